"""Generate the golden fixtures in this directory by running the androidllm
reference itself (numpy path) on seeded inputs.

Run from the repository root, with the path of an androidllm checkout (or
the environment variable ANDROIDLLM_REFERENCE set to it):

    python tests/golden/make_golden.py --reference <androidllm checkout> [--only qwen]

It writes:
  quant.npz     reference quantize/pack/dequant outputs for seeded matrices,
                including K padding, block 32, int8, per-row (embedding)
                blocks, an all-zero block, and the pack known-answer vector of
                the reference's tests/test_quant.py:39-46.
  models.json   sha256 of every shard file the reference writer produces for
                the seeded models below (pins this repository's writer).
  toy.npz       toy Llama (hidden 256, 4 layers, 8/2 heads, head_dim 32, FFN
                688, vocab 32000, all int4 block 64, fp16 embed): hidden states,
                logits, greedy plain and speculative (k=4, 2-layer prefix
                draft) token streams of 128 tokens, stats and top-1/top-2
                margins, and a temperature-1.0 speculative run.
  tiny.npz      the reference test toy (hidden 64, 2 layers, 4/2 heads,
                head_dim 16, FFN 96, vocab 64, int4 block 32): layer states and
                logits.
  minq.npz      a small Qwen-style model (int4 attention, int8 MLP with K
                padding, int8 per-row embedding, untied int8 head): states and
                logits.
  sampling.npz  reference sampler picks for seeded logits and a grid of
                (temperature, top_p, min_p), with the uniform each pick used.
  qwen.npz      the benchmark's layer shapes: 2-layer Qwen2.5-1.5B-shaped target
                (head_dim 128, 12/2 heads, FFN 8960, int4 attention / int8
                MLP, tied int8 per-row 151936 head) and 2-layer Qwen2.5-0.5B-
                shaped draft (head_dim 64, 14/2 heads, FFN 4864, int4), with
                the KV cache of positions 0..775 filled from seeded fp16
                values: layer states of 1-row decode and 5-row verify passes
                at positions 511-771, and argmax / top-2 margin / sha256 /
                sampled entries of the logits.  --only qwen regenerates just
                this file (the reference takes a few minutes at these shapes).

The reference never travels with this repository: only the fixtures do.
"""
import argparse
import hashlib
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from androidllm_b200 import shard as my_shard  # noqa: E402
from androidllm_b200 import synth  # noqa: E402

sys.path.insert(0, HERE)
from qwen_cases import (QWEN_CASES, QWEN_FILL, QWEN_MODELS, qwen_case_tokens,  # noqa: E402
                        qwen_kv_fill, qwen_logit_index)

TOY_PROMPT_SEED = 123
TOY_SEED = 1
TINY = dict(model_type="qwen2", hidden=64, layers=2, heads=4, kv_heads=2, head_dim=16,
            intermediate=96, vocab=64, rope_theta=10000.0, rms_eps=1e-6, max_len=128,
            tied=True, name="tiny")
MINQ = dict(model_type="qwen2", hidden=128, layers=2, heads=4, kv_heads=2, head_dim=32,
            intermediate=344, vocab=1000, rope_theta=1e6, rms_eps=1e-6, max_len=256,
            tied=False, name="minq")
# the toy with an untied fp16 head: its greedy stream is not a single repeated
# token (a tied random-init toy keeps re-picking its input token)
TOYU = dict(synth.CANONS["toy"], tied=False, name="toy-untied")
# (name, canon, seed, shard kwargs)
MODELS = [
    ("toy", synth.CANONS["toy"], TOY_SEED, dict(attn_bits=4, mlp_bits=4, block=64, embed_bits=0)),
    ("tiny", TINY, 7, dict(attn_bits=4, mlp_bits=4, block=32, embed_bits=0)),
    ("minq", MINQ, 3, dict(attn_bits=4, mlp_bits=8, block=64, embed_bits=8)),
    ("toyu", TOYU, 11, dict(attn_bits=4, mlp_bits=4, block=64, embed_bits=0)),
]


def sha(path):
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def write_ref_model(ref_shard, canon, seed, kw, out):
    ref_shard.shard_from_tensors(synth.synth_tensors(canon, seed=seed), canon, out, **kw)
    return {fn: sha(os.path.join(out, fn)) for fn in sorted(os.listdir(out))}


def toy_tokenizer(model_dir):
    """Minimal tokenizer files: the reference engine only enables speculative
    decoding when a tokenizer is present (androidllm/engine.py:337-338)."""
    from androidllm.tokenizer import _bytes_to_unicode
    m = _bytes_to_unicode()
    with open(os.path.join(model_dir, "vocab.txt"), "w", encoding="utf-8") as f:
        f.write("\n".join(["", "<s>", "</s>", "<unk>"] + [m[b] for b in range(256)]) + "\n")
    open(os.path.join(model_dir, "merges.txt"), "w").close()
    with open(os.path.join(model_dir, "special_tokens.json"), "w") as f:
        json.dump({"<s>": 1, "</s>": 2, "<unk>": 3}, f)
    with open(os.path.join(model_dir, "template.txt"), "w") as f:
        f.write("{{messages}}")


def states_and_logits(engine, prompt, n_pos):
    """Resident reference forward: per-layer hidden states for the first
    ``n_pos`` positions, and the logits after the whole prompt."""
    model = engine.model
    layers = [engine._load_layer_raw(i) for i in range(engine.n_layers)]
    kv = model.prepare_kv(len(prompt) + 8)
    states = []
    x = None
    for pos, tok in enumerate(prompt):
        x = model.embed[tok].reshape(1, -1)
        per = []
        for li in range(engine.n_layers):
            x = model.layer_forward(x, layers[li], kv[li], pos)
            per.append(np.array(x, dtype=np.float16).reshape(-1))
        if pos < n_pos:
            states.append(np.stack(per))
    logits = model.logits(x)
    return np.stack(states), logits.reshape(-1).astype(np.float16)


def margins(logit_rows):
    out = []
    for lg in logit_rows:
        s = np.sort(np.asarray(lg, np.float32).reshape(-1))
        out.append(float(s[-1] - s[-2]))
    return np.array(out, np.float32)


def quant_cases(q):
    rng = np.random.default_rng(42)
    cases = []
    for bits in (4, 8):
        for block, shape in ((64, (13, 200)), (64, (64, 128)), (32, (16, 96)), (64, (16, 688)),
                             (64, (8, 1536))):
            w = rng.standard_normal(shape).astype(np.float32) * 0.02
            if shape == (8, 1536):
                w[3, 64:128] = 0.0       # an all-zero block
                w[5, :] = 0.0            # an all-zero row
                w[7, 5] = 1e-7           # a block whose fp16 scale underflows
                w[7, 0:5] = 0.0
                w[7, 6:64] = 0.0
            cases.append((bits, block, w))
    # per-row blocks, as the int8 embedding quantization uses (shard.py:89-94)
    w = rng.standard_normal((24, 256)).astype(np.float32) * 0.02
    cases.append((8, 256, w))
    out = {}
    for i, (bits, block, w) in enumerate(cases):
        qq, sc = q.quantize_matrix(w, bits=bits, block=block)
        packed = q.pack_int4(qq) if bits == 4 else qq.astype(np.int8)
        meta = {"bits": bits, "block": block, "out": qq.shape[0], "in": qq.shape[1]}
        deq = q.dequantize_packed(packed, sc, meta)
        out[f"c{i}_w"] = w
        out[f"c{i}_meta"] = np.array([bits, block, qq.shape[0], qq.shape[1], w.shape[1]], np.int64)
        out[f"c{i}_q"] = qq.astype(np.int32)
        out[f"c{i}_scale"] = sc
        out[f"c{i}_packed"] = packed
        out[f"c{i}_deq"] = deq
    out["n_cases"] = np.array(len(cases))
    kat = np.array([[0, 1, 2, 7, -8, -1, -7, -8, 3, 4],
                    [5, 6, -2, 0, -8, -5, 3, 1, 2, 7]], dtype=np.int32)
    out["kat_q"] = kat
    out["kat_packed"] = q.pack_int4(kat)
    out["kat_unpacked"] = q.unpack_int4(out["kat_packed"], 2, 10)
    return out


def sampling_cases(engine_mod):
    out = {}
    grid = [(0.0, 1.0, 0.0), (1.0, 1.0, 0.0), (0.7, 1.0, 0.0), (1.0, 0.9, 0.0),
            (0.8, 0.9, 0.05), (1.3, 1.0, 0.1), (0.5, 0.5, 0.0)]
    k = 0
    for vocab, n_seeds in ((1000, 4), (32000, 2)):
        for case_seed in range(n_seeds):
            lg = (np.random.default_rng([vocab, case_seed]).standard_normal(vocab) * 2.0)
            lg = lg.astype(np.float16).astype(np.float32)
            for t, tp, mp in grid:
                rng = np.random.default_rng([99, k])
                shadow = np.random.default_rng([99, k])
                pick = engine_mod._sample(lg, t, tp, mp, rng)
                u = shadow.random() if t > 0 else -1.0
                out[f"s{k}_logits"] = lg.astype(np.float16)
                out[f"s{k}_params"] = np.array([t, tp, mp, u], np.float64)
                out[f"s{k}_pick"] = np.array(pick)
                k += 1
    out["n_cases"] = np.array(k)
    return out


def run_toy(LayerStreamingEngine, toy, draft, out_path):
    """Toy Llama runs: states, logits, greedy plain and speculative streams
    (k=4, draft = the target's first 2 layers) and a temperature-1.0 run."""
    my_shard.prefix_draft(toy, draft, 2)
    toy_tokenizer(toy)
    prompt = np.random.default_rng(TOY_PROMPT_SEED).integers(0, 32000, 64).tolist()
    e = LayerStreamingEngine(toy, keep_layers=4)
    states, logits = states_and_logits(e, prompt, 6)

    recorded = []
    orig_score = LayerStreamingEngine._score

    def rec_score(self, x):
        lg = orig_score(self, x)
        recorded.append(np.asarray(lg, np.float32).reshape(-1))
        return lg

    LayerStreamingEngine._score = rec_score
    try:
        plain = e.generate(prompt, max_new_tokens=128, temperature=0.0, top_p=1.0)
    finally:
        LayerStreamingEngine._score = orig_score
    plain_margins = margins(recorded)

    s = LayerStreamingEngine(toy, keep_layers=4, draft_dir=draft, spec_k=4)
    s.draft._keep = 2
    spec = s.generate(prompt, max_new_tokens=128, temperature=0.0, top_p=1.0)
    sp = s.snapshot()["spec"]

    s1 = LayerStreamingEngine(toy, keep_layers=4, draft_dir=draft, spec_k=4)
    s1.draft._keep = 2
    s1._rng = np.random.default_rng(2024)
    spec_t1 = s1.generate(prompt, max_new_tokens=64, temperature=1.0, top_p=1.0)
    sp1 = s1.snapshot()["spec"]

    np.savez_compressed(
        out_path,
        prompt=np.array(prompt, np.int64), states=states, logits=logits,
        plain=np.array(plain, np.int64), plain_margins=plain_margins,
        spec=np.array(spec, np.int64),
        spec_stats=np.array([sp["steps"], sp["draft_tokens"], sp["accepted"], sp["bonus"]],
                            np.int64),
        spec_t1=np.array(spec_t1, np.int64),
        spec_t1_stats=np.array([sp1["steps"], sp1["draft_tokens"], sp1["accepted"],
                                sp1["bonus"]], np.int64))
    print(os.path.basename(out_path), "spec", sp, "t1", sp1, "plain==spec", plain == spec,
          "distinct", len(set(plain)), "min margin", float(plain_margins.min()))


def run_qwen(LayerStreamingEngine, tmp, out_path):
    """Reference layer_forward / logits at the benchmark's shapes over a
    seeded KV cache (the reference has no batched pass: a 5-row verify case is
    5 consecutive single-row forwards, each row through every layer)."""
    out = {}
    for name, canon, seed, kw in QWEN_MODELS:
        d = os.path.join(tmp, name)
        out[f"{name}_files"] = np.array(json.dumps(write_ref_model(sys.modules["androidllm.shard"], canon, seed,
                                                                    kw, d)))
        e = LayerStreamingEngine(d, keep_layers=canon["layers"])
        model = e.model
        layers = [e._load_layer_raw(i) for i in range(canon["layers"])]
        fills = [qwen_kv_fill(canon, seed, li) for li in range(canon["layers"])]
        idx = qwen_logit_index(canon["vocab"])
        states, am, mg, hashes, samples = [], [], [], [], []
        for ci, (rows, pos0) in enumerate(QWEN_CASES):
            kv = model.prepare_kv(QWEN_FILL + 8)
            for li, (k, v) in enumerate(fills):
                kv[li][0][:QWEN_FILL] = k
                kv[li][1][:QWEN_FILL] = v
            toks = qwen_case_tokens(canon, seed, ci)[:rows]
            st = np.zeros((5, canon["layers"], canon["hidden"]), np.float16)
            for r, tok in enumerate(toks):
                x = model.embed[tok].reshape(1, -1)
                for li in range(canon["layers"]):
                    x = model.layer_forward(x, layers[li], kv[li], pos0 + r)
                    st[r, li] = np.asarray(x, np.float16).reshape(-1)
                lg = np.asarray(model.logits(x), np.float32).reshape(-1).astype(np.float16)
                srt = np.sort(lg.astype(np.float32))
                am.append(int(np.argmax(lg)))
                mg.append(float(srt[-1] - srt[-2]))
                hashes.append(hashlib.sha256(lg.tobytes()).hexdigest())
                samples.append(lg[idx])
            states.append(st)
            print(name, "case", ci, rows, pos0, "argmax", am[-rows:], flush=True)
        out[f"{name}_states"] = np.stack(states)
        out[f"{name}_argmax"] = np.array(am, np.int64)
        out[f"{name}_margin"] = np.array(mg, np.float32)
        out[f"{name}_hash"] = np.array(hashes)
        out[f"{name}_sample"] = np.stack(samples)
    out["cases"] = np.array(QWEN_CASES, np.int64)
    np.savez_compressed(out_path, **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ANDROIDLLM_REFERENCE"),
                    help="androidllm checkout (default: $ANDROIDLLM_REFERENCE)")
    ap.add_argument("--only", choices=["qwen"], help="regenerate one fixture file only")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or ANDROIDLLM_REFERENCE) is required")
    sys.path.insert(0, args.reference)
    os.environ["ANDROIDLLM_PREFIX_KV"] = "0"
    from androidllm import engine as ref_engine
    from androidllm import quant as ref_quant
    from androidllm import shard as ref_shard
    from androidllm.engine import LayerStreamingEngine

    # Reference bug: _finalize_kv iterates the target's layer count over the
    # draft's KV list (androidllm/engine.py:266-273 called at :361), so any
    # draft with fewer layers than its target raises IndexError.  The call is
    # a no-op for fp16 caches; iterate the list that was passed instead.
    def _finalize_kv(self, kv, n):
        from androidllm.kv_cache import QuantizedKVCache
        for c in kv:
            if isinstance(c, QuantizedKVCache):
                c.finalize(n)

    LayerStreamingEngine._finalize_kv = _finalize_kv

    if args.only == "qwen":
        with tempfile.TemporaryDirectory() as tmp:
            run_qwen(LayerStreamingEngine, tmp, os.path.join(HERE, "qwen.npz"))
        print("qwen fixture written")
        return

    np.savez_compressed(os.path.join(HERE, "quant.npz"), **quant_cases(ref_quant))
    np.savez_compressed(os.path.join(HERE, "sampling.npz"), **sampling_cases(ref_engine))

    hashes = {}
    with tempfile.TemporaryDirectory() as tmp:
        dirs = {}
        for name, canon, seed, kw in MODELS:
            d = os.path.join(tmp, name)
            hashes[name] = {"seed": seed, "shard": kw, "canon": canon,
                            "files": write_ref_model(ref_shard, canon, seed, kw, d)}
            dirs[name] = d

        for name in ("toy", "toyu"):
            run_toy(LayerStreamingEngine, dirs[name], os.path.join(tmp, name + "_draft"),
                    os.path.join(HERE, name + ".npz"))

        for name, n_pos in (("tiny", 5), ("minq", 5)):
            canon = hashes[name]["canon"]
            prompt = np.random.default_rng(5).integers(0, canon["vocab"], 9).tolist()
            e = LayerStreamingEngine(dirs[name], keep_layers=canon["layers"])
            st, lg = states_and_logits(e, prompt, n_pos)
            np.savez_compressed(os.path.join(HERE, f"{name}.npz"), prompt=np.array(prompt),
                                states=st, logits=lg)

    with open(os.path.join(HERE, "models.json"), "w") as f:
        json.dump(hashes, f, indent=1)
    print("golden fixtures written")


if __name__ == "__main__":
    main()
