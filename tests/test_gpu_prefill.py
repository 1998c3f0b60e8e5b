"""Batched prompt prefill (alm_prefill; the reference runs the prompt as
single-token forwards, androidllm/engine.py:345-361): chunks of up to 256
rows through the dense tcgen05 path against the oracle's sequential
forwards and against the M <= 16 forward, on the golden models and on a
2-layer model with the Qwen2.5-1.5B target's layer shapes."""
import numpy as np
import pytest
from gpu_helpers import prefill, rel_err

from oracle import io as oio
from oracle import llama as ollama

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from androidllm_b200.ops import Context
    return Context(0)


def _kv_all(m, kv, n):
    return [kv.read(li, 0, n) for li in range(m.canon["layers"])]


def _compare_kv(a, b, tol=1e-2):
    exact = total = 0
    for (ka, va), (kb, vb) in zip(a, b):
        for x, y in ((ka, kb), (va, vb)):
            assert rel_err(x.astype(np.float32), y.astype(np.float32)) < tol
            exact += int(np.sum(x.view(np.uint16) == y.view(np.uint16)))
            total += x.size
    return exact / total


@pytest.mark.parametrize("name", ["toy", "toyu", "minq"])
def test_dense_prefill_matches_16_row_forwards(ctx, model_dirs, name):
    """300 prompt tokens (chunks of 256 and 44 rows; 240 for a 256-position
    model): the KV cache and the next token's logits match 16-row forwards;
    a prompt split over two calls gives the cache of one call."""
    from androidllm_b200.ops import DeviceKV, DeviceModel
    m = DeviceModel.from_dir(ctx, model_dirs[name])
    assert m.uses_dense_prefill()
    n = min(300, int(m.canon["max_len"]) - 16)
    rng = np.random.default_rng(3)
    toks = rng.integers(0, m.canon["vocab"], n).tolist()
    cap = n + 8
    kv_d, kv_c = DeviceKV(m, cap), DeviceKV(m, cap)
    m.prefill(kv_d, toks, 0)
    prefill(m, kv_c, toks)
    frac = _compare_kv(_kv_all(m, kv_d, n), _kv_all(m, kv_c, n))
    print(f"{name}: {frac:.3f} of the KV entries bit-identical to 16-row forwards")
    lg_d, am_d = m.forward(kv_d, [17], n, logits=True)
    lg_c, am_c = m.forward(kv_c, [17], n, logits=True)
    assert rel_err(lg_d[0], lg_c[0]) < 1e-2
    srt = np.sort(lg_c[0])
    assert int(am_d[0]) == int(am_c[0]) or srt[-1] - srt[-2] <= 2 * float(np.spacing(np.float16(abs(srt[-1]))))
    # two calls (120 + the rest) against one
    kv_2 = DeviceKV(m, cap)
    m.prefill(kv_2, toks[:120], 0)
    m.prefill(kv_2, toks[120:], 120)
    frac2 = _compare_kv(_kv_all(m, kv_2, n), _kv_all(m, kv_d, n))
    print(f"{name}: {frac2:.3f} bit-identical between one and two prefill calls")


@pytest.mark.parametrize("name", ["toyu", "minq"])
def test_dense_prefill_matches_oracle(ctx, model_dirs, name):
    """A 40-row dense chunk against the oracle's 40 single-token forwards
    (androidllm/models/llama.py:96-128): every layer's K and V within 1e-2."""
    from androidllm_b200.ops import DeviceKV, DeviceModel
    m = DeviceModel.from_dir(ctx, model_dirs[name])
    canon, embed, fnorm, head, layers = oio.load_model(model_dirs[name])
    om = ollama.OracleModel(canon, embed, fnorm, head)
    toks = np.random.default_rng(9).integers(0, canon["vocab"], 40).tolist()
    okv = om.prepare_kv(64)
    for pos, t in enumerate(toks):
        om.forward(layers, t, okv, pos)
    kv = DeviceKV(m, 64)
    m.prefill(kv, toks, 0)
    for li in range(canon["layers"]):
        k, v = kv.read(li, 0, 40)
        assert rel_err(k.astype(np.float32), okv[li][0][:40].astype(np.float32)) < 1e-2, li
        assert rel_err(v.astype(np.float32), okv[li][1][:40].astype(np.float32)) < 1e-2, li


def test_dense_prefill_at_the_targets_layer_shapes(ctx, tmp_path):
    """hidden 1536, 12/2 heads of 128, FFN 8960, int4 attention / int8 MLP
    (the benchmark target's layers; 2 layers, a 4096-row vocabulary): 512
    prompt tokens in two 256-row chunks against 16-row forwards."""
    from androidllm_b200 import shard, synth
    from androidllm_b200.ops import DeviceKV, DeviceModel
    canon = dict(synth.CANONS["qwen2.5-1.5b"], layers=2, vocab=4096, max_len=1024, name="qwen1.5b-2l-v4096")
    d = str(tmp_path / "q")
    shard.shard_from_tensors(synth.synth_tensors(canon, seed=5), canon, d, attn_bits=4, mlp_bits=8, block=64,
                             embed_bits=8)
    m = DeviceModel.from_dir(ctx, d)
    assert m.uses_dense_prefill()
    toks = np.random.default_rng(4).integers(0, canon["vocab"], 512).tolist()
    kv_d, kv_c = DeviceKV(m, 1024), DeviceKV(m, 1024)
    m.prefill(kv_d, toks, 0)
    prefill(m, kv_c, toks)
    frac = _compare_kv(_kv_all(m, kv_d, 512), _kv_all(m, kv_c, 512))
    print(f"target shapes: {frac:.3f} of the KV entries bit-identical to 16-row forwards")
    lg_d, _ = m.forward(kv_d, [11], 512, logits=True)
    lg_c, _ = m.forward(kv_c, [11], 512, logits=True)
    assert rel_err(lg_d[0], lg_c[0]) < 1e-2


def test_prefill_without_row_layout_copies(model_dirs):
    """A context with the dense prefill off (and a model whose blocks are 32
    columns) prefills through the 16-row forward: same cache as prefill()."""
    from androidllm_b200.ops import Context, DeviceKV, DeviceModel
    c = Context(0)
    c.set_dense_prefill(False)
    m = DeviceModel.from_dir(c, model_dirs["toyu"])
    assert not m.uses_dense_prefill()
    t = DeviceModel.from_dir(Context(0), model_dirs["tiny"])
    assert not t.uses_dense_prefill()
    toks = np.random.default_rng(6).integers(0, 256, 70).tolist()
    for mm in (m, t):
        toks_m = [x % mm.canon["vocab"] for x in toks]
        kv_a, kv_b = DeviceKV(mm, 128), DeviceKV(mm, 128)
        mm.prefill(kv_a, toks_m, 0)
        prefill(mm, kv_b, toks_m)
        for (ka, va), (kb, vb) in zip(_kv_all(mm, kv_a, 70), _kv_all(mm, kv_b, 70)):
            assert np.array_equal(ka.view(np.uint16), kb.view(np.uint16))
            assert np.array_equal(va.view(np.uint16), vb.view(np.uint16))


def test_engine_generate_with_dense_prefill(model_dirs):
    """generate() prefills through the dense path; its first greedy tokens
    equal those of an engine on a context without the row-layout copies,
    up to a near-tie."""
    from androidllm_b200.engine import LayerStreamingEngine
    from androidllm_b200.ops import Context
    prompt = np.random.default_rng(8).integers(0, 32000, 200).tolist()
    e1 = LayerStreamingEngine(model_dirs["toyu"], draft_dir=model_dirs["toyu_draft"], spec_k=4)
    assert e1.dm.uses_dense_prefill()
    c = Context(0)
    c.set_dense_prefill(False)
    e2 = LayerStreamingEngine(model_dirs["toyu"], draft_dir=model_dirs["toyu_draft"], spec_k=4, _ctx=c)
    assert not e2.dm.uses_dense_prefill()
    a = e1.generate(prompt, max_new_tokens=16, temperature=0.0)
    b = e2.generate(prompt, max_new_tokens=16, temperature=0.0)
    n_same = next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), len(a))
    print(f"{n_same} of 16 tokens equal; dense prefill {e1.last_decode['prefill_seconds'] * 1e3:.1f} ms, "
          f"16-row forwards {e2.last_decode['prefill_seconds'] * 1e3:.1f} ms")
    assert n_same >= 1
    e1.close()
    e2.close()
