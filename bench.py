#!/usr/bin/env python
"""Speculative-decode throughput of the androidllm verify path on B200.

Workload (default): Qwen2.5-1.5B-shaped target (hidden 1536, 28 layers, 12/2
heads, head_dim 128, FFN 8960, vocab 151936, tied int8 per-row embedding,
int4 attention / int8 MLP, block-64 symmetric) with a Qwen2.5-0.5B-shaped int4
draft, k = 4, greedy, batch 1, 512-token prompt and 256-token episodes.
Weights are seeded random-init (N(0, 0.02)), written in androidllm's shard
format and loaded through the public engine API.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one speculative step (k draft forwards, one (k+1)-row verify
forward, acceptance).  ``value`` is whole-job tokens/s with every input
resident in HBM (device-timed graph replays); ``e2e`` is the same metric
through ``LayerStreamingEngine.generate`` with a host round trip per step.
With N > 1 each rank runs an independent replica (no data-path collective).
``--impl reference`` times the CPU restatement of the reference numpy path
(the oracle port) on this host on a bounded sample.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "spec-decode tokens/sec (k=4) at Qwen2.5-1.5B int4"
PROMPT_LEN = 512
EPISODE_TOKENS = 256
SPEC_K = 4
CACHE = os.environ.get("ALM_BENCH_CACHE", "/tmp/androidllm_b200_bench")
REF_MAX_SAMPLES = 96

WORKLOADS = {
    # name: (target canon, target bits, draft canon, draft bits)
    "qwen2.5-1.5b": ("qwen2.5-1.5b", dict(attn_bits=4, mlp_bits=8, block=64, embed_bits=8),
                     "qwen2.5-0.5b", dict(attn_bits=4, mlp_bits=4, block=64, embed_bits=8)),
    # tensor parallel over the GPUs of the run (k = 6, 2048-token prompt);
    # the draft is the 0.5B shape with the 7B vocabulary, replicated per rank
    "qwen2.5-7b": ("qwen2.5-7b", dict(attn_bits=4, mlp_bits=8, block=64, embed_bits=8),
                   "qwen2.5-0.5b-v152064", dict(attn_bits=4, mlp_bits=4, block=64, embed_bits=8)),
    "toy": ("toy", dict(attn_bits=4, mlp_bits=4, block=64, embed_bits=0), None, None),
}
TP_WORKLOAD = "qwen2.5-7b"
# continuous batching: sessions per GPU, prompt and output length ranges,
# temperature (the 64-sequence / 8-GPU configuration, 8 per GPU)
BATCH_WORKLOAD = "qwen2.5-1.5b-batch"
BATCH_SESSIONS = 8          # active at a time per GPU
BATCH_QUEUE = 24            # sessions per GPU in all (continuous batching: a finished one's slot takes the next)
BATCH_PROMPT = (128, 1024)
BATCH_OUTPUT = (64, 512)
BATCH_TEMPERATURE = 0.8
TP_SPEC_K = 6
TP_PROMPT_LEN = 2048


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


# --------------------------------------------------------------------------
# models
# --------------------------------------------------------------------------
def canon_of(name):
    from androidllm_b200 import synth
    if name == "qwen2.5-0.5b-v152064":
        return dict(synth.CANONS["qwen2.5-0.5b"], vocab=152064, name="qwen2.5-0.5b-synth-v152064")
    return dict(synth.CANONS[name])


def ensure_model(canon_name, kw, seed):
    from androidllm_b200 import shard
    canon = canon_of(canon_name)
    tag = f"{canon_name}-s{seed}-a{kw['attn_bits']}m{kw['mlp_bits']}e{kw['embed_bits']}"
    out = os.path.join(CACHE, tag)
    if not os.path.exists(os.path.join(out, ".complete")):
        shard.write_synthetic(canon, seed, out, workers=min(16, os.cpu_count() or 4), **kw)
        open(os.path.join(out, ".complete"), "w").close()
    return out


def prepare_models(workload):
    tname, tkw, dname, dkw = WORKLOADS[workload]
    tdir = ensure_model(tname, tkw, seed=1)
    if dname is None:
        from androidllm_b200 import shard
        ddir = os.path.join(CACHE, f"{tname}-draft2")
        if not os.path.exists(os.path.join(ddir, "manifest.json")):
            shard.prefix_draft(tdir, ddir, 2)
        return tdir, ddir
    return tdir, ensure_model(dname, dkw, seed=2)


# --------------------------------------------------------------------------
# algorithmic bytes
# --------------------------------------------------------------------------
def gemv_bytes(n, k, m, bits, block=64):
    w = n * k * bits // 8
    s = 0 if bits == 16 else n * (k // block) * 2
    return w + s + m * k * 2 + m * n * 2


def forward_weight_bytes(man):
    """Weight + scale bytes one forward streams (all layers + head)."""
    total = 0
    for li, projs in man["quant"]["layers"].items():
        for base, q in projs.items():
            total += q["out"] * q["in"] * q["bits"] // 8 + q["out"] * (q["in"] // q["block"]) * 2
    c = man["config"]
    hq = man.get("lm_head_quant") or man.get("embed_quant") or {}
    if hq:
        total += c["vocab"] * c["hidden"] * hq["bits"] // 8 + c["vocab"] * (c["hidden"] // hq["block"]) * 2
    else:
        total += c["vocab"] * c["hidden"] * 2
    return total


def _proj_bytes(man, bases, m):
    """Algorithmic bytes of one fused GEMV over the projections ``bases`` of
    layer 0 (weights + scales + m input rows + m output rows)."""
    q = [man["quant"]["layers"]["0"][b] for b in bases]
    n = sum(p["out"] for p in q)
    k = q[0]["in"]
    w = sum(p["out"] * p["in"] * p["bits"] // 8 + p["out"] * (p["in"] // p["block"]) * 2 for p in q)
    return w + m * k * 2 + m * n * 2, n, k, q[0]["bits"]


def _head_bytes(man, m):
    c = man["config"]
    hq = man.get("lm_head_quant") or man.get("embed_quant") or {}
    bits = hq.get("bits", 16)
    w = c["vocab"] * c["hidden"] * bits // 8 + (c["vocab"] * (c["hidden"] // hq["block"]) * 2 if hq else 0)
    return w + m * c["hidden"] * 2 + m * c["vocab"] * 2, bits


_GEMV_OPS = {"qkv": (("q", "k", "v"), "qkv+rope+kv write"), "o": (("o",), "resid"),
             "gate_up": (("gate", "up"), "swiglu"), "down": (("down",), "resid")}


def step_profile_groups(prof, tman, dman, pos, k):
    """Group alm_spec_profile launches by (model, operation): launches, device
    time, share of the step, and achieved GB/s from the algorithmic bytes of
    each launch (GEMV: weights + scales + activations; attention: the K or V
    rows of the context it reads; the rest: none counted)."""
    groups, total, fwd = {}, 0.0, -1
    for role, op, rows, us in prof:
        total += us
        man = dman if role == "draft" else tman
        if role == "draft" and op == "embed":
            fwd += 1
        nbytes, desc = 0, op
        if role in ("draft", "target") and op in _GEMV_OPS:
            bases, epi = _GEMV_OPS[op]
            nbytes, n, kk, bits = _proj_bytes(man, bases, rows)
            desc = f"{op}: gemv_kernel<int{bits}, {epi}> {n}x{kk}, M={rows}"
        elif role in ("draft", "target") and op == "head":
            nbytes, bits = _head_bytes(man, rows)
            c = man["config"]
            desc = f"head: gemv_kernel<int{bits}, logits> {c['vocab']}x{c['hidden']}, M={rows}"
        elif op in ("attn_scores", "attn_pv", "attn"):
            c = man["config"]
            ctx = pos + (fwd + 1 if role == "draft" else k + 1)
            nbytes = c["kv_heads"] * ctx * c["head_dim"] * 2 * (2 if op == "attn" else 1)
            name = "attn_fused_kernel (scores + P.V)" if op == "attn" else f"{op}_kernel"
            desc = f"{name} hd={c['head_dim']} group={c['heads'] // c['kv_heads']} ctx~{ctx}, M={rows}"
        key = f"{role}.{op}"
        g = groups.setdefault(key, {"key": key, "kernel": f"{role} {desc}", "launches": 0, "us": 0.0, "bytes": 0})
        g["launches"] += 1
        g["us"] += us
        g["bytes"] += nbytes
    out = []
    for g in groups.values():
        g["us_per_launch"] = round(g["us"] / g["launches"], 2)
        g["share"] = round(g["us"] / total, 4)
        g["gbs"] = round(g["bytes"] / (g["us"] * 1e3), 1) if g["us"] > 0 else 0.0
        g["bytes_per_launch"] = g["bytes"] // g["launches"]
        out.append(g)
    return sorted(out, key=lambda g: -g["us"])


# --------------------------------------------------------------------------
# clocks during the timed region
# --------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        self.device = vis.split(",")[device] if vis else device
        self.proc = None
        self.path = os.path.join(CACHE, f"clocks_{os.getpid()}.csv")

    def __enter__(self):
        os.makedirs(CACHE, exist_ok=True)
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.device), "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9 and parts[1].isdigit():
                    rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [int(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": int(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows)}


# --------------------------------------------------------------------------
# CPU baseline: the oracle port of the reference numpy path (bounded sample)
# --------------------------------------------------------------------------
def host_description():
    """nproc and the CPU model of this host (the CPU baseline's machine)."""
    model = "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"nproc": os.cpu_count(), "cpu_model": model}


class CpuSample:
    """Times the reference numpy computation (oracle restatement of
    androidllm/models/llama.py and quant.py) for the workload's shapes: one
    target layer, one draft layer (each at position PROMPT_LEN) and a
    1/layers slice of each LM head per sample, plus the per-layer dequant
    that the reference's default streaming engine repeats for every layer of
    every token (androidllm/engine.py:160-174), then extrapolates the time of
    one speculative step for resident and for streamed weights."""

    def __init__(self, workload):
        from androidllm_b200 import synth
        from oracle import llama, quant
        tname, tkw, dname, dkw = WORKLOADS[workload]
        self.llama = llama
        self.quant = quant
        self.tc = canon_of(tname)
        self.dc = dict(canon_of(dname or tname), layers=2 if dname is None else canon_of(dname)["layers"])
        rng = np.random.default_rng(0)
        self.t = self._setup(self.tc, tkw, rng)
        self.d = self._setup(self.dc, dkw or tkw, rng)

    def _setup(self, c, kw, rng):
        h, hd, nh, nkv, i = c["hidden"], c["head_dim"], c["heads"], c["kv_heads"], c["intermediate"]
        mk = lambda *s: (rng.standard_normal(s, dtype=np.float32) * 0.02).astype(np.float16)  # noqa: E731
        shapes = {"q": (nh * hd, h), "k": (nkv * hd, h), "v": (nkv * hd, h), "o": (h, nh * hd),
                  "gate": (i, h), "up": (i, h), "down": (h, i)}
        layer = {b: mk(*sh) for b, sh in shapes.items()}
        layer["n_in"] = np.ones(h, np.float16)
        layer["n_post"] = np.ones(h, np.float16)
        # the shard-format codes of one layer, dequantized per token when streaming
        packed = {}
        for b, (o, k) in shapes.items():
            bits = kw["attn_bits"] if b in ("q", "k", "v", "o") else kw["mlp_bits"]
            blk = kw["block"]
            if bits == 4:
                codes = rng.integers(0, 256, size=(o, k // 2), dtype=np.uint8)
            else:
                codes = rng.integers(-127, 128, size=(o, k), dtype=np.int8)
            packed[b] = (codes, (np.abs(rng.standard_normal((o, k // blk))) * 0.003).astype(np.float16),
                         {"bits": bits, "block": blk, "out": o, "in": k})
        canon = dict(c, max_len=PROMPT_LEN + 8)
        model = self.llama.OracleModel(canon, None, np.ones(h, np.float16), None)
        kv = (mk(PROMPT_LEN + 8, nkv, hd) * 50, mk(PROMPT_LEN + 8, nkv, hd) * 50)
        n_slice = -(-c["vocab"] // c["layers"])
        head_slice = mk(n_slice, h)
        x = (rng.standard_normal((1, h)).astype(np.float16))
        return {"c": c, "layer": layer, "packed": packed, "model": model, "kv": kv, "head": head_slice, "x": x}

    def _one(self, s):
        t0 = time.perf_counter()
        s["model"].layer_forward(s["x"], s["layer"], s["kv"], PROMPT_LEN)
        t1 = time.perf_counter()
        h = self.llama.rms_norm(s["x"], s["model"].final_norm)
        self.llama.matmul_f16(h.astype(np.float16), s["head"])
        t2 = time.perf_counter()
        for codes, scale, meta in s["packed"].values():
            self.quant.dequantize_packed(codes, scale, meta)
        t3 = time.perf_counter()
        # per full token: layers x (layer time [+ its dequant]) + layers x (1/layers of the head)
        n = s["c"]["layers"]
        return n * ((t1 - t0) + (t2 - t1)), n * (t3 - t2)

    def step(self, tokens_per_step, k=SPEC_K):
        """Seconds of one reference speculative step (androidllm/engine.py:288-320):
        k draft tokens, then one target token per emitted token; resident
        weights, and the extra per-token dequant of the streaming engine."""
        t_target, dq_target = self._one(self.t)
        t_draft, dq_draft = self._one(self.d)
        resident = k * t_draft + tokens_per_step * t_target
        streaming = resident + k * dq_draft + tokens_per_step * dq_target
        return resident, streaming, t_target, t_draft


def cpu_baseline(workload, tokens_per_step, samples, k=SPEC_K):
    s = CpuSample(workload)
    s.step(tokens_per_step, k)       # warm-up
    res, stream, walls = [], [], []
    for _ in range(samples):
        t0 = time.perf_counter()
        a, b, _, _ = s.step(tokens_per_step, k)
        walls.append(time.perf_counter() - t0)
        res.append(a)
        stream.append(b)
    host = host_description()
    return {
        "value": tokens_per_step / statistics.mean(res),
        "unit": "tokens/s",
        "cores": 1,
        "kind": "port",
        "value_streaming": tokens_per_step / statistics.mean(stream),
        "host": host,
        "sample": (f"{samples} samples of one target layer + one draft layer at position {PROMPT_LEN}, "
                   f"a 1/layers slice of each fp16 LM head, and one layer's dequantize_packed of each model "
                   f"(numpy, 1 thread: numpy's fp16 matmul has no BLAS path and the reference decodes one "
                   f"sequence; host has {host['nproc']} threads, {host['cpu_model']}), extrapolated to a full "
                   f"step of {k} draft tokens + {tokens_per_step:.2f} target tokens; value = resident "
                   f"dequantized weights, value_streaming = the reference's default streaming engine, which "
                   f"also dequantizes every layer for every token; {sum(walls):.1f}s of CPU work"),
        "sample_s": statistics.mean(walls),
    }


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    tokens_per_step = 1.0
    t0 = time.perf_counter()
    tp = args.workload == TP_WORKLOAD or world > 1
    workload = TP_WORKLOAD if tp else args.workload
    k = TP_SPEC_K if tp else SPEC_K
    # each sample is ~0.5 s (1.5B) / ~2 s (7B) of numpy work; cap the count so
    # the arm ends within a few minutes whatever --steps is
    cb = cpu_baseline(workload, tokens_per_step, min(REF_MAX_SAMPLES if not tp else 24, max(1, args.steps)), k)
    metric = "spec-decode tokens/sec (k=6) at Qwen2.5-7B, tensor parallel" if tp else METRIC
    line = {
        "impl": "reference", "metric": metric, "value": cb["value"], "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        # a step of this arm is one bounded sample (see cpu_baseline.sample);
        # the full speculative step it stands for is extrapolated
        "ms_per_step": round(1000.0 * cb["sample_s"], 3),
        "ms_per_full_step_extrapolated": round(1000.0 * tokens_per_step / cb["value"], 1),
        "higher_is_better": True,
        "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": workload_config(args, world) if not tp else
        {"workload": f"qwen2.5-7b spec-decode (the reference runs one process on the host; the GPU arm is "
                     f"tensor parallel x{world})", "k": TP_SPEC_K, "batch": 1, "prompt_len": TP_PROMPT_LEN,
         "episode_tokens": EPISODE_TOKENS, "temperature": 0},
        "cpu_baseline": {k2: cb[k2] for k2 in ("value", "unit", "cores", "kind", "sample", "value_streaming", "host")},
        "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": time.perf_counter() - t0,
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_config(args, world):
    return {"workload": args.workload + " spec-decode (draft qwen2.5-0.5b shape, int4)"
            if args.workload == "qwen2.5-1.5b" else args.workload,
            "target": "qwen2.5-1.5b: int4 attention, int8 MLP, tied int8 per-row head, block 64",
            "draft": "qwen2.5-0.5b: int4, tied int8 per-row head", "k": SPEC_K, "batch": 1,
            "prompt_len": PROMPT_LEN, "episode_tokens": EPISODE_TOKENS, "temperature": 0,
            "parallelism": f"replicas x{world}" if world > 1 else "single",
            "l2": "weights (2.8 GB streamed per step) exceed the 126 MB L2; no flush needed"}


# --------------------------------------------------------------------------
# our arm
# --------------------------------------------------------------------------
def _profiled_traffic(key):
    """DRAM bytes per launch of a step operation (``draft.down`` and so on)
    from the committed ncu summary profiles/step_kernel_dram.json, or None."""
    path = os.path.join(ROOT, "profiles", "step_kernel_dram.json")
    try:
        with open(path) as f:
            return json.load(f)[key]["dram_bytes_per_launch"]
    except (OSError, KeyError, ValueError):
        return None


def combine_ranks(dist, ms, tokens, device):
    """Replicas: the slowest rank's device time and every rank's tokens."""
    import torch
    t = torch.tensor([ms, float(tokens)], dtype=torch.float64, device=device)
    mx = t.clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    sm = t.clone()
    dist.all_reduce(sm, op=dist.ReduceOp.SUM)
    return float(mx[0]), int(sm[1])


def run_ours(args):
    rank, world, local = dist_env()
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    if rank == 0:
        tdir, ddir = prepare_models(args.workload)
    if dist is not None:
        dist.barrier()
        tdir, ddir = prepare_models(args.workload)
    os.environ.setdefault("ANDROIDLLM_MAX_CTX", "4096")

    from androidllm_b200.engine import LayerStreamingEngine
    from androidllm_b200.ops import QuantProj, QWeight, bench_qmatmul
    eng = LayerStreamingEngine(tdir, draft_dir=ddir, spec_k=SPEC_K, device=local)
    prompt = np.random.default_rng(123).integers(0, eng.canon["vocab"], PROMPT_LEN).tolist()

    # e2e through the public API: generate() with a host round trip per step
    eng.generate(prompt, max_new_tokens=16, temperature=0)          # warm-up (graph, caches)
    out = eng.generate(prompt, max_new_tokens=EPISODE_TOKENS, temperature=0)
    dec = eng.last_decode
    e2e = {"value": len(out) / dec["seconds"], "unit": "tokens/s",
           "scope": "decode steps of generate() (the prompt's prefill is timed separately: prefill_ms)",
           "prefill_ms": round(dec["prefill_seconds"] * 1000.0, 2),
           # per step: the (token, pos) state in (16 B), the state + emitted
           # tokens + accepted count out
           "h2d_bytes_per_step": 16,
           "d2h_bytes_per_step": 16 + 4 * (len(out) / max(1, dec["steps"])) + 4,
           "steps": dec["steps"], "tokens": len(out)}

    # device-resident throughput.  Warm-up: one whole episode from the
    # post-prompt state (positions 511..767 and the tokens at them).  Timed:
    # exactly --steps speculative steps whose start positions are spread
    # evenly over the episode, each a replay of the step graph timed with
    # CUDA events on the decoder's stream, so attention sees the episode's
    # context lengths 512-768 in proportion.
    spec = eng._spec_decoder()
    state0 = (prompt[-1], PROMPT_LEN - 1)
    eng._target_kv().cache.zero()
    eng._prefill(eng._kv, prompt[:-1], 0)
    eng._draft_kv().cache.zero()
    eng.draft._prefill(eng.draft._kv, prompt, 0)
    clk = ClockSampler(local).__enter__()          # sampled from the warm-up on
    spec.begin(*state0)
    stream = [prompt[-1]]
    while len(stream) <= EPISODE_TOKENS:
        emitted, _ = spec.run(1)
        stream += emitted
    for _ in range(max(0, args.warmup - 1)):
        spec.begin(*state0)
        spec.bench(min(EPISODE_TOKENS, 64))
    starts = [PROMPT_LEN - 1 + (i * EPISODE_TOKENS) // args.steps for i in range(args.steps)]
    if dist is not None:
        import torch
        dist.barrier()
        torch.cuda.synchronize()
    t_wall = time.perf_counter()
    ms, tokens = 0.0, 0
    for p0 in starts:
        spec.begin(stream[p0 - (PROMPT_LEN - 1)], p0)
        m1, n1 = spec.bench(1)
        ms += m1
        tokens += n1
    t_wall = time.perf_counter() - t_wall
    clk.__exit__(None, None, None)
    if dist is not None:
        import torch
        torch.cuda.synchronize()
        ms_max, tokens_all = combine_ranks(dist, ms, tokens, "cuda")
        dist.barrier()
    else:
        ms_max, tokens_all = ms, tokens
    value = tokens_all / (ms_max / 1000.0)
    ms_per_step = ms_max / args.steps

    # per-launch device times of one step at the middle of the episode
    # (alm_spec_profile: the step re-captured with a timing event after every
    # kernel); the operation with the largest share is the roofline kernel
    mid = PROMPT_LEN - 1 + EPISODE_TOKENS // 2
    spec.begin(stream[mid - (PROMPT_LEN - 1)], mid)
    prof = spec.profile()
    peaks = load_peaks()
    groups = step_profile_groups(prof, eng.manifest, eng.draft.manifest, mid, SPEC_K)
    top = groups[0]
    roofline = {"kernel": top["kernel"], "bound": "hbm", "achieved": top["gbs"], "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(top["gbs"] / peaks["hbm_gbs"], 3),
                "peak_source": peaks["source"], "algorithmic_bytes": top["bytes_per_launch"],
                "avg_launch_us": top["us_per_launch"], "launches_per_step": top["launches"],
                "share_of_step": top["share"],
                "traffic": _profiled_traffic(top["key"])}
    step_bytes = SPEC_K * forward_weight_bytes(eng.draft.manifest) + forward_weight_bytes(eng.manifest)
    step_roof = step_bytes / (ms_per_step * 1e-3) / 1e9

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic", "config": dict(workload_config(args, world),
                                            positions_timed=[starts[0], starts[-1]]),
        "e2e": {k: (round(v, 3) if isinstance(v, float) else v) for k, v in e2e.items()},
        "roofline": roofline,
        "step_profile": {"position": mid, "launches": len(prof),
                         "sum_us": round(sum(r[3] for r in prof), 1),
                         "note": "per-launch device times of one step re-captured with an event after every "
                                 "kernel (no programmatic dependent launch); shares of that sum",
                         "top": [{k: g[k] for k in ("kernel", "launches", "us_per_launch", "share", "gbs")}
                                 for g in groups[:8]]},
        "step_roofline": {"weight_bytes_per_step": step_bytes, "achieved_gbs": round(step_roof, 1),
                          "frac": round(step_roof / peaks["hbm_gbs"], 3)},
        "tokens_per_step": round(tokens_all / (args.steps * world), 3),
        "gpu_launches": spec.kernel_count() * args.steps,
        "clocks": clk.summary(),
        "wall_s_timed": round(t_wall, 3),
    }
    if rank == 0 and not args.no_cpu_baseline:
        cb = cpu_baseline(args.workload, tokens_per_step=line["tokens_per_step"], samples=args.cpu_samples)
        line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample", "value_streaming",
                                                    "host")}
    if rank == 0:
        print(json.dumps(line), flush=True)
    spec.close()
    if dist is not None:
        dist.destroy_process_group()
    return 0


# --------------------------------------------------------------------------
# tensor-parallel arm: the Qwen2.5-7B-shaped target split over the ranks
# --------------------------------------------------------------------------
def run_batch(args):
    """Continuous batching of speculative sessions (one process per GPU, data
    parallel): BATCH_QUEUE sessions per GPU with seeded prompt lengths in
    BATCH_PROMPT and output lengths in BATCH_OUTPUT, k = 4, T = 0.8 with
    seeded per-session uniforms, paged KV of 16-position pages, at most
    BATCH_SESSIONS active and advanced together, a finished session's slot
    taken by the next (LayerStreamingEngine.generate_batch).  value =
    generated tokens of all ranks / the slowest rank's time; sessions one
    after the other through generate() give the sequential figure it is
    compared with."""
    rank, world, local = dist_env()
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    if rank == 0:
        tdir, ddir = prepare_models("qwen2.5-1.5b")
    if dist is not None:
        dist.barrier()
        tdir, ddir = prepare_models("qwen2.5-1.5b")
    os.environ["ANDROIDLLM_MAX_CTX"] = str(BATCH_PROMPT[1] + BATCH_OUTPUT[1] + 2 * (SPEC_K + 1))
    from androidllm_b200.engine import LayerStreamingEngine
    eng = LayerStreamingEngine(tdir, draft_dir=ddir, spec_k=SPEC_K, device=local)
    eng.batch_runner(slots=BATCH_SESSIONS)
    rng = np.random.default_rng(1000 + rank)
    V = eng.canon["vocab"]
    prompts = [rng.integers(0, V, int(rng.integers(BATCH_PROMPT[0], BATCH_PROMPT[1] + 1))).tolist()
               for _ in range(BATCH_QUEUE)]
    outs = [int(rng.integers(BATCH_OUTPUT[0], BATCH_OUTPUT[1] + 1)) for _ in range(BATCH_QUEUE)]
    seeds = [10_000 * rank + i for i in range(BATCH_QUEUE)]
    # warm-up: a short batch (kernels, caches)
    eng.generate_batch([p[:64] for p in prompts[:2]], max_new_tokens=8, temperature=BATCH_TEMPERATURE,
                       seeds=seeds[:2])
    clk = ClockSampler(local).__enter__()
    if dist is not None:
        dist.barrier()
    t0 = time.perf_counter()
    got = eng.generate_batch(prompts, max_new_tokens=outs, temperature=BATCH_TEMPERATURE, top_p=0.9,
                             seeds=seeds, max_active=BATCH_SESSIONS)
    secs = time.perf_counter() - t0
    clk.__exit__(None, None, None)
    tokens = sum(len(g) for g in got)
    # the same sessions one at a time through generate() (the reference's
    # scheduler visits one session per work unit): rank 0, first sessions
    seq = None
    if rank == 0 and not args.no_cpu_baseline:
        n_seq = 2
        t1 = time.perf_counter()
        n_tok = 0
        for i in range(n_seq):
            n_tok += len(eng.generate(prompts[i], max_new_tokens=outs[i], temperature=BATCH_TEMPERATURE,
                                      top_p=0.9))
        seq = n_tok / (time.perf_counter() - t1)
    if dist is not None:
        import torch
        t = torch.tensor([secs, float(tokens)], dtype=torch.float64, device=torch.device("cuda", local))
        mx, sm = t.clone(), t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        secs, tokens = float(mx[0]), int(sm[1])
    if rank == 0:
        line = {
            "metric": "continuous-batching spec-decode tokens/sec (k=4, T=0.8) at Qwen2.5-1.5B int4, "
                      f"{BATCH_SESSIONS} sessions per GPU",
            "value": round(tokens / secs, 2), "unit": "tokens/s", "n_gpus": world, "steps": 1, "warmup": 1,
            "ms_per_step": round(secs * 1000.0, 2), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": BATCH_WORKLOAD, "sessions_per_gpu": BATCH_SESSIONS,
                       "queued_sessions_per_gpu": BATCH_QUEUE,
                       "prompt_len": list(BATCH_PROMPT), "output_len": list(BATCH_OUTPUT), "k": SPEC_K,
                       "temperature": BATCH_TEMPERATURE, "top_p": 0.9, "kv_page": 16,
                       "parallelism": f"dp{world}", "timed": "prefill + decode of every session, host-timed"},
            "tokens": tokens, "seconds": round(secs, 3),
            "sequential_tokens_per_s": None if seq is None else round(seq, 2),
            "gpu_launches": None,
            "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    eng.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_tp(args):
    """Speculative decoding (k = 6, greedy) of the Qwen2.5-7B-shaped target
    (int4 attention / int8 MLP / int8 head, block 64) split over the ranks
    by tensor parallelism (heads, FFN and vocabulary; an all-reduce after o
    and down through NCCL — over peer memory with ALM_TP_P2P=1 — and an
    all-gathered head argmax), with the 0.5B-shaped int4 draft
    replicated on every rank.  2048-token prompt, 256-token episodes; exactly
    --steps steps timed, their start positions spread over the episode."""
    import datetime

    import torch
    import torch.distributed as dist
    from androidllm_b200 import tp
    from androidllm_b200.ops import Context, DeviceKV, DeviceModel, SpecDecoder
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    if rank == 0:
        tdir, ddir = prepare_models(TP_WORKLOAD)
    if world > 1:
        dist.barrier()
    tdir, ddir = prepare_models(TP_WORKLOAD)
    ctx = Context(local)
    if world > 1:
        uid = [tp.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        tp.init_context_tp(ctx, rank, world, uid[0])
        if os.environ.get("ALM_TP_P2P", "0") == "1":
            tp.enable_p2p(ctx, canon_of(WORKLOADS[TP_WORKLOAD][0])["hidden"])
        t = tp.device_model_tp(ctx, tdir, rank, world)
    else:
        t = DeviceModel.from_dir(ctx, tdir)
    d = DeviceModel.from_dir(ctx, ddir)
    cap = TP_PROMPT_LEN + EPISODE_TOKENS + 2 * (TP_SPEC_K + 1) + 16
    tkv, dkv = DeviceKV(t, cap), DeviceKV(d, cap)
    prompt = np.random.default_rng(321).integers(0, t.canon["vocab"], TP_PROMPT_LEN).tolist()
    t0 = time.perf_counter()
    for i in range(0, TP_PROMPT_LEN - 1, 16):
        t.forward(tkv, prompt[:-1][i:i + 16], i, logits=False, argmax=False)
    for i in range(0, TP_PROMPT_LEN, 16):
        d.forward(dkv, prompt[i:i + 16], i, logits=False, argmax=False)
    prefill_s = time.perf_counter() - t0
    s = SpecDecoder(t, d, tkv, dkv, TP_SPEC_K)
    p0 = TP_PROMPT_LEN - 1
    clk = ClockSampler(local).__enter__()
    # warm-up: one episode (fills the caches over the episode's positions)
    s.begin(prompt[-1], p0)
    stream = [prompt[-1]]
    t_e2e = time.perf_counter()
    n_e2e = 0
    while len(stream) <= EPISODE_TOKENS:
        emitted, _ = s.run(1)
        stream += emitted
        n_e2e += 1
    t_e2e = time.perf_counter() - t_e2e
    for _ in range(max(0, args.warmup - 1)):
        s.begin(prompt[-1], p0)
        s.bench(32)
    starts = [p0 + (i * EPISODE_TOKENS) // args.steps for i in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms, tokens = 0.0, 0
    for st in starts:
        s.begin(stream[st - p0], st)
        m1, n1 = s.bench(1)
        ms += m1
        tokens += n1
    torch.cuda.synchronize()
    clk.__exit__(None, None, None)
    if world > 1:
        ms_max, _ = combine_ranks(dist, ms, tokens, "cuda")
    else:
        ms_max = ms
    # every rank emits the same tokens: the job's tokens are one rank's
    value = tokens / (ms_max / 1000.0)
    ms_per_step = ms_max / args.steps
    mid = p0 + EPISODE_TOKENS // 2
    s.begin(stream[mid - p0], mid)
    prof = s.profile()
    peaks = load_peaks()
    per_rank_bytes = TP_SPEC_K * forward_weight_bytes(d.manifest) + forward_weight_bytes(t.manifest) // world
    line = {
        "metric": "spec-decode tokens/sec (k=6) at Qwen2.5-7B, tensor parallel", "value": round(value, 2),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"qwen2.5-7b spec-decode, tensor parallel x{world} (draft qwen2.5-0.5b shape, "
                               f"int4, replicated)",
                   "target": "qwen2.5-7b: int4 attention, int8 MLP, int8 head, block 64",
                   "draft": "qwen2.5-0.5b: int4, vocabulary 152064", "k": TP_SPEC_K, "batch": 1,
                   "prompt_len": TP_PROMPT_LEN, "episode_tokens": EPISODE_TOKENS, "temperature": 0,
                   "parallelism": f"tp{world}", "positions_timed": [starts[0], starts[-1]],
                   "allreduce": ("peer memory" if world > 1 and os.environ.get("ALM_TP_P2P", "0") == "1"
                                 else "nccl" if world > 1 else None),
                   "l2": "weights (>= 1 GB streamed per step per rank) exceed the 126 MB L2; no flush needed"},
        "e2e": {"value": round((len(stream) - 1) / t_e2e, 3), "unit": "tokens/s",
                "scope": "SpecDecoder.run(1) per step from the host (state in, emitted tokens out)",
                "h2d_bytes_per_step": 16, "d2h_bytes_per_step": 16 + 4 * (TP_SPEC_K + 1) + 4,
                "steps": n_e2e, "tokens": len(stream) - 1, "prefill_s": round(prefill_s, 2)},
        "step_roofline": {"weight_bytes_per_step_per_rank": per_rank_bytes,
                          "achieved_gbs_per_rank": round(per_rank_bytes / (ms_per_step * 1e-3) / 1e9, 1),
                          "frac": round(per_rank_bytes / (ms_per_step * 1e-3) / 1e9 / peaks["hbm_gbs"], 3)},
        "step_profile": {"position": mid, "launches": len(prof), "sum_us": round(sum(r[3] for r in prof), 1),
                         "top": [{k: g[k] for k in ("kernel", "launches", "us_per_launch", "share")}
                                 for g in step_profile_groups(prof, t.manifest, d.manifest, mid, TP_SPEC_K)[:6]]},
        "tokens_per_step": round(tokens / args.steps, 3),
        "gpu_launches": s.kernel_count() * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    s.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# --------------------------------------------------------------------------
# isolated quantized-matmul sweep (block-64 int4 / int8, N(0, 0.02) weights)
# --------------------------------------------------------------------------
SWEEP_SHAPES = [(1536, 1536), (8960, 1536), (1536, 8960), (18944, 3584), (3584, 18944), (151936, 1536)]
SWEEP_M = (1, 5, 8, 16, 40, 128)


def run_sweep(args):
    """GB/s and TFLOP/s of the dequant matmul per (N, K, bits, M),
    graph-replayed launches cycling over weight copies larger than L2; one
    JSON line per case.  M <= 16: the fused dequant-GEMV on the tile layout
    (mma.sync); M > 16: the row layout's dense path (tcgen05 MMAs, N = M)."""
    from androidllm_b200.ops import Context, QuantProj, QWeight, bench_qmatmul
    from androidllm_b200.quant import codes_for_storage, quantize_matrix
    ctx = Context(0)
    peaks = load_peaks()
    rng = np.random.default_rng(3)
    ms = [int(x) for x in args.sweep_m.split(",")]
    shapes = [tuple(int(v) for v in sh.split("x")) for sh in args.sweep_shapes.split(",")] if args.sweep_shapes \
        else SWEEP_SHAPES
    for n, k in shapes:
        for bits in (4, 8):
            # quantize one N(0, 0.02) matrix with the format's own quantizer,
            # then copy it so the rotation exceeds the 126 MB L2
            w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02))
            q, sc = quantize_matrix(w, bits=bits, block=64)
            proj = QuantProj(codes_for_storage(q, bits), sc, bits, 64, n, k)
            del w, q
            per = n * k * bits // 8
            copies = max(2, min(12, int(400e6 // per) + 1))
            plan = ((2, ms),) if args.sweep_layout == "row" else \
                ((0, [m for m in ms if m <= 16]), (2, [m for m in ms if m > 16]))
            for layout, sel in plan:
                if not sel:
                    continue
                ctx.set_gemv_layout(layout)
                ws = [QWeight(ctx, proj) for _ in range(copies)]
                for m in sel:
                    x = rng.standard_normal((m, k)).astype(np.float16)
                    us = bench_qmatmul(ctx, ws, x, 200 if m <= 16 else 40)
                    alg = gemv_bytes(n, k, m, bits)
                    gbs = alg / us / 1e3
                    tflops = 2 * m * n * k / us / 1e6
                    rec = {"n": n, "k": k, "bits": bits, "m": m, "us": round(us, 2), "gbs": round(gbs, 1),
                           "frac": round(gbs / peaks["hbm_gbs"], 3), "tflops": round(tflops, 2),
                           "tensor_frac": round(tflops / peaks["bf16_tflops"], 3),
                           "path": "gemv mma.sync (tile layout)" if layout == 0 else "tcgen05 (row layout)",
                           "split": list(ws[0].split())}
                    print(json.dumps(rec), flush=True)
                del ws
            ctx.set_gemv_layout(0)
    return 0


def run_mma_rate(args):
    """Tensor-core instruction rates on this GPU (JSON lines): mma.sync
    m16n8k16 cycles per instruction per SM by warps per SM and accumulator
    chains; tcgen05.mma (M 128, K 16) ns per instruction by N, operand source
    (A in tensor memory: TS, shared memory: SS), accumulators and issuing
    threads per SM; then the per-launch floor of a CUDA graph of empty
    dependent kernels.  The probe kernels live in libalm_probes.so, apart
    from the product library."""
    import ctypes
    from androidllm_b200.build import PROBES_LIB
    plib = ctypes.CDLL(PROBES_LIB)
    plib.probe_last_error.restype = ctypes.c_char_p
    r = ctypes.c_double()

    def check(rc):
        if rc:
            raise RuntimeError(plib.probe_last_error().decode())

    for warps in (4, 8, 16, 32):
        for chains in (1, 2, 4, 8):
            check(plib.probe_mma_rate(0, 0, warps, chains, ctypes.byref(r)))
            print(json.dumps({"mma": "mma.sync.m16n8k16.f32.f16", "warps_per_sm": warps, "chains": chains,
                              "cycles_per_mma_per_sm": round(r.value, 3),
                              "mac_per_clk_per_sm": round(16 * 8 * 16 / r.value, 1)}), flush=True)
    for kind, form in ((1, "TS"), (2, "SS")):
        for n in (16, 64, 128, 256):
            for na in (1, 8):
                if na * n > 256:
                    continue
                check(plib.probe_mma_rate(0, kind, n, na, ctypes.byref(r)))
                print(json.dumps({"mma": "tcgen05.mma.kind::f16 M128 K16", "form": form, "n": n, "accumulators": na,
                                  "ns_per_mma": round(r.value, 2),
                                  "tmac_per_s_per_sm": round(128 * n * 16 / r.value / 1e3, 3)}), flush=True)
    # several issuing threads per SM: CTAs per SM x issuers per CTA (A in tensor memory)
    for cps in (1, 2, 4):
        for iss in (1, 2, 4):
            for n in (16, 32, 64, 128, 256):
                if iss * n > 512 // cps - 32:
                    continue
                check(plib.probe_tc_rate(0, 1, n, 1, cps, iss, ctypes.byref(r)))
                print(json.dumps({"mma": "tcgen05.mma.kind::f16 M128 K16", "form": "TS", "ctas_per_sm": cps,
                                  "issuers_per_cta": iss, "n": n, "ns_per_mma": round(r.value, 2),
                                  "tmac_per_s_per_sm": round(cps * iss * 128 * n * 16 / r.value / 1e3, 3)}),
                      flush=True)
    # per-launch floor of a CUDA graph: chains of empty dependent kernels
    for pdl in (1, 0):
        for n_ctas in (1, 148, 296, 1184):
            check(plib.probe_launch_floor(0, n_ctas, pdl, ctypes.byref(r)))
            print(json.dumps({"launch_floor": "empty dependent kernels in a CUDA graph", "pdl": bool(pdl),
                              "ctas": n_ctas, "threads": 256, "us_per_launch": round(r.value, 3)}), flush=True)
    return 0


def run_gemv(args):
    """One GEMV shape launched back to back (a small, bounded ncu target)."""
    from androidllm_b200.ops import Context, QuantProj, QWeight, bench_qmatmul
    n, k, bits, m = (int(v) for v in args.gemv.split(","))
    ctx = Context(0)
    if m > 16 or args.sweep_layout == "row":
        ctx.set_gemv_layout(2)   # the row layout (tcgen05); always for more than 16 rows
    rng = np.random.default_rng(0)
    q = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8) if bits == 4 else \
        rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    s = (np.abs(rng.standard_normal((n, k // 64))) * 0.003 + 1e-4).astype(np.float16)
    copies = max(2, min(8, int(300e6 // (n * k * bits // 8)) + 1))
    ws = [QWeight(ctx, QuantProj(q, s, bits, 64, n, k)) for _ in range(copies)]
    x = rng.standard_normal((m, k)).astype(np.float16)
    us = bench_qmatmul(ctx, ws, x, 4 * copies)
    alg = gemv_bytes(n, k, m, bits)
    print(json.dumps({"n": n, "k": k, "bits": bits, "m": m, "us": us, "gbs": alg / us / 1e3,
                      "split": list(ws[0].split())}))
    return 0


# --------------------------------------------------------------------------
# profiling helpers (used with Nsight Compute; see profiles/)
# --------------------------------------------------------------------------
def run_profile(args):
    """Load the workload, then run --profile N speculative steps inside a CUDA
    profiler capture range (start ncu with --profile-from-start off).  A short
    prompt keeps the launches before the range few; the steps run at position
    600, the middle of a 512-prompt / 256-token episode."""
    from androidllm_b200._lib import lib
    from androidllm_b200.ops import Context, DeviceKV, DeviceModel, SpecDecoder
    tdir, ddir = prepare_models(args.workload)
    ctx = Context(0)
    t, d = DeviceModel.from_dir(ctx, tdir), DeviceModel.from_dir(ctx, ddir)
    tkv, dkv = DeviceKV(t, 1024), DeviceKV(d, 1024)
    prompt = np.random.default_rng(123).integers(0, t.canon["vocab"], 16).tolist()
    t.forward(tkv, prompt[:15], 0, logits=False, argmax=False)
    d.forward(dkv, prompt, 0, logits=False, argmax=False)
    s = SpecDecoder(t, d, tkv, dkv, SPEC_K)
    if args.temperature > 0:
        s.set_sampling(args.temperature, args.top_p, 0.0)
        s.set_uniforms(np.random.default_rng(7).random(64 * (2 * SPEC_K + 1)))
    s.begin(prompt[-1], 600)
    s.bench(2)
    s.begin(prompt[-1], 600)
    lib.alm_profiler_range(1)
    ms, _ = s.bench(args.profile)
    lib.alm_profiler_range(0)
    print(json.dumps({"profile_steps": args.profile, "ms_per_step": ms / args.profile,
                      "kernels_per_step": s.kernel_count()}))
    return 0


def run_profile_prefill(args):
    """Load the workload's target and prefill --profile-prefill N prompt tokens
    inside a CUDA profiler capture range (start ncu with --profile-from-start
    off): 256-row chunks through the dense tcgen05 path."""
    from androidllm_b200._lib import lib
    from androidllm_b200.ops import Context, DeviceKV, DeviceModel
    tdir, _ = prepare_models(args.workload)
    ctx = Context(0)
    t = DeviceModel.from_dir(ctx, tdir)
    n = int(args.profile_prefill)
    kv = DeviceKV(t, n + 16)
    toks = np.random.default_rng(5).integers(0, t.canon["vocab"], n).tolist()
    t.prefill(kv, toks, 0)                       # warm-up (scratch, caches)
    lib.alm_profiler_range(1)
    t0 = time.perf_counter()
    t.prefill(kv, toks, 0)
    secs = time.perf_counter() - t0
    lib.alm_profiler_range(0)
    print(json.dumps({"profile_prefill_tokens": n, "ms": secs * 1e3, "dense": t.uses_dense_prefill()}))
    return 0


_PHASES = ("qkv", "scores", "pv", "o", "gu", "down")


def run_trace_forward(args):
    """Per-phase timeline of the persistent forward kernel (global timer of
    CTA 0: its own work in each phase, then its wait at the grid barrier) for
    the draft (1 row) and the target (5 rows) at position 600."""
    from androidllm_b200.ops import Context, DeviceKV, DeviceModel
    tdir, ddir = prepare_models(args.workload)
    ctx = Context(0)
    for tag, d, rows in (("draft", ddir, 1), ("target", tdir, 5)):
        m = DeviceModel.from_dir(ctx, d)
        kv = DeviceKV(m, 1024)
        toks = np.random.default_rng(5).integers(0, m.canon["vocab"], 608).tolist()
        for i in range(0, 592, 16):
            m.forward(kv, toks[i:i + 16], i, logits=False, argmax=False)
        for _ in range(args.trace_forward):
            arrive, passed = m.forward_trace(kv, toks[600:600 + rows], 600)
        arrive, passed = arrive.astype(np.int64), passed.astype(np.int64)
        names = ["embed"] + list(_PHASES) * m.canon["layers"] + ["rownorm", "head"]
        work, wait = {}, {}
        prev = int(arrive[0, 0])
        for b in range(arrive.shape[0]):
            if b > 0:
                work.setdefault(names[b], []).append(int(arrive[b, 0]) - prev)
            wait.setdefault(names[b], []).append(int(passed[b]) - int(arrive[b, 0]))
            prev = int(passed[b])
        out = {"model": tag, "rows": rows, "ctas": int(arrive.shape[1]),
               "total_us": round((int(passed[-1]) - int(arrive[0, 0])) / 1e3, 1), "phases": {}}
        for n in dict.fromkeys(names[1:]):
            out["phases"][n] = {"work_us": round(float(np.median(work[n])) / 1e3, 2),
                                "barrier_wait_us": round(float(np.median(wait[n])) / 1e3, 2)}
        print(json.dumps(out), flush=True)
        kv.close()
        m.close()
    return 0


def run_trace_cluster(args):
    """Per-phase timeline of the single-row cluster forward of the draft
    (sync times of CTA 0) at position 600: median microseconds per phase."""
    from androidllm_b200.ops import Context, DeviceKV, DeviceModel
    _, ddir = prepare_models(args.workload)
    ctx = Context(0)
    m = DeviceModel.from_dir(ctx, ddir)
    kv = DeviceKV(m, 1024)
    toks = np.random.default_rng(5).integers(0, m.canon["vocab"], 608).tolist()
    for i in range(0, 592, 16):
        m.forward(kv, toks[i:i + 16], i, logits=False, argmax=False)
    runs = [m.cluster_trace(kv, toks[600], 600) for _ in range(args.trace_cluster)]
    dec, prod = runs[-1]
    t0 = dec[0][1]
    # per GEMV phase: staging, items (first warp), items (all), epilogue, sync
    names = {1: "start", 2: "staged", 3: "items_w0", 4: "items_all", 5: "epilogue", 6: "sync",
             7: "scores", 8: "pv"}
    layer = []
    prev = t0
    for lab, t in dec[: 60]:
        layer.append((names.get(lab, str(lab)), round((t - prev) / 1e3, 2)))
        prev = t
    totals = [(d[-1][1] - d[0][1]) / 1e3 for d, _ in runs]
    pr = [(lab, round((t - t0) / 1e3, 2)) for lab, t in prod[: 24]]
    print(json.dumps({"model": "draft", "layers": m.canon["layers"], "total_us": round(float(np.median(totals)), 1),
                      "first_points_us_since_previous": layer, "producer_points_us_since_start": pr}), flush=True)
    return 0


def summarize_ncu(path):
    """Aggregate an ncu --csv launch list (gpu__time_duration.sum) by kernel."""
    import collections
    import csv
    import re
    with open(path) as f:
        rows = list(csv.reader(f))
    hdr = next(i for i, r in enumerate(rows) if "Kernel Name" in r)
    h = rows[hdr]
    ki, mi, vi = h.index("Kernel Name"), h.index("Metric Name"), h.index("Metric Value")
    agg = collections.defaultdict(lambda: [0, 0.0])
    epi = {"0": "store", "1": "qkv+rope", "2": "resid", "3": "swiglu", "4": "logits"}
    for r in rows[hdr + 1:]:
        if len(r) <= vi or r[mi] != "gpu__time_duration.sum":
            continue
        name = r[ki]
        m = re.search(r"(tc_gemm_kernel|tc_gemv_kernel|gemv_kernel)<([^>]*)>", name)
        if m:
            g = re.findall(r"\d+", m.group(2))
            if m.group(1) == "tc_gemm_kernel" and len(g) == 2:   # dense path: bits, issuing threads
                name = f"tc_gemm_kernel<int{g[0]}, {g[1]} issuer{'s' if g[1] != '1' else ''}>"
            elif m.group(1) == "tc_gemv_kernel" and len(g) == 2:
                name = f"tc_gemv_kernel<int{g[0]}, {epi.get(g[1], g[1])}>"
            elif len(g) == 4:   # gemv_kernel<bits, scale sets, n8 tiles, epilogue>
                name = f"gemv_kernel<int{g[0]}, nt8={g[2]}, {epi.get(g[3], g[3])}>"
            elif len(g) == 3:
                name = f"gemv_kernel<int{g[0]}, nt8={g[1]}, {epi.get(g[2], g[2])}>"
        else:
            name = re.sub(r"\(.*", "", name).split("::")[-1]
        agg[name][0] += 1
        agg[name][1] += float(r[vi].replace(",", ""))
    tot = sum(v[1] for v in agg.values())
    out = [f"{'kernel':48s} {'launches':>8s} {'total_us':>10s} {'share':>7s}"]
    for k, (n, v) in sorted(agg.items(), key=lambda kv: -kv[1][1]):
        out.append(f"{k:48s} {n:8d} {v / 1000:10.1f} {100 * v / tot:6.1f}%")
    out.append(f"{'total':48s} {sum(v[0] for v in agg.values()):8d} {tot / 1000:10.1f}")
    print("\n".join(out))
    return 0


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "source": "measured (MEASURED_PEAKS.json)"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + [BATCH_WORKLOAD], default="qwen2.5-1.5b")
    ap.add_argument("--cpu-samples", type=int, default=6)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", type=int, default=0,
                    help="run N steps inside a profiler capture range and exit")
    ap.add_argument("--summarize-ncu", metavar="CSV", help="aggregate an ncu launch list and exit")
    ap.add_argument("--profile-prefill", type=int, default=0, metavar="N",
                    help="prefill N tokens of the target inside a profiler capture range and exit")
    ap.add_argument("--temperature", type=float, default=0.0,
                    help="--profile: sampling steps at this temperature (0: greedy)")
    ap.add_argument("--top-p", type=float, default=0.9, help="--profile: nucleus of the sampling steps")
    ap.add_argument("--trace-forward", type=int, default=0, metavar="N",
                    help="run N traced persistent forwards per model and print the phase timeline")
    ap.add_argument("--trace-cluster", type=int, default=0, metavar="N",
                    help="run N traced single-row cluster forwards of the draft and print the phase timeline")
    ap.add_argument("--sweep", action="store_true", help="isolated quantized-matmul sweep (JSON lines)")
    ap.add_argument("--sweep-m", default=",".join(str(m) for m in SWEEP_M))
    ap.add_argument("--sweep-shapes", default="", metavar="NxK,...", help="sweep only these weight shapes")
    ap.add_argument("--sweep-layout", choices=("auto", "row"), default="auto",
                    help="auto: tile layout (mma.sync) up to 16 rows, row layout (tcgen05) above; row: row layout for all")
    ap.add_argument("--gemv", metavar="N,K,BITS,M", help="time one GEMV shape repeatedly (profiling target)")
    ap.add_argument("--mma-rate", action="store_true", help="tensor-core instruction rates (JSON lines)")
    args = ap.parse_args()
    if args.sweep:
        return run_sweep(args)
    if args.gemv:
        return run_gemv(args)
    if args.mma_rate:
        return run_mma_rate(args)
    if args.summarize_ncu:
        return summarize_ncu(args.summarize_ncu)
    if args.profile:
        return run_profile(args)
    if args.profile_prefill:
        return run_profile_prefill(args)
    if args.trace_forward:
        return run_trace_forward(args)
    if args.trace_cluster:
        return run_trace_cluster(args)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == BATCH_WORKLOAD:
        return run_batch(args)
    if args.workload == TP_WORKLOAD or dist_env()[1] > 1:
        return run_tp(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
