"""Python objects over the C ABI: context, quantized weights, device models,
paged KV caches and the speculative decoder.  numpy in, numpy out; device
memory is owned by the library."""
import atexit
import ctypes
import json
import os

import numpy as np

from . import safetensors
from ._lib import ModelConfig, ProjSrc, check, lib, ptr

PROJ_BASES = ("q", "k", "v", "o", "gate", "up", "down")   # androidllm/shard.py:111
# ALM_OP_* codes of include/androidllm_b200.h, in order
OP_NAMES = ("begin", "embed", "qkv", "attn_scores", "attn_pv", "o", "gate_up", "down", "final_norm", "head",
            "argmax", "spec_prep", "spec_accept", "sample", "layers", "attn")

# At interpreter exit the order of finalizers is arbitrary (a context could go
# before the models on it); the process teardown frees device memory anyway.
_EXITING = []
atexit.register(lambda: _EXITING.append(True))


def _f16(a):
    return np.ascontiguousarray(np.asarray(a), dtype=np.float16)


class Context:
    """One device + one stream."""

    def __init__(self, device=0):
        h = ctypes.c_void_p()
        check(lib.alm_ctx_create(int(device), ctypes.byref(h)))
        self.h = h
        self.device = device

    def sync(self):
        check(lib.alm_ctx_sync(self.h))

    def set_persistent(self, enable):
        """Run forwards of <= 8 rows as one persistent kernel or as one launch
        per layer operation (the default); both give bit-identical results."""
        check(lib.alm_ctx_set_persistent(self.h, 1 if enable else 0))

    def set_cluster_forward(self, enable):
        """Single-row forwards of small models as one 16-CTA cluster kernel
        (opt-in, bit-identical, slower on B200 at the draft's shape) or as one
        launch per layer operation (the default)."""
        check(lib.alm_ctx_set_cluster_forward(self.h, 1 if enable else 0))

    def set_tp_p2p(self, enable):
        """Row-split all-reduce over peer memory (after tp.enable_p2p) or NCCL."""
        check(lib.alm_ctx_set_tp_p2p(self.h, 1 if enable else 0))

    def set_attn_fused(self, enable):
        """Attention of decode / verify passes in one launch (opt-in, slower on
        B200 at the benchmark's shapes) or as the two passes (scores, then
        P.V; the default, which the persistent and cluster forwards
        reproduce bit for bit)."""
        check(lib.alm_ctx_set_attn_fused(self.h, 1 if enable else 0))

    def set_dense_prefill(self, enable):
        """Whether models loaded on this context from now on keep row-layout
        copies of their projections so that prefill runs through the dense
        tcgen05 path (default on)."""
        check(lib.alm_ctx_set_dense_prefill(self.h, 1 if enable else 0))

    def set_gemv_layout(self, mode):
        """Layout of weights uploaded from now on: 0 = 16-row tiles (mma.sync
        GEMV, the default), 1 = 128-row records (tcgen05 kernel) for weights of
        4 MB or more, 2 = 128-row records wherever the format allows."""
        check(lib.alm_ctx_set_gemv_layout(self.h, int(mode)))

    def close(self):
        if self.h:
            lib.alm_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        if _EXITING:
            return
        try:
            self.close()
        except Exception:
            pass


_DEFAULT = {}


def default_context(device=0):
    ctx = _DEFAULT.get(device)
    if ctx is None or ctx.h is None:
        ctx = _DEFAULT[device] = Context(device)
    return ctx


class DeviceBuffer:
    def __init__(self, ctx, nbytes):
        h = ctypes.c_void_p()
        check(lib.alm_dev_alloc(ctx.h, int(nbytes), ctypes.byref(h)))
        self.ctx, self.h, self.nbytes = ctx, h, int(nbytes)

    def upload(self, a):
        a = np.ascontiguousarray(a)
        check(lib.alm_copy_h2d(self.ctx.h, self.h, ptr(a), a.nbytes))

    def download(self, out):
        check(lib.alm_copy_d2h(self.ctx.h, ptr(out), self.h, out.nbytes))
        return out

    def free(self):
        if self.h:
            lib.alm_dev_free(self.ctx.h, self.h)
            self.h = None

    def __del__(self):
        if _EXITING:
            return
        try:
            self.free()
        except Exception:
            pass


class QuantProj:
    """One projection in the shard format: codes, scales and manifest meta."""

    def __init__(self, packed, scale, bits, block, out, in_, in_real=None):
        self.bits = int(bits)
        if self.bits == 16:
            self.packed = _f16(packed)
            self.scale = None
        else:
            dt = np.uint8 if self.bits == 4 else np.int8
            self.packed = np.ascontiguousarray(packed, dtype=dt)
            self.scale = _f16(scale)
        self.block = int(block)
        self.out = int(out)
        self.in_ = int(in_)
        self.in_real = int(in_real if in_real is not None else in_)

    @classmethod
    def from_fp16(cls, w):
        w = _f16(w)
        return cls(w, None, 16, 0, w.shape[0], w.shape[1])

    def src(self):
        return ProjSrc(ptr(self.packed), ptr(self.scale), self.bits, self.block, self.out, self.in_,
                       self.in_real)


class QWeight:
    """A weight uploaded and repacked into the tensor-core tile layout."""

    def __init__(self, ctx, proj):
        h = ctypes.c_void_p()
        check(lib.alm_qweight_upload(ctx.h, ptr(proj.packed), ptr(proj.scale), proj.bits, proj.block,
                                     proj.out, proj.in_, proj.in_real, ctypes.byref(h)))
        self.ctx, self.h, self.proj = ctx, h, proj

    def set_split(self, ksw, ksg):
        check(lib.alm_qweight_set_split(self.h, int(ksw), int(ksg)))

    def split(self):
        a, b, c = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        check(lib.alm_qweight_get_split(self.h, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c)))
        return a.value, b.value, c.value

    def dequant(self):
        """fp16 (out, in_real): bit-exact androidllm dequantize_packed (sliced)."""
        out = np.empty((self.proj.out, self.proj.in_real), np.float16)
        check(lib.alm_qweight_dequant(self.ctx.h, self.h, ptr(out)))
        return out

    def matmul(self, x):
        """fp16(x (m, in_real) . W^T), fp32 accumulation; m <= 16, or m <= 256
        for a weight uploaded in the row layout (tcgen05 MMAs)."""
        x = _f16(x)
        m = x.shape[0]
        xb = DeviceBuffer(self.ctx, x.nbytes)
        yb = DeviceBuffer(self.ctx, m * self.proj.out * 2)
        xb.upload(x)
        check(lib.alm_qmatmul(self.ctx.h, self.h, xb.h, x.shape[1], m, yb.h, self.proj.out))
        return yb.download(np.empty((m, self.proj.out), np.float16))

    def free(self):
        if self.h:
            lib.alm_qweight_free(self.h)
            self.h = None

    def __del__(self):
        if _EXITING:
            return
        try:
            self.free()
        except Exception:
            pass


def sample(ctx, logits, temperature, top_p=1.0, min_p=0.0, uniforms=None):
    """alm_sample: engine.py:26-45 on rows of fp16 logits (rows, vocab) with
    the caller's uniform draws (one per row); temperature <= 0 is argmax."""
    lg = _f16(np.atleast_2d(logits))
    rows, vocab = lg.shape
    u = np.ascontiguousarray(np.zeros(rows) if uniforms is None else uniforms, dtype=np.float64).reshape(-1)
    if u.size != rows:
        raise ValueError("one uniform draw per row")
    out = np.empty(rows, np.int32)
    check(lib.alm_sample(ctx.h, ptr(lg), rows, vocab, float(temperature), float(top_p), float(min_p), ptr(u),
                         ptr(out)))
    return out


def probs(ctx, logits, temperature, min_p=0.0):
    """alm_probs: softmax(l / T) rows (min-p filtered) with the rejection
    sampler's fixed arithmetic, fp32 (rows, vocab)."""
    lg = _f16(np.atleast_2d(logits))
    out = np.empty(lg.shape, np.float32)
    check(lib.alm_probs(ctx.h, ptr(lg), lg.shape[0], lg.shape[1], float(temperature), float(min_p), ptr(out)))
    return out


def accept(ctx, target_logits, draft_probs, draft_tokens, temperature, uniforms, min_p=0.0):
    """alm_accept: min(1, p/q) acceptance of k draft tokens against k + 1
    target logit rows; uniforms = k acceptance draws then the resample draw.
    Returns (emitted tokens, number accepted)."""
    lg = _f16(np.atleast_2d(target_logits))
    q = np.ascontiguousarray(np.atleast_2d(draft_probs), dtype=np.float32)
    tok = np.ascontiguousarray(draft_tokens, dtype=np.int32).reshape(-1)
    k = tok.size
    if lg.shape[0] != k + 1 or q.shape != (k, lg.shape[1]):
        raise ValueError("target_logits (k + 1, vocab), draft_probs (k, vocab), draft_tokens (k,)")
    u = np.ascontiguousarray(uniforms, dtype=np.float64).reshape(-1)
    if u.size != k + 1:
        raise ValueError("k + 1 uniform draws: k acceptance draws and the resample draw")
    out = np.empty(k + 1, np.int32)
    n = ctypes.c_int32()
    check(lib.alm_accept(ctx.h, ptr(lg), ptr(q), ptr(tok), k, lg.shape[1], float(temperature), float(min_p),
                         ptr(u), ptr(out), ctypes.byref(n)))
    return out[: n.value + 1].tolist(), n.value


def bench_qmatmul(ctx, weights, x, iters):
    """Mean device time (us) of one dequant-GEMV launch, cycling through
    ``weights`` (QWeight of one shape) so their total can exceed L2."""
    x = _f16(x)
    m = x.shape[0]
    out = weights[0].proj.out
    xb = DeviceBuffer(ctx, x.nbytes)
    yb = DeviceBuffer(ctx, m * out * 2)
    xb.upload(x)
    arr = (ctypes.c_void_p * len(weights))(*[w.h.value for w in weights])
    us = ctypes.c_float()
    check(lib.alm_bench_qmatmul(ctx.h, arr, len(weights), xb.h, m, yb.h, int(iters), ctypes.byref(us)))
    return us.value


def matmul_f16(a, b, ctx=None):
    """``a @ b.T`` for fp16 a (m, k) and b (n, k) on the GPU (androidllm/neon.py:39-51)."""
    a, b = _f16(a), _f16(b)
    ctx = ctx or default_context()
    out = np.empty((a.shape[0], b.shape[0]), np.float16)
    check(lib.alm_matmul_f16_f16(ctx.h, ptr(a), ptr(b), ptr(out), a.shape[0], a.shape[1], b.shape[0]))
    return out


def precompute_rope(head_dim, max_len, theta=10000.0):
    """[cos | sin] table, float64 angles stored fp16 (androidllm/models/llama.py:27-31)."""
    inv = 1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float64) / head_dim))
    ang = np.outer(np.arange(max_len, dtype=np.float64), inv)
    return np.concatenate([np.cos(ang), np.sin(ang)], axis=1).astype(np.float16)


def config_of(canon):
    return ModelConfig(canon["hidden"], canon["layers"], canon["heads"], canon["kv_heads"],
                       canon["head_dim"], canon["intermediate"], canon["vocab"],
                       int(canon["max_len"]), float(canon["rms_eps"]))


def _as_proj(w):
    return w if isinstance(w, QuantProj) else QuantProj.from_fp16(w)


class DeviceModel:
    """A target or draft model resident in HBM (alm_model)."""

    def __init__(self, ctx, canon):
        self.ctx = ctx
        self.canon = dict(canon)
        self.rope = precompute_rope(canon["head_dim"], int(canon["max_len"]), float(canon["rope_theta"]))
        h = ctypes.c_void_p()
        cfg = config_of(canon)
        check(lib.alm_model_create(ctx.h, ctypes.byref(cfg), ptr(self.rope), ctypes.byref(h)))
        self.h = h
        self._layer_src = [None] * canon["layers"]

    # -- assembly ---------------------------------------------------------------
    def set_layer(self, li, layer):
        """``layer``: {q,k,v,o,gate,up,down: QuantProj or fp16 (out, in) array,
        n_in, n_post: fp16 (hidden,)}."""
        projs = [_as_proj(layer[b]) for b in PROJ_BASES]
        arr = (ProjSrc * 7)(*[p.src() for p in projs])
        n_in, n_post = _f16(layer["n_in"]).reshape(-1), _f16(layer["n_post"]).reshape(-1)
        check(lib.alm_model_set_layer(self.h, int(li), arr, ptr(n_in), ptr(n_post)))
        self._layer_src[li] = layer

    def set_embed(self, table, scale=None, bits=16, block=0):
        table = _f16(table) if bits == 16 else np.ascontiguousarray(table)
        scale = None if scale is None else _f16(scale)
        check(lib.alm_model_set_embed(self.h, ptr(table), ptr(scale), int(bits), int(block)))

    def set_final_norm(self, w):
        w = _f16(w).reshape(-1)
        check(lib.alm_model_set_final_norm(self.h, ptr(w)))

    def set_head(self, proj):
        proj = _as_proj(proj)
        src = proj.src()
        check(lib.alm_model_set_head(self.h, ctypes.byref(src)))

    def finalize(self):
        check(lib.alm_model_finalize(self.h))

    def uses_dense_prefill(self):
        """Whether prefill runs its chunks through the dense tcgen05 path."""
        v = ctypes.c_int32()
        check(lib.alm_model_dense_prefill(self.h, ctypes.byref(v)))
        return bool(v.value)

    def max_pass_rows(self):
        """Most rows one forward_seqs pass takes (alm_model_max_pass_rows)."""
        v = ctypes.c_int32()
        check(lib.alm_model_max_pass_rows(self.h, ctypes.byref(v)))
        return v.value

    def prefill(self, kv, tokens, pos0=0, slot=0):
        """Fill kv (slot ``slot``) for positions pos0 .. pos0 + len(tokens) - 1
        (alm_prefill_slot): the prompt's forwards without logits, in chunks of
        up to 256 rows."""
        tok = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        if tok.size:
            check(lib.alm_prefill_slot(self.h, kv.h, int(slot), ptr(tok), int(tok.size), int(pos0)))

    def uses_cluster_forward(self):
        """Whether single-row forwards run as the 16-CTA cluster kernel."""
        v = ctypes.c_int32()
        check(lib.alm_model_cluster_forward(self.h, ctypes.byref(v)))
        return bool(v.value)

    @classmethod
    def from_dir(cls, ctx, model_dir, layers=None):
        """Load an androidllm shard directory straight to the device (no host
        dequantization, androidllm/engine.py:90-116,160-174)."""
        man = load_manifest(model_dir)
        canon = man["config"]
        m = cls(ctx, canon)
        m.manifest = man
        n = canon["layers"] if layers is None else layers
        for i in range(n):
            m.set_layer(i, read_layer(model_dir, man, i))
        emb = os.path.join(model_dir, "embeddings.safetensors")
        eq = man.get("embed_quant") or {}
        if eq:
            m.set_embed(safetensors.read_tensor(emb, "embed.q"), safetensors.read_tensor(emb, "embed.scale"),
                        eq["bits"], eq["block"])
        else:
            m.set_embed(safetensors.read_tensor(emb, "embed"))
        m.set_final_norm(safetensors.read_tensor(os.path.join(model_dir, "norms.safetensors"), "final_norm"))
        if man.get("has_lm_head"):
            path = os.path.join(model_dir, "lm_head.safetensors")
            lq = man.get("lm_head_quant") or {}
            if lq:
                m.set_head(QuantProj(safetensors.read_tensor(path, "lm_head.q"),
                                     safetensors.read_tensor(path, "lm_head.scale"), lq["bits"], lq["block"],
                                     lq["out"], lq["in"]))
            else:
                m.set_head(safetensors.read_tensor(path, "lm_head"))
        m.finalize()
        return m

    # -- compute ------------------------------------------------------------------
    def layer_forward(self, li, kv, x, pos0):
        x = _f16(x)
        x = x.reshape(-1, self.canon["hidden"])
        out = np.empty_like(x)
        check(lib.alm_layer_forward(self.h, int(li), kv.h, ptr(x), x.shape[0], int(pos0), ptr(out)))
        return out

    def head_logits(self, x, want_logits=True):
        x = _f16(x).reshape(-1, self.canon["hidden"])
        rows = x.shape[0]
        lg = np.empty((rows, self.canon["vocab"]), np.float32) if want_logits else None
        am = np.empty(rows, np.int32)
        check(lib.alm_head_logits(self.h, ptr(x), rows, ptr(lg), ptr(am)))
        return lg, am

    def forward(self, kv, tokens, pos0, logits=False, argmax=True):
        tok = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        rows = tok.size
        lg = np.empty((rows, self.canon["vocab"]), np.float32) if logits else None
        am = np.empty(rows, np.int32) if argmax else None
        check(lib.alm_forward(self.h, kv.h, ptr(tok), rows, int(pos0), ptr(lg), ptr(am)))
        return lg, am

    def sample_rows(self, row0, rows, temperature, top_p=1.0, min_p=0.0, uniforms=None):
        """alm_model_sample_rows: sample rows row0 .. row0 + rows - 1 of the last
        forward's logits (one sequence of a multi-sequence pass)."""
        u = np.ascontiguousarray(np.zeros(rows) if uniforms is None else uniforms, dtype=np.float64).reshape(-1)
        out = np.empty(rows, np.int32)
        check(lib.alm_model_sample_rows(self.h, int(row0), int(rows), float(temperature), float(top_p),
                                        float(min_p), ptr(u), ptr(out)))
        return out

    def forward_seqs(self, kv, seqs, logits=False, argmax=True):
        """One pass over several sequences (alm_forward_seqs): ``seqs`` is a
        list of (slot, tokens, pos0); returns per-sequence lists of logits rows
        (or None) and argmax rows (or None)."""
        slots = np.array([int(s) for s, _, _ in seqs], np.int32)
        n_tok = np.array([len(t) for _, t, _ in seqs], np.int32)
        pos = np.array([int(p) for _, _, p in seqs], np.int32)
        tok = np.ascontiguousarray(np.concatenate([np.asarray(t, np.int32).reshape(-1) for _, t, _ in seqs]))
        rows = tok.size
        lg = np.empty((rows, self.canon["vocab"]), np.float32) if logits else None
        am = np.empty(rows, np.int32) if argmax else None
        check(lib.alm_forward_seqs(self.h, kv.h, len(seqs), ptr(slots), ptr(n_tok), ptr(pos), ptr(tok), ptr(lg),
                                   ptr(am)))
        cuts = np.cumsum(n_tok)[:-1]
        return (np.split(lg, cuts) if logits else None), (np.split(am, cuts) if argmax else None)

    def sample(self, rows, temperature, top_p=1.0, min_p=0.0, uniforms=None):
        """alm_model_sample: sample the first rows of the last forward's logits."""
        u = np.ascontiguousarray(np.zeros(rows) if uniforms is None else uniforms, dtype=np.float64).reshape(-1)
        out = np.empty(rows, np.int32)
        check(lib.alm_model_sample(self.h, int(rows), float(temperature), float(top_p), float(min_p), ptr(u),
                                   ptr(out)))
        return out

    def forward_trace(self, kv, tokens, pos0):
        """One persistent forward (with head) recording when every CTA
        finished every phase.  Returns (arrive[n_barriers, n_ctas],
        passed[n_barriers]) in global-timer nanoseconds."""
        tok = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        n_bar = 1 + 6 * self.canon["layers"] + 2
        cap = n_bar * (2 * 148 * 4 + 1)
        buf = np.zeros(cap, np.uint64)
        nb, nc = ctypes.c_int(), ctypes.c_int()
        check(lib.alm_forward_trace(self.h, kv.h, ptr(tok), tok.size, int(pos0), ptr(buf), cap,
                                    ctypes.byref(nb), ctypes.byref(nc)))
        nb, nc = nb.value, nc.value
        return buf[: nb * nc].reshape(nb, nc), buf[nb * nc: nb * nc + nb]

    def cluster_trace(self, kv, token, pos0, cap=1 << 16):
        """One single-row cluster forward (no head) with CTA 0's trace points:
        returns (decoder points, producer points), each a list of (label,
        global-timer ns)."""
        tok = np.ascontiguousarray([token], dtype=np.int32)
        buf = np.zeros(cap, np.uint64)
        nb, nc = ctypes.c_int(), ctypes.c_int()
        check(lib.alm_forward_trace(self.h, kv.h, ptr(tok), 1, int(pos0), ptr(buf), cap,
                                    ctypes.byref(nb), ctypes.byref(nc)))
        if nc.value != 1:
            raise RuntimeError("the model does not run the cluster forward")

        def points(b):
            n = int(b[0])
            return [(int(v) >> 48, int(v) & 0xffffffffffff) for v in b[1:1 + n]]
        return points(buf[: cap // 2]), points(buf[cap // 2:])

    def close(self):
        if self.h:
            lib.alm_model_destroy(self.h)
            self.h = None

    def __del__(self):
        if _EXITING:
            return
        try:
            self.close()
        except Exception:
            pass


def load_manifest(model_dir):
    with open(os.path.join(model_dir, "manifest.json"), encoding="utf-8") as f:
        return json.load(f)


def read_layer(model_dir, man, i):
    """Layer i as QuantProj entries + norms (androidllm/engine.py:160-174 without dequant)."""
    path = os.path.join(model_dir, f"layer_{i}.safetensors")
    header, _ = safetensors.read_header(path)
    layer = {}
    for base, qm in man["quant"]["layers"][str(i)].items():
        layer[base] = QuantProj(safetensors.read_tensor(path, base + ".q", header),
                                safetensors.read_tensor(path, base + ".scale", header),
                                qm["bits"], qm["block"], qm["out"], qm["in"], qm.get("in_real", qm["in"]))
    layer["n_in"] = safetensors.read_tensor(path, "input_layernorm.weight", header)
    layer["n_post"] = safetensors.read_tensor(path, "post_attention_layernorm.weight", header)
    return layer


class DeviceKV:
    """Paged fp16 KV cache of every layer of one model (alm_kv): ``slots``
    sequences of ``max_len`` positions each (single-sequence calls use slot 0)."""

    def __init__(self, model, max_len, page_size=16, slots=1):
        h = ctypes.c_void_p()
        if slots == 1:
            check(lib.alm_kv_create(model.ctx.h, model.h, int(max_len), int(page_size), ctypes.byref(h)))
        else:
            check(lib.alm_kv_create_slots(model.ctx.h, model.h, int(slots), int(max_len), int(page_size),
                                          ctypes.byref(h)))
        self.h = h
        self.model = model
        self.max_len = int(max_len)
        self.page_size = int(page_size)
        self.slots = int(slots)

    def zero(self):
        check(lib.alm_kv_zero(self.h))

    def read(self, layer, pos0, n, slot=0):
        c = self.model.canon
        shape = (n, c["kv_heads"], c["head_dim"])
        k, v = np.empty(shape, np.float16), np.empty(shape, np.float16)
        check(lib.alm_kv_read_slot(self.h, int(slot), int(layer), int(pos0), int(n), ptr(k), ptr(v)))
        return k, v

    def set_pages(self, slot, pages):
        """Map slot's first len(pages) pages to the given physical pages."""
        pg = np.ascontiguousarray(pages, dtype=np.int32).reshape(-1)
        check(lib.alm_kv_set_pages(self.h, int(slot), ptr(pg), int(pg.size)))

    def write(self, layer, pos0, k, v):
        k, v = _f16(k), _f16(v)
        check(lib.alm_kv_write(self.h, int(layer), int(pos0), k.shape[0], ptr(k), ptr(v)))

    def close(self):
        if self.h:
            lib.alm_kv_destroy(self.h)
            self.h = None

    def __del__(self):
        if _EXITING:
            return
        try:
            self.close()
        except Exception:
            pass


class SpecDecoder:
    """Greedy speculative decoding on the device (alm_spec)."""

    def __init__(self, target, draft, target_kv, draft_kv, k):
        h = ctypes.c_void_p()
        check(lib.alm_spec_create(target.h, draft.h, target_kv.h, draft_kv.h, int(k), ctypes.byref(h)))
        self.h = h
        self.k = int(k)
        self._keep = (target, draft, target_kv, draft_kv)
        self._sampling = (0.0, 1.0, 0.0)
        self._uniforms = None

    def begin(self, token, pos, prev=None):
        """Step state: `token` at position `pos` (and the token at pos - 1,
        which the draft refresh forwards again)."""
        if prev is None:
            check(lib.alm_spec_begin(self.h, int(token), int(pos)))
        else:
            check(lib.alm_spec_begin_prev(self.h, int(prev), int(token), int(pos)))

    def set_draft_refresh(self, enable):
        """Re-forward the token at pos - 1 in every step's first draft
        forward (fixes the draft's stale cache entry after an all-accept
        step; off by default, the reference's behaviour)."""
        enable = bool(enable)
        if enable != getattr(self, "_refresh", False):
            check(lib.alm_spec_set_draft_refresh(self.h, 1 if enable else 0))
            self._refresh = enable

    def run(self, n_steps=1):
        """Run n_steps steps; returns (emitted tokens, accepted count per step)."""
        emitted = np.empty(n_steps * (self.k + 1), np.int32)
        n = np.zeros(1, np.int32)
        acc = np.empty(n_steps, np.int32)
        check(lib.alm_spec_run(self.h, int(n_steps), ptr(emitted), ptr(n), ptr(acc)))
        return emitted[: int(n[0])].tolist(), acc.tolist()

    def set_sampling(self, temperature, top_p=1.0, min_p=0.0):
        """Sampling steps at temperature > 0 (greedy at <= 0); re-captures the
        step graph only when the settings change."""
        key = (float(temperature) if temperature > 0 else 0.0, float(top_p), float(min_p))
        if key != self._sampling:
            check(lib.alm_spec_set_sampling(self.h, key[0], key[1], key[2]))
            self._sampling = key

    def set_rejection(self, enable):
        """Sampling steps accept by min(1, p/q) rejection sampling (True) or
        by the reference's rule (False, the default)."""
        enable = bool(enable)
        if enable != getattr(self, "_rejection", False):
            check(lib.alm_spec_set_rejection(self.h, 1 if enable else 0))
            self._rejection = enable

    def set_uniforms(self, uniforms):
        """Load the uniform draws the sampling steps consume (cursor reset)."""
        u = np.ascontiguousarray(uniforms, dtype=np.float64).reshape(-1)
        check(lib.alm_spec_set_uniforms(self.h, ptr(u), u.size))
        self._uniforms = u

    def uniforms_used(self):
        n = ctypes.c_int32()
        check(lib.alm_spec_uniforms_used(self.h, ctypes.byref(n)))
        return n.value

    def bench(self, n_steps):
        """Device-timed replay of n_steps steps: (ms, emitted tokens)."""
        ms, n = ctypes.c_float(), ctypes.c_int32()
        check(lib.alm_spec_bench(self.h, int(n_steps), ctypes.byref(ms), ctypes.byref(n)))
        return ms.value, n.value

    def profile(self, cap=4096):
        """Device time of every kernel launch of one step from the current
        state (alm_spec_profile): a list of (role, op, rows, us), role
        "draft" / "target" / "spec", op the ALM_OP_* name."""
        ops = np.empty(cap, np.int32)
        rows = np.empty(cap, np.int32)
        us = np.empty(cap, np.float32)
        n = ctypes.c_int32()
        check(lib.alm_spec_profile(self.h, cap, ptr(ops), ptr(rows), ptr(us), ctypes.byref(n)))
        roles = {0: "spec", 1: "draft", 2: "target"}
        return [(roles[int(o) // 100], OP_NAMES[int(o) % 100], int(r), float(u))
                for o, r, u in zip(ops[: n.value], rows[: n.value], us[: n.value])]

    def kernel_count(self):
        n = ctypes.c_int32()
        check(lib.alm_spec_kernel_count(self.h, ctypes.byref(n)))
        return n.value

    def state(self):
        t, p = ctypes.c_int32(), ctypes.c_int32()
        check(lib.alm_spec_state(self.h, ctypes.byref(t), ctypes.byref(p)))
        return t.value, p.value

    def close(self):
        if self.h:
            lib.alm_spec_destroy(self.h)
            self.h = None

    def __del__(self):
        if _EXITING:
            return
        try:
            self.close()
        except Exception:
            pass
