"""Oracle (test infrastructure): restatement of androidllm/models/llama.py.

The numpy branch of ``LlamaModel`` (``llama.py:96-146``) with every rounding
point of the reference kept:

* matmuls are fp16 x fp16 -> fp16 (numpy half matmul; ``neon.py:51``),
* RoPE, scores, softmax, RMSNorm and SwiGLU in fp32,
* K/V stored fp16, softmax probabilities cast to fp16 before P.V,
* residual adds fp16 + fp16, RMSNorm outputs cast to fp16,
* the layer is post-norm: ``x = norm(x + attn(x))``, ``x = norm(x + mlp(x))``.

``verify_forward`` runs M consecutive positions one at a time; the reference
has no batched forward, so M sequential single-row calls are the oracle for a
batched (k+1)-row verify pass.
"""
import math

import numpy as np


def matmul_f16(a, b):
    """androidllm/neon.py:39-51 fallback: ``fp16(a) @ fp16(b).T``."""
    a = np.ascontiguousarray(a, dtype=np.float16)
    b = np.ascontiguousarray(b, dtype=np.float16)
    return a @ b.T


def rms_norm(x, w, eps=1e-6):
    """androidllm/models/llama.py:21-24 (fp32 result; callers cast to fp16)."""
    x = x.astype(np.float32)
    ms = np.mean(x * x, axis=-1, keepdims=True)
    return (x / np.sqrt(ms + eps)) * w.astype(np.float32)


def precompute_rope(head_dim, max_len, theta=10000.0):
    """androidllm/models/llama.py:27-31: float64 [cos | sin] table stored fp16."""
    inv = 1.0 / (theta ** (np.arange(0, head_dim, 2) / head_dim))
    ang = np.outer(np.arange(max_len), inv)
    return np.concatenate([np.cos(ang), np.sin(ang)], axis=1).astype(np.float16)


def apply_rope(x, pos, rope):
    """androidllm/models/llama.py:34-45: rotate-half in fp32."""
    half = x.shape[-1] // 2
    c = rope[pos, :half].astype(np.float32)
    s = rope[pos, half:].astype(np.float32)
    x = x.astype(np.float32)
    lo, hi = x[..., :half], x[..., half:]
    return np.concatenate([lo * c - hi * s, lo * s + hi * c], axis=-1)


def swiglu(gate, up):
    """androidllm/models/llama.py:48-50 (fp32)."""
    g = gate.astype(np.float32)
    return g * (1.0 / (1.0 + np.exp(-g))) * up.astype(np.float32)


class OracleModel:
    """Resident-weights model, numpy branch of ``androidllm/models/llama.py:57-164``."""

    def __init__(self, canon, embed, final_norm, lm_head=None):
        self.canon = canon
        self.hidden = canon["hidden"]
        self.heads = canon["heads"]
        self.kv_heads = canon["kv_heads"]
        self.head_dim = canon["head_dim"]
        self.eps = canon["rms_eps"]
        self.embed = embed
        self.final_norm = final_norm
        self.lm_head = lm_head
        self.rope = precompute_rope(self.head_dim, canon["max_len"], canon["rope_theta"])

    def prepare_kv(self, max_len):
        """llama.py:162-164: per-layer zeroed fp16 (max_len, kv_heads, head_dim) pairs."""
        shape = (max_len, self.kv_heads, self.head_dim)
        return [(np.zeros(shape, np.float16), np.zeros(shape, np.float16))
                for _ in range(self.canon["layers"])]

    def layer_forward(self, x, layer, kv, pos):
        """llama.py:96-128 for one row at ``pos``; mutates ``kv`` at ``pos``."""
        hd, nh, nkv = self.head_dim, self.heads, self.kv_heads
        q = matmul_f16(x, layer["q"]).reshape(1, nh, hd)
        k = matmul_f16(x, layer["k"]).reshape(1, nkv, hd)
        v = matmul_f16(x, layer["v"]).reshape(1, nkv, hd)
        q = apply_rope(q, pos, self.rope)
        k = apply_rope(k, pos, self.rope)
        kc, vc = kv
        kc[pos] = k[0].astype(np.float16)
        vc[pos] = v[0].astype(np.float16)
        grp = nh // nkv
        keys = np.repeat(kc[: pos + 1], grp, axis=1).transpose(1, 2, 0)
        vals = np.repeat(vc[: pos + 1], grp, axis=1).transpose(1, 0, 2)
        sc = (q[0][:, None, :].astype(np.float32) @ keys.astype(np.float32)) / math.sqrt(hd)
        p = np.exp(sc - np.max(sc, axis=-1, keepdims=True))
        p = p / np.sum(p, axis=-1, keepdims=True)
        ctx = (p.astype(np.float16) @ vals.astype(np.float16)).reshape(nh, hd)
        o = matmul_f16(ctx.reshape(1, self.hidden), layer["o"])
        x = x + o.reshape(1, self.hidden).astype(np.float16)
        x = rms_norm(x, layer["n_in"], self.eps).astype(np.float16)
        h = swiglu(matmul_f16(x, layer["gate"]), matmul_f16(x, layer["up"]))
        d = matmul_f16(h.reshape(1, -1), layer["down"])
        x = x + d.reshape(1, self.hidden).astype(np.float16)
        return rms_norm(x, layer["n_post"], self.eps).astype(np.float16)

    def head_weight(self):
        return self.lm_head if self.lm_head is not None else self.embed

    def logits(self, x):
        """llama.py:144-146: fp16-rounded logits returned as fp32."""
        h = rms_norm(x, self.final_norm, self.eps)
        return matmul_f16(h.astype(np.float16), self.head_weight()).astype(np.float32)

    def forward(self, layers, token, kv, pos):
        """androidllm/engine.py:255-264 + embedding lookup (engine.py:280)."""
        x = self.embed[token].reshape(1, self.hidden)
        for li, layer in enumerate(layers):
            x = self.layer_forward(x, layer, kv[li], pos)
        return x

    def verify_forward(self, layers, tokens, kv, pos0):
        """M consecutive single-row forwards; returns (M, hidden) fp16 states."""
        return np.concatenate([self.forward(layers, t, kv, pos0 + i)
                               for i, t in enumerate(tokens)], axis=0)
