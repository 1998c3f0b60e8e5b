"""Oracle (test infrastructure): restatement of androidllm/quant.py.

Block-symmetric weight quantization along the input dimension.  All
functions follow the reference's numpy arithmetic exactly, so the oracle's
dequantized matrices are bit-identical to ``dequantize_packed``.
"""
import numpy as np


def quantize_matrix(w, bits=4, block=64):
    """androidllm/quant.py:4-22.

    Pads the input dim with zeros to a block multiple, takes the per-block
    absolute maximum, ``scale = fp16(amax / (2**(bits-1)-1))`` and
    ``q = clip(rint(w / f32(scale)))``.  A block whose scale rounds to 0 in
    fp16 (``quant.py:17`` replaces 0 by ``fp16(1e-8)``, which is again 0) makes
    ``w / 0`` NaN/inf; on x86 numpy turns that into INT_MIN, which the clip
    maps to the most negative code.  That case is restated explicitly.
    """
    w = np.asarray(w, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError("quantize_matrix expects a 2D matrix")
    n_out, n_in = w.shape
    rem = n_in % block
    if rem:
        w = np.concatenate([w, np.zeros((n_out, block - rem), np.float32)], axis=1)
    n_blocks = w.shape[1] // block
    blocks = w.reshape(n_out, n_blocks, block)
    qmax = 2 ** (bits - 1) - 1
    qmin = -(2 ** (bits - 1))
    amax = np.abs(blocks).max(axis=2, keepdims=True)
    scale16 = (amax / np.float32(qmax)).astype(np.float16)
    scale32 = scale16.astype(np.float32)
    zero = scale32 == 0
    with np.errstate(divide="ignore", invalid="ignore"):
        ratio = blocks / np.where(zero, np.float32(1), scale32)
    q = np.clip(np.rint(ratio), qmin, qmax).astype(np.int32)
    q = np.where(zero, np.int32(qmin), q)
    return q.reshape(n_out, n_blocks * block), scale16.reshape(n_out, n_blocks)


def pack_int4(q):
    """androidllm/quant.py:25-33: column 2j -> low nibble, 2j+1 -> high nibble."""
    q = np.asarray(q, dtype=np.int32)
    if q.size % 2:
        raise ValueError("int4 pack needs even element count")
    flat = (q.reshape(-1) & 0xF).astype(np.uint8)
    return (flat[0::2] | (flat[1::2] << 4)).reshape(q.shape[0], -1)


def unpack_int4(packed, out_dim, in_dim):
    """androidllm/quant.py:36-45: two's-complement nibbles back to int32."""
    b = np.asarray(packed, dtype=np.uint8).reshape(-1)
    vals = np.empty(b.size * 2, dtype=np.int32)
    vals[0::2] = b & 0xF
    vals[1::2] = b >> 4
    vals -= (vals >= 8) * 16
    return vals.reshape(out_dim, in_dim)


def dequantize_matrix(q, scale, bits=4):
    """androidllm/quant.py:48-55: fp16(f32(q) * f32(scale repeated per block))."""
    q = np.asarray(q)
    scale = np.asarray(scale, dtype=np.float32)
    block = q.shape[1] // scale.shape[1]
    return (q.astype(np.float32) * np.repeat(scale, block, axis=1)).astype(np.float16)


def dequantize_packed(packed, scale, meta):
    """androidllm/quant.py:58-65: the bit-exact dequant target.

    ``meta`` is one manifest entry ``{bits, block, out, in}``.  int8 weights are
    stored raw (``androidllm/shard.py:112``).
    """
    if meta["bits"] == 4:
        q = unpack_int4(packed, meta["out"], meta["in"]).astype(np.float32)
    else:
        q = np.asarray(packed).astype(np.float32)
    s = np.repeat(np.asarray(scale, dtype=np.float32), meta["block"], axis=1)
    return (q * s).astype(np.float16)
