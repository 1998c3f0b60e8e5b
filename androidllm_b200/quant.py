"""androidllm block-quant format (host side: the shard producer).

The on-disk format is androidllm's (``androidllm/quant.py:4-65``,
``androidllm/shard.py:109-120``), kept unchanged so existing shard
directories load as they are:

* weights ``(out, in)`` are zero-padded along ``in`` to a multiple of
  ``block`` and split into blocks of ``block`` columns;
* per (row, block): ``scale = fp16(max|w| / (2**(bits-1) - 1))`` and
  ``q = clip(round_half_even(w / f32(scale)))``;
* int4 codes are packed two per byte, column ``2j`` in the low nibble;
  int8 codes are stored as raw ``int8``;
* dequantized weight = ``fp16(f32(q) * f32(scale))``.

This module only produces the format (quantize + pack).  Dequantization and
every matmul run on the GPU through :mod:`androidllm_b200.ops`.
"""
import numpy as np


def quantize_matrix(w, bits=4, block=64):
    """Quantize ``w (out, in)`` -> ``(q int32 (out, in_padded), scale fp16)``.

    Same codes and scales as ``androidllm/quant.py:4-22``, including the
    all-zero block case: its fp16 scale underflows to 0 and every code of the
    block becomes the most negative one, which dequantizes to -0.0.
    """
    w = np.asarray(w, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError("quantize_matrix expects a 2D matrix")
    rows, cols = w.shape
    padded = -(-cols // block) * block
    if padded != cols:
        w = np.pad(w, ((0, 0), (0, padded - cols)))
    nb = padded // block
    wb = w.reshape(rows, nb, block)
    lim = 2 ** (bits - 1)
    scale = (np.max(np.abs(wb), axis=2) / np.float32(lim - 1)).astype(np.float16)
    s32 = scale.astype(np.float32)[:, :, None]
    dead = s32 == 0
    with np.errstate(divide="ignore", invalid="ignore"):
        codes = np.rint(wb / np.where(dead, np.float32(1), s32))
    np.clip(codes, -lim, lim - 1, out=codes)
    codes = np.where(dead, np.float32(-lim), codes).astype(np.int32)
    return codes.reshape(rows, padded), scale


def pack_int4(q):
    """Two's-complement nibbles, even column in the low nibble (quant.py:25-33)."""
    q = np.asarray(q)
    if q.size % 2:
        raise ValueError("int4 pack needs even element count")
    u = (q.astype(np.int32) & 0xF).astype(np.uint8).reshape(q.shape[0], -1, 2)
    return u[:, :, 0] | (u[:, :, 1] << 4)


def unpack_int4(packed, out_dim, in_dim):
    """Inverse of :func:`pack_int4` (quant.py:36-45)."""
    b = np.asarray(packed, dtype=np.uint8).reshape(out_dim, -1)
    lo = (b & 0xF).astype(np.int8)
    hi = (b >> 4).astype(np.int8)
    q = np.stack([lo, hi], axis=2).reshape(out_dim, in_dim).astype(np.int32)
    return np.where(q >= 8, q - 16, q)


def codes_for_storage(q, bits):
    """What ``shard.py:112`` writes: packed uint8 for int4, raw int8 otherwise."""
    return pack_int4(q) if bits == 4 else np.asarray(q).astype(np.int8)
