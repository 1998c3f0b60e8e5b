"""GGUF (v3) files loaded straight into device weights.

The reference converts a GGUF file to its shard format by dequantizing every
tensor to fp32 and quantizing it again to 64-column blocks
(androidllm/gguf.py:155-185, 322).  Two GGML block formats are already the
symmetric block quantization the device kernels run on, only with
32-element blocks, so this loader keeps them as they are:

* Q4_0 (18-byte blocks: fp16 d, 16 bytes of 4-bit codes u, value (u - 8) d)
  becomes an int4 projection with 32-column blocks: the code bytes become the
  packed int4 bytes (u ^ 8 is the two's-complement nibble of u - 8), d the
  block scale;
* Q8_0 (34-byte blocks: fp16 d, 32 int8 q, value q d) becomes an int8
  projection with 32-column blocks.

The device dequantizes every such weight to fp16(f32(q) * f32(d)), the fp16
rounding of the value the reference's reader computes in fp32; no second
quantization happens.  F16 / F32 tensors load as fp16.  BF16, Q4_1, Q5_0,
Q5_1 and Q8_1 tensors, which the reference also reads, are decoded on the
host to fp32 with the reference reader's arithmetic and load as fp16.

Element order inside a 4/5-bit block.  The reference's reader puts element
2j in the low nibble of byte j and element 2j + 1 in the high one
(androidllm/gguf.py:179-205), adds the second fp16 of a Q4_1 / Q8_1 block to
every value and centres Q4_1 codes on 8.  llama.cpp's own files put element
j in the low nibble and element j + 16 in the high one, do not centre Q4_1
codes, and keep a sum, not an offset, in Q8_1's second half.  Both read a
Q5 element e's fifth bit from bit e of the block's 32-bit mask.
``order="reference"`` (the default) reads a file the way the reference does;
``order="ggml"`` reads it the way llama.cpp writes it.

Tensor infos may store their dimensions as 64-bit integers (the GGUF
specification) or 32-bit ones (what the reference's reader and its tests'
writer use); both are read.
"""
import os
import struct

import numpy as np

from .ops import DeviceModel, QuantProj

GGUF_ALIGNMENT = 32
T_F32, T_F16, T_Q4_0, T_Q4_1, T_Q5_0, T_Q5_1, T_Q8_0, T_Q8_1, T_BF16 = 0, 1, 2, 3, 6, 7, 8, 9, 30
TYPE_NAMES = {T_F32: "F32", T_F16: "F16", T_Q4_0: "Q4_0", T_Q4_1: "Q4_1", T_Q5_0: "Q5_0", T_Q5_1: "Q5_1",
              T_Q8_0: "Q8_0", T_Q8_1: "Q8_1", T_BF16: "BF16"}
ORDERS = ("reference", "ggml")
_BLOCK = 32
_BLOCK_BYTES = {T_Q4_0: 18, T_Q4_1: 20, T_Q5_0: 22, T_Q5_1: 24, T_Q8_0: 34, T_Q8_1: 36}
_ELEM_BYTES = {T_F32: 4, T_F16: 2, T_BF16: 2}

_SCALAR = {0: ("<B", 1), 1: ("<b", 1), 2: ("<H", 2), 3: ("<h", 2), 4: ("<I", 4), 5: ("<i", 4), 6: ("<f", 4),
           7: ("<?", 1), 10: ("<Q", 8), 11: ("<q", 8), 12: ("<d", 8)}
_STRING, _ARRAY = 8, 9

# GGUF tensor names of one block -> shard layer names (androidllm/gguf.py:211-224)
_LAYER_NAMES = {"attn_q": "q", "attn_k": "k", "attn_v": "v", "attn_output": "o", "ffn_gate": "gate",
                "ffn_up": "up", "ffn_down": "down", "attn_norm": "n_in", "ffn_norm": "n_post"}
# androidllm/gguf.py:226-227
SUPPORTED_ARCH = ("llama", "mistral", "qwen2", "qwen3", "phi3", "starcoder2", "minicpm", "deepseek2")


class _Buf:
    def __init__(self, data):
        self.d = data
        self.p = 0

    def take(self, n):
        if n < 0 or self.p + n > len(self.d):
            raise ValueError("truncated GGUF file")
        b = self.d[self.p:self.p + n]
        self.p += n
        return bytes(b)

    def unpack(self, fmt, n):
        return struct.unpack(fmt, self.take(n))[0]

    def string(self):
        return self.take(self.unpack("<Q", 8)).decode("utf-8", errors="replace")

    def value(self, tag):
        if tag == _STRING:
            return self.string()
        if tag == _ARRAY:
            etag = self.unpack("<I", 4)
            count = self.unpack("<Q", 8)
            return [self.value(etag) for _ in range(count)]
        if tag not in _SCALAR:
            raise ValueError(f"unsupported GGUF value type {tag}")
        fmt, n = _SCALAR[tag]
        return self.unpack(fmt, n)


def tensor_bytes(gtype, dims):
    """Bytes of a tensor of GGML type ``gtype`` with GGUF dims (innermost first)."""
    n = int(np.prod(dims))
    if gtype in _BLOCK_BYTES:
        if n % _BLOCK:
            raise ValueError(f"{TYPE_NAMES[gtype]} tensor of {n} elements is not whole 32-element blocks")
        return n // _BLOCK * _BLOCK_BYTES[gtype]
    if gtype in _ELEM_BYTES:
        return n * _ELEM_BYTES[gtype]
    raise ValueError(f"unsupported GGML type {gtype} (supported: {', '.join(TYPE_NAMES.values())}); "
                     "re-export the model as fp16, Q8_0 or Q4_0")


def _codes_4bit(nib, order):
    """(n, 16) code bytes -> (n, 32) codes 0..15 in element order."""
    lo, hi = nib & 0x0F, nib >> 4
    if order == "ggml":
        return np.concatenate([lo, hi], axis=1)
    u = np.empty((nib.shape[0], 32), np.uint8)
    u[:, 0::2], u[:, 1::2] = lo, hi
    return u


def decode_blocks(gtype, raw, n_elems, order="reference"):
    """Raw bytes of a GGML tensor -> fp32 values in element order
    (androidllm/gguf.py:134-206 for ``order="reference"``)."""
    if order not in ORDERS:
        raise ValueError(f"order must be one of {ORDERS}")
    if gtype == T_F32:
        return np.frombuffer(raw, np.float32, n_elems).copy()
    if gtype == T_F16:
        return np.frombuffer(raw, np.float16, n_elems).astype(np.float32)
    if gtype == T_BF16:
        return (np.frombuffer(raw, np.uint16, n_elems).astype(np.uint32) << 16).view(np.float32)
    if gtype not in _BLOCK_BYTES:
        tensor_bytes(gtype, (n_elems,))
    nb = n_elems // _BLOCK
    buf = np.frombuffer(raw, np.uint8, nb * _BLOCK_BYTES[gtype]).reshape(nb, -1)
    d = buf[:, 0:2].copy().view(np.float16).astype(np.float32)
    second = buf[:, 2:4].copy().view(np.float16).astype(np.float32)
    if gtype in (T_Q8_0, T_Q8_1):
        q = buf[:, 2:34] if gtype == T_Q8_0 else buf[:, 4:36]
        deq = q.view(np.int8).astype(np.float32) * d
        if gtype == T_Q8_1 and order == "reference":
            deq = deq + second
        return deq.reshape(-1)
    if gtype in (T_Q4_0, T_Q4_1):
        u = _codes_4bit(buf[:, 2:18] if gtype == T_Q4_0 else buf[:, 4:20], order).astype(np.int32)
        if gtype == T_Q4_0 or order == "reference":
            u = u - 8
        deq = u.astype(np.float32) * d
        if gtype == T_Q4_1:
            deq = deq + second
        return deq.reshape(-1)
    off = 2 if gtype == T_Q5_0 else 4
    qh = buf[:, off:off + 4].copy().view(np.uint32).reshape(-1, 1)
    fifth = ((qh >> np.arange(32, dtype=np.uint32)[None, :]) & 1).astype(np.int32)
    u = _codes_4bit(buf[:, off + 4:off + 20], order).astype(np.int32) + fifth * 16
    if gtype == T_Q5_0 or order == "reference":
        u = u - 16
    deq = u.astype(np.float32) * d
    if gtype == T_Q5_1:
        deq = deq + second
    return deq.reshape(-1)


class GGUFFile:
    """Header, metadata and tensor table of a GGUF v3 file (data memory-mapped).

    ``order`` chooses how 4/5-bit blocks are read ("reference" or "ggml")."""

    def __init__(self, path, order="reference"):
        if order not in ORDERS:
            raise ValueError(f"order must be one of {ORDERS}")
        self.path = path
        self.order = order
        self._mm = np.memmap(path, dtype=np.uint8, mode="r")
        b = _Buf(self._mm)
        if b.take(4) != b"GGUF":
            raise ValueError(f"not a GGUF file: {path}")
        version = b.unpack("<I", 4)
        if version != 3:
            raise ValueError(f"unsupported GGUF version {version} (want 3)")
        n_tensors = b.unpack("<Q", 8)
        n_kv = b.unpack("<Q", 8)
        self.meta = {}
        for _ in range(n_kv):
            key = b.string()
            self.meta[key] = b.value(b.unpack("<I", 4))
        start = b.p
        size = os.path.getsize(path)
        for dim_fmt, dim_size in (("<Q", 8), ("<I", 4)):
            b.p = start
            try:
                tensors = {}
                for _ in range(n_tensors):
                    name = b.string()
                    n_dim = b.unpack("<I", 4)
                    if not 1 <= n_dim <= 4:
                        raise ValueError("bad tensor rank")
                    dims = tuple(int(b.unpack(dim_fmt, dim_size)) for _ in range(n_dim))
                    gtype = b.unpack("<I", 4)
                    tensors[name] = {"dims": dims, "type": gtype, "offset": b.unpack("<Q", 8)}
                data_start = (b.p + GGUF_ALIGNMENT - 1) // GGUF_ALIGNMENT * GGUF_ALIGNMENT
                if all(t["type"] not in TYPE_NAMES or
                       data_start + t["offset"] + tensor_bytes(t["type"], t["dims"]) <= size
                       for t in tensors.values()):
                    self.tensors, self.data_start = tensors, data_start
                    break
            except (ValueError, struct.error, OverflowError):
                continue
        else:
            raise ValueError(f"cannot read the tensor table of {path}")

    def type_name(self, name):
        t = self.tensors[name]["type"]
        return TYPE_NAMES.get(t, str(t))

    def raw(self, name):
        t = self.tensors[name]
        a = self.data_start + t["offset"]
        return self._mm[a:a + tensor_bytes(t["type"], t["dims"])]

    def shape(self, name):
        return tuple(reversed(self.tensors[name]["dims"]))

    def read_f32(self, name):
        """Any supported tensor dequantized to fp32 (androidllm/gguf.py:134-153)."""
        t = self.tensors[name]
        shape = self.shape(name)
        return decode_blocks(t["type"], self.raw(name).tobytes(), int(np.prod(shape)), self.order).reshape(shape)

    def projection(self, name):
        """The tensor as a shard-format projection (rows = output features):
        Q4_0 / Q8_0 blocks as int4 / int8 with 32-column blocks, the rest fp16."""
        gtype = self.tensors[name]["type"]
        shape = self.shape(name)
        if len(shape) != 2:
            raise ValueError(f"{name}: a projection must be 2-D, got {shape}")
        out, inp = shape
        if gtype in (T_Q4_0, T_Q8_0):
            blk = np.asarray(self.raw(name)).reshape(out, inp // _BLOCK, _BLOCK_BYTES[gtype])
            d = np.ascontiguousarray(blk[:, :, 0:2]).view(np.float16).reshape(out, inp // _BLOCK)
            if gtype == T_Q8_0:
                q = np.ascontiguousarray(blk[:, :, 2:34]).view(np.int8).reshape(out, inp)
                return QuantProj(q, d, 8, _BLOCK, out, inp)
            nib = blk[:, :, 2:18].reshape(-1, 16)
            if self.order == "ggml":
                u = _codes_4bit(nib, "ggml")
                nib = u[:, 0::2] | (u[:, 1::2] << 4)
            packed = (nib ^ np.uint8(0x88)).reshape(out, inp // 2)
            return QuantProj(packed, d, 4, _BLOCK, out, inp)
        return QuantProj.from_fp16(self.fp16(name))

    def fp16(self, name):
        """Any supported tensor as fp16 (Q4_0 / Q8_0 rounded the way the device rounds them)."""
        if self.tensors[name]["type"] == T_F16:
            return np.asarray(self.raw(name)).view(np.float16).reshape(self.shape(name))
        return self.read_f32(name).astype(np.float16)

    def canon(self):
        """androidllm canon config from the metadata (androidllm/gguf.py:230-262;
        tied when there is no output.weight, gguf.py:325-328)."""
        arch = self.meta.get("general.architecture")
        if not arch or arch not in SUPPORTED_ARCH:
            raise ValueError(f"unsupported GGUF architecture: {arch!r} "
                             f"(supported: {', '.join(sorted(SUPPORTED_ARCH))})")

        def get(key, default=0):
            return self.meta.get(f"{arch}.{key}", default)
        hidden = int(get("embedding_length"))
        heads = int(get("attention.head_count"))
        kv_heads = int(get("attention.head_count_kv", heads) or heads)
        vocab = int(get("vocab_size") or 0) or self.shape("token_embd.weight")[0]
        return {"model_type": arch if arch in ("qwen2", "qwen3") else "llama", "hidden": hidden,
                "layers": int(get("block_count")), "heads": heads, "kv_heads": kv_heads,
                "head_dim": hidden // heads, "intermediate": int(get("feed_forward_length")), "vocab": vocab,
                "rope_theta": float(get("rope.freq_base", 10000.0) or 10000.0),
                "rms_eps": float(get("attention.layer_norm_rms_epsilon", 1e-5) or 1e-5),
                "max_len": int(get("attention.max_position_embeddings", 2048) or 2048),
                "tied": "output.weight" not in self.tensors,
                "name": self.meta.get("general.name") or arch}

    def layer(self, i):
        """Block i as {q, k, v, o, gate, up, down: QuantProj, n_in, n_post: fp16}."""
        out = {}
        for gname, base in _LAYER_NAMES.items():
            name = f"blk.{i}.{gname}.weight"
            if name not in self.tensors:
                raise ValueError(f"GGUF has no tensor {name}")
            out[base] = self.fp16(name).reshape(-1) if base in ("n_in", "n_post") else self.projection(name)
        return out


def device_model_from_gguf(ctx, path, max_len=None, order="reference"):
    """Load a GGUF file's model onto the context's device: Q4_0 / Q8_0 blocks
    as they are, everything else as fp16.  The reference's equivalent is
    convert_gguf followed by loading the shards (androidllm/gguf.py:322)."""
    g = GGUFFile(path, order)
    canon = g.canon()
    if max_len:
        canon["max_len"] = int(max_len)
    m = DeviceModel(ctx, canon)
    m.gguf = g
    for i in range(canon["layers"]):
        m.set_layer(i, g.layer(i))
    if g.tensors["token_embd.weight"]["type"] in (T_Q4_0, T_Q8_0):
        p = g.projection("token_embd.weight")
        m.set_embed(p.packed, p.scale, p.bits, p.block)
    else:
        m.set_embed(g.fp16("token_embd.weight"))
    m.set_final_norm(g.fp16("output_norm.weight").reshape(-1))
    if "output.weight" in g.tensors:
        m.set_head(g.projection("output.weight"))
    m.finalize()
    return m


# ---- writing (tests and tooling) ----------------------------------------------
def quantize_q8_0(w):
    """(out, in) fp32 -> Q8_0 blocks (out, in / 32, 34): d = fp16(max|w| / 127),
    q = round(w / d) (a zero block gets d = 0, q = 0)."""
    w = np.asarray(w, np.float32)
    b = w.reshape(w.shape[0], -1, _BLOCK)
    d = (np.max(np.abs(b), axis=-1) / 127.0).astype(np.float16)
    dd = d.astype(np.float32)[..., None]
    q = np.clip(np.round(np.divide(b, dd, out=np.zeros_like(b), where=dd != 0)), -127, 127).astype(np.int8)
    out = np.empty(b.shape[:2] + (34,), np.uint8)
    out[..., 0:2] = d[..., None].view(np.uint8).reshape(d.shape + (2,))
    out[..., 2:] = q.view(np.uint8)
    return out


def quantize_q4_0(w, order="reference"):
    """(out, in) fp32 -> Q4_0 blocks (out, in / 32, 18): d = fp16(max|w| / 7.5),
    codes round(w / d) + 8 clipped to 0..15, nibbles in ``order``."""
    w = np.asarray(w, np.float32)
    b = w.reshape(w.shape[0], -1, _BLOCK)
    d = (np.max(np.abs(b), axis=-1) / 7.5).astype(np.float16)
    dd = d.astype(np.float32)[..., None]
    u = np.clip(np.round(np.divide(b, dd, out=np.zeros_like(b), where=dd != 0)) + 8, 0, 15).astype(np.uint8)
    out = np.empty(b.shape[:2] + (18,), np.uint8)
    out[..., 0:2] = d[..., None].view(np.uint8).reshape(d.shape + (2,))
    if order == "ggml":
        out[..., 2:] = u[..., :16] | (u[..., 16:] << 4)
    else:
        out[..., 2:] = u[..., 0::2] | (u[..., 1::2] << 4)
    return out


class RawTensor:
    """A tensor given as its GGML bytes; ``shape`` is (rows, cols) in numpy order."""

    def __init__(self, gtype, data, shape):
        self.gtype, self.data, self.shape = int(gtype), bytes(data), tuple(int(s) for s in shape)
        if len(self.data) != tensor_bytes(self.gtype, tuple(reversed(self.shape))):
            raise ValueError("raw tensor size does not match its type and shape")


def write_gguf(path, meta, tensors, dims64=True, order="reference"):
    """Write a GGUF v3 file.  meta: {key: str | bool | int | float | list[str]};
    tensors: {name: RawTensor | (type, array)} with array (out, in) fp32 for
    Q4_0 / Q8_0 / F32 and fp16 for F16.  dims64=False writes 32-bit dimensions
    like the reference's tests."""
    def s(x):
        e = x.encode("utf-8")
        return struct.pack("<Q", len(e)) + e

    def val(v):
        if isinstance(v, str):
            return struct.pack("<I", _STRING) + s(v)
        if isinstance(v, bool):
            return struct.pack("<I", 7) + struct.pack("<?", v)
        if isinstance(v, int):
            return struct.pack("<I", 4) + struct.pack("<I", v)
        if isinstance(v, list):
            return struct.pack("<IIQ", _ARRAY, _STRING, len(v)) + b"".join(s(x) for x in v)
        return struct.pack("<I", 6) + struct.pack("<f", float(v))

    blobs, infos, off = [], [], 0
    for name, spec in tensors.items():
        if isinstance(spec, RawTensor):
            gtype, data, shape = spec.gtype, spec.data, spec.shape
        else:
            gtype, arr = spec
            arr = np.asarray(arr)
            shape = arr.shape
            if gtype == T_Q4_0:
                data = quantize_q4_0(arr, order).tobytes()
            elif gtype == T_Q8_0:
                data = quantize_q8_0(arr).tobytes()
            elif gtype == T_F16:
                data = np.ascontiguousarray(arr, np.float16).tobytes()
            elif gtype == T_F32:
                data = np.ascontiguousarray(arr, np.float32).tobytes()
            else:
                raise ValueError(f"write_gguf quantizes only Q4_0 / Q8_0; pass "
                                 f"{TYPE_NAMES.get(gtype, gtype)} as a RawTensor")
        dims = tuple(reversed(shape))
        dfmt = "<" + ("Q" if dims64 else "I") * len(dims)
        infos.append(s(name) + struct.pack("<I", len(dims)) + struct.pack(dfmt, *dims) +
                     struct.pack("<IQ", gtype, off))
        pad = (-len(data)) % GGUF_ALIGNMENT
        blobs.append(data + b"\x00" * pad)
        off += len(data) + pad
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(meta))
    head += b"".join(s(k) + val(v) for k, v in meta.items()) + b"".join(infos)
    head += b"\x00" * ((-len(head)) % GGUF_ALIGNMENT)
    with open(path, "wb") as f:
        f.write(head)
        for bl in blobs:
            f.write(bl)


__all__ = ["GGUFFile", "RawTensor", "decode_blocks", "device_model_from_gguf", "quantize_q4_0", "quantize_q8_0",
           "tensor_bytes", "write_gguf", "ORDERS", "TYPE_NAMES", "SUPPORTED_ARCH"]
