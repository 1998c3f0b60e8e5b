"""Minimal safetensors reader/writer for androidllm shard files.

Format (``androidllm/safetensors.py:23-79``): an 8-byte little-endian header
length, a compact JSON header ``{name: {dtype, shape, data_offsets}}`` and the
raw tensors, each padded to 8 bytes.  Header key order follows insertion
order, so a writer that inserts tensors in the same order produces the same
bytes as androidllm's writer.
"""
import json
import struct

import numpy as np

DTYPES = {
    "F64": np.float64, "F32": np.float32, "F16": np.float16, "BF16": np.uint16,
    "I64": np.int64, "I32": np.int32, "I16": np.int16, "I8": np.int8,
    "U64": np.uint64, "U32": np.uint32, "U16": np.uint16, "U8": np.uint8,
    "BOOL": np.bool_,
}
NAMES = {np.dtype(v): k for k, v in DTYPES.items()}
_ALIGN = 8


def write(path, tensors):
    header, off = {}, 0
    arrays = []
    for name, arr in tensors.items():
        a = np.ascontiguousarray(arr)
        header[name] = {"dtype": NAMES[a.dtype], "shape": list(a.shape),
                        "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes + (-a.nbytes) % _ALIGN
        arrays.append(a)
    raw = json.dumps(header, separators=(",", ":")).encode("utf-8")
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        for a in arrays:
            f.write(a.tobytes())
            f.write(b"\x00" * ((-a.nbytes) % _ALIGN))


def read_header(path):
    with open(path, "rb") as f:
        head = f.read(8)
        if len(head) < 8:
            raise ValueError(f"not a safetensors file: {path}")
        (n,) = struct.unpack("<Q", head)
        header = json.loads(f.read(n))
    return header, 8 + n


def read_tensor(path, name, header=None):
    """Memory-mapped view of one tensor (no copy)."""
    h, start = read_header(path)
    meta = (header or h).get(name)
    if meta is None:
        raise KeyError(f"{name} not in {path}")
    a, _ = meta["data_offsets"]
    return np.memmap(path, dtype=DTYPES[meta["dtype"]], mode="r", offset=start + a,
                     shape=tuple(meta["shape"]))
