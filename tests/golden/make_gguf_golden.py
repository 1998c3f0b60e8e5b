"""Generate gguf.npz by running the androidllm reference's GGUF reader
(androidllm/gguf.py GGUFReader.read_tensor) on the cases of gguf_cases.py.

    python tests/golden/make_gguf_golden.py --reference <androidllm checkout>

The reference's reader raises for any Q4_0 / Q4_1 / Q5_0 / Q5_1 tensor of
more than one 32-element block: it assigns the (blocks, 16) nibble arrays to a
flat slice (androidllm/gguf.py:178, :198), which numpy broadcasts only for a
single block.  Those tensors are therefore decoded here block by block through
the same reference functions (GGUFReader._q4 / _q5 on one block each, the way
the reference's tests/test_gguf.py:208 calls _q8), and the fixture records
that the whole-tensor read raises.  Q5_1 raises even for one block (the
reference reads its 4-byte high mask at byte 6 and its codes at bytes 10..26 of
a 24-byte block, gguf.py:194-196): no reference value exists for it and the
fixture records that instead.

The reference never travels with this repository: only the fixture does.
"""
import argparse
import hashlib
import io
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

from androidllm_b200 import gguf  # noqa: E402
from gguf_cases import BLOCK_SHAPE, BLOCK_TYPES, GGUF_MODELS, block_bytes, write_model  # noqa: E402


def sha(b):
    return hashlib.sha256(b).hexdigest()


_BLOCKWISE = {"Q4_0": (18, "_q4", False), "Q4_1": (20, "_q4", True), "Q5_0": (22, "_q5", False),
              "Q5_1": (24, "_q5", True)}


def ref_decode(reader_cls, r, name):
    """The reference's fp32 decode of one tensor, and whether its whole-tensor
    read raised (then decoded block by block with the reference's functions)."""
    try:
        return np.asarray(r.read_tensor(name), np.float32), False
    except ValueError:
        kind = gguf.TYPE_NAMES.get(r.tensors[name]["type"])
        if kind not in _BLOCKWISE:
            raise
    nbytes, fn, has_sum = _BLOCKWISE[kind]
    shape = tuple(reversed(r.tensors[name]["dims"]))
    n_blocks = int(np.prod(shape)) // 32
    r.f.seek(r.data_start + r.tensors[name]["offset"])
    raw = r.f.read(n_blocks * nbytes)
    dec = getattr(reader_cls, fn)
    try:
        vals = [dec(io.BytesIO(raw[i * nbytes:(i + 1) * nbytes]), (1, 32), has_sum) for i in range(n_blocks)]
    except ValueError:
        return None, True
    return np.concatenate(vals, axis=1).reshape(shape).astype(np.float32), True


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ANDROIDLLM_REFERENCE"),
                    help="androidllm checkout (default: $ANDROIDLLM_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or ANDROIDLLM_REFERENCE) is required")
    sys.path.insert(0, args.reference)
    from androidllm.gguf import GGUFReader

    out = {}
    by_name = {v: k for k, v in gguf.TYPE_NAMES.items()}
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "blocks.gguf")
        tensors = {f"t.{t}": gguf.RawTensor(by_name[t], block_bytes(t), BLOCK_SHAPE) for t in BLOCK_TYPES}
        gguf.write_gguf(path, {"general.architecture": "llama"}, tensors, dims64=False)
        with GGUFReader(path) as r:
            for t in BLOCK_TYPES:
                out[f"block_{t}_raw"] = np.frombuffer(block_bytes(t), np.uint8)
                val, raised = ref_decode(GGUFReader, r, f"t.{t}")
                if val is not None:
                    out[f"block_{t}_ref"] = val
                out[f"block_{t}_whole_read_raises"] = np.array(raised)
                out[f"block_{t}_reference_fails"] = np.array(val is None)
        for name in GGUF_MODELS:
            path = os.path.join(tmp, name + ".gguf")
            write_model(name, path)
            with open(path, "rb") as f:
                out[f"{name}_file_sha"] = np.array(sha(f.read()))
            names, hashes, raised = [], [], []
            with GGUFReader(path) as r:
                for tname in sorted(r.tensors):
                    val, rz = ref_decode(GGUFReader, r, tname)
                    names.append(tname)
                    hashes.append(sha(np.ascontiguousarray(val, np.float32).tobytes()))
                    raised.append(rz)
            out[f"{name}_tensors"] = np.array(names)
            out[f"{name}_f32_sha"] = np.array(hashes)
            out[f"{name}_whole_read_raises"] = np.array(raised)
    np.savez_compressed(os.path.join(HERE, "gguf.npz"), **out)
    print("gguf fixture written")


if __name__ == "__main__":
    main()
