"""GGUF loading on the host: every block type against the reference reader's
decode (tests/golden/gguf.npz, androidllm/gguf.py:134-206), the direct Q4_0 /
Q8_0 projections against the oracle's dequantization, the known-answer vector
of the reference's tests/test_gguf.py:208, both tensor-dimension widths,
both block orders and the errors."""
import hashlib
import os
import struct
import sys

import numpy as np
import pytest
from conftest import GOLDEN, golden

sys.path.insert(0, GOLDEN)
from gguf_cases import BLOCK_SHAPE, BLOCK_TYPES, GGUF_MODELS, GGUF_PROMPT, write_model  # noqa: E402

from androidllm_b200 import gguf  # noqa: E402
from oracle import quant as oquant  # noqa: E402

_BY_NAME = {v: k for k, v in gguf.TYPE_NAMES.items()}


def _sha(b):
    return hashlib.sha256(b).hexdigest()


@pytest.mark.parametrize("t", BLOCK_TYPES)
def test_block_decode_matches_reference(t):
    g = golden("gguf.npz")
    raw = g[f"block_{t}_raw"].tobytes()
    got = gguf.decode_blocks(_BY_NAME[t], raw, BLOCK_SHAPE[0] * BLOCK_SHAPE[1]).reshape(BLOCK_SHAPE)
    if bool(g[f"block_{t}_reference_fails"]):
        # the reference cannot read Q5_1 at all; check the layout directly:
        # d, m (fp16), 32-bit fifth-bit mask, 16 code bytes; value
        # ((interleaved code | bit e << 4) - 16) * d + m in the reference's order
        assert t == "Q5_1"
        blk = np.frombuffer(raw, np.uint8).reshape(-1, 24)
        exp = []
        for b in blk:
            d = float(np.frombuffer(b[0:2].tobytes(), np.float16)[0])
            m = float(np.frombuffer(b[2:4].tobytes(), np.float16)[0])
            qh = struct.unpack("<I", b[4:8].tobytes())[0]
            for e in range(32):
                byte = int(b[8 + e // 2])
                u = (byte & 0xF) if e % 2 == 0 else (byte >> 4)
                u |= ((qh >> e) & 1) << 4
                exp.append(np.float32(np.float32(u - 16) * np.float32(d)) + np.float32(m))
        assert np.array_equal(got.reshape(-1), np.array(exp, np.float32))
        return
    ref = g[f"block_{t}_ref"]
    assert got.dtype == np.float32 and np.array_equal(got.view(np.uint32), ref.view(np.uint32)), t


def test_q8_1_known_answer():
    """androidllm tests/test_gguf.py:208-226: two Q8_1 blocks, value q d + s."""
    d = np.array([2.0, 0.5], np.float16)
    s = np.array([0.25, -0.125], np.float16)
    q = np.array([1, -2, 3, -4, 5, -6, 7, -8] + [0] * 8 + [9, -9, 8, -8, 7, -7, 6, -6, 5, -5, 4, -4, 3, -3, 2, -2]
                 + [1] * 16 + [-1] * 16, np.int8).reshape(2, 32)
    raw = b"".join(d[i:i + 1].tobytes() + s[i:i + 1].tobytes() + q[i].tobytes() for i in range(2))
    got = gguf.decode_blocks(gguf.T_Q8_1, raw, 64).reshape(2, 32)
    exp = q.astype(np.float32) * d[:, None].astype(np.float32) + s[:, None].astype(np.float32)
    assert np.array_equal(got, exp)
    # llama.cpp keeps a sum, not an offset, in the second half
    assert np.array_equal(gguf.decode_blocks(gguf.T_Q8_1, raw, 64, order="ggml").reshape(2, 32),
                          q.astype(np.float32) * d[:, None].astype(np.float32))


@pytest.mark.parametrize("name", sorted(GGUF_MODELS))
def test_model_tensors_match_reference(tmp_path, name):
    g = golden("gguf.npz")
    path = str(tmp_path / f"{name}.gguf")
    write_model(name, path)
    with open(path, "rb") as f:
        assert _sha(f.read()) == str(g[f"{name}_file_sha"]), "the GGUF writer changed: regenerate gguf.npz"
    gf = gguf.GGUFFile(path)
    names = [str(x) for x in g[f"{name}_tensors"]]
    assert sorted(gf.tensors) == names
    for tname, h in zip(names, g[f"{name}_f32_sha"]):
        val = gf.read_f32(tname)
        assert _sha(np.ascontiguousarray(val, np.float32).tobytes()) == str(h), tname
        if gf.tensors[tname]["type"] in (gguf.T_Q4_0, gguf.T_Q8_0):
            p = gf.projection(tname)
            assert p.block == 32 and p.bits == (4 if gf.tensors[tname]["type"] == gguf.T_Q4_0 else 8)
            deq = oquant.dequantize_packed(p.packed, p.scale, {"bits": p.bits, "block": p.block,
                                                                "out": p.out, "in": p.in_})
            # the device's dequantization is the oracle's: fp16 of the reference's fp32 value
            assert np.array_equal(deq.view(np.uint16), val.astype(np.float16).view(np.uint16)), tname
    canon, _ = GGUF_MODELS[name]
    c = gf.canon()
    for k in ("hidden", "layers", "heads", "kv_heads", "head_dim", "intermediate", "vocab", "max_len", "tied"):
        assert c[k] == canon[k], k
    assert c["rope_theta"] == pytest.approx(canon["rope_theta"]) and c["rms_eps"] == pytest.approx(canon["rms_eps"])
    assert max(GGUF_PROMPT) < canon["vocab"]


def test_dims_width_and_block_order(tmp_path):
    """64-bit (GGUF specification) and 32-bit dimensions read the same; a file
    written in llama.cpp's nibble order and read with order="ggml" gives the
    same projections as the reference order."""
    a32, a64, ag = (str(tmp_path / f) for f in ("a32.gguf", "a64.gguf", "ag.gguf"))
    write_model("gguf_b", a32)
    write_model("gguf_b", a64, dims64=True)
    write_model("gguf_b", ag, order="ggml", dims64=True)
    f32, f64, fg = gguf.GGUFFile(a32), gguf.GGUFFile(a64), gguf.GGUFFile(ag, order="ggml")
    assert f32.tensors.keys() == f64.tensors.keys() == fg.tensors.keys()
    for name in f32.tensors:
        assert f32.tensors[name]["dims"] == f64.tensors[name]["dims"]
        assert np.array_equal(f32.read_f32(name), f64.read_f32(name))
        assert np.array_equal(f32.read_f32(name), fg.read_f32(name)), name
        if f32.tensors[name]["type"] == gguf.T_Q4_0:
            assert np.array_equal(f32.projection(name).packed, fg.projection(name).packed)
            assert not np.array_equal(gguf.GGUFFile(ag).projection(name).packed, fg.projection(name).packed)


def test_errors(tmp_path):
    p = str(tmp_path / "x.gguf")
    with open(p, "wb") as f:
        f.write(b"GGML" + b"\0" * 64)
    with pytest.raises(ValueError, match="not a GGUF"):
        gguf.GGUFFile(p)
    with open(p, "wb") as f:
        f.write(b"GGUF" + struct.pack("<IQQ", 2, 0, 0))
    with pytest.raises(ValueError, match="version"):
        gguf.GGUFFile(p)
    # a K-quant tensor (Q4_K = 12) is rejected when read, with the supported list
    head = b"GGUF" + struct.pack("<IQQ", 3, 1, 1)
    key = b"general.architecture"
    head += struct.pack("<Q", len(key)) + key + struct.pack("<IQ", 8, 5) + b"llama"
    nm = b"blk.0.attn_q.weight"
    head += struct.pack("<Q", len(nm)) + nm + struct.pack("<IQQIQ", 2, 256, 4, 12, 0)
    head += b"\0" * ((-len(head)) % 32) + b"\0" * 1024
    with open(p, "wb") as f:
        f.write(head)
    gf = gguf.GGUFFile(p)
    with pytest.raises(ValueError, match="unsupported GGML type 12"):
        gf.projection("blk.0.attn_q.weight")
    with pytest.raises(ValueError, match="unsupported GGUF architecture"):
        write_model("gguf_a", p)
        bad = gguf.GGUFFile(p)
        bad.meta["general.architecture"] = "gpt2"
        bad.canon()
    with pytest.raises(ValueError, match="block order|order must"):
        gguf.GGUFFile(p, order="llama")
    assert os.path.exists(p)
