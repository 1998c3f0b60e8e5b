"""Oracle (test infrastructure): restatement of androidllm/safetensors.py reads.

Only what the oracle needs to load a shard directory: the 8-byte
little-endian header length, the JSON header and raw little-endian tensors
(``androidllm/safetensors.py:45-79``), plus the engine's layer assembly
(``androidllm/engine.py:90-116,160-174``).
"""
import json
import os
import struct

import numpy as np

from . import quant

_DT = {"F64": np.float64, "F32": np.float32, "F16": np.float16, "BF16": np.uint16,
       "I64": np.int64, "I32": np.int32, "I16": np.int16, "I8": np.int8,
       "U64": np.uint64, "U32": np.uint32, "U16": np.uint16, "U8": np.uint8,
       "BOOL": np.bool_}


def read_all(path):
    """Return {name: ndarray} for one safetensors file (copies, not memmaps)."""
    with open(path, "rb") as f:
        (hlen,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(hlen))
        blob = f.read()
    out = {}
    for name, meta in header.items():
        a, b = meta["data_offsets"]
        out[name] = np.frombuffer(blob[a:b], dtype=_DT[meta["dtype"]]).reshape(meta["shape"]).copy()
    return out


def load_model(model_dir):
    """Load a shard dir with every layer dequantized to fp16 (resident).

    Mirrors ``androidllm/engine.py:90-116`` (embed / final norm / lm_head) and
    ``engine.py:160-174`` (per-layer dequant and the ``in_real`` slice).
    Returns ``(canon, embed, final_norm, lm_head_or_None, layers)``.
    """
    with open(os.path.join(model_dir, "manifest.json"), encoding="utf-8") as f:
        man = json.load(f)
    canon = man["config"]
    emb = read_all(os.path.join(model_dir, "embeddings.safetensors"))
    eq = man.get("embed_quant") or {}
    embed = quant.dequantize_packed(emb["embed.q"], emb["embed.scale"], eq) if eq else emb["embed"]
    final_norm = read_all(os.path.join(model_dir, "norms.safetensors"))["final_norm"]
    lm_head = None
    if man.get("has_lm_head"):
        lh = read_all(os.path.join(model_dir, "lm_head.safetensors"))
        lq = man.get("lm_head_quant") or {}
        lm_head = quant.dequantize_packed(lh["lm_head.q"], lh["lm_head.scale"], lq) if lq else lh["lm_head"]
    layers = []
    for i in range(canon["layers"]):
        t = read_all(os.path.join(model_dir, f"layer_{i}.safetensors"))
        layer = {}
        for base, qm in man["quant"]["layers"][str(i)].items():
            deq = quant.dequantize_packed(t[base + ".q"], t[base + ".scale"], qm)
            in_real = qm.get("in_real", qm["in"])
            layer[base] = deq[:, :in_real] if in_real != qm["in"] else deq
        layer["n_in"] = t["input_layernorm.weight"]
        layer["n_post"] = t["post_attention_layernorm.weight"]
        layers.append(layer)
    return canon, embed, final_norm, lm_head, layers
