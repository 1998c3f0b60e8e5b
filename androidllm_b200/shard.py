"""Shard directory writer (androidllm's layer-file + manifest layout).

Produces exactly the files ``androidllm/shard.py:67-152`` produces for the
same input tensors: ``layer_N.safetensors`` (``<base>.q``, ``<base>.scale``,
``input_layernorm.weight``, ``post_attention_layernorm.weight``),
``embeddings.safetensors``, ``norms.safetensors``, an optional
``lm_head.safetensors`` and ``manifest.json`` with per-projection
``{bits, block, out, in, in_real, packed}``.
"""
import json
import os
import shutil

import numpy as np

from . import safetensors
from .quant import codes_for_storage, quantize_matrix

_GLOBAL = {"embed_tokens.weight": "embed", "norm.weight": "final_norm",
           "lm_head.weight": "lm_head"}
_ATTN = ("self_attn.q_proj.weight", "self_attn.k_proj.weight",
         "self_attn.v_proj.weight", "self_attn.o_proj.weight")
_MLP = ("mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight")
_NORMS = ("input_layernorm.weight", "post_attention_layernorm.weight")


def classify(name):
    """HF tensor name -> (kind, key); same classes as androidllm/shard.py:41-56."""
    n = name[len("model."):] if name.startswith("model.") else name
    if n in _GLOBAL:
        return "global", _GLOBAL[n]
    if n.startswith("layers."):
        idx, _, sub = n[len("layers."):].partition(".")
        if sub in _ATTN:
            return "attn", (int(idx), sub[len("self_attn."):])
        if sub in _MLP:
            return "mlp", (int(idx), sub[len("mlp."):])
        if sub in _NORMS:
            return "norm", (int(idx), sub)
    return "other", None


def _quant_global(w, bits):
    q, s = quantize_matrix(w, bits=bits, block=w.shape[1])
    meta = {"bits": bits, "block": int(w.shape[1]), "out": int(w.shape[0]), "in": int(w.shape[1])}
    return codes_for_storage(q, bits), s.astype(np.float16), meta


def shard_from_tensors(source, canon, out, attn_bits=4, mlp_bits=8, block=64, embed_bits=8):
    """Quantize ``source`` ({HF name: array or zero-arg callable}) into ``out``."""
    os.makedirs(out, exist_ok=True)
    layers, qmeta, glob = {}, {}, {}
    embed_quant, head_quant = {}, {}
    for name, src in source.items():
        kind, key = classify(name)
        if kind == "other":
            continue
        w = np.ascontiguousarray(src() if callable(src) else src, dtype=np.float32)
        if kind == "global":
            if key in ("embed", "lm_head") and embed_bits:
                q, s, meta = _quant_global(w, embed_bits)
                glob[key + ".q"], glob[key + ".scale"] = q, s
                if key == "embed":
                    embed_quant = meta
                else:
                    head_quant = meta
            else:
                glob[key] = w.astype(np.float16)
            continue
        li, sub = key
        slot = layers.setdefault(li, {"weights": {}, "norms": {}})
        if kind == "norm":
            slot["norms"][sub] = w.astype(np.float16)
            continue
        bits = attn_bits if kind == "attn" else mlp_bits
        q, s = quantize_matrix(w, bits=bits, block=block)
        base = sub.split("_")[0]
        slot["weights"][base + ".q"] = codes_for_storage(q, bits)
        slot["weights"][base + ".scale"] = s.astype(np.float16)
        qmeta.setdefault(str(li), {})[base] = {
            "bits": bits, "block": block, "out": int(q.shape[0]), "in": int(q.shape[1]),
            "in_real": int(w.shape[1]), "packed": "U8" if bits == 4 else "I8"}
    for li in sorted(layers):
        tensors = dict(layers[li]["weights"])
        tensors.update(layers[li]["norms"])
        safetensors.write(os.path.join(out, f"layer_{li}.safetensors"), tensors)
    safetensors.write(os.path.join(out, "embeddings.safetensors"),
                      {k: v for k, v in glob.items() if k.startswith("embed")})
    safetensors.write(os.path.join(out, "norms.safetensors"), {"final_norm": glob["final_norm"]})
    if "lm_head" in glob or head_quant:
        safetensors.write(os.path.join(out, "lm_head.safetensors"),
                          {k: v for k, v in glob.items() if k.startswith("lm_head")})
    manifest = {
        "format": "androidllm/v1",
        "name": canon["name"],
        "config": canon,
        "quant": {"attn_bits": attn_bits, "mlp_bits": mlp_bits, "block": block, "layers": qmeta},
        "embed_quant": embed_quant,
        "lm_head_quant": head_quant,
        "tied": canon["tied"],
        "has_lm_head": bool(head_quant) or "lm_head" in glob,
    }
    with open(os.path.join(out, "manifest.json"), "w", encoding="utf-8") as f:
        json.dump(manifest, f, indent=2)
    return manifest


def _synth_layer_task(args):
    """Quantize and write one layer of a seeded synthetic model (worker)."""
    from . import synth
    canon, seed, out, li, attn_bits, mlp_bits, block = args
    specs = synth.tensor_specs(canon)
    weights, norms, meta = {}, {}, {}
    prefix = f"model.layers.{li}."
    for idx, (name, shape, kind) in enumerate(specs):
        if not name.startswith(prefix):
            continue
        w = synth.make_tensor(seed, idx, shape, kind)
        k, key = classify(name)
        if k == "norm":
            norms[key[1]] = w.astype(np.float16)
            continue
        bits = attn_bits if k == "attn" else mlp_bits
        q, sc = quantize_matrix(w, bits=bits, block=block)
        base = key[1].split("_")[0]
        weights[base + ".q"] = codes_for_storage(q, bits)
        weights[base + ".scale"] = sc.astype(np.float16)
        meta[base] = {"bits": bits, "block": block, "out": int(q.shape[0]), "in": int(q.shape[1]),
                      "in_real": int(w.shape[1]), "packed": "U8" if bits == 4 else "I8"}
    tensors = dict(weights)
    tensors.update(norms)
    safetensors.write(os.path.join(out, f"layer_{li}.safetensors"), tensors)
    return li, meta


def write_synthetic(canon, seed, out, attn_bits=4, mlp_bits=8, block=64, embed_bits=8, workers=8):
    """Write the seeded synthetic model of ``synth.synth_tensors(canon, seed)``
    as a shard directory, layers in parallel (spawned worker processes).
    Produces the same files as :func:`shard_from_tensors` on those tensors."""
    import multiprocessing as mp

    from . import synth
    os.makedirs(out, exist_ok=True)
    tasks = [(canon, seed, out, li, attn_bits, mlp_bits, block) for li in range(canon["layers"])]
    if workers > 1:
        with mp.get_context("spawn").Pool(workers) as pool:
            results = pool.map(_synth_layer_task, tasks)
    else:
        results = [_synth_layer_task(t) for t in tasks]
    qmeta = {str(li): meta for li, meta in sorted(results)}
    glob_src = {}
    for idx, (name, shape, kind) in enumerate(synth.tensor_specs(canon)):
        if classify(name)[0] == "global":
            glob_src[name] = (idx, shape, kind)
    glob, embed_quant, head_quant = {}, {}, {}
    for name, (idx, shape, kind) in glob_src.items():
        key = classify(name)[1]
        w = synth.make_tensor(seed, idx, shape, kind)
        if key in ("embed", "lm_head") and embed_bits:
            q, sc, meta = _quant_global(w, embed_bits)
            glob[key + ".q"], glob[key + ".scale"] = q, sc
            if key == "embed":
                embed_quant = meta
            else:
                head_quant = meta
        else:
            glob[key] = w.astype(np.float16)
        del w
    safetensors.write(os.path.join(out, "embeddings.safetensors"),
                      {k: v for k, v in glob.items() if k.startswith("embed")})
    safetensors.write(os.path.join(out, "norms.safetensors"), {"final_norm": glob["final_norm"]})
    if "lm_head" in glob or head_quant:
        safetensors.write(os.path.join(out, "lm_head.safetensors"),
                          {k: v for k, v in glob.items() if k.startswith("lm_head")})
    manifest = {
        "format": "androidllm/v1",
        "name": canon["name"],
        "config": canon,
        "quant": {"attn_bits": attn_bits, "mlp_bits": mlp_bits, "block": block, "layers": qmeta},
        "embed_quant": embed_quant,
        "lm_head_quant": head_quant,
        "tied": canon["tied"],
        "has_lm_head": bool(head_quant) or "lm_head" in glob,
    }
    with open(os.path.join(out, "manifest.json"), "w", encoding="utf-8") as f:
        json.dump(manifest, f, indent=2)
    return manifest


def prefix_draft(target_dir, draft_dir, n_layers, name=None):
    """A draft made of the target's first ``n_layers`` layers.

    It shares the target's embeddings, final norm and head (files are copied,
    so each directory stays a self-contained androidllm shard directory).
    """
    os.makedirs(draft_dir, exist_ok=True)
    with open(os.path.join(target_dir, "manifest.json"), encoding="utf-8") as f:
        man = json.load(f)
    canon = dict(man["config"])
    canon["layers"] = int(n_layers)
    canon["name"] = name or canon["name"] + f"-first{n_layers}"
    man["config"] = canon
    man["name"] = canon["name"]
    man["quant"] = dict(man["quant"])
    man["quant"]["layers"] = {str(i): man["quant"]["layers"][str(i)] for i in range(n_layers)}
    files = [f"layer_{i}.safetensors" for i in range(n_layers)]
    files += ["embeddings.safetensors", "norms.safetensors"]
    if man.get("has_lm_head"):
        files.append("lm_head.safetensors")
    for fn in files:
        shutil.copyfile(os.path.join(target_dir, fn), os.path.join(draft_dir, fn))
    with open(os.path.join(draft_dir, "manifest.json"), "w", encoding="utf-8") as f:
        json.dump(man, f, indent=2)
    return man
