"""Tensor-parallel shards of an androidllm model (one process per GPU).

The reference runs every matrix whole in one process
(androidllm/models/llama.py:97-127).  A larger model (the Qwen2.5-7B shape)
is split over the ranks of one node instead:

* attention by heads: each rank keeps a contiguous range of query heads and
  the kv heads they read.  With at least as many kv heads as ranks, each rank
  gets kv_heads / world whole GQA groups; with more ranks than kv heads,
  world / kv_heads ranks share a kv head (each keeps a copy) and split its
  group's query heads as evenly as they go (28 heads over 8 ranks: 4,4,3,4,
  4,3,... by group);
* q, k, v rows of those heads and o columns (its K) of them;
* the FFN by 64-column blocks of the down projection's K: gate and up rows
  and down columns of the same FFN indices;
* the LM head by vocabulary rows (vocab / world each); the embedding stays
  whole on every rank.

Slicing works on the shard format itself (packed int4 / int8 codes and their
fp16 block scales): a column slice on block boundaries keeps each block's
scale, so every rank's dequantized weights are exactly the corresponding
slice of the whole model's.  The device side (alm_model_set_tp) sums the
row-split projections' fp32 partials over the ranks and gathers the head's
per-rank argmax.
"""
import os

import numpy as np

from . import safetensors
from ._lib import check, lib, ptr
from .ops import DeviceModel, QuantProj, load_manifest, read_layer


def nccl_unique_id():
    """A fresh NCCL unique id (128 bytes) for rank 0 to hand to every rank."""
    buf = np.zeros(128, np.uint8)
    check(lib.alm_nccl_unique_id(ptr(buf)))
    return bytes(buf)


def init_context_tp(ctx, rank, world, uid):
    """Join the NCCL communicator of `world` ranks on this context."""
    buf = np.frombuffer(bytes(uid), dtype=np.uint8).copy()
    if buf.size != 128:
        raise ValueError("NCCL unique id must be 128 bytes")
    check(lib.alm_ctx_init_tp(ctx.h, int(rank), int(world), ptr(buf)))


def enable_p2p(ctx, row_floats):
    """Switch the row-split projections' all-reduce from NCCL to the peer-memory
    kernel (alm_tp_p2p_*): every rank opens its receive area, the CUDA IPC
    handles are exchanged over torch.distributed, every rank maps the others'.
    Collective: every rank calls it after init_context_tp, before a forward."""
    import torch.distributed as dist
    h = np.zeros(64, np.uint8)
    check(lib.alm_tp_p2p_open(ctx.h, int(row_floats), ptr(h)))
    handles = [None] * dist.get_world_size()
    dist.all_gather_object(handles, bytes(h))
    buf = np.frombuffer(b"".join(handles), dtype=np.uint8).copy()
    check(lib.alm_tp_p2p_connect(ctx.h, ptr(buf)))
    dist.barrier()


def tp_plan(canon, world, block=64, down_in=None):
    """Per-rank ranges: q heads, kv heads, FFN columns, vocabulary rows.

    ``down_in`` is the stored (padded) K of the down projection; the FFN is
    split on its 64-column blocks."""
    nh, nkv, hd = canon["heads"], canon["kv_heads"], canon["head_dim"]
    inter, vocab = canon["intermediate"], canon["vocab"]
    if vocab % world:
        raise ValueError(f"vocabulary {vocab} does not split over {world} ranks")
    group = nh // nkv
    plans = []
    for r in range(world):
        if world <= nkv:
            if nkv % world:
                raise ValueError(f"{nkv} kv heads do not split over {world} ranks")
            kpr = nkv // world
            k0, k1 = r * kpr, (r + 1) * kpr
            h0, h1 = k0 * group, k1 * group
        else:
            if world % nkv:
                raise ValueError(f"{world} ranks do not split {nkv} kv heads")
            share = world // nkv
            if group < share:
                raise ValueError(f"a group of {group} query heads cannot split over {share} ranks")
            k0 = r // share
            k1 = k0 + 1
            sub = r % share
            sizes = [group // share + (1 if i < group % share else 0) for i in range(share)]
            h0 = k0 * group + sum(sizes[:sub])
            h1 = h0 + sizes[sub]
        if (h0 * hd) % block or (h1 * hd) % block:
            raise ValueError(f"heads {h0}..{h1} of head_dim {hd} do not fall on {block}-column blocks")
        k_pad = down_in if down_in is not None else -(-inter // block) * block
        nblk = k_pad // block
        b0, b1 = r * nblk // world, (r + 1) * nblk // world
        f0, f1 = b0 * block, min(b1 * block, inter)
        if f1 <= f0:
            raise ValueError(f"rank {r} gets no FFN columns")
        plans.append({"heads": (h0, h1), "kv": (k0, k1), "ffn": (f0, f1), "ffn_pad": (b0 * block, b1 * block),
                      "vocab": (r * vocab // world, (r + 1) * vocab // world)})
    return plans


def slice_rows(p, r0, r1):
    """Rows [r0, r1) of a shard-format projection."""
    scale = None if p.scale is None else p.scale[r0:r1]
    return QuantProj(p.packed[r0:r1], scale, p.bits, p.block, r1 - r0, p.in_, p.in_real)


def slice_cols(p, c0, c1, in_real):
    """Columns [c0, c1) (on block boundaries) of a shard-format projection."""
    if p.bits == 16:
        return QuantProj(p.packed[:, c0:c1], None, 16, 0, p.out, c1 - c0, in_real)
    if c0 % p.block or c1 % p.block:
        raise ValueError("column slices must fall on quantization blocks")
    codes = p.packed[:, c0 // 2:c1 // 2] if p.bits == 4 else p.packed[:, c0:c1]
    return QuantProj(codes, p.scale[:, c0 // p.block:c1 // p.block], p.bits, p.block, p.out, c1 - c0, in_real)


def local_canon(canon, plan):
    c = dict(canon)
    c["heads"] = plan["heads"][1] - plan["heads"][0]
    c["kv_heads"] = plan["kv"][1] - plan["kv"][0]
    c["intermediate"] = plan["ffn"][1] - plan["ffn"][0]
    return c


def shard_layer(layer, canon, plan):
    """This rank's slice of one layer ({q,k,v,o,gate,up,down: QuantProj, n_in, n_post})."""
    hd = canon["head_dim"]
    (h0, h1), (k0, k1), (f0, f1) = plan["heads"], plan["kv"], plan["ffn"]
    p0, p1 = plan["ffn_pad"]
    down = layer["down"]
    c1 = min(p1, down.in_)
    return {
        "q": slice_rows(layer["q"], h0 * hd, h1 * hd),
        "k": slice_rows(layer["k"], k0 * hd, k1 * hd),
        "v": slice_rows(layer["v"], k0 * hd, k1 * hd),
        "o": slice_cols(layer["o"], h0 * hd, h1 * hd, (h1 - h0) * hd),
        "gate": slice_rows(layer["gate"], f0, f1),
        "up": slice_rows(layer["up"], f0, f1),
        "down": slice_cols(down, p0, c1, f1 - f0),
        "n_in": layer["n_in"],
        "n_post": layer["n_post"],
    }


def head_rows(model_dir, man, v0, v1):
    """Rows [v0, v1) of the LM head (or of the tied embedding) as a projection."""
    c = man["config"]
    if man.get("has_lm_head"):
        path = os.path.join(model_dir, "lm_head.safetensors")
        lq = man.get("lm_head_quant") or {}
        if lq:
            q = safetensors.read_tensor(path, "lm_head.q")
            s = safetensors.read_tensor(path, "lm_head.scale")
            return QuantProj(q[v0:v1], s[v0:v1], lq["bits"], lq["block"], v1 - v0, lq["in"])
        return QuantProj.from_fp16(safetensors.read_tensor(path, "lm_head")[v0:v1])
    emb = os.path.join(model_dir, "embeddings.safetensors")
    eq = man.get("embed_quant") or {}
    if eq:
        q = safetensors.read_tensor(emb, "embed.q")
        s = safetensors.read_tensor(emb, "embed.scale")
        return QuantProj(q[v0:v1], s[v0:v1], eq["bits"], eq["block"], v1 - v0, c["hidden"])
    return QuantProj.from_fp16(safetensors.read_tensor(emb, "embed")[v0:v1])


def device_model_tp(ctx, model_dir, rank, world):
    """Load this rank's shard of a shard directory onto the context's device
    (the context must have joined with init_context_tp)."""
    man = load_manifest(model_dir)
    canon = man["config"]
    down_in = man["quant"]["layers"]["0"]["down"]["in"]
    plans = tp_plan(canon, world, down_in=down_in)
    plan = plans[rank]
    lc = local_canon(canon, plan)
    m = DeviceModel(ctx, lc)
    m.manifest = man
    m.tp_plan = plan
    v0, v1 = plan["vocab"]
    check(lib.alm_model_set_tp(m.h, v0, v1 - v0))
    for i in range(canon["layers"]):
        m.set_layer(i, shard_layer(read_layer(model_dir, man, i), canon, plan))
    emb = os.path.join(model_dir, "embeddings.safetensors")
    eq = man.get("embed_quant") or {}
    if eq:
        m.set_embed(safetensors.read_tensor(emb, "embed.q"), safetensors.read_tensor(emb, "embed.scale"),
                    eq["bits"], eq["block"])
    else:
        m.set_embed(safetensors.read_tensor(emb, "embed"))
    m.set_final_norm(safetensors.read_tensor(os.path.join(model_dir, "norms.safetensors"), "final_norm"))
    m.set_head(head_rows(model_dir, man, v0, v1))
    m.finalize()
    return m


__all__ = ["nccl_unique_id", "init_context_tp", "enable_p2p", "tp_plan", "slice_rows", "slice_cols", "local_canon",
           "shard_layer", "head_rows", "device_model_tp"]
