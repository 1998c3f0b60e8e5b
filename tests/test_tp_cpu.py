"""Tensor-parallel split and combine on the CPU: two gloo ranks run the
sharded forward in numpy (the oracle's arithmetic on each rank's slices of
the shard-format weights, the row-split projections' fp32 partials summed by
all_reduce, the head's per-rank (max, index) pairs by all_gather) and must
match the whole model's oracle forward (androidllm/models/llama.py:96-146):
logits within 1e-2 and the same argmax.  Also checks that every column and
row slice of the codes dequantizes to exactly the slice of the whole
weight, and the head / kv splits of the plan."""
import math
import os
import socket

import numpy as np
import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _deq(p):
    from oracle.quant import dequantize_packed
    if p.bits == 16:
        return np.asarray(p.packed, np.float16)[:, :p.in_real]
    meta = {"bits": p.bits, "block": p.block, "out": p.out, "in": p.in_}
    return dequantize_packed(np.asarray(p.packed), np.asarray(p.scale), meta)[:, :p.in_real]


def _tp_forward(rank, world, model_dir, tokens, dist):
    """Sharded forward of `tokens` (one position each) on this rank; returns
    the gathered logits of the last position and the combined argmax."""
    import torch
    from androidllm_b200 import tp
    from androidllm_b200.ops import load_manifest, read_layer
    from oracle import llama as ol
    man = load_manifest(model_dir)
    canon = man["config"]
    plan = tp.tp_plan(canon, world, down_in=man["quant"]["layers"]["0"]["down"]["in"])[rank]
    lc = tp.local_canon(canon, plan)
    layers = []
    for i in range(canon["layers"]):
        sl = tp.shard_layer(read_layer(model_dir, man, i), canon, plan)
        layers.append({k: (_deq(v) if k not in ("n_in", "n_post") else np.asarray(v, np.float16))
                       for k, v in sl.items()})
    from oracle import io as oio
    _, embed, fnorm, _, _ = oio.load_model(model_dir)
    v0, v1 = plan["vocab"]
    head = _deq(tp.head_rows(model_dir, man, v0, v1))
    hd, hl, kl = canon["head_dim"], lc["heads"], lc["kv_heads"]
    group = canon["heads"] // canon["kv_heads"]
    h0, k0 = plan["heads"][0], plan["kv"][0]
    rope = ol.precompute_rope(hd, canon["max_len"], canon["rope_theta"])
    eps = canon["rms_eps"]
    kv = [(np.zeros((len(tokens), kl, hd), np.float16), np.zeros((len(tokens), kl, hd), np.float16))
          for _ in layers]

    def allreduce(v):
        t = torch.from_numpy(np.ascontiguousarray(v, np.float32))
        dist.all_reduce(t)
        return t.numpy()

    for pos, tok in enumerate(tokens):
        x = embed[tok].reshape(1, -1)
        for li, L in enumerate(layers):
            q = ol.apply_rope(ol.matmul_f16(x, L["q"]).reshape(1, hl, hd), pos, rope)
            k = ol.apply_rope(ol.matmul_f16(x, L["k"]).reshape(1, kl, hd), pos, rope)
            v = ol.matmul_f16(x, L["v"]).reshape(1, kl, hd)
            kv[li][0][pos] = k[0].astype(np.float16)
            kv[li][1][pos] = v[0].astype(np.float16)
            ctx = np.zeros((hl, hd), np.float16)
            for i in range(hl):
                kvh = (h0 + i) // group - k0
                keys = kv[li][0][:pos + 1, kvh].astype(np.float32)
                sc = (q[0, i].astype(np.float32) @ keys.T) / math.sqrt(hd)
                p = np.exp(sc - sc.max())
                p = p / p.sum()
                ctx[i] = (p.astype(np.float16) @ kv[li][1][:pos + 1, kvh].astype(np.float16))
            o = allreduce(ctx.reshape(1, -1).astype(np.float32) @ L["o"].astype(np.float32).T)
            x = x + o.astype(np.float16)
            x = ol.rms_norm(x, L["n_in"], eps).astype(np.float16)
            h = ol.swiglu(ol.matmul_f16(x, L["gate"]), ol.matmul_f16(x, L["up"]))
            d = allreduce(h.reshape(1, -1).astype(np.float16).astype(np.float32) @ L["down"].astype(np.float32).T)
            x = x + d.astype(np.float16)
            x = ol.rms_norm(x, L["n_post"], eps).astype(np.float16)
    hn = ol.rms_norm(x, fnorm, eps).astype(np.float16)
    local = (hn @ head.T).astype(np.float32)[0]
    j = int(np.argmax(local))
    pairs = torch.tensor([[float(local[j]), float(j + v0)]], dtype=torch.float64)
    gathered = [torch.zeros_like(pairs) for _ in range(world)]
    dist.all_gather(gathered, pairs)
    best = min(gathered, key=lambda t: (-t[0, 0].item(), t[0, 1].item()))
    parts = [torch.zeros(v1 - v0, dtype=torch.float32) for _ in range(world)]
    dist.all_gather(parts, torch.from_numpy(local))
    return np.concatenate([t.numpy() for t in parts]), int(best[0, 1].item())


def _worker(rank, world, port, model_dir, tokens, out_path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        logits, am = _tp_forward(rank, world, model_dir, tokens, dist)
        if rank == 0:
            np.savez(out_path, logits=logits, argmax=am)
    finally:
        dist.destroy_process_group()


@pytest.mark.slow
@pytest.mark.parametrize("name", ["minq", "toy"])
def test_tp2_forward_matches_whole_model(model_dirs, tmp_path, name):
    import torch.multiprocessing as mp
    from oracle import io as oio
    from oracle import llama as ol
    tokens = [5, 17, 300, 3, 44, 0]
    out = str(tmp_path / "tp.npz")
    mp.spawn(_worker, args=(2, _free_port(), model_dirs[name], tokens, out), nprocs=2, join=True)
    got = np.load(out)
    canon, embed, fnorm, head, layers = oio.load_model(model_dirs[name])
    om = ol.OracleModel(canon, embed, fnorm, head)
    kv = om.prepare_kv(len(tokens))
    x = None
    for pos, t in enumerate(tokens):
        x = om.forward(layers, t, kv, pos)
    ref = om.logits(x)[0]
    err = float(np.max(np.abs(got["logits"] - ref)) / np.max(np.abs(ref)))
    assert err < 1e-2, err
    assert int(got["argmax"]) == int(np.argmax(ref))


@pytest.mark.parametrize("name", ["minq", "toy"])
def test_tp_slices_dequantize_to_whole_weight_slices(model_dirs, name):
    from androidllm_b200 import tp
    from androidllm_b200.ops import load_manifest, read_layer
    d = model_dirs[name]
    man = load_manifest(d)
    canon = man["config"]
    whole = read_layer(d, man, 0)
    W = {k: _deq(v) for k, v in whole.items() if k not in ("n_in", "n_post")}
    hd = canon["head_dim"]
    for world in (1, 2):
        plans = tp.tp_plan(canon, world, down_in=whole["down"].in_)
        for plan in plans:
            sl = tp.shard_layer(whole, canon, plan)
            (h0, h1), (k0, k1), (f0, f1) = plan["heads"], plan["kv"], plan["ffn"]
            assert np.array_equal(_deq(sl["q"]).view(np.uint16), W["q"][h0 * hd:h1 * hd].view(np.uint16))
            assert np.array_equal(_deq(sl["k"]).view(np.uint16), W["k"][k0 * hd:k1 * hd].view(np.uint16))
            assert np.array_equal(_deq(sl["o"]).view(np.uint16), W["o"][:, h0 * hd:h1 * hd].view(np.uint16))
            assert np.array_equal(_deq(sl["up"]).view(np.uint16), W["up"][f0:f1].view(np.uint16))
            assert np.array_equal(_deq(sl["down"]).view(np.uint16), W["down"][:, f0:f1].view(np.uint16))
        # every query head, kv head, FFN column and vocabulary row is covered once
        assert sum(p["heads"][1] - p["heads"][0] for p in plans) == canon["heads"]
        assert sum(p["ffn"][1] - p["ffn"][0] for p in plans) == canon["intermediate"]
        assert sum(p["vocab"][1] - p["vocab"][0] for p in plans) == canon["vocab"]


def test_tp_plan_shapes_of_the_7b_split():
    from androidllm_b200 import synth, tp
    c = synth.CANONS["qwen2.5-7b"]
    for world in (1, 2, 4, 8):
        plans = tp.tp_plan(c, world, down_in=18944)
        heads = [p["heads"][1] - p["heads"][0] for p in plans]
        assert sum(heads) == 28
        # each rank's query heads read kv heads it holds
        for p in plans:
            g = 28 // 4
            assert p["kv"][0] == p["heads"][0] // g and p["kv"][1] == (p["heads"][1] - 1) // g + 1
        if world == 8:
            assert sorted(heads) == [3, 3, 3, 3, 4, 4, 4, 4]        # the uneven split
            assert all(p["kv"][1] - p["kv"][0] == 1 for p in plans)   # kv heads replicated
        assert [p["ffn"][1] - p["ffn"][0] for p in plans] == [18944 // world] * world
