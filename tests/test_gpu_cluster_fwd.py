"""The single-row cluster forward (one 16-CTA thread-block cluster runs every
layer) against the per-operation launches it replaces (two-pass attention):
bit-identical logits,
argmax and KV entries, on the golden models and at the benchmark's draft
shape (Qwen2.5-0.5B layers over a 776-position seeded cache), so the
reference parity of the per-operation path carries over; and the draft shape's
logits against the reference's own (tests/golden/qwen.npz)."""
import sys

import numpy as np
import pytest
from conftest import GOLDEN, golden
from gpu_helpers import prefill, rel_err

sys.path.insert(0, GOLDEN)
from qwen_cases import QWEN_CASES, QWEN_FILL, QWEN_MODELS, qwen_case_tokens, qwen_kv_fill, qwen_logit_index  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from androidllm_b200.ops import Context
    c = Context(0)
    c.set_attn_fused(False)   # the cluster kernel reproduces the two attention passes
    c.set_cluster_forward(True)
    yield c
    c.set_cluster_forward(False)


def _both(ctx, m, make_kv, steps):
    """Run `steps` (token, pos) single-row forwards with and without the
    cluster kernel on two caches made by make_kv; returns both results."""
    out = []
    for enable in (True, False):
        ctx.set_cluster_forward(enable)
        kv = make_kv()
        res = [m.forward(kv, [tok], pos, logits=True) for tok, pos in steps]
        out.append((res, kv))
    ctx.set_cluster_forward(True)
    return out


@pytest.mark.parametrize("name", ["toy", "toyu", "minq", "tiny"])
def test_cluster_forward_bit_identical_on_golden_models(ctx, model_dirs, name):
    from androidllm_b200.ops import DeviceKV, DeviceModel
    m = DeviceModel.from_dir(ctx, model_dirs[name])
    assert m.uses_cluster_forward(), f"{name} should fit the cluster forward"
    g = golden(f"{name}.npz")
    prompt = [int(t) for t in g["prompt"]]
    n = len(prompt)

    def make_kv():
        kv = DeviceKV(m, n + 16, 16)
        prefill(m, kv, prompt[:-1])
        return kv

    steps = [(prompt[-1], n - 1)] + [((7 * i + 3) % m.canon["vocab"], n + i) for i in range(6)]
    (a, kva), (b, kvb) = _both(ctx, m, make_kv, steps)
    for (la, ia), (lb, ib) in zip(a, b):
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
        assert np.array_equal(ia, ib)
    for li in range(m.canon["layers"]):
        ka, va = kva.read(li, 0, n + 6)
        kb, vb = kvb.read(li, 0, n + 6)
        assert np.array_equal(ka.view(np.uint16), kb.view(np.uint16))
        assert np.array_equal(va.view(np.uint16), vb.view(np.uint16))


def test_cluster_forward_at_draft_shape(ctx, tmp_path_factory):
    """The benchmark's draft shape (0.5B layers, head_dim 64, 7 query heads
    per kv head, FFN 4864, int4, tied int8 151936 head), 2 layers, over the
    seeded 776-position cache: bit-identical to the per-operation launches,
    and the reference's logits (sampled entries within 1e-2, argmax equal)."""
    from androidllm_b200 import shard, synth
    from androidllm_b200.ops import DeviceKV, DeviceModel
    from oracle import io as oio
    name, canon, seed, kw = QWEN_MODELS[1]
    d = str(tmp_path_factory.mktemp("qd") / name)
    shard.shard_from_tensors(synth.synth_tensors(canon, seed=seed), canon, d, **kw)
    m = DeviceModel.from_dir(ctx, d)
    assert m.uses_cluster_forward()
    embed = oio.load_model(d)[1]
    g = golden("qwen.npz")
    idx = qwen_logit_index(canon["vocab"])

    def make_kv():
        kv = DeviceKV(m, QWEN_FILL + 8, 16)
        for li in range(canon["layers"]):
            kv.write(li, 0, *qwen_kv_fill(canon, seed, li))
        return kv

    row = 0
    for ci, (rows, pos0) in enumerate(QWEN_CASES):
        if rows != 1:
            row += rows
            continue
        tok = qwen_case_tokens(canon, seed, ci)[0]
        (a, _), (b, _) = _both(ctx, m, make_kv, [(tok, pos0)])
        la, ia = a[0]
        lb, ib = b[0]
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32)), ci
        assert rel_err(la[0, idx], g[f"{name}_sample"][row].astype(np.float32)) < 1e-2
        assert int(ia[0]) == int(g[f"{name}_argmax"][row])
        row += 1
    del embed
