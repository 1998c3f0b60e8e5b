"""The persistent forward kernel (one launch per forward of <= 8 rows) against
the per-operation launches with two-pass attention: same device bodies, so
logits, argmax and the paged KV cache must be bit-identical, for decode rows
and verify rows."""
import numpy as np
import pytest
from gpu_helpers import prefill

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from androidllm_b200.ops import Context
    c = Context(0)
    c.set_attn_fused(False)   # the persistent kernel reproduces the two attention passes
    return c


@pytest.fixture(scope="module")
def models(ctx, model_dirs):
    from androidllm_b200.ops import DeviceModel
    return {name: DeviceModel.from_dir(ctx, model_dirs[name]) for name in ("tiny", "minq", "toy", "toyu")}


def _run(ctx, m, toks, persistent):
    from androidllm_b200.ops import DeviceKV
    ctx.set_persistent(persistent)
    try:
        kv = DeviceKV(m, 128, 16)
        prefill(m, kv, toks[:24])            # a 16-row chunk, then an 8-row chunk
        outs = [m.forward(kv, toks[24:29], 24, logits=True)]   # 5 verify rows
        for i in range(3):                   # single-row decode
            outs.append(m.forward(kv, [toks[29 + i]], 29 + i, logits=True))
        cache = [kv.read(li, 0, 32) for li in range(m.canon["layers"])]
        kv.close()
    finally:
        ctx.set_persistent(False)
    return outs, cache


@pytest.mark.parametrize("name", ["tiny", "minq", "toy", "toyu"])
def test_persistent_forward_bit_identical_to_per_op_launches(ctx, models, name):
    m = models[name]
    toks = np.random.default_rng([7, len(name)]).integers(0, m.canon["vocab"], 40).tolist()
    got, got_kv = _run(ctx, m, toks, True)
    ref, ref_kv = _run(ctx, m, toks, False)
    for (lg, am), (lg_r, am_r) in zip(got, ref):
        assert np.array_equal(lg.view(np.uint32), lg_r.view(np.uint32))
        assert np.array_equal(am, am_r)
    for li, ((k, v), (k_r, v_r)) in enumerate(zip(got_kv, ref_kv)):
        assert np.array_equal(k.view(np.uint16), k_r.view(np.uint16)), li
        assert np.array_equal(v.view(np.uint16), v_r.view(np.uint16)), li


def test_persistent_forward_repeats_exactly(ctx, models):
    """Back-to-back launches share the grid-barrier counter: many forwards in a
    row (the counter's base advances every launch) keep producing the same
    rows as a fresh cache."""
    from androidllm_b200.ops import DeviceKV
    m = models["toy"]
    toks = np.random.default_rng(3).integers(0, m.canon["vocab"], 12).tolist()
    first = None
    ctx.set_persistent(True)
    for _ in range(6):
        kv = DeviceKV(m, 64, 16)
        rows = [m.forward(kv, [t], i, logits=True)[0] for i, t in enumerate(toks)]
        kv.close()
        if first is None:
            first = rows
        for a, b in zip(rows, first):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    ctx.set_persistent(False)


def test_spec_decode_through_persistent_forwards(ctx, model_dirs):
    """Speculative greedy decoding whose captured step runs the persistent
    kernel emits exactly the per-op step's stream."""
    from androidllm_b200.ops import DeviceKV, DeviceModel
    from gpu_helpers import greedy_spec
    from conftest import golden
    g = golden("toy.npz")
    t = DeviceModel.from_dir(ctx, model_dirs["toy"])
    d = DeviceModel.from_dir(ctx, model_dirs["toy_draft"])
    prompt = [int(x) for x in g["prompt"]]
    outs = {}
    for persistent in (False, True):
        ctx.set_persistent(persistent)
        try:
            outs[persistent] = greedy_spec(t, d, DeviceKV(t, 256), DeviceKV(d, 256), prompt, 64, 4)
        finally:
            ctx.set_persistent(False)
    assert outs[True] == outs[False]
