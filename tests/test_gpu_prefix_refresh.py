"""Prompt-prefix KV reuse across generate() calls (androidllm/engine.py:245-253,
325-336) and the draft refresh (the fix of the reference's stale draft cache
entry after an all-accept step, engine.py:299-303 vs 318-320)."""
import numpy as np
import pytest
from conftest import golden
from gpu_helpers import greedy_plain

pytestmark = pytest.mark.gpu


def test_prefix_reuse_gives_the_fresh_engines_tokens(model_dirs):
    from androidllm_b200.engine import LayerStreamingEngine
    g = golden("toyu.npz")
    prompt = [int(t) for t in g["prompt"]]
    second = prompt[:40] + [11, 22, 33, 44, 55]
    eng = LayerStreamingEngine(model_dirs["toyu"], draft_dir=model_dirs["toyu_draft"], spec_k=4)
    eng.generate(prompt, max_new_tokens=24, temperature=0.0)
    out = eng.generate(second, max_new_tokens=24, temperature=0.0)
    snap = eng.snapshot()
    assert snap["prefix_kv"] and snap["prefix_calls"] == 1 and snap["prefix_tokens"] == 40
    fresh = LayerStreamingEngine(model_dirs["toyu"], draft_dir=model_dirs["toyu_draft"], spec_k=4)
    assert out == fresh.generate(second, max_new_tokens=24, temperature=0.0)
    eng.close()
    fresh.close()


@pytest.mark.parametrize("k", [1, 4])
def test_draft_refresh_with_the_target_as_its_own_draft(model_dirs, k):
    """With the draft equal to the target every candidate is right; without
    the refresh the draft's cache misses the last candidate of each
    all-accept step and later steps reject, with it every step accepts all
    k.  Emitted tokens equal plain greedy decoding either way."""
    from androidllm_b200.ops import Context, DeviceKV, DeviceModel, SpecDecoder
    from gpu_helpers import prefill
    ctx = Context(0)
    t = DeviceModel.from_dir(ctx, model_dirs["toyu"])
    d = DeviceModel.from_dir(ctx, model_dirs["toyu"])
    g = golden("toyu.npz")
    prompt = [int(x) for x in g["prompt"]]
    n_new = 40
    plain = greedy_plain(t, DeviceKV(t, 256), prompt, n_new)
    rates = {}
    for refresh in (False, True):
        tkv, dkv = DeviceKV(t, 256), DeviceKV(d, 256)
        prefill(t, tkv, prompt[:-1])
        prefill(d, dkv, prompt)
        s = SpecDecoder(t, d, tkv, dkv, k)
        s.set_draft_refresh(refresh)
        s.begin(prompt[-1], len(prompt) - 1, prev=prompt[-2])
        out, acc = [], []
        while len(out) < n_new:
            e, a = s.run(1)
            out += e
            acc += a
        assert out[:n_new] == plain
        rates[refresh] = float(np.mean(np.array(acc) == k))
        s.close()
    print(f"k={k}: steps accepting all candidates without / with the refresh: {rates[False]:.2f} / {rates[True]:.2f}")
    assert rates[True] == 1.0
    assert rates[False] < 1.0
