"""The device sampler (alm_sample, alm_model_sample, the sampling speculative
step) against the oracle's restatement of its fixed arithmetic, token for
token, and the engine's temperature > 0 streams against the reference's
decode rule emulated on the device's logits."""
import numpy as np
import pytest

from oracle import sampling as osamp

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from androidllm_b200.ops import Context
    return Context(0)


def _cases(rng):
    for V in (64, 1000, 32000, 151936):
        for kind in ("normal", "ties", "peaked"):
            if kind == "normal":
                lg = rng.standard_normal(V) * rng.uniform(0.5, 4)
            elif kind == "ties":
                lg = rng.integers(-6, 7, V).astype(np.float64)     # many equal logits
            else:
                lg = rng.standard_normal(V)
                lg[rng.integers(V, size=3)] += 14.0
            lg = lg.astype(np.float16)
            for t, tp, mp in ((0.0, 0.9, 0.0), (0.8, 0.9, 0.0), (1.0, 1.0, 0.0), (1.3, 0.5, 0.05),
                              (0.5, 1.0, 0.05), (1.0, 0.001, 0.0)):
                yield lg, t, tp, mp


def test_sampler_matches_oracle_bit_for_bit(ctx):
    from androidllm_b200.ops import sample
    rng = np.random.default_rng(8)
    n = 0
    for lg, t, tp, mp in _cases(rng):
        us = np.concatenate([[0.0, 0.9999999999], rng.random(6)])
        got = sample(ctx, np.tile(lg, (us.size, 1)), t, tp, mp, us)
        for u, g in zip(us, got):
            want = osamp.sample_fixed(lg.astype(np.float32), t, tp, mp, u)
            assert int(g) == want, (lg.size, t, tp, mp, u)
            n += 1
    assert n > 500


def test_model_sample_uses_the_forward_logits(ctx, model_dirs):
    from androidllm_b200.ops import DeviceKV, DeviceModel
    m = DeviceModel.from_dir(ctx, model_dirs["toy"])
    kv = DeviceKV(m, 64, 16)
    toks = [3, 77, 900, 12, 5]
    lg, _ = m.forward(kv, toks, 0, logits=True)
    us = np.array([0.1, 0.5, 0.93, 0.2, 0.7])
    got = m.sample(5, 0.8, 0.9, 0.0, us)
    for r in range(5):
        assert int(got[r]) == osamp.sample_fixed(lg[r], 0.8, 0.9, 0.0, us[r])


def _emulate(t, d, prompt, n, k, seed, temperature, top_p, min_p):
    """engine.py:322-405 on the host with the device's own logits (single-row
    forwards, which verify rows equal bit for bit) and the oracle's fixed
    sampler: the reference's rule and draw order, independent of the
    engine's graph, uniform stream and acceptance kernel."""
    from androidllm_b200.ops import DeviceKV
    rng = np.random.default_rng(seed)
    draw = lambda lg: osamp.sample_fixed(lg, temperature, top_p, min_p, rng.random())
    # the prompt prefilled the way the engine does it (DeviceModel.prefill)
    tkv = DeviceKV(t, 256, 16)
    t.prefill(tkv, prompt[:-1])
    if d is not None:
        dkv = DeviceKV(d, 256, 16)
        d.prefill(dkv, prompt)
    token, pos, out = prompt[-1], len(prompt) - 1, []
    while len(out) < n:
        if d is None:
            lg, _ = t.forward(tkv, [token], pos, logits=True)
            token = draw(lg[0])
            pos += 1
            out.append(token)
            continue
        cands, dt, dp = [], token, pos
        for _ in range(k):
            lg, _ = d.forward(dkv, [dt], dp, logits=True)
            dt = draw(lg[0])
            cands.append(dt)
            dp += 1
        emitted, tok, tp = [], token, pos
        for c in cands + [None]:
            lg, _ = t.forward(tkv, [tok], tp, logits=True)
            g = draw(lg[0])
            emitted.append(g)
            if g != c:
                break
            tok, tp = c, tp + 1
        out += emitted
        token, pos = emitted[-1], pos + len(emitted)
    return out[:n]


@pytest.mark.parametrize("spec", [False, True])
def test_engine_sampling_stream_follows_reference_rule(model_dirs, spec):
    """generate(temperature=0.8, top_p=0.9) from a seed: the engine's stream
    equals the reference's decode rule emulated on the device's logits."""
    from androidllm_b200.engine import LayerStreamingEngine
    from conftest import golden
    g = golden("toy.npz")
    prompt = [int(x) for x in g["prompt"]]
    kw = dict(draft_dir=model_dirs["toy_draft"], spec_k=4) if spec else {}
    eng = LayerStreamingEngine(model_dirs["toy"], seed=1234, **kw)
    got = eng.generate(prompt, max_new_tokens=24, temperature=0.8, top_p=0.9)
    want = _emulate(eng.dm, eng.draft.dm if spec else None, prompt, 24, 4, 1234, 0.8, 0.9, 0.0)
    assert got == want
    if spec:
        assert eng.stats["spec_accepted"] + eng.stats["spec_bonus"] == 24
    eng.close()


def test_spec_sampling_consumes_the_reference_draw_count(ctx, model_dirs):
    """Each sampling step consumes k draft draws and one draw per target row up
    to the first rejection: k + accepted + 1."""
    from androidllm_b200.ops import DeviceKV, DeviceModel, SpecDecoder
    from gpu_helpers import prefill
    t = DeviceModel.from_dir(ctx, model_dirs["toy"])
    d = DeviceModel.from_dir(ctx, model_dirs["toy_draft"])
    tkv, dkv = DeviceKV(t, 256, 16), DeviceKV(d, 256, 16)
    prompt = [5, 9, 100, 2000, 7]
    prefill(t, tkv, prompt[:-1])
    prefill(d, dkv, prompt)
    s = SpecDecoder(t, d, tkv, dkv, 4)
    s.set_sampling(0.8, 0.9, 0.0)
    s.set_uniforms(np.random.default_rng(3).random(512))
    s.begin(prompt[-1], len(prompt) - 1)
    used = 0
    for _ in range(6):
        emitted, acc = s.run(1)
        used += 4 + acc[0] + 1
        assert s.uniforms_used() == used
        assert len(emitted) == acc[0] + 1
    s.close()
