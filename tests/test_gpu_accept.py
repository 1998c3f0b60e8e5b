"""GPU speculative rejection sampling (alm_probs, alm_accept, and the
speculative decoder's rejection mode) against its oracle,
oracle/sampling.py: probs_repro / sample_probs / accept_rejection.

The reference accepts sampled candidates by its own rule (an independent
target sample must equal the draft sample, androidllm/engine.py:306-320) and
has no min(1, p/q) sampler, so this rule is pinned by its oracle only; the
claim is bit-exact agreement with it given identical logits and draws:
probabilities bit for bit, accepted counts and emitted tokens exactly.
"""
import numpy as np
import pytest

from oracle import sampling as osamp

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from androidllm_b200.ops import Context
    return Context(0)


def _logits(rng, rows, vocab, ties=False):
    lg = (rng.standard_normal((rows, vocab)) * 2.0).astype(np.float16)
    if ties:   # coarse values: many exactly equal logits
        lg = (np.round(lg.astype(np.float32) * 2) / 2).astype(np.float16)
    return lg


@pytest.mark.parametrize("vocab", [1000, 32000, 151936])
@pytest.mark.parametrize("temperature,min_p", [(1.0, 0.0), (0.7, 0.0), (1.3, 0.05), (0.8, 0.1)])
def test_probs_bit_exact(ctx, vocab, temperature, min_p):
    from androidllm_b200.ops import probs
    rng = np.random.default_rng([vocab, int(temperature * 10), int(min_p * 100)])
    lg = _logits(rng, 3, vocab, ties=vocab == 1000)
    got = probs(ctx, lg, temperature, min_p)
    for r in range(lg.shape[0]):
        ref = osamp.probs_repro(lg[r], temperature, min_p)
        assert np.array_equal(got[r].view(np.uint32), ref.view(np.uint32)), r


def _case(rng, k, vocab, temperature, kind):
    """Target logits (k+1, V), draft probs (k, V), candidates drawn from them,
    and k + 1 draws."""
    tl = _logits(rng, k + 1, vocab, ties=kind == "ties")
    if kind == "same":
        dl = tl[:k]
    else:
        dl = (tl[:k].astype(np.float32) + rng.standard_normal((k, vocab)) * 0.7).astype(np.float16)
    min_p_d = 0.05 if kind == "zeros" else 0.0        # zero entries in q
    q = np.stack([osamp.probs_repro(dl[i], temperature, min_p_d) for i in range(k)])
    cand = [osamp.sample_probs(q[i], rng.random()) for i in range(k)]
    u = rng.random(k + 1)
    if kind == "edges":
        u[0], u[-1] = 0.0, np.nextafter(1.0, 0.0)
    return tl, q, cand, u


@pytest.mark.parametrize("kind", ["noisy", "same", "zeros", "ties", "edges"])
@pytest.mark.parametrize("k,vocab", [(1, 1000), (4, 32000), (4, 151936), (7, 5000)])
def test_accept_bit_exact(ctx, kind, k, vocab):
    from androidllm_b200.ops import accept
    rng = np.random.default_rng([k, vocab, len(kind)])
    n_acc = []
    for trial in range(6):
        temperature = (1.0, 0.8, 1.3)[trial % 3]
        min_p = 0.1 if (kind == "zeros" and trial % 2) else 0.0   # zero entries in p too
        tl, q, cand, u = _case(rng, k, vocab, temperature, kind)
        p = np.stack([osamp.probs_repro(tl[i], temperature, min_p) for i in range(k + 1)])
        ref_tok, ref_n = osamp.accept_rejection(p, q, cand, u[:k].astype(np.float32), float(u[k]))
        got_tok, got_n = accept(ctx, tl, q, cand, temperature, u, min_p)
        assert (got_tok, got_n) == (ref_tok, ref_n), (trial, temperature)
        n_acc.append(got_n)
    if kind == "same":
        assert all(n == k for n in n_acc)       # identical distributions: every candidate accepted


def test_accept_rejects_zero_target_probability(ctx):
    """A candidate the target gives probability 0 (min-p filtered) is always
    rejected, and the replacement comes from max(0, p - q)."""
    from androidllm_b200.ops import accept
    rng = np.random.default_rng(3)
    k, vocab, t = 3, 4000, 1.0
    tl = _logits(rng, k + 1, vocab)
    q = np.stack([osamp.probs_repro(tl[i], t) for i in range(k)])
    p = np.stack([osamp.probs_repro(tl[i], t, 0.5) for i in range(k + 1)])
    lowest = int(np.argmin(tl[0].astype(np.float32)))
    assert p[0, lowest] == 0 and q[0, lowest] > 0
    cand = [lowest, 1, 2]
    u = np.array([0.0, 0.5, 0.5, 0.25])
    tok, n = accept(ctx, tl, q, cand, t, u, 0.5)
    assert n == 0 and len(tok) == 1
    assert (p[0] - q[0])[tok[0]] > 0
    assert (tok, n) == osamp.accept_rejection(p, q, cand, u[:k].astype(np.float32), float(u[k]))


def test_spec_decoder_rejection_mode_matches_emulation(models_toy):
    """The speculative decoder in rejection mode at T = 1.0 (k = 4, toy
    target with its 2-layer draft): every step's emitted tokens and accepted
    count equal the oracle's rule applied on the host to the device's own
    logits, with the same draw stream (2k + 1 draws per step)."""
    from androidllm_b200.ops import DeviceKV, SpecDecoder
    from gpu_helpers import prefill
    t, d, prompt = models_toy
    k, temp, n_steps = 4, 1.0, 24
    u = np.random.default_rng(11).random(n_steps * (2 * k + 1) + 16)
    tkv, dkv, tkv2, dkv2 = DeviceKV(t, 512), DeviceKV(d, 512), DeviceKV(t, 512), DeviceKV(d, 512)
    for kv, m, ids in ((tkv, t, prompt[:-1]), (tkv2, t, prompt[:-1]), (dkv, d, prompt), (dkv2, d, prompt)):
        prefill(m, kv, ids)
    s = SpecDecoder(t, d, tkv, dkv, k)
    s.set_sampling(temp, 1.0, 0.0)
    s.set_rejection(True)
    s.set_uniforms(u)
    tok, pos = prompt[-1], len(prompt) - 1
    s.begin(tok, pos)
    cur, accepted_total = 0, 0
    for step in range(n_steps):
        emitted, acc = s.run(1)
        # host emulation over the device's logits
        cands, qs, dtok = [], [], tok
        for i in range(k):
            lg, _ = d.forward(dkv2, [dtok], pos + i, logits=True)
            q = osamp.probs_repro(lg[0], temp)
            qs.append(q)
            dtok = osamp.sample_probs(q, u[cur + i])
            cands.append(dtok)
        lg, _ = t.forward(tkv2, [tok] + cands, pos, logits=True)
        p = np.stack([osamp.probs_repro(lg[j], temp) for j in range(k + 1)])
        ref, n = osamp.accept_rejection(p, np.stack(qs), cands, u[cur + k:cur + 2 * k].astype(np.float32),
                                        float(u[cur + 2 * k]))
        assert (emitted, acc[0]) == (ref, n), step
        cur += 2 * k + 1
        accepted_total += n
        tok, pos = ref[-1], pos + n + 1
    assert s.uniforms_used() == cur
    print(f"rejection mode: {accepted_total} of {n_steps * k} candidates accepted")
    s.close()


@pytest.fixture(scope="module")
def models_toy(ctx, model_dirs):
    from androidllm_b200.ops import DeviceModel
    from conftest import golden
    g = golden("toy.npz")
    return (DeviceModel.from_dir(ctx, model_dirs["toy"]), DeviceModel.from_dir(ctx, model_dirs["toy_draft"]),
            [int(x) for x in g["prompt"]])
