"""GPU parity of the model path against the reference's own outputs
(tests/golden): per-layer hidden states, logits, KV contents, greedy token
streams, and speculative decoding."""
import numpy as np
import pytest
from conftest import golden
from gpu_helpers import greedy_plain, greedy_spec, rel_err, ulp_diff

from oracle import io as oio
from oracle import llama as ollama

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from androidllm_b200.ops import Context
    return Context(0)


@pytest.fixture(scope="module")
def models(ctx, model_dirs):
    from androidllm_b200.ops import DeviceModel
    return {name: DeviceModel.from_dir(ctx, d) for name, d in model_dirs.items()}


def _kv(model, n=512):
    from androidllm_b200.ops import DeviceKV
    return DeviceKV(model, n, 16)


@pytest.mark.parametrize("name", ["tiny", "minq", "toy", "toyu"])
def test_layer_states_match_reference(models, model_dirs, name):
    """layer_forward per position and layer against the reference's states."""
    g = golden(f"{name}.npz")
    m = models[name]
    kv = _kv(m)
    prompt = [int(t) for t in g["prompt"]]
    n_pos = g["states"].shape[0]
    n_exact = n_total = 0
    x = None
    for pos, tok in enumerate(prompt):
        x = _embed(model_dirs[name], tok)
        for li in range(m.canon["layers"]):
            x = m.layer_forward(li, kv, x, pos)
            if pos < n_pos:
                ref = g["states"][pos, li].reshape(1, -1)
                assert rel_err(x, ref) < 1e-2, (pos, li)
                n_exact += int(np.sum(ulp_diff(x, ref) == 0))
                n_total += ref.size
    # rounding points match the reference's, so almost every element is
    # bit-identical (the rest differ by last-bit roundings of fp32 sums)
    print(f"{name}: {n_exact}/{n_total} state elements bit-identical to the reference")
    assert n_exact / n_total > 0.9
    lg, am = m.head_logits(x)
    ref_lg = g["logits"].astype(np.float32)
    assert rel_err(lg[0], ref_lg) < 1e-2
    # last-bit differences accumulate over the prompt's positions; most
    # logits stay bit-identical and all are within one or two fp16 ulps
    exact = float(np.mean(ulp_diff(lg[0], ref_lg) == 0))
    print(f"{name}: {exact:.3f} of the logits bit-identical to the reference")
    assert exact > 0.5
    assert int(am[0]) == int(np.argmax(lg[0]))


_EMBED = {}


def _embed(model_dir, tok):
    """Reference embedding row (the dequantized table, androidllm/engine.py:98-105)."""
    if model_dir not in _EMBED:
        _EMBED[model_dir] = oio.load_model(model_dir)[1]
    return _EMBED[model_dir][tok].reshape(1, -1)


@pytest.mark.parametrize("name", ["toy", "minq"])
def test_verify_rows_equal_sequential_rows(models, name):
    """A (k+1)-row verify forward gives exactly the states, KV entries and
    logits of k+1 single-row forwards."""
    m = models[name]
    rng = np.random.default_rng(1)
    toks = rng.integers(0, m.canon["vocab"], 21).tolist()
    kv1, kv2 = _kv(m), _kv(m)
    from gpu_helpers import prefill
    prefill(m, kv1, toks[:16])
    prefill(m, kv2, toks[:16])
    lg_batch, am_batch = m.forward(kv1, toks[16:21], 16, logits=True)
    seq = [m.forward(kv2, [t], 16 + i, logits=True) for i, t in enumerate(toks[16:21])]
    for i, (lg, am) in enumerate(seq):
        assert np.array_equal(lg[0], lg_batch[i]), i
        assert int(am[0]) == int(am_batch[i])
    for li in range(m.canon["layers"]):
        k1, v1 = kv1.read(li, 0, 21)
        k2, v2 = kv2.read(li, 0, 21)
        assert np.array_equal(k1.view(np.uint16), k2.view(np.uint16))
        assert np.array_equal(v1.view(np.uint16), v2.view(np.uint16))


def test_kv_cache_matches_oracle(models, model_dirs):
    """K (after RoPE) and V written to the paged cache equal the reference's
    fp16 cache entries."""
    name = "minq"
    m = models[name]
    canon, embed, fnorm, head, layers = oio.load_model(model_dirs[name])
    om = ollama.OracleModel(canon, embed, fnorm, head)
    okv = om.prepare_kv(64)
    kv = _kv(m)
    toks = [5, 17, 900, 3, 44, 44, 0]
    for pos, t in enumerate(toks):
        om.forward(layers, t, okv, pos)
    from gpu_helpers import prefill
    prefill(m, kv, toks)
    for li in range(canon["layers"]):
        k, v = kv.read(li, 0, len(toks))
        assert rel_err(k, okv[li][0][: len(toks)]) < 1e-2
        assert rel_err(v, okv[li][1][: len(toks)]) < 1e-2
        assert np.mean(ulp_diff(k, okv[li][0][: len(toks)]) == 0) > 0.99


def test_greedy_stream_toy_identical_to_reference(models):
    """128 greedy tokens on the toy Llama: identical to the reference."""
    g = golden("toy.npz")
    m = models["toy"]
    out = greedy_plain(m, _kv(m, 256), [int(t) for t in g["prompt"]], 128)
    assert out == g["plain"].tolist()


@pytest.mark.parametrize("name", ["toy", "toyu"])
def test_greedy_teacher_forced_matches_reference(models, name):
    """All 128 greedy positions of the reference run, each fed the reference's
    own previous token (teacher forcing, so one near-tie cannot derail the
    rest): the device's pick equals the reference's wherever the reference's
    top-1/top-2 logit margin exceeds one fp16 ulp of its top logit.  The
    untied toy's stream is not one repeated token, and its reference has exact
    fp16 ties (margin 0), which are the only positions allowed to differ."""
    from gpu_helpers import prefill
    g = golden(f"{name}.npz")
    m = models[name]
    kv = _kv(m, 256)
    prompt = [int(t) for t in g["prompt"]]
    ref, margins = g["plain"].tolist(), g["plain_margins"]
    prefill(m, kv, prompt[:-1])
    tok, pos = prompt[-1], len(prompt) - 1
    exceptions, near = [], 0
    for i in range(len(ref)):
        lg, am = m.forward(kv, [tok], pos, logits=True)
        ulp = float(np.spacing(np.float16(abs(float(np.max(lg[0]))))))
        if margins[i] <= ulp:
            near += 1
        if int(am[0]) != ref[i]:
            assert margins[i] <= ulp, f"position {i}: {int(am[0])} vs {ref[i]}, reference margin {margins[i]}"
            exceptions.append(i)
        tok, pos = ref[i], pos + 1
    print(f"{name}: {len(ref) - len(exceptions)}/{len(ref)} picks equal the reference's; "
          f"{near} reference near-ties, differing at {exceptions}")
    if name == "toyu":
        assert len(set(ref)) > 16      # a non-degenerate stream


@pytest.mark.parametrize("name", ["toy", "toyu"])
def test_spec_greedy_equals_plain_greedy_on_device(models, name):
    """Speculative decoding (k=4, 2-layer draft) emits exactly the device's
    plain greedy stream, and its accounting matches the reference's rules."""
    g = golden(f"{name}.npz")
    t, d = models[name], models[name + "_draft"]
    prompt = [int(x) for x in g["prompt"]]
    plain = greedy_plain(t, _kv(t, 256), prompt, 128)
    spec, steps, acc, bonus = greedy_spec(t, d, _kv(t, 256), _kv(d, 256), prompt, 128, 4)
    assert spec == plain
    assert acc + bonus == 128
    if name == "toy":
        # same tokens and same draft decisions as the reference run
        ref_steps, ref_draft, ref_acc, ref_bonus = g["spec_stats"].tolist()
        assert (steps, acc, bonus) == (ref_steps, ref_acc, ref_bonus)


def test_spec_across_the_span_boundary(models):
    """KV caches longer than one 1024-position P.V span: speculative steps
    replay the one-span step graph while every pass fits the first span and
    the span-split graph after it; the stream crossing position 1024 equals
    plain greedy decoding (single-row forwards on either side of the
    boundary) token for token."""
    t, d = models["toyu"], models["toyu_draft"]
    rng = np.random.default_rng(77)
    prompt = rng.integers(0, t.canon["vocab"], 990).tolist()
    plain = greedy_plain(t, _kv(t, 2048), prompt, 96)
    spec, _, _, _ = greedy_spec(t, d, _kv(t, 2048), _kv(d, 2048), prompt, 96, 4)
    assert spec == plain
