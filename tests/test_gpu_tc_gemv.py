"""GPU parity of the row-record layout and its tcgen05 GEMV: device repack +
dequant bit-exact against androidllm's dequantize_packed, GEMV results within
the fp32-summation tolerance of an fp32 reference and independent of the
number of rows, and the model path (residual, SwiGLU and logits epilogues)
against the reference's own states and greedy streams."""
import numpy as np
import pytest
from conftest import golden
from gpu_helpers import greedy_plain, greedy_spec, random_codes, ref_matmul, rel_err, ulp_diff

from oracle import quant as oquant

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from androidllm_b200.ops import Context
    c = Context(0)
    c.set_gemv_layout(2)   # every eligible weight in the row layout
    return c


def _upload(ctx, packed, scale, bits, block, out, k, k_real=None):
    from androidllm_b200.ops import QuantProj, QWeight
    return QWeight(ctx, QuantProj(packed, scale, bits, block, out, k, k_real))


def test_dequant_rows_matches_reference_golden(ctx):
    g = golden("quant.npz")
    n = 0
    for i in range(int(g["n_cases"])):
        bits, block, out, inp, _ = (int(v) for v in g[f"c{i}_meta"])
        if bits not in (4, 8) or block % 64:
            continue
        w = _upload(ctx, g[f"c{i}_packed"], g[f"c{i}_scale"], bits, block, out, inp)
        assert np.array_equal(w.dequant().view(np.uint16), g[f"c{i}_deq"].view(np.uint16)), i
        n += 1
    assert n > 0


SWEEP = [(1536, 1536), (8960, 1536), (1536, 8960), (18944, 3584), (3584, 18944), (151936, 1536)]


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("shape", SWEEP)
def test_dequant_rows_bit_exact_sweep_shapes(ctx, bits, shape):
    rng = np.random.default_rng([bits, *shape, 7])
    n, k = shape
    packed, scale = random_codes(rng, n, k, bits, 64, zero_blocks=3)
    w = _upload(ctx, packed, scale, bits, 64, n, k)
    ref = oquant.dequantize_packed(packed, scale, {"bits": bits, "block": 64, "out": n, "in": k})
    assert np.array_equal(w.dequant().view(np.uint16), ref.view(np.uint16))


def test_dequant_rows_subnormal_scales_and_padding(ctx):
    """Subnormal scales, rows not a multiple of 128, in_real < in."""
    rng = np.random.default_rng(6)
    n, k, k_real = 200, 704, 688
    packed, scale = random_codes(rng, n, k, 4, 64)
    scale[:, :3] = np.array([2 ** -24, 3 * 2 ** -24, 2 ** -15], np.float16)
    w = _upload(ctx, packed, scale, 4, 64, n, k, k_real)
    ref = oquant.dequantize_packed(packed, scale, {"bits": 4, "block": 64, "out": n, "in": k})[:, :k_real]
    assert np.array_equal(w.dequant().view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("bits,block,shape", [(4, 64, (1536, 1536)), (8, 64, (8960, 1536)),
                                              (8, 64, (1536, 8960)), (4, 64, (18944, 3584)),
                                              (8, 1536, (151936, 1536)), (8, 64, (1000, 704)),
                                              (4, 128, (320, 1024))])
@pytest.mark.parametrize("m", [1, 5, 8, 9, 16])
def test_tc_gemv_matches_fp32_reference(ctx, bits, block, shape, m):
    rng = np.random.default_rng([bits, block, m, *shape, 1])
    n, k = shape
    packed, scale = random_codes(rng, n, k, bits, block)
    w = _upload(ctx, packed, scale, bits, block, n, k)
    deq = oquant.dequantize_packed(packed, scale, {"bits": bits, "block": block, "out": n, "in": k})
    x = rng.standard_normal((m, k)).astype(np.float16)
    got = w.matmul(x)
    ref = ref_matmul(x, deq)
    assert rel_err(got, ref) < 1e-2
    assert np.mean(ulp_diff(got, ref) > 1) < 2e-3


@pytest.mark.parametrize("wg,ksg", [(1, 1), (2, 1), (4, 1), (1, 3), (4, 5), (2, 24)])
def test_tc_gemv_every_split(ctx, wg, ksg):
    """Each launch shape (warpgroups per CTA, CTAs along K) is correct and
    row-count independent."""
    rng = np.random.default_rng([wg, ksg])
    n, k = 2048, 1536
    packed, scale = random_codes(rng, n, k, 4, 64)
    w = _upload(ctx, packed, scale, 4, 64, n, k)
    w.set_split(wg, ksg)
    assert w.split()[0] == wg
    deq = oquant.dequantize_packed(packed, scale, {"bits": 4, "block": 64, "out": n, "in": k})
    x = rng.standard_normal((16, k)).astype(np.float16)
    full = w.matmul(x)
    assert rel_err(full, ref_matmul(x, deq)) < 1e-2
    for mm in (1, 7, 9):
        assert np.array_equal(w.matmul(x[:mm]).view(np.uint16), full[:mm].view(np.uint16)), mm


def test_tc_gemv_rows_are_independent_of_m(ctx):
    rng = np.random.default_rng(12)
    for bits, (n, k) in ((4, (9728, 896)), (8, (1536, 8960)), (8, (17920, 1536))):
        packed, scale = random_codes(rng, n, k, bits, 64)
        w = _upload(ctx, packed, scale, bits, 64, n, k)
        x = rng.standard_normal((16, k)).astype(np.float16)
        full = w.matmul(x)
        for mm in (1, 5, 8, 9):
            assert np.array_equal(w.matmul(x[:mm]).view(np.uint16), full[:mm].view(np.uint16)), (bits, n, mm)
        assert np.array_equal(w.matmul(x[3:4]).view(np.uint16), full[3:4].view(np.uint16))


# ---- model path with the row layout --------------------------------------------------


@pytest.fixture(scope="module")
def models(ctx, model_dirs):
    from androidllm_b200.ops import DeviceModel
    return {name: DeviceModel.from_dir(ctx, d) for name, d in model_dirs.items()}


def _kv(model, n=512):
    from androidllm_b200.ops import DeviceKV
    return DeviceKV(model, n, 16)


@pytest.mark.parametrize("name", ["toy", "toyu"])
def test_rows_layer_states_match_reference(models, model_dirs, name):
    g = golden(f"{name}.npz")
    m = models[name]
    kv = _kv(m)
    prompt = [int(t) for t in g["prompt"]]
    n_pos = g["states"].shape[0]
    n_exact = n_total = 0
    from oracle import io as oio
    embed = oio.load_model(model_dirs[name])[1]
    x = None
    for pos, tok in enumerate(prompt):
        x = embed[tok].reshape(1, -1)
        for li in range(m.canon["layers"]):
            x = m.layer_forward(li, kv, x, pos)
            if pos < n_pos:
                ref = g["states"][pos, li].reshape(1, -1)
                assert rel_err(x, ref) < 1e-2, (pos, li)
                n_exact += int(np.sum(ulp_diff(x, ref) == 0))
                n_total += ref.size
    print(f"{name} (row layout): {n_exact}/{n_total} state elements bit-identical to the reference")
    assert n_exact / n_total > 0.9
    lg, am = m.head_logits(x)
    ref_lg = g["logits"].astype(np.float32)
    assert rel_err(lg[0], ref_lg) < 1e-2
    assert int(am[0]) == int(np.argmax(lg[0]))


def test_rows_verify_rows_equal_sequential_rows(models):
    m = models["toy"]
    rng = np.random.default_rng(2)
    toks = rng.integers(0, m.canon["vocab"], 21).tolist()
    kv1, kv2 = _kv(m), _kv(m)
    from gpu_helpers import prefill
    prefill(m, kv1, toks[:16])
    prefill(m, kv2, toks[:16])
    lg_batch, am_batch = m.forward(kv1, toks[16:21], 16, logits=True)
    for i, t in enumerate(toks[16:21]):
        lg, am = m.forward(kv2, [t], 16 + i, logits=True)
        assert np.array_equal(lg[0], lg_batch[i]), i
        assert int(am[0]) == int(am_batch[i])


def test_rows_spec_greedy_equals_plain_greedy(models):
    """Speculative decoding through row-layout weights emits the plain greedy
    stream, and (the summation orders aside) the reference's tokens."""
    g = golden("toy.npz")
    t, d = models["toy"], models["toy_draft"]
    prompt = [int(x) for x in g["prompt"]]
    plain = greedy_plain(t, _kv(t, 256), prompt, 128)
    spec, steps, acc, bonus = greedy_spec(t, d, _kv(t, 256), _kv(d, 256), prompt, 128, 4)
    assert spec == plain
    assert acc + bonus == 128
    print("toy (row layout): %d of 128 greedy tokens equal the reference's before the first difference"
          % next((i for i, (a, b) in enumerate(zip(plain, g["plain"].tolist())) if a != b), 128))


@pytest.mark.parametrize("bits,shape,m", [(4, (2048, 1536), 17), (4, (2048, 1536), 40), (8, (2048, 1536), 128),
                                          (4, (2048, 1536), 256), (8, (1536, 8960), 40), (8, (1536, 8960), 128),
                                          (4, (18944, 3584), 128), (8, (1000, 704), 33), (4, (40000, 1536), 40),
                                          (8, (40000, 1536), 256)])
def test_tc_dense_matches_fp32_reference(ctx, bits, shape, m):
    """More than 16 activation rows: tcgen05 MMAs with N = m (rounded up to
    16) against activations streamed per k-block; 1, 2 or 4 issuing threads
    (fewer on grids of several waves), K splits summed by a separate
    kernel."""
    rng = np.random.default_rng([bits, m, *shape, 3])
    n, k = shape
    packed, scale = random_codes(rng, n, k, bits, 64)
    w = _upload(ctx, packed, scale, bits, 64, n, k)
    deq = oquant.dequantize_packed(packed, scale, {"bits": bits, "block": 64, "out": n, "in": k})
    x = rng.standard_normal((m, k)).astype(np.float16)
    got = w.matmul(x)
    ref = ref_matmul(x, deq)
    assert rel_err(got, ref) < 1e-2
    assert np.mean(ulp_diff(got, ref) > 1) < 2e-3


@pytest.mark.parametrize("m", [24, 96])
def test_tc_dense_unaligned_rows(ctx, m):
    """Activation rows with a stride that is not a multiple of 8 halves take
    the staged dense path (the streamed one needs 16-byte aligned rows); both
    agree with the fp32 reference."""
    from androidllm_b200._lib import check, lib
    from androidllm_b200.ops import DeviceBuffer
    rng = np.random.default_rng([m, 9])
    n, k, ldx = 1024, 1536, 1539
    packed, scale = random_codes(rng, n, k, 4, 64)
    w = _upload(ctx, packed, scale, 4, 64, n, k)
    deq = oquant.dequantize_packed(packed, scale, {"bits": 4, "block": 64, "out": n, "in": k})
    x = rng.standard_normal((m, k)).astype(np.float16)
    xp = np.zeros((m, ldx), np.float16)
    xp[:, :k] = x
    xb, yb = DeviceBuffer(ctx, xp.nbytes), DeviceBuffer(ctx, m * n * 2)
    xb.upload(xp)
    check(lib.alm_qmatmul(ctx.h, w.h, xb.h, ldx, m, yb.h, n))
    got = yb.download(np.empty((m, n), np.float16))
    assert rel_err(got, ref_matmul(x, deq)) < 1e-2
    assert np.array_equal(got.view(np.uint16), w.matmul(x).view(np.uint16)) or rel_err(got, w.matmul(x)) < 1e-2


@pytest.mark.parametrize("bits,m", [(4, 40), (8, 256)])
def test_tc_dense_padded_k(ctx, bits, m):
    """in_real < in: the activation tensor map reads zeros past in_real, so
    the padded weight columns add nothing."""
    rng = np.random.default_rng([bits, m, 11])
    n, k, k_real = 2048, 704, 688
    packed, scale = random_codes(rng, n, k, bits, 64)
    w = _upload(ctx, packed, scale, bits, 64, n, k, k_real)
    deq = oquant.dequantize_packed(packed, scale, {"bits": bits, "block": 64, "out": n, "in": k})[:, :k_real]
    x = rng.standard_normal((m, k_real)).astype(np.float16)
    got = w.matmul(x)
    ref = ref_matmul(x, deq)
    assert rel_err(got, ref) < 1e-2
    assert np.mean(ulp_diff(got, ref) > 1) < 2e-3
