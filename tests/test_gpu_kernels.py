"""GPU parity of the weight path: device repack + dequant (bit-exact against
androidllm's dequantize_packed) and the fused dequant-GEMV (fp32 accumulation,
one fp16 rounding, independent of the number of rows)."""
import numpy as np
import pytest
from conftest import golden
from gpu_helpers import random_codes, ref_matmul, rel_err, ulp_diff

from oracle import quant as oquant

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from androidllm_b200.ops import Context
    return Context(0)


def _upload(ctx, packed, scale, bits, block, out, k, k_real=None):
    from androidllm_b200.ops import QuantProj, QWeight
    return QWeight(ctx, QuantProj(packed, scale, bits, block, out, k, k_real))


def test_dequant_matches_reference_golden(ctx):
    """Every quant case produced by the reference itself, bit for bit."""
    g = golden("quant.npz")
    for i in range(int(g["n_cases"])):
        bits, block, out, inp, _ = (int(v) for v in g[f"c{i}_meta"])
        w = _upload(ctx, g[f"c{i}_packed"], g[f"c{i}_scale"], bits, block, out, inp)
        got = w.dequant()
        assert np.array_equal(got.view(np.uint16), g[f"c{i}_deq"].view(np.uint16)), i


SWEEP = [(1536, 1536), (8960, 1536), (1536, 8960), (18944, 3584), (3584, 18944), (151936, 1536)]


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("shape", SWEEP)
def test_dequant_bit_exact_sweep_shapes(ctx, bits, shape):
    rng = np.random.default_rng([bits, *shape])
    n, k = shape
    packed, scale = random_codes(rng, n, k, bits, 64, zero_blocks=3)
    w = _upload(ctx, packed, scale, bits, 64, n, k)
    got = w.dequant()
    ref = oquant.dequantize_packed(packed, scale, {"bits": bits, "block": 64, "out": n, "in": k})
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))


def test_dequant_subnormal_scales_and_padding(ctx):
    """fp16 subnormal scales and products, K padding with in_real < in."""
    rng = np.random.default_rng(5)
    n, k, k_real = 40, 704, 688
    packed, scale = random_codes(rng, n, k, 4, 64)
    scale[:, :3] = np.array([2 ** -24, 3 * 2 ** -24, 2 ** -15], np.float16)
    w = _upload(ctx, packed, scale, 4, 64, n, k, k_real)
    ref = oquant.dequantize_packed(packed, scale, {"bits": 4, "block": 64, "out": n, "in": k})[:, :k_real]
    assert np.array_equal(w.dequant().view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("bits,block,shape", [(4, 64, (1536, 1536)), (8, 64, (8960, 1536)),
                                              (8, 64, (1536, 8960)), (4, 64, (3584, 18944)),
                                              (8, 1536, (151936, 1536)), (4, 32, (96, 160)),
                                              (8, 64, (1000, 704))])
@pytest.mark.parametrize("m", [1, 5, 8, 16])
def test_gemv_matches_fp32_reference(ctx, bits, block, shape, m):
    rng = np.random.default_rng([bits, block, m, *shape])
    n, k = shape
    packed, scale = random_codes(rng, n, k, bits, block)
    w = _upload(ctx, packed, scale, bits, block, n, k)
    deq = oquant.dequantize_packed(packed, scale, {"bits": bits, "block": block, "out": n, "in": k})
    x = rng.standard_normal((m, k)).astype(np.float16)
    got = w.matmul(x)
    ref = ref_matmul(x, deq)
    # max relative error 1e-2.  In practice the only
    # differences are last-bit roundings of fp32 sums (tensor-core vs BLAS
    # order), so almost every element is within one fp16 ulp.
    assert rel_err(got, ref) < 1e-2
    assert np.mean(ulp_diff(got, ref) > 1) < 2e-3


def test_gemv_rows_are_independent_of_m(ctx):
    """k+1 verify rows give exactly the single-row results (deterministic
    split-K order), so a batched verify pass equals sequential decoding."""
    rng = np.random.default_rng(11)
    for bits, (n, k) in ((4, (2048, 1536)), (8, (1536, 8960)), (8, (17920, 1536))):
        packed, scale = random_codes(rng, n, k, bits, 64)
        w = _upload(ctx, packed, scale, bits, 64, n, k)
        x = rng.standard_normal((16, k)).astype(np.float16)
        full = w.matmul(x)
        for mm in (1, 5, 9):
            part = w.matmul(x[:mm])
            assert np.array_equal(part.view(np.uint16), full[:mm].view(np.uint16)), (bits, n, k, mm)
        assert np.array_equal(w.matmul(x[3:4]).view(np.uint16), full[3:4].view(np.uint16))


def test_fp16_weight_matmul_replaces_neon_kernel(ctx):
    """alm_matmul_f16_f16 has the semantics of androidllm's matmul_f16_f16."""
    from androidllm_b200.ops import matmul_f16
    rng = np.random.default_rng(3)
    a = rng.standard_normal((3, 200)).astype(np.float16)
    b = (rng.standard_normal((77, 200)) * 0.05).astype(np.float16)
    got = matmul_f16(a, b, ctx)
    from oracle.llama import matmul_f16 as ref_mm
    ref = ref_mm(a, b)
    assert rel_err(got, ref) < 1e-2
    assert np.max(ulp_diff(got, ref)) <= 1
