"""alm_qmatmul_noalloc, the dequant-GEMV that allocates no device memory.

Some callers of this library cannot call cudaMalloc once they are running
(real-time loops that cannot take its implicit synchronisation, hosts that
reserve all device memory up front).  This entry point keeps the split-K
scratch of the GEMV in a fixed array inside the library instead.  The test
drives it through the C ABI with a weight whose K is split across CTAs (so
the scratch is really used, asserted through alm_qweight_get_split) and
checks two calls in a row against alm_qmatmul, which allocates its scratch
normally, and against the oracle (dequantize_packed + an fp32 matmul).  A
weight whose split needs more than the fixed array must be rejected.  It
must pass alone in a fresh process and after the other GPU tests.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dev_buffer(lib, ctx, nbytes):
    p = ctypes.c_void_p()
    assert lib.alm_dev_alloc(ctx, nbytes, ctypes.byref(p)) == 0, lib.alm_last_error()
    return p


def _split(lib, w):
    a, b, c = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    assert lib.alm_qweight_get_split(w, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c)) == 0
    return a.value, b.value, c.value


def test_noalloc_gemv_matches_allocating_gemv():
    from androidllm_b200._lib import lib, ptr
    from gpu_helpers import random_codes, ref_matmul, rel_err
    from oracle.quant import dequantize_packed

    ctx = ctypes.c_void_p()
    assert lib.alm_ctx_create(0, ctypes.byref(ctx)) == 0, lib.alm_last_error()
    rng = np.random.default_rng(2024)
    n, k, m = 1536, 8960, 5          # the down projection of the 1.5B shape
    packed, scale = random_codes(rng, n, k, 8, 64)
    w = ctypes.c_void_p()
    assert lib.alm_qweight_upload(ctx, ptr(packed), ptr(scale), 8, 64, n, k, k, ctypes.byref(w)) == 0
    ksw, ksg, _ = _split(lib, w)
    assert ksg > 1, "the default launch shape must split K across CTAs, or the scratch goes unused"
    x = rng.standard_normal((m, k)).astype(np.float16)
    xd = _dev_buffer(lib, ctx, x.nbytes)
    yd = _dev_buffer(lib, ctx, m * n * 2)
    assert lib.alm_copy_h2d(ctx, xd, ptr(x), x.nbytes) == 0

    ref = np.empty((m, n), np.float16)
    assert lib.alm_qmatmul(ctx, w, xd, k, m, yd, n) == 0, lib.alm_last_error()
    assert lib.alm_copy_d2h(ctx, ptr(ref), yd, ref.nbytes) == 0
    oracle = ref_matmul(x, dequantize_packed(packed, scale, {"bits": 8, "block": 64, "out": n, "in": k}))

    for _ in range(2):                 # the shared array keeps the previous call's contents
        got = np.full((m, n), np.nan, np.float16)
        assert lib.alm_copy_h2d(ctx, yd, ptr(got), got.nbytes) == 0
        assert lib.alm_qmatmul_noalloc(ctx, w, xd, k, m, yd, n) == 0, lib.alm_last_error()
        assert lib.alm_copy_d2h(ctx, ptr(got), yd, got.nbytes) == 0
        # same kernel and summation order as alm_qmatmul: identical
        assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))
        # and within the GEMV tolerance of the oracle
        assert rel_err(got, oracle) < 1e-2

    # a split that needs more partial sums than the fixed array holds is rejected
    n2, k2 = 18944, 3584
    p2, s2 = random_codes(rng, n2, k2, 4, 64)
    w2 = ctypes.c_void_p()
    assert lib.alm_qweight_upload(ctx, ptr(p2), ptr(s2), 4, 64, n2, k2, k2, ctypes.byref(w2)) == 0
    assert lib.alm_qweight_set_split(w2, 1, 2) == 0, lib.alm_last_error()
    x2d = _dev_buffer(lib, ctx, k2 * 2)
    y2d = _dev_buffer(lib, ctx, n2 * 2)
    assert lib.alm_qmatmul_noalloc(ctx, w2, x2d, k2, 1, y2d, n2) == 1
    assert b"fixed scratch" in lib.alm_last_error()

    for b in (xd, yd, x2d, y2d):
        lib.alm_dev_free(ctx, b)
    lib.alm_qweight_free(w)
    lib.alm_qweight_free(w2)
    lib.alm_ctx_destroy(ctx)
