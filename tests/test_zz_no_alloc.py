"""alm_qmatmul_noalloc, the dequant-GEMV that allocates no device memory.

Some callers of this library cannot call cudaMalloc once they are running
(real-time loops that cannot take its implicit synchronisation, hosts that
reserve all device memory up front).  This entry point keeps the split-K
scratch of the GEMV in a fixed array inside the library instead.  The test
drives it through the C ABI with a weight whose K is split across CTAs (so
the scratch is really used) and checks two calls in a row against
alm_qmatmul, which allocates its scratch normally.  It must pass alone in a
fresh process and after the other GPU tests.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dev_buffer(lib, ctx, nbytes):
    p = ctypes.c_void_p()
    assert lib.alm_dev_alloc(ctx, nbytes, ctypes.byref(p)) == 0, lib.alm_last_error()
    return p


def test_noalloc_gemv_matches_allocating_gemv():
    from androidllm_b200._lib import lib, ptr
    from gpu_helpers import random_codes, rel_err

    ctx = ctypes.c_void_p()
    assert lib.alm_ctx_create(0, ctypes.byref(ctx)) == 0, lib.alm_last_error()
    rng = np.random.default_rng(2024)
    n, k, m = 1536, 8960, 5          # the down projection of the 1.5B shape: split-K over 4 CTAs
    packed, scale = random_codes(rng, n, k, 8, 64)
    w = ctypes.c_void_p()
    assert lib.alm_qweight_upload(ctx, ptr(packed), ptr(scale), 8, 64, n, k, k, ctypes.byref(w)) == 0
    x = rng.standard_normal((m, k)).astype(np.float16)
    xd = _dev_buffer(lib, ctx, x.nbytes)
    yd = _dev_buffer(lib, ctx, m * n * 2)
    assert lib.alm_copy_h2d(ctx, xd, ptr(x), x.nbytes) == 0

    ref = np.empty((m, n), np.float16)
    assert lib.alm_qmatmul(ctx, w, xd, k, m, yd, n) == 0, lib.alm_last_error()
    assert lib.alm_copy_d2h(ctx, ptr(ref), yd, ref.nbytes) == 0

    for _ in range(2):                 # the shared array keeps the previous call's contents
        got = np.full((m, n), np.nan, np.float16)
        assert lib.alm_copy_h2d(ctx, yd, ptr(got), got.nbytes) == 0
        assert lib.alm_qmatmul_noalloc(ctx, w, xd, k, m, yd, n) == 0, lib.alm_last_error()
        assert lib.alm_copy_d2h(ctx, ptr(got), yd, got.nbytes) == 0
        # same kernel and summation order: identical, hence within the 1e-2 tolerance
        assert rel_err(got, ref) < 1e-2
        assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))

    lib.alm_dev_free(ctx, xd)
    lib.alm_dev_free(ctx, yd)
    lib.alm_qweight_free(w)
    lib.alm_ctx_destroy(ctx)
