"""GEMMs whose TF32 remainder planes are derived in shared memory (FZ_GEMM_SPLIT_IN_KERNEL).

Contract: the product equals, bit for bit, the same call with the remainder planes
written by the separate pass (FZ_GEMM_SPLIT_PASS), for CTA pairs and single CTAs, K-
and MN-major operands, ragged K (the zero-filled edge of the last k-tile), batches and
split K; a supplied plane is not read then but gives the same values; calls the kernel
cannot split for (operands TMA cannot address) fall back to the pass. Both agree with a
float64 product within the GEMM bound |dC| <= 1e-5 (|A| |B|).
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_bits_equal

pytestmark = pytest.mark.gpu

TILES = {"auto": 0, "single": 1, "pair": 2}
PASS, IN_KERNEL = 1, 2


def _split_launches(A):
    n = C.c_int64()
    A.check(A.lib().fz_gemm_split_launches(C.byref(n)))
    return n.value


def _call(A, mode, tiles, batch, M, N, K, da, lda, sA, tA, db, ldb, sB, tB, a_lo=None, b_lo=None):
    L = A.lib()
    out = A.DeviceArray((batch, M, N))
    A.check(L.fz_gemm_set_split(mode))
    A.check(L.fz_gemm_set_tiles(TILES[tiles]))
    try:
        A.check(L.fz_gemm_f32_split(batch, M, N, K, da.ptr, a_lo, lda, sA, int(tA), db.ptr, b_lo, ldb, sB,
                                    int(tB), out.ptr, N, M * N, None))
        A.check(L.fz_kernel_status())
    finally:
        L.fz_gemm_set_split(0)
        L.fz_gemm_set_tiles(0)
    return out.numpy()


def _check_f64(got, a, b, tA, tB, what):
    a64 = np.swapaxes(a, 1, 2).astype(np.float64) if tA else a.astype(np.float64)
    b64 = np.swapaxes(b, 1, 2).astype(np.float64) if tB else b.astype(np.float64)
    want = a64 @ b64
    bound = 1e-5 * (np.abs(a64) @ np.abs(b64))
    err = np.abs(got.astype(np.float64) - want)
    assert np.all(err <= bound), f"{what}: worst |dC| / bound = {float(np.max(err / bound)):.3g}"


CASES = [
    # batch, M, N, K, tA, tB, tiles
    (1, 512, 512, 300, False, False, "single"),   # ragged K: zero-filled edge of the last k-tile
    (1, 1024, 1024, 512, False, True, "pair"),    # CTA pairs, K-major operands
    (1, 1024, 768, 512, True, False, "pair"),     # MN-major A and B
    (1, 1000, 1000, 1000, True, True, "single"),  # MN-major A, K-major B, ragged M, N, K
    (3, 256, 512, 200, False, False, "auto"),     # batch
    (1, 256, 256, 8192, False, False, "auto"),    # split over K: partials summed afterwards
    (64, 512, 512, 512, False, False, "auto"),    # the batched sweep product
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "x".join(map(str, c[:4])) + f"-{'T' if c[4] else 'N'}"
                         f"{'T' if c[5] else 'N'}-{c[6]}")
def test_split_in_kernel_equals_the_remainder_pass(capi, case):
    batch, M, N, K, tA, tB, tiles = case
    rng = np.random.default_rng(batch * 7 + M * 5 + N * 3 + K)
    a = (rng.standard_normal((batch, K, M) if tA else (batch, M, K)) / np.sqrt(K)).astype(np.float32)
    b = (rng.standard_normal((batch, N, K) if tB else (batch, K, N)) / np.sqrt(K)).astype(np.float32)
    da, db = capi.DeviceArray.from_numpy(a), capi.DeviceArray.from_numpy(b)
    args = (batch, M, N, K, da, a.shape[2], a.shape[1] * a.shape[2], tA, db, b.shape[2], b.shape[1] * b.shape[2], tB)
    n0 = _split_launches(capi)
    want = _call(capi, PASS, tiles, *args)
    assert _split_launches(capi) == n0
    got = _call(capi, IN_KERNEL, tiles, *args)
    assert _split_launches(capi) == n0 + 1
    assert_bits_equal(got, want, f"{case}: in-kernel split vs remainder pass")
    _check_f64(got, a, b, tA, tB, str(case))


def test_split_in_kernel_ignores_a_supplied_plane(capi):
    """One plane supplied (A's, from fz_tf32_lo), one missing: the kernel derives both."""
    L = capi.lib()
    M = N = K = 768
    rng = np.random.default_rng(31)
    a = rng.standard_normal((1, M, K)).astype(np.float32)
    b = rng.standard_normal((1, K, N)).astype(np.float32)
    da, db = capi.DeviceArray.from_numpy(a), capi.DeviceArray.from_numpy(b)
    alo = capi.DeviceArray((1, M, K))
    capi.check(L.fz_tf32_lo(alo.ptr, da.ptr, M * K, None))
    args = (1, M, N, K, da, K, M * K, False, db, N, K * N, False)
    want = _call(capi, PASS, "auto", *args, a_lo=alo.ptr)
    n0 = _split_launches(capi)
    got = _call(capi, IN_KERNEL, "auto", *args, a_lo=alo.ptr)
    assert _split_launches(capi) == n0 + 1
    assert_bits_equal(got, want, "one plane supplied")


def test_split_in_kernel_falls_back_when_tma_cannot_read_the_operand(capi):
    """A row pitch of 1001 floats is not a multiple of 16 bytes: the pass copies it."""
    M, N, K = 512, 512, 1001
    rng = np.random.default_rng(32)
    a = rng.standard_normal((1, M, K)).astype(np.float32)
    b = rng.standard_normal((1, K, N)).astype(np.float32)
    da, db = capi.DeviceArray.from_numpy(a), capi.DeviceArray.from_numpy(b)
    args = (1, M, N, K, da, K, M * K, False, db, N, K * N, False)
    want = _call(capi, PASS, "auto", *args)
    n0 = _split_launches(capi)
    got = _call(capi, IN_KERNEL, "auto", *args)
    assert _split_launches(capi) == n0
    assert_bits_equal(got, want, "fallback to the pass")
    _check_f64(got, a, b, False, False, "fallback")


def test_split_mode_argument_check(capi):
    assert capi.lib().fz_gemm_set_split(3) != 0
    capi.check(capi.lib().fz_gemm_set_split(0))
