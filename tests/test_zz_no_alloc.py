"""fz_reduce_noalloc: the reduction entry point that allocates no device memory.

It exists for callers that must not allocate while they run (a runtime that
reserves and accounts for all device memory itself, or a latency-critical loop
that must not grow the allocator's pool). Called through the C ABI, it must give
the same results as fz_reduce -- bit for bit, since it launches the same kernels
with the same split plan -- on two calls in a row, so nothing left in its shared
fixed scratch from one call leaks into the next. This file is collected last so
a failure here comes after every other test has run; it also passes on its own.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_bits_equal

pytestmark = pytest.mark.gpu

# rows split over CTAs, columns split over chunks, and unsplit shapes
SHAPES = [(1, 1 << 22, 1), (8192, 8192, 1), (1, 8192, 8192), (3, 50000, 1),
          (2, 777, 1000), (64 * 256, 64, 64), (5, 3, 7)]


def _noalloc(capi):
    L = capi.lib()
    L.fz_reduce_noalloc.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                    C.c_int64, C.c_void_p]
    return L


@pytest.mark.parametrize("op", ["sum", "mean", "max"])
def test_noalloc_matches_fz_reduce_twice(capi, op):
    L = _noalloc(capi)
    rng = np.random.default_rng(2024)
    for outer, ln, inner in SHAPES:
        for call in range(2):  # two calls in a row, different data
            x = rng.standard_normal((outer, ln, inner)).astype(np.float32)
            dx = capi.DeviceArray.from_numpy(x)
            ref, got = capi.DeviceArray((outer, inner)), capi.DeviceArray((outer, inner))
            capi.check(L.fz_reduce(capi.REDOPS[op], ref.ptr, dx.ptr, outer, ln, inner, None))
            capi.check(L.fz_reduce_noalloc(capi.REDOPS[op], got.ptr, dx.ptr, outer, ln, inner,
                                           None))
            assert_bits_equal(got.numpy(), ref.numpy(), f"{op} {outer}x{ln}x{inner} call {call}")
