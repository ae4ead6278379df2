"""fz_reduce_noalloc: the reduction entry point that allocates no device memory.

It exists for callers that must not allocate while they run (a runtime that
reserves and accounts for all device memory itself, or a latency-critical loop
that must not grow the allocator's pool). Called through the C ABI, it must give
the same results as fz_reduce -- bit for bit, since it launches the same kernels
with the same split plan -- on two calls in a row, so nothing left in its shared
fixed scratch from one call leaks into the next, and the pool must not change
across its calls. This file is collected last so a failure here comes after every
other test has run; it also passes on its own.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_bits_equal

pytestmark = pytest.mark.gpu

# rows split over CTAs (1<<22 and 3x50000 rows), columns split over chunks into the
# fixed array without the cluster kernel ((1,100000,3): 3 columns, no float4 path;
# (1,100000,64): too few column blocks for the cluster kernel at this size), columns
# folded by the cluster kernel ((2,777,1000), (1,8192,8192)), and unsplit shapes
SHAPES = [(1, 1 << 22, 1), (8192, 8192, 1), (1, 8192, 8192), (3, 50000, 1),
          (2, 777, 1000), (64 * 256, 64, 64), (5, 3, 7), (1, 100000, 3), (1, 100000, 64)]


def _noalloc(capi):
    L = capi.lib()
    L.fz_reduce_noalloc.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                    C.c_int64, C.c_void_p]
    L.fz_pool_stats.argtypes = [C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]
    return L


def _pool(capi, L):
    capi.check(L.fz_stream_sync(None))
    r, u = C.c_size_t(), C.c_size_t()
    capi.check(L.fz_pool_stats(C.byref(r), C.byref(u)))
    return r.value, u.value


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
            before = _pool(capi, L)
            capi.check(L.fz_reduce_noalloc(capi.REDOPS[op], got.ptr, dx.ptr, outer, ln, inner,
                                           None))
            assert _pool(capi, L) == before, f"{op} {outer}x{ln}x{inner}: the pool changed"
            assert_bits_equal(got.numpy(), ref.numpy(), f"{op} {outer}x{ln}x{inner} call {call}")


@pytest.mark.parametrize("shape", [(1, 100000, 3), (3, 50000, 1)])
def test_noalloc_matches_oracle(capi, port, shape):
    """Against the oracle's sequential fp32 sum (within 1e-5 * sum|x|) and its max
    (exact), on shapes whose split partials live in the fixed array."""
    L = _noalloc(capi)
    outer, ln, inner = shape
    x = np.random.default_rng(7).standard_normal(shape).astype(np.float32)
    dx, got = capi.DeviceArray.from_numpy(x), capi.DeviceArray((outer, inner))
    for op in ("sum", "max"):
        capi.check(L.fz_reduce_noalloc(capi.REDOPS[op], got.ptr, dx.ptr, outer, ln, inner, None))
        want = port.reduce(op, x, 1)
        if op == "max":
            assert_bits_equal(got.numpy(), want, "max")
        else:
            bound = np.abs(x.astype(np.float64)).sum(axis=1)
            assert np.all(np.abs(got.numpy().astype(np.float64) - want) <= 1e-5 * bound)
