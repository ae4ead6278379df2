"""Device-side random numbers (Philox-4x32-10) against the oracle's restatement.

fz_philox_uniform and fz_philox_dropout must give the oracle's values bit for bit
(the restatement is pinned to the algorithm's published known-answer vectors in
test_oracle_cpu.py), at any offset and size; Random.dropout must equal Nova's Dropout
composition over the same seed's stream, forward and backward.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_bits_equal

pytestmark = pytest.mark.gpu


def _lib(capi):
    L = capi.lib()
    L.fz_philox_uniform.argtypes = [C.c_void_p, C.c_int64, C.c_uint64, C.c_uint64, C.c_float, C.c_float, C.c_void_p]
    L.fz_philox_dropout.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_float, C.c_float, C.c_uint64,
                                    C.c_uint64, C.c_void_p]
    return L


@pytest.mark.parametrize("n,seed,offset,lo,hi", [(1, 1, 0, 0.0, 1.0), (7, 2 ** 40 + 3, 4, -1.0, 1.0),
                                                  ((1 << 22) + 3, 12345, 1 << 32, -3.5, 0.0),
                                                  (1 << 20, 0, 8, 1e-3, 1e-3 + 1e-6)])
def test_uniform_matches_oracle(capi, port, n, seed, offset, lo, hi):
    L = _lib(capi)
    out = capi.DeviceArray((n,))
    capi.check(L.fz_philox_uniform(out.ptr, n, seed, offset, lo, hi, None))
    got = out.numpy()
    assert_bits_equal(got, port.philox_uniform(n, seed, offset, lo, hi), "uniform")
    assert np.all((got >= np.float32(lo)) & (got < np.float32(hi)))


def test_uniform_statistics_and_errors(capi):
    L = _lib(capi)
    n = 1 << 24
    out = capi.DeviceArray((n,))
    capi.check(L.fz_philox_uniform(out.ptr, n, 99, 0, 0.0, 1.0, None))
    u = out.numpy().astype(np.float64)
    assert abs(u.mean() - 0.5) < 1e-3 and abs(u.var() - 1 / 12) < 1e-3
    hist = np.bincount((u * 16).astype(int), minlength=16) / n
    assert np.all(np.abs(hist - 1 / 16) < 1e-3)
    assert L.fz_philox_uniform(out.ptr, n, 99, 2, 0.0, 1.0, None) == 1  # offset not a multiple of 4
    assert L.fz_philox_uniform(out.ptr, n, 99, 0, 1.0, 1.0, None) == 1  # empty range


@pytest.mark.parametrize("n,rate", [(5, 0.5), ((1 << 21) + 1, 0.1), (4096, 0.0)])
def test_dropout_matches_oracle(capi, port, n, rate):
    L = _lib(capi)
    x = np.random.default_rng(n).standard_normal(n).astype(np.float32)
    x[:4] = [0.0, -0.0, np.inf, np.nan][: min(4, n)] if n >= 4 else x[:4]
    keep = np.float32(1.0 - rate)
    dx, do = capi.DeviceArray.from_numpy(x), capi.DeviceArray((n,))
    capi.check(L.fz_philox_dropout(do.ptr, dx.ptr, n, rate, keep, 2024, 16, None))
    with np.errstate(invalid="ignore"):
        assert_bits_equal(do.numpy(), port.philox_dropout(x, rate, keep, 2024, 16), "dropout")


def test_random_dropout_is_novas_composition(capi):
    """Forward and backward of Random.dropout equal Nova's Dropout ops over the same
    seed's device stream, bit for bit, and the stream advances per draw."""
    import nova_b200

    F = nova_b200.fusion
    X = np.random.default_rng(8).standard_normal((300, 257)).astype(np.float32)
    dev = F.CppDevice(F.CppDeviceType.CPU, 0)
    mk = lambda: F.Tensor(list(X.shape), X.ravel(), F.CppDType.FLOAT32, dev, True)
    r1, r2 = F.Random(4), F.Random(4)
    x1, x2 = mk(), mk()
    with F.grad_tape():
        y1 = r1.dropout(x1, 0.25)
        (y1 * y1).backward()
    with F.grad_tape():
        u = r2.uniform_device(list(X.shape), 0.0, 1.0, dev)
        y2 = x2 * (u >= 0.25) / (1 - 0.25)
        (y2 * y2).backward()
    assert_bits_equal(y1.to_numpy(), y2.to_numpy(), "forward")
    assert_bits_equal(x1.get_grad().to_numpy(), x2.get_grad().to_numpy(), "backward")
    kept = (y1.to_numpy() != 0).mean()
    assert abs(kept - 0.75) < 0.01
    y3 = r1.dropout(mk(), 0.25)  # the next draw: another mask
    assert not np.array_equal(y3.to_numpy() != 0, y1.to_numpy() != 0)
