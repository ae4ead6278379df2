"""The collective layer on one GPU: NCCL all-reduce through the C ABI, the Comm
path the data-parallel step runs (watch / collect / flat_prefix) at world size 1,
and the host-side watchdog of fz_comm_wait.

Failures here are made on the host only: a stream held back by a host-side pause
(fz_stream_delay) makes the wait run out; no collective is in flight when the
communicator is aborted, and no device fault is provoked.
"""
import ctypes as C
import os

import numpy as np
import pytest

from conftest import assert_bits_equal

pytestmark = pytest.mark.gpu
os.environ.setdefault("NCCL_NVLS_ENABLE", "0")

FZ_ERR_INVALID, FZ_ERR_TIMEOUT = 1, 6


def _comm(capi):
    L = capi.lib()
    L.fz_comm_unique_id.argtypes = [C.c_char_p]
    L.fz_stream_delay.argtypes = [C.c_void_p, C.c_double]
    uid = C.create_string_buffer(128)
    capi.check(L.fz_comm_unique_id(uid))
    c = C.c_void_p()
    capi.check(L.fz_comm_init(C.byref(c), 1, 0, uid))
    return L, c


def test_one_rank_allreduce(capi):
    L, c = _comm(capi)
    try:
        x = np.random.default_rng(5).standard_normal(1 << 20).astype(np.float32)
        d, o = capi.DeviceArray.from_numpy(x), capi.DeviceArray(x.shape)
        capi.check(L.fz_comm_allreduce(c, d.ptr, o.ptr, x.size, C.c_float(1.0), None))
        assert_bits_equal(o.numpy(), x, "sum over one rank")
        capi.check(L.fz_comm_allreduce(c, d.ptr, d.ptr, x.size, C.c_float(0.5), None))  # in place
        assert_bits_equal(d.numpy(), x * np.float32(0.5), "scaled sum")
        capi.check(L.fz_comm_wait(c, None, 30.0))
    finally:
        capi.check(L.fz_comm_destroy(c))


def test_watchdog_times_out_and_refuses(capi):
    """A stream still busy at the deadline: fz_comm_wait returns FZ_ERR_TIMEOUT after
    aborting the communicator, and later collectives are refused."""
    L, c = _comm(capi)
    s = C.c_void_p()
    capi.check(L.fz_stream_create(C.byref(s)))
    try:
        capi.check(L.fz_comm_wait(c, s, 5.0))  # idle stream: ok
        capi.check(L.fz_stream_delay(s, 1.0))
        assert L.fz_comm_wait(c, s, 0.2) == FZ_ERR_TIMEOUT
        assert b"aborted" in L.fz_last_error()
        buf = capi.DeviceArray((1024,))
        assert L.fz_comm_allreduce(c, buf.ptr, buf.ptr, 1024, C.c_float(1.0), None) == FZ_ERR_INVALID
        capi.check(L.fz_stream_sync(s))  # the pause ends; nothing else was queued
        assert L.fz_stream_delay(s, 61.0) == FZ_ERR_INVALID
    finally:
        capi.check(L.fz_comm_destroy(c))
        capi.check(L.fz_stream_destroy(s))
    capi.check(L.fz_kernel_status())


def test_overlapped_comm_step_equals_plain_step(capi):
    """MLP.step with F.Comm at world size 1 (gradients all-reduced on the side stream
    as the backward completes them, bias gradients cut to the row SGD reads) gives the
    plain step's parameters bit for bit."""
    import api_cases
    import nova_b200
    from nova_b200.mlp import MLP

    F = nova_b200.fusion
    X, Y, Ws, bs = api_cases.mlp_inputs(41, [64, 256, 256, 8], 512)
    bs = [np.linspace(-0.1, 0.1, b.size).astype(np.float32) for b in bs]
    comm = F.Comm(1, 0, F.comm_unique_id())
    try:
        a, b = MLP(F, Ws, bs), MLP(F, Ws, bs)
        for _ in range(2):
            la = a.step(a.tensor(X, True), a.tensor(Y, True), 1e-2, comm).to_numpy()
            lb = b.step(b.tensor(X, True), b.tensor(Y, True), 1e-2).to_numpy()
            comm.wait(30.0)
            assert_bits_equal(la, lb, "loss")
            assert comm.overlapped == 6
        for (Wa, ba), (Wb, bb) in zip(a.numpy_params(), b.numpy_params()):
            assert_bits_equal(Wa, Wb, "W")
            assert_bits_equal(ba, bb, "b")
    finally:
        comm.destroy()
