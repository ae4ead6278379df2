"""Data-parallel MLP step, world size 2 over gloo on CPU.

Each rank runs nova_b200.mlp.MLP.step on its half of the batch through the C++ host
layer (host test double of the C ABI), with a gloo-backed stand-in for the NCCL
Comm that averages the gradient tensors over ranks. The updated weights must equal
the reference's single-process step on the whole batch (oracle/_ref), because each
shard's loss is divided by its own size and the average over ranks undoes that.
The bias follows the reference quirk (SGD applies row 0 of the unreduced [B, U]
gradient): under data parallelism it moves by the average of the shards' row 0,
which is what the reference gives when run on each shard and averaged.
"""
import os
import pathlib
import socket
import sys

import numpy as np
import pytest

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent
DIMS = [16, 32, 32, 4]
BATCH = 24
LR = 1e-2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class GlooComm:
    """Stand-in for fusion.Comm: average tensors over ranks with gloo, then rebind."""

    def __init__(self, F, dist):
        self.F, self.dist = F, dist

    def allreduce_mean(self, tensors):
        import torch

        for t in tensors:
            a = torch.from_numpy(t.to_numpy().copy())
            self.dist.all_reduce(a)
            t.set_values((a / self.dist.get_world_size()).numpy().ravel())


def _gloo_transport(dist, ext_path):
    """Back the host double's collectives with gloo: the C++ Comm (watch / collect,
    flat_prefix, deferral) then runs unchanged over two CPU processes."""
    import ctypes as C

    import torch

    lib = C.CDLL(str(pathlib.Path(ext_path).parent / "libfusion_b200_hostfake.so"))
    FN = C.CFUNCTYPE(C.c_int, C.POINTER(C.c_float), C.c_int64)

    def allreduce(buf, n):
        a = np.ctypeslib.as_array(buf, shape=(n,))
        t = torch.from_numpy(a)  # shares the buffer
        dist.all_reduce(t)
        return 0
    cb = FN(allreduce)
    lib.fake_comm_set_transport(cb)
    return cb  # keep alive


def _worker_overlap(rank, world, port, out_dir, ext_path):
    """The bench's data-parallel path: F.Comm with watch/collect (each gradient
    all-reduced as the backward completes it, bias gradients cut to the row the update
    reads), the transport being gloo instead of NCCL."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import importlib.util

    import torch.distributed as dist

    sys.path[:0] = [str(ROOT), str(HERE)]
    import api_cases
    from nova_b200.mlp import MLP

    dist.init_process_group("gloo", rank=rank, world_size=world)
    spec = importlib.util.spec_from_file_location("hostfake.fusion", ext_path)
    F = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(F)
    keep = _gloo_transport(dist, ext_path)
    comm = F.Comm(world, rank, F.comm_unique_id())
    X, Y, Ws, bs = api_cases.mlp_inputs(31, DIMS, BATCH)
    lo, hi = rank * BATCH // world, (rank + 1) * BATCH // world
    model = MLP(F, Ws, bs)
    loss = model.step(model.tensor(X[lo:hi], True), model.tensor(Y[lo:hi], True), LR, comm)
    comm.wait(30.0)
    np.save(out_dir / f"r{rank}_overlapped.npy", np.array([comm.overlapped]))
    np.save(out_dir / f"r{rank}_loss.npy", loss.to_numpy())
    for i, (W, b) in enumerate(model.numpy_params()):
        np.save(out_dir / f"r{rank}_W{i}.npy", W)
        np.save(out_dir / f"r{rank}_b{i}.npy", b)
    comm.destroy()
    del keep
    dist.barrier()
    dist.destroy_process_group()


def _worker(rank, world, port, out_dir, ext_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import importlib.util

    import torch.distributed as dist

    sys.path[:0] = [str(ROOT), str(HERE)]
    import api_cases
    from nova_b200.mlp import MLP

    dist.init_process_group("gloo", rank=rank, world_size=world)
    spec = importlib.util.spec_from_file_location("hostfake.fusion", ext_path)
    F = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(F)
    X, Y, Ws, bs = api_cases.mlp_inputs(31, DIMS, BATCH)
    lo, hi = rank * BATCH // world, (rank + 1) * BATCH // world
    model = MLP(F, Ws, bs)
    x = model.tensor(X[lo:hi], True)
    y = model.tensor(Y[lo:hi], True)
    model.step(x, y, LR, GlooComm(F, dist))
    for i, (W, b) in enumerate(model.numpy_params()):
        np.save(out_dir / f"r{rank}_W{i}.npy", W)
        np.save(out_dir / f"r{rank}_b{i}.npy", b)
    dist.barrier()
    dist.destroy_process_group()


@pytest.fixture(scope="module")
def fake_ext():
    sys.path.insert(0, str(HERE / "hostfake"))
    import build_fake

    return build_fake.build()


def test_dp2_step_matches_reference_full_batch(tmp_path, fake_ext, ref):
    import torch.multiprocessing as mp

    import api_cases

    mp.spawn(_worker, args=(2, _free_port(), tmp_path, str(fake_ext)), nprocs=2, join=True)
    X, Y, Ws, bs = api_cases.mlp_inputs(31, DIMS, BATCH)
    W_full, _, _ = ref.mlp_step(X, Y, Ws, bs, LR)
    shard_b = []
    for r in range(2):
        lo, hi = r * BATCH // 2, (r + 1) * BATCH // 2
        _, b_r, _ = ref.mlp_step(X[lo:hi], Y[lo:hi], Ws, bs, LR)
        shard_b.append(b_r)
    for i in range(len(DIMS) - 1):
        w0, w1 = np.load(tmp_path / f"r0_W{i}.npy"), np.load(tmp_path / f"r1_W{i}.npy")
        np.testing.assert_array_equal(w0, w1)  # replicas stay identical
        err = np.linalg.norm(w0 - W_full[i]) / np.linalg.norm(W_full[i])
        assert err <= 1e-5, (i, err)
        b0 = np.load(tmp_path / f"r0_b{i}.npy")
        want_b = (shard_b[0][i] + shard_b[1][i]) / 2
        np.testing.assert_allclose(b0, want_b, rtol=1e-5, atol=1e-7)


def _check_dp2_against_reference(tmp_path, ref):
    import api_cases

    X, Y, Ws, bs = api_cases.mlp_inputs(31, DIMS, BATCH)
    W_full, _, _ = ref.mlp_step(X, Y, Ws, bs, LR)
    shard_b = []
    for r in range(2):
        lo, hi = r * BATCH // 2, (r + 1) * BATCH // 2
        _, b_r, _ = ref.mlp_step(X[lo:hi], Y[lo:hi], Ws, bs, LR)
        shard_b.append(b_r)
    for i in range(len(DIMS) - 1):
        w0, w1 = np.load(tmp_path / f"r0_W{i}.npy"), np.load(tmp_path / f"r1_W{i}.npy")
        np.testing.assert_array_equal(w0, w1)  # replicas stay identical
        err = np.linalg.norm(w0 - W_full[i]) / np.linalg.norm(W_full[i])
        assert err <= 1e-5, (i, err)
        b0, b1 = np.load(tmp_path / f"r0_b{i}.npy"), np.load(tmp_path / f"r1_b{i}.npy")
        np.testing.assert_array_equal(b0, b1)
        want_b = (shard_b[0][i] + shard_b[1][i]) / 2
        np.testing.assert_allclose(b0, want_b, rtol=1e-5, atol=1e-7)


def test_dp2_overlapped_comm_matches_reference_full_batch(tmp_path, fake_ext, ref):
    """The Comm path the benchmark runs at N > 1 (watch / collect / flat_prefix), at
    world size 2: same result as the reference's full-batch step, and every gradient
    was handed to the collective while the backward ran."""
    import torch.multiprocessing as mp

    mp.spawn(_worker_overlap, args=(2, _free_port(), tmp_path, str(fake_ext)), nprocs=2, join=True)
    _check_dp2_against_reference(tmp_path, ref)
    for r in range(2):
        assert int(np.load(tmp_path / f"r{r}_overlapped.npy")[0]) == 2 * (len(DIMS) - 1)


def test_comm_wait_timeout_aborts_and_refuses(fake_ext):
    """Watchdog on the host side: a collective stream still busy when Comm.wait's
    deadline passes aborts the communicator, raises, and later collectives are
    refused instead of hanging (stream time emulated by the host double)."""
    import ctypes as C
    import importlib.util

    spec = importlib.util.spec_from_file_location("hostfake.fusion", str(fake_ext))
    F = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(F)
    lib = C.CDLL(str(pathlib.Path(fake_ext).parent / "libfusion_b200_hostfake.so"))
    lib.fz_stream_delay.argtypes = [C.c_void_p, C.c_double]
    comm = F.Comm(1, 0, F.comm_unique_id())
    t = F.Tensor([4], [1.0, 2.0, 3.0, 4.0], F.CppDType.FLOAT32, F.CppDevice(F.CppDeviceType.CPU, 0), True)
    comm.allreduce_mean([t])
    comm.wait(1.0)  # nothing late: returns
    assert lib.fz_stream_delay(None, 1.0) == 0
    with pytest.raises(RuntimeError, match="did not complete"):
        comm.wait(0.2)
    with pytest.raises((RuntimeError, ValueError), match="aborted"):  # FZ_ERR_INVALID
        comm.allreduce_mean([t])
    comm.destroy()


def test_shards_cover_batch_once():
    world, batch = 8, 65536
    rows = [range(r * batch // world, (r + 1) * batch // world) for r in range(world)]
    flat = [i for r in rows for i in r]
    assert flat == list(range(batch))
