"""Parity at the hot path's benchmark configurations, against the oracle.

The kernel tests elsewhere check each op on small and medium shapes; these run the
shapes the benchmark itself times, so the code paths only large problems take (the
CTA-pair GEMM with fused epilogues, K-split weight gradients, the cluster column
reductions, full-size elementwise grids) are held to the same bars:

* linear + ReLU forward, [512,1024] x [1024,512] + bias, through the Python API,
  against the reference CPU path (oracle/_ref);
* the MLP training step at full width (1024-4096-4096-4096-16) on 2048 rows through
  nova_b200.fusion, against the reference's own step (loss, updated parameters) and,
  gradient by gradient, against a float64 restatement of the step that replays each
  implementation's own ReLU decisions;
* the GEMM sweep: square 1024^3 and 4096^3 with B given plainly and transposed, the
  batched [64,512,512]^2, checked against float64 elementwise; 8192^3 and 16384^3
  (too large for a float64 product on the host in seconds) by float64 dot products
  at sampled output elements, a check whose cost does not grow with the output;
* axis reductions of [8192,8192] and the [64,256,64,64] (0,2,3) chain;
* elementwise ops at the sweep's largest size (2^28) and the [16384,16384] + [1,16384]
  row broadcast, bit for bit.

Bars as in the other parity tests: GEMM-bearing results 1e-5 norm-wise and
|dC| <= 1e-5 (|A||B|) elementwise; sums within 1e-5 * sum|x|; max, add/div/broadcast
bit-exact; exp within 2 ulp of glibc.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_bits_equal, ulp_diff

pytestmark = pytest.mark.gpu


def _rel(got, want):
    g, w = np.asarray(got, np.float64).ravel(), np.asarray(want, np.float64).ravel()
    return np.linalg.norm(g - w) / max(np.linalg.norm(w), 1e-30)


def _gemm_stats(capi):
    L = capi.lib()
    out = (C.c_int64 * 4)()
    capi.check(L.fz_gemm_stats(out))
    return {"pair": out[0], "single": out[1], "ksplit": out[2], "epilogue": out[3]}


# ---------------------------------------------------------------- C0: linear + ReLU
def test_linear_relu_512x1024x512(capi, ref):
    import nova_b200

    F = nova_b200.fusion
    rng = np.random.default_rng(1000)
    A = rng.standard_normal((512, 1024)).astype(np.float32)
    B = rng.standard_normal((1024, 512)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, 512).astype(np.float32)
    dev = F.CppDevice(F.CppDeviceType.CPU, 0)

    def t(a):
        return F.Tensor(list(a.shape), a.ravel(), F.CppDType.FLOAT32, dev, False)
    got = (t(A) @ t(B) + t(bias)).maximum(0.0).to_numpy()
    want = ref.binary_scalar("maximum", ref.binary("add", ref.matmul(A, B), bias), 0.0)
    assert _rel(got, want) <= 1e-5
    bound = np.abs(A).astype(np.float64) @ np.abs(B).astype(np.float64) + np.abs(bias)
    assert np.all(np.abs(got.astype(np.float64) - want) <= 1e-5 * bound + 1e-30)


# ---------------------------------------------------------------- C4: the MLP step
def test_mlp_step_full_width(capi, ref):
    """One SGD step of the benchmark's MLP (Kaiming-uniform weights, N(0,1) inputs and
    targets, lr 1e-3) on 2048 rows: the forward and input-gradient GEMMs run on the
    CTA-pair kernel with their bias+ReLU and ReLU-mask programs fused into the
    epilogue, the narrow layers and weight gradients on single CTAs split over K.

    A ReLU's gradient is discontinuous at 0: where a pre-activation lies within the
    GEMMs' rounding error of 0, two correct fp32 implementations may take different
    branches, and each such element moves a whole gradient entry. So the check is, per
    hidden layer and for the whole step:
      * updated parameters and the loss against the reference's step, 1e-5 norm-wise;
      * pre-activations against float64, within the GEMM bars;
      * every ReLU decision that differs from the reference's sits where the float64
        pre-activation is within 1e-5 * (|h| |W|^T + |b|) of 0 (rounding decides it);
      * the loss and every gradient against the float64 restatement of the step run
        with this backend's own ReLU decisions, 1e-5 norm-wise; and the reference's
        against the same restatement with its decisions (which pins the restatement).
    """
    import nova_b200
    import oracle
    from nova_b200.mlp import MLP, init_params

    F = nova_b200.fusion
    dims, rows, lr = [1024, 4096, 4096, 4096, 16], 2048, 1e-3
    Ws, bs = init_params(dims, 4242)
    rng = np.random.default_rng(4243)
    bs = [rng.uniform(-0.05, 0.05, b.shape).astype(np.float32) for b in bs]  # nonzero biases
    X = rng.standard_normal((rows, dims[0])).astype(np.float32)
    Y = rng.standard_normal((rows, dims[-1])).astype(np.float32)

    s0 = _gemm_stats(capi)
    model = MLP(F, Ws, bs)
    flat = [p for pair in model.params for p in pair]
    with F.grad_tape():
        loss = ((model.forward(model.tensor(X, True)) - model.tensor(Y, True)) ** 2)
        loss = loss / loss.size
        loss.backward()
    grads = [p.get_grad().to_numpy() for p in flat]
    for p in flat:
        p -= p.get_grad() * lr
    got_loss = loss.to_numpy()
    got_params = [p.to_numpy() for p in flat]
    s1 = _gemm_stats(capi)
    # this backend's pre-activations (same kernels and bits as inside the step)
    h, ts = model.tensor(X), []
    for i, (W, b) in enumerate(MLP(F, Ws, bs).params):
        t = h @ W.swapaxes(1, 0) + b
        ts.append(t.to_numpy())
        h = t.maximum(0.0)
    # the reference's step, gradients and pre-activations
    W2, b2, want_loss, want_grads = ref.mlp_step(X, Y, Ws, bs, lr, grads=True)
    hr, ref_ts = X, []
    for i in range(len(Ws)):
        t = ref.binary("add", ref.matmul(hr, ref.swapaxes(Ws[i], 0, 1)), bs[i])
        ref_ts.append(t)
        hr = ref.binary_scalar("maximum", t, 0.0)

    assert _rel(got_loss, want_loss) <= 1e-5
    for i in range(len(Ws)):
        assert _rel(got_params[2 * i], W2[i]) <= 1e-5, f"W{i}"
        assert _rel(got_params[2 * i + 1], b2[i]) <= 1e-5, f"b{i}"

    _, _, t64, _ = oracle.mlp_step_f64(X, Y, Ws, bs)
    h64 = X.astype(np.float64)
    for i in range(len(Ws) - 1):
        bound = np.abs(h64) @ np.abs(Ws[i].astype(np.float64)).T + np.abs(bs[i])
        assert _rel(ts[i], t64[i]) <= 1e-5, f"t{i}"
        assert np.all(np.abs(ts[i] - t64[i]) <= 1e-5 * bound), f"t{i} elementwise"
        flips = (ts[i] > 0) != (ref_ts[i] > 0)
        assert np.all(np.abs(t64[i][flips]) <= 1e-5 * bound[flips]), f"layer {i}: a ReLU decision differs away from 0"
        h64 = t64[i] * (t64[i] > 0)

    ours64 = oracle.mlp_step_f64(X, Y, Ws, bs, masks=[t > 0 for t in ts[:-1]])
    ref64 = oracle.mlp_step_f64(X, Y, Ws, bs, masks=[t > 0 for t in ref_ts[:-1]])
    assert _rel(got_loss, ours64[0]) <= 1e-5 and _rel(want_loss, ref64[0]) <= 1e-5
    for i in range(len(Ws)):
        for k, name in ((0, "gW"), (1, "gb")):
            assert grads[2 * i + k].shape == want_grads[i][k].shape
            assert _rel(grads[2 * i + k], ours64[1][i][k]) <= 1e-5, f"{name}{i}"
            assert _rel(want_grads[i][k], ref64[1][i][k]) <= 1e-5, f"reference {name}{i}"
    # the kernels the benchmark's step is made of all ran
    assert s1["pair"] > s0["pair"], s1
    assert s1["epilogue"] > s0["epilogue"], s1
    assert s1["ksplit"] > s0["ksplit"], s1
    assert s1["single"] > s0["single"], s1


# ---------------------------------------------------------------- C3: the GEMM sweep
def _gemm(capi, a, b, tB=False):
    batch, M, K = a.shape
    N = b.shape[1] if tB else b.shape[2]
    da, db, dc = capi.DeviceArray.from_numpy(a), capi.DeviceArray.from_numpy(b), capi.DeviceArray((batch, M, N))
    capi.check(capi.lib().fz_gemm_f32(batch, M, N, K, da.ptr, K, M * K, 0, db.ptr, b.shape[2],
                                      b.shape[1] * b.shape[2], int(tB), dc.ptr, N, M * N, None))
    capi.check(capi.lib().fz_kernel_status())
    out = dc.numpy()
    for arr in (da, db, dc):
        arr.free()
    return out


@pytest.mark.parametrize("batch,n", [(1, 1024), (1, 4096), (64, 512)])
@pytest.mark.parametrize("tB", [False, True])
def test_gemm_sweep_dense(capi, batch, n, tB):
    rng = np.random.default_rng(n + batch + tB)
    s = np.float32(1.0 / np.sqrt(n))  # entries ~ N(0, 1/sqrt(K))
    A = (rng.standard_normal((batch, n, n), dtype=np.float32) * s)
    B = (rng.standard_normal((batch, n, n), dtype=np.float32) * s)
    got = _gemm(capi, A, np.ascontiguousarray(B.transpose(0, 2, 1)) if tB else B, tB)
    A64, B64 = A.astype(np.float64), B.astype(np.float64)
    want = np.matmul(A64, B64)
    assert _rel(got, want) <= 1e-5
    bound = np.matmul(np.abs(A64), np.abs(B64))
    assert np.all(np.abs(got - want) <= 1e-5 * bound + 1e-30)


@pytest.mark.parametrize("n,tB", [(8192, False), (8192, True), (16384, False)])
def test_gemm_sweep_large_sampled(capi, n, tB):
    """Full-size products: float64 dot products at 4096 sampled (row, column) pairs,
    including the first and last rows and columns of the tile grid."""
    rng = np.random.default_rng(n + 7 * tB)
    s = np.float32(1.0 / np.sqrt(n))
    A = rng.standard_normal((1, n, n), dtype=np.float32) * s
    B = rng.standard_normal((1, n, n), dtype=np.float32) * s
    Bin = np.ascontiguousarray(B.transpose(0, 2, 1)) if tB else B
    got = _gemm(capi, A, Bin, tB)[0]
    del Bin
    rows = np.concatenate([[0, n - 1, 255, 256], rng.integers(0, n, 4092)])
    cols = np.concatenate([[0, n - 1, 256, 255], rng.integers(0, n, 4092)])
    a64 = A[0][rows].astype(np.float64)             # [S, K]
    b64 = B[0][:, cols].T.astype(np.float64)        # [S, K]
    want = np.einsum("sk,sk->s", a64, b64)
    bound = np.einsum("sk,sk->s", np.abs(a64), np.abs(b64))
    g = got[rows, cols].astype(np.float64)
    assert np.all(np.abs(g - want) <= 1e-5 * bound + 1e-30)
    assert np.linalg.norm(g - want) / np.linalg.norm(want) <= 1e-5


# ---------------------------------------------------------------- C2: reductions
@pytest.mark.parametrize("op", ["sum", "mean", "max"])
@pytest.mark.parametrize("axis", [0, 1])
def test_reduce_8192_squared(capi, port, op, axis):
    import nova_b200

    F = nova_b200.fusion
    x = np.random.default_rng(2002 + axis).standard_normal((8192, 8192), dtype=np.float32)
    t = F.Tensor([8192, 8192], x.ravel(), F.CppDType.FLOAT32, F.CppDevice(F.CppDeviceType.CPU, 0), False)
    got = getattr(t, op)(axis, False).to_numpy() if op != "max" else None
    if op == "max":  # no reference counterpart in the Python API: through the C ABI
        dx, do = capi.DeviceArray.from_numpy(x), capi.DeviceArray((8192,))
        outer, inner = (1, 8192) if axis == 0 else (8192, 1)
        capi.check(capi.lib().fz_reduce(capi.REDOPS["max"], do.ptr, dx.ptr, outer, 8192, inner, None))
        got = do.numpy()
    want = port.reduce(op, x, axis)
    if op == "max":
        assert_bits_equal(got, want, "max")
        return
    bound = np.abs(x.astype(np.float64)).sum(axis=axis)
    if op == "mean":
        bound /= 8192
    assert np.all(np.abs(got.astype(np.float64) - want) <= 1e-5 * bound + 1e-30)


@pytest.mark.parametrize("op", ["sum", "mean"])
def test_reduce_4d_axes023_chain(capi, ref, op):
    """x.op(3, True).op(2, True).op(0, True) on [64,256,64,64], as the reference can
    only express it (one axis per call); the backend joins the adjacent axes."""
    import nova_b200

    F = nova_b200.fusion
    x = np.random.default_rng(2004).standard_normal((64, 256, 64, 64), dtype=np.float32)
    t = F.Tensor(list(x.shape), x.ravel(), F.CppDType.FLOAT32, F.CppDevice(F.CppDeviceType.CPU, 0), False)
    got = getattr(getattr(getattr(t, op)(3, True), op)(2, True), op)(0, True).to_numpy()
    want = ref.reduce(op, ref.reduce(op, ref.reduce(op, x, 3, True), 2, True), 0, True)
    assert got.shape == want.shape == (1, 256, 1, 1)
    bound = np.abs(x.astype(np.float64)).sum(axis=(0, 2, 3), keepdims=True)
    if op == "mean":
        bound /= 64 * 64 * 64
    assert np.all(np.abs(got.astype(np.float64) - want) <= 1e-5 * bound + 1e-30)


# ---------------------------------------------------------------- C1: elementwise
def test_elementwise_largest_size(capi, port):
    n = 1 << 28
    rng = np.random.default_rng(2028)
    a = rng.uniform(-1, 1, n).astype(np.float32)
    b = rng.uniform(0.5, 2, n).astype(np.float32)
    da, db, do = capi.DeviceArray.from_numpy(a), capi.DeviceArray.from_numpy(b), capi.DeviceArray((n,))
    L = capi.lib()
    capi.check(L.fz_ewise_binary_contig(capi.BINOPS["div"], n, do.ptr, da.ptr, db.ptr, None))
    assert_bits_equal(do.numpy(), port.binary("div", a, b), "div 2^28")
    del b
    db.free()
    x = (rng.random(n, dtype=np.float32) * np.float32(8) - np.float32(4))  # U(-4, 4)
    dx = capi.DeviceArray.from_numpy(x)
    plan = capi.make_plan((n,), [(n,), (n,)])
    capi.check(L.fz_ewise_unary(capi.UNOPS["exp"], C.byref(plan), do.ptr, dx.ptr, None))
    assert ulp_diff(do.numpy(), port.unary("exp", x)).max() <= 2


def test_row_broadcast_16384(capi, port):
    r = 16384
    rng = np.random.default_rng(2016)
    a = rng.uniform(-1, 1, (r, r)).astype(np.float32)
    b = rng.uniform(-1, 1, (1, r)).astype(np.float32)
    plan = capi.make_plan((r, r), [(r, r), (r, r), (1, r)])
    da, db, do = capi.DeviceArray.from_numpy(a), capi.DeviceArray.from_numpy(b), capi.DeviceArray((r, r))
    capi.check(capi.lib().fz_ewise_binary(capi.BINOPS["add"], C.byref(plan), do.ptr, da.ptr, db.ptr, None))
    assert_bits_equal(do.numpy(), port.binary("add", a, b), "[16384,16384] + [1,16384]")
