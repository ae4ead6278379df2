"""The C++ host layer (fusion-IR lowering, autodiff engine, Fusion's op semantics and
quirks) on CPU, through a host-memory test double of the C ABI
(tests/hostfake/fake_fz.cpp), against the reference module's golden outputs.

The double computes every op with the same fp32 semantics as the sm_100a kernels,
so this checks the host logic without a GPU; tests/test_api_gpu.py runs the same
cases on the real kernels."""
import importlib.util
import pathlib
import sys

import numpy as np
import pytest

import api_cases
from conftest import assert_bits_equal
from test_api_gpu import GOLDEN, _compare, _kinds

HERE = pathlib.Path(__file__).resolve().parent


@pytest.fixture(scope="module")
def fake_fusion():
    sys.path.insert(0, str(HERE / "hostfake"))
    import build_fake

    try:
        ext = build_fake.build()
    except Exception as e:  # pragma: no cover
        pytest.skip(f"cannot build the host test double: {e}")
    spec = importlib.util.spec_from_file_location("hostfake.fusion", ext)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_host_layer_matches_reference(fake_fusion):
    res = api_cases.run_all(fake_fusion)
    golden = np.load(GOLDEN / "api_golden.npz")
    kinds = _kinds()
    failures = []
    for key in sorted(golden.files):
        want = golden[key]
        if want.size == 0:
            continue
        try:
            _compare(key, kinds[key], res[key], want)
        except AssertionError as e:
            failures.append(str(e))
    assert not failures, "\n".join(failures)


def test_fusion_off_matches_fusion_on(fake_fusion):
    F = fake_fusion
    F.set_fusion(False)
    try:
        eager = api_cases.run_all(F)
    finally:
        F.set_fusion(True)
    fused = api_cases.run_all(F)
    for k in eager:
        np.testing.assert_array_equal(fused[k].view(np.uint32), eager[k].view(np.uint32), err_msg=k)


def test_lazy_chain_lowers_once(fake_fusion):
    F = fake_fusion
    x = api_cases.T(F, np.arange(12.0).reshape(3, 4))
    b = api_cases.T(F, [1.0, -2.0, 3.0, -4.0])
    y = ((x + b) * 2.0 - 1.0).maximum(0.0)
    assert y.is_pending()
    before = F.stats()["fused_launches"]
    out = y.to_numpy()
    assert F.stats()["fused_launches"] == before + 1
    want = np.maximum((np.arange(12.0).reshape(3, 4) + [1, -2, 3, -4]) * 2 - 1, 0)
    np.testing.assert_array_equal(out, want.astype(np.float32))


def test_inplace_write_keeps_pending_readers(fake_fusion):
    """`p -= g` must not change a pending value that read p earlier."""
    F = fake_fusion
    p = api_cases.T(F, [1.0, 2.0, 3.0])
    q = p * 10.0          # pending, reads p
    p -= api_cases.T(F, [1.0, 1.0, 1.0])
    np.testing.assert_array_equal(q.to_numpy(), [10.0, 20.0, 30.0])
    np.testing.assert_array_equal(p.to_numpy(), [0.0, 1.0, 2.0])


def test_second_backward_zeroes_shared_grads(fake_fusion):
    """Leaf grads alias the engine's grad buffers (reference Engine.hpp:277-283)."""
    F = fake_fusion
    with F.grad_tape():
        a = api_cases.T(F, [1.0, 2.0], True)
        c = a * 3.0
        c.backward()
        g1 = a.get_grad()
        first = g1.to_numpy().copy()
        np.testing.assert_array_equal(first, [3.0, 3.0])


def test_split_planes_follow_values(fake_fusion):
    """A GEMM operand's TF32 remainder plane is split once per buffer and never
    outlives the value: after `-=` or set_values the operand is a new buffer and gets
    a new plane (the test double refuses a plane that does not match its operand)."""
    F = fake_fusion
    rng = np.random.default_rng(5)
    a = rng.standard_normal((8, 12)).astype(np.float32)
    w = rng.standard_normal((12, 4)).astype(np.float32)
    x, W = api_cases.T(F, a), api_cases.T(F, w)
    assert F.split_cache_enabled()
    y1 = (x @ W).to_numpy()
    launches = F.stats()["kernel_launches"]
    y2 = (x @ W).to_numpy()  # both planes cached: one GEMM launch, no splits
    assert F.stats()["kernel_launches"] == launches + 1
    np.testing.assert_array_equal(y1, y2)
    d = rng.standard_normal((12, 4)).astype(np.float32)
    W -= api_cases.T(F, d)
    np.testing.assert_allclose((x @ W).to_numpy(), a.astype(np.float64) @ (w - d), rtol=1e-5, atol=1e-5)
    x.set_values(np.ones(96, np.float32))
    np.testing.assert_allclose((x @ W).to_numpy(), np.ones((8, 12)) @ (w - d), rtol=1e-5, atol=1e-5)
    F.set_split_cache(False)
    try:
        np.testing.assert_allclose((x @ W).to_numpy(), np.ones((8, 12)) @ (w - d), rtol=1e-5, atol=1e-5)
    finally:
        F.set_split_cache(True)


def test_inplace_update_does_not_grow_readers(fake_fusion):
    """`b -= g` leaves b materialised: a parameter updated every step and read by a
    fused consumer must not be re-evaluated from its whole update history."""
    F = fake_fusion
    x = api_cases.T(F, np.ones((4, 3)))
    b = api_cases.T(F, [0.5, -0.5, 1.0])
    g = api_cases.T(F, [0.25, 0.25, 0.25])
    want = np.array([0.5, -0.5, 1.0], np.float32)
    for _ in range(6):
        y = (x + b).maximum(0.0)
        np.testing.assert_array_equal(y.to_numpy(), np.maximum(1.0 + want, 0.0)[None].repeat(4, 0))
        b -= g * 2.0
        want = want - np.float32(0.5)
        assert not b.is_pending()
    np.testing.assert_array_equal(b.to_numpy(), want)


def test_pending_gemm_operand_lowered_with_its_plane(fake_fusion):
    """A pending operand of `@` is lowered together with its TF32 remainder plane (one
    fused program with two outputs), so no separate split pass runs for it."""
    F = fake_fusion
    rng = np.random.default_rng(9)
    x = api_cases.T(F, rng.standard_normal((16, 8)))
    b = api_cases.T(F, rng.standard_normal(8))
    W = api_cases.T(F, rng.standard_normal((8, 4)))
    (x @ W).to_numpy()  # W gets its plane here
    y = (x + b).maximum(0.0)
    assert y.is_pending()
    before = F.stats()["kernel_launches"]
    z = y @ W
    assert F.stats()["kernel_launches"] - before == 1  # the fused program (value + plane)
    assert z.is_pending()  # the GEMM itself waits for its first reader
    want = np.maximum(x.to_numpy() + b.to_numpy(), 0).astype(np.float64) @ W.to_numpy()
    np.testing.assert_allclose(z.to_numpy(), want, rtol=1e-5, atol=1e-6)
    assert F.stats()["kernel_launches"] - before == 2


def test_overlapped_gradient_average_matches_plain_step(fake_fusion):
    """Comm.watch/collect (each gradient all-reduced as the backward completes it) gives
    the same update as the plain step; with one rank the average is the gradient, and
    a bias moves by row 0 of its [B, U] gradient either way."""
    from nova_b200.mlp import MLP

    F = fake_fusion
    X, Y, Ws, bs = api_cases.mlp_inputs(5, [8, 16, 16, 4], 12)
    bs = [np.linspace(-0.1, 0.1, b.size).astype(np.float32) for b in bs]
    plain, over = MLP(F, Ws, bs), MLP(F, Ws, bs)
    comm = F.Comm(1, 0, F.comm_unique_id())
    for _ in range(2):
        lp = plain.step(plain.tensor(X, True), plain.tensor(Y, True), 1e-2)
        lo = over.step(over.tensor(X, True), over.tensor(Y, True), 1e-2, comm)
        np.testing.assert_array_equal(lo.to_numpy(), lp.to_numpy())
        assert comm.overlapped == 6  # every parameter's gradient went out during backward()
    for (Wp, bp), (Wo, bo) in zip(plain.numpy_params(), over.numpy_params()):
        np.testing.assert_array_equal(Wo, Wp)
        np.testing.assert_array_equal(bo, bp)
    comm.destroy()


def test_sibling_gradients_lowered_together(fake_fusion):
    """Multiply backward over two leaves: g0*y and g0*x come out of one fused program
    (one pass over g0, x and y), with the same values as separate lowering."""
    F = fake_fusion
    rng = np.random.default_rng(4)
    a, b, g = (rng.standard_normal((64, 32)).astype(np.float32) for _ in range(3))
    x, y = api_cases.T(F, a, True), api_cases.T(F, b, True)
    gt = api_cases.T(F, g)
    with F.grad_tape():
        z = x * y
        w = z * gt
        before = F.stats()["fused_launches"]
        w.backward()
        after = F.stats()["fused_launches"]
    assert after - before == 1
    np.testing.assert_array_equal(x.get_grad().to_numpy(), (np.ones_like(g) * g) * b)
    np.testing.assert_array_equal(y.get_grad().to_numpy(), (np.ones_like(g) * g) * a)


@pytest.mark.parametrize("op", ["sum", "mean", "max"])
def test_reduction_chains_join_adjacent_axes(fake_fusion, op):
    """x.op(3, True).op(2, True) joins into one reduction over the merged axes (one
    launch), a non-adjacent axis starts a new one; values match numpy's."""
    F = fake_fusion
    rng = np.random.default_rng(11)
    a = rng.standard_normal((4, 5, 6, 7)).astype(np.float32)
    x = api_cases.T(F, a)
    f = {"sum": np.sum, "mean": np.mean, "max": np.max}[op]
    if op == "max" and not hasattr(F.Tensor, "max"):
        pytest.skip("no max reduction in this module")
    before = F.stats()["kernel_launches"]
    y = getattr(getattr(getattr(x, op)(3, True), op)(2, True), op)(0, True)
    got = y.to_numpy()
    assert F.stats()["kernel_launches"] - before == 2  # axes (2, 3) joined, then axis 0
    want = f(a.astype(np.float64), axis=(0, 2, 3), keepdims=True)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)
    # keepdim=False chain over adjacent axes, and a non-adjacent pair
    z = getattr(getattr(x, op)(3), op)(2)
    np.testing.assert_allclose(z.to_numpy(), f(a.astype(np.float64), axis=(2, 3)), rtol=1e-5, atol=1e-5)
    before = F.stats()["kernel_launches"]
    w = getattr(getattr(x, op)(1, True), op)(3, True)
    np.testing.assert_allclose(w.to_numpy(), f(a.astype(np.float64), axis=(1, 3), keepdims=True),
                               rtol=1e-5, atol=1e-5)
    assert F.stats()["kernel_launches"] - before == 2
    # a pending reduction feeding an elementwise op is lowered first
    v = (getattr(x, op)(3, True) + 1.0).to_numpy()
    np.testing.assert_allclose(v, f(a.astype(np.float64), axis=3, keepdims=True) + 1, rtol=1e-5, atol=1e-5)


def test_reduction_chain_edge_cases(fake_fusion):
    """Joined reductions stop where they must: a global reduction after an axis
    reduction, mixed keepdim, different ops, and a chain read twice."""
    F = fake_fusion
    rng = np.random.default_rng(12)
    a = rng.standard_normal((3, 4, 5)).astype(np.float32)
    x = api_cases.T(F, a)
    d = a.astype(np.float64)
    np.testing.assert_allclose(x.sum(2).sum().to_numpy(), [d.sum()], rtol=1e-5)
    np.testing.assert_allclose(x.sum(2, True).sum(1).to_numpy(), d.sum(axis=2, keepdims=True).sum(axis=1),
                               rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(x.mean(2, True).sum(1, True).to_numpy(),
                               d.mean(axis=2, keepdims=True).sum(axis=1, keepdims=True), rtol=1e-5, atol=1e-6)
    y = x.sum(1, True)
    z1 = y.sum(2, True).to_numpy()  # joined with y's pending reduction
    z2 = y.to_numpy()               # y itself is still its own value
    np.testing.assert_allclose(z1, d.sum(axis=(1, 2), keepdims=True), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(z2, d.sum(axis=1, keepdims=True), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(x.sum(0).sum(0).sum(0).to_numpy(), [d.sum()], rtol=1e-5)


def _stat(F, k):
    return F.stats()[k]


def _plain(F, fn):
    """fn() evaluated with every GEMM launched where it is called."""
    F.set_gemm_epilogue(False)
    try:
        return fn()
    finally:
        F.set_gemm_epilogue(True)


def _mlp_layer_inputs(F, seed):
    rng = np.random.default_rng(seed)
    arrs = [rng.standard_normal(s).astype(np.float32) for s in [(32, 8), (8, 16), (16,), (16, 4)]]
    x, W, b, W2 = (api_cases.T(F, a) for a in arrs)
    (x @ W).to_numpy()  # the operands' TF32 remainder planes are made here
    (api_cases.T(F, np.ones((2, 16), np.float32)) @ W2).to_numpy()
    return x, W, b, W2


def test_bias_relu_runs_in_the_gemm_epilogue(fake_fusion):
    """max(x @ W + b, 0) read by the next `@` is written, with its TF32 remainder plane,
    by the epilogue of the x @ W GEMM: one kernel, the product itself not stored (no
    tensor holds it), values equal to the unfused lowering bit for bit."""
    F = fake_fusion
    x, W, b, W2 = _mlp_layer_inputs(F, 11)
    e0, k0, u0 = _stat(F, "epilogue_gemms"), _stat(F, "kernel_launches"), _stat(F, "pool_used_bytes")
    y = ((x @ W) + b).maximum(0.0)
    z = y @ W2
    assert _stat(F, "epilogue_gemms") - e0 == 1
    assert _stat(F, "kernel_launches") - k0 == 1
    assert _stat(F, "pool_used_bytes") - u0 == 2 * y.size * 4  # y and its plane only
    assert z.is_pending()
    want_y, want_z = _plain(F, lambda: (((x @ W) + b).maximum(0.0).to_numpy(),
                                        (((x @ W) + b).maximum(0.0) @ W2).to_numpy()))
    np.testing.assert_array_equal(y.to_numpy(), want_y)
    np.testing.assert_array_equal(z.to_numpy(), want_z)


def test_gemm_epilogue_stores_a_product_still_held(fake_fusion):
    """When a tensor still holds the product, the same epilogue stores it too."""
    F = fake_fusion
    x, W, b, W2 = _mlp_layer_inputs(F, 12)
    e0, k0, u0 = _stat(F, "epilogue_gemms"), _stat(F, "kernel_launches"), _stat(F, "pool_used_bytes")
    t = x @ W
    y = (t + b).maximum(0.0)
    y @ W2
    assert _stat(F, "epilogue_gemms") - e0 == 1
    assert _stat(F, "kernel_launches") - k0 == 1
    assert not t.is_pending()
    assert _stat(F, "pool_used_bytes") - u0 == 3 * y.size * 4  # y, its plane and t
    np.testing.assert_array_equal(t.to_numpy(), _plain(F, lambda: (x @ W).to_numpy()))


def test_pending_product_operand_gets_value_and_plane_from_its_epilogue(fake_fusion):
    F = fake_fusion
    x, W, b, W2 = _mlp_layer_inputs(F, 13)
    e0, k0 = _stat(F, "epilogue_gemms"), _stat(F, "kernel_launches")
    t = x @ W
    z = t @ W2
    assert _stat(F, "epilogue_gemms") - e0 == 1 and _stat(F, "kernel_launches") - k0 == 1
    assert not t.is_pending() and z.is_pending()
    np.testing.assert_array_equal(z.to_numpy(), _plain(F, lambda: ((x @ W) @ W2).to_numpy()))


def test_program_over_two_products_lowers_them_plainly(fake_fusion):
    F = fake_fusion
    x, W, b, W2 = _mlp_layer_inputs(F, 14)
    e0, k0 = _stat(F, "epilogue_gemms"), _stat(F, "kernel_launches")
    y = ((x @ W) + (x @ W) * 2.0).to_numpy()
    assert _stat(F, "epilogue_gemms") == e0
    assert _stat(F, "kernel_launches") - k0 == 3  # two GEMMs and the fused program
    np.testing.assert_array_equal(y, _plain(F, lambda: ((x @ W) + (x @ W) * 2.0).to_numpy()))


@pytest.mark.parametrize("cshape,fused", [((2, 3, 1, 5), True), ((5,), True), ((4, 1), True),
                                          ((2, 1, 4, 5), False), ((3, 4, 5), False)])
def test_epilogue_inputs_broadcast_over_batched_products(fake_fusion, cshape, fused):
    """Inputs whose batch dims flatten into one stride run in the epilogue; others (a
    broadcast batch dim in front of a varying one) fall back to a plain GEMM and a fused
    program; both give the unfused values."""
    F = fake_fusion
    rng = np.random.default_rng(15)
    a = api_cases.T(F, rng.standard_normal((2, 3, 4, 8)))
    w = api_cases.T(F, rng.standard_normal((2, 3, 8, 5)))
    c = api_cases.T(F, rng.standard_normal(cshape))
    e0 = _stat(F, "epilogue_gemms")
    got = ((a @ w) * c - 1.0).to_numpy()
    assert (_stat(F, "epilogue_gemms") - e0 == 1) == fused
    np.testing.assert_array_equal(got, _plain(F, lambda: ((a @ w) * c - 1.0).to_numpy()))


def test_mlp_step_with_gemm_epilogues_matches_plain(fake_fusion):
    """A training step with deferred GEMMs gives the eager-GEMM step's values bit for bit;
    each hidden layer's bias + ReLU and ReLU-mask gradient run in GEMM epilogues."""
    from nova_b200.mlp import MLP

    F = fake_fusion
    X, Y, Ws, bs = api_cases.mlp_inputs(6, [8, 16, 16, 16, 4], 12)
    bs = [np.linspace(-0.1, 0.1, b.size).astype(np.float32) for b in bs]
    fused, plain = MLP(F, Ws, bs), MLP(F, Ws, bs)
    for _ in range(2):
        e0 = _stat(F, "epilogue_gemms")
        lf = fused.step(fused.tensor(X, True), fused.tensor(Y, True), 1e-2).to_numpy()
        # forward: 3 bias+ReLU layers and the output layer's loss gradient; backward: the
        # ReLU-mask input gradients of the 3 hidden layers; update: the 4 weights' SGD
        # steps, run in the epilogues of the weight-gradient GEMMs (W.T is a view, so
        # its gradient's swapaxes is the transposed product, in W's layout)
        assert _stat(F, "epilogue_gemms") - e0 == 11
        lp = _plain(F, lambda: plain.step(plain.tensor(X, True), plain.tensor(Y, True), 1e-2).to_numpy())
        np.testing.assert_array_equal(lf, lp)
    for (Wf, bf), (Wp, bp) in zip(fused.numpy_params(), plain.numpy_params()):
        np.testing.assert_array_equal(Wf, Wp)
        np.testing.assert_array_equal(bf, bp)


def test_swapaxes_view_is_read_in_place_by_gemms(fake_fusion):
    """x @ W.T reads W in the other operand layout and the backward reads it back in
    its own: a training step of a Linear layer transposes nothing, and the weight's
    gradient lands in W's layout straight from the GEMM."""
    F = fake_fusion
    rng = np.random.default_rng(31)
    X, W, b = rng.standard_normal((12, 8)), rng.standard_normal((6, 8)), rng.standard_normal((6,))
    x, w, bt = api_cases.T(F, X, True), api_cases.T(F, W, True), api_cases.T(F, b, True)
    s0 = _stat(F, "swap_materializations")
    with F.grad_tape():
        y = (x @ w.swapaxes(1, 0) + bt).maximum(0.0)
        loss = y * y
        loss.backward()
    gw, gx = w.get_grad().to_numpy(), x.get_grad().to_numpy()
    out = y.to_numpy()
    assert _stat(F, "swap_materializations") == s0
    pre = X.astype(np.float32) @ W.astype(np.float32).T + b.astype(np.float32)
    g = 2 * np.maximum(pre, 0) * (pre > 0)
    np.testing.assert_allclose(out, np.maximum(pre, 0), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(gw, g.T @ X, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(gx, g @ W, rtol=1e-4, atol=1e-5)


def test_swapaxes_view_values_and_copy_semantics(fake_fusion):
    """A view equals the transposed copy wherever it is read; a swapaxes of a view is
    the source; an in-place write to the source later leaves the view's values as they
    were (swapaxes has copy semantics); other axes are transposed at once."""
    F = fake_fusion
    rng = np.random.default_rng(32)
    A = rng.standard_normal((2, 5, 3)).astype(np.float32)
    a = api_cases.T(F, A)
    v = a.swapaxes(2, 1)
    assert v.shape == [2, 3, 5]
    s0 = _stat(F, "swap_materializations")
    back = v.swapaxes(1, 2)
    np.testing.assert_array_equal(back.to_numpy(), A)
    assert _stat(F, "swap_materializations") == s0
    a -= api_cases.T(F, np.ones_like(A))  # rebinds a's storage; v keeps the old value
    np.testing.assert_array_equal((v + 0.0).to_numpy(), A.transpose(0, 2, 1))
    assert _stat(F, "swap_materializations") == s0 + 1  # the elementwise read materialised it
    np.testing.assert_array_equal(v.to_numpy(), A.transpose(0, 2, 1))
    assert _stat(F, "swap_materializations") == s0 + 1  # once
    np.testing.assert_array_equal(a.swapaxes(0, 2).to_numpy(), (A - 1).transpose(2, 1, 0))
    np.testing.assert_array_equal(v.sum(2, False).to_numpy(), A.transpose(0, 2, 1).sum(2))


def test_swapaxes_of_a_pending_product_is_the_transposed_product(fake_fusion):
    F = fake_fusion
    rng = np.random.default_rng(33)
    A, B = rng.standard_normal((7, 4)), rng.standard_normal((4, 9))
    a, b = api_cases.T(F, A), api_cases.T(F, B)
    s0 = _stat(F, "swap_materializations")
    p = a @ b
    assert p.is_pending()
    t = p.swapaxes(0, 1)
    assert t.shape == [9, 7] and t.is_pending()
    got = (t * 2.0).to_numpy()
    assert _stat(F, "swap_materializations") == s0
    want = (A.astype(np.float32) @ B.astype(np.float32)).T * 2
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(p.to_numpy(), want.T / 2, rtol=1e-5, atol=1e-6)


def test_swap_views_off_materialises_like_the_reference(fake_fusion):
    F = fake_fusion
    X = np.arange(12, dtype=np.float32).reshape(3, 4)
    F.set_swap_views(False)
    try:
        s0 = _stat(F, "swap_materializations")
        t = api_cases.T(F, X).swapaxes(1, 0)
        assert not t.is_pending()
        np.testing.assert_array_equal(t.to_numpy(), X.T)
        assert _stat(F, "swap_materializations") == s0
    finally:
        F.set_swap_views(True)


def test_weight_update_keeps_its_remainder_plane(fake_fusion):
    """After a training step the weights' new values carry their TF32 remainder planes
    (written by the update program), so the next forward splits no weight."""
    from nova_b200.mlp import MLP

    F = fake_fusion
    X, Y, Ws, bs = api_cases.mlp_inputs(8, [8, 16, 4], 10)
    m = MLP(F, Ws, bs)
    m.step(m.tensor(X, True), m.tensor(Y, True), 1e-2).to_numpy()
    m.step(m.tensor(X, True), m.tensor(Y, True), 1e-2).to_numpy()
    t0 = _stat(F, "lo_splits")
    m.step(m.tensor(X, True), m.tensor(Y, True), 1e-2).to_numpy()
    # the input batch X is split once (it arrives from the host); no weight is
    assert _stat(F, "lo_splits") - t0 == 1


def test_launch_plans_are_cached_by_shape(fake_fusion):
    """The broadcast plan of a launch is built once per shape set (the plan caching the
    reference leaves as a TODO, PlanMeta.hpp:10-13) and results are unchanged."""
    F = fake_fusion
    rng = np.random.default_rng(40)
    X, B = rng.standard_normal((5, 7)).astype(np.float32), rng.standard_normal((7,)).astype(np.float32)
    x, b = api_cases.T(F, X), api_cases.T(F, B)
    first = (x * b + 1.0).maximum(0.0).to_numpy()
    h0, m0 = _stat(F, "plan_cache_hits"), _stat(F, "plan_cache_misses")
    for _ in range(3):
        np.testing.assert_array_equal((x * b + 1.0).maximum(0.0).to_numpy(), first)
    assert _stat(F, "plan_cache_misses") == m0
    assert _stat(F, "plan_cache_hits") >= h0 + 3
    y = api_cases.T(F, rng.standard_normal((3, 5, 7)))
    (y * b).to_numpy()  # a new shape set: one more plan
    assert _stat(F, "plan_cache_misses") == m0 + 1


def test_device_dropout_is_novas_composition(fake_fusion):
    """Random.dropout equals Nova's Dropout composition, x * (u >= rate) / (1 - rate), over
    the same seed's device stream (u from uniform_device), forward and backward, bit for
    bit; consecutive draws advance the stream."""
    F = fake_fusion
    rng = np.random.default_rng(50)
    X = rng.standard_normal((6, 10)).astype(np.float32)
    X[0, :3] = [0.0, -0.0, np.inf]
    rate = 0.3
    r1, r2 = F.Random(77), F.Random(77)
    x1, x2 = api_cases.T(F, X, True), api_cases.T(F, X, True)
    with F.grad_tape():
        y1 = r1.dropout(x1, rate)
        (y1 * 3.0).backward()
    with F.grad_tape():
        u = r2.uniform_device([6, 10], 0.0, 1.0, F.CppDevice(F.CppDeviceType.CPU, 0))
        y2 = x2 * (u >= rate) / (1 - rate)
        (y2 * 3.0).backward()
    with np.errstate(invalid="ignore"):
        assert_bits_equal(y1.to_numpy(), y2.to_numpy(), "forward")
        assert_bits_equal(x1.get_grad().to_numpy(), x2.get_grad().to_numpy(), "backward")
    assert r1.philox_offset == r2.philox_offset == 60
    d = F.CppDevice(F.CppDeviceType.CPU, 0)
    a, b = F.Random(5).uniform_device([7], -2.0, 3.0, d).to_numpy(), F.Random(5).uniform_device([7], -2.0, 3.0, d)
    np.testing.assert_array_equal(a, b.to_numpy())
    assert np.all((a >= -2.0) & (a < 3.0))
