"""API-level parity cases, written against the `fusion` module interface.

Each case takes a module exposing Fusion's Python API (the reference pybind module
or nova_b200.fusion) and returns named float32 arrays. tests/golden/make_golden.py
runs them through the reference module built from the reference sources and stores
the results in tests/golden/api_golden.npz; tests/test_api_gpu.py runs the same
cases through nova_b200.fusion and compares. Inputs are the reference unit tests'
known-answer vectors (tests/unit/tensor/test_ops.py, test_tensor.py,
tests/unit/activations/test_activations.py) plus seeded random data.
"""
from __future__ import annotations

import numpy as np

# comparison class of each output: "exact" (bitwise), "ulp2", or "rel" (1e-5 norm-wise)
KIND: dict[str, str] = {}


def _dev(F):
    return F.CppDevice(F.CppDeviceType.CPU, 0)


def T(F, data, requires_grad=False):
    a = np.asarray(data, dtype=np.float32)
    shape = list(a.shape) or [1]
    return F.Tensor(shape, a.ravel().tolist(), F.CppDType.FLOAT32, _dev(F), requires_grad)


def _rng(seed):
    return np.random.default_rng(seed)


def case_kat_forward(F):
    out = {}
    kats = [("add", [1, 2, 3], [4, 5, 6]), ("add", [1, 2, 3], [0]), ("add", [0, 2, 3], [1]),
            ("sub", [1, 2, 3], [4, 5, 6]), ("sub", [1, -1, 1], [-1, 1, -1]),
            ("rsub", [1, 2, 3], [4, 5, 6]), ("div", [1, 2, 3], [4, 5, 6]),
            ("div", [2, -4, 10], [-2, 2, 5]), ("div", [0, 0, 0], [1, 1, 1])]
    for i, (op, a, b) in enumerate(kats):
        x, y = T(F, a), T(F, b)
        r = {"add": lambda: x + y, "sub": lambda: x - y, "rsub": lambda: y - x,
             "div": lambda: x / y}[op]()
        out[f"{op}{i}"] = r.to_numpy()
    return out


def case_quirk_scalar_lhs(F):
    """[1]-shaped left operand exchanges operands in the broadcast walk."""
    a = T(F, [10.0])
    b = T(F, [1.0, 2.0, 4.0])
    col = T(F, [[1.0], [2.0]])
    row = T(F, [[1.0, 2.0, 3.0]])
    return {"s_minus_v": (a - b).to_numpy(), "v_minus_s": (b - a).to_numpy(),
            "s_div_v": (a / b).to_numpy(), "v_div_s": (b / a).to_numpy(),
            "s_pow_v": (T(F, [2.0]) ** b).to_numpy(), "v_pow_s": (b ** T(F, [2.0])).to_numpy(),
            "col_minus_row": (col - row).to_numpy(), "row_minus_col": (row - col).to_numpy(),
            "s_max_v": T(F, [0.0]).maximum(T(F, [-1.0, -0.0, np.nan, 2.0])).to_numpy(),
            "s_gt_v": (T(F, [0.5]) > T(F, [0.0, 1.0, 0.5])).to_numpy(),
            "v_ge_s": (T(F, [0.0, 1.0, 0.5]) >= 0.5).to_numpy()}


def case_relu_special(F):
    x = T(F, [-1.0, 0.0, 2.0, -0.0, np.nan, np.inf, -np.inf, 1e-40])
    return {"relu": x.maximum(0.0).to_numpy(), "relu_kat1": T(F, [1.0, 1.0]).maximum(0).to_numpy(),
            "relu_kat2": T(F, [-1.0, 1.0]).maximum(0).to_numpy()}


def case_reductions_kat(F):
    out = {}
    for i, d in enumerate([[1, 2, 3], [[1, 2], [3, 4]], [0, 0, 0]]):
        out[f"sum{i}"] = T(F, d).sum().to_numpy()
        out[f"mean{i}"] = T(F, d).mean().to_numpy()
    m = T(F, [[1, 2], [3, 4]])
    for ax in (0, 1):
        for kd in (False, True):
            out[f"sum_ax{ax}_kd{int(kd)}"] = m.sum(axis=ax, keepdim=kd).to_numpy()
            out[f"mean_ax{ax}_kd{int(kd)}"] = m.mean(axis=ax, keepdim=kd).to_numpy()
    return out


def case_matmul_kat(F):
    a = T(F, [[1.0, 2.0], [3.0, 4.0]])
    b = T(F, [[5.0, 6.0], [7.0, 8.0]])
    c = T(F, [[1.0, 2.0, 3.0]])
    d = T(F, [[10.0], [20.0], [30.0]])
    e = T(F, [[[3, 1], [4, 4]], [[3, 1], [4, 4]]])
    f = T(F, [[[2, 4], [1, 3]], [[4, 2], [4, 3]]])
    return {"mm2": (a @ b).to_numpy(), "mm_row": (c @ d).to_numpy(), "mm3": (e @ f).to_numpy()}


def case_backward_kat(F):
    out = {}
    with F.grad_tape():
        a, b = T(F, [1, 2, 3], True), T(F, [4, 5, 6], True)
        c = a + b
        c.backward()
        out["add_ga"], out["add_gb"] = a.get_grad().to_numpy(), b.get_grad().to_numpy()
    with F.grad_tape():
        a, b = T(F, [1, -1, 1], True), T(F, [-1, 1, -1], True)
        (a - b).backward()
        out["sub_ga"], out["sub_gb"] = a.get_grad().to_numpy(), b.get_grad().to_numpy()
    with F.grad_tape():
        a, b = T(F, [2.0, -4.0], True), T(F, [-1.0, 2.0], True)
        (a / b).backward()
        out["div_ga"], out["div_gb"] = a.get_grad().to_numpy(), b.get_grad().to_numpy()
    with F.grad_tape():
        a, b = T(F, [1.0, 2.0, 3.0], True), T(F, [4.0, 5.0, 6.0], True)
        (a / b).backward()
        out["div2_ga"], out["div2_gb"] = a.get_grad().to_numpy(), b.get_grad().to_numpy()
    with F.grad_tape():
        a = T(F, [[-1.0, -2.0], [3.0, 0.5]], True)
        a.sum().backward()
        out["sum_ga"] = a.get_grad().to_numpy()
    with F.grad_tape():
        A = T(F, [[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]], True)
        B = T(F, [[7.0, 8.0], [9.0, 10.0], [11.0, 12.0]], True)
        (A @ B).sum().backward()
        out["mm_gA"], out["mm_gB"] = A.get_grad().to_numpy(), B.get_grad().to_numpy()
    with F.grad_tape():
        x = T(F, [-1.0, 0.0, 2.0], True)
        x.maximum(0.0).sum().backward()
        out["relu_gx"] = x.get_grad().to_numpy()
    return out


def case_unary_random(F):
    r = _rng(7)
    out = {}
    xe = r.uniform(-4, 4, (37, 5)).astype(np.float32)
    xl = r.uniform(0.01, 10, (37, 5)).astype(np.float32)
    g = r.uniform(-1, 1, (37, 5)).astype(np.float32)
    for name, xv in (("exp", xe), ("log", xl), ("sqrt", xl)):
        with F.grad_tape():
            x = T(F, xv, True)
            y = getattr(x, name)()
            (y * T(F, g)).sum().backward()
            out[name] = y.to_numpy()
            out[name + "_grad"] = x.get_grad().to_numpy()
            KIND[name] = KIND[name + "_grad"] = "exact" if name == "sqrt" else "ulp2"
    return out


def case_binary_random_grads(F):
    """Forward and both grads of each binary op with broadcasting and upstream g."""
    r = _rng(11)
    out = {}
    # traced mul/div/pow/maximum admit a scalar or equal element counts
    # (FUSION_ALLOW_SCALAR_BINARY); add/sub broadcast freely
    shapes = [((6, 5), (6, 5)), ((6, 5), (1,)), ((1,), (6, 5)), ((6, 1), (1, 6)), ((6, 5), (5,))]
    for si, (sa, sb) in enumerate(shapes):
        osh = np.broadcast_shapes(sa, sb)
        ops = ("add", "sub") if si == 4 else ("add", "sub", "mul", "div", "maximum", "pow")
        for op in ops:
            av = r.uniform(0.5, 2, sa).astype(np.float32)
            bv = r.uniform(0.5, 2, sb).astype(np.float32)
            if op == "maximum":
                bv = r.uniform(0.5, 2, sb).astype(np.float32)
            gv = r.uniform(-1, 1, osh).astype(np.float32)
            with F.grad_tape():
                a, b = T(F, av, True), T(F, bv, True)
                y = {"add": lambda: a + b, "sub": lambda: a - b, "mul": lambda: a * b,
                     "div": lambda: a / b, "maximum": lambda: a.maximum(b),
                     "pow": lambda: a ** b}[op]()
                (y * T(F, gv)).sum().backward()
                k = f"{op}_{si}"
                out[k] = y.to_numpy()
                out[k + "_ga"] = a.get_grad().to_numpy()
                out[k + "_gb"] = b.get_grad().to_numpy()
                if op == "pow":
                    KIND[k] = KIND[k + "_ga"] = KIND[k + "_gb"] = "ulp_pow"
    return out


def case_maximum_of_computed_value(F):
    """Maximum whose first operand is computed in the trace: with a second operand that
    needs no gradient (a scalar, a tensor) its backward may read the output for the mask,
    which must give the reference's gradient, NaN, signed zeros and ties included; with a
    second operand that requires grad both gradients come from the operands."""
    out = {}
    xv = np.array([-1.0, -0.0, 0.0, np.nan, 2.0, 1e-30, -1e-30, 0.5, 3.0, -2.0], np.float32)
    gv = np.array([0.5, -0.25, 1.0, 2.0, -1.5, 3.0, 0.75, -1.0, 0.125, 4.0], np.float32)
    yv = np.array([0.5, 0.0, -0.0, 1.0, 2.0, 0.0, 0.0, 0.5, np.nan, -3.0], np.float32)
    with F.grad_tape():
        x = T(F, xv, True)
        (((x * 1.0).maximum(0.0)) * T(F, gv)).sum().backward()
        out["scalar_gx"] = x.get_grad().to_numpy()
    with F.grad_tape():
        x = T(F, xv, True)
        h = (x * 1.0).maximum(T(F, yv))
        (h * T(F, gv)).sum().backward()
        out["tensor"], out["tensor_gx"] = h.to_numpy(), x.get_grad().to_numpy()
    with F.grad_tape():
        x, y = T(F, xv, True), T(F, yv, True)
        ((x * 1.0).maximum(y) * T(F, gv)).sum().backward()
        out["both_gx"], out["both_gy"] = x.get_grad().to_numpy(), y.get_grad().to_numpy()
    return out


def case_reduction_random(F):
    r = _rng(13)
    x = r.standard_normal((7, 33, 9)).astype(np.float32)
    out = {}
    t = T(F, x)
    for ax in (0, 1, 2):
        for kd in (False, True):
            out[f"sum{ax}{int(kd)}"] = t.sum(axis=ax, keepdim=kd).to_numpy()
            out[f"mean{ax}{int(kd)}"] = t.mean(axis=ax, keepdim=kd).to_numpy()
            KIND[f"sum{ax}{int(kd)}"] = KIND[f"mean{ax}{int(kd)}"] = "sum"
    out["sum_all"] = t.sum().to_numpy()
    out["mean_all"] = t.mean().to_numpy()
    KIND["sum_all"] = KIND["mean_all"] = "sum"
    return out


def case_traced_mean_returns_input(F):
    with F.grad_tape():
        x = T(F, [[1.0, 2.0], [3.0, 4.0]], True)
        m = x.mean()
        m.backward()
        return {"traced_mean": m.to_numpy(), "traced_mean_grad": x.get_grad().to_numpy()}


def case_swapaxes(F):
    r = _rng(17)
    x = T(F, r.standard_normal((3, 4, 5)).astype(np.float32))
    with F.grad_tape():
        w = T(F, r.standard_normal((4, 6)).astype(np.float32), True)
        y = w.swapaxes(1, 0)
        (y * T(F, r.uniform(-1, 1, (6, 4)).astype(np.float32))).sum().backward()
        gw = w.get_grad().to_numpy()
    return {"sw01": x.swapaxes(0, 1).to_numpy(), "sw12": x.swapaxes(1, 2).to_numpy(),
            "sw02": x.swapaxes(0, 2).to_numpy(), "swneg": x.swapaxes(-1, -2).to_numpy(),
            "sw_grad": gw}


def _mlp(F, X, Y, Ws, bs, lr, x_requires_grad=True):
    """Nova's Linear/ReLU/MSE/SGD sequence (linear.py:42-48, activations.py:9-10,
    loss_fn.py:14-15, loss.py:34-37, sgd.py:29-44)."""
    params = [(T(F, w, True), T(F, b, True)) for w, b in zip(Ws, bs)]
    with F.grad_tape():
        out = T(F, X, x_requires_grad)
        for i, (W, b) in enumerate(params):
            out = out @ W.swapaxes(W.ndim - 1, W.ndim - 2)
            out = out + b
            if i + 1 < len(params):
                out = out.maximum(0)
        loss = (out - T(F, Y, True)) ** 2
        loss = loss / loss.size
        loss.backward()
    res = {"loss": loss.to_numpy()}
    for i, (W, b) in enumerate(params):
        res[f"gW{i}"] = W.get_grad().to_numpy()
        res[f"gb{i}"] = b.get_grad().to_numpy()
        W -= W.get_grad() * lr
        b -= b.get_grad() * lr
        res[f"W{i}"] = W.to_numpy()
        res[f"b{i}"] = b.to_numpy()
    return res


def mlp_inputs(seed, dims, batch):
    r = _rng(seed)
    X = r.standard_normal((batch, dims[0])).astype(np.float32)
    Y = r.standard_normal((batch, dims[-1])).astype(np.float32)
    Ws = [r.uniform(-np.sqrt(6 / dims[i]), np.sqrt(6 / dims[i]), (dims[i + 1], dims[i])).astype(np.float32)
          for i in range(len(dims) - 1)]
    bs = [r.uniform(-0.1, 0.1, (dims[i + 1],)).astype(np.float32) for i in range(len(dims) - 1)]
    return X, Y, Ws, bs


def case_mlp_step(F):
    X, Y, Ws, bs = mlp_inputs(21, [16, 32, 32, 4], 24)
    res = _mlp(F, X, Y, Ws, bs, 1e-3)
    for k in res:
        KIND[k] = "rel"
    return res


def case_sub_inplace_bias_row0(F):
    b = T(F, [1.0, 2.0, 3.0], True)
    g = T(F, [[0.5, 0.5, 0.5], [9.0, 9.0, 9.0]])
    b -= g
    w = T(F, [[1.0, 2.0], [3.0, 4.0]])
    w -= T(F, [[0.25, 0.5], [1.0, 2.0]])
    return {"bias_row0": b.to_numpy(), "w_inplace": w.to_numpy()}


def case_errors(F):
    """Error behaviour: both back-ends raise for the same misuse."""
    out = {}
    checks = {
        "traced_mul_size_mismatch": lambda: _traced_mul(F),
        "broadcast_mismatch": lambda: T(F, [[1.0, 2.0, 3.0]]) + T(F, [[1.0, 2.0]]),
        "matmul_inner_mismatch": lambda: T(F, [[1.0, 2.0]]) @ T(F, [[1.0, 2.0]]),
        "matmul_rank1": lambda: T(F, [1.0, 2.0]) @ T(F, [[1.0], [2.0]]),
        "set_values_len": lambda: T(F, [1.0, 2.0]).set_values([1.0]),
        "reduce_axis_range": lambda: T(F, [[1.0, 2.0]]).sum(axis=5),
        "backward_no_tape": lambda: T(F, [1.0], True).backward(),
    }
    for k, fn in checks.items():
        try:
            fn()
            out[k] = np.array([0.0], np.float32)
        except (RuntimeError, ValueError, IndexError, TypeError):
            out[k] = np.array([1.0], np.float32)
    return out


def _traced_mul(F):
    with F.grad_tape():
        return T(F, np.ones((6, 5)), True) * T(F, np.ones((5,)), True)


def case_factory_random(F):
    d = _dev(F)
    x = T(F, [[1.0, 2.0], [3.0, 4.0]])
    return {"uniform": F.Random(42).uniform_cpp([3, 4], -1.0, 1.0, d).to_numpy(),
            "zeros_like": F.factory.zeros_like(x).to_numpy(),
            "ones_like": F.factory.ones_like(x).to_numpy(),
            "neg": (-x).to_numpy() if _neg_ok(F, x) else np.zeros((0,), np.float32)}


def _neg_ok(F, x):
    try:
        -x
        return True
    except TypeError:
        return False


CASES = [case_kat_forward, case_quirk_scalar_lhs, case_relu_special, case_reductions_kat,
         case_matmul_kat, case_backward_kat, case_unary_random, case_binary_random_grads,
         case_maximum_of_computed_value, case_reduction_random, case_traced_mean_returns_input,
         case_swapaxes, case_mlp_step,
         case_sub_inplace_bias_row0, case_errors, case_factory_random]


def run_all(F) -> dict[str, np.ndarray]:
    out = {}
    for c in CASES:
        for k, v in c(F).items():
            out[f"{c.__name__}.{k}"] = np.asarray(v, dtype=np.float32)
    return out


def kind_of(key: str) -> str:
    name = key.split(".", 1)[1]
    if key.startswith("case_mlp_step."):
        return "rel"
    if key.startswith("case_matmul_kat.") or key.startswith("case_backward_kat.mm"):
        return "rel"
    if key.startswith("case_swapaxes.sw_grad"):
        return "exact"
    return KIND.get(name, "exact")
