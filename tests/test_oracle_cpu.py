"""Pins the oracle: the C restatement (oracle/fusion_oracle.c) against the reference's
own outputs (golden fixtures from the reference pybind module, and the reference
C++ path loaded through oracle/_ref/libfusion_ref.so), and the golden fixtures
against the known-answer vectors of the reference's unit tests."""
import pathlib

import numpy as np
import pytest

from conftest import assert_bits_equal

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
RNG = np.random.default_rng(99)


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN / "api_golden.npz")


# Expected values written in the reference's unit tests
# (tests/unit/tensor/test_ops.py, test_tensor.py, tests/unit/activations/test_activations.py).
KATS = {
    "case_kat_forward.add0": [5, 7, 9], "case_kat_forward.add1": [1, 2, 3],
    "case_kat_forward.add2": [1, 3, 4], "case_kat_forward.sub3": [-3, -3, -3],
    "case_kat_forward.sub4": [2, -2, 2], "case_kat_forward.rsub5": [3, 3, 3],
    "case_kat_forward.div6": [0.25, 0.4, 0.5], "case_kat_forward.div7": [-1.0, -2.0, 2.0],
    "case_kat_forward.div8": [0, 0, 0],
    "case_reductions_kat.sum0": [6.0], "case_reductions_kat.sum1": [10.0],
    "case_reductions_kat.mean0": [2.0], "case_reductions_kat.mean1": [2.5],
    "case_reductions_kat.sum_ax1_kd0": [3, 7], "case_reductions_kat.sum_ax0_kd0": [4, 6],
    "case_reductions_kat.sum_ax1_kd1": [[3], [7]], "case_reductions_kat.sum_ax0_kd1": [[4, 6]],
    "case_reductions_kat.mean_ax1_kd0": [1.5, 3.5], "case_reductions_kat.mean_ax0_kd1": [[2.0, 3.0]],
    "case_matmul_kat.mm2": [[19, 22], [43, 50]], "case_matmul_kat.mm_row": [[140]],
    "case_matmul_kat.mm3": [[[7, 15], [12, 28]], [[16, 9], [32, 20]]],
    "case_backward_kat.add_ga": [1, 1, 1], "case_backward_kat.sub_gb": [-1, -1, -1],
    "case_backward_kat.div_ga": [-1.0, 0.5], "case_backward_kat.div_gb": [-2.0, 1.0],
    "case_backward_kat.div2_gb": [-0.0625, -0.08, -0.0833333],
    "case_backward_kat.mm_gA": [[15, 19, 23], [15, 19, 23]],
    "case_backward_kat.mm_gB": [[5, 5], [7, 7], [9, 9]],
    "case_relu_special.relu_kat1": [1, 1], "case_relu_special.relu_kat2": [0, 1],
}


@pytest.mark.parametrize("key", sorted(KATS))
def test_golden_matches_reference_unit_tests(golden, key):
    np.testing.assert_array_almost_equal(golden[key], np.array(KATS[key], np.float32), decimal=5)


def test_port_matches_golden_quirks(golden, port):
    g = lambda k: golden["case_quirk_scalar_lhs." + k]
    a, b = np.array([10.0], np.float32), np.array([1.0, 2.0, 4.0], np.float32)
    col, row = np.array([[1.0], [2.0]], np.float32), np.array([[1.0, 2.0, 3.0]], np.float32)
    assert_bits_equal(port.binary("sub", a, b), g("s_minus_v"))
    assert_bits_equal(port.binary("sub", b, a), g("v_minus_s"))
    assert_bits_equal(port.binary("div", a, b), g("s_div_v"))
    assert_bits_equal(port.binary("pow", np.array([2.0], np.float32), b), g("s_pow_v"))
    assert_bits_equal(port.binary("sub", col, row), g("col_minus_row"))
    assert_bits_equal(port.binary("sub", row, col), g("row_minus_col"))
    v = np.array([-1.0, -0.0, np.nan, 2.0], np.float32)
    assert_bits_equal(port.binary("maximum", np.array([0.0], np.float32), v), g("s_max_v"))
    x = np.array([-1.0, 0.0, 2.0, -0.0, np.nan, np.inf, -np.inf, 1e-40], np.float32)
    assert_bits_equal(port.binary("maximum", x, np.array([0.0], np.float32)),
                      golden["case_relu_special.relu"])


def test_port_matches_golden_reductions(golden, port):
    x = np.random.default_rng(13).standard_normal((7, 33, 9)).astype(np.float32)
    for ax in (0, 1, 2):
        for kd in (0, 1):
            assert_bits_equal(port.reduce("sum", x, ax, bool(kd)),
                              golden[f"case_reduction_random.sum{ax}{kd}"])
            assert_bits_equal(port.reduce("mean", x, ax, bool(kd)),
                              golden[f"case_reduction_random.mean{ax}{kd}"])
    assert_bits_equal(port.reduce("sum", x), golden["case_reduction_random.sum_all"])


def test_port_matches_golden_swapaxes(golden, port):
    x = np.random.default_rng(17).standard_normal((3, 4, 5)).astype(np.float32)
    assert_bits_equal(port.swapaxes(x, 0, 1), golden["case_swapaxes.sw01"])
    assert_bits_equal(port.swapaxes(x, 1, 2), golden["case_swapaxes.sw12"])
    assert_bits_equal(port.swapaxes(x, 0, 2), golden["case_swapaxes.sw02"])


BCAST = [((5, 7), (5, 7)), ((5, 7), (7,)), ((5, 1), (5, 7)), ((1,), (4, 3)),
         ((3, 1, 4), (5, 1)), ((10,), (1,)), ((2, 1), (1, 3)), ((1, 1), (1, 1))]


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "pow", "maximum", "gt", "ge"])
def test_port_matches_reference_binary(port, ref, op):
    for sa, sb in BCAST:
        a = RNG.uniform(0.5, 2, sa).astype(np.float32)
        b = RNG.uniform(0.5, 2, sb).astype(np.float32)
        assert_bits_equal(port.binary(op, a, b), ref.binary(op, a, b), f"{op} {sa} {sb}")


@pytest.mark.parametrize("op,lo,hi", [("exp", -4, 4), ("log", 0.01, 10), ("sqrt", 0.01, 10)])
def test_port_matches_reference_unary(port, ref, op, lo, hi):
    a = RNG.uniform(lo, hi, 5000).astype(np.float32)
    assert_bits_equal(port.unary(op, a), ref.unary(op, a), op)


def test_port_matches_reference_reduce_and_layout(port, ref):
    x = RNG.standard_normal((6, 7, 8)).astype(np.float32)
    for op in ("sum", "mean"):
        for ax in (0, 1, 2):
            for kd in (False, True):
                assert_bits_equal(port.reduce(op, x, ax, kd), ref.reduce(op, x, ax, kd))
        assert_bits_equal(port.reduce(op, x), ref.reduce(op, x))
    for a1, a2 in ((0, 1), (1, 2), (0, 2), (-1, -2)):
        assert_bits_equal(port.swapaxes(x, a1, a2), ref.swapaxes(x, a1, a2))


def test_port_matmul_close_to_reference_blas(port, ref):
    a = RNG.standard_normal((3, 17, 33)).astype(np.float32)
    b = RNG.standard_normal((3, 33, 9)).astype(np.float32)
    r, p = ref.matmul(a, b), port.matmul(a, b)
    assert np.linalg.norm(r - p) / np.linalg.norm(r) < 1e-6


def test_reference_backward_formulas_match_golden(golden, ref):
    """ref_backward drives the registry formulas directly; the KAT grads agree."""
    x = np.array([2.0, -4.0], np.float32)
    y = np.array([-1.0, 2.0], np.float32)
    gx, gy = ref.backward("Divide", x, y, np.ones(2, np.float32))
    assert_bits_equal(gx, golden["case_backward_kat.div_ga"])
    assert_bits_equal(gy, golden["case_backward_kat.div_gb"])


def test_reference_mlp_step_matches_golden(golden, ref):
    import api_cases

    X, Y, Ws, bs = api_cases.mlp_inputs(21, [16, 32, 32, 4], 24)
    W2, b2, loss = ref.mlp_step(X, Y, Ws, bs, 1e-3)
    assert_bits_equal(loss, golden["case_mlp_step.loss"])
    for i in range(3):
        assert_bits_equal(W2[i], golden[f"case_mlp_step.W{i}"])
        assert_bits_equal(b2[i], golden[f"case_mlp_step.b{i}"])


def test_philox_restatement_matches_published_vectors(port):
    """The oracle's Philox-4x32-10 (Salmon et al., SC'11) reproduces the published
    known-answer vectors of the algorithm (counter, key -> output)."""
    kat = [((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
           ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
           ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
            (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1))]
    for c, k, want in kat:
        got = port.philox_block(c[0] | c[1] << 32, c[2] | c[3] << 32, k[0] | k[1] << 32)
        assert tuple(got) == want
    u = port.philox_uniform(1 << 16, 9, 0, 0.0, 1.0)
    assert 0.0 <= u.min() and u.max() < 1.0 and abs(u.mean() - 0.5) < 0.01
