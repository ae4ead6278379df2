"""Fusion's Python API on the B200 backend against the reference module's outputs.

Every case of tests/api_cases.py is replayed through nova_b200.fusion and compared
with tests/golden/api_golden.npz, which the reference pybind module (built from
the reference sources) produced for the same inputs.
"""
import pathlib

import numpy as np
import pytest

import api_cases
from conftest import assert_bits_equal, ulp_diff

pytestmark = pytest.mark.gpu
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def _kinds():
    kinds = {}
    for line in (GOLDEN / "api_golden_kinds.txt").read_text().splitlines():
        k, v = line.split()
        kinds[k] = v
    return kinds


@pytest.fixture(scope="module")
def results(capi):
    import nova_b200

    return api_cases.run_all(nova_b200.fusion)


def _compare(key, kind, got, want):
    assert got.shape == want.shape, f"{key}: shape {got.shape} vs {want.shape}"
    if kind == "exact":
        assert_bits_equal(got, want, key)
    elif kind == "ulp2":
        assert ulp_diff(got, want).max() <= 2, key
    elif kind == "ulp_pow":
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-7, err_msg=key)
    elif kind == "sum":
        assert np.all(np.abs(got - want) <= 1e-5 * (np.abs(want) + 1.0)), key
    else:  # "rel": norm-wise relative error of GEMM-bearing results
        err = np.linalg.norm((got - want).ravel().astype(np.float64))
        ref = max(np.linalg.norm(want.ravel().astype(np.float64)), 1e-30)
        assert err / ref <= 1e-5, f"{key}: rel err {err / ref:.3g}"


def test_api_matches_reference(results):
    golden = np.load(GOLDEN / "api_golden.npz")
    kinds = _kinds()
    assert set(golden.files) == set(results), "case sets differ"
    failures = []
    for key in sorted(golden.files):
        want = golden[key]
        if want.size == 0:
            # the reference raises here (e.g. `-x` returns an unbound RawTensor);
            # this backend returns a value instead
            continue
        try:
            _compare(key, kinds[key], results[key], want)
        except AssertionError as e:
            failures.append(str(e))
    assert not failures, "\n".join(failures)


def test_fusion_on_and_off_agree(capi):
    """Lazy fusion only changes how many kernels run, never a bit of the result."""
    import nova_b200

    F = nova_b200.fusion
    F.set_fusion(False)
    try:
        eager = api_cases.run_all(F)
    finally:
        F.set_fusion(True)
    fused = api_cases.run_all(F)
    for k in eager:
        assert_bits_equal(fused[k], eager[k], k)


def test_fused_chain_is_one_kernel(capi):
    """relu(x @ W.T + b) lowers the bias add and ReLU into the GEMM's epilogue (no
    separate launch); with epilogue fusion off, into one fused launch after the GEMM.
    Both give the same bits."""
    import nova_b200

    F = nova_b200.fusion
    x = api_cases.T(F, np.random.default_rng(0).standard_normal((64, 32)))
    w = api_cases.T(F, np.random.default_rng(1).standard_normal((16, 32)))
    b = api_cases.T(F, np.random.default_rng(2).standard_normal((16,)))
    y = (x @ w.swapaxes(1, 0) + b).maximum(0.0)
    assert y.is_pending()
    s0 = F.stats()
    got_epi = y.to_numpy()
    s1 = F.stats()
    assert s1["fused_launches"] == s0["fused_launches"]
    assert s1["epilogue_gemms"] == s0["epilogue_gemms"] + 1
    F.set_gemm_epilogue(False)
    try:
        y = (x @ w.swapaxes(1, 0) + b).maximum(0.0)
        got_plain = y.to_numpy()
        s2 = F.stats()
        assert s2["fused_launches"] == s1["fused_launches"] + 1
        assert s2["epilogue_gemms"] == s1["epilogue_gemms"]
    finally:
        F.set_gemm_epilogue(True)
    assert_bits_equal(got_epi, got_plain, "relu(x W^T + b)")
