"""Shared fixtures. GPU tests are marked `gpu`; everything else runs on CPU."""
import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def port():
    import oracle

    if not oracle.have_port():
        pytest.skip("oracle port not built (make -C oracle port)")
    return oracle.Port()


@pytest.fixture(scope="session")
def ref():
    import oracle

    if not oracle.have_ref():
        pytest.skip("reference oracle not built (make -C oracle ref)")
    return oracle.Ref()


@pytest.fixture(scope="session")
def capi():
    from nova_b200 import capi as A

    if A.device_count() < 1:
        pytest.fail("no sm_100 GPU visible: " + A.lib().fz_last_error().decode())
    A.check(A.lib().fz_set_device(0))
    return A


def ulp_diff(a, b):
    """Distance in units in the last place between fp32 arrays (NaN==NaN -> 0)."""
    a = np.asarray(a, np.float32).ravel()
    b = np.asarray(b, np.float32).ravel()
    ia = a.view(np.int32).astype(np.int64)
    ib = b.view(np.int32).astype(np.int64)
    ia = np.where(ia < 0, np.int64(-2**31) - ia, ia)
    ib = np.where(ib < 0, np.int64(-2**31) - ib, ib)
    d = np.abs(ia - ib)
    both_nan = np.isnan(a) & np.isnan(b)
    d = np.where(both_nan, 0, d)
    return d if d.size else np.zeros(1, np.int64)


def assert_bits_equal(got, want, what=""):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    g, w = got.view(np.uint32), want.view(np.uint32)
    same = (g == w) | (np.isnan(got) & np.isnan(want))
    if not same.all():
        i = int(np.argmin(same.ravel()))
        raise AssertionError(f"{what}: {int((~same).sum())} elements differ; first at {i}: "
                             f"{got.ravel()[i]!r} vs {want.ravel()[i]!r}")
