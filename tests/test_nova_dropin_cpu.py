"""Nova's own Python, unchanged, over this backend's `fusion` module.

A copy of Nova's package (from the reference checkout) gets, in its
nova/src/backend/core/clib/ folder, first the reference's own pybind module (built
from the reference sources into oracle/_ref) and then this backend's module (the C++
host layer, here linked against the host-memory double of the C ABI, since this runs
without a GPU). tests/nova_dropin/run_nova_training.py then trains Nova's Linear /
ReLU / Model / MeanSquaredError / SGD-with-momentum through Nova's unchanged code in
each, and the losses and parameters must agree (1e-5 norm-wise: GEMM-bearing values).
The kernels behind the same host layer are held to the oracle by the GPU tests.
Skipped where the reference checkout is absent (GPU hosts).
"""
import os
import pathlib
import shutil
import subprocess
import sys

import numpy as np
import pytest

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent


def _nova_root():
    env = os.environ.get("FUSION_REFERENCE_ROOT")
    base = pathlib.Path(env) if env else ROOT.parent / "reference"
    return base / "nova"


def _run(tmp, name, modules):
    pkg = tmp / name
    shutil.copytree(_nova_root(), pkg / "nova", ignore=shutil.ignore_patterns("__pycache__", "*.so"))
    clib = pkg / "nova" / "src" / "backend" / "core" / "clib"
    for m in modules:
        shutil.copy(m, clib / m.name)
    out = tmp / f"{name}.npz"
    env = dict(os.environ, PYTHONPATH=str(pkg))
    r = subprocess.run([sys.executable, str(HERE / "nova_dropin" / "run_nova_training.py"), str(out)],
                       env=env, capture_output=True, text=True, cwd=pkg, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    return np.load(out)


@pytest.mark.skipif(not _nova_root().exists(), reason="reference checkout not present")
def test_nova_training_over_this_backend_matches_reference_module(tmp_path):
    ref_so = sorted((ROOT / "oracle" / "_ref").glob("fusion*.so"))
    if not ref_so:
        pytest.skip("reference module not built (make -C oracle ref)")
    sys.path.insert(0, str(HERE / "hostfake"))
    import build_fake

    ours = build_fake.build()
    want = _run(tmp_path, "reference", [ref_so[0]])
    got = _run(tmp_path, "ours", [ours, ours.parent / "libfusion_b200_hostfake.so"])
    assert set(got.files) == set(want.files)
    for k in sorted(want.files):
        g, w = got[k].astype(np.float64), want[k].astype(np.float64)
        assert g.shape == w.shape, k
        err = np.linalg.norm(g - w) / max(np.linalg.norm(w), 1e-30)
        assert err <= 1e-5, f"{k}: rel err {err:.3g}"
