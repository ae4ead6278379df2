"""Generate tests/golden/api_golden.npz from the reference's own pybind module.

Run here (where the reference sources are) after `make -C oracle ref`:
    python tests/golden/make_golden.py
It imports the reference module `fusion` built from fusion/src/Fusion/python/Bindings.cpp
into oracle/_ref/ and runs every case of tests/api_cases.py through it. The GPU tests
replay the same cases through nova_b200.fusion and compare with this file.
"""
import importlib.util
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "tests"))

import api_cases  # noqa: E402


def load_reference_module():
    so = next((ROOT / "oracle" / "_ref").glob("fusion*.so"))
    spec = importlib.util.spec_from_file_location("oracle_ref.fusion", so)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    F = load_reference_module()
    res = api_cases.run_all(F)
    kinds = {k: api_cases.kind_of(k) for k in res}
    np.savez_compressed(HERE / "api_golden.npz", **res)
    (HERE / "api_golden_kinds.txt").write_text("".join(f"{k} {v}\n" for k, v in sorted(kinds.items())))
    print(f"wrote {len(res)} arrays")


if __name__ == "__main__":
    main()
