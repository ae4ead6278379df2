"""B200 (sm_100a) compute backend for Fusion, the tensor library under Nova.

``nova_b200.fusion`` is a drop-in for the pybind module ``fusion`` that Nova
imports (nova/src/backend/core/clib/__init__.py): Tensor, factory, Random,
CppDevice, CppDeviceType, CppDType, grad_tape and autodiff, with the same names,
arguments and error behaviour, running on hand-written sm_100a kernels behind the
C ABI of ``include/fusion_b200.h`` (``libfusion_b200.so``).

There is no CPU path: importing fails loudly when the native libraries have not
been built (``python -m nova_b200.build``).
"""
from __future__ import annotations

import importlib
import pathlib

_PKG = pathlib.Path(__file__).resolve().parent

try:
    fusion = importlib.import_module(".fusion", __name__)
except ImportError as e:  # pragma: no cover - exercised only on unbuilt trees
    raise ImportError(
        "nova_b200: the native module `fusion` is not built or cannot load "
        f"({e}); run `python -m nova_b200.build` on a machine with nvcc"
    ) from e

__all__ = ["fusion"]
