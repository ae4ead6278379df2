"""B200 (sm_100a) compute backend for Fusion, the tensor library under Nova.

``nova_b200.fusion`` is a drop-in for the pybind module ``fusion`` that Nova
imports (nova/src/backend/core/clib/__init__.py): Tensor, factory, Random,
CppDevice, CppDeviceType, CppDType, grad_tape and autodiff, with the same names,
arguments and error behaviour, running on hand-written sm_100a kernels behind the
C ABI of ``include/fusion_b200.h`` (``libfusion_b200.so``).

There is no CPU path: using ``nova_b200.fusion`` fails loudly when the native
libraries have not been built (``python -m nova_b200.build``). The module is
imported on first use so the build script itself can run from an unbuilt tree.
"""
from __future__ import annotations

import importlib

__all__ = ["fusion"]


def __getattr__(name):
    if name == "fusion":
        try:
            mod = importlib.import_module(".fusion", __name__)
        except ImportError as e:
            raise ImportError(
                "nova_b200: the native module `fusion` is not built or cannot load "
                f"({e}); run `python -m nova_b200.build` on a machine with nvcc"
            ) from e
        globals()["fusion"] = mod
        return mod
    raise AttributeError(f"module 'nova_b200' has no attribute {name!r}")
