"""CPU-side checks of the drop-in boundary: the C ABI library and the pybind module
load, export what include/fusion_b200.h and the reference module declare, and fail
loudly (no CPU fallback) when no B200 is present."""
import importlib.util
import pathlib

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]


def test_c_abi_exports_every_declared_symbol():
    from nova_b200 import capi

    lib = capi.lib()
    declared = capi.header_symbols()
    assert len(declared) >= 35
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing


def test_library_is_sm100a_only():
    """The product library carries sm_100a code and no CPU implementation of the ops."""
    so = (ROOT / "nova_b200" / "libfusion_b200.so").read_bytes()
    assert b"sm_100a" in so or b"compute_100a" in so


REFERENCE_API = {
    "module": ["Tensor", "factory", "Random", "CppDevice", "CppDeviceType", "CppDType",
               "grad_tape", "autodiff"],
    "Tensor": ["set_values", "shape", "ndim", "dtype", "size", "name", "requires_grad",
               "to_numpy", "__repr__", "__add__", "__sub__", "__mul__", "__truediv__",
               "__pow__", "__ge__", "__gt__", "__neg__", "__isub__", "sqrt", "exp", "log",
               "sum", "mean", "__matmul__", "maximum", "swapaxes", "backward", "get_grad",
               "rank"],
    "factory": ["fill", "zeros", "ones", "zeros_like", "ones_like"],
}


def test_pybind_module_has_reference_api():
    import nova_b200

    F = nova_b200.fusion
    for name in REFERENCE_API["module"]:
        assert hasattr(F, name), name
    for name in REFERENCE_API["Tensor"]:
        assert hasattr(F.Tensor, name), name
    for name in REFERENCE_API["factory"]:
        assert hasattr(F.factory, name), name
    assert hasattr(F.autodiff, "enabled")
    assert F.CppDeviceType.CUDA.value == 1 and F.CppDType.BOOL.value == 4


def test_reference_module_api_matches_ours():
    """Every public name of the reference module exists in ours."""
    so = list((ROOT / "oracle" / "_ref").glob("fusion*.so"))
    if not so:
        pytest.skip("reference module not built")
    spec = importlib.util.spec_from_file_location("oracle_ref.fusion", so[0])
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    import nova_b200

    ours = nova_b200.fusion
    for name in dir(ref):
        if name.startswith("_"):
            continue
        assert hasattr(ours, name), name
    for name in dir(ref.Tensor):
        if name.startswith("__") and name not in REFERENCE_API["Tensor"]:
            continue
        assert hasattr(ours.Tensor, name), name


def test_no_gpu_fails_loudly():
    import nova_b200

    F = nova_b200.fusion
    if F.device_count() > 0:
        pytest.skip("a GPU is present")
    dev = F.CppDevice(F.CppDeviceType.CPU, 0)
    with pytest.raises(RuntimeError):
        F.Tensor([3], [1.0, 2.0, 3.0], F.CppDType.FLOAT32, dev, False)


def test_device_validation_on_host():
    import nova_b200

    F = nova_b200.fusion
    with pytest.raises(RuntimeError):
        F.CppDevice(F.CppDeviceType.CPU, 1)  # reference: CPU index must be <= 0
    F.CppDevice(F.CppDeviceType.CUDA, 3)  # CUDA ordinals are checked when used


def _epi_program(capi, nodes, nleaves, outs):
    p = capi.Program()
    p.num_nodes, p.num_leaves, p.num_outputs = len(nodes), nleaves, len(outs)
    for i, o in enumerate(outs):
        p.out_node[i] = o
    for i, (kind, op, s0, s1, imm) in enumerate(nodes):
        n = p.nodes[i]
        n.kind, n.op, n.src0, n.src1, n.imm = kind, op, s0, s1, imm
    return p


# (a_mn, b_mn, tile_n, pair): every variant the GEMM dispatch can pick
GEMM_VARIANTS = [(a, b, 256, p) for p in (1, 0) for a in (0, 1) for b in (0, 1)] + \
                [(a, 0, t, 0) for t in (16, 64) for a in (0, 1)]


def test_gemm_epilogues_compile_for_every_kernel_variant():
    """NVRTC (no device needed) compiles each GEMM variant with a generated epilogue:
    relu(P + bias) with its TF32 remainder plane and P, and the ReLU-mask gradient."""
    import ctypes as C

    from nova_b200 import capi

    L = capi.lib()
    B, U, K = capi.NODE_BINARY, capi.NODE_UNARY, capi.NODE_CONST
    fwd = _epi_program(capi, [(B, capi.BINOPS["add"], -1, -2, 0.0), (K, 0, 0, 0, 0.0),
                              (B, capi.BINOPS["maximum"], 0, 1, 0.0), (U, capi.UNOPS["tf32_lo"], 2, 0, 0.0),
                              (U, capi.UNOPS["copy"], -1, 0, 0.0)], 2, [2, 3, 4])
    bwd = _epi_program(capi, [(B, capi.BINOPS["add"], -2, -3, 0.0), (K, 0, 0, 0, 0.0),
                              (B, capi.BINOPS["gt"], 0, 1, 0.0), (B, capi.BINOPS["mul"], -1, 2, 0.0),
                              (U, capi.UNOPS["tf32_lo"], 3, 0, 0.0)], 3, [3, 4])
    row = (capi.EpiInput * 1)(capi.EpiInput(None, 0, 0, 1))
    full_row = (capi.EpiInput * 2)(capi.EpiInput(None, 4096, 64, 1), capi.EpiInput(None, 0, 0, 1))
    for v in GEMM_VARIANTS:
        rc = L.fz_gemm_epilogue_compile(C.byref(fwd), row, *v)
        assert rc == 0, (v, L.fz_last_error())
    for v in [(0, 0, 256, 1), (0, 1, 256, 1), (0, 0, 16, 0)]:
        rc = L.fz_gemm_epilogue_compile(C.byref(bwd), full_row, *v)
        assert rc == 0, (v, L.fz_last_error())
    # more full-shape inputs and outputs: 4-column side-by-side blocks, and the
    # per-output passes when they do not fit the staging tile side by side
    many = _epi_program(capi, [(B, capi.BINOPS["add"], -1, -2, 0.0), (B, capi.BINOPS["add"], 0, -3, 0.0),
                               (B, capi.BINOPS["add"], 1, -4, 0.0), (B, capi.BINOPS["mul"], 2, -5, 0.0),
                               (B, capi.BINOPS["sub"], 3, -6, 0.0)], 6, [1, 2, 3, 4])
    five = (capi.EpiInput * 5)(*[capi.EpiInput(None, 4096, 64, 1)] * 5)
    for v in [(0, 0, 256, 1), (0, 0, 16, 0), (1, 0, 64, 0)]:
        assert L.fz_gemm_epilogue_compile(C.byref(many), five, *v) == 0, (v, L.fz_last_error())
    two = (capi.EpiInput * 5)(*([capi.EpiInput(None, 4096, 64, 1)] * 2 + [capi.EpiInput(None, 0, 0, 1)] * 3))
    for v in [(0, 0, 256, 1), (0, 0, 16, 0)]:
        assert L.fz_gemm_epilogue_compile(C.byref(many), two, *v) == 0, (v, L.fz_last_error())
    # narrow tiles take a K-major B only
    assert L.fz_gemm_epilogue_compile(C.byref(fwd), row, 0, 1, 16, 0) == 1
