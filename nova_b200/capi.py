"""ctypes binding of the C ABI in include/fusion_b200.h (libfusion_b200.so).

This is the binding a Python caller adds to reach the backend without the pybind
module: plain pointers, sizes and POD plans, int status codes turned into
exceptions. The parity tests call the kernels through it.
"""
from __future__ import annotations

import ctypes as C
import pathlib
import re

import numpy as np

_PKG = pathlib.Path(__file__).resolve().parent
LIB_PATH = _PKG / "libfusion_b200.so"
HEADER = _PKG.parent / "include" / "fusion_b200.h"

FZ_MAX_DIMS = 8
FZ_MAX_LEAVES = 12
FZ_MAX_NODES = 48
FZ_MAX_OUTPUTS = 4

BINOPS = {"add": 0, "sub": 1, "mul": 2, "div": 3, "pow": 4, "maximum": 5, "gt": 6, "ge": 7}
UNOPS = {"exp": 0, "log": 1, "sqrt": 2, "copy": 3, "tf32_lo": 4}
REDOPS = {"sum": 0, "mean": 1, "max": 2}
NODE_BINARY, NODE_UNARY, NODE_CONST = 0, 1, 2


class FzError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"fusion_b200 error {code}: {msg}")
        self.code = code


class EwisePlan(C.Structure):
    _fields_ = [
        ("ndim", C.c_int32),
        ("num_operands", C.c_int32),
        ("size", C.c_int64 * FZ_MAX_DIMS),
        ("stride_bytes", (C.c_int64 * FZ_MAX_DIMS) * (FZ_MAX_LEAVES + FZ_MAX_OUTPUTS)),
    ]


class Node(C.Structure):
    _fields_ = [("kind", C.c_int32), ("op", C.c_int32), ("src0", C.c_int32),
                ("src1", C.c_int32), ("imm", C.c_float)]


class Program(C.Structure):
    _fields_ = [("num_nodes", C.c_int32), ("num_leaves", C.c_int32),
                ("num_outputs", C.c_int32), ("out_node", C.c_int32 * FZ_MAX_OUTPUTS),
                ("nodes", Node * FZ_MAX_NODES)]


class EpiInput(C.Structure):
    """fz_epi_input: one input of a GEMM epilogue program (leaf k >= 1)."""
    _fields_ = [("ptr", C.c_void_p), ("batch_stride", C.c_int64), ("row_stride", C.c_int64),
                ("col_stride", C.c_int64)]


class GemmTimingRec(C.Structure):
    _fields_ = [("batch", C.c_int64), ("M", C.c_int64), ("N", C.c_int64), ("K", C.c_int64),
                ("pair", C.c_int32), ("epilogue", C.c_int32), ("splits", C.c_int32),
                ("ms", C.c_float)]


def header_symbols() -> list[str]:
    """Function names declared in include/fusion_b200.h."""
    text = HEADER.read_text()
    return re.findall(r"^\s*(?:const\s+char\s*\*|int64_t|int|void\s*\*)\s*(fz_\w+)\s*\(", text,
                      flags=re.M)


_lib = None


def lib() -> C.CDLL:
    """Load libfusion_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: run `python -m nova_b200.build`")
        L = C.CDLL(str(LIB_PATH))
        L.fz_last_error.restype = C.c_char_p
        L.fz_default_stream.restype = C.c_void_p
        L.fz_launch_count.restype = C.c_int64
        vp, i64, f = C.c_void_p, C.c_int64, C.c_float
        L.fz_malloc.argtypes = [C.POINTER(C.c_void_p), C.c_size_t, vp]
        L.fz_free.argtypes = [vp, vp]
        L.fz_memcpy_h2d.argtypes = [vp, vp, C.c_size_t, vp]
        L.fz_memcpy_d2h.argtypes = [vp, vp, C.c_size_t, vp]
        L.fz_memcpy_d2d.argtypes = [vp, vp, C.c_size_t, vp]
        L.fz_fill_f32.argtypes = [vp, f, i64, vp]
        L.fz_stream_sync.argtypes = [vp]
        L.fz_stream_create.argtypes = [C.POINTER(C.c_void_p)]
        L.fz_stream_destroy.argtypes = [vp]
        L.fz_stream_wait.argtypes = [vp, vp]
        L.fz_upload_stream.restype = C.c_void_p
        L.fz_event_record.argtypes = [C.POINTER(C.c_void_p), vp]
        L.fz_stream_wait_event.argtypes = [vp, vp]
        L.fz_event_destroy.argtypes = [vp]
        L.fz_ewise_binary.argtypes = [C.c_int, C.POINTER(EwisePlan), vp, vp, vp, vp]
        L.fz_ewise_binary_contig.argtypes = [C.c_int, i64, vp, vp, vp, vp]
        L.fz_ewise_unary.argtypes = [C.c_int, C.POINTER(EwisePlan), vp, vp, vp]
        L.fz_sub_inplace.argtypes = [vp, vp, i64, vp]
        L.fz_fused_launch.argtypes = [C.POINTER(Program), C.POINTER(EwisePlan),
                                      C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), vp]
        L.fz_reduce.argtypes = [C.c_int, vp, vp, i64, i64, i64, vp]
        L.fz_swapaxes.argtypes = [vp, vp, C.POINTER(C.c_int64), C.c_int, C.c_int, C.c_int, vp]
        L.fz_gemm_f32.argtypes = [i64, i64, i64, i64, vp, i64, i64, C.c_int, vp, i64, i64,
                                  C.c_int, vp, i64, i64, vp]
        L.fz_gemm_f32_split.argtypes = [i64, i64, i64, i64, vp, vp, i64, i64, C.c_int, vp, vp,
                                        i64, i64, C.c_int, vp, i64, i64, vp]
        L.fz_tf32_lo.argtypes = [vp, vp, i64, vp]
        L.fz_gemm_set_tiles.argtypes = [C.c_int]
        L.fz_gemm_set_tma_stores.argtypes = [C.c_int]
        L.fz_gemm_set_split.argtypes = [C.c_int]
        L.fz_gemm_split_launches.argtypes = [C.POINTER(C.c_int64)]
        L.fz_gemm_f32_epilogue.argtypes = [i64, i64, i64, i64, vp, vp, i64, i64, C.c_int, vp, vp,
                                           i64, i64, C.c_int, C.POINTER(Program),
                                           C.POINTER(EpiInput), C.POINTER(C.c_void_p), i64, i64, vp]
        L.fz_gemm_epilogue_compile.argtypes = [C.POINTER(Program), C.POINTER(EpiInput), C.c_int,
                                               C.c_int, C.c_int, C.c_int]
        L.fz_timer_create.argtypes = [C.POINTER(C.c_void_p)]
        L.fz_timer_start.argtypes = [vp, vp]
        L.fz_timer_stop.argtypes = [vp, vp]
        L.fz_timer_elapsed_ms.argtypes = [vp, C.POINTER(C.c_float)]
        L.fz_timer_destroy.argtypes = [vp]
        L.fz_host_alloc.argtypes = [C.POINTER(C.c_void_p), C.c_size_t]
        L.fz_host_free.argtypes = [vp]
        L.fz_gemm_stats.argtypes = [C.POINTER(C.c_int64)]
        L.fz_gemm_timing.argtypes = [C.c_int]
        L.fz_gemm_timing_read.argtypes = [C.POINTER(GemmTimingRec), C.c_int, C.POINTER(C.c_int)]
        L.fz_comm_init.argtypes = [C.POINTER(C.c_void_p), C.c_int, C.c_int, C.c_char_p]
        L.fz_comm_allreduce.argtypes = [vp, vp, vp, i64, f, vp]
        L.fz_comm_broadcast.argtypes = [vp, vp, i64, C.c_int, vp]
        L.fz_comm_wait.argtypes = [vp, vp, C.c_double]
        L.fz_comm_destroy.argtypes = [vp]
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != 0:
        raise FzError(rc, lib().fz_last_error().decode())


def device_count() -> int:
    n = C.c_int(0)
    rc = lib().fz_device_count(C.byref(n))
    return n.value if rc == 0 else 0


class DeviceArray:
    """An fp32 device buffer from the backend's pool (RAII)."""

    def __init__(self, shape, stream=None):
        self.shape = tuple(int(s) for s in shape)
        self.size = int(np.prod(self.shape)) if self.shape else 1
        self.nbytes = 4 * self.size
        self.stream = stream
        p = C.c_void_p()
        check(lib().fz_malloc(C.byref(p), self.nbytes, stream))
        self.ptr = p.value or 0

    @classmethod
    def from_numpy(cls, a: np.ndarray, stream=None) -> "DeviceArray":
        a = np.ascontiguousarray(a, dtype=np.float32)
        d = cls(a.shape, stream)
        check(lib().fz_memcpy_h2d(d.ptr, a.ctypes.data, a.nbytes, stream))
        return d

    def numpy(self) -> np.ndarray:
        out = np.empty(self.shape, dtype=np.float32)
        check(lib().fz_memcpy_d2h(out.ctypes.data, self.ptr, self.nbytes, self.stream))
        return out

    def free(self):
        if self.ptr:
            lib().fz_free(self.ptr, self.stream)
            self.ptr = 0

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def make_plan(out_shape, operand_shapes) -> EwisePlan:
    """Broadcast plan over `out_shape` for contiguous operands (output first).

    An operand dim of extent 1 facing a larger output dim gets stride 0, as
    stride_bytes_for_binding does (fusion/src/Fusion/core/TensorPlan.cpp:50-65)."""
    nd = len(out_shape)
    p = EwisePlan()
    p.ndim = nd
    p.num_operands = len(operand_shapes)
    for d in range(nd):
        p.size[d] = out_shape[d]
    for k, shp in enumerate(operand_shapes):
        pad = nd - len(shp)
        stride = 1
        st = [0] * nd
        for d in range(nd - 1, -1, -1):
            i = d - pad
            if i < 0:
                st[d] = 0
                continue
            st[d] = 0 if (shp[i] == 1 and out_shape[d] > 1) else stride * 4
            stride *= shp[i]
        for d in range(nd):
            p.stride_bytes[k][d] = st[d]
    return p


def gemm_timing_read(max_records: int = 4096) -> list:
    """The GEMM launches recorded since fz_gemm_timing(1), with their device times."""
    recs = (GemmTimingRec * max_records)()
    n = C.c_int()
    check(lib().fz_gemm_timing_read(recs, max_records, C.byref(n)))
    return list(recs[:n.value])
