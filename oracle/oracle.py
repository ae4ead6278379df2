"""Oracle for the Fusion hot path: the reference CPU path and its C restatement.

TEST INFRASTRUCTURE ONLY. Imported by tests/, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` as the checker; the nova_b200 package never
imports it.

Two back-ends, both loaded with ctypes from ``oracle/_ref`` (built by
``oracle/Makefile``):

* ``Port`` -- ``libfusion_oracle.so``, the C restatement in ``fusion_oracle.c``
  (each function cites the reference file:line it follows).
* ``Ref``  -- ``libfusion_ref.so``, the reference's own C++ sources
  (fusion/src/Fusion/**) compiled with ``ref_harness.cpp``, i.e. the real
  RawTensor operators, registry backward formulas and autodiff engine.
"""
from __future__ import annotations

import ctypes as C
import os
import pathlib

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
REF_DIR = HERE / "_ref"

BINOPS = {"add": 0, "sub": 1, "mul": 2, "div": 3, "pow": 4, "maximum": 5, "gt": 6, "ge": 7}
UNOPS = {"exp": 0, "log": 1, "sqrt": 2}
REDOPS = {"sum": 0, "mean": 1, "max": 2}

_f32p = C.POINTER(C.c_float)
_i64p = C.POINTER(C.c_int64)


def _fp(a: np.ndarray):
    return a.ctypes.data_as(_f32p)


def _shape(a):
    s = np.asarray(a, dtype=np.int64)
    return s, s.ctypes.data_as(_i64p)


class Port:
    """ctypes front-end of the C restatement (fusion_oracle.c)."""

    def __init__(self, path: str | os.PathLike | None = None):
        self.lib = C.CDLL(str(path or REF_DIR / "libfusion_oracle.so"))
        L = self.lib
        L.orc_broadcast_shape.restype = C.c_int
        L.orc_binary.restype = C.c_int
        L.orc_unary.restype = None
        L.orc_reduce.restype = None
        L.orc_matmul.restype = None
        L.orc_swapaxes.restype = None
        L.orc_philox4x32_10.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.POINTER(C.c_uint32)]
        L.orc_philox4x32_10.restype = None
        L.orc_philox_uniform.restype = None
        L.orc_philox_dropout.restype = None

    def broadcast_shape(self, sa, sb):
        a, ap = _shape(sa)
        b, bp = _shape(sb)
        out = np.zeros(max(len(a), len(b)), dtype=np.int64)
        n = self.lib.orc_broadcast_shape(ap, len(a), bp, len(b), out.ctypes.data_as(_i64p))
        if n < 0:
            raise RuntimeError("broadcast: dimension mismatch")
        return tuple(int(v) for v in out[:n])

    def binary(self, op: str, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        a = np.ascontiguousarray(a, dtype=np.float32)
        b = np.ascontiguousarray(b, dtype=np.float32)
        oshape = self.broadcast_shape(a.shape, b.shape)
        out = np.empty(oshape, dtype=np.float32)
        os_, osp = _shape(oshape)
        as_, asp = _shape(a.shape)
        bs_, bsp = _shape(b.shape)
        rc = self.lib.orc_binary(BINOPS[op], _fp(out), osp, len(os_), _fp(a), asp, len(as_),
                                 _fp(b), bsp, len(bs_))
        if rc:
            raise RuntimeError("orc_binary failed")
        return out

    def unary(self, op: str, a: np.ndarray) -> np.ndarray:
        a = np.ascontiguousarray(a, dtype=np.float32)
        out = np.empty_like(a)
        self.lib.orc_unary(UNOPS[op], _fp(out), _fp(a), C.c_int64(a.size))
        return out

    def reduce(self, op: str, a: np.ndarray, axis: int | None = None, keepdim: bool = False):
        a = np.ascontiguousarray(a, dtype=np.float32)
        if axis is None:
            out = np.empty((1,), dtype=np.float32)
            ax = -1
        else:
            ax = axis % a.ndim
            shp = list(a.shape)
            if keepdim:
                shp[ax] = 1
            else:
                del shp[ax]
            out = np.empty(shp, dtype=np.float32)
        s, sp = _shape(a.shape)
        self.lib.orc_reduce(REDOPS[op], _fp(out), _fp(a), sp, a.ndim, ax)
        return out

    def matmul(self, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        a = np.ascontiguousarray(a, dtype=np.float32)
        b = np.ascontiguousarray(b, dtype=np.float32)
        m, k = a.shape[-2:]
        k2, n = b.shape[-2:]
        assert k == k2 and a.shape[:-2] == b.shape[:-2]
        batch = int(np.prod(a.shape[:-2])) if a.ndim > 2 else 1
        out = np.empty(a.shape[:-2] + (m, n), dtype=np.float32)
        self.lib.orc_matmul(_fp(out), _fp(a), _fp(b), C.c_int64(batch), C.c_int64(m),
                            C.c_int64(n), C.c_int64(k))
        return out

    def philox_block(self, ctr_lo: int, ctr_hi: int, key: int) -> list:
        out = (C.c_uint32 * 4)()
        self.lib.orc_philox4x32_10(C.c_uint64(ctr_lo), C.c_uint64(ctr_hi), C.c_uint64(key), out)
        return list(out)

    def philox_uniform(self, n: int, seed: int, offset: int, lo: float, hi: float) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.lib.orc_philox_uniform(_fp(out), C.c_int64(n), C.c_uint64(seed), C.c_uint64(offset),
                                    C.c_float(lo), C.c_float(hi))
        return out

    def philox_dropout(self, x: np.ndarray, rate: float, keep: float, seed: int, offset: int) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        self.lib.orc_philox_dropout(_fp(out), _fp(x), C.c_int64(x.size), C.c_float(rate), C.c_float(keep),
                                    C.c_uint64(seed), C.c_uint64(offset))
        return out

    def swapaxes(self, a: np.ndarray, a1: int, a2: int) -> np.ndarray:
        a = np.ascontiguousarray(a, dtype=np.float32)
        nd = a.ndim
        a1 %= nd
        a2 %= nd
        shp = list(a.shape)
        shp[a1], shp[a2] = shp[a2], shp[a1]
        out = np.empty(shp, dtype=np.float32)
        s, sp = _shape(a.shape)
        self.lib.orc_swapaxes(_fp(out), _fp(a), sp, nd, a1, a2)
        return out


class _RefTensor:
    def __init__(self, lib, h):
        self.lib, self.h = lib, h

    def __del__(self):
        if self.h:
            self.lib.ref_tensor_free(self.h)

    def numpy(self) -> np.ndarray:
        nd = self.lib.ref_tensor_ndim(self.h)
        shp = (C.c_uint64 * nd)()
        self.lib.ref_tensor_shape(self.h, shp)
        out = np.empty(tuple(shp), dtype=np.float32)
        self.lib.ref_tensor_read(self.h, _fp(out))
        return out


class Ref:
    """ctypes front-end of the reference C++ path (ref_harness.cpp)."""

    def __init__(self, path: str | os.PathLike | None = None):
        self.lib = C.CDLL(str(path or REF_DIR / "libfusion_ref.so"))
        L = self.lib
        for name in ("ref_tensor_new", "ref_binary", "ref_binary_scalar", "ref_unary",
                     "ref_reduce", "ref_matmul", "ref_swapaxes"):
            getattr(L, name).restype = C.c_void_p
        L.ref_tensor_free.argtypes = [C.c_void_p]
        L.ref_tensor_ndim.argtypes = [C.c_void_p]
        L.ref_tensor_shape.argtypes = [C.c_void_p, C.POINTER(C.c_uint64)]
        L.ref_tensor_read.argtypes = [C.c_void_p, _f32p]
        L.ref_tensor_numel.restype = C.c_uint64
        L.ref_tensor_numel.argtypes = [C.c_void_p]
        L.ref_binary.argtypes = [C.c_int, C.c_void_p, C.c_void_p]
        L.ref_binary_scalar.argtypes = [C.c_int, C.c_void_p, C.c_float]
        L.ref_unary.argtypes = [C.c_int, C.c_void_p]
        L.ref_reduce.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_int]
        L.ref_matmul.argtypes = [C.c_void_p, C.c_void_p]
        L.ref_swapaxes.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.ref_sub_inplace.argtypes = [C.c_void_p, C.c_void_p]
        L.ref_backward.argtypes = [C.c_char_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                   C.POINTER(C.c_void_p)]
        L.ref_mlp_step.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p),
                                   C.POINTER(C.c_void_p), C.c_int, C.c_float, _f32p]
        L.ref_mlp_step_grads.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p),
                                         C.POINTER(C.c_void_p), C.c_int, C.c_float, _f32p,
                                         C.POINTER(C.c_void_p)]
        L.ref_last_error.restype = C.c_char_p

    def _check(self, h):
        if not h:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return _RefTensor(self.lib, h)

    def tensor(self, a: np.ndarray) -> _RefTensor:
        a = np.ascontiguousarray(a, dtype=np.float32)
        shp = (C.c_uint64 * max(a.ndim, 1))(*(a.shape or (1,)))
        return self._check(self.lib.ref_tensor_new(shp, max(a.ndim, 1), _fp(a)))

    # Input handles are bound to locals so they outlive the call (a temporary's
    # __del__ would free the reference tensor before the C++ side reads it).
    def binary(self, op, a, b):
        ta, tb = self.tensor(a), self.tensor(b)
        return self._check(self.lib.ref_binary(BINOPS[op], ta.h, tb.h)).numpy()

    def binary_scalar(self, op, a, s: float):
        ta = self.tensor(a)
        return self._check(self.lib.ref_binary_scalar(BINOPS[op], ta.h, s)).numpy()

    def unary(self, op, a):
        ta = self.tensor(a)
        return self._check(self.lib.ref_unary(UNOPS[op], ta.h)).numpy()

    def reduce(self, op, a, axis=None, keepdim=False):
        ax = -1 if axis is None else axis % np.ndim(a)
        ta = self.tensor(a)
        return self._check(self.lib.ref_reduce(REDOPS[op], ta.h, ax, int(keepdim))).numpy()

    def matmul(self, a, b):
        ta, tb = self.tensor(a), self.tensor(b)
        return self._check(self.lib.ref_matmul(ta.h, tb.h)).numpy()

    def swapaxes(self, a, a1, a2):
        ta = self.tensor(a)
        return self._check(self.lib.ref_swapaxes(ta.h, a1, a2)).numpy()

    def backward(self, name: str, x, y, g0):
        tx = self.tensor(x)
        ty = self.tensor(y) if y is not None else None
        tg = self.tensor(g0)
        out = (C.c_void_p * 2)()
        n = self.lib.ref_backward(name.encode(), tx.h, ty.h if ty else None, tg.h, out)
        if n <= 0:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return [_RefTensor(self.lib, out[i]).numpy() for i in range(n)]

    def mlp_step(self, X, Y, Ws, bs, lr, grads=False):
        """One reference MLP training step; returns (new Ws, new bs, loss), and with
        grads=True also the gradients [(gW_i, gb_i)] the engine computed."""
        tX, tY = self.tensor(X), self.tensor(Y)
        tW = [self.tensor(w) for w in Ws]
        tb = [self.tensor(b) for b in bs]
        n = len(Ws)
        Wa = (C.c_void_p * n)(*[t.h for t in tW])
        ba = (C.c_void_p * n)(*[t.h for t in tb])
        loss = np.empty((X.shape[0], Ws[-1].shape[0]), dtype=np.float32)
        if not grads:
            rc = self.lib.ref_mlp_step(tX.h, tY.h, Wa, ba, n, C.c_float(lr), _fp(loss))
            if rc:
                raise RuntimeError(self.lib.ref_last_error().decode())
            return [t.numpy() for t in tW], [t.numpy() for t in tb], loss
        ga = (C.c_void_p * (2 * n))()
        rc = self.lib.ref_mlp_step_grads(tX.h, tY.h, Wa, ba, n, C.c_float(lr), _fp(loss), ga)
        hs = [_RefTensor(self.lib, ga[i]) if ga[i] else None for i in range(2 * n)]
        if rc:
            raise RuntimeError(self.lib.ref_last_error().decode())
        gr = [(hs[2 * i].numpy() if hs[2 * i] else None, hs[2 * i + 1].numpy() if hs[2 * i + 1] else None)
              for i in range(n)]
        return [t.numpy() for t in tW], [t.numpy() for t in tb], loss, gr


def have_ref() -> bool:
    return (REF_DIR / "libfusion_ref.so").exists()


def have_port() -> bool:
    return (REF_DIR / "libfusion_oracle.so").exists()


def mlp_step_f64(X, Y, Ws, bs, masks=None):
    """Float64 restatement of the reference MLP step's forward and backward (Nova's
    Linear/ReLU/MSE sequence as the registry differentiates it): pre-activations
    t_l = h_{l-1} W_l^T + b_l (nova/src/blocks/core/linear.py:42-48), h_l = relu(t_l)
    for hidden layers (activations.py:9-10), loss = (out - Y)^2 / size elementwise
    (losses/loss.py:34-37); backward g_L = 2 (out - Y) / size (Pow.hpp:34-51 with the
    Divide backward), gW_l = g_l^T h_{l-1} (MatMul.hpp:55-58 through SwapAxes), gb_l = g_l
    unreduced ([B, U], Add.hpp:41-45), g_{l-1} = (g_l W_l) * (t_{l-1} > 0) (Maximum.hpp:
    34-51; `>=` is `>`). `masks` (one boolean array per hidden layer) replaces the
    ReLU decisions t > 0, so a float32 implementation's own decisions can be replayed
    exactly. Returns loss, [(gW_l, gb_l)], [t_l] (float64) and the masks used."""
    X = np.asarray(X, np.float64)
    Y = np.asarray(Y, np.float64)
    Ws = [np.asarray(w, np.float64) for w in Ws]
    bs = [np.asarray(b, np.float64) for b in bs]
    L = len(Ws)
    hs, ts, used = [X], [], []
    for i in range(L):
        t = hs[-1] @ Ws[i].T + bs[i]
        ts.append(t)
        if i + 1 < L:
            m = (t > 0) if masks is None else np.asarray(masks[i], bool)
            used.append(m)
            hs.append(t * m)
    out = ts[-1]
    loss = (out - Y) ** 2 / out.size
    g = 2.0 * (out - Y) / out.size
    grads = [None] * L
    for i in range(L - 1, -1, -1):
        grads[i] = (g.T @ hs[i], g)
        if i > 0:
            g = (g @ Ws[i]) * used[i - 1]
    return loss, grads, ts, used
