"""GEMMs with a fused epilogue program (fz_gemm_f32_epilogue), through the C ABI.

Contract: the outputs equal, bit for bit, the plain GEMM into a buffer followed by the
same program as one fused elementwise pass over it (fz_fused_launch), for every kernel
variant the dispatch picks: CTA pairs, 256-, 64- and 16-column single-CTA tiles,
MN-major operands, split K (the product formed in a workspace first), K = 0, batches,
ragged extents and output pitches that rule out 16-byte stores.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_bits_equal

pytestmark = pytest.mark.gpu

RNG = np.random.default_rng(77)
TILES = {"auto": 0, "single": 1, "pair": 2}


def _program(A, nodes, nleaves, outs):
    p = A.Program()
    p.num_nodes, p.num_leaves, p.num_outputs = len(nodes), nleaves, len(outs)
    for i, o in enumerate(outs):
        p.out_node[i] = o
    for i, (kind, op, s0, s1, imm) in enumerate(nodes):
        n = p.nodes[i]
        n.kind, n.op, n.src0, n.src1, n.imm = kind, op, s0, s1, imm
    return p


def _programs(A):
    B, U, K = A.NODE_BINARY, A.NODE_UNARY, A.NODE_CONST
    bo, uo = A.BINOPS, A.UNOPS
    return {
        # a hidden layer's forward: relu(P + bias), its TF32 remainder plane, and P
        "bias_relu": ([(B, bo["add"], -1, -2, 0.0), (K, 0, 0, 0, 0.0), (B, bo["maximum"], 0, 1, 0.0),
                       (U, uo["tf32_lo"], 2, 0, 0.0), (U, uo["copy"], -1, 0, 0.0)],
                      ["row"], [2, 3, 4]),
        # its backward: P * (T + bias > 0) with the remainder plane
        "relu_mask": ([(B, bo["add"], -2, -3, 0.0), (K, 0, 0, 0, 0.0), (B, bo["gt"], 0, 1, 0.0),
                       (B, bo["mul"], -1, 2, 0.0), (U, uo["tf32_lo"], 3, 0, 0.0)],
                      ["full", "row"], [3, 4]),
        # two full-shape inputs and four outputs (inputs and outputs share the staging
        # tile in 4-column blocks)
        "two_full_four_out": ([(B, bo["mul"], -1, -2, 0.0), (B, bo["add"], -1, -3, 0.0),
                               (B, bo["sub"], 0, 1, 0.0), (U, uo["copy"], -1, 0, 0.0)],
                              ["full", "full"], [0, 1, 2, 3]),
        # five full-shape inputs and four outputs (too many to share the tile: the
        # inputs are read per output pass)
        "five_full_four_out": ([(B, bo["add"], -1, -2, 0.0), (B, bo["add"], 0, -3, 0.0),
                                (B, bo["add"], 1, -4, 0.0), (B, bo["mul"], 2, -5, 0.0),
                                (B, bo["sub"], 3, -6, 0.0)],
                               ["full"] * 5, [1, 2, 3, 4]),
        # a per-row and a scalar input: exp(P / c_i) - s
        "row_scale_exp": ([(B, bo["div"], -1, -2, 0.0), (U, uo["exp"], 0, 0, 0.0),
                           (B, bo["sub"], 1, -3, 0.0)],
                          ["col", "scalar"], [2]),
    }


def _input(A, kind, batch, M, N):
    """(host array, fz_epi_input strides, shape for the reference plan)."""
    if kind == "row":
        a = RNG.uniform(-0.5, 0.5, (N,)).astype(np.float32)
        return a, (0, 0, 1), (N,)
    if kind == "full":
        a = RNG.standard_normal((batch, M, N)).astype(np.float32)
        return a, (M * N, N, 1), (batch, M, N)
    if kind == "col":
        a = RNG.uniform(1.0, 4.0, (batch, M, 1)).astype(np.float32)
        return a, (M, 1, 0), (batch, M, 1)
    a = np.array([0.25], np.float32)
    return a, (0, 0, 0), (1,)


def _run(A, name, batch, M, N, K, tA, tB, ldc_pad=0, tiles="auto"):
    L = A.lib()
    nodes, kinds, outs = _programs(A)[name]
    prog = _program(A, nodes, 1 + len(kinds), outs)
    a = RNG.standard_normal((batch, K, M) if tA else (batch, M, K)).astype(np.float32)
    b = RNG.standard_normal((batch, N, K) if tB else (batch, K, N)).astype(np.float32)
    da, db = A.DeviceArray.from_numpy(a), A.DeviceArray.from_numpy(b)
    lda, ldb, sA, sB = a.shape[2], b.shape[2], a.shape[1] * a.shape[2], b.shape[1] * b.shape[2]
    ins = [_input(A, k, batch, M, N) for k in kinds]
    dins = [A.DeviceArray.from_numpy(x) for x, _, _ in ins]
    epi_in = (A.EpiInput * max(1, len(ins)))(*[A.EpiInput(d.ptr, *st) for d, (_, st, _) in zip(dins, ins)])
    ldc = N + ldc_pad
    sC = M * ldc
    got = [A.DeviceArray((batch, M, ldc)) for _ in outs]
    want = [A.DeviceArray((batch, M, ldc)) for _ in outs]
    P = A.DeviceArray((batch, M, N))
    capi_outs = lambda arrs: (C.c_void_p * len(arrs))(*[x.ptr for x in arrs])
    A.check(L.fz_gemm_set_tiles(TILES[tiles]))
    try:
        A.check(L.fz_gemm_f32_epilogue(batch, M, N, K, da.ptr, None, lda, sA, int(tA), db.ptr, None,
                                       ldb, sB, int(tB), C.byref(prog), epi_in, capi_outs(got), ldc, sC,
                                       None))
        # the reference product with per-thread stores (the epilogue above uses TMA
        # stores wherever the outputs allow)
        A.check(L.fz_gemm_set_tma_stores(0))
        A.check(L.fz_gemm_f32_split(batch, M, N, K, da.ptr, None, lda, sA, int(tA), db.ptr, None, ldb,
                                    sB, int(tB), P.ptr, N, M * N, None))
    finally:
        L.fz_gemm_set_tiles(0)
        L.fz_gemm_set_tma_stores(1)
    # reference: the program as a fused pass over P
    plan = A.EwisePlan()
    plan.ndim, plan.num_operands = 3, len(outs) + 1 + len(ins)
    for d, v in enumerate((batch, M, N)):
        plan.size[d] = v
    strides = [(sC, ldc, 1)] * len(outs) + [(M * N, N, 1)] + [st for _, st, _ in ins]
    for k, st in enumerate(strides):
        for d in range(3):
            plan.stride_bytes[k][d] = st[d] * 4
    leaves = (C.c_void_p * (1 + len(ins)))(P.ptr, *[d.ptr for d in dins])
    A.check(L.fz_fused_launch(C.byref(prog), C.byref(plan), capi_outs(want), leaves, None))
    A.check(L.fz_kernel_status())
    for k, (g, w) in enumerate(zip(got, want)):
        gv, wv = g.numpy()[..., :N], w.numpy()[..., :N]
        assert_bits_equal(gv, wv, f"{name} output {k}")
    return got


CASES = [
    # batch, M, N, K, tA, tB, ldc pad, tile mode
    (1, 2560, 2048, 256, False, True, 0, "auto"),    # CTA pairs, activations x W^T
    (1, 1024, 1024, 512, False, False, 0, "pair"),   # pairs, MN-major B
    (1, 1024, 1024, 512, True, False, 0, "single"),  # 256-column single CTAs, MN-major A
    (1, 4096, 16, 1024, False, True, 0, "auto"),     # 16-column tiles (output layer)
    (1, 2048, 48, 300, False, False, 0, "auto"),     # 64-column tiles, B transposed first
    (1, 256, 256, 8192, True, False, 0, "auto"),     # split K: product in a workspace
    (3, 300, 270, 100, False, True, 0, "auto"),      # batch, ragged, N % 4 != 0 (scalar stores)
    (2, 520, 264, 64, False, False, 4, "auto"),      # padded output pitch (16-byte stores)
    (1, 130, 260, 40, False, True, 1, "auto"),       # odd output pitch (scalar stores)
    (1, 96, 128, 0, False, True, 0, "auto"),         # K = 0: the program over zeros
]


@pytest.mark.parametrize("name", ["bias_relu", "relu_mask", "row_scale_exp", "two_full_four_out",
                                  "five_full_four_out"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: "x".join(map(str, c[:4])) + f"-{c[7]}")
def test_epilogue_equals_gemm_then_program(capi, name, case):
    _run(capi, name, *case)


@pytest.mark.parametrize("name", ["bias_relu", "relu_mask", "two_full_four_out"])
def test_epilogue_thread_stores(capi, name):
    """The per-thread-store form of the generated epilogues (TMA stores off)."""
    L = capi.lib()
    capi.check(L.fz_gemm_set_tma_stores(0))
    try:
        for case in CASES[:3]:
            _run(capi, name, *case)
    finally:
        L.fz_gemm_set_tma_stores(1)


def test_epilogue_at_a_hidden_layer_size(capi):
    """[8192, 1024] x [4096, 1024]^T with relu(P + b), its plane and P: pairs, in-kernel."""
    _run(capi, "bias_relu", 1, 8192, 4096, 1024, False, True)


def test_epilogue_rejects_bad_programs(capi):
    A, L = capi, capi.lib()
    B = A.NODE_BINARY
    d = A.DeviceArray((64, 64))
    outs = (C.c_void_p * 1)(d.ptr)
    bad_stride = (A.EpiInput * 1)(A.EpiInput(d.ptr, 0, 64, 2))
    prog = _program(A, [(B, A.BINOPS["add"], -1, -2, 0.0)], 2, [0])
    rc = L.fz_gemm_f32_epilogue(1, 64, 64, 64, d.ptr, None, 64, 0, 0, d.ptr, None, 64, 0, 0,
                                C.byref(prog), bad_stride, outs, 64, 64 * 64, None)
    assert rc == 1 and b"column stride" in L.fz_last_error()
    no_leaf = _program(A, [(A.NODE_CONST, 0, 0, 0, 1.0)], 0, [0])
    rc = L.fz_gemm_f32_epilogue(1, 64, 64, 64, d.ptr, None, 64, 0, 0, d.ptr, None, 64, 0, 0,
                                C.byref(no_leaf), None, outs, 64, 64 * 64, None)
    assert rc == 1
