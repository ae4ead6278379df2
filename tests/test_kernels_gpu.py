"""Parity of the sm_100a kernels, called through the C ABI, against the oracle.

Bars (from the hot-path contract): add/sub/mul/div/maximum/comparisons/sqrt and all
index work bit-exact; exp/log within 2 ulp of glibc (the reference's libm); sum/mean
within 1e-5 * sum|x| per output; max exact; GEMM within 1e-5 norm-wise relative error
and 1e-5 * (|A||B|)_ij elementwise.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_bits_equal, ulp_diff

pytestmark = pytest.mark.gpu

RNG = np.random.default_rng(1234)
OPS = ["add", "sub", "mul", "div", "pow", "maximum", "gt", "ge"]


def _inputs(op, sa, sb):
    if op == "pow":
        a = RNG.uniform(0.01, 10, sa).astype(np.float32)
        b = RNG.uniform(-2, 2, sb).astype(np.float32)
    else:
        a = RNG.uniform(-1, 1, sa).astype(np.float32)
        b = (RNG.uniform(0.5, 2, sb) if op == "div" else RNG.uniform(-1, 1, sb)).astype(np.float32)
    if op in ("maximum", "gt", "ge") and a.size > 4 and a.shape == b.shape:
        a.ravel()[:4] = b.ravel()[:4]  # ties
    return a, b


def _check_binary(op, got, want):
    if op == "pow":
        assert ulp_diff(got, want).max() <= 2
    else:
        assert_bits_equal(got, want, op)


@pytest.mark.parametrize("op", OPS)
@pytest.mark.parametrize("n", [1, 3, 4, 1029, (1 << 20) + 3])
def test_binary_contig(capi, port, op, n):
    a, b = _inputs(op, (n,), (n,))
    da, db, do = capi.DeviceArray.from_numpy(a), capi.DeviceArray.from_numpy(b), capi.DeviceArray((n,))
    capi.check(capi.lib().fz_ewise_binary_contig(capi.BINOPS[op], n, do.ptr, da.ptr, db.ptr, None))
    _check_binary(op, do.numpy(), port.binary(op, a, b))


def test_pow_square(capi, port):
    """x ** 2 is the correctly rounded x*x; glibc powf (the reference's std::pow) is
    not always correctly rounded, so the two may differ by 1 ulp."""
    a = RNG.standard_normal(100003).astype(np.float32)
    b = np.full((1,), 2.0, np.float32)
    plan = capi.make_plan(a.shape, [a.shape, a.shape, b.shape])
    da, db, do = capi.DeviceArray.from_numpy(a), capi.DeviceArray.from_numpy(b), capi.DeviceArray(a.shape)
    capi.check(capi.lib().fz_ewise_binary(capi.BINOPS["pow"], C.byref(plan), do.ptr, da.ptr, db.ptr, None))
    got = do.numpy()
    assert_bits_equal(got, a * a, "x**2 == x*x")
    assert ulp_diff(got, port.binary("pow", a, b)).max() <= 1


BCAST = [((5, 7), (7,)), ((4, 1), (4, 9)), ((3, 1, 8), (5, 1)), ((129, 1031), (1, 1031)),
         ((1,), (4, 3)), ((6, 1), (1, 8)), ((2, 3, 4, 5), (3, 1, 5)), ((0, 4), (4,))]


@pytest.mark.parametrize("op", OPS)
@pytest.mark.parametrize("sa,sb", BCAST)
def test_binary_broadcast(capi, port, op, sa, sb):
    """The kernel computes op(a, b) over the broadcast plan exactly as given."""
    a, b = _inputs(op, sa, sb)
    out_shape = np.broadcast_shapes(sa, sb)
    plan = capi.make_plan(out_shape, [out_shape, sa, sb])
    da, db, do = capi.DeviceArray.from_numpy(a), capi.DeviceArray.from_numpy(b), capi.DeviceArray(out_shape)
    capi.check(capi.lib().fz_ewise_binary(capi.BINOPS[op], C.byref(plan), do.ptr, da.ptr, db.ptr, None))
    want = port.binary(op, np.broadcast_to(a, out_shape).copy(), np.broadcast_to(b, out_shape).copy())
    _check_binary(op, do.numpy(), want)


@pytest.mark.parametrize("op,lo,hi", [("exp", -4, 4), ("log", 0.01, 10), ("sqrt", 0.01, 10),
                                      ("copy", -1, 1)])
@pytest.mark.parametrize("n", [1, 7, (1 << 20) + 1])
def test_unary(capi, port, op, lo, hi, n):
    a = RNG.uniform(lo, hi, n).astype(np.float32)
    plan = capi.make_plan((n,), [(n,), (n,)])
    da, do = capi.DeviceArray.from_numpy(a), capi.DeviceArray((n,))
    capi.check(capi.lib().fz_ewise_unary(capi.UNOPS[op], C.byref(plan), do.ptr, da.ptr, None))
    got = do.numpy()
    if op == "copy":
        assert_bits_equal(got, a)
    elif op == "sqrt":
        assert_bits_equal(got, port.unary(op, a), op)
    else:
        assert ulp_diff(got, port.unary(op, a)).max() <= 2


def test_unary_special_values(capi, port):
    a = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1.0, 88.8, -104.0], np.float32)
    for op in ("exp", "log", "sqrt"):
        plan = capi.make_plan(a.shape, [a.shape, a.shape])
        da, do = capi.DeviceArray.from_numpy(a), capi.DeviceArray(a.shape)
        capi.check(capi.lib().fz_ewise_unary(capi.UNOPS[op], C.byref(plan), do.ptr, da.ptr, None))
        with np.errstate(all="ignore"):
            assert ulp_diff(do.numpy(), port.unary(op, a)).max() <= 2, op


def _reduce_gpu(capi, op, x, axis):
    if axis is None:
        outer, ln, inner = 1, x.size, 1
        oshape = (1,)
    else:
        outer = int(np.prod(x.shape[:axis]))
        ln = x.shape[axis]
        inner = int(np.prod(x.shape[axis + 1:]))
        oshape = x.shape[:axis] + x.shape[axis + 1:]
    dx, do = capi.DeviceArray.from_numpy(x), capi.DeviceArray(oshape or (1,))
    capi.check(capi.lib().fz_reduce(capi.REDOPS[op], do.ptr, dx.ptr, outer, ln, inner, None))
    return do.numpy()


@pytest.mark.parametrize("shape,axis", [((1024, 1024), 1), ((1024, 1024), 0), ((513, 1031), 1),
                                        ((513, 1031), 0), ((3, 5, 7), 1), ((7, 9, 64), 2),
                                        ((16, 256, 64, 64), 0), ((1 << 22,), None), ((5,), None),
                                        ((2, 70000), 1), ((70000, 3), 0), ((4096, 8192), 0),
                                        ((3, 2000, 512), 1), ((100, 260), 0), ((1 << 16, 64), 1),
                                        ((999, 200), 1)])
@pytest.mark.parametrize("op", ["sum", "mean", "max"])
def test_reduce(capi, port, shape, axis, op):
    x = RNG.standard_normal(shape).astype(np.float32)
    got = _reduce_gpu(capi, op, x, axis)
    want = port.reduce(op, x, axis)
    assert got.shape == want.reshape(got.shape).shape
    want = want.reshape(got.shape)
    if op == "max":
        assert_bits_equal(got, want, "max")
    else:
        absx = np.abs(x.astype(np.float64))
        bound = (absx.sum() if axis is None else absx.sum(axis=axis)).reshape(got.shape)
        if op == "mean":
            bound = bound / (x.size if axis is None else x.shape[axis])
        assert np.all(np.abs(got.astype(np.float64) - want) <= 1e-5 * bound + 1e-30)


def test_reduce_max_nan_and_zero_sign(capi, port):
    x = np.array([[-0.0, 0.0, -1.0], [1.0, np.nan, 2.0], [-0.0, -0.0, -3.0]], np.float32)
    for axis in (0, 1):
        assert_bits_equal(_reduce_gpu(capi, "max", x, axis), port.reduce("max", x, axis))


@pytest.mark.parametrize("shape", [(4096, 1024), (3000, 64)])
def test_reduce_max_nan_and_zero_sign_split(capi, port, shape):
    """The same rules when a column's rows are split over warps and cluster CTAs (or
    chunks) and when rows are reduced several at a time: NaN anywhere wins, +0 ranks
    above -0, wherever they sit."""
    x = -np.abs(RNG.standard_normal(shape)).astype(np.float32)
    x[:, 0] = -0.0
    x[shape[0] // 2, 1] = 0.0  # one +0 among -0s in a column of negatives
    x[:, 1] = np.where(np.arange(shape[0]) == shape[0] // 2, 0.0, -0.0)
    x[shape[0] - 1, 2] = np.nan
    x[7, shape[1] - 1] = np.nan
    x[3, 5] = np.nan
    for axis in (0, 1):
        assert_bits_equal(_reduce_gpu(capi, "max", x, axis), port.reduce("max", x, axis), f"axis {axis}")


@pytest.mark.parametrize("shape,a1,a2", [((33, 65), 0, 1), ((4096, 1024), 1, 0), ((3, 40, 50), 1, 2),
                                         ((3, 40, 50), 0, 2), ((2, 3, 4, 5), 0, 2),
                                         ((6, 7, 8), 0, 1), ((1, 5), 0, 1), ((5, 1, 3), 0, 1),
                                         ((68, 100), 0, 1), ((8, 12, 20, 36), 1, 3),
                                         ((5, 64, 132), 1, 2), ((4, 4), 0, 1), ((1000, 4), 0, 1)])
def test_swapaxes(capi, port, shape, a1, a2):
    x = RNG.standard_normal(shape).astype(np.float32)
    want = port.swapaxes(x, a1, a2)
    dx, do = capi.DeviceArray.from_numpy(x), capi.DeviceArray(want.shape)
    shp = (C.c_int64 * len(shape))(*shape)
    capi.check(capi.lib().fz_swapaxes(do.ptr, dx.ptr, shp, len(shape), a1, a2, None))
    assert_bits_equal(do.numpy(), want, "swapaxes")


def _gemm(capi, a, b, transA=False, transB=False):
    """C = op(A) @ op(B) for batched [batch, r, c] inputs."""
    batch = a.shape[0]
    M = a.shape[2] if transA else a.shape[1]
    K = a.shape[1] if transA else a.shape[2]
    N = b.shape[1] if transB else b.shape[2]
    da, db, dc = capi.DeviceArray.from_numpy(a), capi.DeviceArray.from_numpy(b), capi.DeviceArray((batch, M, N))
    lda, ldb = a.shape[2], b.shape[2]
    capi.check(capi.lib().fz_gemm_f32(batch, M, N, K, da.ptr, lda, a.shape[1] * a.shape[2], int(transA),
                                      db.ptr, ldb, b.shape[1] * b.shape[2], int(transB),
                                      dc.ptr, N, M * N, None))
    capi.check(capi.lib().fz_kernel_status())
    return dc.numpy()


@pytest.mark.parametrize("batch,M,N,K", [(1, 128, 256, 32), (1, 256, 512, 256), (1, 200, 300, 70),
                                         (1, 1, 5, 3), (3, 65, 33, 17), (1, 512, 512, 1024),
                                         (2, 1000, 129, 257), (1, 256, 512, 4096),
                                         (1, 160, 300, 16384)])
@pytest.mark.parametrize("tA,tB", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm_3xtf32(capi, port, batch, M, N, K, tA, tB):
    s = 1.0 / np.sqrt(K)
    A = (RNG.standard_normal((batch, M, K)) * s).astype(np.float32)
    B = (RNG.standard_normal((batch, K, N)) * s).astype(np.float32)
    a_in = np.ascontiguousarray(A.transpose(0, 2, 1)) if tA else A
    b_in = np.ascontiguousarray(B.transpose(0, 2, 1)) if tB else B
    got = _gemm(capi, a_in, b_in, tA, tB)
    want = port.matmul(A, B)
    err = np.linalg.norm((got - want).ravel()) / max(np.linalg.norm(want.ravel()), 1e-30)
    assert err <= 1e-5, err
    bound = np.einsum("bmk,bkn->bmn", np.abs(A.astype(np.float64)), np.abs(B.astype(np.float64)))
    assert np.all(np.abs(got - want) <= 1e-5 * bound + 1e-30)


@pytest.mark.parametrize("tA,tB", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("batch,M,N,K", [(1, 2560, 2048, 256), (1, 2600, 2100, 200),
                                         (2, 1536, 1792, 64), (1, 2560, 2048, 8192)])
def test_gemm_3xtf32_cta_pairs(capi, batch, M, N, K, tA, tB):
    """Shapes with enough 256 x 256 tiles for the CTA-pair kernel (cta_group::2): ragged
    M and N, K not a multiple of the k-tile, batches, and a K long enough to be split."""
    rng = np.random.default_rng(M + N + K + batch)
    s = 1.0 / np.sqrt(K)
    A = (rng.standard_normal((batch, M, K)) * s).astype(np.float32)
    B = (rng.standard_normal((batch, K, N)) * s).astype(np.float32)
    a_in = np.ascontiguousarray(A.transpose(0, 2, 1)) if tA else A
    b_in = np.ascontiguousarray(B.transpose(0, 2, 1)) if tB else B
    got = _gemm(capi, a_in, b_in, tA, tB)
    want = np.matmul(A.astype(np.float64), B.astype(np.float64))
    err = np.linalg.norm((got - want).ravel()) / np.linalg.norm(want.ravel())
    assert err <= 1e-5, err
    bound = np.matmul(np.abs(A).astype(np.float64), np.abs(B).astype(np.float64))
    assert np.all(np.abs(got - want) <= 1e-5 * bound + 1e-30)


def _gemm_into(capi, a, b, tA, tB, ldc, strideC):
    """fz_gemm_f32 into an output of pitch ldc and slice pitch strideC (padding kept)."""
    batch = a.shape[0]
    M = a.shape[2] if tA else a.shape[1]
    K = a.shape[1] if tA else a.shape[2]
    N = b.shape[1] if tB else b.shape[2]
    da, db = capi.DeviceArray.from_numpy(a), capi.DeviceArray.from_numpy(b)
    dc = capi.DeviceArray.from_numpy(np.full((batch * strideC,), 7.0, np.float32))
    capi.check(capi.lib().fz_gemm_f32(batch, M, N, K, da.ptr, a.shape[2], a.shape[1] * a.shape[2], int(tA),
                                      db.ptr, b.shape[2], b.shape[1] * b.shape[2], int(tB), dc.ptr, ldc,
                                      strideC, None))
    capi.check(capi.lib().fz_kernel_status())
    return dc.numpy()


@pytest.mark.parametrize("batch,M,N,K,pad,tB", [
    (1, 2560, 2048, 256, 0, True),    # CTA pairs
    (1, 300, 200, 100, 0, False),     # single CTAs, ragged M and N
    (2, 520, 264, 64, 4, True),       # batch, padded pitch
    (1, 4096, 16, 512, 0, True),      # 16-column tiles
    (1, 2048, 48, 300, 0, False),     # 64-column tiles
    (1, 256, 256, 8192, 0, False),    # K split: partials stored by TMA
    (1, 130, 260, 40, 1, True),       # odd pitch: per-thread stores either way
])
def test_gemm_tma_stores_match_thread_stores(capi, batch, M, N, K, pad, tB):
    """Outputs written by TMA bulk tensor stores equal per-thread stores bit for bit,
    and neither touches the padding past N."""
    L = capi.lib()
    rng = np.random.default_rng(M * 7 + N + K)
    A = rng.standard_normal((batch, M, K)).astype(np.float32)
    B = rng.standard_normal((batch, N, K) if tB else (batch, K, N)).astype(np.float32)
    ldc = N + pad
    outs = []
    try:
        for on in (1, 0):
            capi.check(L.fz_gemm_set_tma_stores(on))
            outs.append(_gemm_into(capi, A, B, False, tB, ldc, M * ldc))
    finally:
        capi.check(L.fz_gemm_set_tma_stores(1))
    assert_bits_equal(outs[0], outs[1], "tma vs thread stores")
    c = outs[0].reshape(batch, M, ldc)
    assert np.all(c[..., N:] == 7.0)


@pytest.mark.parametrize("tA,tB", [(False, True), (True, False)])
def test_gemm_tile_schedules_agree(capi, tA, tB):
    """The single-CTA and CTA-pair schedules, forced through fz_gemm_set_tiles, give the
    same product (bit for bit here: no K split, same chunk order)."""
    L = capi.lib()
    rng = np.random.default_rng(77)
    M, N, K = 1024, 768, 256  # one promotion chunk: never split over K
    A = rng.standard_normal((1, K, M) if tA else (1, M, K)).astype(np.float32)
    B = rng.standard_normal((1, N, K) if tB else (1, K, N)).astype(np.float32)
    outs = []
    try:
        for mode in (1, 2):  # FZ_GEMM_TILES_SINGLE, FZ_GEMM_TILES_PAIR
            capi.check(L.fz_gemm_set_tiles(mode))
            outs.append(_gemm(capi, A, B, tA, tB))
    finally:
        capi.check(L.fz_gemm_set_tiles(0))
    assert_bits_equal(outs[1], outs[0], "pair vs single")
    assert L.fz_gemm_set_tiles(7) == 1


@pytest.mark.parametrize("M,N,K", [(256, 256, 65536), (4096, 16, 8192)])
def test_gemm_3xtf32_long_k(capi, port, M, N, K):
    """The weight-gradient shapes of the MLP step (K = batch rows) hold 1e-5 too."""
    s = 1.0 / np.sqrt(K)
    A = (RNG.standard_normal((1, K, M)) * s).astype(np.float32)  # given transposed, as x^T
    B = (RNG.standard_normal((1, K, N)) * s).astype(np.float32)
    got = _gemm(capi, A, B, True, False)
    # the oracle's double-accumulation product, via float64 BLAS for speed at this K
    want = (A[0].astype(np.float64).T @ B[0].astype(np.float64))[None]
    err = np.linalg.norm((got - want).ravel()) / np.linalg.norm(want.ravel())
    assert err <= 1e-5, err


def tf32_lo_reference(x):
    """x - hi (hi: x with its 13 low mantissa bits cleared; exact in fp32), rounded to
    the nearest TF32 value, ties to even; non-finite remainders kept."""
    x = np.asarray(x, np.float32)
    hi = (x.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
    with np.errstate(invalid="ignore"):
        r = (x - hi).astype(np.float32)
    u = r.view(np.uint32).astype(np.uint64)
    finite = (u & 0x7F800000) != 0x7F800000
    rn = ((u + 0xFFF + ((u >> 13) & 1)) & 0xFFFFE000) & 0xFFFFFFFF
    return np.where(finite, rn, u).astype(np.uint32).view(np.float32)


def test_tf32_lo_plane_bits(capi):
    """fz_tf32_lo: the remainder x - hi rounded to the nearest TF32 value (ties to even,
    including carries into the exponent), any length. The remainder is below 2^(e-10)
    for x in [2^e, 2^(e+1)), so rounding it to 11 significant bits errs by at most
    2^(e-22): hi + lo is within 2^-22 of x, relatively, or within half the TF32 spacing
    of subnormals (2^-137) where the remainder is subnormal (|x| below about 2^-114)."""
    for n in [1, 3, 4, 1027, (1 << 20) + 5]:
        x = (RNG.standard_normal(n) * 10.0 ** RNG.integers(-30, 30, n)).astype(np.float32)
        if n > 8:
            # x in [2048, 4096) has hi = x rounded down to a multiple of 2, so these
            # remainders are 1 + 2^-11 (a tie, to even: 1), 1 + 3 * 2^-11 (a tie, to
            # even: 1 + 2^-9), 1 + 2^-12 (below a tie), its negative, and 2 - 2^-11
            # (rounds up into the next binade: 2)
            x[:5] = np.array([2049 + 2.0 ** -11, 2049 + 3 * 2.0 ** -11, 2049 + 2.0 ** -12,
                              -(2049 + 3 * 2.0 ** -11), 2050 - 2.0 ** -11], np.float32)
        dx, dl = capi.DeviceArray.from_numpy(x), capi.DeviceArray((n,))
        capi.check(capi.lib().fz_tf32_lo(dl.ptr, dx.ptr, n, None))
        lo = dl.numpy()
        assert_bits_equal(lo, tf32_lo_reference(x), f"tf32 lo n={n}")
        hi = (x.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
        err = np.abs(hi.astype(np.float64) + lo - x.astype(np.float64))
        assert np.all(err <= np.maximum(np.abs(x.astype(np.float64)) * 2.0 ** -22, 2.0 ** -137))


@pytest.mark.parametrize("tA,tB", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("batch,M,N,K", [(1, 300, 520, 260), (2, 128, 256, 1024)])
def test_gemm_split_planes_match_internal_split(capi, batch, M, N, K, tA, tB):
    """fz_gemm_f32_split with caller-supplied lo planes gives fz_gemm_f32's bits."""
    L = capi.lib()
    A = RNG.standard_normal((batch, K, M) if tA else (batch, M, K)).astype(np.float32)
    B = RNG.standard_normal((batch, N, K) if tB else (batch, K, N)).astype(np.float32)
    want = _gemm(capi, A, B, tA, tB)
    da, db, dc = capi.DeviceArray.from_numpy(A), capi.DeviceArray.from_numpy(B), capi.DeviceArray((batch, M, N))
    la, lb = capi.DeviceArray(A.shape), capi.DeviceArray(B.shape)
    capi.check(L.fz_tf32_lo(la.ptr, da.ptr, A.size, None))
    capi.check(L.fz_tf32_lo(lb.ptr, db.ptr, B.size, None))
    capi.check(L.fz_gemm_f32_split(batch, M, N, K, da.ptr, la.ptr, A.shape[2], A.shape[1] * A.shape[2],
                                   int(tA), db.ptr, lb.ptr, B.shape[2], B.shape[1] * B.shape[2], int(tB),
                                   dc.ptr, N, M * N, None))
    capi.check(L.fz_kernel_status())
    assert_bits_equal(dc.numpy(), want, "split planes")


def _program(nodes, nleaves, outs):
    pg = C.pointer(C.c_char())  # placeholder to keep ctypes import used
    del pg
    from nova_b200.capi import Program

    p = Program()
    p.num_nodes = len(nodes)
    p.num_leaves = nleaves
    p.num_outputs = len(outs)
    for i, o in enumerate(outs):
        p.out_node[i] = o
    for i, (kind, op, s0, s1, imm) in enumerate(nodes):
        p.nodes[i].kind, p.nodes[i].op, p.nodes[i].src0, p.nodes[i].src1, p.nodes[i].imm = kind, op, s0, s1, imm
    return p


def test_fused_bias_relu(capi, port):
    """relu(x + b) with a row-broadcast bias, as one fused pass."""
    A = capi
    x = RNG.standard_normal((257, 1024)).astype(np.float32)
    b = RNG.uniform(-0.1, 0.1, (1024,)).astype(np.float32)
    prog = _program([(A.NODE_BINARY, A.BINOPS["add"], -1, -2, 0.0),
                     (A.NODE_CONST, 0, 0, 0, 0.0),
                     (A.NODE_BINARY, A.BINOPS["maximum"], 0, 1, 0.0)], 2, [2])
    plan = A.make_plan(x.shape, [x.shape, x.shape, b.shape])
    dx, db, do = A.DeviceArray.from_numpy(x), A.DeviceArray.from_numpy(b), A.DeviceArray(x.shape)
    outs = (C.c_void_p * 1)(do.ptr)
    leaves = (C.c_void_p * 2)(dx.ptr, db.ptr)
    A.check(A.lib().fz_fused_launch(C.byref(prog), C.byref(plan), outs, leaves, None))
    want = port.binary("maximum", port.binary("add", x, b), np.zeros((1,), np.float32))
    assert_bits_equal(do.numpy(), want, "fused relu(x+b)")


def test_fused_value_and_tf32_remainder(capi):
    """relu(x + b) and its TF32 remainder plane as two outputs of one program, the form
    a pending GEMM operand is lowered in."""
    A = capi
    x = RNG.standard_normal((300, 2048)).astype(np.float32)
    b = RNG.uniform(-0.1, 0.1, (2048,)).astype(np.float32)
    prog = _program([(A.NODE_BINARY, A.BINOPS["add"], -1, -2, 0.0),
                     (A.NODE_CONST, 0, 0, 0, 0.0),
                     (A.NODE_BINARY, A.BINOPS["maximum"], 0, 1, 0.0),
                     (A.NODE_UNARY, A.UNOPS["tf32_lo"], 2, 0, 0.0)], 2, [2, 3])
    plan = A.make_plan(x.shape, [x.shape, x.shape, x.shape, b.shape])
    dx, db = A.DeviceArray.from_numpy(x), A.DeviceArray.from_numpy(b)
    dv, dl = A.DeviceArray(x.shape), A.DeviceArray(x.shape)
    outs = (C.c_void_p * 2)(dv.ptr, dl.ptr)
    leaves = (C.c_void_p * 2)(dx.ptr, db.ptr)
    A.check(A.lib().fz_fused_launch(C.byref(prog), C.byref(plan), outs, leaves, None))
    v = np.maximum((x + b).astype(np.float32), np.float32(0))
    assert_bits_equal(dv.numpy(), v, "value")
    assert_bits_equal(dl.numpy(), tf32_lo_reference(v), "remainder")


def test_fused_divide_backward_two_outputs(capi, port):
    """gx = g/y and gy = ((0 - g) * x) / (y * y) in one pass (Divide backward)."""
    A = capi
    shp = (33, 130)
    g = RNG.uniform(-1, 1, shp).astype(np.float32)
    x = RNG.uniform(-1, 1, shp).astype(np.float32)
    y = RNG.uniform(0.5, 2, shp).astype(np.float32)
    B = A.BINOPS
    nodes = [(A.NODE_BINARY, B["div"], -1, -3, 0.0),     # 0: g / y
             (A.NODE_CONST, 0, 0, 0, 0.0),               # 1: 0
             (A.NODE_BINARY, B["sub"], 1, -1, 0.0),      # 2: 0 - g
             (A.NODE_BINARY, B["mul"], 2, -2, 0.0),      # 3: (0-g) * x
             (A.NODE_BINARY, B["mul"], -3, -3, 0.0),     # 4: y * y
             (A.NODE_BINARY, B["div"], 3, 4, 0.0)]       # 5
    prog = _program(nodes, 3, [0, 5])
    plan = A.make_plan(shp, [shp, shp, shp, shp, shp])
    dg, dx, dy = (A.DeviceArray.from_numpy(v) for v in (g, x, y))
    o1, o2 = A.DeviceArray(shp), A.DeviceArray(shp)
    outs = (C.c_void_p * 2)(o1.ptr, o2.ptr)
    leaves = (C.c_void_p * 3)(dg.ptr, dx.ptr, dy.ptr)
    A.check(A.lib().fz_fused_launch(C.byref(prog), C.byref(plan), outs, leaves, None))
    z = np.zeros(shp, np.float32)
    want_gx = port.binary("div", g, y)
    want_gy = port.binary("div", port.binary("mul", port.binary("sub", z, g), x), port.binary("mul", y, y))
    assert_bits_equal(o1.numpy(), want_gx, "gx")
    assert_bits_equal(o2.numpy(), want_gy, "gy")


def test_sub_inplace_and_fill(capi):
    x = RNG.standard_normal(1001).astype(np.float32)
    y = RNG.standard_normal(1001).astype(np.float32)
    dx, dy = capi.DeviceArray.from_numpy(x), capi.DeviceArray.from_numpy(y)
    capi.check(capi.lib().fz_sub_inplace(dx.ptr, dy.ptr, 1001, None))
    assert_bits_equal(dx.numpy(), x - y)
    capi.check(capi.lib().fz_fill_f32(dx.ptr, C.c_float(1.5), 1001, None))
    assert np.all(dx.numpy() == 1.5)
