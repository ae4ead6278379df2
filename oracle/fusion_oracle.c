/* CPU restatement of the Fusion reference algorithms on the hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the oracle: the parity tests, smoke() and the
 * bench's CPU-baseline leg use it as the checker. The nova_b200 product never links,
 * loads or calls it. Its results are pinned against the reference's own outputs
 * (tests/golden/*.npz, produced by the reference pybind module built from the
 * reference sources by oracle/Makefile) and against the reference's unit-test
 * known-answer vectors.
 *
 * Conventions: fp32 tensors, C-contiguous, shapes as int64 arrays. Every function
 * cites the reference file:line whose behaviour it restates.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

enum { ORC_ADD = 0, ORC_SUB, ORC_MUL, ORC_DIV, ORC_POW, ORC_MAX, ORC_GT, ORC_GE };
enum { ORC_EXP = 0, ORC_LOG, ORC_SQRT };

#define ORC_MAXD 16

/* Scalar functors: fusion/src/Fusion/cpu/simd/SimdTags.hpp:7-77.
 * MaximumSIMD is `a > b ? a : b` (so relu(NaN) = b and relu(-0) = b);
 * comparisons return 1.0f / 0.0f. PowerSIMD is std::pow on floats (powf). */
static float orc_apply(int op, float a, float b) {
  switch (op) {
    case ORC_ADD: return a + b;
    case ORC_SUB: return a - b;
    case ORC_MUL: return a * b;
    case ORC_DIV: return a / b;
    case ORC_POW: return powf(a, b);
    case ORC_MAX: return a > b ? a : b;
    case ORC_GT: return a > b ? 1.0f : 0.0f;
    case ORC_GE: return a >= b ? 1.0f : 0.0f;
  }
  return 0.0f;
}

/* Right-aligned broadcast of two shapes (TensorPlan.cpp:40-48, 67-126).
 * Returns output rank, or -1 on a dimension mismatch. */
int orc_broadcast_shape(const int64_t *as, int an, const int64_t *bs, int bn, int64_t *out) {
  int n = an > bn ? an : bn;
  for (int d = 0; d < n; ++d) {
    int ia = d - (n - an), ib = d - (n - bn);
    int64_t da = ia >= 0 ? as[ia] : 1, db = ib >= 0 ? bs[ib] : 1;
    if (da == db || db == 1) out[d] = da;
    else if (da == 1) out[d] = db;
    else return -1;
  }
  return n;
}

/* fusion::math::{add,sub,mul,div,pow,maximum,greater,greater_equal}
 * (ops/Ewise.hpp:17-55, ops/Comparison.hpp:17-40).
 *
 * Fast path when the two shapes are equal (PlanMeta.hpp:96-108): elementwise.
 * Otherwise the broadcast walk of TensorIter.hpp:122-177 over the plan of
 * PlanMeta.hpp:109-120, whose innermost loop is the last output dim. In that loop
 * simd_traits dispatches on which operand has byte stride 0 (SimdTraits.hpp:26-148):
 * when b's stride is 0 it computes op(a[i], b); when only a's stride is 0 it calls the
 * scalar kernel with the operands exchanged, i.e. op(b[i], a) — so for non-commutative
 * ops the result is op(b, a). a has stride 0 in the last dim exactly when
 * a's last dim is 1 (or absent) and the output's last dim is > 1. */
int orc_binary(int op, float *out, const int64_t *oshape, int on, const float *a,
               const int64_t *as, int an, const float *b, const int64_t *bs, int bn) {
  int same = (an == bn);
  for (int d = 0; same && d < an; ++d) same = (as[d] == bs[d]);
  int64_t total = 1;
  for (int d = 0; d < on; ++d) total *= oshape[d];
  if (same) {
    for (int64_t i = 0; i < total; ++i) out[i] = orc_apply(op, a[i], b[i]);
    return 0;
  }
  if (on > ORC_MAXD) return -1;
  int64_t sa[ORC_MAXD], sb[ORC_MAXD];
  /* element strides of a/b seen from the output index space (0 on broadcast dims) */
  int64_t ra = 1, rb = 1;
  for (int d = on - 1; d >= 0; --d) {
    int ia = d - (on - an), ib = d - (on - bn);
    if (ia >= 0) {
      sa[d] = (as[ia] == 1 && oshape[d] > 1) ? 0 : ra;
      ra *= as[ia];
    } else sa[d] = 0;
    if (ib >= 0) {
      sb[d] = (bs[ib] == 1 && oshape[d] > 1) ? 0 : rb;
      rb *= bs[ib];
    } else sb[d] = 0;
  }
  int swap = (sa[on - 1] == 0 && sb[on - 1] != 0);
  int64_t idx[ORC_MAXD];
  memset(idx, 0, sizeof(idx));
  for (int64_t i = 0; i < total; ++i) {
    int64_t oa = 0, ob = 0;
    for (int d = 0; d < on; ++d) { oa += idx[d] * sa[d]; ob += idx[d] * sb[d]; }
    out[i] = swap ? orc_apply(op, b[ob], a[oa]) : orc_apply(op, a[oa], b[ob]);
    for (int d = on - 1; d >= 0; --d) {
      if (++idx[d] < oshape[d]) break;
      idx[d] = 0;
    }
  }
  return 0;
}

/* fusion::math::{exp,log,sqrt} (ops/Transcendental.hpp:14-33) -> std::exp/log/sqrt
 * on floats (cpu/simd/VecFallback.hpp:41-60). */
void orc_unary(int op, float *out, const float *a, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    float x = a[i];
    out[i] = op == ORC_EXP ? expf(x) : op == ORC_LOG ? logf(x) : sqrtf(x);
  }
}

/* fusion::math::sum over one axis (ops/Reduce.hpp:18-25, TensorIter.hpp:251-297):
 * the output is zero-filled and then accumulated in fp32 in index order along the
 * axis. axis < 0 means the global reduction (PlanMeta.hpp:152-158). mean divides
 * the fp32 sum by (float)reduce_len (Reduce.hpp:27-36). Max is not in the reference;
 * it is the exact maximum (NaN-propagating) over the same index space. */
void orc_reduce(int op, float *out, const float *in, const int64_t *shape, int nd, int axis) {
  int64_t outer = 1, len, inner = 1;
  if (axis < 0) {
    len = 1;
    for (int d = 0; d < nd; ++d) len *= shape[d];
  } else {
    for (int d = 0; d < axis; ++d) outer *= shape[d];
    len = shape[axis];
    for (int d = axis + 1; d < nd; ++d) inner *= shape[d];
  }
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t j = 0; j < inner; ++j) {
      const float *p = in + o * len * inner + j;
      float acc;
      if (op == 2) {
        /* order-independent: any NaN wins; +0 ranks above -0 */
        acc = len > 0 ? p[0] : -INFINITY;
        for (int64_t r = 1; r < len; ++r) {
          float v = p[r * inner];
          if (acc != acc) break;
          if (v != v || v > acc || (v == 0.0f && acc == 0.0f && !signbit(v) && signbit(acc)))
            acc = v;
        }
      } else {
        acc = 0.0f;
        for (int64_t r = 0; r < len; ++r) acc += p[r * inner];
        if (op == 1) acc = acc / (float)len;
      }
      out[o * inner + j] = acc;
    }
}

/* fusion::math::linalg::matmul (ops/Linalg.hpp:76-107): batched row-major NN
 * C[b] = A[b] @ B[b]. The reference calls OpenBLAS cblas_sgemm
 * (cpu/blas/backend/BlasCblas.hpp:19-39), whose fp32 summation order is the
 * library's own; this restatement accumulates in double and rounds once, so it is
 * the more accurate of the two and both are compared under a relative tolerance. */
void orc_matmul(float *c, const float *a, const float *b, int64_t batch, int64_t m,
                int64_t n, int64_t k) {
  for (int64_t bt = 0; bt < batch; ++bt) {
    const float *A = a + bt * m * k, *B = b + bt * k * n;
    float *C = c + bt * m * n;
    for (int64_t i = 0; i < m; ++i)
      for (int64_t j = 0; j < n; ++j) {
        double s = 0.0;
        for (int64_t p = 0; p < k; ++p) s += (double)A[i * k + p] * (double)B[p * n + j];
        C[i * n + j] = (float)s;
      }
  }
}

/* fusion::math::linalg::swapaxes (ops/Linalg.hpp:109-128 -> kernels/Serial.hpp:90-123):
 * materialised copy with two axes exchanged. */
void orc_swapaxes(float *out, const float *in, const int64_t *shape, int nd, int a1, int a2) {
  int64_t total = 1, ist[ORC_MAXD], ost[ORC_MAXD], oshape[ORC_MAXD], idx[ORC_MAXD];
  for (int d = 0; d < nd; ++d) { total *= shape[d]; oshape[d] = shape[d]; }
  oshape[a1] = shape[a2];
  oshape[a2] = shape[a1];
  int64_t r = 1, q = 1;
  for (int d = nd - 1; d >= 0; --d) { ist[d] = r; r *= shape[d]; ost[d] = q; q *= oshape[d]; }
  memset(idx, 0, sizeof(idx));
  for (int64_t i = 0; i < total; ++i) {
    int64_t o = 0;
    for (int d = 0; d < nd; ++d) {
      int dd = d == a1 ? a2 : d == a2 ? a1 : d;
      o += idx[d] * ost[dd];
    }
    out[o] = in[i];
    for (int d = nd - 1; d >= 0; --d) {
      if (++idx[d] < shape[d]) break;
      idx[d] = 0;
    }
  }
  (void)ist;
}

/* Philox-4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11; no reference counterpart: the
 * reference draws from std::mt19937, fusion/src/Fusion/Random.hpp:20-36). Restated
 * from the paper: ten rounds on a 128-bit counter with multipliers 0xD2511F53 and
 * 0xCD9E8D57 and a 64-bit key bumped by 0x9E3779B9 / 0xBB67AE85 between rounds.
 * Stream layout of the device generator: element i of (seed, offset) is lane
 * (offset + i) % 4 of the block at counter (offset + i) / 4; u = (bits >> 8) * 2^-24. */
static void orc_philox(uint64_t ctr, uint64_t key, uint32_t out[4]) {
  uint32_t c[4] = {(uint32_t)ctr, (uint32_t)(ctr >> 32), 0u, 0u};
  uint32_t k0 = (uint32_t)key, k1 = (uint32_t)(key >> 32);
  for (int r = 0; r < 10; ++r) {
    uint64_t p0 = (uint64_t)0xD2511F53u * c[0], p1 = (uint64_t)0xCD9E8D57u * c[2];
    uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  memcpy(out, c, sizeof(c));
}

static float orc_unit(uint32_t bits) { return (float)(bits >> 8) * 5.9604644775390625e-08f; }

/* Raw Philox-4x32-10 block for counter/key (for the published known-answer vectors). */
void orc_philox4x32_10(uint64_t ctr_lo, uint64_t ctr_hi, uint64_t key, uint32_t out[4]) {
  uint32_t c[4] = {(uint32_t)ctr_lo, (uint32_t)(ctr_lo >> 32), (uint32_t)ctr_hi, (uint32_t)(ctr_hi >> 32)};
  uint32_t k0 = (uint32_t)key, k1 = (uint32_t)(key >> 32);
  for (int r = 0; r < 10; ++r) {
    uint64_t p0 = (uint64_t)0xD2511F53u * c[0], p1 = (uint64_t)0xCD9E8D57u * c[2];
    uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0, n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    c[1] = (uint32_t)p1;
    c[3] = (uint32_t)p0;
    c[0] = n0;
    c[2] = n2;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  memcpy(out, c, sizeof(c));
}

void orc_philox_uniform(float *out, int64_t n, uint64_t seed, uint64_t offset, float lo, float hi) {
  const float span = hi - lo;
  for (int64_t i = 0; i < n; ++i) {
    uint32_t r[4];
    orc_philox((offset + (uint64_t)i) / 4, seed, r);
    float v = fmaf(span, orc_unit(r[(offset + (uint64_t)i) % 4]), lo);
    if (v >= hi) v = nextafterf(hi, lo);
    out[i] = v;
  }
}

/* Nova's Dropout, nova/src/blocks/regularisation/dropout.py:17-23: inputs * (u >= rate)
 * / (1 - rate), where Fusion's >= is > (core/RawTensor.hpp:207-209) and the mask is a
 * 1.0 / 0.0 tensor multiplied in. */
void orc_philox_dropout(float *out, const float *x, int64_t n, float rate, float keep, uint64_t seed,
                        uint64_t offset) {
  for (int64_t i = 0; i < n; ++i) {
    uint32_t r[4];
    orc_philox((offset + (uint64_t)i) / 4, seed, r);
    float m = orc_unit(r[(offset + (uint64_t)i) % 4]) > rate ? 1.0f : 0.0f;
    out[i] = (x[i] * m) / keep;
  }
}
