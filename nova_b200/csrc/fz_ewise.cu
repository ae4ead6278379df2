// Elementwise binary and unary kernels for sm_100a.
//
// A launch walks the output index space of an fz_ewise_plan. The host side first
// converts byte strides to element strides, drops size-1 dims and merges adjacent
// dims whose strides chain for every operand, so the usual cases reduce to:
//   * 1 dim, all strides 1            -> plain contiguous stream (fast path)
//   * 1 dim, one operand stride 0     -> scalar operand
//   * 2 dims [rows, cols], a [cols]   -> row broadcast (bias add)
// Plans of 1 or 2 dims with a long inner dim (>= 1024) on the 128-bit path run the
// tiled kernel (no per-element index arithmetic, U loads per thread in flight);
// the rest run the generic kernel, which maps each thread to groups of VEC=4
// consecutive elements of the innermost dim (128-bit loads/stores when every
// operand with inner stride 1 is 16-byte aligned at each row start), with a
// grid-stride loop over groups. Operands with inner stride 0 are loaded once per
// group and replicated.
#include "fz_common.cuh"
#include "fz_ewise_plan.hpp"

namespace {

using fz::EwPlan;

// Offsets of row `r` (the index over every dim but the innermost) for NOPS
// operands; NOPS is a template parameter so the offsets stay in registers.
template <int NOPS, typename IDX>
__device__ __forceinline__ void row_offsets(const EwPlan &p, IDX r, int64_t (&off)[NOPS]) {
#pragma unroll
  for (int k = 0; k < NOPS; ++k) off[k] = 0;
  for (int d = p.ndim - 2; d >= 0; --d) {
    const IDX sz = (IDX)p.size[d];
    const IDX q = r / sz;
    const int64_t i = (int64_t)(r - q * sz);
    r = q;
#pragma unroll
    for (int k = 0; k < NOPS; ++k) off[k] += i * p.stride[k][d];
  }
}

template <int VEC>
struct Vec;
template <>
struct Vec<4> {
  using T = float4;
};

__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ void st4(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }

// Generic kernel: NIN inputs (1 or 2), OP is a binop (NIN=2) or unop (NIN=1).
template <int NIN, int OP, int VEC, typename IDX>
__global__ void __launch_bounds__(256) ewise_kernel(EwPlan p, float *__restrict__ out,
                                                    const float *__restrict__ a,
                                                    const float *__restrict__ b) {
  pdl_wait();
  const int64_t inner = p.ndim ? p.size[p.ndim - 1] : 1;
  const IDX groups_per_row = (IDX)((inner + VEC - 1) / VEC);
  const IDX total = (IDX)p.rows * groups_per_row;
  const int64_t so = p.ndim ? p.stride[0][p.ndim - 1] : 0;
  const int64_t sa = p.ndim ? p.stride[1][p.ndim - 1] : 0;
  const int64_t sb = (NIN == 2 && p.ndim) ? p.stride[2][p.ndim - 1] : 0;
  const IDX step = (IDX)gridDim.x * blockDim.x;
  constexpr int NOPS = NIN + 1;
  int64_t off[NOPS];
#pragma unroll
  for (int k = 0; k < NOPS; ++k) off[k] = 0;
  for (IDX g = (IDX)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += step) {
    IDX row = g / groups_per_row;
    IDX col = (g - row * groups_per_row) * VEC;
    if (p.ndim > 1) row_offsets<NOPS, IDX>(p, row, off);
    if constexpr (VEC == 4) {
      if ((int64_t)col + 4 <= inner) {
        float4 x, y = make_float4(0.f, 0.f, 0.f, 0.f);
        const float *pa = a + off[1] + (int64_t)col * sa;
        if (sa) x = ld4(pa);
        else x = make_float4(*pa, *pa, *pa, *pa);
        if constexpr (NIN == 2) {
          const float *pb = b + off[NIN] + (int64_t)col * sb;
          if (sb) y = ld4(pb);
          else y = make_float4(*pb, *pb, *pb, *pb);
        }
        float4 r;
        if constexpr (NIN == 2) {
          r.x = fzd::binop_t<OP>(x.x, y.x);
          r.y = fzd::binop_t<OP>(x.y, y.y);
          r.z = fzd::binop_t<OP>(x.z, y.z);
          r.w = fzd::binop_t<OP>(x.w, y.w);
        } else {
          r.x = fzd::unop_t<OP>(x.x);
          r.y = fzd::unop_t<OP>(x.y);
          r.z = fzd::unop_t<OP>(x.z);
          r.w = fzd::unop_t<OP>(x.w);
        }
        st4(out + off[0] + (int64_t)col * so, r);
        continue;
      }
    }
    for (int v = 0; v < VEC && (int64_t)col + v < inner; ++v) {
      int64_t c = (int64_t)col + v;
      float x = a[off[1] + c * sa];
      float r;
      if constexpr (NIN == 2) r = fzd::binop_t<OP>(x, b[off[NIN] + c * sb]);
      else r = fzd::unop_t<OP>(x);
      out[off[0] + c * so] = r;
    }
  }
}

// Plans of at most 2 dims ([rows, inner], inner >= 1024) on the 128-bit path: the
// index space is cut into tiles of one row x 1024*U columns and a CTA walks tiles
// blockIdx.x, +gridDim.x, ... (one division per tile, none per element). Each thread
// loads its U float4 groups of a tile (256 groups apart, so every warp access is
// one contiguous 512-byte run) before computing and storing any, keeping U loads
// per operand in flight. Inner strides are 0 (broadcast) or 1.
template <int NIN, int OP, int U>
__global__ void __launch_bounds__(256) ewise_tiles_kernel(EwPlan p, float *__restrict__ out,
                                                          const float *__restrict__ a,
                                                          const float *__restrict__ b) {
  pdl_wait();
  constexpr int64_t TW = 1024 * U;
  const int64_t inner = p.size[p.ndim - 1];
  const int64_t ctiles = (inner + TW - 1) / TW;
  const int64_t total = p.rows * ctiles;
  const bool va = p.stride[1][p.ndim - 1] != 0;
  const bool vb = NIN == 2 && p.stride[2][p.ndim - 1] != 0;
  const int64_t ro = p.ndim > 1 ? p.stride[0][0] : 0, ra = p.ndim > 1 ? p.stride[1][0] : 0;
  const int64_t rb = (NIN == 2 && p.ndim > 1) ? p.stride[2][0] : 0;
  for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
    const int64_t row = t / ctiles;
    const int64_t c0 = (t - row * ctiles) * TW + threadIdx.x * 4;
    const float *pa = a + row * ra;
    const float *pb = NIN == 2 ? b + row * rb : nullptr;
    float *po = out + row * ro;
    float4 x[U], y[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int64_t c = c0 + j * 1024;
      if (c + 4 <= inner) {
        x[j] = va ? ld4(pa + c) : make_float4(*pa, *pa, *pa, *pa);
        if constexpr (NIN == 2) y[j] = vb ? ld4(pb + c) : make_float4(*pb, *pb, *pb, *pb);
      }
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int64_t c = c0 + j * 1024;
      if (c + 4 <= inner) {
        float4 r;
        if constexpr (NIN == 2) {
          r.x = fzd::binop_t<OP>(x[j].x, y[j].x);
          r.y = fzd::binop_t<OP>(x[j].y, y[j].y);
          r.z = fzd::binop_t<OP>(x[j].z, y[j].z);
          r.w = fzd::binop_t<OP>(x[j].w, y[j].w);
        } else {
          r.x = fzd::unop_t<OP>(x[j].x);
          r.y = fzd::unop_t<OP>(x[j].y);
          r.z = fzd::unop_t<OP>(x[j].z);
          r.w = fzd::unop_t<OP>(x[j].w);
        }
        st4(po + c, r);
      } else {
        for (int64_t e = c; e < inner; ++e) {
          const float xa = pa[va ? e : 0];
          if constexpr (NIN == 2) po[e] = fzd::binop_t<OP>(xa, pb[vb ? e : 0]);
          else po[e] = fzd::unop_t<OP>(xa);
        }
      }
    }
  }
}

template <int NIN, int OP>
int launch_op(const EwPlan &p, float *out, const float *a, const float *b, cudaStream_t s) {
  int64_t inner = p.ndim ? p.size[p.ndim - 1] : 1;
  int64_t total = p.rows * inner;
  if (total == 0) return FZ_OK;
  // 128-bit path: every operand walking the inner dim with stride 1 must start
  // each row on a 16-byte boundary; broadcast (stride 0) operands are free.
  bool vec = p.ndim >= 1;
  const float *base[3] = {out, a, b};
  for (int k = 0; vec && k < p.nops; ++k) {
    int64_t si = p.stride[k][p.ndim - 1];
    if (si == 0) continue;
    if (si != 1 || ((uintptr_t)base[k] & 15)) vec = false;
    for (int d = 0; vec && d + 1 < p.ndim; ++d)
      if (p.stride[k][d] % 4) vec = false;
  }
  if (vec && p.ndim <= 2 && inner >= 1024 && p.stride[0][p.ndim - 1] == 1) {
    // one input: 8 float4 per thread in flight; two inputs: 4 of each
    const int U = (NIN == 1 && inner >= 8192) ? 8 : inner >= 4096 ? 4 : inner >= 2048 ? 2 : 1;
    const int64_t tiles = p.rows * ((inner + 1024 * U - 1) / (1024 * U));
    const unsigned grid = (unsigned)(tiles < (int64_t)fz::num_sms() * 8 ? tiles : fz::num_sms() * 8);
    cudaError_t e;
    if (U == 8) e = fz::launch_pdl(ewise_tiles_kernel<NIN, OP, (NIN == 1 ? 8 : 4)>, dim3(grid), dim3(256), 0, s, p, out, a, b);
    else if (U == 4) e = fz::launch_pdl(ewise_tiles_kernel<NIN, OP, 4>, dim3(grid), dim3(256), 0, s, p, out, a, b);
    else if (U == 2) e = fz::launch_pdl(ewise_tiles_kernel<NIN, OP, 2>, dim3(grid), dim3(256), 0, s, p, out, a, b);
    else e = fz::launch_pdl(ewise_tiles_kernel<NIN, OP, 1>, dim3(grid), dim3(256), 0, s, p, out, a, b);
    if (e != cudaSuccess) return fz::cuda_fail(e, "ewise_tiles_kernel launch", __FILE__, __LINE__);
    FZ_CHECK_LAUNCH();
    return FZ_OK;
  }
  int V = vec ? 4 : 1;
  int64_t groups = p.rows * ((inner + V - 1) / V);
  bool i64 = groups > (int64_t)0x7fffffff - (int64_t)fz::num_sms() * 2048;
  unsigned grid = fz::grid_for(groups, 256 * 2, 8);
  cudaError_t e;
  if (vec) {
    if (i64) e = fz::launch_pdl(ewise_kernel<NIN, OP, 4, int64_t>, dim3(grid), dim3(256), 0, s, p, out, a, b);
    else e = fz::launch_pdl(ewise_kernel<NIN, OP, 4, int32_t>, dim3(grid), dim3(256), 0, s, p, out, a, b);
  } else {
    if (i64) e = fz::launch_pdl(ewise_kernel<NIN, OP, 1, int64_t>, dim3(grid), dim3(256), 0, s, p, out, a, b);
    else e = fz::launch_pdl(ewise_kernel<NIN, OP, 1, int32_t>, dim3(grid), dim3(256), 0, s, p, out, a, b);
  }
  if (e != cudaSuccess) return fz::cuda_fail(e, "ewise_kernel launch", __FILE__, __LINE__);
  FZ_CHECK_LAUNCH();
  return FZ_OK;
}

int dispatch_binary(int op, const EwPlan &p, float *out, const float *a, const float *b,
                    cudaStream_t s) {
  switch (op) {
    case FZ_ADD: return launch_op<2, FZ_ADD>(p, out, a, b, s);
    case FZ_SUB: return launch_op<2, FZ_SUB>(p, out, a, b, s);
    case FZ_MUL: return launch_op<2, FZ_MUL>(p, out, a, b, s);
    case FZ_DIV: return launch_op<2, FZ_DIV>(p, out, a, b, s);
    case FZ_POW: return launch_op<2, FZ_POW>(p, out, a, b, s);
    case FZ_MAXIMUM: return launch_op<2, FZ_MAXIMUM>(p, out, a, b, s);
    case FZ_GT: return launch_op<2, FZ_GT>(p, out, a, b, s);
    case FZ_GE: return launch_op<2, FZ_GE>(p, out, a, b, s);
  }
  return fz::fail(FZ_ERR_INVALID, "fz_ewise_binary: unknown op " + std::to_string(op));
}

int dispatch_unary(int op, const EwPlan &p, float *out, const float *a, cudaStream_t s) {
  switch (op) {
    case FZ_EXP: return launch_op<1, FZ_EXP>(p, out, a, nullptr, s);
    case FZ_LOG: return launch_op<1, FZ_LOG>(p, out, a, nullptr, s);
    case FZ_SQRT: return launch_op<1, FZ_SQRT>(p, out, a, nullptr, s);
    case FZ_COPY: return launch_op<1, FZ_COPY>(p, out, a, nullptr, s);
    case FZ_TF32_LO: return launch_op<1, FZ_TF32_LO>(p, out, a, nullptr, s);
  }
  return fz::fail(FZ_ERR_INVALID, "fz_ewise_unary: unknown op " + std::to_string(op));
}

}  // namespace

extern "C" {

int fz_ewise_binary(int op, const fz_ewise_plan *plan, float *out, const float *a,
                    const float *b, void *stream) {
  FZ_REQUIRE(plan, "fz_ewise_binary: null plan");
  EwPlan p;
  int rc = fz::normalize_plan(*plan, 3, p);
  if (rc) return rc;
  if (p.rows == 0) return FZ_OK;
  FZ_REQUIRE(out && a && b, "fz_ewise_binary: null argument");
  return dispatch_binary(op, p, out, a, b, fz::resolve(stream));
}

int fz_ewise_binary_contig(int op, int64_t n, float *out, const float *a, const float *b,
                           void *stream) {
  FZ_REQUIRE(n >= 0, "fz_ewise_binary_contig: negative length");
  if (n == 0) return FZ_OK;
  FZ_REQUIRE(out && a && b, "fz_ewise_binary_contig: null argument");
  EwPlan p = fz::contiguous_plan(n, 3);
  return dispatch_binary(op, p, out, a, b, fz::resolve(stream));
}

int fz_ewise_unary(int op, const fz_ewise_plan *plan, float *out, const float *a,
                   void *stream) {
  FZ_REQUIRE(plan, "fz_ewise_unary: null plan");
  EwPlan p;
  int rc = fz::normalize_plan(*plan, 2, p);
  if (rc) return rc;
  if (p.rows == 0) return FZ_OK;
  FZ_REQUIRE(out && a, "fz_ewise_unary: null argument");
  return dispatch_unary(op, p, out, a, fz::resolve(stream));
}

}  // extern "C"
