// Single-axis reductions (sum / mean / max) for sm_100a.
//
// The input is viewed as a contiguous [outer, len, inner] array and reduced over
// `len`. Two shapes of work:
//   * inner == 1 (reducing the last axis, or everything): rows of `len`
//     contiguous floats. Short rows are reduced by groups of G lanes of a warp
//     (G = 1..32, shuffles within the group); long rows by whole CTAs with
//     128-bit loads, warp shuffles and a shared-memory tree, and when there are
//     too few rows to fill 148 SMs a row is split over several CTAs.
//   * inner > 1 (reducing a leading axis): each thread owns 4 adjacent columns
//     (one float4 per row read, fully coalesced across the warp) and walks `len`;
//     when outer*inner/4 threads cannot fill the GPU, `len` is split: over the 8
//     warps of a CTA and the up to 8 CTAs of a thread-block cluster, folded in a
//     fixed order through shared and distributed shared memory in the same launch
//     (enough columns), or into chunks whose partials a second pass reduces.
// Split row work writes fp32 partials to stream-ordered scratch and a second pass
// reduces them. No atomics: results do not depend on scheduling.
// mean = sum / (float)len with an IEEE division, as fusion::math::mean does
// (fusion/src/Fusion/ops/Reduce.hpp:27-36).
#include <cooperative_groups.h>

#include <mutex>

#include "fz_common.cuh"

namespace {

__device__ __forceinline__ float max_nan(float a, float b) {
  // NaN propagates (as the canonical NaN); otherwise the larger value, +0 ranking
  // above -0: one max.NaN.f32. Order independent, so a tree and a sequential scan
  // agree bit for bit.
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

template <int OP>
struct Red {
  __device__ __forceinline__ static float init() { return OP == FZ_RMAX ? -INFINITY : 0.0f; }
  __device__ __forceinline__ static float op(float a, float b) {
    return OP == FZ_RMAX ? max_nan(a, b) : __fadd_rn(a, b);
  }
};

template <int OP>
__device__ __forceinline__ float finish(float v, int64_t len, bool final) {
  if (OP == FZ_RMEAN && final) return __fdiv_rn(v, (float)len);
  return v;
}

template <int OP, int G>
__device__ __forceinline__ float group_reduce(float v) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) v = Red<OP>::op(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Rows of `len` floats (row stride `ld`), G lanes per row, R consecutive rows per
// group at a time: each lane strides its rows by G (vectorised by 4 when the rows
// are 16-byte aligned) and issues the loads of all R rows before reducing any, so
// short rows still keep R loads per lane in flight.
template <int OP, int G, int R>
__global__ void __launch_bounds__(256) rows_group_kernel(const float *__restrict__ in,
                                                         float *__restrict__ out, int64_t rows,
                                                         int64_t len, int64_t ld,
                                                         int64_t div_len, int final, int vec) {
  pdl_wait();
  const int lane = threadIdx.x % G;
  const int64_t groups_total = (int64_t)gridDim.x * (blockDim.x / G);
  const int64_t nv = vec ? len >> 2 : 0;
  for (int64_t r0 = ((int64_t)blockIdx.x * (blockDim.x / G) + threadIdx.x / G) * R; r0 < rows;
       r0 += groups_total * R) {
    float acc[R];
#pragma unroll
    for (int i = 0; i < R; ++i) acc[i] = Red<OP>::init();
#pragma unroll 4
    for (int64_t j = lane; j < nv; j += G) {
      float4 q[R];
#pragma unroll
      for (int i = 0; i < R; ++i)
        if (r0 + i < rows) q[i] = reinterpret_cast<const float4 *>(in + (r0 + i) * ld)[j];
#pragma unroll
      for (int i = 0; i < R; ++i)
        if (r0 + i < rows)
          acc[i] = Red<OP>::op(acc[i], Red<OP>::op(Red<OP>::op(q[i].x, q[i].y),
                                                   Red<OP>::op(q[i].z, q[i].w)));
    }
#pragma unroll
    for (int i = 0; i < R; ++i) {
      if (r0 + i >= rows) break;
      const float *p = in + (r0 + i) * ld;
      for (int64_t j = (nv << 2) + lane; j < len; j += G) acc[i] = Red<OP>::op(acc[i], p[j]);
    }
#pragma unroll
    for (int i = 0; i < R; ++i) acc[i] = group_reduce<OP, G>(acc[i]);
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < R; ++i)
        if (r0 + i < rows) out[r0 + i] = finish<OP>(acc[i], div_len, final);
    }
  }
}

// Long rows: one CTA per (row, split). Split s covers [s*chunk, min(len, (s+1)*chunk)).
// out has `splits` entries per row.
template <int OP>
__global__ void __launch_bounds__(512) rows_block_kernel(const float *__restrict__ in,
                                                         float *__restrict__ out, int64_t rows,
                                                         int64_t len, int64_t ld, int64_t splits,
                                                         int64_t chunk, int64_t div_len,
                                                         int final, int vec) {
  pdl_wait();
  __shared__ float warp_part[32];
  const int64_t items = rows * splits;
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    const int64_t r = it / splits, s = it - r * splits;
    const int64_t beg = s * chunk;
    const int64_t end = beg + chunk < len ? beg + chunk : len;
    const float *p = in + r * ld;
    float acc = Red<OP>::init();
    if (vec) {  // chunk is a multiple of 4 and rows are 16-byte aligned
      const float4 *p4 = reinterpret_cast<const float4 *>(p + beg);
      int64_t nv = (end - beg) >> 2;
      int64_t j = threadIdx.x;
      for (; j + 3 * (int64_t)blockDim.x < nv; j += 4 * (int64_t)blockDim.x) {
        float4 q0 = p4[j], q1 = p4[j + blockDim.x], q2 = p4[j + 2 * blockDim.x],
               q3 = p4[j + 3 * blockDim.x];
        float t0 = Red<OP>::op(Red<OP>::op(q0.x, q0.y), Red<OP>::op(q0.z, q0.w));
        float t1 = Red<OP>::op(Red<OP>::op(q1.x, q1.y), Red<OP>::op(q1.z, q1.w));
        float t2 = Red<OP>::op(Red<OP>::op(q2.x, q2.y), Red<OP>::op(q2.z, q2.w));
        float t3 = Red<OP>::op(Red<OP>::op(q3.x, q3.y), Red<OP>::op(q3.z, q3.w));
        acc = Red<OP>::op(acc, Red<OP>::op(Red<OP>::op(t0, t1), Red<OP>::op(t2, t3)));
      }
      for (; j < nv; j += blockDim.x) {
        float4 q = p4[j];
        acc = Red<OP>::op(acc, Red<OP>::op(Red<OP>::op(q.x, q.y), Red<OP>::op(q.z, q.w)));
      }
      for (int64_t k = beg + (nv << 2) + threadIdx.x; k < end; k += blockDim.x)
        acc = Red<OP>::op(acc, p[k]);
    } else {
      for (int64_t k = beg + threadIdx.x; k < end; k += blockDim.x) acc = Red<OP>::op(acc, p[k]);
    }
    acc = group_reduce<OP, 32>(acc);
    const int w = threadIdx.x / 32, nw = blockDim.x / 32;
    if ((threadIdx.x & 31) == 0) warp_part[w] = acc;
    __syncthreads();
    if (w == 0) {
      float v = (int)threadIdx.x < nw ? warp_part[threadIdx.x] : Red<OP>::init();
      v = group_reduce<OP, 32>(v);
      if (threadIdx.x == 0) out[it] = finish<OP>(v, div_len, final);
    }
    __syncthreads();
  }
}

// Columns: in is [outer, len, inner]; each thread owns V adjacent columns of one
// outer slice and a chunk of len, with 4 rows in flight. Unsplit it writes
// out[o*inner + c]; split, it writes partials column-major,
// out[(o*inner + c) * splits + s], so the second pass is a row reduction.
template <int OP, int V>
__global__ void __launch_bounds__(256) cols_kernel(const float *__restrict__ in,
                                                   float *__restrict__ out, int64_t outer,
                                                   int64_t len, int64_t inner, int64_t splits,
                                                   int64_t chunk, int64_t div_len) {
  pdl_wait();
  const int64_t cgroups = (inner + V - 1) / V;
  const int64_t items = splits * outer * cgroups;
  const bool split = splits > 1;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < items;
       t += (int64_t)gridDim.x * blockDim.x) {
    int64_t cg = t % cgroups;
    int64_t rest = t / cgroups;
    int64_t o = rest % outer;
    int64_t sp = rest / outer;
    int64_t c = cg * V;
    int64_t beg = sp * chunk, end = beg + chunk < len ? beg + chunk : len;
    const float *p = in + (o * len) * inner + c;
    const int64_t col = o * inner + c;
    if (V == 4 && c + 4 <= inner) {
      float a0 = Red<OP>::init(), a1 = a0, a2 = a0, a3 = a0;
      int64_t r = beg;
      for (; r + 3 < end; r += 4) {
        float4 x0 = *reinterpret_cast<const float4 *>(p + r * inner);
        float4 x1 = *reinterpret_cast<const float4 *>(p + (r + 1) * inner);
        float4 x2 = *reinterpret_cast<const float4 *>(p + (r + 2) * inner);
        float4 x3 = *reinterpret_cast<const float4 *>(p + (r + 3) * inner);
        a0 = Red<OP>::op(a0, Red<OP>::op(Red<OP>::op(x0.x, x1.x), Red<OP>::op(x2.x, x3.x)));
        a1 = Red<OP>::op(a1, Red<OP>::op(Red<OP>::op(x0.y, x1.y), Red<OP>::op(x2.y, x3.y)));
        a2 = Red<OP>::op(a2, Red<OP>::op(Red<OP>::op(x0.z, x1.z), Red<OP>::op(x2.z, x3.z)));
        a3 = Red<OP>::op(a3, Red<OP>::op(Red<OP>::op(x0.w, x1.w), Red<OP>::op(x2.w, x3.w)));
      }
      for (; r < end; ++r) {
        float4 x = *reinterpret_cast<const float4 *>(p + r * inner);
        a0 = Red<OP>::op(a0, x.x);
        a1 = Red<OP>::op(a1, x.y);
        a2 = Red<OP>::op(a2, x.z);
        a3 = Red<OP>::op(a3, x.w);
      }
      if (!split) {
        *reinterpret_cast<float4 *>(out + col) =
            make_float4(finish<OP>(a0, div_len, true), finish<OP>(a1, div_len, true),
                        finish<OP>(a2, div_len, true), finish<OP>(a3, div_len, true));
      } else {
        out[(col + 0) * splits + sp] = a0;
        out[(col + 1) * splits + sp] = a1;
        out[(col + 2) * splits + sp] = a2;
        out[(col + 3) * splits + sp] = a3;
      }
    } else {
      for (int v = 0; v < V && c + v < inner; ++v) {
        float a = Red<OP>::init();
        for (int64_t r = beg; r < end; ++r) a = Red<OP>::op(a, p[r * inner + v]);
        if (!split) out[col + v] = finish<OP>(a, div_len, true);
        else out[(col + v) * splits + sp] = a;
      }
    }
  }
}

// Columns in one pass, with a thread-block cluster along `len`. The CS CTAs of a
// cluster (blockIdx.y = rank) reduce the same 128 columns of one outer slice over
// consecutive row ranges; inside a CTA the 8 warps split the range (rows ty,
// ty + 8, ...; 4 rows in flight per thread) and fold their partials through shared
// memory in warp order, then CTA 0 folds the CTAs' partials through distributed
// shared memory in rank order. The order is fixed, so the result does not depend
// on scheduling, and no scratch memory or second launch is needed.
template <int OP>
__global__ void __launch_bounds__(256, 4) cols_cluster_kernel(const float *__restrict__ in,
                                                           float *__restrict__ out, int64_t outer,
                                                           int64_t len, int64_t inner,
                                                           int64_t rows_per_cta, int64_t div_len) {
  pdl_wait();
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float4 warp_part[8][32];
  __shared__ float4 cta_part[32];
  const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;
  const int64_t cblocks = (inner + 127) / 128;
  const int64_t o = (int64_t)blockIdx.x / cblocks, cb = (int64_t)blockIdx.x - o * cblocks;
  const unsigned rank = cluster.block_rank();
  const unsigned cs = cluster.num_blocks();
  const int64_t c = cb * 128 + tx * 4;
  const int64_t beg = (int64_t)rank * rows_per_cta;
  const int64_t end = beg + rows_per_cta < len ? beg + rows_per_cta : len;
  const float z = Red<OP>::init();
  float4 acc = make_float4(z, z, z, z);
  auto fold = [](float4 a, float4 b) {
    return make_float4(Red<OP>::op(a.x, b.x), Red<OP>::op(a.y, b.y), Red<OP>::op(a.z, b.z),
                       Red<OP>::op(a.w, b.w));
  };
  if (c < inner) {
    const float *p = in + o * len * inner + c;
    int64_t r = beg + ty;
    for (; r + 24 < end; r += 32) {
      const float4 x0 = *reinterpret_cast<const float4 *>(p + r * inner);
      const float4 x1 = *reinterpret_cast<const float4 *>(p + (r + 8) * inner);
      const float4 x2 = *reinterpret_cast<const float4 *>(p + (r + 16) * inner);
      const float4 x3 = *reinterpret_cast<const float4 *>(p + (r + 24) * inner);
      acc = fold(acc, fold(fold(x0, x1), fold(x2, x3)));
    }
    for (; r < end; r += 8) acc = fold(acc, *reinterpret_cast<const float4 *>(p + r * inner));
  }
  warp_part[ty][tx] = acc;
  __syncthreads();
  if (ty == 0) {
    float4 v = warp_part[0][tx];
#pragma unroll
    for (int w = 1; w < 8; ++w) v = fold(v, warp_part[w][tx]);
    cta_part[tx] = v;
  }
  cluster.sync();  // every CTA's partial is in its shared memory
  if (rank == 0 && ty == 0) {
    float4 v = cta_part[tx];
    for (unsigned k = 1; k < cs; ++k) v = fold(v, *cluster.map_shared_rank(&cta_part[tx], k));
    if (c < inner)
      *reinterpret_cast<float4 *>(out + o * inner + c) =
          make_float4(finish<OP>(v.x, div_len, true), finish<OP>(v.y, div_len, true),
                      finish<OP>(v.z, div_len, true), finish<OP>(v.w, div_len, true));
  }
  cluster.sync();  // keep every CTA's shared memory alive until CTA 0 has read it
}

template <int OP>
int launch_cols_cluster(const float *in, float *out, int64_t outer, int64_t len, int64_t inner,
                        int cs, cudaStream_t s) {
  const int64_t cblocks = (inner + 127) / 128;
  const int64_t rows_per_cta = (len + cs - 1) / cs;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(outer * cblocks), (unsigned)cs, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)cs;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // PDL: see fz::launch_pdl
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  FZ_CUDA(cudaLaunchKernelEx(&cfg, cols_cluster_kernel<OP>, in, out, outer, len, inner,
                             rows_per_cta, len));
  fz::note_launch();
  return FZ_OK;
}

template <int OP>
int launch_rows_group(const float *in, float *out, int64_t rows, int64_t len, int64_t ld,
                      int64_t div_len, bool final, cudaStream_t s) {
  int vec = (ld % 4 == 0) && (((uintptr_t)in & 15) == 0);
  int G = 1;
  while (G < 32 && (int64_t)G * 4 * 2 < len) G *= 2;
  // rows in flight per group: short rows take several, long ones fill the lanes alone
  const int R = len <= 256 ? 4 : len <= 1024 ? 2 : 1;
  int64_t per_cta = 256 / G * R;
  unsigned grid = fz::grid_for(rows, per_cta, 8, 4);
#define FZ_RG(g, r)                                                                          \
  if (G == g && R == r) {                                                                    \
    FZ_CUDA(fz::launch_pdl(rows_group_kernel<OP, g, r>, dim3(grid), dim3(256), 0, s, in, out, rows, \
                           len, ld, div_len, (int)final, vec));                              \
  } else
  FZ_RG(1, 4) FZ_RG(2, 4) FZ_RG(4, 4) FZ_RG(8, 4) FZ_RG(16, 4) FZ_RG(32, 4)
  FZ_RG(32, 2) FZ_RG(32, 1) {
    return fz::fail(FZ_ERR_INVALID, "fz_reduce: no row-group kernel for this row length");
  }
#undef FZ_RG
  FZ_CHECK_LAUNCH();
  return FZ_OK;
}

// Where split partials go: `ptr` null means stream-ordered memory from the pool
// (fz_reduce); otherwise a caller-owned buffer of `cap` floats (fz_reduce_noalloc).
struct Scratch {
  float *ptr;
  int64_t cap;
};

int scratch_too_small(int64_t need, int64_t cap) {
  return fz::fail(FZ_ERR_INVALID,
                  "fz_reduce_noalloc: this reduction needs " + std::to_string(need) +
                      " partial sums but the library's fixed scratch holds " + std::to_string(cap) +
                      "; use fz_reduce");
}

int take_scratch(const Scratch &sc, int64_t need, float **part, bool *own, cudaStream_t s) {
  *own = false;
  if (sc.ptr) {
    if (need > sc.cap) return scratch_too_small(need, sc.cap);
    *part = sc.ptr;
    return FZ_OK;
  }
  *own = true;
  return fz_malloc((void **)part, sizeof(float) * need, s);
}

template <int OP>
int launch_rows(const float *in, float *out, int64_t rows, int64_t len, int64_t div_len,
                const Scratch &sc, cudaStream_t s) {
  // short rows, or rows of up to 4K floats when there are enough of them for every warp
  // of a full GPU to own some: lane groups (a whole warp per row above 256 floats)
  if (len <= 2048 || (len <= 4096 && rows >= (int64_t)fz::num_sms() * 8))
    return launch_rows_group<OP>(in, out, rows, len, len, div_len, true, s);
  const int threads = 512;
  const int64_t target_ctas = (int64_t)fz::num_sms() * 4;
  int64_t splits = 1;
  if (rows < target_ctas) {
    splits = (target_ctas + rows - 1) / rows;
    int64_t max_splits = len / 8192;  // keep >= 8K floats per CTA
    if (splits > max_splits) splits = max_splits;
    if (splits < 1) splits = 1;
  }
  int64_t chunk = (len + splits - 1) / splits;
  chunk = (chunk + 3) & ~(int64_t)3;
  splits = (len + chunk - 1) / chunk;
  int vec = (len % 4 == 0) && (((uintptr_t)in & 15) == 0);
  int64_t items = rows * splits;
  unsigned grid = (unsigned)(items < target_ctas * 2 ? items : target_ctas * 2);
  if (splits == 1) {
    FZ_CUDA(fz::launch_pdl(rows_block_kernel<OP>, dim3(grid), dim3(threads), 0, s, in, out, rows, len, len,
                           (int64_t)1, chunk, div_len, 1, vec));
    FZ_CHECK_LAUNCH();
    return FZ_OK;
  }
  float *part = nullptr;
  bool own = false;
  int rc = take_scratch(sc, items, &part, &own, s);
  if (rc) return rc;
  const cudaError_t e = fz::launch_pdl(rows_block_kernel<OP>, dim3(grid), dim3(threads), 0, s, in, part, rows,
                                       len, len, splits, chunk, (int64_t)0, 0, vec);
  if (e != cudaSuccess) return fz::cuda_fail(e, "rows_block_kernel launch", __FILE__, __LINE__);
  FZ_CHECK_LAUNCH();
  // splits <= 4 * SMs, so the second pass is a short-row group reduction
  rc = launch_rows_group<OP>(part, out, rows, splits, splits, div_len, true, s);
  if (own) fz_free(part, s);
  return rc;
}

template <int OP>
int launch_cols(const float *in, float *out, int64_t outer, int64_t len, int64_t inner,
                const Scratch &sc, cudaStream_t s) {
  const bool v4 = (inner % 4 == 0) && (((uintptr_t)in & 15) == 0) && (((uintptr_t)out & 15) == 0);
  const int V = v4 ? 4 : 1;
  const int64_t base = outer * ((inner + V - 1) / V);
  const int64_t target = (int64_t)fz::num_sms() * 1024;  // 4 rows in flight per thread
  int64_t splits = 1;
  if (base < target) {
    splits = (target + base - 1) / base;
    int64_t max_splits = len / 32;  // keep >= 32 rows per thread
    if (splits > max_splits) splits = max_splits;
    if (splits < 1) splits = 1;
  }
  int64_t chunk = (len + splits - 1) / splits;
  splits = (len + chunk - 1) / chunk;
  if (splits > 1 && v4) {
    // one pass through a cluster of up to 8 CTAs per 128 columns, when that fills
    // the GPU (or the whole reduction is small enough that one launch is best)
    const int64_t cblocks = outer * ((inner + 127) / 128);
    const int cs = (int)(len >= 8 * 64 ? 8 : (len + 63) / 64 > 1 ? (len + 63) / 64 : 1);
    if (cblocks < 65536 * 32768LL &&
        (cblocks * cs >= 2 * (int64_t)fz::num_sms() || outer * len * inner <= ((int64_t)1 << 22)))
      return launch_cols_cluster<OP>(in, out, outer, len, inner, cs, s);
  }
  int64_t items = splits * base;
  unsigned grid = fz::grid_for(items, 256, 8, 4);
  float *dst = out;
  bool own = false;
  if (splits > 1) {
    int rc = take_scratch(sc, splits * outer * inner, &dst, &own, s);
    if (rc) return rc;
  }
  if (V == 4)
    FZ_CUDA(fz::launch_pdl(cols_kernel<OP, 4>, dim3(grid), dim3(256), 0, s, in, dst, outer, len, inner, splits,
                           chunk, len));
  else
    FZ_CUDA(fz::launch_pdl(cols_kernel<OP, 1>, dim3(grid), dim3(256), 0, s, in, dst, outer, len, inner, splits,
                           chunk, len));
  FZ_CHECK_LAUNCH();
  if (splits == 1) return FZ_OK;
  // second pass: every output column's `splits` partials are contiguous
  int rc = launch_rows_group<OP>(dst, out, outer * inner, splits, splits, len, true, s);
  if (own) fz_free(dst, s);
  return rc;
}

template <int OP>
int reduce_op(float *out, const float *in, int64_t outer, int64_t len, int64_t inner,
              const Scratch &sc, cudaStream_t s) {
  if (inner == 1) return launch_rows<OP>(in, out, outer, len, len, sc, s);
  return launch_cols<OP>(in, out, outer, len, inner, sc, s);
}

int reduce_entry(int op, float *out, const float *in, int64_t outer, int64_t len, int64_t inner,
                 const Scratch &sc, cudaStream_t s) {
  if (len == 0) {
    float v = op == FZ_RMAX ? -INFINITY : op == FZ_RMEAN ? NAN : 0.0f;
    return fz_fill_f32(out, v, outer * inner, s);
  }
  switch (op) {
    case FZ_RSUM: return reduce_op<FZ_RSUM>(out, in, outer, len, inner, sc, s);
    case FZ_RMEAN: return reduce_op<FZ_RMEAN>(out, in, outer, len, inner, sc, s);
    case FZ_RMAX: return reduce_op<FZ_RMAX>(out, in, outer, len, inner, sc, s);
  }
  return fz::fail(FZ_ERR_INVALID, "fz_reduce: unknown op " + std::to_string(op));
}

}  // namespace

extern "C" int fz_reduce(int op, float *out, const float *in, int64_t outer, int64_t len,
                         int64_t inner, void *stream) {
  FZ_REQUIRE(outer >= 0 && len >= 0 && inner >= 0, "fz_reduce: negative extent");
  if (outer == 0 || inner == 0) return FZ_OK;
  FZ_REQUIRE(out && (in || len == 0), "fz_reduce: null pointer");
  return reduce_entry(op, out, in, outer, len, inner, Scratch{nullptr, 0}, fz::resolve(stream));
}

// ---------------------------------------------------------------------------
// Allocation-free variant of fz_reduce.
//
// Some callers must not allocate device memory while they run: a host runtime
// that reserves the GPU's memory up front and accounts for every byte itself
// (a serving process that pre-partitions HBM between models, for instance), or
// a latency-critical loop where growing the allocator's pool would call into the
// driver. fz_reduce takes its split partials from the stream-ordered pool, so
// this variant takes them from a fixed array compiled into the library instead:
// kNoAllocScratchFloats floats (8 MiB) of device memory that every GPU which
// loads the library holds until the process exits.
//
// It runs fz_reduce's own launcher with the partials pointed at the fixed array,
// so it launches the same kernels with the same split plan and its results are
// bit-identical. It rejects (FZ_ERR_INVALID) any reduction
// whose split plan needs more partials than the array holds. The array's device
// address is looked up with cudaGetSymbolAddress the first time the entry point
// runs on a device, so that first call should come before any stream capture.
// All calls share the array and it keeps the last call's contents; every partial
// is written before it is read, so nothing needs clearing, but calls whose work
// overlaps on the GPU (different streams, or different host threads on one
// device) race on it and must be serialised by the caller.
namespace {

// Size of the fixed array. The split plans above bound the partials a reduction
// needs by the SM count: the row path splits only when rows < 4 * SMs, so it writes
// rows * splits < 8 * SMs partials; the column path splits only when its column
// groups (base) number fewer than 1024 * SMs and writes splits * outer * inner <
// 4 * (1024 * SMs + base) < 8 * 1024 * SMs. 2^21 floats covers every plan on GPUs of
// up to 256 SMs (B200: 148); a GPU with more is refused on first use.
constexpr int64_t kNoAllocScratchFloats = int64_t(1) << 21;
constexpr int64_t kNoAllocPartialsPerSm = 8 * 1024;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

std::mutex g_noalloc_mu;
float *g_noalloc_ptr[64] = {};

int noalloc_scratch(float **p) {
  int dev = 0;
  FZ_CUDA(cudaGetDevice(&dev));
  FZ_REQUIRE(dev >= 0 && dev < 64, "fz_reduce_noalloc: device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    if (kNoAllocPartialsPerSm * fz::num_sms() > kNoAllocScratchFloats)
      return fz::fail(FZ_ERR_INVALID, "fz_reduce_noalloc: this GPU has " + std::to_string(fz::num_sms()) +
                                          " SMs; the fixed scratch covers the split plans of at most " +
                                          std::to_string(kNoAllocScratchFloats / kNoAllocPartialsPerSm));
    void *q = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&q, g_noalloc_scratch);
    if (e != cudaSuccess) return fz::cuda_fail(e, "cudaGetSymbolAddress(scratch)", __FILE__, __LINE__);
    g_noalloc_ptr[dev] = static_cast<float *>(q);
  }
  *p = g_noalloc_ptr[dev];
  return FZ_OK;
}

}  // namespace

extern "C" int fz_reduce_noalloc(int op, float *out, const float *in, int64_t outer, int64_t len,
                                 int64_t inner, void *stream) {
  FZ_REQUIRE(outer >= 0 && len >= 0 && inner >= 0, "fz_reduce_noalloc: negative extent");
  if (outer == 0 || inner == 0) return FZ_OK;
  FZ_REQUIRE(out && (in || len == 0), "fz_reduce_noalloc: null pointer");
  FZ_REQUIRE(op == FZ_RSUM || op == FZ_RMEAN || op == FZ_RMAX,
             "fz_reduce_noalloc: unknown op " + std::to_string(op));
  float *scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return reduce_entry(op, out, in, outer, len, inner, Scratch{scratch, kNoAllocScratchFloats},
                      fz::resolve(stream));
}
