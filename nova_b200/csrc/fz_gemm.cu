// fp32 GEMM in 3xTF32 on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// C[b] = op(A[b]) @ op(B[b]), row-major fp32 in and out.
//
// 3xTF32: x = hi + lo with hi = x with its 13 low mantissa bits cleared (exact in
// TF32) and lo = x - hi (exact in fp32); C = Ah*Bh + Ah*Bl + Al*Bh. The kind::tf32
// MMA ignores the 13 low mantissa bits of its fp32 inputs, so an operand already
// stored K-major ([M, K] for A, [N, K] for B) is its own hi plane and only its lo
// plane is written (lo_kernel); an operand given the other way round is transposed
// into K-major hi and lo planes through shared memory (split_t_kernel).
//
// Main kernel, persistent (one CTA per SM walking 128 x 256 output tiles in grouped
// order), warp-specialised, 320 threads:
//   warp 0     TMA producer: per k-tile of BK = 16 loads A_hi, A_lo (128 x 16) and
//              B_hi, B_lo (256 x 16) into a 4-stage ring of 48 KB (64-byte swizzle)
//   warp 1     allocates 2 x 256 TMEM columns; one lane issues, per 8-wide k-step,
//              tcgen05.mma.kind::tf32 lo*hi, hi*lo, hi*hi, and tcgen05.commit frees
//              each stage. The K range is cut into chunks of 256; each chunk
//              accumulates from zero into one of the two TMEM buffers.
//   warps 2-9  promotion and epilogue: two warps per TMEM lane quarter, each owning
//              128 of the 256 columns, tcgen05.ld every finished chunk and add it
//              into an fp32 register accumulator (IEEE adds), then store C.
// The tensor core's own fp32 accumulation is truncating, so its error grows with
// the number of MMAs folded into one accumulator (about 3e-5 relative at K = 4096
// when a whole tile accumulates in TMEM); promoting every 256 of K bounds it to the
// error of a 256-long chunk and keeps long-K products (weight gradients, K = batch)
// within 1e-5. Double-buffered chunks let the MMAs run on while a chunk is promoted.
//
// Every mbarrier wait is bounded by a %globaltimer deadline; on expiry the kernel
// records an error code in the device's error word (read by fz_kernel_status),
// drains its own TMA loads (bounded), frees TMEM and returns, so a bad launch
// surfaces as an error instead of a hang.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "fz_common.cuh"

namespace {

constexpr int BM = 128;
constexpr int BN = 256;
// k-tile: BK fp32 = one swizzle row (BK = 16 -> 64-byte swizzle, 4 stages of 48 KB;
// BK = 32 -> 128-byte swizzle, 2 stages of 96 KB)
#ifndef FZ_GEMM_BK
#define FZ_GEMM_BK 16
#endif
constexpr int BK = FZ_GEMM_BK;
constexpr int STAGES = BK == 16 ? 4 : 2;
constexpr int SWIZZLE_BYTES = BK * 4;
static_assert(BK == 16 || BK == 32, "BK must be 16 or 32");
constexpr int UMMA_K = 8;  // K of one kind::tf32 MMA
constexpr int TILE_A_BYTES = BM * BK * 4;  // 16 KB
constexpr int TILE_B_BYTES = BN * BK * 4;  // 32 KB
constexpr int STAGE_BYTES = 2 * TILE_A_BYTES + 2 * TILE_B_BYTES;  // 96 KB
constexpr int TMEM_COLS = 256;          // one accumulator buffer (BN fp32 columns)
constexpr int KCHUNK = 16;              // k-tiles per promotion chunk (K = 256)
constexpr int NUM_EPI_WARPS = 8;        // 2 per TMEM lane quarter
constexpr int NUM_THREADS = 64 + 32 * NUM_EPI_WARPS;
constexpr unsigned long long kWaitNs = 4000000000ull;  // 4 s per wait

enum : int { kErrNone = 0, kErrTimeoutFull = 1, kErrTimeoutEmpty = 2, kErrTimeoutAcc = 3 };

// ---------------------------------------------------------------- split pass
__device__ __forceinline__ void split1(float x, float &hi, float &lo) {
  hi = __uint_as_float(__float_as_uint(x) & 0xffffe000u);
  lo = __fsub_rn(x, hi);
}

// src rows are K-major already: src[b][r][k] at b*sb + r*ld + k. Writes the lo
// plane lo[b][r][k] (pitch kp, zero beyond K); the MMA reads src itself as hi. When
// src cannot be addressed by TMA (row pitch not a multiple of 16 bytes, or a
// broadcast batch), `hi` is non-null and receives a copy of src at pitch kp.
__global__ void __launch_bounds__(256) lo_kernel(const float *__restrict__ src, int64_t ld,
                                                 int64_t sb, int64_t rows, int64_t K, int64_t kp,
                                                 int64_t batch, float *__restrict__ lo,
                                                 float *__restrict__ hi) {
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (!hi && ld == kp && K == kp && (batch == 1 || sb == rows * kp) && (((uintptr_t)src | (uintptr_t)lo) & 15) == 0) {
    const int64_t n4 = batch * rows * kp / 4;  // dense rows: one flat float4 stream
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
    float4 *l4 = reinterpret_cast<float4 *>(lo);
    for (int64_t t = t0; t < n4; t += step) {
      float4 x = s4[t];
      float h;
      float4 r;
      split1(x.x, h, r.x);
      split1(x.y, h, r.y);
      split1(x.z, h, r.z);
      split1(x.w, h, r.w);
      l4[t] = r;
    }
    return;
  }
  const int64_t total = batch * rows * kp;
  for (int64_t t = t0; t < total; t += step) {
    int64_t k = t % kp;
    int64_t rest = t / kp;
    int64_t r = rest % rows, bb = rest / rows;
    float x = k < K ? src[bb * sb + r * ld + k] : 0.0f;
    float h, l;
    split1(x, h, l);
    lo[t] = l;
    if (hi) hi[t] = x;
  }
}

// src is [b][k][r] (r contiguous, pitch ld): transpose to [b][r][k] while splitting.
__global__ void __launch_bounds__(256) split_t_kernel(const float *__restrict__ src, int64_t ld,
                                                      int64_t sb, int64_t rows, int64_t K,
                                                      int64_t kp, int64_t batch,
                                                      float *__restrict__ hi,
                                                      float *__restrict__ lo) {
  __shared__ float tile[32][33];
  const int64_t tr = (rows + 31) / 32, tk = (kp + 31) / 32;
  const int64_t total = batch * tr * tk;
  const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;
  for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
    int64_t jr = t % tr;
    int64_t rest = t / tr;
    int64_t jk = rest % tk, b = rest / tk;
    const float *s = src + b * sb;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int64_t k = jk * 32 + ty + 8 * i, r = jr * 32 + tx;
      tile[ty + 8 * i][tx] = (k < K && r < rows) ? s[k * ld + r] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int64_t r = jr * 32 + ty + 8 * i, k = jk * 32 + tx;
      if (r < rows && k < kp) {
        float h, l;
        split1(tile[tx][ty + 8 * i], h, l);
        int64_t o = (b * rows + r) * kp + k;
        hi[o] = h;
        lo[o] = l;
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: true on success, false when the deadline passed or another role
// already reported an error.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > kWaitNs) return false;
  }
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// K-major shared-memory descriptor for rows of SWIZZLE_BYTES (one swizzle atom
// row per tile row): 8-row groups 8*SWIZZLE_BYTES apart (SBO), LBO unused (1),
// descriptor version 1 (bit 46), layout type at bits 61-63: 2 = SWIZZLE_128B,
// 4 = SWIZZLE_64B.
__device__ __forceinline__ uint64_t smem_desc_k(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3fff);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)((8 * SWIZZLE_BYTES) >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)(SWIZZLE_BYTES == 128 ? 2 : 4) << 61;
  return d;
}

// kind::tf32 instruction descriptor: D = F32 (bits 4-5 = 1), A = B = TF32 (2),
// both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr uint32_t make_idesc(int m, int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}
constexpr uint32_t kIdesc = make_idesc(BM, BN);

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(kIdesc), "r"(accum)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct GemmArgs {
  float *C;
  int64_t ldc, strideC;
  int64_t split_stride;  // floats between the partial outputs of consecutive K splits
  int M, N, K, batch;
  int tiles_m, tiles_n, num_tiles, group_m;  // num_tiles counts work units (tiles x K splits)
  int splits, k_per_split;  // K is cut into `splits` ranges of k_per_split (multiple of BK)
  int *err;
};

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Work unit t -> (K split, batch, m block, n block). Units of one K split are
// consecutive; within a batch, bands of group_m row blocks are walked column by
// column, so the units in flight on the 148 SMs share A rows and B columns in L2.
__device__ __forceinline__ void decode_tile(int t, const GemmArgs &a, int &mb, int &nb, int &bz,
                                            int &ks) {
  const int per_batch = a.tiles_m * a.tiles_n;
  const int per_split = per_batch * a.batch;  // units of one K split
  ks = t / per_split;
  t -= ks * per_split;
  bz = t / per_batch;
  const int r = t - bz * per_batch;
  const int band = r / (a.group_m * a.tiles_n);
  const int first_m = band * a.group_m;
  const int rows = min(a.group_m, a.tiles_m - first_m);
  const int in_band = r - band * a.group_m * a.tiles_n;
  mb = first_m + in_band % rows;
  nb = in_band / rows;
}

// k-tiles of unit `ks`: [ks * k_per_split, min(K, (ks + 1) * k_per_split)).
__device__ __forceinline__ int unit_k_tiles(const GemmArgs &a, int ks, int &k_begin) {
  k_begin = ks * a.k_per_split;
  const int k_end = min(a.K, k_begin + a.k_per_split);
  return (k_end - k_begin + BK - 1) / BK;
}

// Persistent kernel: one CTA per SM walks tiles blockIdx.x, +gridDim.x, ...
// K is cut into chunks of KCHUNK k-tiles accumulated alternately in two TMEM
// buffers; warps 2-9 fold each finished chunk into fp32 registers.
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_3xtf32_kernel(const __grid_constant__ CUtensorMap mapAh,
                       const __grid_constant__ CUtensorMap mapAl,
                       const __grid_constant__ CUtensorMap mapBh,
                       const __grid_constant__ CUtensorMap mapBl, GemmArgs args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ uint32_t tmem_base_slot;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 32 * NUM_EPI_WARPS);  // every epilogue thread arrives
    }
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_map(&mapAh);
    prefetch_map(&mapAl);
    prefetch_map(&mapBh);
    prefetch_map(&mapBl);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_base_slot)),
                 "r"(2 * TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_base = tmem_base_slot;

  auto stage_ptr = [&](int s, int which) -> uint8_t * {
    uint8_t *base = smem + (size_t)s * STAGE_BYTES;
    switch (which) {
      case 0: return base;
      case 1: return base + TILE_A_BYTES;
      case 2: return base + 2 * TILE_A_BYTES;
      default: return base + 2 * TILE_A_BYTES + TILE_B_BYTES;
    }
  };

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ TMA producer
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < args.num_tiles; t += gridDim.x) {
        int mb, nb, bz, ks, kb;
        decode_tile(t, args, mb, nb, bz, ks);
        const int nk = unit_k_tiles(args, ks, kb);
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = it % STAGES;
          const uint32_t round = it / STAGES;
          if (it >= STAGES && !mbar_wait(&empty_bar[s], (round - 1) & 1, &abort_flag)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full_bar[s], STAGE_BYTES);
          const int k0 = kb + kt * BK;
          tma_load_3d(stage_ptr(s, 0), &mapAh, &full_bar[s], k0, mb * BM, bz);
          tma_load_3d(stage_ptr(s, 1), &mapAl, &full_bar[s], k0, mb * BM, bz);
          tma_load_3d(stage_ptr(s, 2), &mapBh, &full_bar[s], k0, nb * BN, bz);
          tma_load_3d(stage_ptr(s, 3), &mapBl, &full_bar[s], k0, nb * BN, bz);
        }
      }
      if (!ok) {
        atomicCAS(args.err, kErrNone, kErrTimeoutEmpty);
        abort_flag = 1;
        // drain: wait (bounded) for the loads of the last STAGES issued k-tiles
        for (int i = (it > STAGES ? it - STAGES : 0); i < it; ++i) {
          const int s = i % STAGES;
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(&full_bar[s], (i / STAGES) & 1) && globaltimer() - t0 < kWaitNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------ MMA issuer
      int it = 0, cc = 0;  // k-tile and chunk counters, running across tiles
      bool ok = true;
      for (int t = blockIdx.x; ok && t < args.num_tiles; t += gridDim.x) {
        int mb, nb, bz, ks, kb;
        decode_tile(t, args, mb, nb, bz, ks);
        const int num_k = unit_k_tiles(args, ks, kb);
        for (int kt0 = 0; ok && kt0 < num_k; kt0 += KCHUNK, ++cc) {
          const int b = cc & 1;
          if (cc >= 2 && !mbar_wait(&acc_empty[b], ((cc >> 1) - 1) & 1, &abort_flag)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t d_tmem = tmem_base + (uint32_t)(b * TMEM_COLS);
          const int kend = kt0 + KCHUNK < num_k ? kt0 + KCHUNK : num_k;
          for (int kt = kt0; kt < kend; ++kt, ++it) {
            const int s = it % STAGES;
            if (!mbar_wait(&full_bar[s], (it / STAGES) & 1, &abort_flag)) {
              ok = false;
              break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a_hi = smem_u32(stage_ptr(s, 0)), a_lo = smem_u32(stage_ptr(s, 1));
            const uint32_t b_hi = smem_u32(stage_ptr(s, 2)), b_lo = smem_u32(stage_ptr(s, 3));
#pragma unroll
            for (int kk = 0; kk < BK / UMMA_K; ++kk) {
              const uint32_t off = kk * UMMA_K * 4;  // 32 bytes per k-step in the swizzle row
              const uint64_t dah = smem_desc_k(a_hi + off), dal = smem_desc_k(a_lo + off);
              const uint64_t dbh = smem_desc_k(b_hi + off), dbl = smem_desc_k(b_lo + off);
              const uint32_t first = (kt == kt0 && kk == 0) ? 0u : 1u;
              umma_tf32(d_tmem, dal, dbh, first);  // lo * hi
              umma_tf32(d_tmem, dah, dbl, 1u);     // hi * lo
              umma_tf32(d_tmem, dah, dbh, 1u);     // hi * hi (largest term last)
            }
            umma_commit(&empty_bar[s]);
          }
          if (ok) umma_commit(&acc_full[b]);
        }
      }
      if (!ok) {
        atomicCAS(args.err, kErrNone, kErrTimeoutFull);
        abort_flag = 1;
      }
    }
  } else {
    // ------------------------------------------------------ promotion + epilogue (warps 2..9)
    const int q = warp & 3;             // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;   // which 128 of the 256 columns
    const bool vec = ((args.ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(args.C) & 15) == 0) &&
                     ((args.strideC & 3) == 0);
    int cc = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < args.num_tiles; t += gridDim.x) {
      int mb, nb, bz, ks, kb;
      decode_tile(t, args, mb, nb, bz, ks);
      const int num_k = unit_k_tiles(args, ks, kb);
      float acc[128];
#pragma unroll
      for (int i = 0; i < 128; ++i) acc[i] = 0.0f;
      for (int kt0 = 0; kt0 < num_k; kt0 += KCHUNK, ++cc) {
        const int b = cc & 1;
        if (!mbar_wait(&acc_full[b], (cc >> 1) & 1, &abort_flag)) {
          if (lane == 0) atomicCAS(args.err, kErrNone, kErrTimeoutAcc);
          abort_flag = 1;
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t taddr = tmem_base + (uint32_t)(b * TMEM_COLS + half * 128) +
                               ((uint32_t)(q * 32) << 16);
#pragma unroll
        for (int c0 = 0; c0 < 128; c0 += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + (uint32_t)c0, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[c0 + i] = __fadd_rn(acc[c0 + i], __uint_as_float(r[i]));
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        mbar_arrive(&acc_empty[b]);
      }
      if (!ok) break;
      const int row = mb * BM + q * 32 + lane;
      const int col0 = nb * BN + half * 128;
      if (row < args.M && col0 < args.N) {
        float *crow = args.C + (int64_t)ks * args.split_stride + (int64_t)bz * args.strideC +
                      (int64_t)row * args.ldc + col0;
        if (vec && col0 + 128 <= args.N) {
#pragma unroll
          for (int i = 0; i < 128; i += 4)
            *reinterpret_cast<float4 *>(crow + i) = make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
        } else {
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (col0 + i < args.N) crow[i] = acc[i];
        }
      }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(2 * TMEM_COLS)
                 : "memory");
  }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int get_encoder() {
  static std::once_flag once;
  static int rc = FZ_OK;
  std::call_once(once, []() {
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                                     cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
      rc = fz::fail(FZ_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
      return;
    }
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return rc;
}

// 3D map over a [batch, rows, K] operand (K innermost, row pitch ld floats, batch
// pitch sb floats), box {BK, box_rows, 1}. TMA needs ld*4 and sb*4 to be multiples
// of 16 bytes and the base 16-byte aligned.
int make_map(CUtensorMap *map, const float *base, int64_t rows, int64_t K, int64_t ld, int64_t sb,
             int64_t batch, int box_rows) {
  if (batch == 1) sb = ld * rows;
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 4), (cuuint64_t)(sb * 4)};
  cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void *)base, dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        SWIZZLE_BYTES == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fz::fail(FZ_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  return FZ_OK;
}

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// Number of K splits for a GEMM of `tiles` output tiles. A split turns one tile
// into several units over K ranges (multiples of the 256-wide promotion chunk, at
// least 1024 long) whose fp32 partials are summed afterwards; it pays when the
// tiles fill the 148 SMs poorly (weight gradients: few tiles, K = batch rows).
// Cost model in units of one tile's time per k: waves * K_per_unit, plus the
// partials' write and read at HBM speed.
int choose_splits(int64_t tiles, int64_t M, int64_t N, int64_t K, int64_t batch) {
  const int64_t sms = fz::num_sms();
  const double k_time = 2.65e-8;  // s per k of one 128x256 tile (3 TF32 MMAs at ~1.1 PFLOP/s per GPU)
  int best = 1;
  double best_t = 1e300;
  const int cand[] = {1, 2, 3, 4, 6, 8, 12, 16, 24, 32};
  for (int sp : cand) {
    const int64_t kps = sp == 1 ? K : round_up((K + sp - 1) / sp, (int64_t)BK * KCHUNK);
    if (sp > 1 && kps < 1024) break;
    const int64_t real = (K + kps - 1) / kps;
    const int64_t waves = (tiles * real + sms - 1) / sms;
    double t = (double)waves * (double)kps;
    if (real > 1) t += (double)(real * batch * M * N) * 8.0 / 6.0e12 / k_time;
    if (t < best_t * 0.97) {
      best_t = t;
      best = (int)real;
    }
  }
  return best;
}

// One operand as the (hi, lo) pair the kernel reads, both [batch, rows, K] K-major.
struct Operand {
  const float *hi;
  int64_t hi_ld, hi_sb;
  float *lo;  // plane at pitch kp
};

// Plane floats an operand needs in the workspace (lo always; hi unless the source
// is K-major and TMA-addressable).
bool direct_hi(const float *src, int64_t ld, int64_t sb, bool kmajor, int64_t batch) {
  return kmajor && ld % 4 == 0 && ((uintptr_t)src & 15) == 0 && (batch == 1 || (sb > 0 && sb % 4 == 0));
}

int prepare(const float *src, int64_t ld, int64_t sb, bool kmajor, int64_t rows, int64_t K,
            int64_t kp, int64_t batch, float *ws, Operand *op, cudaStream_t s) {
  const int64_t plane = batch * rows * kp;
  op->lo = ws;
  if (kmajor) {
    const bool direct = direct_hi(src, ld, sb, kmajor, batch);
    float *hi = direct ? nullptr : ws + plane;
    unsigned grid = fz::grid_for(plane / 4 + 1, 256, 8, 4);
    lo_kernel<<<grid, 256, 0, s>>>(src, ld, sb, rows, K, kp, batch, op->lo, hi);
    FZ_CHECK_LAUNCH();
    if (direct) {
      op->hi = src;
      op->hi_ld = ld;
      op->hi_sb = sb;
    } else {
      op->hi = hi;
      op->hi_ld = kp;
      op->hi_sb = rows * kp;
    }
    return FZ_OK;
  }
  float *hi = ws + plane;
  int64_t tiles = batch * ((rows + 31) / 32) * ((kp + 31) / 32);
  unsigned grid = fz::grid_for(tiles, 1, 8, 4);
  split_t_kernel<<<grid, 256, 0, s>>>(src, ld, sb, rows, K, kp, batch, hi, op->lo);
  FZ_CHECK_LAUNCH();
  op->hi = hi;
  op->hi_ld = kp;
  op->hi_sb = rows * kp;
  return FZ_OK;
}

}  // namespace

extern "C" int fz_gemm_f32(int64_t batch, int64_t M, int64_t N, int64_t K, const float *A,
                           int64_t lda, int64_t strideA, int transA, const float *B, int64_t ldb,
                           int64_t strideB, int transB, float *C, int64_t ldc, int64_t strideC,
                           void *stream) {
  FZ_REQUIRE(batch >= 0 && M >= 0 && N >= 0 && K >= 0, "fz_gemm_f32: negative extent");
  if (batch == 0 || M == 0 || N == 0) return FZ_OK;
  FZ_REQUIRE(C, "fz_gemm_f32: null C");
  FZ_REQUIRE(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31) && batch < 65536,
             "fz_gemm_f32: extent too large");
  FZ_REQUIRE(ldc >= N, "fz_gemm_f32: ldc < N");
  cudaStream_t s = fz::resolve(stream);
  if (K == 0) {
    for (int64_t b = 0; b < batch; ++b)
      for (int64_t r = 0; r < M; ++r) {
        int rc = fz_fill_f32(C + b * strideC + r * ldc, 0.0f, N, s);
        if (rc) return rc;
      }
    return FZ_OK;
  }
  FZ_REQUIRE(A && B, "fz_gemm_f32: null operand");
  FZ_REQUIRE(lda >= (transA ? M : K) && ldb >= (transB ? K : N), "fz_gemm_f32: bad leading dim");
  int rc = get_encoder();
  if (rc) return rc;

  const int64_t kp = (K + 3) & ~(int64_t)3;  // 16-byte row pitch for TMA
  const bool a_km = transA == 0, b_km = transB != 0;  // A as [M,K], B as [N,K]
  const int64_t a_plane = batch * M * kp, b_plane = batch * N * kp;
  const int64_t a_need = a_plane * (direct_hi(A, lda, strideA, a_km, batch) ? 1 : 2);
  const int64_t b_need = b_plane * (direct_hi(B, ldb, strideB, b_km, batch) ? 1 : 2);
  float *ws = nullptr;
  rc = fz_malloc((void **)&ws, sizeof(float) * (a_need + b_need), s);
  if (rc) return rc;
  Operand oa{}, ob{};
  rc = prepare(A, lda, strideA, a_km, M, K, kp, batch, ws, &oa, s);
  if (!rc) rc = prepare(B, ldb, strideB, b_km, N, K, kp, batch, ws + a_need, &ob, s);

  CUtensorMap mAh, mAl, mBh, mBl;
  if (!rc) rc = make_map(&mAh, oa.hi, M, K, oa.hi_ld, oa.hi_sb, batch, BM);
  if (!rc) rc = make_map(&mAl, oa.lo, M, K, kp, M * kp, batch, BM);
  if (!rc) rc = make_map(&mBh, ob.hi, N, K, ob.hi_ld, ob.hi_sb, batch, BN);
  if (!rc) rc = make_map(&mBl, ob.lo, N, K, kp, N * kp, batch, BN);
  const int tiles_m = (int)((M + BM - 1) / BM), tiles_n = (int)((N + BN - 1) / BN);
  const int64_t tiles = (int64_t)tiles_m * tiles_n * batch;
  const bool dense_c = ldc == N && (batch == 1 || strideC == M * N);
  const int splits = dense_c ? choose_splits(tiles, M, N, K, batch) : 1;
  const int64_t kps = splits > 1 ? round_up((K + splits - 1) / splits, (int64_t)BK * KCHUNK) : K;
  const int real_splits = (int)((K + kps - 1) / kps);
  const int64_t num_units = tiles * real_splits;
  if (!rc && num_units >= (1ll << 31)) rc = fz::fail(FZ_ERR_INVALID, "fz_gemm_f32: too many tiles");
  float *partial = nullptr;
  if (!rc && real_splits > 1)
    rc = fz_malloc((void **)&partial, sizeof(float) * real_splits * batch * M * N, s);

  int *err = nullptr;
  if (!rc) rc = fz::device_error_word(&err);
  if (!rc) {
    const size_t smem = (size_t)STAGES * STAGE_BYTES + 1024;
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_done[dev]) {
      cudaFuncSetAttribute(gemm_3xtf32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
      attr_done[dev] = true;
    }
    GemmArgs ga{partial ? partial : C, partial ? N : ldc, partial ? M * N : strideC,
                batch * M * N, (int)M, (int)N, (int)K, (int)batch,
                tiles_m, tiles_n, (int)num_units, tiles_m < 16 ? tiles_m : 16,
                real_splits, (int)kps, err};
    const unsigned grid = (unsigned)(num_units < fz::num_sms() ? num_units : fz::num_sms());
    gemm_3xtf32_kernel<<<grid, NUM_THREADS, smem, s>>>(mAh, mAl, mBh, mBl, ga);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) rc = fz::cuda_fail(e, "gemm_3xtf32_kernel launch", __FILE__, __LINE__);
    else fz::note_launch();
    // K-split partials: summed over the splits in a fixed order (deterministic)
    if (!rc && partial) rc = fz_reduce(FZ_RSUM, C, partial, 1, real_splits, batch * M * N, s);
  }
  if (partial) fz_free(partial, s);
  fz_free(ws, s);
  return rc;
}
