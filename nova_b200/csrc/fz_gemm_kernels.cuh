// Device code of the 3xTF32 GEMM kernels (tcgen05 + TMEM + TMA, sm_100a), shared by
// the ahead-of-time build and by runtime compilation with a fused epilogue.
//
// The kernels are templates over an epilogue class EPI whose
//   template <int CPW> static void prefetch(args, ep, bz, row, col0)
// is called when a tile starts (before its MMAs complete) and whose
//   template <int CPW> static void store(args, ep, ks, bz, row, col0, acc)
// receives, per epilogue thread, one output row's CPW consecutive accumulator
// columns [col0, col0 + CPW) in registers and writes them out. StoreEpi stores the
// product (the library's ahead-of-time instances). A fused elementwise program over
// the product is compiled by NVRTC into a generated epilogue class, with this file's
// text (embedded in the library) as the kernel source, so the program's outputs are
// written straight from the accumulators.
#pragma once

#ifdef __CUDACC_RTC__
typedef unsigned char uint8_t;
typedef unsigned int uint32_t;
typedef int int32_t;
typedef unsigned long long uint64_t;
typedef long long int64_t;
typedef unsigned long long uintptr_t;
// layout of the driver's CUtensorMap (128 opaque bytes, 64-byte aligned)
struct __align__(64) CUtensorMap {
  unsigned long long opaque[16];
};
#else
#include <cuda.h>

#include <cstdint>
#endif

namespace fz_gemm_dev {

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
constexpr int MN_CHUNK = 32;              // MN-major tiles: M/N rows per 128-byte swizzle row
constexpr int MN_CHUNK_BYTES = BK * 128;  // one such chunk of a stage tile (BK k-rows)
constexpr int TILE_A_BYTES = BM * BK * 4;  // 16 KB
constexpr int TILE_B_BYTES = BN * BK * 4;  // 32 KB
constexpr int STAGE_BYTES = 2 * TILE_A_BYTES + 2 * TILE_B_BYTES;  // 96 KB
constexpr int TMEM_COLS = 256;          // one accumulator buffer (BN fp32 columns)
// k-tiles per promotion chunk (K = 128). The tensor core's accumulation truncates: each
// MMA added into a TMEM accumulator shifts the sum toward zero by about 0.3 ulp, so the
// relative bias of a chunk grows with its 3 * K / 8 MMAs (about 1.9e-8 per MMA,
// measured); chunks of 128 keep it near 1e-6 per product, against 2e-6 for chunks of
// 256, at about 2 % of the GEMM's time (more handoffs between MMA issuer and promoting
// warps, and less run-ahead of the MMAs while the epilogue stores).
#ifndef FZ_GEMM_KCHUNK
#define FZ_GEMM_KCHUNK 8
#endif
constexpr int KCHUNK = FZ_GEMM_KCHUNK;
constexpr int KSPLIT_GRAN = 16;         // K splits are multiples of this many k-tiles
constexpr int NUM_EPI_WARPS = 8;        // 2 per TMEM lane quarter
// Warp roles: 0 TMA producer, 1 MMA issuer (and TMEM owner), 2-3 idle, 4-11 promotion
// and epilogue. Registers are rebalanced per warpgroup with setmaxnreg: the launch
// gives every thread REG_LAUNCH (12 warps = 3 per SM sub-partition: 168 of the 65536);
// warpgroup 0 (warps 0-3) drops to REG_CTRL and the epilogue warpgroups take what it
// frees, so their 128 fp32 accumulators per thread leave room for the epilogue program.
// The launch check in fz_gemm.cu refuses a kernel whose register count is not
// REG_LAUNCH (the split would not add up: setmaxnreg.inc would wait for registers
// that no warp frees).
constexpr int EPI_WARP0 = 4;
constexpr int NUM_THREADS = 32 * (EPI_WARP0 + NUM_EPI_WARPS);
constexpr int REG_LAUNCH = 168, REG_CTRL = 56, REG_EPI = 224;
static_assert(NUM_THREADS * REG_LAUNCH <= 65536, "registers at launch");
static_assert(128 * REG_CTRL + 32 * NUM_EPI_WARPS * REG_EPI == NUM_THREADS * REG_LAUNCH,
              "setmaxnreg split uses exactly the launch's registers");
static_assert(NUM_EPI_WARPS == 8 && EPI_WARP0 == 4, "two epilogue warpgroups after warpgroup 0");
constexpr unsigned long long kWaitNs = 4000000000ull;  // 4 s per wait
// A producer waits at most this long for the others at a tile boundary, then goes on.
constexpr unsigned long long kTileSyncNs = 200000ull;

enum : int {
  kErrNone = 0, kErrTimeoutFull = 1, kErrTimeoutEmpty = 2, kErrTimeoutAcc = 3, kErrTimeoutSplit = 4,
  kErrTimeoutEpiLoad = 5
};
// Kernels instantiated with SPLIT derive the remainder tiles in shared memory: the TMA
// producer loads the raw operand tiles only, and warps 2-3 (otherwise idle) and the
// eight epilogue warps (between promotions) each write a share of every k-tile's
// remainder tiles beside them; the MMA issuer takes the stage once all ten have.
constexpr int NUM_SPLIT_WARPS = 2 + NUM_EPI_WARPS;
constexpr int SPLIT_SHARE_CTRL = 128;  // float4s of a stage per splitter warp 2 or 3


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

// mbar_wait with cluster-scope acquire: for a barrier that threads of the other CTA of
// a pair release (their shared-memory writes must be visible to this CTA's MMAs).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > kWaitNs) return false;
  }
}

// Wait for a phase without the abort shortcut (draining work already issued), bounded.
__device__ __forceinline__ void mbar_drain(uint64_t *bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity) && globaltimer() - t0 < kWaitNs) {
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

// Kernels are launched with programmatic stream serialization (PDL): wait for the grid
// before in the stream to complete before touching global memory.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void prefetch_map(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// One operand's k-tile [row0, row0 + ROWS) x [k0, k0 + BK) into a stage tile.
// K-major: one box {BK, ROWS}. MN-major: the tile is ROWS / 32 chunks of
// MN_CHUNK_BYTES; a "wide" map (4D: 32 rows, K, chunk, batch) fetches all chunks in
// one box, a narrow one (3D) one chunk per box. Rows past the operand's extent are
// zero-filled by the TMA unit.
template <bool MN, int ROWS>
__device__ __forceinline__ void load_operand(uint8_t *dst, const CUtensorMap *map, uint64_t *bar,
                                             int k0, int row0, int bz, bool wide) {
  if constexpr (MN) {
    if (wide) {
      tma_load_4d(dst, map, bar, 0, k0, row0 / MN_CHUNK, bz);
    } else {
#pragma unroll
      for (int j = 0; j < ROWS / MN_CHUNK; ++j)
        tma_load_3d(dst + j * MN_CHUNK_BYTES, map, bar, row0 + j * MN_CHUNK, k0, bz);
    }
  } else {
    tma_load_3d(dst, map, bar, k0, row0, bz);
  }
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

// MN-major shared-memory descriptor. For 32-bit (TF32) operands the MN-major layout
// is the 128-byte swizzle with 32-byte atomicity (layout type 1): 32-byte units of a
// 128-byte row are permuted by the row index mod 4, in atoms of 4 k-rows x 128 bytes
// (512 B). The tile is stored as chunks of 32 M/N rows, each BK k-rows of 128 bytes;
// LBO = distance between the 32-wide M/N chunks (BK * 128 bytes), SBO = distance
// between 4-row k atoms (512 bytes). The TMA writes this image with
// CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B.
__device__ __forceinline__ uint64_t smem_desc_mn(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3fff);
  d |= (uint64_t)(MN_CHUNK_BYTES >> 4) << 16;
  d |= (uint64_t)(512 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)1 << 61;
  return d;
}

// Descriptor of k-step kk (UMMA_K wide) of a stage tile at `base`.
template <bool MN>
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int kk) {
  if constexpr (MN) return smem_desc_mn(base + (uint32_t)kk * (UMMA_K * 128));  // 8 k-rows
  else return smem_desc_k(base + (uint32_t)kk * (UMMA_K * 4));                  // 32 bytes
}

// kind::tf32 instruction descriptor: D = F32 (bits 4-5 = 1), A = B = TF32 (2),
// A major at bit 15 and B major at bit 16 (0 = K-major, 1 = MN-major), N >> 3 at
// bits 17-22, M >> 4 at bits 24-28.
__host__ __device__ constexpr uint32_t make_idesc(int m, int n, bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 columns of this warp's 32 TMEM lanes into r, without waiting for them
// (tmem_wait_ld), so several loads can be in flight.
__device__ __forceinline__ void tmem_ld_32x32b_x32_async(uint32_t taddr, uint32_t (&r)[32]) {
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
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

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
  int wide;                 // bits 0-3: map Ah, Al, Bh, Bl is a wide (4D) MN-major map
  int *err;
  // CTA pairs' TMA producers meet at each tile boundary: a zeroed counter in global
  // memory (null: they do not), each wait bounded by kTileSyncNs
  unsigned int *tile_sync;
};

// Operands of a fused epilogue program. Leaf 0 of the program is the product; leaf
// k >= 1 reads in[k-1] at bz * in_sb + row * in_sm (+ col when the input varies
// along the columns, a property compiled into the epilogue). Output k is written at
// out[k] + bz * strideC + row * ldc + col. vec: every column-varying input and
// every output allows 16-byte accesses at each row.
//
// tma: the outputs are written by TMA bulk tensor stores from the staging tile,
// through omap[k] (output k; the plain epilogue's C or K-split partials in omap[0]):
// 3D maps {N, M, Z} over fp32 with row pitch ldc, Z = batch (or K splits x batch for
// partials), boxes of {BW, 32, 1}, no swizzle. The TMA unit clips boxes at N and M.
// Plain per-thread stores drain at about 15 GB/s per SM while the mainloop's TMA
// loads run (measured: 9 us per 128 KB output tile per CTA, whatever the access
// pattern), longer than the MMAs can run ahead; bulk stores leave the SM at once.
// imap: with one full-shape input, its load map (the same {N, M, Z} layout and 32 x 32
// boxes in the 128-byte swizzle of tile_put), used by the generated epilogue that
// brings the input into the staging tile by TMA, 32 columns at a time.
constexpr int EPI_MAX_IN = 11;
constexpr int EPI_MAX_OUT = 4;
struct __align__(64) EpiParams {
  CUtensorMap omap[EPI_MAX_OUT];
  CUtensorMap imap;
  const float *in[EPI_MAX_IN];
  long long in_sb[EPI_MAX_IN], in_sm[EPI_MAX_IN];
  float *out[EPI_MAX_OUT];
  int vec;
  int tma;
};

// ---- warp-cooperative epilogue I/O
//
// The 32 lanes of an epilogue warp hold 32 consecutive output rows (lane = row), each
// a run of CPW columns in registers. A lane storing its own row would make every warp
// store touch 32 rows. Instead, per block of EPI_BW columns, the lanes exchange values
// through the warp's private 32 x 32 fp32 staging tile in shared memory. Each row of
// the tile is 8 float4 slots; slot c4 of row r lives at r * 8 + (c4 ^ (r & 7)), so both
// the row-per-lane and the row-per-8-lanes access patterns are free of bank conflicts.
// Global accesses then move whole row segments (EPI_BW / 4 lanes per row).
constexpr int EPI_BW = 16;                   // columns per block (register pressure:
                                             // the 128 accumulators stay live meanwhile)
constexpr int EPI_TILE_BYTES = 32 * 32 * 4;  // per epilogue warp
constexpr int EPI_SMEM_BYTES = NUM_EPI_WARPS * EPI_TILE_BYTES;

__device__ __forceinline__ void tile_put(float4 *t, int r, int c4, float4 v) { t[r * 8 + (c4 ^ (r & 7))] = v; }
__device__ __forceinline__ float4 tile_get(const float4 *t, int r, int c4) { return t[r * 8 + (c4 ^ (r & 7))]; }

// tile rows [0, rows) x columns [0, cols) -> dst (row pitch ld); 16-byte stores when vec
// (dst 16-byte aligned, ld a multiple of 4), else per element.
// `slot`: the block's first float4 slot in each tile row (blocks narrower than the
// tile row may share the tile: an epilogue's inputs and outputs side by side).
template <int BW>
__device__ __forceinline__ void tile_store(const float4 *t, float *dst, long long ld, int rows,
                                           int cols, bool vec, int lane, int slot = 0) {
  constexpr int LPR = BW / 4, RPI = 32 / LPR;  // lanes per row, rows per instruction
  const int c4 = lane % LPR;
#pragma unroll
  for (int r0 = 0; r0 < 32; r0 += RPI) {
    const int r = r0 + lane / LPR;
    if (r < rows) {
      const float4 v = tile_get(t, r, slot + c4);
      float *d = dst + (long long)r * ld + c4 * 4;
      if (vec && c4 * 4 + 4 <= cols) {
        *reinterpret_cast<float4 *>(d) = v;
      } else {
        if (c4 * 4 + 0 < cols) d[0] = v.x;
        if (c4 * 4 + 1 < cols) d[1] = v.y;
        if (c4 * 4 + 2 < cols) d[2] = v.z;
        if (c4 * 4 + 3 < cols) d[3] = v.w;
      }
    }
  }
}

// src (row pitch ld) rows [0, rows) x columns [0, cols) -> tile, zeros elsewhere.
template <int BW>
__device__ __forceinline__ void tile_load(float4 *t, const float *src, long long ld, int rows,
                                          int cols, bool vec, int lane, int slot = 0) {
  constexpr int LPR = BW / 4, RPI = 32 / LPR;
  const int c4 = lane % LPR;
#pragma unroll
  for (int r0 = 0; r0 < 32; r0 += RPI) {
    const int r = r0 + lane / LPR;
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (r < rows) {
      const float *s = src + (long long)r * ld + c4 * 4;
      if (vec && c4 * 4 + 4 <= cols) {
        v = *reinterpret_cast<const float4 *>(s);
      } else {
        if (c4 * 4 + 0 < cols) v.x = s[0];
        if (c4 * 4 + 1 < cols) v.y = s[1];
        if (c4 * 4 + 2 < cols) v.z = s[2];
        if (c4 * 4 + 3 < cols) v.w = s[3];
      }
    }
    tile_put(t, r, slot + c4, v);
  }
}

// Same as tile_load for 16-byte-aligned rows (dst pitch and src pointer multiples of
// 16 bytes), but every lane's copies go global -> shared with cp.async, so all of a
// block's loads are in flight at once and no registers hold them. Past `cols` or
// `rows` the copy reads fewer (or no) bytes and zero-fills the slot; such a copy
// points at src itself, which lies inside the tensor.
template <int BW>
__device__ __forceinline__ void tile_load_async(float4 *t, const float *src, long long ld,
                                                int rows, int cols, int lane, int slot = 0) {
  constexpr int LPR = BW / 4, RPI = 32 / LPR;
  const int c4 = lane % LPR;
#pragma unroll
  for (int r0 = 0; r0 < 32; r0 += RPI) {
    const int r = r0 + lane / LPR;
    const int left = cols - c4 * 4;
    const uint32_t bytes = (r < rows && left > 0) ? 4u * (uint32_t)min(left, 4) : 0u;
    const float *s = bytes ? src + (long long)r * ld + c4 * 4 : src;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                     smem_u32(t + r * 8 + ((slot + c4) ^ (r & 7)))),
                 "l"(s), "r"(bytes)
                 : "memory");
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Pull this lane's row segment [col0, col0 + n) of a full-shape epilogue input into
// L2 (one prefetch per 128-byte line), issued when a tile starts. Only addresses
// inside the segment.
__device__ __forceinline__ void prefetch_row_l2(const float *p, int n) {
  if (n <= 0) return;
  const uintptr_t first = reinterpret_cast<uintptr_t>(p) & ~(uintptr_t)127;
  const uintptr_t last = reinterpret_cast<uintptr_t>(p + n - 1);
  for (uintptr_t a = first; a <= last; a += 128) {
    const uintptr_t q = a < reinterpret_cast<uintptr_t>(p) ? reinterpret_cast<uintptr_t>(p) : a;
    asm volatile("prefetch.global.L2 [%0];" ::"l"(q));
  }
}

// ---- TMA output staging
//
// With TMA stores the warp's 4 KB tile is cut into 32 / BW regions of 32 rows x BW
// floats, row-major (BW * 4 bytes per row), region i at byte i * BW * 128. A lane
// writes its own row of a region; one lane then issues the region's bulk store.
// A region is rewritten only after the stores that read it are done reading
// (cp.async.bulk.wait_group.read by the issuing lane, then a warp barrier).
__device__ __forceinline__ float4 *region_ptr(float4 *tile, int bw, int i) {
  return tile + i * bw * 8;  // bw * 128 bytes = bw * 8 float4
}
__device__ __forceinline__ void region_put(float4 *reg, int bw, int r, int c4, float4 v) {
  reg[r * (bw / 4) + c4] = v;
}
__device__ __forceinline__ float4 region_get(const float4 *reg, int bw, int r, int c4) {
  return reg[r * (bw / 4) + c4];
}
// Wait (lane 0) until at most `pending` committed store groups still read shared
// memory, then let the warp go on.
template <int PENDING>
__device__ __forceinline__ void store_reads_done(int lane, unsigned mask) {
  if (lane == 0) asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(PENDING) : "memory");
  __syncwarp(mask);
}
// The warp's generic-proxy writes to the staged regions become visible to the TMA
// unit; then lane 0 may issue the stores.
__device__ __forceinline__ void staged_for_tma(unsigned mask) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp(mask);
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int x, int y,
                                             int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tma_store_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// End of an epilogue warp's work: its last bulk stores have completed.
__device__ __forceinline__ void tma_stores_drain(const EpiParams &ep, int lane) {
  if (ep.tma && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// An epilogue warp's barrier for TMA loads into its staging tile, the parity of its
// next phase, whether a load is in flight, and the CTA's abort flag (bounded waits as
// in the main loop).
struct EpiSync {
  uint64_t *bar;
  uint32_t phase;
  int pending;
  volatile int *abort;
};

// Start loading the 32 x 32 box of `map` at (x, y, z) into the warp's staging tile
// (128-byte swizzle, zeros past the tensor's edges), once the tile's earlier stores
// have read it.
__device__ __forceinline__ void epi_issue_box(const CUtensorMap *map, float4 *tile, EpiSync &sync, int x, int y,
                                              int z, int lane, unsigned mask) {
  store_reads_done<0>(lane, mask);
  if (lane == 0) {
    mbar_expect_tx(sync.bar, 32 * 32 * 4);
    tma_load_3d(tile, map, sync.bar, x, y, z);
  }
  sync.pending = 1;
}

// Wait for the box in flight. False (after recording the error and letting the load
// land) if the wait ran out.
__device__ __forceinline__ bool epi_wait_box(EpiSync &sync, int lane, unsigned mask, int *err) {
  const bool ok = __all_sync(mask, mbar_wait(sync.bar, sync.phase, sync.abort));
  if (!ok) {
    if (lane == 0) atomicCAS(err, kErrNone, kErrTimeoutEpiLoad);
    *sync.abort = 1;
    mbar_drain(sync.bar, sync.phase);
  }
  sync.phase ^= 1u;
  sync.pending = 0;
  return ok;
}

// A load left in flight (a tile abandoned after an abort) lands before the CTA goes on.
__device__ __forceinline__ void epi_settle(EpiSync &sync) {
  if (sync.pending) {
    mbar_drain(sync.bar, sync.phase);
    sync.phase ^= 1u;
    sync.pending = 0;
  }
}

// L2 prefetch of a 32 x 32 box of `map` by the TMA unit.
__device__ __forceinline__ void tma_prefetch_box(const CUtensorMap *map, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}
// Copy rows [0, rows) x columns [0, cols) of src (row pitch ld, 16-byte aligned rows)
// into region `reg` (zeros elsewhere), every lane's copies in flight at once.
template <int BW>
__device__ __forceinline__ void region_load_async(float4 *reg, const float *src, long long ld,
                                                  int rows, int cols, int lane) {
  constexpr int LPR = BW / 4, RPI = 32 / LPR;
  const int c4 = lane % LPR;
#pragma unroll
  for (int r0 = 0; r0 < 32; r0 += RPI) {
    const int r = r0 + lane / LPR;
    const int left = cols - c4 * 4;
    const uint32_t bytes = (r < rows && left > 0) ? 4u * (uint32_t)min(left, 4) : 0u;
    const float *s = bytes ? src + (long long)r * ld + c4 * 4 : src;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                     smem_u32(reg + r * LPR + c4)),
                 "l"(s), "r"(bytes)
                 : "memory");
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// The plain epilogue: C = product (or this unit's K-split partial), stored through
// the staging tile. `row` is this lane's row; the warp's rows are row - lane + [0, 32).
struct StoreEpi {
  template <int CPW>
  static __device__ __forceinline__ void prefetch(const GemmArgs &, const EpiParams &, int, int, int) {}
  template <int CPW>
  static __device__ __forceinline__ void before_last(const GemmArgs &, const EpiParams &, int, int, int,
                                                     float4 *, EpiSync &) {}
  template <int CPW>
  static __device__ __forceinline__ void store(const GemmArgs &a, const EpiParams &ep, int ks,
                                               int bz, int row, int col0, const float (&acc)[CPW],
                                               float4 *tile, EpiSync &) {
    const int lane = threadIdx.x & 31;
    const int row0 = row - lane;
    const int rows = min(32, a.M - row0);
    if (rows <= 0 || col0 >= a.N) return;  // uniform over the warp
    const unsigned mask = __activemask();
    constexpr int BW = CPW < EPI_BW ? CPW : EPI_BW;
    if (ep.tma && CPW >= 32) {
      // 32-column blocks: the whole 4 KB tile in the 128-byte-swizzled layout of
      // tile_put, one 32 x 32 box per store (the map swizzles the same way). A block
      // is staged once the previous block's store has read the tile (a short wait; a
      // store's fixed cost, about 0.5 us of staging, proxy fence and issue, is what
      // the wider blocks halve).
      const int z = ks * a.batch + bz;
#pragma unroll
      for (int cb = 0; cb < CPW / 32; ++cb) {
        if (col0 + cb * 32 >= a.N) break;
        store_reads_done<0>(lane, mask);
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const int i = cb * 32 + c4 * 4;
          tile_put(tile, lane, c4, make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]));
        }
        staged_for_tma(mask);
        if (lane == 0) {
          tma_store_3d(&ep.omap[0], tile, col0 + cb * 32, row0, z);
          tma_store_commit();
        }
      }
      return;
    }
    if (ep.tma) {
      // two regions: block cb is staged in region cb & 1 while the previous block's
      // store may still read the other
      const int z = ks * a.batch + bz;
#pragma unroll
      for (int cb = 0; cb < CPW / BW; ++cb) {
        if (col0 + cb * BW >= a.N) break;
        float4 *reg = region_ptr(tile, BW, cb & 1);
        // a tile's first block waits for every earlier store (the previous tile may
        // have ended in either region)
        if (cb == 0) store_reads_done<0>(lane, mask);
        else store_reads_done<1>(lane, mask);
#pragma unroll
        for (int c4 = 0; c4 < BW / 4; ++c4) {
          const int i = cb * BW + c4 * 4;
          region_put(reg, BW, lane, c4, make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]));
        }
        staged_for_tma(mask);
        if (lane == 0) {
          tma_store_3d(&ep.omap[0], reg, col0 + cb * BW, row0, z);
          tma_store_commit();
        }
      }
      return;
    }
    float *base = a.C + (int64_t)ks * a.split_stride + (int64_t)bz * a.strideC +
                  (int64_t)row0 * a.ldc + col0;
    const bool vec = ((a.ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.C) & 15) == 0) &&
                     ((a.strideC & 3) == 0) && ((a.split_stride & 3) == 0);
#pragma unroll
    for (int cb = 0; cb < CPW / BW; ++cb) {
      const int cols = min(BW, a.N - col0 - cb * BW);
      if (cols <= 0) break;
#pragma unroll
      for (int c4 = 0; c4 < BW / 4; ++c4) {
        const int i = cb * BW + c4 * 4;
        tile_put(tile, lane, c4, make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]));
      }
      __syncwarp(mask);
      tile_store<BW>(tile, base + cb * BW, a.ldc, rows, cols, vec, lane);
      __syncwarp(mask);
    }
  }
};

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// The TF32 remainder of x, the arithmetic of the remainder pass (lo_kernel): x minus x
// with its 13 low mantissa bits cleared (exact), rounded to the nearest TF32 value,
// ties to even; an Inf or NaN difference passes through. An operand split here
// therefore multiplies bit for bit as one whose remainder plane was written there.
__device__ __forceinline__ float tf32_remainder(float a) {
  uint32_t u = __float_as_uint(__fsub_rn(a, __uint_as_float(__float_as_uint(a) & 0xffffe000u)));
  if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0xfffu + ((u >> 13) & 1u)) & 0xffffe000u;
  return __uint_as_float(u);
}

__device__ __forceinline__ float4 lds_f4(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(a)
               : "memory");
  return v;
}

__device__ __forceinline__ void sts_f4(uint32_t a, float4 v) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

// One warp's share of a stage's remainders: float4s [f0, f0 + 32 * PER) of the stage's
// raw tiles taken as one run (A's A_N4 float4s, then B's, B_OFF bytes into the stage),
// PER per lane and 32 consecutive float4s per access; each remainder goes to the same
// offset in its tile's remainder slot (A_LO or B_LO bytes after the raw tile), the
// swizzled layout in which TMA would have written the remainder plane.
template <int PER, int A_N4, int B_OFF, int A_LO, int B_LO>
__device__ __forceinline__ void split_share(uint32_t stage, int f0, int lane) {
  float4 v[PER];
  uint32_t dst[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int f = f0 + j * 32 + lane;
    const uint32_t src = f < A_N4 ? stage + (uint32_t)f * 16u : stage + (uint32_t)B_OFF + (uint32_t)(f - A_N4) * 16u;
    dst[j] = src + (f < A_N4 ? (uint32_t)A_LO : (uint32_t)B_LO);
    v[j] = lds_f4(src);
  }
#pragma unroll
  for (int j = 0; j < PER; ++j)
    sts_f4(dst[j], make_float4(tf32_remainder(v[j].x), tf32_remainder(v[j].y), tf32_remainder(v[j].z),
                               tf32_remainder(v[j].w)));
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
// buffers; warps 4-11 fold each finished chunk into fp32 registers.
// Per tile width TBN (output columns per tile): 256 for wide products, 64 or 16 for
// narrow ones (a 16-wide output layer would otherwise compute 256 columns for 16).
// Narrow tiles use more stages of smaller k-tiles, within the same ~192 KB.
template <int TBN>
struct TileCfg {
  static constexpr int B_BYTES = TBN * BK * 4;
  static constexpr int STAGE = 2 * TILE_A_BYTES + 2 * B_BYTES;
  static constexpr int NSTAGE = TBN == BN ? STAGES : (192 * 1024) / STAGE;
  static constexpr int TMEM = TBN < 32 ? 32 : TBN;  // TMEM columns per accumulator buffer
  static constexpr int CPW = TBN / 2;               // columns per epilogue warp
  static_assert(TBN == 256 || TBN == 64 || TBN == 16, "tile width");
};

// Add CPW accumulator columns of this warp's TMEM lanes, from `taddr`, into acc.
template <int CPW>
__device__ __forceinline__ void promote_cols(uint32_t taddr, float (&acc)[CPW]) {
  if constexpr (CPW >= 64) {
    // two 32-column loads in flight per wait
#pragma unroll
    for (int c0 = 0; c0 < CPW; c0 += 64) {
      uint32_t r0[32], r1[32];
      tmem_ld_32x32b_x32_async(taddr + (uint32_t)c0, r0);
      tmem_ld_32x32b_x32_async(taddr + (uint32_t)(c0 + 32), r1);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[c0 + i] = __fadd_rn(acc[c0 + i], __uint_as_float(r0[i]));
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[c0 + 32 + i] = __fadd_rn(acc[c0 + 32 + i], __uint_as_float(r1[i]));
    }
  } else if constexpr (CPW >= 32) {
#pragma unroll
    for (int c0 = 0; c0 < CPW; c0 += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(taddr + (uint32_t)c0, r);
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[c0 + i] = __fadd_rn(acc[c0 + i], __uint_as_float(r[i]));
    }
  } else {
    static_assert(CPW == 8, "columns per warp");
    uint32_t r[8];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], __uint_as_float(r[i]));
  }
}

// A_MN / B_MN: the operand is MN-major in global and shared memory (B is K-major
// whenever TBN < 256).
template <bool A_MN, bool B_MN, int TBN, class EPI, bool SPLIT = false>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_3xtf32_kernel(const __grid_constant__ CUtensorMap mapAh,
                       const __grid_constant__ CUtensorMap mapAl,
                       const __grid_constant__ CUtensorMap mapBh,
                       const __grid_constant__ CUtensorMap mapBl, GemmArgs args,
                       const __grid_constant__ EpiParams ep) {
  grid_dependency_wait();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  using T = TileCfg<TBN>;
  constexpr int STAGES = T::NSTAGE;
  constexpr int STAGE_BYTES = T::STAGE;
  constexpr int TILE_B_BYTES = T::B_BYTES;
  constexpr int TMEM_COLS = T::TMEM;
  constexpr int CPW = T::CPW;
  // SPLIT shares of a stage's float4s: warps 2-3 SPLIT_SHARE_CTRL each, then each
  // epilogue warp SPLIT_SHARE_EPI
  constexpr int SPLIT_A_N4 = TILE_A_BYTES / 16;
  constexpr int SPLIT_SHARE_EPI = (SPLIT_A_N4 + TILE_B_BYTES / 16 - 2 * SPLIT_SHARE_CTRL) / NUM_EPI_WARPS;
  static_assert(!SPLIT || (SPLIT_SHARE_EPI % 32 == 0 && 2 * SPLIT_SHARE_CTRL + NUM_EPI_WARPS * SPLIT_SHARE_EPI ==
                                                            SPLIT_A_N4 + TILE_B_BYTES / 16),
                "the shares cover the stage");
  static_assert(TBN == BN || !B_MN, "narrow tiles read B K-major");
  static_assert(!SPLIT || TBN == BN, "remainder tiles in shared memory: full-width tiles only");
  __shared__ __align__(8) uint64_t full_bar[STAGES];   // stage ready for the MMAs
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t raw_full[SPLIT ? STAGES : 1];  // SPLIT: raw tiles landed
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ __align__(8) uint64_t drain_bar;  // MMAs issued before an abort, completed
  __shared__ __align__(8) uint64_t epi_bar[NUM_EPI_WARPS];  // epilogue loads into the staging tiles
  __shared__ uint32_t tmem_base_slot;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  constexpr uint32_t kIdesc = make_idesc(BM, TBN, A_MN, B_MN);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], SPLIT ? NUM_SPLIT_WARPS : 1);
      mbar_init(&empty_bar[s], 1);
      if constexpr (SPLIT) mbar_init(&raw_full[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], NUM_EPI_WARPS);  // one arrival per epilogue warp
    }
    mbar_init(&drain_bar, 1);
    for (int w = 0; w < NUM_EPI_WARPS; ++w) mbar_init(&epi_bar[w], 1);
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

  // registers rebalanced per warpgroup (setmaxnreg at the top of each warpgroup's
  // branch, so the compiler allocates each role within its share)
  if (warp < EPI_WARP0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
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
            const int k0 = kb + kt * BK;
            if constexpr (SPLIT) {  // the raw tiles only; the splitter warps add the remainders
              mbar_expect_tx(&raw_full[s], TILE_A_BYTES + TILE_B_BYTES);
              load_operand<A_MN, BM>(stage_ptr(s, 0), &mapAh, &raw_full[s], k0, mb * BM, bz, args.wide & 1);
              load_operand<B_MN, TBN>(stage_ptr(s, 2), &mapBh, &raw_full[s], k0, nb * TBN, bz, args.wide & 4);
            } else {
              mbar_expect_tx(&full_bar[s], STAGE_BYTES);
              load_operand<A_MN, BM>(stage_ptr(s, 0), &mapAh, &full_bar[s], k0, mb * BM, bz, args.wide & 1);
              load_operand<A_MN, BM>(stage_ptr(s, 1), &mapAl, &full_bar[s], k0, mb * BM, bz, args.wide & 2);
              load_operand<B_MN, TBN>(stage_ptr(s, 2), &mapBh, &full_bar[s], k0, nb * TBN, bz, args.wide & 4);
              load_operand<B_MN, TBN>(stage_ptr(s, 3), &mapBl, &full_bar[s], k0, nb * TBN, bz, args.wide & 8);
            }
          }
        }
        if (!ok) {
          atomicCAS(args.err, kErrNone, kErrTimeoutEmpty);
          abort_flag = 1;
          // drain: wait (bounded) for the loads of the last STAGES issued k-tiles
          for (int i = (it > STAGES ? it - STAGES : 0); i < it; ++i)
            mbar_drain(SPLIT ? &raw_full[i % STAGES] : &full_bar[i % STAGES], (i / STAGES) & 1);
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
                const uint64_t dah = operand_desc<A_MN>(a_hi, kk), dal = operand_desc<A_MN>(a_lo, kk);
                const uint64_t dbh = operand_desc<B_MN>(b_hi, kk), dbl = operand_desc<B_MN>(b_lo, kk);
                const uint32_t first = (kt == kt0 && kk == 0) ? 0u : 1u;
                umma_tf32(d_tmem, dal, dbh, kIdesc, first);  // lo * hi
                umma_tf32(d_tmem, dah, dbl, kIdesc, 1u);     // hi * lo
                umma_tf32(d_tmem, dah, dbh, kIdesc, 1u);     // hi * hi (largest term last)
              }
              umma_commit(&empty_bar[s]);
            }
            if (ok) umma_commit(&acc_full[b]);
          }
        }
        if (!ok) {
          atomicCAS(args.err, kErrNone, kErrTimeoutFull);
          abort_flag = 1;
          // the MMAs already issued complete before TMEM is freed (bounded)
          umma_commit(&drain_bar);
          mbar_drain(&drain_bar, 0);
        }
      }
    } else if constexpr (SPLIT) {
      // ------------------------------------------------------ remainder tiles (warps 2-3)
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < args.num_tiles; t += gridDim.x) {
        int mb, nb, bz, ks, kb;
        decode_tile(t, args, mb, nb, bz, ks);
        const int nk = unit_k_tiles(args, ks, kb);
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = it % STAGES;
          // every lane waits (bounded) and the warp leaves together if any lane gave up
          if (!__all_sync(0xffffffffu, mbar_wait(&raw_full[s], (it / STAGES) & 1, &abort_flag))) {
            ok = false;
            break;
          }
          split_share<SPLIT_SHARE_CTRL / 32, SPLIT_A_N4, 2 * TILE_A_BYTES, TILE_A_BYTES, TILE_B_BYTES>(
              smem_u32(stage_ptr(s, 0)), (warp - 2) * SPLIT_SHARE_CTRL, lane);
          // the remainder tiles, written through the generic proxy, are made visible to
          // the tensor cores' reads before the stage is handed over
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive(&full_bar[s]);
        }
      }
      if (!ok) {
        if (lane == 0) atomicCAS(args.err, kErrNone, kErrTimeoutSplit);
        abort_flag = 1;
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_EPI));
    // ------------------------------------------------------ promotion + epilogue (warps 4..11)
    const int q = warp & 3;                     // TMEM lane quarter this warp may access
    const int half = (warp - EPI_WARP0) >> 2;   // which half of the tile's columns
    float4 *epi_tile = reinterpret_cast<float4 *>(smem + (size_t)STAGES * STAGE_BYTES +
                                                  (size_t)(warp - EPI_WARP0) * EPI_TILE_BYTES);
    EpiSync epi_sync{&epi_bar[warp - EPI_WARP0], 0u, 0, &abort_flag};
    int cc = 0;
    bool ok = true;
    // SPLIT: this warp's share of the remainders, k-tile by k-tile (global index sit),
    // kept up to the end of the chunk after the one it promotes next
    int sit = 0, it_base = 0;
    for (int t = blockIdx.x; ok && t < args.num_tiles; t += gridDim.x) {
      int mb, nb, bz, ks, kb;
      decode_tile(t, args, mb, nb, bz, ks);
      const int num_k = unit_k_tiles(args, ks, kb);
      int next_first = 0;  // SPLIT: k-tiles in the first chunk of this CTA's next tile
      if (SPLIT && t + (int)gridDim.x < args.num_tiles) {
        int mb2, nb2, bz2, ks2, kb2;
        decode_tile(t + (int)gridDim.x, args, mb2, nb2, bz2, ks2);
        const int nk2 = unit_k_tiles(args, ks2, kb2);
        next_first = nk2 < KCHUNK ? nk2 : KCHUNK;
      }
      EPI::template prefetch<CPW>(args, ep, bz, mb * BM + q * 32 + lane, nb * TBN + half * CPW);
      float acc[CPW];
#pragma unroll
      for (int i = 0; i < CPW; ++i) acc[i] = 0.0f;
      for (int kt0 = 0; kt0 < num_k; kt0 += KCHUNK, ++cc) {
        const int b = cc & 1;
        if constexpr (SPLIT) {
          const int target = it_base + (kt0 + KCHUNK < num_k ? (kt0 + 2 * KCHUNK < num_k ? kt0 + 2 * KCHUNK : num_k)
                                                              : num_k + next_first);
          for (; ok && sit < target; ++sit) {
            const int s = sit % STAGES;
            if (!__all_sync(0xffffffffu, mbar_wait(&raw_full[s], (sit / STAGES) & 1, &abort_flag))) {
              if (lane == 0) atomicCAS(args.err, kErrNone, kErrTimeoutSplit);
              abort_flag = 1;
              ok = false;
              break;
            }
            split_share<SPLIT_SHARE_EPI / 32, SPLIT_A_N4, 2 * TILE_A_BYTES, TILE_A_BYTES, TILE_B_BYTES>(
                smem_u32(stage_ptr(s, 0)), 2 * SPLIT_SHARE_CTRL + (warp - EPI_WARP0) * SPLIT_SHARE_EPI, lane);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&full_bar[s]);
          }
          if (!ok) break;
        }
        // the epilogue's first input block, requested while the tile's last chunk is
        // still computed
        if (kt0 + KCHUNK >= num_k)
          EPI::template before_last<CPW>(args, ep, bz, mb * BM + q * 32 + lane, nb * TBN + half * CPW, epi_tile,
                                         epi_sync);
        if (!mbar_wait(&acc_full[b], (cc >> 1) & 1, &abort_flag)) {
          if (lane == 0) atomicCAS(args.err, kErrNone, kErrTimeoutAcc);
          abort_flag = 1;
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t taddr = tmem_base + (uint32_t)(b * TMEM_COLS + half * CPW) +
                               ((uint32_t)(q * 32) << 16);
        promote_cols<CPW>(taddr, acc);
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();  // the whole warp has read the buffer: one arrival for it
        if (lane == 0) mbar_arrive(&acc_empty[b]);
      }
      if (!ok) break;
      EPI::template store<CPW>(args, ep, ks, bz, mb * BM + q * 32 + lane, nb * TBN + half * CPW, acc,
                               epi_tile, epi_sync);
      it_base += num_k;
    }
    epi_settle(epi_sync);
    tma_stores_drain(ep, lane);
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

// ---------------------------------------------------------------- 2-SM (CTA pair) variant
//
// A cluster of two CTAs computes a 256 x 256 output tile with
// tcgen05.mma.cta_group::2: each CTA holds 128 rows of A and 128 rows (N) of B per
// stage, the leader CTA (rank 0) issues the MMAs, the tensor cores read the peer's
// half of each operand from its shared memory, and each CTA's TMEM receives its 128
// rows x 256 columns. Per MMA a CTA reads half of B from its own shared memory
// instead of all of it, and loads a third fewer bytes per k-tile: less shared-memory
// and L2 traffic, and energy, per product. Protocol: both CTAs' TMA loads complete
// their bytes on the leader's full barrier (which the leader's producer armed for the
// pair's bytes); the leader's commits multicast to both CTAs' empty and acc_full
// barriers; the peer's epilogue threads arrive on the leader's acc_empty barriers.
// TMEM is allocated and freed with cta_group::2 by warp 1 of both CTAs. Every wait is
// bounded as in the single-CTA kernel, and both CTAs meet at a cluster barrier before
// freeing TMEM and exiting.
constexpr int PAIR_STAGES = 6;
constexpr int PAIR_TILE_BYTES = BM * BK * 4;             // 128 rows of A or B: 8 KB
constexpr int PAIR_STAGE_BYTES = 4 * PAIR_TILE_BYTES;    // A_hi, A_lo, B_hi, B_lo: 32 KB

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// Shared-memory address of the same variable in the cluster's CTA 0.
__device__ __forceinline__ uint32_t in_leader(const void *p) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(r) : "r"(smem_u32(p)));
  return r;
}

__device__ __forceinline__ void tma_load_3d_pair(void *dst, const CUtensorMap *map, uint32_t bar,
                                                 int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d_pair(void *dst, const CUtensorMap *map, uint32_t bar,
                                                 int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// load_operand for a CTA of a pair: 128 rows, bytes completed on the leader's barrier.
template <bool MN>
__device__ __forceinline__ void load_operand_pair(uint8_t *dst, const CUtensorMap *map, uint32_t bar,
                                                  int k0, int row0, int bz, bool wide) {
  if constexpr (MN) {
    if (wide) {
      tma_load_4d_pair(dst, map, bar, 0, k0, row0 / MN_CHUNK, bz);
    } else {
#pragma unroll
      for (int j = 0; j < BM / MN_CHUNK; ++j)
        tma_load_3d_pair(dst + j * MN_CHUNK_BYTES, map, bar, row0 + j * MN_CHUNK, k0, bz);
    }
  } else {
    tma_load_3d_pair(dst, map, bar, k0, row0, bz);
  }
}

__device__ __forceinline__ void umma_tf32_pair(uint32_t tmem_d, uint64_t a, uint64_t b,
                                               uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}

// Arrive on the barrier at this offset in both CTAs of the pair when the MMAs issued
// so far have completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], m;\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

// Arrive on the leader's barrier at this offset when the MMAs issued so far have completed.
__device__ __forceinline__ void umma_commit_leader(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 1;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], m;\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

template <bool A_MN, bool B_MN, class EPI, bool SPLIT = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap mapAh,
                     const __grid_constant__ CUtensorMap mapAl,
                     const __grid_constant__ CUtensorMap mapBh,
                     const __grid_constant__ CUtensorMap mapBl, GemmArgs args,
                     const __grid_constant__ EpiParams ep) {
  grid_dependency_wait();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full_bar[PAIR_STAGES];
  __shared__ __align__(8) uint64_t empty_bar[PAIR_STAGES];
  __shared__ __align__(8) uint64_t raw_full[SPLIT ? PAIR_STAGES : 1];  // SPLIT: this CTA's raw tiles landed
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ __align__(8) uint64_t drain_bar;  // MMAs issued before an abort, completed
  __shared__ __align__(8) uint64_t epi_bar[NUM_EPI_WARPS];  // epilogue loads into the staging tiles
  __shared__ uint32_t tmem_base_slot;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  constexpr uint32_t kIdesc = make_idesc(2 * BM, BN, A_MN, B_MN);

  if (threadIdx.x == 0) {
    for (int s = 0; s < PAIR_STAGES; ++s) {
      // SPLIT: one arrival per splitter warp of both CTAs (in the leader's barrier)
      mbar_init(&full_bar[s], SPLIT ? 2 * NUM_SPLIT_WARPS : 1);
      mbar_init(&empty_bar[s], 1);
      if constexpr (SPLIT) mbar_init(&raw_full[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * NUM_EPI_WARPS);  // one arrival per epilogue warp of both CTAs
    }
    mbar_init(&drain_bar, 1);
    for (int w = 0; w < NUM_EPI_WARPS; ++w) mbar_init(&epi_bar[w], 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_map(&mapAh);
    prefetch_map(&mapAl);
    prefetch_map(&mapBh);
    prefetch_map(&mapBl);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_base_slot)),
                 "r"(2 * TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_base = tmem_base_slot;

  auto stage_ptr = [&](int s, int which) -> uint8_t * {
    return smem + (size_t)s * PAIR_STAGE_BYTES + (size_t)which * PAIR_TILE_BYTES;
  };

  // registers rebalanced per warpgroup (setmaxnreg at the top of each warpgroup's
  // branch, so the compiler allocates each role within its share)
  if (warp < EPI_WARP0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
    if (warp == 0) {
      if (lane == 0) {
        // ------------------------------------------------------ TMA producer (both CTAs)
        int it = 0;
        bool ok = true;
        // With tile_sync the producers of all pairs start each tile together: pairs that
        // drift apart over K miss in L2 on the operand rows and columns they share (the
        // main loop's traffic turns L2 over in ~15 us), and in lockstep a launch of
        // [65536,4096]x[4096,4096]^T read 10.7 instead of 16.4 GB from DRAM and ran 4 %
        // faster. `need` counts the arrivals due by this boundary: two per pair owning a
        // tile there, so the last partial wave does not wait for pairs that are done.
        int tj = 0;
        unsigned int need = 0;
        for (int t = pair; ok && t < args.num_tiles; t += npairs, ++tj) {
          if (args.tile_sync && tj > 0) {
            const int owners = args.num_tiles - tj * npairs;
            need += 2u * (unsigned int)(owners < npairs ? owners : npairs);
            atomicAdd(args.tile_sync, 1u);
            const uint64_t w0 = globaltimer();
            while (*reinterpret_cast<volatile unsigned int *>(args.tile_sync) < need &&
                   globaltimer() - w0 < kTileSyncNs) {
            }
          }
          int mb, nb, bz, ks, kb;
          decode_tile(t, args, mb, nb, bz, ks);
          const int nk = unit_k_tiles(args, ks, kb);
          const int row_a = mb * 2 * BM + (int)rank * BM, row_b = nb * BN + (int)rank * BM;
          for (int kt = 0; kt < nk; ++kt, ++it) {
            const int s = it % PAIR_STAGES;
            const uint32_t round = it / PAIR_STAGES;
            if (it >= PAIR_STAGES && !mbar_wait(&empty_bar[s], (round - 1) & 1, &abort_flag)) {
              ok = false;
              break;
            }
            const int k0 = kb + kt * BK;
            if constexpr (SPLIT) {
              // this CTA's raw tiles, completed on its own barrier; its splitter warps add
              // the remainders and report to the leader
              mbar_expect_tx(&raw_full[s], 2 * PAIR_TILE_BYTES);
              load_operand<A_MN, BM>(stage_ptr(s, 0), &mapAh, &raw_full[s], k0, row_a, bz, args.wide & 1);
              load_operand<B_MN, BM>(stage_ptr(s, 2), &mapBh, &raw_full[s], k0, row_b, bz, args.wide & 4);
            } else {
              if (leader) mbar_expect_tx(&full_bar[s], 2 * PAIR_STAGE_BYTES);
              const uint32_t fb = in_leader(&full_bar[s]);
              load_operand_pair<A_MN>(stage_ptr(s, 0), &mapAh, fb, k0, row_a, bz, args.wide & 1);
              load_operand_pair<A_MN>(stage_ptr(s, 1), &mapAl, fb, k0, row_a, bz, args.wide & 2);
              load_operand_pair<B_MN>(stage_ptr(s, 2), &mapBh, fb, k0, row_b, bz, args.wide & 4);
              load_operand_pair<B_MN>(stage_ptr(s, 3), &mapBl, fb, k0, row_b, bz, args.wide & 8);
            }
          }
        }
        if (!ok) {
          atomicCAS(args.err, kErrNone, kErrTimeoutEmpty);
          abort_flag = 1;
          if (SPLIT || leader) {  // drain (bounded): the last PAIR_STAGES k-tiles' loads
            for (int i = (it > PAIR_STAGES ? it - PAIR_STAGES : 0); i < it; ++i)
              mbar_drain(SPLIT ? &raw_full[i % PAIR_STAGES] : &full_bar[i % PAIR_STAGES], (i / PAIR_STAGES) & 1);
          }
        }
      }
    } else if (warp == 1) {
      if (lane == 0 && leader) {
        // ------------------------------------------------------ MMA issuer (leader only)
        int it = 0, cc = 0;
        bool ok = true;
        for (int t = pair; ok && t < args.num_tiles; t += npairs) {
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
              const int s = it % PAIR_STAGES;
              if (!(SPLIT ? mbar_wait_cluster(&full_bar[s], (it / PAIR_STAGES) & 1, &abort_flag)
                          : mbar_wait(&full_bar[s], (it / PAIR_STAGES) & 1, &abort_flag))) {
                ok = false;
                break;
              }
              asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
              const uint32_t a_hi = smem_u32(stage_ptr(s, 0)), a_lo = smem_u32(stage_ptr(s, 1));
              const uint32_t b_hi = smem_u32(stage_ptr(s, 2)), b_lo = smem_u32(stage_ptr(s, 3));
  #pragma unroll
              for (int kk = 0; kk < BK / UMMA_K; ++kk) {
                const uint64_t dah = operand_desc<A_MN>(a_hi, kk), dal = operand_desc<A_MN>(a_lo, kk);
                const uint64_t dbh = operand_desc<B_MN>(b_hi, kk), dbl = operand_desc<B_MN>(b_lo, kk);
                const uint32_t first = (kt == kt0 && kk == 0) ? 0u : 1u;
                umma_tf32_pair(d_tmem, dal, dbh, kIdesc, first);  // lo * hi
                umma_tf32_pair(d_tmem, dah, dbl, kIdesc, 1u);     // hi * lo
                umma_tf32_pair(d_tmem, dah, dbh, kIdesc, 1u);     // hi * hi
              }
              umma_commit_pair(&empty_bar[s]);
            }
            if (ok) umma_commit_pair(&acc_full[b]);
          }
        }
        if (!ok) {
          atomicCAS(args.err, kErrNone, kErrTimeoutFull);
          abort_flag = 1;
          // the MMAs already issued (writing both CTAs' TMEM) complete before the pair
          // meets to free TMEM (bounded)
          umma_commit_leader(&drain_bar);
          mbar_drain(&drain_bar, 0);
        }
      }
    } else if constexpr (SPLIT) {
      // ------------------------------------------------------ remainder tiles (warps 2-3, both CTAs)
      int it = 0;
      bool ok = true;
      for (int t = pair; ok && t < args.num_tiles; t += npairs) {
        int mb, nb, bz, ks, kb;
        decode_tile(t, args, mb, nb, bz, ks);
        const int nk = unit_k_tiles(args, ks, kb);
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = it % PAIR_STAGES;
          if (!__all_sync(0xffffffffu, mbar_wait(&raw_full[s], (it / PAIR_STAGES) & 1, &abort_flag))) {
            ok = false;
            break;
          }
          split_share<SPLIT_SHARE_CTRL / 32, PAIR_TILE_BYTES / 16, 2 * PAIR_TILE_BYTES, PAIR_TILE_BYTES,
                      PAIR_TILE_BYTES>(smem_u32(stage_ptr(s, 0)), (warp - 2) * SPLIT_SHARE_CTRL, lane);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            if (leader) mbar_arrive(&full_bar[s]);
            else mbar_arrive_remote(in_leader(&full_bar[s]));
          }
        }
      }
      if (!ok) {
        if (lane == 0) atomicCAS(args.err, kErrNone, kErrTimeoutSplit);
        abort_flag = 1;
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_EPI));
    // ------------------------------------------------------ promotion + epilogue (warps 4..11)
    const int q = warp & 3;
    const int half = (warp - EPI_WARP0) >> 2;
    float4 *epi_tile = reinterpret_cast<float4 *>(smem + (size_t)PAIR_STAGES * PAIR_STAGE_BYTES +
                                                  (size_t)(warp - EPI_WARP0) * EPI_TILE_BYTES);
    EpiSync epi_sync{&epi_bar[warp - EPI_WARP0], 0u, 0, &abort_flag};
    const uint32_t acc_empty_leader0 = in_leader(&acc_empty[0]), acc_empty_leader1 = in_leader(&acc_empty[1]);
    int cc = 0;
    bool ok = true;
    // SPLIT: this warp's share of the remainders, as in the single-CTA kernel; the
    // leader's full barrier counts the ten warps of both CTAs
    constexpr int SPLIT_SHARE_EPI = (2 * (PAIR_TILE_BYTES / 16) - 2 * SPLIT_SHARE_CTRL) / NUM_EPI_WARPS;
    static_assert(SPLIT_SHARE_EPI % 32 == 0, "whole float4s per lane");
    int sit = 0, it_base = 0;
    for (int t = pair; ok && t < args.num_tiles; t += npairs) {
      int mb, nb, bz, ks, kb;
      decode_tile(t, args, mb, nb, bz, ks);
      const int num_k = unit_k_tiles(args, ks, kb);
      int next_first = 0;
      if (SPLIT && t + npairs < args.num_tiles) {
        int mb2, nb2, bz2, ks2, kb2;
        decode_tile(t + npairs, args, mb2, nb2, bz2, ks2);
        const int nk2 = unit_k_tiles(args, ks2, kb2);
        next_first = nk2 < KCHUNK ? nk2 : KCHUNK;
      }
      EPI::template prefetch<128>(args, ep, bz, mb * 2 * BM + (int)rank * BM + q * 32 + lane,
                                  nb * BN + half * 128);
      float acc[128];
#pragma unroll
      for (int i = 0; i < 128; ++i) acc[i] = 0.0f;
      for (int kt0 = 0; kt0 < num_k; kt0 += KCHUNK, ++cc) {
        const int b = cc & 1;
        if constexpr (SPLIT) {
          const int target = it_base + (kt0 + KCHUNK < num_k ? (kt0 + 2 * KCHUNK < num_k ? kt0 + 2 * KCHUNK : num_k)
                                                              : num_k + next_first);
          for (; ok && sit < target; ++sit) {
            const int s = sit % PAIR_STAGES;
            if (!__all_sync(0xffffffffu, mbar_wait(&raw_full[s], (sit / PAIR_STAGES) & 1, &abort_flag))) {
              if (lane == 0) atomicCAS(args.err, kErrNone, kErrTimeoutSplit);
              abort_flag = 1;
              ok = false;
              break;
            }
            split_share<SPLIT_SHARE_EPI / 32, PAIR_TILE_BYTES / 16, 2 * PAIR_TILE_BYTES, PAIR_TILE_BYTES,
                        PAIR_TILE_BYTES>(smem_u32(stage_ptr(s, 0)),
                                         2 * SPLIT_SHARE_CTRL + (warp - EPI_WARP0) * SPLIT_SHARE_EPI, lane);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
              if (leader) mbar_arrive(&full_bar[s]);
              else mbar_arrive_remote(in_leader(&full_bar[s]));
            }
          }
          if (!ok) break;
        }
        if (kt0 + KCHUNK >= num_k)
          EPI::template before_last<128>(args, ep, bz, mb * 2 * BM + (int)rank * BM + q * 32 + lane,
                                         nb * BN + half * 128, epi_tile, epi_sync);
        if (!mbar_wait(&acc_full[b], (cc >> 1) & 1, &abort_flag)) {
          if (lane == 0) atomicCAS(args.err, kErrNone, kErrTimeoutAcc);
          abort_flag = 1;
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t taddr = tmem_base + (uint32_t)(b * TMEM_COLS + half * 128) +
                               ((uint32_t)(q * 32) << 16);
        promote_cols<128>(taddr, acc);
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();  // the whole warp has read the buffer: one arrival for it
        if (lane == 0) {
          if (leader) mbar_arrive(&acc_empty[b]);
          else mbar_arrive_remote(b ? acc_empty_leader1 : acc_empty_leader0);
        }
      }
      if (!ok) break;
      EPI::template store<128>(args, ep, ks, bz, mb * 2 * BM + (int)rank * BM + q * 32 + lane,
                               nb * BN + half * 128, acc, epi_tile, epi_sync);
      it_base += num_k;
    }
    epi_settle(epi_sync);
    tma_stores_drain(ep, lane);
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_sync_all();  // neither CTA frees TMEM or exits while the pair may still use it
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(2 * TMEM_COLS)
                 : "memory");
  }
}


}  // namespace fz_gemm_dev
