// fp32 GEMM in 3xTF32 on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// C[b] = op(A[b]) @ op(B[b]), row-major fp32 in and out.
//
// 3xTF32: x = hi + lo with hi = x with its 13 low mantissa bits cleared (exact in
// TF32) and lo = x - hi (exact in fp32); C = Ah*Bh + Ah*Bl + Al*Bh. The kind::tf32
// MMA ignores the 13 low mantissa bits of its fp32 inputs, so every operand is its
// own hi plane and only its lo plane is written (lo_kernel, same layout as the
// operand). Operands are read in the layout they are stored in: K-major ([M, K] for
// A, [N, K] for B; 64-byte swizzled boxes of 16 k) or MN-major ([K, M] / [K, N], the
// weight-gradient case where K is the batch; boxes of 32 rows x 16 k in the 128-byte
// swizzle with 32-byte atoms), selected per operand by template and the MMA's major bits.
//
// Main kernel, persistent (one CTA per SM walking 128 x 256 output tiles in grouped
// order), warp-specialised, 384 threads (registers rebalanced per warpgroup with
// setmaxnreg: warps 0-3 at 56, the epilogue warpgroups at 224):
//   warp 0     TMA producer: per k-tile of BK = 16 loads A_hi, A_lo (128 x 16) and
//              B_hi, B_lo (256 x 16) into a 4-stage ring of 48 KB
//   warp 1     allocates 2 x 256 TMEM columns; one lane issues, per 8-wide k-step,
//              tcgen05.mma.kind::tf32 lo*hi, hi*lo, hi*hi, and tcgen05.commit frees
//              each stage. The K range is cut into chunks of 128; each chunk
//              accumulates from zero into one of the two TMEM buffers.
//   warps 4-11 promotion and epilogue: two warps per TMEM lane quarter, each owning
//              128 of the 256 columns, tcgen05.ld every finished chunk (two loads in
//              flight per wait) and add it into an fp32 register accumulator (IEEE
//              adds), then store C; one arrival per warp frees the buffer.
// The tensor core's own fp32 accumulation truncates, so its error grows with the
// number of MMAs folded into one accumulator, always toward zero (about 3e-5
// relative at K = 4096 when a whole tile accumulates in TMEM). Promoting every 128 of
// K bounds the bias to that of a 128-long chunk (about 1e-6; 2e-6 with chunks of 256,
// a bias that adds up over the layers of a network), and the TF32 remainder planes
// are rounded to nearest rather than truncated by the MMA. Double-buffered chunks let
// the MMAs run on while a chunk is promoted.
//
// Every mbarrier wait is bounded by a %globaltimer deadline (4 s); on expiry the kernel
// records an error code in the device's error word (read by fz_kernel_status), lets
// the MMAs and TMA loads it already issued complete (bounded), frees TMEM and
// returns, so a bad launch surfaces as an error instead of a hang.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstddef>
#include <cstring>
#include <mutex>
#include <sstream>
#include <string>
#include <unordered_map>
#include <vector>

#include "fz_common.cuh"

#include "fz_gemm_kernels.cuh"

namespace {

using namespace fz_gemm_dev;

// ---------------------------------------------------------------- split pass
__device__ __forceinline__ void split1(float x, float &hi, float &lo) {
  hi = __uint_as_float(__float_as_uint(x) & 0xffffe000u);
  lo = fzd::tf32_lo(x);
}

// src[b][r][k] at b*sb + r*ld + k (k the contiguous index: K for a K-major operand,
// M or N for an MN-major one). Writes the lo plane lo[b][r][k] (pitch kp, zero
// beyond K); the MMA reads src itself as hi. When src cannot be addressed by TMA
// (row pitch not a multiple of 16 bytes, or a broadcast batch), `hi` is non-null and
// receives a copy of src at pitch kp.
__global__ void __launch_bounds__(256) lo_kernel(const float *__restrict__ src, int64_t ld,
                                                 int64_t sb, int64_t rows, int64_t K, int64_t kp,
                                                 int64_t batch, float *__restrict__ lo,
                                                 float *__restrict__ hi) {
  pdl_wait();
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (!hi && ld == kp && K == kp && kp % 4 == 0 && (batch == 1 || sb == rows * kp) &&
      (((uintptr_t)src | (uintptr_t)lo) & 15) == 0) {
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

// Map over one operand plane, K-major ([batch, rows, K], K innermost) or MN-major
// ([batch, K, rows], rows innermost). TMA needs ld*4 and sb*4 to be multiples of 16
// bytes and the base 16-byte aligned; every box starts at an inner coordinate that
// is a multiple of 16 (K-major) or 32 (MN-major) elements, or at 0 (wide).
// K-major: 3D, box {BK, box_rows, 1}, 64-byte swizzle (128-byte for BK = 32).
// MN-major: 128-byte swizzle with 32-byte atoms. When ld is a multiple of 32 floats
// and the rows fill whole 32-row chunks (or the plane is one of ours, padded with
// zeros to its 32-float pitch), the map is "wide": 4D {32 rows, K, rows / 32
// chunks, batch} with a chunk stride of 128 bytes, so one box {32, BK, box_rows /
// 32, 1} lands the whole k-tile in the chunked layout and no read leaves a row's
// pitch. Otherwise 3D {rows, K, batch} with one box {32, BK, 1} per chunk, the TMA
// unit zero-filling past the rows. *wide reports which was made.
int make_map(CUtensorMap *map, const float *base, bool mn, int64_t rows, int64_t K, int64_t ld,
             int64_t sb, int64_t batch, int box_rows, bool padded, bool *wide) {
  if (batch == 1) sb = ld * (mn ? K : rows);
  *wide = mn && ld % MN_CHUNK == 0 && (rows % MN_CHUNK == 0 || padded);
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r;
  if (*wide) {
    cuuint64_t dims[4] = {(cuuint64_t)MN_CHUNK, (cuuint64_t)K,
                          (cuuint64_t)((rows + MN_CHUNK - 1) / MN_CHUNK), (cuuint64_t)batch};
    cuuint64_t strides[3] = {(cuuint64_t)(ld * 4), (cuuint64_t)(MN_CHUNK * 4), (cuuint64_t)(sb * 4)};
    cuuint32_t box[4] = {(cuuint32_t)MN_CHUNK, (cuuint32_t)BK, (cuuint32_t)(box_rows / MN_CHUNK), 1};
    r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void *)base, dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t dims[3] = {(cuuint64_t)(mn ? rows : K), (cuuint64_t)(mn ? K : rows), (cuuint64_t)batch};
    cuuint64_t strides[2] = {(cuuint64_t)(ld * 4), (cuuint64_t)(sb * 4)};
    cuuint32_t box[3] = {mn ? (cuuint32_t)MN_CHUNK : (cuuint32_t)BK,
                         mn ? (cuuint32_t)BK : (cuuint32_t)box_rows, 1};
    const CUtensorMapSwizzle sw = mn ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                 : SWIZZLE_BYTES == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                                        : CU_TENSOR_MAP_SWIZZLE_64B;
    r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void *)base, dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS)
    return fz::fail(FZ_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  return FZ_OK;
}

// Store map of an output: 3D {N, M, Z} over fp32 with row pitch ld and slice pitch sz,
// box {bw, 32, 1}: for bw = 32 the 128-byte swizzle of the staging tile's full-width
// layout (tile_put), else no swizzle (row-major staging regions). false when the
// layout is not one TMA can store (then the epilogue stores per thread).
bool make_out_map(CUtensorMap *map, float *base, int64_t N, int64_t M, int64_t Z, int64_t ld,
                  int64_t sz, int bw) {
  if (Z == 1) sz = ld * M;
  if (!base || ((uintptr_t)base & 15) || (ld * 4) % 16 || (sz * 4) % 16 || bw < 4) return false;
  cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)Z};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 4), (cuuint64_t)(sz * 4)};
  cuuint32_t box[3] = {(cuuint32_t)bw, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void *)base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  bw == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }


// Launch counters by schedule (fz_gemm_stats): CTA-pair launches, single-CTA launches,
// launches split over K, launches with a fused epilogue program compiled in.
std::atomic<int64_t> g_stat_pair{0}, g_stat_single{0}, g_stat_ksplit{0}, g_stat_epilogue{0};
std::atomic<int64_t> g_stat_split_here{0};  // launches deriving remainder tiles in shared memory

// Per-launch device timing of the main GEMM kernel (fz_gemm_timing): an event pair
// recorded around the launch on its stream. Events are pooled and reused.
struct TimedLaunch {
  fz_gemm_timing_rec rec;
  cudaEvent_t start, stop;
};
std::mutex g_timing_mu;
bool g_timing_on = false;
std::vector<TimedLaunch> g_timed;
std::vector<cudaEvent_t> g_event_pool;

cudaEvent_t pooled_event() {
  if (!g_event_pool.empty()) {
    cudaEvent_t e = g_event_pool.back();
    g_event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

// Brackets one main-kernel launch with an event pair while timing is on.
struct LaunchTimer {
  TimedLaunch t{};
  bool on = false;
  cudaStream_t s;
  LaunchTimer(int64_t batch, int64_t M, int64_t N, int64_t K, bool pair, bool epi, int splits,
              cudaStream_t stream)
      : s(stream) {
    std::lock_guard<std::mutex> lk(g_timing_mu);
    if (!g_timing_on || g_timed.size() >= FZ_GEMM_TIMING_MAX) return;
    t.rec = fz_gemm_timing_rec{batch, M, N, K, pair ? 1 : 0, epi ? 1 : 0, splits, 0.0f};
    t.start = pooled_event();
    t.stop = pooled_event();
    on = t.start && t.stop && cudaEventRecord(t.start, s) == cudaSuccess;
  }
  void done(int rc) {
    if (!on) return;
    std::lock_guard<std::mutex> lk(g_timing_mu);
    if (rc == FZ_OK && cudaEventRecord(t.stop, s) == cudaSuccess) {
      g_timed.push_back(t);
    } else {
      g_event_pool.push_back(t.start);
      g_event_pool.push_back(t.stop);
    }
  }
};

std::atomic<int> g_tile_mode{FZ_GEMM_TILES_AUTO};

// Counters for the producers' tile-boundary meetings (GemmArgs::tile_sync): per stream a
// ring of kSyncSlots zeroed words, one per launch in turn; the ring is zeroed again, in
// stream order behind every launch that used it, each time it wraps.
constexpr int kSyncSlots = 1024;
struct SyncRing {
  unsigned int *words = nullptr;
  int next = 0;
};
std::mutex g_sync_mu;
std::unordered_map<cudaStream_t, SyncRing> g_sync_rings;

int tile_sync_slot(cudaStream_t s, unsigned int **slot) {
  std::lock_guard<std::mutex> lk(g_sync_mu);
  SyncRing &r = g_sync_rings[s];
  if (!r.words) {
    FZ_CUDA(cudaMalloc((void **)&r.words, sizeof(unsigned int) * kSyncSlots));
    FZ_CUDA(cudaMemsetAsync(r.words, 0, sizeof(unsigned int) * kSyncSlots, s));
  } else if (r.next == kSyncSlots) {
    FZ_CUDA(cudaMemsetAsync(r.words, 0, sizeof(unsigned int) * kSyncSlots, s));
    r.next = 0;
  }
  *slot = r.words + r.next++;
  return FZ_OK;
}
// Where missing remainder planes come from (fz_gemm_set_split). AUTO takes the separate
// pass: deriving them in shared memory (the SPLIT kernels) measured slower on the sweep's
// products except 1024^3 (0.87x the time; batched 64x512^3 1.3x, 2048^3 1.25x, large
// products 1.5-1.9x), the main loop being bound by shared-memory traffic to which the
// split adds its reads and writes. The SPLIT kernels need no workspace, which callers
// short of memory can choose them for.
std::atomic<int> g_split_mode{FZ_GEMM_SPLIT_AUTO};
// Epilogue outputs through TMA bulk tensor stores where the layout allows (default);
// off: every output stored per thread (fz_gemm_set_tma_stores).
std::atomic<bool> g_tma_stores{true};

// Number of K splits for a GEMM of `tiles` output tiles. A split turns one tile
// into several units over K ranges (multiples of the 256-wide promotion chunk)
// whose fp32 partials are summed afterwards; it pays when the tiles fill the 148
// SMs poorly (weight gradients: few tiles, K = batch rows; small square products).
// Cost model in units of one tile's time per k: waves * K_per_unit, plus the
// partials' write and read at HBM speed.
int choose_splits(int64_t tiles, int64_t M, int64_t N, int64_t K, int64_t batch, int64_t workers) {
  const int64_t sms = workers;
  const double k_time = 2.65e-8;  // s per k of one 128x256 tile (3 TF32 MMAs at ~1.1 PFLOP/s per GPU)
  int best = 1;
  double best_t = 1e300;
  const int cand[] = {1, 2, 3, 4, 6, 8, 12, 16, 24, 32};
  for (int sp : cand) {
    const int64_t kps = sp == 1 ? K : round_up((K + sp - 1) / sp, (int64_t)BK * KSPLIT_GRAN);
    if (sp > 1 && kps < (int64_t)BK * KSPLIT_GRAN) break;
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

// One operand as the (hi, lo) planes the kernel reads, in the operand's own layout:
// outer rows of `inner` contiguous floats (K-major: rows = M or N, inner = K;
// MN-major: rows = K, inner = M or N).
struct Operand {
  bool mn;
  int64_t rows, inner;
  const float *hi;
  int64_t hi_ld, hi_sb;
  const float *lo;
  int64_t lo_ld, lo_sb;
  bool hi_padded = false, lo_padded = false;  // planes written here, zero-padded to their pitch
};

// The raw operand can serve as the hi plane when TMA can address it.
bool direct_hi(const float *src, int64_t ld, int64_t sb, int64_t batch) {
  return ld % 4 == 0 && ((uintptr_t)src & 15) == 0 && (batch == 1 || (sb > 0 && sb % 4 == 0));
}

// Workspace floats the operand needs: none when the caller supplied its lo plane
// and the operand is TMA-addressable; else a lo plane at a 16-byte pitch, plus a
// hi copy when the operand itself is not TMA-addressable.
int64_t workspace_floats(const Operand &o, const float *src, int64_t ld, int64_t sb,
                         const float *lo_given, int64_t batch) {
  const bool direct = direct_hi(src, ld, sb, batch);
  if (direct && lo_given) return 0;
  const int64_t plane = batch * o.rows * (o.mn ? round_up(o.inner, MN_CHUNK) : round_up(o.inner, 4));
  return plane * (direct ? 1 : 2);
}

// Point op at its hi and lo planes, writing into ws what the caller did not supply.
int prepare(const float *src, int64_t ld, int64_t sb, const float *lo_given, int64_t batch,
            float *ws, Operand *op, cudaStream_t s) {
  const bool direct = direct_hi(src, ld, sb, batch);
  if (batch == 1) sb = ld * op->rows;
  if (direct && lo_given) {
    op->hi = src;
    op->lo = lo_given;
    op->hi_ld = op->lo_ld = ld;
    op->hi_sb = op->lo_sb = sb;
    return FZ_OK;
  }
  // row pitch: 16 bytes for TMA; MN-major planes a multiple of 32 floats (wide map)
  const int64_t pitch = op->mn ? round_up(op->inner, MN_CHUNK) : round_up(op->inner, 4);
  const int64_t plane = batch * op->rows * pitch;
  float *lo = ws, *hi = direct ? nullptr : ws + plane;
  unsigned grid = fz::grid_for(plane / 4 + 1, 256, 8, 4);
  FZ_CUDA(fz::launch_pdl(lo_kernel, dim3(grid), dim3(256), 0, s, src, ld, sb, op->rows, op->inner, pitch, batch, lo, hi));
  FZ_CHECK_LAUNCH();
  op->lo = lo;
  op->lo_ld = pitch;
  op->lo_sb = op->rows * pitch;
  op->lo_padded = true;
  if (direct) {
    op->hi = src;
    op->hi_ld = ld;
    op->hi_sb = sb;
  } else {
    op->hi = hi;
    op->hi_ld = pitch;
    op->hi_sb = op->rows * pitch;
    op->hi_padded = true;
  }
  return FZ_OK;
}

// Dynamic shared memory of a kernel variant: stage ring, the epilogue warps' staging
// tiles and alignment slack (at most 225 KB of the 227 KB a CTA may use).
size_t smem_bytes(bool pair, int tbn) {
  size_t ring;
  if (pair) ring = (size_t)PAIR_STAGES * PAIR_STAGE_BYTES;
  else if (tbn == 16) ring = (size_t)TileCfg<16>::NSTAGE * TileCfg<16>::STAGE;
  else if (tbn == 64) ring = (size_t)TileCfg<64>::NSTAGE * TileCfg<64>::STAGE;
  else ring = (size_t)TileCfg<BN>::NSTAGE * TileCfg<BN>::STAGE;
  return ring + EPI_SMEM_BYTES + 1024;
}
static_assert((size_t)PAIR_STAGES * PAIR_STAGE_BYTES + EPI_SMEM_BYTES + 1024 <= 232448 &&
                  (size_t)TileCfg<BN>::NSTAGE * TileCfg<BN>::STAGE + EPI_SMEM_BYTES + 1024 <= 232448 &&
                  (size_t)TileCfg<64>::NSTAGE * TileCfg<64>::STAGE + EPI_SMEM_BYTES + 1024 <= 232448 &&
                  (size_t)TileCfg<16>::NSTAGE * TileCfg<16>::STAGE + EPI_SMEM_BYTES + 1024 <= 232448,
              "shared memory per CTA");

// The kernels split REG_LAUNCH registers per thread between their warpgroups with
// setmaxnreg (warpgroup 0 gives up what the epilogue warpgroups take). A kernel
// compiled to another count would make that split wrong, so it is refused here.
int check_kernel_registers(const void *fn) {
  cudaFuncAttributes fa{};
  FZ_CUDA(cudaFuncGetAttributes(&fa, fn));
  if (fa.numRegs != REG_LAUNCH)
    return fz::fail(FZ_ERR_CUDA, "GEMM kernel compiled to " + std::to_string(fa.numRegs) +
                                     " registers per thread; its warpgroup register split needs " +
                                     std::to_string(REG_LAUNCH));
  return FZ_OK;
}

template <bool A_MN, bool B_MN, int TBN, bool SPLIT = false>
int launch_gemm(const CUtensorMap &mAh, const CUtensorMap &mAl, const CUtensorMap &mBh,
                const CUtensorMap &mBl, const GemmArgs &ga, const EpiParams &ep, unsigned grid,
                bool pair, cudaStream_t s) {
  static bool attr_done[2][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const size_t smem = smem_bytes(pair, TBN);
  if (dev >= 64 || !attr_done[pair][dev]) {
    const void *fn = pair ? (const void *)gemm_pair_kernel<A_MN, B_MN, StoreEpi, SPLIT>
                          : (const void *)gemm_3xtf32_kernel<A_MN, B_MN, TBN, StoreEpi, SPLIT>;
    int rc = check_kernel_registers(fn);
    if (rc) return rc;
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (dev < 64) attr_done[pair][dev] = true;
  }
  if (pair)
    FZ_CUDA(fz::launch_pdl(gemm_pair_kernel<A_MN, B_MN, StoreEpi, SPLIT>, dim3(2 * grid), dim3(NUM_THREADS), smem, s, mAh, mAl, mBh, mBl, ga, ep));
  else
    FZ_CUDA(fz::launch_pdl(gemm_3xtf32_kernel<A_MN, B_MN, TBN, StoreEpi, SPLIT>, dim3(grid), dim3(NUM_THREADS), smem, s, mAh, mAl, mBh, mBl, ga, ep));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fz::cuda_fail(e, "gemm_3xtf32_kernel launch", __FILE__, __LINE__);
  fz::note_launch();
  return FZ_OK;
}

// Kernel for the operand layouts and tile width (narrow tiles read B K-major); `split`:
// the variant that derives the remainder tiles in shared memory (full-width tiles).
int dispatch_gemm(bool a_mn, bool b_mn, int tbn, const CUtensorMap &mAh, const CUtensorMap &mAl,
                  const CUtensorMap &mBh, const CUtensorMap &mBl, const GemmArgs &ga,
                  const EpiParams &ep, unsigned grid, bool pair, bool split, cudaStream_t s) {
  if (split) {
    if (!a_mn && !b_mn) return launch_gemm<false, false, BN, true>(mAh, mAl, mBh, mBl, ga, ep, grid, pair, s);
    if (!a_mn && b_mn) return launch_gemm<false, true, BN, true>(mAh, mAl, mBh, mBl, ga, ep, grid, pair, s);
    if (a_mn && !b_mn) return launch_gemm<true, false, BN, true>(mAh, mAl, mBh, mBl, ga, ep, grid, pair, s);
    return launch_gemm<true, true, BN, true>(mAh, mAl, mBh, mBl, ga, ep, grid, pair, s);
  }
  if (tbn == 16)
    return a_mn ? launch_gemm<true, false, 16>(mAh, mAl, mBh, mBl, ga, ep, grid, false, s)
                : launch_gemm<false, false, 16>(mAh, mAl, mBh, mBl, ga, ep, grid, false, s);
  if (tbn == 64)
    return a_mn ? launch_gemm<true, false, 64>(mAh, mAl, mBh, mBl, ga, ep, grid, false, s)
                : launch_gemm<false, false, 64>(mAh, mAl, mBh, mBl, ga, ep, grid, false, s);
  if (!a_mn && !b_mn) return launch_gemm<false, false, BN>(mAh, mAl, mBh, mBl, ga, ep, grid, pair, s);
  if (!a_mn && b_mn) return launch_gemm<false, true, BN>(mAh, mAl, mBh, mBl, ga, ep, grid, pair, s);
  if (a_mn && !b_mn) return launch_gemm<true, false, BN>(mAh, mAl, mBh, mBl, ga, ep, grid, pair, s);
  return launch_gemm<true, true, BN>(mAh, mAl, mBh, mBl, ga, ep, grid, pair, s);
}

// ---------------------------------------------------------------- fused epilogues
//
// A fused elementwise program over the product (leaf 0) and inputs broadcast into
// the [batch, M, N] output space is compiled into the GEMM kernel: the text of
// fz_gemm_kernels.cuh, the program's scalar evaluator (the same fz_eval the fused
// elementwise kernels use, so each output rounds exactly as there) and a generated
// epilogue class GenEpi, instantiated for the kernel variant by NVRTC and cached per
// (program, input classes, variant).
const char *const kGemmKernelSource =
#include "fz_gemm_kernels.inc"
    ;

static_assert(EPI_MAX_IN + 1 == FZ_MAX_LEAVES && EPI_MAX_OUT == FZ_MAX_OUTPUTS,
              "epilogue operand limits follow the fused-program limits");

struct Epilogue {
  const fz_program *pg = nullptr;
  const fz_epi_input *inputs = nullptr;
  float *const *outputs = nullptr;
};

// Operand setup shared by both epilogue forms: per-row scalars (class 0) and the
// row-segment base pointers of class-1 / class-2 inputs.
void epilogue_operands(std::ostringstream &o, int nin, const int *cls) {
  for (int k = 0; k < nin; ++k) {
    const std::string K = std::to_string(k);
    if (cls[k] == 0)
      o << "    const float s" << K << " = live ? p.in[" << K << "][(long long)bz * p.in_sb[" << K
        << "] + (long long)row * p.in_sm[" << K << "]] : 0.0f;\n";
    else if (cls[k] == 1)
      o << "    const float *g" << K << " = p.in[" << K << "] + (long long)bz * p.in_sb[" << K
        << "] + col0;\n";
    else
      o << "    const float *g" << K << " = p.in[" << K << "] + (long long)bz * p.in_sb[" << K
        << "] + (long long)row0 * p.in_sm[" << K << "] + col0;\n";
  }
}

// Loads of the class-1 input k for columns [c4 * 4, c4 * 4 + 4) of the block (zeros
// past the last column), as u<k>[4].
void epilogue_row_vector(std::ostringstream &o, int k) {
  const std::string K = std::to_string(k);
  o << "        float4 w" << K << " = make_float4(0.0f, 0.0f, 0.0f, 0.0f);\n"
    << "        {\n"
    << "          const float *q = g" << K << " + cb * BW + c4 * 4;\n"
    << "          if (p.vec && c4 * 4 + 4 <= cols) w" << K << " = *reinterpret_cast<const float4 *>(q);\n"
    << "          else {\n"
    << "            if (c4 * 4 + 0 < cols) w" << K << ".x = q[0];\n"
    << "            if (c4 * 4 + 1 < cols) w" << K << ".y = q[1];\n"
    << "            if (c4 * 4 + 2 < cols) w" << K << ".z = q[2];\n"
    << "            if (c4 * 4 + 3 < cols) w" << K << ".w = q[3];\n"
    << "          }\n"
    << "        }\n"
    << "        const float u" << K << "[4] = {w" << K << ".x, w" << K << ".y, w" << K << ".z, w" << K << ".w};\n";
}

// The one-pass block form (see epilogue_class): slots [i * SL, (i + 1) * SL) of each
// tile row hold class-2 input i, then output j at slots (n2 + j) * SL. Each lane
// reads and writes only its own row between the copies in and the stores out, so
// three warp barriers per block order all accesses.
void epilogue_side_by_side(std::ostringstream &o, const fz_program &pg, const int *cls, int sbw) {
  const int nin = pg.num_leaves - 1, nout = pg.num_outputs;
  o << "    constexpr int BW = CPW < " << sbw << " ? CPW : " << sbw << ";\n"
    << "    constexpr int SL = BW / 4;\n";
  epilogue_operands(o, nin, cls);
  o << "#pragma unroll\n"
    << "    for (int cb = 0; cb < CPW / BW; ++cb) {\n"
    << "      const int cols = min(BW, a.N - col0 - cb * BW);\n"
    << "      if (cols <= 0) break;\n";
  std::vector<int> slot(nin, -1);
  int n2 = 0;
  for (int k = 0; k < nin; ++k) {
    if (cls[k] != 2) continue;
    const std::string K = std::to_string(k), S = std::to_string(n2) + " * SL";
    slot[k] = n2++;
    o << "      if (p.vec) tile_load_async<BW>(tile, g" << K << " + cb * BW, p.in_sm[" << K
      << "], rows, cols, lane, " << S << ");\n"
      << "      else tile_load<BW>(tile, g" << K << " + cb * BW, p.in_sm[" << K
      << "], rows, cols, false, lane, " << S << ");\n";
  }
  if (n2) o << "      __syncwarp(mask);\n";
  o << "#pragma unroll\n"
    << "      for (int c4 = 0; c4 < SL; ++c4) {\n";
  for (int k = 0; k < nin; ++k) {
    const std::string K = std::to_string(k);
    if (cls[k] == 1) epilogue_row_vector(o, k);
    if (cls[k] == 2)
      o << "        const float4 x" << K << " = tile_get(tile, lane, " << slot[k] << " * SL + c4);\n"
        << "        const float v" << K << "[4] = {x" << K << ".x, x" << K << ".y, x" << K << ".z, x" << K
        << ".w};\n";
  }
  for (int j = 0; j < nout; ++j) o << "        float r" << j << "[4];\n";
  o << "#pragma unroll\n"
    << "        for (int e = 0; e < 4; ++e) {\n";
  for (int j = 0; j < nout; ++j) o << "          float q" << j << ";\n";
  o << "          fz_eval(acc[cb * BW + c4 * 4 + e], ";
  for (int k = 0; k < nin; ++k)
    o << (cls[k] == 0 ? "s" : cls[k] == 1 ? "u" : "v") << k << (cls[k] == 0 ? "" : "[e]") << ", ";
  for (int j = 0; j < nout; ++j) o << "q" << j << (j + 1 < nout ? ", " : "");
  o << ");\n";
  for (int j = 0; j < nout; ++j) o << "          r" << j << "[e] = q" << j << ";\n";
  o << "        }\n";
  for (int j = 0; j < nout; ++j)
    o << "        tile_put(tile, lane, " << n2 + j << " * SL + c4, make_float4(r" << j << "[0], r" << j
      << "[1], r" << j << "[2], r" << j << "[3]));\n";
  o << "      }\n"
    << "      __syncwarp(mask);\n";
  for (int j = 0; j < nout; ++j)
    o << "      tile_store<BW>(tile, p.out[" << j << "] + ob + cb * BW, a.ldc, rows, cols, p.vec, lane, "
      << n2 + j << " * SL);\n";
  o << "      __syncwarp(mask);\n"
    << "    }\n  }\n};\n";
}

// Regions a TMA-stored epilogue needs per block: its class-2 inputs are copied into
// regions 0..n2-1 and output j is staged in region j (in place over input j: a lane
// reads all inputs of a column group before writing that group's outputs, and only
// its own row). The block width follows from how many fit in the 4 KB tile.
int tma_regions(const fz_program &pg, const int *cls) {
  int n2 = 0;
  for (int k = 0; k + 1 < pg.num_leaves; ++k) n2 += cls[k] == 2;
  return n2 > pg.num_outputs ? n2 : pg.num_outputs;
}
int tma_block_width(const fz_program &pg, const int *cls, int tbn) {
  int n2 = 0;
  for (int k = 0; k + 1 < pg.num_leaves; ++k) n2 += cls[k] == 2;
  if (tbn / 2 >= 32 && n2 == 0) return 32;  // the per-output form (epilogue_tma_wide)
  const int R = tma_regions(pg, cls);
  const int bw = R <= 2 ? 16 : R <= 4 ? 8 : R <= 8 ? 4 : 0;
  return bw < tbn / 2 ? bw : tbn / 2;  // at most the columns per epilogue warp
}

// The TMA form of the generated epilogue (outputs through omap[j]; see EpiParams).
// With one region per block two sets alternate, so a block is staged while the
// previous block's stores still read their region.
void epilogue_tma(std::ostringstream &o, const fz_program &pg, const int *cls, int bw) {
  const int nin = pg.num_leaves - 1, nout = pg.num_outputs, R = tma_regions(pg, cls);
  o << "    constexpr int BW = CPW < " << bw << " ? CPW : " << bw << ";\n"
    << "    constexpr int R = " << R << ";\n"
    << "    constexpr int S = (32 / BW) / R >= 2 ? 2 : 1;\n";
  epilogue_operands(o, nin, cls);
  o << "#pragma unroll\n"
    << "    for (int cb = 0; cb < CPW / BW; ++cb) {\n"
    << "      const int cols = min(BW, a.N - col0 - cb * BW);\n"
    << "      if (cols <= 0) break;\n"
    << "      const int set = S == 2 ? (cb & 1) * R : 0;\n"
    << "      if (S == 1 || cb == 0) store_reads_done<0>(lane, mask);\n"
    << "      else store_reads_done<1>(lane, mask);\n";
  std::vector<int> reg(nin, -1);
  int n2 = 0;
  for (int k = 0; k < nin; ++k) {
    if (cls[k] != 2) continue;
    const std::string K = std::to_string(k);
    reg[k] = n2++;
    o << "      region_load_async<BW>(region_ptr(tile, BW, set + " << reg[k] << "), g" << K
      << " + cb * BW, p.in_sm[" << K << "], rows, cols, lane);\n";
  }
  if (n2) o << "      __syncwarp(mask);\n";
  o << "#pragma unroll\n"
    << "      for (int c4 = 0; c4 < BW / 4; ++c4) {\n";
  for (int k = 0; k < nin; ++k) {
    const std::string K = std::to_string(k);
    if (cls[k] == 1) epilogue_row_vector(o, k);
    if (cls[k] == 2)
      o << "        const float4 x" << K << " = region_get(region_ptr(tile, BW, set + " << reg[k]
        << "), BW, lane, c4);\n"
        << "        const float v" << K << "[4] = {x" << K << ".x, x" << K << ".y, x" << K << ".z, x" << K
        << ".w};\n";
  }
  for (int j = 0; j < nout; ++j) o << "        float r" << j << "[4];\n";
  o << "#pragma unroll\n"
    << "        for (int e = 0; e < 4; ++e) {\n";
  for (int j = 0; j < nout; ++j) o << "          float q" << j << ";\n";
  o << "          fz_eval(acc[cb * BW + c4 * 4 + e], ";
  for (int k = 0; k < nin; ++k)
    o << (cls[k] == 0 ? "s" : cls[k] == 1 ? "u" : "v") << k << (cls[k] == 0 ? "" : "[e]") << ", ";
  for (int j = 0; j < nout; ++j) o << "q" << j << (j + 1 < nout ? ", " : "");
  o << ");\n";
  for (int j = 0; j < nout; ++j) o << "          r" << j << "[e] = q" << j << ";\n";
  o << "        }\n";
  for (int j = 0; j < nout; ++j)
    o << "        region_put(region_ptr(tile, BW, set + " << j << "), BW, lane, c4, make_float4(r" << j
      << "[0], r" << j << "[1], r" << j << "[2], r" << j << "[3]));\n";
  o << "      }\n"
    << "      staged_for_tma(mask);\n"
    << "      if (lane == 0) {\n";
  for (int j = 0; j < nout; ++j)
    o << "        tma_store_3d(&p.omap[" << j << "], region_ptr(tile, BW, set + " << j
      << "), col0 + cb * BW, row0, bz);\n";
  o << "        tma_store_commit();\n"
    << "      }\n"
    << "    }\n  }\n};\n";
}

// The wide TMA form, for warps owning at least 32 columns and programs without
// class-2 inputs: per 32-column block, for each output the program is evaluated over
// the block, staged in the whole tile (128-byte-swizzled tile_put layout) and written
// by one 32 x 32 TMA store. Outputs are stored one at a time, so a block costs nout
// stores of 4 KB (a store has a fixed cost of about 0.5 us: staging, proxy fence and
// issue, timed with %globaltimer). Same box, [8192,4096]x[4096,4096]^T: bias+ReLU with
// three outputs 1.044 -> 1.031 ms against the 8-column region form. With a class-2
// input (loaded per lane into registers) the ReLU-mask gradient measured 1.049 ->
// 1.063 ms, so class-2 inputs keep the region form, whose cp.async copies coalesce.
void epilogue_tma_wide(std::ostringstream &o, const fz_program &pg, const int *cls) {
  const int nin = pg.num_leaves - 1, nout = pg.num_outputs;
  o << "    constexpr int BW = 32;\n";
  epilogue_operands(o, nin, cls);
  o << "#pragma unroll\n"
    << "    for (int cb = 0; cb < CPW / BW; ++cb) {\n"
    << "      const int cols = min(BW, a.N - col0 - cb * BW);\n"
    << "      if (cols <= 0) break;\n";
  for (int j = 0; j < nout; ++j) {
    o << "      {\n"
      << "        float r[BW];\n"
      << "#pragma unroll\n"
      << "        for (int c4 = 0; c4 < BW / 4; ++c4) {\n";
    for (int k = 0; k < nin; ++k)
      if (cls[k] == 1) epilogue_row_vector(o, k);
    o << "#pragma unroll\n"
      << "          for (int e = 0; e < 4; ++e) {\n"
      << "            const int c = c4 * 4 + e;\n";
    for (int q = 0; q < nout; ++q) o << "            float q" << q << ";\n";
    o << "            fz_eval(acc[cb * BW + c], ";
    for (int k = 0; k < nin; ++k)
      o << (cls[k] == 0 ? "s" + std::to_string(k) : "u" + std::to_string(k) + "[e]") << ", ";
    for (int q = 0; q < nout; ++q) o << "q" << q << (q + 1 < nout ? ", " : "");
    o << ");\n"
      << "            r[c] = q" << j << ";\n"
      << "          }\n"
      << "        }\n"
      << "        store_reads_done<0>(lane, mask);\n"
      << "#pragma unroll\n"
      << "        for (int c4 = 0; c4 < BW / 4; ++c4)\n"
      << "          tile_put(tile, lane, c4, make_float4(r[c4 * 4], r[c4 * 4 + 1], r[c4 * 4 + 2], r[c4 * 4 + 3]));\n"
      << "        staged_for_tma(mask);\n"
      << "        if (lane == 0) {\n"
      << "          tma_store_3d(&p.omap[" << j << "], tile, col0 + cb * BW, row0, bz);\n"
      << "          tma_store_commit();\n"
      << "        }\n"
      << "      }\n";
  }
  o << "    }\n  }\n};\n";
}

// The wide TMA form with one full-shape input (class 2): per 32-column block the input's
// 32 x 32 box comes into the warp's staging tile by a TMA load (epi_load_box: 128-byte
// swizzle, zeros past the edges), each lane takes its row into registers, and each
// output is evaluated over the block into the tile and leaves in one 32 x 32 store, as
// in epilogue_tma_wide. Four blocks of one load and nout stores per 128 columns replace
// the region form's eight blocks of 16 columns, each of which waited for a cp.async
// copy of the input and for its stores to read the tile.
void epilogue_tma_wide_in(std::ostringstream &o, const fz_program &pg, const int *cls) {
  const int nin = pg.num_leaves - 1, nout = pg.num_outputs;
  int kin = -1;
  for (int k = 0; k < nin; ++k)
    if (cls[k] == 2) kin = k;
  const std::string KI = std::to_string(kin);
  o << "    constexpr int BW = 32;\n";
  epilogue_operands(o, nin, cls);
  o << "    (void)g" << KI << ";\n"
    << "#pragma unroll\n"
    << "    for (int cb = 0; cb < CPW / BW; ++cb) {\n"
    << "      const int cols = min(BW, a.N - col0 - cb * BW);\n"
    << "      if (cols <= 0) break;\n"
    << "      // block 0's load was started by prefetch, before the tile's last chunk\n"
    << "      if (cb > 0) epi_issue_box(&p.imap, tile, sync, col0 + cb * BW, row0, bz, lane, mask);\n"
    << "      if (!epi_wait_box(sync, lane, mask, a.err)) return;\n"
    << "      float v" << KI << "[BW];\n"
    << "#pragma unroll\n"
    << "      for (int c4 = 0; c4 < BW / 4; ++c4) {\n"
    << "        const float4 t = tile_get(tile, lane, c4);\n"
    << "        v" << KI << "[c4 * 4] = t.x; v" << KI << "[c4 * 4 + 1] = t.y; v" << KI << "[c4 * 4 + 2] = t.z; v" << KI
    << "[c4 * 4 + 3] = t.w;\n"
    << "      }\n"
    << "      __syncwarp(mask);  // every lane has its row before the tile is overwritten\n";
  for (int j = 0; j < nout; ++j) {
    o << "      {\n";
    if (j > 0) o << "        store_reads_done<0>(lane, mask);\n";
    o << "#pragma unroll\n"
      << "        for (int c4 = 0; c4 < BW / 4; ++c4) {\n";
    for (int k = 0; k < nin; ++k)
      if (cls[k] == 1) epilogue_row_vector(o, k);
    o << "          float r[4];\n"
      << "#pragma unroll\n"
      << "          for (int e = 0; e < 4; ++e) {\n"
      << "            const int c = c4 * 4 + e;\n";
    for (int q = 0; q < nout; ++q) o << "            float q" << q << ";\n";
    o << "            fz_eval(acc[cb * BW + c], ";
    for (int k = 0; k < nin; ++k)
      o << (cls[k] == 0 ? "s" + std::to_string(k)
                        : cls[k] == 1 ? "u" + std::to_string(k) + "[e]" : "v" + std::to_string(k) + "[c]")
        << ", ";
    for (int q = 0; q < nout; ++q) o << "q" << q << (q + 1 < nout ? ", " : "");
    o << ");\n"
      << "            r[e] = q" << j << ";\n"
      << "          }\n"
      << "          tile_put(tile, lane, c4, make_float4(r[0], r[1], r[2], r[3]));\n"
      << "        }\n"
      << "        staged_for_tma(mask);\n"
      << "        if (lane == 0) {\n"
      << "          tma_store_3d(&p.omap[" << j << "], tile, col0 + cb * BW, row0, bz);\n"
      << "          tma_store_commit();\n"
      << "        }\n"
      << "      }\n";
  }
  o << "    }\n  }\n};\n";
}

// The one full-shape input of a program, or -1 (none, or more than one).
int single_full_input(const fz_program &pg, const int *cls) {
  int kin = -1;
  for (int k = 0; k + 1 < pg.num_leaves; ++k)
    if (cls[k] == 2) {
      if (kin >= 0) return -1;
      kin = k;
    }
  return kin;
}

// Load map of a full-shape epilogue input: 3D {N, M, Z}, its row and batch pitches,
// 32 x 32 boxes in the staging tile's 128-byte swizzle. false when TMA cannot read
// it (then the region form copies it with cp.async).
bool make_in_map(CUtensorMap *map, const fz_epi_input &in, int64_t N, int64_t M, int64_t Z) {
  const int64_t sm = in.row_stride, sb = Z == 1 ? in.row_stride * M : in.batch_stride;
  if (!in.ptr || ((uintptr_t)in.ptr & 15) || sm < N || (sm * 4) % 16 || sb <= 0 || (sb * 4) % 16) return false;
  cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)Z};
  cuuint64_t strides[2] = {(cuuint64_t)(sm * 4), (cuuint64_t)(sb * 4)};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(in.ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// cls[k] of input k: 0 constant along a row (a per-row value or a scalar), 1 a row
// vector (same for every row: a bias), 2 varying along rows and columns (a tensor of
// the product's shape). Class-2 inputs are read through the warp's staging tile in
// whole row segments; class-1 inputs are the same address for every lane.
std::string epilogue_class(const fz_program &pg, const int *cls, int tma_bw, bool wide_in) {
  const int nin = pg.num_leaves - 1, nout = pg.num_outputs;
  std::ostringstream o;
  // prefetch: called when a tile starts, L2 prefetches of the full-shape inputs' rows
  // lane by lane. before_last: called before the tile's last chunk is promoted; the
  // TMA-input form starts its first block's load into the staging tile there (it lands
  // while the chunk is promoted) and has the TMA unit prefetch the other blocks into L2
  // (a prefetch at the start of the tile would be evicted by the main loop's operand
  // traffic, which turns L2 over every ~15 us).
  o << "struct GenEpi {\n"
    << "  template <int CPW>\n"
    << "  static __device__ __forceinline__ void prefetch(const fz_gemm_dev::GemmArgs &a,\n"
    << "      const fz_gemm_dev::EpiParams &p, int bz, int row, int col0) {\n"
    << "    if (row >= a.M || col0 >= a.N) return;\n"
    << "    const int n = min(CPW, a.N - col0);\n"
    << "    (void)p; (void)bz; (void)n;\n";
  if (!wide_in)
    for (int k = 0; k < nin; ++k)
      if (cls[k] == 2)
        o << "    fz_gemm_dev::prefetch_row_l2(p.in[" << k << "] + (long long)bz * p.in_sb[" << k
          << "] + (long long)row * p.in_sm[" << k << "] + col0, n);\n";
  o << "  }\n"
    << "  template <int CPW>\n"
    << "  static __device__ __forceinline__ void before_last(const fz_gemm_dev::GemmArgs &a,\n"
    << "      const fz_gemm_dev::EpiParams &p, int bz, int row, int col0, float4 *tile,\n"
    << "      fz_gemm_dev::EpiSync &sync) {\n"
    << "    using namespace fz_gemm_dev;\n"
    << "    (void)a; (void)p; (void)bz; (void)row; (void)col0; (void)tile; (void)sync;\n";
  if (wide_in)
    o << "    const int lane = threadIdx.x & 31;\n"
      << "    const int row0 = row - lane;\n"
      << "    if (row0 >= a.M || col0 >= a.N) return;  // uniform over the warp\n"
      << "    const unsigned mask = __activemask();\n"
      << "    epi_issue_box(&p.imap, tile, sync, col0, row0, bz, lane, mask);\n"
      << "    if (lane == 0)\n"
      << "      for (int cb = 1; cb < CPW / 32 && col0 + cb * 32 < a.N; ++cb) tma_prefetch_box(&p.imap, col0 + cb * 32, row0, bz);\n";
  o << "  }\n"
    << "  template <int CPW>\n"
    << "  static __device__ __forceinline__ void store(const fz_gemm_dev::GemmArgs &a,\n"
    << "      const fz_gemm_dev::EpiParams &p, int, int bz, int row, int col0,\n"
    << "      const float (&acc)[CPW], float4 *tile, fz_gemm_dev::EpiSync &sync) {\n"
    << "    using namespace fz_gemm_dev;\n"
    << "    (void)sync;\n"
    << "    const int lane = threadIdx.x & 31;\n"
    << "    const int row0 = row - lane;\n"
    << "    const int rows = min(32, a.M - row0);\n"
    << "    if (rows <= 0 || col0 >= a.N) return;\n"
    << "    const unsigned mask = __activemask();\n"
    << "    const bool live = lane < rows;\n"
    << "    (void)live;\n"
    << "    const long long ob = (long long)bz * a.strideC + (long long)row0 * a.ldc + col0;\n";
  // With full-shape (class-2) inputs, when they and the outputs of one block fit
  // side by side in the staging tile's 8 float4 slots per row, every block runs as
  // one pass: the inputs are copied in, each lane evaluates the program once per
  // group of 4 columns of its row (reading its inputs from the tile, writing every
  // output into its own slots) and the outputs are stored from there, so no copy of
  // the inputs is held in registers beside the accumulators. Measured on
  // [8192,4096]x[4096,4096]^T: the ReLU-mask gradient (one input, two outputs)
  // 1.123 -> 1.105 ms, the K = 16 one of the MLP 1.91 -> 1.60 ms. Without class-2
  // inputs the per-output passes at 16 columns are faster (bias + ReLU with three
  // outputs: 1.056 ms, against 1.085 side by side at 8 columns).
  if (wide_in) {
    epilogue_tma_wide_in(o, pg, cls);
    return o.str();
  }
  if (tma_bw == 32) {
    epilogue_tma_wide(o, pg, cls);
    return o.str();
  }
  if (tma_bw) {
    epilogue_tma(o, pg, cls, tma_bw);
    return o.str();
  }
  int n2 = 0;
  for (int k = 0; k < nin; ++k) n2 += cls[k] == 2;
  const int side = n2 + nout;
  const int sbw = n2 == 0 ? 0 : side <= 2 ? 16 : side <= 4 ? 8 : side <= 8 ? 4 : 0;
  if (sbw) {
    epilogue_side_by_side(o, pg, cls, sbw);
    return o.str();
  }
  o << "    constexpr int BW = CPW < EPI_BW ? CPW : EPI_BW;\n";
  epilogue_operands(o, nin, cls);
  o << "#pragma unroll\n"
    << "    for (int cb = 0; cb < CPW / BW; ++cb) {\n"
    << "      const int cols = min(BW, a.N - col0 - cb * BW);\n"
    << "      if (cols <= 0) break;\n";
  // class-2 inputs: one block of this lane's row, through the tile
  for (int k = 0; k < nin; ++k) {
    if (cls[k] != 2) continue;
    const std::string K = std::to_string(k);
    o << "      float v" << K << "[BW];\n"
      << "      if (p.vec) tile_load_async<BW>(tile, g" << K << " + cb * BW, p.in_sm[" << K << "], rows, cols, lane);\n"
      << "      else tile_load<BW>(tile, g" << K << " + cb * BW, p.in_sm[" << K << "], rows, cols, false, lane);\n"
      << "      __syncwarp(mask);\n"
      << "#pragma unroll\n"
      << "      for (int c4 = 0; c4 < BW / 4; ++c4) {\n"
      << "        const float4 t = tile_get(tile, lane, c4);\n"
      << "        v" << K << "[c4 * 4] = t.x; v" << K << "[c4 * 4 + 1] = t.y; v" << K
      << "[c4 * 4 + 2] = t.z; v" << K << "[c4 * 4 + 3] = t.w;\n"
      << "      }\n"
      << "      __syncwarp(mask);\n";
  }
  // each output: evaluate the block into the tile, then store it in row segments
  for (int j = 0; j < nout; ++j) {
    o << "#pragma unroll\n"
      << "      for (int c4 = 0; c4 < BW / 4; ++c4) {\n"
      << "        float r[4];\n";
    // class-1 inputs: this group of 4 columns (zeros past N)
    for (int k = 0; k < nin; ++k)
      if (cls[k] == 1) epilogue_row_vector(o, k);
    o << "#pragma unroll\n"
      << "        for (int e = 0; e < 4; ++e) {\n"
      << "          const int c = c4 * 4 + e;\n";
    for (int k = 0; k < nout; ++k) o << "          float q" << k << ";\n";
    o << "          fz_eval(acc[cb * BW + c], ";
    for (int k = 0; k < nin; ++k)
      o << (cls[k] == 0 ? "s" + std::to_string(k)
                        : cls[k] == 1 ? "u" + std::to_string(k) + "[e]" : "v" + std::to_string(k) + "[c]")
        << ", ";
    for (int k = 0; k < nout; ++k) o << "q" << k << (k + 1 < nout ? ", " : "");
    o << ");\n"
      << "          r[e] = q" << j << ";\n"
      << "        }\n"
      << "        tile_put(tile, lane, c4, make_float4(r[0], r[1], r[2], r[3]));\n"
      << "      }\n"
      << "      __syncwarp(mask);\n"
      << "      tile_store<BW>(tile, p.out[" << j << "] + ob + cb * BW, a.ldc, rows, cols, p.vec, lane);\n"
      << "      __syncwarp(mask);\n";
  }
  o << "    }\n  }\n};\n";
  return o.str();
}

int input_class(const fz_epi_input &in) {
  return in.col_stride == 0 ? 0 : in.row_stride == 0 ? 1 : 2;
}

struct JitEntry {
  cudaKernel_t kern = nullptr;
  uint64_t attr_devices = 0;  // devices whose shared-memory limit was raised
};
std::mutex g_jit_mu;
std::unordered_map<std::string, JitEntry> g_jit;

std::string epilogue_source(const fz_program &pg, const int *cls, int tma_bw, bool wide_in) {
  return "#define FZ_GEMM_BK " + std::to_string(BK) + "\n" + kGemmKernelSource + "\n" +
         fz::program_eval_source(pg) + epilogue_class(pg, cls, tma_bw, wide_in);
}

std::string epilogue_kernel_name(bool a_mn, bool b_mn, int tbn, bool pair) {
  auto b = [](bool v) { return std::string(v ? "true" : "false"); };
  if (pair) return "&fz_gemm_dev::gemm_pair_kernel<" + b(a_mn) + ", " + b(b_mn) + ", GenEpi>";
  return "&fz_gemm_dev::gemm_3xtf32_kernel<" + b(a_mn) + ", " + b(b_mn) + ", " + std::to_string(tbn) +
         ", GenEpi>";
}

int jit_kernel(const fz_program &pg, const int *cls, bool a_mn, bool b_mn, int tbn, bool pair,
               int tma_bw, bool wide_in, size_t smem, cudaKernel_t *out) {
  std::string key(reinterpret_cast<const char *>(&pg),
                  offsetof(fz_program, nodes) + sizeof(fz_node) * pg.num_nodes);
  for (int k = 0; k + 1 < pg.num_leaves; ++k) key.push_back((char)('0' + cls[k]));
  key += pair ? "P" : "S";
  key.push_back((char)('0' + a_mn));
  key.push_back((char)('0' + b_mn));
  key += std::to_string(tbn);
  key += "T" + std::to_string(tma_bw) + (wide_in ? "I" : "");
  int dev = 0;
  FZ_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_jit_mu);
  JitEntry &e = g_jit[key];
  if (!e.kern) {
    std::vector<char> bin;
    std::string lowered;
    const std::string name = epilogue_kernel_name(a_mn, b_mn, tbn, pair);
    int rc = fz::nvrtc_cubin(epilogue_source(pg, cls, tma_bw, wide_in), "fz_gemm_epilogue.cu", name.c_str(), &bin,
                             &lowered);
    if (rc) return rc;
    cudaLibrary_t lib;
    FZ_CUDA(cudaLibraryLoadData(&lib, bin.data(), nullptr, nullptr, 0, nullptr, nullptr, 0));
    cudaKernel_t kern = nullptr;
    FZ_CUDA(cudaLibraryGetKernel(&kern, lib, lowered.c_str()));
    rc = check_kernel_registers((const void *)kern);
    if (rc) return rc;
    e.kern = kern;
  }
  if (dev >= 64 || !((e.attr_devices >> dev) & 1)) {
    FZ_CUDA(cudaKernelSetAttributeForDevice(e.kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)smem, dev));
    if (dev < 64) e.attr_devices |= 1ull << dev;
  }
  *out = e.kern;
  return FZ_OK;
}

int launch_epilogue_gemm(const Epilogue &E, const int *cls, const EpiParams &ep, bool a_mn,
                         bool b_mn, int tbn, const CUtensorMap &mAh, const CUtensorMap &mAl,
                         const CUtensorMap &mBh, const CUtensorMap &mBl, const GemmArgs &ga,
                         unsigned grid, bool pair, int tma_bw, bool wide_in, cudaStream_t s) {
  const size_t smem = smem_bytes(pair, tbn);
  cudaKernel_t k = nullptr;
  int rc = jit_kernel(*E.pg, cls, a_mn, b_mn, tbn, pair, tma_bw, wide_in, smem, &k);
  if (rc) return rc;
  void *args[] = {const_cast<CUtensorMap *>(&mAh), const_cast<CUtensorMap *>(&mAl),
                  const_cast<CUtensorMap *>(&mBh), const_cast<CUtensorMap *>(&mBl),
                  const_cast<GemmArgs *>(&ga), const_cast<EpiParams *>(&ep)};
  FZ_CUDA(fz::launch_pdl_handle((const void *)k, dim3(pair ? 2 * grid : grid), dim3(NUM_THREADS), smem, s, args));
  fz::note_launch();
  return FZ_OK;
}

// The epilogue program as one fused elementwise pass over a dense product P
// ([batch, M, N]): the form taken when the GEMM splits K or K = 0.
int epilogue_pass(const Epilogue &E, const float *P, int64_t batch, int64_t M, int64_t N,
                  int64_t ldc, int64_t strideC, cudaStream_t s) {
  const fz_program &pg = *E.pg;
  const int nout = pg.num_outputs, nleaf = pg.num_leaves;
  fz_ewise_plan plan{};
  plan.ndim = 3;
  plan.num_operands = nout + nleaf;
  plan.size[0] = batch;
  plan.size[1] = M;
  plan.size[2] = N;
  auto set = [&](int k, int64_t sb, int64_t sm, int64_t sn) {
    plan.stride_bytes[k][0] = sb * 4;
    plan.stride_bytes[k][1] = sm * 4;
    plan.stride_bytes[k][2] = sn * 4;
  };
  for (int k = 0; k < nout; ++k) set(k, strideC, ldc, 1);
  set(nout, M * N, N, 1);
  std::vector<const float *> leaves(nleaf);
  leaves[0] = P;
  for (int k = 1; k < nleaf; ++k) {
    const fz_epi_input &in = E.inputs[k - 1];
    set(nout + k, in.batch_stride, in.row_stride, in.col_stride);
    leaves[k] = in.ptr;
  }
  return fz_fused_launch(&pg, &plan, E.outputs, leaves.data(), s);
}

int check_epilogue(const Epilogue &E, int64_t N, int64_t ldc) {
  FZ_REQUIRE(E.pg && E.outputs, "fz_gemm_f32_epilogue: null program or outputs");
  int rc = fz::validate_program(*E.pg);
  if (rc) return rc;
  const fz_program &pg = *E.pg;
  FZ_REQUIRE(pg.num_leaves >= 1 && pg.num_leaves <= 1 + EPI_MAX_IN,
             "fz_gemm_f32_epilogue: the program needs leaf 0 (the product) and at most " +
                 std::to_string(EPI_MAX_IN) + " inputs");
  FZ_REQUIRE(pg.num_outputs <= EPI_MAX_OUT, "fz_gemm_f32_epilogue: too many outputs");
  FZ_REQUIRE(pg.num_leaves == 1 || E.inputs, "fz_gemm_f32_epilogue: null inputs");
  for (int k = 0; k < pg.num_outputs; ++k) FZ_REQUIRE(E.outputs[k], "fz_gemm_f32_epilogue: null output");
  for (int k = 1; k < pg.num_leaves; ++k) {
    FZ_REQUIRE(E.inputs[k - 1].ptr, "fz_gemm_f32_epilogue: null input");
    FZ_REQUIRE(E.inputs[k - 1].col_stride == 0 || E.inputs[k - 1].col_stride == 1,
               "fz_gemm_f32_epilogue: input column stride must be 0 or 1");
  }
  FZ_REQUIRE(ldc >= N, "fz_gemm_f32_epilogue: ldc < N");
  return FZ_OK;
}

int gemm_impl(int64_t batch, int64_t M, int64_t N, int64_t K, const float *A, const float *A_lo,
              int64_t lda, int64_t strideA, int transA, const float *B, const float *B_lo,
              int64_t ldb, int64_t strideB, int transB, float *C, int64_t ldc, int64_t strideC,
              const Epilogue &E, void *stream) {
  FZ_REQUIRE(batch >= 0 && M >= 0 && N >= 0 && K >= 0, "fz_gemm_f32: negative extent");
  if (E.pg) {
    int rc = check_epilogue(E, N, ldc);
    if (rc) return rc;
  }
  if (batch == 0 || M == 0 || N == 0) return FZ_OK;
  FZ_REQUIRE(C || E.pg, "fz_gemm_f32: null C");
  FZ_REQUIRE(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31) && batch < 65536,
             "fz_gemm_f32: extent too large");
  FZ_REQUIRE(ldc >= N, "fz_gemm_f32: ldc < N");
  cudaStream_t s = fz::resolve(stream);
  if (K == 0) {
    if (E.pg) {
      float *P = nullptr;
      int rc = fz_malloc((void **)&P, sizeof(float) * batch * M * N, s);
      if (!rc) rc = fz_fill_f32(P, 0.0f, batch * M * N, s);
      if (!rc) rc = epilogue_pass(E, P, batch, M, N, ldc, strideC, s);
      fz_free(P, s);
      return rc;
    }
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

  // CTA pairs (256 x 256 tiles, cta_group::2) when there are rows for both halves and
  // enough tiles to keep the pairs busy, or (with at least 1024 rows, so that the
  // 256-row tiles waste little) a product of 8 GFLOP or more, whose K-split units keep
  // them busy: per SM the pair kernel is the faster one (measured with planes supplied:
  // 4096x1024x65536 2.05 against 2.12 ms, 3072x1024x4096 117 against 122 us, 2048^3
  // 68 against 70 us; only 1024^3, 2 GFLOP, ran faster on single CTAs, 19 against 20 us).
  // Single CTAs otherwise, with 16- or 64-column tiles for narrow outputs.
  const int64_t pair_tiles = ((M + 2 * BM - 1) / (2 * BM)) * ((N + BN - 1) / BN) * batch;
  const int mode = g_tile_mode.load(std::memory_order_relaxed);
  const double flops = 2.0 * (double)batch * (double)M * (double)N * (double)K;
  const bool pair = mode == FZ_GEMM_TILES_PAIR ||
                    (mode == FZ_GEMM_TILES_AUTO && M >= 2 * BM && N > 64 &&
                     (pair_tiles * 2 >= fz::num_sms() || (M >= 1024 && flops >= 8.0e9)));
  int tbn = pair || N > 64 ? BN : N > 16 ? 64 : 16;
  // narrow tiles read B K-major: a dense MN-major B ([K, N], N <= 64, a few MB) is
  // transposed into a K-major copy first
  float *bt = nullptr;
  if (tbn < BN && transB == 0) {
    if (ldb == N && (batch == 1 || strideB == K * N) && (((uintptr_t)B) & 15) == 0) {
      rc = fz_malloc((void **)&bt, sizeof(float) * batch * N * K, s);
      const int64_t shp[3] = {batch, K, N};
      if (!rc) rc = fz_swapaxes(bt, B, shp, 3, 1, 2, s);
      if (rc) {
        fz_free(bt, s);
        return rc;
      }
      B = bt;
      B_lo = nullptr;
      ldb = K;
      strideB = N * K;
      transB = 1;
    } else {
      tbn = BN;
    }
  }
  // A as stored: [M, K] (transA = 0, K-major) or [K, M] (MN-major); B: [N, K]
  // (transB != 0, K-major) or [K, N] (MN-major).
  Operand oa{transA != 0, transA ? K : M, transA ? M : K};
  Operand ob{transB == 0, transB ? N : K, transB ? K : N};
  // Remainder planes the caller did not supply: written by a separate pass, or, when
  // asked for (FZ_GEMM_SPLIT_IN_KERNEL), derived in shared memory by the kernel (full-
  // width tiles, plain output, operands TMA can address as they are; a supplied plane
  // is then not read, the values being the same)
  const bool split_here = g_split_mode.load(std::memory_order_relaxed) == FZ_GEMM_SPLIT_IN_KERNEL && !E.pg &&
                          tbn == BN && (!A_lo || !B_lo) && direct_hi(A, lda, strideA, batch) &&
                          direct_hi(B, ldb, strideB, batch);
  float *ws = nullptr;
  if (split_here) {
    for (Operand *op : {&oa, &ob}) {
      const bool is_a = op == &oa;
      op->hi = op->lo = is_a ? A : B;
      op->hi_ld = op->lo_ld = is_a ? lda : ldb;
      op->hi_sb = op->lo_sb = batch == 1 ? op->hi_ld * op->rows : (is_a ? strideA : strideB);
    }
  } else {
    const int64_t a_need = workspace_floats(oa, A, lda, strideA, A_lo, batch);
    const int64_t b_need = workspace_floats(ob, B, ldb, strideB, B_lo, batch);
    if (a_need + b_need) {
      rc = fz_malloc((void **)&ws, sizeof(float) * (a_need + b_need), s);
      if (rc) {
        fz_free(bt, s);
        return rc;
      }
    }
    rc = prepare(A, lda, strideA, A_lo, batch, ws, &oa, s);
    if (!rc) rc = prepare(B, ldb, strideB, B_lo, batch, ws + a_need, &ob, s);
  }

  const int tile_m = pair ? 2 * BM : BM, box_b = pair ? BM : tbn;
  const int64_t workers = pair ? fz::num_sms() / 2 : fz::num_sms();
  CUtensorMap mAh, mAl, mBh, mBl;
  bool wide[4] = {false, false, false, false};
  if (!rc) rc = make_map(&mAh, oa.hi, oa.mn, M, K, oa.hi_ld, oa.hi_sb, batch, BM, oa.hi_padded, &wide[0]);
  if (!rc) rc = make_map(&mAl, oa.lo, oa.mn, M, K, oa.lo_ld, oa.lo_sb, batch, BM, oa.lo_padded, &wide[1]);
  if (!rc) rc = make_map(&mBh, ob.hi, ob.mn, N, K, ob.hi_ld, ob.hi_sb, batch, box_b, ob.hi_padded, &wide[2]);
  if (!rc) rc = make_map(&mBl, ob.lo, ob.mn, N, K, ob.lo_ld, ob.lo_sb, batch, box_b, ob.lo_padded, &wide[3]);
  const int wide_mask = (int)wide[0] | (int)wide[1] << 1 | (int)wide[2] << 2 | (int)wide[3] << 3;
  const int tiles_m = (int)((M + tile_m - 1) / tile_m), tiles_n = (int)((N + tbn - 1) / tbn);
  const int64_t tiles = (int64_t)tiles_m * tiles_n * batch;
  const bool dense_c = ldc == N && (batch == 1 || strideC == M * N);
  const int splits = dense_c || E.pg ? choose_splits(tiles, M, N, K, batch, workers) : 1;
  const int64_t kps = splits > 1 ? round_up((K + splits - 1) / splits, (int64_t)BK * KSPLIT_GRAN) : K;
  const int real_splits = (int)((K + kps - 1) / kps);
  const int64_t num_units = tiles * real_splits;
  if (!rc && num_units >= (1ll << 31)) rc = fz::fail(FZ_ERR_INVALID, "fz_gemm_f32: too many tiles");
  float *partial = nullptr;
  if (!rc && real_splits > 1)
    rc = fz_malloc((void **)&partial, sizeof(float) * real_splits * batch * M * N, s);
  // split K with an epilogue: the partials are summed into a dense product, which the
  // program then reads in one fused pass
  float *product = nullptr;
  if (!rc && E.pg && real_splits > 1) rc = fz_malloc((void **)&product, sizeof(float) * batch * M * N, s);
  // epilogue operands, and the column class of each input compiled into the kernel
  EpiParams ep{};
  int cls[EPI_MAX_IN] = {};
  if (E.pg && !product) {
    bool vec = ldc % 4 == 0 && (batch == 1 || strideC % 4 == 0);
    for (int k = 0; k < E.pg->num_outputs; ++k) {
      ep.out[k] = E.outputs[k];
      vec = vec && ((uintptr_t)E.outputs[k] & 15) == 0;
    }
    for (int k = 0; k + 1 < E.pg->num_leaves; ++k) {
      const fz_epi_input &in = E.inputs[k];
      ep.in[k] = in.ptr;
      ep.in_sb[k] = in.batch_stride;
      ep.in_sm[k] = in.row_stride;
      cls[k] = input_class(in);
      if (cls[k])
        vec = vec && ((uintptr_t)in.ptr & 15) == 0 && in.row_stride % 4 == 0 &&
              (batch == 1 || in.batch_stride % 4 == 0);
    }
    ep.vec = vec;
  }

  int *err = nullptr;
  if (!rc) rc = fz::device_error_word(&err);
  if (!rc) {
    // raster bands of 12 row tiles walked column by column. On [65536,4096]x[4096,4096]^T,
    // bands of 16 / 12 / 8 read 14.3 / 12.6 / 12.9 GB from DRAM per launch in the same
    // time (8.0 ms): the re-reads come mostly from CTA pairs drifting apart in K, not from
    // the band; bands of B columns walked row by row with L2 eviction hints keeping B
    // were measured slower (DRAM is not what bounds these kernels)
    const int band = 12;
    const bool in_kernel = E.pg && !product;
    GemmArgs ga{partial ? partial : in_kernel ? nullptr : C, partial ? N : ldc,
                partial ? M * N : strideC, batch * M * N, (int)M, (int)N, (int)K, (int)batch,
                tiles_m, tiles_n, (int)num_units, tiles_m < band ? tiles_m : band,
                real_splits, (int)kps, wide_mask, err, nullptr};
    // CTA pairs' producers in lockstep for launches of four waves or more (fewer, short
    // tiles measured slower: batched 64x512^3, 3.5 waves, 88 against 84 us)
    if (!rc && pair && num_units >= 4 * workers) rc = tile_sync_slot(s, &ga.tile_sync);
    // persistent grid: one CTA (or CTA pair) per SM (pair of SMs)
    const unsigned grid = (unsigned)(num_units < workers ? num_units : workers);
    (pair ? g_stat_pair : g_stat_single).fetch_add(1, std::memory_order_relaxed);
    if (real_splits > 1) g_stat_ksplit.fetch_add(1, std::memory_order_relaxed);
    if (in_kernel) g_stat_epilogue.fetch_add(1, std::memory_order_relaxed);
    if (split_here) g_stat_split_here.fetch_add(1, std::memory_order_relaxed);
    LaunchTimer timer(batch, M, N, K, pair, in_kernel, real_splits, s);
    // outputs stored by TMA when every output's layout allows it
    if (in_kernel) {
      int bw = tma_block_width(*E.pg, cls, tbn);
      bool tma = ep.vec && bw > 0 && g_tma_stores;
      // one full-shape input and warps owning 32 columns or more: the input comes into
      // the staging tile by TMA as well, and the outputs leave in 32-column boxes
      const int kin = single_full_input(*E.pg, cls);
      const bool wide_in = tma && tbn / 2 >= 32 && kin >= 0 && make_in_map(&ep.imap, E.inputs[kin], N, M, batch);
      if (wide_in) bw = 32;
      for (int k = 0; tma && k < E.pg->num_outputs; ++k)
        tma = make_out_map(&ep.omap[k], E.outputs[k], N, M, batch, ldc, strideC, bw);
      ep.tma = tma;
      rc = launch_epilogue_gemm(E, cls, ep, oa.mn, ob.mn, tbn, mAh, mAl, mBh, mBl, ga, grid, pair,
                                tma ? bw : 0, wide_in && tma, s);
    } else {
      // C, or the K-split partials [split][batch][M][N] as Z = splits x batch slices
      // (32-column swizzled boxes when a warp owns at least 32 columns; see StoreEpi)
      const int sbw = tbn / 2 >= 32 ? 32 : tbn / 2 < EPI_BW ? tbn / 2 : EPI_BW;
      ep.tma = g_tma_stores && (partial ? make_out_map(&ep.omap[0], partial, N, M, real_splits * batch, N,
                                                       M * N, sbw)
                                        : (batch == 1 || strideC % 4 == 0) &&
                                              make_out_map(&ep.omap[0], C, N, M, batch, ldc, strideC, sbw));
      rc = dispatch_gemm(oa.mn, ob.mn, tbn, mAh, mAl, mBh, mBl, ga, ep, grid, pair, split_here, s);
    }
    timer.done(rc);
    // K-split partials: summed over the splits in a fixed order (deterministic)
    if (!rc && partial) rc = fz_reduce(FZ_RSUM, product ? product : C, partial, 1, real_splits, batch * M * N, s);
    if (!rc && product) rc = epilogue_pass(E, product, batch, M, N, ldc, strideC, s);
  }
  if (product) fz_free(product, s);
  if (partial) fz_free(partial, s);
  fz_free(ws, s);
  fz_free(bt, s);
  return rc;
}

}  // namespace

extern "C" int fz_gemm_f32(int64_t batch, int64_t M, int64_t N, int64_t K, const float *A,
                           int64_t lda, int64_t strideA, int transA, const float *B, int64_t ldb,
                           int64_t strideB, int transB, float *C, int64_t ldc, int64_t strideC,
                           void *stream) {
  return gemm_impl(batch, M, N, K, A, nullptr, lda, strideA, transA, B, nullptr, ldb, strideB,
                   transB, C, ldc, strideC, Epilogue{}, stream);
}

extern "C" int fz_gemm_f32_split(int64_t batch, int64_t M, int64_t N, int64_t K, const float *A,
                                 const float *A_lo, int64_t lda, int64_t strideA, int transA,
                                 const float *B, const float *B_lo, int64_t ldb, int64_t strideB,
                                 int transB, float *C, int64_t ldc, int64_t strideC, void *stream) {
  return gemm_impl(batch, M, N, K, A, A_lo, lda, strideA, transA, B, B_lo, ldb, strideB, transB,
                   C, ldc, strideC, Epilogue{}, stream);
}

extern "C" int fz_gemm_f32_epilogue(int64_t batch, int64_t M, int64_t N, int64_t K, const float *A,
                                    const float *A_lo, int64_t lda, int64_t strideA, int transA,
                                    const float *B, const float *B_lo, int64_t ldb, int64_t strideB,
                                    int transB, const fz_program *epi, const fz_epi_input *inputs,
                                    float *const *outputs, int64_t ldc, int64_t strideC,
                                    void *stream) {
  FZ_REQUIRE(epi, "fz_gemm_f32_epilogue: null program");
  Epilogue E{epi, inputs, outputs};
  return gemm_impl(batch, M, N, K, A, A_lo, lda, strideA, transA, B, B_lo, ldb, strideB, transB,
                   nullptr, ldc, strideC, E, stream);
}

extern "C" int fz_gemm_epilogue_compile(const fz_program *epi, const fz_epi_input *inputs,
                                        int a_mn, int b_mn, int tile_n, int pair) {
  FZ_REQUIRE(epi, "fz_gemm_epilogue_compile: null program");
  int rc = fz::validate_program(*epi);
  if (rc) return rc;
  FZ_REQUIRE(epi->num_leaves >= 1 && epi->num_leaves <= 1 + EPI_MAX_IN &&
                 epi->num_outputs <= EPI_MAX_OUT && (epi->num_leaves == 1 || inputs),
             "fz_gemm_epilogue_compile: bad program");
  FZ_REQUIRE(pair ? tile_n == BN : (tile_n == 16 || tile_n == 64 || tile_n == BN),
             "fz_gemm_epilogue_compile: tile width must be 16, 64 or 256 (256 for pairs)");
  FZ_REQUIRE(tile_n == BN || !b_mn, "fz_gemm_epilogue_compile: narrow tiles read B K-major");
  int cls[EPI_MAX_IN] = {};
  for (int k = 0; k + 1 < epi->num_leaves; ++k) cls[k] = input_class(inputs[k]);
  std::vector<char> bin;
  std::string lowered;
  const std::string name = epilogue_kernel_name(a_mn != 0, b_mn != 0, tile_n, pair != 0);
  // every form the launch may pick: per-thread stores, bulk tensor stores from the
  // staging tile, and (one full-shape input, 32 columns or more per warp) the input
  // loaded into the tile by TMA
  int rc2 = fz::nvrtc_cubin(epilogue_source(*epi, cls, 0, false), "fz_gemm_epilogue.cu", name.c_str(), &bin,
                            &lowered);
  const int bw = tma_block_width(*epi, cls, tile_n);
  if (!rc2 && bw)
    rc2 = fz::nvrtc_cubin(epilogue_source(*epi, cls, bw, false), "fz_gemm_epilogue.cu", name.c_str(), &bin,
                          &lowered);
  if (!rc2 && tile_n / 2 >= 32 && single_full_input(*epi, cls) >= 0)
    rc2 = fz::nvrtc_cubin(epilogue_source(*epi, cls, 32, true), "fz_gemm_epilogue.cu", name.c_str(), &bin,
                          &lowered);
  return rc2;
}

extern "C" int fz_tf32_lo(float *lo, const float *x, int64_t n, void *stream) {
  FZ_REQUIRE(n >= 0, "fz_tf32_lo: negative size");
  if (n == 0) return FZ_OK;
  FZ_REQUIRE(lo && x, "fz_tf32_lo: null pointer");
  cudaStream_t s = fz::resolve(stream);
  unsigned grid = fz::grid_for(n / 4 + 1, 256, 8, 4);
  FZ_CUDA(fz::launch_pdl(lo_kernel, dim3(grid), dim3(256), 0, s, x, n, n, 1, n, n, 1, lo, nullptr));
  FZ_CHECK_LAUNCH();
  return FZ_OK;
}

extern "C" int fz_gemm_set_tma_stores(int on) {
  g_tma_stores = on != 0;
  return FZ_OK;
}

extern "C" int fz_gemm_set_tiles(int mode) {
  FZ_REQUIRE(mode == FZ_GEMM_TILES_AUTO || mode == FZ_GEMM_TILES_SINGLE || mode == FZ_GEMM_TILES_PAIR,
             "fz_gemm_set_tiles: unknown mode " + std::to_string(mode));
  g_tile_mode.store(mode, std::memory_order_relaxed);
  return FZ_OK;
}

extern "C" int fz_gemm_set_split(int mode) {
  FZ_REQUIRE(mode == FZ_GEMM_SPLIT_AUTO || mode == FZ_GEMM_SPLIT_PASS || mode == FZ_GEMM_SPLIT_IN_KERNEL,
             "fz_gemm_set_split: unknown mode");
  g_split_mode.store(mode);
  return FZ_OK;
}

extern "C" int fz_gemm_split_launches(int64_t *count) {
  FZ_REQUIRE(count, "fz_gemm_split_launches: null pointer");
  *count = g_stat_split_here.load();
  return FZ_OK;
}

extern "C" int fz_gemm_stats(int64_t counts[4]) {
  FZ_REQUIRE(counts, "fz_gemm_stats: null pointer");
  counts[0] = g_stat_pair.load();
  counts[1] = g_stat_single.load();
  counts[2] = g_stat_ksplit.load();
  counts[3] = g_stat_epilogue.load();
  return FZ_OK;
}

extern "C" int fz_gemm_timing(int on) {
  std::lock_guard<std::mutex> lk(g_timing_mu);
  for (TimedLaunch &t : g_timed) {
    g_event_pool.push_back(t.start);
    g_event_pool.push_back(t.stop);
  }
  g_timed.clear();
  g_timing_on = on != 0;
  return FZ_OK;
}

extern "C" int fz_gemm_timing_read(fz_gemm_timing_rec *out, int max, int *count) {
  FZ_REQUIRE(count && (out || max == 0) && max >= 0, "fz_gemm_timing_read: bad arguments");
  std::lock_guard<std::mutex> lk(g_timing_mu);
  int n = 0;
  for (TimedLaunch &t : g_timed) {
    if (n >= max) break;
    FZ_CUDA(cudaEventSynchronize(t.stop));
    float ms = 0.0f;
    FZ_CUDA(cudaEventElapsedTime(&ms, t.start, t.stop));
    out[n] = t.rec;
    out[n].ms = ms;
    ++n;
  }
  *count = n;
  return FZ_OK;
}
