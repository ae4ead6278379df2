/* fusion_b200.h -- C ABI of the B200 (sm_100a) compute backend for Fusion.
 *
 * Every entry point is `extern "C"`, takes plain pointers, sizes and POD plans,
 * and returns an int status (FZ_OK == 0). On failure the thread-local message
 * from fz_last_error() says what went wrong. No torch or C++ types cross this
 * boundary. Device pointers are CUDA device addresses; streams are cudaStream_t
 * passed as void*. NULL stream means the calling thread's library stream on the
 * current device (fz_default_stream()).
 *
 * Each function names the reference interface it replaces (paths relative to the
 * pytergeist/Nova repository). In the reference those interfaces are C++ templates
 * inside fusion/src/Fusion; the C++ host layer of this project (nova_b200/host)
 * keeps their callers and routes them here.
 */
#ifndef FUSION_B200_H
#define FUSION_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FZ_MAX_DIMS 8     /* loop dims of an elementwise plan (after collapsing) */
#define FZ_MAX_LEAVES 12  /* input tensors of one fused elementwise program */
#define FZ_MAX_NODES 48   /* ops of one fused elementwise program */
#define FZ_MAX_OUTPUTS 4  /* outputs of one fused elementwise program */

enum fz_status {
  FZ_OK = 0,
  FZ_ERR_INVALID = 1,     /* bad argument: shape, pointer, op code, size */
  FZ_ERR_CUDA = 2,        /* a CUDA runtime/driver call failed */
  FZ_ERR_OOM = 3,         /* device allocation failed */
  FZ_ERR_NCCL = 4,        /* an NCCL call failed */
  FZ_ERR_UNSUPPORTED = 5, /* no sm_100 device, or a feature this build lacks */
  FZ_ERR_TIMEOUT = 6,     /* a bounded wait ran out (collective watchdog) */
  FZ_ERR_JIT = 7          /* runtime compilation of a fused program failed */
};

/* Binary ops: the tags of fusion/src/Fusion/cpu/simd/SimdTags.hpp:7-53. */
enum fz_binop {
  FZ_ADD = 0, FZ_SUB = 1, FZ_MUL = 2, FZ_DIV = 3, FZ_POW = 4,
  FZ_MAXIMUM = 5, /* a > b ? a : b (MaximumSIMD) */
  FZ_GT = 6,      /* (a > b) as 1.0f/0.0f (GreaterThanSIMD) */
  FZ_GE = 7       /* (a >= b) as 1.0f/0.0f (GreaterThanEqualSIMD) */
};

/* Unary ops: SimdTags.hpp:55-71 (exp/log/sqrt) plus identity (copy). */
/* FZ_TF32_LO: x minus x with its 13 low mantissa bits cleared, rounded to the nearest
 * TF32 value (ties to even): the remainder plane a 3xTF32 GEMM reads (fz_tf32_lo);
 * not an op of Fusion's API. */
enum fz_unop { FZ_EXP = 0, FZ_LOG = 1, FZ_SQRT = 2, FZ_COPY = 3, FZ_TF32_LO = 4 };

/* Reductions: SumSIMD via reduction_tag (fusion/src/Fusion/core/TensorIter.hpp:251-297);
 * mean = sum / (float)len (fusion/src/Fusion/ops/Reduce.hpp:27-36); max has no
 * reference counterpart (NaN-propagating, +0 ranks above -0). */
enum fz_redop { FZ_RSUM = 0, FZ_RMEAN = 1, FZ_RMAX = 2 };

/* ---- runtime ------------------------------------------------------------ */

/* Thread-local text of the last failure on this thread ("" if none). */
const char *fz_last_error(void);
int fz_version(void);

/* Number of visible CUDA devices of compute capability 10.x. */
int fz_device_count(int *count);
/* Make `device` current for this thread and set up its stream and memory pool.
 * Replaces Device::validate_device (fusion/src/Fusion/device/Device.h:31-33),
 * which only admitted CPU index <= 0. */
int fz_set_device(int device);
int fz_get_device(int *device);
/* The calling thread's stream on the current device (created on first use). */
void *fz_default_stream(void);
int fz_stream_sync(void *stream);
/* The calling thread's upload stream on the current device (created on first use):
 * host-to-device copies issued on it run beside the compute stream's work; a block
 * fz_malloc'd on it and freed on another stream is reused only after that stream has
 * passed the free. Null if the stream could not be created (fz_last_error says why). */
void *fz_upload_stream(void);
/* A second non-blocking stream on the current device (for collectives that overlap the
 * thread's compute stream), and its release. */
int fz_stream_create(void **stream);
int fz_stream_destroy(void *stream);
/* Work submitted to `waiter` after this call starts only once the work submitted to
 * `signaler` before it has finished (an event recorded on `signaler`, waited on by
 * `waiter`; NULL means the thread's stream). The host does not block. */
int fz_stream_wait(void *waiter, void *signaler);
/* An event marking the work submitted to `stream` so far (NULL: the thread's stream);
 * fz_stream_wait_event makes `waiter` wait for it; fz_event_destroy releases it. */
int fz_event_record(void **event, void *stream);
int fz_stream_wait_event(void *waiter, void *event);
int fz_event_destroy(void *event);
int fz_device_sync(void);
/* Queue a host-side pause of `seconds` (0..60) on `stream`: work queued after it starts
 * that much later; nothing runs on the GPU meanwhile. For exercising the host-side
 * watchdog (fz_comm_wait) with a stream that is late, without any device fault.
 * Replaces no reference interface. */
int fz_stream_delay(void *stream, double seconds);

/* Stream-ordered device memory. fz_free(ptr, stream) marks the block free after the
 * work submitted to `stream` so far; it goes back to the free list of the stream it
 * was allocated on, and the next fz_malloc of the same size class there takes it back
 * without a driver call (waiting for `stream` first when that is another stream).
 * Misses go to the device's pool (cudaMallocAsync, release threshold raised).
 * Replaces PoolAllocator::allocate/deallocate
 * (fusion/src/Fusion/alloc/BFCPoolAllocator.cpp:59-111) for tensor storage.
 * fz_free of a pointer fz_malloc did not return fails with FZ_ERR_INVALID. */
int fz_malloc(void **ptr, size_t bytes, void *stream);
int fz_free(void *ptr, void *stream);
/* Return the current device's cached blocks to the driver and trim its pool
 * (synchronises the device). fz_malloc does this by itself before it reports OOM. */
int fz_pool_release(void);
/* reserved: bytes the current device's pool holds (in use, cached or pool-internal);
 * used: bytes handed out by fz_malloc and not freed yet. */
int fz_pool_stats(size_t *reserved, size_t *used);
/* bytes: freed blocks the current device's block cache holds for reuse (not yet
 * returned to the driver pool). */
int fz_pool_cached(size_t *bytes);

/* Copies. d2h waits for the stream so the host buffer is valid on return.
 * Replaces the host std::copy of tensor_to_numpy / set_values
 * (fusion/src/Fusion/python/tensor/Helpers.hpp:14-44, BindTensor.hpp:58-70). */
int fz_memcpy_h2d(void *dst, const void *src, size_t bytes, void *stream);
int fz_memcpy_d2h(void *dst, const void *src, size_t bytes, void *stream);
int fz_memcpy_d2d(void *dst, const void *src, size_t bytes, void *stream);
/* dst[i] = value for i < n. Replaces fill/zeros/ones
 * (fusion/src/Fusion/TensorFactory.hpp:12-36) and RawTensor::clear
 * (fusion/src/Fusion/core/RawTensor.hpp:140-149). */
int fz_fill_f32(float *dst, float value, int64_t n, void *stream);
/* Pinned host memory for staging (H2D/D2H at full PCIe/C2C rate). */
int fz_host_alloc(void **ptr, size_t bytes);
int fz_host_free(void *ptr);

/* Device-side timing of work on a stream: record a start/stop pair around
 * launches and read milliseconds (waits for the stop event). */
int fz_timer_create(void **timer);
int fz_timer_start(void *timer, void *stream);
int fz_timer_stop(void *timer, void *stream);
int fz_timer_elapsed_ms(void *timer, float *ms);
int fz_timer_destroy(void *timer);
/* Number of kernels this library has launched in this process. */
int64_t fz_launch_count(void);
/* Synchronise the current device and report whether any kernel with bounded
 * waits (the GEMM's mbarrier pipeline) gave up since the last call: FZ_OK, or
 * FZ_ERR_TIMEOUT with the kernel's code in fz_last_error(). Clears the record. */
int fz_kernel_status(void);

/* ---- elementwise --------------------------------------------------------- */

/* Loop plan of one elementwise launch: the output index space (outermost dim
 * first) and, per operand, the BYTE stride of each loop dim (0 = broadcast).
 * Operand 0 is the output. Same meaning as LoopDim::size / LoopDim::stride_bytes
 * of BroadcastPlan (fusion/src/Fusion/core/TensorPlan.h:42-68), with the dims
 * stored column-wise. ndim may be 0 (one element). */
typedef struct fz_ewise_plan {
  int32_t ndim;
  int32_t num_operands;
  int64_t size[FZ_MAX_DIMS];
  int64_t stride_bytes[FZ_MAX_LEAVES + FZ_MAX_OUTPUTS][FZ_MAX_DIMS];
} fz_ewise_plan;

/* out = op(a, b) over `plan` (operands: 0 = out, 1 = a, 2 = b), fp32 IEEE,
 * round-to-nearest, no contraction. Operand order is taken as given: the
 * exchange that the reference's scalar-LHS path performs
 * (fusion/src/Fusion/cpu/simd/SimdTraits.hpp:44-47) is decided by the caller.
 * Replaces binary_ewise_tag (fusion/src/Fusion/core/TensorIter.hpp:96-178) and
 * simd_traits<Tag,float>::execute_contiguous (SimdTraits.hpp:26-148). */
int fz_ewise_binary(int op, const fz_ewise_plan *plan, float *out, const float *a,
                    const float *b, void *stream);

/* Contiguous fast path of the above: out[i] = op(a[i], b[i]) for i < n
 * (PlanMeta.hpp:103-107 fastpath; VecFallback.hpp:76-102). */
int fz_ewise_binary_contig(int op, int64_t n, float *out, const float *a,
                           const float *b, void *stream);

/* out = op(a) over `plan` (operands: 0 = out, 1 = a). Replaces unary_ewise_tag
 * (fusion/src/Fusion/core/TensorIter.hpp:180-249) and simd::{exp,log,sqrt}_contiguous
 * (fusion/src/Fusion/cpu/simd/VecFallback.hpp:41-60). exp/log call CUDA's expf/logf,
 * sqrt is the IEEE square root. */
int fz_ewise_unary(int op, const fz_ewise_plan *plan, float *out, const float *a,
                   void *stream);

/* x[i] -= y[i] for i < n, in place: fusion::math::sub_inplace
 * (fusion/src/Fusion/ops/Ewise.hpp:69-83), which forces the contiguous path over
 * x's element count whatever y's shape. */
int fz_sub_inplace(float *x, const float *y, int64_t n, void *stream);

/* ---- fused elementwise programs (fusion IR) ------------------------------ */

/* One node of a fused program. Operand references: values >= 0 name an earlier
 * node; -1-k names leaf k (an input tensor). FZ_NODE_CONST nodes carry their
 * value in `imm`. Binary nodes compute op(src0, src1) with the operand order
 * given (any reference operand exchange is already applied by the caller). */
enum fz_node_kind { FZ_NODE_BINARY = 0, FZ_NODE_UNARY = 1, FZ_NODE_CONST = 2 };
typedef struct fz_node {
  int32_t kind;
  int32_t op;
  int32_t src0, src1;
  float imm;
} fz_node;

/* A fused elementwise program: nodes in topological order, leaves bound to the
 * plan's operands num_outputs..num_outputs+num_leaves-1 and outputs bound to plan
 * operands 0..num_outputs-1 (output k stores node out_node[k]). The program is
 * lowered to CUDA C, compiled for sm_100a by NVRTC once per distinct structure,
 * cached, and launched as a single pass over the plan's index space. There is no
 * reference counterpart: the reference runs each op as its own pass
 * (fusion/src/Fusion/core/TensorIter.hpp:96-249). */
typedef struct fz_program {
  int32_t num_nodes;
  int32_t num_leaves;
  int32_t num_outputs;
  int32_t out_node[FZ_MAX_OUTPUTS];
  fz_node nodes[FZ_MAX_NODES];
} fz_program;

int fz_fused_launch(const fz_program *prog, const fz_ewise_plan *plan,
                    float *const *outputs, const float *const *leaves, void *stream);
/* Number of distinct fused kernels compiled so far in this process. */
int fz_fused_cache_size(void);

/* ---- reductions ---------------------------------------------------------- */

/* Reduce the middle dim of a contiguous [outer, len, inner] view:
 * out[o, i] = red_{r < len} in[o, r, i]. Replaces reduction_tag
 * (fusion/src/Fusion/core/TensorIter.hpp:251-297) driven by make_reduction_meta
 * (fusion/src/Fusion/core/PlanMeta.hpp:148-182); the global reduction is
 * outer = inner = 1. Long reductions are split over CTAs; the partials live in
 * stream-ordered scratch taken from the device pool and released after the launch. */
int fz_reduce(int op, float *out, const float *in, int64_t outer, int64_t len,
              int64_t inner, void *stream);

/* fz_reduce without any device allocation, for callers that must not allocate
 * while they run (a runtime that reserves and accounts for all device memory
 * itself, or a latency-critical loop that must not grow the pool). It has no
 * counterpart in the reference. Split partials go to a fixed 8 MiB array
 * compiled into the library (held on every GPU that loads it until exit) instead
 * of the pool; the kernels and split plan are fz_reduce's, so results are
 * bit-identical. Returns FZ_ERR_INVALID when a reduction's plan needs more
 * partials than the array holds. The first call on a device looks up the array's
 * address (make it before any stream capture). Calls share the array: calls that
 * overlap on the GPU race and must be serialised by the caller. */
int fz_reduce_noalloc(int op, float *out, const float *in, int64_t outer, int64_t len,
                      int64_t inner, void *stream);

/* ---- layout -------------------------------------------------------------- */

/* Materialised swapaxes of a contiguous tensor: out = in with axes a1, a2
 * exchanged. Replaces serial::swapaxes (fusion/src/Fusion/kernels/Serial.hpp:90-123)
 * behind fusion::math::linalg::swapaxes (fusion/src/Fusion/ops/Linalg.hpp:109-128). */
int fz_swapaxes(float *out, const float *in, const int64_t *shape, int ndim, int a1,
                int a2, void *stream);

/* ---- GEMM ---------------------------------------------------------------- */

/* Batched fp32 GEMM in 3xTF32 on the tcgen05 tensor cores (TMEM accumulators,
 * TMA-fed shared-memory tiles): C[b] = op(A[b]) @ op(B[b]) for b < batch, with
 * op(X) = X or X^T (trans flags), element leading dimensions and batch strides.
 * Each fp32 operand is split into a TF32-exact high part and a low remainder
 * and C = Ah*Bh + Ah*Bl + Al*Bh, accumulated in fp32. Row-major throughout.
 * Replaces contraction_tag's BLAS path (fusion/src/Fusion/core/TensorIter.hpp:299-323)
 * and batched_gemm_rowmajor_nn -> cblas_sgemm
 * (fusion/src/Fusion/cpu/blas/backend/BlasCblas.hpp:19-39). */
int fz_gemm_f32(int64_t batch, int64_t M, int64_t N, int64_t K,
                const float *A, int64_t lda, int64_t strideA, int transA,
                const float *B, int64_t ldb, int64_t strideB, int transB,
                float *C, int64_t ldc, int64_t strideC, void *stream);

/* fz_gemm_f32 with the low TF32 remainders of the operands supplied by the caller:
 * A_lo[i] = fz_tf32_lo(A)[i] at A's own leading dimension and batch stride (same for
 * B_lo), so an operand read by several GEMMs (an activation in the forward and the
 * weight-gradient GEMM) is split once. A NULL plane, or an operand TMA cannot
 * address (leading dimension or batch stride not a multiple of 4 floats, base not
 * 16-byte aligned, broadcast batch), is split here as in fz_gemm_f32. */
int fz_gemm_f32_split(int64_t batch, int64_t M, int64_t N, int64_t K,
                      const float *A, const float *A_lo, int64_t lda, int64_t strideA, int transA,
                      const float *B, const float *B_lo, int64_t ldb, int64_t strideB, int transB,
                      float *C, int64_t ldc, int64_t strideC, void *stream);
/* One input of a GEMM epilogue program (program leaf k >= 1 reads inputs[k-1];
 * leaf 0 is the product). At output element (b, i, j) it reads
 * ptr[b * batch_stride + i * row_stride + j * col_stride], col_stride 0 or 1: a
 * bias row bias[j] has batch_stride = row_stride = 0 and col_stride = 1, a
 * same-shape tensor row_stride = its row pitch, a per-row value col_stride = 0. */
typedef struct fz_epi_input {
  const float *ptr;
  int64_t batch_stride, row_stride, col_stride;
} fz_epi_input;

/* GEMM with a fused elementwise epilogue. With P[b] = op(A[b]) @ op(B[b]) computed
 * as by fz_gemm_f32_split, the program `epi` (declared below) is evaluated at every
 * output element (b, i, j) with leaf 0 = P[b][i][j] and leaf k = inputs[k-1] at
 * (b, i, j); output k is stored at outputs[k][b * strideC + i * ldc + j]. The results
 * equal, bit for bit, fz_gemm_f32_split into a buffer followed by fz_fused_launch of
 * `epi` over it; P itself is stored only if the program outputs it (an FZ_COPY node
 * of leaf 0). The program is compiled into the epilogue of the GEMM kernel (NVRTC,
 * cached per program structure, input classes and kernel variant), so P never goes
 * through HBM; when the GEMM splits K (few output tiles) or K = 0, P is formed in a
 * workspace and the program runs as one fused pass over it. At most FZ_MAX_LEAVES - 1
 * inputs and FZ_MAX_OUTPUTS outputs. No reference counterpart: the reference runs
 * the product and each following op as separate passes
 * (fusion/src/Fusion/core/TensorIter.hpp:96-249, 299-323). */
struct fz_program;
int fz_gemm_f32_epilogue(int64_t batch, int64_t M, int64_t N, int64_t K,
                         const float *A, const float *A_lo, int64_t lda, int64_t strideA, int transA,
                         const float *B, const float *B_lo, int64_t ldb, int64_t strideB, int transB,
                         const struct fz_program *epi, const fz_epi_input *inputs,
                         float *const *outputs, int64_t ldc, int64_t strideC, void *stream);
/* Compile (NVRTC only: no device is needed, nothing is loaded or cached) the GEMM
 * kernel variant with `epi` as its epilogue: A / B MN-major (a_mn, b_mn), output
 * tile width tile_n (16, 64 or 256; narrow tiles take a K-major B), CTA pair (tile_n
 * 256). Returns FZ_ERR_JIT with the compiler log in fz_last_error on failure. */
int fz_gemm_epilogue_compile(const struct fz_program *epi, const fz_epi_input *inputs,
                             int a_mn, int b_mn, int tile_n, int pair);
/* lo[i] = tf32_rn(x[i] - tf32_hi(x[i])) for i < n: tf32_hi clears the 13 low mantissa
 * bits (what the MMA reads for x), the difference is exact, and tf32_rn rounds it to the
 * nearest TF32 value, ties to even (the plane fz_gemm_f32_split takes). */
int fz_tf32_lo(float *lo, const float *x, int64_t n, void *stream);
/* GEMM tile schedule for the calls that follow (process-wide): FZ_GEMM_TILES_AUTO picks
 * CTA pairs (256 x 256 tiles, tcgen05 cta_group::2) for products with at least 256 rows,
 * more than 64 columns and enough tiles to occupy every SM pair, single CTAs otherwise
 * (128 x 256 tiles, or 128 x 64 / 128 x 16 for outputs of at most 64 / 16 columns);
 * SINGLE and PAIR force one schedule (a pair schedule on fewer rows computes zero rows).
 * Both meet the same error bounds; with the same K split (none, or the same count) an
 * output element is accumulated from the same K chunks in the same order. */
enum fz_gemm_tiles { FZ_GEMM_TILES_AUTO = 0, FZ_GEMM_TILES_SINGLE = 1, FZ_GEMM_TILES_PAIR = 2 };
int fz_gemm_set_tiles(int mode);
/* How GEMM kernels write their outputs, for the calls that follow (process-wide):
 * on (default), through TMA bulk tensor stores from shared-memory staging tiles
 * wherever every output is 16-byte aligned with a pitch of a multiple of 4 floats;
 * off, by per-thread stores. Results are identical either way. Replaces no reference
 * interface (the reference's cblas_sgemm writes C directly). */
int fz_gemm_set_tma_stores(int on);
/* Where the TF32 remainder planes that a GEMM call is not given come from, for the calls
 * that follow (process-wide): FZ_GEMM_SPLIT_PASS and FZ_GEMM_SPLIT_AUTO (default), a
 * separate pass writes each into a workspace before the GEMM; FZ_GEMM_SPLIT_IN_KERNEL,
 * the GEMM kernel derives them in shared memory from the raw operand tiles and needs no
 * workspace (full-width tiles, plain output, operands TMA can address; other calls use
 * the pass). The in-kernel split is slower on B200 for all but single-wave products
 * (1024^3: 0.87x the time; batched 64x512^3 1.3x; large products 1.5-1.9x), hence
 * not the default. Results are identical bit for bit. Replaces
 * no reference interface. fz_gemm_split_launches: how many launches so far derived
 * them in shared memory. */
enum fz_gemm_split { FZ_GEMM_SPLIT_AUTO = 0, FZ_GEMM_SPLIT_PASS = 1, FZ_GEMM_SPLIT_IN_KERNEL = 2 };
int fz_gemm_set_split(int mode);
int fz_gemm_split_launches(int64_t *count);
/* Launches of the GEMM kernels so far in this process, by schedule: counts[0] CTA-pair
 * launches, [1] single-CTA launches, [2] launches split over K, [3] launches with a
 * fused epilogue program. Instrumentation for tests and measurement; replaces no
 * reference interface. */
int fz_gemm_stats(int64_t counts[4]);
/* Device time of each GEMM main-kernel launch (instrumentation; no reference
 * counterpart). fz_gemm_timing(1) clears the records and starts recording a CUDA
 * event pair around every launch on its own stream, up to FZ_GEMM_TIMING_MAX
 * launches; fz_gemm_timing(0) clears and stops. fz_gemm_timing_read waits for the
 * recorded launches and copies up to `max` records, in launch order. */
#define FZ_GEMM_TIMING_MAX 4096
typedef struct fz_gemm_timing_rec {
  int64_t batch, M, N, K;
  int32_t pair;      /* CTA-pair kernel */
  int32_t epilogue;  /* fused epilogue program compiled in */
  int32_t splits;    /* K splits (partials summed by a separate launch, not timed here) */
  float ms;          /* event-timed duration of the launch */
} fz_gemm_timing_rec;
int fz_gemm_timing(int on);
int fz_gemm_timing_read(fz_gemm_timing_rec *out, int max, int *count);

/* ---- device-side random numbers (Philox-4x32-10) ------------------------- */

/* Counter-based generator, a device-side alternative to Random::uniform_base
 * (fusion/src/Fusion/Random.hpp:20-36, std::mt19937 on the host, whose stream it does
 * not reproduce). Element i of the stream (seed, offset) is lane (offset + i) % 4 of
 * Philox-4x32-10 at counter (offset + i) / 4 under key seed; u = (bits >> 8) * 2^-24.
 * offset must be a multiple of 4; out 16-byte aligned. */
int fz_philox_uniform(float *out, int64_t n, uint64_t seed, uint64_t offset, float lo, float hi,
                      void *stream);
/* Nova's Dropout (nova/src/blocks/regularisation/dropout.py:17-23) in one pass with
 * the mask drawn in the kernel: out[i] = (x[i] * (u_i > rate ? 1 : 0)) / keep, u_i the
 * stream's uniform in [0, 1), keep = fp32(1 - rate) as Nova passes it (Fusion's `>=`
 * is `>`). No mask tensor is written. */
int fz_philox_dropout(float *out, const float *x, int64_t n, float rate, float keep, uint64_t seed,
                      uint64_t offset, void *stream);

/* ---- collectives (data-parallel MLP step) -------------------------------- */

#define FZ_UNIQUE_ID_BYTES 128
/* NCCL unique id for rank 0 to share with the other ranks. */
int fz_comm_unique_id(unsigned char id[FZ_UNIQUE_ID_BYTES]);
/* Join a communicator of `world` ranks on the current device. */
int fz_comm_init(void **comm, int world, int rank,
                 const unsigned char id[FZ_UNIQUE_ID_BYTES]);
/* fp32 all-reduce of `count` floats from `send` into `recv` (may be the same
 * buffer): sum over ranks, then multiply by `scale` (1/world for a mean). */
int fz_comm_allreduce(void *comm, const float *send, float *recv, int64_t count, float scale,
                      void *stream);
/* Start / end a group of collectives issued back to back (one NCCL launch). */
int fz_comm_group_start(void);
int fz_comm_group_end(void);
int fz_comm_broadcast(void *comm, float *buf, int64_t count, int root, void *stream);
/* Wait for `stream` with a host-side deadline; on expiry abort the communicator
 * and return FZ_ERR_TIMEOUT instead of blocking for ever. */
int fz_comm_wait(void *comm, void *stream, double timeout_s);
int fz_comm_destroy(void *comm);

#ifdef __cplusplus
}
#endif
#endif /* FUSION_B200_H */
