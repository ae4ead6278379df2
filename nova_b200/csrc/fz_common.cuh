// Shared definitions of the sm_100a backend: status plumbing, the launch counter,
// op functors with IEEE round-to-nearest fp32 semantics, and grid sizing.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>
#include <utility>
#include <vector>

#include "fusion_b200.h"

namespace fz {

// Thread-local last error message (fz_last_error).
void set_error(const std::string &msg);
void clear_error();
int fail(int code, const std::string &msg);
int cuda_fail(cudaError_t e, const char *what, const char *file, int line);

// Kernel launch accounting (fz_launch_count).
void note_launch(int n = 1);

cudaStream_t resolve(void *stream);
// Per-device int in global memory where kernels with bounded waits record a
// nonzero code when a wait expires; read and cleared by fz_kernel_status.
int device_error_word(int **word);
int num_sms();

// Fused-program support shared by the elementwise and GEMM-epilogue compilers
// (fz_fused.cu): validation, the CUDA C of a program's scalar evaluator fz_eval, and
// NVRTC compilation for sm_100a (name_expr, when given, is lowered into *lowered).
int validate_program(const fz_program &pg);
std::string program_eval_source(const fz_program &pg);
int nvrtc_cubin(const std::string &src, const char *name, const char *name_expr,
                std::vector<char> *cubin, std::string *lowered);

// Grid size for a streaming kernel: enough CTAs to cover `work_items` at
// `per_cta` items each, capped at `waves` full waves of resident CTAs (148 SMs).
inline unsigned grid_for(int64_t work_items, int64_t per_cta, int ctas_per_sm, int waves = 1) {
  int64_t need = (work_items + per_cta - 1) / per_cta;
  int64_t cap = (int64_t)num_sms() * ctas_per_sm * waves;
  if (need > cap) need = cap;
  if (need < 1) need = 1;
  return (unsigned)need;
}

// Programmatic dependent launch (PDL): `kernel` is launched on `s` with programmatic
// stream serialization, so its launch and scheduling overlap the tail of the kernel
// before it in the stream instead of starting after it has drained. The kernel must
// execute pdl_wait() before it reads or writes global memory: that returns once the
// preceding grid has completed and its memory operations are visible.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args &&...args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The same for a kernel handle (runtime-compiled kernels) and its argument array.
inline cudaError_t launch_pdl_handle(const void *kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                     void **args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, kernel, args);
}

}  // namespace fz

// First statement of a kernel launched with fz::launch_pdl: wait for the preceding
// grid in the stream (a no-op when the launch had no programmatic dependency).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

#define FZ_CUDA(call)                                                        \
  do {                                                                       \
    cudaError_t fz_e_ = (call);                                              \
    if (fz_e_ != cudaSuccess) return fz::cuda_fail(fz_e_, #call, __FILE__, __LINE__); \
  } while (0)

#define FZ_CHECK_LAUNCH()                                                    \
  do {                                                                       \
    cudaError_t fz_e_ = cudaGetLastError();                                  \
    if (fz_e_ != cudaSuccess) return fz::cuda_fail(fz_e_, "kernel launch", __FILE__, __LINE__); \
    fz::note_launch();                                                       \
  } while (0)

#define FZ_REQUIRE(cond, msg)                                                \
  do {                                                                       \
    if (!(cond)) return fz::fail(FZ_ERR_INVALID, msg);                       \
  } while (0)

// ---- device-side op functors (SimdTags.hpp:7-71 semantics) -----------------
// __f*_rn intrinsics pin round-to-nearest and forbid FMA contraction, so each op
// rounds exactly once as the reference's scalar loops do.
namespace fzd {

__device__ __forceinline__ float pow_f(float a, float b) {
  // std::pow on floats (glibc powf) is correctly rounded; a*a is the correctly
  // rounded square, so the common exponent 2 is bit-exact. Other exponents use
  // CUDA's powf.
  if (b == 2.0f) return __fmul_rn(a, a);
  return powf(a, b);
}

__device__ __forceinline__ float binop(int op, float a, float b) {
  switch (op) {
    case FZ_ADD: return __fadd_rn(a, b);
    case FZ_SUB: return __fsub_rn(a, b);
    case FZ_MUL: return __fmul_rn(a, b);
    case FZ_DIV: return __fdiv_rn(a, b);
    case FZ_POW: return pow_f(a, b);
    case FZ_MAXIMUM: return a > b ? a : b;
    case FZ_GT: return a > b ? 1.0f : 0.0f;
    case FZ_GE: return a >= b ? 1.0f : 0.0f;
  }
  return 0.0f;
}

template <int OP>
__device__ __forceinline__ float binop_t(float a, float b) {
  if constexpr (OP == FZ_ADD) return __fadd_rn(a, b);
  else if constexpr (OP == FZ_SUB) return __fsub_rn(a, b);
  else if constexpr (OP == FZ_MUL) return __fmul_rn(a, b);
  else if constexpr (OP == FZ_DIV) return __fdiv_rn(a, b);
  else if constexpr (OP == FZ_POW) return pow_f(a, b);
  else if constexpr (OP == FZ_MAXIMUM) return a > b ? a : b;
  else if constexpr (OP == FZ_GT) return a > b ? 1.0f : 0.0f;
  else return a >= b ? 1.0f : 0.0f;
}

// TF32 remainder plane of x: x - hi (hi = x with its 13 low mantissa bits cleared,
// the value a kind::tf32 MMA reads for x; the difference is exact in fp32), rounded
// to the nearest TF32 value, ties to even. The MMA reads the plane exactly, so
// hi + lo represents x to 2^-22 relative with an unbiased error (truncating the
// remainder to TF32 inside the MMA would bias every product toward zero).
__device__ __forceinline__ float tf32_lo(float a) {
  uint32_t u = __float_as_uint(__fsub_rn(a, __uint_as_float(__float_as_uint(a) & 0xffffe000u)));
  if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0xfffu + ((u >> 13) & 1u)) & 0xffffe000u;
  return __uint_as_float(u);
}

template <int OP>
__device__ __forceinline__ float unop_t(float a) {
  if constexpr (OP == FZ_EXP) return expf(a);
  else if constexpr (OP == FZ_LOG) return logf(a);
  else if constexpr (OP == FZ_SQRT) return __fsqrt_rn(a);
  else if constexpr (OP == FZ_TF32_LO) return tf32_lo(a);
  else return a;
}

}  // namespace fzd
