// Device-side counter-based random numbers: Philox-4x32-10.
//
// Philox (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3",
// SC'11) maps a 128-bit counter and a 64-bit key to four 32-bit outputs through ten
// rounds of two 32x32->64 multiplies (multipliers 0xD2511F53 and 0xCD9E8D57), the key
// bumped by the Weyl constants 0x9E3779B9 and 0xBB67AE85 between rounds. Being a pure
// function of (counter, key), every element is generated independently, by any
// thread, in any order: element i of a stream with key `seed` at position `offset`
// takes lane (offset + i) % 4 of the block whose counter is (offset + i) / 4 (64 bits,
// upper counter words zero). A uniform in [0, 1) is the output's top 24 bits times
// 2^-24 (exact in fp32); [lo, hi) is fmaf(hi - lo, u, lo), pulled below hi where the
// rounding reaches it.
//
// The reference's Random draws from std::mt19937 on the host
// (fusion/src/Fusion/Random.hpp:20-36) and Nova's Dropout builds its mask from such a
// draw (nova/src/blocks/regularisation/dropout.py:17-23); that sequential stream
// cannot be produced in parallel, so these generators give different (equally
// distributed) numbers. Random.uniform_cpp keeps the reference's stream; these are the
// device-side alternative (no host generation, no upload, and for dropout no random
// tensor in HBM at all: the mask is drawn inside the kernel that applies it).
#include <cstdint>

#include "fz_common.cuh"

namespace {

struct U4 {
  uint32_t x, y, z, w;
};

__device__ __forceinline__ U4 philox4x32_10(uint64_t ctr, uint64_t key) {
  uint32_t c0 = (uint32_t)ctr, c1 = (uint32_t)(ctr >> 32), c2 = 0u, c3 = 0u;
  uint32_t k0 = (uint32_t)key, k1 = (uint32_t)(key >> 32);
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
    const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return U4{c0, c1, c2, c3};
}

__device__ __forceinline__ float to_range(uint32_t bits, float lo, float span, float hi) {
  const float u = (float)(bits >> 8) * 5.9604644775390625e-08f;  // 2^-24
  float v = __fmaf_rn(span, u, lo);
  if (v >= hi) v = nextafterf(hi, lo);  // the largest float below hi
  return v;
}

__device__ __forceinline__ uint32_t lane(const U4 &r, int k) {
  return k == 0 ? r.x : k == 1 ? r.y : k == 2 ? r.z : r.w;
}

// One Philox block (4 values) per thread per iteration; `offset` is a multiple of 4,
// so element i's block is offset/4 + i/4 and its lane i % 4.
__global__ void __launch_bounds__(256) uniform_kernel(float *__restrict__ out, int64_t n, uint64_t seed,
                                                      uint64_t base, float lo, float hi) {
  pdl_wait();
  const float span = hi - lo;
  const int64_t blocks = (n + 3) / 4;
  for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < blocks;
       b += (int64_t)gridDim.x * blockDim.x) {
    const U4 r = philox4x32_10(base + (uint64_t)b, seed);
    const int64_t i = b * 4;
    if (i + 4 <= n) {
      reinterpret_cast<float4 *>(out)[b] = make_float4(to_range(r.x, lo, span, hi), to_range(r.y, lo, span, hi),
                                                       to_range(r.z, lo, span, hi), to_range(r.w, lo, span, hi));
    } else {
      for (int k = 0; i + k < n; ++k) out[i + k] = to_range(lane(r, k), lo, span, hi);
    }
  }
}

// out = (x * m) / keep with m = (u > rate) ? 1 : 0 and u the stream's uniform in
// [0, 1): Nova's Dropout, inputs * (uniform >= rate) / (1 - rate), in one pass, each op
// rounded as the unfused ops are. Fusion's `>=` computes `>` (RawTensor.hpp:207-209),
// hence the strict comparison; keep is the divisor as Nova passes it, fp32(1 - rate).
__global__ void __launch_bounds__(256) dropout_kernel(float *__restrict__ out, const float *__restrict__ x,
                                                      int64_t n, float rate, float keep, uint64_t seed,
                                                      uint64_t base) {
  pdl_wait();
  const int64_t blocks = (n + 3) / 4;
  for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < blocks;
       b += (int64_t)gridDim.x * blockDim.x) {
    const U4 r = philox4x32_10(base + (uint64_t)b, seed);
    const int64_t i = b * 4;
    auto one = [&](uint32_t bits, float v) {
      const float u = (float)(bits >> 8) * 5.9604644775390625e-08f;
      const float m = u > rate ? 1.0f : 0.0f;
      return __fdiv_rn(__fmul_rn(v, m), keep);
    };
    if (i + 4 <= n) {
      const float4 v = reinterpret_cast<const float4 *>(x)[b];
      reinterpret_cast<float4 *>(out)[b] = make_float4(one(r.x, v.x), one(r.y, v.y), one(r.z, v.z), one(r.w, v.w));
    } else {
      for (int k = 0; i + k < n; ++k) out[i + k] = one(lane(r, k), x[i + k]);
    }
  }
}

}  // namespace

extern "C" int fz_philox_uniform(float *out, int64_t n, uint64_t seed, uint64_t offset, float lo, float hi,
                                 void *stream) {
  FZ_REQUIRE(n >= 0, "fz_philox_uniform: negative size");
  if (n == 0) return FZ_OK;
  FZ_REQUIRE(out, "fz_philox_uniform: null pointer");
  FZ_REQUIRE(((uintptr_t)out & 15) == 0, "fz_philox_uniform: output must be 16-byte aligned");
  FZ_REQUIRE(offset % 4 == 0, "fz_philox_uniform: offset must be a multiple of 4");
  FZ_REQUIRE(lo < hi, "fz_philox_uniform: need min < max");
  const int64_t blocks = (n + 3) / 4;
  FZ_CUDA(fz::launch_pdl(uniform_kernel, dim3(fz::grid_for(blocks, 256 * 4, 8)), dim3(256), 0, fz::resolve(stream),
                         out, n, seed, offset / 4, lo, hi));
  FZ_CHECK_LAUNCH();
  return FZ_OK;
}

extern "C" int fz_philox_dropout(float *out, const float *x, int64_t n, float rate, float keep,
                                 uint64_t seed, uint64_t offset, void *stream) {
  FZ_REQUIRE(n >= 0, "fz_philox_dropout: negative size");
  if (n == 0) return FZ_OK;
  FZ_REQUIRE(out && x, "fz_philox_dropout: null pointer");
  FZ_REQUIRE((((uintptr_t)out | (uintptr_t)x) & 15) == 0, "fz_philox_dropout: operands must be 16-byte aligned");
  FZ_REQUIRE(offset % 4 == 0, "fz_philox_dropout: offset must be a multiple of 4");
  FZ_REQUIRE(rate >= 0.0f && rate < 1.0f && keep > 0.0f, "fz_philox_dropout: rate must be in [0, 1)");
  const int64_t blocks = (n + 3) / 4;
  FZ_CUDA(fz::launch_pdl(dropout_kernel, dim3(fz::grid_for(blocks, 256 * 4, 8)), dim3(256), 0, fz::resolve(stream),
                         out, x, n, rate, keep, seed, offset / 4));
  FZ_CHECK_LAUNCH();
  return FZ_OK;
}
