// Normalised elementwise loop plan shared by the AOT kernels and the fused-program
// launcher: element strides, size-1 dims dropped, chained dims merged.
#pragma once

#include <cstdint>
#include <string>

#include "fusion_b200.h"

namespace fz {

int fail(int code, const std::string &msg);

constexpr int kMaxOps = FZ_MAX_LEAVES + FZ_MAX_OUTPUTS;

struct EwPlan {
  int32_t ndim;   // collapsed loop dims; the last one is the vectorised inner dim
  int32_t nops;   // operands (outputs first)
  int64_t rows;   // product of all dims but the last (1 if ndim <= 1)
  int64_t size[FZ_MAX_DIMS];
  int64_t stride[kMaxOps][FZ_MAX_DIMS];  // element strides
};

inline EwPlan contiguous_plan(int64_t n, int nops) {
  EwPlan p{};
  p.ndim = 1;
  p.nops = nops;
  p.rows = 1;
  p.size[0] = n;
  for (int k = 0; k < nops; ++k) p.stride[k][0] = 1;
  return p;
}

// Byte strides -> element strides; drop size-1 dims; merge dim d into d+1 when
// stride[k][d] == stride[k][d+1] * size[d+1] for every operand k.
inline int normalize_plan(const fz_ewise_plan &in, int nops, EwPlan &p) {
  if (in.ndim < 0 || in.ndim > FZ_MAX_DIMS)
    return fail(FZ_ERR_INVALID, "elementwise plan: ndim out of range");
  if (in.num_operands != nops && !(nops < 0 && in.num_operands > 0 && in.num_operands <= kMaxOps))
    return fail(FZ_ERR_INVALID, "elementwise plan: wrong operand count");
  nops = in.num_operands;
  p = EwPlan{};
  p.nops = nops;
  int nd = 0;
  for (int d = 0; d < in.ndim; ++d) {
    if (in.size[d] < 0) return fail(FZ_ERR_INVALID, "elementwise plan: negative extent");
    if (in.size[d] == 0) {  // empty output: nothing to do
      p.ndim = 1;
      p.rows = 0;
      p.size[0] = 0;
      return 0;
    }
    if (in.size[d] == 1) continue;
    p.size[nd] = in.size[d];
    for (int k = 0; k < nops; ++k) {
      int64_t sb = in.stride_bytes[k][d];
      if (sb % 4) return fail(FZ_ERR_INVALID, "elementwise plan: stride not a multiple of 4 bytes");
      p.stride[k][nd] = sb / 4;
    }
    ++nd;
  }
  // merge from the innermost outwards
  int w = 0;
  for (int d = 0; d < nd; ++d) {
    if (w > 0) {
      bool chain = true;
      for (int k = 0; k < nops && chain; ++k)
        chain = p.stride[k][w - 1] == p.stride[k][d] * p.size[d];
      if (chain) {
        p.size[w - 1] *= p.size[d];
        for (int k = 0; k < nops; ++k) p.stride[k][w - 1] = p.stride[k][d];
        continue;
      }
    }
    p.size[w] = p.size[d];
    for (int k = 0; k < nops; ++k) p.stride[k][w] = p.stride[k][d];
    ++w;
  }
  if (w == 0) {  // a single element
    p.ndim = 1;
    p.size[0] = 1;
    for (int k = 0; k < nops; ++k) p.stride[k][0] = 0;
    p.rows = 1;
    return 0;
  }
  p.ndim = w;
  p.rows = 1;
  for (int d = 0; d + 1 < w; ++d) p.rows *= p.size[d];
  return 0;
}

}  // namespace fz
