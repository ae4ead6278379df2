// Fused elementwise programs: lowering to CUDA C, NVRTC compilation for sm_100a,
// caching and launch.
//
// A program is a small DAG of fp32 ops over up to FZ_MAX_LEAVES input tensors,
// each broadcast into a common output index space by its own strides (the loop
// plan built by the host from Fusion's broadcast planner). The generated kernel
// reads every leaf once and writes every output once: one HBM pass per tensor
// instead of one pass per op. Each op rounds exactly as the unfused op does
// (__f*_rn intrinsics, -fmad=false), so fusing never changes a bit of the result.
//
// The generated source is specialised on the program, the per-operand class of
// the innermost stride (0 = broadcast, 1 = unit, other = general), the vector
// width (4 when every unit-stride operand is 16-byte aligned at each row), the
// index width and the loop form (tiled over rows x 1024*U columns for plans of at
// most 2 dims with a long inner dim, else a generic ND grid-stride loop). Shapes and strides stay runtime parameters, so one compiled kernel
// serves every shape with the same structure.
#include <cuda.h>
#include <nvrtc.h>

#include <cstring>
#include <mutex>
#include <cstdio>
#include <cstdlib>
#include <sstream>
#include <string>
#include <unordered_map>
#include <vector>

#include "fz_common.cuh"
#include "fz_ewise_plan.hpp"

namespace {

constexpr int kMaxOps = FZ_MAX_LEAVES + FZ_MAX_OUTPUTS;

// Kernel parameter block; the generated source declares the same layout.
struct FusedParams {
  long long rows;
  int ndim;
  int nops;
  long long size[FZ_MAX_DIMS];
  long long stride[kMaxOps][FZ_MAX_DIMS];
  float *ptr[kMaxOps];
};

const char *kPrelude = R"(
#define FZ_MAX_DIMS 8
#define FZ_MAX_OPS 16
struct FusedParams {
  long long rows;
  int ndim;
  int nops;
  long long size[FZ_MAX_DIMS];
  long long stride[FZ_MAX_OPS][FZ_MAX_DIMS];
  float *ptr[FZ_MAX_OPS];
};
__device__ __forceinline__ float fz_pow(float a, float b) {
  if (b == 2.0f) return __fmul_rn(a, a);
  return powf(a, b);
}
__device__ __forceinline__ float fz_max(float a, float b) { return a > b ? a : b; }
__device__ __forceinline__ float fz_gt(float a, float b) { return a > b ? 1.0f : 0.0f; }
__device__ __forceinline__ float fz_ge(float a, float b) { return a >= b ? 1.0f : 0.0f; }
__device__ __forceinline__ float fz_tf32_lo(float a) {
  unsigned u = __float_as_uint(__fsub_rn(a, __uint_as_float(__float_as_uint(a) & 0xffffe000u)));
  if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0xfffu + ((u >> 13) & 1u)) & 0xffffe000u;
  return __uint_as_float(u);
}
)";

std::string binop_expr(int op, const std::string &a, const std::string &b) {
  switch (op) {
    case FZ_ADD: return "__fadd_rn(" + a + ", " + b + ")";
    case FZ_SUB: return "__fsub_rn(" + a + ", " + b + ")";
    case FZ_MUL: return "__fmul_rn(" + a + ", " + b + ")";
    case FZ_DIV: return "__fdiv_rn(" + a + ", " + b + ")";
    case FZ_POW: return "fz_pow(" + a + ", " + b + ")";
    case FZ_MAXIMUM: return "fz_max(" + a + ", " + b + ")";
    case FZ_GT: return "fz_gt(" + a + ", " + b + ")";
    case FZ_GE: return "fz_ge(" + a + ", " + b + ")";
  }
  return "";
}

std::string unop_expr(int op, const std::string &a) {
  switch (op) {
    case FZ_EXP: return "expf(" + a + ")";
    case FZ_LOG: return "logf(" + a + ")";
    case FZ_SQRT: return "__fsqrt_rn(" + a + ")";
    case FZ_COPY: return a;
    case FZ_TF32_LO: return "fz_tf32_lo(" + a + ")";
  }
  return "";
}

int validate(const fz_program &pg) {
  if (pg.num_nodes < 1 || pg.num_nodes > FZ_MAX_NODES)
    return fz::fail(FZ_ERR_INVALID, "fused program: node count out of range");
  if (pg.num_leaves < 0 || pg.num_leaves > FZ_MAX_LEAVES)
    return fz::fail(FZ_ERR_INVALID, "fused program: leaf count out of range");
  if (pg.num_outputs < 1 || pg.num_outputs > FZ_MAX_OUTPUTS)
    return fz::fail(FZ_ERR_INVALID, "fused program: output count out of range");
  for (int i = 0; i < pg.num_nodes; ++i) {
    const fz_node &n = pg.nodes[i];
    int nsrc = n.kind == FZ_NODE_BINARY ? 2 : n.kind == FZ_NODE_UNARY ? 1 : 0;
    if (n.kind < 0 || n.kind > FZ_NODE_CONST)
      return fz::fail(FZ_ERR_INVALID, "fused program: bad node kind");
    if (n.kind == FZ_NODE_BINARY && (n.op < FZ_ADD || n.op > FZ_GE))
      return fz::fail(FZ_ERR_INVALID, "fused program: bad binary op");
    if (n.kind == FZ_NODE_UNARY && (n.op < FZ_EXP || n.op > FZ_TF32_LO))
      return fz::fail(FZ_ERR_INVALID, "fused program: bad unary op");
    const int32_t srcs[2] = {n.src0, n.src1};
    for (int k = 0; k < nsrc; ++k) {
      int s = srcs[k];
      if (s >= 0 ? s >= i : (-1 - s) >= pg.num_leaves)
        return fz::fail(FZ_ERR_INVALID, "fused program: operand reference out of range");
    }
  }
  for (int k = 0; k < pg.num_outputs; ++k)
    if (pg.out_node[k] < 0 || pg.out_node[k] >= pg.num_nodes)
      return fz::fail(FZ_ERR_INVALID, "fused program: output node out of range");
  return FZ_OK;
}

std::string ref_name(int s) { return s >= 0 ? "t" + std::to_string(s) : "l" + std::to_string(-1 - s); }

// cls[k]: inner-stride class of operand k (0 broadcast, 1 unit, 2 general)
// Tiled form for plans of at most 2 dims on the 128-bit path with inner >= 1024:
// tiles of one row x 1024*U columns walked by whole CTAs, one division per tile,
// each thread loading its U float4 groups of every leaf before evaluating.
void generate_tiles(std::ostringstream &o, const fz_program &pg, const int *cls, int U) {
  const int nout = pg.num_outputs, nleaf = pg.num_leaves, nops = nout + nleaf;
  o << "extern \"C\" __global__ void __launch_bounds__(256) fz_fused(const FusedParams p) {\n"
    << "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n"
    << "  const long long inner = p.size[p.ndim - 1];\n"
    << "  const long long TW = " << 1024 * U << ";\n"
    << "  const long long ctiles = (inner + TW - 1) / TW;\n"
    << "  const long long total = p.rows * ctiles;\n";
  for (int k = 0; k < nops; ++k)
    o << "  const long long r" << k << " = p.ndim > 1 ? p.stride[" << k << "][0] : 0;\n";
  o << "  for (long long t = blockIdx.x; t < total; t += gridDim.x) {\n"
    << "    const long long row = t / ctiles;\n"
    << "    const long long c0 = (t - row * ctiles) * TW + threadIdx.x * 4;\n";
  for (int k = 0; k < nops; ++k)
    o << "    float *b" << k << " = p.ptr[" << k << "] + row * r" << k << ";\n";
  for (int lk = 0; lk < nleaf; ++lk) o << "    float4 v" << lk << "[" << U << "];\n";
  o << "#pragma unroll\n    for (int j = 0; j < " << U << "; ++j) {\n"
    << "      const long long c = c0 + j * 1024;\n"
    << "      if (c + 4 <= inner) {\n";
  for (int k = nout; k < nops; ++k) {
    const int lk = k - nout;
    if (cls[k] == 1)
      o << "        v" << lk << "[j] = *reinterpret_cast<const float4 *>(b" << k << " + c);\n";
    else
      o << "        { const float s = b" << k << "[0]; v" << lk << "[j] = make_float4(s, s, s, s); }\n";
  }
  o << "      }\n    }\n";
  o << "#pragma unroll\n    for (int j = 0; j < " << U << "; ++j) {\n"
    << "      const long long c = c0 + j * 1024;\n"
    << "      if (c + 4 <= inner) {\n";
  for (int k = 0; k < nout; ++k) o << "        float4 q" << k << ";\n";
  const char *lanes[4] = {"x", "y", "z", "w"};
  for (int ln = 0; ln < 4; ++ln) {
    o << "        fz_eval(";
    for (int lk = 0; lk < nleaf; ++lk) o << "v" << lk << "[j]." << lanes[ln] << ", ";
    for (int k = 0; k < nout; ++k) o << "q" << k << "." << lanes[ln] << (k + 1 < nout ? ", " : "");
    o << ");\n";
  }
  for (int k = 0; k < nout; ++k)
    o << "        *reinterpret_cast<float4 *>(b" << k << " + c) = q" << k << ";\n";
  o << "      } else {\n"
    << "        for (long long e = c; e < inner; ++e) {\n";
  for (int k = nout; k < nops; ++k)
    o << "          const float e" << (k - nout) << " = b" << k << "[" << (cls[k] == 1 ? "e" : "0") << "];\n";
  for (int k = 0; k < nout; ++k) o << "          float s" << k << ";\n";
  o << "          fz_eval(";
  for (int lk = 0; lk < nleaf; ++lk) o << "e" << lk << ", ";
  for (int k = 0; k < nout; ++k) o << "s" << k << (k + 1 < nout ? ", " : "");
  o << ");\n";
  for (int k = 0; k < nout; ++k) o << "          b" << k << "[e] = s" << k << ";\n";
  o << "        }\n      }\n    }\n  }\n}\n";
}

// The prelude and the scalar evaluator fz_eval(l0.., &o0..) of a program.
void generate_eval(std::ostringstream &o, const fz_program &pg) {
  o << kPrelude;
  const int nout = pg.num_outputs, nleaf = pg.num_leaves;
  o << "__device__ __forceinline__ void fz_eval(";
  for (int k = 0; k < nleaf; ++k) o << "float l" << k << ", ";
  for (int k = 0; k < nout; ++k) o << "float &o" << k << (k + 1 < nout ? ", " : "");
  o << ") {\n";
  for (int i = 0; i < pg.num_nodes; ++i) {
    const fz_node &n = pg.nodes[i];
    o << "  const float t" << i << " = ";
    if (n.kind == FZ_NODE_BINARY) o << binop_expr(n.op, ref_name(n.src0), ref_name(n.src1));
    else if (n.kind == FZ_NODE_UNARY) o << unop_expr(n.op, ref_name(n.src0));
    else {
      uint32_t bits;
      std::memcpy(&bits, &n.imm, 4);
      o << "__int_as_float(" << (int32_t)bits << ")";
    }
    o << ";\n";
  }
  for (int k = 0; k < nout; ++k) o << "  o" << k << " = t" << pg.out_node[k] << ";\n";
  o << "}\n";
}

std::string generate(const fz_program &pg, const int *cls, int vec, bool i64, int tiles_u) {
  std::ostringstream o;
  generate_eval(o, pg);
  const int nout = pg.num_outputs, nleaf = pg.num_leaves, nops = nout + nleaf;
  if (tiles_u) {
    generate_tiles(o, pg, cls, tiles_u);
    return o.str();
  }
  const char *IDX = i64 ? "long long" : "int";
  o << "extern \"C\" __global__ void __launch_bounds__(256) fz_fused(const FusedParams p) {\n"
    << "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n"
    << "  typedef " << IDX << " IDX;\n"
    << "  const long long inner = p.size[p.ndim - 1];\n"
    << "  const IDX gpr = (IDX)((inner + " << vec - 1 << ") / " << vec << ");\n"
    << "  const IDX total = (IDX)p.rows * gpr;\n"
    << "  const IDX step = (IDX)gridDim.x * blockDim.x;\n";
  for (int k = 0; k < nops; ++k)
    o << "  const long long si" << k << " = p.stride[" << k << "][p.ndim - 1];\n";
  o << "  for (IDX g = (IDX)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += step) {\n"
    << "    IDX row = g / gpr;\n"
    << "    const long long col = (long long)(g - row * gpr) * " << vec << ";\n";
  for (int k = 0; k < nops; ++k) o << "    long long off" << k << " = 0;\n";
  o << "    for (int d = p.ndim - 2; d >= 0; --d) {\n"
    << "      const IDX sz = (IDX)p.size[d];\n"
    << "      const IDX q = row / sz;\n"
    << "      const long long i = (long long)(row - q * sz);\n"
    << "      row = q;\n";
  for (int k = 0; k < nops; ++k) o << "      off" << k << " += i * p.stride[" << k << "][d];\n";
  o << "    }\n";
  if (vec == 4) {
    o << "    if (col + 4 <= inner) {\n";
    for (int k = nout; k < nops; ++k) {
      int lk = k - nout;
      o << "      const float *pl" << lk << " = p.ptr[" << k << "] + off" << k << ";\n";
      if (cls[k] == 1)
        o << "      const float4 v" << lk << " = *reinterpret_cast<const float4 *>(pl" << lk
          << " + col);\n";
      else
        o << "      const float s" << lk << " = pl" << lk << "[0];\n"
          << "      const float4 v" << lk << " = make_float4(s" << lk << ", s" << lk << ", s" << lk
          << ", s" << lk << ");\n";
    }
    for (int k = 0; k < nout; ++k) o << "      float4 r" << k << ";\n";
    const char *lanes[4] = {"x", "y", "z", "w"};
    for (int ln = 0; ln < 4; ++ln) {
      o << "      fz_eval(";
      for (int lk = 0; lk < nleaf; ++lk) o << "v" << lk << "." << lanes[ln] << ", ";
      for (int k = 0; k < nout; ++k) o << "r" << k << "." << lanes[ln] << (k + 1 < nout ? ", " : "");
      o << ");\n";
    }
    for (int k = 0; k < nout; ++k)
      o << "      *reinterpret_cast<float4 *>(p.ptr[" << k << "] + off" << k << " + col) = r" << k
        << ";\n";
    o << "      continue;\n    }\n";
  }
  o << "    for (int v = 0; v < " << vec << " && col + v < inner; ++v) {\n"
    << "      const long long c = col + v;\n";
  for (int k = nout; k < nops; ++k)
    o << "      const float e" << (k - nout) << " = p.ptr[" << k << "][off" << k << " + c * si" << k
      << "];\n";
  for (int k = 0; k < nout; ++k) o << "      float q" << k << ";\n";
  o << "      fz_eval(";
  for (int lk = 0; lk < nleaf; ++lk) o << "e" << lk << ", ";
  for (int k = 0; k < nout; ++k) o << "q" << k << (k + 1 < nout ? ", " : "");
  o << ");\n";
  for (int k = 0; k < nout; ++k)
    o << "      p.ptr[" << k << "][off" << k << " + c * si" << k << "] = q" << k << ";\n";
  o << "    }\n  }\n}\n";
  return o.str();
}

struct Cache {
  std::mutex mu;
  std::unordered_map<std::string, cudaKernel_t> kernels;
};
Cache &cache() {
  static Cache c;
  return c;
}

int compile(const std::string &src, cudaKernel_t *out) {
  std::vector<char> bin;
  int rc = fz::nvrtc_cubin(src, "fz_fused.cu", nullptr, &bin, nullptr);
  if (rc) return rc;
  cudaLibrary_t lib;
  cudaError_t e = cudaLibraryLoadData(&lib, bin.data(), nullptr, nullptr, 0, nullptr, nullptr, 0);
  if (e != cudaSuccess) return fz::cuda_fail(e, "cudaLibraryLoadData(fused)", __FILE__, __LINE__);
  e = cudaLibraryGetKernel(out, lib, "fz_fused");
  if (e != cudaSuccess) return fz::cuda_fail(e, "cudaLibraryGetKernel(fused)", __FILE__, __LINE__);
  return FZ_OK;
}

}  // namespace

namespace fz {

int validate_program(const fz_program &pg) { return validate(pg); }

std::string program_eval_source(const fz_program &pg) {
  std::ostringstream o;
  generate_eval(o, pg);
  return o.str();
}

int nvrtc_cubin(const std::string &src, const char *name, const char *name_expr,
                std::vector<char> *cubin, std::string *lowered) {
  nvrtcProgram prog;
  nvrtcResult r = nvrtcCreateProgram(&prog, src.c_str(), name, 0, nullptr, nullptr);
  if (r != NVRTC_SUCCESS) return fail(FZ_ERR_JIT, std::string("nvrtcCreateProgram: ") + nvrtcGetErrorString(r));
  if (name_expr) nvrtcAddNameExpression(prog, name_expr);
  // FZ_NVRTC_VERBOSE=1 prints ptxas' resource usage (registers, spills, shared
  // memory) of every runtime-compiled kernel to stderr.
  static const bool verbose = std::getenv("FZ_NVRTC_VERBOSE") != nullptr;
  const char *opts[] = {"--gpu-architecture=sm_100a", "--fmad=false", "--std=c++17", "-lineinfo",
                        "--ptxas-options=-v"};
  r = nvrtcCompileProgram(prog, verbose ? 5 : 4, opts);
  if (r == NVRTC_SUCCESS && verbose) {
    size_t n = 0;
    nvrtcGetProgramLogSize(prog, &n);
    std::string log(n, '\0');
    nvrtcGetProgramLog(prog, log.data());
    std::fprintf(stderr, "[fz nvrtc] %s (%s):\n%s\n", name, name_expr ? name_expr : "", log.c_str());
  }
  if (r != NVRTC_SUCCESS) {
    size_t n = 0;
    nvrtcGetProgramLogSize(prog, &n);
    std::string log(n, '\0');
    nvrtcGetProgramLog(prog, log.data());
    nvrtcDestroyProgram(&prog);
    return fail(FZ_ERR_JIT, std::string("NVRTC compilation of ") + name + " failed: " + log);
  }
  if (name_expr && lowered) {
    const char *ln = nullptr;
    nvrtcGetLoweredName(prog, name_expr, &ln);
    *lowered = ln ? ln : "";
  }
  size_t nbin = 0;
  nvrtcGetCUBINSize(prog, &nbin);
  cubin->resize(nbin);
  nvrtcGetCUBIN(prog, cubin->data());
  nvrtcDestroyProgram(&prog);
  return FZ_OK;
}

}  // namespace fz

extern "C" {

int fz_fused_launch(const fz_program *prog, const fz_ewise_plan *plan, float *const *outputs,
                    const float *const *leaves, void *stream) {
  FZ_REQUIRE(prog && plan && outputs, "fz_fused_launch: null argument");
  int rc = validate(*prog);
  if (rc) return rc;
  const int nout = prog->num_outputs, nleaf = prog->num_leaves, nops = nout + nleaf;
  FZ_REQUIRE(plan->num_operands == nops, "fz_fused_launch: plan operand count != outputs + leaves");
  FZ_REQUIRE(nleaf == 0 || leaves, "fz_fused_launch: null leaves");
  fz::EwPlan p;
  rc = fz::normalize_plan(*plan, nops, p);
  if (rc) return rc;
  const int64_t inner = p.size[p.ndim - 1];
  const int64_t total = p.rows * inner;
  if (total == 0) return FZ_OK;
  if (p.rows == 0) return FZ_OK;
  float *ptrs[kMaxOps] = {};
  for (int k = 0; k < nout; ++k) {
    FZ_REQUIRE(outputs[k], "fz_fused_launch: null output");
    ptrs[k] = outputs[k];
  }
  for (int k = 0; k < nleaf; ++k) {
    FZ_REQUIRE(leaves[k], "fz_fused_launch: null leaf");
    ptrs[nout + k] = const_cast<float *>(leaves[k]);
  }
  int cls[kMaxOps];
  bool vec = true;
  for (int k = 0; k < nops; ++k) {
    int64_t si = p.stride[k][p.ndim - 1];
    cls[k] = si == 0 ? 0 : si == 1 ? 1 : 2;
    if (k < nout && cls[k] != 1) vec = false;  // outputs must be unit-stride to vectorise
    if (cls[k] == 2) vec = false;
    if (cls[k] == 1) {
      if ((uintptr_t)ptrs[k] & 15) vec = false;
      for (int d = 0; d + 1 < p.ndim; ++d)
        if (p.stride[k][d] % 4) vec = false;
    }
  }
  const int V = vec ? 4 : 1;
  const int64_t groups = p.rows * ((inner + V - 1) / V);
  const bool i64 = groups > (int64_t)0x7fffffff - (int64_t)fz::num_sms() * 2048;
  // tiled form: one leaf keeps 8 float4 per thread in flight, more leaves 4 each
  const int U = (vec && p.ndim <= 2 && inner >= 1024)
                    ? ((nleaf <= 1 && inner >= 8192) ? 8 : inner >= 4096 ? 4 : inner >= 2048 ? 2 : 1)
                    : 0;
  // cache key: program bytes + specialisation
  std::string key(reinterpret_cast<const char *>(prog), offsetof(fz_program, nodes) +
                                                            sizeof(fz_node) * prog->num_nodes);
  for (int k = 0; k < nops; ++k) key.push_back((char)('0' + cls[k]));
  key.push_back((char)V);
  key.push_back(i64 ? 'L' : 'I');
  key.push_back((char)('0' + U));
  cudaKernel_t kern = nullptr;
  {
    Cache &c = cache();
    std::lock_guard<std::mutex> lk(c.mu);
    auto it = c.kernels.find(key);
    if (it != c.kernels.end()) {
      kern = it->second;
    } else {
      rc = compile(generate(*prog, cls, V, i64, U), &kern);
      if (rc) return rc;
      c.kernels.emplace(key, kern);
    }
  }
  FusedParams fp{};
  fp.rows = p.rows;
  fp.ndim = p.ndim;
  fp.nops = nops;
  for (int d = 0; d < p.ndim; ++d) fp.size[d] = p.size[d];
  for (int k = 0; k < nops; ++k) {
    for (int d = 0; d < p.ndim; ++d) fp.stride[k][d] = p.stride[k][d];
    fp.ptr[k] = ptrs[k];
  }
  unsigned grid;
  if (U) {
    const int64_t tiles = p.rows * ((inner + 1024 * U - 1) / (1024 * U));
    grid = (unsigned)(tiles < (int64_t)fz::num_sms() * 8 ? tiles : fz::num_sms() * 8);
  } else {
    grid = fz::grid_for(groups, 256 * 2, 8);
  }
  void *args[] = {&fp};
  FZ_CUDA(fz::launch_pdl_handle((const void *)kern, dim3(grid), dim3(256), 0, fz::resolve(stream), args));
  fz::note_launch();
  return FZ_OK;
}

int fz_fused_cache_size(void) {
  Cache &c = cache();
  std::lock_guard<std::mutex> lk(c.mu);
  return (int)c.kernels.size();
}

}  // extern "C"
