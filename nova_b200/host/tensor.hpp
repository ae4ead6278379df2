// Fusion's tensor value type and op API over B200 device storage.
//
// RawTensor keeps the reference's shape/strides/dtype/device value semantics
// (fusion/src/Fusion/core/RawTensor.hpp:36-318): copies are shallow and share one
// Storage, so in-place writes through any copy are seen by all of them.
//
// Storage holds an Expr, the node of the fusion IR:
//   * Leaf  -- a materialised device buffer (HBM, from the stream-ordered pool)
//   * Const -- a value broadcast over a shape (zeros_like, ones_like, scalars)
//   * Unary / Binary -- a pending elementwise op over other Exprs
// Elementwise ops build pending nodes instead of running; a node is lowered to one
// fused sm_100a kernel when its value is first needed (a GEMM, reduction, transpose,
// host read-back, or the size limit of a fused program). Lowering turns the node
// into a Leaf in place, so every holder sees the result and nothing is computed
// twice. In-place writes (`-=`, set_values, clear) rebind the Storage to a new Expr
// and leave the old one to pending readers, which keeps program order without
// copies.
#pragma once

#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "fusion_b200.h"

namespace fusion_b200 {

// ---- error convention: FUSION_CHECK-style std::runtime_error ---------------
[[noreturn]] void throw_check(const char *file, int line, const std::string &msg);
void fz_check(int rc, const char *what);

#define FB_CHECK(cond, msg)                                                          \
  do {                                                                                \
    if (!(cond)) ::fusion_b200::throw_check(__FILE__, __LINE__, (msg));               \
  } while (0)

// ---- device / dtype (fusion/src/Fusion/device/Device.h, core/Dtype.h) -------
enum class DeviceType : int { CPU = 0, CUDA = 1, METAL = 2 };
enum class DType : int { FLOAT32 = 0, FLOAT64 = 1, INT32 = 2, INT64 = 3, BOOL = 4 };

// Device tag. Every tensor of this backend lives in HBM of a CUDA device; a CPU
// tag (Nova's default) places it on the calling thread's current CUDA device.
// Index rules: CPU admits idx <= 0 as the reference does; CUDA admits -1 (the
// current device) or 0 .. device_count-1.
struct Device {
  DeviceType type{DeviceType::CPU};
  int idx{-1};
  Device() = default;
  Device(DeviceType t, int i = -1);
  bool operator==(const Device &o) const { return type == o.type && idx == o.idx; }
  bool is_cpu() const { return type == DeviceType::CPU; }
  bool is_cuda() const { return type == DeviceType::CUDA; }
  int cuda_index() const;  // the CUDA ordinal the data lives on
};

size_t dtype_size(DType d);

// ---- device memory -----------------------------------------------------------
// Device storage of one value. A buffer is written once, by the kernel or copy that
// produces it, before anything reads it; later values (in-place ops, set_values,
// all-reduce results) go to new buffers. So data derived from the values, like the
// TF32 remainder plane a GEMM reads, can be kept with the buffer.
struct DeviceBuffer {
  float *ptr = nullptr;
  size_t numel = 0;
  int device = 0;
  std::shared_ptr<DeviceBuffer> tf32_lo;  // fz_tf32_lo(ptr), made by the first GEMM reading it
  void *ready = nullptr;  // event after the producing work, recorded by flush() for read-backs
  void mark_ready();      // (re)record `ready` at the current point of the thread's stream
  explicit DeviceBuffer(size_t n);
  DeviceBuffer(size_t n, void *stream);  // allocated for first use on `stream`
  ~DeviceBuffer();
  DeviceBuffer(const DeviceBuffer &) = delete;
  DeviceBuffer &operator=(const DeviceBuffer &) = delete;
};

// A GEMM whose launch is deferred (Expr::Gemm): the operands as the GEMM reads them,
// materialised, with their TF32 remainder planes, kept alive by the node.
struct GemmSpec {
  int64_t batch = 1, M = 0, N = 0, K = 0;
  const float *pa = nullptr, *la = nullptr, *pb = nullptr, *lb = nullptr;
  int64_t lda = 0, sA = 0, ldb = 0, sB = 0;
  int transA = 0, transB = 0;
  std::shared_ptr<DeviceBuffer> keep_a, keep_b, keep_la, keep_lb;
};

// ---- fusion IR node --------------------------------------------------------------
struct Expr {
  // Reduce: a pending single- or multi-axis reduction of `a` (fz_redop in op), kept
  // pending so a following reduction over an adjacent axis can join it (one pass over
  // the merged axes); lowered by itself, never inside an elementwise program.
  // Gemm: a pending product [batch..., M, N] (`gemm`). The first elementwise program
  // lowered over it runs in the GEMM's epilogue (fz_gemm_f32_epilogue), and the
  // product itself is stored only if something else still holds the node; lowered by
  // any other reader, it is a plain GEMM into a buffer.
  // Swap: `a` with its last two axes exchanged (swapaxes(-1, -2), Nova's `.T`), kept as
  // a view: a GEMM reads the source in the other operand layout, a swapaxes of it
  // gives the source back, and any other reader gets it materialised by the
  // transpose kernel.
  enum Kind { Leaf, Const, Unary, Binary, Reduce, Gemm, Swap } kind;
  int op = 0;  // fz_binop / fz_unop / fz_redop
  std::vector<size_t> shape;
  std::shared_ptr<Expr> a, b;
  std::shared_ptr<GemmSpec> gemm;     // Gemm
  std::shared_ptr<DeviceBuffer> buf;  // Leaf
  float imm = 0.0f;                   // Const
  int red_lo = 0, red_hi = 0;         // Reduce: axes [red_lo, red_hi] of a's shape
  bool red_keep = false;              // Reduce: reduced axes kept as extent 1
  int nodes_ub = 1;                   // upper bounds used by the fusion size policy
  int leaves_ub = 0;
  bool gemm_below = false;            // a pending GEMM may sit in this DAG (never false if one does)
  size_t numel() const;
};
using ExprPtr = std::shared_ptr<Expr>;

struct Storage {
  ExprPtr expr;
  explicit Storage(ExprPtr e) : expr(std::move(e)) {}
  // Materialise (if pending) and return the device pointer.
  float *data();
  size_t numel() const { return expr->numel(); }
};

// Fusion policy switches (fusion enabled by default).
void set_fusion_enabled(bool on);
bool fusion_enabled();
// Keep each GEMM operand's TF32 remainder plane with its buffer, so an operand read
// by several GEMMs is split once (on by default; off frees the memory it holds on to
// for buffers made later).
void set_split_cache_enabled(bool on);
bool split_cache_enabled();
// Defer GEMM launches so that the elementwise program reading a product runs in the
// GEMM's epilogue (on by default; off launches every GEMM where it is called).
void set_gemm_epilogue_enabled(bool on);
bool gemm_epilogue_enabled();
// GEMMs launched with a fused epilogue program so far in this process.
int64_t epilogue_gemms();
// Lower a pending node to one fused kernel (no-op for a Leaf).
void materialize(const ExprPtr &e);
// Keep `swapaxes(-1, -2)` pending as a view (on by default; off materialises every
// swapaxes where it is called, as the reference does).
void set_swap_views_enabled(bool on);
bool swap_views_enabled();
int64_t swap_materializations();
// TF32 remainder planes split by a separate pass (fz_tf32_lo) so far: operands whose
// plane no producing kernel wrote (host uploads, values lowered without a plane).
int64_t lo_splits();
// Launch plans (per-operand broadcast strides over the output, chained dims merged)
// are cached by the shapes they are built from: hits and misses so far.
int64_t plan_cache_hits();
int64_t plan_cache_misses();
// Lower a pending node and its TF32 remainder plane in one fused pass (GEMM operands).
void materialize_with_lo(const ExprPtr &e);
// Lower several pending nodes of one shape as outputs of one fused program.
void materialize_group(const std::vector<ExprPtr> &eps);
int64_t fused_launches();

class RawTensor {
 public:
  RawTensor() = default;
  // From host data (copied to the device).
  RawTensor(std::vector<size_t> shape, const float *data, DType dtype, Device device);
  RawTensor(std::vector<size_t> shape, const std::vector<float> &data, DType dtype, Device device);
  // Zero-initialised.
  RawTensor(std::vector<size_t> shape, DType dtype, Device device);
  // From an Expr (internal).
  RawTensor(ExprPtr e, DType dtype, Device device);

  static RawTensor full(const std::vector<size_t> &shape, float value, DType dtype, Device device);
  // A tensor over an existing device buffer (numel = product of shape).
  static RawTensor from_buffer(std::shared_ptr<DeviceBuffer> buf, std::vector<size_t> shape,
                               DType dtype, Device device);
  static RawTensor scalar(float v, DType dtype, Device device) { return full({1}, v, dtype, device); }

  DType dtype() const { return dtype_; }
  size_t dtype_size() const { return fusion_b200::dtype_size(dtype_); }
  size_t rank() const { return shape_.size(); }
  size_t ndims() const { return shape_.size(); }
  const std::vector<size_t> &shape() const { return shape_; }
  std::vector<int64_t> strides() const { return strides_; }
  Device device() const { return device_; }
  bool is_contiguous() const { return true; }
  bool is_initialised() const { return storage_ != nullptr; }
  bool empty() const { return !storage_ || storage_->numel() == 0; }
  size_t size() const { return storage_ ? storage_->numel() : 0; }
  size_t flat_size() const { return size(); }
  const std::shared_ptr<Storage> &storage() const { return storage_; }
  ExprPtr expr() const { return storage_ ? storage_->expr : nullptr; }
  bool pending() const { return storage_ && storage_->expr->kind != Expr::Leaf; }

  // Device pointer (materialises a pending value).
  float *data() const;
  // Host copy of the values.
  std::vector<float> to_host() const;
  void to_host(float *dst) const;

  // In-place writes, visible to every shallow copy.
  void set_values(const float *src, size_t n);
  // Point the storage at an already computed device buffer of the same size.
  void rebind_buffer(std::shared_ptr<DeviceBuffer> buf);
  void clear();                           // zero (RawTensor.hpp:140-149)
  void assign(const RawTensor &other);    // RawTensor.hpp:151-157
  RawTensor &operator-=(const RawTensor &other);  // sub_inplace (ops/Ewise.hpp:69-83)

  RawTensor operator+(const RawTensor &o) const;
  RawTensor operator-(const RawTensor &o) const;
  RawTensor operator*(const RawTensor &o) const;
  RawTensor operator/(const RawTensor &o) const;
  RawTensor operator>(const RawTensor &o) const;
  RawTensor operator>=(const RawTensor &o) const;  // the reference calls greater (RawTensor.hpp:207-209)
  RawTensor maximum(const RawTensor &o) const;
  RawTensor pow(const RawTensor &o) const;
  RawTensor operator+(float s) const;
  RawTensor operator-(float s) const;
  RawTensor operator*(float s) const;
  RawTensor operator/(float s) const;
  RawTensor operator>=(float s) const;
  RawTensor maximum(float s) const;
  RawTensor pow(float s) const;
  RawTensor sqrt() const;
  RawTensor log() const;
  RawTensor exp() const;
  RawTensor sum(size_t axis, bool keepdim) const;
  RawTensor mean(size_t axis, bool keepdim) const;
  RawTensor max(size_t axis, bool keepdim) const;
  RawTensor matmul(const RawTensor &o) const;
  RawTensor swapaxes(int a1, int a2) const;

  std::string repr() const;
  std::string shape_str() const;

 private:
  std::shared_ptr<Storage> storage_;
  std::vector<size_t> shape_;
  std::vector<int64_t> strides_;
  DType dtype_{DType::FLOAT32};
  Device device_{};
  void set_contiguous_strides();
};

constexpr size_t kGlobalReduceAxis = static_cast<size_t>(-1);

namespace math {
RawTensor binary(int op, const RawTensor &x, const RawTensor &y);
RawTensor unary(int op, const RawTensor &x);
RawTensor reduce(int op, const RawTensor &x, size_t axis, bool keepdim);
// C = op(A) @ op(B) over the last two dims, batch dims equal (ops/Linalg.hpp:76-107).
RawTensor matmul(const RawTensor &A, const RawTensor &B, bool transA = false, bool transB = false);
RawTensor swapaxes(const RawTensor &x, int a1, int a2);
void sub_inplace(RawTensor &x, const RawTensor &y);
// (x * (u > rate)) / keep with u the Philox stream (seed, offset) in [0, 1): Nova's
// Dropout composition in one pass (fz_philox_dropout), the mask never stored.
RawTensor dropout(const RawTensor &x, float rate, float keep, uint64_t seed, uint64_t offset);
// n values of the Philox stream (seed, offset) in [lo, hi) (fz_philox_uniform).
RawTensor philox_uniform(const std::vector<size_t> &shape, float lo, float hi, uint64_t seed,
                         uint64_t offset, DType dtype, Device device);
RawTensor flat_prefix(const RawTensor &x, size_t n, const std::vector<size_t> &shape);
}  // namespace math

RawTensor zeros_like(const RawTensor &t);
RawTensor ones_like(const RawTensor &t);

// Make the calling thread's CUDA device current for `d` and return its ordinal.
int bind_device(const Device &d);

}  // namespace fusion_b200
