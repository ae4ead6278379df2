// Fusion's autodiff layer over the B200 tensor: ADTensor, the tape Engine, the
// op registry and the thread-local engine context.
//
// Semantics follow the reference exactly, because they are observable:
//   * tracing only under an installed engine with grad enabled and an input that
//     requires grad (autodiff/AutodiffMode.hpp:34-42, Dispatch.hpp:43-101);
//   * value ids: inputs tracked on first use, op outputs allocated after the
//     forward (Engine.hpp:48-63, 120-126; Graph.hpp build_node with static arity 0);
//   * backward runs every node of the tape in reverse Kahn order, seeding the
//     root with ones and missing output grads with zeros, and accumulates input
//     grads by `dst = src` (sharing storage) or `dst = dst + src`
//     (Engine.hpp:65-102, 277-336; Sort.hpp:36-74);
//   * leaf grads share storage with the engine's grad buffers, so a second
//     backward on the same engine, which clears those buffers, zeroes them
//     (Engine.hpp:277-283, ADTensor.hpp:144-154);
//   * the op formulas and their quirks (registry/**): traced mean returns its
//     input, >= is >, Add aliases g0 for both inputs, no broadcast reduction.
// The op results are the lazy RawTensors of tensor.hpp, so each backward formula
// becomes one fused kernel at the point its value is consumed. Gradients of
// inputs that no reader can observe (untracked, non-leaf inputs such as the [1]
// scalar of `maximum(0)`) are not computed.
#pragma once

#include <memory>
#include <functional>
#include <optional>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "tensor.hpp"

namespace fusion_b200 {

using ValueID = int64_t;
using NodeID = int64_t;

struct OpParam {
  size_t axis = kGlobalReduceAxis;
  bool keepdim = false;
  int axis1 = 0, axis2 = 0;
  // Dropout: the Philox stream (seed, offset) its mask is drawn from, the rate and
  // the divisor keep = fp32(1 - rate)
  uint64_t rng_seed = 0, rng_offset = 0;
  float rate = 0.0f, keep = 1.0f;
};

struct OpContext {
  std::unordered_map<std::string, RawTensor> saved;
  std::unordered_map<std::string, int> ints;
  OpParam param;  // the op's parameters, for backward formulas that need them
  const RawTensor &load(const std::string &k) const;
};

enum class OpKind {
  Add, Subtract, Multiply, Divide, Pow, Maximum, GreaterThan, GreaterThanEqual,
  MatMul, Exp, Log, Sqrt, Sum, Mean, SwapAxes,
  Dropout  // no reference op: Nova's Dropout composition with a device-drawn mask
};
const char *op_name(OpKind k);

// Forward of registry op `k` (runs under a no-grad guard in the engine).
std::vector<RawTensor> op_forward(OpKind k, OpContext &ctx, const std::vector<RawTensor> &in,
                                  const OpParam &p);
// Backward: `need[j]` false means input j's gradient cannot be observed and may be
// returned uninitialised.
std::vector<RawTensor> op_backward(OpKind k, OpContext &ctx, const RawTensor &g0,
                                   const std::vector<bool> &need);

struct TapeNode {
  OpKind kind;
  OpContext ctx;
  std::vector<ValueID> inputs, outputs;
};

struct BackwardResult {
  std::unordered_map<int64_t, RawTensor> grads;
};

class Engine {
 public:
  Engine() = default;
  Engine(const Engine &) = delete;
  Engine &operator=(const Engine &) = delete;

  ValueID apply(OpKind k, const std::vector<RawTensor> &ins, const std::vector<ValueID> &vids,
                const OpParam &p);
  BackwardResult backward(ValueID seed);
  ValueID track_input(const RawTensor &raw, bool requires_grad);
  RawTensor materialise(ValueID vid) const;
  bool has_value(ValueID vid) const;
  size_t num_nodes() const { return nodes_.size(); }

 private:
  std::vector<TapeNode> nodes_;
  std::vector<NodeID> produced_by_;
  std::vector<std::vector<NodeID>> consumed_by_;
  std::vector<RawTensor> val_, grad_;
  std::unordered_set<int64_t> requires_grad_set_;
  int64_t value_counter_ = 0;

  ValueID new_input_value();
  ValueID new_intermediate_value();
  std::vector<NodeID> topo_order() const;
};

// Called during Engine::backward, on the engine's thread, as soon as the gradient of a
// leaf value that requires grad is complete (every node reading it has contributed), so
// a caller can start using it (an all-reduce on another stream) while the rest of the
// backward is still being computed. Thread-local; an empty function removes it.
using GradReadyHook = std::function<void(ValueID, const RawTensor &)>;
void set_grad_ready_hook(GradReadyHook hook);

// thread-local engine slot (EngineContext.hpp:10-25)
Engine *engine_instance();
void set_engine_instance(Engine *e);
bool grad_enabled();
void set_grad_enabled(bool on);
// autodiff.enabled(state): installs / removes a thread-local default engine
// (autodiff/AutodiffBridge.hpp).
void set_autodiff_enabled(bool on);

class NoGradGuard {
 public:
  NoGradGuard();
  ~NoGradGuard();
  NoGradGuard(const NoGradGuard &) = delete;
  NoGradGuard &operator=(const NoGradGuard &) = delete;

 private:
  bool prev_;
};

class EngineScope {
 public:
  void enter() {
    set_engine_instance(&eng_);
    active_ = true;
  }
  void exit() {
    set_engine_instance(nullptr);
    active_ = false;
  }
  ~EngineScope() {
    if (active_) exit();
  }
  Engine &engine() { return eng_; }

 private:
  Engine eng_;
  bool active_ = false;
};

class ADTensor {
 public:
  ADTensor() = default;
  explicit ADTensor(RawTensor raw, bool requires_grad = false)
      : raw_(std::move(raw)), requires_grad_(requires_grad) {}
  ADTensor(const ADTensor &o);
  ADTensor &operator=(const ADTensor &o);
  ~ADTensor();

  const RawTensor &raw() const { return raw_; }
  RawTensor &raw() { return raw_; }
  std::vector<size_t> shape() const { return raw_.shape(); }
  size_t rank() const { return raw_.rank(); }
  size_t flat_size() const { return raw_.flat_size(); }
  Device device() const { return raw_.device(); }
  DType dtype() const { return raw_.dtype(); }

  ValueID vid() const { return vid_; }
  void set_vid(ValueID v) { vid_ = v; }
  bool has_vid() const { return vid_ >= 0; }
  bool requires_grad() const { return requires_grad_; }
  void set_requires_grad(bool v) { requires_grad_ = v; }

  ValueID ensure_vid();
  void backward();
  std::optional<ADTensor> grad() const;

  ADTensor binary_op(OpKind k, const ADTensor &other) const;
  ADTensor binary_scalar(OpKind k, float s) const;
  ADTensor unary_op(OpKind k, const OpParam &p = {}) const;

 private:
  RawTensor raw_;
  std::shared_ptr<RawTensor> grad_;
  ValueID vid_ = -1;
  bool requires_grad_ = false;

  void set_leaf();
  void attach_grads(BackwardResult &res) const;
  friend class Engine;
};

}  // namespace fusion_b200
