// Autodiff engine and op registry (see autodiff.hpp for the semantics kept).
#include "autodiff.hpp"

#include <algorithm>
#include <queue>
#include <sstream>

namespace fusion_b200 {

// ---------------------------------------------------------------- context
static thread_local Engine *t_engine = nullptr;
static thread_local bool t_grad_enabled = true;
static thread_local std::vector<ADTensor *> t_leaf_tensors;

Engine *engine_instance() { return t_engine; }
void set_engine_instance(Engine *e) { t_engine = e; }
bool grad_enabled() { return t_grad_enabled; }
void set_grad_enabled(bool on) { t_grad_enabled = on; }

void set_autodiff_enabled(bool on) {
  t_grad_enabled = on;
  static thread_local Engine default_engine;
  set_engine_instance(on ? &default_engine : nullptr);
}

NoGradGuard::NoGradGuard() : prev_(t_grad_enabled) { t_grad_enabled = false; }
NoGradGuard::~NoGradGuard() { t_grad_enabled = prev_; }

static Engine &current_engine() {
  FB_CHECK(t_engine != nullptr, "No Engine instance set in context");
  return *t_engine;
}

const RawTensor &OpContext::load(const std::string &k) const {
  auto it = saved.find(k);
  FB_CHECK(it != saved.end(), "Context::load: key not found: " + k);
  return it->second;
}

const char *op_name(OpKind k) {
  switch (k) {
    case OpKind::Add: return "Add";
    case OpKind::Subtract: return "Subtract";
    case OpKind::Multiply: return "Multiply";
    case OpKind::Divide: return "Divide";
    case OpKind::Pow: return "Pow";
    case OpKind::Maximum: return "Maximum";
    case OpKind::GreaterThan: return "GreaterThan";
    case OpKind::GreaterThanEqual: return "GreaterThanEqual";
    case OpKind::MatMul: return "MatMul";
    case OpKind::Exp: return "Exp";
    case OpKind::Log: return "Log";
    case OpKind::Sqrt: return "Sqrt";
    case OpKind::Sum: return "Sum";
    case OpKind::Mean: return "Mean";
    case OpKind::SwapAxes: return "SwapAxes";
    case OpKind::Dropout: return "Dropout";
  }
  return "?";
}

// ---------------------------------------------------------------- registry
// FUSION_ALLOW_SCALAR_BINARY (fusion/src/Fusion/common/Checks.hpp:48-66): the traced
// Multiply/Divide/Pow/Maximum accept a scalar operand or equal element counts only.
static void allow_scalar_binary(const RawTensor &a, const RawTensor &b, const char *where) {
  const long long s1 = (long long)a.size(), s2 = (long long)b.size();
  const bool sc1 = a.ndims() == 0 || s1 == 1, sc2 = b.ndims() == 0 || s2 == 1;
  if (!(sc1 || sc2 || s1 == s2)) {
    std::ostringstream os;
    os << "FUSION_ALLOW_SCALAR_BINARY failed @ " << where
       << ": Elementwise op requires scalars or equal element counts; got size(" << s1
       << ") vs size(" << s2 << ")";
    throw std::runtime_error(os.str());
  }
}

// Forward/backward formulas of fusion/src/Fusion/autodiff/registry/** restated.
std::vector<RawTensor> op_forward(OpKind k, OpContext &ctx, const std::vector<RawTensor> &in,
                                  const OpParam &p) {
  const RawTensor &x = in.at(0);
  switch (k) {
    case OpKind::Add: return {x + in.at(1)};
    case OpKind::Subtract: return {x - in.at(1)};
    case OpKind::Multiply:
      allow_scalar_binary(x, in.at(1), "Multiply");
      ctx.saved["x"] = x;
      ctx.saved["y"] = in.at(1);
      return {x * in.at(1)};
    case OpKind::Divide:
      ctx.saved["x"] = x;
      ctx.saved["y"] = in.at(1);
      allow_scalar_binary(x, in.at(1), "Divide");
      return {x / in.at(1)};
    case OpKind::Pow:
      allow_scalar_binary(x, in.at(1), "Pow");
      ctx.saved["x"] = x;
      ctx.saved["y"] = in.at(1);
      return {x.pow(in.at(1))};
    case OpKind::Maximum: {
      allow_scalar_binary(x, in.at(1), "Maximum");
      RawTensor out = x.maximum(in.at(1));
      ctx.saved["y"] = in.at(1);
      // x's gradient mask (x > y) equals (max(x, y) > y) for every pair of values (x > y:
      // the max is x; otherwise it is y, and y > y is false, NaN included), so when the
      // engine marked the node (y needs no gradient and x is the engine's own value) the
      // backward reads the output, which later ops keep anyway, instead of x: a ReLU
      // after a GEMM then does not keep (and store) the product for its backward
      if (ctx.ints.count("mask_from_out")) ctx.saved["out"] = out;
      else ctx.saved["x"] = x;
      return {out};
    }
    case OpKind::GreaterThan:
    case OpKind::GreaterThanEqual: {
      const RawTensor &y = in.at(1);
      ctx.saved["x"] = x;
      ctx.saved["y"] = y;
      FB_CHECK(x.size() == y.size(), k == OpKind::GreaterThan
                                          ? "GreaterThan: input size mismatch"
                                          : "GreaterThanEqual: input size mismatch");
      return {k == OpKind::GreaterThan ? x > y : x >= y};
    }
    case OpKind::MatMul: {
      const RawTensor &y = in.at(1);
      ctx.saved["x"] = x;
      ctx.saved["y"] = y;
      FB_CHECK(x.rank() >= 2 && y.rank() >= 2, "MatMul: rank must be >= 2");
      FB_CHECK(x.shape().back() == y.shape()[y.rank() - 2], "MatMul: inner dims mismatch");
      return {x.matmul(y)};
    }
    case OpKind::Exp: ctx.saved["x"] = x; return {x.exp()};
    case OpKind::Log: ctx.saved["x"] = x; return {x.log()};
    case OpKind::Sqrt: ctx.saved["x"] = x; return {x.sqrt()};
    case OpKind::Sum:
      ctx.saved["x"] = x;
      return {x.sum(p.axis, p.keepdim)};
    case OpKind::Mean: {
      // registry/Reduction/Mean.hpp:26-28 computes the mean and returns its input
      ctx.saved["x"] = x;
      RawTensor unused = x.mean(p.axis, p.keepdim);
      (void)unused;
      return {x};
    }
    case OpKind::Dropout:
      ctx.param = p;
      return {math::dropout(x, p.rate, p.keep, p.rng_seed, p.rng_offset)};
    case OpKind::SwapAxes:
      FB_CHECK(p.axis1 != p.axis2, "SwapAxes: axes must be different");
      ctx.ints["axis1"] = p.axis1;
      ctx.ints["axis2"] = p.axis2;
      return {x.swapaxes(p.axis1, p.axis2)};
  }
  throw std::runtime_error("unknown op");
}

std::vector<RawTensor> op_backward(OpKind k, OpContext &ctx, const RawTensor &g0,
                                   const std::vector<bool> &need) {
  FB_CHECK(!g0.empty() || g0.is_initialised(), std::string(op_name(k)) + "::backward: upstream grad is empty");
  auto want = [&](size_t j) { return j < need.size() ? (bool)need[j] : true; };
  switch (k) {
    case OpKind::Add: return {g0, g0};  // Add.hpp:41-45: both alias g0
    case OpKind::Subtract:
      return {g0, want(1) ? zeros_like(g0) - g0 : RawTensor()};
    case OpKind::Multiply: {
      const RawTensor &x = ctx.load("x"), &y = ctx.load("y");
      return {want(0) ? g0 * y : RawTensor(), want(1) ? g0 * x : RawTensor()};
    }
    case OpKind::Divide: {
      const RawTensor &x = ctx.load("x"), &y = ctx.load("y");
      return {want(0) ? g0 / y : RawTensor(),
              want(1) ? ((zeros_like(g0) - g0) * x) / (y * y) : RawTensor()};
    }
    case OpKind::Pow: {
      const RawTensor &x = ctx.load("x"), &y = ctx.load("y");
      return {want(0) ? (y * x.pow(y - 1.0f)) * g0 : RawTensor(),
              want(1) ? (x.pow(y) * x.log()) * g0 : RawTensor()};
    }
    case OpKind::Maximum: {
      const RawTensor &y = ctx.load("y");
      if (ctx.saved.count("out")) {
        FB_CHECK(!want(1), "Maximum::backward: the second operand's gradient needs the first operand");
        return {want(0) ? g0 * (ctx.load("out") >= y) : RawTensor(), RawTensor()};
      }
      const RawTensor &x = ctx.load("x");
      return {want(0) ? g0 * (x >= y) : RawTensor(), want(1) ? g0 * (y > x) : RawTensor()};
    }
    case OpKind::GreaterThan:
    case OpKind::GreaterThanEqual: {
      const RawTensor &x = ctx.load("x"), &y = ctx.load("y");
      return {zeros_like(x), zeros_like(y)};
    }
    case OpKind::MatMul: {
      // MatMul.hpp:55-58: gx = g0 @ swapaxes(y), gy = swapaxes(x) @ g0; the
      // transposes are folded into the GEMM's operand modes (same values).
      const RawTensor &x = ctx.load("x"), &y = ctx.load("y");
      return {want(0) ? math::matmul(g0, y, false, true) : RawTensor(),
              want(1) ? math::matmul(x, g0, true, false) : RawTensor()};
    }
    case OpKind::Exp: return {g0 * ctx.load("x").exp()};
    case OpKind::Log: return {g0 / ctx.load("x")};
    case OpKind::Sqrt: return {g0 / (ctx.load("x").sqrt() * 2.0f)};
    case OpKind::Sum: {
      const RawTensor &x = ctx.load("x");
      return {g0.flat_size() == 1 ? ones_like(x) * g0 : g0};
    }
    case OpKind::Mean: {
      const RawTensor &x = ctx.load("x");
      RawTensor gx = g0.flat_size() == 1 ? ones_like(x) * g0 : g0;
      return {gx * static_cast<float>(1.0 / static_cast<double>(x.size()))};
    }
    case OpKind::SwapAxes:
      return {g0.swapaxes(ctx.ints.at("axis1"), ctx.ints.at("axis2"))};
    case OpKind::Dropout: {
      // the composition's backward, Divide (g0 / keep) then Multiply (* mask), gives
      // (g0 / keep) * m, which equals (g0 * m) / keep for m in {0, 1} bit for bit
      // (signed zeros and NaNs included): the same kernel redraws the same mask
      const OpParam &q = ctx.param;
      return {math::dropout(g0, q.rate, q.keep, q.rng_seed, q.rng_offset)};
    }
  }
  throw std::runtime_error("unknown op");
}

// ---------------------------------------------------------------- engine
ValueID Engine::new_input_value() {
  ValueID v = value_counter_++;
  if ((int64_t)produced_by_.size() <= v) produced_by_.resize(v + 1, -1);
  produced_by_[v] = -1;
  return v;
}

ValueID Engine::new_intermediate_value() {
  ValueID v = value_counter_++;
  if ((int64_t)produced_by_.size() <= v) produced_by_.resize(v + 1, -1);
  if ((int64_t)consumed_by_.size() <= v) consumed_by_.resize(v + 1);
  return v;
}

ValueID Engine::track_input(const RawTensor &raw, bool requires_grad) {
  ValueID v = new_input_value();
  if ((int64_t)val_.size() <= v) val_.resize(v + 1);
  val_[v] = raw;
  if (produced_by_[v] == -1 && requires_grad) requires_grad_set_.insert(v);
  return v;
}

bool Engine::has_value(ValueID v) const {
  if (v < 0 || v >= (int64_t)val_.size()) return false;
  if (v >= (int64_t)produced_by_.size()) return false;
  return val_[v].is_initialised();
}

// Engine::materialise deep-copies the value (Engine.hpp:128-134); here the copy
// is a second Storage over the same immutable Expr, so in-place writes through
// either side stay private to it.
RawTensor Engine::materialise(ValueID v) const {
  const RawTensor &src = val_.at(v);
  return RawTensor(src.expr(), src.dtype(), src.device());
}

ValueID Engine::apply(OpKind k, const std::vector<RawTensor> &ins,
                      const std::vector<ValueID> &vids, const OpParam &p) {
  NodeID nid = (NodeID)nodes_.size();
  nodes_.push_back(TapeNode{k, {}, {}, {}});
  for (size_t i = 0; i < ins.size(); ++i) {
    ValueID v = vids[i];
    nodes_[nid].inputs.push_back(v);
    if ((int64_t)consumed_by_.size() <= v) consumed_by_.resize(v + 1);
    consumed_by_[v].push_back(nid);
  }
  // Maximum whose second operand needs no gradient (neither produced by a node nor a
  // leaf that requires grad; the same test the backward applies) and whose first
  // operand is a value the engine produced (no caller holds it to write in place):
  // its backward may take the mask from the output (see op_forward)
  if (k == OpKind::Maximum && vids.size() == 2) {
    const ValueID vx = vids[0], vy = vids[1];
    const bool y_needs = produced_by_[vy] != -1 || requires_grad_set_.count(vy);
    if (!y_needs && produced_by_[vx] != -1) nodes_[nid].ctx.ints["mask_from_out"] = 1;
  }
  std::vector<RawTensor> out;
  {
    NoGradGuard ng;
    out = op_forward(k, nodes_[nid].ctx, ins, p);
  }
  FB_CHECK(!out.empty(), "Engine::apply: forward produced empty outputs");
  for (size_t i = 0; i < out.size(); ++i) {
    ValueID v = new_intermediate_value();
    produced_by_[v] = nid;
    nodes_[nid].outputs.push_back(v);
    if ((int64_t)val_.size() <= v) val_.resize(v + 1);
    val_[v] = out[i];
  }
  return nodes_[nid].outputs[0];
}

// Kahn's algorithm over every node, in-degree = inputs produced by a node
// (autodiff/Sort.hpp:21-74).
std::vector<NodeID> Engine::topo_order() const {
  const size_t n = nodes_.size();
  std::vector<size_t> indeg(n, 0);
  for (size_t i = 0; i < n; ++i)
    for (ValueID v : nodes_[i].inputs)
      if (produced_by_[v] != -1) ++indeg[i];
  std::queue<NodeID> q;
  for (size_t i = 0; i < n; ++i)
    if (indeg[i] == 0) q.push((NodeID)i);
  std::vector<NodeID> order;
  order.reserve(n);
  while (!q.empty()) {
    NodeID id = q.front();
    q.pop();
    order.push_back(id);
    for (ValueID o : nodes_[id].outputs)
      if (o < (int64_t)consumed_by_.size())
        for (NodeID c : consumed_by_[o])
          if (--indeg[c] == 0) q.push(c);
  }
  if (order.size() != n)
    throw std::runtime_error("Number of nodes greater than indegree vec - graph contains cycles!");
  return order;
}

static thread_local GradReadyHook t_grad_ready_hook;
void set_grad_ready_hook(GradReadyHook hook) { t_grad_ready_hook = std::move(hook); }

BackwardResult Engine::backward(ValueID seed) {
  grad_.resize(val_.size());
  for (auto &g : grad_)
    if (g.is_initialised()) g.clear();
  std::vector<NodeID> order = topo_order();
  grad_[seed] = ones_like(val_[seed]);
  // readers left per value, to tell the hook when a leaf's gradient is complete
  const GradReadyHook hook = t_grad_ready_hook;
  std::vector<int> readers_left;
  if (hook) {
    readers_left.assign(val_.size(), 0);
    for (const TapeNode &nd : nodes_)
      for (ValueID v : nd.inputs) ++readers_left[v];
  }
  for (auto it = order.rbegin(); it != order.rend(); ++it) {
    TapeNode &n = nodes_[*it];
    FB_CHECK(!n.outputs.empty(), "node has no outputs in backward()");
    ValueID out = n.outputs[0];
    FB_CHECK((size_t)out < val_.size(), std::string("val index OOB in backward: ") + op_name(n.kind));
    FB_CHECK(val_[out].is_initialised(), std::string("val missing for node output: ") + op_name(n.kind));
    if (!grad_[out].is_initialised()) grad_[out] = zeros_like(val_[out]);
    std::vector<bool> need(n.inputs.size());
    for (size_t j = 0; j < n.inputs.size(); ++j) {
      ValueID v = n.inputs[j];
      need[j] = produced_by_[v] != -1 || requires_grad_set_.count(v);
    }
    std::vector<RawTensor> gin;
    try {
      gin = op_backward(n.kind, n.ctx, grad_[out], need);
    } catch (const std::exception &e) {
      throw std::runtime_error(std::string("apply_backward threw in op ") + op_name(n.kind) +
                               ": " + e.what());
    }
    FB_CHECK(gin.size() == n.inputs.size(), "backward arity mismatch");
    // An intermediate value's gradient is read by this node alone (its producer) and
    // never returned: drop it, so a pending product inside it is not kept alive (and
    // stored) only for this table.
    if (out != seed && produced_by_[out] != -1 && !requires_grad_set_.count(out)) grad_[out] = RawTensor();
    // Both operands are leaves that require grad (their gradients are final values):
    // lower the two pending gradients together, one pass over the shared upstream
    // gradient and operands (e.g. Multiply: g0*y and g0*x read g0, x, y once).
    if (gin.size() == 2 && n.inputs[0] != n.inputs[1] && gin[0].is_initialised() &&
        gin[1].is_initialised() && gin[0].pending() && gin[1].pending() &&
        gin[0].shape() == gin[1].shape()) {
      bool leaves = true;
      for (ValueID v : n.inputs)
        leaves = leaves && produced_by_[v] == -1 && requires_grad_set_.count(v) &&
                 !grad_[v].is_initialised();
      if (leaves) materialize_group({gin[0].expr(), gin[1].expr()});
    }
    for (size_t j = 0; j < n.inputs.size(); ++j) {
      if (!gin[j].is_initialised()) continue;  // unobservable gradient, not computed
      RawTensor &dst = grad_[n.inputs[j]];
      if (!dst.is_initialised()) dst = gin[j];
      else dst = dst + gin[j];
    }
    if (hook)
      for (ValueID v : n.inputs)
        if (--readers_left[v] == 0 && produced_by_[v] == -1 && requires_grad_set_.count(v) &&
            grad_[v].is_initialised())
          hook(v, grad_[v]);
  }
  BackwardResult r;
  for (int64_t v : requires_grad_set_) r.grads.try_emplace(v, grad_[v]);
  FB_CHECK(!r.grads.empty(), "backward result is empty - no gradients to attatch");
  return r;
}

// ---------------------------------------------------------------- ADTensor
ADTensor::ADTensor(const ADTensor &o) = default;
ADTensor &ADTensor::operator=(const ADTensor &o) = default;

ADTensor::~ADTensor() {
  auto &v = t_leaf_tensors;
  v.erase(std::remove(v.begin(), v.end(), this), v.end());
}

void ADTensor::set_leaf() {
  if (requires_grad_) t_leaf_tensors.push_back(this);
}

ValueID ADTensor::ensure_vid() {
  Engine &eng = current_engine();
  if (vid_ >= 0 && eng.has_value(vid_)) {
    set_leaf();
    return vid_;
  }
  vid_ = eng.track_input(raw_, requires_grad_);
  set_leaf();
  return vid_;
}

void ADTensor::attach_grads(BackwardResult &res) const {
  for (ADTensor *leaf : t_leaf_tensors) {
    if (!leaf->has_vid()) continue;
    auto it = res.grads.find(leaf->vid());
    if (it != res.grads.end()) leaf->grad_ = std::make_shared<RawTensor>(it->second);
  }
  t_leaf_tensors.clear();
}

void ADTensor::backward() {
  Engine &eng = current_engine();
  ValueID v = ensure_vid();
  BackwardResult r = eng.backward(v);
  attach_grads(r);
}

std::optional<ADTensor> ADTensor::grad() const {
  if (!grad_ || !grad_->is_initialised()) return std::nullopt;
  return ADTensor(*grad_, false);
}

static RawTensor eager_binary(OpKind k, const RawTensor &x, const RawTensor &y) {
  switch (k) {
    case OpKind::Add: return x + y;
    case OpKind::Subtract: return x - y;
    case OpKind::Multiply: return x * y;
    case OpKind::Divide: return x / y;
    case OpKind::Pow: return x.pow(y);
    case OpKind::Maximum: return x.maximum(y);
    case OpKind::GreaterThan: return x > y;
    case OpKind::GreaterThanEqual: return x >= y;
    case OpKind::MatMul: return x.matmul(y);
    default: break;
  }
  throw std::runtime_error("not a binary op");
}

// autodiff::binary (autodiff/Dispatch.hpp:82-101)
ADTensor ADTensor::binary_op(OpKind k, const ADTensor &other) const {
  const bool needs_grad = grad_enabled() && (requires_grad_ || other.requires_grad_);
  if (!needs_grad || !engine_instance()) {
    return ADTensor(eager_binary(k, raw_, other.raw_), requires_grad_ || other.requires_grad_);
  }
  Engine &eng = current_engine();
  ValueID vx = const_cast<ADTensor *>(this)->ensure_vid();
  ValueID vy = const_cast<ADTensor &>(other).ensure_vid();
  ValueID out = eng.apply(k, {raw_, other.raw_}, {vx, vy}, OpParam{});
  ADTensor r(eng.materialise(out), needs_grad);
  r.set_vid(out);
  return r;
}

// ADTensor scalar overloads wrap the scalar as a [1] tensor without grad
// (autodiff/ADTensor.hpp:54-58, 173-213).
ADTensor ADTensor::binary_scalar(OpKind k, float s) const {
  ADTensor other(RawTensor::scalar(s, raw_.dtype(), raw_.device()), false);
  return binary_op(k, other);
}

// autodiff::unary (autodiff/Dispatch.hpp:43-80)
ADTensor ADTensor::unary_op(OpKind k, const OpParam &p) const {
  const bool needs_grad = grad_enabled() && requires_grad_;
  if (!needs_grad || !engine_instance()) {
    RawTensor out;
    switch (k) {
      case OpKind::Exp: out = raw_.exp(); break;
      case OpKind::Log: out = raw_.log(); break;
      case OpKind::Sqrt: out = raw_.sqrt(); break;
      case OpKind::Sum: out = raw_.sum(p.axis, p.keepdim); break;
      case OpKind::Mean: out = raw_.mean(p.axis, p.keepdim); break;
      case OpKind::SwapAxes: out = raw_.swapaxes(p.axis1, p.axis2); break;
      case OpKind::Dropout: out = math::dropout(raw_, p.rate, p.keep, p.rng_seed, p.rng_offset); break;
      default: throw std::runtime_error("not a unary op");
    }
    return ADTensor(out, requires_grad_);
  }
  Engine &eng = current_engine();
  ValueID vx = const_cast<ADTensor *>(this)->ensure_vid();
  ValueID out = eng.apply(k, {raw_}, {vx}, p);
  ADTensor r(eng.materialise(out), requires_grad_);
  r.set_vid(out);
  return r;
}

}  // namespace fusion_b200
