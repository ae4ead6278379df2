// C-ABI harness over the reference Fusion CPU path (oracle infrastructure only).
//
// This file is compiled together with the reference's own headers and sources
// (fusion/src/Fusion/**, TensorPlan.cpp, BFCPoolAllocator.cpp, CPUSubAllocator.cpp)
// by oracle/Makefile into oracle/_ref/libfusion_ref.so. It is the checker and the
// timed CPU baseline; nothing in the nova_b200 package links or loads it.
//
// Every entry point drives the reference's public C++ API exactly as its callers do:
//   * RawTensor operators -> fusion::math::* (fusion/src/Fusion/core/RawTensor.hpp:159-241)
//   * registry forward/backward formulas (fusion/src/Fusion/autodiff/registry/**)
//   * ADTensor + EngineScope for the traced MLP step (autodiff/ADTensor.hpp,
//     autodiff/EngineContext.hpp:43-74), mirroring nova/src/blocks/core/linear.py:42-48,
//     nova/src/blocks/activations/activations.py:9-10, nova/src/losses/loss.py:34-37 and
//     nova/src/optim/sgd.py:29-44.
#include "Fusion/autodiff/AutodiffBridge.hpp"
#include "Fusion/autodiff/AutodiffMode.hpp"
#include "Fusion/autodiff/EngineContext.hpp"
#include "Fusion/TensorFactory.hpp"
#include "Fusion/Random.hpp"
#include "Fusion/Tensor.h"
#include "Fusion/autodiff/ADTensor.hpp"

#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

using RT = RawTensor<float>;
using AT = ADTensor<float>;

namespace {
thread_local std::string g_err;

struct Handle {
   RT t;
};

Handle *wrap(RT &&t) { return new Handle{std::move(t)}; }

template <class F> auto guard(F &&f) -> decltype(f()) {
   try {
      return f();
   } catch (const std::exception &e) {
      g_err = e.what();
   } catch (...) {
      g_err = "unknown exception";
   }
   return decltype(f()){};
}

const Device kCpu{DeviceType::CPU, 0};

enum BinOp { kAdd = 0, kSub, kMul, kDiv, kPow, kMax, kGt, kGe };
enum UnOp { kExp = 0, kLog, kSqrt };
enum RedOp { kSum = 0, kMean };

RT binary(int op, const RT &a, const RT &b) {
   switch (op) {
   case kAdd: return a + b;
   case kSub: return a - b;
   case kMul: return a * b;
   case kDiv: return a / b;
   case kPow: return a.pow(b);
   case kMax: return a.maximum(b);
   case kGt: return a > b;
   case kGe: return a >= b;
   }
   throw std::runtime_error("ref_binary: bad op");
}

RT unary(int op, const RT &a) {
   switch (op) {
   case kExp: return a.exp();
   case kLog: return a.log();
   case kSqrt: return a.sqrt();
   }
   throw std::runtime_error("ref_unary: bad op");
}

// Runs one registry op's forward then backward on upstream grad g0, the way
// Engine::backward drives it (autodiff/Engine.hpp:74-89).
template <class Op>
std::vector<RT> run_backward(const std::vector<const RT *> &ins, const RT &g0,
                             std::any param = {}) {
   Op op;
   Context<float> ctx;
   AutodiffMeta<float> in;
   for (const RT *t : ins) in.push_back(*t);
   in.op_param = std::move(param);
   AutodiffMeta<float> out = op.forward(ctx, in);
   AutodiffMeta<float> gout;
   gout.push_back(g0);
   AutodiffMeta<float> gin = op.backward(ctx, gout);
   std::vector<RT> res;
   for (auto &g : gin) res.push_back(g);
   return res;
}
} // namespace

extern "C" {

const char *ref_last_error() { return g_err.c_str(); }

void *ref_tensor_new(const uint64_t *shape, int ndim, const float *data) {
   return guard([&]() -> void * {
      std::vector<size_t> s(shape, shape + ndim);
      size_t n = 1;
      for (auto d : s) n *= d;
      std::vector<float> v(data, data + n);
      return wrap(RT(s, std::move(v), DType::FLOAT32, kCpu));
   });
}

void ref_tensor_free(void *h) { delete static_cast<Handle *>(h); }

int ref_tensor_ndim(void *h) { return (int)static_cast<Handle *>(h)->t.rank(); }

void ref_tensor_shape(void *h, uint64_t *out) {
   auto s = static_cast<Handle *>(h)->t.shape();
   for (size_t i = 0; i < s.size(); ++i) out[i] = s[i];
}

uint64_t ref_tensor_numel(void *h) { return static_cast<Handle *>(h)->t.flat_size(); }

void ref_tensor_read(void *h, float *out) {
   const RT &t = static_cast<Handle *>(h)->t;
   std::memcpy(out, t.get_ptr(), t.flat_size() * sizeof(float));
}

void *ref_binary(int op, void *a, void *b) {
   return guard([&]() -> void * {
      return wrap(binary(op, static_cast<Handle *>(a)->t, static_cast<Handle *>(b)->t));
   });
}

// RawTensor scalar overloads build a [1] tensor (core/RawTensor.hpp:30-34,159-185).
void *ref_binary_scalar(int op, void *a, float s) {
   return guard([&]() -> void * {
      const RT &x = static_cast<Handle *>(a)->t;
      switch (op) {
      case kAdd: return wrap(x + s);
      case kSub: return wrap(x - s);
      case kMul: return wrap(x * s);
      case kDiv: return wrap(x / s);
      case kPow: return wrap(x.pow(s));
      case kMax: return wrap(x.maximum(s));
      case kGe: return wrap(x >= s);
      }
      throw std::runtime_error("ref_binary_scalar: bad op");
   });
}

void *ref_unary(int op, void *a) {
   return guard([&]() -> void * { return wrap(unary(op, static_cast<Handle *>(a)->t)); });
}

// axis < 0 with keepdim == 0 selects the global reduction (ops/Reduce.hpp, PlanMeta.hpp:152).
void *ref_reduce(int op, void *a, int64_t axis, int keepdim) {
   return guard([&]() -> void * {
      const RT &x = static_cast<Handle *>(a)->t;
      size_t ax = axis < 0 ? (size_t)-1 : (size_t)axis;
      if (op == kSum) return wrap(x.sum(ax, keepdim != 0));
      if (op == kMean) return wrap(x.mean(ax, keepdim != 0));
      throw std::runtime_error("ref_reduce: bad op");
   });
}

void *ref_matmul(void *a, void *b) {
   return guard([&]() -> void * {
      return wrap(static_cast<Handle *>(a)->t.matmul(static_cast<Handle *>(b)->t));
   });
}

void *ref_swapaxes(void *a, int a1, int a2) {
   return guard([&]() -> void * { return wrap(static_cast<Handle *>(a)->t.swapaxes(a1, a2)); });
}

int ref_sub_inplace(void *a, void *b) {
   return guard([&]() -> int {
      static_cast<Handle *>(a)->t -= static_cast<Handle *>(b)->t;
      return 1;
   }) ? 0 : -1;
}

// Backward formulas of the registry ops. Writes up to two grads into out[0..1]
// and returns how many were produced (0 on error).
int ref_backward(const char *name, void *x, void *y, void *g0, void **out) {
   return guard([&]() -> int {
      std::string n(name);
      const RT &g = static_cast<Handle *>(g0)->t;
      const RT *X = &static_cast<Handle *>(x)->t;
      const RT *Y = y ? &static_cast<Handle *>(y)->t : nullptr;
      std::vector<RT> r;
      if (n == "Add") r = run_backward<Add<float>>({X, Y}, g);
      else if (n == "Subtract") r = run_backward<Subtract<float>>({X, Y}, g);
      else if (n == "Multiply") r = run_backward<Multiply<float>>({X, Y}, g);
      else if (n == "Divide") r = run_backward<Divide<float>>({X, Y}, g);
      else if (n == "Pow") r = run_backward<Pow<float>>({X, Y}, g);
      else if (n == "Maximum") r = run_backward<Maximum<float>>({X, Y}, g);
      else if (n == "MatMul") r = run_backward<MatMul<float>>({X, Y}, g);
      else if (n == "Exp") r = run_backward<Exp<float>>({X}, g);
      else if (n == "Log") r = run_backward<Log<float>>({X}, g);
      else if (n == "Sqrt") r = run_backward<Sqrt<float>>({X}, g);
      else throw std::runtime_error("ref_backward: unknown op " + n);
      for (size_t i = 0; i < r.size(); ++i) out[i] = wrap(std::move(r[i]));
      return (int)r.size();
   });
}

// One MLP training step through the reference autodiff engine, as Nova's Python
// layer issues it: under a fresh grad_tape, for each Linear layer
// `out = x @ W.T` then `out = out + b`, ReLU via maximum(0) on all but the last
// layer; loss = ((pred - y) ** 2) / loss.size; loss.backward(); then SGD
// `p -= grad * lr` for every W and b. The input batch tensor is created with
// requires_grad=True, the default of nova's Tensor constructor
// (nova/src/backend/core/_tensor.py:32-48).
//
// W[i] / b[i] are handles updated in place. loss_out receives the loss tensor
// ([B, out_dim]) when non-null.
// One step as ref_mlp_step; grads_out (2 * nlayers handles, nullable) receives each
// kernel's and bias's gradient as the engine left it (gW_i at 2i, gb_i at 2i + 1).
int ref_mlp_step_grads(void *X, void *Y, void **W, void **b, int nlayers, float lr,
                       float *loss_out, void **grads_out) {
   return guard([&]() -> int {
      std::vector<AT> Ws, bs;
      Ws.reserve(nlayers);
      bs.reserve(nlayers);
      for (int i = 0; i < nlayers; ++i) {
         Ws.emplace_back(static_cast<Handle *>(W[i])->t, true);
         bs.emplace_back(static_cast<Handle *>(b[i])->t, true);
      }
      AT x(static_cast<Handle *>(X)->t, true);
      AT y(static_cast<Handle *>(Y)->t, true);
      {
         EngineScope<float> scope;
         scope.enter();
         AT out = x;
         for (int i = 0; i < nlayers; ++i) {
            AT kT = Ws[i].swapaxes((int)Ws[i].rank() - 1, (int)Ws[i].rank() - 2);
            out = out.matmul(kT);
            out = out + bs[i];
            if (i + 1 < nlayers) out = out.maximum(0.0f);
         }
         AT diff = out - y;
         AT sq = diff.pow(2.0f);
         AT loss = sq / (float)sq.flat_size();
         loss.backward();
         if (loss_out)
            std::memcpy(loss_out, loss.raw().get_ptr(), loss.flat_size() * sizeof(float));
         scope.exit();
      }
      for (int i = 0; i < nlayers; ++i) {
         int slot = 0;
         for (AT *p : {&Ws[i], &bs[i]}) {
            auto g = p->grad();
            if (grads_out) grads_out[2 * i + slot] = g ? wrap(RT(g->raw())) : nullptr;
            ++slot;
            if (!g) continue;
            AT step = *g * lr;
            p->raw() -= step.raw();
         }
      }
      return 1;
   }) ? 0 : -1;
}

int ref_mlp_step(void *X, void *Y, void **W, void **b, int nlayers, float lr,
                 float *loss_out) {
   return ref_mlp_step_grads(X, Y, W, b, nlayers, lr, loss_out, nullptr);
}

} // extern "C"
