// pybind11 module `fusion`: the Python API that Nova imports
// (nova/src/backend/core/clib/__init__.py:1-3), with the names, argument meaning
// and error behaviour of the reference module (fusion/src/Fusion/python/Bindings.cpp,
// tensor/BindTensor.hpp, factory/BindFactory.hpp, random/BindRandom.hpp), backed by
// the B200 tensor of this project.
#include <pybind11/numpy.h>
#include <pybind11/operators.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <numeric>
#include <optional>
#include <random>
#include <sstream>

#include "autodiff.hpp"

namespace py = pybind11;
using namespace fusion_b200;

namespace {

size_t prod(const std::vector<size_t> &s) {
  return std::accumulate(s.begin(), s.end(), (size_t)1, std::multiplies<size_t>());
}

// Random<T>::uniform_base (fusion/src/Fusion/Random.hpp:20-36): mt19937 with
// uniform_real_distribution<float>, generated on the host, then uploaded.
// The same seed also keys a device-side Philox-4x32-10 stream (fz_philox_*), for draws
// made on the GPU: uniform_device and dropout. Its position advances by each draw's
// size (rounded up to 4), so consecutive draws differ and a replayed sequence of draws
// repeats. It does not reproduce the mt19937 stream of uniform_cpp.
struct Random {
  std::mt19937 engine;
  uint64_t seed = 0, offset = 0;
  explicit Random(uint32_t s) : engine(s), seed(s) {}
  ADTensor uniform(const std::vector<size_t> &shape, float lo, float hi, Device dev) {
    std::vector<float> data;
    size_t n = prod(shape);
    data.reserve(n);
    std::uniform_real_distribution<float> dist(lo, hi);
    for (size_t i = 0; i < n; ++i) data.push_back(dist(engine));
    return ADTensor(RawTensor(shape, data, DType::FLOAT32, dev), false);
  }
  uint64_t advance(size_t n) {
    const uint64_t at = offset;
    offset += (n + 3) / 4 * 4;
    return at;
  }
  ADTensor uniform_device(const std::vector<size_t> &shape, float lo, float hi, Device dev) {
    const uint64_t at = advance(prod(shape));
    return ADTensor(math::philox_uniform(shape, lo, hi, seed, at, DType::FLOAT32, dev), false);
  }
  // Nova's Dropout (nova/src/blocks/regularisation/dropout.py:17-23):
  // inputs * (uniform >= rate) / (1 - rate), with `>=` computing `>` as Fusion's does,
  // in one kernel and traced as one op whose backward redraws the mask.
  ADTensor dropout(const ADTensor &x, double rate) {
    if (!(rate >= 0.0 && rate < 1.0)) throw std::invalid_argument("dropout: rate must be in [0, 1)");
    OpParam p;
    p.rng_seed = seed;
    p.rng_offset = advance(x.raw().size());
    p.rate = (float)rate;
    p.keep = (float)(1.0 - rate);
    return x.unary_op(OpKind::Dropout, p);
  }
};

py::array_t<float> to_numpy(const ADTensor &t) {
  const auto &shape = t.shape();
  std::vector<ssize_t> sh(shape.begin(), shape.end());
  py::array_t<float> arr(sh);
  t.raw().to_host(static_cast<float *>(arr.request().ptr));
  return arr;
}

RawTensor raw_from_array(const std::vector<size_t> &shape, py::array_t<float, py::array::c_style | py::array::forcecast> a,
                         DType dt, Device dev) {
  size_t total = prod(shape);
  if ((size_t)a.size() != total) throw std::invalid_argument("shape* must equal data.size()");
  return RawTensor(shape, a.data(), dt, dev);
}

struct GradTape {
  EngineScope scope;
};

// NCCL communicator over the GPUs of one data-parallel job (one process per GPU).
struct Comm {
  void *c = nullptr;
  int world = 1, rank = 0;
  void *side = nullptr;  // stream for all-reduces that overlap the backward
  struct Watched {
    ADTensor *param;
    ValueID vid;
    std::optional<RawTensor> avg;  // averaged gradient (what the update reads)
    std::optional<RawTensor> sent;  // the reduced values, kept alive until collect()
  };
  std::vector<Watched> watched;
  // Gradients announced while still pending, reduced at the next announcement (or in
  // collect()): by then the backward has usually lowered them as part of a larger
  // program (a bias gradient is the operand of the next GEMMs), where reducing at once
  // would force its pending product to be computed on its own first.
  std::vector<std::pair<Watched *, RawTensor>> deferred;
  int overlapped = 0;  // gradients the last backward handed over while it ran
  Comm(int w, int r, py::bytes uid) : world(w), rank(r) {
    std::string id = uid;
    if (id.size() != FZ_UNIQUE_ID_BYTES) throw std::invalid_argument("Comm: unique id must be 128 bytes");
    fz_check(fz_comm_init(&c, w, r, reinterpret_cast<const unsigned char *>(id.data())), "fz_comm_init");
  }
  ~Comm() { destroy(); }
  void destroy() {
    if (!watched.empty()) set_grad_ready_hook({});
    deferred.clear();
    watched.clear();
    if (c) fz_comm_destroy(c);
    c = nullptr;
    if (side) fz_stream_destroy(side);
    side = nullptr;
  }
  // All-reduce (average) what `param -= grad * lr` reads from grad: all of it, or its
  // first param.size values when the gradient is larger (a bias gradient that keeps the
  // batch dimension), on the side stream after the work that produced it.
  void reduce_into(Watched &w, const RawTensor &g) {
    const size_t n = w.param->raw().size();
    RawTensor src = g.size() > n ? math::flat_prefix(g, n, w.param->raw().shape()) : g;
    const float *in = src.data();
    auto out = std::make_shared<DeviceBuffer>(src.size());
    fz_check(fz_stream_wait(side, nullptr), "fz_stream_wait");
    fz_check(fz_comm_allreduce(c, in, out->ptr, (int64_t)src.size(), 1.0f / (float)world, side),
             "fz_comm_allreduce");
    w.avg = RawTensor::from_buffer(out, src.shape(), src.dtype(), src.device());
    w.sent = std::move(src);
  }
  // Average the gradients of `params` over ranks while the backward runs: each one is
  // all-reduced on a second stream as soon as the engine has completed it, so the
  // transfers overlap the backward of the earlier layers. Call after the forward and
  // before backward(); collect() returns the averaged gradients. Every rank issues the
  // all-reduces in the engine's (deterministic) completion order.
  void watch(const std::vector<ADTensor *> &params) {
    if (!c) throw std::runtime_error("Comm: destroyed");
    if (!side) fz_check(fz_stream_create(&side), "fz_stream_create");
    watched.clear();
    for (ADTensor *p : params) watched.push_back(Watched{p, p->has_vid() ? p->vid() : -1, {}, {}});
    deferred.clear();
    set_grad_ready_hook([this](ValueID v, const RawTensor &g) {
      flush_deferred();
      for (Watched &w : watched)
        if (w.vid == v && w.vid >= 0 && !w.avg) {
          if (g.pending()) deferred.emplace_back(&w, g);
          else reduce_into(w, g);
        }
    });
  }
  void flush_deferred() {
    for (auto &d : deferred)
      if (!d.first->avg) reduce_into(*d.first, d.second);
    deferred.clear();
  }
  // The averaged gradients of the watched parameters (None where a parameter got no
  // gradient). Gradients the backward did not announce are reduced here, in parameter
  // order. The thread's stream then waits for the side stream.
  std::vector<py::object> collect() {
    set_grad_ready_hook({});
    flush_deferred();
    overlapped = 0;
    for (Watched &w : watched) overlapped += w.avg ? 1 : 0;
    for (Watched &w : watched)
      if (!w.avg) {
        std::optional<ADTensor> g = w.param->grad();
        if (g) reduce_into(w, g->raw());
      }
    if (side) fz_check(fz_stream_wait(nullptr, side), "fz_stream_wait");
    std::vector<py::object> out;
    for (Watched &w : watched)
      out.push_back(w.avg ? py::cast(ADTensor(*w.avg, false)) : py::none());
    watched.clear();
    return out;
  }
  // Average each tensor over ranks, out of place, then rebind the tensor's storage
  // to the result so pending readers of the old value keep it. All reductions are
  // issued as one NCCL group.
  void allreduce_mean(const std::vector<ADTensor *> &ts) {
    if (!c) throw std::runtime_error("Comm: destroyed");
    std::vector<std::shared_ptr<DeviceBuffer>> outs;
    std::vector<const float *> ins;
    for (ADTensor *t : ts) {
      ins.push_back(t->raw().data());
      outs.push_back(std::make_shared<DeviceBuffer>(t->raw().size()));
    }
    fz_check(fz_comm_group_start(), "fz_comm_group_start");
    for (size_t i = 0; i < ts.size(); ++i)
      fz_check(fz_comm_allreduce(c, ins[i], outs[i]->ptr, (int64_t)ts[i]->raw().size(),
                                 1.0f / (float)world, nullptr),
               "fz_comm_allreduce");
    fz_check(fz_comm_group_end(), "fz_comm_group_end");
    for (size_t i = 0; i < ts.size(); ++i) ts[i]->raw().rebind_buffer(outs[i]);
  }
  void broadcast(const std::vector<ADTensor *> &ts, int root) {
    if (!c) throw std::runtime_error("Comm: destroyed");
    for (ADTensor *t : ts) {
      auto buf = std::make_shared<DeviceBuffer>(t->raw().size());
      fz_check(fz_memcpy_d2d(buf->ptr, t->raw().data(), t->raw().size() * 4, nullptr), "fz_memcpy_d2d");
      fz_check(fz_comm_broadcast(c, buf->ptr, (int64_t)t->raw().size(), root, nullptr), "fz_comm_broadcast");
      t->raw().rebind_buffer(buf);
    }
  }
  void wait(double timeout_s) {
    if (!c) throw std::runtime_error("Comm: destroyed");
    fz_check(fz_comm_wait(c, nullptr, timeout_s), "fz_comm_wait");
  }
};

}  // namespace

PYBIND11_MODULE(fusion, m) {
  m.doc() = "Fusion Tensor module exposing Tensor<float> (for composition) on the B200 backend";

  py::class_<Device>(m, "CppDevice", py::module_local())
      .def(py::init([](DeviceType t, int idx) { return Device(t, idx); }), py::arg("type"),
           py::arg("index") = -1)
      .def_property_readonly("type", [](const Device &d) { return d.type; })
      .def_property_readonly("index", [](const Device &d) { return d.idx; });

  py::enum_<DeviceType>(m, "CppDeviceType", py::module_local())
      .value("CPU", DeviceType::CPU)
      .value("CUDA", DeviceType::CUDA)
      .value("METAL", DeviceType::METAL);

  py::enum_<DType>(m, "CppDType", py::module_local())
      .value("FLOAT32", DType::FLOAT32)
      .value("FLOAT64", DType::FLOAT64)
      .value("INT32", DType::INT32)
      .value("INT64", DType::INT64)
      .value("BOOL", DType::BOOL);

  using T = ADTensor;
  py::class_<T>(m, "Tensor", py::module_local())
      .def(py::init([](const std::vector<size_t> &shape, DType dt, Device dev, bool rg) {
             return T(RawTensor(shape, dt, dev), rg);
           }),
           py::arg("shape"), py::arg("dtype"), py::arg("device"), py::arg("requires_grad"),
           "Construct a Tensor of given shape, zero-initialized. Optionally set requires_grad.")
      .def(py::init([](const std::vector<size_t> &shape,
                       py::array_t<float, py::array::c_style | py::array::forcecast> data, DType dt,
                       Device dev, bool rg) { return T(raw_from_array(shape, data, dt, dev), rg); }),
           py::arg("shape"), py::arg("data"), py::arg("dtype"), py::arg("device"),
           py::arg("requires_grad"),
           "Construct a Tensor from a shape list and flat data (list or array).")
      .def(
          "set_values",
          [](T &t, py::array_t<float, py::array::c_style | py::array::forcecast> vals) {
            size_t expected = t.flat_size();
            if ((size_t)vals.size() != expected)
              throw std::invalid_argument("set_values: expected " + std::to_string(expected) +
                                          " elements, got " + std::to_string(vals.size()));
            t.raw().set_values(vals.data(), expected);
          },
          py::arg("values"), "Fill the Tensor with a flat list of length prod(shape).")
      .def_property_readonly("shape", [](const T &t) { return t.shape(); })
      .def_property_readonly("ndim", [](const T &t) { return t.rank(); })
      .def_property_readonly("dtype", [](const T &) { return py::dtype::of<float>(); })
      .def_property_readonly("size", &T::flat_size)
      .def_property_readonly("name", [](const T &) { return std::string("ADTensor"); })
      .def_property_readonly("device", [](const T &t) { return t.device(); })
      .def_property("requires_grad", &T::requires_grad, &T::set_requires_grad)
      .def("to_numpy", &to_numpy, "Return a NumPy copy of the Tensor's contents.")
      .def("__repr__", [](const T &t) { return t.raw().repr(); })
      .def("__add__", [](const T &a, const T &b) { return a.binary_op(OpKind::Add, b); }, py::is_operator())
      .def("__add__", [](const T &a, float b) { return a.binary_scalar(OpKind::Add, b); }, py::is_operator())
      .def("__sub__", [](const T &a, const T &b) { return a.binary_op(OpKind::Subtract, b); }, py::is_operator())
      .def("__sub__", [](const T &a, float b) { return a.binary_scalar(OpKind::Subtract, b); }, py::is_operator())
      .def("__mul__", [](const T &a, const T &b) { return a.binary_op(OpKind::Multiply, b); }, py::is_operator())
      .def("__mul__", [](const T &a, float b) { return a.binary_scalar(OpKind::Multiply, b); }, py::is_operator())
      .def("__truediv__", [](const T &a, const T &b) { return a.binary_op(OpKind::Divide, b); }, py::is_operator())
      .def("__truediv__", [](const T &a, float b) { return a.binary_scalar(OpKind::Divide, b); }, py::is_operator())
      .def("__pow__", [](const T &a, const T &b) { return a.binary_op(OpKind::Pow, b); }, py::is_operator())
      .def("__pow__", [](const T &a, float b) { return a.binary_scalar(OpKind::Pow, b); }, py::is_operator())
      .def("__ge__", [](const T &a, const T &b) { return a.binary_op(OpKind::GreaterThanEqual, b); }, py::is_operator())
      .def("__ge__", [](const T &a, float b) { return a.binary_scalar(OpKind::GreaterThanEqual, b); }, py::is_operator())
      .def("__gt__", [](const T &a, const T &b) { return a.binary_op(OpKind::GreaterThan, b); }, py::is_operator())
      .def(
          "__neg__",
          // BindTensor.hpp:120-126 computes zeros_like(raw) - raw (an untracked result)
          [](const T &t) { return T(zeros_like(t.raw()) - t.raw(), false); }, py::is_operator())
      .def(
          "__isub__",
          [](T &a, const T &b) -> T & {
            a.raw() -= b.raw();
            return a;
          },
          py::is_operator())
      .def("sqrt", [](const T &t) { return t.unary_op(OpKind::Sqrt); })
      .def("exp", [](const T &t) { return t.unary_op(OpKind::Exp); })
      .def("log", [](const T &t) { return t.unary_op(OpKind::Log); })
      .def("sum", [](const T &t) { return t.unary_op(OpKind::Sum, OpParam{kGlobalReduceAxis, false}); })
      .def(
          "sum",
          [](const T &t, size_t axis, bool keepdim) { return t.unary_op(OpKind::Sum, OpParam{axis, keepdim}); },
          py::arg("axis"), py::arg("keepdim") = false)
      .def("mean", [](const T &t) { return t.unary_op(OpKind::Mean, OpParam{kGlobalReduceAxis, false}); })
      .def(
          "mean",
          [](const T &t, size_t axis, bool keepdim) { return t.unary_op(OpKind::Mean, OpParam{axis, keepdim}); },
          py::arg("axis"), py::arg("keepdim") = false)
      .def(
          "max",
          // New reduction (no reference counterpart); untracked, like comparisons' values.
          [](const T &t, py::object axis, bool keepdim) {
            size_t ax = axis.is_none() ? kGlobalReduceAxis : axis.cast<size_t>();
            return T(t.raw().max(ax, keepdim), false);
          },
          py::arg("axis") = py::none(), py::arg("keepdim") = false)
      .def("__matmul__", [](const T &a, const T &b) { return a.binary_op(OpKind::MatMul, b); })
      .def("maximum", [](const T &a, const T &b) { return a.binary_op(OpKind::Maximum, b); }, py::is_operator())
      .def("maximum", [](const T &a, float b) { return a.binary_scalar(OpKind::Maximum, b); }, py::is_operator())
      .def(
          "swapaxes",
          [](const T &t, int a1, int a2) {
            OpParam p;
            p.axis1 = a1;
            p.axis2 = a2;
            return t.unary_op(OpKind::SwapAxes, p);
          },
          py::arg("axis1"), py::arg("axis2"))
      .def("backward", &T::backward)
      .def("get_grad", &T::grad)
      .def("rank", &T::rank)
      .def("is_pending", [](const T &t) { return t.raw().pending(); },
           "True while the value is an unlowered node of the fusion IR.");

  auto fac = m.def_submodule("factory", "factory functions for Tensor<float>");
  fac.def("fill", [](const std::vector<size_t> &s, float v, Device d) {
    return T(RawTensor::full(s, v, DType::FLOAT32, d), false);
  }, py::arg("shape"), py::arg("value"), py::arg("device"));
  fac.def("zeros", [](const std::vector<size_t> &s, Device d) {
    return T(RawTensor::full(s, 0.0f, DType::FLOAT32, d), false);
  }, py::arg("shape"), py::arg("device"));
  fac.def("ones", [](const std::vector<size_t> &s, Device d) {
    return T(RawTensor::full(s, 1.0f, DType::FLOAT32, d), false);
  }, py::arg("shape"), py::arg("device"));
  fac.def("zeros_like", [](const T &t) { return T(zeros_like(t.raw()), t.requires_grad()); },
          py::arg("other"));
  fac.def("ones_like", [](const T &t) { return T(ones_like(t.raw()), t.requires_grad()); },
          py::arg("other"));

  py::class_<Random>(m, "Random", py::module_local())
      .def(py::init<uint32_t>(), py::arg("seed") = std::random_device{}())
      .def("uniform_device", &Random::uniform_device, py::arg("shape"), py::arg("min"), py::arg("max"),
           py::arg("device"),
           "Uniform values in [min, max) drawn on the GPU from this seed's Philox-4x32-10 stream "
           "(not the mt19937 stream of uniform_cpp).")
      .def("dropout", &Random::dropout, py::arg("x"), py::arg("rate"),
           "Nova's Dropout, x * (u >= rate) / (1 - rate) with u drawn on the GPU, in one kernel; "
           "traced by autodiff (the backward redraws the mask).")
      .def_readonly("philox_offset", &Random::offset)
      .def("uniform_cpp", &Random::uniform, py::arg("shape"), py::arg("min"), py::arg("max"),
           py::arg("device"));

  py::class_<GradTape>(m, "grad_tape", py::module_local())
      .def(py::init<>())
      .def(
          "__enter__",
          [](GradTape &self) -> GradTape & {
            self.scope.enter();
            return self;
          },
          py::return_value_policy::reference)
      .def("__exit__", [](GradTape &self, const py::object &, const py::object &, const py::object &) {
        self.scope.exit();
        return false;
      });

  auto ad = m.def_submodule("autodiff", "Autodiff control");
  ad.def(
      "enabled",
      [](py::object state) {
        if (!state.is_none()) set_autodiff_enabled(state.cast<bool>());
        return grad_enabled();
      },
      py::arg("state") = py::none(),
      "Get or set whether autodiff is enabled for this thread. When enabled, a default "
      "Engine is installed in the EngineContext.");

  // ---- backend controls (no reference counterpart) ------------------------
  m.def("set_device", [](int d) { fz_check(fz_set_device(d), "fz_set_device"); }, py::arg("index"),
        "Make CUDA device `index` current for this thread.");
  m.def("device_count", []() {
    int n = 0;
    fz_device_count(&n);
    return n;
  });
  m.def("synchronize", []() {
    fz_check(fz_stream_sync(nullptr), "fz_stream_sync");
    fz_check(fz_kernel_status(), "fz_kernel_status");
  }, "Wait for this thread's stream and surface any kernel-side bounded-wait error.");
  m.def("set_fusion", &set_fusion_enabled, py::arg("enabled"),
        "Enable (default) or disable lazy elementwise fusion.");
  m.def("fusion_enabled", &fusion_enabled);
  m.def("flat_prefix", [](const T &t, const T &like) {
          return T(math::flat_prefix(t.raw(), like.raw().size(), like.raw().shape()), false);
        }, py::arg("tensor"), py::arg("like"),
        "The first like.size values of tensor (flat order) as a new tensor shaped like `like`: "
        "what `like -= tensor` reads.");
  m.def("set_split_cache", &set_split_cache_enabled, py::arg("enabled"),
        "Keep GEMM operands' TF32 remainder planes with their buffers (default on).");
  m.def("split_cache_enabled", &split_cache_enabled);
  m.def("set_swap_views", &set_swap_views_enabled, py::arg("enabled"),
        "Keep swapaxes of the last two axes (Nova's .T) as a view that GEMMs read in place "
        "(default on); off materialises every swapaxes where it is called.");
  m.def("swap_views_enabled", &swap_views_enabled);
  m.def("set_gemm_epilogue", &set_gemm_epilogue_enabled, py::arg("enabled"),
        "Defer each GEMM so the elementwise program reading its product runs in the GEMM's "
        "epilogue (default on); off launches every GEMM where it is called.");
  m.def("gemm_epilogue_enabled", &gemm_epilogue_enabled);
  m.def("empty_cache", []() { fz_check(fz_pool_release(), "fz_pool_release"); },
        "Return this device's cached blocks to the driver (synchronises the device).");
  m.def("flush", [](const T &t) {
          t.raw().data();
          t.raw().expr()->buf->mark_ready();
        }, py::arg("tensor"),
        "Lower a pending tensor to device memory now; a later to_numpy() then reads it back "
        "as soon as it is ready, without waiting for work submitted after the flush.");
  m.def("stats", []() {
    py::dict d;
    d["kernel_launches"] = fz_launch_count();
    d["fused_launches"] = fused_launches();
    d["epilogue_gemms"] = epilogue_gemms();
    d["swap_materializations"] = swap_materializations();
    d["lo_splits"] = lo_splits();
    d["plan_cache_hits"] = plan_cache_hits();
    d["plan_cache_misses"] = plan_cache_misses();
    d["fused_kernels_compiled"] = fz_fused_cache_size();
    size_t r = 0, u = 0;
    if (fz_pool_stats(&r, &u) == FZ_OK) {
      d["pool_reserved_bytes"] = r;
      d["pool_used_bytes"] = u;
    }
    return d;
  });
  m.def("device_ptr", [](const T &t) { return reinterpret_cast<uintptr_t>(t.raw().data()); },
        py::arg("tensor"), "Device address of the tensor's data (lowers it if pending).");

  m.def("comm_unique_id", []() {
    unsigned char id[FZ_UNIQUE_ID_BYTES];
    fz_check(fz_comm_unique_id(id), "fz_comm_unique_id");
    return py::bytes(reinterpret_cast<const char *>(id), FZ_UNIQUE_ID_BYTES);
  }, "NCCL unique id (128 bytes) for rank 0 to share with the other ranks.");
  py::class_<Comm>(m, "Comm", py::module_local())
      .def(py::init<int, int, py::bytes>(), py::arg("world"), py::arg("rank"), py::arg("unique_id"))
      .def_readonly("world", &Comm::world)
      .def_readonly("rank", &Comm::rank)
      .def("allreduce_mean", &Comm::allreduce_mean, py::arg("tensors"),
           "Average tensors over all ranks (one NCCL group, out of place).")
      .def("watch", &Comm::watch, py::arg("params"),
           "Average these parameters' gradients over ranks as the backward completes them "
           "(on a second stream, overlapping the rest of the backward).")
      .def_readonly("overlapped", &Comm::overlapped,
                    "How many of the last collect()'s gradients were reduced during the backward.")
      .def("collect", &Comm::collect,
           "The averaged gradients of the watched parameters, in order (None if none).")
      .def("broadcast", &Comm::broadcast, py::arg("tensors"), py::arg("root") = 0)
      .def("wait", &Comm::wait, py::arg("timeout_s"),
           "Wait for this rank's stream with a deadline; on expiry abort the communicator "
           "and raise.")
      .def("destroy", &Comm::destroy);
}
