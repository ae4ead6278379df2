// RawTensor, device storage and the fusion IR lowering (see tensor.hpp).
#include "tensor.hpp"

#include <algorithm>
#include <cstring>
#include <numeric>
#include <sstream>
#include <unordered_map>
#include <unordered_set>

namespace fusion_b200 {

// ---------------------------------------------------------------- errors
void throw_check(const char *file, int line, const std::string &msg) {
  // Same text shape as FUSION_CHECK (fusion/src/Fusion/common/Checks.hpp:14-29).
  std::ostringstream os;
  os << "FUSION_CHECK failed @ " << file << ":" << line << ": " << msg;
  throw std::runtime_error(os.str());
}

void fz_check(int rc, const char *what) {
  if (rc == FZ_OK) return;
  std::string msg = std::string(what) + ": " + fz_last_error();
  if (rc == FZ_ERR_OOM) throw std::bad_alloc();
  if (rc == FZ_ERR_INVALID) throw std::invalid_argument(msg);
  throw std::runtime_error(msg);
}

// ---------------------------------------------------------------- device
static int device_count_cached() {
  static int n = -1;
  if (n < 0) {
    int c = 0;
    n = fz_device_count(&c) == FZ_OK ? c : 0;
  }
  return n;
}

Device::Device(DeviceType t, int i) : type(t), idx(i) {
  if (t == DeviceType::CPU) FB_CHECK(i <= 0, "Invalid device index");
  else if (t == DeviceType::CUDA) FB_CHECK(i >= -1, "Invalid device index");
  else throw std::runtime_error("Unsupported device");
}

int Device::cuda_index() const {
  if (type == DeviceType::CUDA && idx >= 0) return idx;
  int d = 0;
  fz_check(fz_get_device(&d), "fz_get_device");
  return d;
}

int bind_device(const Device &d) {
  int want = d.cuda_index();
  int cur = -1;
  fz_get_device(&cur);
  if (cur != want || fz_default_stream() == nullptr) {
    FB_CHECK(want < device_count_cached(), "Invalid device index");
    fz_check(fz_set_device(want), "fz_set_device");
  }
  return want;
}

size_t dtype_size(DType d) {
  switch (d) {
    case DType::FLOAT32: return 4;
    case DType::FLOAT64: return 8;
    case DType::INT32: return 4;
    case DType::INT64: return 8;
    case DType::BOOL: return 1;
  }
  throw std::runtime_error("Unknown DType");
}

// ---------------------------------------------------------------- memory
DeviceBuffer::DeviceBuffer(size_t n) : DeviceBuffer(n, nullptr) {}

DeviceBuffer::DeviceBuffer(size_t n, void *stream) : numel(n) {
  fz_get_device(&device);
  void *p = nullptr;
  fz_check(fz_malloc(&p, n * sizeof(float), stream), "fz_malloc");
  ptr = static_cast<float *>(p);
}

DeviceBuffer::~DeviceBuffer() {
  if (ready) fz_event_destroy(ready);
  if (ptr) fz_free(ptr, nullptr);
}

void DeviceBuffer::mark_ready() {
  if (ready) fz_event_destroy(ready);
  ready = nullptr;
  fz_check(fz_event_record(&ready, nullptr), "fz_event_record");
}

size_t Expr::numel() const {
  size_t n = 1;
  for (auto s : shape) n *= s;
  return n;
}

// ---------------------------------------------------------------- fusion IR
static bool g_fusion = true;
static bool g_split_cache = true;
void set_split_cache_enabled(bool on) { g_split_cache = on; }
bool split_cache_enabled() { return g_split_cache; }
static bool g_gemm_epilogue = true;
void set_gemm_epilogue_enabled(bool on) { g_gemm_epilogue = on; }
bool gemm_epilogue_enabled() { return g_gemm_epilogue; }
static int64_t g_epilogue_gemms = 0;
int64_t epilogue_gemms() { return g_epilogue_gemms; }
static int64_t g_fused_launches = 0;
constexpr int kNodeLimit = 40;   // below FZ_MAX_NODES, leaving room for dedupe slack
constexpr int kLeafLimit = 10;   // below FZ_MAX_LEAVES

static int64_t g_lo_splits = 0;  // separate split passes (planes not made by a producer)
int64_t lo_splits() { return g_lo_splits; }
static bool g_swap_views = true;
static int64_t g_swap_materializations = 0;
void set_swap_views_enabled(bool on) { g_swap_views = on; }
bool swap_views_enabled() { return g_swap_views; }
int64_t swap_materializations() { return g_swap_materializations; }

void set_fusion_enabled(bool on) { g_fusion = on; }
bool fusion_enabled() { return g_fusion; }
int64_t fused_launches() { return g_fused_launches; }

static ExprPtr make_leaf(std::shared_ptr<DeviceBuffer> buf, std::vector<size_t> shape) {
  auto e = std::make_shared<Expr>();
  e->kind = Expr::Leaf;
  e->shape = std::move(shape);
  e->buf = std::move(buf);
  e->nodes_ub = 0;
  e->leaves_ub = 1;
  return e;
}

static ExprPtr make_const(float v, std::vector<size_t> shape) {
  auto e = std::make_shared<Expr>();
  e->kind = Expr::Const;
  e->shape = std::move(shape);
  e->imm = v;
  e->nodes_ub = 1;
  e->leaves_ub = 0;
  return e;
}

float *Storage::data() {
  if (expr->kind != Expr::Leaf) materialize(expr);
  return expr->buf ? expr->buf->ptr : nullptr;
}

// Right-aligned broadcast of two shapes (TensorPlan.cpp:40-48, 67-126 rules).
static std::vector<size_t> broadcast_shape(const std::vector<size_t> &a, const std::vector<size_t> &b) {
  size_t n = std::max(a.size(), b.size());
  std::vector<size_t> out(n);
  for (size_t d = 0; d < n; ++d) {
    long ia = (long)d - (long)(n - a.size()), ib = (long)d - (long)(n - b.size());
    size_t da = ia >= 0 ? a[ia] : 1, db = ib >= 0 ? b[ib] : 1;
    if (da == db || db == 1) out[d] = da;
    else if (da == 1) out[d] = db;
    else throw std::runtime_error("broadcast: dimension mismatch");
  }
  return out;
}

// Element strides of a contiguous operand of shape `s` seen from output shape
// `out`: 0 on broadcast dims (TensorPlan.cpp:50-65).
// An operand with more dims than `out` (a flat-prefix evaluation, below) sits at
// index 0 along its extra leading dims.
static void operand_strides(const std::vector<size_t> &s, const std::vector<size_t> &out,
                            int64_t *st) {
  const long nd = (long)out.size(), pad = nd - (long)s.size();
  int64_t r = 1;
  for (long d = (long)nd - 1; d >= 0; --d) {
    long i = d - pad;
    if (i < 0) {
      st[d] = 0;
      continue;
    }
    st[d] = (s[i] == 1 && out[d] > 1) ? 0 : r;
    r *= (int64_t)s[i];
  }
}

static void lower_gemm(Expr *e);
static void lower_swap(Expr *e);

namespace {
struct Lowering {
  fz_program prog{};
  std::unordered_map<const Expr *, int> node_of;
  std::vector<const Expr *> leaves;
  std::unordered_map<const float *, int> leaf_of_buf;  // dedupe equal buffers of equal shape
  bool overflow = false;
  const Expr *acc = nullptr;  // epilogue programs: the pending GEMM read as leaf 0

  Lowering() = default;
  explicit Lowering(const Expr *product) : acc(product) { leaves.push_back(product); }

  int leaf_index(const Expr *e) {
    auto it = leaf_of_buf.find(e->buf->ptr);
    if (it != leaf_of_buf.end() && leaves[it->second]->shape == e->shape) return it->second;
    if ((int)leaves.size() >= FZ_MAX_LEAVES) {
      overflow = true;
      return 0;
    }
    leaves.push_back(e);
    leaf_of_buf[e->buf->ptr] = (int)leaves.size() - 1;
    return (int)leaves.size() - 1;
  }

  // Returns an operand reference (>= 0 node, < 0 leaf).
  int visit(const Expr *e) {
    if (overflow) return 0;
    if (e == acc) return -1;
    // any other pending GEMM is a plain product read as a leaf, and a pending
    // swapaxes view is materialised and read as a leaf
    if (e->kind == Expr::Gemm) lower_gemm(const_cast<Expr *>(e));
    if (e->kind == Expr::Swap) lower_swap(const_cast<Expr *>(e));
    if (e->kind == Expr::Leaf) return -1 - leaf_index(e);
    auto it = node_of.find(e);
    if (it != node_of.end()) return it->second;
    int s0 = 0, s1 = 0;
    if (e->kind == Expr::Unary || e->kind == Expr::Binary) s0 = visit(e->a.get());
    if (e->kind == Expr::Binary) s1 = visit(e->b.get());
    if (overflow) return 0;
    if (prog.num_nodes >= FZ_MAX_NODES) {
      overflow = true;
      return 0;
    }
    fz_node &n = prog.nodes[prog.num_nodes];
    n.kind = e->kind == Expr::Binary ? FZ_NODE_BINARY : e->kind == Expr::Unary ? FZ_NODE_UNARY : FZ_NODE_CONST;
    n.op = e->op;
    n.src0 = s0;
    n.src1 = s1;
    n.imm = e->imm;
    node_of[e] = prog.num_nodes;
    return prog.num_nodes++;
  }
};

// Merge chained dims on the host (for ranks above FZ_MAX_DIMS), operands share `size`.
int collapse(std::vector<int64_t> &size, std::vector<std::vector<int64_t>> &st) {
  std::vector<int64_t> s2;
  std::vector<std::vector<int64_t>> st2(st.size());
  for (size_t d = 0; d < size.size(); ++d) {
    if (size[d] == 1) continue;
    if (!s2.empty()) {
      bool chain = true;
      for (size_t k = 0; k < st.size() && chain; ++k) chain = st2[k].back() == st[k][d] * size[d];
      if (chain) {
        s2.back() *= size[d];
        for (size_t k = 0; k < st.size(); ++k) st2[k].back() = st[k][d];
        continue;
      }
    }
    s2.push_back(size[d]);
    for (size_t k = 0; k < st.size(); ++k) st2[k].push_back(st[k][d]);
  }
  size.swap(s2);
  st.swap(st2);
  return (int)size.size();
}
}  // namespace

// ---- launch-plan cache (the shape caching fusion/src/Fusion/core/PlanMeta.hpp:10-13
// leaves as a TODO): the plan of `nout` outputs of shape `out` and operands of the
// given shapes depends on the shapes only, so it is built once per shape set.
namespace {
struct PlanKeyHash {
  size_t operator()(const std::vector<int64_t> &k) const {
    size_t h = 1469598103934665603ull;
    for (int64_t v : k) h = (h ^ (size_t)v) * 1099511628211ull;
    return h;
  }
};
thread_local std::unordered_map<std::vector<int64_t>, fz_ewise_plan, PlanKeyHash> t_plans;
int64_t g_plan_hits = 0, g_plan_misses = 0;
constexpr size_t kPlanCacheMax = 4096;
}  // namespace
int64_t plan_cache_hits() { return g_plan_hits; }
int64_t plan_cache_misses() { return g_plan_misses; }

static const fz_ewise_plan &cached_plan(const std::vector<size_t> &out, int nout,
                                        const std::vector<const std::vector<size_t> *> &ins) {
  std::vector<int64_t> key;
  key.reserve(2 + out.size() + 4 * ins.size());
  key.push_back(nout);
  key.push_back((int64_t)out.size());
  for (size_t d : out) key.push_back((int64_t)d);
  for (const auto *s : ins) {
    key.push_back(-1 - (int64_t)s->size());
    for (size_t d : *s) key.push_back((int64_t)d);
  }
  auto it = t_plans.find(key);
  if (it != t_plans.end()) {
    ++g_plan_hits;
    return it->second;
  }
  ++g_plan_misses;
  const int nops = nout + (int)ins.size();
  std::vector<int64_t> size(out.begin(), out.end());
  std::vector<std::vector<int64_t>> st(nops, std::vector<int64_t>(out.size()));
  for (int k = 0; k < nout; ++k) operand_strides(out, out, st[k].data());
  for (size_t k = 0; k < ins.size(); ++k) operand_strides(*ins[k], out, st[nout + k].data());
  if ((int)size.size() > FZ_MAX_DIMS) collapse(size, st);
  FB_CHECK((int)size.size() <= FZ_MAX_DIMS, "fused elementwise: too many non-mergeable dims");
  fz_ewise_plan plan{};
  plan.ndim = (int32_t)size.size();
  plan.num_operands = nops;
  for (int d = 0; d < plan.ndim; ++d) {
    plan.size[d] = size[d];
    for (int k = 0; k < nops; ++k) plan.stride_bytes[k][d] = st[k][d] * 4;
  }
  if (t_plans.size() >= kPlanCacheMax) t_plans.clear();
  return t_plans.emplace(std::move(key), plan).first->second;
}

// Launch a lowered program whose outputs (all of out_shape) go to `outs`.
static void launch_program(const Lowering &L, const std::vector<size_t> &out_shape,
                           const std::vector<float *> &outs) {
  std::vector<const std::vector<size_t> *> ins;
  ins.reserve(L.leaves.size());
  for (const Expr *l : L.leaves) ins.push_back(&l->shape);
  const fz_ewise_plan plan = cached_plan(out_shape, (int)outs.size(), ins);
  std::vector<const float *> leaf_ptrs;
  for (auto *l : L.leaves) leaf_ptrs.push_back(l->buf->ptr);
  fz_check(fz_fused_launch(&L.prog, &plan, outs.data(), leaf_ptrs.data(), nullptr), "fz_fused_launch");
  ++g_fused_launches;
}

// A single binary op over two leaves runs on the ahead-of-time kernels.
static bool try_single_op(Expr *e, float *out_ptr) {
  if (e->kind == Expr::Binary && e->a->kind == Expr::Leaf && e->b->kind == Expr::Leaf) {
    const auto &os = e->shape;
    if (e->a->shape == os && e->b->shape == os) {
      fz_check(fz_ewise_binary_contig(e->op, (int64_t)e->numel(), out_ptr, e->a->buf->ptr,
                                      e->b->buf->ptr, nullptr), "fz_ewise_binary_contig");
      return true;
    }
    if (os.size() <= FZ_MAX_DIMS) {
      const fz_ewise_plan &plan = cached_plan(os, 1, {&e->a->shape, &e->b->shape});
      fz_check(fz_ewise_binary(e->op, &plan, out_ptr, e->a->buf->ptr, e->b->buf->ptr, nullptr),
               "fz_ewise_binary");
      return true;
    }
  }
  if (e->kind == Expr::Unary && e->a->kind == Expr::Leaf && e->a->shape == e->shape) {
    fz_ewise_plan plan{};
    plan.ndim = 1;
    plan.num_operands = 2;
    plan.size[0] = (int64_t)e->numel();
    plan.stride_bytes[0][0] = plan.stride_bytes[1][0] = 4;
    fz_check(fz_ewise_unary(e->op, &plan, out_ptr, e->a->buf->ptr, nullptr), "fz_ewise_unary");
    return true;
  }
  if (e->kind == Expr::Const) {
    fz_check(fz_fill_f32(out_ptr, e->imm, (int64_t)e->numel(), nullptr), "fz_fill_f32");
    return true;
  }
  return false;
}

// Values at flat indices [0, prod(shape[k:])) of a pending node, i.e. the slice
// at index 0 of its first k dims, lowered into a fresh buffer.
static std::shared_ptr<DeviceBuffer> materialize_prefix(const ExprPtr &ep, size_t k) {
  std::vector<size_t> sub(ep->shape.begin() + (long)k, ep->shape.end());
  size_t n = 1;
  for (auto v : sub) n *= v;
  auto out = std::make_shared<DeviceBuffer>(n);
  if (n == 0) return out;
  Lowering L;
  int root = L.visit(ep.get());
  if (L.overflow) return nullptr;
  L.prog.num_leaves = (int32_t)L.leaves.size();
  L.prog.num_outputs = 1;
  L.prog.out_node[0] = root;
  launch_program(L, sub, {out->ptr});
  return out;
}

// [outer, len, inner] view of a Reduce node over its input's shape.
static void reduce_view(const Expr &e, int64_t &outer, int64_t &len, int64_t &inner) {
  const auto &s = e.a->shape;
  outer = len = inner = 1;
  for (int d = 0; d < (int)s.size(); ++d) {
    if (d < e.red_lo) outer *= (int64_t)s[d];
    else if (d <= e.red_hi) len *= (int64_t)s[d];
    else inner *= (int64_t)s[d];
  }
}

// A swapaxes(-1, -2) view read by something other than a GEMM or a swapaxes: the
// source (lowered first if pending) transposed into a buffer by the transpose kernel.
static void lower_swap(Expr *e) {
  if (e->a->kind != Expr::Leaf) materialize(e->a);
  const std::vector<size_t> &src = e->a->shape;
  std::vector<int64_t> shp(src.begin(), src.end());
  const int nd = (int)shp.size();
  auto out = std::make_shared<DeviceBuffer>(e->numel());
  if (e->numel() > 0)
    fz_check(fz_swapaxes(out->ptr, e->a->buf->ptr, shp.data(), nd, nd - 2, nd - 1, nullptr), "fz_swapaxes");
  ++g_swap_materializations;
  e->kind = Expr::Leaf;
  e->buf = std::move(out);
  e->a.reset();
  e->nodes_ub = 0;
  e->leaves_ub = 1;
}

// A pending GEMM lowered by itself: the product into a buffer.
static void lower_gemm(Expr *e) {
  const GemmSpec &g = *e->gemm;
  auto out = std::make_shared<DeviceBuffer>(e->numel());
  fz_check(fz_gemm_f32_split(g.batch, g.M, g.N, g.K, g.pa, g.la, g.lda, g.sA, g.transA, g.pb,
                             g.lb, g.ldb, g.sB, g.transB, out->ptr, g.N, g.M * g.N, nullptr),
           "fz_gemm_f32_split");
  e->kind = Expr::Leaf;
  e->buf = std::move(out);
  e->gemm.reset();
  e->nodes_ub = 0;
  e->leaves_ub = 1;
}

namespace {
// The DAG under a set of roots, as the epilogue lowering needs it.
struct EpiScan {
  std::unordered_set<const Expr *> seen, roots;
  std::unordered_map<const Expr *, int> in_edges;           // parent edges inside the DAG
  std::unordered_map<const Expr *, const ExprPtr *> owner;  // a parent's pointer to the node
  std::vector<const Expr *> ops;                            // Unary / Binary nodes
  const Expr *gemm = nullptr;
  int gemms = 0;
  bool ok = true;

  void scan(const Expr *e, const ExprPtr *from) {
    if (from) {
      ++in_edges[e];
      owner.emplace(e, from);
    }
    if (!seen.insert(e).second) return;
    switch (e->kind) {
      case Expr::Leaf:
      case Expr::Const: return;
      case Expr::Reduce:
      case Expr::Swap: ok = false; return;
      case Expr::Gemm:
        gemm = e;
        ++gemms;
        return;
      case Expr::Unary:
        ops.push_back(e);
        scan(e->a.get(), &e->a);
        return;
      case Expr::Binary:
        ops.push_back(e);
        scan(e->a.get(), &e->a);
        scan(e->b.get(), &e->b);
        return;
    }
  }
  // References to e from outside the DAG (tensors, saved contexts, other programs).
  long external(const Expr *e) const {
    auto it = owner.find(e);
    if (it == owner.end()) return 1;
    auto jt = in_edges.find(e);
    return it->second->use_count() - (jt == in_edges.end() ? 0 : jt->second);
  }
};

bool reaches(const Expr *e, const Expr *target, std::unordered_map<const Expr *, bool> &memo) {
  if (e == target) return true;
  if (e->kind != Expr::Unary && e->kind != Expr::Binary) return false;
  auto it = memo.find(e);
  if (it != memo.end()) return it->second;
  bool r = reaches(e->a.get(), target, memo) || (e->kind == Expr::Binary && reaches(e->b.get(), target, memo));
  memo[e] = r;
  return r;
}

// How an input of shape `s` reads from the product's [batch..., M, N] index space:
// strides along the (flattened) batch, the rows and the columns. False when the batch
// dims do not flatten into one stride.
bool epilogue_input(const std::vector<size_t> &s, const std::vector<size_t> &out, const float *ptr,
                    fz_epi_input *in) {
  const size_t nd = out.size();
  if (s.size() > nd || nd < 2) return false;
  int64_t st[64];
  if (nd > 64) return false;
  operand_strides(s, out, st);
  in->ptr = ptr;
  in->col_stride = st[nd - 1];
  in->row_stride = st[nd - 2];
  if (in->col_stride != 0 && in->col_stride != 1) return false;
  // batch offset = bz * batch_stride for the flat batch index bz
  int64_t sb = 0, inner = 1;
  bool have = false;
  for (long d = (long)nd - 3; d >= 0; --d) {
    if (out[d] == 1) continue;
    if (!have) {
      sb = st[d];
      have = true;
    } else if (st[d] != sb * inner) {
      return false;
    }
    inner *= (int64_t)out[d];
  }
  in->batch_stride = sb;
  return true;
}
}  // namespace

// Lower pending nodes that read exactly one pending GEMM (and leaves broadcast into its
// product as rows, columns or batch slices) as the outputs of that GEMM's epilogue:
// one kernel writes every root (and, for roots with want_lo, its TF32 remainder plane)
// straight from the accumulators. The product is stored as well only when something
// outside these roots still holds the GEMM node. Returns false, having done nothing,
// when the roots do not qualify.
static bool try_epilogue(const std::vector<ExprPtr> &roots, const std::vector<bool> &want_lo) {
  if (!g_gemm_epilogue || !g_fusion || roots.empty()) return false;
  bool any = false;  // no pending GEMM under any root: nothing to scan
  for (const ExprPtr &r : roots) any = any || r->gemm_below;
  if (!any) return false;
  EpiScan S;
  for (const ExprPtr &r : roots) S.roots.insert(r.get());
  for (const ExprPtr &r : roots) S.scan(r.get(), nullptr);
  if (!S.ok || S.gemms != 1) return false;
  Expr *G = const_cast<Expr *>(S.gemm);
  const std::vector<size_t> &oshape = G->shape;
  for (const ExprPtr &r : roots)
    if (r->shape != oshape) return false;
  const bool g_root = S.roots.count(G) > 0;
  bool g_needed = false;
  if (!g_root) {
    g_needed = S.external(G) > 0;
    std::unordered_map<const Expr *, bool> memo;
    for (const Expr *x : S.ops)
      if (!g_needed && !S.roots.count(x) && S.external(x) > 0 && reaches(x, G, memo)) g_needed = true;
  }
  Lowering L(G);
  std::vector<int> refs;
  for (const ExprPtr &r : roots) refs.push_back(L.visit(r.get()));
  if (L.overflow) return false;
  auto add_node = [&](int kind, int op, int src) {
    if (L.prog.num_nodes >= FZ_MAX_NODES) return -1;
    fz_node &n = L.prog.nodes[L.prog.num_nodes];
    n.kind = kind;
    n.op = op;
    n.src0 = src;
    n.src1 = 0;
    n.imm = 0.0f;
    return L.prog.num_nodes++;
  };
  std::vector<int> outs;
  for (int &r : refs) {
    if (r < 0) r = add_node(FZ_NODE_UNARY, FZ_COPY, r);  // a root that is the product itself
    if (r < 0) return false;
    outs.push_back(r);
  }
  int nlo = 0;
  for (size_t k = 0; k < roots.size(); ++k)
    if (want_lo[k]) {
      const int n = add_node(FZ_NODE_UNARY, FZ_TF32_LO, refs[k]);
      if (n < 0) return false;
      outs.push_back(n);
      ++nlo;
    }
  if (g_needed) {
    const int n = add_node(FZ_NODE_UNARY, FZ_COPY, -1);
    if (n < 0) return false;
    outs.push_back(n);
  }
  if ((int)outs.size() > FZ_MAX_OUTPUTS) return false;
  std::vector<fz_epi_input> inputs(L.leaves.size() - 1);
  for (size_t k = 1; k < L.leaves.size(); ++k)
    if (!epilogue_input(L.leaves[k]->shape, oshape, L.leaves[k]->buf->ptr, &inputs[k - 1])) return false;
  L.prog.num_leaves = (int32_t)L.leaves.size();
  L.prog.num_outputs = (int32_t)outs.size();
  for (size_t k = 0; k < outs.size(); ++k) L.prog.out_node[k] = outs[k];

  const GemmSpec &g = *G->gemm;
  const size_t n = G->numel();
  std::vector<std::shared_ptr<DeviceBuffer>> bufs;
  std::vector<float *> ptrs;
  for (size_t k = 0; k < outs.size(); ++k) {
    bufs.push_back(std::make_shared<DeviceBuffer>(n));
    ptrs.push_back(bufs.back()->ptr);
  }
  fz_check(fz_gemm_f32_epilogue(g.batch, g.M, g.N, g.K, g.pa, g.la, g.lda, g.sA, g.transA, g.pb,
                                g.lb, g.ldb, g.sB, g.transB, &L.prog,
                                inputs.empty() ? nullptr : inputs.data(), ptrs.data(), g.N,
                                g.M * g.N, nullptr),
           "fz_gemm_f32_epilogue");
  ++g_epilogue_gemms;
  size_t next_lo = roots.size();
  for (size_t k = 0; k < roots.size(); ++k) {
    Expr *e = roots[k].get();
    if (want_lo[k]) bufs[k]->tf32_lo = bufs[next_lo++];
    e->kind = Expr::Leaf;
    e->buf = bufs[k];
    e->a.reset();
    e->b.reset();
    e->gemm.reset();
    e->nodes_ub = 0;
    e->leaves_ub = 1;
  }
  if (g_needed) {
    G->kind = Expr::Leaf;
    G->buf = bufs.back();
    G->gemm.reset();
    G->nodes_ub = 0;
    G->leaves_ub = 1;
  }
  return true;
}

void materialize(const ExprPtr &ep) {
  Expr *e = ep.get();
  if (e->kind == Expr::Leaf) return;
  if (e->kind == Expr::Swap) {
    lower_swap(e);
    return;
  }
  if (e->kind == Expr::Gemm) {
    lower_gemm(e);
    return;
  }
  if ((e->kind == Expr::Unary || e->kind == Expr::Binary) && e->numel() > 0 &&
      try_epilogue({ep}, {false}))
    return;
  if (e->kind == Expr::Reduce) {
    if (e->a->kind != Expr::Leaf) materialize(e->a);
    int64_t outer, len, inner;
    reduce_view(*e, outer, len, inner);
    auto out = std::make_shared<DeviceBuffer>(e->numel());
    if (e->numel() > 0)
      fz_check(fz_reduce(e->op, out->ptr, e->a->buf->ptr, outer, len, inner, nullptr), "fz_reduce");
    e->kind = Expr::Leaf;
    e->buf = std::move(out);
    e->a.reset();
    e->nodes_ub = 0;
    e->leaves_ub = 1;
    return;
  }
  auto out = std::make_shared<DeviceBuffer>(e->numel());
  if (e->numel() > 0 && !try_single_op(e, out->ptr)) {
    Lowering L;
    int root = L.visit(e);
    if (L.overflow) {
      // too large for one program: materialise the operands first, then retry
      if (e->a) materialize(e->a);
      if (e->b) materialize(e->b);
      materialize(ep);
      return;
    }
    L.prog.num_leaves = (int32_t)L.leaves.size();
    L.prog.num_outputs = 1;
    L.prog.out_node[0] = root;
    launch_program(L, e->shape, {out->ptr});
  }
  e->kind = Expr::Leaf;
  e->buf = std::move(out);
  e->a.reset();
  e->b.reset();
  e->nodes_ub = 0;
  e->leaves_ub = 1;
}

// Lower a pending node together with its TF32 remainder plane (the lo plane a 3xTF32
// GEMM reads), as two outputs of one fused program: the plane costs one extra write
// instead of a second pass over the value. The plane is kept with the new buffer.
void materialize_with_lo(const ExprPtr &ep) {
  Expr *e = ep.get();
  if (e->kind == Expr::Leaf || e->kind == Expr::Const || e->kind == Expr::Reduce ||
      e->kind == Expr::Swap || e->numel() == 0) {
    materialize(ep);
    return;
  }
  if (try_epilogue({ep}, {true})) return;
  if (e->kind == Expr::Gemm) {
    lower_gemm(e);
    return;
  }
  Lowering L;
  const int root = L.visit(e);
  if (L.overflow || root < 0 || L.prog.num_nodes >= FZ_MAX_NODES) {
    materialize(ep);
    return;
  }
  fz_node &n = L.prog.nodes[L.prog.num_nodes];
  n.kind = FZ_NODE_UNARY;
  n.op = FZ_TF32_LO;
  n.src0 = root;
  n.src1 = 0;
  n.imm = 0.0f;
  const int lo_node = L.prog.num_nodes++;
  L.prog.num_leaves = (int32_t)L.leaves.size();
  L.prog.num_outputs = 2;
  L.prog.out_node[0] = root;
  L.prog.out_node[1] = lo_node;
  auto out = std::make_shared<DeviceBuffer>(e->numel());
  auto lo = std::make_shared<DeviceBuffer>(e->numel());
  launch_program(L, e->shape, {out->ptr, lo->ptr});
  out->tf32_lo = std::move(lo);
  e->kind = Expr::Leaf;
  e->buf = std::move(out);
  e->a.reset();
  e->b.reset();
  e->nodes_ub = 0;
  e->leaves_ub = 1;
}

// Lower several pending nodes of one shape as the outputs of one fused program
// (sibling gradients of a binary op read the same upstream gradient and operands: one
// pass instead of one per output). Falls back to lowering them one by one.
void materialize_group(const std::vector<ExprPtr> &eps) {
  std::vector<ExprPtr> todo;
  for (const ExprPtr &e : eps)
    if (e && e->kind == Expr::Reduce) materialize(e);
  for (const ExprPtr &e : eps)
    if (e && e->kind != Expr::Leaf && e->kind != Expr::Const && e->numel() > 0 &&
        std::find(todo.begin(), todo.end(), e) == todo.end())
      todo.push_back(e);
  bool grouped = todo.size() >= 2 && (int)todo.size() <= FZ_MAX_OUTPUTS;
  for (const ExprPtr &e : todo) grouped = grouped && e->shape == todo[0]->shape;
  if (grouped && try_epilogue(todo, std::vector<bool>(todo.size(), false))) return;
  if (grouped) {
    Lowering L;
    std::vector<int> roots;
    for (const ExprPtr &e : todo) roots.push_back(L.visit(e.get()));
    for (int r : roots) grouped = grouped && r >= 0;
    if (grouped && !L.overflow) {
      L.prog.num_leaves = (int32_t)L.leaves.size();
      L.prog.num_outputs = (int32_t)todo.size();
      std::vector<std::shared_ptr<DeviceBuffer>> bufs;
      std::vector<float *> outs;
      for (size_t k = 0; k < todo.size(); ++k) {
        L.prog.out_node[k] = roots[k];
        bufs.push_back(std::make_shared<DeviceBuffer>(todo[k]->numel()));
        outs.push_back(bufs.back()->ptr);
      }
      launch_program(L, todo[0]->shape, outs);
      for (size_t k = 0; k < todo.size(); ++k) {
        Expr *e = todo[k].get();
        e->kind = Expr::Leaf;
        e->buf = bufs[k];
        e->a.reset();
        e->b.reset();
        e->nodes_ub = 0;
        e->leaves_ub = 1;
      }
      return;
    }
  }
  for (const ExprPtr &e : todo) materialize(e);
}

static ExprPtr make_op(Expr::Kind kind, int op, ExprPtr a, ExprPtr b, std::vector<size_t> shape) {
  // reductions are lowered on their own, never inside an elementwise program, and an
  // elementwise op reads a swapaxes view materialised
  if (a && (a->kind == Expr::Reduce || a->kind == Expr::Swap)) materialize(a);
  if (b && (b->kind == Expr::Reduce || b->kind == Expr::Swap)) materialize(b);
  // size policy: keep every pending program within the fused-kernel limits
  auto nodes = [&]() { return 1 + a->nodes_ub + (b ? b->nodes_ub : 0); };
  auto leaves = [&]() { return a->leaves_ub + (b ? b->leaves_ub : 0); };
  while (nodes() > kNodeLimit || leaves() > kLeafLimit) {
    ExprPtr &big = (!b || a->nodes_ub + a->leaves_ub >= b->nodes_ub + b->leaves_ub) ? a : b;
    FB_CHECK(big->kind != Expr::Leaf, "fusion policy: cannot shrink program");
    materialize(big);
  }
  auto e = std::make_shared<Expr>();
  e->kind = kind;
  e->op = op;
  e->nodes_ub = nodes();
  e->leaves_ub = leaves();
  e->gemm_below = a->gemm_below || (b && b->gemm_below);
  e->a = std::move(a);
  e->b = std::move(b);
  e->shape = std::move(shape);
  if (!g_fusion) materialize(e);
  return e;
}

// ---------------------------------------------------------------- RawTensor
// The calling thread's upload stream; null from the library means it could not be
// created, and the copy must not fall back to another stream silently.
static void *upload_stream() {
  void *up = fz_upload_stream();
  if (!up) fz_check(FZ_ERR_CUDA, "fz_upload_stream");
  return up;
}

void RawTensor::set_contiguous_strides() {
  strides_.assign(shape_.size(), 0);
  int64_t r = 1;
  for (long i = (long)shape_.size() - 1; i >= 0; --i) {
    strides_[i] = r;
    r *= (int64_t)shape_[i];
  }
}

RawTensor::RawTensor(std::vector<size_t> shape, const float *data, DType dtype, Device device)
    : shape_(std::move(shape)), dtype_(dtype), device_(device) {
  FB_CHECK(!shape_.empty(), "Tensor: empty shape");
  bind_device(device_);
  set_contiguous_strides();
  size_t n = 1;
  for (auto s : shape_) n *= s;
  // Uploaded on the thread's upload stream, beside whatever the compute stream is
  // still running (the next step's inputs while the current step computes). The host
  // waits for the copy itself, so `data` may be reused or freed on return as with a
  // synchronous copy; compute work submitted afterwards is ordered after it.
  void *up = upload_stream();
  auto buf = std::make_shared<DeviceBuffer>(n, up);
  if (n) {
    fz_check(fz_memcpy_h2d(buf->ptr, data, n * sizeof(float), up), "fz_memcpy_h2d");
    fz_check(fz_stream_sync(up), "fz_stream_sync(upload)");
    fz_check(fz_stream_wait(nullptr, up), "fz_stream_wait");
  }
  storage_ = std::make_shared<Storage>(make_leaf(std::move(buf), shape_));
}

RawTensor::RawTensor(std::vector<size_t> shape, const std::vector<float> &data, DType dtype,
                     Device device)
    : RawTensor(shape, data.data(), dtype, device) {
  size_t n = 1;
  for (auto s : shape_) n *= s;
  FB_CHECK(data.size() == n, "Tensor: data size != product(shape)");
}

RawTensor::RawTensor(std::vector<size_t> shape, DType dtype, Device device)
    : shape_(std::move(shape)), dtype_(dtype), device_(device) {
  FB_CHECK(!shape_.empty(), "Tensor: empty shape");
  bind_device(device_);
  set_contiguous_strides();
  storage_ = std::make_shared<Storage>(make_const(0.0f, shape_));
}

RawTensor::RawTensor(ExprPtr e, DType dtype, Device device)
    : shape_(e->shape), dtype_(dtype), device_(device) {
  set_contiguous_strides();
  storage_ = std::make_shared<Storage>(std::move(e));
}

RawTensor RawTensor::full(const std::vector<size_t> &shape, float value, DType dtype, Device device) {
  FB_CHECK(!shape.empty(), "Tensor: empty shape");
  bind_device(device);
  return RawTensor(make_const(value, shape), dtype, device);
}

float *RawTensor::data() const {
  FB_CHECK(storage_, "uninitialised tensor");
  return storage_->data();
}

void RawTensor::to_host(float *dst) const {
  size_t n = size();
  if (!n) return;
  float *p = data();
  // read back on the upload stream once the compute stream has produced the value;
  // for a value flushed earlier that point is its ready event, so the copy does not
  // wait for compute work submitted since (the next step)
  void *up = upload_stream();
  const DeviceBuffer *b = expr()->buf.get();
  if (b && b->ready) fz_check(fz_stream_wait_event(up, b->ready), "fz_stream_wait_event");
  else fz_check(fz_stream_wait(up, nullptr), "fz_stream_wait");
  fz_check(fz_memcpy_d2h(dst, p, n * sizeof(float), up), "fz_memcpy_d2h");
}

std::vector<float> RawTensor::to_host() const {
  std::vector<float> v(size());
  to_host(v.data());
  return v;
}

void RawTensor::set_values(const float *src, size_t n) {
  FB_CHECK(storage_, "uninitialised tensor");
  auto buf = std::make_shared<DeviceBuffer>(n);
  if (n) fz_check(fz_memcpy_h2d(buf->ptr, src, n * sizeof(float), nullptr), "fz_memcpy_h2d");
  storage_->expr = make_leaf(std::move(buf), shape_);
}

RawTensor RawTensor::from_buffer(std::shared_ptr<DeviceBuffer> buf, std::vector<size_t> shape,
                                 DType dtype, Device device) {
  size_t n = 1;
  for (size_t d : shape) n *= d;
  FB_CHECK(buf && buf->numel == n, "from_buffer: size mismatch");
  return RawTensor(make_leaf(std::move(buf), std::move(shape)), dtype, device);
}

void RawTensor::rebind_buffer(std::shared_ptr<DeviceBuffer> buf) {
  FB_CHECK(storage_, "uninitialised tensor");
  FB_CHECK(buf && buf->numel == size(), "rebind_buffer: size mismatch");
  storage_->expr = make_leaf(std::move(buf), shape_);
}

void RawTensor::clear() {
  if (!storage_ || storage_->numel() == 0) return;
  storage_->expr = make_const(0.0f, storage_->expr->shape);
}

void RawTensor::assign(const RawTensor &other) {
  if (!storage_) {
    *this = other;
    return;
  }
  storage_->expr = other.storage_->expr;
}

RawTensor &RawTensor::operator-=(const RawTensor &other) {
  math::sub_inplace(*this, other);
  return *this;
}

RawTensor RawTensor::operator+(const RawTensor &o) const { return math::binary(FZ_ADD, *this, o); }
RawTensor RawTensor::operator-(const RawTensor &o) const { return math::binary(FZ_SUB, *this, o); }
RawTensor RawTensor::operator*(const RawTensor &o) const { return math::binary(FZ_MUL, *this, o); }
RawTensor RawTensor::operator/(const RawTensor &o) const { return math::binary(FZ_DIV, *this, o); }
RawTensor RawTensor::operator>(const RawTensor &o) const { return math::binary(FZ_GT, *this, o); }
RawTensor RawTensor::operator>=(const RawTensor &o) const { return math::binary(FZ_GT, *this, o); }
RawTensor RawTensor::maximum(const RawTensor &o) const { return math::binary(FZ_MAXIMUM, *this, o); }
RawTensor RawTensor::pow(const RawTensor &o) const { return math::binary(FZ_POW, *this, o); }
// Scalar overloads build a [1] tensor (RawTensor.hpp:30-34, 159-185).
RawTensor RawTensor::operator+(float s) const { return *this + scalar(s, dtype_, device_); }
RawTensor RawTensor::operator-(float s) const { return *this - scalar(s, dtype_, device_); }
RawTensor RawTensor::operator*(float s) const { return *this * scalar(s, dtype_, device_); }
RawTensor RawTensor::operator/(float s) const { return *this / scalar(s, dtype_, device_); }
RawTensor RawTensor::operator>=(float s) const { return *this >= scalar(s, dtype_, device_); }
RawTensor RawTensor::maximum(float s) const { return maximum(scalar(s, dtype_, device_)); }
RawTensor RawTensor::pow(float s) const { return pow(scalar(s, dtype_, device_)); }
RawTensor RawTensor::sqrt() const { return math::unary(FZ_SQRT, *this); }
RawTensor RawTensor::log() const { return math::unary(FZ_LOG, *this); }
RawTensor RawTensor::exp() const { return math::unary(FZ_EXP, *this); }
RawTensor RawTensor::sum(size_t axis, bool keepdim) const { return math::reduce(FZ_RSUM, *this, axis, keepdim); }
RawTensor RawTensor::mean(size_t axis, bool keepdim) const { return math::reduce(FZ_RMEAN, *this, axis, keepdim); }
RawTensor RawTensor::max(size_t axis, bool keepdim) const { return math::reduce(FZ_RMAX, *this, axis, keepdim); }
RawTensor RawTensor::matmul(const RawTensor &o) const { return math::matmul(*this, o); }
RawTensor RawTensor::swapaxes(int a1, int a2) const { return math::swapaxes(*this, a1, a2); }

std::string RawTensor::shape_str() const {
  std::ostringstream os;
  os << '(';
  for (size_t i = 0; i < shape_.size(); ++i) os << shape_[i] << (i + 1 < shape_.size() ? "," : "");
  os << ')';
  return os.str();
}

// operator<< format of the reference (RawTensor.hpp:243-262).
std::string RawTensor::repr() const {
  std::ostringstream os;
  if (!storage_) return "Tensor(unsupported storage type)";
  auto v = to_host();
  os << "Tensor(";
  for (size_t i = 0; i < v.size(); ++i) {
    os << v[i];
    if (i + 1 < v.size()) os << ", ";
  }
  os << ")" << std::endl;
  return os.str();
}

RawTensor zeros_like(const RawTensor &t) { return RawTensor::full(t.shape(), 0.0f, DType::FLOAT32, t.device()); }
RawTensor ones_like(const RawTensor &t) { return RawTensor::full(t.shape(), 1.0f, DType::FLOAT32, t.device()); }

// ---------------------------------------------------------------- ops
namespace math {

static void check_pair(const RawTensor &x, const RawTensor &y) {
  FB_CHECK(x.is_initialised(), "binary ewise: LHS uninitialised");
  FB_CHECK(y.is_initialised(), "binary ewise: RHS uninitialised");
  FB_CHECK(x.dtype() == y.dtype(), "dtypes do not match!");
  FB_CHECK(x.device() == y.device(), "devices do not match!");
}

// fusion::math::{add,sub,mul,div,pow,maximum,greater} (ops/Ewise.hpp:17-55,
// ops/Comparison.hpp:17-40). Equal shapes take the contiguous fast path
// (PlanMeta.hpp:100-108); otherwise the broadcast walk, whose innermost loop
// hands the operands to the scalar kernel exchanged when only the left operand
// has stride 0 in the last dim (SimdTraits.hpp:30-31 and peers), so op(b, a).
RawTensor binary(int op, const RawTensor &x, const RawTensor &y) {
  check_pair(x, y);
  const bool same = x.shape() == y.shape();
  std::vector<size_t> out = same ? x.shape() : broadcast_shape(x.shape(), y.shape());
  const bool swap = !same && x.shape().back() == 1 && out.back() > 1;
  ExprPtr a = x.expr(), b = y.expr();
  if (swap) std::swap(a, b);
  return RawTensor(make_op(Expr::Binary, op, std::move(a), std::move(b), out), x.dtype(), x.device());
}

RawTensor unary(int op, const RawTensor &x) {
  FB_CHECK(x.is_initialised(), "unary ewise: uninitialised tensor");
  return RawTensor(make_op(Expr::Unary, op, x.expr(), nullptr, x.shape()), x.dtype(), x.device());
}

// fusion::math::sum/mean (ops/Reduce.hpp:18-36) via make_reduction_meta
// (PlanMeta.hpp:148-182): axis == (size_t)-1 with keepdim == false is the global
// reduction to shape [1]; otherwise one axis, removed or kept as 1.
// fusion::math::sum/mean/max over one axis (ops/Reduce.hpp:18-36). The result is a
// pending Reduce node; when x is itself a pending reduction of the same op and keepdim
// over the axes next to `axis`, the two join into one reduction over the merged axes
// of x's input (x.sum(3, True).sum(2, True) reads its input once, as rows of
// shape[2]*shape[3]). mean joins as one sum divided by the merged length. Joined
// sums add in a different order than the chained calls: the result stays within the
// reductions' error bound, not bit for bit.
RawTensor reduce(int op, const RawTensor &x, size_t axis, bool keepdim) {
  FB_CHECK(x.is_initialised(), "reduction: uninitialised tensor");
  const auto &s = x.shape();
  std::vector<size_t> oshape;
  if (axis == kGlobalReduceAxis && !keepdim) {
    oshape = {1};
  } else {
    if (axis >= s.size()) throw std::runtime_error("axis out of range");
    for (size_t d = 0; d < s.size(); ++d) {
      if (d == axis) {
        if (keepdim) oshape.push_back(1);
      } else {
        oshape.push_back(s[d]);
      }
    }
    if (oshape.empty()) oshape = {1};
  }
  ExprPtr xe = x.expr();
  auto e = std::make_shared<Expr>();
  e->kind = Expr::Reduce;
  e->op = op;
  e->shape = oshape;
  e->red_keep = keepdim;
  if (axis == kGlobalReduceAxis && !keepdim) {
    if (xe->kind == Expr::Reduce) materialize(xe);
    e->a = xe;
    e->red_lo = 0;
    e->red_hi = (int)s.size() - 1;
    return RawTensor(e, x.dtype(), x.device());
  }
  // join a pending reduction of the same op and keepdim over the adjacent axes
  if (xe->kind == Expr::Reduce && xe->op == op && xe->red_keep == keepdim &&
      !(xe->red_lo == 0 && xe->red_hi + 1 == (int)xe->a->shape.size() && !keepdim)) {
    // axis of xe's input that `axis` names
    const int removed = keepdim ? 0 : xe->red_hi - xe->red_lo + 1;
    const int ax = (int)axis < xe->red_lo ? (int)axis : (int)axis + removed;
    if (ax == xe->red_lo - 1 || ax == xe->red_hi + 1) {
      e->a = xe->a;
      e->red_lo = ax < xe->red_lo ? ax : xe->red_lo;
      e->red_hi = ax > xe->red_hi ? ax : xe->red_hi;
      return RawTensor(e, x.dtype(), x.device());
    }
  }
  if (xe->kind == Expr::Reduce) materialize(xe);
  e->a = xe;
  e->red_lo = e->red_hi = (int)axis;
  return RawTensor(e, x.dtype(), x.device());
}

// The TF32 remainder plane of a materialised GEMM operand, split on first use and
// kept with its buffer; null (the GEMM splits it itself) when caching is off or the
// GEMM could not read it directly (pitch or batch stride not a multiple of 4 floats,
// broadcast batch).
static bool split_plane_usable(int64_t ld, int64_t stride, size_t batch) {
  return split_cache_enabled() && ld % 4 == 0 && stride % 4 == 0 && !(batch > 1 && stride == 0);
}

static const float *tf32_lo_plane(const RawTensor &t, int64_t ld, int64_t stride, size_t batch) {
  if (!split_plane_usable(ld, stride, batch)) return nullptr;
  ExprPtr e = t.expr();
  if (!e || e->kind != Expr::Leaf || !e->buf) return nullptr;
  DeviceBuffer &b = *e->buf;
  if (!b.tf32_lo) {
    auto lo = std::make_shared<DeviceBuffer>(b.numel);
    fz_check(fz_tf32_lo(lo->ptr, b.ptr, (int64_t)b.numel, nullptr), "fz_tf32_lo");
    b.tf32_lo = std::move(lo);
    ++g_lo_splits;
  }
  return b.tf32_lo->ptr;
}

// An operand that is a swapaxes(-1, -2) view is read as its source in the other
// layout (K-major <-> MN-major): W.T in `x @ W.T` is W read K-major, and the
// backward's `g @ swapaxes(W.T)` is W read MN-major; nothing is transposed.
static RawTensor gemm_operand(const RawTensor &T, bool &trans) {
  const ExprPtr &e = T.expr();
  if (e->kind != Expr::Swap) return T;
  trans = !trans;
  return RawTensor(e->a, T.dtype(), T.device());
}

RawTensor matmul(const RawTensor &A0, const RawTensor &B0, bool transA, bool transB) {
  FB_CHECK(A0.is_initialised(), "matmul: A uninitialised");
  FB_CHECK(B0.is_initialised(), "matmul: B uninitialised");
  FB_CHECK(A0.dtype() == B0.dtype(), "matmul: dtype mismatch");
  FB_CHECK(A0.device() == B0.device(), "matmul: device mismatch");
  const RawTensor A = gemm_operand(A0, transA), B = gemm_operand(B0, transB);
  const auto &as = A.shape(), &bs = B.shape();
  if (as.size() < 2 || bs.size() < 2) throw std::runtime_error("matmul: expected rank >= 2");
  const size_t ar = as.size(), br = bs.size();
  const size_t M = transA ? as[ar - 1] : as[ar - 2], Ka = transA ? as[ar - 2] : as[ar - 1];
  const size_t Kb = transB ? bs[br - 1] : bs[br - 2], N = transB ? bs[br - 2] : bs[br - 1];
  if (Ka != Kb) throw std::runtime_error("matmul: inner dimension mismatch");
  if (ar != br) throw std::runtime_error("matmul: batch rank mismatch (implement broadcasting/padding)");
  std::vector<size_t> oshape;
  size_t batch = 1, ba = 1, bb = 1;
  for (size_t d = 0; d + 2 < ar; ++d) {
    size_t o = as[d] == bs[d] ? as[d] : (as[d] == 1 ? bs[d] : (bs[d] == 1 ? as[d] : 0));
    if (o == 0) throw std::runtime_error("broadcast: dimension mismatch");
    oshape.push_back(o);
    batch *= o;
    ba *= as[d];
    bb *= bs[d];
  }
  FB_CHECK((ba == batch || ba == 1) && (bb == batch || bb == 1),
           "matmul: batch dims broadcast only as a whole");
  oshape.push_back(M);
  oshape.push_back(N);
  const int64_t lda = (int64_t)as[ar - 1], ldb = (int64_t)bs[br - 1];
  const int64_t sA = ba == 1 ? 0 : (int64_t)(as[ar - 1] * as[ar - 2]);
  const int64_t sB = bb == 1 ? 0 : (int64_t)(bs[br - 1] * bs[br - 2]);
  // pending operands are lowered with their remainder planes in the same pass
  if (A.pending() && split_plane_usable(lda, sA, batch)) materialize_with_lo(A.expr());
  if (B.pending() && split_plane_usable(ldb, sB, batch)) materialize_with_lo(B.expr());
  auto g = std::make_shared<GemmSpec>();
  g->pa = A.data();
  g->pb = B.data();
  g->la = tf32_lo_plane(A, lda, sA, batch);
  g->lb = tf32_lo_plane(B, ldb, sB, batch);
  g->keep_a = A.expr()->buf;
  g->keep_b = B.expr()->buf;
  if (g->la) g->keep_la = A.expr()->buf->tf32_lo;
  if (g->lb) g->keep_lb = B.expr()->buf->tf32_lo;
  g->batch = (int64_t)batch;
  g->M = (int64_t)M;
  g->N = (int64_t)N;
  g->K = (int64_t)Ka;
  g->lda = lda;
  g->sA = sA;
  g->ldb = ldb;
  g->sB = sB;
  g->transA = transA;
  g->transB = transB;
  auto e = std::make_shared<Expr>();
  e->kind = Expr::Gemm;
  e->shape = oshape;
  e->gemm = std::move(g);
  e->nodes_ub = 0;
  e->leaves_ub = 1;
  e->gemm_below = true;
  // launched where its value is first needed: inside the epilogue of the program that
  // reads it, or as a plain product
  if (!g_gemm_epilogue || batch * M * N == 0) lower_gemm(e.get());
  return RawTensor(std::move(e), A.dtype(), A.device());
}

// The pending product (A B)^T as the pending product B^T A^T: the operands trade
// places and layouts, nothing is transposed. The swapaxes of a weight gradient
// (SwapAxes backward of `W.T`) so lands in W's layout straight from the GEMM.
static ExprPtr transposed_gemm(const Expr &g) {
  const GemmSpec &s = *g.gemm;
  auto t = std::make_shared<GemmSpec>();
  t->batch = s.batch;
  t->M = s.N;
  t->N = s.M;
  t->K = s.K;
  t->pa = s.pb;
  t->la = s.lb;
  t->lda = s.ldb;
  t->sA = s.sB;
  t->transA = !s.transB;
  t->pb = s.pa;
  t->lb = s.la;
  t->ldb = s.lda;
  t->sB = s.sA;
  t->transB = !s.transA;
  t->keep_a = s.keep_b;
  t->keep_la = s.keep_lb;
  t->keep_b = s.keep_a;
  t->keep_lb = s.keep_la;
  auto e = std::make_shared<Expr>();
  e->kind = Expr::Gemm;
  e->shape = g.shape;
  std::swap(e->shape[e->shape.size() - 1], e->shape[e->shape.size() - 2]);
  e->gemm = std::move(t);
  e->nodes_ub = 0;
  e->leaves_ub = 1;
  e->gemm_below = true;
  return e;
}

// fusion::math::linalg::swapaxes (ops/Linalg.hpp:109-128) has copy semantics: rank < 2
// or equal axes give an unchanged copy, other axes a transposed copy. A swap of the
// last two axes (Nova's `.T`, _tensor.py:91-98) is kept as a view (Expr::Swap) that
// the consumer resolves: a GEMM reads the source in the other layout, a swapaxes of a
// view gives back the source, a pending product becomes the transposed product, and
// any other reader materialises it. Values are never shared with later in-place
// writes: those rebind the source's Storage to a new Expr, and the view keeps the old.
RawTensor swapaxes(const RawTensor &x, int a1, int a2) {
  FB_CHECK(x.is_initialised(), "swapaxes: uninitialised tensor");
  const int nd = (int)x.rank();
  if (nd < 2) return RawTensor(x.expr(), x.dtype(), x.device());
  auto norm = [&](int a) {
    int r = a < 0 ? a + nd : a;
    if (r < 0 || r >= nd) throw std::out_of_range("axis out of range");
    return r;
  };
  const int n1 = norm(a1), n2 = norm(a2);
  if (n1 == n2) return RawTensor(x.expr(), x.dtype(), x.device());
  std::vector<size_t> oshape = x.shape();
  std::swap(oshape[n1], oshape[n2]);
  const ExprPtr &xe = x.expr();
  if (g_swap_views && std::min(n1, n2) == nd - 2 && std::max(n1, n2) == nd - 1) {
    if (xe->kind == Expr::Swap) return RawTensor(xe->a, x.dtype(), x.device());
    if (xe->kind == Expr::Gemm) return RawTensor(transposed_gemm(*xe), x.dtype(), x.device());
    auto e = std::make_shared<Expr>();
    e->kind = Expr::Swap;
    e->shape = oshape;
    e->a = xe;
    e->nodes_ub = 0;
    e->leaves_ub = 1;
    return RawTensor(std::move(e), x.dtype(), x.device());
  }
  std::vector<int64_t> shp(x.shape().begin(), x.shape().end());
  const float *in = x.data();
  auto buf = std::make_shared<DeviceBuffer>(x.size());
  fz_check(fz_swapaxes(buf->ptr, in, shp.data(), nd, n1, n2, nullptr), "fz_swapaxes");
  return RawTensor(make_leaf(std::move(buf), oshape), x.dtype(), x.device());
}

// When y is pending and its first n values are the slice at index 0 of its leading
// dims (the [U] bias minus row 0 of a [B, U] gradient), lower just that slice into
// a buffer instead of all of y; null otherwise (read y itself).
static std::shared_ptr<DeviceBuffer> prefix_values(const RawTensor &y, size_t n) {
  if (!y.pending() || y.size() <= n || y.expr()->kind == Expr::Reduce) return nullptr;
  const auto &ys = y.shape();
  size_t tail = 1;
  for (size_t k = ys.size(); k-- > 0;) {
    tail *= ys[k];
    if (tail == n) return materialize_prefix(y.expr(), k);
    if (tail > n) break;
  }
  return nullptr;
}

// fusion::math::sub_inplace (ops/Ewise.hpp:69-83): x[i] -= y[i] for i < x.size,
// reading y flat whatever its shape. Implemented by rebinding x's storage to the
// new value, so pending readers of the old value are unaffected.
void sub_inplace(RawTensor &x, const RawTensor &y) {
  FB_CHECK(x.is_initialised() && y.is_initialised(), "sub_inplace: uninitialised tensor");
  if (x.shape() == y.shape()) {
    // lowered now, as one fused program with y's pending ops: an updated value (a
    // parameter) is read again and again, and left pending it would be inlined into
    // every reader, growing by one term with every update. A value whose previous
    // one was split for a GEMM (a weight) gets its TF32 remainder plane from the same
    // program, so the next GEMM reading it needs no split pass.
    const ExprPtr &old = x.expr();
    const bool split = split_cache_enabled() && old->kind == Expr::Leaf && old->buf && old->buf->tf32_lo;
    x.storage()->expr = make_op(Expr::Binary, FZ_SUB, x.expr(), y.expr(), x.shape());
    if (split) materialize_with_lo(x.storage()->expr);
    else materialize(x.storage()->expr);
    return;
  }
  const size_t n = x.size();
  FB_CHECK(y.size() >= n, "sub_inplace: right-hand side has fewer elements than the tensor");
  const float *px = x.data();
  // Only y's first n values are read.
  std::shared_ptr<DeviceBuffer> prefix = prefix_values(y, n);
  const float *py = prefix ? prefix->ptr : y.data();
  auto buf = std::make_shared<DeviceBuffer>(n);
  fz_check(fz_ewise_binary_contig(FZ_SUB, (int64_t)n, buf->ptr, px, py, nullptr),
           "fz_ewise_binary_contig");
  x.storage()->expr = make_leaf(std::move(buf), x.shape());
}

RawTensor dropout(const RawTensor &x, float rate, float keep, uint64_t seed, uint64_t offset) {
  FB_CHECK(x.is_initialised(), "dropout: uninitialised tensor");
  FB_CHECK(rate >= 0.0f && rate < 1.0f, "dropout: rate must be in [0, 1)");
  const float *px = x.data();
  auto buf = std::make_shared<DeviceBuffer>(x.size());
  fz_check(fz_philox_dropout(buf->ptr, px, (int64_t)x.size(), rate, keep, seed, offset, nullptr),
           "fz_philox_dropout");
  return RawTensor(make_leaf(std::move(buf), x.shape()), x.dtype(), x.device());
}

RawTensor philox_uniform(const std::vector<size_t> &shape, float lo, float hi, uint64_t seed,
                         uint64_t offset, DType dtype, Device device) {
  FB_CHECK(!shape.empty(), "Tensor: empty shape");
  bind_device(device);
  size_t n = 1;
  for (size_t d : shape) n *= d;
  auto buf = std::make_shared<DeviceBuffer>(n);
  fz_check(fz_philox_uniform(buf->ptr, (int64_t)n, seed, offset, lo, hi, nullptr), "fz_philox_uniform");
  return RawTensor(make_leaf(std::move(buf), shape), dtype, device);
}

// The first n values of x (flat order) as a tensor of `shape` (n elements).
RawTensor flat_prefix(const RawTensor &x, size_t n, const std::vector<size_t> &shape) {
  FB_CHECK(x.is_initialised(), "flat_prefix: uninitialised tensor");
  FB_CHECK(x.size() >= n, "flat_prefix: the tensor has fewer than n elements");
  size_t m = 1;
  for (size_t d : shape) m *= d;
  FB_CHECK(m == n, "flat_prefix: shape does not hold n elements");
  std::shared_ptr<DeviceBuffer> buf = prefix_values(x, n);
  if (!buf) {
    buf = std::make_shared<DeviceBuffer>(n);
    if (n) fz_check(fz_memcpy_d2d(buf->ptr, x.data(), n * sizeof(float), nullptr), "fz_memcpy_d2d");
  }
  return RawTensor(make_leaf(std::move(buf), shape), x.dtype(), x.device());
}

}  // namespace math
}  // namespace fusion_b200
