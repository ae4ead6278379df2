// Host-memory test double of the C ABI in include/fusion_b200.h.
//
// TEST INFRASTRUCTURE ONLY. It lets the CPU test suite run the C++ host layer
// (nova_b200/host: the fusion-IR lowering, the autodiff engine, Fusion's op
// semantics and quirks) without a GPU: tests/hostfake/build_fake.py links a copy
// of the pybind module against this library in tests/hostfake/_build/. The
// product library nova_b200/libfusion_b200.so never contains or loads it, and it
// is never a fallback: it exists so host-logic bugs surface on CPU before a GPU
// run. "Device" pointers here are host pointers; every op is a scalar loop with
// the IEEE fp32 semantics the sm_100a kernels implement.
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <set>
#include <string>
#include <vector>

#include "fusion_b200.h"

namespace {
thread_local std::string g_err;
int64_t g_launches = 0;
std::set<std::string> g_programs;

int fail(int code, const std::string &m) {
  g_err = m;
  return code;
}

float binop(int op, float a, float b) {
  switch (op) {
    case FZ_ADD: return a + b;
    case FZ_SUB: return a - b;
    case FZ_MUL: return a * b;
    case FZ_DIV: return a / b;
    case FZ_POW: return b == 2.0f ? a * a : std::pow(a, b);
    case FZ_MAXIMUM: return a > b ? a : b;
    case FZ_GT: return a > b ? 1.0f : 0.0f;
    case FZ_GE: return a >= b ? 1.0f : 0.0f;
  }
  return 0.0f;
}

static float tf32_lo1(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  u &= 0xffffe000u;
  float h;
  std::memcpy(&h, &u, 4);
  float r = x - h;
  std::memcpy(&u, &r, 4);
  if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0xfffu + ((u >> 13) & 1u)) & 0xffffe000u;
  std::memcpy(&r, &u, 4);
  return r;
}

float unop(int op, float a) {
  switch (op) {
    case FZ_EXP: return std::exp(a);
    case FZ_LOG: return std::log(a);
    case FZ_SQRT: return std::sqrt(a);
    case FZ_TF32_LO: return tf32_lo1(a);
    default: return a;
  }
}

// Visit every index of a plan; fn(offsets in elements of each operand).
template <class Fn>
void walk(const fz_ewise_plan &p, Fn fn) {
  int64_t total = 1;
  for (int d = 0; d < p.ndim; ++d) total *= p.size[d];
  std::vector<int64_t> idx(p.ndim > 0 ? p.ndim : 1, 0);
  std::vector<int64_t> off(p.num_operands);
  for (int64_t i = 0; i < total; ++i) {
    for (int k = 0; k < p.num_operands; ++k) {
      int64_t o = 0;
      for (int d = 0; d < p.ndim; ++d) o += idx[d] * p.stride_bytes[k][d] / 4;
      off[k] = o;
    }
    fn(off.data());
    for (int d = p.ndim - 1; d >= 0; --d) {
      if (++idx[d] < p.size[d]) break;
      idx[d] = 0;
    }
  }
}
}  // namespace

extern "C" {

const char *fz_last_error(void) { return g_err.c_str(); }
int fz_version(void) { return 1; }
int fz_device_count(int *c) { *c = 1; return FZ_OK; }
int fz_set_device(int d) { return d == 0 ? FZ_OK : fail(FZ_ERR_INVALID, "Invalid device index"); }
int fz_get_device(int *d) { *d = 0; return FZ_OK; }
void *fz_default_stream(void) { static int s; return &s; }
int fz_stream_sync(void *) { return FZ_OK; }
int fz_device_sync(void) { return FZ_OK; }
// live allocations, so pool_used_bytes reports what the host keeps
std::map<void *, size_t> g_live;
size_t g_live_bytes = 0;
int fz_malloc(void **p, size_t bytes, void *) {
  *p = nullptr;
  if (!bytes) return FZ_OK;
  *p = std::aligned_alloc(256, (bytes + 255) & ~(size_t)255);
  if (!*p) return fail(FZ_ERR_OOM, "host allocation failed");
  g_live[*p] = bytes;
  g_live_bytes += bytes;
  return FZ_OK;
}
int fz_free(void *p, void *) {
  auto it = g_live.find(p);
  if (it != g_live.end()) {
    g_live_bytes -= it->second;
    g_live.erase(it);
  }
  std::free(p);
  return FZ_OK;
}
int fz_pool_release(void) { return FZ_OK; }
int fz_pool_stats(size_t *r, size_t *u) { if (r) *r = g_live_bytes; if (u) *u = g_live_bytes; return FZ_OK; }
int fz_memcpy_h2d(void *d, const void *s, size_t n, void *) { if (n) std::memcpy(d, s, n); return FZ_OK; }
int fz_memcpy_d2h(void *d, const void *s, size_t n, void *) { if (n) std::memcpy(d, s, n); return FZ_OK; }
int fz_memcpy_d2d(void *d, const void *s, size_t n, void *) { if (n) std::memmove(d, s, n); return FZ_OK; }
int fz_fill_f32(float *d, float v, int64_t n, void *) { for (int64_t i = 0; i < n; ++i) d[i] = v; ++g_launches; return FZ_OK; }
int fz_host_alloc(void **p, size_t b) { return fz_malloc(p, b ? b : 1, nullptr); }
int fz_host_free(void *p) { std::free(p); return FZ_OK; }
int fz_timer_create(void **t) { *t = std::malloc(1); return FZ_OK; }
int fz_timer_start(void *, void *) { return FZ_OK; }
int fz_timer_stop(void *, void *) { return FZ_OK; }
int fz_timer_elapsed_ms(void *, float *ms) { *ms = 0.0f; return FZ_OK; }
int fz_timer_destroy(void *t) { std::free(t); return FZ_OK; }
int64_t fz_launch_count(void) { return g_launches; }
int fz_kernel_status(void) { return FZ_OK; }

int fz_ewise_binary(int op, const fz_ewise_plan *p, float *out, const float *a, const float *b, void *) {
  if (p->num_operands != 3) return fail(FZ_ERR_INVALID, "elementwise plan: wrong operand count");
  walk(*p, [&](const int64_t *o) { out[o[0]] = binop(op, a[o[1]], b[o[2]]); });
  ++g_launches;
  return FZ_OK;
}
int fz_ewise_binary_contig(int op, int64_t n, float *out, const float *a, const float *b, void *) {
  for (int64_t i = 0; i < n; ++i) out[i] = binop(op, a[i], b[i]);
  ++g_launches;
  return FZ_OK;
}
int fz_ewise_unary(int op, const fz_ewise_plan *p, float *out, const float *a, void *) {
  walk(*p, [&](const int64_t *o) { out[o[0]] = unop(op, a[o[1]]); });
  ++g_launches;
  return FZ_OK;
}
int fz_sub_inplace(float *x, const float *y, int64_t n, void *) {
  for (int64_t i = 0; i < n; ++i) x[i] = x[i] - y[i];
  ++g_launches;
  return FZ_OK;
}

int fz_fused_launch(const fz_program *pg, const fz_ewise_plan *p, float *const *outs,
                    const float *const *leaves, void *) {
  if (p->num_operands != pg->num_outputs + pg->num_leaves)
    return fail(FZ_ERR_INVALID, "fz_fused_launch: plan operand count != outputs + leaves");
  g_programs.insert(std::string(reinterpret_cast<const char *>(pg->nodes),
                                sizeof(fz_node) * pg->num_nodes));
  std::vector<float> t(pg->num_nodes);
  walk(*p, [&](const int64_t *o) {
    auto val = [&](int s) { return s >= 0 ? t[s] : leaves[-1 - s][o[pg->num_outputs + (-1 - s)]]; };
    for (int i = 0; i < pg->num_nodes; ++i) {
      const fz_node &n = pg->nodes[i];
      t[i] = n.kind == FZ_NODE_BINARY ? binop(n.op, val(n.src0), val(n.src1))
             : n.kind == FZ_NODE_UNARY ? unop(n.op, val(n.src0)) : n.imm;
    }
    for (int k = 0; k < pg->num_outputs; ++k) outs[k][o[k]] = t[pg->out_node[k]];
  });
  ++g_launches;
  return FZ_OK;
}
int fz_fused_cache_size(void) { return (int)g_programs.size(); }

int fz_reduce(int op, float *out, const float *in, int64_t outer, int64_t len, int64_t inner, void *) {
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t j = 0; j < inner; ++j) {
      const float *q = in + o * len * inner + j;
      float acc = op == FZ_RMAX ? -INFINITY : 0.0f;
      for (int64_t r = 0; r < len; ++r) {
        float v = q[r * inner];
        if (op == FZ_RMAX) {
          if (acc != acc) continue;
          if (v != v || v > acc || (v == 0.0f && acc == 0.0f && !std::signbit(v))) acc = v;
        } else {
          acc += v;
        }
      }
      if (op == FZ_RMEAN) acc = acc / (float)len;
      out[o * inner + j] = acc;
    }
  ++g_launches;
  return FZ_OK;
}

int fz_swapaxes(float *out, const float *in, const int64_t *shape, int nd, int a1, int a2, void *) {
  if (a1 < 0) a1 += nd;
  if (a2 < 0) a2 += nd;
  std::vector<int64_t> os(shape, shape + nd), ist(nd), ost(nd), idx(nd, 0);
  std::swap(os[a1], os[a2]);
  int64_t r = 1, q = 1, total = 1;
  for (int d = nd - 1; d >= 0; --d) {
    ist[d] = r; r *= shape[d];
    ost[d] = q; q *= os[d];
    total *= shape[d];
  }
  for (int64_t i = 0; i < total; ++i) {
    int64_t o = 0;
    for (int d = 0; d < nd; ++d) o += idx[d] * ost[d == a1 ? a2 : d == a2 ? a1 : d];
    out[o] = in[i];
    for (int d = nd - 1; d >= 0; --d) {
      if (++idx[d] < shape[d]) break;
      idx[d] = 0;
    }
  }
  ++g_launches;
  return FZ_OK;
}

int fz_gemm_f32(int64_t batch, int64_t M, int64_t N, int64_t K, const float *A, int64_t lda,
                int64_t sA, int tA, const float *B, int64_t ldb, int64_t sB, int tB, float *C,
                int64_t ldc, int64_t sC, void *) {
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t i = 0; i < M; ++i)
      for (int64_t j = 0; j < N; ++j) {
        double s = 0;
        for (int64_t k = 0; k < K; ++k) {
          float x = tA ? A[b * sA + k * lda + i] : A[b * sA + i * lda + k];
          float y = tB ? B[b * sB + j * ldb + k] : B[b * sB + k * ldb + j];
          s += (double)x * (double)y;
        }
        C[b * sC + i * ldc + j] = (float)s;
      }
  ++g_launches;
  return FZ_OK;
}


int64_t g_epilogue_launches = 0;
int fz_gemm_f32_epilogue(int64_t batch, int64_t M, int64_t N, int64_t K, const float *A,
                         const float *A_lo, int64_t lda, int64_t sA, int tA, const float *B,
                         const float *B_lo, int64_t ldb, int64_t sB, int tB,
                         const struct fz_program *pg, const fz_epi_input *inputs,
                         float *const *outs, int64_t ldc, int64_t sC, void *st) {
  if (!pg || pg->num_leaves < 1 || pg->num_leaves > FZ_MAX_LEAVES || pg->num_outputs > FZ_MAX_OUTPUTS)
    return fail(FZ_ERR_INVALID, "fz_gemm_f32_epilogue: bad program");
  std::vector<float> P((size_t)(batch * M * N));
  int64_t before = g_launches;
  int rc = fz_gemm_f32_split(batch, M, N, K, A, A_lo, lda, sA, tA, B, B_lo, ldb, sB, tB, P.data(), N,
                             M * N, st);
  if (rc) return rc;
  fz_ewise_plan plan{};
  plan.ndim = 3;
  plan.num_operands = pg->num_outputs + pg->num_leaves;
  plan.size[0] = batch;
  plan.size[1] = M;
  plan.size[2] = N;
  auto set = [&](int k, int64_t b, int64_t m, int64_t n) {
    plan.stride_bytes[k][0] = b * 4;
    plan.stride_bytes[k][1] = m * 4;
    plan.stride_bytes[k][2] = n * 4;
  };
  for (int k = 0; k < pg->num_outputs; ++k) set(k, sC, ldc, 1);
  std::vector<const float *> leaves(pg->num_leaves);
  leaves[0] = P.data();
  set(pg->num_outputs, M * N, N, 1);
  for (int k = 1; k < pg->num_leaves; ++k) {
    const fz_epi_input &in = inputs[k - 1];
    if (in.col_stride != 0 && in.col_stride != 1)
      return fail(FZ_ERR_INVALID, "fz_gemm_f32_epilogue: input column stride must be 0 or 1");
    leaves[k] = in.ptr;
    set(pg->num_outputs + k, in.batch_stride, in.row_stride, in.col_stride);
  }
  rc = fz_fused_launch(pg, &plan, outs, leaves.data(), st);
  g_launches = before + 1;  // one kernel on the device
  ++g_epilogue_launches;
  return rc;
}
int fz_gemm_epilogue_compile(const struct fz_program *, const fz_epi_input *, int, int, int, int) {
  return FZ_OK;
}

int fz_stream_create(void **s) { static int token; *s = &token; return FZ_OK; }
void *fz_upload_stream(void) { static int token; return &token; }
int fz_event_record(void **e, void *) { static int token; *e = &token; return FZ_OK; }
int fz_stream_wait_event(void *, void *) { return FZ_OK; }
int fz_event_destroy(void *) { return FZ_OK; }
int fz_stream_destroy(void *) { return FZ_OK; }
int fz_stream_wait(void *, void *) { return FZ_OK; }
int fz_gemm_set_tma_stores(int) { return FZ_OK; }
int fz_gemm_set_tiles(int mode) { return mode >= 0 && mode <= 2 ? FZ_OK : fail(FZ_ERR_INVALID, "fz_gemm_set_tiles: unknown mode"); }

int fz_tf32_lo(float *lo, const float *x, int64_t n, void *) {
  for (int64_t i = 0; i < n; ++i) lo[i] = tf32_lo1(x[i]);
  ++g_launches;
  return FZ_OK;
}

// A supplied lo plane must hold the remainders of the operand's current values:
// a stale plane (the host reusing one after the operand changed) is an error here.
static int check_lo(const float *X, const float *X_lo, int64_t rows, int64_t cols, int64_t ld,
                    int64_t sb, int64_t batch, const char *name) {
  if (!X_lo) return FZ_OK;
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t r = 0; r < rows; ++r)
      for (int64_t c = 0; c < cols; ++c) {
        const int64_t o = b * sb + r * ld + c;
        const float want = tf32_lo1(X[o]);
        if (std::memcmp(&want, &X_lo[o], 4) != 0)
          return fail(FZ_ERR_INVALID, std::string("fz_gemm_f32_split: stale lo plane for ") + name);
      }
  return FZ_OK;
}

int fz_gemm_f32_split(int64_t batch, int64_t M, int64_t N, int64_t K, const float *A,
                      const float *A_lo, int64_t lda, int64_t sA, int tA, const float *B,
                      const float *B_lo, int64_t ldb, int64_t sB, int tB, float *C, int64_t ldc,
                      int64_t sC, void *st) {
  int rc = check_lo(A, A_lo, tA ? K : M, tA ? M : K, lda, sA, sA ? batch : 1, "A");
  if (!rc) rc = check_lo(B, B_lo, tB ? N : K, tB ? K : N, ldb, sB, sB ? batch : 1, "B");
  if (rc) return rc;
  return fz_gemm_f32(batch, M, N, K, A, lda, sA, tA, B, ldb, sB, tB, C, ldc, sC, st);
}

// Collectives. With a transport set (fake_comm_set_transport: a host callback that sums
// a buffer over the ranks of a host process group, e.g. gloo), communicators of more
// than one rank work and fz_comm_allreduce sums through it; otherwise world must be 1.
// Stream time is emulated for the watchdog: fz_stream_delay marks the streams busy for
// that long, and fz_comm_wait with a shorter timeout then aborts the communicator and
// fails as the real one does.
typedef int (*fake_allreduce_fn)(float *buf, int64_t n);
static fake_allreduce_fn g_transport = nullptr;
static double g_busy_s = 0.0;
struct FakeComm {
  int world;
  bool aborted;
};
void fake_comm_set_transport(fake_allreduce_fn fn) { g_transport = fn; }

int fz_stream_delay(void *, double seconds) {
  if (!(seconds >= 0.0 && seconds <= 60.0)) return fail(FZ_ERR_INVALID, "fz_stream_delay: seconds must be in [0, 60]");
  g_busy_s += seconds;
  return FZ_OK;
}
// Philox-4x32-10 (Salmon et al., SC'11), the device generator's stream layout.
static void philox(uint64_t ctr, uint64_t key, uint32_t c[4]) {
  c[0] = (uint32_t)ctr; c[1] = (uint32_t)(ctr >> 32); c[2] = 0; c[3] = 0;
  uint32_t k0 = (uint32_t)key, k1 = (uint32_t)(key >> 32);
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0], p1 = (uint64_t)0xCD9E8D57u * c[2];
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0, n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    c[1] = (uint32_t)p1; c[3] = (uint32_t)p0; c[0] = n0; c[2] = n2;
    k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
  }
}
static float philox_unit(uint64_t seed, uint64_t i) {
  uint32_t c[4];
  philox(i / 4, seed, c);
  return (float)(c[i % 4] >> 8) * 5.9604644775390625e-08f;
}
int fz_philox_uniform(float *out, int64_t n, uint64_t seed, uint64_t offset, float lo, float hi, void *) {
  if (offset % 4 || !(lo < hi)) return fail(FZ_ERR_INVALID, "fz_philox_uniform: bad arguments");
  for (int64_t i = 0; i < n; ++i) {
    float v = std::fmaf(hi - lo, philox_unit(seed, offset + (uint64_t)i), lo);
    out[i] = v >= hi ? std::nextafterf(hi, lo) : v;
  }
  ++g_launches;
  return FZ_OK;
}
int fz_philox_dropout(float *out, const float *x, int64_t n, float rate, float keep, uint64_t seed,
                      uint64_t offset, void *) {
  if (offset % 4 || !(rate >= 0.0f && rate < 1.0f)) return fail(FZ_ERR_INVALID, "fz_philox_dropout: bad arguments");
  for (int64_t i = 0; i < n; ++i) {
    const float m = philox_unit(seed, offset + (uint64_t)i) > rate ? 1.0f : 0.0f;
    out[i] = (x[i] * m) / keep;
  }
  ++g_launches;
  return FZ_OK;
}

int fz_comm_unique_id(unsigned char id[FZ_UNIQUE_ID_BYTES]) { std::memset(id, 0, FZ_UNIQUE_ID_BYTES); return FZ_OK; }
int fz_comm_init(void **c, int world, int, const unsigned char *) {
  if (world != 1 && !g_transport) return fail(FZ_ERR_UNSUPPORTED, "host test double: world must be 1");
  *c = new FakeComm{world, false};
  return FZ_OK;
}
int fz_comm_allreduce(void *comm, const float *s, float *r, int64_t n, float scale, void *) {
  FakeComm *c = static_cast<FakeComm *>(comm);
  if (c->aborted) return fail(FZ_ERR_INVALID, "fz_comm_allreduce: communicator was aborted");
  if (r != s) std::memmove(r, s, sizeof(float) * (size_t)n);
  if (c->world > 1 && g_transport(r, n) != 0) return fail(FZ_ERR_NCCL, "host transport failed");
  for (int64_t i = 0; i < n; ++i) r[i] = r[i] * scale;
  return FZ_OK;
}
int fz_comm_group_start(void) { return FZ_OK; }
int fz_comm_group_end(void) { return FZ_OK; }
int fz_comm_broadcast(void *, float *, int64_t, int, void *) { return FZ_OK; }
int fz_comm_wait(void *comm, void *, double timeout_s) {
  FakeComm *c = static_cast<FakeComm *>(comm);
  const bool late = g_busy_s > timeout_s;
  g_busy_s = 0.0;
  if (late) {
    c->aborted = true;
    return fail(FZ_ERR_TIMEOUT, "collective did not complete within " + std::to_string(timeout_s) +
                                    " s; communicator aborted");
  }
  return FZ_OK;
}
int fz_comm_destroy(void *c) { delete static_cast<FakeComm *>(c); return FZ_OK; }

}  // extern "C"
