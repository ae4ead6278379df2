// Runtime plumbing of the sm_100a backend: errors, devices, per-thread streams,
// the stream-ordered memory pool, copies, fills and device timers.
#include <atomic>
#include <cstring>
#include <mutex>
#include <thread>
#include <chrono>
#include <string>
#include <unordered_map>
#include <vector>

#include "fz_common.cuh"

namespace fz {

static thread_local std::string g_err;
static std::atomic<int64_t> g_launches{0};

void set_error(const std::string &msg) { g_err = msg; }
void clear_error() { g_err.clear(); }

int fail(int code, const std::string &msg) {
  g_err = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char *what, const char *file, int line) {
  char buf[512];
  snprintf(buf, sizeof(buf), "CUDA error %d (%s) in %s at %s:%d", (int)e,
           cudaGetErrorString(e), what, file, line);
  g_err = buf;
  return e == cudaErrorMemoryAllocation ? FZ_ERR_OOM : FZ_ERR_CUDA;
}

void note_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

constexpr int kMaxDevices = 16;

struct DeviceState {
  std::once_flag once;
  int sms = 0;
  int ok = 0;
};
static DeviceState g_dev[kMaxDevices];
static thread_local cudaStream_t t_stream[kMaxDevices] = {};

static int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

// One-time per-device setup: check the architecture and keep freed pool blocks
// cached (release threshold = max) so steady-state allocation never calls the driver.
static int setup_device(int d) {
  DeviceState &st = g_dev[d];
  int rc = FZ_OK;
  std::call_once(st.once, [&]() {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, d) != cudaSuccess) {
      rc = fail(FZ_ERR_CUDA, "cudaGetDeviceProperties failed");
      return;
    }
    if (p.major != 10) {
      rc = fail(FZ_ERR_UNSUPPORTED,
                "fusion_b200 needs a compute capability 10.x (B200, sm_100a) device; got " +
                    std::to_string(p.major) + "." + std::to_string(p.minor));
      return;
    }
    st.sms = p.multiProcessorCount;
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, d) == cudaSuccess) {
      uint64_t thr = UINT64_MAX;
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
    }
    st.ok = 1;
  });
  if (rc != FZ_OK) return rc;
  if (!st.ok) return fail(FZ_ERR_UNSUPPORTED, "device setup failed earlier");
  return FZ_OK;
}

cudaStream_t resolve(void *stream) {
  if (stream) return (cudaStream_t)stream;
  int d = current_device();
  if (!t_stream[d]) {
    setup_device(d);
    cudaStreamCreateWithFlags(&t_stream[d], cudaStreamNonBlocking);
  }
  return t_stream[d];
}

static int *g_err_word[kMaxDevices] = {};
static std::mutex g_err_mu;

int device_error_word(int **word) {
  int d = current_device();
  std::lock_guard<std::mutex> lk(g_err_mu);
  if (!g_err_word[d]) {
    int *p = nullptr;
    cudaError_t e = cudaMalloc(&p, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(error word)", __FILE__, __LINE__);
    e = cudaMemset(p, 0, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(error word)", __FILE__, __LINE__);
    g_err_word[d] = p;
  }
  *word = g_err_word[d];
  return FZ_OK;
}

int num_sms() {
  int d = current_device();
  if (!g_dev[d].sms) setup_device(d);
  return g_dev[d].sms ? g_dev[d].sms : 148;
}

}  // namespace fz

using namespace fz;

namespace {
__global__ void fill_kernel(float *__restrict__ dst, float v, int64_t n) {
  pdl_wait();
  int64_t nv = n >> 2;
  float4 q = make_float4(v, v, v, v);
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  float4 *d4 = reinterpret_cast<float4 *>(dst);
  for (int64_t j = i; j < nv; j += stride) __stcs(d4 + j, q);
  for (int64_t j = (nv << 2) + i; j < n; j += stride) dst[j] = v;
}

__global__ void sub_inplace_kernel(float *__restrict__ x, const float *__restrict__ y, int64_t n) {
  pdl_wait();
  int64_t nv = n >> 2;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  float4 *x4 = reinterpret_cast<float4 *>(x);
  const float4 *y4 = reinterpret_cast<const float4 *>(y);
  for (int64_t j = i; j < nv; j += stride) {
    float4 a = x4[j], b = __ldcs(y4 + j);
    a.x = __fsub_rn(a.x, b.x);
    a.y = __fsub_rn(a.y, b.y);
    a.z = __fsub_rn(a.z, b.z);
    a.w = __fsub_rn(a.w, b.w);
    x4[j] = a;
  }
  for (int64_t j = (nv << 2) + i; j < n; j += stride) x[j] = __fsub_rn(x[j], y[j]);
}

struct Timer {
  cudaEvent_t a = nullptr, b = nullptr;
};
}  // namespace

extern "C" {

const char *fz_last_error(void) { return g_err.c_str(); }
int fz_version(void) { return 1; }

int fz_device_count(int *count) {
  FZ_REQUIRE(count, "fz_device_count: null pointer");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    *count = 0;
    cudaGetLastError();
    return cuda_fail(e, "cudaGetDeviceCount", __FILE__, __LINE__);
  }
  int good = 0;
  for (int d = 0; d < n; ++d) {
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d);
    if (major == 10) ++good;
  }
  *count = good;
  return FZ_OK;
}

int fz_set_device(int device) {
  int n = 0;
  FZ_CUDA(cudaGetDeviceCount(&n));
  FZ_REQUIRE(device >= 0 && device < n && device < kMaxDevices, "Invalid device index");
  FZ_CUDA(cudaSetDevice(device));
  int rc = setup_device(device);
  if (rc) return rc;
  resolve(nullptr);
  return FZ_OK;
}

int fz_get_device(int *device) {
  FZ_REQUIRE(device, "fz_get_device: null pointer");
  FZ_CUDA(cudaGetDevice(device));
  return FZ_OK;
}

void *fz_default_stream(void) { return (void *)resolve(nullptr); }

int fz_stream_sync(void *stream) {
  FZ_CUDA(cudaStreamSynchronize(resolve(stream)));
  return FZ_OK;
}

int fz_event_record(void **event, void *stream) {
  FZ_REQUIRE(event, "fz_event_record: null pointer");
  cudaEvent_t e = nullptr;
  FZ_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  cudaError_t rc = cudaEventRecord(e, resolve(stream));
  if (rc != cudaSuccess) {
    cudaEventDestroy(e);
    return cuda_fail(rc, "fz_event_record", __FILE__, __LINE__);
  }
  *event = (void *)e;
  return FZ_OK;
}

int fz_stream_wait_event(void *waiter, void *event) {
  FZ_REQUIRE(event, "fz_stream_wait_event: null event");
  FZ_CUDA(cudaStreamWaitEvent(resolve(waiter), (cudaEvent_t)event, 0));
  return FZ_OK;
}

int fz_event_destroy(void *event) {
  if (event) FZ_CUDA(cudaEventDestroy((cudaEvent_t)event));
  return FZ_OK;
}

int release_stream_blocks(cudaStream_t s);  // block cache, below

static thread_local cudaStream_t t_upload[kMaxDevices] = {};

void *fz_upload_stream(void) {
  int d = current_device();
  if (!t_upload[d]) {
    setup_device(d);
    cudaStream_t s = nullptr;
    cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
      // reported through fz_last_error; the caller gets null and must not copy
      cuda_fail(e, "creating the upload stream", __FILE__, __LINE__);
      return nullptr;
    }
    t_upload[d] = s;
  }
  return (void *)t_upload[d];
}

int fz_stream_create(void **stream) {
  FZ_REQUIRE(stream, "fz_stream_create: null pointer");
  cudaStream_t s = nullptr;
  FZ_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  *stream = (void *)s;
  return FZ_OK;
}

int fz_stream_destroy(void *stream) {
  if (!stream) return FZ_OK;
  cudaStream_t s = (cudaStream_t)stream;
  // The block cache keys free lists by stream handle, and a later fz_stream_create
  // may return the same handle: hand this stream's cached blocks back to the pool now
  // (each free ordered after the stream's work, and after its free point when it was
  // freed elsewhere), and re-home its live blocks to the thread's compute stream, so
  // their eventual free does not file them under a handle that no longer exists.
  int rc = release_stream_blocks(s);
  if (rc) return rc;
  FZ_CUDA(cudaStreamDestroy(s));
  return FZ_OK;
}

int fz_stream_wait(void *waiter, void *signaler) {
  cudaStream_t w = resolve(waiter), g = resolve(signaler);
  if (w == g) return FZ_OK;
  cudaEvent_t e = nullptr;
  FZ_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  cudaError_t rc = cudaEventRecord(e, g);
  if (rc == cudaSuccess) rc = cudaStreamWaitEvent(w, e, 0);
  cudaEventDestroy(e);  // released once the wait no longer needs it
  if (rc != cudaSuccess) return cuda_fail(rc, "fz_stream_wait", __FILE__, __LINE__);
  return FZ_OK;
}

namespace {
void CUDART_CB host_pause(void *arg) {
  double *secs = static_cast<double *>(arg);
  std::this_thread::sleep_for(std::chrono::duration<double>(*secs));
  delete secs;
}
}  // namespace

int fz_stream_delay(void *stream, double seconds) {
  FZ_REQUIRE(seconds >= 0.0 && seconds <= 60.0, "fz_stream_delay: seconds must be in [0, 60]");
  double *arg = new double(seconds);
  cudaError_t e = cudaLaunchHostFunc(resolve(stream), host_pause, arg);
  if (e != cudaSuccess) {
    delete arg;
    return cuda_fail(e, "fz_stream_delay", __FILE__, __LINE__);
  }
  return FZ_OK;
}

int fz_device_sync(void) {
  FZ_CUDA(cudaDeviceSynchronize());
  return FZ_OK;
}

// Block cache in front of the stream-ordered pool, in the role of Fusion's
// PoolAllocator (fusion/src/Fusion/alloc/BFCPoolAllocator.cpp:59-111). A freed
// block goes back onto the free list of the stream it was allocated on (its home),
// keyed by size class; the next allocation of that class on that stream takes it
// back without calling the driver. Work on one stream runs in order, so a block
// freed on its home stream is reused with no event; a block freed on another stream
// (an upload buffer allocated on the upload stream and last read by the compute
// stream) carries an event recorded at the free, which the home stream waits on
// before reusing it. A training step allocates the same sizes every step, so in the
// steady state no allocation reaches cudaMallocAsync; that call can block the host
// for tens to hundreds of milliseconds in the driver while it maps pool pages,
// long enough to leave the GPU idle behind it.
namespace {
struct CachedBlock {
  void *ptr;
  cudaEvent_t ready;  // recorded where the block was freed, if not on its home stream
};
struct FreeLists {
  int device = 0;
  std::unordered_map<size_t, std::vector<CachedBlock>> by_size;
};
struct LiveBlock {
  size_t size;
  int device;
  cudaStream_t home;
};
std::mutex g_cache_mu;
std::unordered_map<void *, LiveBlock> g_live;
std::unordered_map<cudaStream_t, FreeLists> g_free;
size_t g_live_bytes[fz::kMaxDevices] = {};
size_t g_cached_bytes[fz::kMaxDevices] = {};

// Size classes: 512 B granules below 1 MiB, 2 MiB granules above (the driver
// pool maps in 2 MiB pages, so a larger granule wastes nothing there).
size_t size_class(size_t bytes) {
  const size_t small = 512, large = (size_t)2 << 20;
  return bytes < ((size_t)1 << 20) ? (bytes + small - 1) / small * small
                                   : (bytes + large - 1) / large * large;
}

// Give every cached block of `device` back to the driver pool and trim the pool.
// The device is synchronised first, so the blocks can be freed on any stream.
int release_cached(int device) {
  std::vector<void *> blocks;
  std::vector<cudaEvent_t> events;
  {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    for (auto it = g_free.begin(); it != g_free.end();) {
      if (it->second.device != device) {
        ++it;
        continue;
      }
      for (auto &kv : it->second.by_size)
        for (const CachedBlock &c : kv.second) {
          blocks.push_back(c.ptr);
          if (c.ready) events.push_back(c.ready);
        }
      it = g_free.erase(it);
    }
    g_cached_bytes[device] = 0;
  }
  int prev = 0;
  FZ_CUDA(cudaGetDevice(&prev));
  FZ_CUDA(cudaSetDevice(device));
  cudaStream_t s = fz::resolve(nullptr);
  cudaError_t e = cudaDeviceSynchronize();
  for (cudaEvent_t ev : events) cudaEventDestroy(ev);
  for (void *p : blocks)
    if (e == cudaSuccess) e = cudaFreeAsync(p, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaMemPool_t pool;
  if (e == cudaSuccess) e = cudaDeviceGetDefaultMemPool(&pool, device);
  if (e == cudaSuccess) e = cudaMemPoolTrimTo(pool, 0);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return fz::cuda_fail(e, "releasing cached device blocks", __FILE__, __LINE__);
  return FZ_OK;
}
}  // namespace

// The block cache's part of fz_stream_destroy (see there).
int release_stream_blocks(cudaStream_t s) {
  std::vector<CachedBlock> blocks;
  {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    auto it = g_free.find(s);
    if (it != g_free.end()) {
      for (auto &kv : it->second.by_size) {
        for (const CachedBlock &c : kv.second) blocks.push_back(c);
        g_cached_bytes[it->second.device] -= kv.first * kv.second.size();
      }
      g_free.erase(it);
    }
    bool have = false;
    for (const auto &kv : g_live) have = have || kv.second.home == s;
    if (have) {
      const cudaStream_t home = resolve(nullptr);
      for (auto &kv : g_live)
        if (kv.second.home == s) kv.second.home = home;
    }
  }
  cudaError_t e = cudaSuccess;
  for (const CachedBlock &c : blocks) {
    if (c.ready && e == cudaSuccess) e = cudaStreamWaitEvent(s, c.ready, 0);
    if (e == cudaSuccess) e = cudaFreeAsync(c.ptr, s);
    if (c.ready) cudaEventDestroy(c.ready);
  }
  if (e != cudaSuccess) return cuda_fail(e, "fz_stream_destroy: returning cached blocks", __FILE__, __LINE__);
  return FZ_OK;
}

int fz_malloc(void **ptr, size_t bytes, void *stream) {
  FZ_REQUIRE(ptr, "fz_malloc: null pointer");
  *ptr = nullptr;
  if (bytes == 0) return FZ_OK;
  // size classes are multiples of 512 B, so every block can feed 128-bit and TMA accesses
  const size_t sz = size_class(bytes);
  cudaStream_t s = resolve(stream);
  int d = current_device();
  {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    auto it = g_free.find(s);
    if (it != g_free.end()) {
      auto jt = it->second.by_size.find(sz);
      if (jt != it->second.by_size.end() && !jt->second.empty()) {
        // A block freed on its home stream is reusable at once; one freed on another
        // stream only when that stream has passed the free. Waiting for a free point that
        // lies ahead (the upload of step i+2 taking the buffer step i+1 is still reading)
        // would serialise the streams, so such blocks are skipped and, if none is ready,
        // new memory is taken: a rotation of buffers forms instead.
        auto &v = jt->second;
        for (size_t k = v.size(); k-- > 0;) {
          const CachedBlock c = v[k];
          if (c.ready) {
            const cudaError_t q = cudaEventQuery(c.ready);
            if (q == cudaErrorNotReady) {
              // make sure the answer is not left as the thread's last error, where the
              // next launch check would read it
              if (cudaPeekAtLastError() == cudaErrorNotReady) cudaGetLastError();
              continue;
            }
            if (q != cudaSuccess) return cuda_fail(q, "cudaEventQuery(cached block)", __FILE__, __LINE__);
          }
          v.erase(v.begin() + (long)k);
          if (c.ready) cudaEventDestroy(c.ready);
          g_cached_bytes[d] -= sz;
          g_live.emplace(c.ptr, LiveBlock{sz, d, s});
          g_live_bytes[d] += sz;
          *ptr = c.ptr;
          return FZ_OK;
        }
      }
    }
  }
  cudaError_t e = cudaMallocAsync(ptr, sz, s);
  if (e == cudaErrorMemoryAllocation) {
    // the pool is full: hand the cached blocks back and try once more
    cudaGetLastError();
    int rc = release_cached(d);
    if (rc) return rc;
    e = cudaMallocAsync(ptr, sz, s);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    *ptr = nullptr;
    return fail(FZ_ERR_OOM, "device allocation of " + std::to_string(bytes) +
                                " bytes failed: " + cudaGetErrorString(e));
  }
  std::lock_guard<std::mutex> lk(g_cache_mu);
  g_live.emplace(*ptr, LiveBlock{sz, d, s});
  g_live_bytes[d] += sz;
  return FZ_OK;
}

int fz_free(void *ptr, void *stream) {
  if (!ptr) return FZ_OK;
  cudaStream_t s = resolve(stream);
  std::lock_guard<std::mutex> lk(g_cache_mu);
  auto it = g_live.find(ptr);
  FZ_REQUIRE(it != g_live.end(), "fz_free: pointer was not returned by fz_malloc or was freed already");
  const LiveBlock b = it->second;
  cudaEvent_t ready = nullptr;
  if (s != b.home) {  // freed where it was last used, not where it lives
    cudaError_t e = cudaEventCreateWithFlags(&ready, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(ready, s);
    if (e != cudaSuccess) return cuda_fail(e, "fz_free: recording the free point", __FILE__, __LINE__);
  }
  g_live.erase(it);
  g_live_bytes[b.device] -= b.size;
  FreeLists &fl = g_free[b.home];
  fl.device = b.device;
  fl.by_size[b.size].push_back(CachedBlock{ptr, ready});
  g_cached_bytes[b.device] += b.size;
  return FZ_OK;
}

int fz_pool_release(void) {
  int d = 0;
  FZ_CUDA(cudaGetDevice(&d));
  FZ_REQUIRE(d < kMaxDevices, "fz_pool_release: device index out of range");
  return release_cached(d);
}

int fz_pool_cached(size_t *bytes) {
  FZ_REQUIRE(bytes, "fz_pool_cached: null pointer");
  int d = 0;
  FZ_CUDA(cudaGetDevice(&d));
  std::lock_guard<std::mutex> lk(g_cache_mu);
  *bytes = d < kMaxDevices ? g_cached_bytes[d] : 0;
  return FZ_OK;
}

int fz_pool_stats(size_t *reserved, size_t *used) {
  int d = 0;
  FZ_CUDA(cudaGetDevice(&d));
  cudaMemPool_t pool;
  FZ_CUDA(cudaDeviceGetDefaultMemPool(&pool, d));
  uint64_t r = 0;
  FZ_CUDA(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemCurrent, &r));
  if (reserved) *reserved = r;
  if (used) {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    *used = d < kMaxDevices ? g_live_bytes[d] : 0;
  }
  return FZ_OK;
}

int fz_memcpy_h2d(void *dst, const void *src, size_t bytes, void *stream) {
  if (!bytes) return FZ_OK;
  FZ_REQUIRE(dst && src, "fz_memcpy_h2d: null pointer");
  FZ_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, resolve(stream)));
  return FZ_OK;
}

int fz_memcpy_d2h(void *dst, const void *src, size_t bytes, void *stream) {
  if (!bytes) return FZ_OK;
  FZ_REQUIRE(dst && src, "fz_memcpy_d2h: null pointer");
  cudaStream_t s = resolve(stream);
  FZ_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s));
  FZ_CUDA(cudaStreamSynchronize(s));
  return FZ_OK;
}

int fz_memcpy_d2d(void *dst, const void *src, size_t bytes, void *stream) {
  if (!bytes) return FZ_OK;
  FZ_REQUIRE(dst && src, "fz_memcpy_d2d: null pointer");
  FZ_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, resolve(stream)));
  return FZ_OK;
}

int fz_fill_f32(float *dst, float value, int64_t n, void *stream) {
  if (n <= 0) return FZ_OK;
  FZ_REQUIRE(dst, "fz_fill_f32: null pointer");
  FZ_REQUIRE(((uintptr_t)dst & 15) == 0, "fz_fill_f32: destination must be 16-byte aligned");
  unsigned grid = grid_for((n + 3) / 4, 256 * 4, 8);
  FZ_CUDA(fz::launch_pdl(fill_kernel, dim3(grid), dim3(256), 0, resolve(stream), dst, value, n));
  FZ_CHECK_LAUNCH();
  return FZ_OK;
}

int fz_sub_inplace(float *x, const float *y, int64_t n, void *stream) {
  if (n <= 0) return FZ_OK;
  FZ_REQUIRE(x && y, "fz_sub_inplace: null pointer");
  FZ_REQUIRE((((uintptr_t)x | (uintptr_t)y) & 15) == 0,
             "fz_sub_inplace: operands must be 16-byte aligned");
  unsigned grid = grid_for((n + 3) / 4, 256 * 2, 8);
  FZ_CUDA(fz::launch_pdl(sub_inplace_kernel, dim3(grid), dim3(256), 0, resolve(stream), x, y, n));
  FZ_CHECK_LAUNCH();
  return FZ_OK;
}

int fz_host_alloc(void **ptr, size_t bytes) {
  FZ_REQUIRE(ptr, "fz_host_alloc: null pointer");
  FZ_CUDA(cudaMallocHost(ptr, bytes ? bytes : 1));
  return FZ_OK;
}

int fz_host_free(void *ptr) {
  if (ptr) FZ_CUDA(cudaFreeHost(ptr));
  return FZ_OK;
}

int fz_timer_create(void **timer) {
  FZ_REQUIRE(timer, "fz_timer_create: null pointer");
  Timer *t = new Timer;
  FZ_CUDA(cudaEventCreate(&t->a));
  FZ_CUDA(cudaEventCreate(&t->b));
  *timer = t;
  return FZ_OK;
}

int fz_timer_start(void *timer, void *stream) {
  FZ_REQUIRE(timer, "fz_timer_start: null timer");
  FZ_CUDA(cudaEventRecord(static_cast<Timer *>(timer)->a, resolve(stream)));
  return FZ_OK;
}

int fz_timer_stop(void *timer, void *stream) {
  FZ_REQUIRE(timer, "fz_timer_stop: null timer");
  FZ_CUDA(cudaEventRecord(static_cast<Timer *>(timer)->b, resolve(stream)));
  return FZ_OK;
}

int fz_timer_elapsed_ms(void *timer, float *ms) {
  FZ_REQUIRE(timer && ms, "fz_timer_elapsed_ms: null pointer");
  Timer *t = static_cast<Timer *>(timer);
  FZ_CUDA(cudaEventSynchronize(t->b));
  FZ_CUDA(cudaEventElapsedTime(ms, t->a, t->b));
  return FZ_OK;
}

int fz_timer_destroy(void *timer) {
  if (!timer) return FZ_OK;
  Timer *t = static_cast<Timer *>(timer);
  cudaEventDestroy(t->a);
  cudaEventDestroy(t->b);
  delete t;
  return FZ_OK;
}

int64_t fz_launch_count(void) { return g_launches.load(); }

int fz_kernel_status(void) {
  int *w = nullptr;
  int rc = device_error_word(&w);
  if (rc) return rc;
  int v = 0;
  FZ_CUDA(cudaDeviceSynchronize());
  FZ_CUDA(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost));
  if (v) {
    FZ_CUDA(cudaMemset(w, 0, sizeof(int)));
    return fail(FZ_ERR_TIMEOUT, "a kernel's bounded wait expired (code " + std::to_string(v) + ")");
  }
  return FZ_OK;
}

}  // extern "C"
