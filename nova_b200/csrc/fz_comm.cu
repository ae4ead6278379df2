// NCCL collectives for the data-parallel MLP step (one process per GPU).
//
// The gradient exchange is an in-place fp32 all-reduce over NVLink 5 / NVSwitch
// (NCCL picks NVLS in-switch reduction when the fabric offers it), followed by a
// scale to turn the sum into a mean. A host-side watchdog (fz_comm_wait) bounds
// the wait for the communication stream and aborts the communicator on expiry,
// so a rank that died or never joined ends the step with FZ_ERR_TIMEOUT.
#include <nccl.h>

#include <chrono>
#include <cmath>
#include <cstring>
#include <thread>

#include "fz_common.cuh"

namespace {

struct Comm {
  ncclComm_t comm = nullptr;
  int world = 1, rank = 0;
  bool aborted = false;
};

int nccl_fail(ncclResult_t r, const char *what) {
  return fz::fail(FZ_ERR_NCCL, std::string(what) + " failed: " + ncclGetErrorString(r));
}

__global__ void scale_kernel(float *__restrict__ x, float s, int64_t n) {
  int64_t nv = n >> 2;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  float4 *x4 = reinterpret_cast<float4 *>(x);
  for (int64_t j = i; j < nv; j += stride) {
    float4 v = x4[j];
    v.x = __fmul_rn(v.x, s);
    v.y = __fmul_rn(v.y, s);
    v.z = __fmul_rn(v.z, s);
    v.w = __fmul_rn(v.w, s);
    x4[j] = v;
  }
  for (int64_t j = (nv << 2) + i; j < n; j += stride) x[j] = __fmul_rn(x[j], s);
}

}  // namespace

extern "C" {

int fz_comm_unique_id(unsigned char id[FZ_UNIQUE_ID_BYTES]) {
  FZ_REQUIRE(id, "fz_comm_unique_id: null pointer");
  static_assert(sizeof(ncclUniqueId) == FZ_UNIQUE_ID_BYTES, "ncclUniqueId size");
  ncclUniqueId uid;
  ncclResult_t r = ncclGetUniqueId(&uid);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  std::memcpy(id, &uid, sizeof(uid));
  return FZ_OK;
}

int fz_comm_init(void **comm, int world, int rank, const unsigned char id[FZ_UNIQUE_ID_BYTES]) {
  FZ_REQUIRE(comm && id, "fz_comm_init: null pointer");
  FZ_REQUIRE(world >= 1 && rank >= 0 && rank < world, "fz_comm_init: bad rank/world");
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  Comm *c = new Comm;
  c->world = world;
  c->rank = rank;
  ncclResult_t r = ncclCommInitRank(&c->comm, world, uid, rank);
  if (r != ncclSuccess) {
    delete c;
    return nccl_fail(r, "ncclCommInitRank");
  }
  *comm = c;
  return FZ_OK;
}

int fz_comm_allreduce(void *comm, const float *send, float *recv, int64_t count, float scale,
                      void *stream) {
  FZ_REQUIRE(comm, "fz_comm_allreduce: null communicator");
  if (count == 0) return FZ_OK;
  FZ_REQUIRE(send && recv && count > 0, "fz_comm_allreduce: bad buffer");
  Comm *c = static_cast<Comm *>(comm);
  FZ_REQUIRE(!c->aborted, "fz_comm_allreduce: communicator was aborted");
  cudaStream_t s = fz::resolve(stream);
  // scale 1 -> sum; scale 1/world -> NCCL's average (no extra kernel, so the call
  // is safe inside an fz_comm_group_start/end group); any other scale -> sum then
  // a scaling pass (not allowed inside a group).
  const bool avg = scale != 1.0f && std::fabs(scale * (float)c->world - 1.0f) < 1e-6f;
  ncclResult_t r = ncclAllReduce(send, recv, (size_t)count, ncclFloat, avg ? ncclAvg : ncclSum,
                                 c->comm, s);
  if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce");
  if (scale != 1.0f && !avg) {
    FZ_REQUIRE(((uintptr_t)recv & 15) == 0, "fz_comm_allreduce: buffer must be 16-byte aligned");
    unsigned grid = fz::grid_for((count + 3) / 4, 256 * 2, 8);
    scale_kernel<<<grid, 256, 0, s>>>(recv, scale, count);
    FZ_CHECK_LAUNCH();
  }
  return FZ_OK;
}

int fz_comm_group_start(void) {
  ncclResult_t r = ncclGroupStart();
  return r == ncclSuccess ? FZ_OK : nccl_fail(r, "ncclGroupStart");
}

int fz_comm_group_end(void) {
  ncclResult_t r = ncclGroupEnd();
  return r == ncclSuccess ? FZ_OK : nccl_fail(r, "ncclGroupEnd");
}

int fz_comm_broadcast(void *comm, float *buf, int64_t count, int root, void *stream) {
  FZ_REQUIRE(comm, "fz_comm_broadcast: null communicator");
  if (count == 0) return FZ_OK;
  Comm *c = static_cast<Comm *>(comm);
  FZ_REQUIRE(!c->aborted, "fz_comm_broadcast: communicator was aborted");
  FZ_REQUIRE(root >= 0 && root < c->world, "fz_comm_broadcast: bad root");
  ncclResult_t r =
      ncclBroadcast(buf, buf, (size_t)count, ncclFloat, root, c->comm, fz::resolve(stream));
  if (r != ncclSuccess) return nccl_fail(r, "ncclBroadcast");
  return FZ_OK;
}

int fz_comm_wait(void *comm, void *stream, double timeout_s) {
  FZ_REQUIRE(comm, "fz_comm_wait: null communicator");
  Comm *c = static_cast<Comm *>(comm);
  cudaStream_t s = fz::resolve(stream);
  auto t0 = std::chrono::steady_clock::now();
  while (true) {
    cudaError_t e = cudaStreamQuery(s);
    if (e == cudaSuccess) return FZ_OK;
    if (e != cudaErrorNotReady) return fz::cuda_fail(e, "cudaStreamQuery", __FILE__, __LINE__);
    ncclResult_t async_err = ncclSuccess;
    ncclCommGetAsyncError(c->comm, &async_err);
    if (async_err != ncclSuccess && async_err != ncclInProgress) {
      ncclCommAbort(c->comm);
      c->aborted = true;
      return nccl_fail(async_err, "collective (async error)");
    }
    double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > timeout_s) {
      ncclCommAbort(c->comm);
      c->aborted = true;
      return fz::fail(FZ_ERR_TIMEOUT, "collective did not complete within " +
                                          std::to_string(timeout_s) + " s; communicator aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

int fz_comm_destroy(void *comm) {
  if (!comm) return FZ_OK;
  Comm *c = static_cast<Comm *>(comm);
  if (!c->aborted && c->comm) ncclCommDestroy(c->comm);
  delete c;
  return FZ_OK;
}

}  // extern "C"
