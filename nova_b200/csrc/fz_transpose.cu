// Materialised swapaxes for sm_100a.
//
// A contiguous tensor with axes a1 < a2 exchanged is viewed as
//   in  [P, A, Q, B, R]  ->  out [P, B, Q, A, R]
// with A = shape[a1], B = shape[a2]. When R == 1 (the last axis takes part, as in
// the W.T / x.T of a Linear layer) each of the P*Q [A, B] planes is transposed
// through shared memory so both the reads and the writes are coalesced rows:
// 64 x 64 tiles with 16-byte accesses and overlapped tiles when the extents and
// pitches allow it, else 32 x 32 tiles addressed by a 3D grid. When R > 1 whole
// R-runs move together and a vectorised gather copy is used.
#include "fz_common.cuh"

namespace {

constexpr int kTile = 32;
constexpr int kRows = 8;

// One 32 x 32 tile of one [A, B] plane per CTA: blockIdx.x walks the tiles along B,
// blockIdx.y those along A and blockIdx.z the P*Q planes, each dimension grid-
// striding when it exceeds the launch limits, so no index is ever divided.
__global__ void __launch_bounds__(kTile *kRows) transpose_tiles(const float *__restrict__ in,
                                                               float *__restrict__ out, int64_t P,
                                                               int64_t Q, int64_t A, int64_t B) {
  pdl_wait();
  __shared__ float tile[kTile][kTile + 1];
  const int64_t ta = (A + kTile - 1) / kTile, tb = (B + kTile - 1) / kTile;
  const int tx = threadIdx.x % kTile, ty = threadIdx.x / kTile;
  for (int64_t pq = blockIdx.z; pq < P * Q; pq += gridDim.z) {
    const int64_t p = pq / Q, q = pq - p * Q;  // once per plane
    const float *src = in + p * A * Q * B + q * B;  // element (i, j) at i*Q*B + j
    float *dst = out + p * B * Q * A + q * A;       // element (j, i) at j*Q*A + i
    for (int64_t ib = blockIdx.y; ib < ta; ib += gridDim.y) {
      for (int64_t jb = blockIdx.x; jb < tb; jb += gridDim.x) {
        const int64_t i0 = ib * kTile, j0 = jb * kTile;
#pragma unroll
        for (int k = 0; k < kTile / kRows; ++k) {
          const int64_t i = i0 + ty + k * kRows, j = j0 + tx;
          if (i < A && j < B) tile[ty + k * kRows][tx] = src[i * Q * B + j];
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kTile / kRows; ++k) {
          const int64_t j = j0 + ty + k * kRows, i = i0 + tx;
          if (j < B && i < A) dst[j * Q * A + i] = tile[tx][ty + k * kRows];
        }
        __syncthreads();
      }
    }
  }
}

// Fast path for R == 1 when A, B and both row pitches (Q*B, Q*A) are multiples of 4
// floats and the bases are 16-byte aligned: 64 x 64 tiles moved with float4 loads
// and stores through a 64 x 65 shared tile (two-way bank conflicts on either side),
// by persistent CTAs that issue the next tile's loads before writing the current
// tile out, so global reads and writes overlap. Tile indices are decoded with IDX
// (32-bit when the tile count allows) once per tile.
constexpr int kBig = 64;

struct TileIdx {
  const float *src;
  float *dst;
  int64_t i0, j0;
};

template <typename IDX>
__device__ __forceinline__ TileIdx decode_tile64(IDX t, IDX per_plane, IDX tb, IDX Q,
                                                 const float *in, float *out, int64_t A,
                                                 int64_t B) {
  const IDX pq = t / per_plane, rem = t - pq * per_plane;
  const IDX ib = rem / tb, jb = rem - ib * tb;
  const IDX p = pq / Q, q = pq - p * Q;
  TileIdx r;
  r.src = in + (int64_t)p * A * (int64_t)Q * B + (int64_t)q * B;
  r.dst = out + (int64_t)p * B * (int64_t)Q * A + (int64_t)q * A;
  r.i0 = (int64_t)ib * kBig;
  r.j0 = (int64_t)jb * kBig;
  return r;
}

template <typename IDX>
__global__ void __launch_bounds__(256, 4) transpose64_kernel(const float *__restrict__ in,
                                                          float *__restrict__ out, int64_t P,
                                                          int64_t Q, int64_t A, int64_t B) {
  pdl_wait();
  __shared__ float tile[kBig][kBig + 1];
  const IDX ta = (IDX)((A + kBig - 1) / kBig), tb = (IDX)((B + kBig - 1) / kBig);
  const IDX per_plane = ta * tb;
  const IDX total = (IDX)(P * Q) * per_plane;
  const int64_t in_ld = Q * B, out_ld = Q * A;  // row pitches in floats
  const int hi = threadIdx.x >> 4, lo = threadIdx.x & 15;
  IDX t = blockIdx.x;
  if (t >= total) return;
  TileIdx cur = decode_tile64<IDX>(t, per_plane, tb, (IDX)Q, in, out, A, B);
  float4 v[4];
  auto load = [&](const TileIdx &x) {
    const int64_t j = x.j0 + lo * 4;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int64_t i = x.i0 + hi + 16 * m;
      if (i < A && j < B) v[m] = *reinterpret_cast<const float4 *>(x.src + i * in_ld + j);
    }
  };
  load(cur);
  while (true) {
    __syncthreads();  // the previous tile's store phase has read the shared tile
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      float *row = &tile[hi + 16 * m][lo * 4];
      row[0] = v[m].x;
      row[1] = v[m].y;
      row[2] = v[m].z;
      row[3] = v[m].w;
    }
    __syncthreads();
    const IDX tn = t + (IDX)gridDim.x;
    const bool more = tn < total;
    TileIdx nxt = cur;
    if (more) {
      nxt = decode_tile64<IDX>(tn, per_plane, tb, (IDX)Q, in, out, A, B);
      load(nxt);
    }
    const int64_t i = cur.i0 + lo * 4;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int c = hi + 16 * m;
      const int64_t j = cur.j0 + c;
      if (j < B && i < A)
        *reinterpret_cast<float4 *>(cur.dst + j * out_ld + i) =
            make_float4(tile[lo * 4][c], tile[lo * 4 + 1][c], tile[lo * 4 + 2][c],
                        tile[lo * 4 + 3][c]);
    }
    if (!more) break;
    t = tn;
    cur = nxt;
  }
}

// R > 1: out[p, j, q, i, r] = in[p, i, q, j, r]; each thread copies V floats of a run.
template <int V>
__global__ void __launch_bounds__(256) transpose_runs(const float *__restrict__ in,
                                                     float *__restrict__ out, int64_t P, int64_t A,
                                                     int64_t Q, int64_t B, int64_t R) {
  pdl_wait();
  const int64_t rv = R / V;
  const int64_t total = P * B * Q * A * rv;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = (t % rv) * V;
    int64_t rest = t / rv;
    int64_t i = rest % A;
    rest /= A;
    int64_t q = rest % Q;
    rest /= Q;
    int64_t j = rest % B;
    int64_t p = rest / B;
    const float *s = in + (((p * A + i) * Q + q) * B + j) * R + r;
    float *d = out + (((p * B + j) * Q + q) * A + i) * R + r;
    if constexpr (V == 4)
      *reinterpret_cast<float4 *>(d) = *reinterpret_cast<const float4 *>(s);
    else
      *d = *s;
  }
}

}  // namespace

extern "C" int fz_swapaxes(float *out, const float *in, const int64_t *shape, int ndim, int a1,
                           int a2, void *stream) {
  FZ_REQUIRE(shape && ndim >= 0 && ndim <= 32, "fz_swapaxes: bad shape");
  int64_t total = 1;
  for (int d = 0; d < ndim; ++d) {
    FZ_REQUIRE(shape[d] >= 0, "fz_swapaxes: negative extent");
    total *= shape[d];
  }
  if (total == 0) return FZ_OK;
  FZ_REQUIRE(out && in, "fz_swapaxes: null pointer");
  cudaStream_t s = fz::resolve(stream);
  if (ndim < 2) return fz_memcpy_d2d(out, in, total * sizeof(float), s);
  if (a1 < 0) a1 += ndim;
  if (a2 < 0) a2 += ndim;
  FZ_REQUIRE(a1 >= 0 && a1 < ndim && a2 >= 0 && a2 < ndim, "fz_swapaxes: axis out of range");
  if (a1 == a2) return fz_memcpy_d2d(out, in, total * sizeof(float), s);
  if (a1 > a2) {
    int t = a1;
    a1 = a2;
    a2 = t;
  }
  int64_t P = 1, Q = 1, R = 1, A = shape[a1], B = shape[a2];
  for (int d = 0; d < a1; ++d) P *= shape[d];
  for (int d = a1 + 1; d < a2; ++d) Q *= shape[d];
  for (int d = a2 + 1; d < ndim; ++d) R *= shape[d];
  if (A == 1 || B == 1) {
    if (Q == 1 || (A == 1 && B == 1)) return fz_memcpy_d2d(out, in, total * sizeof(float), s);
  }
  const bool fast = R == 1 && A % 4 == 0 && B % 4 == 0 && (Q * A) % 4 == 0 && (Q * B) % 4 == 0 &&
                    (((uintptr_t)in | (uintptr_t)out) & 15) == 0;
  if (fast) {
    const int64_t tiles = P * Q * ((A + kBig - 1) / kBig) * ((B + kBig - 1) / kBig);
    // one wave of persistent CTAs (four fit on an SM at this kernel's register count)
    const unsigned grid = (unsigned)(tiles < (int64_t)fz::num_sms() * 4 ? tiles : fz::num_sms() * 4);
    if (tiles < ((int64_t)1 << 31) && P * Q < ((int64_t)1 << 31))
      FZ_CUDA(fz::launch_pdl(transpose64_kernel<uint32_t>, dim3(grid), dim3(256), 0, s, in, out, P, Q, A, B));
    else
      FZ_CUDA(fz::launch_pdl(transpose64_kernel<int64_t>, dim3(grid), dim3(256), 0, s, in, out, P, Q, A, B));
  } else if (R == 1) {
    const int64_t ta = (A + kTile - 1) / kTile, tb = (B + kTile - 1) / kTile;
    dim3 grid((unsigned)(tb < 0x7fffffff ? tb : 0x7fffffff), (unsigned)(ta < 65535 ? ta : 65535),
              (unsigned)(P * Q < 65535 ? P * Q : 65535));
    FZ_CUDA(fz::launch_pdl(transpose_tiles, grid, dim3(kTile * kRows), 0, s, in, out, P, Q, A, B));
  } else {
    bool v4 = R % 4 == 0 && (((uintptr_t)in | (uintptr_t)out) & 15) == 0;
    int64_t items = total / (v4 ? 4 : 1);
    unsigned grid = fz::grid_for(items, 256, 8, 4);
    if (v4) FZ_CUDA(fz::launch_pdl(transpose_runs<4>, dim3(grid), dim3(256), 0, s, in, out, P, A, Q, B, R));
    else FZ_CUDA(fz::launch_pdl(transpose_runs<1>, dim3(grid), dim3(256), 0, s, in, out, P, A, Q, B, R));
  }
  FZ_CHECK_LAUNCH();
  return FZ_OK;
}
