// RMSNorm: y = x * rsqrt(mean(x^2) + eps) * w, fp32 math, one rounding.
//
// The row lives in registers between the sum-of-squares pass and the scale
// pass, so x crosses HBM exactly once (read) and y once (write); the weight
// row is re-read from L1/L2.  A row is owned by TPR threads (a warp for short
// rows, up to 1024 threads for long ones) each holding VPT 16-byte vectors;
// partial sums meet through warp shuffles and, for TPR > 32, one shared-memory
// exchange.  The reference uses one block per row with a shared-memory tree
// reduction and reads x twice (aot_kernel/csrc/norm/rmsnorm.cu:111-182).
// Rows whose byte length is not a multiple of 16 take a scalar two-pass
// kernel, as the reference does (rmsnorm.cu:205-209).
#include "common.h"
#include "vec.cuh"

namespace aotk {
namespace {

constexpr int kBlock = 256;

template <typename T, int VPT, int TPR>
__device__ __forceinline__ void load_row(const T* __restrict__ x, int64_t row, int64_t rows,
                                         int cols, int t, uint4 (&v)[VPT]) {
  constexpr int E = Elem<T>::kPerVec;
  const int n_vec = cols / E;
  const bool live = row < rows;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (live ? row : 0) * (int64_t)cols);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = t + i * TPR;
    if (live && idx < n_vec) v[i] = ld_stream(xr + idx);
    else v[i] = make_uint4(0u, 0u, 0u, 0u);
  }
}

// Persistent over row groups: a block owns RPB rows at a time and, before
// reducing them, issues the loads of the group it will handle next, so each
// SM keeps two groups of rows in flight and the grid is a single wave.
template <typename T, int VPT, int TPR>
__global__ void __launch_bounds__(TPR > kBlock ? TPR : kBlock)
    rmsnorm_vec_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y,
                       int64_t rows, int cols, float eps) {
  constexpr int E = Elem<T>::kPerVec;
  constexpr int THREADS = TPR > kBlock ? TPR : kBlock;
  constexpr int RPB = THREADS / TPR;  // rows per block
  constexpr int WPR = TPR / 32;       // warps per row
  // 1024-thread blocks get 64 registers per thread: no room for a second row copy.
  constexpr bool kPrefetch = THREADS < 1024;
  __shared__ float partial[2][RPB][WPR > 1 ? WPR : 1];

  const int sub = threadIdx.x / TPR;  // row slot in this block
  const int t = threadIdx.x % TPR;    // thread index within the row
  const int n_vec = cols / E;
  const int64_t groups = (rows + RPB - 1) / RPB;
  const uint4* wr = reinterpret_cast<const uint4*>(w);

  uint4 cur[VPT];
  int64_t g = blockIdx.x;
  load_row<T, VPT, TPR>(x, g * RPB + sub, rows, cols, t, cur);
  for (int iter = 0; g < groups; g += gridDim.x, ++iter) {
    uint4 nxt[VPT];
    if constexpr (kPrefetch) load_row<T, VPT, TPR>(x, (g + gridDim.x) * RPB + sub, rows, cols, t, nxt);

    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      float f[E];
      Elem<T>::unpack(cur[i], f);
#pragma unroll
      for (int e = 0; e < E; ++e) ss = fmaf(f[e], f[e], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if constexpr (WPR > 1) {
      // Two partial buffers alternate so one barrier per group suffices.
      if ((t & 31) == 0) partial[iter & 1][sub][t / 32] = ss;
      __syncthreads();
      ss = 0.0f;
#pragma unroll
      for (int k = 0; k < WPR; ++k) ss += partial[iter & 1][sub][k];
    }
    const float rstd = rsqrtf(ss / (float)cols + eps);
    const int64_t row = g * RPB + sub;
    if (row < rows) {
      uint4* yr = reinterpret_cast<uint4*>(y + row * (int64_t)cols);
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int idx = t + i * TPR;
        if (idx < n_vec) {
          float f[E], gw[E];
          Elem<T>::unpack(cur[i], f);
          Elem<T>::unpack(ld_cached(wr + idx), gw);
#pragma unroll
          for (int e = 0; e < E; ++e) f[e] = f[e] * rstd * gw[e];
          st_stream(yr + idx, Elem<T>::pack(f));
        }
      }
    }
    if constexpr (kPrefetch) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) cur[i] = nxt[i];
    } else {
      load_row<T, VPT, TPR>(x, (g + gridDim.x) * RPB + sub, rows, cols, t, cur);
    }
  }
}

// Any row length: one block per row, two passes over x (the second mostly hits L2).
template <typename T>
__global__ void __launch_bounds__(kBlock) rmsnorm_scalar_kernel(const T* __restrict__ x,
                                                                const T* __restrict__ w,
                                                                T* __restrict__ y, int64_t cols,
                                                                float eps) {
  __shared__ float partial[kBlock / 32];
  const T* xr = x + (int64_t)blockIdx.x * cols;
  T* yr = y + (int64_t)blockIdx.x * cols;
  float ss = 0.0f;
  for (int64_t c = threadIdx.x; c < cols; c += kBlock) {
    const float f = Elem<T>::to_f(xr[c]);
    ss = fmaf(f, f, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x / 32] = ss;
  __syncthreads();
  ss = 0.0f;
#pragma unroll
  for (int k = 0; k < kBlock / 32; ++k) ss += partial[k];
  const float rstd = rsqrtf(ss / (float)cols + eps);
  for (int64_t c = threadIdx.x; c < cols; c += kBlock) {
    yr[c] = Elem<T>::from_f(Elem<T>::to_f(xr[c]) * rstd * Elem<T>::to_f(w[c]));
  }
}

template <typename T, int VPT, int TPR>
int launch_vec(const T* x, const T* w, T* y, int64_t rows, int cols, float eps, cudaStream_t s) {
  constexpr int THREADS = TPR > kBlock ? TPR : kBlock;
  constexpr int RPB = THREADS / TPR;
  DeviceInfo info;
  if (int st = current_device_info(&info)) return st;
  auto kernel = rmsnorm_vec_kernel<T, VPT, TPR>;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, THREADS, 0) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int64_t groups = (rows + RPB - 1) / RPB;
  const int64_t capacity = (int64_t)per_sm * info.sm_count;
  const int64_t blocks = groups < capacity ? groups : capacity;
  kernel<<<(unsigned)blocks, THREADS, 0, s>>>(x, w, y, rows, cols, eps);
  return check_launch("aotk_rmsnorm_forward");
}

template <typename T>
int launch(const void* xv, const void* wv, void* yv, int64_t rows, int64_t cols, float eps,
           cudaStream_t s) {
  const T* x = static_cast<const T*>(xv);
  const T* w = static_cast<const T*>(wv);
  T* y = static_cast<T*>(yv);
  constexpr int E = Elem<T>::kPerVec;
  const bool vec_ok = cols % E == 0 && aligned16(x) && aligned16(w) && aligned16(y);
  const int64_t n_vec = cols / E;
  if (vec_ok && n_vec <= 8 * 1024) {
    const int nv = (int)n_vec;
    const int c = (int)cols;
    // Short rows: one warp per row with 1..8 vectors per lane.
    if (nv <= 32) return launch_vec<T, 1, 32>(x, w, y, rows, c, eps, s);
    if (nv <= 64) return launch_vec<T, 2, 32>(x, w, y, rows, c, eps, s);
    if (nv <= 128) return launch_vec<T, 4, 32>(x, w, y, rows, c, eps, s);
    if (nv <= 256) return launch_vec<T, 8, 32>(x, w, y, rows, c, eps, s);
    // Long rows: 8 vectors per thread, 64..1024 threads per row.
    if (nv <= 512) return launch_vec<T, 8, 64>(x, w, y, rows, c, eps, s);
    if (nv <= 1024) return launch_vec<T, 8, 128>(x, w, y, rows, c, eps, s);
    if (nv <= 2048) return launch_vec<T, 8, 256>(x, w, y, rows, c, eps, s);
    if (nv <= 4096) return launch_vec<T, 8, 512>(x, w, y, rows, c, eps, s);
    return launch_vec<T, 8, 1024>(x, w, y, rows, c, eps, s);
  }
  if (rows > 0x7fffffffLL) return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_rmsnorm_forward: too many rows");
  rmsnorm_scalar_kernel<T><<<(unsigned)rows, kBlock, 0, s>>>(x, w, y, cols, eps);
  return check_launch("aotk_rmsnorm_forward");
}

}  // namespace
}  // namespace aotk

extern "C" int aotk_rmsnorm_forward(void* out, const void* x, const void* weight, int64_t rows,
                                    int64_t cols, double eps, int dtype, void* stream) {
  using namespace aotk;
  if (rows < 0 || cols < 0) return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_rmsnorm_forward: negative size");
  if (rows == 0 || cols == 0) return AOTK_OK;
  if (!out || !x || !weight) return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_rmsnorm_forward: null pointer");
  if (cols > 0x7fffffffLL) return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_rmsnorm_forward: row too long");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float e = static_cast<float>(eps);
  switch (dtype) {
    case AOTK_FLOAT32: return launch<float>(x, weight, out, rows, cols, e, s);
    case AOTK_FLOAT16: return launch<__half>(x, weight, out, rows, cols, e, s);
    case AOTK_BFLOAT16: return launch<__nv_bfloat16>(x, weight, out, rows, cols, e, s);
    default: return fail(AOTK_ERR_UNSUPPORTED, "aotk_rmsnorm_forward: unsupported dtype %d", dtype);
  }
}
