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
//
// The residual variant (aotk_add_rmsnorm_forward) first forms h = x + residual
// rounded to the element type - what `rmsnorm(x + residual)` sees when the
// addition is a separate 16-bit op - writes h out as the next residual and
// normalises h, all in the same pass: x and residual are read once, h and y
// written once.
#include "common.h"
#include "sm100.cuh"
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
// With kRes, the loaded vectors are x and residual and the row is their
// rounded sum h, which is also written to h_out.
// With kStats the kernel writes only the row statistic rstd (fp32, to
// `stats`) and no normalised row.
template <typename T, int VPT, int TPR, bool kRes, bool kStats = false>
__global__ void __launch_bounds__(TPR > kBlock ? TPR : kBlock)
    rmsnorm_vec_kernel(const T* __restrict__ x, const T* __restrict__ res, const T* __restrict__ w,
                       T* __restrict__ y, T* __restrict__ h_out, int64_t rows, int cols,
                       float eps, float* __restrict__ stats = nullptr) {
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

  // Programmatic dependent launch: the next kernel may start its prologue
  // now; x (and the residual) may come from the previous kernel, so nothing
  // is read before it has completed.
  sm100::pdl_launch_dependents();
  sm100::pdl_wait_prior();
  uint4 cur[VPT], cur_r[kRes ? VPT : 1];
  int64_t g = blockIdx.x;
  load_row<T, VPT, TPR>(x, g * RPB + sub, rows, cols, t, cur);
  if constexpr (kRes) load_row<T, VPT, TPR>(res, g * RPB + sub, rows, cols, t, cur_r);
  for (int iter = 0; g < groups; g += gridDim.x, ++iter) {
    uint4 nxt[VPT], nxt_r[kRes ? VPT : 1];
    if constexpr (kPrefetch) {
      load_row<T, VPT, TPR>(x, (g + gridDim.x) * RPB + sub, rows, cols, t, nxt);
      if constexpr (kRes) load_row<T, VPT, TPR>(res, (g + gridDim.x) * RPB + sub, rows, cols, t, nxt_r);
    }
    const int64_t row = g * RPB + sub;
    if constexpr (kRes) {
      // h = round(x + residual); the normalisation below sees exactly h.
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        float a[E], b[E];
        Elem<T>::unpack(cur[i], a);
        Elem<T>::unpack(cur_r[i], b);
#pragma unroll
        for (int e = 0; e < E; ++e) a[e] += b[e];
        cur[i] = Elem<T>::pack(a);
        const int idx = t + i * TPR;
        if (row < rows && idx < n_vec)
          st_stream(reinterpret_cast<uint4*>(h_out + row * (int64_t)cols) + idx, cur[i]);
      }
    }

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
    if constexpr (kStats) {
      if (row < rows && t == 0) stats[row] = rstd;
    } else if (row < rows) {
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
      for (int i = 0; i < VPT; ++i) {
        cur[i] = nxt[i];
        if constexpr (kRes) cur_r[i] = nxt_r[i];
      }
    } else {
      load_row<T, VPT, TPR>(x, (g + gridDim.x) * RPB + sub, rows, cols, t, cur);
      if constexpr (kRes) load_row<T, VPT, TPR>(res, (g + gridDim.x) * RPB + sub, rows, cols, t, cur_r);
    }
  }
}

// Any row length: one block per row, two passes over the row (the second
// mostly hits L2).  With a residual, pass one also writes h = round(x + r) and
// pass two reads h back.
template <typename T, bool kRes>
__global__ void __launch_bounds__(kBlock) rmsnorm_scalar_kernel(const T* __restrict__ x,
                                                                const T* __restrict__ res,
                                                                const T* __restrict__ w,
                                                                T* __restrict__ y,
                                                                T* __restrict__ h_out,
                                                                int64_t cols, float eps) {
  __shared__ float partial[kBlock / 32];
  const int64_t off = (int64_t)blockIdx.x * cols;
  float ss = 0.0f;
  for (int64_t c = threadIdx.x; c < cols; c += kBlock) {
    float f = Elem<T>::to_f(x[off + c]);
    if constexpr (kRes) {
      const T h = Elem<T>::from_f(f + Elem<T>::to_f(res[off + c]));
      h_out[off + c] = h;
      f = Elem<T>::to_f(h);
    }
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
  const T* src = kRes ? h_out : x;  // each thread re-reads only what it wrote
  for (int64_t c = threadIdx.x; c < cols; c += kBlock) {
    y[off + c] = Elem<T>::from_f(Elem<T>::to_f(src[off + c]) * rstd * Elem<T>::to_f(w[c]));
  }
}

template <typename T, int VPT, int TPR, bool kRes, bool kStats = false>
int launch_vec(const T* x, const T* r, const T* w, T* y, T* h, int64_t rows, int cols, float eps,
               cudaStream_t s, float* stats = nullptr) {
  constexpr int THREADS = TPR > kBlock ? TPR : kBlock;
  constexpr int RPB = THREADS / TPR;
  DeviceInfo info;
  if (int st = current_device_info(&info)) return st;
  auto kernel = rmsnorm_vec_kernel<T, VPT, TPR, kRes, kStats>;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, THREADS, 0) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int64_t groups = (rows + RPB - 1) / RPB;
  const int64_t capacity = (int64_t)per_sm * info.sm_count;
  const int64_t blocks = groups < capacity ? groups : capacity;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks, 1, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, x, r, w, y, h, rows, cols, eps, stats);
  if (e != cudaSuccess)
    return fail(AOTK_ERR_CUDA, "aotk_rmsnorm_forward launch: %s", cudaGetErrorString(e));
  return check_launch("aotk_rmsnorm_forward");
}

template <typename T, bool kRes>
int launch(const void* xv, const void* rv, const void* wv, void* yv, void* hv, int64_t rows,
           int64_t cols, float eps, cudaStream_t s) {
  const T* x = static_cast<const T*>(xv);
  const T* r = static_cast<const T*>(rv);
  const T* w = static_cast<const T*>(wv);
  T* y = static_cast<T*>(yv);
  T* h = static_cast<T*>(hv);
  constexpr int E = Elem<T>::kPerVec;
  const bool vec_ok = cols % E == 0 && aligned16(x) && aligned16(w) && aligned16(y) &&
                      (!kRes || (aligned16(r) && aligned16(h)));
  const int64_t n_vec = cols / E;
  // The residual variant keeps two copies (x, r) of the row per thread: at
  // most 4 vectors per thread, twice the threads per row.
  constexpr int kMaxVpt = kRes ? 4 : 8;
  if (vec_ok && n_vec <= kMaxVpt * 1024) {
    const int nv = (int)n_vec;
    const int c = (int)cols;
    // Short rows: one warp per row with 1..kMaxVpt vectors per lane.
    if (nv <= 32) return launch_vec<T, 1, 32, kRes>(x, r, w, y, h, rows, c, eps, s);
    if (nv <= 64) return launch_vec<T, 2, 32, kRes>(x, r, w, y, h, rows, c, eps, s);
    if (nv <= 128) return launch_vec<T, 4, 32, kRes>(x, r, w, y, h, rows, c, eps, s);
    constexpr int V = kMaxVpt;
    if (nv <= V * 32) return launch_vec<T, V, 32, kRes>(x, r, w, y, h, rows, c, eps, s);
    // Long rows: kMaxVpt vectors per thread, 64..1024 threads per row.
    if (nv <= V * 64) return launch_vec<T, V, 64, kRes>(x, r, w, y, h, rows, c, eps, s);
    if (nv <= V * 128) return launch_vec<T, V, 128, kRes>(x, r, w, y, h, rows, c, eps, s);
    if (nv <= V * 256) return launch_vec<T, V, 256, kRes>(x, r, w, y, h, rows, c, eps, s);
    if (nv <= V * 512) return launch_vec<T, V, 512, kRes>(x, r, w, y, h, rows, c, eps, s);
    return launch_vec<T, V, 1024, kRes>(x, r, w, y, h, rows, c, eps, s);
  }
  if (rows > 0x7fffffffLL) return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_rmsnorm_forward: too many rows");
  rmsnorm_scalar_kernel<T, kRes><<<(unsigned)rows, kBlock, 0, s>>>(x, r, w, y, h, cols, eps);
  return check_launch("aotk_rmsnorm_forward");
}

template <bool kRes>
int dispatch(const void* x, const void* r, const void* w, void* y, void* h, int64_t rows,
             int64_t cols, double eps, int dtype, void* stream, const char* name) {
  if (rows < 0 || cols < 0) return fail(AOTK_ERR_INVALID_ARGUMENT, "%s: negative size", name);
  if (rows == 0 || cols == 0) return AOTK_OK;
  if (!y || !x || !w || (kRes && (!r || !h)))
    return fail(AOTK_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (cols > 0x7fffffffLL) return fail(AOTK_ERR_INVALID_ARGUMENT, "%s: row too long", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float e = static_cast<float>(eps);
  switch (dtype) {
    case AOTK_FLOAT32: return launch<float, kRes>(x, r, w, y, h, rows, cols, e, s);
    case AOTK_FLOAT16: return launch<__half, kRes>(x, r, w, y, h, rows, cols, e, s);
    case AOTK_BFLOAT16: return launch<__nv_bfloat16, kRes>(x, r, w, y, h, rows, cols, e, s);
    default: return fail(AOTK_ERR_UNSUPPORTED, "%s: unsupported dtype %d", name, dtype);
  }
}

// rstd[row] = rsqrt(mean(x[row]^2) + eps) in fp32 and nothing else: the row
// statistic of rms_norm for callers that fold the normalisation into a GEMM
// (x @ (diag(w) W) scaled by rstd per row, aotk_gemm_silu_mul_rowscale).
// Long rows take rmsnorm_vec_kernel in statistics-only mode; this kernel
// serves short and unaligned rows: one warp per row, 16-byte loads, 8 in
// flight per lane; x is read once.
template <typename T, bool kVec>
__global__ void __launch_bounds__(kBlock) rms_rstd_kernel(const T* __restrict__ x,
                                                          float* __restrict__ rstd, int64_t rows,
                                                          int64_t cols, float eps) {
  constexpr int E = Elem<T>::kPerVec;
  const int64_t row = (int64_t)blockIdx.x * (kBlock / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float ss = 0.0f;
  if constexpr (kVec) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * cols);
    const int64_t n_vec = cols / E;
    for (int64_t v0 = lane; v0 < n_vec; v0 += 8 * 32) {
      uint4 v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int64_t idx = v0 + i * 32;
        v[i] = idx < n_vec ? ld_stream(xr + idx) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float f[E];
        Elem<T>::unpack(v[i], f);
#pragma unroll
        for (int e = 0; e < E; ++e) ss = fmaf(f[e], f[e], ss);
      }
    }
  } else {
    for (int64_t c = lane; c < cols; c += 32) {
      const float f = Elem<T>::to_f(x[row * cols + c]);
      ss = fmaf(f, f, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) rstd[row] = rsqrtf(ss / (float)cols + eps);
}

template <typename T>
int launch_rstd(const void* xv, float* rstd, int64_t rows, int64_t cols, float eps,
                cudaStream_t s) {
  const T* x = static_cast<const T*>(xv);
  constexpr int E = Elem<T>::kPerVec;
  const int64_t n_vec = cols / E;
  // Rows that fit the persistent vector kernel use it in statistics-only
  // mode (the same row layout and prefetch as rms_norm, no output row).
  if (cols % E == 0 && aligned16(x) && n_vec <= 8 * 1024 && n_vec > 128) {
    const int nv = (int)n_vec, c = (int)cols;
    const T* none = nullptr;
    T* none_out = nullptr;
#define AOTK_RSTD_VEC(TPR) \
  launch_vec<T, 8, TPR, false, true>(x, none, none, none_out, none_out, rows, c, eps, s, rstd)
    if (nv <= 8 * 32) return AOTK_RSTD_VEC(32);
    if (nv <= 8 * 64) return AOTK_RSTD_VEC(64);
    if (nv <= 8 * 128) return AOTK_RSTD_VEC(128);
    if (nv <= 8 * 256) return AOTK_RSTD_VEC(256);
    if (nv <= 8 * 512) return AOTK_RSTD_VEC(512);
    return AOTK_RSTD_VEC(1024);
#undef AOTK_RSTD_VEC
  }
  const int64_t blocks = (rows + kBlock / 32 - 1) / (kBlock / 32);
  if (blocks > 0x7fffffffLL) return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_rmsnorm_rstd: too many rows");
  if (cols % E == 0 && aligned16(x))
    rms_rstd_kernel<T, true><<<(unsigned)blocks, kBlock, 0, s>>>(x, rstd, rows, cols, eps);
  else
    rms_rstd_kernel<T, false><<<(unsigned)blocks, kBlock, 0, s>>>(x, rstd, rows, cols, eps);
  return check_launch("aotk_rmsnorm_rstd");
}

}  // namespace
}  // namespace aotk

extern "C" int aotk_rmsnorm_rstd(float* rstd, const void* x, int64_t rows, int64_t cols, double eps,
                                 int dtype, void* stream) {
  using namespace aotk;
  if (rows < 0 || cols < 0) return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_rmsnorm_rstd: negative size");
  if (rows == 0) return AOTK_OK;
  if (!rstd || (cols > 0 && !x)) return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_rmsnorm_rstd: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float e = static_cast<float>(eps);
  switch (dtype) {
    case AOTK_FLOAT32: return launch_rstd<float>(x, rstd, rows, cols, e, s);
    case AOTK_FLOAT16: return launch_rstd<__half>(x, rstd, rows, cols, e, s);
    case AOTK_BFLOAT16: return launch_rstd<__nv_bfloat16>(x, rstd, rows, cols, e, s);
    default: return fail(AOTK_ERR_UNSUPPORTED, "aotk_rmsnorm_rstd: unsupported dtype %d", dtype);
  }
}

extern "C" int aotk_rmsnorm_forward(void* out, const void* x, const void* weight, int64_t rows,
                                    int64_t cols, double eps, int dtype, void* stream) {
  return aotk::dispatch<false>(x, nullptr, weight, out, nullptr, rows, cols, eps, dtype, stream,
                               "aotk_rmsnorm_forward");
}

extern "C" int aotk_add_rmsnorm_forward(void* out, void* residual_out, const void* x,
                                        const void* residual, const void* weight, int64_t rows,
                                        int64_t cols, double eps, int dtype, void* stream) {
  return aotk::dispatch<true>(x, residual, weight, out, residual_out, rows, cols, eps, dtype,
                              stream, "aotk_add_rmsnorm_forward");
}
