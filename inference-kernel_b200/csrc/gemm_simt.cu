// SIMT GEMM for the shapes and types the tensor-core paths do not take:
// FLOAT32 inputs, K or N not a multiple of 8, or pointers without 16-byte
// alignment.  64 x 64 output tile per 256-thread block, 4 x 4 outputs per
// thread, K staged through shared memory 16 at a time, fp32 accumulation and
// one rounding per output; every global access is bounds-checked.
// Stands in for the reference's naive tier (aot_kernel/csrc/gemm/gemm.cu:14-104),
// whose WMMA fragment loads read past M/N on partial tiles (gemm.cu:39-43).
#include "common.h"
#include "vec.cuh"

namespace aotk {
namespace {

constexpr int TM = 64, TN = 64, TK = 16;

template <typename T>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const T* __restrict__ a,
                                                        const T* __restrict__ b, T* __restrict__ c,
                                                        int64_t M, int64_t N, int64_t K) {
  __shared__ float sa[TK][TM + 4];
  __shared__ float sb[TK][TN + 4];
  const int tx = threadIdx.x % 16;  // column group
  const int ty = threadIdx.x / 16;  // row group
  const int64_t m0 = (int64_t)blockIdx.y * TM;
  const int64_t n0 = (int64_t)blockIdx.x * TN;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += TK) {
    // 64 x 16 tile of A and 16 x 64 tile of B: 1024 elements each, 4 per thread.
    for (int i = threadIdx.x; i < TM * TK; i += 256) {
      const int r = i / TK, kk = i % TK;
      const int64_t gm = m0 + r, gk = k0 + kk;
      sa[kk][r] = (gm < M && gk < K) ? Elem<T>::to_f(a[gm * K + gk]) : 0.0f;
    }
    for (int i = threadIdx.x; i < TK * TN; i += 256) {
      const int kk = i / TN, cc = i % TN;
      const int64_t gk = k0 + kk, gn = n0 + cc;
      sb[kk][cc] = (gk < K && gn < N) ? Elem<T>::to_f(b[gk * N + gn]) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = sa[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = sb[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t gm = m0 + ty + 16 * i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gn = n0 + tx + 16 * j;
      if (gn < N) c[gm * N + gn] = Elem<T>::from_f(acc[i][j]);
    }
  }
}

template <typename T>
int launch(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K,
           cudaStream_t s) {
  const int64_t gx = (N + TN - 1) / TN, gy = (M + TM - 1) / TM;
  if (gx > 0x7fffffffLL || gy > 65535)
    return fail(AOTK_ERR_INVALID_ARGUMENT, "simt gemm: problem too large (M=%lld N=%lld)",
                (long long)M, (long long)N);
  gemm_simt_kernel<T><<<dim3((unsigned)gx, (unsigned)gy), 256, 0, s>>>(
      static_cast<const T*>(a), static_cast<const T*>(b), static_cast<T*>(c), M, N, K);
  return check_launch("simt gemm");
}

}  // namespace

// Shared by aotk_gemm and the aotk_gemm_opt fallback.
int gemm_simt(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K, int dtype,
              void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case AOTK_FLOAT32: return launch<float>(c, a, b, M, N, K, s);
    case AOTK_FLOAT16: return launch<__half>(c, a, b, M, N, K, s);
    case AOTK_BFLOAT16: return launch<__nv_bfloat16>(c, a, b, M, N, K, s);
    default: return fail(AOTK_ERR_UNSUPPORTED, "gemm: unsupported dtype %d", dtype);
  }
}

}  // namespace aotk
