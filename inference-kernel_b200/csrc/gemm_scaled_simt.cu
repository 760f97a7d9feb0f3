// SIMT scaled GEMM on 8-bit operands: C = (A * B) * scale_a * scale_b for
// every shape, dtype combination and alignment aotk_scaled_gemm accepts.  The
// path for shapes the tcgen05 kernel's TMA cannot address (K or N not a
// multiple of 16, unaligned pointers) - the reference's test shapes
// (130, 64, 130) and (129, 257, 193) among them.
//
// 64 x 64 output tile per 256-thread block, 4 x 4 outputs per thread, K
// staged 32 at a time through shared memory.  fp8 bytes are decoded once
// when staged (exact in fp32) and accumulated in fp32; int8 products are
// accumulated in int32 (exact) and converted at the end, as the reference's
// fp32 accumulator of int32 dot products is while |acc| < 2^24.
//
// Replaces the reference's Triton kernels _scaled_gemm_kernel and
// _scaled_gemm_kernel_optimized (jit_kernel/gemm.py:86-123, 144-196).
#include <cuda_fp8.h>

#include "common.h"
#include "gemm_internal.h"
#include "vec.cuh"

#include <type_traits>

namespace aotk {
namespace {

constexpr int kTile = 64;
constexpr int kTK = 32;

// Input kinds: 0 = int8, 1 = e4m3, 2 = e5m2.
template <int kKind>
struct In8 {
  using Acc = typename std::conditional<kKind != 0, float, int>::type;
  __device__ __forceinline__ static Acc load(const uint8_t* p) {
    if constexpr (kKind != 0) {
      const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(*p),
                                                   kKind == 1 ? __NV_E4M3 : __NV_E5M2);
      return __half2float(__half(h));
    } else {
      return static_cast<int>(static_cast<int8_t>(*p));
    }
  }
};

template <typename TOut>
__device__ __forceinline__ void store_out(TOut* p, float v) {
  if constexpr (std::is_same<TOut, float>::value)
    *p = v;
  else
    *p = Elem<TOut>::from_f(v);
}

template <int kKind, typename TOut>
__global__ void __launch_bounds__(256) scaled_gemm_simt_kernel(
    TOut* __restrict__ C, const uint8_t* __restrict__ A, const uint8_t* __restrict__ B,
    const float* __restrict__ sa, const float* __restrict__ sb, int sa_step, int sb_step, int M,
    int N, int K) {
  using Acc = typename In8<kKind>::Acc;
  __shared__ Acc sA[kTK][kTile + 1];  // [k][m]
  __shared__ Acc sB[kTK][kTile];      // [k][n]
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * kTile, n0 = blockIdx.x * kTile;
  Acc acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += kTK) {
    for (int i = threadIdx.x; i < kTile * kTK; i += 256) {
      const int r = i / kTK, k = i % kTK;  // A: consecutive threads along K
      const int gm = m0 + r, gk = k0 + k;
      sA[k][r] = (gm < M && gk < K) ? In8<kKind>::load(A + static_cast<size_t>(gm) * K + gk) : Acc(0);
      const int kb = i / kTile, c = i % kTile;  // B: consecutive threads along N
      const int gkb = k0 + kb, gn = n0 + c;
      sB[kb][c] = (gkb < K && gn < N) ? In8<kKind>::load(B + static_cast<size_t>(gkb) * N + gn) : Acc(0);
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < kTK; ++k) {
      Acc a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = sA[k][ty + 16 * i];
        b[i] = sB[k][tx + 16 * i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += a[i] * b[j];
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty + 16 * i;
    if (gm >= M) continue;
    const float s_row = sa[static_cast<size_t>(gm) * sa_step];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx + 16 * j;
      if (gn >= N) continue;
      const float v = (static_cast<float>(acc[i][j]) * s_row) * sb[static_cast<size_t>(gn) * sb_step];
      store_out(C + static_cast<size_t>(gm) * N + gn, v);
    }
  }
}

template <int kKind>
int launch(void* c, const void* a, const void* b, const float* sa, const float* sb, int step,
           int M, int N, int K, int out_dtype, cudaStream_t s) {
  const dim3 grid((N + kTile - 1) / kTile, (M + kTile - 1) / kTile);
  const auto* A = static_cast<const uint8_t*>(a);
  const auto* B = static_cast<const uint8_t*>(b);
  if (out_dtype == AOTK_BFLOAT16)
    scaled_gemm_simt_kernel<kKind, __nv_bfloat16><<<grid, 256, 0, s>>>(
        static_cast<__nv_bfloat16*>(c), A, B, sa, sb, step, step, M, N, K);
  else if (out_dtype == AOTK_FLOAT16)
    scaled_gemm_simt_kernel<kKind, __half><<<grid, 256, 0, s>>>(static_cast<__half*>(c), A, B, sa,
                                                               sb, step, step, M, N, K);
  else
    scaled_gemm_simt_kernel<kKind, float><<<grid, 256, 0, s>>>(static_cast<float*>(c), A, B, sa, sb,
                                                              step, step, M, N, K);
  return check_launch("scaled gemm (SIMT)");
}

}  // namespace

int gemm_scaled_simt(void* c, const void* a, const void* b, const float* scale_a,
                     const float* scale_b, int64_t M, int64_t N, int64_t K, int in_dtype,
                     int out_dtype, int scale_mode, void* stream) {
  if (M == 0 || N == 0) return AOTK_OK;
  if ((M + kTile - 1) / kTile > 65535)
    return fail(AOTK_ERR_UNSUPPORTED, "aotk_scaled_gemm_simt: M = %lld too large", (long long)M);
  const int step = scale_mode == AOTK_SCALE_ROW ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int m = (int)M, n = (int)N, k = (int)K;
  if (in_dtype == AOTK_FLOAT8_E4M3)
    return launch<1>(c, a, b, scale_a, scale_b, step, m, n, k, out_dtype, s);
  if (in_dtype == AOTK_FLOAT8_E5M2)
    return launch<2>(c, a, b, scale_a, scale_b, step, m, n, k, out_dtype, s);
  return launch<0>(c, a, b, scale_a, scale_b, step, m, n, k, out_dtype, s);
}

}  // namespace aotk
