// Activation kernels: silu, relu and the fused silu(gate) * up.
//
// These are pure HBM-streaming kernels (2 bytes read + 2 written per bf16
// element for silu/relu, 4 + 2 for silu_mul).  Each thread moves 16-byte
// vectors, issues all UNROLL loads of an iteration before any math so that
// UNROLL * 16 bytes per thread are in flight, and walks the tensor with a
// grid-stride loop over a grid of exactly one wave of resident blocks.  The reference runs one
// scalar element per thread with 458 752 blocks at [8192, 14336]
// (aot_kernel/csrc/activation/silu.cu:14-19, :29-39).  Every kernel here is
// launched with programmatic dependent launch: it lets the next kernel on the
// stream start its prologue at once, and touches global memory only after
// griddepcontrol.wait, so its own launch and setup overlap the tail of the
// kernel before it.
#include "common.h"
#include "sm100.cuh"
#include "vec.cuh"

#include <mutex>

namespace aotk {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;
constexpr int kBlocksPerSm = 8;

struct SiluOp {
  __device__ __forceinline__ static float apply(float x) { return silu_f(x); }
};
struct ReluOp {
  // max(x, 0) propagating NaN like torch.relu.
  __device__ __forceinline__ static float apply(float x) { return x > 0.0f || x != x ? x : 0.0f; }
};

// Unary map over n_vec 16-byte vectors.
template <typename T, typename Op>
__global__ void __launch_bounds__(kThreads) unary_vec_kernel(const uint4* __restrict__ x,
                                                             uint4* __restrict__ y, int64_t n_vec) {
  constexpr int E = Elem<T>::kPerVec;
  sm100::pdl_launch_dependents();
  sm100::pdl_wait_prior();
  const int64_t step = (int64_t)gridDim.x * kThreads * kUnroll;
  for (int64_t base = (int64_t)blockIdx.x * kThreads * kUnroll + threadIdx.x; base < n_vec;
       base += step) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + (int64_t)u * kThreads;
      if (i < n_vec) v[u] = ld_stream(x + i);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + (int64_t)u * kThreads;
      if (i < n_vec) {
        float f[E];
        Elem<T>::unpack(v[u], f);
#pragma unroll
        for (int e = 0; e < E; ++e) f[e] = Op::apply(f[e]);
        st_stream(y + i, Elem<T>::pack(f));
      }
    }
  }
}

// Scalar remainder / unaligned fallback.
template <typename T, typename Op>
__global__ void __launch_bounds__(kThreads) unary_scalar_kernel(const T* __restrict__ x,
                                                                T* __restrict__ y, int64_t n) {
  sm100::pdl_launch_dependents();
  sm100::pdl_wait_prior();
  const int64_t step = (int64_t)gridDim.x * kThreads;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += step) {
    y[i] = Elem<T>::from_f(Op::apply(Elem<T>::to_f(x[i])));
  }
}

// silu(gate) * up over a [rows, cols] view with row strides (in elements);
// vectorised along the row when every row start is 16-byte aligned.
template <typename T>
__global__ void __launch_bounds__(kThreads) silu_mul_vec_kernel(
    const T* __restrict__ gate, int64_t gate_stride, const T* __restrict__ up, int64_t up_stride,
    T* __restrict__ out, int64_t out_stride, int64_t rows, int64_t vec_per_row) {
  constexpr int E = Elem<T>::kPerVec;
  const int64_t n_vec = rows * vec_per_row;
  sm100::pdl_launch_dependents();
  sm100::pdl_wait_prior();
  const int64_t step = (int64_t)gridDim.x * kThreads * kUnroll;
  for (int64_t base = (int64_t)blockIdx.x * kThreads * kUnroll + threadIdx.x; base < n_vec;
       base += step) {
    uint4 g[kUnroll], u4[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + (int64_t)u * kThreads;
      if (i < n_vec) {
        const int64_t r = i / vec_per_row;
        const int64_t c = (i - r * vec_per_row) * E;
        g[u] = ld_stream(reinterpret_cast<const uint4*>(gate + r * gate_stride + c));
        u4[u] = ld_stream(reinterpret_cast<const uint4*>(up + r * up_stride + c));
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + (int64_t)u * kThreads;
      if (i < n_vec) {
        const int64_t r = i / vec_per_row;
        const int64_t c = (i - r * vec_per_row) * E;
        float fg[E], fu[E];
        Elem<T>::unpack(g[u], fg);
        Elem<T>::unpack(u4[u], fu);
#pragma unroll
        for (int e = 0; e < E; ++e) fg[e] = silu_f(fg[e]) * fu[e];
        st_stream(reinterpret_cast<uint4*>(out + r * out_stride + c), Elem<T>::pack(fg));
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) silu_mul_scalar_kernel(
    const T* __restrict__ gate, int64_t gate_stride, const T* __restrict__ up, int64_t up_stride,
    T* __restrict__ out, int64_t out_stride, int64_t rows, int64_t cols) {
  const int64_t n = rows * cols;
  sm100::pdl_launch_dependents();
  sm100::pdl_wait_prior();
  const int64_t step = (int64_t)gridDim.x * kThreads;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += step) {
    const int64_t r = i / cols;
    const int64_t c = i - r * cols;
    const float g = Elem<T>::to_f(gate[r * gate_stride + c]);
    const float u = Elem<T>::to_f(up[r * up_stride + c]);
    out[r * out_stride + c] = Elem<T>::from_f(silu_f(g) * u);
  }
}

// Blocks of `kernel` that are resident at once on one SM of the current
// device (cached per kernel and device; at most kBlocksPerSm).
int resident_per_sm(const void* kernel, const DeviceInfo& info) {
  struct Entry {
    const void* kernel;
    int device, n;
  };
  static std::mutex mu;
  static Entry cache[64];
  static int count = 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < count; ++i)
    if (cache[i].kernel == kernel && cache[i].device == info.device) return cache[i].n;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kThreads, 0) != cudaSuccess || n < 1)
    n = 1;
  if (n > kBlocksPerSm) n = kBlocksPerSm;
  if (count < 64) cache[count++] = Entry{kernel, info.device, n};
  return n;
}

// Grid of the grid-stride kernels: one wave of resident blocks (a grid
// larger than what fits would run its last blocks as a partial second wave).
int grid_for(const void* kernel, int64_t work_items, int per_block, const DeviceInfo& info) {
  const int64_t want = (work_items + per_block - 1) / per_block;
  const int64_t cap = (int64_t)info.sm_count * resident_per_sm(kernel, info);
  return (int)(want < cap ? (want > 0 ? want : 1) : cap);
}

// Launches `kernel` on `grid` blocks of kThreads with programmatic stream
// serialisation and turns a launch error into AOTK_ERR_CUDA.
template <typename... Params, typename... Args>
int launch_pdl(void (*kernel)(Params...), int grid, cudaStream_t stream, const char* name,
               Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
  if (e != cudaSuccess) return fail(AOTK_ERR_CUDA, "%s launch: %s", name, cudaGetErrorString(e));
  return check_launch(name);
}

template <typename T, typename Op>
int launch_unary(void* out, const void* x, int64_t n, cudaStream_t stream, const char* name) {
  DeviceInfo info;
  if (int st = current_device_info(&info)) return st;
  constexpr int E = Elem<T>::kPerVec;
  int64_t head = 0;  // elements covered by the vector kernel
  if (aligned16(out) && aligned16(x)) {
    const int64_t n_vec = n / E;
    if (n_vec > 0) {
      auto kernel = unary_vec_kernel<T, Op>;
      const int grid = grid_for(reinterpret_cast<const void*>(kernel), n_vec, kThreads * kUnroll, info);
      if (int st = launch_pdl(kernel, grid, stream, name, static_cast<const uint4*>(x),
                              static_cast<uint4*>(out), n_vec))
        return st;
    }
    head = n_vec * E;
  }
  const int64_t tail = n - head;
  if (tail > 0) {
    auto kernel = unary_scalar_kernel<T, Op>;
    const int grid = grid_for(reinterpret_cast<const void*>(kernel), tail, kThreads, info);
    if (int st = launch_pdl(kernel, grid, stream, name, static_cast<const T*>(x) + head,
                            static_cast<T*>(out) + head, tail))
      return st;
  }
  return AOTK_OK;
}

template <typename Op>
int dispatch_unary(void* out, const void* x, int64_t n, int dtype, void* stream, const char* name) {
  if (n < 0) return fail(AOTK_ERR_INVALID_ARGUMENT, "%s: negative size %lld", name, (long long)n);
  if (n == 0) return AOTK_OK;
  if (!out || !x) return fail(AOTK_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case AOTK_FLOAT32: return launch_unary<float, Op>(out, x, n, s, name);
    case AOTK_FLOAT16: return launch_unary<__half, Op>(out, x, n, s, name);
    case AOTK_BFLOAT16: return launch_unary<__nv_bfloat16, Op>(out, x, n, s, name);
    default: return fail(AOTK_ERR_UNSUPPORTED, "%s: unsupported dtype %d", name, dtype);
  }
}

template <typename T>
int launch_silu_mul(void* out, int64_t out_stride, const void* gate, int64_t gate_stride,
                    const void* up, int64_t up_stride, int64_t rows, int64_t cols,
                    cudaStream_t stream) {
  DeviceInfo info;
  if (int st = current_device_info(&info)) return st;
  constexpr int E = Elem<T>::kPerVec;
  const bool vec_ok = aligned16(out) && aligned16(gate) && aligned16(up) && cols % E == 0 &&
                      out_stride % E == 0 && gate_stride % E == 0 && up_stride % E == 0;
  if (vec_ok) {
    const int64_t vpr = cols / E;
    auto kernel = silu_mul_vec_kernel<T>;
    const int grid =
        grid_for(reinterpret_cast<const void*>(kernel), rows * vpr, kThreads * kUnroll, info);
    return launch_pdl(kernel, grid, stream, "aotk_silu_mul_forward", static_cast<const T*>(gate),
                      gate_stride, static_cast<const T*>(up), up_stride, static_cast<T*>(out),
                      out_stride, rows, vpr);
  }
  auto kernel = silu_mul_scalar_kernel<T>;
  const int grid = grid_for(reinterpret_cast<const void*>(kernel), rows * cols, kThreads, info);
  return launch_pdl(kernel, grid, stream, "aotk_silu_mul_forward", static_cast<const T*>(gate),
                    gate_stride, static_cast<const T*>(up), up_stride, static_cast<T*>(out),
                    out_stride, rows, cols);
}

}  // namespace
}  // namespace aotk

extern "C" int aotk_silu_forward(void* out, const void* x, int64_t n, int dtype, void* stream) {
  return aotk::dispatch_unary<aotk::SiluOp>(out, x, n, dtype, stream, "aotk_silu_forward");
}

extern "C" int aotk_relu_forward(void* out, const void* x, int64_t n, int dtype, void* stream) {
  return aotk::dispatch_unary<aotk::ReluOp>(out, x, n, dtype, stream, "aotk_relu_forward");
}

extern "C" int aotk_silu_mul_forward(void* out, int64_t out_stride, const void* gate,
                                     int64_t gate_stride, const void* up, int64_t up_stride,
                                     int64_t rows, int64_t cols, int dtype, void* stream) {
  using namespace aotk;
  if (rows < 0 || cols < 0)
    return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_silu_mul_forward: negative size");
  if (rows == 0 || cols == 0) return AOTK_OK;
  if (!out || !gate || !up) return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_silu_mul_forward: null pointer");
  if (out_stride < cols || gate_stride < cols || up_stride < cols)
    return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_silu_mul_forward: row stride smaller than cols");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case AOTK_FLOAT32:
      return launch_silu_mul<float>(out, out_stride, gate, gate_stride, up, up_stride, rows, cols, s);
    case AOTK_FLOAT16:
      return launch_silu_mul<__half>(out, out_stride, gate, gate_stride, up, up_stride, rows, cols, s);
    case AOTK_BFLOAT16:
      return launch_silu_mul<__nv_bfloat16>(out, out_stride, gate, gate_stride, up, up_stride, rows,
                                            cols, s);
    default:
      return fail(AOTK_ERR_UNSUPPORTED, "aotk_silu_mul_forward: unsupported dtype %d", dtype);
  }
}
