// Device helpers for the HBM-streaming kernels: 16-byte vector loads/stores
// and the float <-> element conversions of the three supported types.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

namespace aotk {

// Read-only 16-byte load that bypasses L1 allocation (each byte is read once).
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// 16-byte load through L1 (for data reused by several warps, e.g. norm weights).
__device__ __forceinline__ uint4 ld_cached(const uint4* p) { return __ldg(p); }

__device__ __forceinline__ void st_stream(uint4* p, const uint4& v) {
  asm volatile("st.global.L1::no_allocate.v4.u32 [%0], {%1, %2, %3, %4};"
               :
               : "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Element traits: E elements per 16-byte vector, unpack to / pack from floats.
template <typename T>
struct Elem;

template <>
struct Elem<float> {
  static constexpr int kPerVec = 4;
  __device__ __forceinline__ static float to_f(float v) { return v; }
  __device__ __forceinline__ static float from_f(float v) { return v; }
  __device__ __forceinline__ static void unpack(const uint4& v, float* f) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
  }
};

template <>
struct Elem<__nv_bfloat16> {
  static constexpr int kPerVec = 8;
  __device__ __forceinline__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  __device__ __forceinline__ static float2 unpack2(uint32_t u) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&u);
    return __bfloat1622float2(h);
  }
  __device__ __forceinline__ static uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static void unpack(const uint4& v, float* f) {
    float2 t;
    t = unpack2(v.x); f[0] = t.x; f[1] = t.y;
    t = unpack2(v.y); f[2] = t.x; f[3] = t.y;
    t = unpack2(v.z); f[4] = t.x; f[5] = t.y;
    t = unpack2(v.w); f[6] = t.x; f[7] = t.y;
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
  }
};

template <>
struct Elem<__half> {
  static constexpr int kPerVec = 8;
  __device__ __forceinline__ static float to_f(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from_f(float v) { return __float2half_rn(v); }
  __device__ __forceinline__ static float2 unpack2(uint32_t u) {
    __half2 h = *reinterpret_cast<__half2*>(&u);
    return __half22float2(h);
  }
  __device__ __forceinline__ static uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static void unpack(const uint4& v, float* f) {
    float2 t;
    t = unpack2(v.x); f[0] = t.x; f[1] = t.y;
    t = unpack2(v.y); f[2] = t.x; f[3] = t.y;
    t = unpack2(v.z); f[4] = t.x; f[5] = t.y;
    t = unpack2(v.w); f[6] = t.x; f[7] = t.y;
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
  }
};

// silu(x) = x * sigmoid(x) = x / (1 + e^-x), with the hardware exponential and
// reciprocal; for x -> -inf the denominator overflows to +inf and the result
// is -0, for x -> +inf it is x.
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

}  // namespace aotk
