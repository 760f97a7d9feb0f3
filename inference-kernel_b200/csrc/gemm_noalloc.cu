// GEMM entry point for callers that cannot allocate device memory.
//
// aotk_gemm_opt_ws needs a scratch workspace for the K-split last wave of the
// persistent tcgen05 kernel.  Some hosts have no way to provide one: a program
// that binds only this C ABI through an FFI (a plugin inside another runtime,
// with no CUDA allocator of its own to call into), or a latency-critical
// serving loop that must never call cudaMalloc because cudaMalloc can
// synchronise the device and block on the driver.  For them the scratch lives
// in a fixed array compiled into this library instead.
//
// The array below is ordinary device global memory of kStaticScratchBytes on
// every GPU where this library's kernels are loaded, held until the process
// exits.  Host code must not hand the symbol itself to a kernel: on the host
// the name only stands for the variable.  Its device address is looked up
// once per device with cudaGetSymbolAddress, with that device current, the
// first time the entry point runs on it (retried until a lookup succeeds).
#include <cuda_runtime.h>

#include <mutex>

#include "common.h"
#include "gemm_internal.h"

// 24 MiB: the largest K-split workspace on a 148-SM B200 is 148 partial tiles of
// 128 x 256 fp32 (18.5 MiB) plus the per-tile counters.
constexpr size_t kStaticScratchBytes = 24u << 20;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

namespace aotk {
namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_static_scratch on the current device.  Only a
// successful lookup is cached: a lookup that failed (inside a stream capture,
// say, or on a transient driver error) is retried on the next call.
int static_scratch(int device, void** ptr) {
  if (device < 0 || device >= kMaxDevices)
    return fail(AOTK_ERR_CUDA, "device ordinal %d out of range", device);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[device] == nullptr) {
    void* p = nullptr;
    cudaError_t err = cudaGetSymbolAddress(&p, g_static_scratch);
    if (err != cudaSuccess || p == nullptr) {
      if (err != cudaSuccess) cudaGetLastError();  // not sticky: leave no error behind
      return fail(AOTK_ERR_CUDA, "cudaGetSymbolAddress(static scratch) on device %d: %s", device,
                  cudaGetErrorString(err));
    }
    g_scratch_ptr[device] = p;
  }
  *ptr = g_scratch_ptr[device];
  return AOTK_OK;
}

}  // namespace
}  // namespace aotk

extern "C" int aotk_gemm_opt_noalloc(void* c, const void* a, const void* b, int64_t M, int64_t N,
                                     int64_t K, int dtype, void* stream) {
  using namespace aotk;
  size_t need = 0;
  if (int st = aotk_gemm_opt_workspace_size(M, N, K, dtype, &need)) return st;
  if (need > kStaticScratchBytes)
    return fail(AOTK_ERR_UNSUPPORTED,
                "aotk_gemm_opt_noalloc: M=%lld N=%lld K=%lld needs %zu bytes of scratch, the "
                "library's static scratch holds %zu; use aotk_gemm_opt_ws with a workspace",
                (long long)M, (long long)N, (long long)K, need, kStaticScratchBytes);
  if (need == 0) return aotk_gemm_opt_ws(c, a, b, M, N, K, dtype, nullptr, 0, stream);
  DeviceInfo info;
  if (int st = current_device_info(&info)) return st;
  void* scratch = nullptr;
  if (int st = static_scratch(info.device, &scratch)) return st;
  return aotk_gemm_opt_ws(c, a, b, M, N, K, dtype, scratch, kStaticScratchBytes, stream);
}
