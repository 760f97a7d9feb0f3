// Status/error plumbing and the per-device property cache.
#include "common.h"

#include <mutex>

namespace aotk {

namespace {
thread_local char g_last_error[512] = "no error";

constexpr int kMaxDevices = 64;
DeviceInfo g_info[kMaxDevices];
std::once_flag g_info_once[kMaxDevices];
}  // namespace

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    return fail(AOTK_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(err));
  }
  return AOTK_OK;
}

int current_device_info(DeviceInfo* info) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return fail(AOTK_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxDevices) return fail(AOTK_ERR_CUDA, "device ordinal %d out of range", dev);
  int status = AOTK_OK;
  std::call_once(g_info_once[dev], [&] {
    DeviceInfo d;
    d.device = dev;
    cudaError_t e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (e == cudaSuccess)
      e = cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) {
      status = fail(AOTK_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
      d.device = -1;
    }
    g_info[dev] = d;
  });
  if (status != AOTK_OK) return status;
  if (g_info[dev].device < 0) return fail(AOTK_ERR_CUDA, "device %d properties unavailable", dev);
  *info = g_info[dev];
  return AOTK_OK;
}

int require_sm100(const DeviceInfo& info) {
  if (info.cc_major != 10) {
    return fail(AOTK_ERR_DEVICE, "tcgen05 kernels need an sm_100 device, found sm_%d%d",
                info.cc_major, info.cc_minor);
  }
  return AOTK_OK;
}

}  // namespace aotk

extern "C" const char* aotk_last_error(void) { return aotk::g_last_error; }

extern "C" int aotk_version(void) { return 100; }
