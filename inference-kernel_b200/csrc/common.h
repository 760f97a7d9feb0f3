// Host-side helpers shared by the kernel translation units: status codes,
// the per-thread error message behind aotk_last_error(), and a per-device
// cache of the properties the launchers size their grids from.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "aotk.h"

namespace aotk {

// Records a formatted message for aotk_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);

// Checks the launch that was just issued; turns a CUDA error into AOTK_ERR_CUDA.
int check_launch(const char* what);

struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0;
  int cc_minor = 0;
  int max_smem_optin = 0;
};

// Properties of the current device (cached per device ordinal).
int current_device_info(DeviceInfo* info);

// Requires an sm_100-family device for the tcgen05 / TMA kernels.
int require_sm100(const DeviceInfo& info);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int elem_size(int dtype) { return dtype == AOTK_FLOAT32 ? 4 : 2; }

inline bool valid_dtype(int dtype) {
  return dtype == AOTK_FLOAT32 || dtype == AOTK_FLOAT16 || dtype == AOTK_BFLOAT16;
}

}  // namespace aotk
