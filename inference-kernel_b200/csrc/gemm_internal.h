// Internal interface between the GEMM kernels and the C-ABI dispatcher.
#pragma once

#include <cstdint>

#include "common.h"

namespace aotk {

// Persistent tcgen05 kernel (gemm_tc.cu).  With a workspace of at least
// gemm_tc_workspace_size() bytes (256-byte aligned, contents irrelevant) the
// partial last wave of tiles is split along K; without one it runs whole.
int gemm_tc(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K, int dtype,
            void* workspace, size_t ws_bytes, void* stream);
size_t gemm_tc_workspace_size(int64_t M, int64_t N, int64_t K, int sm_count);

// Persistent tcgen05 GEMM whose epilogue applies silu(gate) * up: b is
// [K, N2] with gate and up interleaved in blocks of 128 columns, act is
// [M, N2 / 2] (gemm_tc.cu).  With row_scale (fp32 [M], may be null) both
// accumulators of row m are multiplied by row_scale[m] first.  Workspace as
// for gemm_tc with N = N2.
int gemm_silu_mul(void* act, const void* a, const void* b, const float* row_scale, int64_t M,
                  int64_t N2, int64_t K, int dtype, void* workspace, size_t ws_bytes,
                  void* stream);

// The persistent kernel's schedule for a problem on `sm_count` SMs (no device
// access): out[0..9] = grid, tiles, whole-tile rounds, first tail tile,
// halves, K splits, K blocks per split, tail work items, K blocks, workspace
// bytes (gemm_tc.cu).
int gemm_tc_schedule(int64_t M, int64_t N, int64_t K, int elem_bytes, int sm_count,
                     bool with_workspace, int64_t* out);

// Persistent tcgen05 GEMM on 8-bit operands (e4m3 or int8, kind::f8f6f4 /
// kind::i8) with the dequantisation epilogue C = (A * B) * scale_a * scale_b
// (gemm_tc.cu).  The caller has checked shapes, alignment and dtypes
// (scaled_tc_eligible); workspace as for gemm_tc.
int gemm_scaled_tc(void* c, const void* a, const void* b, const float* scale_a,
                   const float* scale_b, int64_t M, int64_t N, int64_t K, int in_dtype,
                   int out_dtype, int scale_mode, void* workspace, size_t ws_bytes, void* stream);
size_t gemm_scaled_tc_workspace_size(int64_t M, int64_t N, int64_t K, int sm_count);

// SIMT scaled GEMM for every shape (gemm_scaled_simt.cu).
int gemm_scaled_simt(void* c, const void* a, const void* b, const float* scale_a,
                     const float* scale_b, int64_t M, int64_t N, int64_t K, int in_dtype,
                     int out_dtype, int scale_mode, void* stream);

// Persistent tcgen05 GEMM on CTA pairs, 256 x 256 tiles (gemm_tc2.cu).
int gemm_tc2(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K, int dtype,
             void* stream);
// The same on 256 x 512 tiles (one 512-column accumulator per CTA).
int gemm_tc2_wide(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                  int dtype, void* stream);
// A pair kernel (256 x 512 tiles when `wide`, else 256 x 256) with
// gemm_silu_mul's epilogue (interleaved [K, N2] weight, act [M, N2 / 2],
// optional fp32 row scale).
int gemm_tc2_silu_mul(void* act, const void* a, const void* b, const float* row_scale, int64_t M,
                      int64_t N2, int64_t K, int dtype, bool wide, void* stream);

// Which kernel aotk_gemm_opt runs for a TMA-eligible 16-bit problem on
// `sm_count` SMs (pure host arithmetic): AOTK_PATH_SKINNY, AOTK_PATH_TC,
// AOTK_PATH_TC2 or AOTK_PATH_TC2_WIDE (gemm_dispatch.cu).
int gemm_opt_path(int64_t M, int64_t N, int64_t K, int sm_count, bool with_workspace);
int tc2_watchdog(uint32_t* status, bool clear);

// Persistent tcgen05 GEMM fused with an all-reduce of C over NVSwitch
// multicast memory (gemm_tc.cu).
int gemm_allreduce(const void* a, const void* b, int64_t M, int64_t N, int64_t K, int dtype,
                   const aotk_allreduce_buffers* bufs, void* stream);
int gemm_allreduce_tiles(int64_t M, int64_t N);

// Swap-AB split-K tcgen05 kernel for M <= kSkinnyMaxM (gemm_skinny.cu).
constexpr int64_t kSkinnyMaxM = 128;
int gemm_skinny(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K, int dtype,
                void* stream);

// SIMT kernel for every dtype and shape (gemm_simt.cu).
int gemm_simt(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K, int dtype,
              void* stream);

// Launches the bounded-wait self-test kernel (gemm_tc.cu).
int watchdog_selftest(void* stream);

// Watchdog words of the tensor-core kernels (OR-ed into *status).
int tc_watchdog(uint32_t* status, bool clear);
int skinny_watchdog(uint32_t* status, bool clear);

// Raises the dynamic shared-memory limit of `kernel` to `bytes` once per device.
int ensure_dynamic_smem(const void* kernel, int bytes, const DeviceInfo& info);

// Preconditions shared by the TMA-fed kernels: 16-bit dtype, K % 8 == 0,
// N % 8 == 0 (16-byte row strides), 16-byte aligned bases, 32-bit extents.
bool tc_eligible(const void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                 int dtype);
int check_tc_preconditions(const char* who, const void* c, const void* a, const void* b, int64_t M,
                           int64_t N, int64_t K, int dtype);

}  // namespace aotk
