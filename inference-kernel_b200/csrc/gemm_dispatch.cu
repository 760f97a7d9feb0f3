// C-ABI GEMM entry points and the path selection of aotk_gemm_opt.
//
// Path choice (all fp32 accumulation, one rounding per output; with a
// workspace the persistent kernel also splits its partial last wave along K):
//   16-bit, TMA-addressable, M <= 128  -> skinny swap-AB split-K kernel
//                                          (decode; HBM-bound on the weight)
//   16-bit, TMA-addressable, M > 128   -> the CTA-pair kernel on 256 x 512
//                                          or 256 x 256 tiles or the
//                                          persistent 1-CTA kernel on 128 x
//                                          256 tiles, by the cost model of
//                                          gemm_opt_path
//   anything else                       -> SIMT kernel
// aotk_scaled_gemm (8-bit inputs): K % 16 == 0, N % 16 == 0, aligned -> the
// persistent kernel on kind::f8f6f4 / kind::i8, else its SIMT kernel.
// The reference routes in its Python wrapper instead: fp16/bf16 with
// K % 16 == 0 to gemm_opt, everything else to the naive tier
// (aot_kernel/gemm.py:39-42).
#include <cuda_runtime.h>

#include <mutex>

#include "common.h"
#include "gemm_internal.h"

namespace aotk {

namespace {

struct SmemKey {
  const void* kernel;
  int device;
};

std::mutex g_smem_mu;
SmemKey g_smem_done[256];
int g_smem_count = 0;

int validate_common(const char* who, const void* c, const void* a, const void* b, int64_t M,
                    int64_t N, int64_t K, int dtype) {
  if (M < 0 || N < 0 || K < 0)
    return fail(AOTK_ERR_INVALID_ARGUMENT, "%s: negative size (M=%lld N=%lld K=%lld)", who,
                (long long)M, (long long)N, (long long)K);
  if (!valid_dtype(dtype)) return fail(AOTK_ERR_UNSUPPORTED, "%s: unsupported dtype %d", who, dtype);
  if (M > 0 && N > 0 && (!c || (K > 0 && (!a || !b))))
    return fail(AOTK_ERR_INVALID_ARGUMENT, "%s: null pointer", who);
  return AOTK_OK;
}

// C = 0 when K == 0 (an empty sum), matching `a @ b` for an empty inner dim.
int zero_output(void* c, int64_t M, int64_t N, int dtype, void* stream) {
  cudaError_t e = cudaMemsetAsync(c, 0, (size_t)(M * N * elem_size(dtype)),
                                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(AOTK_ERR_CUDA, "gemm: cudaMemsetAsync: %s", cudaGetErrorString(e));
  return AOTK_OK;
}

}  // namespace

int ensure_dynamic_smem(const void* kernel, int bytes, const DeviceInfo& info) {
  std::lock_guard<std::mutex> lock(g_smem_mu);
  for (int i = 0; i < g_smem_count; ++i) {
    if (g_smem_done[i].kernel == kernel && g_smem_done[i].device == info.device) return AOTK_OK;
  }
  if (bytes > info.max_smem_optin)
    return fail(AOTK_ERR_DEVICE, "kernel needs %d bytes of shared memory, device allows %d", bytes,
                info.max_smem_optin);
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess)
    return fail(AOTK_ERR_CUDA, "cudaFuncSetAttribute(smem=%d): %s", bytes, cudaGetErrorString(e));
  if (g_smem_count < 256) g_smem_done[g_smem_count++] = SmemKey{kernel, info.device};
  return AOTK_OK;
}

bool tc_eligible(const void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                 int dtype) {
  if (dtype != AOTK_FLOAT16 && dtype != AOTK_BFLOAT16) return false;
  if (K % 8 != 0 || N % 8 != 0) return false;
  if (M >= (1LL << 31) || N >= (1LL << 31) || K >= (1LL << 31)) return false;
  return aligned16(a) && aligned16(b) && aligned16(c);
}

int check_tc_preconditions(const char* who, const void* c, const void* a, const void* b, int64_t M,
                           int64_t N, int64_t K, int dtype) {
  if (int st = validate_common(who, c, a, b, M, N, K, dtype)) return st;
  if (M == 0 || N == 0 || K == 0)
    return fail(AOTK_ERR_INVALID_ARGUMENT, "%s: empty problem (M=%lld N=%lld K=%lld)", who,
                (long long)M, (long long)N, (long long)K);
  if (!tc_eligible(c, a, b, M, N, K, dtype))
    return fail(AOTK_ERR_UNSUPPORTED,
                "%s: needs fp16/bf16, K %% 8 == 0, N %% 8 == 0 and 16-byte aligned pointers "
                "(dtype=%d M=%lld N=%lld K=%lld)",
                who, dtype, (long long)M, (long long)N, (long long)K);
  return AOTK_OK;
}

// Cost model behind aotk_gemm_opt's choice among the 1-CTA kernel (128 x 256
// tiles over all SMs, its partial last wave cut into N halves or K splits by
// plan_tc) and the CTA-pair kernel on 256 x 256 or 256 x 512 tiles (over SM
// pairs).  Time is counted in rounds of 128 x 256 x K work per SM; a 256 x 256
// pair tile is one such unit per SM, a 256 x 512 one two; all three kernels
// cut a partial last round of at most half their slots into N halves.  The
// pair kernels'
// throughput advantage on whole rounds is what was measured on B200 with each
// kernel running back to back for 0.6 s at the 1 kW power cap (as GEMMs run
// inside a model step): 256 x 256 1.04-1.08x, 256 x 512 1.07-1.10x the 1-CTA
// kernel (8192^3, 4096 x 8192 x 57344, 8192 x 4096 x 28672, 4096 x 28672 x
// 8192).  Below K = 4096 the pair kernels are not chosen (untimed there; the
// 256 x 512 tile's epilogue is not overlapped with the next tile).  The cut
// last wave of the 1-CTA kernel is charged more than its share of the work
// (N halves 0.6 of a round, a 4-way K split 0.35: tails run at lower
// efficiency than whole tiles).  A pair kernel is chosen when it beats the
// 1-CTA kernel's cost by 2 %.
int gemm_opt_path(int64_t M, int64_t N, int64_t K, int sm_count, bool with_workspace) {
  constexpr double kPairGain = 1.05;
  constexpr double kWideGain = 1.09;
  constexpr double kMargin = 0.98;
  if (M <= kSkinnyMaxM) {
    // M in (96, 128]: the 1-CTA kernel (one 128-row band of tiles, B read
    // once, no split-K reduction) beats the skinny kernel, whose cluster
    // reduction grows with M, once its whole tiles fill 3/4 of the SMs
    // (measured at 128 x 4096 x 28672: 54.5 vs 61.2 us; with 16-32 tiles
    // the skinny kernel stays ahead by 1.4-1.6x).
    const int64_t tiles = (N + 255) / 256;
    return M > 96 && 4 * tiles >= 3 * static_cast<int64_t>(sm_count) ? AOTK_PATH_TC
                                                                      : AOTK_PATH_SKINNY;
  }
  if (K < 4096 || sm_count < 2) return AOTK_PATH_TC;
  int64_t sch[10];
  if (gemm_tc_schedule(M, N, K, 2, sm_count, with_workspace, sch) != AOTK_OK) return AOTK_PATH_TC;
  double tc = static_cast<double>(sch[2]);  // rounds of whole tiles
  if (sch[4]) tc += 0.6;                    // last wave as N halves
  else if (sch[5] > 1) tc += 0.35;          // last wave as K splits
  const int64_t pairs = sm_count / 2;
  // Rounds of pair tiles: a last round of at most half the pairs runs as N
  // halves (charged 0.6 of a round, as for the 1-CTA kernel).
  auto rounds = [&](int64_t tiles) {
    const int64_t rem = tiles % pairs;
    return static_cast<double>(tiles / pairs) + (rem == 0 ? 0.0 : (2 * rem <= pairs ? 0.6 : 1.0));
  };
  const double pair = rounds(((M + 255) / 256) * ((N + 255) / 256)) / kPairGain;
  const double wide = 2.0 * rounds(((M + 255) / 256) * ((N + 511) / 512)) / kWideGain;
  if (wide <= pair && wide < kMargin * tc) return AOTK_PATH_TC2_WIDE;
  if (pair < wide && pair < kMargin * tc) return AOTK_PATH_TC2;
  return AOTK_PATH_TC;
}

}  // namespace aotk

extern "C" int aotk_gemm_opt_ws(void* c, const void* a, const void* b, int64_t M, int64_t N,
                                int64_t K, int dtype, void* workspace, size_t workspace_bytes,
                                void* stream) {
  using namespace aotk;
  if (int st = validate_common("aotk_gemm_opt", c, a, b, M, N, K, dtype)) return st;
  if (dtype == AOTK_FLOAT32)
    return fail(AOTK_ERR_UNSUPPORTED, "aotk_gemm_opt: tensor-core path supports fp16/bf16 only");
  if (M == 0 || N == 0) return AOTK_OK;
  if (K == 0) return zero_output(c, M, N, dtype, stream);
  if (tc_eligible(c, a, b, M, N, K, dtype)) {
    DeviceInfo info;
    if (int st = current_device_info(&info)) return st;
    const bool with_ws =
        workspace != nullptr && workspace_bytes >= gemm_tc_workspace_size(M, N, K, info.sm_count);
    switch (gemm_opt_path(M, N, K, info.sm_count, with_ws)) {
      case AOTK_PATH_SKINNY:
        return gemm_skinny(c, a, b, M, N, K, dtype, stream);
      case AOTK_PATH_TC2_WIDE:
        return gemm_tc2_wide(c, a, b, M, N, K, dtype, stream);
      case AOTK_PATH_TC2:
        return gemm_tc2(c, a, b, M, N, K, dtype, stream);
      default:
        return gemm_tc(c, a, b, M, N, K, dtype, workspace, workspace_bytes, stream);
    }
  }
  return gemm_simt(c, a, b, M, N, K, dtype, stream);
}

extern "C" int aotk_gemm_opt(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                             int dtype, void* stream) {
  return aotk_gemm_opt_ws(c, a, b, M, N, K, dtype, nullptr, 0, stream);
}

extern "C" int aotk_gemm_opt_workspace_size(int64_t M, int64_t N, int64_t K, int dtype,
                                            size_t* bytes) {
  using namespace aotk;
  if (!bytes) return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_gemm_opt_workspace_size: null pointer");
  *bytes = 0;
  if (M < 0 || N < 0 || K < 0)
    return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_gemm_opt_workspace_size: negative size");
  if (dtype != AOTK_FLOAT16 && dtype != AOTK_BFLOAT16) return AOTK_OK;
  if (M <= kSkinnyMaxM || K % 8 != 0 || N % 8 != 0) return AOTK_OK;
  DeviceInfo info;
  if (int st = current_device_info(&info)) return st;
  // The pair kernels need no scratch; one is chosen without a workspace
  // whenever it is chosen with one (the 1-CTA kernel only gets slower).
  if (gemm_opt_path(M, N, K, info.sm_count, true) != AOTK_PATH_TC) return AOTK_OK;
  *bytes = gemm_tc_workspace_size(M, N, K, info.sm_count);
  return AOTK_OK;
}

extern "C" int aotk_gemm(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                         int dtype, void* stream) {
  using namespace aotk;
  if (int st = validate_common("aotk_gemm", c, a, b, M, N, K, dtype)) return st;
  if (M == 0 || N == 0) return AOTK_OK;
  return gemm_simt(c, a, b, M, N, K, dtype, stream);
}

extern "C" int aotk_gemm_tc(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                            int dtype, void* stream) {
  return aotk::gemm_tc(c, a, b, M, N, K, dtype, nullptr, 0, stream);
}

extern "C" int aotk_gemm_tc2(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                             int dtype, void* stream) {
  return aotk::gemm_tc2(c, a, b, M, N, K, dtype, stream);
}

extern "C" int aotk_gemm_tc2w(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                              int dtype, void* stream) {
  return aotk::gemm_tc2_wide(c, a, b, M, N, K, dtype, stream);
}

extern "C" int aotk_gemm_path(int64_t M, int64_t N, int64_t K, int sm_count, int with_workspace,
                              int* path) {
  using namespace aotk;
  if (!path || M <= 0 || N <= 0 || K <= 0 || sm_count <= 0)
    return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_gemm_path: bad arguments");
  if (K % 8 != 0 || N % 8 != 0 || M >= (1LL << 31) || N >= (1LL << 31) || K >= (1LL << 31)) {
    *path = AOTK_PATH_SIMT;
    return AOTK_OK;
  }
  *path = gemm_opt_path(M, N, K, sm_count, with_workspace != 0);
  return AOTK_OK;
}

extern "C" int aotk_gemm_skinny(void* c, const void* a, const void* b, int64_t M, int64_t N,
                                int64_t K, int dtype, void* stream) {
  return aotk::gemm_skinny(c, a, b, M, N, K, dtype, stream);
}

extern "C" int aotk_gemm_silu_mul_workspace_size(int64_t M, int64_t I, int64_t K, int dtype,
                                                 size_t* bytes) {
  using namespace aotk;
  if (!bytes) return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_gemm_silu_mul_workspace_size: null pointer");
  *bytes = 0;
  if (M < 0 || I < 0 || K < 0)
    return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_gemm_silu_mul_workspace_size: negative size");
  if (dtype != AOTK_FLOAT16 && dtype != AOTK_BFLOAT16) return AOTK_OK;
  DeviceInfo info;
  if (int st = current_device_info(&info)) return st;
  if (M > kSkinnyMaxM && gemm_opt_path(M, 2 * I, K, info.sm_count, true) != AOTK_PATH_TC)
    return AOTK_OK;
  *bytes = gemm_tc_workspace_size(M, 2 * I, K, info.sm_count);
  return AOTK_OK;
}

namespace aotk {
namespace {

// gemm_silu_mul on the kernel aotk_gemm_path names for the [K, 2I] product:
// a CTA-pair kernel or the persistent 1-CTA kernel (also for M <= 128, which
// has no skinny silu_mul variant).
int silu_mul_dispatch(void* act, const void* a, const void* b, const float* row_scale, int64_t M,
                      int64_t N2, int64_t K, int dtype, void* workspace, size_t workspace_bytes,
                      void* stream) {
  if (tc_eligible(act, a, b, M, N2, K, dtype) && N2 % 256 == 0 && M > kSkinnyMaxM) {
    DeviceInfo info;
    if (int st = current_device_info(&info)) return st;
    const bool with_ws = workspace != nullptr &&
                         workspace_bytes >= gemm_tc_workspace_size(M, N2, K, info.sm_count);
    const int path = gemm_opt_path(M, N2, K, info.sm_count, with_ws);
    if (path == AOTK_PATH_TC2_WIDE || path == AOTK_PATH_TC2)
      return gemm_tc2_silu_mul(act, a, b, row_scale, M, N2, K, dtype, path == AOTK_PATH_TC2_WIDE,
                               stream);
  }
  return gemm_silu_mul(act, a, b, row_scale, M, N2, K, dtype, workspace, workspace_bytes, stream);
}

}  // namespace
}  // namespace aotk

extern "C" int aotk_gemm_silu_mul(void* act, const void* a, const void* b_gate_up, int64_t M,
                                  int64_t I, int64_t K, int dtype, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  using namespace aotk;
  if (I < 0) return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_gemm_silu_mul: negative size");
  if (M == 0 || I == 0) return AOTK_OK;
  return silu_mul_dispatch(act, a, b_gate_up, nullptr, M, 2 * I, K, dtype, workspace,
                           workspace_bytes, stream);
}

extern "C" int aotk_gemm_silu_mul_rowscale(void* act, const void* a, const void* b_gate_up,
                                           const float* row_scale, int64_t M, int64_t I, int64_t K,
                                           int dtype, void* workspace, size_t workspace_bytes,
                                           void* stream) {
  using namespace aotk;
  if (I < 0) return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_gemm_silu_mul_rowscale: negative size");
  if (M == 0 || I == 0) return AOTK_OK;
  if (!row_scale)
    return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_gemm_silu_mul_rowscale: null row_scale");
  return silu_mul_dispatch(act, a, b_gate_up, row_scale, M, 2 * I, K, dtype, workspace,
                           workspace_bytes, stream);
}

namespace aotk {
namespace {

bool scaled_in_dtype(int d) {
  return d == AOTK_FLOAT8_E4M3 || d == AOTK_FLOAT8_E5M2 || d == AOTK_INT8;
}

int validate_scaled(const char* who, const void* c, const void* a, const void* b, const float* sa,
                    const float* sb, int64_t M, int64_t N, int64_t K, int in_dtype, int out_dtype,
                    int scale_mode) {
  if (M < 0 || N < 0 || K < 0)
    return fail(AOTK_ERR_INVALID_ARGUMENT, "%s: negative size (M=%lld N=%lld K=%lld)", who,
                (long long)M, (long long)N, (long long)K);
  if (!scaled_in_dtype(in_dtype))
    return fail(AOTK_ERR_UNSUPPORTED, "%s: input dtype %d is not FLOAT8_E4M3, FLOAT8_E5M2 or INT8",
                who, in_dtype);
  if (!valid_dtype(out_dtype))
    return fail(AOTK_ERR_UNSUPPORTED, "%s: unsupported output dtype %d", who, out_dtype);
  if (scale_mode != AOTK_SCALE_TENSOR && scale_mode != AOTK_SCALE_ROW)
    return fail(AOTK_ERR_INVALID_ARGUMENT, "%s: unknown scale mode %d", who, scale_mode);
  if (M > 0 && N > 0 && (!c || !sa || !sb || (K > 0 && (!a || !b))))
    return fail(AOTK_ERR_INVALID_ARGUMENT, "%s: null pointer", who);
  return AOTK_OK;
}

// The tcgen05 kernel reads A / B rows through TMA (16-byte row strides: K and
// N multiples of 16 bytes) and B's scales as float4.
bool scaled_tc_eligible(const void* c, const void* a, const void* b, const float* sb, int64_t M,
                        int64_t N, int64_t K, int scale_mode) {
  if (K <= 0 || K % 16 != 0 || N % 16 != 0) return false;
  if (M >= (1LL << 31) || N >= (1LL << 31) || K >= (1LL << 31)) return false;
  if (scale_mode == AOTK_SCALE_ROW && !aligned16(sb)) return false;
  return aligned16(a) && aligned16(b) && aligned16(c);
}

}  // namespace
}  // namespace aotk

extern "C" int aotk_scaled_gemm_workspace_size(int64_t M, int64_t N, int64_t K, int in_dtype,
                                               size_t* bytes) {
  using namespace aotk;
  if (!bytes) return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_scaled_gemm_workspace_size: null pointer");
  *bytes = 0;
  if (M < 0 || N < 0 || K < 0)
    return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_scaled_gemm_workspace_size: negative size");
  if (!scaled_in_dtype(in_dtype)) return AOTK_OK;
  if (K % 16 != 0 || N % 16 != 0) return AOTK_OK;
  DeviceInfo info;
  if (int st = current_device_info(&info)) return st;
  *bytes = gemm_scaled_tc_workspace_size(M, N, K, info.sm_count);
  return AOTK_OK;
}

extern "C" int aotk_scaled_gemm_tc(void* c, const void* a, const void* b, const float* scale_a,
                                   const float* scale_b, int64_t M, int64_t N, int64_t K,
                                   int in_dtype, int out_dtype, int scale_mode, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  using namespace aotk;
  const char* who = "aotk_scaled_gemm_tc";
  if (int st = validate_scaled(who, c, a, b, scale_a, scale_b, M, N, K, in_dtype, out_dtype,
                               scale_mode))
    return st;
  if (M == 0 || N == 0 || K == 0)
    return fail(AOTK_ERR_INVALID_ARGUMENT, "%s: empty problem (M=%lld N=%lld K=%lld)", who,
                (long long)M, (long long)N, (long long)K);
  if (!scaled_tc_eligible(c, a, b, scale_b, M, N, K, scale_mode))
    return fail(AOTK_ERR_UNSUPPORTED,
                "%s: needs K %% 16 == 0, N %% 16 == 0 and 16-byte aligned A, B, C and row scales "
                "(M=%lld N=%lld K=%lld)",
                who, (long long)M, (long long)N, (long long)K);
  return gemm_scaled_tc(c, a, b, scale_a, scale_b, M, N, K, in_dtype, out_dtype, scale_mode,
                        workspace, workspace_bytes, stream);
}

extern "C" int aotk_scaled_gemm_simt(void* c, const void* a, const void* b, const float* scale_a,
                                     const float* scale_b, int64_t M, int64_t N, int64_t K,
                                     int in_dtype, int out_dtype, int scale_mode, void* stream) {
  using namespace aotk;
  if (int st = validate_scaled("aotk_scaled_gemm_simt", c, a, b, scale_a, scale_b, M, N, K,
                               in_dtype, out_dtype, scale_mode))
    return st;
  return gemm_scaled_simt(c, a, b, scale_a, scale_b, M, N, K, in_dtype, out_dtype, scale_mode,
                          stream);
}

extern "C" int aotk_scaled_gemm(void* c, const void* a, const void* b, const float* scale_a,
                                const float* scale_b, int64_t M, int64_t N, int64_t K, int in_dtype,
                                int out_dtype, int scale_mode, void* workspace,
                                size_t workspace_bytes, void* stream) {
  using namespace aotk;
  if (int st = validate_scaled("aotk_scaled_gemm", c, a, b, scale_a, scale_b, M, N, K, in_dtype,
                               out_dtype, scale_mode))
    return st;
  if (M == 0 || N == 0) return AOTK_OK;
  if (K == 0) return zero_output(c, M, N, out_dtype, stream);
  if (scaled_tc_eligible(c, a, b, scale_b, M, N, K, scale_mode))
    return gemm_scaled_tc(c, a, b, scale_a, scale_b, M, N, K, in_dtype, out_dtype, scale_mode,
                          workspace, workspace_bytes, stream);
  return gemm_scaled_simt(c, a, b, scale_a, scale_b, M, N, K, in_dtype, out_dtype, scale_mode,
                          stream);
}

extern "C" int aotk_gemm_schedule(int64_t M, int64_t N, int64_t K, int elem_bytes, int sm_count,
                                  int with_workspace, int64_t* out) {
  using namespace aotk;
  if (!out) return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_gemm_schedule: null pointer");
  return gemm_tc_schedule(M, N, K, elem_bytes, sm_count, with_workspace != 0, out);
}

extern "C" int aotk_gemm_allreduce_tiles(int64_t M, int64_t N, int64_t* tiles) {
  using namespace aotk;
  if (!tiles || M < 0 || N < 0)
    return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_gemm_allreduce_tiles: bad arguments");
  *tiles = gemm_allreduce_tiles(M, N);
  return AOTK_OK;
}

extern "C" int aotk_gemm_allreduce(const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                                   int dtype, const aotk_allreduce_buffers* bufs, void* stream) {
  return aotk::gemm_allreduce(a, b, M, N, K, dtype, bufs, stream);
}

extern "C" int aotk_watchdog_status(int device, uint32_t* status, int clear) {
  using namespace aotk;
  if (!status) return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_watchdog_status: null pointer");
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e == cudaSuccess) e = cudaSetDevice(device);
  if (e != cudaSuccess) return fail(AOTK_ERR_CUDA, "aotk_watchdog_status: %s", cudaGetErrorString(e));
  *status = 0;
  int st = tc_watchdog(status, clear != 0);
  if (st == AOTK_OK) st = skinny_watchdog(status, clear != 0);
  if (st == AOTK_OK) st = tc2_watchdog(status, clear != 0);
  cudaSetDevice(prev);
  return st;
}

extern "C" int aotk_watchdog_selftest(void* stream) { return aotk::watchdog_selftest(stream); }
