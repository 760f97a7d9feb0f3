/* The C ABI exercised from plain C (no torch, no CUDA headers): a host
 * program that links libaotk.so and calls entry points whose argument checks
 * complete before any device work, so it runs on a machine without a GPU.
 * Prints one line per check and exits non-zero on the first failure. */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "aotk.h"

static int expect(const char* what, int got, int want) {
  if (got != want) {
    printf("FAIL %s: status %d, expected %d (%s)\n", what, got, want, aotk_last_error());
    return 1;
  }
  printf("ok %s -> %d%s%s\n", what, got, got ? ": " : "", got ? aotk_last_error() : "");
  return 0;
}

int main(void) {
  char dummy[64];
  void* p = dummy; /* never dereferenced: every call below fails or returns early */
  int bad = 0;
  if (aotk_version() < 100) {
    printf("FAIL version %d\n", aotk_version());
    return 1;
  }
  bad |= expect("gemm_opt fp32 rejected", aotk_gemm_opt(p, p, p, 4, 4, 4, AOTK_FLOAT32, NULL),
                AOTK_ERR_UNSUPPORTED);
  bad |= expect("gemm negative M", aotk_gemm(p, p, p, -1, 4, 4, AOTK_BFLOAT16, NULL),
                AOTK_ERR_INVALID_ARGUMENT);
  bad |= expect("gemm empty is a no-op", aotk_gemm_opt(p, p, p, 0, 16, 16, AOTK_BFLOAT16, NULL),
                AOTK_OK);
  bad |= expect("rmsnorm null output",
                aotk_rmsnorm_forward(NULL, p, p, 4, 8, 1e-6, AOTK_BFLOAT16, NULL),
                AOTK_ERR_INVALID_ARGUMENT);
  bad |= expect("scaled_gemm 16-bit input rejected",
                aotk_scaled_gemm(p, p, p, (const float*)p, (const float*)p, 4, 4, 4,
                                 AOTK_BFLOAT16, AOTK_BFLOAT16, AOTK_SCALE_TENSOR, NULL, 0, NULL),
                AOTK_ERR_UNSUPPORTED);
  bad |= expect("gemm_host fp32 rejected",
                aotk_gemm_host(p, p, p, 4, 4, 4, AOTK_FLOAT32, p, p, p, NULL, 0, NULL),
                AOTK_ERR_UNSUPPORTED);
  int64_t sched[12];
  memset(sched, 0, sizeof(sched));
  bad |= expect("schedule of 8192^3 on 148 SMs",
                aotk_gemm_schedule(8192, 8192, 8192, 2, 148, 1, sched), AOTK_OK);
  if (sched[0] != 148 || sched[1] != 2048) {
    printf("FAIL schedule grid %lld tiles %lld\n", (long long)sched[0], (long long)sched[1]);
    bad = 1;
  }
  return bad;
}
