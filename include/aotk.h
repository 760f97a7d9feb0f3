/*
 * aotk.h - C ABI of the B200 (sm_100a) dense-linear inference kernels.
 *
 * Every entry point takes plain device pointers, element counts and a CUDA
 * stream handle (cudaStream_t passed as void*, NULL = legacy default stream),
 * launches asynchronously on that stream and returns a status code.  No entry
 * point allocates device memory, synchronises the device or keeps state
 * between calls apart from per-device launch configuration set up on first
 * use.  Pointers must belong to the current device (cudaSetDevice).
 *
 * The operator names mirror the reference's torch operator library
 * (aot_kernel/csrc/registration.cc:10-25 of gongyisheng/inference-kernel):
 * each aotk_<op> is what the TORCH_LIBRARY kernel <op> does once its tensors
 * are reduced to pointers, so a torch binding is a thin adapter (see
 * aot_kernel/csrc/registration.cc in this package) and a non-torch caller
 * binds the same symbols through ctypes / cffi / dlopen.
 *
 * Layouts: all matrices are row-major and dense in the last dimension.
 * GEMM: C[M,N] = A[M,K] * B[K,N], 16-bit inputs, fp32 accumulation, one
 * rounding to the output type (the contract of ref.gemm = `a @ b`,
 * ref/gemm.py:4-5).
 */
#ifndef AOTK_H_
#define AOTK_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define AOTK_API __attribute__((visibility("default")))
#else
#define AOTK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types.  The 8-bit types are inputs of aotk_scaled_gemm only. */
enum aotk_dtype {
  AOTK_FLOAT32 = 0,
  AOTK_FLOAT16 = 1,
  AOTK_BFLOAT16 = 2,
  AOTK_FLOAT8_E4M3 = 3, /* OCP e4m3 "fn": bias 7, no infinities, 0x7F / 0xFF NaN */
  AOTK_INT8 = 4,
  AOTK_FLOAT8_E5M2 = 5  /* OCP e5m2: bias 15, IEEE-style infinities and NaNs */
};

/* Granularity of the dequantisation scales of aotk_scaled_gemm. */
enum aotk_scale_mode {
  AOTK_SCALE_TENSOR = 0, /* scale_a and scale_b each hold one fp32 value */
  AOTK_SCALE_ROW = 1     /* scale_a[M] per row of A, scale_b[N] per column of B */
};

/* Status codes returned by every entry point. */
enum aotk_status {
  AOTK_OK = 0,
  AOTK_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad stride   */
  AOTK_ERR_UNSUPPORTED = 2,      /* dtype / alignment this entry cannot serve  */
  AOTK_ERR_CUDA = 3,             /* a CUDA runtime call failed                 */
  AOTK_ERR_DEVICE = 4            /* current device is not an sm_100 part       */
};

/* Message describing the last non-OK status returned on the calling thread. */
AOTK_API const char* aotk_last_error(void);

/* Library version, major * 10000 + minor * 100 + patch. */
AOTK_API int aotk_version(void);

/* ---- activation -------------------------------------------------------- */

/* out[i] = x[i] / (1 + exp(-x[i])), computed in fp32, rounded once.
 * Replaces silu_forward(Tensor! out, Tensor x)
 * (aot_kernel/csrc/activation/silu.cu:22-41, registration.cc:14-15). */
AOTK_API int aotk_silu_forward(void* out, const void* x, int64_t n, int dtype, void* stream);

/* out[i] = max(x[i], 0).
 * Replaces relu_forward(Tensor! out, Tensor x)
 * (aot_kernel/csrc/activation/relu.cu:22-41, registration.cc:11-12). */
AOTK_API int aotk_relu_forward(void* out, const void* x, int64_t n, int dtype, void* stream);

/* out[r, c] = silu(gate[r, c]) * up[r, c] for r < rows, c < cols, computed in
 * fp32 and rounded once.  *_stride are element strides between rows, so gate
 * and up may be the two column halves of one fused [rows, 2*cols] GEMM output.
 * No reference counterpart: the reference composes ref.silu(gate) * up
 * (ref/activation.py:15-16). */
AOTK_API int aotk_silu_mul_forward(void* out, int64_t out_stride, const void* gate, int64_t gate_stride,
                          const void* up, int64_t up_stride, int64_t rows, int64_t cols,
                          int dtype, void* stream);

/* ---- norm ------------------------------------------------------------- */

/* out[r, :] = x[r, :] * rsqrt(mean(x[r, :]^2) + eps) * weight, fp32 math,
 * one rounding; x is [rows, cols] dense, weight is [cols].
 * Replaces rmsnorm_forward(Tensor! out, Tensor x, Tensor weight, float eps)
 * (aot_kernel/csrc/norm/rmsnorm.cu:185-239, registration.cc:17-18). */
AOTK_API int aotk_rmsnorm_forward(void* out, const void* x, const void* weight, int64_t rows,
                         int64_t cols, double eps, int dtype, void* stream);

/* h = x + residual rounded to `dtype`, written to residual_out, and
 * out = rmsnorm(h, weight, eps) as aotk_rmsnorm_forward computes it - one pass
 * over x and residual.  What the reference computes as ref.rmsnorm(x + r, w)
 * with the addition a separate 16-bit op (ref/norm.py:11-12); no fused
 * counterpart in the reference.  residual_out may alias residual. */
AOTK_API int aotk_add_rmsnorm_forward(void* out, void* residual_out, const void* x,
                                      const void* residual, const void* weight, int64_t rows,
                                      int64_t cols, double eps, int dtype, void* stream);

/* rstd[r] = rsqrt(mean(x[r, :]^2) + eps) in fp32 (rms_norm's row statistic,
 * for folding the normalisation into the next GEMM: see
 * aotk_gemm_silu_mul_rowscale).  x is [rows, cols] dense; one read of x.  No
 * reference counterpart. */
AOTK_API int aotk_rmsnorm_rstd(float* rstd, const void* x, int64_t rows, int64_t cols, double eps,
                               int dtype, void* stream);

/* ---- gemm ------------------------------------------------------------- */

/* Tensor-core GEMM for FLOAT16 / BFLOAT16 (FLOAT32 returns AOTK_ERR_UNSUPPORTED,
 * as the reference's gemm_opt rejects it).  Picks the skinny split-K tcgen05
 * kernel (M <= 128, except M > 96 with at least 3/4 of the SMs' worth of
 * 256-column tiles), a CTA-pair kernel (256 x 512 or 256 x 256 tiles) or the
 * persistent 1-CTA tcgen05 kernel (whichever aotk_gemm_path names for the
 * shape) or, for shapes TMA cannot address (K or N not a multiple of 8,
 * pointers not 16-byte aligned), the SIMT kernel.
 * Replaces gemm_opt(Tensor! out, Tensor a, Tensor b)
 * (aot_kernel/csrc/gemm/gemm_opt.cu:165-195, registration.cc:23-24). */
AOTK_API int aotk_gemm_opt(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                  int dtype, void* stream);

/* aotk_gemm_opt with caller-provided scratch.  Bytes needed for (M, N, K,
 * dtype) on the current device come from aotk_gemm_opt_workspace_size (0 when
 * the problem has no use for it).  With at least that many bytes, 256-byte
 * aligned (contents irrelevant: the call resets what it uses), the persistent
 * kernel splits the tiles of its partial last wave along K across all SMs and
 * reduces the fp32 partials in split order, so results stay deterministic.
 * With less, it behaves exactly like aotk_gemm_opt.  Calls that share a
 * workspace must be ordered on one stream.
 * Same reference counterpart as aotk_gemm_opt. */
AOTK_API int aotk_gemm_opt_ws(void* c, const void* a, const void* b, int64_t M, int64_t N,
                              int64_t K, int dtype, void* workspace, size_t workspace_bytes,
                              void* stream);
AOTK_API int aotk_gemm_opt_workspace_size(int64_t M, int64_t N, int64_t K, int dtype,
                                          size_t* bytes);

/* aotk_gemm_opt_ws for callers that cannot allocate device memory: hosts that
 * reach this library only through its C ABI (an FFI plugin with no CUDA
 * allocator of its own) and serving loops that must not call cudaMalloc,
 * which can synchronise the device.  The K-split scratch comes from a 24 MiB
 * array compiled into the library (device global memory, held on every GPU
 * where the library's kernels are loaded until the process exits).  The
 * entry point calls no cudaMalloc, cudaFree or allocating library routine.
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress; kept once it succeeds, retried while it fails);
 * make that first call before any stream capture.  Every call on a device shares the one array and resets the
 * part it needs, so calls whose kernels overlap on the GPU (different streams
 * without ordering) race and corrupt each other's results; order them on one
 * stream.  Problems needing more scratch than the array holds return
 * AOTK_ERR_UNSUPPORTED.  No counterpart in the reference. */
AOTK_API int aotk_gemm_opt_noalloc(void* c, const void* a, const void* b, int64_t M, int64_t N,
                                   int64_t K, int dtype, void* stream);

/* aotk_gemm_opt on host-resident operands: c_host[M, N] = a_host[M, K] *
 * b_host[K, N], FLOAT16 / BFLOAT16, through caller-provided device buffers
 * a_dev [M, K], b_dev [K, N], c_dev [M, N] of the same dtype.  B is copied in
 * first, then A in blocks of 128-row multiples (about M/8, the last eighth
 * in four smaller blocks to shorten the tail); the GEMM of
 * block i runs on `stream` as soon as its rows have landed while the next
 * block is still in flight, and block i of C is copied out while later blocks
 * compute, so inbound copies, GEMMs and outbound copies overlap.  Host
 * buffers should be page-locked for the copies to run asynchronously.  The
 * call is ordered on `stream` like one operation: work queued on `stream`
 * before it completes before its copies start, and work queued after it sees
 * c_host filled once the stream reaches it (synchronise before reading
 * c_host on the host).  Two copy streams and a few events per device are
 * created on first use and kept.  workspace as for aotk_gemm_opt_ws, sized by
 * aotk_gemm_host_workspace_size (NULL / 0: none).  No reference counterpart:
 * the reference's callers copy with torch and call gemm. */
AOTK_API int aotk_gemm_host(void* c_host, const void* a_host, const void* b_host, int64_t M,
                            int64_t N, int64_t K, int dtype, void* a_dev, void* b_dev, void* c_dev,
                            void* workspace, size_t workspace_bytes, void* stream);
AOTK_API int aotk_gemm_host_workspace_size(int64_t M, int64_t N, int64_t K, int dtype,
                                           size_t* bytes);

/* Any-dtype, any-shape GEMM (SIMT, fp32 accumulation).
 * Replaces gemm(Tensor! out, Tensor a, Tensor b)
 * (aot_kernel/csrc/gemm/gemm.cu:106-157, registration.cc:20-21). */
AOTK_API int aotk_gemm(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K,
              int dtype, void* stream);

/* Path-pinned variants of aotk_gemm_opt, for tests and benchmarks that must
 * exercise one kernel.  They return AOTK_ERR_UNSUPPORTED where the kernel's
 * preconditions (listed with each) do not hold instead of falling back. */

/* Persistent warp-specialised tcgen05 kernel, 128 x 256 tiles.
 * Needs FLOAT16/BFLOAT16, K % 8 == 0, N % 8 == 0, 16-byte aligned pointers. */
AOTK_API int aotk_gemm_tc(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                 int dtype, void* stream);

/* Persistent tcgen05 kernel on CTA pairs (cta_group::2, 2-CTA clusters),
 * 256 x 256 tiles: each CTA of a pair stages 128 rows of A and 128 columns of
 * B, one MMA of M = 256 reads both.  Same preconditions as aotk_gemm_tc. */
AOTK_API int aotk_gemm_tc2(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                           int dtype, void* stream);

/* The CTA-pair kernel on 256 x 512 tiles: two MMAs of M = 256, N = 256 per K
 * step into one 512-column accumulator per CTA (all of TMEM); each CTA stages
 * 128 rows of A and 256 columns of B.  Half the operand bytes per flop of the
 * 1-CTA kernel.  Same preconditions as aotk_gemm_tc. */
AOTK_API int aotk_gemm_tc2w(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                            int dtype, void* stream);

enum {
  AOTK_PATH_SIMT = 0,      /* aotk_gemm's SIMT kernel */
  AOTK_PATH_SKINNY = 1,    /* aotk_gemm_skinny */
  AOTK_PATH_TC = 2,        /* aotk_gemm_tc */
  AOTK_PATH_TC2_WIDE = 3,  /* aotk_gemm_tc2w */
  AOTK_PATH_TC2 = 4        /* aotk_gemm_tc2 */
};

/* The kernel aotk_gemm_opt_ws picks for a 16-bit problem on a device with
 * `sm_count` SMs, given a workspace (with_workspace != 0) or not; assumes
 * TMA-addressable operands (K % 8 == 0, N % 8 == 0, aligned pointers), else
 * the path is AOTK_PATH_SIMT.  Pure host arithmetic: a cost model of whole
 * rounds of tiles over the SMs (the 1-CTA kernel's cut last wave included)
 * with the pair kernel's measured throughput advantage.  No reference
 * counterpart (the reference has one tensor-core kernel). */
AOTK_API int aotk_gemm_path(int64_t M, int64_t N, int64_t K, int sm_count, int with_workspace,
                            int* path);

/* Skinny (decode) kernel: computes C^T = B^T A^T on tcgen05 with the weight
 * streamed by TMA and K split across a thread-block cluster whose partial sums
 * are reduced through distributed shared memory.  Same preconditions as
 * aotk_gemm_tc plus M <= 128. */
AOTK_API int aotk_gemm_skinny(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                     int dtype, void* stream);

/* ---- gemm fused with silu(gate) * up ------------------------------------ */

/* act[M, I] = silu(A @ W_gate) * (A @ W_up), fp32 accumulation, silu and
 * product in fp32 from the accumulators, one rounding - the gate/up
 * projection and the activation of a gated MLP in one kernel (the
 * [M, 2I] gate/up product never reaches memory).  b_gate_up is [K, 2I]
 * with W_gate and W_up interleaved in blocks of 128 columns:
 * columns [256j, 256j + 128) = W_gate[:, 128j : 128j + 128], columns
 * [256j + 128, 256j + 256) = W_up[:, 128j : 128j + 128]; I % 128 == 0,
 * K % 8 == 0, FLOAT16/BFLOAT16, 16-byte aligned pointers.  Runs on the
 * kernel aotk_gemm_path names for the [M, K] x [K, 2I] product - a
 * CTA-pair kernel (a 256 x 512 tile holds two gate/up block pairs, a 256 x
 * 256 one) or the persistent 1-CTA kernel (also for M <= 128); for the
 * latter a workspace of aotk_gemm_silu_mul_workspace_size bytes (0 when a
 * pair kernel is chosen) enables the K-split last wave as in
 * aotk_gemm_opt_ws.  No reference counterpart (the reference composes
 * ref.silu(a @ W_gate) * (a @ W_up)). */
AOTK_API int aotk_gemm_silu_mul(void* act, const void* a, const void* b_gate_up, int64_t M,
                                int64_t I, int64_t K, int dtype, void* workspace,
                                size_t workspace_bytes, void* stream);
AOTK_API int aotk_gemm_silu_mul_workspace_size(int64_t M, int64_t I, int64_t K, int dtype,
                                               size_t* bytes);

/* aotk_gemm_silu_mul with a per-row scale of both projections:
 * act[m, :] = silu(s_m (A @ W_gate)[m, :]) * (s_m (A @ W_up)[m, :]), s =
 * row_scale[M] fp32.  With A = x, s = rstd from aotk_rmsnorm_rstd and the
 * norm weight folded into the rows of the gate/up weight (W' = diag(w) W,
 * rounded once), this is the gate/up projection of rms_norm(x, w) without
 * the normalised activations ever being written: rms_norm as the GEMM's
 * prologue.  Numerically it differs from the unfused composition by where
 * the roundings fall (W' instead of the normalised x).  Same layout and
 * preconditions as aotk_gemm_silu_mul.  No reference counterpart. */
AOTK_API int aotk_gemm_silu_mul_rowscale(void* act, const void* a, const void* b_gate_up,
                                         const float* row_scale, int64_t M, int64_t I, int64_t K,
                                         int dtype, void* workspace, size_t workspace_bytes,
                                         void* stream);

/* ---- scaled (dequantising) 8-bit gemm ----------------------------------- */

/* C[M, N] = (acc[m, n] * scale_a[m]) * scale_b[n] rounded once to out_dtype,
 * acc = A[M, K] * B[K, N] with A and B both FLOAT8_E4M3 or both FLOAT8_E5M2
 * (fp32 accumulation) or both INT8 (exact integer accumulation, converted to
 * fp32).  scale_a /
 * scale_b are dense fp32 device vectors of 1 value each (AOTK_SCALE_TENSOR)
 * or M and N values (AOTK_SCALE_ROW).  out_dtype BFLOAT16, FLOAT16 or
 * FLOAT32.  K % 16 == 0, N % 16 == 0 and 16-byte aligned A, B, C, scale_b
 * run on the persistent tcgen05 kernel (kind::f8f6f4 / kind::i8, 128 x 256
 * tiles, the scales applied to the TMEM accumulator in the epilogue); other
 * shapes on a SIMT kernel.  A workspace of aotk_scaled_gemm_workspace_size
 * bytes enables the K-split last wave as in aotk_gemm_opt_ws (NULL / 0: none).
 * Replaces scaled_gemm(a, b, scale_a, scale_b, out_dtype, optimized)
 * (jit_kernel/gemm.py:199-248; kernels jit_kernel/gemm.py:86-123 and
 * 144-196: fp32 accumulator, acc * scale_a[:, None] * scale_b[None, :]). */
AOTK_API int aotk_scaled_gemm(void* c, const void* a, const void* b, const float* scale_a,
                              const float* scale_b, int64_t M, int64_t N, int64_t K, int in_dtype,
                              int out_dtype, int scale_mode, void* workspace,
                              size_t workspace_bytes, void* stream);
AOTK_API int aotk_scaled_gemm_workspace_size(int64_t M, int64_t N, int64_t K, int in_dtype,
                                             size_t* bytes);

/* Path-pinned variants of aotk_scaled_gemm: the tcgen05 kernel (returns
 * AOTK_ERR_UNSUPPORTED where its preconditions do not hold) and the SIMT
 * kernel (every shape). */
AOTK_API int aotk_scaled_gemm_tc(void* c, const void* a, const void* b, const float* scale_a,
                                 const float* scale_b, int64_t M, int64_t N, int64_t K,
                                 int in_dtype, int out_dtype, int scale_mode, void* workspace,
                                 size_t workspace_bytes, void* stream);
AOTK_API int aotk_scaled_gemm_simt(void* c, const void* a, const void* b, const float* scale_a,
                                   const float* scale_b, int64_t M, int64_t N, int64_t K,
                                   int in_dtype, int out_dtype, int scale_mode, void* stream);

/* ---- gemm fused with the tensor-parallel all-reduce -------------------- */

/* Buffers of one rank for aotk_gemm_allreduce.  `part` and the output are
 * [M, N] row-major buffers of the GEMM's dtype allocated symmetrically on all
 * ranks and bound to NVSwitch multicast objects (NVLS); the *_multicast
 * fields are the multicast addresses of the two.  counters / done are
 * zero-initialised uint32 words in memory every rank can access: counters
 * needs aotk_gemm_allreduce_tiles(M, N) entries, done one; peer_counters[r]
 * and peer_done[r] (device arrays of `world` pointers) are rank r's words as
 * mapped on this GPU.  epoch is 1 on the first call and grows by 1 per call,
 * identically on every rank. */
typedef struct aotk_allreduce_buffers {
  int rank;
  int world;
  void* part;
  uint64_t part_multicast;
  uint64_t out_multicast;
  uint32_t* counters;
  uint32_t* const* peer_counters;
  uint32_t* done;
  uint32_t* const* peer_done;
  uint32_t epoch;
} aotk_allreduce_buffers;

/* Number of output tiles (arrival counters) of an [M, N] aotk_gemm_allreduce. */
AOTK_API int aotk_gemm_allreduce_tiles(int64_t M, int64_t N, int64_t* tiles);

/* out = sum over ranks of A_r[M, K] * B_r[K, N], on every rank of a
 * tensor-parallel group (one process per GPU), in one kernel: each rank's
 * persistent tcgen05 GEMM stores its partial tiles into `part`, and as the
 * W partials of a tile arrive, the tile's owner rank (one of W, rotating) sums them
 * through the switch (multimem.ld_reduce, fp32 accumulation) and writes the
 * 16-bit result into every rank's output (multimem.st), overlapping the
 * transfer with the rest of the GEMM.  FLOAT16/BFLOAT16, K % 8 == 0,
 * N % 8 == 0.  All ranks must call with the same M, N, K, dtype and epoch;
 * every wait is bounded (~1 s) and a timeout sets watchdog bit 64.
 * Replaces the down projection + NCCL all-reduce of the tensor-parallel MLP
 * block (no reference counterpart: the reference has no multi-GPU code). */
AOTK_API int aotk_gemm_allreduce(const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                                 int dtype, const aotk_allreduce_buffers* bufs, void* stream);

/* The persistent tcgen05 kernel's tile schedule for an [M, N, K] problem of
 * elem_bytes-byte operands (2: fp16/bf16, 1: the scaled 8-bit GEMM) on a
 * device with sm_count SMs, with or without a K-split workspace; pure host
 * arithmetic, no device access.  out[10] receives: grid, tiles (128 x 256),
 * whole-tile rounds, first tail tile, halves (1: tail tiles run as two
 * 128 x 128 halves), K splits per tail tile, K blocks per split, tail work
 * items, K blocks, workspace bytes needed.  For tests and capacity planning. */
AOTK_API int aotk_gemm_schedule(int64_t M, int64_t N, int64_t K, int elem_bytes, int sm_count,
                                int with_workspace, int64_t* out);

/* Watchdog word of the tcgen05 kernels on `device`: a bit mask of pipeline
 * waits that gave up after their time limit (0 = healthy).  Persistent
 * kernel: 1 producer, 2 MMA, 4 epilogue, 64 peer / flag wait, 128 self-test,
 * 2048 K-split partials; skinny kernel: 8, 16, 32; CTA-pair kernel: 256,
 * 512, 1024.  Synchronises the
 * device.  clear != 0 resets it to 0 after reading. */
AOTK_API int aotk_watchdog_status(int device, uint32_t* status, int clear);

/* Runs the kernels' bounded waits with nothing to wait for - an mbarrier
 * phase no one completes, then a flag no one sets - on `stream`.  Each gives
 * up after about a second and sets watchdog bit 128 and 64 respectively; the
 * kernel then returns and the context stays usable.  Tests the failure path
 * without faulting or hanging the GPU.  No reference counterpart. */
AOTK_API int aotk_watchdog_selftest(void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AOTK_H_ */
