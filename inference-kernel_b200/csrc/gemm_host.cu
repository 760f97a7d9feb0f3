// GEMM on host-resident operands: C_host = A_host * B_host with the
// host <-> device transfers overlapped with the tensor-core work.
//
// A caller whose matrices live in host memory would otherwise copy A and B
// in, run the GEMM and copy C out one after another, so the PCIe link idles
// during the GEMM and carries one direction at a time.  Here A is cut into
// row blocks: B goes in first, then each A block; the GEMM of block i starts
// as soon as A_i has landed (the copy of A_{i+1} continues meanwhile), and the
// copy-out of C_i starts as soon as its GEMM ends, in the other direction of
// the full-duplex link.  The step then costs about the inbound bytes at link
// speed plus one block's GEMM and copy-out.
//
// Two copy streams per device (inbound, outbound) and a pool of events are
// created on first use and kept (calls on one device are serialised while
// they enqueue, see gemm_host); the GEMM blocks run on the caller's stream,
// which at return is ordered after the last copy-out, so the call behaves as
// one stream-ordered operation.  Host buffers should be page-locked
// (cudaHostAlloc / cudaHostRegister) for the copies to overlap.
#include <cuda_runtime.h>

#include <mutex>

#include "common.h"
#include "gemm_internal.h"

extern "C" int aotk_gemm_opt_ws(void* c, const void* a, const void* b, int64_t M, int64_t N,
                                int64_t K, int dtype, void* workspace, size_t workspace_bytes,
                                void* stream);
extern "C" int aotk_gemm_opt_workspace_size(int64_t M, int64_t N, int64_t K, int dtype,
                                            size_t* bytes);

namespace aotk {
namespace {

constexpr int kMaxDevices = 64;
constexpr int kMaxBlocks = 16;
constexpr int kRowAlign = 128;  // the tcgen05 tile height

struct HostPipe {
  std::mutex mu;  // one call's enqueue sequence at a time (the events are shared)
  cudaStream_t in = nullptr, out = nullptr;
  cudaEvent_t start = nullptr, end = nullptr;
  cudaEvent_t a_ready[kMaxBlocks] = {};
  cudaEvent_t c_ready[kMaxBlocks] = {};
  int status = AOTK_OK;
};

HostPipe g_pipe[kMaxDevices];
std::once_flag g_pipe_once[kMaxDevices];

int pipe_for(int device, HostPipe** p) {
  if (device < 0 || device >= kMaxDevices)
    return fail(AOTK_ERR_CUDA, "device ordinal %d out of range", device);
  std::call_once(g_pipe_once[device], [device] {
    HostPipe& h = g_pipe[device];
    cudaError_t e = cudaStreamCreateWithFlags(&h.in, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&h.out, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h.start, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h.end, cudaEventDisableTiming);
    for (int i = 0; i < kMaxBlocks && e == cudaSuccess; ++i) {
      e = cudaEventCreateWithFlags(&h.a_ready[i], cudaEventDisableTiming);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h.c_ready[i], cudaEventDisableTiming);
    }
    if (e != cudaSuccess)
      h.status = fail(AOTK_ERR_CUDA, "aotk_gemm_host: stream/event setup: %s", cudaGetErrorString(e));
  });
  if (g_pipe[device].status != AOTK_OK) return g_pipe[device].status;
  *p = &g_pipe[device];
  return AOTK_OK;
}

// Row blocks of A: about M/8 rows each (whole 128-row tiles), except that
// the last eighth is cut in four.  Every block after the last inbound byte
// is tail - its GEMM and its copy-out - so the last blocks are kept small,
// while the bulk stays in large blocks whose per-copy and per-launch cost is
// amortised (at M = N = K = 8192 on B200, sixteen equal blocks took 6.06 ms
// per call against 5.82 ms for eight; seven of 1024 rows and four of 256
// took 5.94 ms against 6.00 ms for eight equal blocks on the same box).
// Returns the number of blocks.
int block_plan(int64_t M, int64_t (&rows)[kMaxBlocks]) {
  auto up = [](int64_t r) {
    r = (r + kRowAlign - 1) / kRowAlign * kRowAlign;
    return r < kRowAlign ? static_cast<int64_t>(kRowAlign) : r;
  };
  const int64_t big = up((M + 7) / 8);
  int n = 0;
  int64_t left = M;
  while (left > big && n < 8) {
    rows[n++] = big;
    left -= big;
  }
  const int64_t small = up((left + 3) / 4);
  while (left > 0 && n < kMaxBlocks - 1) {
    rows[n] = left < small ? left : small;
    left -= rows[n++];
  }
  if (left > 0) rows[n++] = left;  // not reached for M > 0: at most 8 + 4 blocks
  return n;
}

#define AOTK_HOST_CHECK(expr)                                                                  \
  do {                                                                                         \
    cudaError_t e_ = (expr);                                                                   \
    if (e_ != cudaSuccess)                                                                     \
      return fail(AOTK_ERR_CUDA, "aotk_gemm_host: %s: %s", #expr, cudaGetErrorString(e_));    \
  } while (0)

int gemm_host(void* c_host, const void* a_host, const void* b_host, int64_t M, int64_t N,
              int64_t K, int dtype, void* a_dev, void* b_dev, void* c_dev, void* workspace,
              size_t workspace_bytes, void* stream_v) {
  if (M < 0 || N < 0 || K < 0)
    return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_gemm_host: negative size");
  if (dtype != AOTK_FLOAT16 && dtype != AOTK_BFLOAT16)
    return fail(AOTK_ERR_UNSUPPORTED, "aotk_gemm_host: fp16/bf16 only (dtype %d)", dtype);
  if (M == 0 || N == 0) return AOTK_OK;
  if (!c_host || !c_dev || (K > 0 && (!a_host || !b_host || !a_dev || !b_dev)))
    return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_gemm_host: null pointer");
  int device = 0;
  AOTK_HOST_CHECK(cudaGetDevice(&device));
  HostPipe* p = nullptr;
  if (int st = pipe_for(device, &p)) return st;
  // Calls from several host threads enqueue one after another: each call's
  // event records and the waits on them are issued together, so a wait never
  // picks up another call's record.  The copies of calls on one device share
  // the two copy streams and therefore run in call order.
  std::lock_guard<std::mutex> lock(p->mu);
  cudaStream_t s = static_cast<cudaStream_t>(stream_v);
  const size_t es = 2;
  int64_t rows[kMaxBlocks];
  const int nblocks = block_plan(M, rows);

  // Everything already queued on the caller's stream (an earlier call's
  // GEMMs, which read a_dev / b_dev and write c_dev) precedes the copies.
  AOTK_HOST_CHECK(cudaEventRecord(p->start, s));
  AOTK_HOST_CHECK(cudaStreamWaitEvent(p->in, p->start, 0));
  AOTK_HOST_CHECK(cudaStreamWaitEvent(p->out, p->start, 0));
  if (K > 0)
    AOTK_HOST_CHECK(cudaMemcpyAsync(b_dev, b_host, static_cast<size_t>(K) * N * es,
                                    cudaMemcpyHostToDevice, p->in));
  int64_t r0 = 0;
  for (int i = 0; i < nblocks; r0 += rows[i], ++i) {
    const int64_t m = rows[i];
    if (K > 0)
      AOTK_HOST_CHECK(cudaMemcpyAsync(static_cast<char*>(a_dev) + r0 * K * es,
                                      static_cast<const char*>(a_host) + r0 * K * es,
                                      static_cast<size_t>(m) * K * es, cudaMemcpyHostToDevice,
                                      p->in));
    AOTK_HOST_CHECK(cudaEventRecord(p->a_ready[i], p->in));
  }
  r0 = 0;
  for (int i = 0; i < nblocks; r0 += rows[i], ++i) {
    const int64_t m = rows[i];
    AOTK_HOST_CHECK(cudaStreamWaitEvent(s, p->a_ready[i], 0));
    char* c_blk = static_cast<char*>(c_dev) + r0 * N * es;
    if (int st = aotk_gemm_opt_ws(c_blk, static_cast<const char*>(a_dev) + r0 * K * es, b_dev, m,
                                  N, K, dtype, workspace, workspace_bytes, s))
      return st;
    AOTK_HOST_CHECK(cudaEventRecord(p->c_ready[i], s));
    AOTK_HOST_CHECK(cudaStreamWaitEvent(p->out, p->c_ready[i], 0));
    AOTK_HOST_CHECK(cudaMemcpyAsync(static_cast<char*>(c_host) + r0 * N * es, c_blk,
                                    static_cast<size_t>(m) * N * es, cudaMemcpyDeviceToHost,
                                    p->out));
  }
  AOTK_HOST_CHECK(cudaEventRecord(p->end, p->out));
  AOTK_HOST_CHECK(cudaStreamWaitEvent(s, p->end, 0));
  return AOTK_OK;
}

}  // namespace
}  // namespace aotk

extern "C" int aotk_gemm_host_workspace_size(int64_t M, int64_t N, int64_t K, int dtype,
                                             size_t* bytes) {
  using namespace aotk;
  if (!bytes || M < 0 || N < 0 || K < 0)
    return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_gemm_host_workspace_size: bad arguments");
  *bytes = 0;
  if (M == 0) return AOTK_OK;
  int64_t rows[kMaxBlocks];
  const int n = block_plan(M, rows);
  for (int i = 0; i < n; ++i) {
    size_t b = 0;
    if (int st = aotk_gemm_opt_workspace_size(rows[i], N, K, dtype, &b)) return st;
    if (b > *bytes) *bytes = b;
  }
  return AOTK_OK;
}

extern "C" int aotk_gemm_host(void* c_host, const void* a_host, const void* b_host, int64_t M,
                              int64_t N, int64_t K, int dtype, void* a_dev, void* b_dev,
                              void* c_dev, void* workspace, size_t workspace_bytes, void* stream) {
  return aotk::gemm_host(c_host, a_host, b_host, M, N, K, dtype, a_dev, b_dev, c_dev, workspace,
                         workspace_bytes, stream);
}
