// Persistent, warp-specialised tcgen05 GEMM: C[M,N] = A[M,K] * B[K,N].
//
// One CTA per SM walks output tiles of 128 x BN (grouped raster for L2
// reuse).  Six warps split the work:
//   warp 0      TMA producer: per K block (one 128-byte swizzle row of
//               elements: 64 16-bit or 128 8-bit), one 128-row box of A
//               (K-major) and BN / box-width boxes of B (N-major), all
//               128-byte swizzled, into a STAGES-deep shared-memory ring
//               guarded by full/empty mbarriers;
//   warp 1      MMA issuer: allocates 2 * BN TMEM columns (two 32-bit
//               accumulators), issues tcgen05.mma M=128 N=BN (kind::f16 for
//               fp16/bf16, K=16; kind::f8f6f4 / kind::i8 for the scaled
//               8-bit GEMM, K=32) with A K-major and B MN-major straight from
//               the swizzled stages (no transpose pass), and commits each
//               stage back to the producer and each finished accumulator to
//               the epilogue;
//   warps 2-5   epilogue: tcgen05.ld of their 32-lane TMEM quarter, the
//               variant's arithmetic (none, silu(gate) * up, dequantisation
//               scales), packing to the output type, swizzled 32-row staging
//               boxes and TMA stores (double buffered per warp).  The
//               accumulator is handed back as soon as it is read, so the
//               next tile's main loop overlaps this tile's stores.
// Schedule: whole tiles are dealt round-robin to the CTAs.  A partial last
// wave is cut to occupy more SMs (plan_tc): into two N halves per tile (an
// MMA of N = BN/2 each; no workspace, results identical to whole tiles) or,
// for a small remainder, long K and a caller-provided workspace, into S K
// ranges whose fp32 partial tiles meet in the workspace: the unit that
// arrives last (atomic counter per tile) waits for the others' partials,
// adds them to its own accumulator in split order - so the output is
// deterministic - and stores the result.
// Every pipeline wait is bounded (sm100.cuh): on a timeout the kernel records
// a watchdog bit, lets the other roles drop out, drains its in-flight copies
// and frees TMEM before returning.
//
// Replaces the reference's WMMA/cp.async kernel gemm_wmma_pipe_kernel
// (aot_kernel/csrc/gemm/gemm_opt.cu:30-195): 128 x 128 x 32 tiles, 2 stages,
// one CTA per tile, fp32 epilogue through shared memory.
#include "common.h"
#include "gemm_internal.h"
#include "sm100.cuh"
#include "tmap.h"
#include "vec.cuh"

#include <type_traits>

namespace aotk {
namespace {

using namespace sm100;

__device__ unsigned g_tc_watchdog;

constexpr int kBM = 128;
constexpr int kThreads = 192;       // plain GEMM: producer, MMA, 4 epilogue warps
constexpr int kThreadsFused = 320;  // + 4 all-reduce warps (gemm_allreduce)
// M tiles per raster group.  Groups of 8 and 32, and L2 eviction hints on
// the operand loads (evict_last on A, evict_first on B) measured within
// +-3 % of this on the shapes of the path, none better throughout.
constexpr int kGroupM = 16;
constexpr int kMaxSplits = 4;
// K blocks below which a K split does not pay for its partial-tile traffic
// (measured on B200: a 4-way split of 64 K blocks lost to whole tiles, of 128
// K blocks it cut the kernel time by 13 %).
constexpr int kSplitMinKblocks = 128;

// Watchdog bits of this kernel (the skinny kernel uses 8-32, the CTA-pair
// kernel 256-1024; aotk_watchdog_status ORs all of them).
enum : unsigned {
  kWdProducer = 1u,
  kWdMma = 2u,
  kWdEpilogue = 4u,
  kWdSplit = 2048u,  // the last K-split unit gave up waiting for the other partials
  kWdPeer = 64u,
  kWdSelfTest = 128u
};

__device__ unsigned g_never_set;  // stays 0: the self-test's flag that nothing sets

// Operand kinds: element size, the tcgen05 MMA that consumes them and its
// instruction-descriptor formats.  A K block is one 128-byte swizzle row of
// elements (kBK); one MMA consumes 32 bytes of it (kUmmaK elements).
template <typename T>
struct Op16 {
  static constexpr int kBytes = 2;
  static constexpr bool kIntAcc = false;
  static constexpr uint32_t idesc(int m, int n) {
    return idesc_f16(std::is_same<T, __nv_bfloat16>::value, m, n, false, true);
  }
  __device__ __forceinline__ static void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id,
                                             bool acc) {
    umma_f16(d, a, b, id, acc);
  }
};
struct OpE4m3 {
  static constexpr int kBytes = 1;
  static constexpr bool kIntAcc = false;
  static constexpr uint32_t idesc(int m, int n) { return idesc_make(1u, 0u, m, n, false, true); }
  __device__ __forceinline__ static void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id,
                                             bool acc) {
    umma_f8f6f4(d, a, b, id, acc);
  }
};
struct OpE5m2 {
  static constexpr int kBytes = 1;
  static constexpr bool kIntAcc = false;
  static constexpr uint32_t idesc(int m, int n) { return idesc_make(1u, 1u, m, n, false, true); }
  __device__ __forceinline__ static void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id,
                                             bool acc) {
    umma_f8f6f4(d, a, b, id, acc);
  }
};
struct OpS8 {
  static constexpr int kBytes = 1;
  static constexpr bool kIntAcc = true;  // s32 accumulator
  static constexpr uint32_t idesc(int m, int n) { return idesc_make(2u, 1u, m, n, false, true); }
  __device__ __forceinline__ static void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id,
                                             bool acc) {
    umma_i8(d, a, b, id, acc);
  }
};

template <int kInBytes>
struct OpShape {
  static constexpr int kBK = 128 / kInBytes;    // elements per K block
  static constexpr int kUmmaK = 32 / kInBytes;  // elements per MMA
};

template <int BN, int STAGES, int kInBytes = 2>
struct TcLayout {
  static constexpr int kBK = OpShape<kInBytes>::kBK;
  static constexpr int kBoxN = 128 / kInBytes;  // N elements per B box
  static constexpr uint32_t kABytes = kBM * 128;
  static constexpr uint32_t kBBox = kBK * 128;  // one kBoxN (N) x kBK (K) box
  static constexpr uint32_t kBBytes = (BN / kBoxN) * kBBox;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kCBuf = 32 * 128;  // 32 rows x 64 columns x 2 bytes
  static constexpr uint32_t kOffA = 0;
  static constexpr uint32_t kOffB = kOffA + STAGES * kABytes;
  static constexpr uint32_t kOffC = kOffB + STAGES * kBBytes;
  static constexpr uint32_t kOffBar = kOffC + 4 * 2 * kCBuf;
  static constexpr uint32_t kNumBars = 2 * STAGES + 5;  // full, empty, tmem full/empty x2, drain
  static constexpr uint32_t kOffMisc = kOffBar + kNumBars * 8;
  static constexpr uint32_t kBytes = kOffMisc + 16;
  static constexpr uint32_t kAlloc = kBytes + 1024;  // base is rounded up to 1 KB
  static constexpr uint32_t kTmemCols = 2 * BN;
  static_assert(BN % 64 == 0 && BN <= 256, "BN must be 64..256 in steps of 64");
  static_assert(kTmemCols <= 512, "two accumulators must fit in TMEM");
  // The last K-split unit stages up to 4 partials x 16 x 128 x 16 bytes in the ring.
  static_assert(4 * 16 * 128 * 16 <= STAGES * kStageBytes, "stage ring too small for partials");
};

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& mb, int& nb) {
  const int per_group = kGroupM * tiles_n;
  const int g = tile / per_group;
  const int first_m = g * kGroupM;
  const int gm = min(tiles_m - first_m, kGroupM);
  const int local = tile - g * per_group;
  mb = first_m + local % gm;
  nb = local / gm;
}

// Work list shared by the producer, MMA and epilogue roles of a CTA.  Tiles
// before split_begin run whole; the tail tiles from split_begin on run either
// as two halves of 128 x BN/2 (halves != 0: twice the CTAs, no reduction) or
// as `splits` K ranges whose fp32 partials meet in the workspace.
struct TcSched {
  int tiles_m, tiles_n, num_tiles, kblocks;
  int full_rounds;    // rounds of whole tiles: tile = cta + r * grid, tile < split_begin
  int split_begin;    // first tail tile (num_tiles when none)
  int halves;         // 1: tail tiles run as two N halves
  int splits;         // K units per tail tile (1 with halves)
  int kb_per_split;
  int units;          // tail work items: (num_tiles - split_begin) * (halves ? 2 : splits)
  float* ws;          // [units][kBM][BN] fp32 partial tiles (K splits)
  unsigned* counters; // [2][num_tiles - split_begin]: arrivals, then partials stored
};

struct WorkItem {
  int tile, kb0, kb1;
  int unit;  // >= 0: K-split unit (index into the workspace); -1 otherwise
  int half;  // 0 / 1: N half of the tile; -1: the whole width
};

__device__ __forceinline__ bool work_item(const TcSched& s, int i, WorkItem& w) {
  if (i < s.full_rounds) {
    w.tile = blockIdx.x + i * gridDim.x;
    if (w.tile >= s.split_begin) return false;
    w.kb0 = 0;
    w.kb1 = s.kblocks;
    w.unit = -1;
    w.half = -1;
    return true;
  }
  const int u = blockIdx.x + (i - s.full_rounds) * gridDim.x;
  if (u >= s.units) return false;
  if (s.halves) {
    w.tile = s.split_begin + (u >> 1);
    w.half = u & 1;
    w.kb0 = 0;
    w.kb1 = s.kblocks;
    w.unit = -1;
    return true;
  }
  w.tile = s.split_begin + u / s.splits;
  w.kb0 = (u % s.splits) * s.kb_per_split;
  w.kb1 = min(s.kblocks, w.kb0 + s.kb_per_split);
  w.unit = u;
  w.half = -1;
  return true;
}

// Global column of B box `j` of a work item (j counts the boxes the item
// loads).  A half item loads BN/2 columns: for silu_mul tiles, whose columns
// are [gate | up], the half takes the matching quarter of each.
template <int BN, int kBoxN, bool kSiluMul>
__device__ __forceinline__ int b_box_col(int nb, int half, int j) {
  if (half < 0) return nb * BN + j * kBoxN;
  if constexpr (kSiluMul) {
    constexpr int kPerPart = BN / 4 / kBoxN;  // boxes per quarter
    const int part = j / kPerPart;            // 0: gate, 1: up
    return nb * BN + part * (BN / 2) + half * (BN / 4) + (j % kPerPart) * kBoxN;
  }
  return nb * BN + half * (BN / 2) + j * kBoxN;
}

// float4 index, within one unit's partial tile, of 16-byte group j (columns
// 4j..4j+3 of 64-column chunk c) of the row held by `lane` of epilogue warp
// wq (0..3).  Consecutive lanes are consecutive, so warp accesses coalesce.
__device__ __forceinline__ int partial_index(int c, int wq, int j, int lane) {
  return ((c * 4 + wq) * 16 + j) * 32 + lane;
}

__device__ __forceinline__ void epilogue_bar_sync() {
  asm volatile("bar.sync 1, 128;" ::: "memory");  // warps 2..5 only
}

// 16-byte asynchronous global -> shared copy (L2 only) and its completion.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}
__device__ __forceinline__ float4 ld_shared_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void st_global_v4(float* p, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

// Fused all-reduce of the output over W ranks (one process per GPU) through
// NVSwitch multicast memory.  Each rank stores its partial tile into its own
// `part` buffer, then bumps the tile's arrival counter on every rank.  Every
// rank reduces a 1/W slice of the rows of every tile it computed: once all W
// partials of the tile have arrived, its all-reduce warps read the slice's
// sum through the multicast address of `part` (multimem.ld_reduce, fp32
// accumulation) and write it to every rank's `out` through the multicast
// address of `out` (multimem.st).  So in every round of tiles every CTA of
// every rank has reduction work, and the last round's tiles are reduced by
// all W ranks at once.  Counters only grow: call number e (epoch, from 1)
// waits for W*e arrivals.  A final done counter per rank (W * grid * e) tells
// each rank when every rank has written its slices.
struct ArParams {
  int rank, world;
  uint64_t part_mc, out_mc;        // multicast addresses of part / out
  unsigned* counters;              // this rank's per-tile arrival counters
  unsigned* const* peer_counters;  // [world] each rank's counters (peer-mapped)
  unsigned* done;                  // this rank's done counter
  unsigned* const* peer_done;      // [world] each rank's done counter
  unsigned epoch;
};

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
// Relaxed system-scope add: after a fence.acq_rel.sys by the same thread it
// completes a release pattern (the fence orders everything before it - the
// partial tile's stores, made visible to this thread by the bulk waits and
// the barrier - ahead of the add), without the per-operation wait of a
// release add.
__device__ __forceinline__ void red_relaxed_sys_add(unsigned* p, unsigned v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_gpu_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void comm_bar_sync() {
  asm volatile("bar.sync 2, 128;" ::: "memory");  // warps 6..9 only
}
// Waits until *p >= target, which a peer rank's kernel raises.  Ranks are
// separate host processes whose launches can drift apart by far more than
// the ~1 s a pipeline wait allows (interpreter pauses, first-call set-up), so
// cross-rank waits are bounded in wall time (%globaltimer) at 10 s instead;
// only a peer that never arrives ends one.  On a timeout: raises *abort, ORs
// `code` into *status and returns false.
constexpr unsigned long long kPeerWaitLimitNs = 10000000000ull;
__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool wait_at_least(const unsigned* p, unsigned target,
                                              volatile int* abort, unsigned* status,
                                              unsigned code = kWdPeer) {
  if (static_cast<int>(ld_acquire_sys(p) - target) >= 0) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (static_cast<int>(ld_acquire_sys(p) - target) < 0) {
    if (*abort) return false;
    if (globaltimer_ns() - t0 > kPeerWaitLimitNs) {
      *abort = 1;
      atomicOr(status, code);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void ld_reduce_bf16x8(uint64_t mc, uint4& v) {
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
}
__device__ __forceinline__ void ld_reduce_f16x8(uint64_t mc, uint4& v) {
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
}
__device__ __forceinline__ void multimem_st16(uint64_t mc, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Epilogue variants of the persistent kernel.
enum : int {
  kEpiStore = 0,      // C tile -> TMA store
  kEpiAllReduce = 1,  // partial tile -> `part`, all-reduce warps (ArParams)
  kEpiSiluMul = 2,    // tile = [gate_j | up_j] (128 + 128 columns) -> silu(gate) * up, 128 columns
  kEpiScaled = 3      // C = (acc * scale_a[row]) * scale_b[col] (ScaleParams)
};

// Dequantisation scales of the scaled epilogue: fp32 vectors read with a step
// of 0 (one scale for the whole operand) or 1 (one per row of A / column of B).
struct ScaleParams {
  const float* sa;
  const float* sb;
  int sa_step, sb_step;
};

// 16-bit or fp32 output element; stores and packs of 2 or 4 values.
template <typename T>
__device__ __forceinline__ void store4(T* p, float a, float b, float c, float d) {
  if constexpr (std::is_same<T, float>::value) {
    *reinterpret_cast<float4*>(p) = make_float4(a, b, c, d);
  } else {
    uint2 o;
    o.x = Elem<T>::pack2(a, b);
    o.y = Elem<T>::pack2(c, d);
    *reinterpret_cast<uint2*>(p) = o;
  }
}

// Scale factor of column `col` of B: four consecutive columns (col % 4 == 0).
// Columns at or beyond n read as 0; n % 4 == 0, so a group is all in or out.
__device__ __forceinline__ float4 load_sb4(const ScaleParams& sc, int col, int n) {
  if (sc.sb_step == 0) {
    const float v = __ldg(sc.sb);
    return make_float4(v, v, v, v);
  }
  if (col >= n) return make_float4(0.f, 0.f, 0.f, 0.f);
  return __ldg(reinterpret_cast<const float4*>(sc.sb + col));
}

template <typename Op, typename T, int BN, int STAGES, int kEpi>
__global__ void __launch_bounds__(kEpi == kEpiAllReduce ? kThreadsFused : kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, T* __restrict__ C, int M, int N, int K,
                   uint32_t idesc, TcSched sched, ArParams ar, ScaleParams sc) {
  constexpr bool kFused = kEpi == kEpiAllReduce;
  constexpr bool kSiluMul = kEpi == kEpiSiluMul;
  constexpr bool kScaled = kEpi == kEpiScaled;
  // Columns of C per tile and in total (the silu_mul epilogue halves both).
  constexpr int kOutCols = kSiluMul ? BN / 2 : BN;
  const int n_out = kSiluMul ? N / 2 : N;
  using L = TcLayout<BN, STAGES, Op::kBytes>;
  constexpr int kBK = L::kBK;
  constexpr int kUmmaK = OpShape<Op::kBytes>::kUmmaK;
  const uint32_t idesc_half = (idesc & ~(0x3Fu << 17)) | (static_cast<uint32_t>(BN / 2 / 8) << 17);
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw);
  const uint32_t sA = base + L::kOffA;
  const uint32_t sB = base + L::kOffB;
  const uint32_t sC = base + L::kOffC;
  const uint32_t bar0 = base + L::kOffBar;
  const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);
  unsigned* wd = &g_tc_watchdog;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_m = sched.tiles_m;
  const int tiles_n = sched.tiles_n;
  volatile int* last_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 8);

  // Programmatic dependent launch: the next kernel on the stream may start
  // its own prologue as SMs free up; this one touches global memory only
  // after pdl_wait_prior() below, once the previous kernel has completed.
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait_prior();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      auto load_a = [&](uint32_t dst, int x, int y, uint32_t bar) { tma_load_2d(dst, &tmA, x, y, bar); };
      auto load_b = [&](uint32_t dst, int x, int y, uint32_t bar) { tma_load_2d(dst, &tmB, x, y, bar); };
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      WorkItem w;
      for (int i = 0; ok && work_item(sched, i, w); ++i) {
        int mb, nb;
        tile_coords(w.tile, tiles_m, tiles_n, mb, nb);
        const int nbox = (w.half < 0 ? BN : BN / 2) / L::kBoxN;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, wd, kWdProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb = full_bar(stage);
          mbar_arrive_expect_tx(fb, L::kABytes + nbox * L::kBBox);
          load_a(sA + stage * L::kABytes, kb * kBK, mb * kBM, fb);
          // Straight-line issue (constant trip counts): a runtime loop here
          // cost 8 % of whole-tile throughput on B200.
          if (w.half < 0) {
#pragma unroll
            for (int j = 0; j < BN / L::kBoxN; ++j)
              load_b(sB + stage * L::kBBytes + j * L::kBBox, nb * BN + j * L::kBoxN, kb * kBK, fb);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 2 / L::kBoxN; ++j)
              load_b(sB + stage * L::kBBytes + j * L::kBBox,
                     b_box_col<BN, L::kBoxN, kSiluMul>(nb, w.half, j), kb * kBK, fb);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Loads already issued must land before this CTA may exit.
      int s = stage;
      uint32_t p = phase;
      for (int i = 0; i < STAGES && i < issued; ++i) {
        if (--s < 0) {
          s = STAGES - 1;
          p ^= 1u;
        }
        mbar_drain(full_bar(s), p);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      WorkItem w;
      for (int i = 0; ok && work_item(sched, i, w); ++i) {
        if (!mbar_wait_bounded(tempty_bar(acc), acc_phase ^ 1u, abort_flag, wd, kWdMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        // A half item is one MMA of N = BN/2 over the boxes it loaded.
        const uint32_t id = w.half < 0 ? idesc : idesc_half;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait_bounded(full_bar(stage), phase, abort_flag, wd, kWdMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = sA + stage * L::kABytes;
          const uint32_t b0 = sB + stage * L::kBBytes;
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            // A: K-major, advance 32 B inside the swizzle row.
            // B: MN-major, advance kUmmaK K rows (atoms of 8 rows x 128 B).
            const uint64_t ad = sdesc_sw128(a0 + k * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(b0 + k * kUmmaK * 128, L::kBBox, 1024);
            Op::mma(d_tmem, ad, bd, id, kb > w.kb0 || k > 0);
          }
          umma_commit(empty_bar(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(tfull_bar(acc));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Every MMA issued by this thread completes before TMEM is released.
      umma_commit(drain_bar);
      mbar_drain(drain_bar, 0);
    }
    __syncwarp();
  } else if (warp < 6) {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t cbuf = sC + (warp - 2) * 2 * L::kCBuf;
    int acc = 0;
    uint32_t acc_phase = 0;
    int nstore = 0;
    const uint64_t c_policy = l2_policy_evict_first();
    // Packs 64 fp32 values of this lane's row into T, stages them in
    // 128-byte-swizzled boxes of 32 rows x 128 bytes (one box for 16-bit T,
    // two for fp32) and TMA-stores each box at (x + its first column, y).
    constexpr int kBoxCols = 128 / static_cast<int>(sizeof(T));
    auto store_chunk = [&](const float (&f)[64], int x, int y) {
#pragma unroll
      for (int h = 0; h < 64 / kBoxCols; ++h) {
        uint32_t pk[32];
        if constexpr (sizeof(T) == 4) {
#pragma unroll
          for (int i = 0; i < 32; ++i) pk[i] = __float_as_uint(f[h * 32 + i]);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) pk[i] = Elem<T>::pack2(f[2 * i], f[2 * i + 1]);
        }
        const uint32_t buf = cbuf + (nstore & 1) * L::kCBuf;
        if (nstore >= 2 && lane == 0) bulk_wait_read<1>();
        __syncwarp();
        // Row `lane` of the box, 16-byte chunk j stored at j ^ (row % 8).
        const uint32_t row = buf + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          st_shared_v4(row + ((j ^ (lane & 7)) << 4), pk[4 * j], pk[4 * j + 1], pk[4 * j + 2],
                       pk[4 * j + 3]);
        }
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) {
          // C is written once and not re-read here: evict it first so the A
          // and B tiles other CTAs still need stay in L2.
          tma_store_2d_hint(&tmC, buf, x + h * kBoxCols, y, c_policy);
          bulk_commit();
        }
        ++nstore;
      }
    };
    WorkItem w;
    for (int i = 0; work_item(sched, i, w); ++i) {
      int mb, nb;
      tile_coords(w.tile, tiles_m, tiles_n, mb, nb);
      int ok = 1;
      if (lane == 0) ok = mbar_wait_bounded(tfull_bar(acc), acc_phase, abort_flag, wd, kWdEpilogue);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t trow = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                            static_cast<uint32_t>(acc * BN);
      const int row_in_tile = q * 32 + lane;
      const int store_y = mb * kBM + q * 32;
      const int slot = w.tile - sched.split_begin;
      // K-split unit: the unit that completes the tile (the last to arrive)
      // sums all partials in split order; the others leave theirs in the
      // workspace.  Learn which one this is before draining TMEM.
      bool split_last = false;
      if constexpr (!kFused) {
        if (w.unit >= 0) {
          if (warp == 2 && lane == 0) {
            const unsigned prev = atomicAdd(&sched.counters[slot], 1u);
            *last_flag = prev == static_cast<unsigned>(sched.splits - 1) ? 1 : 0;
          }
          epilogue_bar_sync();
          split_last = *last_flag != 0;
          epilogue_bar_sync();  // last_flag is rewritten by the next unit
          if (!split_last) {
            // Partial layout [chunk][warp][16-byte group][lane]: each warp
            // store (and the last unit's load) covers 512 contiguous bytes.
            float* dst = sched.ws + static_cast<size_t>(w.unit) * kBM * BN;
#pragma unroll 1
            for (int c = 0; c < BN / 64; ++c) {
              uint32_t r[64];
              tmem_ld_32x32b_x32(trow + c * 64, r);
              tmem_ld_32x32b_x32(trow + c * 64 + 32, r + 32);
              tmem_wait_ld();
              if constexpr (Op::kIntAcc) {
#pragma unroll
                for (int j = 0; j < 64; ++j)
                  r[j] = __float_as_uint(static_cast<float>(static_cast<int>(r[j])));
              }
              if (c == BN / 64 - 1) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(tempty_bar(acc));
              }
#pragma unroll
              for (int j = 0; j < 16; ++j)
                st_global_v4(dst + 4 * partial_index(c, warp - 2, j, lane), r[4 * j], r[4 * j + 1],
                             r[4 * j + 2], r[4 * j + 3]);
            }
            // All four warps' rows are written: count the partial in.
            __threadfence();
            epilogue_bar_sync();
            if (warp == 2 && lane == 0)
              red_release_gpu_add(sched.counters + sched.units / sched.splits + slot, 1u);
            if (++acc == 2) {
              acc = 0;
              acc_phase ^= 1u;
            }
            continue;
          }
          // Last arriver: the other S - 1 units have arrived, so they are
          // running and about to publish their partials; wait (bounded).
          if (warp == 2 && lane == 0)
            *last_flag = wait_at_least(sched.counters + sched.units / sched.splits + slot,
                                       static_cast<unsigned>(sched.splits - 1), abort_flag, wd,
                                       kWdSplit)
                             ? 1
                             : 0;
          epilogue_bar_sync();
          const bool ready = *last_flag != 0;
          epilogue_bar_sync();
          if (!ready) break;
          __threadfence();
        }
      }
      // 64 accumulator columns [tcol, tcol + 64) of this lane's row as fp32;
      // for the last K-split unit, the sum of all S partials in split order.
      // The other units' partial rows are fetched with cp.async into the A/B
      // stage ring - idle by now, since a K-split unit is always its CTA's
      // last work item and its MMAs have consumed every stage - laid out
      // [split][16-byte group][thread] so each warp access is contiguous.
      auto acc_chunk = [&](int tcol, float (&f)[64]) {
        uint32_t r[64];
        tmem_ld_32x32b_x32(trow + tcol, r);
        tmem_ld_32x32b_x32(trow + tcol + 32, r + 32);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 64; ++j)
          f[j] = Op::kIntAcc ? static_cast<float>(static_cast<int>(r[j])) : __uint_as_float(r[j]);
        if (!split_last) return;
        const int me = w.unit % sched.splits;
        const uint32_t et = threadIdx.x - 64;  // 0..127
        const size_t unit_stride = static_cast<size_t>(kBM) * BN;
        const float* base = sched.ws + static_cast<size_t>(slot) * sched.splits * unit_stride;
        auto slot_addr = [&](int sp, int j) { return sA + ((sp * 16 + j) * 128 + et) * 16; };
#pragma unroll 1
        for (int sp = 0; sp < sched.splits; ++sp) {
          if (sp == me) continue;
#pragma unroll
          for (int j = 0; j < 16; ++j)
            cp_async16(slot_addr(sp, j),
                       base + sp * unit_stride + 4 * partial_index(tcol / 64, warp - 2, j, lane));
        }
        cp_async_wait_all();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
          for (int sp = 0; sp < sched.splits; ++sp) {
            const float4 v = sp == me ? make_float4(f[4 * j], f[4 * j + 1], f[4 * j + 2], f[4 * j + 3])
                                      : ld_shared_f4(slot_addr(sp, j));
            if (sp == 0) {
              sum = v;
            } else {
              sum.x += v.x;
              sum.y += v.y;
              sum.z += v.z;
              sum.w += v.w;
            }
          }
          f[4 * j] = sum.x;
          f[4 * j + 1] = sum.y;
          f[4 * j + 2] = sum.z;
          f[4 * j + 3] = sum.w;
        }
      };
      // Accumulator columns this item holds: BN, or BN / 2 for a half tile.
      const int ncols = w.half < 0 ? BN : BN / 2;
      bool chunks_done = false;
      if constexpr (kSiluMul) {
        // The accumulator holds [gate | up], ncols / 2 columns each.
        const int nch = ncols / 128;
#pragma unroll 1
        for (int c = 0; c < nch; ++c) {
          float g[64], u[64];
          acc_chunk(c * 64, g);
          acc_chunk(ncols / 2 + c * 64, u);
          if (c == nch - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(acc));
          }
          const int store_x = nb * kOutCols + (w.half < 0 ? 0 : w.half * (kOutCols / 2)) + c * 64;
          if (store_x >= n_out || store_y >= M) continue;
          if (sc.sa != nullptr) {
            // Row scale (an rms_norm rstd folded out of A): gate and up
            // accumulators are both linear in the row.
            const int row = mb * kBM + row_in_tile;
            const float rs = row < M ? __ldg(sc.sa + row) : 0.f;
#pragma unroll
            for (int j = 0; j < 64; ++j) {
              g[j] *= rs;
              u[j] *= rs;
            }
          }
#pragma unroll
          for (int j = 0; j < 64; ++j) g[j] = silu_f(g[j]) * u[j];
          store_chunk(g, store_x, store_y);
        }
        chunks_done = true;
      }
      const int nch = ncols / 64;
#pragma unroll 1
      for (int c = 0; c < nch && !chunks_done; ++c) {
        float f[64];
        acc_chunk(c * 64, f);
        if (c == nch - 1) {
          // Accumulator fully read: hand it back to the MMA warp.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(tempty_bar(acc));
        }
        const int store_x = nb * BN + (w.half < 0 ? 0 : w.half * (BN / 2)) + c * 64;
        if (store_x >= N || store_y >= M) continue;  // box entirely outside C
        if constexpr (kScaled) {
          const int row = mb * kBM + row_in_tile;
          const float sa = row < M ? __ldg(sc.sa + static_cast<size_t>(row) * sc.sa_step) : 0.f;
#pragma unroll
          for (int j = 0; j < 64; j += 4) {
            const float4 sb = load_sb4(sc, store_x + j, N);
            f[j] = (f[j] * sa) * sb.x;
            f[j + 1] = (f[j + 1] * sa) * sb.y;
            f[j + 2] = (f[j + 2] * sa) * sb.z;
            f[j + 3] = (f[j + 3] * sa) * sb.w;
          }
        }
        store_chunk(f, store_x, store_y);
      }
      if constexpr (kFused) {
        // The partial tile is in `part` once each warp's stores complete;
        // after all four epilogue warps, count it in on every rank: one
        // system-scope fence, then relaxed adds (a release pattern).  A
        // release add per rank, and a system fence on every thread, each
        // waited for the memory system in turn: measured at 8 ranks they
        // made the epilogue ~45 us per tile, twice the tile's MMA time.
        if (lane == 0) {
          bulk_wait_all();
          fence_proxy_async_global();
          fence_sys();
        }
        __syncwarp();
        epilogue_bar_sync();
        if (warp == 2 && lane == 0) {
          fence_sys();
          for (int p = 0; p < ar.world; ++p) red_relaxed_sys_add(ar.peer_counters[p] + w.tile, 1u);
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  } else if constexpr (kFused) {
    // ---------------- all-reduce (warps 6..9) ----------------
    // Same work list as the epilogue; for each tile, wait for all W partials,
    // then reduce this rank's slice of its rows through the switch and
    // broadcast the sum.
    const int ct = threadIdx.x - 192;  // 0..127
    volatile int* peer_ok = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 12);
    constexpr int kVecPerRow = BN * 2 / 16;
    const int slice_rows = (kBM + ar.world - 1) / ar.world;
    const int row0 = ar.rank * slice_rows;
    const int nvec = max(0, min(kBM, row0 + slice_rows) - row0) * kVecPerRow;
    WorkItem w;
    for (int i = 0; work_item(sched, i, w); ++i) {
      if (ct == 0)
        *peer_ok = wait_at_least(ar.counters + w.tile, ar.epoch * ar.world, abort_flag, wd) ? 1 : 0;
      comm_bar_sync();
      const bool ok = *peer_ok != 0;
      comm_bar_sync();
      if (!ok) break;
      int mb, nb;
      tile_coords(w.tile, tiles_m, tiles_n, mb, nb);
      constexpr int kInFlight = 8;  // 16-byte reductions per thread in flight
#pragma unroll 1
      for (int v0 = ct; v0 < nvec; v0 += kInFlight * 128) {
        uint4 val[kInFlight];
        uint64_t off[kInFlight];
        bool live[kInFlight];
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) {
          const int v = v0 + u * 128;
          const int gr = mb * kBM + row0 + v / kVecPerRow;
          const int gc = nb * BN + (v % kVecPerRow) * 8;
          // N % 8 == 0: a 16-byte vector is all in range or all out
          live[u] = v < nvec && gr < M && gc < N;
          off[u] = (static_cast<uint64_t>(gr) * N + gc) * sizeof(T);
          if (live[u]) {
            if constexpr (sizeof(T) == 2 && std::is_same<T, __nv_bfloat16>::value)
              ld_reduce_bf16x8(ar.part_mc + off[u], val[u]);
            else
              ld_reduce_f16x8(ar.part_mc + off[u], val[u]);
          }
        }
#pragma unroll
        for (int u = 0; u < kInFlight; ++u)
          if (live[u]) multimem_st16(ar.out_mc + off[u], val[u]);
      }
    }
    // Every rank has written its slices of every tile once all W * grid CTAs
    // have checked in on this rank.
    fence_sys();
    comm_bar_sync();
    if (ct == 0) {
      fence_sys();
      for (int p = 0; p < ar.world; ++p) red_relaxed_sys_add(ar.peer_done[p], 1u);
      wait_at_least(ar.done, ar.epoch * ar.world * gridDim.x, abort_flag, wd);
    }
    comm_bar_sync();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// Exercises the bounded waits with nothing to wait for: an mbarrier phase that
// no thread or copy completes (gives up after kWaitLimitCycles, ~1 s), then a
// flag that nothing sets (gives up after kPeerWaitLimitNs, 10 s).  Each
// records its watchdog bit; the kernel returns.
__global__ void watchdog_selftest_kernel() {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_addr(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_wait_bounded(smem_addr(&bar), 0, &abort_flag, &g_tc_watchdog, kWdSelfTest);
    abort_flag = 0;
    wait_at_least(&g_never_set, 1u, &abort_flag, &g_tc_watchdog);
  }
}

struct TcPlan {
  int grid;
  TcSched sched;
  size_t ws_bytes;       // 0: no K-split phase
  size_t counter_bytes;  // leading part of the workspace holding the counters
};

// Tile schedule for the device.  Whole tiles go round-robin over the SMs; a
// partial last wave of `rem` tiles (or a single partial wave) is cut so that
// it keeps more SMs busy:
//   * rem <= sms / 4, K >= kSplitMinKblocks blocks, workspace given: each tile
//     is cut along K into S = min(4, sms / rem) units whose fp32 partials the
//     last-arriving unit sums (deterministically, in split order) - the tail
//     lasts about 1/S of a tile plus the read of S - 1 partials;
//   * otherwise rem <= sms / 2: each tile runs as two N halves on two SMs -
//     the tail lasts half a tile, with no reduction and results identical to
//     whole tiles;
//   * otherwise the tail runs whole.
TcPlan plan_tc(int M, int N, int K, int BN, int bk, int sms, bool allow_split, bool allow_halves) {
  TcPlan p{};
  TcSched& s = p.sched;
  s.tiles_m = (M + kBM - 1) / kBM;
  s.tiles_n = (N + BN - 1) / BN;
  s.num_tiles = s.tiles_m * s.tiles_n;
  s.kblocks = (K + bk - 1) / bk;
  const int full = s.num_tiles / sms;
  const int rem = s.num_tiles - full * sms;
  p.grid = s.num_tiles < sms ? s.num_tiles : sms;
  s.full_rounds = (s.num_tiles + p.grid - 1) / p.grid;
  s.split_begin = s.num_tiles;
  s.halves = 0;
  s.splits = 1;
  s.kb_per_split = s.kblocks;
  s.units = 0;
  if (rem == 0) return p;
  int S = 1;
  if (allow_split && rem * kMaxSplits <= sms && s.kblocks >= kSplitMinKblocks) S = kMaxSplits;
  if (S > 1) {
    p.grid = sms;
    s.full_rounds = full;
    s.split_begin = full * sms;
    s.kb_per_split = (s.kblocks + S - 1) / S;
    s.splits = (s.kblocks + s.kb_per_split - 1) / s.kb_per_split;  // every split non-empty
    s.units = rem * s.splits;
    p.counter_bytes =
        (2 * static_cast<size_t>(rem) * sizeof(unsigned) + 255) & ~static_cast<size_t>(255);
    p.ws_bytes = p.counter_bytes + static_cast<size_t>(s.units) * kBM * BN * sizeof(float);
    return p;
  }
  if (allow_halves && 2 * rem <= sms) {
    p.grid = full > 0 ? sms : 2 * rem;
    s.full_rounds = full;
    s.split_begin = full * sms;
    s.halves = 1;
    s.units = 2 * rem;
  }
  return p;
}

// Tensor map over a row-major matrix of T (16-bit or fp32).
template <typename T>
int make_tmap_of(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_cols,
                 uint32_t box_rows) {
  if constexpr (std::is_same<T, float>::value)
    return make_tmap_2d_f32(map, base, rows, cols, cols, box_cols, box_rows);
  else
    return make_tmap_2d_16bit(map, base, std::is_same<T, __nv_bfloat16>::value, rows, cols, cols,
                              box_cols, box_rows);
}

// Launches the persistent kernel on operands of kind Op (Op16<T> for the
// 16-bit GEMMs, OpE4m3 / OpE5m2 / OpS8 for the scaled GEMM) with output type T.
template <typename Op, typename T, int BN, int STAGES, int kEpi = kEpiStore>
int launch_tc(void* c, const void* a, const void* b, int M, int N, int K, void* workspace,
              size_t ws_bytes, cudaStream_t stream, const DeviceInfo& info,
              const ArParams* ar = nullptr, const ScaleParams* scales = nullptr) {
  using L = TcLayout<BN, STAGES, Op::kBytes>;
  constexpr bool kFused = kEpi == kEpiAllReduce;
  auto kernel = gemm_tc_kernel<Op, T, BN, STAGES, kEpi>;
  if (int st = ensure_dynamic_smem(reinterpret_cast<const void*>(kernel), L::kAlloc, info)) return st;
  // The fused all-reduce counts whole tiles: its tail always runs whole.
  constexpr bool kHalves = !kFused;
  TcPlan p = plan_tc(M, N, K, BN, L::kBK, info.sm_count, workspace != nullptr, kHalves);
  if (p.ws_bytes > 0 && (ws_bytes < p.ws_bytes || (reinterpret_cast<uintptr_t>(workspace) & 255)))
    p = plan_tc(M, N, K, BN, L::kBK, info.sm_count, false, kHalves);
  if (p.ws_bytes > 0) {
    p.sched.counters = static_cast<unsigned*>(workspace);
    p.sched.ws = reinterpret_cast<float*>(static_cast<char*>(workspace) + p.counter_bytes);
    cudaError_t e = cudaMemsetAsync(workspace, 0, p.counter_bytes, stream);
    if (e != cudaSuccess)
      return fail(AOTK_ERR_CUDA, "tcgen05 gemm: counter reset: %s", cudaGetErrorString(e));
  }
  CUtensorMap ta, tb, tc;
  if constexpr (Op::kBytes == 1) {
    if (int st = make_tmap_2d_8bit(&ta, a, M, K, K, L::kBK, kBM)) return st;
    if (int st = make_tmap_2d_8bit(&tb, b, K, N, N, L::kBoxN, L::kBK)) return st;
  } else {
    if (int st = make_tmap_of<T>(&ta, a, M, K, L::kBK, kBM)) return st;
    if (int st = make_tmap_of<T>(&tb, b, K, N, L::kBoxN, L::kBK)) return st;
  }
  const int n_out = kEpi == kEpiSiluMul ? N / 2 : N;
  if (int st = make_tmap_of<T>(&tc, c, M, n_out, 128 / sizeof(T), 32)) return st;
  const uint32_t idesc = Op::idesc(kBM, BN);  // A K-major, B MN-major
  ArParams arp{};
  if (ar) arp = *ar;
  ScaleParams scp{};
  if (scales) scp = *scales;
  // Launched with programmatic stream serialisation (see the kernel's
  // prologue): barrier set-up, TMEM allocation and descriptor prefetch
  // overlap the tail of the previous kernel.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.grid), 1, 1);
  cfg.blockDim = dim3(kFused ? kThreadsFused : kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, ta, tb, tc, static_cast<T*>(c), M, N, K, idesc,
                                     p.sched, arp, scp);
  if (e != cudaSuccess)
    return fail(AOTK_ERR_CUDA, "tcgen05 gemm launch (grid %d): %s", p.grid, cudaGetErrorString(e));
  return check_launch("tcgen05 gemm");
}

constexpr int kTcBN = 256;
constexpr int kTcStages = 4;

}  // namespace

size_t gemm_tc_workspace_size(int64_t M, int64_t N, int64_t K, int sm_count) {
  if (M <= 0 || N <= 0 || K <= 0 || M >= (1LL << 31) || N >= (1LL << 31) || K >= (1LL << 31))
    return 0;
  return plan_tc((int)M, (int)N, (int)K, kTcBN, OpShape<2>::kBK, sm_count, true, true).ws_bytes;
}

int gemm_tc(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K, int dtype,
            void* workspace, size_t ws_bytes, void* stream) {
  DeviceInfo info;
  if (int st = current_device_info(&info)) return st;
  if (int st = require_sm100(info)) return st;
  if (int st = check_tc_preconditions("aotk_gemm_tc", c, a, b, M, N, K, dtype)) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int m = (int)M, n = (int)N, k = (int)K;
  if (dtype == AOTK_BFLOAT16)
    return launch_tc<Op16<__nv_bfloat16>, __nv_bfloat16, kTcBN, kTcStages, kEpiStore>(
        c, a, b, m, n, k, workspace, ws_bytes, s, info);
  return launch_tc<Op16<__half>, __half, kTcBN, kTcStages, kEpiStore>(c, a, b, m, n, k, workspace,
                                                                      ws_bytes, s, info);
}

int gemm_silu_mul(void* act, const void* a, const void* b, const float* row_scale, int64_t M,
                  int64_t N2, int64_t K, int dtype, void* workspace, size_t ws_bytes,
                  void* stream) {
  DeviceInfo info;
  if (int st = current_device_info(&info)) return st;
  if (int st = require_sm100(info)) return st;
  if (int st = check_tc_preconditions("aotk_gemm_silu_mul", act, a, b, M, N2, K, dtype)) return st;
  if (N2 % kTcBN != 0)
    return fail(AOTK_ERR_UNSUPPORTED,
                "aotk_gemm_silu_mul: interleaved width 2*I = %lld must be a multiple of %d",
                (long long)N2, kTcBN);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int m = (int)M, n = (int)N2, k = (int)K;
  const ScaleParams rs{row_scale, nullptr, 1, 0};
  if (dtype == AOTK_BFLOAT16)
    return launch_tc<Op16<__nv_bfloat16>, __nv_bfloat16, kTcBN, kTcStages, kEpiSiluMul>(
        act, a, b, m, n, k, workspace, ws_bytes, s, info, nullptr, &rs);
  return launch_tc<Op16<__half>, __half, kTcBN, kTcStages, kEpiSiluMul>(
      act, a, b, m, n, k, workspace, ws_bytes, s, info, nullptr, &rs);
}

size_t gemm_scaled_tc_workspace_size(int64_t M, int64_t N, int64_t K, int sm_count) {
  if (M <= 0 || N <= 0 || K <= 0 || M >= (1LL << 31) || N >= (1LL << 31) || K >= (1LL << 31))
    return 0;
  return plan_tc((int)M, (int)N, (int)K, kTcBN, OpShape<1>::kBK, sm_count, true, true).ws_bytes;
}

namespace {

template <typename Op>
int launch_scaled(void* c, const void* a, const void* b, int m, int n, int k, int out_dtype,
                  const ScaleParams& sc, void* workspace, size_t ws_bytes, cudaStream_t s,
                  const DeviceInfo& info) {
  if (out_dtype == AOTK_BFLOAT16)
    return launch_tc<Op, __nv_bfloat16, kTcBN, kTcStages, kEpiScaled>(c, a, b, m, n, k, workspace,
                                                                      ws_bytes, s, info, nullptr, &sc);
  if (out_dtype == AOTK_FLOAT16)
    return launch_tc<Op, __half, kTcBN, kTcStages, kEpiScaled>(c, a, b, m, n, k, workspace,
                                                               ws_bytes, s, info, nullptr, &sc);
  return launch_tc<Op, float, kTcBN, kTcStages, kEpiScaled>(c, a, b, m, n, k, workspace, ws_bytes,
                                                            s, info, nullptr, &sc);
}

}  // namespace

int gemm_scaled_tc(void* c, const void* a, const void* b, const float* scale_a,
                   const float* scale_b, int64_t M, int64_t N, int64_t K, int in_dtype,
                   int out_dtype, int scale_mode, void* workspace, size_t ws_bytes, void* stream) {
  DeviceInfo info;
  if (int st = current_device_info(&info)) return st;
  if (int st = require_sm100(info)) return st;
  ScaleParams sc{scale_a, scale_b, scale_mode == AOTK_SCALE_ROW ? 1 : 0,
                 scale_mode == AOTK_SCALE_ROW ? 1 : 0};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int m = (int)M, n = (int)N, k = (int)K;
  if (in_dtype == AOTK_FLOAT8_E4M3)
    return launch_scaled<OpE4m3>(c, a, b, m, n, k, out_dtype, sc, workspace, ws_bytes, s, info);
  if (in_dtype == AOTK_FLOAT8_E5M2)
    return launch_scaled<OpE5m2>(c, a, b, m, n, k, out_dtype, sc, workspace, ws_bytes, s, info);
  return launch_scaled<OpS8>(c, a, b, m, n, k, out_dtype, sc, workspace, ws_bytes, s, info);
}

int gemm_tc_schedule(int64_t M, int64_t N, int64_t K, int elem_bytes, int sm_count,
                     bool with_workspace, int64_t* out) {
  if (M <= 0 || N <= 0 || K <= 0 || M >= (1LL << 31) || N >= (1LL << 31) || K >= (1LL << 31) ||
      (elem_bytes != 1 && elem_bytes != 2) || sm_count <= 0)
    return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_gemm_schedule: bad arguments");
  const int bk = elem_bytes == 1 ? OpShape<1>::kBK : OpShape<2>::kBK;
  const TcPlan p = plan_tc((int)M, (int)N, (int)K, kTcBN, bk, sm_count, with_workspace, true);
  const TcSched& s = p.sched;
  out[0] = p.grid;
  out[1] = s.num_tiles;
  out[2] = s.full_rounds;
  out[3] = s.split_begin;
  out[4] = s.halves;
  out[5] = s.splits;
  out[6] = s.kb_per_split;
  out[7] = s.units;
  out[8] = s.kblocks;
  out[9] = static_cast<int64_t>(p.ws_bytes);
  return AOTK_OK;
}

int gemm_allreduce_tiles(int64_t M, int64_t N) {
  return static_cast<int>(((M + kBM - 1) / kBM) * ((N + kTcBN - 1) / kTcBN));
}

int gemm_allreduce(const void* a, const void* b, int64_t M, int64_t N, int64_t K, int dtype,
                   const aotk_allreduce_buffers* bufs, void* stream) {
  DeviceInfo info;
  if (int st = current_device_info(&info)) return st;
  if (int st = require_sm100(info)) return st;
  if (!bufs) return fail(AOTK_ERR_INVALID_ARGUMENT, "aotk_gemm_allreduce: null buffers");
  if (int st = check_tc_preconditions("aotk_gemm_allreduce", bufs->part, a, b, M, N, K, dtype))
    return st;
  if (bufs->world < 1 || bufs->rank < 0 || bufs->rank >= bufs->world || bufs->epoch == 0 ||
      !bufs->part_multicast || !bufs->out_multicast || !bufs->counters || !bufs->peer_counters ||
      !bufs->done || !bufs->peer_done)
    return fail(AOTK_ERR_INVALID_ARGUMENT,
                "aotk_gemm_allreduce: incomplete buffers (rank %d of %d, epoch %u)", bufs->rank,
                bufs->world, bufs->epoch);
  if ((bufs->part_multicast & 15u) || (bufs->out_multicast & 15u))
    return fail(AOTK_ERR_INVALID_ARGUMENT,
                "aotk_gemm_allreduce: multicast addresses not 16-byte aligned");
  ArParams ar{};
  ar.rank = bufs->rank;
  ar.world = bufs->world;
  ar.part_mc = bufs->part_multicast;
  ar.out_mc = bufs->out_multicast;
  ar.counters = bufs->counters;
  ar.peer_counters = bufs->peer_counters;
  ar.done = bufs->done;
  ar.peer_done = bufs->peer_done;
  ar.epoch = bufs->epoch;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int m = (int)M, n = (int)N, k = (int)K;
  if (dtype == AOTK_BFLOAT16)
    return launch_tc<Op16<__nv_bfloat16>, __nv_bfloat16, kTcBN, kTcStages, kEpiAllReduce>(
        bufs->part, a, b, m, n, k, nullptr, 0, s, info, &ar);
  return launch_tc<Op16<__half>, __half, kTcBN, kTcStages, kEpiAllReduce>(
      bufs->part, a, b, m, n, k, nullptr, 0, s, info, &ar);
}

int watchdog_selftest(void* stream) {
  watchdog_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>();
  return check_launch("watchdog self-test");
}

int tc_watchdog(uint32_t* status, bool clear) {
  unsigned v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_watchdog, sizeof(v));
  if (e != cudaSuccess) return fail(AOTK_ERR_CUDA, "watchdog read: %s", cudaGetErrorString(e));
  if (clear) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_tc_watchdog, &zero, sizeof(zero));
    if (e != cudaSuccess) return fail(AOTK_ERR_CUDA, "watchdog clear: %s", cudaGetErrorString(e));
  }
  *status |= v;
  return AOTK_OK;
}

}  // namespace aotk
