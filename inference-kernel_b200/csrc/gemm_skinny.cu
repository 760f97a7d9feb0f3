// Skinny (decode-shaped) GEMM, M <= 128: C[M,N] = A[M,K] * B[K,N].
//
// At small M the cost is streaming the weight B from HBM, so the kernel is
// organised around that stream:
//   * swap AB: the MMA computes C^T = B^T * A^T, so the weight's N dimension
//     fills the 128-row MMA (M_mma = 128 output columns per CTA) and the
//     activation rows become the MMA's N (16..128, padded by TMA zero fill);
//     B is read N-major straight from its row-major layout (MN-major operand)
//     and A K-major;
//   * split K across a thread-block cluster of S CTAs (S <= 8) so that
//     ceil(N/128) * S CTAs keep every SM streaming; each CTA runs a TMA ->
//     tcgen05 pipeline over its K slice and leaves a 128 x MP fp32 partial
//     tile in its own shared memory;
//   * the S partials are summed in a fixed order through distributed shared
//     memory (each CTA reduces 1/S of the tile by reading its peers), so
//     there is no global workspace, no atomics, no second launch, and the
//     result is rounded to 16 bits once.
// Warp roles: 0 = TMA producer, 1 = MMA issuer + TMEM owner, 2..5 = TMEM
// readers; all 6 warps take part in the cluster reduction.
//
// The reference has no small-M path: gemm_wmma_pipe_kernel pads M to its
// 128-row tile (aot_kernel/csrc/gemm/gemm_opt.cu:174-192).
#include "common.h"
#include "gemm_internal.h"
#include "sm100.cuh"
#include "tmap.h"
#include "vec.cuh"

#include <mutex>

namespace aotk {
namespace {

using namespace sm100;

__device__ unsigned g_sk_watchdog;

constexpr int kThreads = 192;
constexpr int kTileN = 128;  // output columns per CTA (= MMA M)
constexpr int kBK = 64;
constexpr int kUmmaK = 16;
constexpr int kMaxCluster = 8;

enum : unsigned { kWdProducer = 8u, kWdMma = 16u, kWdEpilogue = 32u };

template <int MP, int STAGES>
struct SkLayout {
  static constexpr uint32_t kBtBox = kBK * 128;  // 64 (N) x 64 (K) box of the weight
  static constexpr uint32_t kBtBytes = 2 * kBtBox;
  static constexpr uint32_t kABytes = MP * 128;  // MP rows x 64 K
  static constexpr uint32_t kStageBytes = kBtBytes + kABytes;
  static constexpr uint32_t kOffBt = 0;
  static constexpr uint32_t kOffA = STAGES * kBtBytes;
  static constexpr uint32_t kRing = kOffA + STAGES * kABytes;
  static constexpr uint32_t kPartialBytes = MP * kTileN * 4;  // aliases the drained ring
  static constexpr uint32_t kOffBar = kRing > kPartialBytes ? kRing : kPartialBytes;
  static constexpr uint32_t kNumBars = 2 * STAGES + 1;  // full, empty, done
  static constexpr uint32_t kOffMisc = kOffBar + kNumBars * 8;
  static constexpr uint32_t kBytes = kOffMisc + 16;
  static constexpr uint32_t kAlloc = kBytes + 1024;
  static constexpr uint32_t kTmemCols = MP < 32 ? 32 : MP;
  static_assert(MP % 16 == 0 && MP <= 128, "MP must be 16..128 in steps of 16");
  static_assert(kABytes % 1024 == 0, "A stages stay 1 KB aligned (swizzle atoms)");
};

template <typename T, int MP, int STAGES>
__global__ void __launch_bounds__(kThreads, 2)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ CUtensorMap tmA, T* __restrict__ c, int M, int N,
                       int K, int kb_per_split, uint32_t idesc) {
  using L = SkLayout<MP, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw);
  const uint32_t sBt = base + L::kOffBt;
  const uint32_t sA = base + L::kOffA;
  const uint32_t bar0 = base + L::kOffBar;
  const uint32_t done_bar = bar0 + 8u * (2 * STAGES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);
  float* partial = reinterpret_cast<float*>(smem);  // [MP][128] fp32, after the main loop
  unsigned* wd = &g_sk_watchdog;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t split = cluster_ctarank();
  uint32_t S;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(S));
  const int n0 = static_cast<int>(blockIdx.x / S) * kTileN;
  const int kblocks = (K + kBK - 1) / kBK;
  const int kb0 = static_cast<int>(split) * kb_per_split;
  const int kb1 = min(kblocks, kb0 + kb_per_split);  // the host guarantees kb1 > kb0

  // The next kernel may start its own prologue now; this kernel reads global
  // memory only after pdl_wait_prior() below.
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmA);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(done_bar, 1);
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

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      pdl_wait_prior();  // inputs may come from the previous kernel on the stream
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, wd, kWdProducer)) break;
        const uint32_t fb = full_bar(stage);
        mbar_arrive_expect_tx(fb, L::kStageBytes);
        const uint32_t bt = sBt + stage * L::kBtBytes;
        tma_load_2d(bt, &tmB, n0, kb * kBK, fb);
        tma_load_2d(bt + L::kBtBox, &tmB, n0 + 64, kb * kBK, fb);
        tma_load_2d(sA + stage * L::kABytes, &tmA, kb * kBK, 0, fb);
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
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
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_bounded(full_bar(stage), phase, abort_flag, wd, kWdMma)) break;
        tc_fence_after();
        const uint32_t bt = sBt + stage * L::kBtBytes;
        const uint32_t at = sA + stage * L::kABytes;
#pragma unroll
        for (int k = 0; k < kBK / kUmmaK; ++k) {
          // MMA A = weight tile (MN-major: 2 column blocks of 64, 8 KB apart);
          // MMA B = activation rows (K-major, 32 B per 16-element step).
          const uint64_t ad = sdesc_sw128(bt + k * kUmmaK * 128, L::kBtBox, 1024);
          const uint64_t bd = sdesc_sw128(at + k * kUmmaK * 2, 16, 1024);
          umma_f16(tmem_base, ad, bd, idesc, kb > kb0 || k > 0);
        }
        umma_commit(empty_bar(stage));
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      umma_commit(done_bar);
      mbar_drain(done_bar, 0);
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    int ok = 1;
    if (lane == 0) ok = mbar_wait_bounded(done_bar, 0, abort_flag, wd, kWdEpilogue);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok) {
      tc_fence_after();
      const int nl = q * 32 + lane;  // output column within the tile = TMEM lane
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
      if constexpr (MP == 16) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(taddr, r);
        tmem_wait_ld();
#pragma unroll
        for (int m = 0; m < 16; ++m) partial[m * kTileN + nl] = __uint_as_float(r[m]);
      } else {
#pragma unroll 1
        for (int c0 = 0; c0 < MP; c0 += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + c0, r);
          tmem_wait_ld();
#pragma unroll
          for (int m = 0; m < 32; ++m) partial[(c0 + m) * kTileN + nl] = __uint_as_float(r[m]);
        }
      }
    }
  }

  tc_fence_before();
  // Partials of every CTA in the cluster are complete and visible.
  cluster_sync();

  // This CTA sums float4 slots [f_begin, f_end) of the 128 x MP tile over all
  // S partials, in rank order, and writes the rounded result.
  {
    constexpr int kF4 = MP * kTileN / 4;
    const int f_begin = static_cast<int>((static_cast<uint32_t>(kF4) * split) / S);
    const int f_end = static_cast<int>((static_cast<uint32_t>(kF4) * (split + 1)) / S);
    const uint32_t part_addr = smem_addr(partial);
    for (int f = f_begin + threadIdx.x; f < f_end; f += kThreads) {
      const int m = f / (kTileN / 4);
      const int n = n0 + (f % (kTileN / 4)) * 4;
      if (m >= M || n >= N) continue;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (uint32_t j = 0; j < S; ++j) {
        const float4 v = ld_dsmem_f32x4(map_to_rank(part_addr + static_cast<uint32_t>(f) * 16u, j));
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      // N % 8 == 0 and n % 4 == 0, so n + 3 < N: one 8-byte store.
      uint2 o;
      o.x = Elem<T>::pack2(acc.x, acc.y);
      o.y = Elem<T>::pack2(acc.z, acc.w);
      *reinterpret_cast<uint2*>(c + static_cast<int64_t>(m) * N + n) = o;
    }
  }

  // No CTA leaves while a peer may still read its shared memory.
  __syncwarp();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// A kernel with the skinny kernel's block shape and no TMEM, used only for
// occupancy queries: the driver reports one block per SM for any kernel that
// allocates TMEM (it cannot know how many columns each CTA takes), while two
// skinny CTAs - at most 128 + 128 of the 512 columns - do run side by side on
// an SM when shared memory allows, and clusters pack accordingly.
__global__ void __launch_bounds__(kThreads, 2) skinny_shadow_kernel() {}

// Clusters of `cs` skinny CTAs with `smem` bytes each that can be resident at
// once on the device (cached per device, cluster size and shared-memory size).
int resident_clusters(int cs, int smem, const DeviceInfo& info, int* out) {
  struct Entry {
    int device, cs, smem, n;
  };
  static std::mutex mu;
  static Entry cache[64];
  static int count = 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < count; ++i) {
    if (cache[i].device == info.device && cache[i].cs == cs && cache[i].smem == smem) {
      *out = cache[i].n;
      return AOTK_OK;
    }
  }
  if (int st = ensure_dynamic_smem(reinterpret_cast<const void*>(skinny_shadow_kernel), smem, info))
    return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(cs), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cs);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  cudaError_t e = cudaOccupancyMaxActiveClusters(&n, skinny_shadow_kernel, &cfg);
  if (e != cudaSuccess)
    return fail(AOTK_ERR_CUDA, "skinny gemm: cluster occupancy (size %d): %s", cs,
                cudaGetErrorString(e));
  if (count < 64) cache[count++] = Entry{info.device, cs, smem, n};
  *out = n;
  return AOTK_OK;
}

template <typename T, int MP, int STAGES>
int launch_skinny(void* c, const void* a, const void* b, int M, int N, int K, bool bf16,
                  cudaStream_t stream, const DeviceInfo& info) {
  using L = SkLayout<MP, STAGES>;
  auto kernel = gemm_skinny_kernel<T, MP, STAGES>;
  if (int st = ensure_dynamic_smem(reinterpret_cast<const void*>(kernel), L::kAlloc, info)) return st;
  CUtensorMap tb, ta;
  if (int st = make_tmap_2d_16bit(&tb, b, bf16, K, N, N, 64, kBK)) return st;
  if (int st = make_tmap_2d_16bit(&ta, a, bf16, M, K, K, kBK, MP)) return st;

  const int ntiles = (N + kTileN - 1) / kTileN;
  const int kblocks = (K + kBK - 1) / kBK;
  // One wave: every CTA streams an equal share of the weight at the same time.
  // The split is the largest cluster size (<= 8, <= K blocks) whose `ntiles`
  // clusters are all resident at once - up to two CTAs per SM - so that the
  // most weight bytes are in flight from the first K block on.  Measured on
  // B200 (graph-free back-to-back launches): M = 1 x K = 4096 x N = 6144
  // 13.0 -> 11.1 us against one CTA per SM (S = SMs / strips); M = 128 x
  // K = 14336 x N = 4096 32.3 -> 27.8 us against S = SMs / strips.  Larger
  // clusters that do not fit in one wave lose up to 2x.
  int S = 1;
  for (int cs = kMaxCluster < kblocks ? kMaxCluster : kblocks; cs > 1; --cs) {
    int resident = 0;
    if (int st = resident_clusters(cs, static_cast<int>(L::kAlloc), info, &resident)) return st;
    if (ntiles <= resident) {
      S = cs;
      break;
    }
  }
  const int kbps = (kblocks + S - 1) / S;
  S = (kblocks + kbps - 1) / kbps;  // every split owns at least one K block

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(ntiles * S), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(S);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // Programmatic dependent launch: the prologue (barrier init, TMEM
  // allocation, descriptor prefetch) overlaps the previous kernel's tail.
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const uint32_t idesc = idesc_f16(bf16, kTileN, MP, /*a_mn_major=*/true, /*b_mn_major=*/false);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, tb, ta, static_cast<T*>(c), M, N, K, kbps, idesc);
  if (e != cudaSuccess)
    return fail(AOTK_ERR_CUDA, "skinny gemm launch (cluster %d, grid %d): %s", S, ntiles * S,
                cudaGetErrorString(e));
  return check_launch("skinny gemm");
}

// Ring depth per activation width: two CTAs fit per SM (about 100-112 KB of
// shared memory each), which also lets clusters pack two CTAs onto one SM.
template <typename T>
int dispatch_mp(void* c, const void* a, const void* b, int M, int N, int K, bool bf16,
                cudaStream_t s, const DeviceInfo& info) {
  if (M <= 16) return launch_skinny<T, 16, 6>(c, a, b, M, N, K, bf16, s, info);
  if (M <= 32) return launch_skinny<T, 32, 5>(c, a, b, M, N, K, bf16, s, info);
  if (M <= 64) return launch_skinny<T, 64, 4>(c, a, b, M, N, K, bf16, s, info);
  return launch_skinny<T, 128, 3>(c, a, b, M, N, K, bf16, s, info);
}

}  // namespace

int gemm_skinny(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K, int dtype,
                void* stream) {
  DeviceInfo info;
  if (int st = current_device_info(&info)) return st;
  if (int st = require_sm100(info)) return st;
  if (int st = check_tc_preconditions("aotk_gemm_skinny", c, a, b, M, N, K, dtype)) return st;
  if (M > kSkinnyMaxM)
    return fail(AOTK_ERR_UNSUPPORTED, "aotk_gemm_skinny: M=%lld exceeds %lld", (long long)M,
                (long long)kSkinnyMaxM);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == AOTK_BFLOAT16)
    return dispatch_mp<__nv_bfloat16>(c, a, b, (int)M, (int)N, (int)K, true, s, info);
  return dispatch_mp<__half>(c, a, b, (int)M, (int)N, (int)K, false, s, info);
}

int skinny_watchdog(uint32_t* status, bool clear) {
  unsigned v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_sk_watchdog, sizeof(v));
  if (e != cudaSuccess) return fail(AOTK_ERR_CUDA, "watchdog read: %s", cudaGetErrorString(e));
  if (clear) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_sk_watchdog, &zero, sizeof(zero));
    if (e != cudaSuccess) return fail(AOTK_ERR_CUDA, "watchdog clear: %s", cudaGetErrorString(e));
  }
  *status |= v;
  return AOTK_OK;
}

}  // namespace aotk
