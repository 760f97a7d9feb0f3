// Persistent tcgen05 GEMM on CTA pairs: C[M,N] = A[M,K] * B[K,N].
//
// A cluster of two CTAs (on two SMs) computes 256 x BNP output tiles with
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16), BNP = 256 (one MMA per
// K step) or 512 (two, into a 512-column accumulator that fills TMEM):
//   * CTA r of the pair TMA-loads rows [m0 + 128r, +128) of A and, for each
//     256-column MMA h, columns [n0 + 256h + 128r, +128) of B into its own
//     shared memory; the MMA reads both CTAs' halves.  Per 64-deep K block an
//     SM stages 32 KB for 128 x 256 x 64 of MMA work (BNP = 256) or 48 KB for
//     128 x 512 x 64 (BNP = 512) - against 48 KB for 128 x 256 x 64 in the
//     1-CTA kernel - so the wide tile moves half as many operand bytes per
//     flop through L2 and shared memory, and its 4-stage ring covers twice
//     the MMA time.  On B200, where these GEMMs run at the 1 kW power cap,
//     fewer bytes moved per flop show up as clock and tensor-pipe occupancy
//     (8192^3: 1.08-1.11x the 1-CTA kernel).  No load is multicast.
//   * The full barrier of a stage lives in the first CTA: its producer
//     expects the bytes of both CTAs' loads, the second CTA's loads complete
//     their bytes there.  The first CTA's MMA warp issues all MMAs and its
//     commits arrive on the empty / accumulator-full barriers of both CTAs.
//   * Each CTA's four epilogue warps read their 128 accumulator rows from
//     their own TMEM (BNP = 256: two 256-column accumulators, so the epilogue
//     of one tile overlaps the MMAs of the next; BNP = 512: one, so the next
//     tile's MMAs wait for its read-out; splitting the read-out over eight
//     warps measured no faster), release the accumulator on the first CTA's
//     barrier and TMA-store 32 x 64 boxes of C.
// Every wait is bounded (sm100.cuh); both CTAs meet at a cluster barrier
// before TMEM is freed and before either exits.
#include <type_traits>

#include "common.h"
#include "gemm_internal.h"
#include "sm100.cuh"
#include "tmap.h"
#include "vec.cuh"

namespace aotk {
namespace {

using namespace sm100;

__device__ unsigned g_tc2_watchdog;

constexpr int kBM = 256;      // rows per pair tile (128 per CTA)
constexpr int kHalf = 128;
constexpr int kBK = 64;
constexpr int kUmmaK = 16;
constexpr int kThreads = 192;  // producer, MMA and 4 epilogue warps
constexpr int kGroupM = 8;    // M pair-tiles per raster group
constexpr uint32_t kTmemCols = 512;  // all of TMEM: 2 x 256 or 1 x 512 accumulator columns

enum : unsigned { kWdProducer = 256u, kWdMma = 512u, kWdEpilogue = 1024u };

// BNP = columns per pair tile: 256 (one MMA of N = 256 per K step, two
// accumulators so the epilogue of one tile overlaps the next tile's MMAs) or
// 512 (two MMAs of N = 256 per K step into one 512-column accumulator, which
// fills TMEM: each SM then stages 48 KB of operands per 128 x 512 x 64 of
// MMA work instead of 32 KB per 128 x 256 x 64).
template <int STAGES, int BNP>
struct Tc2Layout {
  static constexpr int kMmas = BNP / 256;               // MMAs of N = 256 per K step
  static constexpr int kAccs = BNP == 256 ? 2 : 1;      // accumulators in TMEM
  static constexpr uint32_t kABytes = kHalf * kBK * 2;  // this CTA's 128 rows of A
  static constexpr uint32_t kBBox = kBK * 128;          // 64 (N) x 64 (K)
  static constexpr int kBBoxes = BNP / 2 / 64;          // this CTA's BNP / 2 columns of B
  static constexpr uint32_t kBBytes = kBBoxes * kBBox;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kPairStageBytes = 2 * kStageBytes;
  static constexpr uint32_t kCBuf = 32 * 128;
  static constexpr uint32_t kOffA = 0;
  static constexpr uint32_t kOffB = kOffA + STAGES * kABytes;
  static constexpr uint32_t kOffC = kOffB + STAGES * kBBytes;
  static constexpr uint32_t kOffBar = kOffC + 4 * 2 * kCBuf;
  static constexpr uint32_t kNumBars = 2 * STAGES + 5;  // full, empty, tfull x2, tempty x2, drain
  static constexpr uint32_t kOffMisc = kOffBar + kNumBars * 8;
  static constexpr uint32_t kBytes = kOffMisc + 16;
  static constexpr uint32_t kAlloc = kBytes + 1024;
  static_assert(BNP == 256 || BNP == 512, "pair tiles are 256 or 512 columns wide");
  static_assert(kAccs * BNP <= static_cast<int>(kTmemCols), "accumulators must fit in TMEM");
};

__device__ __forceinline__ void pair_tile_coords(int tile, int tiles_m, int tiles_n, int& mb,
                                                 int& nb) {
  const int per_group = kGroupM * tiles_n;
  const int g = tile / per_group;
  const int first_m = g * kGroupM;
  const int gm = min(tiles_m - first_m, kGroupM);
  const int local = tile - g * per_group;
  mb = first_m + local % gm;
  nb = local / gm;
}

// Work item i of a pair: its whole tiles (tile < tail_begin, round robin
// over the pairs), then at most one half of a tail tile (half = 0 or 1, N
// columns [BNP/2 half, BNP/2 half + BNP/2) of the tile; for silu_mul the
// matching gate and up columns: 64 + 64 of a 256-column tile, one whole
// [gate | up] block of a 512-column tile).  Without a cut tail, tail_begin
// equals the tile count.
__device__ __forceinline__ bool pair_item(int i, int pair, int num_pairs, int num_tiles,
                                          int tail_begin, int& tile, int& half) {
  const int whole = tail_begin > pair ? (tail_begin - pair + num_pairs - 1) / num_pairs : 0;
  if (i < whole) {
    tile = pair + i * num_pairs;
    half = -1;
    return true;
  }
  const int u = pair + (i - whole) * num_pairs;
  if (u >= 2 * (num_tiles - tail_begin)) return false;
  tile = tail_begin + u / 2;
  half = u % 2;
  return true;
}

// kSiluMul: B is a gate/up weight interleaved in blocks of 128 columns
// ([gate_j | up_j], N = 2I) and the kernel writes act = silu(g) * u ([M, I],
// through tmC), with both accumulators of row m first multiplied by
// row_scale[m] when row_scale is given.
template <typename T, int STAGES, int BNP, bool kSiluMul>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, int M, int N, int K, uint32_t idesc,
                    const float* __restrict__ row_scale, int tail_begin) {
  using L = Tc2Layout<STAGES, BNP>;
  constexpr int kBN = BNP;
  const int n_out = kSiluMul ? N / 2 : N;  // columns of the output
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
  unsigned* wd = &g_tc2_watchdog;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: issues the MMAs
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int num_pairs = static_cast<int>(gridDim.x >> 1);
  const int tiles_m = (M + kBM - 1) / kBM;
  const int tiles_n = (N + kBN - 1) / kBN;
  const int num_tiles = tiles_m * tiles_n;
  const int kblocks = (K + kBK - 1) / kBK;
  // A half tail item is one MMA per K step: N = 128 for 256-column tiles,
  // N = 256 (the tile's first MMA) for 512-column tiles.
  const uint32_t idesc_half =
      BNP == 256 ? (idesc & ~(0x3Fu << 17)) | ((128u >> 3) << 17) : idesc;

  // The next kernel on the stream may start its prologue as SMs free up.
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
      mbar_init(tempty_bar(a), 8);  // 4 epilogue warps in each CTA of the pair
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_addr(tmem_slot), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs initialised before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Global memory is touched only from here on, once the previous kernel on
  // the stream has completed (programmatic dependent launch).
  pdl_wait_prior();

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      int tile, half;
      for (int i = 0; ok && pair_item(i, pair, num_pairs, num_tiles, tail_begin, tile, half);
           ++i) {
        int mb, nb;
        pair_tile_coords(tile, tiles_m, tiles_n, mb, nb);
        const int row0 = mb * kBM + static_cast<int>(rank) * kHalf;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, wd, kWdProducer)) {
            ok = false;
            break;
          }
          // The stage's bytes are counted on the first CTA's full barrier.
          const uint32_t fb = map_to_rank(full_bar(stage), 0);
          if (rank == 0)
            mbar_arrive_expect_tx(full_bar(stage),
                                  half < 0 ? L::kPairStageBytes
                                           : 2 * (L::kABytes + (L::kBBoxes / 2) * L::kBBox));
          tma_load_2d_pair(sA + stage * L::kABytes, &tmA, kb * kBK, row0, fb);
          if (half < 0) {
            // Box j feeds MMA j / 2 (columns [256 h, 256 h + 256) of the
            // tile), of which this CTA stages [128 rank, 128 rank + 128).
#pragma unroll
            for (int j = 0; j < L::kBBoxes; ++j)
              tma_load_2d_pair(
                  sB + stage * L::kBBytes + j * L::kBBox, &tmB,
                  nb * kBN + (j / 2) * 256 + static_cast<int>(rank) * kHalf + (j % 2) * 64,
                  kb * kBK, fb);
          } else if constexpr (BNP == 256) {
            // One 64-column box per CTA: columns [128 half + 64 rank, +64),
            // or for silu_mul gate (rank 0) / up (rank 1) columns 64 half on.
            const int col = kSiluMul ? nb * kBN + static_cast<int>(rank) * 128 + half * 64
                                     : nb * kBN + half * 128 + static_cast<int>(rank) * 64;
            tma_load_2d_pair(sB + stage * L::kBBytes, &tmB, col, kb * kBK, fb);
          } else {
            // The boxes of MMA `half` alone: columns [256 half, 256 half +
            // 256) of the tile (for silu_mul one [gate | up] block), of which
            // this CTA stages [128 rank, 128 rank + 128).
#pragma unroll
            for (int j = 0; j < 2; ++j)
              tma_load_2d_pair(sB + stage * L::kBBytes + j * L::kBBox, &tmB,
                               nb * kBN + half * 256 + static_cast<int>(rank) * kHalf + j * 64,
                               kb * kBK, fb);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // The first CTA's full barriers see every load of the pair: drain there.
      if (rank == 0) {
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
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer (first CTA only) ----------------
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      int tile, half;
      for (int i = 0; ok && pair_item(i, pair, num_pairs, num_tiles, tail_begin, tile, half);
           ++i) {
        if (!mbar_wait_bounded(tempty_bar(acc), acc_phase ^ 1u, abort_flag, wd, kWdMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_bounded(full_bar(stage), phase, abort_flag, wd, kWdMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = sA + stage * L::kABytes;
          const uint32_t b0 = sB + stage * L::kBBytes;
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            const uint64_t ad = sdesc_sw128(a0 + k * kUmmaK * 2, 16, 1024);
            if (half < 0) {
#pragma unroll
              for (int h = 0; h < L::kMmas; ++h) {
                const uint64_t bd =
                    sdesc_sw128(b0 + h * 2 * L::kBBox + k * kUmmaK * 128, L::kBBox, 1024);
                umma_f16_pair(d_tmem + h * 256, ad, bd, idesc, kb > 0 || k > 0);
              }
            } else {
              const uint64_t bd = sdesc_sw128(b0 + k * kUmmaK * 128, L::kBBox, 1024);
              umma_f16_pair(d_tmem, ad, bd, idesc_half, kb > 0 || k > 0);
            }
          }
          umma_commit_pair(empty_bar(stage), 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(tfull_bar(acc), 0x3);
        if (++acc == L::kAccs) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      umma_commit_pair(drain_bar, 0x3);
      mbar_drain(drain_bar, 0);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..5, both CTAs) ----------------
    const int q = warp & 3;
    const uint32_t cbuf = sC + (warp - 2) * 2 * L::kCBuf;
    int acc = 0;
    uint32_t acc_phase = 0;
    int nstore = 0;
    int tile, half;
    for (int i = 0; pair_item(i, pair, num_pairs, num_tiles, tail_begin, tile, half); ++i) {
      int mb, nb;
      pair_tile_coords(tile, tiles_m, tiles_n, mb, nb);
      int ok = 1;
      if (lane == 0) ok = mbar_wait_bounded(tfull_bar(acc), acc_phase, abort_flag, wd, kWdEpilogue);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t trow = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                            static_cast<uint32_t>(acc * kBN);
      const int store_y = mb * kBM + static_cast<int>(rank) * kHalf + q * 32;
      // After this warp's last TMEM load of the tile: hand the accumulator
      // back on the first CTA's barrier.
      auto release_if_last = [&](bool last) {
        if (!last) return;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(map_to_rank(tempty_bar(acc), 0));
      };
      // Output chunks of 64 columns: kBN / 64 of C, or (silu_mul) kBN / 128 of
      // act, each from a 64-column gate chunk and the up chunk 128 columns on.
      // A half item holds kBN / 2 accumulator columns: kBN / 128 chunks of
      // C, or kBN / 256 act chunks from gate columns [0, kBN / 4) and up
      // columns [kBN / 4, kBN / 2).
      const int out_chunks =
          half >= 0 ? (kSiluMul ? kBN / 256 : kBN / 128) : (kSiluMul ? kBN / 128 : kBN / 64);
      const int row = store_y + lane;
      float rs = 1.f;
      if (kSiluMul && row_scale != nullptr) rs = row < M ? __ldg(row_scale + row) : 0.f;
#pragma unroll 1
      for (int c = 0; c < out_chunks; ++c) {
        float f[64];
        int store_x;
        if constexpr (kSiluMul) {
          // Interleaved weight: tile columns [256 j, 256 j + 256) hold
          // [gate block | up block] of 128 each.
          const int gcol = half >= 0 ? c * 64 : (c / 2) * 256 + (c % 2) * 64;
          const int ucol = gcol + (half >= 0 ? kBN / 4 : 128);
          uint32_t g[64], u[64];
          tmem_ld_32x32b_x32(trow + gcol, g);
          tmem_ld_32x32b_x32(trow + gcol + 32, g + 32);
          tmem_ld_32x32b_x32(trow + ucol, u);
          tmem_ld_32x32b_x32(trow + ucol + 32, u + 32);
          tmem_wait_ld();
          release_if_last(c == out_chunks - 1);
#pragma unroll
          for (int j = 0; j < 64; ++j)
            f[j] = silu_f(__uint_as_float(g[j]) * rs) * (__uint_as_float(u[j]) * rs);
          store_x = nb * (kBN / 2) + (half >= 0 ? half * (kBN / 4) : 0) + c * 64;
        } else {
          uint32_t r[64];
          tmem_ld_32x32b_x32(trow + c * 64, r);
          tmem_ld_32x32b_x32(trow + c * 64 + 32, r + 32);
          tmem_wait_ld();
          release_if_last(c == out_chunks - 1);
#pragma unroll
          for (int j = 0; j < 64; ++j) f[j] = __uint_as_float(r[j]);
          store_x = nb * kBN + (half >= 0 ? half * (kBN / 2) : 0) + c * 64;
        }
        if (store_x >= n_out || store_y >= M) continue;
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) pk[i] = Elem<T>::pack2(f[2 * i], f[2 * i + 1]);
        const uint32_t buf = cbuf + (nstore & 1) * L::kCBuf;
        if (nstore >= 2 && lane == 0) bulk_wait_read<1>();
        __syncwarp();
        const uint32_t srow = buf + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          st_shared_v4(srow + ((j ^ (lane & 7)) << 4), pk[4 * j], pk[4 * j + 1], pk[4 * j + 2],
                       pk[4 * j + 3]);
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, buf, store_x, store_y);
          bulk_commit();
        }
        ++nstore;
      }
      if (++acc == L::kAccs) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  // Neither CTA frees TMEM or exits while its pair may still use its shared
  // memory (MMA operands, barriers) or its TMEM.
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

template <typename T, int STAGES, int BNP, bool kSiluMul>
int launch_tc2(void* c, const void* a, const void* b, const float* row_scale, int M, int N, int K,
               bool bf16, cudaStream_t stream, const DeviceInfo& info) {
  using L = Tc2Layout<STAGES, BNP>;
  constexpr int kBN = BNP;
  auto kernel = gemm_tc2_kernel<T, STAGES, BNP, kSiluMul>;
  if (int st = ensure_dynamic_smem(reinterpret_cast<const void*>(kernel), L::kAlloc, info)) return st;
  const int n_out = kSiluMul ? N / 2 : N;
  CUtensorMap ta, tb, tc;
  if (int st = make_tmap_2d_16bit(&ta, a, bf16, M, K, K, kBK, kHalf)) return st;
  if (int st = make_tmap_2d_16bit(&tb, b, bf16, K, N, N, 64, kBK)) return st;
  if (int st = make_tmap_2d_16bit(&tc, c, bf16, M, n_out, n_out, 64, 32)) return st;
  const int tiles = ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
  const int max_pairs = info.sm_count / 2;
  int pairs = tiles < max_pairs ? tiles : max_pairs;
  int tail_begin = tiles;
  // A partial last round of at most half the pairs is cut into N halves
  // (twice the pairs, half a tile each).
  const int full = tiles / max_pairs;
  const int rem = tiles - full * max_pairs;
  if (rem > 0 && 2 * rem <= max_pairs) {
    pairs = full > 0 ? max_pairs : 2 * rem;
    tail_begin = full * max_pairs;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // Programmatic dependent launch: the prologue (barrier init, TMEM
  // allocation, descriptor prefetch) overlaps the previous kernel's tail.
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  // Every MMA is M = 256 (128 rows per CTA) x N = 256.
  const uint32_t idesc = idesc_f16(bf16, kBM, 256, /*a_mn_major=*/false, /*b_mn_major=*/true);
  cudaError_t e =
      cudaLaunchKernelEx(&cfg, kernel, ta, tb, tc, M, N, K, idesc, row_scale, tail_begin);
  if (e != cudaSuccess)
    return fail(AOTK_ERR_CUDA, "tcgen05 pair gemm launch: %s", cudaGetErrorString(e));
  return check_launch("tcgen05 pair gemm");
}

constexpr int kTc2Stages = 6;      // 256-column pair tiles: 6 x 32 KB stages
constexpr int kTc2WideStages = 4;  // 512-column pair tiles: 4 x 48 KB stages

}  // namespace

int gemm_tc2(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K, int dtype,
             void* stream) {
  DeviceInfo info;
  if (int st = current_device_info(&info)) return st;
  if (int st = require_sm100(info)) return st;
  if (int st = check_tc_preconditions("aotk_gemm_tc2", c, a, b, M, N, K, dtype)) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int m = (int)M, n = (int)N, k = (int)K;
  if (dtype == AOTK_BFLOAT16)
    return launch_tc2<__nv_bfloat16, kTc2Stages, 256, false>(c, a, b, nullptr, m, n, k, true, s,
                                                             info);
  return launch_tc2<__half, kTc2Stages, 256, false>(c, a, b, nullptr, m, n, k, false, s, info);
}

int gemm_tc2_wide(void* c, const void* a, const void* b, int64_t M, int64_t N, int64_t K,
                  int dtype, void* stream) {
  DeviceInfo info;
  if (int st = current_device_info(&info)) return st;
  if (int st = require_sm100(info)) return st;
  if (int st = check_tc_preconditions("aotk_gemm_tc2w", c, a, b, M, N, K, dtype)) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int m = (int)M, n = (int)N, k = (int)K;
  if (dtype == AOTK_BFLOAT16)
    return launch_tc2<__nv_bfloat16, kTc2WideStages, 512, false>(c, a, b, nullptr, m, n, k, true,
                                                                 s, info);
  return launch_tc2<__half, kTc2WideStages, 512, false>(c, a, b, nullptr, m, n, k, false, s, info);
}

int gemm_tc2_silu_mul(void* act, const void* a, const void* b, const float* row_scale, int64_t M,
                      int64_t N2, int64_t K, int dtype, bool wide, void* stream) {
  DeviceInfo info;
  if (int st = current_device_info(&info)) return st;
  if (int st = require_sm100(info)) return st;
  if (int st = check_tc_preconditions("aotk_gemm_silu_mul", act, a, b, M, N2, K, dtype)) return st;
  if (N2 % 256 != 0)
    return fail(AOTK_ERR_UNSUPPORTED,
                "aotk_gemm_silu_mul: interleaved width 2*I = %lld must be a multiple of 256",
                (long long)N2);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int m = (int)M, n = (int)N2, k = (int)K;
  const bool bf16 = dtype == AOTK_BFLOAT16;
  if (wide) {
    if (bf16)
      return launch_tc2<__nv_bfloat16, kTc2WideStages, 512, true>(act, a, b, row_scale, m, n, k,
                                                                  true, s, info);
    return launch_tc2<__half, kTc2WideStages, 512, true>(act, a, b, row_scale, m, n, k, false, s,
                                                         info);
  }
  if (bf16)
    return launch_tc2<__nv_bfloat16, kTc2Stages, 256, true>(act, a, b, row_scale, m, n, k, true, s,
                                                            info);
  return launch_tc2<__half, kTc2Stages, 256, true>(act, a, b, row_scale, m, n, k, false, s, info);
}

int tc2_watchdog(uint32_t* status, bool clear) {
  unsigned v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc2_watchdog, sizeof(v));
  if (e != cudaSuccess) return fail(AOTK_ERR_CUDA, "watchdog read: %s", cudaGetErrorString(e));
  if (clear) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_tc2_watchdog, &zero, sizeof(zero));
    if (e != cudaSuccess) return fail(AOTK_ERR_CUDA, "watchdog clear: %s", cudaGetErrorString(e));
  }
  *status |= v;
  return AOTK_OK;
}

}  // namespace aotk
