// bf16 grouped expert GEMMs on CTA pairs (tcgen05.mma.cta_group::2, "2-SM" MMA).
//
// Same math as the single-CTA kernel in gemm_tc.cu (reference python/vesper/model.py:295-298:
// gemm1 h = ERA(x We_gate^T + b) * (x We_up^T + b), gemm2 y = h Wd^T + b), computed on
// 256 x 256 output tiles by a cluster of two CTAs on two SMs:
//   * each CTA loads its own 128 rows of A and its own half (128 rows) of B per k-block
//     into its own shared memory (6-stage ring, 32 KB per stage); both CTAs' copies count
//     on the leader CTA's barrier;
//   * the leader's MMA thread issues tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16):
//     the pair's tensor cores read A from their own CTA and B from both, and each CTA's TMEM
//     receives its 128 accumulator rows;
//   * the leader's commits arrive on both CTAs' barriers (commit multicast); each CTA's
//     epilogue drains its own TMEM rows and reports back to the leader.
// Per CTA this moves 32 KB per k-block for a 128 x 256 x 64 slice instead of 48 KB, and the
// same shared memory holds 6 stages instead of 4.  Expert segments are padded to 256 rows so
// both halves of a pair tile belong to one expert.  For gemm1 the B tile is [128 gate rows |
// 128 up rows]: the leader loads the gate half, the follower the up half, and the pair's
// accumulator holds gate in columns 0..127 and up in 128..255 for every row.
//
// All waits are bounded (kWaitLimitNs) and report a status code; no TMA multicast is used
// (each CTA fetches only its own tile from this GPU's own memory).
#include <stdio.h>

#include "common.cuh"
#include "kernels.h"

namespace vmoe {
namespace {

constexpr int BK = 64;
constexpr int PAIR_M = 2 * kTileM;          // 256 rows per pair tile
constexpr int BN = 256;                      // output columns per pair tile
constexpr uint32_t A_BYTES = kTileM * BK * 2;       // 16 KB: this CTA's 128 rows
constexpr uint32_t B_BYTES = (BN / 2) * BK * 2;     // 16 KB: this CTA's half of B
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int STAGES = 6;
constexpr uint32_t TMEM_COLS = 2 * BN;              // two accumulators of this CTA's rows
constexpr uint32_t IDESC = umma_idesc_bf16(PAIR_M, BN);

struct PairShared {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];  // leader's are used: 8 arrivals (4 epilogue warps x 2 CTAs)
  uint64_t done;
  uint32_t tmem_base;
  int abort;
};

constexpr size_t SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + sizeof(PairShared) + 64;

__device__ __forceinline__ bool aborted(const PairShared* sh) {
  return *reinterpret_cast<const volatile int*>(&sh->abort) != 0;
}
__device__ __forceinline__ void set_abort(PairShared* sh, int* status, int code) {
  *reinterpret_cast<volatile int*>(&sh->abort) = 1;
  report(status, code);
}

__device__ __forceinline__ int pair_expert_of(const TcGemmArgs& args, int m) {
  const int e = args.tile_expert[m];
  if (static_cast<unsigned>(e) < static_cast<unsigned>(args.num_experts)) return e;
  report(args.status, kStatusBadExpert);
  return 0;
}

enum PairEpi { kPairPlain = 0, kPairGated = 1, kPairGluBwd = 2, kPairPush = 3 };

// Tile index -> (m tile, n tile).  Row-major over (m, n) unless args.band_n = b > 0: then
// each expert's tiles (its m tiles form one run of tile_expert, written contiguously by the
// plan) are taken in bands of b n tiles, every m tile of the expert for band 0, then band 1,
// ...: a wave of consecutive tiles shares a few A tiles and b B tiles, and the expert's A and
// the band's B stay in L2 while the band lasts.  Either order is a permutation of the same
// tiles inside each expert's range of tile indices.  A CTA's tiles ascend, so the run bounds
// are found by a short scan only when the CTA moves to another expert's run.
struct TileOrder {
  int m0 = 0, m1 = 0;  // the current expert run [m0, m1) of m tiles
  __device__ __forceinline__ void coords(const TcGemmArgs& args, int num_m, int n_tiles,
                                         int tile, int& m, int& n) {
    const int mt = tile / n_tiles;
    const int nb = args.band_n;
    if (nb <= 0 || nb >= n_tiles || !args.tile_expert) {
      m = mt;
      n = tile - mt * n_tiles;
      return;
    }
    if (mt < m0 || mt >= m1) {
      const int e = args.tile_expert[mt];
      m0 = mt;
      while (m0 > 0 && args.tile_expert[m0 - 1] == e) --m0;
      m1 = mt + 1;
      while (m1 < num_m && args.tile_expert[m1] == e) ++m1;
    }
    const int cnt = m1 - m0;
    const int l = tile - m0 * n_tiles;  // 0 .. cnt * n_tiles - 1
    const int full = n_tiles / nb;      // whole bands; then one band of the rest
    const int band = l / (cnt * nb);
    if (band < full) {
      const int r = l - band * cnt * nb;
      m = m0 + r / nb;
      n = band * nb + r % nb;
    } else {
      const int w = n_tiles - full * nb;
      const int r = l - full * cnt * nb;
      m = m0 + r / w;
      n = full * nb + r % w;
    }
  }
};

// push epilogue staging: per epilogue warp 32 rows x 64 bf16 columns, 144-byte row pitch
constexpr int PUSH_PITCH = 72;  // elements
constexpr uint32_t PUSH_STG_BYTES = 4 * 32 * PUSH_PITCH * 2;

__device__ __forceinline__ void st_peer_v4(char* p, uint4 v) {
  *reinterpret_cast<uint4*>(p) = v;
}

// Epilogue warps per CTA: four (one per TMEM lane quarter), eight for the gated gate|up
// epilogue and the GLU backward, whose per-element work (ERA, or ERA and its derivative with
// two loads and two stores) outlasts a short tile's main loop with four (32 k-blocks at
// d_model 2048): two warps share each lane quarter, each taking half the columns.
template <int EPI>
constexpr int pair_epi_warps() { return EPI == kPairGluBwd || EPI == kPairGated ? 8 : 4; }
template <int EPI>
constexpr int pair_threads() { return 64 + 32 * pair_epi_warps<EPI>(); }

template <int EPI>
__global__ void __launch_bounds__(pair_threads<EPI>(), 1)
tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap a_map,
                    const __grid_constant__ CUtensorMap b_map, const TcGemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t a_s = base;
  const uint32_t b_s = base + STAGES * A_BYTES;
  PairShared* sh = reinterpret_cast<PairShared*>(gbase + STAGES * STAGE_BYTES);
  // push staging (kPairPush only) sits after the shared state
  __nv_bfloat16* push_stg = reinterpret_cast<__nv_bfloat16*>(
      gbase + ((STAGES * STAGE_BYTES + sizeof(PairShared) + 127) & ~static_cast<size_t>(127)));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&sh->full[s]), 1);
      mbar_init(smem_u32(&sh->empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&sh->tfull[a]), 1);
      mbar_init(smem_u32(&sh->tempty[a]), 2 * pair_epi_warps<EPI>());
    }
    mbar_init(smem_u32(&sh->done), 1);
    sh->abort = 0;
    fence_mbar_init();
    prefetch_tmap(&a_map);
    prefetch_tmap(&b_map);
  }
  cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA arrive or copy
  if (warp == 1) tmem_alloc_pair(smem_u32(&sh->tmem_base), TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  const int n_tiles = args.n_tiles, k_blocks = args.k_blocks;
  int num_m = *args.num_m_tiles;
  if (num_m > args.max_m_tiles || num_m < 0) {
    if (threadIdx.x == 0) report(args.status, kStatusBadTileCount);
    num_m = num_m < 0 ? 0 : args.max_m_tiles;
  }
  const int total = num_m * n_tiles;
  const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int it = 0;
      TileOrder order;
      for (int tile = pair; tile < total; tile += num_pairs) {
        int m, n;
        order.coords(args, num_m, n_tiles, tile, m, n);
        const int e = pair_expert_of(args, m);
        const int a_row = m * PAIR_M + static_cast<int>(rank) * kTileM;
        const int b_row = e * args.b_rows_per_expert + n * BN + static_cast<int>(rank) * (BN / 2);
        bool ok = true;
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(smem_u32(&sh->empty[s]), ph ^ 1)) {
            set_abort(sh, args.status, kStatusTimeoutProducer);
            ok = false;
            break;
          }
          if (aborted(sh)) { ok = false; break; }
          const uint32_t fb = smem_u32(&sh->full[s]);
          if (leader) mbar_arrive_expect_tx(fb, 2 * STAGE_BYTES);
          const uint32_t fb_leader = mapa_shared(fb, 0);
          tma_load_2d_pair(a_s + s * A_BYTES, &a_map, fb_leader, kb * BK, a_row);
          tma_load_2d_pair(b_s + s * B_BYTES, &b_map, fb_leader, kb * BK, b_row);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader only) ----------------
    if (leader && lane == 0) {
      int it = 0, local = 0;
      for (int tile = pair; tile < total; tile += num_pairs, ++local) {
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait_cluster(smem_u32(&sh->tempty[acc]), aph ^ 1)) {
          set_abort(sh, args.status, kStatusTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(smem_u32(&sh->full[s]), ph)) {
            set_abort(sh, args.status, kStatusTimeoutMma);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = a_s + s * A_BYTES, b_addr = b_s + s * B_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            umma_bf16_pair(d_tmem, umma_desc_sw128(a_addr + k * 32),
                           umma_desc_sw128(b_addr + k * 32), IDESC, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(smem_u32(&sh->empty[s]), 0x3);  // frees the stage in both CTAs
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&sh->tfull[acc]), 0x3);  // both CTAs' epilogues may read
        if (aborted(sh)) break;
      }
      umma_commit_pair(smem_u32(&sh->done), 0x1);
      if (!mbar_wait(smem_u32(&sh->done), 0)) report(args.status, kStatusTimeoutDrain);
    }
  } else {
    // ---------------- epilogue (warps 2..5, both CTAs) ----------------
    const int q = warp & 3;                     // TMEM lane quarter this warp may access
    const int part = (warp - 2) >> 2;  // which share of the columns (eight epilogue warps)
    int local = 0;
    TileOrder order;
    for (int tile = pair; tile < total; tile += num_pairs, ++local) {
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      const bool got = mbar_wait(smem_u32(&sh->tfull[acc]), aph);
      __syncwarp();
      if (!__all_sync(0xffffffffu, got)) {
        if (lane == 0) set_abort(sh, args.status, kStatusTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      int m, n;
      order.coords(args, num_m, n_tiles, tile, m, n);
      const int e = pair_expert_of(args, m);
      const int64_t row = static_cast<int64_t>(m) * PAIR_M + rank * kTileM + q * 32 + lane;
      const uint32_t t_row = tmem + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      __nv_bfloat16* outp = static_cast<__nv_bfloat16*>(args.out) + row * args.ldo;
      if constexpr (EPI == kPairGated) {
        const float* bias = args.bias + static_cast<int64_t>(e) * args.bias_ld + n * BN;
        outp += n * (BN / 2);
        // training: also keep the pre-activations for the backward (tile layout: gate | up)
        __nv_bfloat16* gup = args.gu_out ? static_cast<__nv_bfloat16*>(args.gu_out) +
                                               row * args.gu_ld + n * BN
                                         : nullptr;
        constexpr int kColsG = (BN / 2) / (pair_epi_warps<EPI>() / 4);  // gate columns per warp
#pragma unroll 1
        for (int c = part * kColsG; c < (part + 1) * kColsG; c += 32) {
          float g[32], u[32];
          tmem_ld32(t_row + c, g);
          tmem_ld32(t_row + BN / 2 + c, u);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            g[j] += bias[c + j];
            u[j] += bias[BN / 2 + c + j];
          }
          if (gup) {
            uint32_t pg[16], pu[16];
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              pg[j / 2] = pack_bf16x2(g[j], g[j + 1]);
              pu[j / 2] = pack_bf16x2(u[j], u[j + 1]);
            }
            uint4* dg = reinterpret_cast<uint4*>(gup + c);
            uint4* du = reinterpret_cast<uint4*>(gup + BN / 2 + c);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              dg[v] = make_uint4(pg[4 * v], pg[4 * v + 1], pg[4 * v + 2], pg[4 * v + 3]);
              du[v] = make_uint4(pu[4 * v], pu[4 * v + 1], pu[4 * v + 2], pu[4 * v + 3]);
            }
          }
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float h0 = era_fast(g[j], args.gamma) * u[j];
            const float h1 = era_fast(g[j + 1], args.gamma) * u[j + 1];
            packed[j / 2] = pack_bf16x2(h0, h1);
          }
          uint4* dst = reinterpret_cast<uint4*>(outp + c);
#pragma unroll
          for (int v = 0; v < 4; ++v)
            dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
        }
      } else if constexpr (EPI == kPairGluBwd) {
        // accumulator = dh for I columns [n*BN, n*BN + BN); g, u at their interleaved
        // positions (128-column blocks: gate then up) of the saved pre-activations
        const __nv_bfloat16* gurow = static_cast<const __nv_bfloat16*>(args.gu_in) + row * args.gu_ld;
        constexpr int kCols = BN / (pair_epi_warps<EPI>() / 4);
#pragma unroll 1
        for (int c = part * kCols; c < (part + 1) * kCols; c += 32) {
          const int i0 = n * BN + c;
          if (i0 >= args.i_valid) break;
          const int gcol = (i0 / 128) * 256 + (i0 & 127);
          float dh[32], g[32], u[32];
          tmem_ld32(t_row + c, dh);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            load16_to_f(gurow + gcol + 8 * v, g + 8 * v);
            load16_to_f(gurow + gcol + 128 + 8 * v, u + 8 * v);
          }
          uint32_t pg[16], pu[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float a0, d0, a1, d1;
            era_and_grad_fast(g[j], args.gamma, a0, d0);
            era_and_grad_fast(g[j + 1], args.gamma, a1, d1);
            pg[j / 2] = pack_bf16x2(dh[j] * u[j] * d0, dh[j + 1] * u[j + 1] * d1);
            pu[j / 2] = pack_bf16x2(dh[j] * a0, dh[j + 1] * a1);
          }
          uint4* dg = reinterpret_cast<uint4*>(outp + gcol);
          uint4* du = reinterpret_cast<uint4*>(outp + gcol + 128);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            dg[v] = make_uint4(pg[4 * v], pg[4 * v + 1], pg[4 * v + 2], pg[4 * v + 3]);
            du[v] = make_uint4(pu[4 * v], pu[4 * v + 1], pu[4 * v + 2], pu[4 * v + 3]);
          }
        }
      } else if constexpr (EPI == kPairPush) {
        // this thread's row goes back to the rank that sent it (epoch-tagged address)
        const float* bias = args.bias + static_cast<int64_t>(e) * args.bias_ld + n * BN;
        const int64_t ret = args.push_ret[row];
        char* dst = nullptr;
        if (static_cast<unsigned>(ret >> 32) == args.push_epoch) {
          const int src = static_cast<int>((ret >> 24) & 0xFF);
          const int64_t j = ret & 0xFFFFFF;
          if (src < args.push_G && j < args.push_back_rows)
            dst = args.push_peers[src] + args.push_back_off +
                  (j * args.ldo + static_cast<int64_t>(n) * BN) * 2;
        }
        __nv_bfloat16* stg = push_stg + q * 32 * PUSH_PITCH;
#pragma unroll 1
        for (int c = 0; c < BN; c += 64) {
          float v[64];
          tmem_ld32(t_row + c, v);
          tmem_ld32(t_row + c + 32, v + 32);
          uint32_t packed[32];
#pragma unroll
          for (int j = 0; j < 64; j += 2)
            packed[j / 2] = pack_bf16x2(v[j] + bias[c + j], v[j + 1] + bias[c + j + 1]);
          __syncwarp();
          uint4* srow = reinterpret_cast<uint4*>(stg + lane * PUSH_PITCH);
#pragma unroll
          for (int u = 0; u < 8; ++u)
            srow[u] = make_uint4(packed[4 * u], packed[4 * u + 1], packed[4 * u + 2], packed[4 * u + 3]);
          __syncwarp();
          // eight lanes per row: 128 contiguous bytes of one row per group of eight lanes,
          // four rows per pass, eight passes for the warp's 32 rows
#pragma unroll
          for (int rr = 0; rr < 8; ++rr) {
            const int r = rr * 4 + (lane >> 3), seg = lane & 7;
            const unsigned long long d =
                __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(dst), r);
            if (d) {
              const uint4 val = reinterpret_cast<const uint4*>(stg + r * PUSH_PITCH)[seg];
              st_peer_v4(reinterpret_cast<char*>(d) + c * 2 + seg * 16, val);
            }
          }
        }
      } else {
        // plain: + bias (none when args.bias is null)
        const float* bias = args.bias ? args.bias + static_cast<int64_t>(e) * args.bias_ld + n * BN
                                      : nullptr;
        outp += n * BN;
        const bool store = args.row_limit <= 0 || row < args.row_limit;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v32[32];
          tmem_ld32(t_row + c, v32);
          if (!store) continue;
          if (bias) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v32[j] += bias[c + j];
          }
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) packed[j / 2] = pack_bf16x2(v32[j], v32[j + 1]);
          uint4* dst = reinterpret_cast<uint4*>(outp + c);
#pragma unroll
          for (int v = 0; v < 4; ++v)
            dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&sh->tempty[acc]), 0));
    }
  }

  // pushed rows must be visible to the peers before the signal that follows this kernel
  if constexpr (EPI == kPairPush) __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0 && aborted(sh)) {
    // copies issued by this CTA land on the leader's barriers; give any still in flight a
    // bounded time to finish before the shared memory is released
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 200000ull) {
    }
  }
  cluster_sync_all();  // the leader's MMAs (which read both CTAs' smem) are complete
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
}

}  // namespace

namespace {
template <int EPI>
cudaError_t launch_pair(const CUtensorMap& a_map, const CUtensorMap& b_map, const TcGemmArgs& args,
                        int64_t max_pair_tiles, int num_sms, cudaStream_t s) {
  auto kern = tc_gemm_pair_kernel<EPI>;
  constexpr size_t smem_bytes = SMEM_BYTES + (EPI == kPairPush ? PUSH_STG_BYTES + 128 : 0);
  static_assert(smem_bytes <= 232448, "shared memory budget");
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem_bytes));
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(pair_threads<EPI>(), 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // as many CTA pairs as can be resident at once (persistent), no more than the work
  cfg.gridDim = dim3(static_cast<unsigned>(num_sms & ~1), 1, 1);
  int max_clusters = 0;
  err = cudaOccupancyMaxActiveClusters(&max_clusters, reinterpret_cast<const void*>(kern), &cfg);
  if (err != cudaSuccess) return err;
  if (max_clusters < 1) return cudaErrorInvalidConfiguration;
  int64_t work = max_pair_tiles * args.n_tiles;
  if (work < 1) work = 1;
  int64_t pairs = work < max_clusters ? work : max_clusters;
  if (pairs > num_sms / 2) pairs = num_sms / 2;  // the caller's SM budget
  if (pairs < 1) pairs = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  err = cudaLaunchKernelEx(&cfg, kern, a_map, b_map, args);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_tc_gemm_pair(bool gated, const CUtensorMap& a_map, const CUtensorMap& b_map,
                                const TcGemmArgs& args, int64_t max_pair_tiles, int num_sms,
                                cudaStream_t s) {
  if (gated) return launch_pair<kPairGated>(a_map, b_map, args, max_pair_tiles, num_sms, s);
  return launch_pair<kPairPlain>(a_map, b_map, args, max_pair_tiles, num_sms, s);
}

cudaError_t launch_tc_gemm_pair_push(const CUtensorMap& a_map, const CUtensorMap& b_map,
                                     const TcGemmArgs& args, int64_t max_pair_tiles, int num_sms,
                                     cudaStream_t s) {
  if (!args.push_ret || !args.push_peers || !args.bias || args.push_G < 1 || args.push_G > 256)
    return cudaErrorInvalidValue;
  return launch_pair<kPairPush>(a_map, b_map, args, max_pair_tiles, num_sms, s);
}

cudaError_t launch_tc_gemm_pair_glu_bwd(const CUtensorMap& a_map, const CUtensorMap& b_map,
                                        const TcGemmArgs& args, int64_t max_pair_tiles,
                                        int num_sms, cudaStream_t s) {
  if (!args.gu_in || args.i_valid <= 0) return cudaErrorInvalidValue;
  return launch_pair<kPairGluBwd>(a_map, b_map, args, max_pair_tiles, num_sms, s);
}

}  // namespace vmoe
