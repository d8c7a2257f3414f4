// Grouped weight-gradient GEMM on the tensor cores (tcgen05 + TMEM + TMA), fp32 out.
//
// For every expert e:  dW_e[M, N] = sum over the rows r of e's segment of  A[r, :]^T B[r, :]
// -- the nn.Linear weight gradient dW = dY^T X that autograd forms for every expert's
// Linear in MoELayer.forward (python/vesper/model.py:295-298, 322) -- with the token rows as
// the reduction (K) dimension, and the bias gradient db_e = sum over the same rows of A.
//
// Both operands stay in their row-major activation layout ([rows, M] and [rows, N]): the
// tiles are loaded "MN-major" (TMA boxes of 64 columns x 64 rows, 128-byte swizzle: every
// 128-byte shared row holds 64 consecutive M (or N) elements of one token row) and the MMA
// reads them transposed (instruction-descriptor A/B major bits; descriptor leading byte
// offset = 8 KB between 64-wide column chunks, stride byte offset = 1 KB between 8-row
// groups), so no transposed copy of any activation is ever written.  The K range of a tile
// is its expert's segment [offs[e], offs[e+1]) (a multiple of 64 rows): experts with more
// tokens run longer K loops, empty experts write zeros.  With bias outputs, every (expert,
// M tile) gets one more work item whose B operand is a constant K-major ones row (N = 16):
// its column 0 is the segment's column sums of A.
//
// One CTA per SM, persistent over (expert, M tile, N tile) work items; warp 0 is the TMA
// producer (A 128 x 64 + B 256 x 64 per stage, 4 stages), warp 1 allocates TMEM (two
// 128 x 256 fp32 accumulators) and issues tcgen05.mma M128 N256 K16, warps 2..5 drain the
// accumulator (tcgen05.ld) and write fp32 rows straight into the caller's gradient tensor,
// un-padding (and for the gate|up weight, de-interleaving) on the way.  Every wait is
// bounded; no TMA multicast is used.
#include <stdio.h>

#include "common.cuh"
#include "kernels.h"

namespace vmoe {
namespace {

constexpr int BK = 64;
constexpr int BN = 256;
constexpr uint32_t CHUNK_BYTES = 64 * BK * 2;   // one 64-column x 64-row box: 8 KB
constexpr uint32_t A_BYTES = 2 * CHUNK_BYTES;   // 128 M columns
constexpr uint32_t B_BYTES = 4 * CHUNK_BYTES;   // 256 N columns
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int STAGES = 4;
constexpr uint32_t ONES_BYTES = 16 * 128;       // 16-row K-major ones tile (row 0 = 1)
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr uint32_t kMajorA = 1u << 15, kMajorB = 1u << 16;  // operand read MN-major
constexpr uint32_t IDESC = umma_idesc_bf16(kTileM, BN) | kMajorA | kMajorB;
constexpr uint32_t IDESC_BIAS = umma_idesc_bf16(kTileM, 16) | kMajorA;  // B: K-major ones

// Descriptor of an MN-major operand chunk sequence: 128-byte swizzle, 64-element MN chunks
// CHUNK_BYTES apart (leading byte offset), 8-row K groups 1024 bytes apart (stride).
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(CHUNK_BYTES >> 4) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

struct WgShared {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t done;
  uint32_t tmem_base;
  int abort;
  int issued;
  int consumed;
};

// per epilogue warp: a 32 x 32 fp32 block (pitch 33) turned from row-per-thread into
// row-per-store, so every store instruction writes 128 contiguous bytes of one row
constexpr int STG_PITCH = 33;
constexpr uint32_t STG_BYTES = 4 * 32 * STG_PITCH * 4;

constexpr size_t SMEM_BYTES =
    1024 + STAGES * STAGE_BYTES + ONES_BYTES + STG_BYTES + sizeof(WgShared) + 64;

// Destination row of M row `mrow` (plain, or the gate|up de-interleave), null if outside.
__device__ __forceinline__ float* wg_dst_row(const WgradArgs& a, int e, int mrow) {
  int which = 0, i = mrow;
  if (a.mode == 1) {
    which = (mrow / 128) & 1;
    i = (mrow / 256) * 128 + (mrow & 127);
  }
  if (i >= a.m_valid) return nullptr;
  return (which ? a.out2 : a.out) + static_cast<int64_t>(e) * a.out_expert_stride +
         static_cast<int64_t>(i) * a.ld_out;
}

// Drain one 128 x 256 accumulator tile (this warp's 32 rows starting at M row mrow0).
__device__ __forceinline__ void wg_store_tile(const WgradArgs& a, int e, int mrow0, int ncol0,
                                              uint32_t t_row, bool have_acc, float* stg,
                                              int lane) {
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    float v[32];
    if (have_acc) {
      tmem_ld32(t_row + c, v);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = 0.f;
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 32; ++j) stg[lane * STG_PITCH + j] = v[j];
    __syncwarp();
    const int col = ncol0 + c + lane;
#pragma unroll 4
    for (int r = 0; r < 32; ++r) {
      float* dst = wg_dst_row(a, e, mrow0 + r);
      if (dst && col < a.n_valid) dst[col] = stg[r * STG_PITCH + lane];
    }
  }
}

__device__ __forceinline__ bool aborted(const WgShared* sh) {
  return *reinterpret_cast<const volatile int*>(&sh->abort) != 0;
}
__device__ __forceinline__ void set_abort(WgShared* sh, int* status, int code) {
  *reinterpret_cast<volatile int*>(&sh->abort) = 1;
  report(status, code);
}

// K blocks [kb0, kb0 + nk) of expert e's segment (bounded by the operands' row count).
__device__ __forceinline__ void seg_blocks(const WgradArgs& a, int e, int& kb0, int& nk) {
  int r0 = 0, r1 = a.seg_rows_host;
  if (a.seg_offs) {
    r0 = a.seg_offs[e];
    r1 = a.seg_offs[e + 1];
  }
  if (r0 < 0 || r1 < r0 || r1 > a.rows_total || (r0 % BK) || (r1 % BK)) {
    report(a.status, kStatusBadSlot);
    kb0 = 0;
    nk = 0;
    return;
  }
  kb0 = r0 / BK;
  nk = (r1 - r0) / BK;
}

struct Work {
  int e, m, n;
  bool bias;
};

__device__ __forceinline__ Work work_of(const WgradArgs& a, int tile) {
  const int nt = a.n_tiles + (a.bias_out ? 1 : 0);
  const int per_expert = a.m_tiles * nt;
  Work w;
  w.e = tile / per_expert;
  const int mn = tile - w.e * per_expert;
  w.m = mn / nt;
  w.n = mn - w.m * nt;
  w.bias = w.n == a.n_tiles;
  return w;
}

__global__ void __launch_bounds__(192, 1)
wgrad_kernel(const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap b_map,
             const WgradArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t a_s = base;
  const uint32_t b_s = base + STAGES * A_BYTES;
  const uint32_t ones_s = base + STAGES * STAGE_BYTES;
  float* stg_all = reinterpret_cast<float*>(gbase + STAGES * STAGE_BYTES + ONES_BYTES);
  auto* sh = reinterpret_cast<WgShared*>(gbase + STAGES * STAGE_BYTES + ONES_BYTES + STG_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  {  // the bias tiles' B operand: row 0 = 64 bf16 ones, rows 1..15 zero
    uint32_t* ones = reinterpret_cast<uint32_t*>(gbase + STAGES * STAGE_BYTES);
    for (int i = threadIdx.x; i < static_cast<int>(ONES_BYTES / 4); i += blockDim.x)
      ones[i] = i < 32 ? 0x3F803F80u : 0u;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&sh->full[s]), 1);
      mbar_init(smem_u32(&sh->empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&sh->tfull[a]), 1);
      mbar_init(smem_u32(&sh->tempty[a]), 4);
    }
    mbar_init(smem_u32(&sh->done), 1);
    sh->abort = 0;
    sh->issued = 0;
    sh->consumed = 0;
    fence_mbar_init();
    prefetch_tmap(&a_map);
    prefetch_tmap(&b_map);
  }
  if (warp == 1) tmem_alloc(smem_u32(&sh->tmem_base), TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  const int total = args.num_experts * args.m_tiles * (args.n_tiles + (args.bias_out ? 1 : 0));

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
        const Work w = work_of(args, tile);
        int kb0, nk;
        seg_blocks(args, w.e, kb0, nk);
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(smem_u32(&sh->empty[s]), ph ^ 1)) {
            set_abort(sh, args.status, kStatusTimeoutProducer);
            ok = false;
            break;
          }
          if (aborted(sh)) { ok = false; break; }
          const uint32_t fb = smem_u32(&sh->full[s]);
          const int row = (kb0 + kb) * BK;
          mbar_arrive_expect_tx(fb, w.bias ? A_BYTES : STAGE_BYTES);
#pragma unroll
          for (int j = 0; j < 2; ++j)
            tma_load_2d(a_s + s * A_BYTES + j * CHUNK_BYTES, &a_map, fb, w.m * kTileM + 64 * j, row);
          if (!w.bias) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              tma_load_2d(b_s + s * B_BYTES + j * CHUNK_BYTES, &b_map, fb, w.n * BN + 64 * j, row);
          }
          *reinterpret_cast<volatile int*>(&sh->issued) = it + 1;
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, local = 0;
      for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++local) {
        const Work w = work_of(args, tile);
        int kb0, nk;
        seg_blocks(args, w.e, kb0, nk);
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(smem_u32(&sh->tempty[acc]), aph ^ 1)) {
          set_abort(sh, args.status, kStatusTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb, ++it) {
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
            const uint32_t accum = (kb | k) != 0 ? 1u : 0u;
            // 16 K rows = two 8-row groups further on
            const uint64_t a_desc = desc_mn_sw128(a_addr + k * 2048);
            if (w.bias)
              umma_bf16(d_tmem, a_desc, umma_desc_sw128(ones_s + k * 32), IDESC_BIAS, accum);
            else
              umma_bf16(d_tmem, a_desc, desc_mn_sw128(b_addr + k * 2048), IDESC, accum);
          }
          umma_commit(smem_u32(&sh->empty[s]));
          *reinterpret_cast<volatile int*>(&sh->consumed) = it + 1;
        }
        if (!ok) break;
        umma_commit(smem_u32(&sh->tfull[acc]));  // with nk == 0: arrives at once
        if (aborted(sh)) break;
      }
      umma_commit(smem_u32(&sh->done));
      if (!mbar_wait(smem_u32(&sh->done), 0)) report(args.status, kStatusTimeoutDrain);
    }
  } else {
    const int q = warp & 3;
    int local = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++local) {
      const Work w = work_of(args, tile);
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      const bool got = mbar_wait(smem_u32(&sh->tfull[acc]), aph);
      __syncwarp();
      if (!__all_sync(0xffffffffu, got)) {
        if (lane == 0) set_abort(sh, args.status, kStatusTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      int kb0, nk;
      seg_blocks(args, w.e, kb0, nk);
      const int mrow = w.m * kTileM + q * 32 + lane;  // row of this expert's M dimension
      // destination row: plain, or the gate|up de-interleave of the packed 2*Ipad rows
      int which = 0, i = mrow;
      if (args.mode == 1) {
        which = (mrow / 128) & 1;
        i = (mrow / 256) * 128 + (mrow & 127);
      }
      const bool row_ok = i < args.m_valid;
      const uint32_t t_row = tmem + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      if (w.bias) {
        float v[16];
        if (nk > 0) {
          tmem_ld16(t_row, v);
        } else {
          v[0] = 0.f;
        }
        if (row_ok)
          ((which && args.bias_out2) ? args.bias_out2 : args.bias_out)
              [static_cast<int64_t>(w.e) * args.m_valid + i] = v[0];
      } else {
        wg_store_tile(args, w.e, mrow - lane, w.n * BN, t_row, nk > 0, stg_all + q * 32 * STG_PITCH,
                      lane);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&sh->tempty[acc]));
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && aborted(sh)) {
    const int issued = *reinterpret_cast<volatile int*>(&sh->issued);
    const int consumed = *reinterpret_cast<volatile int*>(&sh->consumed);
    for (int i = consumed; i < issued; ++i) {
      if (!mbar_wait(smem_u32(&sh->full[i % STAGES]), (i / STAGES) & 1)) {
        report(args.status, kStatusTimeoutDrain);
        break;
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---- the same on CTA pairs (tcgen05.mma.cta_group::2) -----------------------------------
// 256 x 256 pair tiles: CTA `rank` loads its own 128 M columns of A and its own 128 of the
// 256 N columns of B per 64-row K block (16 + 16 KB, 6 stages), the leader's MMA thread
// issues M256 N256 K16 for both, each CTA's TMEM receives its 128 accumulator rows.  Copies
// of both CTAs complete on the leader's barrier; commits arrive on both CTAs' barriers.
constexpr int PAIR_M = 2 * kTileM;
constexpr uint32_t P_A_BYTES = 2 * CHUNK_BYTES;  // this CTA's 128 M columns
constexpr uint32_t P_B_BYTES = 2 * CHUNK_BYTES;  // this CTA's 128 of the 256 N columns
constexpr uint32_t P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
constexpr int P_STAGES = 6;
constexpr uint32_t P_IDESC = umma_idesc_bf16(PAIR_M, BN) | kMajorA | kMajorB;
constexpr uint32_t P_IDESC_BIAS = umma_idesc_bf16(PAIR_M, 16) | kMajorA;

struct PairWgShared {
  uint64_t full[P_STAGES];
  uint64_t empty[P_STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];  // the leader's: 8 arrivals (4 epilogue warps x 2 CTAs)
  uint64_t done;
  uint32_t tmem_base;
  int abort;
};

constexpr size_t P_SMEM_BYTES =
    1024 + P_STAGES * P_STAGE_BYTES + ONES_BYTES + STG_BYTES + sizeof(PairWgShared) + 64;

__device__ __forceinline__ bool p_aborted(const PairWgShared* sh) {
  return *reinterpret_cast<const volatile int*>(&sh->abort) != 0;
}
__device__ __forceinline__ void p_set_abort(PairWgShared* sh, int* status, int code) {
  *reinterpret_cast<volatile int*>(&sh->abort) = 1;
  report(status, code);
}

__global__ void __launch_bounds__(192, 1)
wgrad_pair_kernel(const __grid_constant__ CUtensorMap a_map,
                  const __grid_constant__ CUtensorMap b_map, const WgradArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t a_s = base;
  const uint32_t b_s = base + P_STAGES * P_A_BYTES;
  const uint32_t ones_s = base + P_STAGES * P_STAGE_BYTES;
  float* stg_all = reinterpret_cast<float*>(gbase + P_STAGES * P_STAGE_BYTES + ONES_BYTES);
  auto* sh = reinterpret_cast<PairWgShared*>(gbase + P_STAGES * P_STAGE_BYTES + ONES_BYTES +
                                             STG_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  {
    uint32_t* ones = reinterpret_cast<uint32_t*>(gbase + P_STAGES * P_STAGE_BYTES);
    for (int i = threadIdx.x; i < static_cast<int>(ONES_BYTES / 4); i += blockDim.x)
      ones[i] = i < 32 ? 0x3F803F80u : 0u;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(smem_u32(&sh->full[s]), 1);
      mbar_init(smem_u32(&sh->empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&sh->tfull[a]), 1);
      mbar_init(smem_u32(&sh->tempty[a]), 8);
    }
    mbar_init(smem_u32(&sh->done), 1);
    sh->abort = 0;
    fence_mbar_init();
    prefetch_tmap(&a_map);
    prefetch_tmap(&b_map);
  }
  cluster_sync_all();
  if (warp == 1) tmem_alloc_pair(smem_u32(&sh->tmem_base), TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  const int total = args.num_experts * args.m_tiles * (args.n_tiles + (args.bias_out ? 1 : 0));
  const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int tile = pair; tile < total; tile += num_pairs) {
        const Work w = work_of(args, tile);
        int kb0, nk;
        seg_blocks(args, w.e, kb0, nk);
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % P_STAGES;
          const uint32_t ph = (it / P_STAGES) & 1;
          if (!mbar_wait(smem_u32(&sh->empty[s]), ph ^ 1)) {
            p_set_abort(sh, args.status, kStatusTimeoutProducer);
            ok = false;
            break;
          }
          if (p_aborted(sh)) { ok = false; break; }
          const uint32_t fb = smem_u32(&sh->full[s]);
          if (leader) mbar_arrive_expect_tx(fb, w.bias ? 2 * P_A_BYTES : 2 * P_STAGE_BYTES);
          const uint32_t fb_leader = mapa_shared(fb, 0);
          const int row = (kb0 + kb) * BK;
#pragma unroll
          for (int j = 0; j < 2; ++j)
            tma_load_2d_pair(a_s + s * P_A_BYTES + j * CHUNK_BYTES, &a_map, fb_leader,
                             w.m * PAIR_M + static_cast<int>(rank) * kTileM + 64 * j, row);
          if (!w.bias) {
#pragma unroll
            for (int j = 0; j < 2; ++j)
              tma_load_2d_pair(b_s + s * P_B_BYTES + j * CHUNK_BYTES, &b_map, fb_leader,
                               w.n * BN + static_cast<int>(rank) * (BN / 2) + 64 * j, row);
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      int it = 0, local = 0;
      for (int tile = pair; tile < total; tile += num_pairs, ++local) {
        const Work w = work_of(args, tile);
        int kb0, nk;
        seg_blocks(args, w.e, kb0, nk);
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait_cluster(smem_u32(&sh->tempty[acc]), aph ^ 1)) {
          p_set_abort(sh, args.status, kStatusTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % P_STAGES;
          const uint32_t ph = (it / P_STAGES) & 1;
          if (!mbar_wait(smem_u32(&sh->full[s]), ph)) {
            p_set_abort(sh, args.status, kStatusTimeoutMma);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = a_s + s * P_A_BYTES, b_addr = b_s + s * P_B_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint32_t accum = (kb | k) != 0 ? 1u : 0u;
            const uint64_t a_desc = desc_mn_sw128(a_addr + k * 2048);
            if (w.bias)
              umma_bf16_pair(d_tmem, a_desc, umma_desc_sw128(ones_s + k * 32), P_IDESC_BIAS, accum);
            else
              umma_bf16_pair(d_tmem, a_desc, desc_mn_sw128(b_addr + k * 2048), P_IDESC, accum);
          }
          umma_commit_pair(smem_u32(&sh->empty[s]), 0x3);
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&sh->tfull[acc]), 0x3);
        if (p_aborted(sh)) break;
      }
      umma_commit_pair(smem_u32(&sh->done), 0x1);
      if (!mbar_wait(smem_u32(&sh->done), 0)) report(args.status, kStatusTimeoutDrain);
    }
  } else {
    const int q = warp & 3;
    int local = 0;
    for (int tile = pair; tile < total; tile += num_pairs, ++local) {
      const Work w = work_of(args, tile);
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      const bool got = mbar_wait(smem_u32(&sh->tfull[acc]), aph);
      __syncwarp();
      if (!__all_sync(0xffffffffu, got)) {
        if (lane == 0) p_set_abort(sh, args.status, kStatusTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      int kb0, nk;
      seg_blocks(args, w.e, kb0, nk);
      const int mrow = w.m * PAIR_M + static_cast<int>(rank) * kTileM + q * 32 + lane;
      int which = 0, i = mrow;
      if (args.mode == 1) {
        which = (mrow / 128) & 1;
        i = (mrow / 256) * 128 + (mrow & 127);
      }
      const bool row_ok = i < args.m_valid;
      const uint32_t t_row = tmem + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      if (w.bias) {
        float v[16];
        if (nk > 0) {
          tmem_ld16(t_row, v);
        } else {
          v[0] = 0.f;
        }
        if (row_ok)
          ((which && args.bias_out2) ? args.bias_out2 : args.bias_out)
              [static_cast<int64_t>(w.e) * args.m_valid + i] = v[0];
      } else {
        wg_store_tile(args, w.e, mrow - lane, w.n * BN, t_row, nk > 0, stg_all + q * 32 * STG_PITCH,
                      lane);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&sh->tempty[acc]), 0));
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && p_aborted(sh)) {
    // copies issued by this CTA land on the leader's barriers; give any still in flight a
    // bounded time to finish before the shared memory is released
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 200000ull) {
    }
  }
  cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
}

}  // namespace

cudaError_t launch_wgrad_pair(const CUtensorMap& a_map, const CUtensorMap& b_map,
                              const WgradArgs& args, int num_sms, cudaStream_t s) {
  if (args.mode == 1 && !args.out2) return cudaErrorInvalidValue;
  if (args.mode == 1 && args.bias_out && !args.bias_out2) return cudaErrorInvalidValue;
  cudaError_t err = cudaFuncSetAttribute(wgrad_pair_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(P_SMEM_BYTES));
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = P_SMEM_BYTES;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(num_sms & ~1), 1, 1);
  int max_clusters = 0;
  err = cudaOccupancyMaxActiveClusters(&max_clusters, reinterpret_cast<const void*>(&wgrad_pair_kernel),
                                       &cfg);
  if (err != cudaSuccess) return err;
  if (max_clusters < 1) return cudaErrorInvalidConfiguration;
  int64_t work = static_cast<int64_t>(args.num_experts) * args.m_tiles *
                 (args.n_tiles + (args.bias_out ? 1 : 0));
  if (work < 1) work = 1;
  int64_t pairs = work < max_clusters ? work : max_clusters;
  if (pairs > num_sms / 2) pairs = num_sms / 2;
  if (pairs < 1) pairs = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  err = cudaLaunchKernelEx(&cfg, wgrad_pair_kernel, a_map, b_map, args);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

cudaError_t launch_wgrad(const CUtensorMap& a_map, const CUtensorMap& b_map, const WgradArgs& args,
                         int num_sms, cudaStream_t s) {
  if (args.mode == 1 && !args.out2) return cudaErrorInvalidValue;
  if (args.mode == 1 && args.bias_out && !args.bias_out2) return cudaErrorInvalidValue;
  cudaError_t err = cudaFuncSetAttribute(wgrad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(SMEM_BYTES));
  if (err != cudaSuccess) return err;
  const int64_t work = static_cast<int64_t>(args.num_experts) * args.m_tiles *
                       (args.n_tiles + (args.bias_out ? 1 : 0));
  const int grid = static_cast<int>(work < num_sms ? (work > 0 ? work : 1) : num_sms);
  wgrad_kernel<<<grid, 192, SMEM_BYTES, s>>>(a_map, b_map, args);
  return cudaGetLastError();
}

}  // namespace vmoe
