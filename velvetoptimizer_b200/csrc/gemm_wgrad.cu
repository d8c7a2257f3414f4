// Grouped weight-gradient GEMM on the tensor cores (tcgen05 + TMEM + TMA), fp32 out.
//
// For every expert e:  dW_e[M, N] = sum over the rows r of e's segment of  A[r, :]^T B[r, :]
// -- the nn.Linear weight gradient dW = dY^T X that autograd forms for every expert's
// Linear in MoELayer.forward (python/vesper/model.py:295-298, 322) -- with the token rows as
// the reduction (K) dimension.  Both operands are stored transposed (A^T [M_total, R],
// B^T [N_total, R], rows contiguous along R) so every operand tile is K-major like the
// forward GEMMs'; the K range of a tile is its expert's segment [offs[e], offs[e+1]) (a
// multiple of 64 rows), so experts with more tokens simply run longer K loops and empty
// experts write zeros.
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
constexpr uint32_t A_BYTES = kTileM * BK * 2;  // 16 KB
constexpr uint32_t B_BYTES = BN * BK * 2;      // 32 KB
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int STAGES = 4;
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr uint32_t IDESC = umma_idesc_bf16(kTileM, BN);

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

constexpr size_t SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + sizeof(WgShared) + 64;

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

__global__ void __launch_bounds__(192, 1)
wgrad_kernel(const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap b_map,
             const WgradArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t a_s = base;
  const uint32_t b_s = base + STAGES * A_BYTES;
  auto* sh = reinterpret_cast<WgShared*>(gbase + STAGES * STAGE_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

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
  const int per_expert = args.m_tiles * args.n_tiles;
  const int total = args.num_experts * per_expert;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
        const int e = tile / per_expert, mn = tile - e * per_expert;
        const int m = mn / args.n_tiles, n = mn - m * args.n_tiles;
        int kb0, nk;
        seg_blocks(args, e, kb0, nk);
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
          mbar_arrive_expect_tx(fb, STAGE_BYTES);
          tma_load_2d(a_s + s * A_BYTES, &a_map, fb, (kb0 + kb) * BK, m * kTileM);
          tma_load_2d(b_s + s * B_BYTES, &b_map, fb, (kb0 + kb) * BK, n * BN);
          *reinterpret_cast<volatile int*>(&sh->issued) = it + 1;
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, local = 0;
      for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++local) {
        const int e = tile / per_expert;
        int kb0, nk;
        seg_blocks(args, e, kb0, nk);
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
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16(d_tmem, umma_desc_sw128(a_addr + k * 32), umma_desc_sw128(b_addr + k * 32),
                      IDESC, (kb | k) != 0 ? 1u : 0u);
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
      const int e = tile / per_expert, mn = tile - e * per_expert;
      const int m = mn / args.n_tiles, n = mn - m * args.n_tiles;
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
      seg_blocks(args, e, kb0, nk);
      const int mrow = m * kTileM + q * 32 + lane;  // row of this expert's M dimension
      // destination row: plain, or the gate|up de-interleave of the packed 2*Ipad rows
      float* dst = nullptr;
      if (args.mode == 0) {
        if (mrow < args.m_valid)
          dst = args.out + static_cast<int64_t>(e) * args.out_expert_stride +
                static_cast<int64_t>(mrow) * args.ld_out;
      } else {
        const int which = (mrow / 128) & 1, i = (mrow / 256) * 128 + (mrow & 127);
        if (i < args.m_valid)
          dst = (which ? args.out2 : args.out) + static_cast<int64_t>(e) * args.out_expert_stride +
                static_cast<int64_t>(i) * args.ld_out;
      }
      const uint32_t t_row = tmem + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        float v[32];
        if (nk > 0) {
          tmem_ld32(t_row + c, v);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0.f;
        }
        const int col = n * BN + c;
        if (dst) {
          if (col + 32 <= args.n_valid && args.vec_ok) {
            float4* d4 = reinterpret_cast<float4*>(dst + col);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col + j < args.n_valid) dst[col + j] = v[j];
          }
        }
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

}  // namespace

cudaError_t launch_wgrad(const CUtensorMap& a_map, const CUtensorMap& b_map, const WgradArgs& args,
                         int num_sms, cudaStream_t s) {
  if (args.mode == 1 && !args.out2) return cudaErrorInvalidValue;
  cudaError_t err = cudaFuncSetAttribute(wgrad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(SMEM_BYTES));
  if (err != cudaSuccess) return err;
  const int64_t work = static_cast<int64_t>(args.num_experts) * args.m_tiles * args.n_tiles;
  const int grid = static_cast<int>(work < num_sms ? (work > 0 ? work : 1) : num_sms);
  wgrad_kernel<<<grid, 192, SMEM_BYTES, s>>>(a_map, b_map, args);
  return cudaGetLastError();
}

}  // namespace vmoe
