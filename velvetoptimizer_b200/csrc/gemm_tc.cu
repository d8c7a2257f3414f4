// bf16 grouped expert GEMMs on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Reference math (python/vesper/model.py):
//   gated (gemm1): h = ERA(x_e Wg_e^T + bg_e) * (x_e Wu_e^T + bu_e)   :295-297, ERA :69-76
//   plain (gemm2): y = h Wd_e^T + bd_e                                :298
//
// Design (one CTA per SM, persistent over (M tile, N tile) work items):
//   warp 0      TMA producer: A tile [128 x 64] and B tile [256 x 64] per k-block into a
//               4-stage ring of 128B-swizzled shared-memory buffers;
//   warp 1      allocates 512 TMEM columns (two 128 x 256 fp32 accumulators) and one
//               thread issues tcgen05.mma (M=128, N=256, K=16) four times per k-block;
//   warps 2..5  epilogue: tcgen05.ld of their 32 TMEM lanes, bias + ERA(gate) * up (or
//               bias only), bf16 convert, store; the accumulator is double-buffered so
//               the epilogue of tile i overlaps the main loop of tile i+1.
// The gate/up weights are packed so that one 256-row B tile holds 128 gate rows followed
// by the 128 up rows of the same output columns: one MMA chain produces both operands
// of the gated product, and the activation never leaves the SM before it is multiplied.
//
// Every mbarrier wait is bounded (kWaitLimitNs); on a timeout the kernel records a code
// in the status word, stops issuing work, waits (bounded) for its own copies and MMAs in
// flight, frees TMEM and returns.  No TMA multicast is used.
#include <cudaTypedefs.h>
#include <stdio.h>

#include "common.cuh"
#include "kernels.h"

namespace vmoe {
namespace {

constexpr int BN = 256, BK = 64, STAGES = 4;
constexpr uint32_t A_BYTES = kTileM * BK * 2;  // 16 KB
constexpr uint32_t B_BYTES = BN * BK * 2;      // 32 KB
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t TMEM_COLS = 2 * BN;         // 512: two accumulators
constexpr uint32_t IDESC = umma_idesc_bf16(kTileM, BN);

struct TcShared {
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

constexpr size_t SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + sizeof(TcShared) + 64;

__device__ __forceinline__ bool aborted(const TcShared* sh) {
  return *reinterpret_cast<const volatile int*>(&sh->abort) != 0;
}
__device__ __forceinline__ void set_abort(TcShared* sh, int* status, int code) {
  *reinterpret_cast<volatile int*>(&sh->abort) = 1;
  report(status, code);
}

// Expert of M tile m, clamped into range (a bad map only produces a status code).
__device__ __forceinline__ int expert_of(const TcGemmArgs& args, int m) {
  const int e = args.tile_expert[m];
  if (static_cast<unsigned>(e) < static_cast<unsigned>(args.num_experts)) return e;
  report(args.status, kStatusBadExpert);
  return 0;
}

template <bool GATED>
__global__ void __launch_bounds__(192, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap b_map,
               const TcGemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t a_s = base;
  const uint32_t b_s = base + STAGES * A_BYTES;
  TcShared* sh = reinterpret_cast<TcShared*>(gbase + STAGES * STAGE_BYTES);

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

  const int n_tiles = args.n_tiles, k_blocks = args.k_blocks;
  int num_m = *args.num_m_tiles;
  if (num_m > args.max_m_tiles || num_m < 0) {  // never write past the output buffer
    if (threadIdx.x == 0) report(args.status, kStatusBadTileCount);
    num_m = num_m < 0 ? 0 : args.max_m_tiles;
  }
  const int total = num_m * n_tiles;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int it = 0;
      for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
        const int m = tile / n_tiles, n = tile - m * n_tiles;
        const int e = expert_of(args, m);
        const int a_row = m * kTileM;
        const int b_row = e * args.b_rows_per_expert + n * BN;
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
          mbar_arrive_expect_tx(fb, STAGE_BYTES);
          tma_load_2d(a_s + s * A_BYTES, &a_map, fb, kb * BK, a_row);
          tma_load_2d(b_s + s * B_BYTES, &b_map, fb, kb * BK, b_row);
          *reinterpret_cast<volatile int*>(&sh->issued) = it + 1;
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int it = 0, local = 0;
      for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(smem_u32(&sh->tempty[acc]), aph ^ 1)) {
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
            umma_bf16(d_tmem, umma_desc_sw128(a_addr + k * 32), umma_desc_sw128(b_addr + k * 32),
                      IDESC, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(smem_u32(&sh->empty[s]));
          *reinterpret_cast<volatile int*>(&sh->consumed) = it + 1;
        }
        if (!ok) break;
        umma_commit(smem_u32(&sh->tfull[acc]));
        if (aborted(sh)) break;
      }
      // every MMA this thread issued has completed once `done` flips
      umma_commit(smem_u32(&sh->done));
      if (!mbar_wait(smem_u32(&sh->done), 0)) report(args.status, kStatusTimeoutDrain);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int local = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      const bool got = mbar_wait(smem_u32(&sh->tfull[acc]), aph);
      __syncwarp();
      if (!__all_sync(0xffffffffu, got)) {
        if (lane == 0) set_abort(sh, args.status, kStatusTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      const int m = tile / n_tiles, n = tile - m * n_tiles;
      const int e = expert_of(args, m);
      const int64_t row = static_cast<int64_t>(m) * kTileM + q * 32 + lane;
      const uint32_t t_row = tmem + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      __nv_bfloat16* outp = static_cast<__nv_bfloat16*>(args.out) + row * args.ldo;
      const float* bias = args.bias + static_cast<int64_t>(e) * args.bias_ld + n * BN;
      if constexpr (GATED) {
        outp += n * (BN / 2);
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
          float g[32], u[32];
          tmem_ld32(t_row + c, g);
          tmem_ld32(t_row + BN / 2 + c, u);
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float h0 = era_fast(g[j] + bias[c + j], args.gamma) * (u[j] + bias[BN / 2 + c + j]);
            const float h1 =
                era_fast(g[j + 1] + bias[c + j + 1], args.gamma) * (u[j + 1] + bias[BN / 2 + c + j + 1]);
            packed[j / 2] = pack_bf16x2(h0, h1);
          }
          uint4* dst = reinterpret_cast<uint4*>(outp + c);
#pragma unroll
          for (int v = 0; v < 4; ++v)
            dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
        }
      } else {
        outp += n * BN;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v32[32];
          tmem_ld32(t_row + c, v32);
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2)
            packed[j / 2] = pack_bf16x2(v32[j] + bias[c + j], v32[j + 1] + bias[c + j + 1]);
          uint4* dst = reinterpret_cast<uint4*>(outp + c);
#pragma unroll
          for (int v = 0; v < 4; ++v)
            dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&sh->tempty[acc]));
    }
  }

  __syncthreads();
  // after an abort: wait (bounded) for TMA loads that were issued but never consumed
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

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

}  // namespace

bool make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                    uint32_t box_rows, char* err, size_t err_len) {
  auto encode = get_encode_fn();
  if (!encode) {
    snprintf(err, err_len, "cuTensorMapEncodeTiled is unavailable from the driver");
    return false;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (ld * 2) % 16 || rows == 0 || cols == 0) {
    snprintf(err, err_len, "tensor map: base %p / row pitch %llu elements not 16-byte aligned",
             base, static_cast<unsigned long long>(ld));
    return false;
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    snprintf(err, err_len, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
    return false;
  }
  return true;
}

cudaError_t launch_tc_gemm(bool gated, const CUtensorMap& a_map, const CUtensorMap& b_map,
                           const TcGemmArgs& args, int64_t max_tiles, int num_sms,
                           cudaStream_t s) {
  const int64_t work = max_tiles * args.n_tiles;
  const int grid = static_cast<int>(work < num_sms ? (work > 0 ? work : 1) : num_sms);
  cudaError_t err;
  if (gated) {
    err = cudaFuncSetAttribute(tc_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(SMEM_BYTES));
    if (err != cudaSuccess) return err;
    tc_gemm_kernel<true><<<grid, 192, SMEM_BYTES, s>>>(a_map, b_map, args);
  } else {
    err = cudaFuncSetAttribute(tc_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(SMEM_BYTES));
    if (err != cudaSuccess) return err;
    tc_gemm_kernel<false><<<grid, 192, SMEM_BYTES, s>>>(a_map, b_map, args);
  }
  return cudaGetLastError();
}

}  // namespace vmoe
