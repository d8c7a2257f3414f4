// Decode-sized grouped expert GEMMs on the 5th-generation tensor cores, operands swapped.
//
// Reference math (python/vesper/model.py:295-298, per expert e over its n_e routed rows):
//   phase 1 (gate|up): h = ERA(x_e Wg_e^T + bg_e) * (x_e Wu_e^T + bu_e)     (ERA :69-76)
//   phase 2 (down)   : y = h_e Wd_e^T + bd_e
// In a decode batch an expert receives a handful of rows (64 tokens, top-2 over 8 experts:
// 16 rows each) while its weights are tens of megabytes, so the layer is bound by reading
// every active expert's weights once from HBM.  The row-tiled GEMMs would pad each expert's
// rows to a 256-row MMA tile.  Here the weights are the MMA's M operand (128 output features
// per tile, K-major exactly as packed) and the expert's rows are the N operand, N = its
// segment length (a multiple of 16, at most 256) written into the instruction descriptor
// per work item at run time:
//   D^T [128 features x N rows] = W_block [128 x K] . X_e^T
// so the tensor cores do only the useful products and the weight stream sets the pace.
//
// Work items are (active expert, 128-row weight block), spread over a persistent grid:
// first every phase-1 item, then every phase-2 item.  A phase-1 block is 64 gate rows plus
// the 64 up rows of the same features (two 64-row TMA boxes into one 128-row stage), so TMEM
// lanes 0..63 hold gate and 64..127 up for the same features; the up warps hand their values
// to the gate warps through shared memory.  Experts that received no rows are skipped: their
// weights are never read.
//
// Both phases in one launch: a phase-2 item of expert e needs all of e's h rows, so each
// phase-1 epilogue publishes its stored block on a per-expert counter (release) and the
// producer of a phase-2 item waits until the counter reaches the expert's block count
// (acquire, bounded) before its TMA reads h.  Phase-1 items never wait, and every CTA takes
// its items in ascending order, so the waits always end; the launch is cooperative (all CTAs
// resident, or the launch fails).  The down GEMM's weight stream then starts on the SMs that
// run out of gate|up work instead of after a second launch, filling the first phase's last
// partial wave.  The phases can also run as separate launches (a null counter array).
//
// Roles (192 threads, one CTA per SM):
//   warp 0      TMA producer: per k-block one 16 KB weight tile and N/16 row tiles of the
//               expert's activations (16-row boxes) into a ring of 128B-swizzled stages;
//   warp 1      TMEM allocator (two accumulators of 256 columns) and MMA issuer
//               (tcgen05.mma M = 128, N = rows, K = 16, four per k-block);
//   warps 2..5  epilogue: tcgen05.ld of 16 columns (rows) at a time, bias, ERA * up (phase
//               1) and bf16 stores into the row-major output; the accumulator is released
//               as soon as it has been read, so the next item's main loop overlaps.
// Every wait is bounded (kWaitLimitNs) and reports a status code; after an abort the kernel
// drains its own copies and MMAs (bounded) and frees TMEM.  No TMA multicast is used.
#include <stdio.h>

#include "common.cuh"
#include "kernels.h"

namespace vmoe {
namespace {

constexpr int BK = 64;
constexpr uint32_t A_BYTES = 128 * BK * 2;     // 16 KB: 128 weight rows x 64 K
constexpr uint32_t B_ROW_BYTES = BK * 2;       // 128 B: one activation row x 64 K
constexpr uint32_t B_BOX_ROWS = 16;            // rows per activation TMA box
constexpr int kMaxStages = 12;
constexpr uint32_t kAccCols = 256;             // one accumulator: up to 256 rows (N)
constexpr uint32_t kTmemCols = 2 * kAccCols;
constexpr size_t kSmemDyn = 232448;            // the whole opt-in shared memory of a CTA

struct DecShared {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t done;
  uint32_t tmem_base;
  int abort;
  int issued;
  int consumed;
  int n_act;
  int stages;                      // ring depth for the largest segment of this forward
  uint32_t b_slot;                 // bytes of one stage's row tile (largest segment x 128)
  int ep_ok[2][4];                 // epilogue: each warp's wait result, per item parity
  int act_e[kDecodeMaxExperts];    // experts with rows, ascending id
  int act_seg[kDecodeMaxExperts];  // first row of the expert's segment
  int act_n[kDecodeMaxExperts];    // its rows, a multiple of 16 in [16, 256]
  float xch[2][64][17];            // up values handed to the gate warps (17: no bank conflicts)
};

// shared state first (fixed place), then the ring of stages, 1024-byte aligned
constexpr uint32_t kSharedBytes = (sizeof(DecShared) + 1023) & ~1023u;
constexpr uint32_t kRingBytes = static_cast<uint32_t>(kSmemDyn) - 1024 - kSharedBytes;

__device__ __forceinline__ bool aborted(const DecShared* sh) {
  return *reinterpret_cast<const volatile int*>(&sh->abort) != 0;
}
__device__ __forceinline__ void set_abort(DecShared* sh, int* status, int code) {
  *reinterpret_cast<volatile int*>(&sh->abort) = 1;
  report(status, code);
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ void store_bf16(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// generic-proxy global memory accesses ordered with async-proxy (TMA) ones
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Item -> (phase, active-expert index, block): n1 phase-1 items of bpe1 blocks per expert,
// then phase-2 items of bpe2 blocks per expert.
struct Item {
  bool gated;
  int a, blk;
};
__device__ __forceinline__ Item item_of(int item, int n1, int bpe1, int bpe2) {
  Item it;
  it.gated = item < n1;
  const int j = it.gated ? item : item - n1;
  const int bpe = it.gated ? bpe1 : bpe2;
  it.a = j / bpe;
  it.blk = j - it.a * bpe;
  return it;
}

__global__ void __launch_bounds__(192, 1)
decode_gemm_kernel(const __grid_constant__ CUtensorMap a1_map,
                   const __grid_constant__ CUtensorMap b1_map,
                   const __grid_constant__ CUtensorMap a2_map,
                   const __grid_constant__ CUtensorMap b2_map, const DecodeGemmArgs args) {
  pdl_wait_and_trigger();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  DecShared* sh = reinterpret_cast<DecShared*>(smem_raw + (base - raw));
  const uint32_t ring = base + kSharedBytes;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    sh->abort = 0;
    sh->issued = 0;
    sh->consumed = 0;
    // the experts that received rows, in ascending id, with their segments
    int n = 0, widest = kDecodeRowAlign;
    const int E = args.num_experts < kDecodeMaxExperts ? args.num_experts : kDecodeMaxExperts;
    for (int e = 0; e < E; ++e) {
      const int seg = args.offs[e], len = args.offs[e + 1] - seg;
      if (len <= 0) continue;
      int rows = len;
      if (rows > args.n_max || (rows & 15) || seg < 0 ||
          static_cast<int64_t>(seg) + rows > args.max_rows) {
        report(args.status, kStatusBadTileCount);  // never read or write past the buffers
        continue;
      }
      sh->act_e[n] = e;
      sh->act_seg[n] = seg;
      sh->act_n[n] = rows;
      widest = rows > widest ? rows : widest;
      ++n;
    }
    sh->n_act = n;
    // as many stages as the ring holds for this forward's widest segment (not the widest
    // possible one): more weight tiles in flight per SM
    sh->b_slot = static_cast<uint32_t>(widest) * B_ROW_BYTES;
    int st = static_cast<int>(kRingBytes / (A_BYTES + sh->b_slot));
    sh->stages = st > kMaxStages ? kMaxStages : st;
    for (int s = 0; s < sh->stages; ++s) {
      mbar_init(smem_u32(&sh->full[s]), 1);
      mbar_init(smem_u32(&sh->empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&sh->tfull[a]), 1);
      mbar_init(smem_u32(&sh->tempty[a]), 4);
    }
    mbar_init(smem_u32(&sh->done), 1);
    fence_mbar_init();
    if (args.bpe1 > 0) { prefetch_tmap(&a1_map); prefetch_tmap(&b1_map); }
    if (args.bpe2 > 0) { prefetch_tmap(&a2_map); prefetch_tmap(&b2_map); }
  }
  if (warp == 1) tmem_alloc(smem_u32(&sh->tmem_base), kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  const int bpe1 = args.bpe1, bpe2 = args.bpe2;
  const int n1 = sh->n_act * bpe1;
  const int total = n1 + sh->n_act * bpe2;
  const int stages = sh->stages;
  const uint32_t b_slot = sh->b_slot;
  const uint32_t a_s = ring;
  const uint32_t b_s = ring + static_cast<uint32_t>(stages) * A_BYTES;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total && ok; item += gridDim.x) {
        const Item w = item_of(item, n1, bpe1, bpe2);
        const int e = sh->act_e[w.a], seg = sh->act_seg[w.a], rows = sh->act_n[w.a];
        if (!w.gated && args.ready) {
          // the down GEMM of expert e reads every row of e's h: wait until all of e's
          // gate|up blocks are stored (their epilogues count them), then order the TMA
          // reads after those stores
          const int* cnt = args.ready + e;
          if (ld_acquire_gpu(cnt) < bpe1) {
            const uint64_t t0 = globaltimer_ns();
            uint32_t spins = 0;
            while (ld_acquire_gpu(cnt) < bpe1) {
              if ((++spins & 63u) == 0 && (aborted(sh) || globaltimer_ns() - t0 > kWaitLimitNs)) {
                set_abort(sh, args.status, kStatusTimeoutProducer);
                ok = false;
                break;
              }
            }
            if (!ok) break;
          }
          fence_proxy_async_global();
        }
        // phase 1: gate rows [256 j + 64 hh, +64) and the up rows 128 further of block blk;
        // phase 2: down rows [128 blk, +128)
        const CUtensorMap* am = w.gated ? &a1_map : &a2_map;
        const CUtensorMap* bm = w.gated ? &b1_map : &b2_map;
        const int a_row = w.gated ? e * args.a_rows1 + 256 * (w.blk >> 1) + 64 * (w.blk & 1)
                                  : e * args.a_rows2 + 128 * w.blk;
        const int k_blocks = w.gated ? args.k_blocks1 : args.k_blocks2;
        const uint32_t tx = A_BYTES + static_cast<uint32_t>(rows) * B_ROW_BYTES;
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const int s = it % stages;
          const uint32_t ph = (it / stages) & 1;
          if (!mbar_wait(smem_u32(&sh->empty[s]), ph ^ 1)) {
            set_abort(sh, args.status, kStatusTimeoutProducer);
            ok = false;
            break;
          }
          if (aborted(sh)) { ok = false; break; }
          const uint32_t fb = smem_u32(&sh->full[s]);
          mbar_arrive_expect_tx(fb, tx);
          const uint32_t a_dst = a_s + s * A_BYTES;
          if (w.gated) {
            tma_load_2d(a_dst, am, fb, kb * BK, a_row);
            tma_load_2d(a_dst + A_BYTES / 2, am, fb, kb * BK, a_row + 128);
          } else {
            tma_load_2d(a_dst, am, fb, kb * BK, a_row);
          }
          const uint32_t b_dst = b_s + s * b_slot;
          for (int r = 0; r < rows; r += B_BOX_ROWS)
            tma_load_2d(b_dst + r * B_ROW_BYTES, bm, fb, kb * BK, seg + r);
          *reinterpret_cast<volatile int*>(&sh->issued) = it + 1;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int it = 0, local = 0;
      for (int item = blockIdx.x; item < total; item += gridDim.x, ++local) {
        const Item w = item_of(item, n1, bpe1, bpe2);
        const uint32_t idesc = umma_idesc_bf16(128, sh->act_n[w.a]);
        const int k_blocks = w.gated ? args.k_blocks1 : args.k_blocks2;
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(smem_u32(&sh->tempty[acc]), aph ^ 1)) {
          set_abort(sh, args.status, kStatusTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * kAccCols;
        bool ok = true;
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const int s = it % stages;
          const uint32_t ph = (it / stages) & 1;
          if (!mbar_wait(smem_u32(&sh->full[s]), ph)) {
            set_abort(sh, args.status, kStatusTimeoutMma);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = a_s + s * A_BYTES, b_addr = b_s + s * b_slot;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16(d_tmem, umma_desc_sw128(a_addr + k * 32), umma_desc_sw128(b_addr + k * 32),
                      idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(smem_u32(&sh->empty[s]));
          *reinterpret_cast<volatile int*>(&sh->consumed) = it + 1;
        }
        if (!ok) break;
        umma_commit(smem_u32(&sh->tfull[acc]));
        if (aborted(sh)) break;
      }
      umma_commit(smem_u32(&sh->done));
      if (!mbar_wait(smem_u32(&sh->done), 0)) report(args.status, kStatusTimeoutDrain);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;  // TMEM lane quarter: rows (features) 32q .. 32q + 31
    __nv_bfloat16* hout = static_cast<__nv_bfloat16*>(args.h);
    __nv_bfloat16* yout = static_cast<__nv_bfloat16*>(args.y);
    int chunk = 0;           // 16-row chunks handed over so far (alternates the xch buffers)
    int local = 0;
    for (int item = blockIdx.x; item < total; item += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      const bool got = mbar_wait(smem_u32(&sh->tfull[acc]), aph);
      __syncwarp();
      const bool warp_ok = __all_sync(0xffffffffu, got);
      // the four warps meet at named barriers (the gate|up hand-over, the completion count),
      // so they must agree on going on: each publishes its own (bounded) wait's result and
      // all read the four after the barrier (the flags of item i + 1 are written only after
      // every warp passed item i's later barriers, so a double buffer suffices)
      if (lane == 0) sh->ep_ok[local & 1][q] = warp_ok ? 1 : 0;
      epi_bar();
      const int* okf = sh->ep_ok[local & 1];
      if (!(okf[0] && okf[1] && okf[2] && okf[3])) {
        if (lane == 0 && !warp_ok) set_abort(sh, args.status, kStatusTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      const Item w = item_of(item, n1, bpe1, bpe2);
      const int e = sh->act_e[w.a], seg = sh->act_seg[w.a], rows = sh->act_n[w.a];
      const uint32_t t_row = tmem + (static_cast<uint32_t>(q * 32) << 16) + acc * kAccCols;
      const bool limit = args.row_limit > 0;
      if (w.gated) {
        // feature f of this lane (gate warps q = 0, 1; the up warps q = 2, 3 hold the same
        // features' up values); packed bias: gate at 256 j + c, up at 256 j + 128 + c
        const int fl = 32 * (q & 1) + lane;                  // 0..63 within the block
        const int f = 64 * w.blk + fl;                       // feature (column of h)
        const int64_t bcol = static_cast<int64_t>(e) * args.bias1_ld + 256 * (w.blk >> 1) +
                             64 * (w.blk & 1) + fl;
        const float bg = args.bias1[bcol], bu = args.bias1[bcol + 128];
        for (int c = 0; c < rows; c += 16, ++chunk) {
          float (*x)[17] = sh->xch[chunk & 1];
          float v[16];
          tmem_ld16(t_row + c, v);
          if (q >= 2) {
#pragma unroll
            for (int j = 0; j < 16; ++j) x[fl][j] = v[j] + bu;
          }
          epi_bar();
          if (q < 2) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int64_t r = static_cast<int64_t>(seg) + c + j;
              if (!limit || r < args.row_limit)
                store_bf16(hout + r * args.ldh + f, era_fast(v[j] + bg, args.gamma) * x[fl][j]);
            }
          }
        }
        if (args.ready) {
          // publish this block of e's h rows to the down GEMM's producers: every storing
          // thread orders its stores (also for the TMA's async proxy), the four warps meet,
          // then one release-add counts the block
          fence_proxy_async_global();
          __threadfence();
          epi_bar();
          if (q == 2 && lane == 0) red_release_gpu_add(args.ready + e, 1);
        }
      } else {
        const int f = 128 * w.blk + 32 * q + lane;  // output feature (column of y)
        const float bias = args.bias2 ? args.bias2[static_cast<int64_t>(e) * args.bias2_ld + f] : 0.f;
        for (int c = 0; c < rows; c += 16) {
          float v[16];
          tmem_ld16(t_row + c, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int64_t r = static_cast<int64_t>(seg) + c + j;
            if (!limit || r < args.row_limit) store_bf16(yout + r * args.ldy + f, v[j] + bias);
          }
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
      if (!mbar_wait(smem_u32(&sh->full[i % stages]), (i / stages) & 1)) {
        report(args.status, kStatusTimeoutDrain);
        break;
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

int decode_gemm_stages(int n_max) {
  const int s = static_cast<int>(kRingBytes / (A_BYTES + static_cast<uint32_t>(n_max) * B_ROW_BYTES));
  return s > kMaxStages ? kMaxStages : s;
}

cudaError_t launch_decode_gemm(const CUtensorMap& a1_map, const CUtensorMap& b1_map,
                               const CUtensorMap& a2_map, const CUtensorMap& b2_map,
                               const DecodeGemmArgs& args, int64_t max_items, int num_sms,
                               cudaStream_t s) {
  const bool fused = args.bpe1 > 0 && args.bpe2 > 0;
  if (args.n_max < 16 || args.n_max > static_cast<int>(kAccCols) || (args.n_max & 15) ||
      args.num_experts < 1 || args.num_experts > kDecodeMaxExperts || args.bpe1 < 0 ||
      args.bpe2 < 0 || (args.bpe1 == 0 && args.bpe2 == 0) || !args.offs ||
      (args.bpe1 > 0 && (!args.h || !args.bias1 || args.k_blocks1 < 1)) ||
      (args.bpe2 > 0 && (!args.y || args.k_blocks2 < 1)) || (fused && !args.ready))
    return cudaErrorInvalidValue;
  if (decode_gemm_stages(args.n_max) < 2) return cudaErrorInvalidValue;
  static_assert(kRingBytes / (A_BYTES + kAccCols * B_ROW_BYTES) >= 2, "two stages of the widest");
  constexpr size_t smem = kSmemDyn;
  cudaError_t err = cudaFuncSetAttribute(decode_gemm_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  int64_t grid = max_items < num_sms ? max_items : num_sms;
  if (grid < 1) grid = 1;
  if (!fused)  // programmatic dependent launch when the caller's scope asks for it
    return launch_kernel(decode_gemm_kernel, dim3(static_cast<unsigned>(grid)), dim3(192), smem,
                         s, a1_map, b1_map, a2_map, b2_map, args);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // a phase-2 item waits for other CTAs' work
  attr[0].val.cooperative = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_gemm_kernel, a1_map, b1_map, a2_map, b2_map, args);
}

}  // namespace vmoe
