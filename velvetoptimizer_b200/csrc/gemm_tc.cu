// bf16 GEMMs on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), three epilogues.
//
// Reference math (python/vesper/model.py):
//   kGated  (expert gemm1): h = ERA(x_e Wg_e^T + bg_e) * (x_e Wu_e^T + bu_e)  :295-297, ERA :69-76
//   kPlain  (expert gemm2): y = h Wd_e^T + bd_e                               :298
//   kRouter (router)      : logits = x W_r^T + b_r, softmax, top-K, renormalise :322-329, plus
//                           the per-128-token expert histogram and probability sums the
//                           dispatch and the load-balancing loss (:366-385) consume
//   kRouterLN             : the same router on LayerNorm(x) (the ffn_norm of :418) without
//                           materialising the normalised rows: the B operand holds
//                           W' = W_r * ln_w, and two more MMAs per k-step on the x tile that
//                           is already in shared memory give every token's sum (x against a
//                           ones row) and sum of squares (the diagonal of x x^T); the epilogue
//                           forms mean / rstd and logits = rstd (x W'^T - mean c) + b' with
//                           c = row sums of W' and b' = b_r + W_r ln_b (folded at load time)
//
// Design (one CTA per SM, persistent over (M tile, N tile) work items):
//   warp 0      TMA producer: A tile [128 x 64] and B tile [BN x 64] per k-block into a
//               ring of 128B-swizzled shared-memory stages (4 stages at BN = 256, 8 at <= 64);
//   warp 1      allocates TMEM (two 128 x BN fp32 accumulators) and one thread issues
//               tcgen05.mma (M = 128, N = BN, K = 16) four times per k-block;
//   warps 2..5  epilogue: tcgen05.ld of their 32 TMEM lanes (one row per thread); the
//               accumulator is double-buffered so the epilogue of tile i overlaps the main
//               loop of tile i + 1.
// The gate/up weights are packed so that one 256-row B tile holds 128 gate rows followed by
// the 128 up rows of the same output columns: one MMA chain produces both operands of the
// gated product, and the activation never leaves the SM before it is multiplied.  The router
// keeps each token's E logits in registers: softmax, top-K and the weights never touch HBM.
//
// Every mbarrier wait is bounded (kWaitLimitNs); on a timeout the kernel records a code in
// the status word, stops issuing work, waits (bounded) for its own copies and MMAs in flight,
// frees TMEM and returns.  No TMA multicast is used.
#include <cudaTypedefs.h>
#include <stdio.h>

#include "common.cuh"
#include "kernels.h"

namespace vmoe {
namespace {

enum Epi { kPlain = 0, kGated = 1, kRouter = 2, kRouterLN = 3 };

// kRouterLN accumulator columns: [0, BN) logits, kSumCol.. the x-sum block (N 16),
// kSqCol.. x x^T (N 128); one accumulator spans kLnAccCols columns.
constexpr int kSumCol = 64, kSqCol = 128, kLnAccCols = 256;
constexpr uint32_t kOnesBytes = 16 * 128;  // 16-row K-major ones tile (row 0 = 1, rest 0)

constexpr int BK = 64;

// AR = rows of A a stage holds: 128 (a full M tile), or 32 for the router of a decode batch
// routed in blocks of at most 32 tokens.  Such a stage is 4 KB of A, so the ring is deep
// enough (32 stages) to have every k-block of a token block in flight at once; the MMA is
// still M = 128 and reads past the slot into other stages' shared memory for rows 32..127,
// whose accumulator rows the epilogue never uses.
template <int BN, int AR = 128>
struct TcCfg {
  static constexpr uint32_t A_BYTES = AR * BK * 2;
  static constexpr uint32_t B_BYTES = BN * BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES_FIT = static_cast<int>((200u * 1024u) / STAGE_BYTES);
  static constexpr int STAGES_MAX = AR == 128 ? 8 : 32;
  static constexpr int STAGES = STAGES_FIT > STAGES_MAX ? STAGES_MAX : STAGES_FIT;
  static constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;  // power of two for BN in {16..256}
  static constexpr uint32_t IDESC = umma_idesc_bf16(kTileM, BN);
  // an M = 128 MMA on the last stage's A slot reads 16 KB from its start
  static_assert(AR == 128 || (STAGES - 1) * A_BYTES + 16384 <= STAGES * STAGE_BYTES,
                "the MMA's reads past a short A slot stay inside the ring");
};

template <int STAGES>
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
  // router epilogue scratch (E <= 64), one set per epilogue group
  int ep_ok[2][4];
  int hist[2][64];
  float psum[2][4][64];
  float bias[64];  // router bias (and the LayerNorm router's folded-weight row sums), staged
  float ln_c[64];  // once per CTA so that the epilogue makes no global loads
};

template <int BN, int EPI = kPlain, int AR = 128>
constexpr size_t tc_smem_bytes() {
  return 1024 + TcCfg<BN, AR>::STAGES * TcCfg<BN, AR>::STAGE_BYTES +
         (EPI == kRouterLN ? kOnesBytes : 0) + sizeof(TcShared<TcCfg<BN, AR>::STAGES>) + 64;
}

template <int STAGES>
__device__ __forceinline__ bool aborted(const TcShared<STAGES>* sh) {
  return *reinterpret_cast<const volatile int*>(&sh->abort) != 0;
}
template <int STAGES>
__device__ __forceinline__ void set_abort(TcShared<STAGES>* sh, int* status, int code) {
  *reinterpret_cast<volatile int*>(&sh->abort) = 1;
  report(status, code);
}

// Expert of M tile m, clamped into range (a bad map only produces a status code).
__device__ __forceinline__ int expert_of(const TcGemmArgs& args, int m) {
  if (!args.tile_expert) return 0;
  const int e = args.tile_expert[m];
  if (static_cast<unsigned>(e) < static_cast<unsigned>(args.num_experts)) return e;
  report(args.status, kStatusBadExpert);
  return 0;
}

// The router runs two epilogue groups of four warps (one per TMEM accumulator, so they take
// alternate tiles and one group's routing math overlaps the other's); the GEMM epilogues run
// one.  Group g synchronises on named barrier 1 + g.
template <int EPI>
constexpr int tc_epi_groups() { return EPI == kRouter || EPI == kRouterLN ? 2 : 1; }
template <int EPI>
constexpr int tc_threads() { return 64 + 128 * tc_epi_groups<EPI>(); }

__device__ __forceinline__ void epilogue_bar(int grp) {  // the 4 warps of one epilogue group
  asm volatile("bar.sync %0, 128;" ::"r"(1 + grp) : "memory");
}

// Column sums over the warp's 32 lanes of v[0..31] (a reduce-scatter: lane l returns column
// l).  Each level adds the same pairs, in the same order, as the xor butterfly
// v += shfl_xor(v, o) for o = 16..1, so the sums are bit-identical to that butterfly's, with
// 31 shuffles instead of 160.
__device__ __forceinline__ float warp_column_sums(float (&v)[32], int lane) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = up ? v[i] : v[i + o];
      const float keep = up ? v[i + o] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0];
}

// Router epilogue for one 128-token tile by epilogue group `grp`: each thread owns one
// token's logits.  The accumulator is released (tempty_bar) as soon as it has been read.
template <int BN, int STAGES, bool LN>
__device__ __forceinline__ void router_epilogue(const TcGemmArgs& args, TcShared<STAGES>* sh,
                                                uint32_t t_row, uint32_t tempty_bar, int grp,
                                                int m, int q, int lane) {
  float lg[BN];
#pragma unroll
  for (int c = 0; c < BN; c += 16) tmem_ld16(t_row + c, lg + c);
  float sum_x = 0.f, ss = 0.f;
  if constexpr (LN) {
    // this token's sum (column kSumCol) and sum of squares (its own diagonal entry of x x^T)
    float sx[16], sq[32];
    tmem_ld16(t_row + kSumCol, sx);
    tmem_ld32(t_row + kSqCol + q * 32, sq);
#pragma unroll
    for (int j = 0; j < 32; ++j) ss = j == lane ? sq[j] : ss;
    sum_x = sx[0];
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(tempty_bar);
  const int E = args.num_experts, K = args.top_k;
  // routing block m holds tokens [m * rr, (m + 1) * rr); rows of the tile past rr hold
  // stale shared memory (their accumulator rows are never used)
  const int rr = args.route_rows > 0 ? args.route_rows : kTileM;
  const int64_t t = static_cast<int64_t>(m) * rr + q * 32 + lane;
  const bool valid = q * 32 + lane < rr && t < args.tokens;
  if constexpr (LN) {
    const float inv_h = 1.0f / static_cast<float>(args.ln_h);
    const float mean = sum_x * inv_h;
    const float var = fmaxf(fmaf(ss, inv_h, -mean * mean), 0.f);
    const float rstd = 1.0f / sqrtf(var + args.ln_eps);
    if (valid) args.ln_stats[t] = make_float2(mean, rstd);
#pragma unroll
    for (int e = 0; e < BN; ++e)
      lg[e] = e < E ? fmaf(rstd, fmaf(-mean, sh->ln_c[e], lg[e]), sh->bias[e]) : -INFINITY;
  } else {
#pragma unroll
    for (int e = 0; e < BN; ++e) lg[e] = e < E ? lg[e] + sh->bias[e] : -INFINITY;
  }
  if (valid && args.logits) {
    float* dst = args.logits + t * E;
#pragma unroll
    for (int e = 0; e < BN; ++e)
      if (e < E) dst[e] = lg[e];
  }
  // softmax (model.py:323): exp(l - max) / sum, summed in ascending expert order
  // (the maximum as a tree: fmaxf is exact, so the order does not matter, and the tree has
  // depth log2(N) instead of a chain of N dependent instructions)
  float mt[BN / 2];
#pragma unroll
  for (int i = 0; i < BN / 2; ++i) mt[i] = fmaxf(lg[i], lg[i + BN / 2]);
#pragma unroll
  for (int w = BN / 4; w >= 1; w >>= 1)
#pragma unroll
    for (int i = 0; i < w; ++i) mt[i] = fmaxf(mt[i], mt[i + w]);
  const float mx = mt[0];
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < BN; ++e) {
    const float p = e < E ? expf(lg[e] - mx) : 0.f;
    lg[e] = p;
    s += p;
  }
  // one division, then products: BN correctly rounded divisions cost microseconds of this
  // latency-bound epilogue (one warp per SM sub-partition); the probabilities differ from
  // the quotients by at most a rounding of the reciprocal
  const float inv_s = 1.0f / s;
#pragma unroll
  for (int e = 0; e < BN; ++e) lg[e] = lg[e] * inv_s;
  // top-K by (p desc, index asc) (model.py:326): strict '>' keeps the lowest index.  The
  // selection runs twice (the first pass sums the selected probabilities, the second writes
  // them renormalised and counts them) instead of keeping the chosen indices in a
  // dynamically indexed array, which would live in local memory: under the router's HBM
  // stream every local-memory miss is an L2 round trip of about a microsecond.
  auto select = [&](uint64_t& taken, int& best, float& bv) {
    best = -1;
    bv = -INFINITY;
#pragma unroll
    for (int e = 0; e < BN; ++e) {
      const bool free_e = e < E && !((taken >> e) & 1ull);
      if (free_e && (best < 0 || lg[e] > bv)) { best = e; bv = lg[e]; }
    }
    taken |= 1ull << best;
  };
  const int et = q * 32 + lane;  // 0..127 over the group's four warps
  epilogue_bar(grp);             // the group's previous readers of hist / psum are done
  if (et < E) sh->hist[grp][et] = 0;
  epilogue_bar(grp);
  float vsum = 0.f;
  uint64_t taken = 0;
  for (int k = 0; k < K; ++k) {
    int best;
    float bv;
    select(taken, best, bv);
    vsum += bv;
  }
  if (valid) {
    uint64_t again = 0;
    for (int k = 0; k < K; ++k) {
      int best;
      float bv;
      select(again, best, bv);
      args.topk_idx[t * K + k] = best;
      args.topk_w[t * K + k] = bv / vsum;  // model.py:329
      atomicAdd(&sh->hist[grp][best], 1);
    }
  }
  // per-tile probability column sums, fixed reduction order: over each warp's 32 tokens,
  // then over the four warps
#pragma unroll
  for (int c0 = 0; c0 < BN; c0 += 32) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int j = c0 + i < BN ? c0 + i : BN - 1;  // (N 16: lanes 16..31 sum zeros)
      v[i] = c0 + i < BN && j < E && valid ? lg[j] : 0.f;
    }
    const float col = warp_column_sums(v, lane);
    if (c0 + lane < E) sh->psum[grp][q][c0 + lane] = col;
  }
  epilogue_bar(grp);
  if (et < E) {
    args.psum[static_cast<int64_t>(m) * E + et] =
        ((sh->psum[grp][0][et] + sh->psum[grp][1][et]) + sh->psum[grp][2][et]) +
        sh->psum[grp][3][et];
    args.hist[static_cast<int64_t>(m) * E + et] = sh->hist[grp][et];
  }
}

template <int EPI, int BN, int AR = 128>
__global__ void __launch_bounds__(tc_threads<EPI>(), 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap b_map,
               const TcGemmArgs args) {
  using Cfg = TcCfg<BN, AR>;
  constexpr uint32_t A_BYTES = Cfg::A_BYTES;
  constexpr int STAGES = Cfg::STAGES;
  constexpr bool LN = EPI == kRouterLN;
  constexpr bool ROUTER = EPI == kRouter || EPI == kRouterLN;
  constexpr uint32_t TCOLS = LN ? 2 * kLnAccCols : Cfg::TMEM_COLS;
  constexpr uint32_t ACC_COLS = LN ? kLnAccCols : BN;
  static_assert(!LN || BN <= kSumCol, "the LayerNorm router keeps E <= 64 logit columns");
  pdl_wait_and_trigger();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t a_s = base;
  const uint32_t b_s = base + STAGES * A_BYTES;
  const uint32_t ones_s = base + STAGES * Cfg::STAGE_BYTES;  // kRouterLN only
  auto* sh = reinterpret_cast<TcShared<STAGES>*>(gbase + STAGES * Cfg::STAGE_BYTES +
                                                 (LN ? kOnesBytes : 0));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if constexpr (LN) {
    // row 0 of the 16-row tile is 64 bf16 ones (0x3F80), rows 1..15 zero; with one 128-byte
    // row per K-block the 128B swizzle leaves row 0 in place
    uint32_t* ones = reinterpret_cast<uint32_t*>(gbase + STAGES * Cfg::STAGE_BYTES);
    for (int i = threadIdx.x; i < static_cast<int>(kOnesBytes / 4); i += blockDim.x)
      ones[i] = i < 32 ? 0x3F803F80u : 0u;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to tcgen05.mma
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
  if constexpr (ROUTER) {
    for (int i = threadIdx.x; i < args.num_experts && i < 64; i += blockDim.x) {
      sh->bias[i] = args.bias[i];
      if constexpr (LN) sh->ln_c[i] = args.ln_c[i];
    }
  }
  if (warp == 1) tmem_alloc(smem_u32(&sh->tmem_base), TCOLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  const int n_tiles = args.n_tiles, k_blocks = args.k_blocks;
  int num_m = args.num_m_tiles ? *args.num_m_tiles : args.m_tiles_host;
  if (num_m > args.max_m_tiles || num_m < 0) {  // never write past the output buffer
    if (threadIdx.x == 0) report(args.status, kStatusBadTileCount);
    num_m = num_m < 0 ? 0 : args.max_m_tiles;
  }
  const int total = num_m * n_tiles;

  // the router's tiles may hold fewer than 128 tokens (a decode batch routed in small
  // blocks over more SMs): the x box then has route_rows rows
  // (launch_tc_router picks AR = 32 only for route_rows <= 32: a_rows never exceeds AR)
  const int a_rows = ROUTER && args.route_rows > 0 ? args.route_rows : kTileM;
  const uint32_t stage_tx = static_cast<uint32_t>(a_rows) * BK * 2 + Cfg::B_BYTES;
  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int it = 0;
      for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
        const int m = tile / n_tiles, n = tile - m * n_tiles;
        const int e = expert_of(args, m);
        const int a_row = m * a_rows;
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
          mbar_arrive_expect_tx(fb, stage_tx);
          tma_load_2d(a_s + s * A_BYTES, &a_map, fb, kb * BK, a_row);
          tma_load_2d(b_s + s * Cfg::B_BYTES, &b_map, fb, kb * BK, b_row);
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
        const uint32_t d_tmem = tmem + acc * ACC_COLS;
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
          const uint32_t a_addr = a_s + s * A_BYTES, b_addr = b_s + s * Cfg::B_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t a_desc = umma_desc_sw128(a_addr + k * 32);
            const uint32_t accum = (kb | k) != 0 ? 1u : 0u;
            umma_bf16(d_tmem, a_desc, umma_desc_sw128(b_addr + k * 32), Cfg::IDESC, accum);
            if constexpr (LN) {
              umma_bf16(d_tmem + kSumCol, a_desc, umma_desc_sw128(ones_s + k * 32),
                        umma_idesc_bf16(kTileM, 16), accum);
              umma_bf16(d_tmem + kSqCol, a_desc, a_desc, umma_idesc_bf16(kTileM, 128), accum);
            }
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
    // ---------------- epilogue (warps 2..5, and 6..9 for the router) ----------------
    // group g takes this CTA's tiles g, g + G, g + 2G, ... (G groups); with two groups each
    // one owns one of the two TMEM accumulators
    constexpr int G = tc_epi_groups<EPI>();
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int grp = (warp - 2) >> 2;
    int k_local = 0;
    for (int tile = blockIdx.x + grp * gridDim.x; tile < total;
         tile += G * gridDim.x, ++k_local) {
      const int local = k_local * G + grp;  // this CTA's tiles before this one
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      const bool got = mbar_wait(smem_u32(&sh->tfull[acc]), aph);
      __syncwarp();
      const bool warp_ok = __all_sync(0xffffffffu, got);
      if constexpr (ROUTER) {
        // the router epilogue synchronises the group's four warps, so they must agree on
        // whether to go on (each warp's wait above is bounded)
        if (lane == 0) sh->ep_ok[grp][q] = warp_ok ? 1 : 0;
        epilogue_bar(grp);
        const bool all_ok =
            sh->ep_ok[grp][0] && sh->ep_ok[grp][1] && sh->ep_ok[grp][2] && sh->ep_ok[grp][3];
        if (!all_ok) {
          if (lane == 0 && !warp_ok) set_abort(sh, args.status, kStatusTimeoutEpilogue);
          break;
        }
      } else if (!warp_ok) {
        if (lane == 0) set_abort(sh, args.status, kStatusTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      const int m = tile / n_tiles, n = tile - m * n_tiles;
      const uint32_t t_row = tmem + (static_cast<uint32_t>(q * 32) << 16) + acc * ACC_COLS;
      if constexpr (ROUTER) {
        router_epilogue<BN, STAGES, LN>(args, sh, t_row, smem_u32(&sh->tempty[acc]), grp, m, q,
                                        lane);
        continue;  // the router epilogue released the accumulator after reading it
      } else {
        const int e = expert_of(args, m);
        const int64_t row = static_cast<int64_t>(m) * kTileM + q * 32 + lane;
        __nv_bfloat16* outp = static_cast<__nv_bfloat16*>(args.out) + row * args.ldo;
        const float* bias =
            args.bias ? args.bias + static_cast<int64_t>(e) * args.bias_ld + n * BN : nullptr;
        if constexpr (EPI == kGated) {
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
              const float h1 = era_fast(g[j + 1] + bias[c + j + 1], args.gamma) *
                               (u[j + 1] + bias[BN / 2 + c + j + 1]);
              packed[j / 2] = pack_bf16x2(h0, h1);
            }
            uint4* dst = reinterpret_cast<uint4*>(outp + c);
#pragma unroll
            for (int v = 0; v < 4; ++v)
              dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
          }
        } else {
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
    tmem_dealloc(tmem, TCOLS);
  }
}

template <int EPI, int BN, int AR = 128>
cudaError_t launch_cfg(const CUtensorMap& a_map, const CUtensorMap& b_map, const TcGemmArgs& args,
                       int64_t work, int num_sms, cudaStream_t s) {
  constexpr size_t smem = tc_smem_bytes<BN, EPI, AR>();
  static_assert(smem <= 232448, "shared memory budget");
  const int grid = static_cast<int>(work < num_sms ? (work > 0 ? work : 1) : num_sms);
  auto kern = tc_gemm_kernel<EPI, BN, AR>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  return launch_kernel(kern, dim3(grid), dim3(tc_threads<EPI>()), smem, s, a_map, b_map, args);
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
  if (gated) return launch_cfg<kGated, 256>(a_map, b_map, args, work, num_sms, s);
  return launch_cfg<kPlain, 256>(a_map, b_map, args, work, num_sms, s);
}

int tc_router_width(int E) {
  if (E <= 16) return 16;
  if (E <= 32) return 32;
  if (E <= 64) return 64;
  return 0;  // wider routers use the CUDA-core kernel
}

cudaError_t launch_tc_router(const CUtensorMap& x_map, const CUtensorMap& w_map,
                             const TcGemmArgs& args, int num_sms, cudaStream_t s, bool ln) {
  if (args.route_rows < 0 || args.route_rows > kTileM || args.route_rows % 16)
    return cudaErrorInvalidValue;
  const int64_t work = args.m_tiles_host;
  const bool short_blocks = args.route_rows > 0 && args.route_rows <= 32;
  if (ln) {
    if (!args.ln_stats || !args.ln_c || args.ln_h <= 0) return cudaErrorInvalidValue;
    if (short_blocks) {
      switch (tc_router_width(args.num_experts)) {
        case 16: return launch_cfg<kRouterLN, 16, 32>(x_map, w_map, args, work, num_sms, s);
        case 32: return launch_cfg<kRouterLN, 32, 32>(x_map, w_map, args, work, num_sms, s);
        case 64: return launch_cfg<kRouterLN, 64, 32>(x_map, w_map, args, work, num_sms, s);
        default: return cudaErrorInvalidValue;
      }
    }
    switch (tc_router_width(args.num_experts)) {
      case 16: return launch_cfg<kRouterLN, 16>(x_map, w_map, args, work, num_sms, s);
      case 32: return launch_cfg<kRouterLN, 32>(x_map, w_map, args, work, num_sms, s);
      case 64: return launch_cfg<kRouterLN, 64>(x_map, w_map, args, work, num_sms, s);
      default: return cudaErrorInvalidValue;
    }
  }
  if (short_blocks) {
    switch (tc_router_width(args.num_experts)) {
      case 16: return launch_cfg<kRouter, 16, 32>(x_map, w_map, args, work, num_sms, s);
      case 32: return launch_cfg<kRouter, 32, 32>(x_map, w_map, args, work, num_sms, s);
      case 64: return launch_cfg<kRouter, 64, 32>(x_map, w_map, args, work, num_sms, s);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (tc_router_width(args.num_experts)) {
    case 16: return launch_cfg<kRouter, 16>(x_map, w_map, args, work, num_sms, s);
    case 32: return launch_cfg<kRouter, 32>(x_map, w_map, args, work, num_sms, s);
    case 64: return launch_cfg<kRouter, 64>(x_map, w_map, args, work, num_sms, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace vmoe
