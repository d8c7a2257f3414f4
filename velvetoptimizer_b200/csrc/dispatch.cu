// Token dispatch and combine: the data-movement half of the MoE forward.
//
// Reference behaviour (python/vesper/model.py):
//   :339-349  for each expert in ascending order, the tokens that chose it, in ascending
//             token order (token_mask.nonzero()), are gathered: x_e = x_flat[token_idx];
//   :337,354-357 out starts at zero and receives index_add_(token_idx, y_e * w_e) for
//             e = 0..E-1 in that order;
//   :366-385  aux = E * sum_e (count_e / (T*K)) * mean_t p[t, e].
//
// B200 layout: the permuted activations are one expert-major buffer whose expert
// segments are padded to multiples of 128 rows (the grouped-GEMM M tile), so that every
// M tile belongs to one expert and no GEMM tile needs a row mask.  Slots are assigned
// without atomics: slot(t, k) = offs[e] + (tokens of earlier 128-token blocks that chose e)
// + (rank of t among this block's tokens that chose e), which is the reference's stable
// order and makes every run bit-identical.
#include "common.cuh"
#include "kernels.h"

namespace vmoe {
namespace {

// Fixed-shape warp sum (xor butterfly): the scan's per-warp partial probability sums.
__device__ __forceinline__ float warp_sum_fixed(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Switch load-balancing loss (model.py:366-385) from the per-expert counts and probability
// sums, summed in ascending expert order.
__device__ __forceinline__ float aux_loss_of(const int* counts, const float* psum_tot, int64_t T,
                                             int E, int K) {
  const float inv_tk = 1.0f / static_cast<float>(T * K);
  const float inv_t = 1.0f / static_cast<float>(T);
  float s = 0.f;
  for (int e = 0; e < E; ++e) {
    const float f = static_cast<float>(counts[e]) * inv_tk;
    const float p = psum_tot[e] * inv_t;
    s += f * p;
  }
  return static_cast<float>(E) * s;
}

// ---- 1. per-expert exclusive scan over routing blocks --------------------------------
// grid = E, block = 256: column e of hist[nblk][E] -> excl[nblk][E], counts[e]; column
// sums of psum in a fixed order.
__global__ void __launch_bounds__(256)
scan_blocks_kernel(const int* __restrict__ hist, const float* __restrict__ psum, int nblk, int E,
                   int* __restrict__ excl, int* __restrict__ counts, float* __restrict__ psum_tot) {
  pdl_wait_and_trigger();
  const int e = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (nblk + 255) / 256;
  const int b0 = min(nblk, tid * per), b1 = min(nblk, b0 + per);
  int local = 0;
  float ps = 0.f;
  for (int b = b0; b < b1; ++b) {
    local += hist[static_cast<int64_t>(b) * E + e];
    ps += psum[static_cast<int64_t>(b) * E + e];
  }
  // block exclusive scan of `local` (warp shuffles, then warp totals)
  __shared__ int wsum[8];
  __shared__ float wps[8];
  int inc = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += n;
  }
  // fixed-shape tree for the float sum
  const float fs = warp_sum_fixed(ps);
  if (lane == 31) wsum[warp] = inc;
  if (lane == 0) wps[warp] = fs;
  __syncthreads();
  int wbase = 0;
  for (int w = 0; w < warp; ++w) wbase += wsum[w];
  int run = wbase + inc - local;
  for (int b = b0; b < b1; ++b) {
    excl[static_cast<int64_t>(b) * E + e] = run;
    run += hist[static_cast<int64_t>(b) * E + e];
  }
  if (tid == 0) {
    int tot = 0;
    float pt = 0.f;
    for (int w = 0; w < 8; ++w) { tot += wsum[w]; pt += wps[w]; }
    counts[e] = tot;
    psum_tot[e] = pt;
  }
}

// ---- 2. expert offsets, M-tile map, aux loss ------------------------------------------
// one block of 1024 threads (E <= 1024)
__global__ void __launch_bounds__(1024)
plan_kernel(const int* __restrict__ counts, const float* __restrict__ psum_tot, int64_t T, int E,
            int K, int64_t capacity, int row_align, int* __restrict__ offs,
            int* __restrict__ tile_expert, int* __restrict__ num_tiles, float* __restrict__ aux,
            int32_t* __restrict__ counts_out, int* __restrict__ zero_e) {
  pdl_wait_and_trigger();
  __shared__ int pad_s[1024];
  __shared__ int off_s[1025];
  const int tid = threadIdx.x;
  if (tid < E) {
    int kept = counts[tid];
    if (capacity > 0 && kept > capacity) kept = static_cast<int>(capacity);
    pad_s[tid] = (kept + row_align - 1) / row_align * row_align;
    if (counts_out) counts_out[tid] = counts[tid];
  }
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) { off_s[e] = run; run += pad_s[e]; }
    off_s[E] = run;
    if (num_tiles) *num_tiles = run / row_align;
    if (aux) *aux = aux_loss_of(counts, psum_tot, T, E, K);
  }
  __syncthreads();
  for (int e = tid; e <= E; e += blockDim.x) offs[e] = off_s[e];
  if (zero_e)
    for (int e = tid; e < E; e += blockDim.x) zero_e[e] = 0;
  if (tile_expert && tid < E) {  // one entry per row_align-row GEMM tile
    const int t0 = off_s[tid] / row_align, nt = pad_s[tid] / row_align;
    for (int j = 0; j < nt; ++j) tile_expert[t0 + j] = tid;
  }
}

// ---- 2b. segments of one token chunk with carried rows ---------------------------------
// Expert e's segment in a chunk's buffer holds the rows carried in from the previous chunk
// (carry_in[e], placed first) and then this chunk's new rows (counts[e]).  Only whole
// row_align-row tiles are computed; the rows past the last whole tile are carried out to the
// next chunk, except that every carried-in row is computed now (a row waits at most one
// chunk) and a chunk flagged `last` computes everything (its last tiles padded).
// one block of 1024 threads (E <= 1024)
__global__ void __launch_bounds__(1024)
plan_carry_kernel(const int* __restrict__ counts, const int* __restrict__ carry_in, int E,
                  int last, int row_align, int* __restrict__ offs, int* __restrict__ computed,
                  int* __restrict__ carry_out, int* __restrict__ tile_expert,
                  int* __restrict__ num_tiles) {
  __shared__ int pad_s[1024];
  __shared__ int off_s[1025];
  const int tid = threadIdx.x;
  if (tid < E) {
    const int cin = carry_in[tid], n = cin + counts[tid];
    const int whole = n / row_align * row_align;
    const int comp = (!last && whole >= cin) ? whole : (n + row_align - 1) / row_align * row_align;
    pad_s[tid] = comp;
    computed[tid] = comp;
    carry_out[tid] = n > comp ? n - comp : 0;
  }
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) { off_s[e] = run; run += pad_s[e]; }
    off_s[E] = run;
    *num_tiles = run / row_align;
  }
  __syncthreads();
  for (int e = tid; e <= E; e += blockDim.x) offs[e] = off_s[e];
  if (tid < E) {
    const int t0 = off_s[tid] / row_align, nt = pad_s[tid] / row_align;
    for (int j = 0; j < nt; ++j) tile_expert[t0 + j] = tid;
  }
}

// ---- 3. slot assignment + gather -----------------------------------------------------
// grid = (nblk, S), block = 128 (one thread per token of the routing block).  The S blocks
// of one routing block all derive its slots (cheap) and each copies every S-th group of
// four tokens' rows, so that a small batch's rows are copied by many SMs; only the first
// writes slot_of and the carry lists.  With a carry
// (DispatchCarry::computed set) the token chunk's new rows follow the carried-in rows of
// each segment, rows past the computed part go to the carry-out list instead of the buffer,
// and slots are numbered from slot_base (the buffer's first row in a ring of buffers).
struct DispatchCarry {
  const int* carry_in;  // [E]
  const int* computed;  // [E] rows of each segment computed in this chunk (null: no carry)
  int* list_out;        // [E][kCarryCap] global (token, k) indices carried out
  int64_t t0;           // global index of the chunk's first token
  int64_t slot_base;
};

template <typename T, bool LN>
__global__ void __launch_bounds__(128)
dispatch_kernel(const T* __restrict__ x, const int32_t* __restrict__ topk_idx,
                const int* __restrict__ excl, const int* __restrict__ offs, int64_t T_tok, int H,
                int E, int K, int64_t capacity, int* __restrict__ slot_of, T* __restrict__ x_perm,
                int64_t xp_ld, int* status, const float2* __restrict__ ln_stats,
                const float* __restrict__ ln_w, const float* __restrict__ ln_b,
                const DispatchCarry carry, int rb, const DispatchPlan plan) {
  pdl_wait_and_trigger();
  extern __shared__ uint32_t dsm[];
  uint32_t* masks = dsm;                            // [4 warps][E] token bitmasks
  int* wbase = reinterpret_cast<int*>(dsm + 4 * E);  // [4][E]
  int* slots = wbase + 4 * E;                        // [128][K]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t blk = blockIdx.x;
  const int64_t t = blk * rb + tid;  // rb tokens per routing block (<= 128 threads)
  const bool valid = tid < rb && t < T_tok;

  for (int i = tid; i < 4 * E; i += 128) masks[i] = 0u;
  const int* excl_row = plan.hist ? nullptr : excl + blk * E;  // this block's prefixes [E]
  if (plan.hist) {
    // the scan and the plan of a decode-sized batch, in every CTA: this routing block's
    // prefixes and the expert offsets from the router's histograms (the same sums as the
    // scan and plan kernels); the first CTA also writes the plan's outputs
    int* excl_s = slots + kTileM * K;  // [E]
    int* offs_s = excl_s + E;          // [E + 1]
    int* cnt_s = offs_s + E + 1;       // [E]
    int* pad_s = cnt_s + E;            // [E]
    float* ptot_s = reinterpret_cast<float*>(pad_s + E);  // [E]
    const int nblk = static_cast<int>(gridDim.x);
    const bool first = blockIdx.x == 0 && blockIdx.y == 0;
    for (int e = tid; e < E; e += 128) {
      int run = 0, mine = 0;
      for (int b = 0; b < nblk; ++b) {
        if (b == blk) mine = run;
        run += plan.hist[static_cast<int64_t>(b) * E + e];
      }
      excl_s[e] = mine;
      cnt_s[e] = run;
      const int kept = capacity > 0 && run > capacity ? static_cast<int>(capacity) : run;
      pad_s[e] = (kept + plan.row_align - 1) / plan.row_align * plan.row_align;
    }
    if (first) {  // probability sums: lane b holds block b's (nblk <= 32), fixed tree
      for (int e = warp; e < E; e += 4) {
        const float v = lane < nblk ? plan.psum[static_cast<int64_t>(lane) * E + e] : 0.f;
        const float tot = warp_sum_fixed(v);
        if (lane == 0) ptot_s[e] = tot;
      }
    }
    __syncthreads();
    if (tid == 0) {
      int run = 0;
      for (int e = 0; e < E; ++e) { offs_s[e] = run; run += pad_s[e]; }
      offs_s[E] = run;
      if (first && plan.aux) *plan.aux = aux_loss_of(cnt_s, ptot_s, T_tok, E, K);
    }
    __syncthreads();
    if (first) {
      for (int e = tid; e <= E; e += 128) plan.offs_out[e] = offs_s[e];
      if (plan.counts_out)
        for (int e = tid; e < E; e += 128) plan.counts_out[e] = cnt_s[e];
      if (plan.zero)
        for (int i = tid; i < plan.zero_n; i += 128) plan.zero[i] = 0;
    }
    excl_row = excl_s;
    offs = offs_s;
  }
  __syncthreads();
  if (valid) {
    for (int k = 0; k < K; ++k) {
      const int e = topk_idx[t * K + k];
      atomicOr(&masks[warp * E + e], 1u << lane);
    }
  }
  __syncthreads();
  for (int e = tid; e < E; e += 128) {
    int run = 0;
    for (int w = 0; w < 4; ++w) { wbase[w * E + e] = run; run += __popc(masks[w * E + e]); }
  }
  __syncthreads();
  const uint32_t lt = (1u << lane) - 1u;
  for (int k = 0; k < K; ++k) {
    int slot = -1;  // row of x_perm (relative to x_perm)
    if (valid) {
      const int e = topk_idx[t * K + k];
      const int rank = excl_row[e] + wbase[warp * E + e] + __popc(masks[warp * E + e] & lt);
      if (carry.computed) {
        const int pos = carry.carry_in[e] + rank;  // position in the segment
        const int over = pos - carry.computed[e];
        if (over < 0) {
          slot = offs[e] + pos;
        } else if (over < kCarryCap) {
          if (blockIdx.y == 0)
            carry.list_out[e * kCarryCap + over] = static_cast<int>((carry.t0 + t) * K + k);
        } else {
          report(status, kStatusBadSlot);
        }
      } else if (capacity <= 0 || rank < capacity) {
        slot = offs[e] + rank;
      }
      if (slot >= offs[e + 1]) { report(status, kStatusBadSlot); slot = -1; }
      // a carried-out row gets its slot from the next chunk (carry_rows_kernel)
      if (blockIdx.y == 0)
        slot_of[t * K + k] = slot >= 0 ? static_cast<int>(carry.slot_base + slot) : -1;
    }
    slots[tid * K + k] = slot;
  }
  __syncthreads();
  // gather: each warp copies whole rows with 16-byte vectors, reading x[t] once
  constexpr int V = Vec16<T>::N;
  const int nvec = H / V;
  const int ntok = static_cast<int>(T_tok - blk * rb < rb ? T_tok - blk * rb : rb);
  for (int i = warp + 4 * static_cast<int>(blockIdx.y); i < ntok; i += 4 * static_cast<int>(gridDim.y)) {
    const T* src = x + (blk * rb + i) * static_cast<int64_t>(H);
    float2 st = make_float2(0.f, 0.f);
    if constexpr (LN) st = ln_stats[blk * rb + i];
    for (int v0 = 0; v0 < nvec; v0 += 32 * 4) {
      uint4 buf[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int v = v0 + u * 32 + lane;
        if (v < nvec) {
          buf[u] = reinterpret_cast<const uint4*>(src)[v];
          if constexpr (LN) {  // (x - mean) * rstd * w + b, rounded to the dtype (model.py:418)
            float f[V];
            load16_to_f(reinterpret_cast<const T*>(&buf[u]), f);
            // w / b as 16-byte vectors (V floats from a 4V-byte aligned offset)
            const float4* w4 = reinterpret_cast<const float4*>(ln_w + v * V);
            const float4* b4 = reinterpret_cast<const float4*>(ln_b + v * V);
#pragma unroll
            for (int q = 0; q < V / 4; ++q) {
              const float4 w = w4[q], b = b4[q];
              f[4 * q + 0] = fmaf((f[4 * q + 0] - st.x) * st.y, w.x, b.x);
              f[4 * q + 1] = fmaf((f[4 * q + 1] - st.x) * st.y, w.y, b.y);
              f[4 * q + 2] = fmaf((f[4 * q + 2] - st.x) * st.y, w.z, b.z);
              f[4 * q + 3] = fmaf((f[4 * q + 3] - st.x) * st.y, w.w, b.w);
            }
            store16_from_f(reinterpret_cast<T*>(&buf[u]), f);
          }
        }
      }
      for (int k = 0; k < K; ++k) {
        const int s = slots[i * K + k];
        if (s < 0) continue;
        uint4* dst = reinterpret_cast<uint4*>(x_perm + static_cast<int64_t>(s) * xp_ld);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int v = v0 + u * 32 + lane;
          if (v < nvec) dst[v] = buf[u];
        }
      }
    }
  }
}

// ---- 3b. carried-in rows ---------------------------------------------------------------
// grid = E, block = 256: expert e's carried-in (token, k) rows go to the first carry_in[e]
// rows of its segment, one warp per row (x holds every token of the batch).
template <typename T>
__global__ void __launch_bounds__(256)
carry_rows_kernel(const T* __restrict__ x, int H, int K, const int* __restrict__ list_in,
                  const int* __restrict__ carry_in, const int* __restrict__ offs,
                  T* __restrict__ x_perm, int64_t xp_ld, int64_t slot_base,
                  int* __restrict__ slot_of, int* status) {
  const int e = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = carry_in[e];
  if (n > kCarryCap) {
    if (threadIdx.x == 0) report(status, kStatusBadSlot);
    return;
  }
  constexpr int V = Vec16<T>::N;
  const int nvec = H / V;
  for (int j = warp; j < n; j += 8) {
    const int idx = list_in[e * kCarryCap + j];
    const int64_t t = idx / K;
    const int row = offs[e] + j;
    const uint4* src = reinterpret_cast<const uint4*>(x + t * H);
    uint4* dst = reinterpret_cast<uint4*>(x_perm + static_cast<int64_t>(row) * xp_ld);
    for (int v = lane; v < nvec; v += 32) dst[v] = src[v];
    if (lane == 0) slot_of[idx] = static_cast<int>(slot_base + row);
  }
}

// ---- 4. combine --------------------------------------------------------------------
// fp32 accumulation in ascending expert order (model.py:339-357).  `wpt` warps (1, 2, 4 or
// 8) share one token's row, each taking every wpt-th 32-vector column group, so a small
// batch still spreads over the SMs; the per-element sum is the same for any wpt.  KMAX
// bounds top_k at compile time: the K rows of each 16-byte column chunk are loaded before
// any is summed, so their loads are in flight together.
template <typename T, int KMAX>
__global__ void __launch_bounds__(256)
combine_kernel(const T* __restrict__ y, int64_t y_ld, const int32_t* __restrict__ topk_idx,
               const float* __restrict__ topk_w, const int* __restrict__ slot_of, int64_t T_tok,
               int H, int K, T* out, const T* resid, int wpt) {
  pdl_wait_and_trigger();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * (8 / wpt) + warp / wpt;
  const int part = warp % wpt;
  if (t >= T_tok) return;
  // the token's K (expert, slot, weight) triples sorted by expert id
  int ord_e[KMAX], ord_s[KMAX];
  float ord_w[KMAX];
  int n = 0;
  for (int k = 0; k < K; ++k) {
    const int e = topk_idx[t * K + k];
    const int s = slot_of[t * K + k];
    const float w = topk_w[t * K + k];
    int j = n++;
    while (j > 0 && ord_e[j - 1] > e) {
      ord_e[j] = ord_e[j - 1]; ord_s[j] = ord_s[j - 1]; ord_w[j] = ord_w[j - 1];
      --j;
    }
    ord_e[j] = e; ord_s[j] = s; ord_w[j] = w;
  }
  constexpr int V = Vec16<T>::N;
  const int nvec = H / V;
  T* orow = out + t * static_cast<int64_t>(H);
  for (int v = part * 32 + lane; v < nvec; v += 32 * wpt) {
    uint4 raw[KMAX];
#pragma unroll
    for (int j = 0; j < KMAX; ++j)
      if (j < n && ord_s[j] >= 0)
        raw[j] = reinterpret_cast<const uint4*>(y + static_cast<int64_t>(ord_s[j]) * y_ld)[v];
    float acc[V];
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] = 0.f;
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
      if (j >= n || ord_s[j] < 0) continue;  // dropped by capacity
      float f[V];
      load16_to_f(reinterpret_cast<const T*>(&raw[j]), f);
      const float w = ord_w[j];
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(f[i], w));  // (y*w) then add
    }
    if (resid) {
      // hidden_states + ffn_out (model.py:425): ffn_out is rounded to the dtype first;
      // each thread reads its resid vector before it writes the same out vector
      float r[V];
      load16_to_f(resid + t * static_cast<int64_t>(H) + v * V, r);
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] = __fadd_rn(r[i], Elt<T>::to_f(Elt<T>::from_f(acc[i])));
    }
    store16_from_f(orow + v * V, acc);
  }
}

// ---- 5. aux loss of a batch routed in chunks -----------------------------------------
// counts[c] / psum_tot[c] are chunk c's per-expert routed rows and probability sums; the
// loss of the whole batch is E * sum_e (sum_c counts) / (T*K) * (sum_c psum) / T, summed
// over chunks and experts in a fixed order (model.py:366-385).
__global__ void aux_merge_kernel(const char* ws, size_t stride, size_t counts_off,
                                 size_t psum_off, int chunks, int64_t T, int E, int K, float* aux) {
  if (threadIdx.x != 0) return;
  const float inv_tk = 1.0f / static_cast<float>(T * K);
  const float inv_t = 1.0f / static_cast<float>(T);
  float s = 0.f;
  for (int e = 0; e < E; ++e) {
    int c_e = 0;
    float p_e = 0.f;
    for (int c = 0; c < chunks; ++c) {
      c_e += reinterpret_cast<const int*>(ws + c * stride + counts_off)[e];
      p_e += reinterpret_cast<const float*>(ws + c * stride + psum_off)[e];
    }
    s += (static_cast<float>(c_e) * inv_tk) * (p_e * inv_t);
  }
  *aux = static_cast<float>(E) * s;
}

// ---- 6. dense layer: every tile is expert 0 -------------------------------------------
__global__ void fill_tiles_kernel(int* __restrict__ tile_expert, int n, int* __restrict__ num_tiles) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    tile_expert[i] = 0;
  if (blockIdx.x == 0 && threadIdx.x == 0) *num_tiles = n;
}

}  // namespace

cudaError_t launch_fill_tiles(int* tile_expert, int n, int* num_tiles, cudaStream_t s) {
  fill_tiles_kernel<<<(n + 255) / 256 > 0 ? (n + 255) / 256 : 1, 256, 0, s>>>(tile_expert, n,
                                                                            num_tiles);
  return cudaGetLastError();
}

cudaError_t launch_aux_merge_ws(const void* ws, size_t stride, size_t counts_off, size_t psum_off,
                                int chunks, int64_t T, int E, int K, float* aux, cudaStream_t s) {
  aux_merge_kernel<<<1, 32, 0, s>>>(static_cast<const char*>(ws), stride, counts_off, psum_off,
                                    chunks, T, E, K, aux);
  return cudaGetLastError();
}

cudaError_t launch_scan_blocks(const int* hist, const float* psum, int nblk, int E, int* excl,
                               int* counts, float* psum_tot, cudaStream_t s) {
  return launch_kernel(scan_blocks_kernel, dim3(E), dim3(256), 0, s, hist, psum, nblk, E, excl,
                       counts, psum_tot);
}

cudaError_t launch_plan(const int* counts, const float* psum_tot, int64_t T, int E, int K,
                        int64_t capacity, int row_align, int* offs, int* tile_expert,
                        int* num_tiles, float* aux, int32_t* counts_out, cudaStream_t s,
                        int* zero_e) {
  return launch_kernel(plan_kernel, dim3(1), dim3(1024), 0, s, counts, psum_tot, T, E, K,
                       capacity, row_align, offs, tile_expert, num_tiles, aux, counts_out, zero_e);
}

cudaError_t launch_plan_carry(const int* counts, const int* carry_in, int E, bool last,
                              int row_align, int* offs, int* computed, int* carry_out,
                              int* tile_expert, int* num_tiles, cudaStream_t s) {
  plan_carry_kernel<<<1, 1024, 0, s>>>(counts, carry_in, E, last ? 1 : 0, row_align, offs,
                                       computed, carry_out, tile_expert, num_tiles);
  return cudaGetLastError();
}

namespace {
template <typename T, bool LN>
cudaError_t dispatch_as(const void* x, const int32_t* topk_idx, const int* excl, const int* offs,
                 int64_t T_tok, int H, int E, int K, int64_t capacity, int* slot_of, void* x_perm,
                 int64_t xp_ld, int* status, const LnArgs* ln, cudaStream_t s,
                 const DispatchCarry& carry, int rb, const DispatchPlan& plan) {
  const unsigned nblk = static_cast<unsigned>((T_tok + rb - 1) / rb);
  if (nblk == 0) return cudaSuccess;  // no tokens: nothing to place
  if (plan.hist && (nblk > 32 || E > 1024 || carry.computed || !plan.psum || !plan.offs_out ||
                    plan.row_align < 1))
    return cudaErrorInvalidValue;
  const size_t smem = (8 * static_cast<size_t>(E) + static_cast<size_t>(kTileM) * K +
                       (plan.hist ? 5 * static_cast<size_t>(E) + 1 : 0)) * 4;
  auto kern = dispatch_kernel<T, LN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  // copy slices per routing block: about 2048 CTAs in all (some 14 per SM, whose row loads
  // in flight hide the HBM latency: 4 slices per block took the 65,536-token top-4 dispatch
  // at H 4096 from 0.573 to 0.493 ms), at most one slice per four tokens
  unsigned slices = (2048u + nblk - 1) / nblk;
  const unsigned groups = static_cast<unsigned>((T_tok < rb ? T_tok : rb) + 3) / 4;
  if (slices > groups) slices = groups;
  if (slices > 32) slices = 32;
  if (slices < 1) slices = 1;
  return launch_kernel(kern, dim3(nblk, slices), dim3(128), smem, s, static_cast<const T*>(x),
                       topk_idx, excl, offs, T_tok, H, E, K, capacity, slot_of,
                       static_cast<T*>(x_perm), xp_ld, status, LN ? ln->stats : nullptr,
                       LN ? ln->weight : nullptr, LN ? ln->bias : nullptr, carry, rb, plan);
}
}  // namespace

cudaError_t launch_dispatch(int dtype, const void* x, const int32_t* topk_idx, const int* excl,
                            const int* offs, int64_t T, int H, int E, int K, int64_t capacity,
                            int* slot_of, void* x_perm, int64_t xp_ld, int* status,
                            const LnArgs* ln, cudaStream_t s, int rb, const DispatchPlan* plan) {
  if (rb < 1 || rb > kTileM) return cudaErrorInvalidValue;
  const DispatchCarry none{nullptr, nullptr, nullptr, 0, 0};
  const DispatchPlan p = plan ? *plan : DispatchPlan{};
  if (dtype == kF32) {
    if (ln) return dispatch_as<float, true>(x, topk_idx, excl, offs, T, H, E, K, capacity, slot_of, x_perm, xp_ld, status, ln, s, none, rb, p);
    return dispatch_as<float, false>(x, topk_idx, excl, offs, T, H, E, K, capacity, slot_of, x_perm, xp_ld, status, ln, s, none, rb, p);
  }
  if (ln) return dispatch_as<__nv_bfloat16, true>(x, topk_idx, excl, offs, T, H, E, K, capacity, slot_of, x_perm, xp_ld, status, ln, s, none, rb, p);
  return dispatch_as<__nv_bfloat16, false>(x, topk_idx, excl, offs, T, H, E, K, capacity, slot_of, x_perm, xp_ld, status, ln, s, none, rb, p);
}

cudaError_t launch_dispatch_carry(int dtype, const void* x, const int32_t* topk_idx,
                                  const int* excl, const int* offs, int64_t T, int H, int E,
                                  int K, int* slot_of, void* x_perm, int64_t xp_ld,
                                  const int* carry_in, const int* computed, int* list_out,
                                  int64_t t0, int64_t slot_base, int* status, cudaStream_t s) {
  const DispatchCarry carry{carry_in, computed, list_out, t0, slot_base};
  const DispatchPlan none{};
  if (dtype == kF32)
    return dispatch_as<float, false>(x, topk_idx, excl, offs, T, H, E, K, 0, slot_of, x_perm, xp_ld, status, nullptr, s, carry, kTileM, none);
  return dispatch_as<__nv_bfloat16, false>(x, topk_idx, excl, offs, T, H, E, K, 0, slot_of, x_perm, xp_ld, status, nullptr, s, carry, kTileM, none);
}

cudaError_t launch_carry_rows(int dtype, const void* x, int H, int E, int K, const int* list_in,
                              const int* carry_in, const int* offs, void* x_perm, int64_t xp_ld,
                              int64_t slot_base, int* slot_of, int* status, cudaStream_t s) {
  if (dtype == kF32)
    carry_rows_kernel<float><<<E, 256, 0, s>>>(static_cast<const float*>(x), H, K, list_in, carry_in,
                                               offs, static_cast<float*>(x_perm), xp_ld, slot_base,
                                               slot_of, status);
  else
    carry_rows_kernel<__nv_bfloat16><<<E, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), H, K, list_in, carry_in, offs,
        static_cast<__nv_bfloat16*>(x_perm), xp_ld, slot_base, slot_of, status);
  return cudaGetLastError();
}

cudaError_t launch_combine(int dtype, const void* y, int64_t y_ld, const int32_t* topk_idx,
                           const float* topk_w, const int* slot_of, int64_t T, int H, int K,
                           void* out, const void* resid, cudaStream_t s) {
  if (K > 32) return cudaErrorInvalidValue;
  if (T <= 0) return cudaSuccess;
  // warps per token: enough blocks for about two per SM (8 for a decode batch, 1 from
  // about 2,400 tokens up)
  int wpt = 1;
  while (wpt < 8 && T * wpt < 2 * 148 * 8) wpt *= 2;
  const unsigned grid = static_cast<unsigned>((T * wpt + 7) / 8);
  auto go = [&](auto kern, auto* yy, auto* o, auto* r) {
    return launch_kernel(kern, dim3(grid), dim3(256), 0, s, yy, y_ld, topk_idx, topk_w, slot_of,
                         T, H, K, o, r, wpt);
  };
  if (dtype == kF32) {
    const float* yy = static_cast<const float*>(y);
    float* o = static_cast<float*>(out);
    const float* r = static_cast<const float*>(resid);
    if (K <= 2) return go(combine_kernel<float, 2>, yy, o, r);
    if (K <= 4) return go(combine_kernel<float, 4>, yy, o, r);
    if (K <= 8) return go(combine_kernel<float, 8>, yy, o, r);
    return go(combine_kernel<float, 32>, yy, o, r);
  }
  const __nv_bfloat16* yy = static_cast<const __nv_bfloat16*>(y);
  __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
  const __nv_bfloat16* r = static_cast<const __nv_bfloat16*>(resid);
  if (K <= 2) return go(combine_kernel<__nv_bfloat16, 2>, yy, o, r);
  if (K <= 4) return go(combine_kernel<__nv_bfloat16, 4>, yy, o, r);
  if (K <= 8) return go(combine_kernel<__nv_bfloat16, 8>, yy, o, r);
  return go(combine_kernel<__nv_bfloat16, 32>, yy, o, r);
}

}  // namespace vmoe
