// Fused router: logits = x W_r^T + b_r, softmax, top-K with lowest-index tie-break,
// renormalised gate weights, and per-128-token-block expert histogram / probability sums.
//
// Reference: python/vesper/model.py:314,322 (router Linear), :323 (softmax), :326
// (torch.topk), :329 (renormalise), :366-385 (the sums the load-balancing loss needs).
//
// With a fused pre-norm (LayerNorm of python/vesper/model.py:418 folded into this read of
// x), ln_stats_kernel first computes every token's mean and 1/sqrt(var + eps) (two passes
// over the row, fp32), and the router normalises x while it stages it: the normalised rows
// never go to HBM.
//
// One CTA routes 128 tokens.  The [128 x E] logit tile is computed on CUDA cores from
// 32-column chunks of x and W_r staged in shared memory (fp32 accumulation, inputs of
// either dtype); then one thread per token does softmax and selection.  The per-block
// histogram and probability sums are written without atomics to global memory, so the
// downstream scan and loss are deterministic.
#include "common.cuh"
#include "kernels.h"

namespace vmoe {
namespace {

constexpr int kThreads = 256;
constexpr int kChunk = 32;
constexpr int kMaxTopK = 32;

// one warp per token: mean, then the centred sum of squares (the row is re-read from L1/L2)
template <typename T>
__global__ void __launch_bounds__(256)
ln_stats_kernel(const T* __restrict__ x, int64_t T_tok, int H, float eps, float2* __restrict__ stats) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (t >= T_tok) return;
  constexpr int V = Vec16<T>::N;
  const T* row = x + t * H;
  const int nvec = H / V;
  float s = 0.f;
  for (int v = lane; v < nvec; v += 32) {
    float f[V];
    load16_to_f(row + v * V, f);
#pragma unroll
    for (int i = 0; i < V; ++i) s += f[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / static_cast<float>(H);
  float q = 0.f;
  for (int v = lane; v < nvec; v += 32) {
    float f[V];
    load16_to_f(row + v * V, f);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const float d = f[i] - mean;
      q = fmaf(d, d, q);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  if (lane == 0) stats[t] = make_float2(mean, 1.0f / sqrtf(q / static_cast<float>(H) + eps));
}

template <typename T, int EB, bool LN>
__global__ void __launch_bounds__(kThreads)
router_kernel(const T* __restrict__ x, const T* __restrict__ w_r, const float* __restrict__ b_r,
              int64_t T_tok, int H, int E, int K, float* __restrict__ logits_out,
              int32_t* __restrict__ topk_idx, float* __restrict__ topk_w, int* __restrict__ hist,
              float* __restrict__ psum, const float2* __restrict__ ln_stats,
              const float* __restrict__ ln_w, const float* __restrict__ ln_b) {
  constexpr int TE = EB / 8;          // experts per thread
  constexpr int PITCH = kChunk + 1;   // padded smem row (floats)
  extern __shared__ float sm[];
  float* xs = sm;                      // [128][PITCH]
  float* ws = sm + kTileM * PITCH;     // [EB][PITCH]
  __shared__ int hist_s[EB];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t tok0 = static_cast<int64_t>(blockIdx.x) * kTileM;
  const int valid = static_cast<int>(T_tok - tok0 < kTileM ? T_tok - tok0 : kTileM);
  constexpr int V = Vec16<T>::N;  // elements per 16-byte vector

  for (int e = tid; e < EB; e += kThreads) hist_s[e] = 0;

  float acc[4][TE];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int j = 0; j < TE; ++j) acc[r][j] = 0.f;

  for (int h0 = 0; h0 < H; h0 += kChunk) {
    // stage x[tok0 .. +128][h0 .. +32] and W_r[0 .. EB][h0 .. +32] as fp32
    for (int v = tid; v < kTileM * (kChunk / V); v += kThreads) {
      const int row = v / (kChunk / V), c = (v % (kChunk / V)) * V;
      float f[V];
      if (row < valid && h0 + c < H) {
        load16_to_f(x + (tok0 + row) * H + h0 + c, f);
        if constexpr (LN) {
          // the reference's normalised row, rounded to the activation dtype (model.py:418)
          const float2 st = ln_stats[tok0 + row];
#pragma unroll
          for (int i = 0; i < V; ++i)
            f[i] = Elt<T>::to_f(Elt<T>::from_f(
                fmaf((f[i] - st.x) * st.y, ln_w[h0 + c + i], ln_b[h0 + c + i])));
        }
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) f[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < V; ++i) xs[row * PITCH + c + i] = f[i];
    }
    for (int v = tid; v < EB * (kChunk / V); v += kThreads) {
      const int row = v / (kChunk / V), c = (v % (kChunk / V)) * V;
      float f[V];
      if (row < E && h0 + c < H) {
        load16_to_f(w_r + static_cast<int64_t>(row) * H + h0 + c, f);
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) f[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < V; ++i) ws[row * PITCH + c + i] = f[i];
    }
    __syncthreads();
#pragma unroll 4
    for (int hh = 0; hh < kChunk; ++hh) {
      float a[4], b[TE];
#pragma unroll
      for (int r = 0; r < 4; ++r) a[r] = xs[(lane + 32 * r) * PITCH + hh];
#pragma unroll
      for (int j = 0; j < TE; ++j) b[j] = ws[(warp + 8 * j) * PITCH + hh];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int j = 0; j < TE; ++j) acc[r][j] = fmaf(a[r], b[j], acc[r][j]);
    }
    __syncthreads();
  }

  // logits (+ bias) into shared memory [128][EB + 1]
  float* lg = sm;
  constexpr int LP = EB + 1;
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int j = 0; j < TE; ++j) {
      const int e = warp + 8 * j;
      lg[(lane + 32 * r) * LP + e] = e < E ? acc[r][j] + b_r[e] : 0.f;
    }
  __syncthreads();

  if (tid < valid) {
    const int64_t t = tok0 + tid;
    float* row = lg + tid * LP;
    if (logits_out) {
      for (int e = 0; e < E; ++e) logits_out[t * E + e] = row[e];
    }
    // softmax (model.py:323): exp(l - max) / sum
    float m = -INFINITY;
    for (int e = 0; e < E; ++e) m = fmaxf(m, row[e]);
    float s = 0.f;
    for (int e = 0; e < E; ++e) {
      const float p = expf(row[e] - m);
      row[e] = p;
      s += p;
    }
    for (int e = 0; e < E; ++e) row[e] = row[e] / s;
    // top-K by (p desc, index asc) (model.py:326); strict '>' keeps the lowest index
    uint32_t taken[EB / 32 > 0 ? EB / 32 : 1];
#pragma unroll
    for (int i = 0; i < (EB / 32 > 0 ? EB / 32 : 1); ++i) taken[i] = 0u;
    float val[kMaxTopK];
    float vsum = 0.f;
    for (int k = 0; k < K; ++k) {
      int best = -1;
      float bv = -INFINITY;
      for (int e = 0; e < E; ++e) {
        if ((taken[e >> 5] >> (e & 31)) & 1u) continue;
        const float p = row[e];
        if (best < 0 || p > bv) { best = e; bv = p; }
      }
      taken[best >> 5] |= 1u << (best & 31);
      topk_idx[t * K + k] = best;
      val[k] = bv;
      vsum += bv;
      atomicAdd(&hist_s[best], 1);
    }
    for (int k = 0; k < K; ++k) topk_w[t * K + k] = val[k] / vsum;  // model.py:329
  }
  __syncthreads();
  // per-block histogram and probability column sums (fixed order: deterministic)
  for (int e = tid; e < E; e += kThreads) {
    float s = 0.f;
    for (int i = 0; i < valid; ++i) s += lg[i * LP + e];
    psum[static_cast<int64_t>(blockIdx.x) * E + e] = s;
    hist[static_cast<int64_t>(blockIdx.x) * E + e] = hist_s[e];
  }
}

struct RouterCall {
  const void* x;
  const void* w_r;
  const float* b_r;
  int64_t T;
  int H, E, K;
  float* logits;
  int32_t* idx;
  float* w;
  int* hist;
  float* psum;
  const LnArgs* ln;
};

template <typename T, int EB, bool LN>
cudaError_t launch_eb(const RouterCall& c, cudaStream_t s) {
  const size_t stage = static_cast<size_t>(kTileM + EB) * (kChunk + 1);
  const size_t logit = static_cast<size_t>(kTileM) * (EB + 1);
  const size_t bytes = (stage > logit ? stage : logit) * sizeof(float);
  auto kern = router_kernel<T, EB, LN>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(bytes));
  if (err != cudaSuccess) return err;
  const unsigned nblk = static_cast<unsigned>((c.T + kTileM - 1) / kTileM);
  kern<<<nblk, kThreads, bytes, s>>>(
      static_cast<const T*>(c.x), static_cast<const T*>(c.w_r), c.b_r, c.T, c.H, c.E, c.K,
      c.logits, c.idx, c.w, c.hist, c.psum, LN ? c.ln->stats : nullptr,
      LN ? c.ln->weight : nullptr, LN ? c.ln->bias : nullptr);
  return cudaGetLastError();
}

template <typename T, bool LN>
cudaError_t launch_t(const RouterCall& c, cudaStream_t s) {
  if (c.E <= 8) return launch_eb<T, 8, LN>(c, s);
  if (c.E <= 16) return launch_eb<T, 16, LN>(c, s);
  if (c.E <= 32) return launch_eb<T, 32, LN>(c, s);
  if (c.E <= 64) return launch_eb<T, 64, LN>(c, s);
  if (c.E <= 128) return launch_eb<T, 128, LN>(c, s);
  return launch_eb<T, 256, LN>(c, s);
}

template <typename T>
cudaError_t launch_stats_then_router(const RouterCall& c, cudaStream_t s) {
  if (!c.ln) return launch_t<T, false>(c, s);
  ln_stats_kernel<T><<<static_cast<unsigned>((c.T + 7) / 8), 256, 0, s>>>(
      static_cast<const T*>(c.x), c.T, c.H, c.ln->eps, c.ln->stats);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  return launch_t<T, true>(c, s);
}

}  // namespace

cudaError_t launch_router(int dtype, const void* x, const void* w_r, const float* b_r, int64_t T,
                          int H, int E, int K, float* logits, int32_t* topk_idx, float* topk_w,
                          int* hist, float* psum, const LnArgs* ln, cudaStream_t s) {
  const RouterCall c{x, w_r, b_r, T, H, E, K, logits, topk_idx, topk_w, hist, psum, ln};
  if (dtype == kF32) return launch_stats_then_router<float>(c, s);
  return launch_stats_then_router<__nv_bfloat16>(c, s);
}

}  // namespace vmoe
