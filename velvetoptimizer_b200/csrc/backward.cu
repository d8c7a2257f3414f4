// Data-movement and routing half of the MoE backward (bf16 activations, fp32 math).
//
// Autograd of MoELayer.forward (python/vesper/model.py:317-385) restated per kernel:
//   combine_bwd  out += y_e * w_e (:354-357)     -> dy = w * dout, dw = <dout, y>
//   router_bwd   w = p_k / sum p_k (:329), aux = E sum_e f_e mean_t p (:366-385),
//                p = softmax(logits) (:323)       -> dlogits
//   gather_dx    x_e = x[token_idx] (:348-349)    -> dx[t] = sum over its rows of dx_rows
//   transpose    K-contiguous operands for the weight-gradient GEMMs (dW = dY^T X), with the
//                column sums of every 64-row block (bias gradients) on the way
// Every reduction runs in a fixed order (no atomics), so the backward is deterministic.
#include "common.cuh"
#include "kernels.h"

namespace vmoe {
namespace {

// ---- transpose -------------------------------------------------------------------------
// 64 x 64 tiles through shared memory with 16-byte loads and stores; block 256; grid
// (dst_cols / 64, dst_rows / 64, batch).  Tile rows are stored with their 8-column chunks
// rotated by (row / 8) so that the column reads of the store phase hit 16 distinct banks.
constexpr int kTP = 72;  // shared row pitch (elements): 144 bytes, 16-byte aligned rows

__device__ __forceinline__ int tpos(int r, int c) { return 8 * (((c >> 3) + (r >> 3)) & 7) + (c & 7); }

__global__ void __launch_bounds__(256)
transpose_bf16_kernel(const __nv_bfloat16* __restrict__ src, int64_t rows, int64_t cols,
                      int64_t src_ld, int64_t src_bs, __nv_bfloat16* __restrict__ dst,
                      int64_t dst_rows, int64_t dst_cols, int64_t dst_bs,
                      float* __restrict__ colsum) {
  __shared__ __align__(16) __nv_bfloat16 tile[64 * kTP];
  const int tid = threadIdx.x;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * 64;  // source rows = dst columns
  const int64_t c0 = static_cast<int64_t>(blockIdx.y) * 64;  // source cols = dst rows
  const int b = blockIdx.z;
  const __nv_bfloat16* sb = src + b * src_bs;
  const bool vec_src = (src_ld & 7) == 0 && (reinterpret_cast<uintptr_t>(sb) & 15) == 0;
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int i = tid + 256 * it;
    const int rr = i >> 3, ch = i & 7;
    const int64_t r = r0 + rr, c = c0 + 8 * ch;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < rows) {
      if (vec_src && c + 8 <= cols) {
        v = *reinterpret_cast<const uint4*>(sb + r * src_ld + c);
      } else {
        __align__(16) __nv_bfloat16 e[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) e[j] = c + j < cols ? sb[r * src_ld + c + j] : __float2bfloat16_rn(0.f);
        v = *reinterpret_cast<const uint4*>(e);
      }
    }
    *reinterpret_cast<uint4*>(tile + rr * kTP + tpos(rr, 8 * ch)) = v;
  }
  __syncthreads();
  if (colsum && tid < 64) {  // this 64-row block's column sums, rows in ascending order
    const int cc = tid;
    const int64_t nrb = (rows + 63) / 64;
    if (c0 + cc < cols && blockIdx.x < nrb) {
      float s = 0.f;
      for (int rr = 0; rr < 64; ++rr) s += __bfloat162float(tile[rr * kTP + tpos(rr, cc)]);
      colsum[(static_cast<int64_t>(b) * nrb + blockIdx.x) * cols + c0 + cc] = s;
    }
  }
  __nv_bfloat16* db = dst + b * dst_bs;
  const bool vec_dst = (dst_cols & 7) == 0 && (reinterpret_cast<uintptr_t>(db) & 15) == 0;
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int i = tid + 256 * it;
    const int cc = i >> 3, ch = i & 7;  // dst row c0 + cc, dst columns r0 + 8 ch .. + 8
    const int64_t drow = c0 + cc, dcol = r0 + 8 * ch;
    if (drow >= dst_rows) continue;
    __align__(16) __nv_bfloat16 e[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int rr = 8 * ch + j;
      e[j] = tile[rr * kTP + tpos(rr, cc)];
    }
    if (vec_dst && dcol + 8 <= dst_cols) {
      *reinterpret_cast<uint4*>(db + drow * dst_cols + dcol) = *reinterpret_cast<const uint4*>(e);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (dcol + j < dst_cols) db[drow * dst_cols + dcol + j] = e[j];
    }
  }
}

// ---- zero the padding rows of the expert segments -------------------------------------
__global__ void zero_pad_rows_kernel(char* __restrict__ buf, int64_t ld_bytes, int64_t row_bytes,
                                     const int* __restrict__ offs, const int* __restrict__ counts,
                                     int64_t capacity) {
  const int e = blockIdx.y;
  int kept = counts[e];
  if (capacity > 0 && kept > capacity) kept = static_cast<int>(capacity);
  const int64_t r0 = offs[e] + kept, r1 = offs[e + 1];
  const int64_t nvec = row_bytes / 16;
  const int64_t total = (r1 - r0) * nvec;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = r0 + i / nvec, v = i % nvec;
    reinterpret_cast<uint4*>(buf + r * ld_bytes)[v] = make_uint4(0u, 0u, 0u, 0u);
  }
}

// ---- combine backward: one warp per token -----------------------------------------------
// KMAX bounds top_k at compile time so the per-slot state stays in registers and the K row
// loads of each 16-byte column chunk are issued together.
template <int KMAX>
__global__ void __launch_bounds__(256)
combine_bwd_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ y,
                   int64_t y_ld, const int32_t* __restrict__ topk_idx,
                   const float* __restrict__ topk_w, const int* __restrict__ slot_of, int64_t T,
                   int H, int K, __nv_bfloat16* __restrict__ dy, int64_t dy_ld,
                   float* __restrict__ dw) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  int slot[KMAX];
  float wk[KMAX], dot[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    slot[k] = k < K ? slot_of[t * K + k] : -1;
    wk[k] = k < K ? topk_w[t * K + k] : 0.f;
    dot[k] = 0.f;
  }
  const int nvec = H / 8;
  const __nv_bfloat16* drow = dout + t * static_cast<int64_t>(H);
  for (int v = lane; v < nvec; v += 32) {
    const uint4 dv = reinterpret_cast<const uint4*>(drow)[v];
    uint4 yv[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
      if (slot[k] >= 0) yv[k] = reinterpret_cast<const uint4*>(y + static_cast<int64_t>(slot[k]) * y_ld)[v];
    float d[8];
    load16_to_f(reinterpret_cast<const __nv_bfloat16*>(&dv), d);
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      if (slot[k] < 0) continue;
      float f[8], o[8];
      load16_to_f(reinterpret_cast<const __nv_bfloat16*>(&yv[k]), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        dot[k] = fmaf(d[i], f[i], dot[k]);
        o[i] = d[i] * wk[k];
      }
      store16_from_f(dy + static_cast<int64_t>(slot[k]) * dy_ld + v * 8, o);
    }
  }
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    if (k >= K) break;
    float s = dot[k];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) dw[t * K + k] = slot[k] < 0 ? 0.f : s;
  }
}

// ---- router backward: one thread per token, 128 tokens per block ------------------------
__global__ void __launch_bounds__(128)
router_bwd_kernel(const float* __restrict__ logits, const int32_t* __restrict__ topk_idx,
                  const float* __restrict__ dw, const int32_t* __restrict__ counts, int64_t T,
                  int E, int K, const float* __restrict__ daux_ptr, float* __restrict__ dlogits,
                  __nv_bfloat16* __restrict__ dl_bf16, int e_ld, float* __restrict__ blocksum) {
  extern __shared__ float rs[];  // [128][E + 1]
  const int tid = threadIdx.x;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * 128 + tid;
  const int LP = E + 1;
  float* row = rs + tid * LP;
  const bool valid = t < T;
  if (valid) {
    // softmax as the forward (model.py:323)
    float mx = -INFINITY;
    for (int e = 0; e < E; ++e) mx = fmaxf(mx, logits[t * E + e]);
    float s = 0.f;
    for (int e = 0; e < E; ++e) {
      const float p = expf(logits[t * E + e] - mx);
      row[e] = p;
      s += p;
    }
    for (int e = 0; e < E; ++e) row[e] = row[e] / s;
    // top-K renormalisation (model.py:329): w_k = p_k / S
    float S = 0.f, wdw = 0.f;
    for (int k = 0; k < K; ++k) S += row[topk_idx[t * K + k]];
    for (int k = 0; k < K; ++k) wdw += (row[topk_idx[t * K + k]] / S) * dw[t * K + k];
    // dp: the aux loss term on every expert (counts carry no gradient), plus the K chosen
    const float daux = daux_ptr ? *daux_ptr : 0.f;
    const float aux_c = daux * static_cast<float>(E) / (static_cast<float>(T) * static_cast<float>(T * K));
    float pdp = 0.f;
    float dpk[32];
    for (int k = 0; k < K; ++k) dpk[k] = (dw[t * K + k] - wdw) / S;
    // dl = p * (dp - sum p dp) (softmax backward); first sum p dp
    for (int e = 0; e < E; ++e) {
      float dp = aux_c * static_cast<float>(counts[e]);
      for (int k = 0; k < K; ++k)
        if (topk_idx[t * K + k] == e) dp += dpk[k];
      pdp = fmaf(row[e], dp, pdp);
    }
    for (int e = 0; e < E; ++e) {
      float dp = aux_c * static_cast<float>(counts[e]);
      for (int k = 0; k < K; ++k)
        if (topk_idx[t * K + k] == e) dp += dpk[k];
      const float dl = row[e] * (dp - pdp);
      row[e] = dl;
      dlogits[t * E + e] = dl;
      dl_bf16[t * e_ld + e] = __float2bfloat16_rn(dl);
    }
    for (int e = E; e < e_ld; ++e) dl_bf16[t * e_ld + e] = __float2bfloat16_rn(0.f);
  } else {
    for (int e = 0; e < E; ++e) row[e] = 0.f;
  }
  __syncthreads();
  // per-block column sums over the 128 tokens in ascending order (bias gradient)
  for (int e = tid; e < E; e += 128) {
    float s = 0.f;
    for (int i = 0; i < 128; ++i) s += rs[i * LP + e];
    blocksum[static_cast<int64_t>(blockIdx.x) * E + e] = s;
  }
}

// ---- dx gather: one warp per token ---------------------------------------------------
__global__ void __launch_bounds__(256)
gather_dx_kernel(const __nv_bfloat16* __restrict__ dxr, int64_t dxr_ld,
                 const __nv_bfloat16* __restrict__ dxr_router, int64_t router_ld,
                 const int32_t* __restrict__ topk_idx, const int* __restrict__ slot_of, int64_t T,
                 int H, int K, __nv_bfloat16* __restrict__ dx) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  int ord_e[32], ord_s[32];
  int n = 0;
  for (int k = 0; k < K; ++k) {  // the token's rows sorted by expert id
    const int e = topk_idx[t * K + k], s = slot_of[t * K + k];
    int j = n++;
    while (j > 0 && ord_e[j - 1] > e) {
      ord_e[j] = ord_e[j - 1];
      ord_s[j] = ord_s[j - 1];
      --j;
    }
    ord_e[j] = e;
    ord_s[j] = s;
  }
  const int nvec = H / 8;
  for (int v = lane; v < nvec; v += 32) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int j = 0; j < n; ++j) {
      if (ord_s[j] < 0) continue;
      float f[8];
      load16_to_f(dxr + static_cast<int64_t>(ord_s[j]) * dxr_ld + v * 8, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += f[i];
    }
    if (dxr_router) {
      float f[8];
      load16_to_f(dxr_router + t * router_ld + v * 8, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += f[i];
    }
    store16_from_f(dx + t * static_cast<int64_t>(H) + v * 8, acc);
  }
}

// ---- per-expert sums of row-block partials ---------------------------------------------
__global__ void segment_sum_kernel(const float* __restrict__ part, int64_t part_ld,
                                   const int* __restrict__ offs, int nblk_host, int cols,
                                   int blk_rows, float* __restrict__ out, float* __restrict__ out2,
                                   int valid, bool interleave) {
  const int e = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  const int b0 = offs ? offs[e] / blk_rows : 0;
  const int b1 = offs ? offs[e + 1] / blk_rows : nblk_host;
  float s = 0.f;
  for (int b = b0; b < b1; ++b) s += part[static_cast<int64_t>(b) * part_ld + c];
  if (!interleave) {
    if (c < valid) out[static_cast<int64_t>(e) * valid + c] = s;
  } else {
    const int which = (c / 128) & 1, i = (c / 256) * 128 + (c & 127);
    if (i < valid) (which ? out2 : out)[static_cast<int64_t>(e) * valid + i] = s;
  }
}

}  // namespace

cudaError_t launch_transpose_bf16(const void* src, int64_t rows, int64_t cols, int64_t src_ld,
                                  int64_t src_batch_stride, int batch, void* dst,
                                  int64_t dst_rows, int64_t dst_cols, int64_t dst_batch_stride,
                                  float* colsum, cudaStream_t s) {
  if (dst_rows < cols || dst_cols < rows) return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>((dst_cols + 63) / 64), static_cast<unsigned>((dst_rows + 63) / 64),
                  static_cast<unsigned>(batch));
  transpose_bf16_kernel<<<grid, 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(src), rows, cols, src_ld, src_batch_stride,
      static_cast<__nv_bfloat16*>(dst), dst_rows, dst_cols, dst_batch_stride, colsum);
  return cudaGetLastError();
}

cudaError_t launch_zero_pad_rows(void* buf, int64_t ld_bytes, int64_t row_bytes, const int* offs,
                                 const int* counts, int E, int64_t capacity, cudaStream_t s) {
  if (row_bytes % 16 || ld_bytes % 16) return cudaErrorInvalidValue;
  zero_pad_rows_kernel<<<dim3(8, static_cast<unsigned>(E)), 256, 0, s>>>(
      static_cast<char*>(buf), ld_bytes, row_bytes, offs, counts, capacity);
  return cudaGetLastError();
}

cudaError_t launch_combine_bwd(const void* dout, const void* y, int64_t y_ld,
                               const int32_t* topk_idx, const float* topk_w, const int* slot_of,
                               int64_t T, int H, int K, void* dy, int64_t dy_ld, float* dw,
                               cudaStream_t s) {
  if (K > 32 || H % 8) return cudaErrorInvalidValue;
  const unsigned grid = static_cast<unsigned>((T + 7) / 8);
  const auto* d = static_cast<const __nv_bfloat16*>(dout);
  const auto* yy = static_cast<const __nv_bfloat16*>(y);
  auto* o = static_cast<__nv_bfloat16*>(dy);
  if (K <= 2)
    combine_bwd_kernel<2><<<grid, 256, 0, s>>>(d, yy, y_ld, topk_idx, topk_w, slot_of, T, H, K, o, dy_ld, dw);
  else if (K <= 4)
    combine_bwd_kernel<4><<<grid, 256, 0, s>>>(d, yy, y_ld, topk_idx, topk_w, slot_of, T, H, K, o, dy_ld, dw);
  else if (K <= 8)
    combine_bwd_kernel<8><<<grid, 256, 0, s>>>(d, yy, y_ld, topk_idx, topk_w, slot_of, T, H, K, o, dy_ld, dw);
  else
    combine_bwd_kernel<32><<<grid, 256, 0, s>>>(d, yy, y_ld, topk_idx, topk_w, slot_of, T, H, K, o, dy_ld, dw);
  return cudaGetLastError();
}

cudaError_t launch_router_bwd(const float* logits, const int32_t* topk_idx, const float* dw,
                              const int32_t* counts, int64_t T, int E, int K, const float* daux,
                              float* dlogits, void* dl_bf16, int e_ld, float* dl_blocksum,
                              cudaStream_t s) {
  if (K > 32) return cudaErrorInvalidValue;
  const size_t smem = static_cast<size_t>(128) * (E + 1) * sizeof(float);
  cudaError_t err = cudaFuncSetAttribute(router_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  router_bwd_kernel<<<static_cast<unsigned>((T + 127) / 128), 128, smem, s>>>(
      logits, topk_idx, dw, counts, T, E, K, daux, dlogits, static_cast<__nv_bfloat16*>(dl_bf16),
      e_ld, dl_blocksum);
  return cudaGetLastError();
}

cudaError_t launch_gather_dx(const void* dxr, int64_t dxr_ld, const void* dxr_router,
                             int64_t router_ld, const int32_t* topk_idx, const int* slot_of,
                             int64_t T, int H, int K, void* dx, cudaStream_t s) {
  if (K > 32 || H % 8) return cudaErrorInvalidValue;
  gather_dx_kernel<<<static_cast<unsigned>((T + 7) / 8), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(dxr), dxr_ld, static_cast<const __nv_bfloat16*>(dxr_router),
      router_ld, topk_idx, slot_of, T, H, K, static_cast<__nv_bfloat16*>(dx));
  return cudaGetLastError();
}

cudaError_t launch_segment_sum(const float* part, int64_t part_ld, const int* offs, int E,
                               int cols, int blk_rows, float* out, float* out2, int valid,
                               bool interleave, cudaStream_t s) {
  // offs == nullptr: one segment of E row blocks (E is then the block count)
  const int nseg = offs ? E : 1;
  segment_sum_kernel<<<dim3(static_cast<unsigned>((cols + 255) / 256), static_cast<unsigned>(nseg)),
                       256, 0, s>>>(part, part_ld, offs, offs ? 0 : E, cols, blk_rows, out, out2,
                                    valid, interleave);
  return cudaGetLastError();
}

}  // namespace vmoe
