// fp32 grouped expert GEMMs on CUDA cores: the fp32 path, whose tolerance (1e-5
// norm-relative against the reference's fp32 forward) rules out the tensor cores' tf32.
//
// gemm1: h = ERA(A Wg_e^T + bg_e) * (A Wu_e^T + bu_e)   (python/vesper/model.py:295-297)
// gemm2: y = A Wd_e^T + bd_e                            (python/vesper/model.py:298)
// A is the expert-major permuted buffer; each 128-row M tile belongs to the expert in
// tile_expert[], and the number of live tiles is read on the device (no host sync).
// A CTA computes a 64 x 64 output tile with 256 threads, 4 x 4 outputs each.
#include "common.cuh"
#include "kernels.h"

namespace vmoe {
namespace {

constexpr int BM = 64, BN = 64, BK = 16;

template <bool GATED>
__global__ void __launch_bounds__(256)
simt_gemm_kernel(const float* __restrict__ a, int64_t lda, const float* __restrict__ w0,
                 const float* __restrict__ w1, const float* __restrict__ b0,
                 const float* __restrict__ b1, float* __restrict__ c, int64_t ldc, int N, int K,
                 float gamma, const int* __restrict__ tile_expert, const int* __restrict__ num_tiles,
                 int num_experts, int* status) {
  const int mt = blockIdx.y / (kTileM / BM);
  if (mt >= *num_tiles) return;
  int e = tile_expert[mt];
  if (static_cast<unsigned>(e) >= static_cast<unsigned>(num_experts)) {
    if (threadIdx.x == 0) report(status, kStatusBadExpert);
    return;
  }
  const int64_t row0 = static_cast<int64_t>(blockIdx.y) * BM;
  const int n0 = blockIdx.x * BN;
  const float* wa = w0 + static_cast<int64_t>(e) * N * K;
  const float* wb = GATED ? w1 + static_cast<int64_t>(e) * N * K : nullptr;

  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  __shared__ float Cs[GATED ? BK : 1][GATED ? BN + 4 : 1];

  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  float acc0[4][4], acc1[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) { acc0[i][j] = 0.f; acc1[i][j] = 0.f; }

  // loader mapping: 64 rows x 16 k = 256 float4 slots -> one per thread
  const int lr = tid >> 2, lk = (tid & 3) * 4;
  for (int k0 = 0; k0 < K; k0 += BK) {
    {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k0 + lk < K) v = *reinterpret_cast<const float4*>(a + (row0 + lr) * lda + k0 + lk);
      As[lk + 0][lr] = v.x; As[lk + 1][lr] = v.y; As[lk + 2][lr] = v.z; As[lk + 3][lr] = v.w;
      float4 u = make_float4(0.f, 0.f, 0.f, 0.f);
      if (n0 + lr < N && k0 + lk < K)
        u = *reinterpret_cast<const float4*>(wa + static_cast<int64_t>(n0 + lr) * K + k0 + lk);
      Bs[lk + 0][lr] = u.x; Bs[lk + 1][lr] = u.y; Bs[lk + 2][lr] = u.z; Bs[lk + 3][lr] = u.w;
      if constexpr (GATED) {
        float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
        if (n0 + lr < N && k0 + lk < K)
          g = *reinterpret_cast<const float4*>(wb + static_cast<int64_t>(n0 + lr) * K + k0 + lk);
        Cs[lk + 0][lr] = g.x; Cs[lk + 1][lr] = g.y; Cs[lk + 2][lr] = g.z; Cs[lk + 3][lr] = g.w;
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float av[4], bv[4], cv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
      if constexpr (GATED) {
#pragma unroll
        for (int j = 0; j < 4; ++j) cv[j] = Cs[kk][tx * 4 + j];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc0[i][j] = fmaf(av[i], bv[j], acc0[i][j]);
          if constexpr (GATED) acc1[i][j] = fmaf(av[i], cv[j], acc1[i][j]);
        }
    }
    __syncthreads();
  }
  // epilogue
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = row0 + ty * 4 + i;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= N) continue;
      float v = acc0[i][j] + b0[static_cast<int64_t>(e) * N + n];
      if constexpr (GATED) {
        const float u = acc1[i][j] + b1[static_cast<int64_t>(e) * N + n];
        v = era_precise(v, gamma) * u;
      }
      c[r * ldc + n] = v;
    }
  }
}

}  // namespace

cudaError_t launch_simt_gemm1(const float* a, int64_t lda, const float* wg, const float* wu,
                              const float* bg, const float* bu, float* h, int64_t ldh, int N,
                              int K, float gamma, const int* tile_expert, const int* num_tiles,
                              int64_t max_tiles, int num_experts, int* status, cudaStream_t s) {
  dim3 grid((N + BN - 1) / BN, static_cast<unsigned>(max_tiles * (kTileM / BM)));
  simt_gemm_kernel<true><<<grid, 256, 0, s>>>(a, lda, wg, wu, bg, bu, h, ldh, N, K, gamma,
                                              tile_expert, num_tiles, num_experts, status);
  return cudaGetLastError();
}

cudaError_t launch_simt_gemm2(const float* a, int64_t lda, const float* wd, const float* bd,
                              float* y, int64_t ldy, int N, int K, const int* tile_expert,
                              const int* num_tiles, int64_t max_tiles, int num_experts,
                              int* status, cudaStream_t s) {
  dim3 grid((N + BN - 1) / BN, static_cast<unsigned>(max_tiles * (kTileM / BM)));
  simt_gemm_kernel<false><<<grid, 256, 0, s>>>(a, lda, wd, nullptr, bd, nullptr, y, ldy, N, K,
                                               0.f, tile_expert, num_tiles, num_experts, status);
  return cudaGetLastError();
}

}  // namespace vmoe
