// Expert-parallel exchange fused into the kernels over NVLink peer memory.
//
// Every rank owns one symmetric region (same layout on every GPU, mapped into every peer
// through CUDA IPC):
//   sig        uint32 [3][G]   epoch flags: [0] counts published, [1] rows dispatched,
//                              [2] expert outputs ready; flag [k][s] is written by rank s
//   all_counts int32  [G][E]   routed rows per (source rank, global expert)
//   recv       [cap_rows, H]   rows for this rank's local experts, one segment per local
//                              expert padded to 128-row GEMM tiles, sources in rank order
//   y          [cap_rows, H]   expert outputs, same layout
//
// One forward, with no host synchronisation and no collective library:
//   publish  : write my counts[E] into every peer's all_counts[me], then raise sig[0][me]
//   dispatch : wait for every sig[0]; from all_counts every block derives every
//              destination's layout, assigns each (token, k) its row in the owner's recv
//              (sources in rank order, tokens ascending) and stores the token row straight
//              into the owner's memory (16-byte NVLink stores); the last block to finish
//              raises sig[1][me] on every peer; block 0 writes this rank's GEMM tile map
//   wait(1)  : local rows complete -> the grouped GEMMs run on recv (local memory) -> y
//   signal(2), wait(2)
//   combine  : each token reads its K expert rows from the owners' y (NVLink loads) and
//              sums them in ascending expert order in fp32 -- the single-GPU arithmetic,
//              so outputs are bit-identical to the one-GPU forward.
// Push mode (bf16 with the CTA-pair GEMMs): the dispatch also writes every row's return
// address (epoch, source rank, t*K + k) into the owner's `ret`; the down GEMM's epilogue
// stores each output row straight into its source rank's return buffer `back` over NVLink,
// tile by tile while the GEMM runs (the GEMM -> exchange step is one kernel), and the
// combine reads the token's rows from local memory in the same order.
// Flags hold the forward's epoch (monotonic), so nothing is reset between forwards; the
// stream order of the stages on every rank rules out reuse races (a rank republishes its
// counts only after its combine, which waited for every peer's experts, which waited for
// every dispatch).  Every spin is bounded by kWaitLimitNs and reports a status code.
// No TMA or any bulk copy touches peer memory: peers are read and written with plain
// vector loads and stores only.
#include "common.cuh"
#include "kernels.h"

namespace vmoe {
namespace {

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned* sig_ptr(const P2PArgs& a, int rank, int which, int src) {
  return reinterpret_cast<unsigned*>(a.peer_base[rank] + a.sig_off) + which * a.G + src;
}

// Wait until flag [which][s] >= epoch for every source s (bounded).  Returns false on timeout.
__device__ bool wait_all(const P2PArgs& a, int which) {
  const unsigned* sig = reinterpret_cast<const unsigned*>(a.peer_base[a.me] + a.sig_off) + which * a.G;
  const uint64_t t0 = globaltimer_ns();
  for (int s = 0; s < a.G; ++s) {
    uint32_t it = 0;
    while (static_cast<int>(ld_acquire_sys(sig + s) - a.epoch) < 0) {
      if ((++it & 255u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
  }
  return true;
}

__global__ void p2p_publish_kernel(P2PArgs a, const int* __restrict__ counts) {
  for (int d = 0; d < a.G; ++d) {
    int* dst = reinterpret_cast<int*>(a.peer_base[d] + a.counts_off) + a.me * a.E;
    for (int e = threadIdx.x; e < a.E; e += blockDim.x) dst[e] = counts[e];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < a.G) st_release_sys(sig_ptr(a, threadIdx.x, 0, a.me), a.epoch);
}

__global__ void p2p_wait_kernel(P2PArgs a, int which) {
  if (threadIdx.x == 0 && !wait_all(a, which)) report(a.status, kStatusTimeoutPeer);
}

__global__ void p2p_signal_kernel(P2PArgs a, int which) {
  __threadfence_system();
  if (threadIdx.x < a.G) st_release_sys(sig_ptr(a, threadIdx.x, which, a.me), a.epoch);
}

// grid = (max(1, nblk), S) blocks of 128 threads (one thread per token of a 128-token
// block): the S blocks of a routing block all derive its rows (cheap) and each copies every
// S-th group of four tokens, so that many CTAs keep row stores in flight over NVLink; only
// the first writes the block's row map and return addresses
template <typename T>
__global__ void __launch_bounds__(128)
p2p_dispatch_kernel(P2PArgs a, const T* __restrict__ x, const int32_t* __restrict__ topk_idx,
                    const int* __restrict__ excl, int64_t T_tok) {
  extern __shared__ uint32_t dsm[];
  const int E = a.E, K = a.K, G = a.G, El = a.El;
  uint32_t* masks = dsm;                                  // [4][E]
  int* wbase = reinterpret_cast<int*>(dsm + 4 * E);      // [4][E]
  int* base_s = wbase + 4 * E;                           // [E] my first row at each owner
  int* cnt = base_s + E;                                 // [G][E] all_counts
  int* slot_rank = cnt + G * E;                          // [128][K]
  int* slot_row = slot_rank + kTileM * K;                // [128][K]
  __shared__ int ok_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t blk = blockIdx.x;

  if (tid == 0) {
    ok_s = wait_all(a, 0) ? 1 : 0;
    if (!ok_s) report(a.status, kStatusTimeoutPeer);
  }
  for (int i = tid; i < 4 * E; i += 128) masks[i] = 0u;
  __syncthreads();
  const bool ok = ok_s != 0;
  const bool first = blockIdx.y == 0;
  if (!ok && blk == 0 && first && tid == 0) *a.num_tiles = 0;  // no GEMM work after a failed wait
  if (ok) {
    const int* all_counts = reinterpret_cast<const int*>(a.peer_base[a.me] + a.counts_off);
    for (int i = tid; i < G * E; i += 128) cnt[i] = all_counts[i];
  }
  __syncthreads();
  if (ok) {
    // my first row in the owner's recv buffer for every global expert
    for (int e = tid; e < E; e += 128) {
      const int d = e / El, el = e - d * El;
      int64_t off = 0;
      for (int j = 0; j < el; ++j) {
        int64_t n = 0;
        for (int s = 0; s < G; ++s) n += cnt[s * E + d * El + j];
        off += (n + a.row_align - 1) / a.row_align * a.row_align;
      }
      for (int s = 0; s < a.me; ++s) off += cnt[s * E + e];
      const int64_t end = off + cnt[a.me * E + e];
      if (end > a.cap_rows) {
        report(a.status, kStatusCapacity);
        base_s[e] = -1;
      } else {
        base_s[e] = static_cast<int>(off);
      }
    }
    // block 0 writes this rank's tile map (segments of its local experts)
    if (blk == 0 && first && tid == 0) {
      *a.num_tiles = 0;
      int64_t t0 = 0;
      for (int el = 0; el < El; ++el) {
        int64_t n = 0;
        for (int s = 0; s < G; ++s) n += cnt[s * E + a.me * El + el];
        const int64_t tiles = (n + a.row_align - 1) / a.row_align;
        if ((t0 + tiles) * a.row_align > a.cap_rows) { report(a.status, kStatusCapacity); break; }
        for (int64_t j = 0; j < tiles; ++j) a.tile_expert[t0 + j] = el;
        t0 += tiles;
      }
      *a.num_tiles = static_cast<int>(t0);
    }
  }
  const int64_t t = blk * kTileM + tid;
  const bool valid = ok && t < T_tok;
  if (valid) {
    for (int k = 0; k < K; ++k) atomicOr(&masks[warp * E + topk_idx[t * K + k]], 1u << lane);
  }
  __syncthreads();
  for (int e = tid; e < E; e += 128) {
    int run = 0;
    for (int w = 0; w < 4; ++w) { wbase[w * E + e] = run; run += __popc(masks[w * E + e]); }
  }
  __syncthreads();
  const uint32_t lt = (1u << lane) - 1u;
  for (int k = 0; k < K; ++k) {
    int d = -1, row = -1;
    if (valid) {
      const int e = topk_idx[t * K + k];
      if (base_s[e] >= 0) {
        d = e / El;
        row = base_s[e] + excl[blk * E + e] + wbase[warp * E + e] + __popc(masks[warp * E + e] & lt);
      }
    }
    if (t < T_tok && first) {  // -1 also when the wait gave up: the combine then skips the row
      a.dest_rank[t * K + k] = d;
      a.dest_row[t * K + k] = row;
      if (a.push && d >= 0) {
        // the row's return address in the owner's memory: where its expert output goes
        const int64_t j = t * K + k;
        reinterpret_cast<int64_t*>(a.peer_base[d] + a.ret_off)[row] =
            (static_cast<int64_t>(a.epoch) << 32) | (static_cast<int64_t>(a.me) << 24) | j;
      }
    }
    slot_rank[tid * K + k] = d;
    slot_row[tid * K + k] = row;
  }
  __syncthreads();
  // copy: each warp reads a token row once and stores it to its K owners over NVLink
  constexpr int V = Vec16<T>::N;
  const int nvec = static_cast<int>(a.H / V);
  const int64_t left = T_tok - blk * kTileM;
  const int ntok = ok ? static_cast<int>(left < kTileM ? (left > 0 ? left : 0) : kTileM) : 0;
  for (int i = warp + 4 * static_cast<int>(blockIdx.y); i < ntok;
       i += 4 * static_cast<int>(gridDim.y)) {
    const T* src = x + (blk * kTileM + i) * a.H;
    for (int v0 = 0; v0 < nvec; v0 += 32 * 4) {
      uint4 buf[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int v = v0 + u * 32 + lane;
        if (v < nvec) buf[u] = reinterpret_cast<const uint4*>(src)[v];
      }
      for (int k = 0; k < K; ++k) {
        const int d = slot_rank[i * K + k];
        if (d < 0) continue;
        uint4* dst = reinterpret_cast<uint4*>(a.peer_base[d] + a.recv_off +
                                              static_cast<int64_t>(slot_row[i * K + k]) * a.H * sizeof(T));
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int v = v0 + u * 32 + lane;
          if (v < nvec) dst[v] = buf[u];
        }
      }
    }
  }
  // completion: the last block to finish raises the dispatch flag on every rank
  __threadfence_system();
  __syncthreads();
  if (tid == 0) {
    const int done = atomicAdd(a.block_counter, 1);
    if (done == static_cast<int>(gridDim.x * gridDim.y) - 1) {
      __threadfence_system();
      *a.block_counter = 0;
      for (int d = 0; d < G; ++d) st_release_sys(sig_ptr(a, d, 1, a.me), a.epoch);
    }
  }
}

// one warp per token; the same fixed-order fp32 arithmetic as the single-GPU combine.  KMAX
// bounds top_k at compile time: the K rows of each 16-byte column chunk are loaded (over
// NVLink) before any is summed, so the remote loads are in flight together instead of one
// after another.
template <typename T, int KMAX>
__global__ void __launch_bounds__(256)
p2p_combine_kernel(P2PArgs a, const int32_t* __restrict__ topk_idx, const float* __restrict__ topk_w,
                   int64_t T_tok, T* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (t >= T_tok) return;
  const int K = a.K;
  int ord_e[KMAX];
  const T* ord_y[KMAX];
  float ord_w[KMAX];
  int n = 0;
  for (int k = 0; k < K; ++k) {  // the token's rows sorted by expert id
    const int e = topk_idx[t * K + k];
    const int d = a.dest_rank[t * K + k], r = a.dest_row[t * K + k];
    const float w = topk_w[t * K + k];
    const T* y = (d < 0 || d >= a.G || r < 0 || r >= a.cap_rows)
                     ? nullptr
                     : reinterpret_cast<const T*>(a.peer_base[d] + a.y_off) + static_cast<int64_t>(r) * a.H;
    int j = n++;
    while (j > 0 && ord_e[j - 1] > e) {
      ord_e[j] = ord_e[j - 1]; ord_y[j] = ord_y[j - 1]; ord_w[j] = ord_w[j - 1];
      --j;
    }
    ord_e[j] = e; ord_y[j] = y; ord_w[j] = w;
  }
  constexpr int V = Vec16<T>::N;
  const int nvec = static_cast<int>(a.H / V);
  T* orow = out + t * a.H;
  for (int v = lane; v < nvec; v += 32) {
    uint4 raw[KMAX];
#pragma unroll
    for (int j = 0; j < KMAX; ++j)
      if (j < n && ord_y[j]) raw[j] = reinterpret_cast<const uint4*>(ord_y[j])[v];
    float acc[V];
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] = 0.f;
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
      if (j >= n || !ord_y[j]) continue;
      float f[V];
      load16_to_f(reinterpret_cast<const T*>(&raw[j]), f);
      const float w = ord_w[j];
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(f[i], w));
    }
    store16_from_f(orow + v * V, acc);
  }
}

// push mode: the K rows of every token are already in this rank's return buffer
template <typename T>
__global__ void __launch_bounds__(256)
p2p_combine_local_kernel(P2PArgs a, const int32_t* __restrict__ topk_idx,
                         const float* __restrict__ topk_w, int64_t T_tok, T* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (t >= T_tok) return;
  const int K = a.K;
  int ord_e[32], ord_j[32];
  float ord_w[32];
  int n = 0;
  for (int k = 0; k < K; ++k) {
    const int e = topk_idx[t * K + k];
    const int d = a.dest_rank[t * K + k];
    const int jrow = (d >= 0 && d < a.G && t * K + k < a.back_rows) ? static_cast<int>(t * K + k) : -1;
    const float w = topk_w[t * K + k];
    int j = n++;
    while (j > 0 && ord_e[j - 1] > e) {
      ord_e[j] = ord_e[j - 1]; ord_j[j] = ord_j[j - 1]; ord_w[j] = ord_w[j - 1];
      --j;
    }
    ord_e[j] = e; ord_j[j] = jrow; ord_w[j] = w;
  }
  constexpr int V = Vec16<T>::N;
  const int nvec = static_cast<int>(a.H / V);
  const T* back = reinterpret_cast<const T*>(a.peer_base[a.me] + a.back_off);
  T* orow = out + t * a.H;
  for (int v = lane; v < nvec; v += 32) {
    float acc[V];
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] = 0.f;
    for (int j = 0; j < n; ++j) {
      if (ord_j[j] < 0) continue;
      float f[V];
      load16_to_f(back + static_cast<int64_t>(ord_j[j]) * a.H + v * V, f);
      const float w = ord_w[j];
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(f[i], w));
    }
    store16_from_f(orow + v * V, acc);
  }
}

}  // namespace

cudaError_t launch_p2p_combine_local(int dtype, const P2PArgs& a, const int32_t* topk_idx,
                                     const float* topk_w, int64_t T, void* out, size_t min_smem,
                                     cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (!a.push) return cudaErrorInvalidValue;
  const unsigned grid = static_cast<unsigned>((T + 7) / 8);
  if (dtype == kF32) {
    auto kern = p2p_combine_local_kernel<float>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(min_smem));
    kern<<<grid, 256, min_smem, s>>>(a, topk_idx, topk_w, T, static_cast<float*>(out));
  } else {
    auto kern = p2p_combine_local_kernel<__nv_bfloat16>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(min_smem));
    kern<<<grid, 256, min_smem, s>>>(a, topk_idx, topk_w, T, static_cast<__nv_bfloat16*>(out));
  }
  return cudaGetLastError();
}

cudaError_t launch_p2p_publish(const P2PArgs& a, const int* counts, cudaStream_t s) {
  p2p_publish_kernel<<<1, 256, 0, s>>>(a, counts);
  return cudaGetLastError();
}

cudaError_t launch_p2p_wait(const P2PArgs& a, int which, cudaStream_t s) {
  p2p_wait_kernel<<<1, 32, 0, s>>>(a, which);
  return cudaGetLastError();
}

cudaError_t launch_p2p_signal(const P2PArgs& a, int which, cudaStream_t s) {
  p2p_signal_kernel<<<1, 32, 0, s>>>(a, which);
  return cudaGetLastError();
}

size_t p2p_dispatch_smem(int E, int K, int G) {
  return (8 * static_cast<size_t>(E) + E + static_cast<size_t>(G) * E +
          2 * static_cast<size_t>(kTileM) * K) * 4;
}

cudaError_t launch_p2p_dispatch(int dtype, const P2PArgs& a, const void* x,
                                const int32_t* topk_idx, const int* excl, int64_t T,
                                size_t min_smem, bool spread, cudaStream_t s) {
  const unsigned nblk = static_cast<unsigned>((T + kTileM - 1) / kTileM);
  // copy slices per routing block with `spread`: about 2048 CTAs in all, at most 32 (one per
  // four tokens); else one CTA per routing block
  unsigned slices = (2048u + (nblk > 0 ? nblk : 1u) - 1) / (nblk > 0 ? nblk : 1u);
  if (slices > 32) slices = 32;
  if (!spread) slices = 1;
  const dim3 grid(nblk > 0 ? nblk : 1, slices);
  size_t smem = p2p_dispatch_smem(a.E, a.K, a.G);
  if (smem < min_smem) smem = min_smem;  // see launch_p2p_combine
  if (dtype == kF32) {
    auto kern = p2p_dispatch_kernel<float>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    kern<<<grid, 128, smem, s>>>(a, static_cast<const float*>(x), topk_idx, excl, T);
  } else {
    auto kern = p2p_dispatch_kernel<__nv_bfloat16>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    kern<<<grid, 128, smem, s>>>(a, static_cast<const __nv_bfloat16*>(x), topk_idx, excl, T);
  }
  return cudaGetLastError();
}

// `min_smem` > 0 makes each block claim that much shared memory (unused by the kernel) so
// the transfer kernels cannot share an SM with a GEMM CTA and run only on the SMs the GEMMs
// leave free: the GEMMs keep full speed while the links are busy.
cudaError_t launch_p2p_combine(int dtype, const P2PArgs& a, const int32_t* topk_idx,
                               const float* topk_w, int64_t T, void* out, size_t min_smem,
                               cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (a.K > 32) return cudaErrorInvalidValue;
  const unsigned grid = static_cast<unsigned>((T + 7) / 8);
  auto go = [&](auto kern, auto* o) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(min_smem));
    kern<<<grid, 256, min_smem, s>>>(a, topk_idx, topk_w, T, o);
  };
  if (dtype == kF32) {
    float* o = static_cast<float*>(out);
    if (a.K <= 2) go(p2p_combine_kernel<float, 2>, o);
    else if (a.K <= 4) go(p2p_combine_kernel<float, 4>, o);
    else if (a.K <= 8) go(p2p_combine_kernel<float, 8>, o);
    else go(p2p_combine_kernel<float, 32>, o);
  } else {
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
    if (a.K <= 2) go(p2p_combine_kernel<__nv_bfloat16, 2>, o);
    else if (a.K <= 4) go(p2p_combine_kernel<__nv_bfloat16, 4>, o);
    else if (a.K <= 8) go(p2p_combine_kernel<__nv_bfloat16, 8>, o);
    else go(p2p_combine_kernel<__nv_bfloat16, 32>, o);
  }
  return cudaGetLastError();
}

}  // namespace vmoe
