// Weight packing at load time: copy the caller's nn.Linear weights into the layouts the
// expert GEMMs read, with zero padding to the tile sizes, and fold the FlyLoRA branch.
//
// FlyLoRALinear.forward is base(x) + s * lora_up(lora_down(x)) (python/vesper/model.py:123-126)
// with biases on both LoRA linears (:116-117).  It is linear in x, so
//   W_eff = W + s * U D,      b_eff = b + s * (U b_D + b_U)
// gives the same function; W_eff is formed in fp32 and rounded once to the storage dtype.
//
// Gate/up interleave (bf16 path): for G = 128, rows [128 j, 128 j + 128) of gate go to
// rows [256 j, 256 j + 128) of the packed matrix and the same rows of up to
// [256 j + 128, 256 j + 256), so one 256-row B tile carries both halves of the GLU.
#include "common.cuh"
#include "kernels.h"

namespace vmoe {
namespace {

__device__ __forceinline__ int64_t map_row(int o, int interleave, int which) {
  if (interleave <= 0) return o;
  return static_cast<int64_t>(o / interleave) * 2 * interleave + which * interleave + o % interleave;
}

template <typename T>
__global__ void pack_weight_kernel(PackArgs a) {
  const T* src = static_cast<const T*>(a.src);
  const T* ld = static_cast<const T*>(a.lora_down);
  const T* lu = static_cast<const T*>(a.lora_up);
  T* dst = static_cast<T*>(a.dst);
  const int opad = a.interleave > 0 ? a.dst_rows_per_expert / 2 : a.dst_rows_per_expert;
  const int64_t total = static_cast<int64_t>(a.E) * opad * a.Kpad;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int k = static_cast<int>(i % a.Kpad);
    const int64_t eo = i / a.Kpad;
    const int o = static_cast<int>(eo % opad);
    const int e = static_cast<int>(eo / opad);
    float v = 0.f;
    if (o < a.O && k < a.Kin) {
      v = Elt<T>::to_f(src[(static_cast<int64_t>(e) * a.O + o) * a.Kin + k]);
      if (ld && lu && a.R > 0) {
        float l = 0.f;
        for (int r = 0; r < a.R; ++r)
          l = fmaf(Elt<T>::to_f(lu[(static_cast<int64_t>(e) * a.O + o) * a.R + r]),
                   Elt<T>::to_f(ld[(static_cast<int64_t>(e) * a.R + r) * a.Kin + k]), l);
        v += a.scaling * l;
      }
    }
    const int64_t row = static_cast<int64_t>(e) * a.dst_rows_per_expert + map_row(o, a.interleave, a.which);
    dst[row * a.Kpad + k] = Elt<T>::from_f(v);
  }
}

template <typename T>
__global__ void pack_bias_kernel(PackBiasArgs a) {
  const T* b = static_cast<const T*>(a.b);
  const T* lu = static_cast<const T*>(a.lora_up);
  const T* bd = static_cast<const T*>(a.lora_down_b);
  const T* bu = static_cast<const T*>(a.lora_up_b);
  const int opad = a.interleave > 0 ? a.dst_per_expert / 2 : a.dst_per_expert;
  const int64_t total = static_cast<int64_t>(a.E) * opad;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int o = static_cast<int>(i % opad);
    const int e = static_cast<int>(i / opad);
    float v = 0.f;
    if (o < a.O) {
      const int64_t eo = static_cast<int64_t>(e) * a.O + o;
      if (b) v = Elt<T>::to_f(b[eo]);
      if (lu && a.R > 0) {
        float l = 0.f;
        if (bd)
          for (int r = 0; r < a.R; ++r)
            l = fmaf(Elt<T>::to_f(lu[eo * a.R + r]), Elt<T>::to_f(bd[static_cast<int64_t>(e) * a.R + r]), l);
        if (bu) l += Elt<T>::to_f(bu[eo]);
        v += a.scaling * l;
      }
    }
    a.dst[static_cast<int64_t>(e) * a.dst_per_expert + map_row(o, a.interleave, a.which)] = v;
  }
}

// One block per expert row e: w_out[e, :] = bf16(W_r[e, :] * ln_w), then in a fixed
// order c[e] = sum_j w_out[e, j] and b_out[e] = b_r[e] + sum_j W_r[e, j] * ln_b[j].
__global__ void __launch_bounds__(256)
fold_router_ln_kernel(const __nv_bfloat16* __restrict__ w_r, const float* __restrict__ b_r,
                      const float* __restrict__ ln_w, const float* __restrict__ ln_b, int H,
                      __nv_bfloat16* __restrict__ w_out, float* __restrict__ b_out,
                      float* __restrict__ c_out) {
  const int e = blockIdx.x, tid = threadIdx.x;
  float c = 0.f, b = 0.f;
  for (int j = tid; j < H; j += blockDim.x) {
    const float w = __bfloat162float(w_r[static_cast<int64_t>(e) * H + j]);
    const __nv_bfloat16 f = __float2bfloat16_rn(w * ln_w[j]);
    w_out[static_cast<int64_t>(e) * H + j] = f;
    c += __bfloat162float(f);
    b = fmaf(w, ln_b[j], b);
  }
  __shared__ float sc[256], sb[256];
  sc[tid] = c;
  sb[tid] = b;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (tid < o) {
      sc[tid] += sc[tid + o];
      sb[tid] += sb[tid + o];
    }
    __syncthreads();
  }
  if (tid == 0) {
    c_out[e] = sc[0];
    b_out[e] = b_r[e] + sb[0];
  }
}

template <typename T>
__global__ void to_f32_kernel(const T* __restrict__ src, int64_t n, float fill, float* __restrict__ dst) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = src ? Elt<T>::to_f(src[i]) : fill;
}

}  // namespace

cudaError_t launch_fold_router_ln(const void* w_r, const float* b_r, const float* ln_w,
                                  const float* ln_b, int E, int H, void* w_out, float* b_out,
                                  float* c_out, cudaStream_t s) {
  fold_router_ln_kernel<<<E, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(w_r), b_r, ln_w, ln_b,
                                          H, static_cast<__nv_bfloat16*>(w_out), b_out, c_out);
  return cudaGetLastError();
}

cudaError_t launch_to_f32(int dtype, const void* src, int64_t n, float fill, float* dst,
                          cudaStream_t s) {
  const unsigned grid = static_cast<unsigned>((n + 255) / 256 > 0 ? (n + 255) / 256 : 1);
  if (dtype == kF32)
    to_f32_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(src), n, fill, dst);
  else
    to_f32_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(src), n,
                                                      fill, dst);
  return cudaGetLastError();
}

cudaError_t launch_pack_weight(const PackArgs& a, cudaStream_t s) {
  if (a.dtype == kF32)
    pack_weight_kernel<float><<<148 * 8, 256, 0, s>>>(a);
  else
    pack_weight_kernel<__nv_bfloat16><<<148 * 8, 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_pack_bias(const PackBiasArgs& a, cudaStream_t s) {
  if (a.dtype == kF32)
    pack_bias_kernel<float><<<148, 256, 0, s>>>(a);
  else
    pack_bias_kernel<__nv_bfloat16><<<148, 256, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace vmoe
