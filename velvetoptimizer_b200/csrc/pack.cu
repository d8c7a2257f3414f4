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

}  // namespace

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
