// Fused AdamW step with the post-step weight abs-max.
//
// The reference trains its hidden weights with torch.optim.AdamW(fused=True)
// (src/models/parametrizations.py:311) and, after every step, re-reads each
// Quartet weight to cache max|w| for the next forward
// (quartet2/python/quartet2/linear.py:259-270, register_optimizer_hook).
// Here one pass does both: it updates the fp32 weight and moments and
// reduces max|bf16(w_new)| (the value the hook computes), optionally writing the
// bf16 copy of the new weight that the forward quantizes.
//
// Update (AdamW with decoupled weight decay, in the operation order of
// torch's fused AdamW):
//   w -= lr*wd * w
//   m  = beta1*m + (1-beta1)*g
//   v  = beta2*v + (1-beta2)*g*g
//   w -= (lr / (1 - beta1^t)) * m / (sqrt(v) / sqrt(1 - beta2^t) + eps)
#pragma once
#include "common.cuh"

namespace q2b {

struct AdamParams {
  float lr_wd;        // lr * weight_decay
  float beta1, one_minus_beta1;
  float beta2, one_minus_beta2;
  float step_size;    // lr / (1 - beta1^t)
  float bc2_sqrt;     // sqrt(1 - beta2^t)
  float eps;
};

__device__ __forceinline__ float adamw_one(float& w, float& m, float& v, float g, const AdamParams& a) {
  w -= a.lr_wd * w;
  m = a.beta1 * m + a.one_minus_beta1 * g;
  v = a.beta2 * v + a.one_minus_beta2 * g * g;
  const float denom = sqrtf(v) / a.bc2_sqrt + a.eps;
  w -= a.step_size * m / denom;
  // |bf16(w)|: the forward quantizes the bf16 copy of the weight, and the
  // reference's hook takes the abs-max of that copy (bf16 rounding is
  // monotone, so this equals bf16(max |w|))
  return fabsf(__bfloat162float(__float2bfloat16_rn(w)));
}

// grad is fp32 (kGradBf16 = false) or bf16.  wb (optional) receives bf16(w).
// amax (optional) accumulates the fp32 bits of max|bf16(w)| with atomicMax; the
// caller zeroes it first.  Vector path for 16-byte aligned tensors (four
// elements per thread per iteration), scalar path otherwise.
template <bool kGradBf16>
__global__ void __launch_bounds__(256) adamw_amax_kernel(float* __restrict__ w, float* __restrict__ m,
                                                         float* __restrict__ v, const void* __restrict__ grad,
                                                         int64_t n, AdamParams a, __nv_bfloat16* __restrict__ wb,
                                                         unsigned* __restrict__ amax, int vec) {
  float mx = 0.f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  int64_t done = 0;
  if (vec) {
    const int64_t n4 = n / 4;
    for (int64_t i = tid; i < n4; i += stride) {
      float4 wv = reinterpret_cast<float4*>(w)[i];
      float4 mv = reinterpret_cast<float4*>(m)[i];
      float4 vv = reinterpret_cast<float4*>(v)[i];
      float g0, g1, g2, g3;
      if constexpr (kGradBf16) {
        const uint2 gb = reinterpret_cast<const uint2*>(grad)[i];
        g0 = __uint_as_float(gb.x << 16);
        g1 = __uint_as_float(gb.x & 0xFFFF0000u);
        g2 = __uint_as_float(gb.y << 16);
        g3 = __uint_as_float(gb.y & 0xFFFF0000u);
      } else {
        const float4 gf = reinterpret_cast<const float4*>(grad)[i];
        g0 = gf.x; g1 = gf.y; g2 = gf.z; g3 = gf.w;
      }
      mx = fmaxf(mx, adamw_one(wv.x, mv.x, vv.x, g0, a));
      mx = fmaxf(mx, adamw_one(wv.y, mv.y, vv.y, g1, a));
      mx = fmaxf(mx, adamw_one(wv.z, mv.z, vv.z, g2, a));
      mx = fmaxf(mx, adamw_one(wv.w, mv.w, vv.w, g3, a));
      reinterpret_cast<float4*>(w)[i] = wv;
      reinterpret_cast<float4*>(m)[i] = mv;
      reinterpret_cast<float4*>(v)[i] = vv;
      if (wb != nullptr)
        reinterpret_cast<uint2*>(wb)[i] = make_uint2(pack_bf16x2(wv.x, wv.y), pack_bf16x2(wv.z, wv.w));
    }
    done = n4 * 4;
  }
  for (int64_t i = done + tid; i < n; i += stride) {
    float g;
    if constexpr (kGradBf16)
      g = __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(grad)[i]) << 16);
    else
      g = reinterpret_cast<const float*>(grad)[i];
    float wi = w[i], mi = m[i], vi = v[i];
    mx = fmaxf(mx, adamw_one(wi, mi, vi, g, a));
    w[i] = wi;
    m[i] = mi;
    v[i] = vi;
    if (wb != nullptr) wb[i] = __float2bfloat16_rn(wi);
  }
  if (amax == nullptr) return;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < (blockDim.x >> 5); ++k) mx = fmaxf(mx, red[k]);
    atomicMax(amax, __float_as_uint(mx));
  }
}

}  // namespace q2b
