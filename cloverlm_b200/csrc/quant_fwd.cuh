// Forward NVFP4 quantization (round-to-nearest and four-over-six) and the
// tensor abs-max reduction that feeds it.
//
// Semantics follow quartet2/csrc/round_four_six.cu:24-123 of the reference
// (four_six_fp4_kernel<6,4> / <6>): per 16-element group an E4M3 scale
// s8 = e4m3(absmax * (so / v) / ts) for candidate v in {6, 4} (RNE: {6}),
// codes = e2m1_rn(x / (s8' * ts)) with s8' = (s8 == 0 ? 1 : s8), and the
// candidate with the strictly lower squared error is kept (a tie keeps 6).
// Reciprocals are IEEE-rounded (the reference uses rcp.approx).
//
// Work decomposition: one thread per 8 consecutive bf16 (one 16-byte load);
// lane pairs (2j, 2j+1) hold one 16-element group.  A warp covers 256
// consecutive elements, so its loads and code stores are fully coalesced;
// lane 8q gathers the four scale bytes of its k-tile with shuffles and writes
// them as one 32-bit word of the blocked layout.  Every thread keeps kUnroll
// independent 16-byte loads in flight.
#pragma once
#include "common.cuh"

namespace q2b {

constexpr int kQuantThreads = 256;
constexpr int kQuantUnroll = 4;

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Per-tensor lookup tables indexed by the E4M3 scale byte (0..127):
//   factor[s8]  = 1 / (s8' * ts)   (s8' = 1 when s8 == 0)
//   descale[s8] = e4m3(s8) * ts    (0 stays 0)
struct QuantTables {
  float factor[128];
  float descale[128];
};

__device__ __forceinline__ void fill_quant_tables(QuantTables& t, float ts) {
  for (int i = threadIdx.x; i < 128; i += blockDim.x) {
    float s = e4m3_to_f32(static_cast<uint32_t>(i));
    float s_round = (s == 0.f) ? 1.f : s;
    t.factor[i] = rcp_rn(s_round * ts);
    t.descale[i] = s * ts;
  }
}

// Quantize my 8 values with one candidate; returns the group's squared error
// (both lanes of the pair get the same value).
__device__ __forceinline__ float quant_candidate(const float (&x)[8], float gabs, float inv_val_so, float inv_ts,
                                                 const QuantTables& tab, uint32_t& codes, uint32_t& s8) {
  const float s_group = gabs * inv_val_so;
  s8 = cvt_e4m3(s_group * inv_ts);
  const float f = tab.factor[s8];
  codes = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float2 w = fmul2(make_float2(x[2 * k], x[2 * k + 1]), make_float2(f, f));
    codes |= cvt_e2m1x2(w.x, w.y) << (8 * k);
  }
  const float nd = -tab.descale[s8];
  float2 sum = make_float2(0.f, 0.f);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float2 dq = f16x2_to_f32x2(e2m1x2_to_f16x2((codes >> (8 * k)) & 0xFFu));
    float2 d = ffma2(dq, make_float2(nd, nd), make_float2(x[2 * k], x[2 * k + 1]));
    sum = ffma2(d, d, sum);
  }
  const float local = sum.x + sum.y;
  return local + __shfl_xor_sync(0xffffffffu, local, 1);
}

template <bool kFourSix>
__global__ void __launch_bounds__(kQuantThreads) quant_fwd_kernel(uint32_t* __restrict__ codes,
                                                                  uint8_t* __restrict__ sf,
                                                                  float* __restrict__ ts_out,
                                                                  const uint4* __restrict__ x,
                                                                  const float* __restrict__ amax_ptr,
                                                                  float scale_override, int64_t nvecs,
                                                                  int64_t groups_per_row) {
  __shared__ QuantTables tab;
  const float amax = *amax_ptr;
  const float inv_scales_max = kFourSix ? 1.f / 256.f : 1.f / 448.f;
  const float one_over_six = 1.f / 6.f;
  const float inv_val_max = scale_override * one_over_six;
  const float ts = (amax == 0.f) ? 1.f : amax * inv_scales_max * inv_val_max;
  if (blockIdx.x == 0 && threadIdx.x == 0) *ts_out = ts;
  fill_quant_tables(tab, ts);
  __syncthreads();

  const float inv_ts = rcp_rn(ts);
  const float inv6 = (1.f / 6.f) * scale_override;
  const float inv4 = (1.f / 4.f) * scale_override;
  const int lane = threadIdx.x & 31;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t n_ktiles = groups_per_row >> 2;

  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; base < nvecs;
       base += stride * kQuantUnroll) {
    uint4 v[kQuantUnroll];
#pragma unroll
    for (int u = 0; u < kQuantUnroll; ++u) {
      const int64_t idx = base + u * stride;
      if (idx < nvecs) v[u] = __ldcs(x + idx);
    }
#pragma unroll
    for (int u = 0; u < kQuantUnroll; ++u) {
      const int64_t idx = base + u * stride;
      if (idx >= nvecs) break;  // warp-uniform: nvecs is a multiple of 32
      float xv[8] = {bf16lo(v[u].x), bf16hi(v[u].x), bf16lo(v[u].y), bf16hi(v[u].y),
                     bf16lo(v[u].z), bf16hi(v[u].z), bf16lo(v[u].w), bf16hi(v[u].w)};
      float a = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) a = fmaxf(a, fabsf(xv[k]));
      const float gabs = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));

      uint32_t c6, s6;
      const float e6 = quant_candidate(xv, gabs, inv6, inv_ts, tab, c6, s6);
      uint32_t c = c6, s = s6;
      if constexpr (kFourSix) {
        uint32_t c4, s4;
        const float e4 = quant_candidate(xv, gabs, inv4, inv_ts, tab, c4, s4);
        if (e4 < e6) { c = c4; s = s4; }
      }
      __stcs(codes + idx, c);
      // gather the scale bytes of groups 4q..4q+3 (lanes 8q, 8q+2, 8q+4, 8q+6)
      const uint32_t b1 = __shfl_down_sync(0xffffffffu, s, 2);
      const uint32_t b2 = __shfl_down_sync(0xffffffffu, s, 4);
      const uint32_t b3 = __shfl_down_sync(0xffffffffu, s, 6);
      if ((lane & 7) == 0) {
        const int64_t grp = idx >> 1;
        const int64_t row = grp / groups_per_row;
        const int64_t kb = grp - row * groups_per_row;
        const int64_t off = (((row >> 7) * n_ktiles + (kb >> 2)) << 9) | ((row & 31) << 4) | (((row >> 5) & 3) << 2);
        *reinterpret_cast<uint32_t*>(sf + off) = s | (b1 << 8) | (b2 << 16) | (b3 << 24);
      }
    }
  }
}

// |x| max over n bf16 values; *out must be zero on entry (atomicMax on the
// fp32 bit pattern, valid for non-negative values).
__global__ void __launch_bounds__(256) abs_max_kernel(unsigned* __restrict__ out, const uint4* __restrict__ x,
                                                      int64_t nvec, const uint16_t* __restrict__ tail,
                                                      int64_t ntail) {
  float m = 0.f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < nvec; i += 4 * stride) {
    uint4 a = __ldcs(x + i), b = __ldcs(x + i + stride), c = __ldcs(x + i + 2 * stride),
          d = __ldcs(x + i + 3 * stride);
    const uint32_t w[16] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
#pragma unroll
    for (int k = 0; k < 16; ++k) m = fmaxf(m, fmaxf(fabsf(bf16lo(w[k])), fabsf(bf16hi(w[k]))));
  }
  for (; i < nvec; i += stride) {
    uint4 a = __ldcs(x + i);
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) m = fmaxf(m, fmaxf(fabsf(bf16lo(w[k])), fabsf(bf16hi(w[k]))));
  }
  if (blockIdx.x == 0) {
    for (int64_t t = threadIdx.x; t < ntail; t += blockDim.x)
      m = fmaxf(m, fabsf(__uint_as_float(static_cast<uint32_t>(tail[t]) << 16)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < (blockDim.x >> 5); ++k) m = fmaxf(m, red[k]);
    atomicMax(out, __float_as_uint(m));
  }
}

}  // namespace q2b
