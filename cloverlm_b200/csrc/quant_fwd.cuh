// Forward NVFP4 quantization (round-to-nearest and four-over-six) and the
// tensor abs-max reduction that feeds it.
//
// Semantics follow quartet2/csrc/round_four_six.cu:24-123 of the reference
// (four_six_fp4_kernel<6,4> / <6>): per 16-element group an E4M3 scale
// s8 = e4m3(absmax * (so / v) / ts) for candidate v in {6, 4} (RNE: {6}),
// codes = e2m1_rn(x / (s8' * ts)) with s8' = (s8 == 0 ? 1 : s8), and the
// candidate with the strictly lower squared error is kept (a tie keeps 6).
// Reciprocals use rcp.approx.ftz at the same points as the reference, so
// codes and scales match its kernels bit for bit, rounding ties included.
//
// Work decomposition: one thread per 16-element group (one 32-byte load), a
// warp covers 512 consecutive elements, so its loads and 8-byte code stores
// are fully coalesced; lane 4q gathers the four scale bytes of its k-tile with
// shuffles and writes them as one 32-bit word of the blocked layout.
#pragma once
#include "common.cuh"

namespace q2b {


__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Abs-max of a group's 16 bf16 values (eight packed words): a tree of packed
// max(|a|, |b|) (the result's sign is the xor of the inputs' and is dropped at
// the end), exact and order-independent like any maximum.
__device__ __forceinline__ uint32_t maxabs_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ float group_absmax16(const uint32_t (&w)[8]) {
  const uint32_t m = maxabs_bf16x2(maxabs_bf16x2(maxabs_bf16x2(w[0], w[1]), maxabs_bf16x2(w[2], w[3])),
                                   maxabs_bf16x2(maxabs_bf16x2(w[4], w[5]), maxabs_bf16x2(w[6], w[7]))) &
                     0x7FFF7FFFu;
  return fmaxf(bf16lo(m), bf16hi(m));
}

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
    t.factor[i] = rcp_approx_ftz(s_round * ts);
    t.descale[i] = s * ts;
  }
}

// ---------------------------------------------------------------------------
// v2: one thread per 16-element group (a 32-byte load), so the group's
// abs-max and squared errors need no shuffles; row/column of the group come
// from a 64-bit multiply-high by a precomputed reciprocal instead of a
// division.  Errors are accumulated on signed values: x - q * descale is, bit
// for bit, +-(|x| - |q| * descale) (q has the sign of x or is zero, and
// rounding is symmetric), so d*d equals the magnitude form the reference uses.
__device__ __forceinline__ void ldg256(const void* p, uint32_t (&r)[8]) {
  asm volatile("ld.global.nc.L1::no_allocate.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "l"(p));
}

__device__ __forceinline__ float quant16(const float (&xs)[16], float gabs, float inv_c,
                                         float inv_ts, const QuantTables& tab, uint2& codes, uint32_t& s8) {
  s8 = cvt_e4m3(gabs * inv_c * inv_ts);
  const float f = tab.factor[s8];
  const float nd = -tab.descale[s8];
  uint32_t h[8];
#pragma unroll
  for (int hw = 0; hw < 2; ++hw) {  // 8 values -> one code word
    float w[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 p = fmul2(make_float2(xs[8 * hw + 2 * k], xs[8 * hw + 2 * k + 1]), make_float2(f, f));
      w[2 * k] = p.x;
      w[2 * k + 1] = p.y;
    }
    uint32_t (&hb)[4] = *reinterpret_cast<uint32_t (*)[4]>(h + 4 * hw);
    cvt_e2m1x8_back(w, hw == 0 ? codes.x : codes.y, hb);
  }
  // signed errors: a code carries its input's sign (or is zero), so x - q*s is
  // exactly +-(|x| - |q|*s) (a fused multiply-add of negated inputs is the
  // negated exact result) and its square is the magnitude form's, bit for bit
  float2 s0 = make_float2(0.f, 0.f), s1 = make_float2(0.f, 0.f);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 q0 = f16x2_to_f32x2(h[k]);
    const float2 d0 = ffma2(q0, make_float2(nd, nd), make_float2(xs[2 * k], xs[2 * k + 1]));
    s0 = ffma2(d0, d0, s0);
    const float2 q1 = f16x2_to_f32x2(h[4 + k]);
    const float2 d1 = ffma2(q1, make_float2(nd, nd), make_float2(xs[8 + 2 * k], xs[8 + 2 * k + 1]));
    s1 = ffma2(d1, d1, s1);
  }
  return (s0.x + s0.y) + (s1.x + s1.y);
}

template <bool kFourSix>
__global__ void __launch_bounds__(256) quant_fwd_v2_kernel(uint2* __restrict__ codes, uint8_t* __restrict__ sf,
                                                           float* __restrict__ ts_out,
                                                           const uint16_t* __restrict__ x,
                                                           const float* __restrict__ amax_ptr, float scale_override,
                                                           uint32_t ngroups, uint32_t gpr, uint64_t gpr_magic) {
  __shared__ QuantTables tab;
  const float amax = *amax_ptr;
  const float inv_scales_max = kFourSix ? 1.f / 256.f : 1.f / 448.f;
  const float one_over_six = 1.f / 6.f;
  const float inv_val_max = scale_override * one_over_six;
  const float ts = (amax == 0.f) ? 1.f : amax * inv_scales_max * inv_val_max;
  if (blockIdx.x == 0 && threadIdx.x == 0) *ts_out = ts;
  fill_quant_tables(tab, ts);
  __syncthreads();

  const float inv_ts = rcp_approx_ftz(ts);
  const float inv6 = (1.f / 6.f) * scale_override;
  const float inv4 = (1.f / 4.f) * scale_override;
  const int lane = threadIdx.x & 31;
  const uint32_t stride = gridDim.x * blockDim.x;
  const uint32_t n_kt = gpr >> 2;
  // whole warps stay in the loop (the scale gather below shuffles across the
  // warp); lanes past the end load nothing and store nothing
  const uint32_t ngroups_up = (ngroups + 31u) & ~31u;
  // the next group's 32 bytes are loaded while this one is quantized
  uint32_t wn[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const uint32_t g0 = blockIdx.x * blockDim.x + threadIdx.x;
  if (g0 < ngroups) ldg256(x + static_cast<uint64_t>(g0) * 16, wn);
  for (uint32_t g = g0; g < ngroups_up; g += stride) {
    const bool valid = g < ngroups;
    uint32_t w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) w[k] = wn[k];
    if (static_cast<uint64_t>(g) + stride < ngroups) ldg256(x + (static_cast<uint64_t>(g) + stride) * 16, wn);
    float xs[16];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      xs[2 * k] = bf16lo(w[k]);
      xs[2 * k + 1] = bf16hi(w[k]);
    }
    const float gabs = group_absmax16(w);
    uint2 c;
    uint32_t s;
    const float e6 = quant16(xs, gabs, inv6, inv_ts, tab, c, s);
    if constexpr (kFourSix) {
      uint2 c4;
      uint32_t s4;
      const float e4 = quant16(xs, gabs, inv4, inv_ts, tab, c4, s4);
      if (e4 < e6) { c = c4; s = s4; }
    }
    if (valid) __stcs(codes + g, c);
    const uint32_t b1 = __shfl_down_sync(0xffffffffu, s, 1);
    const uint32_t b2 = __shfl_down_sync(0xffffffffu, s, 2);
    const uint32_t b3 = __shfl_down_sync(0xffffffffu, s, 3);
    if (valid && (lane & 3) == 0) {
      const uint32_t row = static_cast<uint32_t>(__umul64hi(static_cast<uint64_t>(g), gpr_magic));
      const uint32_t kb = g - row * gpr;
      const uint64_t off = ((static_cast<uint64_t>(row >> 7) * n_kt + (kb >> 2)) << 9) | ((row & 31) << 4) |
                           (((row >> 5) & 3) << 2);
      *reinterpret_cast<uint32_t*>(sf + off) = s | (b1 << 8) | (b2 << 16) | (b3 << 24);
    }
  }
}

// ---------------------------------------------------------------------------
// Small-input path of the inference linear: abs-max, tensor scale and
// four-over-six (or RNE) quantization of x [rows, cols] in ONE launch of a
// single thread-block cluster.  Each CTA reduces the abs-max of its share of
// the groups, the CTAs exchange their maxima through distributed shared
// memory, and every CTA then quantizes its share exactly as
// quant_fwd_v2_kernel does.  Scale words of the padding rows of the last
// 128-row block (rows..ceil(rows/128)*128-1) are written as zero.
constexpr int kRowsClusterCtas = 8;
constexpr int kRowsThreads = 512;

template <bool kFourSix>
__global__ void __launch_bounds__(kRowsThreads) quant_rows_cluster_kernel(
    uint2* __restrict__ codes, uint8_t* __restrict__ sf, float* __restrict__ ts_out, const uint16_t* __restrict__ x,
    float scale_override, uint32_t rows, uint32_t ngroups, uint32_t gpr, uint64_t gpr_magic) {
  __shared__ QuantTables tab;
  __shared__ float red[kRowsThreads / 32];
  __shared__ float cta_max;
  const uint32_t rank = cluster_ctarank();
  const int lane = threadIdx.x & 31;
  const uint32_t stride = kRowsClusterCtas * kRowsThreads;
  const uint32_t first = rank * kRowsThreads + threadIdx.x;

  // phase 1: abs-max of this CTA's groups
  float m = 0.f;
  for (uint32_t g = first; g < ngroups; g += stride) {
    uint32_t w[8];
    ldg256(x + static_cast<uint64_t>(g) * 16, w);
#pragma unroll
    for (int k = 0; k < 8; ++k) m = fmaxf(m, fmaxf(fabsf(bf16lo(w[k])), fabsf(bf16hi(w[k]))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < kRowsThreads / 32; ++k) m = fmaxf(m, red[k]);
    cta_max = m;
  }
  cluster_sync();  // every CTA's cta_max is written
  float amax = 0.f;
#pragma unroll
  for (int r = 0; r < kRowsClusterCtas; ++r) amax = fmaxf(amax, ld_shared_cluster_f32(map_to_rank(smem_u32(&cta_max), r)));
  cluster_sync();  // no CTA leaves (or reuses cta_max) while another still reads it

  // phase 2: quantization, as quant_fwd_v2_kernel
  const float inv_scales_max = kFourSix ? 1.f / 256.f : 1.f / 448.f;
  const float inv_val_max = scale_override * (1.f / 6.f);
  const float ts = (amax == 0.f) ? 1.f : amax * inv_scales_max * inv_val_max;
  if (rank == 0 && threadIdx.x == 0) *ts_out = ts;
  fill_quant_tables(tab, ts);
  __syncthreads();
  const float inv_ts = rcp_approx_ftz(ts);
  const float inv6 = (1.f / 6.f) * scale_override;
  const float inv4 = (1.f / 4.f) * scale_override;
  const uint32_t n_kt = gpr >> 2;
  // whole warps stay in the loop (the scale gather shuffles across the warp)
  const uint32_t ngroups_up = (ngroups + 31u) & ~31u;
  for (uint32_t g = first; g < ngroups_up; g += stride) {
    const bool valid = g < ngroups;
    uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (valid) ldg256(x + static_cast<uint64_t>(g) * 16, w);
    float xs[16];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      xs[2 * k] = bf16lo(w[k]);
      xs[2 * k + 1] = bf16hi(w[k]);
    }
    const float gabs = group_absmax16(w);
    uint2 c;
    uint32_t sc;
    const float e6 = quant16(xs, gabs, inv6, inv_ts, tab, c, sc);
    if constexpr (kFourSix) {
      uint2 c4;
      uint32_t s4;
      const float e4 = quant16(xs, gabs, inv4, inv_ts, tab, c4, s4);
      if (e4 < e6) { c = c4; sc = s4; }
    }
    if (valid) codes[g] = c;
    const uint32_t b1 = __shfl_down_sync(0xffffffffu, sc, 1);
    const uint32_t b2 = __shfl_down_sync(0xffffffffu, sc, 2);
    const uint32_t b3 = __shfl_down_sync(0xffffffffu, sc, 3);
    if (valid && (lane & 3) == 0) {
      const uint32_t row = static_cast<uint32_t>(__umul64hi(static_cast<uint64_t>(g), gpr_magic));
      const uint32_t kb = g - row * gpr;
      const uint64_t off = ((static_cast<uint64_t>(row >> 7) * n_kt + (kb >> 2)) << 9) | ((row & 31) << 4) |
                           (((row >> 5) & 3) << 2);
      *reinterpret_cast<uint32_t*>(sf + off) = sc | (b1 << 8) | (b2 << 16) | (b3 << 24);
    }
  }
  // zero scale words of the padding rows (one 32-bit word = 4 groups of a row)
  const uint32_t rows_pad = (rows + 127) & ~127u;
  const uint32_t pad_words = (rows_pad - rows) * n_kt;
  for (uint32_t i = first; i < pad_words; i += stride) {
    const uint32_t row = rows + i / n_kt, kt = i % n_kt;
    const uint64_t off = ((static_cast<uint64_t>(row >> 7) * n_kt + kt) << 9) | ((row & 31) << 4) |
                         (((row >> 5) & 3) << 2);
    *reinterpret_cast<uint32_t*>(sf + off) = 0u;
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

// y = relu(a)^2 (bf16, from the fp32 square of the bf16 input) and
// *amax = max |y| in one pass: the MLP activation feeding a Quartet layer
// together with the abs-max that layer's quantizer needs.  *amax must be zero
// on entry.  a and y 16-byte aligned; the tail (n % 8) runs in block 0.
__global__ void __launch_bounds__(256) relu2_abs_max_kernel(uint4* __restrict__ y, unsigned* __restrict__ amax,
                                                            const uint4* __restrict__ a, int64_t nvec,
                                                            uint16_t* __restrict__ y_tail,
                                                            const uint16_t* __restrict__ a_tail, int64_t ntail) {
  float m = 0.f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const uint4 v = __ldcs(a + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float lo = fmaxf(bf16lo(w[k]), 0.f), hi = fmaxf(bf16hi(w[k]), 0.f);
      o[k] = pack_bf16x2(lo * lo, hi * hi);
      m = fmaxf(m, fmaxf(bf16lo(o[k]), bf16hi(o[k])));
    }
    y[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if (blockIdx.x == 0) {
    for (int64_t t = threadIdx.x; t < ntail; t += blockDim.x) {
      const float r = fmaxf(__uint_as_float(static_cast<uint32_t>(a_tail[t]) << 16), 0.f);
      const uint32_t b = pack_bf16x2(r * r, 0.f) & 0xFFFFu;
      y_tail[t] = static_cast<uint16_t>(b);
      m = fmaxf(m, __uint_as_float(b << 16));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < (blockDim.x >> 5); ++k) m = fmaxf(m, red[k]);
    atomicMax(amax, __float_as_uint(m));
  }
}

}  // namespace q2b
