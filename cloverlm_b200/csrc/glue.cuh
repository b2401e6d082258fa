// The elementwise operations between the Quartet-II linears of a CloverLM
// block (src/models/transformer.py:338-397, src/models/mlp.py:113-118), each
// fused into one HBM pass:
//
//  * rope_norm_fwd / rope_norm_bwd: rotary position embedding of a query or
//    key head vector (transformer.py:39-74, base 1024, interleaved pairs),
//    the sphere norm after it (mlp.py:5-6, F.normalize, eps 1e-12) and, for
//    queries, the learned per-head attention scale (transformer.py:307-310,
//    177-185: Q = scale * Q with softmax scale 1);
//  * add_rmsnorm_amax / rmsnorm_bwd: the post-sublayer RMSNorm with learned
//    weight and the residual add (transformer.py:380-395), emitting the fp32
//    residual, its bf16 copy and the abs-max of that copy, so the next
//    Quartet layer quantizes without another pass over its input;
//  * relu2_bwd: the gradient of the MLP activation relu(a)^2 (mlp.py:34-38).
//
// All tensors are contiguous; bf16 vectors are read and written 16 bytes at
// a time.
#pragma once
#include "common.cuh"

namespace q2b {

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float bf_round(float v) { return __uint_as_float(pack_bf16x2(v, 0.f) << 16); }

// ---------------------------------------------------------------- RoPE + norm
// One 16-lane half warp per 128-element head vector, 8 elements (4 rotation
// pairs) per lane.  x: bf16 [rows, H, 128], row r at position r % seq;
// cs: (cos, sin) fp32 [seq, 64].  out = scale[h] * n / max(|n|, 1e-12) with
// n = bf16(rope(x)) (the reference rounds the rotated vector to the input's
// dtype before normalizing); norm_out[r, h] = max(|n|, 1e-12).
constexpr int kRopeThreads = 256;

__global__ void __launch_bounds__(kRopeThreads) rope_norm_fwd_kernel(
    uint4* __restrict__ out, float* __restrict__ norm_out, const uint4* __restrict__ x,
    const float2* __restrict__ cs, const float* __restrict__ scale, int64_t nvec, int H, int seq) {
  const int lane = threadIdx.x & 15;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * (kRopeThreads / 16);
  for (int64_t v0 = static_cast<int64_t>(blockIdx.x) * (kRopeThreads / 16); v0 < nvec; v0 += stride) {
    const int64_t v = v0 + (threadIdx.x >> 4);
    const bool ok = v < nvec;
    uint4 w = make_uint4(0, 0, 0, 0);
    if (ok) w = __ldcs(x + v * 16 + lane);
    // head vectors stay below 2^31 (the launchers check): 32-bit division, not a 64-bit one
    const uint32_t row = static_cast<uint32_t>(v) / static_cast<uint32_t>(H);
    const int h = static_cast<int>(v - row * H);
    const int pos = static_cast<int>(row % static_cast<uint32_t>(seq));
    const uint32_t win[4] = {w.x, w.y, w.z, w.w};
    float y[8];
    float ss = 0.f;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float xe = bf_lo(win[p]), xo = bf_hi(win[p]);
      const float2 c = ok ? cs[pos * 64 + lane * 4 + p] : make_float2(0.f, 0.f);
      // Y = X*cos + X_*sin with X_ = (-x_odd, x_even): two products, then the sum
      y[2 * p] = bf_round(__fadd_rn(__fmul_rn(xe, c.x), __fmul_rn(-xo, c.y)));
      y[2 * p + 1] = bf_round(__fadd_rn(__fmul_rn(xo, c.x), __fmul_rn(xe, c.y)));
      ss = fmaf(y[2 * p], y[2 * p], ss);
      ss = fmaf(y[2 * p + 1], y[2 * p + 1], ss);
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float d = fmaxf(sqrtf(ss), 1e-12f);
    const float s = (scale != nullptr && ok) ? scale[h] : 1.f;
    // one IEEE reciprocal per vector instead of eight divisions: n * (1/d) is within an
    // ulp of n / d before the bf16 rounding of the output
    const float inv_d = __frcp_rn(d);
    uint32_t o4[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) o4[p] = pack_bf16x2(y[2 * p] * inv_d * s, y[2 * p + 1] * inv_d * s);
    if (ok) {
      out[v * 16 + lane] = make_uint4(o4[0], o4[1], o4[2], o4[3]);
      if (lane == 0) norm_out[v] = d;
    }
  }
}

// Gradient of rope_norm_fwd.  With n̂ = out / s (the normalized vector):
//   dscale[h] += sum(dout * n̂)            (over every row of head h)
//   dn = (s*dout - n̂ * (n̂ . s*dout)) / d  (normalization)
//   dx = rope^T(dn)                        (the rotation transposed)
// The bf16 rounding between rotation and norm passes the gradient through.
// Per-head partial sums collect in shared memory and reach dscale with one
// atomic per head and block.
__global__ void __launch_bounds__(kRopeThreads) rope_norm_bwd_kernel(
    uint4* __restrict__ dx, float* __restrict__ dscale, const uint4* __restrict__ dout,
    const uint4* __restrict__ out, const float* __restrict__ norm, const float2* __restrict__ cs,
    const float* __restrict__ scale, int64_t nvec, int H, int seq) {
  __shared__ float acc[64];
  for (int i = threadIdx.x; i < 64; i += kRopeThreads) acc[i] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 15;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * (kRopeThreads / 16);
  // the next head vector's gradient and output are loaded while this one is processed
  const int64_t first = static_cast<int64_t>(blockIdx.x) * (kRopeThreads / 16) + (threadIdx.x >> 4);
  uint4 gn = make_uint4(0, 0, 0, 0), on = make_uint4(0, 0, 0, 0);
  if (first < nvec) {
    gn = __ldcs(dout + first * 16 + lane);
    on = __ldcs(out + first * 16 + lane);
  }
  for (int64_t v0 = static_cast<int64_t>(blockIdx.x) * (kRopeThreads / 16); v0 < nvec; v0 += stride) {
    const int64_t v = v0 + (threadIdx.x >> 4);
    const bool ok = v < nvec;
    const uint4 g = gn, o = on;
    if (v + stride < nvec) {
      gn = __ldcs(dout + (v + stride) * 16 + lane);
      on = __ldcs(out + (v + stride) * 16 + lane);
    }
    // head vectors stay below 2^31 (the launchers check): 32-bit division, not a 64-bit one
    const uint32_t row = static_cast<uint32_t>(v) / static_cast<uint32_t>(H);
    const int h = static_cast<int>(v - row * H);
    const int pos = static_cast<int>(row % static_cast<uint32_t>(seq));
    const float s = (scale != nullptr && ok) ? scale[h] : 1.f;
    const float inv_s = 1.f / s;
    const float d = ok ? norm[v] : 1.f;
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, ow[4] = {o.x, o.y, o.z, o.w};
    float n[8], dn[8];
    float dot = 0.f, ds = 0.f;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      n[2 * p] = bf_lo(ow[p]) * inv_s;
      n[2 * p + 1] = bf_hi(ow[p]) * inv_s;
      const float g0 = bf_lo(gw[p]), g1 = bf_hi(gw[p]);
      ds = fmaf(g0, n[2 * p], fmaf(g1, n[2 * p + 1], ds));
      dn[2 * p] = g0 * s;
      dn[2 * p + 1] = g1 * s;
      dot = fmaf(n[2 * p], dn[2 * p], fmaf(n[2 * p + 1], dn[2 * p + 1], dot));
    }
#pragma unroll
    for (int sh = 8; sh > 0; sh >>= 1) {
      dot += __shfl_xor_sync(0xffffffffu, dot, sh);
      ds += __shfl_xor_sync(0xffffffffu, ds, sh);
    }
    const float inv_d = 1.f / d;
    uint32_t r4[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float dy0 = (dn[2 * p] - n[2 * p] * dot) * inv_d;
      const float dy1 = (dn[2 * p + 1] - n[2 * p + 1] * dot) * inv_d;
      const float2 c = ok ? cs[pos * 64 + lane * 4 + p] : make_float2(0.f, 0.f);
      r4[p] = pack_bf16x2(dy0 * c.x + dy1 * c.y, dy1 * c.x - dy0 * c.y);
    }
    if (ok) {
      dx[v * 16 + lane] = make_uint4(r4[0], r4[1], r4[2], r4[3]);
      if (dscale != nullptr && lane == 0) atomicAdd(&acc[h], ds);
    }
  }
  if (dscale == nullptr) return;
  __syncthreads();
  for (int i = threadIdx.x; i < H; i += kRopeThreads)
    if (acc[i] != 0.f) atomicAdd(dscale + i, acc[i]);
}

// ---------------------------------------------------------- residual RMSNorm
// One block per row (grid-stride), d a multiple of 8.
//   rstd = 1 / sqrt(mean(y^2) + eps)
//   x_out = x + (y * rstd) * w        (fp32 residual stream)
//   xb_out = bf16(x_out); *amax = max |xb_out| (atomicMax on the fp32 bits;
//   the host zeroes it first)
constexpr int kNormThreads = 256;
constexpr int kNormMaxVecs = 2;  // d <= 2 * 8 * 256 = 4096

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int k = 0; k < kNormThreads / 32; ++k) t += red[k];
  return t;
}

__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_amax_kernel(
    float* __restrict__ x_out, uint4* __restrict__ xb_out, float* __restrict__ rstd_out,
    unsigned* __restrict__ amax, const float* __restrict__ x, const uint4* __restrict__ y,
    const float* __restrict__ w, int64_t rows, int d, float eps) {
  __shared__ float red[kNormThreads / 32];
  const int nv = d >> 3;
  float m = 0.f;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    uint4 yv[kNormMaxVecs];
    float4 xv[kNormMaxVecs][2];  // the residual's 8 values, loaded before the reduction needs them
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < kNormMaxVecs; ++k) {
      const int c = threadIdx.x + k * kNormThreads;
      yv[k] = make_uint4(0, 0, 0, 0);
      if (c < nv) {
        yv[k] = __ldcs(y + r * nv + c);
        const float4* xp = reinterpret_cast<const float4*>(x + (r * nv + c) * 8);
        xv[k][0] = __ldcs(xp);
        xv[k][1] = __ldcs(xp + 1);
      }
      const uint32_t a[4] = {yv[k].x, yv[k].y, yv[k].z, yv[k].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float lo = bf_lo(a[q]), hi = bf_hi(a[q]);
        ss = fmaf(lo, lo, fmaf(hi, hi, ss));
      }
    }
    const float rstd = 1.f / sqrtf(block_sum(ss, red) / static_cast<float>(d) + eps);
    if (threadIdx.x == 0) rstd_out[r] = rstd;
#pragma unroll
    for (int k = 0; k < kNormMaxVecs; ++k) {
      const int c = threadIdx.x + k * kNormThreads;
      if (c >= nv) continue;
      const float4* wp = reinterpret_cast<const float4*>(w + c * 8);
      const float4 x0 = xv[k][0], x1 = xv[k][1];
      const float4 w0 = wp[0], w1 = wp[1];
      const uint32_t a[4] = {yv[k].x, yv[k].y, yv[k].z, yv[k].w};
      const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
      const float ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      float o[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        o[2 * q] = xs[2 * q] + (bf_lo(a[q]) * rstd) * ws[2 * q];
        o[2 * q + 1] = xs[2 * q + 1] + (bf_hi(a[q]) * rstd) * ws[2 * q + 1];
      }
      float4* op = reinterpret_cast<float4*>(x_out + (r * nv + c) * 8);
      op[0] = make_float4(o[0], o[1], o[2], o[3]);
      op[1] = make_float4(o[4], o[5], o[6], o[7]);
      uint32_t b[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        b[q] = pack_bf16x2(o[2 * q], o[2 * q + 1]);
        m = fmaxf(m, fmaxf(fabsf(bf_lo(b[q])), fabsf(bf_hi(b[q]))));
      }
      xb_out[r * nv + c] = make_uint4(b[0], b[1], b[2], b[3]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < kNormThreads / 32; ++k) m = fmaxf(m, red[k]);
    atomicMax(amax, __float_as_uint(m));
  }
}

// Gradient of add_rmsnorm_amax.  g = g32 (+ gb, the gradient reaching the bf16
// copy, when not null) is the gradient of the block output; then
//   dx = g                                     (fp32, written to dx_out; may be g32)
//   dy = rstd * (g*w - yhat * mean(g*w*yhat))  (bf16), yhat = y * rstd
//   dw_partial[block, :] = sum over the block's rows of g * yhat
__global__ void __launch_bounds__(kNormThreads) rmsnorm_bwd_kernel(
    float* dx_out, uint4* __restrict__ dy_out, float* __restrict__ dw_partial,
    const float* g32, const uint4* __restrict__ gb, const uint4* __restrict__ y,
    const float* __restrict__ rstd_in, const float* __restrict__ w, int64_t rows, int d) {
  __shared__ float red[kNormThreads / 32];
  const int nv = d >> 3;
  float dw[kNormMaxVecs][8];
#pragma unroll
  for (int k = 0; k < kNormMaxVecs; ++k)
#pragma unroll
    for (int q = 0; q < 8; ++q) dw[k][q] = 0.f;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float rstd = rstd_in[r];
    float gv[kNormMaxVecs][8], yh[kNormMaxVecs][8];
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < kNormMaxVecs; ++k) {
      const int c = threadIdx.x + k * kNormThreads;
      if (c >= nv) {
#pragma unroll
        for (int q = 0; q < 8; ++q) gv[k][q] = yh[k][q] = 0.f;
        continue;
      }
      const float4* gp = reinterpret_cast<const float4*>(g32 + (r * nv + c) * 8);
      const float4 g0 = __ldcs(gp), g1 = __ldcs(gp + 1);
      float t[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      if (gb != nullptr) {
        const uint4 b = __ldcs(gb + r * nv + c);
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          t[2 * q] += bf_lo(bw[q]);
          t[2 * q + 1] += bf_hi(bw[q]);
        }
      }
      const uint4 yv = __ldcs(y + r * nv + c);
      const uint32_t yw[4] = {yv.x, yv.y, yv.z, yv.w};
      const float4* wp = reinterpret_cast<const float4*>(w + c * 8);
      const float4 w0 = wp[0], w1 = wp[1];
      const float ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        gv[k][q] = t[q];
        yh[k][q] = ((q & 1) ? bf_hi(yw[q >> 1]) : bf_lo(yw[q >> 1])) * rstd;
        dot = fmaf(t[q] * ws[q], yh[k][q], dot);
      }
      float4* xo = reinterpret_cast<float4*>(dx_out + (r * nv + c) * 8);
      xo[0] = make_float4(t[0], t[1], t[2], t[3]);
      xo[1] = make_float4(t[4], t[5], t[6], t[7]);
    }
    const float mean = block_sum(dot, red) / static_cast<float>(d);
#pragma unroll
    for (int k = 0; k < kNormMaxVecs; ++k) {
      const int c = threadIdx.x + k * kNormThreads;
      if (c >= nv) continue;
      const float4* wp = reinterpret_cast<const float4*>(w + c * 8);
      const float4 w0 = wp[0], w1 = wp[1];
      const float ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float a = rstd * (gv[k][2 * q] * ws[2 * q] - yh[k][2 * q] * mean);
        const float b = rstd * (gv[k][2 * q + 1] * ws[2 * q + 1] - yh[k][2 * q + 1] * mean);
        o[q] = pack_bf16x2(a, b);
        dw[k][2 * q] = fmaf(gv[k][2 * q], yh[k][2 * q], dw[k][2 * q]);
        dw[k][2 * q + 1] = fmaf(gv[k][2 * q + 1], yh[k][2 * q + 1], dw[k][2 * q + 1]);
      }
      dy_out[r * nv + c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
#pragma unroll
  for (int k = 0; k < kNormMaxVecs; ++k) {
    const int c = threadIdx.x + k * kNormThreads;
    if (c >= nv) continue;
    float4* p = reinterpret_cast<float4*>(dw_partial + static_cast<int64_t>(blockIdx.x) * d + c * 8);
    p[0] = make_float4(dw[k][0], dw[k][1], dw[k][2], dw[k][3]);
    p[1] = make_float4(dw[k][4], dw[k][5], dw[k][6], dw[k][7]);
  }
}

// ---------------------------------------------------------------- ReLU^2 grad
// da = bf16(2 * relu(a) * g) for n bf16 values (n a multiple of 8); da may be g.
__global__ void __launch_bounds__(256) relu2_bwd_kernel(uint4* da, const uint4* __restrict__ a, const uint4* g,
                                                        int64_t nvec) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const uint4 av = __ldcs(a + i), gv = __ldcs(g + i);
    const uint32_t aw[4] = {av.x, av.y, av.z, av.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      o[k] = pack_bf16x2(2.f * fmaxf(bf_lo(aw[k]), 0.f) * bf_lo(gw[k]),
                         2.f * fmaxf(bf_hi(aw[k]), 0.f) * bf_hi(gw[k]));
    da[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ------------------------------------------------- softmax cross-entropy rows
// One CTA per row of bf16 logits [rows, V] (V a multiple of 8): an online
// max / sum-of-exponentials pass gives lse = max + log(sum exp(x - max)), then
// row_loss[r] = lse - x[t] and, in place, the gradient of the mean loss
// bf16((exp(x - lse) - [j == t]) * inv_n) -- F.cross_entropy of the reference's
// get_loss (src/data/utils_data.py:293-318) and its backward, for one chunk of
// rows of the tied head, with one read and one write of the logits.
constexpr int kXentThreads = 256;

// (m, s) <- the running max and sum of exp(x - max) of the union of two parts
__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  if (m2 > m) { s = s * expf(m - m2) + s2; m = m2; } else if (m2 != -INFINITY) { s += s2 * expf(m2 - m); }
}

__global__ void __launch_bounds__(kXentThreads) softmax_xent_kernel(uint4* logits, float* __restrict__ row_loss,
                                                                    const int64_t* __restrict__ targets, float inv_n,
                                                                    int64_t V) {
  __shared__ float red_m[kXentThreads / 32], red_s[kXentThreads / 32];
  __shared__ float lse_sh;
  const int64_t row = blockIdx.x;
  uint4* x = logits + row * (V / 8);
  const int64_t nv = V / 8;
  float m = -INFINITY, s = 0.f;
  for (int64_t i = threadIdx.x; i < nv; i += kXentThreads) {
    const uint4 v = x[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    float lm = -INFINITY;
#pragma unroll
    for (int k = 0; k < 4; ++k) lm = fmaxf(lm, fmaxf(bf_lo(w[k]), bf_hi(w[k])));
    float ls = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) ls += expf(bf_lo(w[k]) - lm) + expf(bf_hi(w[k]) - lm);
    online_merge(m, s, lm, ls);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { red_m[warp] = m; red_s[warp] = s; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = red_m[0], S = red_s[0];
    for (int k = 1; k < kXentThreads / 32; ++k) online_merge(M, S, red_m[k], red_s[k]);
    const float lse = M + logf(S);
    lse_sh = lse;
    const int64_t t = targets[row];
    const uint16_t tb = reinterpret_cast<const uint16_t*>(x)[t];
    row_loss[row] = lse - __uint_as_float(static_cast<uint32_t>(tb) << 16);
  }
  __syncthreads();
  const float lse = lse_sh;
  const int64_t t = targets[row];
  for (int64_t i = threadIdx.x; i < nv; i += kXentThreads) {
    const uint4 v = x[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float p0 = expf(bf_lo(w[k]) - lse), p1 = expf(bf_hi(w[k]) - lse);
      const int64_t j = i * 8 + 2 * k;
      if (j == t) p0 -= 1.f;
      if (j + 1 == t) p1 -= 1.f;
      o[k] = pack_bf16x2(p0 * inv_n, p1 * inv_n);
    }
    x[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace q2b
