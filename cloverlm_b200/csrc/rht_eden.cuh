// Backward quantizer, pass 1: 128-point rotation on the tensor cores followed
// by EDEN rounding, for bf16 inputs (the output gradient E) and for NVFP4
// inputs (requantization of the saved forward operands).
//
// Reference semantics (paths relative to the reference project root):
//   rotation     quartet2/csrc/rht128_eden.cu:10-137 and rht.py:65-82 -- the
//                effective matrix is swizzle_hadamard(H) built from the 16x128
//                slice by Sylvester extension (or a full 128x128 matrix for
//                quant_had_eden, group_transform_and_eden.cu).
//   EDEN         quartet2/csrc/had128_utils.cuh:155-229 -- per 16 rotated
//                values: m3 = trunc4(absmax / fp4_max), codes = e2m1_rn(v / m3),
//                fixed = m3 * sum(w^2) / sum(w * q) kept as bf16, global max of
//                the bf16 fixed scales by atomicMax.
//   requant      quartet2/csrc/rht128_requant.cu:79-262 -- codes * e4m3 * ts
//                rounded to bf16, transposed, rotated along the old rows.
//
// B200 design.  A CTA owns one SM and walks 128x128 tiles of the input.
//   * bf16 input: one TMA warp streams each tile (two 64-column boxes, 128-byte
//     swizzle) into a 4-stage ring.  NVFP4 input: four producer warps load the
//     codes and scales with vector loads, dequantize and write the bf16 tile
//     in the same swizzled layout.
//   * One MMA warp issues tcgen05.mma kind::f16 M=128 N=128 K=16 x 8 with the
//     rotation matrix (32 KB, built in shared memory once per CTA) as the B
//     operand.  The same shared-memory tile serves as a K-major A operand
//     (rotation along the contiguous dimension: `rows` output) and as an
//     MN-major A operand (rotation along the row dimension: transposed `cols`
//     output), so E and E^T are both produced from ONE read of E.
//   * fp32 results land in TMEM, one buffer per group of four epilogue warps
//     (one warp per TMEM lane quarter, 32 output rows); the groups take tiles
//     in turn (two per orientation for the dual output, four for one
//     orientation).  A thread runs EDEN on whole 16-groups of its row with no
//     shuffles, writing the code bytes and bf16 scales of each chunk.
// Scratch scales are written in the blocked 128x4 layout so the scale pass
// (sr_scales.cuh) is a flat, fully coalesced map.
#pragma once
#include <cfloat>
#include <cuda.h>
#include "common.cuh"

namespace q2b {

enum RhtInput : int { kInBf16 = 0, kInFp4 = 1 };
enum RhtOut : int { kOutRows = 1, kOutCols = 2, kOutBoth = 3 };

struct RhtParams {
  int64_t M, N;                 // input is [M, N] (bf16), or codes [M, N/2] (NVFP4)
  const uint8_t* x_codes;       // NVFP4 input
  const uint8_t* x_sf;          //   blocked scales of the input
  const float* x_ts;            //   input tensor scale
  const uint16_t* h;            // rotation: 16x128 Sylvester slice or full 128x128 (bf16 bits)
  int h_rows;                   // 16 or 128
  uint8_t* codes_r;             // rows output: codes [M, N/2]
  uint16_t* scratch_r;          //   bf16 fixed scales, blocked [M, N/16]
  unsigned* max_r;              //   max of the bf16 fixed scales (fp32 bits)
  uint8_t* codes_c;             // cols output: codes [N, M/2]
  uint16_t* scratch_c;          //   blocked [N, M/16]
  unsigned* max_c;
  float inv_fp4_max;
};


constexpr uint32_t kTileBytes = 128 * 128 * 2;  // one bf16 tile
constexpr uint32_t kHalfBytes = 128 * 128;      // one 64-column half of a tile

template <int kIn, int kOut>
struct RhtCfg {
  static constexpr int kNumOut = (kOut == kOutBoth) ? 2 : 1;
  // NVFP4 input: one loader warp streams the codes (TMA) and scales (bulk
  // copy) of each tile into a shared-memory ring; eight converter warps
  // dequantize them into the bf16 tile.  bf16 input: one TMA warp.
  static constexpr int kConvWarps = (kIn == kInBf16) ? 0 : 8;
  static constexpr int kProdWarps = kConvWarps + 1;
  static constexpr int kLoadWarp = kConvWarps;  // the last producer warp issues the loads
  static constexpr int kMmaWarp = kProdWarps;
  static constexpr int kEpiWarp0 = kProdWarps + 1;
  // TMEM buffers, taken by tiles in turn: two for the dual output (2 x 256
  // columns), four for one orientation (4 x 128).  Groups of 4 epilogue warps
  // (one per TMEM lane quarter, per orientation) take tiles in turn too; the
  // number of groups divides the number of buffers.
  static constexpr int kTmemBufs = (kNumOut == 2) ? 2 : 4;
  static constexpr int kEpiWarps = 16;
  static constexpr int kEpiGroups = kEpiWarps / (4 * kNumOut);
  static_assert(kTmemBufs % kEpiGroups == 0, "groups must divide buffers");
  static constexpr int kThreads = 32 * (kProdWarps + 1 + kEpiWarps);
  static constexpr uint32_t kColsPerBuf = 128 * kNumOut;
  // tcgen05.alloc takes a power of two of at least 32 columns
  static constexpr uint32_t kTmemUsed = kTmemBufs * kColsPerBuf;
  static constexpr uint32_t kTmemCols = kTmemUsed <= 128 ? 128 : (kTmemUsed <= 256 ? 256 : 512);
  static_assert(kTmemUsed <= 512, "TMEM overflow");
  // columns per TMEM load of a one-orientation epilogue warp, double-buffered:
  // 16 keeps the 800-thread requant block within 80 registers a thread
  static constexpr int kLdCols = (kIn == kInFp4) ? 16 : 32;
  // NVFP4 input ring: per stage the tile's codes (128 rows x 64 bytes) and its
  // two 512-byte blocks of scales
  static constexpr int kRawStages = (kIn == kInFp4) ? 4 : 0;
  // bf16 tiles in the ring: three for bf16 input (measured: 4, 5 and 6 stages
  // run slower -- more shared memory in flight and less L1 did not buy bandwidth)
  static constexpr int kStages = (kIn == kInBf16) ? 3 : 4;
  static constexpr uint32_t kRawBytes = 128 * 64 + 1024;
  // shared memory: [H 32K][stages x 32K][raw stages x 9K][barriers]
  static constexpr uint32_t kSmemBytes = 1024 + kTileBytes * (1 + kStages) + kRawStages * kRawBytes + 256;
};

// Byte offset of bf16 element (r, c) of a 128x128 tile stored as two 64-column
// halves of 128 rows x 128 bytes with the 128-byte swizzle (16-byte chunk
// index XOR row % 8).
__device__ __forceinline__ uint32_t tile_off(int r, int c) {
  const int half = c >> 6, q = (c & 63) >> 3;
  return half * kHalfBytes + r * 128 + (((q ^ (r & 7)) << 4) | ((c & 7) << 1));
}

// Build the rotation matrix B[p, c] (p = output index, c = input index) in
// the K-major swizzled layout.
__device__ __forceinline__ void build_rotation(uint8_t* hs, const uint16_t* h, int h_rows, int tid, int nthreads) {
  for (int i = tid; i < 128 * 16; i += nthreads) {
    const int p = i >> 4, q = i & 15;  // q: 16-byte chunk of 8 elements, c = 8q
    uint4 v;
    if (h_rows == 16) {
      const int k = (p >> 6) << 6, l = (p & 63) >> 4, j = p & 15;
      const int R = k + 4 * l + (j & 3) + 16 * (j >> 2);
      v = *reinterpret_cast<const uint4*>(h + (R & 15) * 128 + 8 * q);
      if (__popc((R >> 4) & (q >> 1)) & 1) {
        v.x ^= 0x80008000u; v.y ^= 0x80008000u; v.z ^= 0x80008000u; v.w ^= 0x80008000u;
      }
    } else {
      v = *reinterpret_cast<const uint4*>(h + p * 128 + 8 * q);
    }
    *reinterpret_cast<uint4*>(hs + tile_off(p, 8 * q)) = v;
  }
}

// EDEN on 16 rotated values; writes 8 code bytes (as two words) and returns
// the bf16-rounded fixed scale as fp32.
__device__ __forceinline__ float eden16(const uint32_t* r, float inv_fp4_max, uint32_t& w0, uint32_t& w1,
                                        uint32_t& fixed_bf16) {
  // abs-max with three-input maxima (max is exact and order-independent)
  float v[16];
#pragma unroll
  for (int t = 0; t < 16; ++t) v[t] = fabsf(__uint_as_float(r[t]));
  const float a0 = fmax3(v[0], v[1], v[2]), a1 = fmax3(v[3], v[4], v[5]), a2 = fmax3(v[6], v[7], v[8]);
  const float a3 = fmax3(v[9], v[10], v[11]), a4 = fmax3(v[12], v[13], v[14]);
  const float amax = fmaxf(fmax3(a0, a1, a2), fmax3(a3, a4, v[15]));
  const float scale = amax * inv_fp4_max;
  float m3 = __uint_as_float(__float_as_uint(scale) & 0xFFF80000u);
  float f;
  if (fabsf(m3) < FLT_MIN) { m3 = 0.f; f = 0.f; } else { f = rcp_approx_ftz(m3); }
  float2 xx = make_float2(0.f, 0.f), xy = make_float2(0.f, 0.f);
  uint32_t c[2];
#pragma unroll
  for (int hw = 0; hw < 2; ++hw) {  // 8 values -> one code word
    float w[8];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 p = fmul2(make_float2(__uint_as_float(r[8 * hw + 2 * t]), __uint_as_float(r[8 * hw + 2 * t + 1])),
                             make_float2(f, f));
      w[2 * t] = p.x;
      w[2 * t + 1] = p.y;
    }
    uint32_t h2[4];
    cvt_e2m1x8_back(w, c[hw], h2);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 wv = make_float2(w[2 * t], w[2 * t + 1]);
      const float2 back = f16x2_to_f32x2(h2[t]);
      xx = ffma2(wv, wv, xx);
      xy = ffma2(wv, back, xy);
    }
  }
  const float xx_t = xx.x + xx.y, xy_t = xy.x + xy.y;
  const float corr = (xy_t == 0.f) ? 1.f : xx_t * rcp_approx_ftz(xy_t);
  const float fixed = m3 * corr;
  w0 = c[0];
  w1 = c[1];
  const uint32_t hb = pack_bf16x2(fixed, 0.f) & 0xFFFFu;
  fixed_bf16 = hb;
  return __uint_as_float(hb << 16);
}

#ifdef Q2B_RHT_STATS
// Instrumented builds only: cycle counts of CTA 0 of the last launch's roles (0 producer warp 0:
// waiting for a free stage, 1: converting, 2: loop total; 3 MMA: waiting for a TMEM buffer,
// 4: waiting for a stage, 5: loop total, 6: tiles; 7 epilogue warp 0: waiting for its tile,
// 8: TMEM loads, 9 producer warp 0: waiting for its prefetched codes, 10: epilogue loop total).  Counted in registers, added at exit.
__device__ long long g_rht_stats[12];
#define Q2B_R_T(v) const long long v = clock64();
#define Q2B_R_ADD(i, val) q2b_rs[i] += (val);
#else
#define Q2B_R_T(v)
#define Q2B_R_ADD(i, val)
#endif

template <int kIn, int kOut>
__global__ void __launch_bounds__(RhtCfg<kIn, kOut>::kThreads, 1)
    rht_eden_kernel(const __grid_constant__ CUtensorMap tmap_x, const RhtParams p) {
  using Cfg = RhtCfg<kIn, kOut>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* hs = smem;
  uint8_t* tiles = smem + kTileBytes;
  uint8_t* raw = tiles + Cfg::kStages * kTileBytes;  // NVFP4 input ring
  uint64_t* full = reinterpret_cast<uint64_t*>(raw + Cfg::kRawStages * Cfg::kRawBytes);
  uint64_t* empty = full + Cfg::kStages;
  uint64_t* tfull = empty + Cfg::kStages;
  uint64_t* tempty = tfull + 4;
  uint64_t* drain = tempty + 4;  // the MMA warp's final commit: no MMA in flight at dealloc
  uint64_t* rfull = drain + 1;  // NVFP4 input ring: codes + scales landed
  uint64_t* rempty = rfull + 4;  //   ... and read by every converter thread
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(rempty + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // tile indices stay below 2^31 (the launcher checks), so the per-tile
  // row/column split is a 32-bit division, not a 64-bit software one
  const uint32_t tiles_n = static_cast<uint32_t>(p.N >> 7);
  const int64_t ntiles = (p.M >> 7) * static_cast<int64_t>(tiles_n);
#ifdef Q2B_RHT_STATS
  long long q2b_rs[12] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
#endif

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&full[s], kIn == kInBf16 ? 1 : 32 * Cfg::kConvWarps);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < Cfg::kRawStages; ++s) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], 32 * Cfg::kConvWarps);
    }
    for (int b = 0; b < Cfg::kTmemBufs; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4 * Cfg::kNumOut);  // the group(s) of epilogue warps of this buffer
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (threadIdx.x == 0) prefetch_tmap(&tmap_x);
  if (warp == Cfg::kMmaWarp) {
    tmem_alloc(tmem_holder, Cfg::kTmemCols);
    tmem_relinquish();
  }
  build_rotation(hs, p.h, p.h_rows, threadIdx.x, Cfg::kThreads);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp < Cfg::kProdWarps) {
    // ------------------------------------------------------------ producer
    if constexpr (kIn == kInBf16) {
      if (lane == 0) {
        const uint64_t policy = policy_evict_first();
        int it = 0;
        for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
          const int slot = it % Cfg::kStages;
          const uint32_t ph = (it / Cfg::kStages) & 1;
          if (!mbar_wait(&empty[slot], ph ^ 1, kTimeoutSmemEmpty)) break;
          const uint32_t t32 = static_cast<uint32_t>(t);
          const int tm = static_cast<int>(t32 / tiles_n), tn = static_cast<int>(t32 % tiles_n);
          uint8_t* dst = tiles + slot * kTileBytes;
          mbar_arrive_expect_tx(&full[slot], kTileBytes);
          tma_load_2d_hint(dst, &tmap_x, &full[slot], tn * 128, tm * 128, policy);
          tma_load_2d_hint(dst + kHalfBytes, &tmap_x, &full[slot], tn * 128 + 64, tm * 128, policy);
        }
        // drain: make sure no copy is still landing when the CTA retires
        const int issued = it;
        for (int k = issued > Cfg::kStages ? issued - Cfg::kStages : 0; k < issued; ++k)
          mbar_wait(&full[k % Cfg::kStages], (k / Cfg::kStages) & 1, kTimeoutProducer);
      }
    } else if (warp == Cfg::kLoadWarp) {
      // NVFP4 input, loader: the tile's 128 x 64 code bytes by TMA and its two
      // contiguous 512-byte scale blocks (blocked layout: 128 rows x 4 groups
      // each) by one bulk copy, on one barrier
      if (lane == 0) {
        const int64_t n_kt = p.N >> 6;  // 4-group column blocks of the scales
        int it = 0;
        for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
          const int slot = it % Cfg::kRawStages;
          const uint32_t ph = (it / Cfg::kRawStages) & 1;
          if (!mbar_wait(&rempty[slot], ph ^ 1, kTimeoutSmemEmpty)) break;
          const uint32_t t32 = static_cast<uint32_t>(t);
          const int tm = static_cast<int>(t32 / tiles_n), tn = static_cast<int>(t32 % tiles_n);
          uint8_t* dst = raw + slot * Cfg::kRawBytes;
          mbar_arrive_expect_tx(&rfull[slot], Cfg::kRawBytes);
          tma_load_2d(dst, &tmap_x, &rfull[slot], tn * 64, tm * 128);
          bulk_load(dst + 128 * 64, p.x_sf + ((static_cast<int64_t>(tm) * n_kt + 2 * tn) << 9), 1024, &rfull[slot]);
        }
        const int issued = it;
        for (int k = issued > Cfg::kRawStages ? issued - Cfg::kRawStages : 0; k < issued; ++k)
          mbar_wait(&rfull[k % Cfg::kRawStages], (k / Cfg::kRawStages) & 1, kTimeoutProducer);
      }
    } else {
      // NVFP4 input, converters: each thread dequantizes pairs of 16-element
      // groups of the tile (16 code bytes + 2 scale bytes -> 64 bytes of
      // bf16) from the ring into the swizzled bf16 tile; four consecutive
      // lanes cover one row's 64 code bytes, so a warp reads 512 contiguous
      // bytes.
      const int pt = threadIdx.x;  // 0 .. 32*kConvWarps-1
      const float x_ts = *p.x_ts;
      constexpr int kItems = 128 * 4 / (32 * Cfg::kConvWarps);  // (row, group pair) items per thread
      int it = 0;
      Q2B_R_T(_pl)
      for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
        const int rs = it % Cfg::kRawStages;
        Q2B_R_T(_p0)
        if (!mbar_wait(&rfull[rs], (it / Cfg::kRawStages) & 1, kTimeoutTmaFull)) break;
        Q2B_R_ADD(9, clock64() - _p0)
        const uint8_t* src = raw + rs * Cfg::kRawBytes;
        uint4 qc[kItems];
        uint32_t sc[kItems];
#pragma unroll
        for (int u = 0; u < kItems; ++u) {
          const int item = pt + u * 32 * Cfg::kConvWarps;
          const int r = item >> 2, gp = item & 3;  // row, pair of 16-col groups of the tile
          qc[u] = *reinterpret_cast<const uint4*>(src + r * 64 + gp * 16);
          const int kb = 2 * gp;  // even: the pair's two scale bytes are adjacent
          sc[u] = *reinterpret_cast<const uint16_t*>(src + 128 * 64 + (((kb >> 2) << 9) | ((r & 31) << 4) |
                                                                       (((r >> 5) & 3) << 2) | (kb & 3)));
        }
        mbar_arrive(&rempty[rs]);
        const int slot = it % Cfg::kStages;
        const uint32_t ph = (it / Cfg::kStages) & 1;
        Q2B_R_T(_p1)
        if (!mbar_wait(&empty[slot], ph ^ 1, kTimeoutSmemEmpty)) break;
        Q2B_R_T(_p2)
        Q2B_R_ADD(0, _p2 - _p1)
        uint8_t* dst = tiles + slot * kTileBytes;
#pragma unroll
        for (int u = 0; u < kItems; ++u) {
          const int item = pt + u * 32 * Cfg::kConvWarps;
          const int r = item >> 2, gp = item & 3;
#pragma unroll
          for (int k = 0; k < 2; ++k) {  // the pair's two groups
            const int g = 2 * gp + k;
            const float gs = e4m3_to_f32((sc[u] >> (8 * k)) & 0xFFu) * x_ts;
#pragma unroll
            for (int half = 0; half < 2; ++half) {  // 8 elements -> one 16-byte chunk
              const uint32_t w = k == 0 ? (half ? qc[u].y : qc[u].x) : (half ? qc[u].w : qc[u].z);
              uint32_t o[4], hq[4];
              e2m1x8_to_f16x2(w, hq);
#pragma unroll
              for (int b = 0; b < 4; ++b) {
                const float2 dq = f16x2_to_f32x2(hq[b]);
                const float2 v = fmul2(dq, make_float2(gs, gs));
                o[b] = pack_bf16x2(v.x, v.y);
              }
              *reinterpret_cast<uint4*>(dst + tile_off(r, 16 * g + 8 * half)) = make_uint4(o[0], o[1], o[2], o[3]);
            }
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(&full[slot]);
        Q2B_R_ADD(1, clock64() - _p2)
      }
      Q2B_R_ADD(2, clock64() - _pl)
    }
  } else if (warp == Cfg::kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    const uint32_t id_rows = idesc_bf16(128, 128, false, false);
    const uint32_t id_cols = idesc_bf16(128, 128, true, false);
    const bool lead = lane == 0;
    const uint64_t h_desc0 = smem_desc(smem_u32(hs), 0, 1024, kLayoutSW128);
    const uint64_t rows_desc0 = smem_desc(smem_u32(tiles), 0, 1024, kLayoutSW128);
    const uint64_t cols_desc0 = smem_desc(smem_u32(tiles), kHalfBytes, 1024, kLayoutSW128);
    int it = 0;
    bool ok = true;
    Q2B_R_T(_ml)
    for (int64_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++it) {
      const int slot = it % Cfg::kStages;
      const uint32_t ph = (it / Cfg::kStages) & 1;
      const int buf = it % Cfg::kTmemBufs;
      const uint32_t bph = (it / Cfg::kTmemBufs) & 1;
      Q2B_R_T(_m0)
      ok = mbar_wait(&tempty[buf], bph ^ 1, kTimeoutTmemEmpty);
      Q2B_R_T(_m1)
      ok = ok && mbar_wait(&full[slot], ph, kTimeoutTmaFull);
      Q2B_R_ADD(3, _m1 - _m0)
      Q2B_R_ADD(4, clock64() - _m1)
      Q2B_R_ADD(6, 1)
      if (!ok) break;
      tc_fence_after();
      // converged warp, one lane issuing through a predicate; descriptors are
      // the per-CTA bases plus compile-time offsets (start address >> 4 in
      // the low bits)
      const uint64_t slot_off = (slot * kTileBytes) >> 4;
      const uint32_t d = tmem + buf * Cfg::kColsPerBuf;
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint64_t bdesc = h_desc0 + (((s >> 2) * kHalfBytes + (s & 3) * 32) >> 4);
        if constexpr ((kOut & kOutRows) != 0)
          umma_bf16_if(lead, d, rows_desc0 + slot_off + (((s >> 2) * kHalfBytes + (s & 3) * 32) >> 4), bdesc,
                       id_rows, s > 0);
        if constexpr ((kOut & kOutCols) != 0)
          umma_bf16_if(lead, d + ((kOut & kOutRows) ? 128 : 0), cols_desc0 + slot_off + ((s * 2048) >> 4), bdesc,
                       id_cols, s > 0);
      }
      tc_commit_if(lead, &empty[slot]);
      tc_commit_if(lead, &tfull[buf]);
      __syncwarp();
    }
    Q2B_R_ADD(5, clock64() - _ml)
    if (lane == 0) {
      tc_commit(drain);
      mbar_wait(drain, 0, kTimeoutProducer);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - Cfg::kEpiWarp0;   // 0 .. kEpiWarps-1
    const int q = warp & 3;                // TMEM lane quarter this warp may access
    const int orient = (kOut == kOutBoth) ? (e >> 3) : (kOut == kOutRows ? 0 : 1);  // 0 rows, 1 cols
    // Groups of epilogue warps take tiles in turn (tile i is drained from
    // TMEM buffer i % kTmemBufs), each warp draining its 32 rows x 128
    // columns in chunks: while one group waits for its TMEM loads the others
    // compute.
    const int grp = (e >> 2) % Cfg::kEpiGroups;
    const uint32_t col_base = (kOut == kOutBoth && orient == 1) ? 128 : 0;
    uint8_t* codes = orient == 0 ? p.codes_r : p.codes_c;
    uint16_t* scratch = orient == 0 ? p.scratch_r : p.scratch_c;
    unsigned* maxp = orient == 0 ? p.max_r : p.max_c;
    const int64_t out_cols = orient == 0 ? p.N : p.M;  // length of an output row
    const int64_t n_kblk = out_cols >> 4, n_kt = n_kblk >> 2;
    constexpr int kLd = Cfg::kLdCols, kNLd = 128 / kLd;
    float run_max = 0.f;
    Q2B_R_T(_el)
    for (int it = grp;; it += Cfg::kEpiGroups) {
      const int64_t t = blockIdx.x + static_cast<int64_t>(it) * gridDim.x;
      if (t >= ntiles) break;
      const int buf = it % Cfg::kTmemBufs;
      const uint32_t bph = (it / Cfg::kTmemBufs) & 1;
      Q2B_R_T(_w0)
      if (!mbar_wait(&tfull[buf], bph, kTimeoutTmemFull)) break;
      Q2B_R_ADD(7, clock64() - _w0)
      tc_fence_after();
      const uint32_t t32 = static_cast<uint32_t>(t);
      const int64_t tm = t32 / tiles_n, tn = t32 % tiles_n;
      const int64_t orow = (orient == 0 ? tm : tn) * 128 + q * 32 + lane;
      const int64_t ogrp = orient == 0 ? tn : tm;  // 128-group index along the output row
      const uint32_t taddr0 = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * Cfg::kColsPerBuf + col_base;
      if constexpr (Cfg::kNumOut == 2) {
        // dual output: two TMEM buffers only, so the hand-off comes first --
        // two 64-column round trips, the buffer released after the second load
        constexpr int kChunk = 64, kNChunks = 2, kG = 4;
#pragma unroll
        for (int ch = 0; ch < kNChunks; ++ch) {
          uint8_t* crow = codes + orow * (out_cols >> 1) + ogrp * 64 + ch * (kChunk / 2);
          const uint32_t taddr = taddr0 + ch * kChunk;
          uint32_t r[kChunk / 32][32];
#pragma unroll
          for (int h = 0; h < kChunk / 32; ++h) tmem_ld_32x32b_x32(taddr + 32 * h, r[h]);
          Q2B_R_T(_l1)
          tmem_ld_wait();
          Q2B_R_ADD(8, clock64() - _l1)
          if (ch == kNChunks - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_relaxed(&tempty[buf]);  // TMEM hand-off only
          }
          uint32_t cw[2 * kG], fs[kG];
#pragma unroll
          for (int g = 0; g < kG; ++g)
            run_max = fmaxf(run_max, eden16(r[g >> 1] + 16 * (g & 1), p.inv_fp4_max, cw[2 * g], cw[2 * g + 1], fs[g]));
#pragma unroll
          for (int v = 0; v < kG / 2; ++v)
            __stcs(reinterpret_cast<uint4*>(crow + 16 * v), make_uint4(cw[4 * v], cw[4 * v + 1], cw[4 * v + 2], cw[4 * v + 3]));
          const int64_t kb = ogrp * 8 + ch * kG;
          const int64_t so = (((orow >> 7) * n_kt + (kb >> 2)) << 9) | ((orow & 31) << 4) | (((orow >> 5) & 3) << 2) |
                             (kb & 3);
          *reinterpret_cast<uint2*>(scratch + so) = make_uint2(fs[0] | (fs[1] << 16), fs[2] | (fs[3] << 16));
        }
      } else {
        // one orientation (four TMEM buffers): loads run one chunk ahead of
        // the EDEN arithmetic (two register buffers), so only the first load
        // of a tile is exposed
        uint32_t r[2][kLd];
        uint32_t cw[4], fs[4];
        tmem_ld_cols<kLd>(taddr0, r[0]);
        Q2B_R_T(_l1)
        tmem_ld_wait_regs<kLd>(r[0]);
        Q2B_R_ADD(8, clock64() - _l1)
#pragma unroll
        for (int l = 0; l < kNLd; ++l) {
          if (l + 1 < kNLd) {
            tmem_ld_cols<kLd>(taddr0 + (l + 1) * kLd, r[(l + 1) & 1]);
          } else {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_relaxed(&tempty[buf]);  // TMEM hand-off only
          }
#pragma unroll
          for (int gg = 0; gg < kLd / 16; ++gg) {
            const int g = l * (kLd / 16) + gg;  // 16-column group of the tile's row
            run_max = fmaxf(run_max, eden16(r[l & 1] + 16 * gg, p.inv_fp4_max, cw[2 * (g & 1)], cw[2 * (g & 1) + 1],
                                            fs[g & 3]));
            if ((g & 1) == 1)
              __stcs(reinterpret_cast<uint4*>(codes + orow * (out_cols >> 1) + ogrp * 64 + (g >> 1) * 16),
                     make_uint4(cw[0], cw[1], cw[2], cw[3]));
            if ((g & 3) == 3) {
              const int64_t kb = ogrp * 8 + (g - 3);
              const int64_t so = (((orow >> 7) * n_kt + (kb >> 2)) << 9) | ((orow & 31) << 4) |
                                 (((orow >> 5) & 3) << 2) | (kb & 3);
              *reinterpret_cast<uint2*>(scratch + so) = make_uint2(fs[0] | (fs[1] << 16), fs[2] | (fs[3] << 16));
            }
          }
          if (l + 1 < kNLd) tmem_ld_wait_regs<kLd>(r[(l + 1) & 1]);
        }
      }
    }
    Q2B_R_ADD(10, clock64() - _el)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) run_max = fmaxf(run_max, __shfl_xor_sync(0xffffffffu, run_max, o));
    if (lane == 0) atomicMax(maxp, __float_as_uint(run_max));
  }

#ifdef Q2B_RHT_STATS
  // roles' lane 0: producer warp 0, the MMA warp, epilogue warp 0
  if (blockIdx.x == 0 && lane == 0 && (warp == 0 || warp == Cfg::kMmaWarp || warp == Cfg::kEpiWarp0))
    for (int i = 0; i < 12; ++i)
      if (q2b_rs[i] != 0) atomicAdd(reinterpret_cast<unsigned long long*>(&g_rht_stats[i]),
                                    static_cast<unsigned long long>(q2b_rs[i]));
#endif
  tc_fence_before();
  __syncthreads();
  // this CTA's work is issued: the SR pass (a programmatic dependent launch) may be scheduled;
  // its griddepcontrol.wait still orders it after every write of this grid
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (warp == Cfg::kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// Pass 2: scale of the whole tensor from the global max, then stochastic
// rounding of every bf16 fixed scale to E4M3 (utils.cuh:336-386,
// group_transform_and_eden.cu:210-268 of the reference).  Scratch and output
// are both in the blocked layout; noise for scale i is 16 bits of
// Philox-4x32-10(key = seed, counter = i / 8).
__device__ __forceinline__ uint4 philox4x32_10(uint64_t seed, uint32_t ctr) {
  uint32_t c0 = ctr, c1 = 0, c2 = 0, c3 = 0;
  uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    // one widening multiply gives both halves of each 32 x 32 -> 64 product
    const uint64_t p0 = static_cast<uint64_t>(0xD2511F53u) * c0;
    const uint64_t p1 = static_cast<uint64_t>(0xCD9E8D57u) * c2;
    const uint32_t n0 = static_cast<uint32_t>(p1 >> 32) ^ c1 ^ k0;
    const uint32_t n2 = static_cast<uint32_t>(p0 >> 32) ^ c3 ^ k1;
    c0 = n0; c1 = static_cast<uint32_t>(p1); c2 = n2; c3 = static_cast<uint32_t>(p0);
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return make_uint4(c0, c1, c2, c3);
}

// The value whose round-to-nearest E4M3 conversion is the stochastic rounding
// of `in` with 16 bits of noise: inside E4M3's normal range the 20 mantissa
// bits below E4M3's 3 are truncated or rounded up against the noise; outside
// it (saturation, subnormals) `in` is converted as it is.
__device__ __forceinline__ float sr_e4m3_pre(float in, uint32_t noise16) {
  const float a = fabsf(in);
  if (a > 448.f || a < 0.015625f) return in;
  const uint32_t mask = 0x000FFFFFu;
  const uint32_t threshold = (noise16 << 4) & mask;
  uint32_t bits = __float_as_uint(in);
  bits = ((bits & mask) > threshold) ? (bits | mask) : (bits & ~mask);
  return __uint_as_float(bits);
}

// Two values -> two E4M3 bytes (lo in the low byte), round-to-nearest, saturating.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b16 h;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 h, %1, %2;\n\t"
      "cvt.u32.u16 %0, h;\n\t}"
      : "=r"(r)
      : "f"(hi), "f"(lo));
  return r;
}

// Eight consecutive blocked scales: scratch group i -> sf group i.
__device__ __forceinline__ void sr8(uint2* __restrict__ sf, const uint4* __restrict__ scratch, float f, uint64_t seed,
                                    int64_t i) {
  const uint4 s = __ldcg(scratch + i);
  const uint4 rnd = philox4x32_10(seed, static_cast<uint32_t>(i));
  const uint32_t w[4] = {s.x, s.y, s.z, s.w};
  const uint32_t nz[4] = {rnd.x, rnd.y, rnd.z, rnd.w};
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float x = __uint_as_float((j & 1) ? (w[j >> 1] & 0xFFFF0000u) : (w[j >> 1] << 16)) * f;
    v[j] = sr_e4m3_pre(x, (j & 1) ? (nz[j >> 1] >> 16) : (nz[j >> 1] & 0xFFFFu));
  }
  const uint32_t o0 = cvt_e4m3x2(v[0], v[1]) | (cvt_e4m3x2(v[2], v[3]) << 16);
  const uint32_t o1 = cvt_e4m3x2(v[4], v[5]) | (cvt_e4m3x2(v[6], v[7]) << 16);
  __stcs(sf + i, make_uint2(o0, o1));
}

// Tensor scale from the global max and the reciprocal the SR pass multiplies by.
__device__ __forceinline__ float sr_factor(float max_scale, float inv_fp8_max, float* gs_out) {
  float gs = max_scale * inv_fp8_max;
  float f;
  if (fabsf(gs) < FLT_MIN) { gs = 0.f; f = 0.f; } else { f = rcp_approx_ftz(gs); }
  *gs_out = gs;
  return f;
}

__global__ void __launch_bounds__(256) sr_scales_kernel(uint2* __restrict__ sf, float* __restrict__ ts_out,
                                                        const uint4* __restrict__ scratch,
                                                        const unsigned* __restrict__ max_bits, float inv_fp8_max,
                                                        uint64_t seed, int64_t n8) {
  // launched as a programmatic dependent of the EDEN kernel: the CTAs may start while its last
  // CTAs finish, and wait here until its writes (scratch, max word) are visible
  asm volatile("griddepcontrol.wait;" ::: "memory");
  float gs;
  const float f = sr_factor(__uint_as_float(*max_bits), inv_fp8_max, &gs);
  if (blockIdx.x == 0 && threadIdx.x == 0) *ts_out = gs;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += stride)
    sr8(sf, scratch, f, seed, i);
}


}  // namespace q2b
