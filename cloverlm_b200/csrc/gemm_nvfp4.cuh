// NVFP4 x NVFP4 -> bf16 GEMM on the 5th-generation tensor cores.
//
//   D[m, n] = alpha * sum_k (a[m,k] * sfa[m, k/16]) * (b[n,k] * sfb[n, k/16])
//
// A [M, K] and B [N, K] are packed E2M1 codes, K-major (both Quartet GEMMs --
// forward, dgrad, wgrad -- are "TN"), scales are UE4M3 in the blocked 128x4
// layout, alpha is a device fp32 scalar.  This replaces the reference's
// _fp4_mm -> flashinfer.mm_fp4(backend="cudnn") (quartet2/python/quartet2/
// linear.py:34-56), whose kernel is closed.
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A box 128x128B and B box BNx128B with the
//               128-byte swizzle, plus the matching 512-byte scale chunks with
//               plain bulk copies, into a kStages ring (mbarrier complete_tx).
//   warp 1      TMEM owner and MMA issuer: per 256-element K block, tcgen05.cp
//               moves the scale chunks smem -> TMEM (32x128b, broadcast to the
//               four lane quarters), then four tcgen05.mma.kind::mxf4nvf4
//               .block_scale.block16 (M=128, N=BN, K=64) accumulate in TMEM.
//   warps 2..9  epilogue: tcgen05.ld of the fp32 accumulator, * alpha, bf16,
//               16-byte stores.
// No cluster, no multicast: every CTA fetches its own operands.
#pragma once
#include <cuda.h>
#include "common.cuh"

namespace q2b {

struct GemmParams {
  int64_t M, N, K;      // M rounded up to whole 128-row tiles
  const uint8_t* sfa;   // blocked [M, K/16]
  const uint8_t* sfb;   // blocked [N, K/16]
  const float* alpha;
  const float* alpha_b; // optional second factor of alpha (nullptr = 1)
  void* D;              // [m_valid, N] row-major, bf16 (or fp32 for the kOutF32 kernels)
  const uint16_t* aux;  // kEpiRelu2Bwd: the MLP pre-activation a, bf16 [M, N] row-major
  unsigned* amax;       // kEpiRelu2: max |relu(D)^2| (fp32 bits, atomicMax; zeroed by the launcher)
  int64_t m_valid;      // rows of A and D that exist (A rows past it read as zero through TMA)
  int splits;           // K split into this many ranges per output tile (1 = none)
  float* ws;            // splits > 1: fp32 partial tiles [tiles][128][BN], zero between calls
  unsigned* counters;   // splits > 1: arrival counters [tiles][epilogue warps], zero between calls
  int raster_rows = 1;  // pair kernel: row tiles per raster group (1 = row-major tile order)
};

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BKB = 128;                 // bytes of K per stage (256 fp4)
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kAccBufs = BN == 256 ? 1 : 2;
  static constexpr uint32_t kABytes = BM * BKB;   // 16 KB
  static constexpr uint32_t kBBytes = BN * BKB;
  static constexpr uint32_t kSfaBytes = 4 * 512;
  static constexpr uint32_t kSfbBytes = (BN / 128) * 4 * 512;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;
  // TMEM: accumulators in [0, 256); one scale-factor column set per stage
  // after them (A: 4 K steps x 4 columns, B: 4 K steps x BN/32 columns).
  static constexpr uint32_t kSfSetCols = 16 + 4 * (BN / 32);
  static constexpr uint32_t kSfBase = 256;
  static constexpr uint32_t kTmemCols = 512;
  static_assert(kSfBase + kStages * kSfSetCols <= kTmemCols, "TMEM overflow");
  static constexpr int kEpiWarps = 8;
#ifndef Q2B_GEMM_SF_WARPS
#define Q2B_GEMM_SF_WARPS 6
#endif
  // scale copies are issued by kSfWarps warps (A scales / B scales) because
  // tcgen05 issue blocks per thread: two issuing threads copy concurrently
  static constexpr int kSfWarps = Q2B_GEMM_SF_WARPS;
  static constexpr int kEpiWarp0 = 2 + kSfWarps;
  static constexpr int kThreads = 32 * (kEpiWarp0 + kEpiWarps);
  static constexpr uint32_t kSmemBytes = 1024 + kStages * kStageBytes + 512;
};

// Warp roles:
//   0  TMA producer      (waits empty[s], loads A/B/scales, arrives full[s])
//   1  MMA issuer        (waits sfready[s], 4 x tcgen05.mma, commits empty[s])
//   2  scale-copy issuer (waits full[s], tcgen05.cp of the stage's scales into
//                         TMEM column set s, commits sfready[s])
//   3+ epilogue
// The scale copies run on their own warp because tcgen05.cp and tcgen05.mma
// issued by one thread serialize with each other in this pipeline, while
// copies issued by a second warp overlap the MMAs of earlier stages.  Column
// set s is free again when full[s] fires, because the producer reloads stage
// s only after the MMAs that read set s have completed (empty[s]).
template <int BN, bool kOutF32 = false, bool kAccum = false>
__global__ void __launch_bounds__(GemmCfg<BN>::kThreads, 1)
    gemm_nvfp4_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const GemmParams p) {
  using Cfg = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kStages * Cfg::kStageBytes);
  uint64_t* empty = full + Cfg::kStages;
  uint64_t* sfready = empty + Cfg::kStages;
  uint64_t* tfull = sfready + Cfg::kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;  // every tcgen05 issuer's final commit: nothing in flight at dealloc
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tiles_n = p.N / BN;
  const int64_t ntiles = (p.M / Cfg::BM) * tiles_n;
  const int splits = p.splits;
  const int64_t nunits = ntiles * splits;  // work unit = (output tile, K range)
  const int64_t nkb = (p.K + 255) / 256;
  const int64_t n_kt = p.K / 64;  // 64-element scale chunks along K
  const int tail_nk = static_cast<int>((p.K % 256) / 64);  // K steps in a partial last block (0 = none)

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&sfready[s], Cfg::kSfWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], Cfg::kEpiWarps);
    }
    mbar_init(drain, 1 + Cfg::kSfWarps);
    fence_barrier_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t smem_base = smem_u32(smem);

  // Producer, scale-copy and MMA loops run on converged warps with one lane
  // issuing (predicated tcgen05 instructions, a short lane-0 block for the
  // loads): a loop run by one diverged lane pays for every branch.
  const bool lead = lane == 0;
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int64_t it = 0;
    bool ok = true;
    for (int64_t u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
      const int64_t t = u / splits, sp = u % splits;
      const int64_t tm = t / tiles_n, tn = t % tiles_n;
      for (int64_t kb = sp * nkb / splits; kb < (sp + 1) * nkb / splits; ++kb, ++it) {
        const int slot = static_cast<int>(it % Cfg::kStages);
        const uint32_t ph = static_cast<uint32_t>(it / Cfg::kStages) & 1;
        if (!warp_wait(&empty[slot], ph ^ 1, kTimeoutSmemEmpty)) { ok = false; break; }
        if (lead) {
          const int nk = (kb == nkb - 1 && tail_nk) ? tail_nk : 4;
          uint8_t* st = smem + slot * Cfg::kStageBytes;
          const uint32_t sf_bytes = nk * 512u;
          mbar_arrive_expect_tx(&full[slot], Cfg::kABytes + Cfg::kBBytes + sf_bytes * (1 + BN / 128));
          tma_load_2d(st, &tmap_a, &full[slot], static_cast<int>(kb * 128), static_cast<int>(tm * Cfg::BM));
          tma_load_2d(st + Cfg::kABytes, &tmap_b, &full[slot], static_cast<int>(kb * 128),
                      static_cast<int>(tn * BN));
          bulk_load(st + Cfg::kABytes + Cfg::kBBytes, p.sfa + ((tm * n_kt + kb * 4) << 9), sf_bytes, &full[slot]);
#pragma unroll
          for (int v = 0; v < BN / 128; ++v)
            bulk_load(st + Cfg::kABytes + Cfg::kBBytes + Cfg::kSfaBytes + v * 2048,
                      p.sfb + (((tn * (BN / 128) + v) * n_kt + kb * 4) << 9), sf_bytes, &full[slot]);
        }
        __syncwarp();
      }
    }
    const int64_t issued = it;
    for (int64_t k = issued > Cfg::kStages ? issued - Cfg::kStages : 0; k < issued; ++k)
      warp_wait(&full[k % Cfg::kStages], static_cast<uint32_t>(k / Cfg::kStages) & 1, kTimeoutProducer);
  } else if (warp >= 2 && warp < 2 + Cfg::kSfWarps) {
    // ------------------------------------------------------------ scale copies
    const int me = warp - 2;
    constexpr int kPerStep = 1 + BN / 128;
    // descriptors of stage 0's scale chunks; stage s adds s * kStageBytes
    const uint64_t sfa_d0 = smem_desc(smem_base + Cfg::kABytes + Cfg::kBBytes, 0, 128, kLayoutNone);
    const uint64_t sfb_d0 = sfa_d0 + (Cfg::kSfaBytes >> 4);
    int slot = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int64_t u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
      const int64_t sp = u % splits;
      for (int64_t kb = sp * nkb / splits; kb < (sp + 1) * nkb / splits; ++kb) {
        if (!warp_wait(&full[slot], ph, kTimeoutTmaFull)) { ok = false; break; }
        tc_fence_after();
        const int nk = (kb == nkb - 1 && tail_nk) ? tail_nk : 4;
        const uint64_t so = static_cast<uint64_t>((slot * Cfg::kStageBytes) >> 4);
        const uint32_t set = tmem + Cfg::kSfBase + slot * Cfg::kSfSetCols;
        // copies in TMEM column order (A steps, then B steps x halves);
        // each warp takes a contiguous block of them
        const int ncp = nk * kPerStep;
        const int lo = me * ncp / Cfg::kSfWarps, hi = (me + 1) * ncp / Cfg::kSfWarps;
        for (int c = lo; c < hi; ++c) {
          if (c < nk) {
            tmem_cp_32x128b_x4_if(lead, set + 4 * c, sfa_d0 + so + 32 * c);
          } else {
            const int b = c - nk, j = b / (BN / 128), v = b % (BN / 128);
            tmem_cp_32x128b_x4_if(lead, set + 16 + (BN / 32) * j + 4 * v, sfb_d0 + so + 128 * v + 32 * j);
          }
        }
        tc_commit_if(lead, &sfready[slot]);
        if (++slot == Cfg::kStages) { slot = 0; ph ^= 1; }
      }
    }
    tc_commit_if(lead, drain);
    warp_wait(drain, 0, kTimeoutProducer);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    const uint32_t idesc = idesc_nvf4(Cfg::BM, BN);
    const uint64_t a_d0 = smem_desc(smem_base, 0, 1024, kLayoutSW128);
    const uint64_t b_d0 = smem_desc(smem_base + Cfg::kABytes, 0, 1024, kLayoutSW128);
    const uint32_t sf0 = tmem + Cfg::kSfBase;
    int slot = 0;
    uint32_t ph = 0;
    int64_t tc = 0;
    bool ok = true;
    for (int64_t u = blockIdx.x; u < nunits && ok; u += gridDim.x, ++tc) {
      const int buf = static_cast<int>(tc % Cfg::kAccBufs);
      const uint32_t bph = static_cast<uint32_t>(tc / Cfg::kAccBufs) & 1;
      if (!warp_wait(&tempty[buf], bph ^ 1, kTimeoutTmemEmpty)) break;
      tc_fence_after();
      const uint32_t d = tmem + buf * BN;
      const int64_t sp = u % splits, kb0 = sp * nkb / splits;
      for (int64_t kb = kb0; kb < (sp + 1) * nkb / splits; ++kb) {
        if (!warp_wait(&sfready[slot], ph, kTimeoutTmaFull)) { ok = false; break; }
        tc_fence_after();
        const uint64_t so = static_cast<uint64_t>((slot * Cfg::kStageBytes) >> 4);
        const uint32_t set = sf0 + slot * Cfg::kSfSetCols;
        const uint64_t ad = a_d0 + so, bd = b_d0 + so;
        if (kb == nkb - 1 && tail_nk) {
          for (int j = 0; j < tail_nk; ++j)
            umma_nvf4_if(lead, d, ad + 2 * j, bd + 2 * j, idesc, set + 4 * j, set + 16 + (BN / 32) * j,
                         (kb > kb0 || j > 0) ? 1u : 0u);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            umma_nvf4_if(lead, d, ad + 2 * j, bd + 2 * j, idesc, set + 4 * j, set + 16 + (BN / 32) * j,
                         (kb > kb0 || j > 0) ? 1u : 0u);
        }
        tc_commit_if(lead, &empty[slot]);
        if (++slot == Cfg::kStages) { slot = 0; ph ^= 1; }
      }
      if (!ok) break;
      tc_commit_if(lead, &tfull[buf]);
    }
    tc_commit_if(lead, drain);
    warp_wait(drain, 0, kTimeoutProducer);
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - Cfg::kEpiWarp0;
    const int q = warp & 3;  // TMEM lane quarter
    constexpr int kColsPerWarp = BN / 2;
    const int c0 = (e >> 2) * kColsPerWarp;
    const float alpha = *p.alpha * (p.alpha_b != nullptr ? *p.alpha_b : 1.f);
    int64_t tc = 0;
    for (int64_t u = blockIdx.x; u < nunits; u += gridDim.x, ++tc) {
      const int buf = static_cast<int>(tc % Cfg::kAccBufs);
      const uint32_t bph = static_cast<uint32_t>(tc / Cfg::kAccBufs) & 1;
      if (!mbar_wait(&tfull[buf], bph, kTimeoutTmemFull)) break;
      tc_fence_after();
      const int64_t t = u / splits;
      const int64_t tm = t / tiles_n, tn = t % tiles_n;
      const int trow = q * 32 + lane;
      const int64_t row = tm * Cfg::BM + trow;
      const bool live = row < p.m_valid;
      __nv_bfloat16* drow = static_cast<__nv_bfloat16*>(p.D) + row * p.N + tn * BN + c0;
      float* frow = static_cast<float*>(p.D) + row * p.N + tn * BN + c0;
      const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * BN + c0;
      constexpr int kChunks = kColsPerWarp / 32;
      if constexpr (BN == 128) {
        if (splits > 1) {
          // Split-K: add this K range's partial (times alpha) into the fp32
          // tile in the workspace; the unit that arrives last converts the
          // tile to bf16, stores it and zeroes the workspace and counter.
          uint32_t r[kChunks][32];
#pragma unroll
          for (int ch = 0; ch < kChunks; ++ch) tmem_ld_32x32b_x32(taddr + ch * 32, r[ch]);
          tmem_ld_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_relaxed(&tempty[buf]);  // TMEM hand-off only
          float* wrow = p.ws + t * (Cfg::BM * BN) + trow * BN + c0;
          if (live) {
#pragma unroll
            for (int ch = 0; ch < kChunks; ++ch)
#pragma unroll
              for (int k = 0; k < 8; ++k)
                red_add_v4(wrow + ch * 32 + 4 * k, __uint_as_float(r[ch][4 * k]) * alpha,
                           __uint_as_float(r[ch][4 * k + 1]) * alpha, __uint_as_float(r[ch][4 * k + 2]) * alpha,
                           __uint_as_float(r[ch][4 * k + 3]) * alpha);
          }
          // each epilogue warp owns a 32-row x 64-column region of the tile
          // and its own arrival counter, so no barrier spans warps
          __threadfence();
          __syncwarp();
          unsigned* ctr = p.counters + t * Cfg::kEpiWarps + e;
          int last = 0;
          if (lane == 0) last = atomicAdd(ctr, 1u) == static_cast<unsigned>(splits - 1);
          last = __shfl_sync(0xffffffffu, last, 0);
          if (last) {
            __threadfence();
            if (live) {
#pragma unroll
              for (int ch = 0; ch < kChunks; ++ch) {
                uint32_t o[16];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                  const float4 v = __ldcg(reinterpret_cast<const float4*>(wrow + ch * 32 + 4 * k));
                  if constexpr (kOutF32) {
                    reinterpret_cast<float4*>(frow + ch * 32)[k] = v;
                  } else {
                    o[2 * k] = pack_bf16x2(v.x, v.y);
                    o[2 * k + 1] = pack_bf16x2(v.z, v.w);
                  }
                  __stcg(reinterpret_cast<float4*>(wrow + ch * 32 + 4 * k), make_float4(0.f, 0.f, 0.f, 0.f));
                }
                if constexpr (!kOutF32) {
                  uint4* dst = reinterpret_cast<uint4*>(drow + ch * 32);
#pragma unroll
                  for (int k = 0; k < 4; ++k)
                    dst[k] = make_uint4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
                }
              }
            }
            if (lane == 0) *ctr = 0u;
          }
          continue;
        }
      }
      // Drain the whole accumulator slice into registers first (scaled and
      // packed to bf16 pairs in two halves, which halves the live registers)
      // and hand the TMEM buffer back to the MMA warp at once; the global
      // stores then overlap the next tile's MMAs.
      constexpr int kHalf = kChunks > 1 ? kChunks / 2 : 1;
      if constexpr (kOutF32) {
        // fp32 output: each 32-column chunk goes out as soon as it is loaded
        // (the accumulator is released after the last chunk's load)
#pragma unroll
        for (int ch = 0; ch < kChunks; ++ch) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + ch * 32, r);
          tmem_ld_wait();
          if (ch == kChunks - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_relaxed(&tempty[buf]);  // TMEM hand-off only
          }
          if (live) {
            float4* dst = reinterpret_cast<float4*>(frow + ch * 32);
#pragma unroll
            for (int k = 0; k < 8; ++k)
              dst[k] = make_float4(__uint_as_float(r[4 * k]) * alpha, __uint_as_float(r[4 * k + 1]) * alpha,
                                   __uint_as_float(r[4 * k + 2]) * alpha, __uint_as_float(r[4 * k + 3]) * alpha);
          }
        }
        continue;
      }
      uint32_t o[kChunks][16];
#pragma unroll
      for (int h0 = 0; h0 < kChunks; h0 += kHalf) {
        uint32_t r[kHalf][32];
#pragma unroll
        for (int ch = 0; ch < kHalf; ++ch) tmem_ld_32x32b_x32(taddr + (h0 + ch) * 32, r[ch]);
        tmem_ld_wait();
#pragma unroll
        for (int ch = 0; ch < kHalf; ++ch)
#pragma unroll
          for (int k = 0; k < 16; ++k)
            o[h0 + ch][k] = pack_bf16x2(__uint_as_float(r[ch][2 * k]) * alpha, __uint_as_float(r[ch][2 * k + 1]) * alpha);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_relaxed(&tempty[buf]);  // TMEM hand-off only
      if (live) {
#pragma unroll
        for (int ch = 0; ch < kChunks; ++ch) {
          uint4* dst = reinterpret_cast<uint4*>(drow + ch * 32);
          if constexpr (kAccum) {
            // D += bf16(alpha * acc): bf16 adds of the existing output (the row is this lane's)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint4 d = dst[k];
              const uint32_t dw[4] = {d.x, d.y, d.z, d.w};
              uint32_t sum[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint32_t v = o[ch][4 * k + j];
                sum[j] = pack_bf16x2(__uint_as_float(dw[j] << 16) + __uint_as_float(v << 16),
                                     __uint_as_float(dw[j] & 0xFFFF0000u) + __uint_as_float(v & 0xFFFF0000u));
              }
              dst[k] = make_uint4(sum[0], sum[1], sum[2], sum[3]);
            }
          } else {
#pragma unroll
            for (int k = 0; k < 4; ++k)
              dst[k] = make_uint4(o[ch][4 * k], o[ch][4 * k + 1], o[ch][4 * k + 2], o[ch][4 * k + 3]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

}  // namespace q2b

namespace q2b {

// ---------------------------------------------------------------------------
// 2-SM variant: a cluster of two CTAs (an SM pair) computes a 256x256 output
// tile with tcgen05.mma.cta_group::2 (M=256 across the pair, N=256).  Each CTA
// loads its own 128 rows of A and its own 128-row half of B, so per SM a K
// block needs 16 + 16 KB of operands instead of 16 + 32 KB, and five stages
// fit.  Scale factors: each CTA holds the A scales of its rows and the B
// scales of all 256 columns (four-way lane-replicated, as tcgen05.cp 32x128b
// .warpx4 writes them); one 2-CTA copy instruction fills both CTAs' TMEM.
//   leader (rank 0): TMA warp, MMA warp, two groups of three scale-copy warps,
//                    epilogue; its full[] barriers count the bytes of BOTH
//                    CTAs (.cta_group::2 TMA completes on the leader's
//                    barrier), its tempty[] collects both CTAs' epilogue warps.
//   peer   (rank 1): TMA warp and epilogue.
// A warp issues tcgen05.cp at ~76 cycles each and copies cost tensor-pipe
// time once MMAs depend on them, so a K block's twelve copies are split over
// three warps (A scales, B scales of columns 0-127, of 128-255), and two such
// groups take alternate K blocks.  Issue loops run on converged warps with one
// lane issuing through a predicate.  The epilogue writes D with TMA stores from
// a per-warp staging buffer and hands TMEM back with a relaxed arrive.
// Every wait is bounded; both CTAs meet at a cluster barrier before TMEM is
// freed and before exit, so no CTA leaves while its peer can still touch its
// shared memory or TMEM.
struct Gemm2Cfg {
  static constexpr int kStages = 5;
  static constexpr uint32_t kABytes = 128 * 128;            // this CTA's 128 rows x 128 B of K
  static constexpr uint32_t kBBytes = 128 * 128;            // this CTA's half of B
  static constexpr uint32_t kSfaBytes = 2048;               // 4 chunks (one per K=64 step) of 128 rows
  static constexpr uint32_t kSfbBytes = 4096;               // 2 x 128 rows x 4 chunks
  static constexpr uint32_t kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;  // 38 KB
  static constexpr uint32_t kSfSetCols = 48, kSfBase = 256, kTmemCols = 512;
  static_assert(kSfBase + kStages * kSfSetCols <= kTmemCols, "TMEM overflow");
#ifndef Q2B_GEMM2_EPI_WARPS
#define Q2B_GEMM2_EPI_WARPS 16
#endif
  static constexpr int kEpiWarps = Q2B_GEMM2_EPI_WARPS;  // 4 per TMEM lane quarter, 64 columns each
#ifndef Q2B_GEMM2_SF_GROUPS
#define Q2B_GEMM2_SF_GROUPS 2
#endif
  // Scale-copy warps: groups of three (A scales, B scales of columns 0-127,
  // of columns 128-255) that take K blocks in turn.  Copies cost tensor-pipe
  // time and a single warp issues them at ~76 cycles each, so one warp per K
  // block would make each block's copies a ~900-cycle serial step.
  static constexpr int kSfGroups = Q2B_GEMM2_SF_GROUPS;
  static_assert(kSfGroups >= 1 && kSfGroups <= 3, "2 + 3 * kSfGroups + epilogue warps must fit the block");
  static constexpr int kSfWarps = 3 * kSfGroups;
  static constexpr int kEpiWarp0 = 2 + kSfWarps;
  static constexpr int kThreads = 32 * (kEpiWarp0 + kEpiWarps);
  // epilogue staging after the ring and the barriers: 2 KB per epilogue warp
  static constexpr uint32_t kStagingPerWarp = 32 * 32 * 2;
  static constexpr uint32_t kStagingOff = (kStages * kStageBytes + 512 + 1023) / 1024 * 1024;
  static constexpr uint32_t kSmemBytes = 1024 + kStagingOff + kEpiWarps * kStagingPerWarp;
  static_assert(kSmemBytes <= 232448, "shared memory");
};

// Output tile t -> (row tile, column tile) in groups of `group` row tiles:
// consecutive tiles (the CTAs of one wave) walk a group's rows fastest, so a
// wave touches about `group` A panels and 74 / group B panels instead of
// 74 / tiles_n A panels and all tiles_n B panels; with long K the panels a
// wave streams then fit L2 together.  group = 1 is row-major order.
__device__ __forceinline__ void tile_coords(int64_t t, int64_t tiles_m, int64_t tiles_n, int64_t group, int64_t& tm,
                                            int64_t& tn) {
  const int64_t per = group * tiles_n;
  const int64_t grp = t / per, in = t - grp * per;
  const int64_t m0 = grp * group;
  const int64_t gs = tiles_m - m0 < group ? tiles_m - m0 : group;
  tm = m0 + in % gs;
  tn = in / gs;
}

#ifdef Q2B_GEMM2_STATS
// Instrumented builds only: cycle counts of CTA 0's roles (0 MMA: total, 1 MMA: waiting for
// scales, 2 MMA: waiting for the accumulator, 3 K blocks, 4 copy warp 0: waiting for stages,
// 5 producer: waiting for free slots, 6 epilogue warp 0: waiting for tiles, 7 tiles,
// 8 / 9 epilogue warp 0: issuing / waiting for its TMEM loads).  Counted in registers and
// added to the global counters once at exit, so the counting stays off the timed paths.
__device__ long long g_gemm2_stats[12];
#define Q2B_S_T(v) const long long v = clock64();
#define Q2B_S_ADD(i, val) q2b_st[i] += (val);
#else
#define Q2B_S_T(v)
#define Q2B_S_ADD(i, val)
#endif

// Arrive on the leader CTA's copy of `bar` when this thread's prior 2-CTA
// tcgen05 ops complete.
__device__ __forceinline__ void tc_commit_pair_leader(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 1;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Warp roles (both CTAs unless noted):
//   0  TMA producer; its loads complete on the LEADER's full[s]
//   1  MMA issuer (leader): waits sfready[s], cta_group::2 MMAs, multicast-commits empty[s]
//   2..kEpiWarp0-1  scale-copy issuers (leader): every warp waits full[s] of each stage in
//      order; on its group's K blocks it issues its third of the stage's cta_group::2
//      tcgen05.cp into TMEM set s and commits sfready[s] (three arrivals complete it)
//   kEpiWarp0+  epilogue: drains its own TMEM rows, arrives on the leader's tempty
// Epilogues of the pair kernel (D = alpha * A B^T is formed in fp32 first):
//   kEpiBf16      D bf16
//   kEpiF32       D fp32 (weight gradients of fp32 master weights)
//   kEpiRelu2     D = bf16(alpha*acc), the MLP pre-activation a, and D2 = bf16(relu(a)^2), the
//                 activation the next Quartet layer quantizes, plus *amax = max D2: the MLP's
//                 first linear, its ReLU^2 and the second linear's input abs-max in one pass
//                 (src/models/mlp.py:34-38,113-118)
//   kEpiRelu2Bwd  D = bf16(2 * relu(a) * bf16(alpha*acc)) with a = aux: the second linear's
//                 dgrad followed by the ReLU^2 backward, without writing and re-reading dH
//   kEpiBf16Add   D += bf16(alpha*acc), added in place by TMA reductions: the input gradient of
//                 several layers that read one activation (Q, K and V) summed in the dgrad GEMMs
enum GemmEpi : int { kEpiBf16 = 0, kEpiF32 = 1, kEpiRelu2 = 2, kEpiRelu2Bwd = 3, kEpiBf16Add = 4 };

template <int kEpi = kEpiBf16>
__global__ void __launch_bounds__(Gemm2Cfg::kThreads, 1)
    gemm_nvfp4_2sm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                          const __grid_constant__ CUtensorMap tmap_sfa, const __grid_constant__ CUtensorMap tmap_sfb,
                          const __grid_constant__ CUtensorMap tmap_d, const __grid_constant__ CUtensorMap tmap_d2,
                          const GemmParams p) {
  using Cfg = Gemm2Cfg;
  constexpr bool kOutF32 = kEpi == kEpiF32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kStages * Cfg::kStageBytes);
  uint64_t* empty = full + Cfg::kStages;
  uint64_t* sfready = empty + Cfg::kStages;
  uint64_t* tfull = sfready + Cfg::kStages;
  uint64_t* tempty = tfull + 1;
  uint64_t* drain = tempty + 1;  // leader's tcgen05 issuers' final commits: nothing in flight at dealloc
  uint64_t* auxbar = drain + 1;  // kEpiRelu2Bwd: one per epilogue warp, its TMA load of the a box
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(auxbar + Cfg::kEpiWarps);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#ifdef Q2B_GEMM2_STATS
  long long q2b_st[12] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
#endif
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int64_t cluster_id = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int64_t tiles_n = (p.N + 255) / 256;  // a last half tile reads zeros and stores nothing past N
  const int64_t tiles_m = (p.M + 255) / 256;
  const int64_t ntiles = tiles_m * tiles_n;
  const int64_t nkb = (p.K + 255) / 256;
  const int64_t n_kt = p.K / 64;
  const int tail_nk = static_cast<int>((p.K % 256) / 64);

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&sfready[s], 3);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, 2 * Cfg::kEpiWarps);
    mbar_init(drain, 1 + Cfg::kSfWarps);
    for (int w = 0; w < Cfg::kEpiWarps; ++w) mbar_init(&auxbar[w], 1);
    fence_barrier_init();
  }
  if (threadIdx.x == 32) {
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
    prefetch_tmap(&tmap_sfa);
    prefetch_tmap(&tmap_sfb);
  }
  cluster_sync();  // both CTAs resident, barriers initialized
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t smem_base = smem_u32(smem);

  // The producer, scale-copy and MMA warps run their loops with all 32 lanes
  // converged and one lane issuing (predicated tcgen05 instructions, a short
  // lane-0 block for the TMA): a loop run by one diverged lane pays for every
  // branch, and the MMA issue rate drops to a third of the pipe's.
  const bool lead = lane == 0;
  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    int64_t it = 0;
    bool ok = true;
    for (int64_t t = cluster_id; t < ntiles && ok; t += nclusters) {
      int64_t tm, tn;
      tile_coords(t, tiles_m, tiles_n, p.raster_rows, tm, tn);
      const int a_row = static_cast<int>(tm * 256 + rank * 128);
      const int b_row = static_cast<int>(tn * 256 + rank * 128);
      const int64_t sfa_chunk0 = (tm * 2 + rank) * n_kt;
      const int64_t sfb_chunk0 = (tn * 2) * n_kt;
      for (int64_t kb = 0; kb < nkb; ++kb, ++it) {
        const int slot = static_cast<int>(it % Cfg::kStages);
        const uint32_t ph = static_cast<uint32_t>(it / Cfg::kStages) & 1;
        Q2B_S_T(_p0)
        if (!warp_wait(&empty[slot], ph ^ 1, kTimeoutSmemEmpty)) { ok = false; break; }
        Q2B_S_ADD(5, clock64() - _p0)
        if (lead) {
          uint8_t* st = smem + slot * Cfg::kStageBytes;
          const uint32_t bar = map_to_rank(smem_u32(&full[slot]), 0);
          if (leader) mbar_arrive_expect_tx(&full[slot], 2 * Cfg::kStageBytes);
          tma_load_2d_pair(st, &tmap_a, bar, static_cast<int>(kb * 128), a_row);
          tma_load_2d_pair(st + Cfg::kABytes, &tmap_b, bar, static_cast<int>(kb * 128), b_row);
          // scale chunks: 512 B each, viewed as rows of 256 B
          tma_load_2d_pair(st + Cfg::kABytes + Cfg::kBBytes, &tmap_sfa, bar, 0,
                           static_cast<int>((sfa_chunk0 + kb * 4) * 2));
          tma_load_2d_pair(st + Cfg::kABytes + Cfg::kBBytes + Cfg::kSfaBytes, &tmap_sfb, bar, 0,
                           static_cast<int>((sfb_chunk0 + kb * 4) * 2));
          tma_load_2d_pair(st + Cfg::kABytes + Cfg::kBBytes + Cfg::kSfaBytes + 2048, &tmap_sfb, bar, 0,
                           static_cast<int>((sfb_chunk0 + n_kt + kb * 4) * 2));
        }
        __syncwarp();
      }
    }
    // drain: every issued stage is released by the MMAs (or the watchdog tripped)
    const int64_t issued = it;
    for (int64_t k = issued > Cfg::kStages ? issued - Cfg::kStages : 0; k < issued; ++k)
      warp_wait(&empty[k % Cfg::kStages], static_cast<uint32_t>(k / Cfg::kStages) & 1, kTimeoutProducer);
  } else if (warp >= 2 && warp < Cfg::kEpiWarp0) {
    // ------------------------------------------------------------ scale copies (leader)
    if (leader) {
      const int me = warp - 2, part = me % 3, group = me / 3;
      const uint64_t sfa_d0 = smem_desc(smem_base + Cfg::kABytes + Cfg::kBBytes, 0, 128, kLayoutNone);
      const uint64_t sfb_d0 = sfa_d0 + (Cfg::kSfaBytes >> 4);
      // this warp's part of a K block: A scales into columns 4j, B scales of
      // columns 0-127 into 16+8j, of columns 128-255 into 20+8j
      const uint64_t src0 = part == 0 ? sfa_d0 : (part == 1 ? sfb_d0 : sfb_d0 + 128);
      const uint32_t col0 = part == 0 ? 0 : (part == 1 ? 16 : 20);
      const uint32_t col_step = part == 0 ? 4 : 8;
      const int64_t my_tiles = cluster_id < ntiles ? (ntiles - 1 - cluster_id) / nclusters + 1 : 0;
      const int64_t total = my_tiles * nkb;
      // Every copy warp waits for every K block's stage in order, copying only
      // for its own group's blocks: a parity wait is only unambiguous when the
      // previous phase of that barrier is known to be complete, and TMA loads
      // of different stages may land out of order.
      for (int64_t i = 0; i < total; ++i) {
        const int slot = static_cast<int>(i % Cfg::kStages);
        const uint32_t ph = static_cast<uint32_t>(i / Cfg::kStages) & 1;
        const int64_t kb = i % nkb;
        Q2B_S_T(_c0)
        if (!warp_wait(&full[slot], ph, kTimeoutTmaFull)) break;
        if (me == 0) { Q2B_S_ADD(4, clock64() - _c0) }
        if (i % Cfg::kSfGroups != group) continue;
        tc_fence_after();
        const uint64_t src = src0 + ((slot * Cfg::kStageBytes) >> 4);
        const uint32_t set = tmem + Cfg::kSfBase + slot * Cfg::kSfSetCols + col0;
        const int nk = (kb == nkb - 1 && tail_nk) ? tail_nk : 4;
        for (int j = 0; j < nk; ++j) tmem_cp_32x128b_x4_pair_if(lead, set + col_step * j, src + 32 * j);
        tc_commit_pair_leader_if(lead, &sfready[slot]);
      }
      tc_commit_pair_leader_if(lead, drain);
      warp_wait(drain, 0, kTimeoutProducer);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue (leader)
    if (leader) {
      const uint32_t idesc = idesc_nvf4(256, 256);
      const uint64_t a_d0 = smem_desc(smem_base, 0, 1024, kLayoutSW128);
      const uint64_t b_d0 = smem_desc(smem_base + Cfg::kABytes, 0, 1024, kLayoutSW128);
      int slot = 0;
      uint32_t ph = 0;
      int64_t tc = 0;
      bool ok = true;
      Q2B_S_T(_m00)
      for (int64_t t = cluster_id; t < ntiles && ok; t += nclusters, ++tc) {
        const uint32_t bph = static_cast<uint32_t>(tc) & 1;
        Q2B_S_T(_m0)
        if (!warp_wait(tempty, bph ^ 1, kTimeoutTmemEmpty)) break;
        Q2B_S_ADD(2, clock64() - _m0)
        tc_fence_after();
        for (int64_t kb = 0; kb < nkb; ++kb) {
          Q2B_S_T(_m1)
          if (!warp_wait(&sfready[slot], ph, kTimeoutTmaFull)) { ok = false; break; }
          Q2B_S_ADD(1, clock64() - _m1)
          Q2B_S_ADD(3, 1)
          tc_fence_after();
          const uint64_t so = (slot * Cfg::kStageBytes) >> 4;
          const uint32_t set = tmem + Cfg::kSfBase + slot * Cfg::kSfSetCols;
          const uint64_t a_d = a_d0 + so, b_d = b_d0 + so;
          if (kb != nkb - 1 || tail_nk == 0) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              umma_nvf4_pair_if(lead, tmem, a_d + 2 * j, b_d + 2 * j, idesc, set + 4 * j, set + 16 + 8 * j,
                                (kb > 0 || j > 0) ? 1u : 0u);
          } else {
            for (int j = 0; j < tail_nk; ++j)
              umma_nvf4_pair_if(lead, tmem, a_d + 2 * j, b_d + 2 * j, idesc, set + 4 * j, set + 16 + 8 * j,
                                (kb > 0 || j > 0) ? 1u : 0u);
          }
          tc_commit_pair_if(lead, &empty[slot]);
          if (++slot == Cfg::kStages) { slot = 0; ph ^= 1; }
        }
        if (!ok) break;
        tc_commit_pair_if(lead, tfull);
      }
      Q2B_S_ADD(0, clock64() - _m00)
      tc_commit_pair_leader_if(lead, drain);
      warp_wait(drain, 0, kTimeoutProducer);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    // Each warp drains its 32 rows x 64 columns with one TMEM round trip,
    // releases the accumulator, then scales to bf16 and writes two 32 x 32
    // boxes through its 2 KB staging buffer (64-byte swizzle) with TMA
    // stores: coalesced writes, where per-lane 16-byte row stores slowed the
    // whole mainloop (a third of the forward GEMM's time at K = 3584).
    const int e = warp - Cfg::kEpiWarp0;
    const int q = warp & 3;
    constexpr int kCols = 256 / (Cfg::kEpiWarps / 4);  // columns per warp
    const int c0 = (e >> 2) * kCols;
    const float alpha = *p.alpha * (p.alpha_b != nullptr ? *p.alpha_b : 1.f);
    const uint32_t tempty_leader = map_to_rank(smem_u32(tempty), 0);
    uint8_t* stage = smem + Cfg::kStagingOff + e * Cfg::kStagingPerWarp;
    float relu2_max = 0.f;
    uint32_t aux_phase = 0;
    int64_t tc = 0;
    for (int64_t t = cluster_id; t < ntiles; t += nclusters, ++tc) {
      // tile coordinates before the wait: the drain is on the MMA's critical path
      int64_t tm, tn;
      tile_coords(t, tiles_m, tiles_n, p.raster_rows, tm, tn);
      const int row0 = static_cast<int>(tm * 256 + rank * 128 + q * 32);
      const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + c0;
      Q2B_S_T(_e0)
      if (!mbar_wait(tfull, static_cast<uint32_t>(tc) & 1, kTimeoutTmemFull)) break;
      if (e == 0) { Q2B_S_ADD(6, clock64() - _e0) Q2B_S_ADD(7, 1) }
      Q2B_S_T(_e1)
      tc_fence_after();
      uint32_t r[kCols / 32][32];
#pragma unroll
      for (int ch = 0; ch < kCols / 32; ++ch) tmem_ld_32x32b_x32(taddr + ch * 32, r[ch]);
      Q2B_S_T(_e2)
      tmem_ld_wait();
      Q2B_S_T(_e3)
      tc_fence_before();
      Q2B_S_T(_e4)
      __syncwarp();
      Q2B_S_T(_e5)
      // relaxed: only tensor memory changes hands, its reads already complete
      if (lane == 0) mbar_arrive_cluster_relaxed(tempty_leader);
      if (e == 0) { Q2B_S_ADD(8, _e2 - _e1) Q2B_S_ADD(9, _e3 - _e2) Q2B_S_ADD(10, _e4 - _e3) Q2B_S_ADD(11, _e5 - _e4) }
      // one box = 32 rows x 64 bytes: 32 bf16 columns, or 16 fp32 columns
      constexpr int kBoxCols = kOutF32 ? 16 : 32;
      // write one box of this warp's rows through the staging buffer with a TMA store
      auto store_box = [&](const uint32_t (&o)[16], const CUtensorMap* map, int col) {
        // the previous box's store must have read the staging buffer
        if (lane == 0) bulk_wait_group_read0();
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 4; ++k)  // 16-byte chunk k of row `lane`, 64-byte swizzle
          *reinterpret_cast<uint4*>(stage + lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4)) =
              make_uint4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if constexpr (kEpi == kEpiBf16Add)
            tma_reduce_add_2d(map, stage, col, row0);
          else
            tma_store_2d(map, stage, col, row0);
          bulk_commit_group();
        }
      };
#pragma unroll
      for (int bx = 0; bx < kCols / kBoxCols; ++bx) {
        const int col = static_cast<int>(tn * 256 + c0 + bx * kBoxCols);
        uint32_t o[16];
        if constexpr (kOutF32) {
#pragma unroll
          for (int k = 0; k < 16; ++k)
            o[k] = __float_as_uint(__uint_as_float(r[bx >> 1][16 * (bx & 1) + k]) * alpha);
        } else {
#pragma unroll
          for (int k = 0; k < 16; ++k)
            o[k] = pack_bf16x2(__uint_as_float(r[bx][2 * k]) * alpha, __uint_as_float(r[bx][2 * k + 1]) * alpha);
        }
        if constexpr (kEpi == kEpiRelu2Bwd) {
          // da = 2 * relu(a) * g, g the bf16 dgrad value: the a box comes into this warp's
          // staging buffer by TMA (once the previous store has read it), in the store's layout
          if (lane == 0) {
            bulk_wait_group_read0();
            mbar_arrive_expect_tx(&auxbar[e], 32 * 64);
            tma_load_2d(stage, &tmap_d2, &auxbar[e], col, row0);
          }
          __syncwarp();
          if (!mbar_wait(&auxbar[e], aux_phase, kTimeoutTmaFull)) break;
          aux_phase ^= 1u;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint4 av = *reinterpret_cast<const uint4*>(stage + lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4));
            const uint32_t aw[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t g = o[4 * k + j];
              const float a0 = fmaxf(__uint_as_float(aw[j] << 16), 0.f);
              const float a1 = fmaxf(__uint_as_float(aw[j] & 0xFFFF0000u), 0.f);
              o[4 * k + j] = pack_bf16x2(2.f * a0 * __uint_as_float(g << 16),
                                         2.f * a1 * __uint_as_float(g & 0xFFFF0000u));
            }
          }
        }
        store_box(o, &tmap_d, col);
        if constexpr (kEpi == kEpiRelu2) {
          // h = relu(a)^2 from the bf16 pre-activation just stored
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float a0 = fmaxf(__uint_as_float(o[k] << 16), 0.f);
            const float a1 = fmaxf(__uint_as_float(o[k] & 0xFFFF0000u), 0.f);
            o[k] = pack_bf16x2(a0 * a0, a1 * a1);
            relu2_max = fmaxf(relu2_max, fmaxf(__uint_as_float(o[k] << 16), __uint_as_float(o[k] & 0xFFFF0000u)));
          }
          store_box(o, &tmap_d2, col);
        }
      }
    }
    if (lane == 0) bulk_wait_group0();
    __syncwarp();
    if constexpr (kEpi == kEpiRelu2) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) relu2_max = fmaxf(relu2_max, __shfl_xor_sync(0xffffffffu, relu2_max, o));
      if (lane == 0) atomicMax(p.amax, __float_as_uint(relu2_max));
    }
  }

#ifdef Q2B_GEMM2_STATS
  if (blockIdx.x == 0 && lane == 0)
    for (int i = 0; i < 12; ++i)
      if (q2b_st[i] != 0) atomicAdd(reinterpret_cast<unsigned long long*>(&g_gemm2_stats[i]),
                                    static_cast<unsigned long long>(q2b_st[i]));
#endif
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, Cfg::kTmemCols);
  }
  cluster_sync();
}


// ---------------------------------------------------------------------------
// FP4 tensor-core ceiling (measurement only).  Each SM pair issues `iters`
// back-to-back cta_group::2 M256 N256 K64 block-scaled MMAs
// (2*256*256*64 FLOP each) on operands resident in shared memory: pseudo-random
// E2M1 codes and E4M3 scales in [0.5, 1.875], so the datapath toggles as in a
// real GEMM.  No loads and no scale copies inside the loop: the rate is the
// tensor pipe's own ceiling on this part, the denominator the GEMM kernels'
// roofline fraction is quoted against.
struct PeakCfg {
  static constexpr uint32_t kOpBytes = 2 * 128 * 128;  // A and this CTA's half of B, K = 256
  static constexpr uint32_t kSfBytes = 2048 + 4096;
  static constexpr uint32_t kUsedBytes = 1024 + kOpBytes + kSfBytes + 256;
  // more than half an SM's shared memory: one CTA per SM, so no two pairs share a tensor pipe
  static constexpr uint32_t kSmemBytes = 120 * 1024;
  static constexpr int kThreads = 64;
};

__global__ void __launch_bounds__(PeakCfg::kThreads, 1) fp4_mma_peak_kernel(int iters, long long* cycles) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* drain = reinterpret_cast<uint64_t*>(smem + PeakCfg::kOpBytes + PeakCfg::kSfBytes);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  const int warp = threadIdx.x >> 5;
  const uint32_t rank = cluster_ctarank();
  for (uint32_t i = threadIdx.x; i < PeakCfg::kOpBytes / 4; i += blockDim.x) {
    uint32_t h = (i + 1u) * 0x9E3779B1u ^ (blockIdx.x * 0x85EBCA77u);
    h ^= h >> 15;
    reinterpret_cast<uint32_t*>(smem)[i] = h * 0x2C1B3C6Du;
  }
  for (uint32_t i = threadIdx.x; i < PeakCfg::kSfBytes; i += blockDim.x)
    smem[PeakCfg::kOpBytes + i] = static_cast<uint8_t>(0x30u + ((i * 7u) & 0xFu));  // 0.5 .. 1.875
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  cluster_sync();
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  if (rank == 0 && warp == 1) {
    const bool lead = (threadIdx.x & 31) == 0;
    const uint32_t base = smem_u32(smem);
    const uint64_t sf_d0 = smem_desc(base + PeakCfg::kOpBytes, 0, 128, kLayoutNone);
    const uint64_t sfb_d0 = sf_d0 + (2048 >> 4);
    const uint32_t set = tmem + 256;
    // one K block's scale sets, copied once; every MMA reads them
    for (int j = 0; j < 4; ++j) {
      tmem_cp_32x128b_x4_pair_if(lead, set + 4 * j, sf_d0 + 32 * j);
      tmem_cp_32x128b_x4_pair_if(lead, set + 16 + 8 * j, sfb_d0 + 32 * j);
      tmem_cp_32x128b_x4_pair_if(lead, set + 20 + 8 * j, sfb_d0 + 128 + 32 * j);
    }
    const uint32_t idesc = idesc_nvf4(256, 256);
    const uint64_t a_d0 = smem_desc(base, 0, 1024, kLayoutSW128);
    const uint64_t b_d0 = smem_desc(base + 128 * 128, 0, 1024, kLayoutSW128);
    const long long c0 = clock64();
    uint64_t g0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g0));
    for (int i = 0; i < iters; ++i) {
      const int j = i & 3;
      umma_nvf4_pair_if(lead, tmem, a_d0 + 2 * j, b_d0 + 2 * j, idesc, set + 4 * j, set + 16 + 8 * j,
                        i > 0 ? 1u : 0u);
    }
    tc_commit_pair_leader_if(lead, drain);
    warp_wait(drain, 0, kTimeoutProducer);
    if (lead && cycles != nullptr && blockIdx.x == 0) {
      uint64_t g1;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g1));
      cycles[0] = clock64() - c0;
      cycles[1] = static_cast<long long>(g1 - g0);
    }
  }
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
  cluster_sync();
}

}  // namespace q2b
