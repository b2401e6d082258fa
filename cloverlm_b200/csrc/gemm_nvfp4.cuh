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
  int64_t M, N, K;
  const uint8_t* sfa;   // blocked [M, K/16]
  const uint8_t* sfb;   // blocked [N, K/16]
  const float* alpha;
  __nv_bfloat16* D;     // [M, N] row-major
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
  static constexpr uint32_t kSfaCol = 256;        // TMEM column of the A scales (16 cols)
  static constexpr uint32_t kSfbCol = 272;        // B scales (16 or 32 cols)
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kEpiWarps = 8;
  static constexpr int kThreads = 32 * (2 + kEpiWarps);
  static constexpr uint32_t kSmemBytes = 1024 + kStages * kStageBytes + 256;
};

template <int BN>
__global__ void __launch_bounds__(GemmCfg<BN>::kThreads, 1)
    gemm_nvfp4_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const GemmParams p) {
  using Cfg = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kStages * Cfg::kStageBytes);
  uint64_t* empty = full + Cfg::kStages;
  uint64_t* tfull = empty + Cfg::kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tiles_m = p.M / Cfg::BM, tiles_n = p.N / BN;
  const int64_t ntiles = tiles_m * tiles_n;
  const int64_t nkb = (p.K + 255) / 256;
  const int64_t n_kt = p.K / 64;  // 64-element scale chunks along K

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], Cfg::kEpiWarps);
    }
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int64_t it = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const int64_t tm = t / tiles_n, tn = t % tiles_n;
        for (int64_t kb = 0; kb < nkb; ++kb, ++it) {
          const int slot = static_cast<int>(it % Cfg::kStages);
          const uint32_t ph = static_cast<uint32_t>(it / Cfg::kStages) & 1;
          if (!mbar_wait(&empty[slot], ph ^ 1, kTimeoutSmemEmpty)) { ok = false; break; }
          const int nk = static_cast<int>((p.K - kb * 256) / 64 < 4 ? (p.K - kb * 256) / 64 : 4);
          uint8_t* st = smem + slot * Cfg::kStageBytes;
          const uint32_t sf_bytes = nk * 512u;
          mbar_arrive_expect_tx(&full[slot], Cfg::kABytes + Cfg::kBBytes + sf_bytes * (1 + BN / 128));
          tma_load_2d(st, &tmap_a, &full[slot], static_cast<int>(kb * 128), static_cast<int>(tm * Cfg::BM));
          tma_load_2d(st + Cfg::kABytes, &tmap_b, &full[slot], static_cast<int>(kb * 128),
                      static_cast<int>(tn * BN));
          bulk_load(st + Cfg::kABytes + Cfg::kBBytes, p.sfa + ((tm * n_kt + kb * 4) << 9), sf_bytes, &full[slot]);
#pragma unroll
          for (int u = 0; u < BN / 128; ++u)
            bulk_load(st + Cfg::kABytes + Cfg::kBBytes + Cfg::kSfaBytes + u * 2048,
                      p.sfb + (((tn * (BN / 128) + u) * n_kt + kb * 4) << 9), sf_bytes, &full[slot]);
        }
      }
      const int64_t issued = it;
      for (int64_t k = issued > Cfg::kStages ? issued - Cfg::kStages : 0; k < issued; ++k)
        mbar_wait(&full[k % Cfg::kStages], static_cast<uint32_t>(k / Cfg::kStages) & 1, kTimeoutProducer);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    const uint32_t idesc = idesc_nvf4(Cfg::BM, BN);
    int64_t it = 0, tc = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++tc) {
      const int buf = static_cast<int>(tc % Cfg::kAccBufs);
      const uint32_t bph = static_cast<uint32_t>(tc / Cfg::kAccBufs) & 1;
      if (!mbar_wait(&tempty[buf], bph ^ 1, kTimeoutTmemEmpty)) break;
      tc_fence_after();
      const uint32_t d = tmem + buf * BN;
      for (int64_t kb = 0; kb < nkb; ++kb, ++it) {
        const int slot = static_cast<int>(it % Cfg::kStages);
        const uint32_t ph = static_cast<uint32_t>(it / Cfg::kStages) & 1;
        if (!mbar_wait(&full[slot], ph, kTimeoutTmaFull)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
          const int nk = static_cast<int>((p.K - kb * 256) / 64 < 4 ? (p.K - kb * 256) / 64 : 4);
          const uint32_t st = smem_u32(smem + slot * Cfg::kStageBytes);
          const uint32_t sfa_s = st + Cfg::kABytes + Cfg::kBBytes;
          const uint32_t sfb_s = sfa_s + Cfg::kSfaBytes;
          for (int j = 0; j < nk; ++j) {
            tmem_cp_32x128b_x4(tmem + Cfg::kSfaCol + 4 * j, smem_desc(sfa_s + 512 * j, 0, 128, kLayoutNone));
#pragma unroll
            for (int u = 0; u < BN / 128; ++u)
              tmem_cp_32x128b_x4(tmem + Cfg::kSfbCol + (BN / 32) * j + 4 * u,
                                 smem_desc(sfb_s + u * 2048 + 512 * j, 0, 128, kLayoutNone));
          }
          for (int j = 0; j < nk; ++j) {
            const uint64_t adesc = smem_desc(st + 32 * j, 0, 1024, kLayoutSW128);
            const uint64_t bdesc = smem_desc(st + Cfg::kABytes + 32 * j, 0, 1024, kLayoutSW128);
            umma_nvf4(d, adesc, bdesc, idesc, tmem + Cfg::kSfaCol + 4 * j, tmem + Cfg::kSfbCol + (BN / 32) * j,
                      (kb > 0 || j > 0) ? 1u : 0u);
          }
          tc_commit(&empty[slot]);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (lane == 0) tc_commit(&tfull[buf]);
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - 2;
    const int q = warp & 3;  // TMEM lane quarter
    constexpr int kColsPerWarp = BN / 2;
    const int c0 = (e >> 2) * kColsPerWarp;
    const float alpha = *p.alpha;
    int64_t tc = 0;
    for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++tc) {
      const int buf = static_cast<int>(tc % Cfg::kAccBufs);
      const uint32_t bph = static_cast<uint32_t>(tc / Cfg::kAccBufs) & 1;
      if (!mbar_wait(&tfull[buf], bph, kTimeoutTmemFull)) break;
      tc_fence_after();
      const int64_t tm = t / tiles_n, tn = t % tiles_n;
      const int64_t row = tm * Cfg::BM + q * 32 + lane;
      __nv_bfloat16* drow = p.D + row * p.N + tn * BN + c0;
      const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * BN + c0;
#pragma unroll 1
      for (int ch = 0; ch < kColsPerWarp / 32; ++ch) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + ch * 32, r);
        tmem_ld_wait();
        if (ch == kColsPerWarp / 32 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[buf]);
        }
        uint32_t o[16];
#pragma unroll
        for (int k = 0; k < 16; ++k)
          o[k] = pack_bf16x2(__uint_as_float(r[2 * k]) * alpha, __uint_as_float(r[2 * k + 1]) * alpha);
        uint4* dst = reinterpret_cast<uint4*>(drow + ch * 32);
#pragma unroll
        for (int k = 0; k < 4; ++k) dst[k] = make_uint4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
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
