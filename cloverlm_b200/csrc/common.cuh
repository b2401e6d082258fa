// Shared device helpers for the sm_100a kernels of libq2b: mbarriers with
// bounded waits, TMA loads, tcgen05 (TMEM allocation, UMMA issue, TMEM loads,
// TMEM copies), shared-memory matrix descriptors and number-format
// conversions written as inline PTX.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#if !defined(__CUDA_ARCH__) || (__CUDA_ARCH__ >= 1000)
#define Q2B_SM100 1
#endif

namespace q2b {

// ---------------------------------------------------------------- watchdog
// Every spin-wait in these kernels is bounded.  A wait that runs out records
// a code here (first writer wins) and the kernel unwinds without touching the
// data it was waiting for; the host reads and clears it via q2b_device_status.
enum WatchdogCode : unsigned {
  kOk = 0,
  kTimeoutTmaFull = 1,
  kTimeoutSmemEmpty = 2,
  kTimeoutTmemFull = 3,
  kTimeoutTmemEmpty = 4,
  kTimeoutProducer = 5,
  kTimeoutSelfTest = 6,  // q2b_watchdog_selftest: a wait nobody completes, by construction
};

// Defined once: the library is compiled as a single translation unit.
__device__ unsigned g_watchdog = 0;

// ~2 s at 2 GHz before a wait is declared stuck.
constexpr long long kWaitCycles = 4000000000ll;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void record_timeout(unsigned code) {
  atomicCAS(&g_watchdog, 0u, code);
}

__device__ __forceinline__ bool watchdog_tripped() {
  return *static_cast<volatile unsigned*>(&g_watchdog) != 0u;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Returns false (and
// records `code`) if it did not complete within `limit` SM cycles, or if
// another wait in the grid already gave up.
__device__ __forceinline__ bool mbar_wait_limit(uint64_t* bar, uint32_t parity, unsigned code, long long limit) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 1023u) == 0u) {
      if (watchdog_tripped()) return false;
      if (clock64() - start > limit) {
        record_timeout(code);
        return false;
      }
    }
  }
  return true;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned code) {
  return mbar_wait_limit(bar, parity, code, kWaitCycles);
}

// Health check of the timeout path: one thread waits, with a short limit, on
// a shared-memory barrier that nothing arrives on, so the wait runs out,
// records kTimeoutSelfTest and the kernel returns.  No copy, MMA or tensor
// memory is involved, so nothing is left in flight.
__global__ void watchdog_selftest_kernel(long long limit_cycles) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    mbar_wait_limit(&bar, 0, kTimeoutSelfTest, limit_cycles);
  }
  __syncwarp();
}

// Vector fp32 reduction into global memory (performed at L2).
__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy (TMA, UMMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Plain (untiled) bulk copy global -> shared; both addresses 16-B aligned,
// size a multiple of 16.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------- tcgen05
// TMEM allocation: executed by one full warp; writes the base address to smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrive (once) on an mbarrier when all previously issued tcgen05 async ops
// of this thread have completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// The same, issued by the lanes where `issue` holds: a converged warp issues
// through a predicate instead of a branch around one lane.
__device__ __forceinline__ void umma_bf16_if(bool issue, uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "setp.ne.b32 q, %5, 0;\n\t"
      "@q tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(issue ? 1u : 0u));
}

// D[tmem] (+)= A[smem] * B[smem]^T, bf16 inputs, fp32 accumulation.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Block-scaled NVFP4 MMA: E2M1 A/B from smem, UE4M3 scales (one per 16
// elements along K) from TMEM, fp32 accumulation.  K = 64 per instruction.
__device__ __forceinline__ void umma_nvf4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
      : "memory");
}

// Copy 32 rows x 128 bits from smem to TMEM, broadcast to all four lane
// quarters (the scale-factor layout of block-scaled UMMA).
__device__ __forceinline__ void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Each thread of the warp reads 32 consecutive 32-bit columns of its lane.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Wait for the outstanding TMEM loads, with the destination registers of the
// load being waited for tied to the wait: with a later load in flight the
// compiler may not read (or copy) these registers before this point.
template <int kN>
__device__ __forceinline__ void tmem_ld_wait_regs(uint32_t (&r)[kN]) {
  static_assert(kN == 16 || kN == 32, "16 or 32 registers");
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :: "memory");
  if constexpr (kN == 32)
    asm volatile(""
                 : "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]),
                   "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                   "+r"(r[30]), "+r"(r[31]));
}

template <int kN>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[kN]) {
  if constexpr (kN == 32) tmem_ld_32x32b_x32(taddr, r); else tmem_ld_32x32b_x16(taddr, r);
}

// Shared-memory matrix descriptor (sm_100 format): start address, leading and
// stride byte offsets (all >> 4), fixed version 1 at bit 46, layout type in
// bits 61-63 (0 none, 2 = 128-byte swizzle, 4 = 64-byte, 6 = 32-byte).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

constexpr uint32_t kLayoutSW128 = 2;
constexpr uint32_t kLayoutNone = 0;

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 D.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                      // D format f32
         | (1u << 7)                    // A bf16
         | (1u << 10)                   // B bf16
         | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// Instruction descriptor for kind::mxf4nvf4 with E2M1 A/B, UE4M3 scales.
__host__ __device__ constexpr uint32_t idesc_nvf4(int M, int N) {
  return (1u << 7)     // A E2M1
         | (1u << 10)  // B E2M1
         | (static_cast<uint32_t>(N >> 3) << 17)  // scale format bit 23 = 0 -> UE4M3
         | (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------- formats
// Two fp32 -> packed E2M1 (round to nearest even, saturating): `lo` goes to
// the low nibble (the even element).
__device__ __forceinline__ uint32_t cvt_e2m1x2(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b8 b;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b, %1, %2;\n\t"
      "cvt.u32.u8 %0, b;\n\t}"
      : "=r"(r)
      : "f"(hi), "f"(lo));
  return r;
}

// Two fp32 -> packed E2M1 byte (as in cvt_e2m1x2) and, from the same byte
// register, its two decoded values as fp16x2 -- one asm block, so the byte
// never round-trips through a 32-bit register between the conversions.
// Eight values -> one word of E2M1 codes (value 2j in the low nibble of byte
// j, round-to-nearest-even, saturating) and the four f16x2 pairs the codes
// decode to; the code bytes are packed in registers, with no byte extraction.
__device__ __forceinline__ void cvt_e2m1x8_back(const float (&v)[8], uint32_t& word, uint32_t (&back)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %8, %7;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %10, %9;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %12, %11;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %4, b3;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(word), "=r"(back[0]), "=r"(back[1]), "=r"(back[2]), "=r"(back[3])
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
}

__device__ __forceinline__ void cvt_e2m1x2_back(float lo, float hi, uint32_t& byte, uint32_t& back_h2) {
  asm("{\n\t.reg .b8 b;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b, %2, %3;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b;\n\t"
      "cvt.u32.u8 %0, b;\n\t}"
      : "=r"(byte), "=r"(back_h2)
      : "f"(hi), "f"(lo));
}

// Packed E2M1 byte -> two fp16 values (low nibble in the low half).
// One word of eight E2M1 codes -> four f16x2 pairs (pair j from byte j).
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t word, uint32_t (&h)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(word));
}

__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
  uint32_t r;
  asm("{\n\t.reg .b8 b;\n\t"
      "cvt.u8.u32 b, %1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b;\n\t}"
      : "=r"(r)
      : "r"(byte));
  return r;
}

__device__ __forceinline__ float2 f16x2_to_f32x2(uint32_t h2) {
  float a, b;
  asm("{\n\t.reg .f16 lo, hi;\n\t"
      "mov.b32 {lo, hi}, %2;\n\t"
      "cvt.f32.f16 %0, lo;\n\t"
      "cvt.f32.f16 %1, hi;\n\t}"
      : "=f"(a), "=f"(b)
      : "r"(h2));
  return make_float2(a, b);
}

// fp32 -> E4M3 (round to nearest even, saturating to 448).
__device__ __forceinline__ uint32_t cvt_e4m3(float v) {
  uint32_t r;
  asm("{\n\t.reg .b16 h;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 h, %1, %1;\n\t"
      "cvt.u32.u16 %0, h;\n\t}"
      : "=r"(r)
      : "f"(v));
  return r & 0xFFu;
}

// E4M3 byte -> fp32 (exact).
__device__ __forceinline__ float e4m3_to_f32(uint32_t byte) {
  uint32_t h2;
  asm("{\n\t.reg .b16 b;\n\t"
      "cvt.u16.u32 b, %1;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, b;\n\t}"
      : "=r"(h2)
      : "r"(byte & 0xFFu));
  return f16x2_to_f32x2(h2).x;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Correctly rounded fp32 reciprocal (IEEE round to nearest).
__device__ __forceinline__ float rcp_rn(float x) { return __frcp_rn(x); }

// The hardware's approximate reciprocal (rcp.approx.ftz.f32), the instruction
// the reference's quantizers use for every scale reciprocal
// (quartet2/csrc/utils.cuh:412-428, round_four_six.cu:25-31,
// had128_utils.cuh:193,210, group_transform_and_eden.cu:222).  Using the same
// instruction at the same points makes codes and scales bit-identical to the
// reference's at rounding ties, where an IEEE reciprocal can land one ulp
// away and flip the rounding.
__device__ __forceinline__ float rcp_approx_ftz(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ float2 fmul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// Blocked 128x4 scale-factor layout offset of (row, 16-element block kblk).
__host__ __device__ __forceinline__ int64_t sf_offset(int64_t row, int64_t kblk, int64_t n_kblk) {
  const int64_t n_ktiles = n_kblk >> 2;
  return (((row >> 7) * n_ktiles + (kblk >> 2)) << 9) | ((row & 31) << 4) | (((row >> 5) & 3) << 2) | (kblk & 3);
}

}  // namespace q2b

namespace q2b {
// ---------------------------------------------------------------- clusters / 2-SM
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// shared::cluster address of the object at `smem_addr` (a shared::cta address)
// in the CTA of the cluster with the given rank.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}

__device__ __forceinline__ float ld_shared_cluster_f32(uint32_t cluster_addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
  return v;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// Relaxed arrive: no release of the thread's prior memory operations.  For a
// hand-off of tensor memory only (the reads already completed by
// tcgen05.wait::ld, ordered by tcgen05.fence::before_thread_sync), where a
// cluster-scope release would wait ~2 k cycles for the warp's outstanding
// stores.
__device__ __forceinline__ void mbar_arrive_relaxed(uint64_t* bar) {
  asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// TMA tile load into this CTA's shared memory whose completion is counted on
// an mbarrier that may live in either CTA of the pair (`bar_cluster`).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const void* tmap, uint32_t bar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Arrive (once) on the mbarrier at the same offset in both CTAs of the pair
// when all prior tcgen05 ops of this thread have completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void umma_nvf4_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                               uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
      : "memory");
}

// The same MMA and commit issued only where `issue` is set, without a branch:
// the whole warp runs the issue loop converged and one lane issues.
__device__ __forceinline__ void umma_nvf4_pair_if(bool issue, uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                  uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "setp.ne.b32 q, %7, 0;\n\t"
      "@q tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate), "r"(issue ? 1u : 0u)
      : "memory");
}

__device__ __forceinline__ void tc_commit_pair_if(bool issue, uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\t.reg .pred q;\n\tmov.b16 m, 3;\n\t"
      "setp.ne.b32 q, %1, 0;\n\t"
      "@q tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar)), "r"(issue ? 1u : 0u)
      : "memory");
}

__device__ __forceinline__ void tc_commit_pair_leader_if(bool issue, uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\t.reg .pred q;\n\tmov.b16 m, 1;\n\t"
      "setp.ne.b32 q, %1, 0;\n\t"
      "@q tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar)), "r"(issue ? 1u : 0u)
      : "memory");
}

__device__ __forceinline__ void tmem_cp_32x128b_x4_pair_if(bool issue, uint32_t taddr, uint64_t sdesc) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t"
      "@q tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;\n\t}" ::"r"(taddr), "l"(sdesc), "r"(issue ? 1u : 0u)
      : "memory");
}

// TMA tensor store shared -> global of one box at (x, y), tracked as a bulk
// group of the issuing thread (no multicast; the destination is local memory).
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
// TMA tensor reduction shared -> global: the box is added element-wise into global memory
// (the tensor map's element type; local memory only), tracked as a bulk group.
__device__ __forceinline__ void tma_reduce_add_2d(const void* tmap, const void* smem_src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   tmap),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until the thread's bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until the thread's bulk stores have completed.
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// 1-CTA forms of the predicated issue helpers.
__device__ __forceinline__ void umma_nvf4_if(bool issue, uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "setp.ne.b32 q, %7, 0;\n\t"
      "@q tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate), "r"(issue ? 1u : 0u)
      : "memory");
}

__device__ __forceinline__ void tc_commit_if(bool issue, uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %1, 0;\n\t"
      "@q tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar)),
      "r"(issue ? 1u : 0u)
      : "memory");
}

__device__ __forceinline__ void tmem_cp_32x128b_x4_if(bool issue, uint32_t taddr, uint64_t sdesc) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t"
      "@q tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;\n\t}" ::"r"(taddr), "l"(sdesc), "r"(issue ? 1u : 0u)
      : "memory");
}

// Three-input maximum (sm_100): NaN inputs are ignored as by fmaxf.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Bounded wait by a whole warp; the result is the same in every lane (false if
// any lane's wait gave up), so the warp's control flow stays converged.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, unsigned code) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, code));
}

// Scale-factor copy into both CTAs' TMEM, each from its own shared memory.
__device__ __forceinline__ void tmem_cp_32x128b_x4_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
}  // namespace q2b
