// libq2b: host side of the C ABI declared in include/q2b.h.  The whole
// library is one translation unit (kernels are header-only .cuh files).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/q2b.h"
#include "common.cuh"
#include "gemm_nvfp4.cuh"
#include "quant_fwd.cuh"
#include "rht_eden.cuh"
#include "optim.cuh"
#include "glue.cuh"

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

#define Q2B_CUDA(call)                                                                               \
  do {                                                                                               \
    cudaError_t e_ = (call);                                                                         \
    if (e_ != cudaSuccess) {                                                                         \
      cudaGetLastError();                                                                            \
      return fail(Q2B_ERR_CUDA, "%s failed: %s (%s)", #call, cudaGetErrorName(e_), cudaGetErrorString(e_)); \
    }                                                                                                \
  } while (0)

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

#define Q2B_REQUIRE_PTR(p)                                                                          \
  do {                                                                                              \
    if ((p) == nullptr) return fail(Q2B_ERR_INVALID, "Pointer `%s` is null", #p);                   \
    if (!aligned16(p)) return fail(Q2B_ERR_INVALID, "Pointer `%s` is not aligned to 16 bytes", #p); \
  } while (0)

#define Q2B_REQUIRE_NONNULL(p) \
  do {                         \
    if ((p) == nullptr) return fail(Q2B_ERR_INVALID, "Pointer `%s` is null", #p); \
  } while (0)

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  bool ready = false;
  int sms = 0;
  int cc_major = 0;
  int cc_minor = 0;
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_mu;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;

template <typename K>
cudaError_t set_smem(K kernel, uint32_t bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
}

// One-time per-device setup: device properties, kernel shared-memory limits,
// the driver's tensor-map encoder.
int device_setup(int* dev_out, int* sms_out) {
  int dev = 0;
  Q2B_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(Q2B_ERR_DEVICE, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    Q2B_CUDA(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
    Q2B_CUDA(cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev));
    Q2B_CUDA(cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev));
    if (d.cc_major != 10 || d.cc_minor != 0)
      return fail(Q2B_ERR_DEVICE, "libq2b is built for sm_100a; device %d is sm_%d%d", dev, d.cc_major, d.cc_minor);
    if (g_encode == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      Q2B_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
      if (fn == nullptr || q != cudaDriverEntryPointSuccess)
        return fail(Q2B_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
    using namespace q2b;
    Q2B_CUDA(set_smem(rht_eden_kernel<kInBf16, kOutRows>, RhtCfg<kInBf16, kOutRows>::kSmemBytes));
    Q2B_CUDA(set_smem(rht_eden_kernel<kInBf16, kOutCols>, RhtCfg<kInBf16, kOutCols>::kSmemBytes));
    Q2B_CUDA(set_smem(rht_eden_kernel<kInBf16, kOutBoth>, RhtCfg<kInBf16, kOutBoth>::kSmemBytes));
    Q2B_CUDA(set_smem(rht_eden_kernel<kInFp4, kOutCols>, RhtCfg<kInFp4, kOutCols>::kSmemBytes));
    Q2B_CUDA(set_smem(gemm_nvfp4_kernel<256, false>, GemmCfg<256>::kSmemBytes));
    Q2B_CUDA(set_smem(gemm_nvfp4_kernel<128, false>, GemmCfg<128>::kSmemBytes));
    Q2B_CUDA(set_smem(gemm_nvfp4_kernel<256, true>, GemmCfg<256>::kSmemBytes));
    Q2B_CUDA(set_smem(gemm_nvfp4_kernel<128, true>, GemmCfg<128>::kSmemBytes));
    Q2B_CUDA(set_smem(gemm_nvfp4_2sm_kernel<kEpiBf16>, Gemm2Cfg::kSmemBytes));
    Q2B_CUDA(set_smem(gemm_nvfp4_2sm_kernel<kEpiF32>, Gemm2Cfg::kSmemBytes));
    Q2B_CUDA(set_smem(gemm_nvfp4_2sm_kernel<kEpiRelu2>, Gemm2Cfg::kSmemBytes));
    Q2B_CUDA(set_smem(gemm_nvfp4_2sm_kernel<kEpiRelu2Bwd>, Gemm2Cfg::kSmemBytes));
    Q2B_CUDA(set_smem(gemm_nvfp4_2sm_kernel<kEpiBf16Add>, Gemm2Cfg::kSmemBytes));
    Q2B_CUDA(set_smem(gemm_nvfp4_kernel<256, false, true>, GemmCfg<256>::kSmemBytes));
    Q2B_CUDA(set_smem(gemm_nvfp4_kernel<128, false, true>, GemmCfg<128>::kSmemBytes));
    Q2B_CUDA(set_smem(fp4_mma_peak_kernel, PeakCfg::kSmemBytes));
    d.ready = true;
  }
  *dev_out = dev;
  *sms_out = d.sms;
  return Q2B_OK;
}

// 2-D tensor map over a row-major [rows, inner] matrix with a box of
// box_inner x box_rows elements and the 128-byte swizzle.
int make_tmap(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
              uint64_t rows, uint32_t box_inner, uint32_t box_rows,
              CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * elem_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(Q2B_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return Q2B_OK;
}

int check_dims128(const char* what, int64_t a, int64_t b) {
  if (a <= 0 || b <= 0) return fail(Q2B_ERR_INVALID, "%s: dimensions must be positive (got %lld x %lld)", what,
                                    static_cast<long long>(a), static_cast<long long>(b));
  if (a % 128 != 0) return fail(Q2B_ERR_INVALID, "%s: rows must be divisible by 128 (got %lld)", what,
                                static_cast<long long>(a));
  if (b % 128 != 0) return fail(Q2B_ERR_INVALID, "%s: cols must be divisible by 128 (got %lld)", what,
                                static_cast<long long>(b));
  if (a * b / 8 >= (int64_t(1) << 40)) return fail(Q2B_ERR_INVALID, "%s: tensor too large", what);
  return Q2B_OK;
}

int launch_sr(void* sf, float* ts, const void* scratch, const unsigned* maxp, float fp8_max, uint64_t seed,
              int64_t nscales, int sms, cudaStream_t st) {
  const int64_t n8 = nscales / 8;
  const int64_t want = (n8 + 255) / 256;
  const int blocks = static_cast<int>(want < int64_t(sms) * 8 ? want : int64_t(sms) * 8);
  // programmatic dependent launch: scheduled as the EDEN kernel drains, the kernel waits
  // (griddepcontrol.wait) for its results before reading them
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(blocks), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  Q2B_CUDA(cudaLaunchKernelEx(&cfg, q2b::sr_scales_kernel, reinterpret_cast<uint2*>(sf), ts,
                              reinterpret_cast<const uint4*>(scratch), maxp, 1.f / fp8_max, seed, n8));
  return Q2B_OK;
}

}  // namespace

namespace {

int rht_check_h(const void* h, int h_rows) {
  Q2B_REQUIRE_PTR(h);
  if (h_rows != 16 && h_rows != 128)
    return fail(Q2B_ERR_INVALID, "rotation matrix must have 16 (Hadamard slice) or 128 rows, got %d", h_rows);
  return Q2B_OK;
}

template <int kIn, int kOut>
int launch_rht(const CUtensorMap& tmap, const q2b::RhtParams& p, int sms, cudaStream_t st) {
  using Cfg = q2b::RhtCfg<kIn, kOut>;
  const int64_t ntiles = (p.M / 128) * (p.N / 128);
  if (ntiles >= (int64_t(1) << 31))
    return fail(Q2B_ERR_INVALID, "rht128: %lld x %lld is too large (more than 2^31 tiles of 128 x 128)",
                static_cast<long long>(p.M), static_cast<long long>(p.N));
  const int grid = static_cast<int>(ntiles < sms ? ntiles : sms);
  q2b::rht_eden_kernel<kIn, kOut><<<grid, Cfg::kThreads, Cfg::kSmemBytes, st>>>(tmap, p);
  Q2B_CUDA(cudaGetLastError());
  return Q2B_OK;
}

}  // namespace

extern "C" {

int q2b_version(void) { return 100; }

const char* q2b_last_error(void) { return g_err; }

int q2b_device_status(unsigned* code) {
  Q2B_REQUIRE_NONNULL(code);
  Q2B_CUDA(cudaDeviceSynchronize());
  unsigned v = 0, zero = 0;
  Q2B_CUDA(cudaMemcpyFromSymbol(&v, q2b::g_watchdog, sizeof(unsigned)));
  Q2B_CUDA(cudaMemcpyToSymbol(q2b::g_watchdog, &zero, sizeof(unsigned)));
  *code = v;
  return Q2B_OK;
}

// ---------------------------------------------------------------- block glue
int q2b_rope_norm_fwd(void* out, float* norm_out, const void* x, const float* cos_sin, const float* scale,
                      int64_t rows, int heads, int seq, void* stream) {
  Q2B_REQUIRE_PTR(out);
  Q2B_REQUIRE_PTR(x);
  Q2B_REQUIRE_NONNULL(norm_out);
  Q2B_REQUIRE_NONNULL(cos_sin);
  if (rows <= 0 || heads <= 0 || heads > 64 || seq <= 0)
    return fail(Q2B_ERR_INVALID, "rope_norm: rows, heads (1..64) and seq must be positive");
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  const int64_t nvec = rows * heads;
  if (nvec >= (int64_t(1) << 31)) return fail(Q2B_ERR_INVALID, "rope_norm: rows * heads must be below 2^31");
  const int64_t blocks = std::min<int64_t>((nvec + 15) / 16, static_cast<int64_t>(sms) * 16);
  q2b::rope_norm_fwd_kernel<<<static_cast<unsigned>(blocks), q2b::kRopeThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint4*>(out), norm_out, static_cast<const uint4*>(x), reinterpret_cast<const float2*>(cos_sin),
      scale, nvec, heads, seq);
  Q2B_CUDA(cudaGetLastError());
  return Q2B_OK;
}

int q2b_rope_norm_bwd(void* dx, float* dscale, const void* dout, const void* out, const float* norm,
                      const float* cos_sin, const float* scale, int64_t rows, int heads, int seq, void* stream) {
  Q2B_REQUIRE_PTR(dx);
  Q2B_REQUIRE_PTR(dout);
  Q2B_REQUIRE_PTR(out);
  Q2B_REQUIRE_NONNULL(norm);
  Q2B_REQUIRE_NONNULL(cos_sin);
  if (rows <= 0 || heads <= 0 || heads > 64 || seq <= 0)
    return fail(Q2B_ERR_INVALID, "rope_norm: rows, heads (1..64) and seq must be positive");
  if ((dscale == nullptr) != (scale == nullptr))
    return fail(Q2B_ERR_INVALID, "rope_norm_bwd: dscale and scale are given together or not at all");
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  const int64_t nvec = rows * heads;
  if (nvec >= (int64_t(1) << 31)) return fail(Q2B_ERR_INVALID, "rope_norm: rows * heads must be below 2^31");
  const int64_t blocks = std::min<int64_t>((nvec + 15) / 16, static_cast<int64_t>(sms) * 8);
  q2b::rope_norm_bwd_kernel<<<static_cast<unsigned>(blocks), q2b::kRopeThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint4*>(dx), dscale, static_cast<const uint4*>(dout), static_cast<const uint4*>(out), norm,
      reinterpret_cast<const float2*>(cos_sin), scale, nvec, heads, seq);
  Q2B_CUDA(cudaGetLastError());
  return Q2B_OK;
}

int q2b_add_rmsnorm_amax(float* x_out, void* xb_out, float* rstd_out, float* amax, const float* x, const void* y,
                         const float* w, int64_t rows, int d, float eps, void* stream) {
  Q2B_REQUIRE_PTR(x_out);
  Q2B_REQUIRE_PTR(xb_out);
  Q2B_REQUIRE_PTR(x);
  Q2B_REQUIRE_PTR(y);
  Q2B_REQUIRE_PTR(w);
  Q2B_REQUIRE_NONNULL(rstd_out);
  Q2B_REQUIRE_NONNULL(amax);
  if (rows <= 0 || d <= 0 || d % 8 != 0 || d > 8 * q2b::kNormThreads * q2b::kNormMaxVecs)
    return fail(Q2B_ERR_INVALID, "add_rmsnorm_amax: d must be a positive multiple of 8 up to %d",
                8 * q2b::kNormThreads * q2b::kNormMaxVecs);
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Q2B_CUDA(cudaMemsetAsync(amax, 0, sizeof(float), st));
  const int64_t blocks = std::min<int64_t>(rows, static_cast<int64_t>(sms) * 8);
  q2b::add_rmsnorm_amax_kernel<<<static_cast<unsigned>(blocks), q2b::kNormThreads, 0, st>>>(
      x_out, static_cast<uint4*>(xb_out), rstd_out, reinterpret_cast<unsigned*>(amax), x,
      static_cast<const uint4*>(y), w, rows, d, eps);
  Q2B_CUDA(cudaGetLastError());
  return Q2B_OK;
}

int q2b_rmsnorm_bwd(float* dx, void* dy, float* dw_partial, int64_t partial_rows, const float* g, const void* gb,
                    const void* y, const float* rstd, const float* w, int64_t rows, int d, void* stream) {
  Q2B_REQUIRE_PTR(dx);
  Q2B_REQUIRE_PTR(dy);
  Q2B_REQUIRE_PTR(dw_partial);
  Q2B_REQUIRE_PTR(g);
  Q2B_REQUIRE_PTR(y);
  Q2B_REQUIRE_PTR(w);
  Q2B_REQUIRE_NONNULL(rstd);
  if (gb != nullptr && !aligned16(gb)) return fail(Q2B_ERR_INVALID, "Pointer `gb` is not aligned to 16 bytes");
  if (rows <= 0 || d <= 0 || d % 8 != 0 || d > 8 * q2b::kNormThreads * q2b::kNormMaxVecs)
    return fail(Q2B_ERR_INVALID, "rmsnorm_bwd: d must be a positive multiple of 8 up to %d",
                8 * q2b::kNormThreads * q2b::kNormMaxVecs);
  if (partial_rows <= 0 || partial_rows > rows)
    return fail(Q2B_ERR_INVALID, "rmsnorm_bwd: partial_rows must be in [1, rows]");
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  q2b::rmsnorm_bwd_kernel<<<static_cast<unsigned>(partial_rows), q2b::kNormThreads, 0,
                            static_cast<cudaStream_t>(stream)>>>(dx, static_cast<uint4*>(dy), dw_partial, g,
                                                                 static_cast<const uint4*>(gb),
                                                                 static_cast<const uint4*>(y), rstd, w, rows, d);
  Q2B_CUDA(cudaGetLastError());
  return Q2B_OK;
}

int q2b_relu2_bwd(void* da, const void* a, const void* g, int64_t n, void* stream) {
  Q2B_REQUIRE_PTR(da);
  Q2B_REQUIRE_PTR(a);
  Q2B_REQUIRE_PTR(g);
  if (n <= 0 || n % 8 != 0) return fail(Q2B_ERR_INVALID, "relu2_bwd: n must be a positive multiple of 8");
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  const int64_t nvec = n / 8;
  const int64_t blocks = std::min<int64_t>((nvec + 255) / 256, static_cast<int64_t>(sms) * 8);
  q2b::relu2_bwd_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint4*>(da), static_cast<const uint4*>(a), static_cast<const uint4*>(g), nvec);
  Q2B_CUDA(cudaGetLastError());
  return Q2B_OK;
}

int q2b_softmax_xent_bf16(void* logits, float* row_loss, const int64_t* targets, float inv_n, int64_t rows, int64_t V,
                          void* stream) {
  Q2B_REQUIRE_PTR(logits);
  Q2B_REQUIRE_NONNULL(row_loss);
  Q2B_REQUIRE_NONNULL(targets);
  if (rows <= 0 || rows >= (int64_t(1) << 31)) return fail(Q2B_ERR_INVALID, "softmax_xent: rows must be in [1, 2^31)");
  if (V <= 0 || V % 8 != 0) return fail(Q2B_ERR_INVALID, "softmax_xent: V must be a positive multiple of 8");
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  q2b::softmax_xent_kernel<<<static_cast<unsigned>(rows), q2b::kXentThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint4*>(logits), row_loss, targets, inv_n, V);
  Q2B_CUDA(cudaGetLastError());
  return Q2B_OK;
}

int q2b_watchdog_poll(unsigned* host_word, void* stream) {
  Q2B_REQUIRE_NONNULL(host_word);
  Q2B_CUDA(cudaMemcpyFromSymbolAsync(host_word, q2b::g_watchdog, sizeof(unsigned), 0, cudaMemcpyDeviceToHost,
                                     static_cast<cudaStream_t>(stream)));
  return Q2B_OK;
}

int q2b_watchdog_selftest(int64_t wait_cycles, void* stream) {
  if (wait_cycles < 1024 || wait_cycles > q2b::kWaitCycles)
    return fail(Q2B_ERR_INVALID, "watchdog_selftest: wait_cycles must be in [1024, %lld]", q2b::kWaitCycles);
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  q2b::watchdog_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(wait_cycles);
  Q2B_CUDA(cudaGetLastError());
  return Q2B_OK;
}

int q2b_abs_max(float* out, const void* x, int64_t n, void* stream) {
  Q2B_REQUIRE_PTR(x);
  Q2B_REQUIRE_NONNULL(out);
  if (n <= 0) return fail(Q2B_ERR_INVALID, "abs_max: n must be positive");
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Q2B_CUDA(cudaMemsetAsync(out, 0, sizeof(float), st));
  const int64_t nvec = n / 8;
  const int64_t want = (nvec + 255) / 256;
  const int blocks = static_cast<int>(want < 1 ? 1 : (want < int64_t(sms) * 8 ? want : int64_t(sms) * 8));
  q2b::abs_max_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<unsigned*>(out), static_cast<const uint4*>(x), nvec,
                                              static_cast<const uint16_t*>(x) + nvec * 8, n - nvec * 8);
  Q2B_CUDA(cudaGetLastError());
  return Q2B_OK;
}

int q2b_adamw_step(float* w, float* exp_avg, float* exp_avg_sq, const void* grad, int grad_bf16, int64_t n,
                   float lr, float beta1, float beta2, float eps, float weight_decay, int64_t step, void* w_bf16,
                   float* amax, void* stream) {
  Q2B_REQUIRE_NONNULL(w);
  Q2B_REQUIRE_NONNULL(exp_avg);
  Q2B_REQUIRE_NONNULL(exp_avg_sq);
  Q2B_REQUIRE_NONNULL(grad);
  if (n <= 0) return fail(Q2B_ERR_INVALID, "adamw: n must be positive");
  if (step < 1) return fail(Q2B_ERR_INVALID, "adamw: step must be >= 1 (got %lld)", (long long)step);
  if (!(beta1 >= 0.f && beta1 < 1.f) || !(beta2 >= 0.f && beta2 < 1.f))
    return fail(Q2B_ERR_INVALID, "adamw: betas must lie in [0, 1)");
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  q2b::AdamParams a;
  const double bc1 = 1.0 - std::pow(static_cast<double>(beta1), static_cast<double>(step));
  const double bc2 = 1.0 - std::pow(static_cast<double>(beta2), static_cast<double>(step));
  a.lr_wd = lr * weight_decay;
  a.beta1 = beta1;
  a.one_minus_beta1 = 1.f - beta1;
  a.beta2 = beta2;
  a.one_minus_beta2 = 1.f - beta2;
  a.step_size = static_cast<float>(lr / bc1);
  a.bc2_sqrt = static_cast<float>(std::sqrt(bc2));
  a.eps = eps;
  auto al = [](const void* p, uintptr_t m) { return (reinterpret_cast<uintptr_t>(p) & m) == 0; };
  const int vec = al(w, 15) && al(exp_avg, 15) && al(exp_avg_sq, 15) && al(grad, grad_bf16 ? 7 : 15) &&
                  (w_bf16 == nullptr || al(w_bf16, 7));
  if (amax != nullptr) Q2B_CUDA(cudaMemsetAsync(amax, 0, sizeof(float), st));
  const int64_t want = (n / 4 + 255) / 256;
  const int blocks = static_cast<int>(want < 1 ? 1 : (want < int64_t(sms) * 8 ? want : int64_t(sms) * 8));
  auto* wb = static_cast<__nv_bfloat16*>(w_bf16);
  auto* am = reinterpret_cast<unsigned*>(amax);
  if (grad_bf16)
    q2b::adamw_amax_kernel<true><<<blocks, 256, 0, st>>>(w, exp_avg, exp_avg_sq, grad, n, a, wb, am, vec);
  else
    q2b::adamw_amax_kernel<false><<<blocks, 256, 0, st>>>(w, exp_avg, exp_avg_sq, grad, n, a, wb, am, vec);
  Q2B_CUDA(cudaGetLastError());
  return Q2B_OK;
}

int q2b_relu2_abs_max(void* y, float* amax, const void* a, int64_t n, void* stream) {
  Q2B_REQUIRE_PTR(y);
  Q2B_REQUIRE_PTR(a);
  Q2B_REQUIRE_NONNULL(amax);
  if (n <= 0) return fail(Q2B_ERR_INVALID, "relu2_abs_max: n must be positive");
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Q2B_CUDA(cudaMemsetAsync(amax, 0, sizeof(float), st));
  const int64_t nvec = n / 8;
  const int64_t want = (nvec + 255) / 256;
  const int blocks = static_cast<int>(want < 1 ? 1 : (want < int64_t(sms) * 8 ? want : int64_t(sms) * 8));
  q2b::relu2_abs_max_kernel<<<blocks, 256, 0, st>>>(static_cast<uint4*>(y), reinterpret_cast<unsigned*>(amax),
                                                    static_cast<const uint4*>(a), nvec,
                                                    static_cast<uint16_t*>(y) + nvec * 8,
                                                    static_cast<const uint16_t*>(a) + nvec * 8, n - nvec * 8);
  Q2B_CUDA(cudaGetLastError());
  return Q2B_OK;
}

static int quant_fwd_impl(void* codes, void* sf, float* ts, const void* x, const float* amax, float scale_override,
                          int64_t rows, int64_t cols, int mode, void* stream, bool ragged) {
  if (mode != Q2B_MODE_RNE && mode != Q2B_MODE_FOUR_SIX)
    return fail(Q2B_ERR_INVALID, "quant_fwd: unknown mode %d", mode);
  const char* name = mode == Q2B_MODE_RNE ? "rtn_fp4" : "four_six_fp4";
  if (cols % 128 != 0) return fail(Q2B_ERR_INVALID, "%s: cols must be divisible by 128", name);
  if (ragged) {
    if (rows <= 0) return fail(Q2B_ERR_INVALID, "%s: rows must be positive", name);
  } else if (int r = check_dims128(name, rows, cols)) {
    return r;
  }
  Q2B_REQUIRE_PTR(codes);
  Q2B_REQUIRE_PTR(sf);
  Q2B_REQUIRE_PTR(x);
  Q2B_REQUIRE_NONNULL(ts);
  Q2B_REQUIRE_NONNULL(amax);
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t ngroups = rows * cols / 16;
  if (ngroups >= (int64_t(1) << 32)) return fail(Q2B_ERR_INVALID, "%s: tensor too large", name);
  if ((reinterpret_cast<uintptr_t>(x) & 31u) != 0)
    return fail(Q2B_ERR_INVALID, "Pointer `x` is not aligned to 32 bytes");
  const uint32_t gpr = static_cast<uint32_t>(cols / 16);
  // ceil(2^64 / gpr): floor(g * magic / 2^64) == g / gpr exactly for every 32-bit g
  const uint64_t magic = ~uint64_t(0) / gpr + 1;
  const int64_t want = (ngroups + 255) / 256;
  const int blocks = static_cast<int>(want < int64_t(sms) * 8 ? want : int64_t(sms) * 8);
  if (mode == Q2B_MODE_FOUR_SIX)
    q2b::quant_fwd_v2_kernel<true><<<blocks, 256, 0, st>>>(
        static_cast<uint2*>(codes), static_cast<uint8_t*>(sf), ts, static_cast<const uint16_t*>(x), amax,
        scale_override, static_cast<uint32_t>(ngroups), gpr, magic);
  else
    q2b::quant_fwd_v2_kernel<false><<<blocks, 256, 0, st>>>(
        static_cast<uint2*>(codes), static_cast<uint8_t*>(sf), ts, static_cast<const uint16_t*>(x), amax,
        scale_override, static_cast<uint32_t>(ngroups), gpr, magic);
  Q2B_CUDA(cudaGetLastError());
  return Q2B_OK;
}

int q2b_quant_fwd(void* codes, void* sf, float* ts, const void* x, const float* amax, float scale_override,
                  int64_t rows, int64_t cols, int mode, void* stream) {
  return quant_fwd_impl(codes, sf, ts, x, amax, scale_override, rows, cols, mode, stream, false);
}

int q2b_quant_fwd_ragged(void* codes, void* sf, float* ts, const void* x, const float* amax, float scale_override,
                         int64_t rows, int64_t cols, int mode, void* stream) {
  return quant_fwd_impl(codes, sf, ts, x, amax, scale_override, rows, cols, mode, stream, true);
}

int q2b_quant_rows_fused(void* codes, void* sf, float* ts, const void* x, float scale_override, int64_t rows,
                         int64_t cols, int mode, void* stream) {
  if (mode != Q2B_MODE_RNE && mode != Q2B_MODE_FOUR_SIX)
    return fail(Q2B_ERR_INVALID, "quant_rows_fused: unknown mode %d", mode);
  if (cols <= 0 || cols % 128 != 0) return fail(Q2B_ERR_INVALID, "quant_rows_fused: cols must be divisible by 128");
  if (rows <= 0) return fail(Q2B_ERR_INVALID, "quant_rows_fused: rows must be positive");
  Q2B_REQUIRE_PTR(codes);
  Q2B_REQUIRE_PTR(sf);
  Q2B_REQUIRE_PTR(x);
  Q2B_REQUIRE_NONNULL(ts);
  if ((reinterpret_cast<uintptr_t>(x) & 31u) != 0)
    return fail(Q2B_ERR_INVALID, "Pointer `x` is not aligned to 32 bytes");
  const int64_t ngroups = rows * cols / 16;
  if (ngroups >= (int64_t(1) << 31)) return fail(Q2B_ERR_INVALID, "quant_rows_fused: tensor too large");
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  const uint32_t gpr = static_cast<uint32_t>(cols / 16);
  const uint64_t magic = ~uint64_t(0) / gpr + 1;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = q2b::kRowsClusterCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(q2b::kRowsClusterCtas, 1, 1);
  cfg.blockDim = dim3(q2b::kRowsThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto* c = static_cast<uint2*>(codes);
  auto* s = static_cast<uint8_t*>(sf);
  auto* xx = static_cast<const uint16_t*>(x);
  if (mode == Q2B_MODE_FOUR_SIX)
    Q2B_CUDA(cudaLaunchKernelEx(&cfg, q2b::quant_rows_cluster_kernel<true>, c, s, ts, xx, scale_override,
                                static_cast<uint32_t>(rows), static_cast<uint32_t>(ngroups), gpr, magic));
  else
    Q2B_CUDA(cudaLaunchKernelEx(&cfg, q2b::quant_rows_cluster_kernel<false>, c, s, ts, xx, scale_override,
                                static_cast<uint32_t>(rows), static_cast<uint32_t>(ngroups), gpr, magic));
  return Q2B_OK;
}

int q2b_rht_eden(void* codes, void* sf, float* ts, void* scratch, unsigned* scratch_max, const void* h, int h_rows,
                 const void* x, uint64_t seed, float fp4_max, float fp8_max, int64_t M, int64_t N, int transpose,
                 void* stream) {
  if (int r = check_dims128("rht128_eden", M, N)) return r;
  Q2B_REQUIRE_PTR(codes);
  Q2B_REQUIRE_PTR(sf);
  Q2B_REQUIRE_PTR(scratch);
  Q2B_REQUIRE_PTR(x);
  Q2B_REQUIRE_NONNULL(ts);
  Q2B_REQUIRE_NONNULL(scratch_max);
  if (int r = rht_check_h(h, h_rows)) return r;
  if (!(fp4_max > 0.f) || !(fp8_max > 0.f)) return fail(Q2B_ERR_INVALID, "fp4_max and fp8_max must be positive");
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap tmap;
  if (int r = make_tmap(&tmap, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, 64, 128)) return r;
  q2b::RhtParams p{};
  p.M = M;
  p.N = N;
  p.h = static_cast<const uint16_t*>(h);
  p.h_rows = h_rows;
  p.inv_fp4_max = 1.f / fp4_max;
  Q2B_CUDA(cudaMemsetAsync(scratch_max, 0, sizeof(unsigned), st));
  int r;
  if (transpose) {
    p.codes_c = static_cast<uint8_t*>(codes);
    p.scratch_c = static_cast<uint16_t*>(scratch);
    p.max_c = scratch_max;
    r = launch_rht<q2b::kInBf16, q2b::kOutCols>(tmap, p, sms, st);
  } else {
    p.codes_r = static_cast<uint8_t*>(codes);
    p.scratch_r = static_cast<uint16_t*>(scratch);
    p.max_r = scratch_max;
    r = launch_rht<q2b::kInBf16, q2b::kOutRows>(tmap, p, sms, st);
  }
  if (r) return r;
  return launch_sr(sf, ts, scratch, scratch_max, fp8_max, seed, M * N / 16, sms, st);
}

// ---------------------------------------------------------------------------
// Allocation-free q2b_rht_eden.  Its scratch (bf16 pre-rounding scales, then
// the uint32 max word at the end) is this file-scope device array; host code
// must not pass the symbol itself to a kernel -- on the host it names a
// stand-in, not device memory -- but the address cudaGetSymbolAddress returns
// for the current device.
}  // extern "C"

namespace {
static __device__ __align__(256) unsigned char g_noalloc_scratch[Q2B_NOALLOC_SCRATCH_BYTES + 256];
void* g_noalloc_addr[kMaxDevices] = {};
CUcontext g_noalloc_ctx[kMaxDevices] = {};
std::mutex g_noalloc_mu;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn g_ctx_get_current = nullptr;

// The device address of g_noalloc_scratch on device `dev`, looked up with
// cudaGetSymbolAddress while that device is current and cached together with
// the current context: if the context changes (cudaDeviceReset, or a context
// torn down and created again reloads the module), the address is looked up
// again instead of reusing a stale one.
int noalloc_scratch(int dev, unsigned char** out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_ctx_get_current == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    Q2B_CUDA(cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q));
    if (fn == nullptr || q != cudaDriverEntryPointSuccess)
      return fail(Q2B_ERR_CUDA, "cuCtxGetCurrent is not available from the driver");
    g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
  }
  CUcontext ctx = nullptr;
  if (g_ctx_get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr)
    return fail(Q2B_ERR_CUDA, "no current CUDA context for the static scratch lookup");
  if (g_noalloc_addr[dev] == nullptr || g_noalloc_ctx[dev] != ctx) {
    void* p = nullptr;
    Q2B_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    if (p == nullptr) return fail(Q2B_ERR_CUDA, "cudaGetSymbolAddress returned a null scratch address");
    g_noalloc_addr[dev] = p;
    g_noalloc_ctx[dev] = ctx;
  }
  *out = static_cast<unsigned char*>(g_noalloc_addr[dev]);
  return Q2B_OK;
}
}  // namespace

extern "C" {

int q2b_rht_eden_noalloc(void* codes, void* sf, float* ts, const void* h, int h_rows, const void* x, uint64_t seed,
                         float fp4_max, float fp8_max, int64_t M, int64_t N, int transpose, void* stream) {
  if (int r = check_dims128("rht128_eden_noalloc", M, N)) return r;
  if (M * N > Q2B_NOALLOC_MAX_ELEMS)
    return fail(Q2B_ERR_INVALID,
                "rht128_eden_noalloc: M*N = %lld exceeds the static scratch limit of %lld elements "
                "(use q2b_rht_eden with caller-provided scratch)",
                static_cast<long long>(M * N), static_cast<long long>(Q2B_NOALLOC_MAX_ELEMS));
  Q2B_REQUIRE_PTR(codes);
  Q2B_REQUIRE_PTR(sf);
  Q2B_REQUIRE_PTR(x);
  Q2B_REQUIRE_NONNULL(ts);
  if (int r = rht_check_h(h, h_rows)) return r;
  if (!(fp4_max > 0.f) || !(fp8_max > 0.f)) return fail(Q2B_ERR_INVALID, "fp4_max and fp8_max must be positive");
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  unsigned char* scratch = nullptr;
  if (int r = noalloc_scratch(dev, &scratch)) return r;
  unsigned* scratch_max = reinterpret_cast<unsigned*>(scratch + Q2B_NOALLOC_SCRATCH_BYTES);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap tmap;
  if (int r = make_tmap(&tmap, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, 64, 128)) return r;
  q2b::RhtParams p{};
  p.M = M;
  p.N = N;
  p.h = static_cast<const uint16_t*>(h);
  p.h_rows = h_rows;
  p.inv_fp4_max = 1.f / fp4_max;
  Q2B_CUDA(cudaMemsetAsync(scratch_max, 0, sizeof(unsigned), st));
  int r;
  if (transpose) {
    p.codes_c = static_cast<uint8_t*>(codes);
    p.scratch_c = reinterpret_cast<uint16_t*>(scratch);
    p.max_c = scratch_max;
    r = launch_rht<q2b::kInBf16, q2b::kOutCols>(tmap, p, sms, st);
  } else {
    p.codes_r = static_cast<uint8_t*>(codes);
    p.scratch_r = reinterpret_cast<uint16_t*>(scratch);
    p.max_r = scratch_max;
    r = launch_rht<q2b::kInBf16, q2b::kOutRows>(tmap, p, sms, st);
  }
  if (r) return r;
  return launch_sr(sf, ts, scratch, scratch_max, fp8_max, seed, M * N / 16, sms, st);
}

int q2b_rht_eden_dual(void* codes_r, void* sf_r, float* ts_r, void* scratch_r, unsigned* max_r, void* codes_c,
                      void* sf_c, float* ts_c, void* scratch_c, unsigned* max_c, const void* h, int h_rows,
                      const void* x, uint64_t seed_r, uint64_t seed_c, float fp4_max, float fp8_max, int64_t M,
                      int64_t N, void* stream) {
  if (int r = check_dims128("rht128_eden_dual", M, N)) return r;
  Q2B_REQUIRE_PTR(codes_r);
  Q2B_REQUIRE_PTR(sf_r);
  Q2B_REQUIRE_PTR(scratch_r);
  Q2B_REQUIRE_PTR(codes_c);
  Q2B_REQUIRE_PTR(sf_c);
  Q2B_REQUIRE_PTR(scratch_c);
  Q2B_REQUIRE_PTR(x);
  Q2B_REQUIRE_NONNULL(ts_r);
  Q2B_REQUIRE_NONNULL(ts_c);
  Q2B_REQUIRE_NONNULL(max_r);
  Q2B_REQUIRE_NONNULL(max_c);
  if (max_r == max_c) return fail(Q2B_ERR_INVALID, "rht128_eden_dual: the two outputs need distinct max words");
  if (int r = rht_check_h(h, h_rows)) return r;
  if (!(fp4_max > 0.f) || !(fp8_max > 0.f)) return fail(Q2B_ERR_INVALID, "fp4_max and fp8_max must be positive");
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap tmap;
  if (int r = make_tmap(&tmap, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, 64, 128)) return r;
  q2b::RhtParams p{};
  p.M = M;
  p.N = N;
  p.h = static_cast<const uint16_t*>(h);
  p.h_rows = h_rows;
  p.inv_fp4_max = 1.f / fp4_max;
  p.codes_r = static_cast<uint8_t*>(codes_r);
  p.scratch_r = static_cast<uint16_t*>(scratch_r);
  p.max_r = max_r;
  p.codes_c = static_cast<uint8_t*>(codes_c);
  p.scratch_c = static_cast<uint16_t*>(scratch_c);
  p.max_c = max_c;
  Q2B_CUDA(cudaMemsetAsync(max_r, 0, sizeof(unsigned), st));
  Q2B_CUDA(cudaMemsetAsync(max_c, 0, sizeof(unsigned), st));
  if (int r = launch_rht<q2b::kInBf16, q2b::kOutBoth>(tmap, p, sms, st)) return r;
  if (int r = launch_sr(sf_r, ts_r, scratch_r, max_r, fp8_max, seed_r, M * N / 16, sms, st)) return r;
  return launch_sr(sf_c, ts_c, scratch_c, max_c, fp8_max, seed_c, M * N / 16, sms, st);
}

int q2b_rht_requant(void* codes, void* sf, float* ts, void* scratch, unsigned* scratch_max, const void* h,
                    int h_rows, const void* x_codes, const void* x_sf, const float* x_ts, uint64_t seed,
                    float fp4_max, float fp8_max, int64_t M, int64_t N, void* stream) {
  if (int r = check_dims128("rht128_requant", M, N)) return r;
  Q2B_REQUIRE_PTR(codes);
  Q2B_REQUIRE_PTR(sf);
  Q2B_REQUIRE_PTR(scratch);
  Q2B_REQUIRE_PTR(x_codes);
  Q2B_REQUIRE_PTR(x_sf);
  Q2B_REQUIRE_NONNULL(x_ts);
  Q2B_REQUIRE_NONNULL(ts);
  Q2B_REQUIRE_NONNULL(scratch_max);
  if (int r = rht_check_h(h, h_rows)) return r;
  if (!(fp4_max > 0.f) || !(fp8_max > 0.f)) return fail(Q2B_ERR_INVALID, "fp4_max and fp8_max must be positive");
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  q2b::RhtParams p{};
  p.M = M;
  p.N = N;
  p.x_codes = static_cast<const uint8_t*>(x_codes);
  p.x_sf = static_cast<const uint8_t*>(x_sf);
  p.x_ts = x_ts;
  p.h = static_cast<const uint16_t*>(h);
  p.h_rows = h_rows;
  p.inv_fp4_max = 1.f / fp4_max;
  p.codes_c = static_cast<uint8_t*>(codes);
  p.scratch_c = static_cast<uint16_t*>(scratch);
  p.max_c = scratch_max;
  Q2B_CUDA(cudaMemsetAsync(scratch_max, 0, sizeof(unsigned), st));
  CUtensorMap tmap;  // the codes, [M, N/2] bytes, 64-byte x 128-row boxes
  if (int r = make_tmap(&tmap, x_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N / 2, M, 64, 128,
                        CU_TENSOR_MAP_SWIZZLE_NONE))
    return r;
  if (int r = launch_rht<q2b::kInFp4, q2b::kOutCols>(tmap, p, sms, st)) return r;
  return launch_sr(sf, ts, scratch, scratch_max, fp8_max, seed, M * N / 16, sms, st);
}

}  // extern "C"

namespace {

// Output tiles of the 1-SM kernel at BN=128 and the K split that fills the
// SMs when there are too few of them (decode-sized M).  A split keeps at
// least two 256-wide K blocks per unit.
struct SplitPlan {
  int64_t tiles;
  int splits;
};

SplitPlan plan_split(int64_t m_valid, int64_t N, int64_t K, int sms) {
  const int64_t tiles = ((m_valid + 127) / 128) * (N / 128);
  const int64_t nkb = (K + 255) / 256;
  int64_t splits = 1;
  if (tiles * 2 <= sms) {
    splits = sms / tiles;
    if (splits > nkb / 2) splits = nkb / 2;
    if (splits < 1) splits = 1;
  }
  return {tiles, static_cast<int>(splits)};
}

int64_t split_ws_bytes(const SplitPlan& sp) {
  if (sp.splits <= 1) return 0;
  // fp32 tile slabs, then one counter per (tile, epilogue warp)
  return sp.tiles * 128 * 128 * 4 + sp.tiles * q2b::GemmCfg<128>::kEpiWarps * 4;
}

// Whether the 2-SM pair kernel takes this problem (256-aligned, enough tiles to fill the pairs).
// The pair kernel covers M and N in 256-wide tiles; a last half tile (M or N = 128 mod 256) is
// read as zeros past the end by TMA (A, B and both scale maps are bounded by the real extent)
// and its stores are clipped to the real extent, so multiples of 128 suffice.
bool takes_pair_kernel(int64_t m_valid, int64_t N, int sms, const void* D) {
  const int64_t M = (m_valid + 127) / 128 * 128;
  return m_valid % 128 == 0 && N % 128 == 0 && sms >= 2 && ((M + 255) / 256) * ((N + 255) / 256) * 2 >= sms &&
         (reinterpret_cast<uintptr_t>(D) & 15u) == 0;
}

int gemm_launch(void* D, const void* A, const void* B, const void* sfa, const void* sfb, const float* alpha,
                const float* alpha_b, int64_t m_valid, int64_t N, int64_t K, void* ws, int64_t ws_bytes,
                void* stream, bool out_f32 = false, int epi = q2b::kEpiBf16, void* D2 = nullptr,
                const void* aux = nullptr, float* amax = nullptr) {
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t M = (m_valid + 127) / 128 * 128;
  CUtensorMap ta, tb;
  q2b::GemmParams p{M, N, K, static_cast<const uint8_t*>(sfa), static_cast<const uint8_t*>(sfb), alpha, alpha_b,
                    D, static_cast<const uint16_t*>(aux), reinterpret_cast<unsigned*>(amax), m_valid, 1, nullptr,
                    nullptr};
  if (out_f32) epi = q2b::kEpiF32;
  if (int r = make_tmap(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, m_valid, 128, 128)) return r;
#ifndef Q2B_GEMM_NO_2SM
  if (takes_pair_kernel(m_valid, N, sms, D)) {
    // 2-SM pairs: 256x256 tiles, one cluster of two CTAs per SM pair; D written by TMA stores.
    // Long K: tiles in groups of 8 row tiles, so one wave's K panels fit L2 (a 256-row panel
    // is 128 x K bytes: 2 MB at K = 16384, and row-major waves touch every column panel)
    p.raster_rows = K >= 16384 ? 8 : 1;
    CUtensorMap tsa, tsb, td;
    // store boxes of 32 rows x 64 bytes (32 bf16 or 16 fp32 columns), 64-byte swizzle
    CUtensorMap td2;
    if (int r = out_f32 ? make_tmap(&td, D, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, M, 16, 32, CU_TENSOR_MAP_SWIZZLE_64B)
                        : make_tmap(&td, D, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
      return r;
    if (epi == q2b::kEpiRelu2) {
      if (int r = make_tmap(&td2, D2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
        return r;
    } else if (epi == q2b::kEpiRelu2Bwd) {
      // the pre-activation, loaded box by box in the store's layout
      if (int r = make_tmap(&td2, aux, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
        return r;
    } else {
      td2 = td;
    }
    if (int r = make_tmap(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, N, 128, 128)) return r;
    if (int r = make_tmap(&tsa, sfa, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 256, M * K / 16 / 256, 256, 8,
                          CU_TENSOR_MAP_SWIZZLE_NONE))
      return r;
    if (int r = make_tmap(&tsb, sfb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 256, N * K / 16 / 256, 256, 8,
                          CU_TENSOR_MAP_SWIZZLE_NONE))
      return r;
    const int64_t tiles = ((M + 255) / 256) * ((N + 255) / 256);
    const int64_t pairs = tiles < sms / 2 ? tiles : sms / 2;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
    cfg.blockDim = dim3(q2b::Gemm2Cfg::kThreads, 1, 1);
    cfg.dynamicSmemBytes = q2b::Gemm2Cfg::kSmemBytes;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    switch (epi) {
      case q2b::kEpiF32:
        Q2B_CUDA(cudaLaunchKernelEx(&cfg, q2b::gemm_nvfp4_2sm_kernel<q2b::kEpiF32>, ta, tb, tsa, tsb, td, td2, p));
        break;
      case q2b::kEpiRelu2:
        Q2B_CUDA(cudaLaunchKernelEx(&cfg, q2b::gemm_nvfp4_2sm_kernel<q2b::kEpiRelu2>, ta, tb, tsa, tsb, td, td2, p));
        break;
      case q2b::kEpiRelu2Bwd:
        Q2B_CUDA(cudaLaunchKernelEx(&cfg, q2b::gemm_nvfp4_2sm_kernel<q2b::kEpiRelu2Bwd>, ta, tb, tsa, tsb, td, td2, p));
        break;
      case q2b::kEpiBf16Add:
        Q2B_CUDA(cudaLaunchKernelEx(&cfg, q2b::gemm_nvfp4_2sm_kernel<q2b::kEpiBf16Add>, ta, tb, tsa, tsb, td, td2, p));
        break;
      default:
        Q2B_CUDA(cudaLaunchKernelEx(&cfg, q2b::gemm_nvfp4_2sm_kernel<q2b::kEpiBf16>, ta, tb, tsa, tsb, td, td2, p));
    }
    return Q2B_OK;
  }
#endif
  const bool accum = epi == q2b::kEpiBf16Add;
  const SplitPlan sp = plan_split(m_valid, N, K, sms);
  const bool split = !accum && sp.splits > 1 && ws != nullptr && ws_bytes >= split_ws_bytes(sp);
  if (N % 256 == 0 && !split && (M / 128) * (N / 256) * 2 >= sms) {
    if (int r = make_tmap(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, N, 128, 256)) return r;
    const int64_t tiles = (M / 128) * (N / 256);
    const int grid = static_cast<int>(tiles < sms ? tiles : sms);
    if (out_f32)
      q2b::gemm_nvfp4_kernel<256, true><<<grid, q2b::GemmCfg<256>::kThreads, q2b::GemmCfg<256>::kSmemBytes, st>>>(ta, tb, p);
    else if (accum)
      q2b::gemm_nvfp4_kernel<256, false, true><<<grid, q2b::GemmCfg<256>::kThreads, q2b::GemmCfg<256>::kSmemBytes, st>>>(ta, tb, p);
    else
      q2b::gemm_nvfp4_kernel<256, false><<<grid, q2b::GemmCfg<256>::kThreads, q2b::GemmCfg<256>::kSmemBytes, st>>>(ta, tb, p);
  } else {
    if (int r = make_tmap(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, N, 128, 128)) return r;
    int64_t units = sp.tiles;
    if (split) {
      p.splits = sp.splits;
      p.ws = static_cast<float*>(ws);
      p.counters = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(ws) + sp.tiles * 128 * 128 * 4);
      units = sp.tiles * sp.splits;
    }
    const int grid = static_cast<int>(units < sms ? units : sms);
    if (out_f32)
      q2b::gemm_nvfp4_kernel<128, true><<<grid, q2b::GemmCfg<128>::kThreads, q2b::GemmCfg<128>::kSmemBytes, st>>>(ta, tb, p);
    else if (accum)
      q2b::gemm_nvfp4_kernel<128, false, true><<<grid, q2b::GemmCfg<128>::kThreads, q2b::GemmCfg<128>::kSmemBytes, st>>>(ta, tb, p);
    else
      q2b::gemm_nvfp4_kernel<128, false><<<grid, q2b::GemmCfg<128>::kThreads, q2b::GemmCfg<128>::kSmemBytes, st>>>(ta, tb, p);
  }
  Q2B_CUDA(cudaGetLastError());
  return Q2B_OK;
}

int check_gemm_args(const char* name, void* D, const void* A, const void* B, const void* sfa, const void* sfb,
                    const float* alpha, int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return fail(Q2B_ERR_INVALID, "%s: empty problem", name);
  if (N % 128 != 0) return fail(Q2B_ERR_INVALID, "%s: N must be divisible by 128 (got %lld)", name, (long long)N);
  if (K % 64 != 0) return fail(Q2B_ERR_INVALID, "%s: K must be divisible by 64 (got %lld)", name, (long long)K);
  Q2B_REQUIRE_PTR(D);
  Q2B_REQUIRE_PTR(A);
  Q2B_REQUIRE_PTR(B);
  Q2B_REQUIRE_PTR(sfa);
  Q2B_REQUIRE_PTR(sfb);
  Q2B_REQUIRE_NONNULL(alpha);
  return Q2B_OK;
}

}  // namespace

extern "C" {

int q2b_gemm_nvfp4(void* D, const void* A, const void* B, const void* sfa, const void* sfb, const float* alpha,
                   int64_t M, int64_t N, int64_t K, void* stream) {
  if (M > 0 && M % 128 != 0) return fail(Q2B_ERR_INVALID, "fp4_mm: M must be divisible by 128 (got %lld)", (long long)M);
  if (int r = check_gemm_args("fp4_mm", D, A, B, sfa, sfb, alpha, M, N, K)) return r;
  return gemm_launch(D, A, B, sfa, sfb, alpha, nullptr, M, N, K, nullptr, 0, stream);
}

int q2b_gemm_nvfp4_f32(float* D, const void* A, const void* B, const void* sfa, const void* sfb, const float* alpha,
                       int64_t M, int64_t N, int64_t K, void* stream) {
  if (M > 0 && M % 128 != 0)
    return fail(Q2B_ERR_INVALID, "fp4_mm_f32: M must be divisible by 128 (got %lld)", (long long)M);
  if (int r = check_gemm_args("fp4_mm_f32", D, A, B, sfa, sfb, alpha, M, N, K)) return r;
  return gemm_launch(D, A, B, sfa, sfb, alpha, nullptr, M, N, K, nullptr, 0, stream, true);
}

int q2b_gemm_nvfp4_add(void* D, const void* A, const void* B, const void* sfa, const void* sfb, const float* alpha,
                       int64_t M, int64_t N, int64_t K, void* stream) {
  if (M > 0 && M % 128 != 0)
    return fail(Q2B_ERR_INVALID, "fp4_mm_add: M must be divisible by 128 (got %lld)", (long long)M);
  if (int r = check_gemm_args("fp4_mm_add", D, A, B, sfa, sfb, alpha, M, N, K)) return r;
  return gemm_launch(D, A, B, sfa, sfb, alpha, nullptr, M, N, K, nullptr, 0, stream, false, q2b::kEpiBf16Add);
}

int q2b_gemm_nvfp4_relu2(void* A_out, void* H_out, float* amax, const void* A, const void* B, const void* sfa,
                         const void* sfb, const float* alpha, int64_t M, int64_t N, int64_t K, void* stream) {
  if (M > 0 && M % 128 != 0)
    return fail(Q2B_ERR_INVALID, "fp4_mm_relu2: M must be divisible by 128 (got %lld)", (long long)M);
  if (int r = check_gemm_args("fp4_mm_relu2", A_out, A, B, sfa, sfb, alpha, M, N, K)) return r;
  Q2B_REQUIRE_PTR(H_out);
  Q2B_REQUIRE_NONNULL(amax);
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Q2B_CUDA(cudaMemsetAsync(amax, 0, sizeof(float), st));
  if (takes_pair_kernel(M, N, sms, A_out))
    return gemm_launch(A_out, A, B, sfa, sfb, alpha, nullptr, M, N, K, nullptr, 0, stream, false, q2b::kEpiRelu2,
                       H_out, nullptr, amax);
  // other shapes: the GEMM, then the one-pass ReLU^2 + abs-max kernel (same results)
  if (int r = gemm_launch(A_out, A, B, sfa, sfb, alpha, nullptr, M, N, K, nullptr, 0, stream)) return r;
  return q2b_relu2_abs_max(H_out, amax, A_out, M * N, stream);
}

int q2b_gemm_nvfp4_relu2_bwd(void* dA, const void* a, const void* A, const void* B, const void* sfa, const void* sfb,
                             const float* alpha, int64_t M, int64_t N, int64_t K, void* stream) {
  if (M > 0 && M % 128 != 0)
    return fail(Q2B_ERR_INVALID, "fp4_mm_relu2_bwd: M must be divisible by 128 (got %lld)", (long long)M);
  if (int r = check_gemm_args("fp4_mm_relu2_bwd", dA, A, B, sfa, sfb, alpha, M, N, K)) return r;
  Q2B_REQUIRE_PTR(a);
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  if (takes_pair_kernel(M, N, sms, dA))
    return gemm_launch(dA, A, B, sfa, sfb, alpha, nullptr, M, N, K, nullptr, 0, stream, false, q2b::kEpiRelu2Bwd,
                       nullptr, a, nullptr);
  // other shapes: the GEMM into dA, then the ReLU^2 backward in place
  if (int r = gemm_launch(dA, A, B, sfa, sfb, alpha, nullptr, M, N, K, nullptr, 0, stream)) return r;
  return q2b_relu2_bwd(dA, a, dA, M * N, stream);
}

int64_t q2b_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0 || N % 128 != 0) return 0;
  int dev, sms;
  if (device_setup(&dev, &sms)) return -1;
  return split_ws_bytes(plan_split(M, N, K, sms));
}

int q2b_gemm_nvfp4_ex(void* D, const void* A, const void* B, const void* sfa, const void* sfb, const float* alpha,
                      const float* alpha_b, int64_t M, int64_t N, int64_t K, void* workspace, int64_t workspace_bytes,
                      void* stream) {
  if (int r = check_gemm_args("fp4_mm_ex", D, A, B, sfa, sfb, alpha, M, N, K)) return r;
  if (workspace != nullptr && (reinterpret_cast<uintptr_t>(workspace) & 15u) != 0)
    return fail(Q2B_ERR_INVALID, "fp4_mm_ex: workspace must be 16-byte aligned");
  return gemm_launch(D, A, B, sfa, sfb, alpha, alpha_b, M, N, K, workspace, workspace_bytes, stream);
}

int q2b_fp4_mma_peak(int iters, long long* cycles, void* stream) {
  if (iters <= 0 || iters % 4 != 0 || iters > (1 << 24)) return fail(Q2B_ERR_INVALID, "fp4_mma_peak: iters must be a positive multiple of 4 up to 2^24");
  int dev, sms;
  if (int r = device_setup(&dev, &sms)) return r;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(sms / 2 * 2), 1, 1);
  cfg.blockDim = dim3(q2b::PeakCfg::kThreads, 1, 1);
  cfg.dynamicSmemBytes = q2b::PeakCfg::kSmemBytes;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  Q2B_CUDA(cudaLaunchKernelEx(&cfg, q2b::fp4_mma_peak_kernel, iters, cycles));
  return Q2B_OK;
}

#ifdef Q2B_GEMM2_STATS
// Instrumented builds only: read and clear the pair GEMM's cycle counters.
int q2b_gemm2_stats(long long* out) {
  Q2B_CUDA(cudaMemcpyFromSymbol(out, q2b::g_gemm2_stats, sizeof(long long) * 12));
  long long zero[12] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
  Q2B_CUDA(cudaMemcpyToSymbol(q2b::g_gemm2_stats, zero, sizeof(zero)));
  return Q2B_OK;
}
#endif

#ifdef Q2B_RHT_STATS
// Instrumented builds only: read and clear the RHT/EDEN kernel's cycle counters.
int q2b_rht_stats(long long* out) {
  Q2B_CUDA(cudaMemcpyFromSymbol(out, q2b::g_rht_stats, sizeof(long long) * 12));
  long long zero[12] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
  Q2B_CUDA(cudaMemcpyToSymbol(q2b::g_rht_stats, zero, sizeof(zero)));
  return Q2B_OK;
}
#endif

}  // extern "C"
