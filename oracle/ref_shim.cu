// ref_shim.cu -- TEST INFRASTRUCTURE ONLY.
//
// Exposes the reference's own CUDA quantizers (compiled from the sources in
// the reference tree, see oracle/Makefile `ref` target) through a C ABI so
// the GPU tests can pin the CPU oracle against the real reference on a B200.
// Only the launcher declarations below are restated (from the signatures in
// quartet2/csrc/binding.cpp:29-56); nothing of the reference is copied.
#include <cuda_bf16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>
#include <cstdio>
#include <exception>

void rtn_fp4(__nv_fp4x4_e2m1* y, __nv_fp8_e4m3* sf, float* ts, const nv_bfloat16* x, const float* amax,
             float so, long rows, long cols);
void four_six_fp4(__nv_fp4x4_e2m1* y, __nv_fp8_e4m3* sf, float* ts, const nv_bfloat16* x, const float* amax,
                  float so, long rows, long cols);
void transform_rht128_eden(__nv_fp4x2_storage_t* y, __nv_fp8_e4m3* sf, float* ts, nv_bfloat16* scratch,
                           unsigned* max_scale, const nv_bfloat16* h, const nv_bfloat16* x, long seed, float fp4_max,
                           float fp8_max, int M, int N, bool transpose);
void group_transform_128_eden(__nv_fp4x2_storage_t* y, __nv_fp8_e4m3* sf, float* ts, nv_bfloat16* scratch,
                              unsigned* max_scale, const nv_bfloat16* h, const nv_bfloat16* x, long seed,
                              float fp4_max, float fp8_max, int M, int N, bool transpose);
void rht128_requant(__nv_fp4x2_storage_t* y, __nv_fp8_e4m3* sf, float* ts, nv_bfloat16* scratch,
                    unsigned* max_scale, const nv_bfloat16* h, const __nv_fp4x2_storage_t* x,
                    const __nv_fp8_e4m3* x_sf, const float* x_ts, long seed, float fp4_max, float fp8_max, int M,
                    int N);

static char g_msg[512];

template <typename F>
static int guarded(F f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    snprintf(g_msg, sizeof(g_msg), "%s", e.what());
    return 1;
  }
}

extern "C" {
const char* qref_last_error() { return g_msg; }

int qref_quant_fwd(void* y, void* sf, float* ts, const void* x, const float* amax, float so, long rows, long cols,
                   int four_six) {
  return guarded([&] {
    if (four_six)
      four_six_fp4((__nv_fp4x4_e2m1*)y, (__nv_fp8_e4m3*)sf, ts, (const nv_bfloat16*)x, amax, so, rows, cols);
    else
      rtn_fp4((__nv_fp4x4_e2m1*)y, (__nv_fp8_e4m3*)sf, ts, (const nv_bfloat16*)x, amax, so, rows, cols);
  });
}

int qref_rht128_eden(void* y, void* sf, float* ts, void* scratch, unsigned* mx, const void* h, const void* x,
                     long seed, float fp4_max, float fp8_max, int M, int N, int transpose, int full_h) {
  return guarded([&] {
    if (full_h)
      group_transform_128_eden((__nv_fp4x2_storage_t*)y, (__nv_fp8_e4m3*)sf, ts, (nv_bfloat16*)scratch, mx,
                               (const nv_bfloat16*)h, (const nv_bfloat16*)x, seed, fp4_max, fp8_max, M, N,
                               transpose != 0);
    else
      transform_rht128_eden((__nv_fp4x2_storage_t*)y, (__nv_fp8_e4m3*)sf, ts, (nv_bfloat16*)scratch, mx,
                            (const nv_bfloat16*)h, (const nv_bfloat16*)x, seed, fp4_max, fp8_max, M, N,
                            transpose != 0);
  });
}

int qref_rht128_requant(void* y, void* sf, float* ts, void* scratch, unsigned* mx, const void* h, const void* x,
                        const void* x_sf, const float* x_ts, long seed, float fp4_max, float fp8_max, int M, int N) {
  return guarded([&] {
    rht128_requant((__nv_fp4x2_storage_t*)y, (__nv_fp8_e4m3*)sf, ts, (nv_bfloat16*)scratch, mx,
                   (const nv_bfloat16*)h, (const __nv_fp4x2_storage_t*)x, (const __nv_fp8_e4m3*)x_sf, x_ts, seed,
                   fp4_max, fp8_max, M, N);
  });
}
}
