/*
 * q2b.h -- C ABI of libq2b, the B200 (sm_100a) implementation of the
 * Quartet-II NVFP4 linear-layer hot path of IST-DASLab/CloverLM.
 *
 * Every entry point takes raw device pointers, sizes and a cudaStream_t (as
 * void*), launches asynchronously on that stream, allocates no device memory
 * and returns Q2B_OK or an error code; q2b_last_error() then describes the
 * failure (thread-local).  Callers own every buffer, including scratch.
 *
 * Layouts (shared with the reference):
 *   bf16 tensors      row-major, 16-byte aligned.
 *   E2M1 codes        uint8 [rows, cols/2]; the low nibble holds the even element.
 *   E4M3 scales       one byte per 16 elements along a row, stored in the
 *                     blocked 128x4 layout: offset of (row r, block k) with
 *                     n = cols/16 blocks per row is
 *                     ((r/128 * n/4 + k/4) << 9) | (r%32)<<4 | ((r/32)%4)<<2 | k%4
 *                     (reference quartet2/csrc/utils.cuh:392-410).
 *   tensor scale      one fp32 in device memory; value = code * scale * ts.
 * Shape rules: rows and cols multiples of 128 (reference quant.py:117-121).
 * Paths in comments are relative to the reference project root.
 */
#ifndef Q2B_H
#define Q2B_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  Q2B_OK = 0,
  Q2B_ERR_INVALID = 1, /* bad shape, null or misaligned pointer, bad mode */
  Q2B_ERR_CUDA = 2,    /* a CUDA runtime/driver call failed */
  Q2B_ERR_DEVICE = 3   /* current device is not an sm_100 (B200-class) GPU */
};

enum { Q2B_MODE_RNE = 0, Q2B_MODE_FOUR_SIX = 1 };

/* Library version (major*10000 + minor*100 + patch). */
int q2b_version(void);

/* Message for the last failing call on this thread ("" if none). */
const char* q2b_last_error(void);

/* Reads and clears the device-side watchdog word of the current device: 0 if
 * no kernel wait ever timed out, else the code of the first wait that gave up.
 * Synchronizes the device.
 * A trip stays set until this call clears it, and while it is set every
 * libq2b kernel leaves at its first wait that is not already satisfied, so
 * outputs written after a trip are invalid.  Codes: 1 TMA data not arrived,
 * 2 shared-memory stage not released, 3 accumulator not ready, 4 accumulator
 * not drained, 5 producer/drain wait, 6 q2b_watchdog_selftest.
 * No counterpart in the reference (its kernels spin without a bound). */
int q2b_device_status(unsigned* code);

/* Copies the watchdog word of the current device to *host_word (pinned host
 * memory) asynchronously on `stream`, without clearing it and without
 * synchronizing: a training loop polls it once per step and checks the value
 * when the stream has passed the copy.
 * No counterpart in the reference. */
int q2b_watchdog_poll(unsigned* host_word, void* stream);

/* Exercises the timeout path: launches one thread that waits, with a limit of
 * wait_cycles SM cycles (1024 .. 4e9), on a barrier nothing completes.  The
 * wait gives up and records code 6 in the watchdog word (read it with
 * q2b_device_status).  Nothing is left in flight; later launches run normally
 * once the word is cleared.
 * No counterpart in the reference. */
int q2b_watchdog_selftest(int64_t wait_cycles, void* stream);

/* out[0] = max |x| over n bf16 values (fp32).
 * Replaces: abs_max (torch.compile reduction), quartet2/python/quartet2/linear.py:146-148. */
int q2b_abs_max(float* out, const void* x, int64_t n, void* stream);

/* y = relu(a)^2 for n bf16 values and out[0] = max |y| (fp32) in one pass.
 * a and y 16-byte aligned.
 * Replaces: the MLP activation ReLU2 (src/models/mlp.py:34-38) and the
 * abs-max pass of the next Quartet layer's forward (linear.py:146-148,179-183). */
int q2b_relu2_abs_max(void* y, float* amax, const void* a, int64_t n, void* stream);

/* Forward RTN quantization of bf16 x [rows, cols] to NVFP4 with tensor scale
 * from *amax; mode Q2B_MODE_RNE or Q2B_MODE_FOUR_SIX.
 * Replaces: rtn_fp4 / four_six_fp4, quartet2/csrc/round_four_six.cu:125-153
 * (bound in quartet2/csrc/binding.cpp, used by quant.py:114-138). */
int q2b_quant_fwd(void* codes, void* sf, float* ts, const void* x, const float* amax, float scale_override,
                  int64_t rows, int64_t cols, int mode, void* stream);

/* q2b_quant_fwd for any rows >= 1 (cols a multiple of 128).  codes are
 * [rows, cols/2]; sf is the blocked layout of ceil(rows/128)*128 rows, of
 * which only the rows that exist are written (the caller zero-fills the
 * rest once).  Serves the inference linear without padding its input.
 * Replaces: the 128-row F.pad + four_six_fp4 of QuartetIILinearMethod.apply,
 * src/evals/vllm_plugin/quartet2_quant.py:110-128. */
int q2b_quant_fwd_ragged(void* codes, void* sf, float* ts, const void* x, const float* amax, float scale_override,
                         int64_t rows, int64_t cols, int mode, void* stream);

/* Abs-max, tensor scale and quantization of x [rows, cols] in one launch (a
 * single cluster of 8 CTAs that exchange their partial maxima through
 * distributed shared memory), with the scale words of the padding rows of
 * the last 128-row block written as zero: the caller needs no amax buffer and
 * no zero-fill.  For small inputs (decode-sized rows); large ones are faster
 * through q2b_abs_max + q2b_quant_fwd_ragged.  Outputs as q2b_quant_fwd_ragged.
 * Replaces: abs_max + F.pad + four_six_fp4 of QuartetIILinearMethod.apply,
 * src/evals/vllm_plugin/quartet2_quant.py:110-128. */
int q2b_quant_rows_fused(void* codes, void* sf, float* ts, const void* x, float scale_override, int64_t rows,
                         int64_t cols, int mode, void* stream);

/* Rotation by the 128-point randomized Hadamard transform (h: h_rows = 16,
 * the top slice, extended by Sylvester's construction and row-swizzled as
 * quartet2/python/quartet2/rht.py:65-82) or by an explicit 128x128 matrix
 * (h_rows = 128), then EDEN quantization with a stochastically rounded E4M3
 * scale (seed keys the noise).  x is bf16 [M, N]; transpose = 0 quantizes
 * rows (codes [M, N/2]), transpose = 1 quantizes x^T (codes [N, M/2]).
 * scratch: bf16 [M*N/16]; scratch_max: one uint32.
 * Replaces: transform_rht128_eden, quartet2/csrc/rht128_eden.cu:171-177, and
 * group_transform_128_eden, quartet2/csrc/group_transform_and_eden.cu:321-329. */
int q2b_rht_eden(void* codes, void* sf, float* ts, void* scratch, unsigned* scratch_max, const void* h, int h_rows,
                 const void* x, uint64_t seed, float fp4_max, float fp8_max, int64_t M, int64_t N, int transpose,
                 void* stream);

/* Allocation-free variant of q2b_rht_eden.  No counterpart in the reference.
 *
 * For callers that may not allocate device memory at all -- for example code
 * running inside a host framework that owns every device byte through its own
 * pool and hands an operator only its input and output buffers, or a
 * latency-critical path where cudaMalloc's implicit device synchronization is
 * not acceptable -- this entry point needs no scratch from the caller.  The
 * bf16 pre-rounding scales and the max word live in one static device buffer
 * inside libq2b (Q2B_NOALLOC_SCRATCH_BYTES plus 256 bytes, held on every GPU
 * that loads the library until the process exits).  Inputs and outputs are as
 * for q2b_rht_eden.
 *
 * Limit: M * N <= Q2B_NOALLOC_MAX_ELEMS (one bf16 scale per 16 elements);
 * larger inputs are rejected with Q2B_ERR_INVALID.
 * The first call on a device looks up the buffer's device address (once per
 * device and CUDA context, under a lock; a reset device is looked up again);
 * make that first call before any stream capture.
 * All calls share the one buffer: calls whose kernels overlap on the GPU
 * (different streams, or different host threads, without ordering) race and
 * produce wrong results -- serialize them.  The max word is cleared on every
 * call; the scale area is fully overwritten before it is read. */
#define Q2B_NOALLOC_SCRATCH_BYTES (16ll << 20)
#define Q2B_NOALLOC_MAX_ELEMS (Q2B_NOALLOC_SCRATCH_BYTES * 8)
int q2b_rht_eden_noalloc(void* codes, void* sf, float* ts, const void* h, int h_rows, const void* x, uint64_t seed,
                         float fp4_max, float fp8_max, int64_t M, int64_t N, int transpose, void* stream);

/* Both orientations of q2b_rht_eden from one read of x: the row output uses
 * (codes_r, sf_r, ts_r, scratch_r, max_r, seed_r), the transposed output
 * (codes_c, ..., seed_c).  Equal, element for element, to two q2b_rht_eden
 * calls with transpose = 0 and 1.
 * Replaces: the two rht128_quant_eden calls on the output gradient in
 * Quartet_II_fn.backward, quartet2/python/quartet2/linear.py:222,229. */
int q2b_rht_eden_dual(void* codes_r, void* sf_r, float* ts_r, void* scratch_r, unsigned* max_r, void* codes_c,
                      void* sf_c, float* ts_c, void* scratch_c, unsigned* max_c, const void* h, int h_rows,
                      const void* x, uint64_t seed_r, uint64_t seed_c, float fp4_max, float fp8_max, int64_t M,
                      int64_t N, void* stream);

/* Requantization of an NVFP4 tensor (codes [M, N/2], blocked scales, tensor
 * scale *x_ts): dequantize to bf16, transpose, rotate along the old rows,
 * EDEN.  Output codes [N, M/2], scales blocked [N, M/16].
 * Replaces: rht128_requant, quartet2/csrc/rht128_requant.cu:303-311. */
int q2b_rht_requant(void* codes, void* sf, float* ts, void* scratch, unsigned* scratch_max, const void* h,
                    int h_rows, const void* x_codes, const void* x_sf, const float* x_ts, uint64_t seed,
                    float fp4_max, float fp8_max, int64_t M, int64_t N, void* stream);

/* D[M, N] (bf16) = *alpha * dequant(A[M, K]) @ dequant(B[N, K])^T for NVFP4
 * operands (codes K-major, blocked scales).  M, N multiples of 128, K of 64.
 * Replaces: _fp4_mm -> flashinfer.mm_fp4(..., backend="cudnn"),
 * quartet2/python/quartet2/linear.py:34-56. */
int q2b_gemm_nvfp4(void* D, const void* A, const void* B, const void* sfa, const void* sfb, const float* alpha,
                   int64_t M, int64_t N, int64_t K, void* stream);

/* q2b_gemm_nvfp4 with an fp32 D[M, N] (*alpha * the fp32 accumulator, not
 * rounded to bf16): the weight gradient of a layer whose master weight is fp32
 * comes out in the parameter's dtype, with no separate bf16 -> fp32 pass.
 * No counterpart in the reference (its wgrad GEMM writes bf16, which autograd
 * then casts to the fp32 parameter's dtype). */
int q2b_gemm_nvfp4_f32(float* D, const void* A, const void* B, const void* sfa, const void* sfb, const float* alpha,
                       int64_t M, int64_t N, int64_t K, void* stream);

/* D += bf16(*alpha * A B^T) for a bf16 D [M, N] that already holds a value:
 * each element becomes the bf16 sum of the old value and the bf16-rounded
 * product (TMA reductions on the 2-SM path).  Used to sum the input gradients
 * of the layers that read one activation (the attention projections).
 * Replaces: dx = dx_q + dx_k + dx_v, the autograd accumulation of the three
 * projections' input gradients (src/models/transformer.py:341-344). */
int q2b_gemm_nvfp4_add(void* D, const void* A, const void* B, const void* sfa, const void* sfb, const float* alpha,
                       int64_t M, int64_t N, int64_t K, void* stream);

/* The MLP's first linear with its activation in the GEMM epilogue: A_out =
 * bf16(*alpha * A B^T) (the pre-activation a, [M, N]), H_out = bf16(relu(a)^2)
 * and *amax = max H_out (fp32, written by the call).  Shapes as
 * q2b_gemm_nvfp4; shapes the 2-SM kernel does not take run the GEMM and then
 * q2b_relu2_abs_max (same results).
 * Replaces: l1 = Quartet_II_linear -> ReLU2 -> abs_max of the l2 input,
 * src/models/mlp.py:34-38,113-118, quartet2/python/quartet2/linear.py:179-183. */
int q2b_gemm_nvfp4_relu2(void* A_out, void* H_out, float* amax, const void* A, const void* B, const void* sfa,
                         const void* sfb, const float* alpha, int64_t M, int64_t N, int64_t K, void* stream);

/* The second MLP linear's dgrad with the ReLU^2 backward in the epilogue:
 * dA = bf16(2 * relu(a) * bf16(*alpha * A B^T)), a the saved pre-activation
 * (bf16 [M, N]).  Other shapes: the GEMM, then q2b_relu2_bwd in place.
 * Replaces: the dX GEMM of l2's backward (linear.py:222-225) followed by the
 * autograd backward of relu(x)**2 (src/models/mlp.py:34-38). */
int q2b_gemm_nvfp4_relu2_bwd(void* dA, const void* a, const void* A, const void* B, const void* sfa, const void* sfb,
                             const float* alpha, int64_t M, int64_t N, int64_t K, void* stream);

/* q2b_gemm_nvfp4 for any M >= 1 (N a multiple of 128, K of 64), scaled by
 * *alpha times *alpha_b when alpha_b is not null (the two tensor scales,
 * so no separate product kernel runs).  A is
 * [M, K/2] (rows past M are read as zero), sfa the blocked scales of
 * ceil(M/128)*128 rows, D [M, N] (only rows < M are written).  When the
 * output has too few 128x128 tiles to fill the GPU (decode-sized M), K is
 * split across CTAs and the partial tiles are summed in fp32 in `workspace`
 * (q2b_gemm_workspace_bytes(M, N, K) bytes, 16-byte aligned, zero-filled
 * once by the caller; every call leaves it zero again).  With a smaller or
 * null workspace the call runs unsplit.  Calls that share a workspace must
 * not overlap on the GPU.
 * Replaces: the padded _fp4_mm of QuartetIILinearMethod.apply and its row
 * slice, src/evals/vllm_plugin/quartet2_quant.py:125-137. */
int q2b_gemm_nvfp4_ex(void* D, const void* A, const void* B, const void* sfa, const void* sfb, const float* alpha,
                      const float* alpha_b, int64_t M, int64_t N, int64_t K, void* workspace, int64_t workspace_bytes,
                      void* stream);

/* Workspace bytes q2b_gemm_nvfp4_ex uses for this shape on the current
 * device (0 = it never splits K); -1 if no device is usable.
 * No counterpart in the reference (its GEMM library manages its own). */
int64_t q2b_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K);

/* One AdamW step (decoupled weight decay, torch's fused-AdamW operation
 * order) on n fp32 weights w with fp32 moments exp_avg / exp_avg_sq and an
 * fp32 (grad_bf16 = 0) or bf16 (grad_bf16 = 1) gradient; step is the 1-based
 * step count after this update.  In the same pass: *amax = max |w_new| (fp32,
 * device; written even when it stays 0) when amax is not null, and
 * w_bf16[i] = bf16(w_new[i]) when w_bf16 is not null.  Any alignment; 16-byte
 * aligned tensors take the vector path.
 * Replaces: torch.optim.AdamW(fused=True) (src/models/parametrizations.py:311)
 * followed by the weight abs-max pass of register_optimizer_hook,
 * quartet2/python/quartet2/linear.py:259-270. */
int q2b_adamw_step(float* w, float* exp_avg, float* exp_avg_sq, const void* grad, int grad_bf16, int64_t n,
                   float lr, float beta1, float beta2, float eps, float weight_decay, int64_t step, void* w_bf16,
                   float* amax, void* stream);

/* ---- CloverLM block glue (the training step around the Quartet linears) ----
 * No counterparts as single kernels in the reference: each fuses a chain of
 * PyTorch elementwise ops of src/models/transformer.py / mlp.py into one pass.
 *
 * RoPE (base-1024 table, interleaved pairs) + sphere norm (eps 1e-12) +
 * optional per-head scale of x bf16 [rows, heads, 128] (row r at position
 * r % seq): out = scale[h] * n / max(|n|, 1e-12) with n = bf16(rope(x));
 * norm_out [rows, heads] fp32 keeps max(|n|, 1e-12) for the backward.
 * cos_sin: fp32 [seq, 64, 2] (cos, sin).  scale: fp32 [heads] or NULL.
 * Replaces: apply_rope + sphere_norm + Q = scale * Q,
 * src/models/transformer.py:63-74,357-363,177-185. */
int q2b_rope_norm_fwd(void* out, float* norm_out, const void* x, const float* cos_sin, const float* scale,
                      int64_t rows, int heads, int seq, void* stream);

/* Gradient of q2b_rope_norm_fwd: dx bf16 [rows, heads, 128] from dout and the
 * forward's out and norm_out; dscale[h] += sum over rows of dout * out / scale
 * (dscale and scale both NULL when there is no scale; the caller zeroes it). */
int q2b_rope_norm_bwd(void* dx, float* dscale, const void* dout, const void* out, const float* norm,
                      const float* cos_sin, const float* scale, int64_t rows, int heads, int seq, void* stream);

/* Residual RMSNorm with the next Quartet layer's abs-max: for rows of d
 * (a multiple of 8, at most 4096) values, rstd = 1/sqrt(mean(y^2) + eps),
 * x_out = x + (y * rstd) * w (fp32), xb_out = bf16(x_out), *amax =
 * max |xb_out|, rstd_out[r] = rstd.  x, x_out, w fp32; y, xb_out bf16.
 * Replaces: Y = out_att_norm(Y); Y__ = X + Y (and the MLP's), followed by the
 * next Quartet_II_fn's abs_max of its input, src/models/transformer.py:380-395,
 * quartet2/python/quartet2/linear.py:179-183. */
int q2b_add_rmsnorm_amax(float* x_out, void* xb_out, float* rstd_out, float* amax, const float* x, const void* y,
                         const float* w, int64_t rows, int d, float eps, void* stream);

/* Gradient of q2b_add_rmsnorm_amax: with g = g (fp32) + gb (bf16, may be
 * NULL), dx = g (fp32; dx may be g), dy = rstd * (g*w - yhat * mean(g*w*yhat))
 * (bf16, yhat = y * rstd), and dw_partial [partial_rows, d] fp32 holds the
 * per-block sums of g * yhat (partial_rows blocks; the caller sums them). */
int q2b_rmsnorm_bwd(float* dx, void* dy, float* dw_partial, int64_t partial_rows, const float* g, const void* gb,
                    const void* y, const float* rstd, const float* w, int64_t rows, int d, void* stream);

/* da = bf16(2 * relu(a) * g) for n (a multiple of 8) bf16 values.
 * Replaces: the autograd backward of relu(x)**2, src/models/mlp.py:34-38. */
int q2b_relu2_bwd(void* da, const void* a, const void* g, int64_t n, void* stream);

/* Cross-entropy of rows of bf16 logits [rows, V] (V a multiple of 8) against int64 targets:
 * row_loss[r] = logsumexp(x_r) - x_r[t_r] (fp32), and the logits are overwritten with the
 * gradient of inv_n * sum(row_loss): bf16((softmax(x_r) - onehot(t_r)) * inv_n).
 * Replaces: F.cross_entropy of get_loss (src/data/utils_data.py:293-318) and its autograd
 * backward, applied per chunk of rows of the tied output head. */
int q2b_softmax_xent_bf16(void* logits, float* row_loss, const int64_t* targets, float inv_n, int64_t rows, int64_t V,
                          void* stream);

/* Measurement: one SM pair per two SMs issues `iters` back-to-back
 * cta_group::2 M256 N256 K64 NVFP4 block-scaled MMAs on operands resident in
 * shared memory (2*256*256*64 FLOP each; total FLOP = (SMs/2) * iters * that).
 * Time it with events on `stream`: the tensor pipe's FP4 ceiling, against
 * which the GEMM's roofline fraction is quoted.  iters: a multiple of 4.
 * cycles (device, optional, 2 entries): SM cycles and globaltimer
 * nanoseconds of the first pair's issue loop.
 * No counterpart in the reference (its FP4 GEMM is a library call). */
int q2b_fp4_mma_peak(int iters, long long* cycles, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* Q2B_H */
