/*
 * fvq.h -- C ABI of the B200 (sm_100a) NVFP4 transformer-FFN library (libfvq.so).
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * passed as void*.  Nothing allocates: outputs and workspaces belong to the
 * caller.  Work is enqueued on the given stream; no entry point synchronises
 * the host (except fvq_read_device_error).  Return value: FVQ_OK (0) or a
 * negative FVQ_E* status; fvq_last_error() gives a message for the calling
 * host thread.
 *
 * Tensor conventions (the reference's, so buffers are interchangeable):
 *   bf16 tensors are uint16_t bit patterns, row-major.
 *   NVFP4 codes: uint8 [rows, k/2], element 2j in the low nibble of byte j.
 *   Scale factors: E4M3 bytes, one per 16 elements, in the 128x4 swizzled
 *     layout [pad128(rows)/128][k/64][32][4][4] (pad128(rows) * k/16 bytes);
 *     rows past `rows` hold zero.
 *   Global scales: device fp32 scalars, g = 2688 / max(amax, 1e-12) computed
 *     as reciprocal(amax) * 2688 (two fp32 roundings).
 *
 * Shape limits: k % 64 == 0 for the quantizer; the GEMM needs k % 256 == 0
 * and n % 256 == 0 (d_model 1536 and d_ff 8960 both qualify).
 * Alignment: bf16 inputs of the quantizer (and of linear / ffn) 32 bytes,
 * every other pointer 16 bytes.
 */
#ifndef FVQ_H_
#define FVQ_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FVQ_OK 0
#define FVQ_EINVAL (-1)     /* bad shape, null pointer or bad mode */
#define FVQ_EALIGN (-2)     /* pointer not 16-byte aligned */
#define FVQ_ECUDA (-3)      /* CUDA runtime / driver error */
#define FVQ_EDEVICE (-4)    /* device is not sm_100 */
#define FVQ_EWORKSPACE (-5) /* workspace too small */
#define FVQ_ETIMEOUT (-6)   /* a bounded device wait gave up (fvq_read_device_error) */

/* GEMM epilogues */
#define FVQ_EPI_BF16 0      /* y = bf16(alpha*acc), then y = bf16(y + bias) if bias */
#define FVQ_EPI_GELU_AMAX 1 /* FVQ_EPI_BF16, then h = bf16(gelu_tanh(y)) and
                               atomic max of |h| into *amax_out (fp32 bits) */

/* Library version (major*10000 + minor*100 + patch). */
int fvq_version(void);

/* Message for the last failing call made by this host thread. */
const char* fvq_last_error(void);

/*
 * Bytes of workspace fvq_amax needs.  The workspace must be zeroed once
 * before its first use; every call leaves it zeroed again.
 */
size_t fvq_amax_workspace_bytes(void);

/*
 * amax = max |x| over `numel` bf16 values; g = 2688 / max(amax, 1e-12).
 * Replaces the reference's global_scale() -- the Triton _partial_amax
 * kernel and its torch tail (ffn_quantization.py:15-19, :29-32).
 * Either output may be NULL.  numel == 0 gives amax = 0.
 */
int fvq_amax(const uint16_t* x, int64_t numel, float* amax_out, float* g_out,
             void* workspace, size_t workspace_bytes, void* stream);

/*
 * NVFP4 quantization with a given global scale: codes and swizzled E4M3
 * scale factors.  Replaces flashinfer.nvfp4_quantize(x, g) with its default
 * 128x4 layout as called at ffn_quantization.py:47 and :64.
 * `g` points to the fp32 encode scale on the device.
 */
int fvq_nvfp4_quantize(const uint16_t* x, int64_t rows, int64_t k, const float* g,
                       uint8_t* codes, uint8_t* sf, void* stream);

/*
 * global_scale + nvfp4_quantize in one call (ffn_quantization.py:63-64):
 * g_out receives the encode scale it used.  `amax_in` may be NULL (then the
 * amax pass runs first, using `workspace`); if not NULL it must hold
 * max |x| already (e.g. from an FVQ_EPI_GELU_AMAX epilogue) and no amax
 * pass runs.
 */
int fvq_nvfp4_quantize_dynamic(const uint16_t* x, int64_t rows, int64_t k,
                               const float* amax_in, float* g_out,
                               uint8_t* codes, uint8_t* sf,
                               void* workspace, size_t workspace_bytes, void* stream);

/*
 * Block-scaled NVFP4 GEMM on tcgen05 tensor cores:
 *   out[m, n] = epilogue(alpha * sum_k A[m,k] * W[n,k]),  alpha = 1 / (g_a * g_w)
 * A: codes [m, k/2] + swizzled sf; W: codes [n, k/2] + swizzled sf (the
 * nn.Linear weight layout).  Replaces flashinfer.mm_fp4(q, qweight.t(), s,
 * scale.t(), alpha=1./(g*global_sf), out_dtype=bf16, backend='cutlass')
 * followed by `out + self.bias` (ffn_quantization.py:65-69), with the bias
 * add's double rounding kept.  `bias` may be NULL.  `amax_out` is required
 * for FVQ_EPI_GELU_AMAX (the caller zeroes it before the first tile runs).
 */
int fvq_nvfp4_gemm(const uint8_t* a_codes, const uint8_t* a_sf, const float* g_a,
                   const uint8_t* w_codes, const uint8_t* w_sf, const float* g_w,
                   const uint16_t* bias, uint16_t* out, int64_t m, int64_t n, int64_t k,
                   int epilogue, float* amax_out, void* stream);

/*
 * Weight preparation with no reference counterpart.  The W scales of an
 * [n, k] weight (128x4 layout) rewritten as the GEMM's 128-lane tensor-memory
 * scale copies read them: each 512-byte atom four times, the two 128-row
 * halves of a 256-row N block interleaved per 64-deep K step, so that one K
 * tile's W scales take four copies instead of eight.  n % 256 == 0,
 * k % 256 == 0; the output holds fvq_w_scales_replicated_bytes(n, k) =
 * 4 * n * k / 16 bytes.  fvq_nvfp4_ffn does this for its second linear on
 * every call; callers with fixed weights can do it once.
 */
size_t fvq_w_scales_replicated_bytes(int64_t n, int64_t k);
int fvq_replicate_w_scales(const uint8_t* w_sf, int64_t n, int64_t k, uint8_t* w_sf_rep,
                           void* stream);

/*
 * fvq_nvfp4_gemm with the FVQ_EPI_BF16 epilogue and the W scales in the
 * replicated layout of fvq_replicate_w_scales; bit-identical results.  No
 * reference counterpart (the reference's mm_fp4 takes the 128x4 layout, which
 * fvq_nvfp4_gemm and fvq_nvfp4_mm accept).
 */
int fvq_nvfp4_gemm_wrep(const uint8_t* a_codes, const uint8_t* a_sf, const float* g_a,
                        const uint8_t* w_codes, const uint8_t* w_sf_rep, const float* g_w,
                        const uint16_t* bias, uint16_t* out, int64_t m, int64_t n, int64_t k,
                        void* stream);

/*
 * The same GEMM with a precomputed device alpha (fp32 scalar) instead of the
 * two global scales: the exact argument list of flashinfer.mm_fp4 as the
 * reference calls it (ffn_quantization.py:65-67), plus the optional bias of
 * :68-69.  FVQ_EPI_BF16 epilogue.
 */
int fvq_nvfp4_mm(const uint8_t* a_codes, const uint8_t* a_sf, const uint8_t* w_codes,
                 const uint8_t* w_sf, const float* alpha, const uint16_t* bias, uint16_t* out,
                 int64_t m, int64_t n, int64_t k, void* stream);

/* One nn.Linear replaced by QuantLinear (ffn_quantization.py:54-70). */
typedef struct fvq_linear {
  const uint8_t* qweight;   /* [out_features, in_features/2] */
  const uint8_t* scale;     /* swizzled, pad128(out_features) * in_features/16 */
  const float* global_sf;   /* device fp32 scalar */
  const uint16_t* bias;     /* bf16 [out_features] or NULL */
  int64_t in_features;
  int64_t out_features;
} fvq_linear;

/* Bytes of workspace fvq_nvfp4_linear needs for `rows` rows. */
size_t fvq_nvfp4_linear_workspace_bytes(int64_t rows, int64_t in_features);

/* QuantLinear.forward: y = bias + mm_fp4(nvfp4_quantize(x, global_scale(x)), W). */
int fvq_nvfp4_linear(const uint16_t* x, int64_t rows, const fvq_linear* lin, uint16_t* y,
                     void* workspace, size_t workspace_bytes, void* stream);

/*
 * QuantLinear.forward for callers that cannot allocate device memory (code
 * running inside another runtime's memory arena, plugins handed only their
 * input and output buffers, callers that must not touch the allocator while
 * work is in flight).  No counterpart in the reference; no workspace
 * argument: the scratch that fvq_nvfp4_linear takes as a workspace comes from
 * a fixed 16 MiB array built into the library (fvq_noalloc_scratch_bytes),
 * which every GPU that loads the library holds until the process exits.
 * Calls whose fvq_nvfp4_linear_workspace_bytes(rows, in_features) exceeds it
 * return FVQ_EWORKSPACE.  The first call in each CUDA context (a device's
 * primary context, or a caller's own driver-API context) looks the array's
 * address up with cudaGetSymbolAddress and caches it under the context's
 * unique id, so a cudaDeviceReset or another context is looked up again; make
 * that first call before any stream capture.  All calls share the array, so
 * calls that overlap on the GPU race.  Nothing is allocated by this call.
 */
int fvq_nvfp4_linear_noalloc(const uint16_t* x, int64_t rows, const fvq_linear* lin, uint16_t* y,
                             void* stream);
size_t fvq_noalloc_scratch_bytes(void);

/* Bytes of workspace fvq_nvfp4_ffn needs for `rows` tokens. */
size_t fvq_nvfp4_ffn_workspace_bytes(int64_t rows, int64_t d_model, int64_t d_ff);

/*
 * The whole FFN the reference installs into (ffn_quantization.py:77-80 swaps
 * ffn[0] and ffn[2] of nn.Sequential(Linear, GELU(tanh), Linear)):
 *   y = QuantLinear2(bf16(gelu_tanh(QuantLinear1(x))))
 * with the same global scales and roundings as the reference.  GELU and the
 * amax of the intermediate are computed in GEMM1's epilogue.
 * The workspace must be zeroed once before its first use.
 */
int fvq_nvfp4_ffn(const uint16_t* x, int64_t rows, const fvq_linear* lin1, const fvq_linear* lin2,
                  uint16_t* y, void* workspace, size_t workspace_bytes, void* stream);

/*
 * No counterpart in the reference (whose DiT blocks put attention between two
 * FFNs): fvq_nvfp4_ffn for a stack of FFNs that feed each other directly, each
 * call handing the next the max |y| it already knows.  x_amax (NULL: computed
 * as fvq_nvfp4_ffn does) is max |x| as the previous call's y_amax gave it;
 * then the first launch quantizes x without its own pass over x.  y_amax
 * (NULL: not produced) receives max |y| (bf16 magnitudes, NaN ignored, as
 * fvq_amax takes them) from the second GEMM's epilogue; the call sets it to 0
 * itself, after its first launch.  y_amax must not alias x_amax.  Same
 * workspace as fvq_nvfp4_ffn; the output equals fvq_nvfp4_ffn's bit for bit.
 */
int fvq_nvfp4_ffn_chain(const uint16_t* x, int64_t rows, const fvq_linear* lin1,
                        const fvq_linear* lin2, uint16_t* y, const float* x_amax, float* y_amax,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * The FFN with the intermediate never stored in bf16: GEMM1's epilogue applies bias and
 * GELU and quantizes h to NVFP4 itself (codes and 128x4-swizzled E4M3 scales, the
 * activation quantizer's exact per-block recipe), with a provisional encode scale
 *   g = 2^-headroom_log2 * 2688 / max(*amax_hint, 1e-12)      (headroom_log2 in [0, 30])
 * instead of the reference's 2688 / amax(h); GEMM2 uses alpha = 1 / (g * g_w2).  Three
 * launches.  No reference counterpart as a call: it replaces the same
 * nn.Sequential(QuantLinear, GELU(tanh), QuantLinear) as fvq_nvfp4_ffn
 * (ffn_quantization.py:77-80) but is not bit-exact with it unless *amax_hint equals
 * amax(h) times a power of two (a block's codes depend on g only through its
 * mantissa); otherwise it is an equally accurate but different quantization of h.
 *   amax_hint: device fp32, an estimate of max |h| (a calibrated value, or the previous
 *              call's amax_seen: delayed scaling).  Read, never written.
 *   headroom_log2: g is divided by 2^headroom_log2 (exactly), leaving room for h to
 *              exceed the hint by that factor before a block's scale saturates.
 *   amax_seen: device fp32 or NULL; receives max |h| of this call (zeroed by the call's
 *              first launch, so it must not alias amax_hint).
 *   flags:     device u32 or NULL; OR-ed with 1 when a block's scale value
 *              g * vmax / 6 exceeded 448 and was clipped (the hint was too small: rerun
 *              fvq_nvfp4_ffn), 2 when a nonzero block's scale rounded to zero.  The
 *              caller zeroes it.
 * Workspace: fvq_nvfp4_ffn_fused_workspace_bytes (no bf16 intermediate).
 */
size_t fvq_nvfp4_ffn_fused_workspace_bytes(int64_t rows, int64_t d_model, int64_t d_ff);
int fvq_nvfp4_ffn_fused(const uint16_t* x, int64_t rows, const fvq_linear* lin1,
                        const fvq_linear* lin2, uint16_t* y, const float* amax_hint,
                        int headroom_log2, float* amax_seen, uint32_t* flags, void* workspace,
                        size_t workspace_bytes, void* stream);
/* fvq_nvfp4_ffn_fused with CUDA events around its three launches; synchronises and
 * writes the device times (ms) to kernel_ms[0..2].  Instrumentation. */
int fvq_nvfp4_ffn_fused_profile(const uint16_t* x, int64_t rows, const fvq_linear* lin1,
                                const fvq_linear* lin2, uint16_t* y, const float* amax_hint,
                                int headroom_log2, float* amax_seen, uint32_t* flags,
                                void* workspace, size_t workspace_bytes, void* stream,
                                float* kernel_ms);

/*
 * The DiT block around the FFN -- the caller of block.ffn that the reference's
 * installer patches (ffn_quantization.py:77-80); the block itself is upstream
 * code, not part of the reference.  adaLN-modulated input and gated residual:
 *   u   = bf16(bf16(LN(x) * bf16(1 + scale)) + shift)
 *   out = bf16(x + bf16(gate * FFN(u)))
 * LN without affine: bf16((x - mean) * rsqrtf(var + eps)), mean and biased
 * variance of the row in fp32; shift, scale, gate: bf16 [d_model]; every
 * elementwise step one bf16 rounding (torch's semantics on bf16 tensors).
 * FFN(u) is fvq_nvfp4_ffn's result; u is never stored (the first launch
 * normalises, modulates and quantizes x in one pass) and the gated residual
 * is applied in the second GEMM's epilogue.  d_model % 8 == 0 and <= 2048
 * (and the FFN's d_model % 64 == 0); pointers 16-byte
 * aligned, the workspace (fvq_nvfp4_ffn_block_workspace_bytes, zeroed once)
 * 32-byte aligned.
 */
size_t fvq_nvfp4_ffn_block_workspace_bytes(int64_t rows, int64_t d_model, int64_t d_ff);
/* The block's input step alone: u as above, [rows, d] bf16. */
int fvq_ln_modulate(const uint16_t* x, int64_t rows, int64_t d, const uint16_t* shift,
                    const uint16_t* scale, float eps, uint16_t* u, void* stream);
int fvq_nvfp4_ffn_block(const uint16_t* x, int64_t rows, const uint16_t* shift,
                        const uint16_t* scale, const uint16_t* gate, float eps,
                        const fvq_linear* lin1, const fvq_linear* lin2, uint16_t* out,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * Instrumentation with no reference counterpart: fvq_nvfp4_ffn with CUDA
 * events around its four launches (amax+quantize of x, GEMM1 with bias, GELU
 * and amax, quantize of the intermediate, GEMM2 with bias).  Synchronises on
 * the last event and writes the four device times in milliseconds to
 * kernel_ms[0..3].
 */
int fvq_nvfp4_ffn_profile(const uint16_t* x, int64_t rows, const fvq_linear* lin1,
                          const fvq_linear* lin2, uint16_t* y, void* workspace,
                          size_t workspace_bytes, void* stream, float* kernel_ms);
/* The same instrumentation around fvq_nvfp4_ffn_chain. */
int fvq_nvfp4_ffn_chain_profile(const uint16_t* x, int64_t rows, const fvq_linear* lin1,
                                const fvq_linear* lin2, uint16_t* y, const float* x_amax,
                                float* y_amax, void* workspace, size_t workspace_bytes,
                                void* stream, float* kernel_ms);

/*
 * ---------------------------------------------------------------------------
 * FP8 (E4M3) W8A8 mode: the reference's QuantLinear(mode='fp8')
 * (ffn_quantization.py:6-13, :22-26, :45-46, :57-60) and its per-tensor
 * activation quantizer (decoder_fp8.py:9-24, shared by lq_fp8.py:24-31).
 *
 * E4M3 tensors are uint8 bytes of float8_e4m3fn values, row-major.  Row
 * scales are fp32, one per row ([rows] -- the reference's [rows, 1]).  The
 * reference divides with Triton's fp32 `/` (div.full.f32 on the GPU); these
 * kernels issue the same instruction.
 * ---------------------------------------------------------------------------
 */

/*
 * Per-row quantization, the reference's row_quant(x) (ffn_quantization.py:22-26,
 * Triton _row_quant :6-13):
 *   scale[r] = max(max_k |x[r,k]| / 448, 1e-12);  q[r,k] = e4m3_rn_satfinite(x[r,k] / scale[r])
 * k % 8 == 0 and k <= 16384; x and q 16-byte aligned.
 */
int fvq_fp8_row_quantize(const uint16_t* x, int64_t rows, int64_t k, uint8_t* q, float* scale,
                         void* stream);

/*
 * Per-tensor quantization, the reference's quantize_activation(x)
 * (decoder_fp8.py:17-24, and FP8Conv3d.quantize, lq_fp8.py:24-31): the amax of
 * _partial_amax (the same kernel as fvq_amax), scale = max(amax / 448, 1e-12)
 * evaluated as torch does (amax times the fp32 reciprocal of 448) and written
 * to *scale, then
 *   q = e4m3(min(max(x / scale, -448), 448))
 * over `numel` elements in memory order (any dense layout, channels_last
 * included).  The workspace (fvq_fp8_tensor_quantize_workspace_bytes) must be
 * zeroed once before its first use; every call leaves it zeroed again.
 * x 16-byte aligned, q 8-byte aligned.
 */
size_t fvq_fp8_tensor_quantize_workspace_bytes(void);
int fvq_fp8_tensor_quantize(const uint16_t* x, int64_t numel, uint8_t* q, float* scale,
                            void* workspace, size_t workspace_bytes, void* stream);

/*
 * E4M3 GEMM on tcgen05 tensor cores (kind::f8f6f4) with row-wise scales:
 *   out[m, n] = bf16((sum_k A[m,k] W[n,k]) * scale_a[m] * scale_w[n]),  then
 *   out = bf16(out + bias[n]) if bias
 * Replaces torch._scaled_mm(q, qweight.t(), scale_a=s, scale_b=scale.t(),
 * out_dtype=bf16, use_fast_accum=False) and the bias add that follows it
 * (ffn_quantization.py:58-60, :68-69).  A [m, k], W [n, k] (the nn.Linear
 * layout).  n % 256 == 0, k % 128 == 0, k <= 16384.
 */
int fvq_fp8_scaled_mm(const uint8_t* a, const float* scale_a, const uint8_t* w,
                      const float* scale_w, const uint16_t* bias, uint16_t* out, int64_t m,
                      int64_t n, int64_t k, void* stream);

/* One nn.Linear replaced by QuantLinear(linear, 'fp8') (ffn_quantization.py:45-46). */
typedef struct fvq_linear_fp8 {
  const uint8_t* qweight;   /* E4M3 [out_features, in_features] */
  const float* scale;       /* fp32 [out_features], the weight's row scales */
  const uint16_t* bias;     /* bf16 [out_features] or NULL */
  int64_t in_features;
  int64_t out_features;
} fvq_linear_fp8;

/* QuantLinear.forward in mode 'fp8': y = bias + scaled_mm(row_quant(x), W). */
size_t fvq_fp8_linear_workspace_bytes(int64_t rows, int64_t in_features);
int fvq_fp8_linear(const uint16_t* x, int64_t rows, const fvq_linear_fp8* lin, uint16_t* y,
                   void* workspace, size_t workspace_bytes, void* stream);

/*
 * The whole FFN in mode 'fp8': y = QuantLinear2(bf16(gelu_tanh(QuantLinear1(x))))
 * with the reference's row scales and roundings.  GELU and the per-row max |h|
 * the second row quantizer needs are computed in GEMM1's epilogue.  Four
 * launches; the workspace needs no initialisation.
 */
size_t fvq_fp8_ffn_workspace_bytes(int64_t rows, int64_t d_model, int64_t d_ff);
int fvq_fp8_ffn(const uint16_t* x, int64_t rows, const fvq_linear_fp8* lin1,
                const fvq_linear_fp8* lin2, uint16_t* y, void* workspace, size_t workspace_bytes,
                void* stream);

/*
 * Instrumentation with no reference counterpart: fvq_fp8_ffn with CUDA events
 * around its four launches (quantize x, GEMM1 + bias + GELU + row maxima,
 * quantize h, GEMM2 + bias); synchronises and writes the four device times in
 * milliseconds to kernel_ms[0..3].
 */
int fvq_fp8_ffn_profile(const uint16_t* x, int64_t rows, const fvq_linear_fp8* lin1,
                        const fvq_linear_fp8* lin2, uint16_t* y, void* workspace,
                        size_t workspace_bytes, void* stream, float* kernel_ms);

/*
 * ---------------------------------------------------------------------------
 * Pillow-exact bicubic resize of the input pipeline (reference pil_exact_gpu.py:
 * 30-150, used by chunked_input.py:111-113).
 * ---------------------------------------------------------------------------
 *
 * RGB uint8 frames [frames, in_h, in_w, 3] resized to out_w x out_h exactly as
 * Pillow's Image.resize(..., BICUBIC) does (22-bit fixed-point separable
 * passes, horizontal first, each rounded and clipped to uint8), cropped to
 * [crop_y, crop_y + crop_h) x [crop_x, crop_x + crop_w), and written as
 *   dst_u8:   uint8 [frames, crop_h, crop_w, 3]        (resize_exact_gpu), and/or
 *   dst_bf16: bf16 [frames, 3, crop_h, crop_w] of p / 255 * 2 - 1 (fp32, then
 *             bf16) -- normalize_exact_gpu(resize_exact_gpu(frames)) in one pass.
 * Either output may be NULL (not both).  Upscaling only (out_h >= in_h,
 * out_w >= in_w); crop_w % 8 == 0; frames <= 65535; outputs 16-byte aligned.
 * The reference's geometry is 426x240 -> 1704x960, crop (32, 20, 896, 1664).
 */
int fvq_pil_resize(const uint8_t* src, int64_t frames, int64_t in_h, int64_t in_w, int64_t out_h,
                   int64_t out_w, int64_t crop_y, int64_t crop_x, int64_t crop_h, int64_t crop_w,
                   uint8_t* dst_u8, uint16_t* dst_bf16, void* stream);

/*
 * normalize_exact_gpu on its own (pil_exact_gpu.py:115-150): uint8 pixels
 * [frames, h, w, 3] at element strides (stride_frame, stride_row, stride_col;
 * the three channels adjacent) -> bf16 [frames, 3, h, w] of p / 255 * 2 - 1.
 * w % 8 == 0; dst 16-byte aligned.
 */
int fvq_pil_normalize(const uint8_t* src, int64_t frames, int64_t h, int64_t w,
                      int64_t stride_frame, int64_t stride_row, int64_t stride_col, uint16_t* dst,
                      void* stream);

/*
 * Test support: out[i] = div.full.f32(a[i], b[i]) on the device, the division
 * the FP8 quantizers (and the reference's Triton `/`) use.
 */
int fvq_div_full_probe(const float* a, const float* b, float* out, int64_t n, void* stream);

/*
 * Test support: out[i] = rcp.approx.ftz.f32(in[i]) on the device, the
 * reciprocal the quantizer uses (so a CPU oracle can use measured values).
 */
int fvq_rcp_approx_probe(const float* in, float* out, int64_t n, void* stream);

/*
 * Test support: out[i] = bf16(gelu_tanh(in[i])) through the GEMM epilogue's
 * GELU path (a per-CTA table over |x| in [2^-20, 8) plus the exact fp32
 * formula elsewhere), so it can be compared with torch over all 65536 inputs.
 */
int fvq_gelu_bf16_probe(const uint16_t* in, uint16_t* out, int64_t count, void* stream);

/*
 * Library setting with no reference counterpart: NVFP4 GEMMs with the plain
 * bf16 epilogue whose m is a multiple of 256 (fvq_nvfp4_gemm with
 * FVQ_EPI_BF16, fvq_nvfp4_gemm_wrep, the second GEMM of fvq_nvfp4_ffn and,
 * in mode 1, the gated-residual GEMM of fvq_nvfp4_ffn_block) run on pairs of
 * SMs (clusters of two CTAs sharing 256 x 256 tiles, tcgen05 cta_group::2).
 * mode 0 selects the one-SM kernel, 1 (the default) the pair kernel reading
 * the W scales in their library layout, 2 the pair kernel reading the
 * replicated copy where the caller has one.  All modes give the same bits.
 * Applies to later launches from any thread; FVQ_EINVAL for other modes.
 */
int fvq_set_gemm_pairing(int mode);

/*
 * Library setting with no reference counterpart: which FP8 GEMMs (fvq_fp8_scaled_mm,
 * fvq_fp8_linear, fvq_fp8_ffn) run on pairs of SMs (clusters of two CTAs sharing
 * 256 x 256 tiles, tcgen05 cta_group::2) instead of one SM per 128 x 256 tile:
 * mode 0 none, 1 those with the plain bias epilogue (the default; the GELU epilogue
 * of fvq_fp8_ffn's first GEMM runs faster on one SM), 2 all.  Every mode gives the
 * same bits.  Applies to later launches.
 */
int fvq_set_fp8_gemm_pairing(int mode);

/*
 * Bounded device waits: a GEMM whose pipeline wait exceeds the limit sets a
 * device error word and returns early (after letting its own copies and MMAs
 * drain).  fvq_set_wait_limit changes the limit, in nanoseconds of wall time
 * per wait (0 restores the default of 2 s), for later launches.  The limit is
 * process-wide: it applies to launches from every host thread, so a short
 * limit set by one thread also shortens the waits of other threads' calls.
 * fvq_read_device_error synchronises `stream`, returns the error word
 * (0 = none) in *flags and clears it.
 */
int fvq_set_wait_limit(uint64_t nanoseconds);
int fvq_read_device_error(void* stream, uint32_t* flags);

#ifdef __cplusplus
}
#endif

#endif /* FVQ_H_ */
