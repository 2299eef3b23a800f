// fvq_internal.h -- launchers shared between the kernel files and the C ABI.
#pragma once

#include <cstddef>
#include <cstdint>
#include <mutex>
#include <cuda_runtime.h>

namespace fvq {

// Bits of the device error word.
constexpr uint32_t kErrWaitProducer = 1u << 0;  // producer gave up on an empty stage
constexpr uint32_t kErrWaitMma = 1u << 1;       // MMA warp gave up on a full stage / accumulator
constexpr uint32_t kErrWaitEpilogue = 1u << 2;  // epilogue gave up on the accumulator
constexpr uint32_t kErrWaitTeardown = 1u << 3;  // teardown gave up on in-flight work
constexpr uint32_t kErrSmemAlign = 1u << 4;     // dynamic shared memory not 1024-byte aligned
constexpr uint32_t kErrWaitGrid = 1u << 5;      // fused quantizer gave up at its grid barrier

// Bound on any single pipeline wait inside a kernel (wall time, ns).
constexpr uint64_t kDefaultWaitLimit = 2000000000ull;

// amax workspace: [0] arrival counter, [2] amax bits, partials from byte 64.
constexpr int kAmaxMaxBlocks = 2048;
// amax workspace words: arrival counter, barrier generation, amax bits, the
// grid barrier's per-group counters, then one partial maximum per CTA
constexpr int kWsCounter = 0;
constexpr int kWsGeneration = 1;
constexpr int kWsAmax = 2;
constexpr int kWsGroups = 32;          // up to 32 group counters (words 32..127)
constexpr int kBarrierGroup = 64;      // CTAs per group counter
constexpr int kWsPartial = 128;
constexpr size_t kAmaxWorkspaceBytes = (kWsPartial + kAmaxMaxBlocks) * 4;
static_assert(kAmaxMaxBlocks / kBarrierGroup <= kWsPartial - kWsGroups, "group counters");

inline int64_t pad_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }
inline size_t sf_bytes(int64_t rows, int64_t k) {
  return static_cast<size_t>(pad_up(rows, 128) * pad_up(k / 16, 4));
}

int sm_count();

// Per-context caches.  The device address of a __device__ symbol of this library and a
// kernel's function attributes belong to a CUDA context, not to a device ordinal: after
// cudaDeviceReset, or under a caller's own driver-API context, the module is loaded
// again, possibly at another address.  Values are therefore cached under the unique id
// of the calling thread's current context (cuCtxGetId; ids are never reused).
uint64_t current_context_id();  // 0 when no context is current or the query failed

class ContextCache {
 public:
  bool get(uint64_t ctx, void** value) {
    std::lock_guard<std::mutex> lock(mu_);
    for (int i = 0; i < n_; ++i)
      if (ids_[i] == ctx) {
        *value = vals_[i];
        return true;
      }
    return false;
  }
  void put(uint64_t ctx, void* value) {
    std::lock_guard<std::mutex> lock(mu_);
    for (int i = 0; i < n_; ++i)
      if (ids_[i] == ctx) {
        vals_[i] = value;
        return;
      }
    const int slot = n_ < kSlots ? n_++ : static_cast<int>(next_++ % kSlots);  // oldest goes
    ids_[slot] = ctx;
    vals_[slot] = value;
  }

 private:
  static constexpr int kSlots = 64;
  std::mutex mu_;
  uint64_t ids_[kSlots] = {};
  void* vals_[kSlots] = {};
  int n_ = 0;
  uint64_t next_ = 0;
};

// cudaGetSymbolAddress of `symbol` in the current context, cached per context.
cudaError_t context_symbol_address(ContextCache& cache, const void* symbol, void** out);
// cudaFuncSetAttribute(fn, MaxDynamicSharedMemorySize, bytes) once per context.
cudaError_t ensure_max_dynamic_smem(ContextCache& cache, const void* fn, int bytes);

// Record a message for fvq_last_error() and return `code` (fvq_api.cu).
int report_error(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));

// Kernels (fvq_quant.cu)
cudaError_t launch_amax(const uint16_t* x, int64_t numel, float* amax_out, float* g_out,
                        uint32_t* ws, float* zero_word, cudaStream_t st);
// scratch_input: x is a scratch buffer nothing reads afterwards; it is walked from its
// end and its 128-byte lines are dropped from L2 after reading (no write-back).
cudaError_t launch_quantize(const uint16_t* x, int64_t rows, int64_t k, const float* g,
                            const float* amax, float* g_out, uint8_t* codes, uint8_t* sf,
                            float* zero_word, cudaStream_t st, bool scratch_input = false);
cudaError_t launch_rcp_probe(const float* in, float* out, int64_t n, cudaStream_t st);
// amax + global scale + quantize of x in one cooperative launch; with rep_dst != NULL it
// also writes the replicated W scales of an [rep_n, rep_k] weight.  ws: the amax workspace
// (counter ws[0] and generation ws[1] left re-armed), ws[2] receives amax.
cudaError_t launch_amax_quantize(const uint16_t* x, int64_t rows, int64_t k, float* g_out,
                                 uint8_t* codes, uint8_t* sf, uint32_t* ws, float* zero_word,
                                 const uint8_t* rep_src, int64_t rep_n, int64_t rep_k,
                                 uint8_t* rep_dst, uint64_t wait_limit, uint32_t* err_word,
                                 cudaStream_t st);
// launch_amax_quantize of u = bf16(bf16(LN(x) * bf16(1 + scale)) + shift) (LayerNorm
// without affine, as launch_ln_modulate) without writing u: pass 1 keeps each row's
// (mean, rstd) in stats[2 * rows] and takes max |u|, pass 2 recomputes u from x.
// k % 64 == 0 and k <= 2048.
cudaError_t launch_amax_quantize_ln(const uint16_t* x, int64_t rows, int64_t k,
                                    const uint16_t* shift, const uint16_t* scale, float eps,
                                    float* stats, float* g_out, uint8_t* codes, uint8_t* sf,
                                    uint32_t* ws, float* zero_word, const uint8_t* rep_src,
                                    int64_t rep_n, int64_t rep_k, uint8_t* rep_dst,
                                    uint64_t wait_limit, uint32_t* err_word, cudaStream_t st);
// W scales (128x4 layout, n % 256 == 0, k % 256 == 0) -> the replicated layout the
// GEMM's 128x256b scale copies read; 4 * n * k / 16 bytes.
cudaError_t launch_replicate_w_scales(const uint8_t* sf, int64_t n, int64_t k, uint8_t* rep,
                                      cudaStream_t st);

// GEMM (fvq_gemm.cu)
// Epilogue 3 (GEMM1 quantizing its own output): bias, GELU and the amax as epilogue 1,
// then NVFP4 codes [m, n/2] and 128x4-swizzled E4M3 scales of the result with the
// provisional encode scale g = 2^-headroom_log2 * 2688 / max(*amax_hint, 1e-12), written
// to `codes` / `sf` (no bf16 output).  g_used (optional) receives g; flags (optional) collects
// kQuantSaturated (a block's scale value g * vmax / 6 exceeded 448 and was clipped)
// and kQuantUnderflow (a nonzero block's scale rounded to zero).
constexpr uint32_t kQuantSaturated = 1u << 0;
constexpr uint32_t kQuantUnderflow = 1u << 1;
struct QuantOut {
  uint8_t* codes = nullptr;
  uint8_t* sf = nullptr;
  const float* amax_hint = nullptr;
  int headroom_log2 = 0;
  float* g_used = nullptr;
  uint32_t* flags = nullptr;
  float* zero_word = nullptr;  // epilogue 1: set to 0 before any tile (a later GEMM's amax target)
};
cudaError_t launch_gemm(const uint8_t* a_codes, const uint8_t* a_sf, const float* g_a,
                        const uint8_t* w_codes, const uint8_t* w_sf, const float* g_w,
                        const float* alpha, const uint16_t* bias, uint16_t* out, int64_t m, int64_t n, int64_t k,
                        int epilogue, float* amax_out, uint64_t wait_limit, cudaStream_t st,
                        const char** why, const uint8_t* w_sf_rep = nullptr,
                        const uint16_t* residual = nullptr, const uint16_t* gate = nullptr,
                        const QuantOut* qo = nullptr);
// epilogue 2 (replicated W scales only): out = bf16(residual + bf16(gate[n] * y)), y the
// epilogue-0 result -- the gated residual of a DiT block around its FFN.
// Epilogues 0 and 2 with amax_out: max |out| over the real rows (bf16 magnitudes, NaN
// ignored, as launch_amax takes it) is maxed into *amax_out, which must start at 0;
// epilogue 1 with qo->zero_word: that word is set to 0 before any tile (so that a later
// GEMM of the same sequence can max into it).
// FVQ_EPI_BF16 GEMMs with replicated W scales, alpha from the global scales and
// m % 256 == 0 run on SM pairs (nvfp4_gemm_pair_kernel) when enabled.
void set_gemm_pairing(int mode);  // 0 off, 1 pairs (raw W scales), 2 pairs (replicated)
bool gemm_pairs(int64_t m, int epilogue);
// The plain-epilogue GEMM of m rows runs on SM pairs reading W scales in their
// library layout (pairing mode 1), so it needs no replicated copy of them.
bool gemm_pairs_raw_scales(int64_t m);
cudaError_t launch_gelu_probe(const uint16_t* in, uint16_t* out, int64_t count, cudaStream_t st);
// E4M3 GEMM with per-row A scales and per-column W scales (fvq_gemm.cu); epilogue 1:
// bias, GELU and per-row max |h| (fp32 bits) into row_amax.  k % 128 == 0, n % 256 == 0.
cudaError_t launch_fp8_gemm(const uint8_t* a, const float* sa, const uint8_t* w, const float* sw,
                            const uint16_t* bias, uint16_t* out, int64_t m, int64_t n, int64_t k,
                            int epilogue, uint32_t* row_amax, uint64_t wait_limit, cudaStream_t st,
                            const char** why);

// FP8 GEMMs on SM pairs (fp8_gemm_pair_kernel, 256 x 256 tiles) or one SM per tile:
// 0 never pairs, 1 pairs the plain-epilogue GEMMs (default), 2 pairs all.
void set_fp8_gemm_pairing(int mode);

// FP8 quantizers (fvq_fp8.cu).  Row: one scale per row, k % 8 == 0 and
// k <= fp8_row_quant_max_k(); row_amax != NULL supplies each row's max |x| (fp32
// bits); zero_rows != NULL gets zero in each row's word.  Tensor: one scale from a
// device amax.
int64_t fp8_row_quant_max_k();
cudaError_t launch_fp8_row_quant(const uint16_t* x, int64_t rows, int64_t k, uint8_t* q,
                                 float* scale, const uint32_t* row_amax, uint32_t* zero_rows,
                                 cudaStream_t st);
cudaError_t launch_fp8_tensor_quant(const uint16_t* x, int64_t numel, const float* amax,
                                    uint8_t* q, float* scale, cudaStream_t st);
cudaError_t launch_div_full_probe(const float* a, const float* b, float* out, int64_t n,
                                  cudaStream_t st);
// Pillow-exact bicubic upscale + crop (+ bf16 normalisation), and the normalisation on
// its own (fvq_resize.cu).  smem_needed receives the CTA's shared memory; a plan that does
// not fit returns cudaErrorInvalidValue.
cudaError_t launch_pil_resize(const uint8_t* src, int64_t frames, int in_h, int in_w, int out_h,
                              int out_w, int crop_y, int crop_x, int crop_h, int crop_w,
                              uint8_t* dst_u8, uint16_t* dst_bf16, size_t* smem_needed,
                              cudaStream_t st);
cudaError_t launch_pil_normalize(const uint8_t* src, int64_t frames, int h, int w, int64_t sb,
                                 int64_t sy, int64_t sx, uint16_t* dst, cudaStream_t st);
// u = bf16(bf16(LN(x) * bf16(1 + scale)) + shift), one warp per row, d % 8 == 0, d <= 2048
// (fvq_block.cu).
cudaError_t launch_ln_modulate(const uint16_t* x, int64_t rows, int64_t d, const uint16_t* shift,
                               const uint16_t* scale, float eps, uint16_t* u, cudaStream_t st);
cudaError_t set_error_word(uint32_t v, cudaStream_t st);
uint32_t* error_word_ptr();   // device address of the error word (current device)
cudaError_t read_error_word(uint32_t* v, cudaStream_t st);

}  // namespace fvq
