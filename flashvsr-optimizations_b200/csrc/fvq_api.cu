// fvq_api.cu -- the extern "C" boundary (include/fvq.h): argument checks,
// status codes, per-thread error text, workspace carving and the call
// sequences of QuantLinear.forward and the FFN.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/fvq.h"
#include "fvq_internal.h"

namespace {

thread_local std::string g_last_error;
// Process-wide bound on device waits (fvq_set_wait_limit); read by every launch path from
// any host thread, hence atomic.
std::atomic<uint64_t> g_wait_limit_ns{fvq::kDefaultWaitLimit};
uint64_t wait_limit() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(FVQ_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
// the quantizer reads bf16 inputs in 32-byte vectors
bool aligned32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31u) == 0; }

int check_device() {
  static int ok_cache[64] = {0};  // 0 unknown, 1 ok, -1 bad
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev >= 0 && dev < 64 && ok_cache[dev] == 1) return FVQ_OK;
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) {
    return fail(FVQ_EDEVICE, "device %d is sm_%d%d; this library is built for sm_100a (B200)", dev,
                major, minor);
  }
  if (dev >= 0 && dev < 64) ok_cache[dev] = 1;
  return FVQ_OK;
}

constexpr size_t kAlign = 256;
size_t round_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Workspace carving shared by linear and ffn.
struct Carve {
  uint8_t* base;
  size_t off = 0;
  explicit Carve(void* b) : base(static_cast<uint8_t*>(b)) {}
  uint8_t* take(size_t bytes) {
    uint8_t* p = base ? base + off : nullptr;
    off += round_up(bytes);
    return p;
  }
};

constexpr size_t kScalarBytes = 256;  // g_x, g_h, amax_h, spare

int check_quant_shape(int64_t rows, int64_t k, const char* who) {
  if (rows <= 0) return fail(FVQ_EINVAL, "%s: rows must be > 0 (got %lld)", who, (long long)rows);
  if (k <= 0 || k % 64 != 0)
    return fail(FVQ_EINVAL, "%s: k must be a positive multiple of 64 (got %lld)", who,
                (long long)k);
  if (rows > (int64_t(1) << 31) || k > (int64_t(1) << 24) ||
      (rows + 128) * (k / 16) >= (int64_t(1) << 31))
    return fail(FVQ_EINVAL, "%s: shape too large (pad128(rows) * k / 16 must stay below 2^31)",
                who);
  return FVQ_OK;
}

int check_gemm_shape(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || m > (int64_t(1) << 30))
    return fail(FVQ_EINVAL, "fvq_nvfp4_gemm: m must be in [1, 2^30] (got %lld)", (long long)m);
  if (n <= 0 || n % 256 != 0)
    return fail(FVQ_EINVAL, "fvq_nvfp4_gemm: n must be a positive multiple of 256 (got %lld)",
                (long long)n);
  if (k <= 0 || k % 256 != 0)
    return fail(FVQ_EINVAL, "fvq_nvfp4_gemm: k must be a positive multiple of 256 (got %lld)",
                (long long)k);
  if (n * k / 2 > (int64_t(1) << 31) || m * (k / 2) > (int64_t(1) << 40))
    return fail(FVQ_EINVAL, "fvq_nvfp4_gemm: operand too large");
  return FVQ_OK;
}

int gemm_impl(const uint8_t* a_codes, const uint8_t* a_sf, const float* g_a,
              const uint8_t* w_codes, const uint8_t* w_sf, const float* g_w, const float* alpha,
              const uint16_t* bias, uint16_t* out, int64_t m, int64_t n, int64_t k, int epilogue,
              float* amax_out, cudaStream_t st, const uint8_t* w_sf_rep = nullptr,
              const uint16_t* residual = nullptr, const uint16_t* gate = nullptr) {
  const char* why = nullptr;
  cudaError_t e = fvq::launch_gemm(a_codes, a_sf, g_a, w_codes, w_sf, g_w, alpha, bias, out, m, n, k,
                                   epilogue, amax_out, wait_limit(), st, &why, w_sf_rep, residual,
                                   gate);
  if (e != cudaSuccess) {
    if (why) return fail(FVQ_ECUDA, "fvq_nvfp4_gemm: %s", why);
    return cuda_fail(e, "fvq_nvfp4_gemm launch");
  }
  return FVQ_OK;
}

}  // namespace

namespace fvq {
int report_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}
}  // namespace fvq

extern "C" {

int fvq_version(void) { return 100; }

const char* fvq_last_error(void) { return g_last_error.c_str(); }

size_t fvq_amax_workspace_bytes(void) { return round_up(fvq::kAmaxWorkspaceBytes); }

int fvq_amax(const uint16_t* x, int64_t numel, float* amax_out, float* g_out, void* workspace,
             size_t workspace_bytes, void* stream) {
  if (numel < 0) return fail(FVQ_EINVAL, "fvq_amax: numel < 0");
  if (numel > 0 && x == nullptr) return fail(FVQ_EINVAL, "fvq_amax: x is NULL");
  if (workspace == nullptr) return fail(FVQ_EINVAL, "fvq_amax: workspace is NULL");
  if (workspace_bytes < fvq_amax_workspace_bytes())
    return fail(FVQ_EWORKSPACE, "fvq_amax: workspace needs %zu bytes, got %zu",
                fvq_amax_workspace_bytes(), workspace_bytes);
  if (!aligned16(x) || !aligned16(workspace))
    return fail(FVQ_EALIGN, "fvq_amax: x and workspace must be 16-byte aligned");
  if (int rc = check_device()) return rc;
  cudaError_t e = fvq::launch_amax(x, numel, amax_out, g_out, static_cast<uint32_t*>(workspace),
                                   nullptr, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fvq_amax launch");
  return FVQ_OK;
}

int fvq_nvfp4_quantize(const uint16_t* x, int64_t rows, int64_t k, const float* g,
                       uint8_t* codes, uint8_t* sf, void* stream) {
  if (int rc = check_quant_shape(rows, k, "fvq_nvfp4_quantize")) return rc;
  if (!x || !g || !codes || !sf) return fail(FVQ_EINVAL, "fvq_nvfp4_quantize: NULL pointer");
  if (!aligned32(x) || !aligned16(codes) || !aligned16(sf))
    return fail(FVQ_EALIGN, "fvq_nvfp4_quantize: x must be 32-byte aligned, codes and sf 16-byte");
  if (int rc = check_device()) return rc;
  cudaError_t e = fvq::launch_quantize(x, rows, k, g, nullptr, nullptr, codes, sf, nullptr,
                                       static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fvq_nvfp4_quantize launch");
  return FVQ_OK;
}

int fvq_nvfp4_quantize_dynamic(const uint16_t* x, int64_t rows, int64_t k, const float* amax_in,
                               float* g_out, uint8_t* codes, uint8_t* sf, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (int rc = check_quant_shape(rows, k, "fvq_nvfp4_quantize_dynamic")) return rc;
  if (!x || !codes || !sf) return fail(FVQ_EINVAL, "fvq_nvfp4_quantize_dynamic: NULL pointer");
  if (!aligned32(x) || !aligned16(codes) || !aligned16(sf))
    return fail(FVQ_EALIGN,
                "fvq_nvfp4_quantize_dynamic: x must be 32-byte aligned, codes and sf 16-byte");
  if (int rc = check_device()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float* amax = amax_in;
  if (amax == nullptr) {
    if (workspace == nullptr || workspace_bytes < fvq_amax_workspace_bytes())
      return fail(FVQ_EWORKSPACE, "fvq_nvfp4_quantize_dynamic: workspace needs %zu bytes",
                  fvq_amax_workspace_bytes());
    if (!aligned16(workspace))
      return fail(FVQ_EALIGN, "fvq_nvfp4_quantize_dynamic: workspace must be 16-byte aligned");
    // amax, global scale and quantization in one launch
    uint32_t* ws = static_cast<uint32_t*>(workspace);
    cudaError_t e = fvq::launch_amax_quantize(x, rows, k, g_out, codes, sf, ws, nullptr, nullptr, 0,
                                              0, nullptr, wait_limit(), fvq::error_word_ptr(), st);
    if (e != cudaSuccess) return cuda_fail(e, "fvq_nvfp4_quantize_dynamic launch");
    return FVQ_OK;
  }
  cudaError_t e = fvq::launch_quantize(x, rows, k, nullptr, amax, g_out, codes, sf, nullptr, st);
  if (e != cudaSuccess) return cuda_fail(e, "fvq_nvfp4_quantize_dynamic launch");
  return FVQ_OK;
}

int fvq_nvfp4_gemm(const uint8_t* a_codes, const uint8_t* a_sf, const float* g_a,
                   const uint8_t* w_codes, const uint8_t* w_sf, const float* g_w,
                   const uint16_t* bias, uint16_t* out, int64_t m, int64_t n, int64_t k,
                   int epilogue, float* amax_out, void* stream) {
  if (int rc = check_gemm_shape(m, n, k)) return rc;
  if (!a_codes || !a_sf || !g_a || !w_codes || !w_sf || !g_w || !out)
    return fail(FVQ_EINVAL, "fvq_nvfp4_gemm: NULL pointer");
  if (epilogue != FVQ_EPI_BF16 && epilogue != FVQ_EPI_GELU_AMAX)
    return fail(FVQ_EINVAL, "fvq_nvfp4_gemm: unknown epilogue %d", epilogue);
  if (epilogue == FVQ_EPI_GELU_AMAX && amax_out == nullptr)
    return fail(FVQ_EINVAL, "fvq_nvfp4_gemm: FVQ_EPI_GELU_AMAX needs amax_out");
  if (!aligned16(a_codes) || !aligned16(a_sf) || !aligned16(w_codes) || !aligned16(w_sf) ||
      !aligned16(out) || !aligned16(bias))
    return fail(FVQ_EALIGN, "fvq_nvfp4_gemm: operands, scales, bias and out must be 16-byte aligned");
  if (int rc = check_device()) return rc;
  return gemm_impl(a_codes, a_sf, g_a, w_codes, w_sf, g_w, nullptr, bias, out, m, n, k, epilogue,
                   epilogue == FVQ_EPI_GELU_AMAX ? amax_out : nullptr,
                   static_cast<cudaStream_t>(stream));
}

size_t fvq_w_scales_replicated_bytes(int64_t n, int64_t k) {
  if (n <= 0 || k <= 0) return 0;
  return static_cast<size_t>(4 * n * (k / 16));
}

int fvq_replicate_w_scales(const uint8_t* w_sf, int64_t n, int64_t k, uint8_t* w_sf_rep,
                           void* stream) {
  if (n <= 0 || n % 256 != 0 || k <= 0 || k % 256 != 0)
    return fail(FVQ_EINVAL, "fvq_replicate_w_scales: n and k must be positive multiples of 256 "
                "(got %lld, %lld)", (long long)n, (long long)k);
  if (!w_sf || !w_sf_rep) return fail(FVQ_EINVAL, "fvq_replicate_w_scales: NULL pointer");
  if (!aligned16(w_sf) || !aligned16(w_sf_rep))
    return fail(FVQ_EALIGN, "fvq_replicate_w_scales: pointers must be 16-byte aligned");
  if (int rc = check_device()) return rc;
  cudaError_t e = fvq::launch_replicate_w_scales(w_sf, n, k, w_sf_rep,
                                                 static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fvq_replicate_w_scales launch");
  return FVQ_OK;
}

int fvq_nvfp4_gemm_wrep(const uint8_t* a_codes, const uint8_t* a_sf, const float* g_a,
                        const uint8_t* w_codes, const uint8_t* w_sf_rep, const float* g_w,
                        const uint16_t* bias, uint16_t* out, int64_t m, int64_t n, int64_t k,
                        void* stream) {
  if (int rc = check_gemm_shape(m, n, k)) return rc;
  if (!a_codes || !a_sf || !g_a || !w_codes || !w_sf_rep || !g_w || !out)
    return fail(FVQ_EINVAL, "fvq_nvfp4_gemm_wrep: NULL pointer");
  if (!aligned16(a_codes) || !aligned16(a_sf) || !aligned16(w_codes) || !aligned16(w_sf_rep) ||
      !aligned16(out) || !aligned16(bias))
    return fail(FVQ_EALIGN,
                "fvq_nvfp4_gemm_wrep: operands, scales, bias and out must be 16-byte aligned");
  if (int rc = check_device()) return rc;
  return gemm_impl(a_codes, a_sf, g_a, w_codes, nullptr, g_w, nullptr, bias, out, m, n, k,
                   FVQ_EPI_BF16, nullptr, static_cast<cudaStream_t>(stream), w_sf_rep);
}

int fvq_nvfp4_mm(const uint8_t* a_codes, const uint8_t* a_sf, const uint8_t* w_codes,
                 const uint8_t* w_sf, const float* alpha, const uint16_t* bias, uint16_t* out,
                 int64_t m, int64_t n, int64_t k, void* stream) {
  if (int rc = check_gemm_shape(m, n, k)) return rc;
  if (!a_codes || !a_sf || !w_codes || !w_sf || !alpha || !out)
    return fail(FVQ_EINVAL, "fvq_nvfp4_mm: NULL pointer");
  if (!aligned16(a_codes) || !aligned16(a_sf) || !aligned16(w_codes) || !aligned16(w_sf) ||
      !aligned16(out) || !aligned16(bias))
    return fail(FVQ_EALIGN, "fvq_nvfp4_mm: operands, scales, bias and out must be 16-byte aligned");
  if (int rc = check_device()) return rc;
  return gemm_impl(a_codes, a_sf, nullptr, w_codes, w_sf, nullptr, alpha, bias, out, m, n, k,
                   FVQ_EPI_BF16, nullptr, static_cast<cudaStream_t>(stream));
}

size_t fvq_nvfp4_linear_workspace_bytes(int64_t rows, int64_t in_features) {
  if (rows <= 0 || in_features <= 0) return 0;
  Carve c(nullptr);
  c.take(fvq::kAmaxWorkspaceBytes);
  c.take(kScalarBytes);
  c.take(static_cast<size_t>(rows * in_features / 2));
  c.take(fvq::sf_bytes(rows, in_features));
  return c.off;
}

static int check_linear(const fvq_linear* lin, const char* who) {
  if (lin == nullptr) return fail(FVQ_EINVAL, "%s: linear descriptor is NULL", who);
  if (!lin->qweight || !lin->scale || !lin->global_sf)
    return fail(FVQ_EINVAL, "%s: qweight, scale and global_sf are required", who);
  if (lin->in_features <= 0 || lin->in_features % 256 != 0 || lin->out_features <= 0 ||
      lin->out_features % 256 != 0)
    return fail(FVQ_EINVAL, "%s: in/out features must be positive multiples of 256 (got %lld, %lld)",
                who, (long long)lin->in_features, (long long)lin->out_features);
  if (!aligned16(lin->qweight) || !aligned16(lin->scale) || !aligned16(lin->bias))
    return fail(FVQ_EALIGN, "%s: weight buffers must be 16-byte aligned", who);
  return FVQ_OK;
}

int fvq_nvfp4_linear(const uint16_t* x, int64_t rows, const fvq_linear* lin, uint16_t* y,
                     void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_linear(lin, "fvq_nvfp4_linear")) return rc;
  if (int rc = check_quant_shape(rows, lin->in_features, "fvq_nvfp4_linear")) return rc;
  if (!x || !y || !workspace) return fail(FVQ_EINVAL, "fvq_nvfp4_linear: NULL pointer");
  const size_t need = fvq_nvfp4_linear_workspace_bytes(rows, lin->in_features);
  if (workspace_bytes < need)
    return fail(FVQ_EWORKSPACE, "fvq_nvfp4_linear: workspace needs %zu bytes, got %zu", need,
                workspace_bytes);
  if (!aligned32(x) || !aligned16(y) || !aligned16(workspace))
    return fail(FVQ_EALIGN, "fvq_nvfp4_linear: x must be 32-byte aligned, y and workspace 16-byte");
  if (int rc = check_device()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t k = lin->in_features;
  Carve c(workspace);
  uint32_t* amax_ws = reinterpret_cast<uint32_t*>(c.take(fvq::kAmaxWorkspaceBytes));
  float* scalars = reinterpret_cast<float*>(c.take(kScalarBytes));
  uint8_t* codes = c.take(static_cast<size_t>(rows * k / 2));
  uint8_t* sf = c.take(fvq::sf_bytes(rows, k));
  cudaError_t e = fvq::launch_amax_quantize(x, rows, k, &scalars[0], codes, sf, amax_ws, nullptr,
                                            nullptr, 0, 0, nullptr, wait_limit(),
                                            fvq::error_word_ptr(), st);
  if (e != cudaSuccess) return cuda_fail(e, "fvq_nvfp4_linear quantize launch");
  return gemm_impl(codes, sf, &scalars[0], lin->qweight, lin->scale, lin->global_sf, nullptr,
                   lin->bias, y,
                   rows, lin->out_features, k, FVQ_EPI_BF16, nullptr, st);
}

size_t fvq_nvfp4_ffn_workspace_bytes(int64_t rows, int64_t d_model, int64_t d_ff) {
  if (rows <= 0 || d_model <= 0 || d_ff <= 0) return 0;
  Carve c(nullptr);
  c.take(fvq::kAmaxWorkspaceBytes);
  c.take(kScalarBytes);
  c.take(static_cast<size_t>(rows * d_model / 2));
  c.take(fvq::sf_bytes(rows, d_model));
  c.take(static_cast<size_t>(rows * d_ff * 2));
  c.take(static_cast<size_t>(rows * d_ff / 2));
  c.take(fvq::sf_bytes(rows, d_ff));
  c.take(static_cast<size_t>(4 * d_model * (d_ff / 16)));  // W2 scales, replicated
  return c.off;
}

namespace {

// The FFN launch sequence.  ev: NULL, or 5 events recorded before the first
// launch and after each of the four (for fvq_nvfp4_ffn_profile).  residual and
// gate (both or neither): GEMM2 writes the gated residual residual + gate * FFN(x).
// x_amax (optional): max |x| given, so the first launch only quantizes x; y_amax
// (optional): receives max |y| from GEMM2's epilogue (fvq_nvfp4_ffn_chain).
// LnModulate: the DiT block's input step, applied to x inside the first launch.
struct LnModulate {
  const uint16_t* shift;
  const uint16_t* scale;
  float eps;
  float* stats;  // [2 * rows] floats of scratch
};

int ffn_impl(const uint16_t* x, int64_t rows, const fvq_linear* lin1, const fvq_linear* lin2,
             uint16_t* y, void* workspace, size_t workspace_bytes, cudaStream_t st,
             cudaEvent_t* ev, const uint16_t* residual = nullptr, const uint16_t* gate = nullptr,
             const LnModulate* ln = nullptr, const float* x_amax = nullptr,
             float* y_amax = nullptr) {
  if (int rc = check_linear(lin1, "fvq_nvfp4_ffn (linear 1)")) return rc;
  if (int rc = check_linear(lin2, "fvq_nvfp4_ffn (linear 2)")) return rc;
  if (lin1->out_features != lin2->in_features || lin2->out_features != lin1->in_features)
    return fail(FVQ_EINVAL, "fvq_nvfp4_ffn: linear shapes do not chain (%lld->%lld, %lld->%lld)",
                (long long)lin1->in_features, (long long)lin1->out_features,
                (long long)lin2->in_features, (long long)lin2->out_features);
  if (int rc = check_quant_shape(rows, lin1->in_features, "fvq_nvfp4_ffn")) return rc;
  if (!x || !y || !workspace) return fail(FVQ_EINVAL, "fvq_nvfp4_ffn: NULL pointer");
  const int64_t d = lin1->in_features, f = lin1->out_features;
  const size_t need = fvq_nvfp4_ffn_workspace_bytes(rows, d, f);
  if (workspace_bytes < need)
    return fail(FVQ_EWORKSPACE, "fvq_nvfp4_ffn: workspace needs %zu bytes, got %zu", need,
                workspace_bytes);
  if (!aligned32(x) || !aligned16(y) || !aligned16(workspace))
    return fail(FVQ_EALIGN, "fvq_nvfp4_ffn: x must be 32-byte aligned, y and workspace 16-byte");
  if (int rc = check_device()) return rc;
  Carve c(workspace);
  uint32_t* amax_ws = reinterpret_cast<uint32_t*>(c.take(fvq::kAmaxWorkspaceBytes));
  float* scalars = reinterpret_cast<float*>(c.take(kScalarBytes));
  uint8_t* codes_x = c.take(static_cast<size_t>(rows * d / 2));
  uint8_t* sf_x = c.take(fvq::sf_bytes(rows, d));
  uint16_t* h = reinterpret_cast<uint16_t*>(c.take(static_cast<size_t>(rows * f * 2)));
  uint8_t* codes_h = c.take(static_cast<size_t>(rows * f / 2));
  uint8_t* sf_h = c.take(fvq::sf_bytes(rows, f));
  uint8_t* sf_w2_rep = c.take(static_cast<size_t>(4 * d * (f / 16)));
  // GEMM2 on SM pairs reads W2's scales as they are: skip the replicated copy
  if (fvq::gemm_pairs_raw_scales(rows)) sf_w2_rep = nullptr;
  float* g_x = &scalars[0];
  float* g_h = &scalars[1];
  float* amax_h = &scalars[2];
  auto mark = [&](int i) {
    if (ev != nullptr) cudaEventRecord(ev[i], st);
  };
  mark(0);
  // 1. amax(x) -> g_x -> x in NVFP4, one launch; it also zeroes amax_h before GEMM1
  //    accumulates into it and, when GEMM2 runs on one SM per tile, writes the W2
  //    scales in the layout of its 128x256b scale copies
  //    (for the DiT block: of u = LN(x) * (1 + scale) + shift, computed on the fly)
  //    (with x_amax given: a plain quantize of x with g_x from it, and the W2 scale copy, if
  //    needed, as a launch of its own)
  cudaError_t e = cudaSuccess;
  if (ln != nullptr) {
    e = fvq::launch_amax_quantize_ln(x, rows, d, ln->shift, ln->scale, ln->eps, ln->stats, g_x,
                                     codes_x, sf_x, amax_ws, amax_h, lin2->scale, d, f, sf_w2_rep,
                                     wait_limit(), fvq::error_word_ptr(), st);
  } else if (x_amax != nullptr) {
    e = fvq::launch_quantize(x, rows, d, nullptr, x_amax, g_x, codes_x, sf_x, amax_h, st);
    if (e == cudaSuccess && sf_w2_rep != nullptr)
      e = fvq::launch_replicate_w_scales(lin2->scale, d, f, sf_w2_rep, st);
  } else {
    e = fvq::launch_amax_quantize(x, rows, d, g_x, codes_x, sf_x, amax_ws, amax_h, lin2->scale, d,
                                  f, sf_w2_rep, wait_limit(), fvq::error_word_ptr(), st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "fvq_nvfp4_ffn quantize(x) launch");
  mark(1);
  // 2. h = bf16(gelu(bf16(bf16(alpha1 * acc) + b1))), amax_h = max |h|; y_amax zeroed for
  //    step 4
  {
    fvq::QuantOut q;
    q.zero_word = y_amax;
    const char* why = nullptr;
    e = fvq::launch_gemm(codes_x, sf_x, g_x, lin1->qweight, lin1->scale, lin1->global_sf, nullptr,
                         lin1->bias, h, rows, f, d, FVQ_EPI_GELU_AMAX, amax_h, wait_limit(), st,
                         &why, nullptr, nullptr, nullptr, &q);
    if (e != cudaSuccess) {
      if (why) return fail(FVQ_ECUDA, "fvq_nvfp4_ffn GEMM1: %s", why);
      return cuda_fail(e, "fvq_nvfp4_ffn GEMM1 launch");
    }
  }
  mark(2);
  // 3. h -> NVFP4 with g_h = 2688 / max(amax_h, 1e-12); h is scratch, so its lines
  //    are dropped from L2 once read
  e = fvq::launch_quantize(h, rows, f, nullptr, amax_h, g_h, codes_h, sf_h, nullptr, st,
                           /*scratch_input=*/true);
  if (e != cudaSuccess) return cuda_fail(e, "fvq_nvfp4_ffn quantize(h) launch");
  mark(3);
  // 4. y = bf16(bf16(alpha2 * acc) + b2)  [then bf16(residual + bf16(gate * y))]
  if (int rc = gemm_impl(codes_h, sf_h, g_h, lin2->qweight, lin2->scale, lin2->global_sf, nullptr,
                         lin2->bias, y, rows, d, f, residual ? 2 : FVQ_EPI_BF16, y_amax, st,
                         sf_w2_rep, residual, gate))
    return rc;
  mark(4);
  return FVQ_OK;
}

}  // namespace

int fvq_nvfp4_ffn(const uint16_t* x, int64_t rows, const fvq_linear* lin1, const fvq_linear* lin2,
                  uint16_t* y, void* workspace, size_t workspace_bytes, void* stream) {
  return ffn_impl(x, rows, lin1, lin2, y, workspace, workspace_bytes,
                  static_cast<cudaStream_t>(stream), nullptr);
}

int fvq_nvfp4_ffn_chain(const uint16_t* x, int64_t rows, const fvq_linear* lin1,
                        const fvq_linear* lin2, uint16_t* y, const float* x_amax, float* y_amax,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (y_amax != nullptr && static_cast<const void*>(y_amax) == static_cast<const void*>(x_amax))
    return fail(FVQ_EINVAL, "fvq_nvfp4_ffn_chain: y_amax must not alias x_amax (the call zeroes "
                "y_amax while its first launch may still read x_amax)");
  if (x_amax != nullptr && !aligned4(x_amax))
    return fail(FVQ_EALIGN, "fvq_nvfp4_ffn_chain: x_amax must be 4-byte aligned");
  if (y_amax != nullptr && !aligned4(y_amax))
    return fail(FVQ_EALIGN, "fvq_nvfp4_ffn_chain: y_amax must be 4-byte aligned");
  return ffn_impl(x, rows, lin1, lin2, y, workspace, workspace_bytes,
                  static_cast<cudaStream_t>(stream), nullptr, nullptr, nullptr, nullptr, x_amax,
                  y_amax);
}

size_t fvq_nvfp4_ffn_fused_workspace_bytes(int64_t rows, int64_t d_model, int64_t d_ff) {
  if (rows <= 0 || d_model <= 0 || d_ff <= 0) return 0;
  Carve c(nullptr);
  c.take(fvq::kAmaxWorkspaceBytes);
  c.take(kScalarBytes);
  c.take(static_cast<size_t>(rows * d_model / 2));
  c.take(fvq::sf_bytes(rows, d_model));
  c.take(static_cast<size_t>(rows * d_ff / 2));
  c.take(fvq::sf_bytes(rows, d_ff));
  c.take(static_cast<size_t>(4 * d_model * (d_ff / 16)));  // W2 scales, replicated
  return c.off;
}

namespace {

// The FFN with the intermediate quantized inside GEMM1's epilogue (three launches):
// amax + quantize of x (which also zeroes the amax word GEMM1 maxes into) -> GEMM1 with
// bias, GELU, amax and NVFP4 quantization of h with g = 2688 / max(*amax_hint, 1e-12)
// -> GEMM2 with alpha = 1 / (g * g_w2).  ev: NULL or 4 events (profile).
int ffn_fused_impl(const uint16_t* x, int64_t rows, const fvq_linear* lin1, const fvq_linear* lin2,
                   uint16_t* y, const float* amax_hint, int headroom_log2, float* amax_seen,
                   uint32_t* flags, void* workspace, size_t workspace_bytes, cudaStream_t st,
                   cudaEvent_t* ev) {
  if (int rc = check_linear(lin1, "fvq_nvfp4_ffn_fused (linear 1)")) return rc;
  if (int rc = check_linear(lin2, "fvq_nvfp4_ffn_fused (linear 2)")) return rc;
  if (lin1->out_features != lin2->in_features || lin2->out_features != lin1->in_features)
    return fail(FVQ_EINVAL, "fvq_nvfp4_ffn_fused: linear shapes do not chain");
  if (int rc = check_quant_shape(rows, lin1->in_features, "fvq_nvfp4_ffn_fused")) return rc;
  if (!x || !y || !workspace || !amax_hint)
    return fail(FVQ_EINVAL, "fvq_nvfp4_ffn_fused: NULL pointer");
  if (headroom_log2 < 0 || headroom_log2 > 30)
    return fail(FVQ_EINVAL, "fvq_nvfp4_ffn_fused: headroom_log2 must be in [0, 30] (got %d)",
                headroom_log2);
  if (amax_seen != nullptr && amax_seen == amax_hint)
    return fail(FVQ_EINVAL, "fvq_nvfp4_ffn_fused: amax_seen must not alias amax_hint "
                "(the call zeroes amax_seen before it reads the hint)");
  const int64_t d = lin1->in_features, f = lin1->out_features;
  const size_t need = fvq_nvfp4_ffn_fused_workspace_bytes(rows, d, f);
  if (workspace_bytes < need)
    return fail(FVQ_EWORKSPACE, "fvq_nvfp4_ffn_fused: workspace needs %zu bytes, got %zu", need,
                workspace_bytes);
  if (!aligned32(x) || !aligned16(y) || !aligned16(workspace))
    return fail(FVQ_EALIGN, "fvq_nvfp4_ffn_fused: x must be 32-byte aligned, y and workspace 16-byte");
  if (int rc = check_device()) return rc;
  Carve c(workspace);
  uint32_t* amax_ws = reinterpret_cast<uint32_t*>(c.take(fvq::kAmaxWorkspaceBytes));
  float* scalars = reinterpret_cast<float*>(c.take(kScalarBytes));
  uint8_t* codes_x = c.take(static_cast<size_t>(rows * d / 2));
  uint8_t* sf_x = c.take(fvq::sf_bytes(rows, d));
  uint8_t* codes_h = c.take(static_cast<size_t>(rows * f / 2));
  uint8_t* sf_h = c.take(fvq::sf_bytes(rows, f));
  uint8_t* sf_w2_rep = c.take(static_cast<size_t>(4 * d * (f / 16)));
  if (fvq::gemm_pairs_raw_scales(rows)) sf_w2_rep = nullptr;
  float* g_x = &scalars[0];
  float* g_h = &scalars[1];
  float* amax_h = amax_seen != nullptr ? amax_seen : &scalars[2];
  auto mark = [&](int i) {
    if (ev != nullptr) cudaEventRecord(ev[i], st);
  };
  mark(0);
  cudaError_t e = fvq::launch_amax_quantize(x, rows, d, g_x, codes_x, sf_x, amax_ws, amax_h,
                                            lin2->scale, d, f, sf_w2_rep, wait_limit(),
                                            fvq::error_word_ptr(), st);
  if (e != cudaSuccess) return cuda_fail(e, "fvq_nvfp4_ffn_fused quantize(x) launch");
  mark(1);
  fvq::QuantOut qo;
  qo.codes = codes_h;
  qo.sf = sf_h;
  qo.amax_hint = amax_hint;
  qo.headroom_log2 = headroom_log2;
  qo.g_used = g_h;
  qo.flags = flags;
  const char* why = nullptr;
  e = fvq::launch_gemm(codes_x, sf_x, g_x, lin1->qweight, lin1->scale, lin1->global_sf, nullptr,
                       lin1->bias, nullptr, rows, f, d, 3, amax_h, wait_limit(), st, &why, nullptr,
                       nullptr, nullptr, &qo);
  if (e != cudaSuccess) {
    if (why) return fail(FVQ_ECUDA, "fvq_nvfp4_ffn_fused GEMM1: %s", why);
    return cuda_fail(e, "fvq_nvfp4_ffn_fused GEMM1 launch");
  }
  mark(2);
  if (int rc = gemm_impl(codes_h, sf_h, g_h, lin2->qweight, lin2->scale, lin2->global_sf, nullptr,
                         lin2->bias, y, rows, d, f, FVQ_EPI_BF16, nullptr, st, sf_w2_rep))
    return rc;
  mark(3);
  return FVQ_OK;
}

}  // namespace

int fvq_nvfp4_ffn_fused(const uint16_t* x, int64_t rows, const fvq_linear* lin1,
                        const fvq_linear* lin2, uint16_t* y, const float* amax_hint,
                        int headroom_log2, float* amax_seen, uint32_t* flags, void* workspace,
                        size_t workspace_bytes, void* stream) {
  return ffn_fused_impl(x, rows, lin1, lin2, y, amax_hint, headroom_log2, amax_seen, flags,
                        workspace, workspace_bytes, static_cast<cudaStream_t>(stream), nullptr);
}

int fvq_nvfp4_ffn_fused_profile(const uint16_t* x, int64_t rows, const fvq_linear* lin1,
                                const fvq_linear* lin2, uint16_t* y, const float* amax_hint,
                                int headroom_log2, float* amax_seen, uint32_t* flags, void* workspace,
                                size_t workspace_bytes, void* stream, float* kernel_ms) {
  if (kernel_ms == nullptr)
    return fail(FVQ_EINVAL, "fvq_nvfp4_ffn_fused_profile: kernel_ms is NULL");
  if (int rc = check_device()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaEvent_t ev[4];
  int made = 0;
  for (; made < 4; ++made) {
    if (cudaEventCreate(&ev[made]) != cudaSuccess) break;
  }
  int rc = FVQ_OK;
  if (made < 4) {
    rc = fail(FVQ_ECUDA, "fvq_nvfp4_ffn_fused_profile: cudaEventCreate failed");
  } else {
    rc = ffn_fused_impl(x, rows, lin1, lin2, y, amax_hint, headroom_log2, amax_seen, flags,
                        workspace, workspace_bytes, st, ev);
    if (rc == FVQ_OK) {
      cudaError_t e = cudaEventSynchronize(ev[3]);
      for (int i = 0; e == cudaSuccess && i < 3; ++i)
        e = cudaEventElapsedTime(&kernel_ms[i], ev[i], ev[i + 1]);
      if (e != cudaSuccess) rc = cuda_fail(e, "fvq_nvfp4_ffn_fused_profile timing");
    }
  }
  for (int i = 0; i < made; ++i) cudaEventDestroy(ev[i]);
  return rc;
}

int fvq_ln_modulate(const uint16_t* x, int64_t rows, int64_t d, const uint16_t* shift,
                    const uint16_t* scale, float eps, uint16_t* u, void* stream) {
  if (rows <= 0 || d <= 0 || d % 8 != 0 || d > 2048)
    return fail(FVQ_EINVAL, "fvq_ln_modulate: rows > 0 and d a multiple of 8 up to 2048 "
                "(got %lld, %lld)", (long long)rows, (long long)d);
  if (!(eps >= 0.0f)) return fail(FVQ_EINVAL, "fvq_ln_modulate: eps must be >= 0");
  if (!x || !shift || !scale || !u) return fail(FVQ_EINVAL, "fvq_ln_modulate: NULL pointer");
  if (!aligned16(x) || !aligned16(shift) || !aligned16(scale) || !aligned16(u))
    return fail(FVQ_EALIGN, "fvq_ln_modulate: pointers must be 16-byte aligned");
  if (int rc = check_device()) return rc;
  cudaError_t e = fvq::launch_ln_modulate(x, rows, d, shift, scale, eps, u,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fvq_ln_modulate launch");
  return FVQ_OK;
}

size_t fvq_nvfp4_ffn_block_workspace_bytes(int64_t rows, int64_t d_model, int64_t d_ff) {
  if (rows <= 0 || d_model <= 0 || d_ff <= 0) return 0;
  // the FFN's workspace, then (mean, rstd) of every row
  return fvq_nvfp4_ffn_workspace_bytes(rows, d_model, d_ff) +
         round_up(static_cast<size_t>(rows) * 2 * sizeof(float));
}

int fvq_nvfp4_ffn_block(const uint16_t* x, int64_t rows, const uint16_t* shift,
                        const uint16_t* scale, const uint16_t* gate, float eps,
                        const fvq_linear* lin1, const fvq_linear* lin2, uint16_t* out,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_linear(lin1, "fvq_nvfp4_ffn_block (linear 1)")) return rc;
  if (int rc = check_linear(lin2, "fvq_nvfp4_ffn_block (linear 2)")) return rc;
  const int64_t d = lin1->in_features;
  if (lin2->out_features != d)
    return fail(FVQ_EINVAL, "fvq_nvfp4_ffn_block: the FFN must map d_model back to d_model");
  if (d > 2048 || d % 8 != 0)
    return fail(FVQ_EINVAL, "fvq_nvfp4_ffn_block: d_model must be a multiple of 8 up to 2048 "
                "(got %lld)", (long long)d);
  if (!(eps >= 0.0f)) return fail(FVQ_EINVAL, "fvq_nvfp4_ffn_block: eps must be >= 0");
  if (!x || !shift || !scale || !gate || !out || !workspace)
    return fail(FVQ_EINVAL, "fvq_nvfp4_ffn_block: NULL pointer");
  if (rows <= 0) return fail(FVQ_EINVAL, "fvq_nvfp4_ffn_block: rows must be > 0");
  const size_t need = fvq_nvfp4_ffn_block_workspace_bytes(rows, d, lin1->out_features);
  if (workspace_bytes < need)
    return fail(FVQ_EWORKSPACE, "fvq_nvfp4_ffn_block: workspace needs %zu bytes, got %zu", need,
                workspace_bytes);
  if (!aligned16(x) || !aligned16(shift) || !aligned16(scale) || !aligned16(gate) ||
      !aligned16(out) || !aligned32(workspace))
    return fail(FVQ_EALIGN, "fvq_nvfp4_ffn_block: pointers must be 16-byte aligned, the "
                "workspace 32-byte");
  if (int rc = check_device()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the FFN's workspace first, so that its zero-state amax counters sit at offset 0
  // whatever the row count; the rows' LayerNorm statistics after it.  u itself is
  // never stored: the first launch normalises, modulates and quantizes x in one go.
  const size_t ffn_bytes = fvq_nvfp4_ffn_workspace_bytes(rows, d, lin1->out_features);
  float* stats = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + ffn_bytes);
  const LnModulate ln{shift, scale, eps, stats};
  return ffn_impl(x, rows, lin1, lin2, out, workspace, ffn_bytes, st, nullptr, x, gate, &ln);
}

namespace {

int ffn_profile_impl(const uint16_t* x, int64_t rows, const fvq_linear* lin1,
                     const fvq_linear* lin2, uint16_t* y, const float* x_amax, float* y_amax,
                     void* workspace, size_t workspace_bytes, void* stream, float* kernel_ms) {
  if (kernel_ms == nullptr) return fail(FVQ_EINVAL, "fvq_nvfp4_ffn_profile: kernel_ms is NULL");
  if (y_amax != nullptr && static_cast<const void*>(y_amax) == static_cast<const void*>(x_amax))
    return fail(FVQ_EINVAL, "fvq_nvfp4_ffn_chain_profile: y_amax must not alias x_amax");
  if (int rc = check_device()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaEvent_t ev[5];
  int made = 0;
  for (; made < 5; ++made) {
    if (cudaEventCreate(&ev[made]) != cudaSuccess) break;
  }
  int rc = FVQ_OK;
  if (made < 5) {
    rc = fail(FVQ_ECUDA, "fvq_nvfp4_ffn_profile: cudaEventCreate failed");
  } else {
    rc = ffn_impl(x, rows, lin1, lin2, y, workspace, workspace_bytes, st, ev, nullptr, nullptr,
                  nullptr, x_amax, y_amax);
    if (rc == FVQ_OK) {
      cudaError_t e = cudaEventSynchronize(ev[4]);
      for (int i = 0; e == cudaSuccess && i < 4; ++i)
        e = cudaEventElapsedTime(&kernel_ms[i], ev[i], ev[i + 1]);
      if (e != cudaSuccess) rc = cuda_fail(e, "fvq_nvfp4_ffn_profile timing");
    }
  }
  for (int i = 0; i < made; ++i) cudaEventDestroy(ev[i]);
  return rc;
}

}  // namespace

int fvq_nvfp4_ffn_profile(const uint16_t* x, int64_t rows, const fvq_linear* lin1,
                          const fvq_linear* lin2, uint16_t* y, void* workspace,
                          size_t workspace_bytes, void* stream, float* kernel_ms) {
  return ffn_profile_impl(x, rows, lin1, lin2, y, nullptr, nullptr, workspace, workspace_bytes,
                          stream, kernel_ms);
}

int fvq_nvfp4_ffn_chain_profile(const uint16_t* x, int64_t rows, const fvq_linear* lin1,
                                const fvq_linear* lin2, uint16_t* y, const float* x_amax,
                                float* y_amax, void* workspace, size_t workspace_bytes,
                                void* stream, float* kernel_ms) {
  return ffn_profile_impl(x, rows, lin1, lin2, y, x_amax, y_amax, workspace, workspace_bytes,
                          stream, kernel_ms);
}

// ---------------------------------------------------------------- FP8 (W8A8) mode

int fvq_fp8_row_quantize(const uint16_t* x, int64_t rows, int64_t k, uint8_t* q, float* scale,
                         void* stream) {
  if (rows <= 0 || rows > (int64_t(1) << 31) - 1)
    return fail(FVQ_EINVAL, "fvq_fp8_row_quantize: rows must be in [1, 2^31) (got %lld)",
                (long long)rows);
  if (k <= 0 || k % 8 != 0 || k > fvq::fp8_row_quant_max_k())
    return fail(FVQ_EINVAL, "fvq_fp8_row_quantize: k must be a positive multiple of 8 up to %lld "
                "(got %lld)", (long long)fvq::fp8_row_quant_max_k(), (long long)k);
  if (!x || !q || !scale) return fail(FVQ_EINVAL, "fvq_fp8_row_quantize: NULL pointer");
  if (!aligned16(x) || !aligned16(q) || (reinterpret_cast<uintptr_t>(scale) & 3u) != 0)
    return fail(FVQ_EALIGN, "fvq_fp8_row_quantize: x and q must be 16-byte aligned, scale 4-byte");
  if (int rc = check_device()) return rc;
  cudaError_t e = fvq::launch_fp8_row_quant(x, rows, k, q, scale, nullptr, nullptr,
                                            static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fvq_fp8_row_quantize launch");
  return FVQ_OK;
}

size_t fvq_fp8_tensor_quantize_workspace_bytes(void) {
  return round_up(fvq::kAmaxWorkspaceBytes) + kScalarBytes;
}

int fvq_fp8_tensor_quantize(const uint16_t* x, int64_t numel, uint8_t* q, float* scale,
                            void* workspace, size_t workspace_bytes, void* stream) {
  if (numel <= 0)
    return fail(FVQ_EINVAL, "fvq_fp8_tensor_quantize: numel must be > 0 (got %lld)",
                (long long)numel);
  if (!x || !q || !scale || !workspace) return fail(FVQ_EINVAL, "fvq_fp8_tensor_quantize: NULL pointer");
  if (workspace_bytes < fvq_fp8_tensor_quantize_workspace_bytes())
    return fail(FVQ_EWORKSPACE, "fvq_fp8_tensor_quantize: workspace needs %zu bytes, got %zu",
                fvq_fp8_tensor_quantize_workspace_bytes(), workspace_bytes);
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(q) & 7u) != 0 || !aligned16(workspace))
    return fail(FVQ_EALIGN,
                "fvq_fp8_tensor_quantize: x and workspace must be 16-byte aligned, q 8-byte");
  if (int rc = check_device()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carve c(workspace);
  uint32_t* amax_ws = reinterpret_cast<uint32_t*>(c.take(fvq::kAmaxWorkspaceBytes));
  float* amax = reinterpret_cast<float*>(c.take(kScalarBytes));
  cudaError_t e = fvq::launch_amax(x, numel, amax, nullptr, amax_ws, nullptr, st);
  if (e != cudaSuccess) return cuda_fail(e, "fvq_fp8_tensor_quantize amax launch");
  e = fvq::launch_fp8_tensor_quant(x, numel, amax, q, scale, st);
  if (e != cudaSuccess) return cuda_fail(e, "fvq_fp8_tensor_quantize launch");
  return FVQ_OK;
}

namespace {

int check_fp8_gemm(const uint8_t* a, const float* sa, const uint8_t* w, const float* sw,
                   const uint16_t* bias, const uint16_t* out, int64_t m, int64_t n, int64_t k,
                   const char* who) {
  if (m <= 0 || m > (int64_t(1) << 30))
    return fail(FVQ_EINVAL, "%s: m must be in [1, 2^30] (got %lld)", who, (long long)m);
  if (n <= 0 || n % 256 != 0)
    return fail(FVQ_EINVAL, "%s: n must be a positive multiple of 256 (got %lld)", who,
                (long long)n);
  if (k <= 0 || k % 128 != 0 || k > fvq::fp8_row_quant_max_k())
    return fail(FVQ_EINVAL, "%s: k must be a positive multiple of 128 up to %lld (got %lld)", who,
                (long long)fvq::fp8_row_quant_max_k(), (long long)k);
  if (n * k > (int64_t(1) << 31) || m * k > (int64_t(1) << 40))
    return fail(FVQ_EINVAL, "%s: operand too large", who);
  if (!a || !sa || !w || !sw || !out) return fail(FVQ_EINVAL, "%s: NULL pointer", who);
  if (!aligned16(a) || !aligned16(w) || !aligned16(sw) || !aligned16(out) || !aligned16(bias) ||
      (reinterpret_cast<uintptr_t>(sa) & 3u) != 0)
    return fail(FVQ_EALIGN, "%s: operands, W scales, bias and out must be 16-byte aligned", who);
  return FVQ_OK;
}

int fp8_gemm_impl(const uint8_t* a, const float* sa, const uint8_t* w, const float* sw,
                  const uint16_t* bias, uint16_t* out, int64_t m, int64_t n, int64_t k,
                  int epilogue, uint32_t* row_amax, cudaStream_t st) {
  const char* why = nullptr;
  cudaError_t e = fvq::launch_fp8_gemm(a, sa, w, sw, bias, out, m, n, k, epilogue, row_amax,
                                       wait_limit(), st, &why);
  if (e != cudaSuccess) {
    if (why) return fail(FVQ_ECUDA, "fp8 GEMM: %s", why);
    return cuda_fail(e, "fp8 GEMM launch");
  }
  return FVQ_OK;
}

int check_fp8_linear(const fvq_linear_fp8* lin, const char* who) {
  if (lin == nullptr) return fail(FVQ_EINVAL, "%s: linear descriptor is NULL", who);
  if (!lin->qweight || !lin->scale)
    return fail(FVQ_EINVAL, "%s: qweight and scale are required", who);
  if (lin->in_features <= 0 || lin->in_features % 128 != 0 ||
      lin->in_features > fvq::fp8_row_quant_max_k() || lin->out_features <= 0 ||
      lin->out_features % 256 != 0)
    return fail(FVQ_EINVAL,
                "%s: in_features must be a positive multiple of 128 up to %lld and out_features "
                "a positive multiple of 256 (got %lld, %lld)",
                who, (long long)fvq::fp8_row_quant_max_k(), (long long)lin->in_features,
                (long long)lin->out_features);
  if (!aligned16(lin->qweight) || !aligned16(lin->scale) || !aligned16(lin->bias))
    return fail(FVQ_EALIGN, "%s: weight buffers must be 16-byte aligned", who);
  return FVQ_OK;
}

int check_fp8_rows(int64_t rows, const char* who) {
  if (rows <= 0 || rows > (int64_t(1) << 30))
    return fail(FVQ_EINVAL, "%s: rows must be in [1, 2^30] (got %lld)", who, (long long)rows);
  return FVQ_OK;
}

}  // namespace

int fvq_fp8_scaled_mm(const uint8_t* a, const float* scale_a, const uint8_t* w,
                      const float* scale_w, const uint16_t* bias, uint16_t* out, int64_t m,
                      int64_t n, int64_t k, void* stream) {
  if (int rc = check_fp8_gemm(a, scale_a, w, scale_w, bias, out, m, n, k, "fvq_fp8_scaled_mm"))
    return rc;
  if (int rc = check_device()) return rc;
  return fp8_gemm_impl(a, scale_a, w, scale_w, bias, out, m, n, k, FVQ_EPI_BF16, nullptr,
                       static_cast<cudaStream_t>(stream));
}

size_t fvq_fp8_linear_workspace_bytes(int64_t rows, int64_t in_features) {
  if (rows <= 0 || in_features <= 0) return 0;
  Carve c(nullptr);
  c.take(static_cast<size_t>(rows * in_features));
  c.take(static_cast<size_t>(rows * 4));
  return c.off;
}

int fvq_fp8_linear(const uint16_t* x, int64_t rows, const fvq_linear_fp8* lin, uint16_t* y,
                   void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_fp8_linear(lin, "fvq_fp8_linear")) return rc;
  if (int rc = check_fp8_rows(rows, "fvq_fp8_linear")) return rc;
  if (!x || !y || !workspace) return fail(FVQ_EINVAL, "fvq_fp8_linear: NULL pointer");
  const size_t need = fvq_fp8_linear_workspace_bytes(rows, lin->in_features);
  if (workspace_bytes < need)
    return fail(FVQ_EWORKSPACE, "fvq_fp8_linear: workspace needs %zu bytes, got %zu", need,
                workspace_bytes);
  if (!aligned16(x) || !aligned16(y) || !aligned16(workspace))
    return fail(FVQ_EALIGN, "fvq_fp8_linear: x, y and workspace must be 16-byte aligned");
  if (int rc = check_device()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t k = lin->in_features;
  Carve c(workspace);
  uint8_t* q = c.take(static_cast<size_t>(rows * k));
  float* s = reinterpret_cast<float*>(c.take(static_cast<size_t>(rows * 4)));
  cudaError_t e = fvq::launch_fp8_row_quant(x, rows, k, q, s, nullptr, nullptr, st);
  if (e != cudaSuccess) return cuda_fail(e, "fvq_fp8_linear quantize launch");
  return fp8_gemm_impl(q, s, lin->qweight, lin->scale, lin->bias, y, rows, lin->out_features, k,
                       FVQ_EPI_BF16, nullptr, st);
}

size_t fvq_fp8_ffn_workspace_bytes(int64_t rows, int64_t d_model, int64_t d_ff) {
  if (rows <= 0 || d_model <= 0 || d_ff <= 0) return 0;
  Carve c(nullptr);
  c.take(static_cast<size_t>(rows * 4));          // per-row max |h|
  c.take(static_cast<size_t>(rows * d_model));    // x in E4M3
  c.take(static_cast<size_t>(rows * 4));          // x row scales
  c.take(static_cast<size_t>(rows * d_ff * 2));   // h
  c.take(static_cast<size_t>(rows * d_ff));       // h in E4M3
  c.take(static_cast<size_t>(rows * 4));          // h row scales
  return c.off;
}

namespace {

int fp8_ffn_impl(const uint16_t* x, int64_t rows, const fvq_linear_fp8* lin1,
                 const fvq_linear_fp8* lin2, uint16_t* y, void* workspace, size_t workspace_bytes,
                 cudaStream_t st, cudaEvent_t* ev) {
  if (int rc = check_fp8_linear(lin1, "fvq_fp8_ffn (linear 1)")) return rc;
  if (int rc = check_fp8_linear(lin2, "fvq_fp8_ffn (linear 2)")) return rc;
  if (lin1->out_features != lin2->in_features || lin2->out_features != lin1->in_features)
    return fail(FVQ_EINVAL, "fvq_fp8_ffn: linear shapes do not chain (%lld->%lld, %lld->%lld)",
                (long long)lin1->in_features, (long long)lin1->out_features,
                (long long)lin2->in_features, (long long)lin2->out_features);
  if (int rc = check_fp8_rows(rows, "fvq_fp8_ffn")) return rc;
  if (!x || !y || !workspace) return fail(FVQ_EINVAL, "fvq_fp8_ffn: NULL pointer");
  const int64_t d = lin1->in_features, f = lin1->out_features;
  const size_t need = fvq_fp8_ffn_workspace_bytes(rows, d, f);
  if (workspace_bytes < need)
    return fail(FVQ_EWORKSPACE, "fvq_fp8_ffn: workspace needs %zu bytes, got %zu", need,
                workspace_bytes);
  if (!aligned16(x) || !aligned16(y) || !aligned16(workspace))
    return fail(FVQ_EALIGN, "fvq_fp8_ffn: x, y and workspace must be 16-byte aligned");
  if (int rc = check_device()) return rc;
  Carve c(workspace);
  uint32_t* row_amax = reinterpret_cast<uint32_t*>(c.take(static_cast<size_t>(rows * 4)));
  uint8_t* q_x = c.take(static_cast<size_t>(rows * d));
  float* s_x = reinterpret_cast<float*>(c.take(static_cast<size_t>(rows * 4)));
  uint16_t* h = reinterpret_cast<uint16_t*>(c.take(static_cast<size_t>(rows * f * 2)));
  uint8_t* q_h = c.take(static_cast<size_t>(rows * f));
  float* s_h = reinterpret_cast<float*>(c.take(static_cast<size_t>(rows * 4)));
  auto mark = [&](int i) {
    if (ev != nullptr) cudaEventRecord(ev[i], st);
  };
  mark(0);
  // 1. x -> E4M3 with per-row scales; also zeroes the per-row maxima GEMM1 accumulates
  cudaError_t e = fvq::launch_fp8_row_quant(x, rows, d, q_x, s_x, nullptr, row_amax, st);
  if (e != cudaSuccess) return cuda_fail(e, "fvq_fp8_ffn quantize(x) launch");
  mark(1);
  // 2. h = bf16(gelu(bf16(bf16(acc * s_x * s_w1) + b1))), row_amax = max |h| per row
  if (int rc = fp8_gemm_impl(q_x, s_x, lin1->qweight, lin1->scale, lin1->bias, h, rows, f, d,
                             FVQ_EPI_GELU_AMAX, row_amax, st))
    return rc;
  mark(2);
  // 3. h -> E4M3 with per-row scales from row_amax (step 1 of the next call re-zeroes it)
  e = fvq::launch_fp8_row_quant(h, rows, f, q_h, s_h, row_amax, nullptr, st);
  if (e != cudaSuccess) return cuda_fail(e, "fvq_fp8_ffn quantize(h) launch");
  mark(3);
  // 4. y = bf16(bf16(acc * s_h * s_w2) + b2)
  if (int rc = fp8_gemm_impl(q_h, s_h, lin2->qweight, lin2->scale, lin2->bias, y, rows, d, f,
                             FVQ_EPI_BF16, nullptr, st))
    return rc;
  mark(4);
  return FVQ_OK;
}

}  // namespace

int fvq_fp8_ffn(const uint16_t* x, int64_t rows, const fvq_linear_fp8* lin1,
                const fvq_linear_fp8* lin2, uint16_t* y, void* workspace, size_t workspace_bytes,
                void* stream) {
  return fp8_ffn_impl(x, rows, lin1, lin2, y, workspace, workspace_bytes,
                      static_cast<cudaStream_t>(stream), nullptr);
}

int fvq_fp8_ffn_profile(const uint16_t* x, int64_t rows, const fvq_linear_fp8* lin1,
                        const fvq_linear_fp8* lin2, uint16_t* y, void* workspace,
                        size_t workspace_bytes, void* stream, float* kernel_ms) {
  if (kernel_ms == nullptr) return fail(FVQ_EINVAL, "fvq_fp8_ffn_profile: kernel_ms is NULL");
  if (int rc = check_device()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaEvent_t ev[5];
  int made = 0;
  for (; made < 5; ++made) {
    if (cudaEventCreate(&ev[made]) != cudaSuccess) break;
  }
  int rc = FVQ_OK;
  if (made < 5) {
    rc = fail(FVQ_ECUDA, "fvq_fp8_ffn_profile: cudaEventCreate failed");
  } else {
    rc = fp8_ffn_impl(x, rows, lin1, lin2, y, workspace, workspace_bytes, st, ev);
    if (rc == FVQ_OK) {
      cudaError_t e = cudaEventSynchronize(ev[4]);
      for (int i = 0; e == cudaSuccess && i < 4; ++i)
        e = cudaEventElapsedTime(&kernel_ms[i], ev[i], ev[i + 1]);
      if (e != cudaSuccess) rc = cuda_fail(e, "fvq_fp8_ffn_profile timing");
    }
  }
  for (int i = 0; i < made; ++i) cudaEventDestroy(ev[i]);
  return rc;
}

int fvq_div_full_probe(const float* a, const float* b, float* out, int64_t n, void* stream) {
  if (n < 0 || (n > 0 && (!a || !b || !out))) return fail(FVQ_EINVAL, "fvq_div_full_probe: bad args");
  if (int rc = check_device()) return rc;
  cudaError_t e = fvq::launch_div_full_probe(a, b, out, n, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fvq_div_full_probe launch");
  return FVQ_OK;
}

// ---------------------------------------------------------------- Pillow-exact resize

int fvq_pil_resize(const uint8_t* src, int64_t frames, int64_t in_h, int64_t in_w, int64_t out_h,
                   int64_t out_w, int64_t crop_y, int64_t crop_x, int64_t crop_h, int64_t crop_w,
                   uint8_t* dst_u8, uint16_t* dst_bf16, void* stream) {
  if (frames <= 0 || frames > 65535)
    return fail(FVQ_EINVAL, "fvq_pil_resize: frames must be in [1, 65535] (got %lld)",
                (long long)frames);
  if (in_h <= 0 || in_w <= 0 || out_h < in_h || out_w < in_w || out_h > 32768 || out_w > 32768)
    return fail(FVQ_EINVAL, "fvq_pil_resize: only upscaling is supported, sizes in [1, 32768] "
                "(got %lldx%lld -> %lldx%lld)", (long long)in_w, (long long)in_h,
                (long long)out_w, (long long)out_h);
  if (crop_y < 0 || crop_x < 0 || crop_h <= 0 || crop_w <= 0 || crop_y + crop_h > out_h ||
      crop_x + crop_w > out_w)
    return fail(FVQ_EINVAL, "fvq_pil_resize: the crop must lie inside the output");
  if (crop_w % 8 != 0)
    return fail(FVQ_EINVAL, "fvq_pil_resize: crop_w must be a multiple of 8 (got %lld)",
                (long long)crop_w);
  if (!src || (!dst_u8 && !dst_bf16)) return fail(FVQ_EINVAL, "fvq_pil_resize: NULL pointer");
  if (!aligned16(dst_u8) || !aligned16(dst_bf16))
    return fail(FVQ_EALIGN, "fvq_pil_resize: outputs must be 16-byte aligned");
  if (int rc = check_device()) return rc;
  size_t smem = 0;
  cudaError_t e = fvq::launch_pil_resize(
      src, frames, static_cast<int>(in_h), static_cast<int>(in_w), static_cast<int>(out_h),
      static_cast<int>(out_w), static_cast<int>(crop_y), static_cast<int>(crop_x),
      static_cast<int>(crop_h), static_cast<int>(crop_w), dst_u8, dst_bf16, &smem,
      static_cast<cudaStream_t>(stream));
  if (e == cudaErrorInvalidValue)
    return fail(FVQ_EINVAL, "fvq_pil_resize: a tile needs %zu bytes of shared memory (input too "
                "wide for its scale)", smem);
  if (e != cudaSuccess) return cuda_fail(e, "fvq_pil_resize launch");
  return FVQ_OK;
}

int fvq_pil_normalize(const uint8_t* src, int64_t frames, int64_t h, int64_t w,
                      int64_t stride_frame, int64_t stride_row, int64_t stride_col, uint16_t* dst,
                      void* stream) {
  if (frames <= 0 || h <= 0 || w <= 0 || w % 8 != 0)
    return fail(FVQ_EINVAL, "fvq_pil_normalize: frames, h > 0 and w a positive multiple of 8");
  if (stride_col < 3 || stride_row < stride_col * w || stride_frame < stride_row * h)
    return fail(FVQ_EINVAL, "fvq_pil_normalize: strides must describe non-overlapping HWC pixels");
  if (!src || !dst) return fail(FVQ_EINVAL, "fvq_pil_normalize: NULL pointer");
  if (!aligned16(dst)) return fail(FVQ_EALIGN, "fvq_pil_normalize: dst must be 16-byte aligned");
  if (int rc = check_device()) return rc;
  cudaError_t e = fvq::launch_pil_normalize(src, frames, static_cast<int>(h), static_cast<int>(w),
                                            stride_frame, stride_row, stride_col, dst,
                                            static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fvq_pil_normalize launch");
  return FVQ_OK;
}

int fvq_rcp_approx_probe(const float* in, float* out, int64_t n, void* stream) {
  if (n < 0 || (n > 0 && (!in || !out))) return fail(FVQ_EINVAL, "fvq_rcp_approx_probe: bad args");
  if (int rc = check_device()) return rc;
  cudaError_t e = fvq::launch_rcp_probe(in, out, n, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fvq_rcp_approx_probe launch");
  return FVQ_OK;
}

int fvq_gelu_bf16_probe(const uint16_t* in, uint16_t* out, int64_t count, void* stream) {
  if (count < 0 || (count > 0 && (!in || !out)))
    return fail(FVQ_EINVAL, "fvq_gelu_bf16_probe: bad args");
  if (int rc = check_device()) return rc;
  cudaError_t e = fvq::launch_gelu_probe(in, out, count, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fvq_gelu_bf16_probe launch");
  return FVQ_OK;
}

int fvq_set_gemm_pairing(int mode) {
  if (mode < 0 || mode > 2)
    return fail(FVQ_EINVAL, "fvq_set_gemm_pairing: mode must be 0, 1 or 2 (got %d)", mode);
  fvq::set_gemm_pairing(mode);
  return FVQ_OK;
}

int fvq_set_fp8_gemm_pairing(int mode) {
  if (mode < 0 || mode > 2)
    return fail(FVQ_EINVAL, "fvq_set_fp8_gemm_pairing: mode must be 0, 1 or 2 (got %d)", mode);
  fvq::set_fp8_gemm_pairing(mode);
  return FVQ_OK;
}

int fvq_set_wait_limit(uint64_t nanoseconds) {
  g_wait_limit_ns.store(nanoseconds == 0 ? fvq::kDefaultWaitLimit : nanoseconds,
                        std::memory_order_relaxed);
  return FVQ_OK;
}

int fvq_read_device_error(void* stream, uint32_t* flags) {
  if (flags == nullptr) return fail(FVQ_EINVAL, "fvq_read_device_error: flags is NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  cudaError_t e = fvq::read_error_word(&v, st);
  if (e != cudaSuccess) return cuda_fail(e, "fvq_read_device_error");
  *flags = v;
  if (v != 0) {
    e = fvq::set_error_word(0, st);
    if (e != cudaSuccess) return cuda_fail(e, "fvq_read_device_error clear");
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "fvq_read_device_error clear");
  }
  return FVQ_OK;
}

}  // extern "C"
