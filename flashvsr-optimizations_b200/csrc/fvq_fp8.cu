// fvq_fp8.cu -- HBM-bound E4M3 (FP8) quantizers of the reference's W8A8 paths.
//
//   row quantizer    : reference ffn_quantization.py:6-13 (_row_quant) and :22-26
//                      (row_quant), used by QuantLinear(mode='fp8') on weights and
//                      activations:
//                        scale[r] = max(div(max_k |x[r, k]|, 448), 1e-12)
//                        q[r, k]  = e4m3_rn_satfinite(div(x[r, k], scale[r]))
//   tensor quantizer : reference decoder_fp8.py:9-24 (_quantize, quantize_activation),
//                      shared by lq_fp8.py:24-31:
//                        scale = max(amax * fl(1/448), 1e-12)      (torch's tensor / 448.)
//                        q     = e4m3_rn(min(max(div(x, scale), -448), 448))
//
// `div` is the reference's Triton fp32 division `x / scale`, which Triton's
// NVIDIA backend emits as div.full.f32 (an approximate divide, not IEEE
// rounded); these kernels issue that same instruction, so the codes match the
// reference bit for bit on the GPU.
//
// The row quantizer runs one CTA of 256 threads per row (one warp per row for
// rows of at most 2048 elements): the row is read once
// into registers (16-byte loads, up to 8 per thread, so K <= 16384), reduced to
// its max |x|, then divided and converted in place.  With a precomputed row
// maximum (the FP8 GEMM1 epilogue's per-row max |h|) it skips the reduction.
// The per-element division is replaced by two multiplies whose E4M3 codes
// bracket div.full's, with the division issued where they disagree (quantize8).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "fvq_internal.h"
#include "fvq_ptx.cuh"

namespace fvq {

namespace {

constexpr int kRowThreads = 256;
constexpr int kRowMaxVec = 8;                      // 16-byte words per thread
constexpr int kTensorThreads = 256;
constexpr int kTensorUnroll = 4;
constexpr float kInv448 = 1.0f / 448.0f;             // fp32 reciprocal, round to nearest

__device__ __forceinline__ float div_full(float a, float b) {
  float q;
  asm("div.full.f32 %0, %1, %2;" : "=f"(q) : "f"(a), "f"(b));
  return q;
}

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// per-halfword unsigned maximum; on |bf16| bit patterns (non-NaN) it orders magnitudes
__device__ __forceinline__ uint32_t max_u16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Two floats -> two E4M3 bytes (`lo` in bits 0-7), round to nearest even, satfinite.
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// E4M3 codes of x / scale without a division per element.  With r =
// rcp.rn(scale), the products x * r * (1 -+ 2^-18) (through per-row constants
// r_lo, r_hi; three roundings of at most 2^-24 each) lie below and above every
// value within 2^-22 (relative) of the exact quotient, and div.full.f32's
// result is one of those (its documented maximum error is 2 ulp).  Round-to-nearest-even
// conversion is monotonic, so when the two ends of the bracket convert to the
// same code (one paired cvt per end), that is the code of div.full(x, scale);
// otherwise -- a rounding midpoint lies inside the bracket, about 6e-5 of
// Gaussian-like data -- the division itself is issued.  Zeros, fp32 subnormals
// and saturating values need no special case: both ends agree on them.
// kClamp (the tensor quantizer): quotients are clamped to [-448, 448] before
// the conversion, as the reference does (NaN clamps to -448 like Triton's
// NaN-ignoring maximum).
constexpr float kBracketLo = 1.0f - 0x1p-18f;
constexpr float kBracketHi = 1.0f + 0x1p-18f;

// (lo, hi) * (r, r) in one mul.rn.f32x2
__device__ __forceinline__ void mul2(float lo, float hi, float r, float& plo, float& phi) {
  uint64_t v, rr, p;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(lo), "f"(hi));
  asm("mov.b64 %0, {%1, %1};" : "=l"(rr) : "f"(r));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(p) : "l"(v), "l"(rr));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(plo), "=f"(phi) : "l"(p));
}

__device__ __forceinline__ float clamp448(float v) { return fminf(fmaxf(v, -448.0f), 448.0f); }

template <bool kClamp>
__device__ __forceinline__ uint32_t e4m3_pair(float lo, float hi) {
  if (kClamp) {
    lo = clamp448(lo);
    hi = clamp448(hi);
  }
  return e4m3x2(lo, hi);
}

// Eight bf16 values (one 16-byte word) -> eight E4M3 codes of div.full(x, scale).
template <bool kClamp>
__device__ __forceinline__ uint2 quantize8(uint4 v, float scale, float r_lo, float r_hi) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t c[4];
  uint32_t differ = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float lo = __uint_as_float(w[j] << 16), hi = __uint_as_float(w[j] & 0xFFFF0000u);
    float dl, dh, ul, uh;
    mul2(lo, hi, r_lo, dl, dh);
    mul2(lo, hi, r_hi, ul, uh);
    c[j] = e4m3_pair<kClamp>(dl, dh);
    if (c[j] != e4m3_pair<kClamp>(ul, uh)) differ |= 1u << j;  // pair j unsettled
  }
  if (__builtin_expect(differ != 0, 0)) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (differ & (1u << j)) {
        const float lo = __uint_as_float(w[j] << 16), hi = __uint_as_float(w[j] & 0xFFFF0000u);
        c[j] = e4m3_pair<kClamp>(div_full(lo, scale), div_full(hi, scale));
      }
    }
  }
  return make_uint2(c[0] | (c[1] << 16), c[2] | (c[3] << 16));
}

// scale = max(div(amax, 448), 1e-12): _row_quant's `tl.maximum(tl.max(|x|)/448., 1.e-12)`.
__device__ __forceinline__ float row_scale(float amax) {
  return fmaxf(div_full(amax, 448.0f), 1e-12f);
}

// One CTA per row.  kVec: 16-byte words per thread (the row has k/8 of them).
// row_amax != nullptr: its word for the row holds max |x| (fp32 bits) and the
// reduction is skipped.  zero_rows != nullptr: the row's word there is set to
// zero (arming the per-row maxima a later GEMM epilogue accumulates).
template <int kVec>
__global__ void __launch_bounds__(kRowThreads) fp8_row_quant_kernel(
    const uint16_t* __restrict__ x, int k, uint8_t* __restrict__ q, float* __restrict__ scale_out,
    const uint32_t* __restrict__ row_amax, uint32_t* zero_rows) {
  __shared__ uint32_t warp_max[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const int nvec = k / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * k);
  uint32_t amax_bits = row_amax != nullptr ? __ldg(row_amax + row) : 0u;
  uint4 v[kVec];
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int j = threadIdx.x + i * kRowThreads;
    v[i] = j < nvec ? ld_nc_v4(xr + j) : make_uint4(0, 0, 0, 0);
  }
  if (row_amax == nullptr) {
    uint32_t m2 = 0;  // max |x| of the low and high halves, packed
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
      m2 = max_u16x2(m2, max_u16x2(v[i].x & 0x7FFF7FFFu, v[i].y & 0x7FFF7FFFu));
      m2 = max_u16x2(m2, max_u16x2(v[i].z & 0x7FFF7FFFu, v[i].w & 0x7FFF7FFFu));
    }
    uint32_t m = __reduce_max_sync(0xFFFFFFFFu, max(m2 & 0xFFFFu, m2 >> 16));
    if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
    __syncthreads();
    m = warp_max[0];
#pragma unroll
    for (int w = 1; w < kRowThreads / 32; ++w) m = max(m, warp_max[w]);
    amax_bits = m << 16;
  }
  const float s = row_scale(__uint_as_float(amax_bits));
  const float r = __frcp_rn(s);
  const float r_lo = __fmul_rn(r, kBracketLo), r_hi = __fmul_rn(r, kBracketHi);
  if (threadIdx.x == 0) {
    scale_out[row] = s;
    if (zero_rows != nullptr) zero_rows[row] = 0u;
  }
  uint2* qr = reinterpret_cast<uint2*>(q + row * k);
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int j = threadIdx.x + i * kRowThreads;
    if (j < nvec) qr[j] = quantize8<false>(v[i], s, r_lo, r_hi);
  }
}

// Rows of at most 2048 elements: one warp per row, eight rows per CTA, the row
// maximum reduced within the warp.  Same arithmetic as fp8_row_quant_kernel.
template <int kVec>
__global__ void __launch_bounds__(kRowThreads) fp8_row_quant_warp_kernel(
    const uint16_t* __restrict__ x, int64_t rows, int k, uint8_t* __restrict__ q,
    float* __restrict__ scale_out, const uint32_t* __restrict__ row_amax, uint32_t* zero_rows) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (kRowThreads / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nvec = k / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * k);
  uint32_t amax_bits = row_amax != nullptr ? __ldg(row_amax + row) : 0u;
  uint4 v[kVec];
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int j = lane + i * 32;
    v[i] = j < nvec ? ld_nc_v4(xr + j) : make_uint4(0, 0, 0, 0);
  }
  if (row_amax == nullptr) {
    uint32_t m2 = 0;
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
      m2 = max_u16x2(m2, max_u16x2(v[i].x & 0x7FFF7FFFu, v[i].y & 0x7FFF7FFFu));
      m2 = max_u16x2(m2, max_u16x2(v[i].z & 0x7FFF7FFFu, v[i].w & 0x7FFF7FFFu));
    }
    amax_bits = __reduce_max_sync(0xFFFFFFFFu, max(m2 & 0xFFFFu, m2 >> 16)) << 16;
  }
  const float s = row_scale(__uint_as_float(amax_bits));
  const float r = __frcp_rn(s);
  const float r_lo = __fmul_rn(r, kBracketLo), r_hi = __fmul_rn(r, kBracketHi);
  if (lane == 0) {
    scale_out[row] = s;
    if (zero_rows != nullptr) zero_rows[row] = 0u;
  }
  uint2* qr = reinterpret_cast<uint2*>(q + row * k);
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int j = lane + i * 32;
    if (j < nvec) qr[j] = quantize8<false>(v[i], s, r_lo, r_hi);
  }
}

// Per-tensor quantizer: scale from the device amax as torch evaluates
// `(amax / 448.).clamp_min(1e-12)` -- a CUDA tensor divided by a Python scalar
// is multiplied by the scalar's fp32 reciprocal -- then a grid-stride pass over
// 16-byte words and a scalar tail.
__global__ void __launch_bounds__(kTensorThreads) fp8_tensor_quant_kernel(
    const uint16_t* __restrict__ x, int64_t numel, const float* __restrict__ amax,
    uint8_t* __restrict__ q, float* __restrict__ scale_out) {
  const float s = fmaxf(__fmul_rn(*amax, kInv448), 1e-12f);
  const float r = __frcp_rn(s);
  const float r_lo = __fmul_rn(r, kBracketLo), r_hi = __fmul_rn(r, kBracketHi);
  if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = s;
  const int64_t nvec = numel / 8;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  uint2* qv = reinterpret_cast<uint2*>(q);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kTensorThreads;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kTensorThreads) + threadIdx.x; i < nvec;
       i += kTensorUnroll * stride) {
    uint4 v[kTensorUnroll];
#pragma unroll
    for (int u = 0; u < kTensorUnroll; ++u) {
      const int64_t j = i + u * stride;
      v[u] = j < nvec ? ld_nc_v4(xv + j) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kTensorUnroll; ++u) {
      const int64_t j = i + u * stride;
      if (j < nvec) qv[j] = quantize8<true>(v[u], s, r_lo, r_hi);
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < (numel & 7)) {
    const int64_t e = nvec * 8 + threadIdx.x;
    const float f = __uint_as_float(static_cast<uint32_t>(x[e]) << 16);
    q[e] = static_cast<uint8_t>(e4m3x2(clamp448(div_full(f, s)), 0.0f) & 0xFFu);
  }
}

__global__ void div_full_probe_kernel(const float* a, const float* b, float* out, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = div_full(a[i], b[i]);
}

template <int kVec>
void row_quant_warp_launch(const uint16_t* x, int64_t rows, int k, uint8_t* q, float* scale,
                           const uint32_t* row_amax, uint32_t* zero_rows, cudaStream_t st) {
  constexpr int kRowsPerCta = kRowThreads / 32;
  const int64_t blocks = (rows + kRowsPerCta - 1) / kRowsPerCta;
  fp8_row_quant_warp_kernel<kVec><<<static_cast<unsigned>(blocks), kRowThreads, 0, st>>>(
      x, rows, k, q, scale, row_amax, zero_rows);
}

template <int kVec>
void row_quant_launch(const uint16_t* x, int64_t rows, int k, uint8_t* q, float* scale,
                      const uint32_t* row_amax, uint32_t* zero_rows, cudaStream_t st) {
  fp8_row_quant_kernel<kVec><<<static_cast<unsigned>(rows), kRowThreads, 0, st>>>(
      x, k, q, scale, row_amax, zero_rows);
}

}  // namespace

int64_t fp8_row_quant_max_k() { return static_cast<int64_t>(kRowThreads) * kRowMaxVec * 8; }

cudaError_t launch_fp8_row_quant(const uint16_t* x, int64_t rows, int64_t k, uint8_t* q,
                                 float* scale, const uint32_t* row_amax, uint32_t* zero_rows,
                                 cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const int ki = static_cast<int>(k);
  if (k <= 2048) {  // one warp per row
    switch (static_cast<int>((k / 8 + 31) / 32)) {
      case 0:
      case 1: row_quant_warp_launch<1>(x, rows, ki, q, scale, row_amax, zero_rows, st); break;
      case 2: row_quant_warp_launch<2>(x, rows, ki, q, scale, row_amax, zero_rows, st); break;
      case 3:
      case 4: row_quant_warp_launch<4>(x, rows, ki, q, scale, row_amax, zero_rows, st); break;
      case 5:
      case 6: row_quant_warp_launch<6>(x, rows, ki, q, scale, row_amax, zero_rows, st); break;
      default: row_quant_warp_launch<8>(x, rows, ki, q, scale, row_amax, zero_rows, st); break;
    }
    return cudaGetLastError();
  }
  const int words = static_cast<int>((k / 8 + kRowThreads - 1) / kRowThreads);
  switch (words) {
    case 0:
    case 1: row_quant_launch<1>(x, rows, ki, q, scale, row_amax, zero_rows, st); break;
    case 2: row_quant_launch<2>(x, rows, ki, q, scale, row_amax, zero_rows, st); break;
    case 3: row_quant_launch<3>(x, rows, ki, q, scale, row_amax, zero_rows, st); break;
    case 4: row_quant_launch<4>(x, rows, ki, q, scale, row_amax, zero_rows, st); break;
    case 5: row_quant_launch<5>(x, rows, ki, q, scale, row_amax, zero_rows, st); break;
    case 6: row_quant_launch<6>(x, rows, ki, q, scale, row_amax, zero_rows, st); break;
    case 7:
    case 8: row_quant_launch<8>(x, rows, ki, q, scale, row_amax, zero_rows, st); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_fp8_tensor_quant(const uint16_t* x, int64_t numel, const float* amax,
                                    uint8_t* q, float* scale, cudaStream_t st) {
  const int64_t nvec = numel / 8;
  int64_t blocks = (nvec + kTensorThreads * kTensorUnroll - 1) / (kTensorThreads * kTensorUnroll);
  if (blocks < 1) blocks = 1;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  fp8_tensor_quant_kernel<<<static_cast<unsigned>(blocks), kTensorThreads, 0, st>>>(x, numel, amax,
                                                                                    q, scale);
  return cudaGetLastError();
}

cudaError_t launch_div_full_probe(const float* a, const float* b, float* out, int64_t n,
                                  cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  div_full_probe_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(a, b, out, n);
  return cudaGetLastError();
}

}  // namespace fvq
