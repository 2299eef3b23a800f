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
// The row quantizer runs one CTA of 256 threads per row: the row is read once
// into registers (16-byte loads, up to 8 per thread, so K <= 16384), reduced to
// its max |x|, then divided and converted in place.  With a precomputed row
// maximum (the FP8 GEMM1 epilogue's per-row max |h|) it skips the reduction and
// resets that word to zero for the next use.
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

// max |bf16| of both halves (bit patterns; non-NaN magnitudes order as integers)
__device__ __forceinline__ uint32_t absmax_pair(uint32_t m, uint32_t w) {
  const uint32_t a = w & 0x7FFF7FFFu;
  return max(m, max(a & 0xFFFFu, a >> 16));
}

// Two floats -> two E4M3 bytes (`lo` in bits 0-7), round to nearest even, satfinite.
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Eight bf16 values (one 16-byte word) divided by `scale` -> eight E4M3 bytes.
__device__ __forceinline__ uint2 quantize8_row(uint4 v, float scale) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t p[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float lo = __uint_as_float(w[j] << 16), hi = __uint_as_float(w[j] & 0xFFFF0000u);
    p[j] = e4m3x2(div_full(lo, scale), div_full(hi, scale));
  }
  return make_uint2(p[0] | (p[1] << 16), p[2] | (p[3] << 16));
}

// The tensor quantizer's variant: the quotient is clamped to [-448, 448] first.
__device__ __forceinline__ float clamp448(float v) { return fminf(fmaxf(v, -448.0f), 448.0f); }

__device__ __forceinline__ uint2 quantize8_clamped(uint4 v, float scale) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t p[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float lo = __uint_as_float(w[j] << 16), hi = __uint_as_float(w[j] & 0xFFFF0000u);
    p[j] = e4m3x2(clamp448(div_full(lo, scale)), clamp448(div_full(hi, scale)));
  }
  return make_uint2(p[0] | (p[1] << 16), p[2] | (p[3] << 16));
}

// scale = max(div(amax, 448), 1e-12): _row_quant's `tl.maximum(tl.max(|x|)/448., 1.e-12)`.
__device__ __forceinline__ float row_scale(float amax) {
  return fmaxf(div_full(amax, 448.0f), 1e-12f);
}

// One CTA per row.  kVec: 16-byte words per thread (the row has k/8 of them).
// row_amax != nullptr: its word for the row holds max |x| (fp32 bits); the
// reduction is skipped and the word is reset to zero after use.  zero_rows !=
// nullptr: the row's word there is set to zero (arming the per-row maxima a
// later GEMM epilogue accumulates).
template <int kVec>
__global__ void __launch_bounds__(kRowThreads) fp8_row_quant_kernel(
    const uint16_t* __restrict__ x, int k, uint8_t* __restrict__ q, float* __restrict__ scale_out,
    uint32_t* row_amax, uint32_t* zero_rows) {
  __shared__ uint32_t warp_max[kRowThreads / 32];
  __shared__ float row_scale_s;
  const int64_t row = blockIdx.x;
  const int nvec = k / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * k);
  uint4 v[kVec];
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int j = threadIdx.x + i * kRowThreads;
    v[i] = j < nvec ? ld_nc_v4(xr + j) : make_uint4(0, 0, 0, 0);
  }
  if (row_amax == nullptr) {
    uint32_t m = 0;
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
      m = absmax_pair(m, v[i].x);
      m = absmax_pair(m, v[i].y);
      m = absmax_pair(m, v[i].z);
      m = absmax_pair(m, v[i].w);
    }
    m = __reduce_max_sync(0xFFFFFFFFu, m);
    if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t t = warp_max[0];
#pragma unroll
      for (int w = 1; w < kRowThreads / 32; ++w) t = max(t, warp_max[w]);
      const float s = row_scale(__uint_as_float(t << 16));
      row_scale_s = s;
      scale_out[row] = s;
    }
  } else if (threadIdx.x == 0) {
    const float s = row_scale(__uint_as_float(row_amax[row]));
    row_amax[row] = 0u;
    row_scale_s = s;
    scale_out[row] = s;
  }
  __syncthreads();
  if (zero_rows != nullptr && threadIdx.x == 0) zero_rows[row] = 0u;
  const float s = row_scale_s;
  uint2* qr = reinterpret_cast<uint2*>(q + row * k);
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int j = threadIdx.x + i * kRowThreads;
    if (j < nvec) qr[j] = quantize8_row(v[i], s);
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
      if (j < nvec) qv[j] = quantize8_clamped(v[u], s);
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
void row_quant_launch(const uint16_t* x, int64_t rows, int k, uint8_t* q, float* scale,
                      uint32_t* row_amax, uint32_t* zero_rows, cudaStream_t st) {
  fp8_row_quant_kernel<kVec><<<static_cast<unsigned>(rows), kRowThreads, 0, st>>>(
      x, k, q, scale, row_amax, zero_rows);
}

}  // namespace

int64_t fp8_row_quant_max_k() { return static_cast<int64_t>(kRowThreads) * kRowMaxVec * 8; }

cudaError_t launch_fp8_row_quant(const uint16_t* x, int64_t rows, int64_t k, uint8_t* q,
                                 float* scale, uint32_t* row_amax, uint32_t* zero_rows,
                                 cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const int words = static_cast<int>((k / 8 + kRowThreads - 1) / kRowThreads);
  const int ki = static_cast<int>(k);
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
