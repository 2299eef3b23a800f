// fvq_quant.cu -- HBM-bound kernels of the activation quantizer.
//
//   amax kernel     : max |x| over a bf16 tensor, then g = 2688 / max(amax, 1e-12)
//                     (reference ffn_quantization.py:15-19, :29-32).
//   quantize kernel : NVFP4 codes + 128x4-swizzled E4M3 block scales
//                     (reference: flashinfer.nvfp4_quantize, ffn_quantization.py:47, :64).
//
// Both stream the input once with wide non-allocating loads, several in flight
// per thread, on a grid of up to (SM count x 8) CTAs of 256 threads.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "fvq_internal.h"
#include "fvq_ptx.cuh"

namespace fvq {

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 8;   // 16-byte loads in flight per thread in the amax pass

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Packed bf16 maximum (max.bf16x2); on non-negative non-NaN values it orders
// exactly like the bit patterns.
__device__ __forceinline__ uint32_t bmax2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// max of |bf16| over the 8 values of a uint4, as a bf16 bit pattern in the low 16 bits.
__device__ __forceinline__ uint32_t absmax8(uint4 v) {
  const uint32_t m = bmax2(bmax2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu),
                           bmax2(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu));
  return max(m & 0xFFFFu, m >> 16);
}

// four bytes (low 8 bits of each argument) -> one word, b0 lowest
__device__ __forceinline__ uint32_t pack4(uint32_t b0, uint32_t b1, uint32_t b2, uint32_t b3) {
  uint32_t lo, hi, r;
  asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(lo) : "r"(b0), "r"(b1));
  asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(hi) : "r"(b2), "r"(b3));
  asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(r) : "r"(lo), "r"(hi));
  return r;
}

__device__ __forceinline__ int64_t pad_up_dev(int64_t r) { return (r + 127) / 128 * 128; }

// g = reciprocal(max(amax, 1e-12)) * 2688 with IEEE rounding at each step,
// as torch evaluates 2688. / t on a device tensor.
__device__ __forceinline__ float encode_scale(float amax) {
  float m = fmaxf(amax, 1e-12f);
  return __fmul_rn(__frcp_rn(m), 2688.0f);
}

// ---------------------------------------------------------------- amax
__global__ void __launch_bounds__(kThreads) amax_kernel(const uint16_t* __restrict__ x,
                                                        int64_t numel, float* amax_out,
                                                        float* g_out, uint32_t* ws,
                                                        float* zero_word) {
  __shared__ uint32_t warp_max[kThreads / 32];
  __shared__ bool is_last;
  if (zero_word != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *zero_word = 0.0f;

  const int64_t nvec = numel / 8;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * kThreads;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  uint32_t m = 0;
  int64_t i = tid;
  for (; i + (kUnroll - 1) * nthreads < nvec; i += kUnroll * nthreads) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) v[u] = ld_stream(xv + i + u * nthreads);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) m = max(m, absmax8(v[u]));
  }
  for (; i < nvec; i += nthreads) m = max(m, absmax8(ld_stream(xv + i)));
  // ragged tail (numel % 8)
  for (int64_t t = nvec * 8 + tid; t < numel; t += nthreads) m = max(m, x[t] & 0x7FFFu);

  m = __reduce_max_sync(0xFFFFFFFFu, m);
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t bm = 0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) bm = max(bm, warp_max[w]);
    ws[16 + blockIdx.x] = bm;
    __threadfence();
    uint32_t prev = atomicAdd(&ws[0], 1u);
    is_last = (prev == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last) return;
  // last CTA: reduce the per-CTA maxima, publish, and re-arm the counter.
  __threadfence();
  uint32_t bm = 0;
  for (int b = threadIdx.x; b < static_cast<int>(gridDim.x); b += kThreads)
    bm = max(bm, __ldcg(&ws[16 + b]));
  bm = __reduce_max_sync(0xFFFFFFFFu, bm);
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = bm;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t r = 0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) r = max(r, warp_max[w]);
    const float amax = __uint_as_float(r << 16);
    ws[2] = __float_as_uint(amax);
    if (amax_out) *amax_out = amax;
    if (g_out) *g_out = encode_scale(amax);
    ws[0] = 0;
  }
}

// ---------------------------------------------------------------- quantize
// One thread per 16-element scale block (a 32-byte load); consecutive threads
// take consecutive blocks, so a warp streams 1 KB per load instruction and
// writes 256 contiguous code bytes.  The four scale bytes of a 64-column group
// (held by 4 consecutive lanes) are gathered into one 32-bit store.  Blocks
// past the last row, up to pad128(rows), only write zero scale words.
__device__ __forceinline__ void ld_stream_v8(const void* p, uint32_t (&r)[8]) {
  asm volatile("ld.global.nc.L1::no_allocate.v8.u32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "l"(p));
}

constexpr int kQuantUnroll = 2;

__global__ void __launch_bounds__(kThreads) quantize_kernel(
    const uint16_t* __restrict__ x, int64_t rows, int64_t k, const float* __restrict__ g_ptr,
    const float* __restrict__ amax_ptr, float* g_out, uint8_t* __restrict__ codes,
    uint8_t* __restrict__ sf, float* zero_word) {
  const float g = amax_ptr != nullptr ? encode_scale(*amax_ptr) : *g_ptr;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (g_out != nullptr) *g_out = g;
    if (zero_word != nullptr) *zero_word = 0.0f;
  }
  const float r6 = rcp_approx_ftz(6.0f);
  const float rg = rcp_approx_ftz(g);

  const int lane = threadIdx.x & 31;
  const int64_t bpr = k / 16;                      // scale blocks per row
  const int64_t gpr = k / 64;                      // 64-column groups per row
  const int64_t n_real = rows * bpr;
  const int64_t n_all = pad_up_dev(rows) * bpr;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  const uint32_t* xw = reinterpret_cast<const uint32_t*>(x);

  for (int64_t base = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; base - lane < n_all;
       base += stride * kQuantUnroll) {
    uint32_t v[kQuantUnroll][8];
#pragma unroll
    for (int u = 0; u < kQuantUnroll; ++u) {
      const int64_t b = base + u * stride;
      if (b < n_real) {
        ld_stream_v8(xw + b * 8, v[u]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[u][j] = 0;
      }
    }
#pragma unroll
    for (int u = 0; u < kQuantUnroll; ++u) {
      const int64_t b = base + u * stride;
      // warp-uniform exit: the warp's blocks are consecutive
      if (b - lane >= n_all) break;
      const uint32_t* w = v[u];
      const uint32_t m2 = bmax2(bmax2(bmax2(w[0] & 0x7FFF7FFFu, w[1] & 0x7FFF7FFFu),
                                      bmax2(w[2] & 0x7FFF7FFFu, w[3] & 0x7FFF7FFFu)),
                                bmax2(bmax2(w[4] & 0x7FFF7FFFu, w[5] & 0x7FFF7FFFu),
                                      bmax2(w[6] & 0x7FFF7FFFu, w[7] & 0x7FFF7FFFu)));
      const uint32_t bm = max(m2 & 0xFFFFu, m2 >> 16);   // block max |x|, bf16 bits (exact)
      const float vmax = __uint_as_float(bm << 16);
      const uint32_t s8 = f32_to_e4m3(mul_ftz(g, mul_ftz(vmax, r6)));
      const float sfv = e4m3_to_f32(s8);
      // vmax != 0 under flush-to-zero: a subnormal maximum counts as zero
      const float os = (bm >= 0x0080u) ? rcp_approx_ftz(mul_ftz(sfv, rg)) : 0.0f;
      uint32_t byte[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        byte[j] = f32x2_to_e2m1x2(mul_ftz(__uint_as_float(w[j] << 16), os),
                                  mul_ftz(__uint_as_float(w[j] & 0xFFFF0000u), os));
      }
      const uint32_t c0 = pack4(byte[0], byte[1], byte[2], byte[3]);
      const uint32_t c1 = pack4(byte[4], byte[5], byte[6], byte[7]);
      // gather the group's 4 scale bytes into its first lane (b % 4 == lane % 4)
      const int lead = lane & ~3;
      const uint32_t s1 = __shfl_sync(0xFFFFFFFFu, s8, lead + 1);
      const uint32_t s2 = __shfl_sync(0xFFFFFFFFu, s8, lead + 2);
      const uint32_t s3 = __shfl_sync(0xFFFFFFFFu, s8, lead + 3);
      if (b < n_real) {
        *reinterpret_cast<uint2*>(codes + b * 8) = make_uint2(c0, c1);
      }
      if ((lane & 3) == 0 && b < n_all) {
        // block indices stay below 2^31 (checked by the host), so 32-bit division
        const uint32_t b32 = static_cast<uint32_t>(b);
        const uint32_t row32 = b32 / static_cast<uint32_t>(bpr);
        const int64_t row = row32;
        const int64_t kc = (b32 - row32 * static_cast<uint32_t>(bpr)) >> 2;
        const uint32_t word = (b < n_real) ? (s8 | (s1 << 8) | (s2 << 16) | (s3 << 24)) : 0u;
        const int64_t off = (row >> 7) * (gpr * 512) + kc * 512 + (row & 31) * 16 +
                            ((row & 127) >> 5) * 4;
        *reinterpret_cast<uint32_t*>(sf + off) = word;
      }
    }
  }
}

__global__ void rcp_probe_kernel(const float* in, float* out, int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = rcp_approx_ftz(in[i]);
}

}  // namespace

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

cudaError_t launch_amax(const uint16_t* x, int64_t numel, float* amax_out, float* g_out,
                        uint32_t* ws, float* zero_word, cudaStream_t st) {
  const int64_t nvec = numel / 8 + 1;
  int64_t blocks = (nvec + kThreads * kUnroll - 1) / (kThreads * kUnroll);
  blocks = blocks < 1 ? 1 : blocks;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks > kAmaxMaxBlocks) blocks = kAmaxMaxBlocks;
  amax_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(x, numel, amax_out, g_out, ws,
                                                                  zero_word);
  return cudaGetLastError();
}

cudaError_t launch_quantize(const uint16_t* x, int64_t rows, int64_t k, const float* g,
                            const float* amax, float* g_out, uint8_t* codes, uint8_t* sf,
                            float* zero_word, cudaStream_t st) {
  const int64_t n_all = pad_up(rows, 128) * (k / 16);
  int64_t blocks = (n_all + kThreads * kQuantUnroll - 1) / (kThreads * kQuantUnroll);
  blocks = blocks < 1 ? 1 : blocks;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  quantize_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(x, rows, k, g, amax, g_out,
                                                                      codes, sf, zero_word);
  return cudaGetLastError();
}

cudaError_t launch_rcp_probe(const float* in, float* out, int64_t n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const int64_t blocks = (n + 255) / 256;
  rcp_probe_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(in, out, n);
  return cudaGetLastError();
}

}  // namespace fvq
