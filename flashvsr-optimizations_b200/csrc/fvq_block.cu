// fvq_block.cu -- the DiT block around the FFN (the caller of block.ffn in the
// reference's installer, ffn_quantization.py:77-80): adaLN-modulated input and
// gated residual,
//
//   u   = bf16(bf16(LN(x) * bf16(1 + scale)) + shift)      LN without affine, eps
//   out = bf16(x + bf16(gate * FFN(u)))                      (GEMM2's epilogue 2)
//
// each elementwise step one bf16 rounding, as torch evaluates it on bf16
// tensors.  LN(x) = bf16((x - mean) * rsqrtf(var + eps)) with mean and the
// biased variance of the row in fp32.
//
// ln_modulate_kernel: one warp per row (d <= 2048, d % 8 == 0), the row held
// in registers; mean, then the variance around it, each reduced across the
// warp.  HBM-bound: one read of x, one write of u.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "fvq_internal.h"

namespace fvq {

namespace {

constexpr int kLnThreads = 256;

__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

template <int kVec>
__global__ void __launch_bounds__(kLnThreads) ln_modulate_kernel(
    const uint16_t* __restrict__ x, int64_t rows, int d, const uint16_t* __restrict__ shift,
    const uint16_t* __restrict__ scale, float eps, uint16_t* __restrict__ u) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (kLnThreads / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nvec = d / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * d);
  uint4 v[kVec];
  float sum = 0.0f;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int j = lane + i * 32;
    v[i] = j < nvec ? __ldg(xr + j) : make_uint4(0, 0, 0, 0);
    const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
    for (int q = 0; q < 4; ++q)
      sum += __uint_as_float(w[q] << 16) + __uint_as_float(w[q] & 0xFFFF0000u);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
  const float mean = sum / static_cast<float>(d);
  float sq = 0.0f;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int j = lane + i * 32;
    if (j >= nvec) continue;
    const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float a = __uint_as_float(w[q] << 16) - mean, b = __uint_as_float(w[q] & 0xFFFF0000u) - mean;
      sq += a * a + b * b;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xFFFFFFFFu, sq, o);
  const float rstd = rsqrtf(sq / static_cast<float>(d) + eps);
  const uint4* sh4 = reinterpret_cast<const uint4*>(shift);
  const uint4* sc4 = reinterpret_cast<const uint4*>(scale);
  uint4* ur = reinterpret_cast<uint4*>(u + row * d);
  const uint32_t one2 = 0x3F803F80u;  // bf16 (1, 1)
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int j = lane + i * 32;
    if (j >= nvec) continue;
    const uint4 s = __ldg(sh4 + j), c = __ldg(sc4 + j);
    const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
    const uint32_t sw[4] = {s.x, s.y, s.z, s.w}, cw[4] = {c.x, c.y, c.z, c.w};
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float lo = (__uint_as_float(w[q] << 16) - mean) * rstd;
      const float hi = (__uint_as_float(w[q] & 0xFFFF0000u) - mean) * rstd;
      const uint32_t n2 = pack_bf16x2(lo, hi);
      o[q] = add_bf16x2(mul_bf16x2(n2, add_bf16x2(one2, cw[q])), sw[q]);
    }
    ur[j] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <int kVec>
void ln_launch(const uint16_t* x, int64_t rows, int d, const uint16_t* shift, const uint16_t* scale,
               float eps, uint16_t* u, cudaStream_t st) {
  const int64_t blocks = (rows + kLnThreads / 32 - 1) / (kLnThreads / 32);
  ln_modulate_kernel<kVec><<<static_cast<unsigned>(blocks), kLnThreads, 0, st>>>(x, rows, d, shift,
                                                                                  scale, eps, u);
}

}  // namespace

cudaError_t launch_ln_modulate(const uint16_t* x, int64_t rows, int64_t d, const uint16_t* shift,
                               const uint16_t* scale, float eps, uint16_t* u, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const int di = static_cast<int>(d);
  switch (static_cast<int>((d / 8 + 31) / 32)) {
    case 0:
    case 1: ln_launch<1>(x, rows, di, shift, scale, eps, u, st); break;
    case 2: ln_launch<2>(x, rows, di, shift, scale, eps, u, st); break;
    case 3:
    case 4: ln_launch<4>(x, rows, di, shift, scale, eps, u, st); break;
    case 5:
    case 6: ln_launch<6>(x, rows, di, shift, scale, eps, u, st); break;
    case 7:
    case 8: ln_launch<8>(x, rows, di, shift, scale, eps, u, st); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace fvq
