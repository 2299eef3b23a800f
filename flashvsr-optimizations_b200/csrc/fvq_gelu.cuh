// fvq_gelu.cuh -- bf16 GELU (tanh approximation) exactly as torch evaluates it for bf16
// inputs (the fp32 formula, one rounding to bf16), used by the GEMM epilogues.
//
// A bf16 input has 65536 values.  Inputs with exponent field in [107, 130) (|x| in
// [2^-20, 8)) are tabulated (computed with the exact fp32 formula, gelu_table_init); the
// rest take short exact paths (gelu_bf16).  The range reaches down to 2^-20 because the
// intermediate of a deep stack is small: its pre-activations shrink to a standard
// deviation near 0.02, where 1% of them lie below 2^-12.  Entry index:
// ((bits & 0x7FFF) - 0x3580) + sign * 2944, 2 x 2944 entries (11.5 KB).
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

namespace fvq {

constexpr uint32_t kGeluTabLo = 107u << 7;       // 0x3580 = 2^-20
constexpr uint32_t kGeluTabSpan = 23u << 7;      // 0xB80: magnitudes below 8.0
constexpr int kGeluTabEntries = 2 * kGeluTabSpan;
constexpr int kGeluTabBytes = kGeluTabEntries * 2;
static_assert(kGeluTabBytes % 16 == 0, "table keeps what follows it 16-byte aligned");

// GELU, tanh approximation, evaluated in fp32 as torch does for bf16 inputs.
__device__ __forceinline__ float gelu_tanh(float x) {
  const float kBeta = 0.7978845608028654f;  // sqrt(2 / pi)
  const float kKappa = 0.044715f;
  const float x_cube = x * x * x;
  const float inner = kBeta * (x + kKappa * x_cube);
  return 0.5f * x * (1.0f + tanhf(inner));
}

__device__ __noinline__ inline uint32_t gelu_bf16_exact(uint32_t x_bits) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(gelu_tanh(__uint_as_float(x_bits << 16))));
}

__device__ __forceinline__ void gelu_table_init(uint16_t* tab, int tid, int nthreads) {
  for (int i = tid; i < kGeluTabEntries; i += nthreads) {
    const uint32_t neg = static_cast<uint32_t>(i) >= kGeluTabSpan ? 1u : 0u;
    const uint32_t off = static_cast<uint32_t>(i) - neg * kGeluTabSpan;
    tab[i] = static_cast<uint16_t>(gelu_bf16_exact((neg << 15) | (kGeluTabLo + off)));
  }
}

// bf16(gelu(x)) for |x| < 2^-12 (zeros and subnormals included).  There the fp32
// formula is 0.5x * (1 + t) with |t| = |tanh(sqrt(2/pi)(x + 0.044715x^3))| < 2^-12: for
// a normal x, 0.5x is a bf16 value and the factor (1 + t) moves it by far less than
// half a bf16 ulp, so the result rounds back to 0.5x; for a subnormal x, t is so small
// that 1 + t == 1 in fp32.  Either way the result is bf16_rn(0.5x) (0.5x exact in
// fp32, then one rounding).  The GPU test compares every bf16 input with torch.
__device__ __forceinline__ uint32_t gelu_bf16_tiny(uint32_t x_bits) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(__fmul_rn(__uint_as_float(x_bits << 16), 0.5f)));
}

// bf16(gelu(x)) for a bf16 input, bit-identical to the exact formula.  For
// 8 <= |x| (finite, and +inf) the fp32 tanh saturates to +-1, so the formula
// gives x itself for positive x and -0 for negative x; below 2^-20 see
// gelu_bf16_tiny; only -inf and NaN evaluate the formula.
__device__ __forceinline__ uint32_t gelu_bf16(uint32_t x_bits, const uint16_t* tab) {
  const uint32_t mag = x_bits & 0x7FFFu;
  const uint32_t off = mag - kGeluTabLo;
  if (off < kGeluTabSpan) return tab[off + ((x_bits >> 15) & 1u) * kGeluTabSpan];
  if (mag < kGeluTabLo) return gelu_bf16_tiny(x_bits);
  if (mag < 0x7F80u) return (x_bits & 0x8000u) ? 0x8000u : x_bits;
  if (x_bits == 0x7F80u) return x_bits;
  return gelu_bf16_exact(x_bits);
}

__device__ __noinline__ inline uint32_t gelu_bf16x2_slow(uint32_t hv, const uint16_t* tab) {
  return gelu_bf16(hv & 0xFFFFu, tab) | (gelu_bf16(hv >> 16, tab) << 16);
}

__device__ __forceinline__ uint32_t min_u16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("min.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t max_u16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
  uint32_t r;
  asm("ld.shared.u16 %0, [%1];" : "=r"(r) : "r"(addr));
  return r;
}

// GELU of four bf16x2 words.  Per word both magnitude offsets are formed in one
// 32-bit subtraction and clamped to the last entry in one min.u16x2, so the two
// lookups stay inside the table whatever the input; a negative half adds the
// table's span to its index.  There is no branch between the eight lookups, so all
// can be in flight at once; a word with a half that was clamped (outside
// [2^-20, 8), or a borrow from the low half) is redone through gelu_bf16 afterwards.
// tab_base is the table's shared-memory address.
__device__ __forceinline__ void gelu_bf16x2_x4(uint32_t (&w)[4], uint32_t tab_base,
                                               const uint16_t* tab) {
  uint32_t res[4];
  uint32_t slow = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t d = (w[j] & 0x7FFF7FFFu) - ((kGeluTabLo << 16) | kGeluTabLo);
    const uint32_t c = min_u16x2(d, ((kGeluTabSpan - 1) << 16) | (kGeluTabSpan - 1));
    const uint32_t off2 = (c + ((w[j] >> 15) & 0x00010001u) * kGeluTabSpan) << 1;
    res[j] = __byte_perm(lds_u16(tab_base + (off2 & 0xFFFFu)), lds_u16(tab_base + (off2 >> 16)),
                         0x5410);
    slow |= static_cast<uint32_t>(c != d) << j;
  }
  if (slow != 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if ((slow >> j) & 1u) res[j] = gelu_bf16x2_slow(w[j], tab);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) w[j] = res[j];
}

}  // namespace fvq
