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

// max of |bf16| over the 8 values of a uint4, as a bf16 bit pattern in the low 16 bits.
__device__ __forceinline__ uint32_t absmax8(uint4 v) {
  const uint32_t m = bmax2(bmax2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu),
                           bmax2(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu));
  return max(m & 0xFFFFu, m >> 16);
}

// max |x| over the 16-byte words first, first + stride, ... below nvec: batches
// of kUnroll independent loads (the last batch predicated), so every thread
// keeps kUnroll loads in flight even when it has fewer than kUnroll words.
__device__ __forceinline__ uint32_t absmax_words(const uint4* __restrict__ xv, int64_t nvec,
                                                 int64_t first, int64_t stride) {
  uint32_t m = 0;
  for (int64_t i = first; i < nvec; i += kUnroll * stride) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t j = i + u * stride;
      v[u] = j < nvec ? ld_stream(xv + j) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) m = max(m, absmax8(v[u]));
  }
  return m;
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
  uint32_t m = absmax_words(reinterpret_cast<const uint4*>(x), nvec, tid, nthreads);
  // ragged tail (numel % 8)
  for (int64_t t = nvec * 8 + tid; t < numel; t += nthreads) m = max(m, x[t] & 0x7FFFu);

  m = __reduce_max_sync(0xFFFFFFFFu, m);
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t bm = 0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) bm = max(bm, warp_max[w]);
    ws[kWsPartial + blockIdx.x] = bm;
    __threadfence();
    uint32_t prev = atomicAdd(&ws[kWsCounter], 1u);
    is_last = (prev == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last) return;
  // last CTA: reduce the per-CTA maxima, publish, and re-arm the counter.
  __threadfence();
  uint32_t bm = 0;
  for (int b = threadIdx.x; b < static_cast<int>(gridDim.x); b += kThreads)
    bm = max(bm, __ldcg(&ws[kWsPartial + b]));
  bm = __reduce_max_sync(0xFFFFFFFFu, bm);
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = bm;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t r = 0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) r = max(r, warp_max[w]);
    const float amax = __uint_as_float(r << 16);
    ws[kWsAmax] = __float_as_uint(amax);
    if (amax_out) *amax_out = amax;
    if (g_out) *g_out = encode_scale(amax);
    ws[kWsCounter] = 0;
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

// floor(n / d) for every n < 2^31 as umulhi(n, magic) >> shift, with
// l = ceil(log2 d), magic = ceil(2^(31 + l) / d) < 2^32 and shift = l - 1:
// the product overestimates n / d by less than n / 2^(31 + l) < 1 / d, which
// never reaches the next integer.
struct Div31 {
  uint32_t magic, shift;
};

Div31 make_div31(uint32_t d) {  // d >= 2
  uint32_t l = 0;
  while ((1ull << l) < d) ++l;
  const uint64_t num = 1ull << (31 + l);
  return Div31{static_cast<uint32_t>((num + d - 1) / d), l - 1};
}


__device__ __forceinline__ void discard_l2_line(const void* p) {
  asm volatile("discard.global.L2 [%0], 128;" ::"l"(p) : "memory");
}

// Element transform applied to each 16-value block of x before it is quantized
// (block index b in row-major block order, the block's eight bf16x2 words).
// load(b) fetches what the transform needs for block b; it is issued together
// with the block's own loads, one batch ahead.
struct NoXform {
  struct Aux {};
  __device__ __forceinline__ Aux load(uint32_t) const { return Aux{}; }
  __device__ __forceinline__ void operator()(uint32_t, uint32_t (&)[8], const Aux&) const {}
};

// Quantize x with encode scale g.  The work is cut into chunks of 32 blocks
// (1 KB of x, one per warp step); this warp takes chunks warp_first,
// warp_first + warp_stride, ...  kReverse walks the chunks from the end of x
// (the part a producer kernel wrote last, most likely still in L2).
// kDiscard drops each fully read 128-byte line of x from L2 without a
// write-back: only for a scratch input that nothing reads afterwards.
// Xform (NoXform unless given) maps each real block before its maximum is taken.
template <bool kReverse, bool kDiscard, class Xform = NoXform>
__device__ __forceinline__ void quantize_blocks(const uint16_t* __restrict__ x, uint32_t rows,
                                                uint32_t bpr, float g, uint8_t* __restrict__ codes,
                                                uint8_t* __restrict__ sf, uint32_t warp_first,
                                                uint32_t warp_stride, Div31 div,
                                                const Xform& xf = Xform()) {
  const float r6 = rcp_approx_ftz(6.0f);
  const float rg = rcp_approx_ftz(g);

  const uint32_t lane = threadIdx.x & 31;
  const uint32_t gpr = bpr / 4;                    // 64-column groups per row
  const uint32_t n_real = rows * bpr;              // < 2^31 (checked by the host)
  const uint32_t n_all = ((rows + 127) / 128 * 128) * bpr;
  const uint32_t n_chunks = (n_all + 31) / 32;
  const uint32_t* xw = reinterpret_cast<const uint32_t*>(x);

  // software pipeline: the next batch's loads are issued before this batch is
  // processed, so each thread keeps 2 * kQuantUnroll blocks of loads in flight
  using Aux = typename Xform::Aux;
  uint32_t vn[kQuantUnroll][8];
  Aux an[kQuantUnroll];
  auto load_batch = [&](uint32_t c0, uint32_t (&dst)[kQuantUnroll][8], Aux (&adst)[kQuantUnroll]) {
#pragma unroll
    for (int u = 0; u < kQuantUnroll; ++u) {
      const uint32_t cu = c0 + u * warp_stride;
      const uint32_t ch = kReverse ? n_chunks - 1 - cu : cu;
      const uint32_t b = ch * 32 + lane;
      if (cu < n_chunks && b < n_real) {
        ld_stream_v8(xw + static_cast<size_t>(b) * 8, dst[u]);
        adst[u] = xf.load(b);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) dst[u][j] = 0;
        adst[u] = Aux{};
      }
    }
  };
  load_batch(warp_first, vn, an);
  for (uint32_t c = warp_first; c < n_chunks; c += warp_stride * kQuantUnroll) {
    uint32_t v[kQuantUnroll][8];
    Aux a[kQuantUnroll];
    uint32_t chunk[kQuantUnroll];
#pragma unroll
    for (int u = 0; u < kQuantUnroll; ++u) {
      const uint32_t cu = c + u * warp_stride;
      chunk[u] = kReverse ? n_chunks - 1 - cu : cu;
      a[u] = an[u];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[u][j] = vn[u][j];
    }
    load_batch(c + warp_stride * kQuantUnroll, vn, an);
#pragma unroll
    for (int u = 0; u < kQuantUnroll; ++u) {
      if (c + u * warp_stride >= n_chunks) break;  // warp-uniform
      const uint32_t b = chunk[u] * 32 + lane;
      uint32_t w[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) w[j] = v[u][j];
      if (b < n_real) xf(b, w, a[u]);
      uint32_t c0, c1;
      const uint32_t s8 = quantize_block16(w, g, r6, rg, c0, c1);
      // gather the group's 4 scale bytes into its first lane (b % 4 == lane % 4)
      const uint32_t lead = lane & ~3u;
      const uint32_t s1 = __shfl_sync(0xFFFFFFFFu, s8, lead + 1);
      const uint32_t s2 = __shfl_sync(0xFFFFFFFFu, s8, lead + 2);
      const uint32_t s3 = __shfl_sync(0xFFFFFFFFu, s8, lead + 3);
      if (b < n_real) {
        *reinterpret_cast<uint2*>(codes + static_cast<size_t>(b) * 8) = make_uint2(c0, c1);
      }
      if ((lane & 3) == 0 && b < n_all) {
        const uint32_t row = __umulhi(b, div.magic) >> div.shift;
        const uint32_t kc = (b - row * bpr) >> 2;
        const uint32_t word = (b < n_real) ? (s8 | (s1 << 8) | (s2 << 16) | (s3 << 24)) : 0u;
        const size_t off = static_cast<size_t>(row >> 7) * (gpr * 512) + kc * 512 +
                           (row & 31) * 16 + ((row & 127) >> 5) * 4;
        *reinterpret_cast<uint32_t*>(sf + off) = word;
      }
      if (kDiscard) {
        __syncwarp();  // every lane has consumed its part of the chunk
        const uint32_t line_first_block = chunk[u] * 32 + lane * 4;
        if (lane < 8 && line_first_block + 4 <= n_real)
          discard_l2_line(xw + static_cast<size_t>(line_first_block) * 8);
      }
    }
  }
}

template <bool kReverse, bool kDiscard>
__global__ void __launch_bounds__(kThreads) quantize_kernel(
    const uint16_t* __restrict__ x, uint32_t rows, uint32_t bpr, const float* __restrict__ g_ptr,
    const float* __restrict__ amax_ptr, float* g_out, uint8_t* __restrict__ codes,
    uint8_t* __restrict__ sf, float* zero_word, Div31 div) {
  // launched as a programmatic dependent of the GEMM that wrote x
  grid_launch_dependents();
  grid_dependency_wait();
  const float g = amax_ptr != nullptr ? encode_scale(*amax_ptr) : *g_ptr;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (g_out != nullptr) *g_out = g;
    if (zero_word != nullptr) *zero_word = 0.0f;
  }
  constexpr uint32_t kWarps = kThreads / 32;
  quantize_blocks<kReverse, kDiscard>(x, rows, bpr, g, codes, sf,
                                      blockIdx.x * kWarps + (threadIdx.x >> 5), gridDim.x * kWarps,
                                      div);
}

// ---------------------------------------------------------------- W scale replication
// The GEMM's W scales for one 256-row N block and one 64-deep K step are two
// 512-byte atoms of the 128x4 layout (rows 0-127 and 128-255).  The tensor
// cores want each atom in all four 32-lane TMEM sub-partitions; a
// 128-lane x 256-bit tcgen05.cp does that in one instruction when the source
// row i already holds line i % 32 of both atoms.  This kernel writes that
// source: for N block nb, K step j, half h and replica r the 512-byte atom
// (2*nb + h, j) goes to byte ((((nb * k64 + j) * 2 + h) * 4 + r) * 512), so
// one K tile (four K steps) is 16 KB contiguous.
__global__ void __launch_bounds__(kThreads) replicate_w_scales_kernel(const uint4* __restrict__ sf,
                                                                       int64_t k64, int64_t total16,
                                                                       uint4* __restrict__ rep) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t o = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; o < total16;
       o += stride) {
    const int64_t x16 = o & 31;          // 16-byte word within the 512-byte atom
    const int64_t h = (o >> 7) & 1;      // o >> 5 = replica index bits, >> 7 = half
    const int64_t jb = o >> 8;           // nb * k64 + j
    const int64_t nb = jb / k64, j = jb - nb * k64;
    rep[o] = __ldg(sf + ((2 * nb + h) * k64 + j) * 32 + x16);
  }
}

// ---------------------------------------------------------------- fused amax + quantize
// One cooperative launch for the dynamic quantization of an activation:
//   pass 1: max |x| over this CTA's grid-stride share, published to ws[kWsPartial + cta]
//           (plus, optionally, a share of the W-scale replication above);
//   grid barrier (grid_barrier): the last CTA to arrive advances the generation
//           word ws[kWsGeneration], the others wait for it to change (bounded by
//           wait_limit ns: on expiry the CTA flags kErrWaitGrid and skips pass 2);
//   pass 2: every CTA reduces the published maxima to the same amax, forms
//           g = 2688 / max(amax, 1e-12) and quantizes its share of x, which pass 1
//           has just brought into L2.
// The cooperative launch makes all CTAs co-resident, so the barrier cannot wait
// on a CTA that has not started.
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid barrier for thread 0 of each CTA, in two levels so that no counter sees
// more than 64 arrivals: the last CTA of each group of 64 arrives at the top
// counter, the last of those advances the generation word.  Counters are
// reset by their last arrival, so the next launch finds them at zero.
// Returns false (and flags kErrWaitGrid) if the generation did not change
// within wait_limit ns.
__device__ bool grid_barrier(uint32_t* ws, uint32_t gen, uint64_t wait_limit, uint32_t* err_word) {
  const uint32_t ngroups = (gridDim.x + kBarrierGroup - 1) / kBarrierGroup;
  const uint32_t group = blockIdx.x / kBarrierGroup;
  const uint32_t in_group = min(static_cast<uint32_t>(kBarrierGroup), gridDim.x - group * kBarrierGroup);
  __threadfence();
  if (atomicAdd(&ws[kWsGroups + group], 1u) == in_group - 1) {
    ws[kWsGroups + group] = 0;
    __threadfence();
    if (atomicAdd(&ws[kWsCounter], 1u) == ngroups - 1) {
      ws[kWsCounter] = 0;
      __threadfence();
      st_release_gpu(&ws[kWsGeneration], gen + 1);
      return true;
    }
  }
  const uint64_t t0 = global_timer_ns();
  uint32_t sleep_ns = 32;
  while (ld_acquire_gpu(&ws[kWsGeneration]) == gen) {
    if (global_timer_ns() - t0 > wait_limit) {
      atomicOr(err_word, kErrWaitGrid);
      return false;
    }
    __nanosleep(sleep_ns);
    if (sleep_ns < 256) sleep_ns *= 2;
  }
  return true;
}

__global__ void __launch_bounds__(kThreads) amax_quantize_kernel(
    const uint16_t* __restrict__ x, int64_t rows, int64_t k, float* g_out,
    uint8_t* __restrict__ codes, uint8_t* __restrict__ sf, uint32_t* ws, float* zero_word,
    const uint4* __restrict__ rep_src, int64_t rep_k64, int64_t rep_total16,
    uint4* __restrict__ rep_dst, uint64_t wait_limit, uint32_t* err_word, Div31 div) {
  __shared__ uint32_t warp_max[kThreads / 32];
  __shared__ int go;
  grid_launch_dependents();  // the GEMM that follows may start its prologue
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * kThreads;
  uint32_t gen = 0;
  if (threadIdx.x == 0) gen = ld_acquire_gpu(&ws[kWsGeneration]);

  // pass 1: amax share
  const int64_t numel = rows * k;                  // k % 64 == 0: no ragged tail
  const int64_t nvec = numel / 8;
  uint32_t m = absmax_words(reinterpret_cast<const uint4*>(x), nvec, tid, nthreads);
  // W-scale replication share
  for (int64_t o = tid; o < rep_total16; o += nthreads) {
    const int64_t x16 = o & 31, h = (o >> 7) & 1, jb = o >> 8;
    const int64_t nb = jb / rep_k64, j = jb - nb * rep_k64;
    rep_dst[o] = __ldg(rep_src + ((2 * nb + h) * rep_k64 + j) * 32 + x16);
  }
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t bm = 0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) bm = max(bm, warp_max[w]);
    ws[kWsPartial + blockIdx.x] = bm;
    go = grid_barrier(ws, gen, wait_limit, err_word) ? 1 : 0;
  }
  __syncthreads();
  if (!go) return;

  // pass 2: the same amax in every CTA, then quantize
  uint32_t bm = 0;
  for (int b = threadIdx.x; b < static_cast<int>(gridDim.x); b += kThreads)
    bm = max(bm, __ldcg(&ws[kWsPartial + b]));
  bm = __reduce_max_sync(0xFFFFFFFFu, bm);
  __syncthreads();                     // warp_max reuse
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = bm;
  __syncthreads();
  uint32_t r = 0;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) r = max(r, warp_max[w]);
  const float amax = __uint_as_float(r << 16);
  const float g = encode_scale(amax);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    ws[kWsAmax] = __float_as_uint(amax);
    if (g_out != nullptr) *g_out = g;
    if (zero_word != nullptr) *zero_word = 0.0f;
  }
  constexpr uint32_t kWarps = kThreads / 32;
  quantize_blocks<false, false>(x, static_cast<uint32_t>(rows), static_cast<uint32_t>(k / 16), g,
                                codes, sf, blockIdx.x * kWarps + (threadIdx.x >> 5),
                                gridDim.x * kWarps, div);
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
                            float* zero_word, cudaStream_t st, bool scratch_input) {
  const int64_t n_all = pad_up(rows, 128) * (k / 16);
  const int64_t chunks = (n_all + 31) / 32;
  int64_t blocks = (chunks + (kThreads / 32) * kQuantUnroll - 1) / ((kThreads / 32) * kQuantUnroll);
  blocks = blocks < 1 ? 1 : blocks;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  const Div31 div = make_div31(static_cast<uint32_t>(k / 16));
  const uint32_t r = static_cast<uint32_t>(rows), bpr = static_cast<uint32_t>(k / 16);
  // the discard works on whole 128-byte lines
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(kThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // read from the end: an input the previous kernel just wrote (the intermediate, or the
  // previous layer's output in a stack) has its last-written lines still in L2
  if (scratch_input && (reinterpret_cast<uintptr_t>(x) & 127) == 0)
    return cudaLaunchKernelEx(&cfg, quantize_kernel<true, true>, x, r, bpr, g, amax, g_out, codes,
                              sf, zero_word, div);
  return cudaLaunchKernelEx(&cfg, quantize_kernel<true, false>, x, r, bpr, g, amax, g_out, codes,
                            sf, zero_word, div);
}

cudaError_t launch_replicate_w_scales(const uint8_t* sf, int64_t n, int64_t k, uint8_t* rep,
                                     cudaStream_t st) {
  const int64_t total16 = n * (k / 16) * 4 / 16;   // 4 replicas of n * k/16 scale bytes
  if (total16 <= 0) return cudaSuccess;
  int64_t blocks = (total16 + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  replicate_w_scales_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(
      reinterpret_cast<const uint4*>(sf), k / 64, total16, reinterpret_cast<uint4*>(rep));
  return cudaGetLastError();
}

cudaError_t launch_amax_quantize(const uint16_t* x, int64_t rows, int64_t k, float* g_out,
                                 uint8_t* codes, uint8_t* sf, uint32_t* ws, float* zero_word,
                                 const uint8_t* rep_src, int64_t rep_n, int64_t rep_k,
                                 uint8_t* rep_dst, uint64_t wait_limit, uint32_t* err_word,
                                 cudaStream_t st) {
  static int resident[64] = {0};   // CTAs of this kernel per SM, per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (resident[dev] == 0) {
    int nb = 0;
    cudaError_t e =
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, amax_quantize_kernel, kThreads, 0);
    if (e != cudaSuccess) return e;
    resident[dev] = nb > 0 ? nb : 1;
  }
  const int64_t n_all = pad_up(rows, 128) * (k / 16);
  int64_t blocks = (n_all + kThreads * kQuantUnroll - 1) / (kThreads * kQuantUnroll);
  blocks = blocks < 1 ? 1 : blocks;
  const int64_t cap = static_cast<int64_t>(sm_count()) * resident[dev];
  if (blocks > cap) blocks = cap;
  if (blocks > kAmaxMaxBlocks) blocks = kAmaxMaxBlocks;
  const uint4* rsrc = reinterpret_cast<const uint4*>(rep_src);
  uint4* rdst = reinterpret_cast<uint4*>(rep_dst);
  int64_t rep_k64 = rep_k / 64 > 0 ? rep_k / 64 : 1;
  int64_t rep_total16 = rep_dst != nullptr ? rep_n * (rep_k / 16) * 4 / 16 : 0;
  Div31 div = make_div31(static_cast<uint32_t>(k / 16));
  void* args[] = {&x, &rows, &k, &g_out, &codes, &sf, &ws, &zero_word, &rsrc, &rep_k64,
                  &rep_total16, &rdst, &wait_limit, &err_word, &div};
  return cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(amax_quantize_kernel),
                                     dim3(static_cast<unsigned>(blocks)), dim3(kThreads), args, 0,
                                     st);
}

namespace {

// ---------------------------------------------------------------- LayerNorm + modulation fused in
// The DiT block's FFN input u = bf16(bf16(LN(x) * bf16(1 + scale)) + shift) (LN without
// affine), quantized without writing u: pass 1 takes each row's mean and rstd exactly as
// ln_modulate_kernel does (one warp per row, same lane layout and summation order), keeps
// them in `stats` and takes max |u|; pass 2 recomputes u block by block from x and quantizes.
__device__ __forceinline__ uint32_t ln_pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t ln_add_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t ln_mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// u of one bf16x2 word of x, given the row's mean and rstd and the column pair's
// bf16x2 words of (1 + scale) and shift.
__device__ __forceinline__ uint32_t ln_modulate_word(uint32_t xw, float mean, float rstd,
                                                     uint32_t one_scale, uint32_t shift) {
  const float lo = (__uint_as_float(xw << 16) - mean) * rstd;
  const float hi = (__uint_as_float(xw & 0xFFFF0000u) - mean) * rstd;
  return ln_add_bf16x2(ln_mul_bf16x2(ln_pack_bf16x2(lo, hi), one_scale), shift);
}

struct LnModXform {
  const float2* stats;      // [rows] (mean, rstd)
  const uint4* shift;       // [d / 8]
  const uint4* scale;
  uint32_t bpr;             // 16-value blocks per row
  Div31 div;
  using Aux = float2;       // the block's row statistics, fetched with the block
  __device__ __forceinline__ float2 load(uint32_t b) const {
    return __ldcg(stats + (__umulhi(b, div.magic) >> div.shift));
  }
  __device__ __forceinline__ void operator()(uint32_t b, uint32_t (&w)[8], const float2& st) const {
    const uint32_t row = __umulhi(b, div.magic) >> div.shift;
    const uint32_t blk = b - row * bpr;
    const uint4 s0 = __ldg(shift + 2 * blk), s1 = __ldg(shift + 2 * blk + 1);
    const uint4 c0 = __ldg(scale + 2 * blk), c1 = __ldg(scale + 2 * blk + 1);
    const uint32_t sw[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const uint32_t cw[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
    for (int j = 0; j < 8; ++j)
      w[j] = ln_modulate_word(w[j], st.x, st.y, ln_add_bf16x2(0x3F803F80u, cw[j]), sw[j]);
  }
};

template <int kVec>
__global__ void __launch_bounds__(kThreads, kVec >= 8 ? 2 : 3) amax_quantize_ln_kernel(
    const uint16_t* __restrict__ x, int64_t rows, int64_t k, const uint16_t* __restrict__ shift,
    const uint16_t* __restrict__ scale, float eps, float2* __restrict__ stats, float* g_out,
    uint8_t* __restrict__ codes, uint8_t* __restrict__ sf, uint32_t* ws, float* zero_word,
    const uint4* __restrict__ rep_src, int64_t rep_k64, int64_t rep_total16,
    uint4* __restrict__ rep_dst, uint64_t wait_limit, uint32_t* err_word, Div31 div) {
  __shared__ uint32_t warp_max[kThreads / 32];
  __shared__ int go;
  grid_launch_dependents();  // the GEMM that follows may start its prologue
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * kThreads;
  const int lane = threadIdx.x & 31;
  uint32_t gen = 0;
  if (threadIdx.x == 0) gen = ld_acquire_gpu(&ws[kWsGeneration]);

  // pass 1: per-row statistics and max |u| (one warp per row)
  const int d = static_cast<int>(k), nvec = d / 8;
  const uint4* sh4 = reinterpret_cast<const uint4*>(shift);
  const uint4* sc4 = reinterpret_cast<const uint4*>(scale);
  uint32_t m2 = 0;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kThreads / 32);
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5);
       row < rows; row += warps) {
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
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
      const int j = lane + i * 32;
      if (j >= nvec) continue;
      const uint4 s = __ldg(sh4 + j), c = __ldg(sc4 + j);
      const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
      const uint32_t sw[4] = {s.x, s.y, s.z, s.w}, cw[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t u = ln_modulate_word(w[q], mean, rstd, ln_add_bf16x2(0x3F803F80u, cw[q]), sw[q]);
        m2 = bmax2(m2, u & 0x7FFF7FFFu);
      }
    }
    if (lane == 0) stats[row] = make_float2(mean, rstd);
  }
  uint32_t m = max(m2 & 0xFFFFu, m2 >> 16);
  // W-scale replication share
  for (int64_t o = tid; o < rep_total16; o += nthreads) {
    const int64_t x16 = o & 31, h = (o >> 7) & 1, jb = o >> 8;
    const int64_t nb = jb / rep_k64, j = jb - nb * rep_k64;
    rep_dst[o] = __ldg(rep_src + ((2 * nb + h) * rep_k64 + j) * 32 + x16);
  }
  __threadfence();  // the row statistics are read by other CTAs after the grid barrier
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t bm = 0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) bm = max(bm, warp_max[w]);
    ws[kWsPartial + blockIdx.x] = bm;
    go = grid_barrier(ws, gen, wait_limit, err_word) ? 1 : 0;
  }
  __syncthreads();
  if (!go) return;

  // pass 2: the same amax in every CTA, then quantize u recomputed from x
  uint32_t bm = 0;
  for (int b = threadIdx.x; b < static_cast<int>(gridDim.x); b += kThreads)
    bm = max(bm, __ldcg(&ws[kWsPartial + b]));
  bm = __reduce_max_sync(0xFFFFFFFFu, bm);
  __syncthreads();                     // warp_max reuse
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = bm;
  __syncthreads();
  uint32_t r = 0;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) r = max(r, warp_max[w]);
  const float amax = __uint_as_float(r << 16);
  const float g = encode_scale(amax);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    ws[kWsAmax] = __float_as_uint(amax);
    if (g_out != nullptr) *g_out = g;
    if (zero_word != nullptr) *zero_word = 0.0f;
  }
  constexpr uint32_t kWarps = kThreads / 32;
  const LnModXform xf{stats, sh4, sc4, static_cast<uint32_t>(k / 16), div};
  quantize_blocks<false, false>(x, static_cast<uint32_t>(rows), static_cast<uint32_t>(k / 16), g,
                                codes, sf, blockIdx.x * kWarps + (threadIdx.x >> 5),
                                gridDim.x * kWarps, div, xf);
}

template <int kVec>
cudaError_t launch_aq_ln_t(const uint16_t* x, int64_t rows, int64_t k, const uint16_t* shift,
                           const uint16_t* scale, float eps, float2* stats, float* g_out,
                           uint8_t* codes, uint8_t* sf, uint32_t* ws, float* zero_word,
                           const uint8_t* rep_src, int64_t rep_n, int64_t rep_k, uint8_t* rep_dst,
                           uint64_t wait_limit, uint32_t* err_word, cudaStream_t st) {
  static int resident[64] = {0};   // CTAs of this kernel per SM, per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (resident[dev] == 0) {
    int nb = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &nb, amax_quantize_ln_kernel<kVec>, kThreads, 0);
    if (e != cudaSuccess) return e;
    resident[dev] = nb > 0 ? nb : 1;
  }
  const int64_t n_all = pad_up(rows, 128) * (k / 16);
  int64_t blocks = (n_all + kThreads * kQuantUnroll - 1) / (kThreads * kQuantUnroll);
  blocks = blocks < 1 ? 1 : blocks;
  const int64_t cap = static_cast<int64_t>(sm_count()) * resident[dev];
  if (blocks > cap) blocks = cap;
  if (blocks > kAmaxMaxBlocks) blocks = kAmaxMaxBlocks;
  const uint4* rsrc = reinterpret_cast<const uint4*>(rep_src);
  uint4* rdst = reinterpret_cast<uint4*>(rep_dst);
  int64_t rep_k64 = rep_k / 64 > 0 ? rep_k / 64 : 1;
  int64_t rep_total16 = rep_dst != nullptr ? rep_n * (rep_k / 16) * 4 / 16 : 0;
  Div31 div = make_div31(static_cast<uint32_t>(k / 16));
  void* args[] = {&x, &rows, &k, &shift, &scale, &eps, &stats, &g_out, &codes, &sf, &ws,
                  &zero_word, &rsrc, &rep_k64, &rep_total16, &rdst, &wait_limit, &err_word, &div};
  return cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(amax_quantize_ln_kernel<kVec>),
                                     dim3(static_cast<unsigned>(blocks)), dim3(kThreads), args, 0,
                                     st);
}

}  // namespace

cudaError_t launch_amax_quantize_ln(const uint16_t* x, int64_t rows, int64_t k,
                                    const uint16_t* shift, const uint16_t* scale, float eps,
                                    float* stats, float* g_out, uint8_t* codes, uint8_t* sf,
                                    uint32_t* ws, float* zero_word, const uint8_t* rep_src,
                                    int64_t rep_n, int64_t rep_k, uint8_t* rep_dst,
                                    uint64_t wait_limit, uint32_t* err_word, cudaStream_t st) {
  float2* st2 = reinterpret_cast<float2*>(stats);
  switch (static_cast<int>((k / 8 + 31) / 32)) {
    case 0:
    case 1: return launch_aq_ln_t<1>(x, rows, k, shift, scale, eps, st2, g_out, codes, sf, ws, zero_word, rep_src, rep_n, rep_k, rep_dst, wait_limit, err_word, st);
    case 2: return launch_aq_ln_t<2>(x, rows, k, shift, scale, eps, st2, g_out, codes, sf, ws, zero_word, rep_src, rep_n, rep_k, rep_dst, wait_limit, err_word, st);
    case 3:
    case 4: return launch_aq_ln_t<4>(x, rows, k, shift, scale, eps, st2, g_out, codes, sf, ws, zero_word, rep_src, rep_n, rep_k, rep_dst, wait_limit, err_word, st);
    case 5:
    case 6: return launch_aq_ln_t<6>(x, rows, k, shift, scale, eps, st2, g_out, codes, sf, ws, zero_word, rep_src, rep_n, rep_k, rep_dst, wait_limit, err_word, st);
    case 7:
    case 8: return launch_aq_ln_t<8>(x, rows, k, shift, scale, eps, st2, g_out, codes, sf, ws, zero_word, rep_src, rep_n, rep_k, rep_dst, wait_limit, err_word, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_rcp_probe(const float* in, float* out, int64_t n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const int64_t blocks = (n + 255) / 256;
  rcp_probe_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(in, out, n);
  return cudaGetLastError();
}

}  // namespace fvq
