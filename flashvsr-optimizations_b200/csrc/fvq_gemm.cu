// fvq_gemm.cu -- block-scaled NVFP4 GEMM on sm_100a tensor cores.
//
//   out[m, n] = epilogue(alpha * sum_k A[m, k] W[n, k]),  alpha = 1 / (g_a * g_w)
//
// Replaces flashinfer.mm_fp4(..., backend='cutlass') plus the bias add that
// follows it (reference ffn_quantization.py:65-69).  Design:
//   * persistent CTAs (one per SM), 128 x 256 output tile, 256-deep K tiles;
//   * warp 0: TMA producer (A and W codes through 128B-swizzled tensor maps,
//     the scale factors as contiguous 2 KB bulk copies -- the 128x4 swizzled
//     layout keeps a 128-row x 256-K scale tile contiguous);
//   * warp 1: owns TMEM (512 columns: fp32 accumulator in 0-255, A scales in
//     256-271, W scales in 272-303), moves scales smem -> TMEM with
//     tcgen05.cp and issues tcgen05.mma.kind::mxf4nvf4 (K = 64 per MMA);
//   * warps 2-17: epilogue; each thread owns one accumulator row and 64
//     columns, pulls them into registers, forms bf16(alpha*acc), frees the
//     accumulator for the next tile, then adds the bias and (GEMM1) applies
//     GELU through a shared-memory table, tracks max |h| and writes the
//     warp's 32 x 64 block through a swizzled staging buffer with one TMA
//     tensor store, or (GEMM2) stores from registers, while the next tile's
//     MMAs run.
// Every CTA loads its own tiles (no loads shared across a CTA cluster).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "fvq_gelu.cuh"
#include "fvq_internal.h"
#include "fvq_ptx.cuh"

namespace fvq {

__device__ uint32_t g_device_error = 0;

namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 256;
constexpr int BKB = BK / 2;                      // bytes of codes per row per K tile
constexpr int kABytes = BM * BKB;                // 16 KB
constexpr int kBBytes = BN * BKB;                // 32 KB
constexpr int kSfaBytes = BM * (BK / 16);        // 2 KB
constexpr int kSfbBytes = BN * (BK / 16);        // 4 KB
constexpr int kSfbRepBytes = 4 * kSfbBytes;      // 16 KB: W scales replicated for 128x256b copies
constexpr int kEpiWarps = 16;                    // 4 per TMEM lane quadrant, 64 columns each
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kNumThreads = 64 + kEpiThreads;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSfaCol = 256;                // A scales: 16 columns (4 K-steps x 4)
constexpr uint32_t kSfbCol = 272;                // W scales: 8 columns per K-step
constexpr int kMaxResidentKSteps = (512 - 272) / 8;  // W scales of up to K = 1920 stay in TMEM
constexpr int kBarrierBytes = 256;
constexpr int kStagingBytes = BM * BN * 2;       // bf16 tile staged for coalesced stores

constexpr int kStageRowBytes = 128;              // one epilogue row: 64 bf16 columns
constexpr int kWarpStagingBytes = 32 * kStageRowBytes;

// Shared-memory plan.  kResident: the W scales of the CTA's single N block
// are loaded into TMEM once (K <= 1920), so stages carry only A, W and A scales.
// kRepSfb: stages carry the W scales already replicated four times (16 KB per
// K tile), moved to TMEM with four 128x256b copies instead of eight
// 32x128b.warpx4 copies.
// kEpi 3 (GEMM1 quantizing its own output) writes NVFP4 codes and scales straight
// from registers: it needs no staging buffer, so four resident stages fit, and in resident mode
// the W scales are preloaded through the last stage's buffer (kPreloadInStage: the
// producer fills that stage only after the MMA warp's copies out of it completed).
template <int kEpi, bool kResident, bool kRepSfb = false>
struct Plan {
  static constexpr int kStageBytes =
      kABytes + kBBytes + kSfaBytes + (kResident ? 0 : (kRepSfb ? kSfbRepBytes : kSfbBytes));
  static constexpr bool kStaged = kEpi == 1;
  static constexpr int kStages =
      kEpi == 3 ? (kResident ? 4 : 3) : (!kStaged ? (kRepSfb ? 3 : 4) : (kResident ? 3 : 2));
  static constexpr bool kGelu = kEpi == 1 || kEpi == 3;
  static constexpr bool kPreloadInStage = kResident && !kStaged;
  static constexpr int kStagingOff = kStages * kStageBytes;
  static constexpr int kTableOff = kStagingOff + (kStaged ? kStagingBytes : 0);
  static constexpr int kBarrierOff = kTableOff + (kGelu ? kGeluTabBytes : 0);
  static constexpr int kSmemBytes = kBarrierOff + kBarrierBytes;
};
static_assert(Plan<1, true>::kSmemBytes <= 232448, "GEMM1 resident plan exceeds shared memory");
static_assert(Plan<1, false>::kSmemBytes <= 232448, "GEMM1 streaming plan exceeds shared memory");
static_assert(Plan<3, true>::kSmemBytes <= 232448, "quantizing GEMM1 plan exceeds shared memory");
static_assert(Plan<3, false>::kSmemBytes <= 232448, "quantizing GEMM1 plan exceeds shared memory");
static_assert(2 * (kMaxResidentKSteps * 512) <= Plan<3, true>::kStageBytes,
              "resident W scales must fit one stage buffer");
static_assert(Plan<0, false>::kSmemBytes <= 232448, "GEMM2 plan exceeds shared memory");
static_assert(Plan<0, false, true>::kSmemBytes <= 232448, "GEMM2 replicated plan exceeds shared memory");

// Instruction descriptor, kind::mxf4nvf4: A/B E2M1 (1), UE4M3 scales (0),
// K-major A and B, N = 256 (>>3 at bit 17), M = 128 (>>4 at bit 24).
constexpr uint32_t kIdesc = (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
                            (static_cast<uint32_t>(BM >> 4) << 24);
// N = 128: one half of a W tile (tail tiles split in two, see TileSeq)
constexpr uint32_t kIdescHalf = (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN / 2 >> 3) << 17) |
                                (static_cast<uint32_t>(BM >> 4) << 24);

template <int kStages>
struct Barriers {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full;
  uint64_t acc_empty;
  uint64_t teardown;
  uint64_t sfb_full;
  uint64_t sfb_free;   // the resident W scales' copies to TMEM completed (kPreloadInStage)
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Barriers<4>) <= kBarrierBytes, "barrier area");

template <class B>
__device__ __forceinline__ void flag_error(B* bars, uint32_t bit) {
  atomicOr(&g_device_error, bit);
  *reinterpret_cast<volatile int*>(&bars->abort_flag) = 1;
}

template <class B>
__device__ __forceinline__ bool aborted(B* bars) {
  return *reinterpret_cast<volatile int*>(&bars->abort_flag) != 0;
}

// aborted() as lane 0 of a converged warp sees it, for every lane.
template <class B>
__device__ __forceinline__ bool warp_aborted(B* bars) {
  return __shfl_sync(0xFFFFFFFFu, aborted(bars) ? 1 : 0, 0) != 0;
}

// flag_error from one lane of a converged warp.
template <class B>
__device__ __forceinline__ void warp_flag_error(B* bars, uint32_t bit) {
  if (elect_one()) flag_error(bars, bit);
  __syncwarp();
}

// Two floats -> two bf16 (round to nearest even) in one cvt.rn.bf16x2.f32.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// alpha * (lo, hi) with one mul.rn.f32x2 (two IEEE products), rounded to a bf16x2 pair.
__device__ __forceinline__ uint32_t scale_pack_bf16x2(uint32_t lo_bits, uint32_t hi_bits,
                                                      uint64_t alpha2) {
  uint64_t v, p;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "r"(lo_bits), "r"(hi_bits));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(p) : "l"(v), "l"(alpha2));
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(p));
  return pack_bf16x2(lo, hi);
}

// bf16x2 product, one rounding of the exact product (two 8-bit mantissas fit in fp32, so
// torch's fp32 multiply followed by a bf16 rounding gives the same value).
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// bf16x2 add, one rounding of the exact sum.  For two bf16 operands this equals
// torch's fp32 add followed by a bf16 rounding: the fp32 sum is exact unless
// the exponents differ by more than 16, and then it lies far from a bf16 tie.
__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Tiles of one CTA.  Streaming: tile t = blockIdx + i*grid, M-block fastest.
// Resident: the CTA keeps one N block (blockIdx % NB) and strides over M blocks.
// kSplitTail (streaming only): when the tiles past the last full round of the
// grid number at most half the grid, each of them is split into two N = 128
// halves, one per CTA, so that the last round takes about half as long;
// `half` is -1 for a whole tile, else 0 or 1.
template <bool kResident, bool kSplitTail>
struct TileSeq {
  int count, nb_fixed, mb0, mb_step, num_m_blocks, full_rounds;
  bool split;
  __device__ TileSeq(int num_m, int num_n) : num_m_blocks(num_m) {
    const int c = blockIdx.x, g = gridDim.x;
    split = false;
    full_rounds = 0;
    if (kResident) {
      nb_fixed = c % num_n;
      mb0 = c / num_n;
      mb_step = (g - 1 - nb_fixed) / num_n + 1;
      count = mb0 < num_m ? (num_m - 1 - mb0) / mb_step + 1 : 0;
    } else {
      const int tiles = num_m * num_n;
      nb_fixed = 0;
      mb0 = 0;
      mb_step = 0;
      count = c < tiles ? (tiles - 1 - c) / g + 1 : 0;
      const int rounds = tiles / g, rest = tiles - rounds * g;
      if (kSplitTail && rounds > 0 && rest > 0 && 2 * rest <= g) {
        split = true;
        full_rounds = rounds;
        count = rounds + (c < 2 * rest ? 1 : 0);
      }
    }
  }
  __device__ void at(int i, int& mb, int& nb, int& half) const {
    half = -1;
    if (kResident) {
      mb = mb0 + i * mb_step;
      nb = nb_fixed;
    } else {
      int t = blockIdx.x + i * gridDim.x;
      if (split && i == full_rounds) {
        t = full_rounds * gridDim.x + (blockIdx.x >> 1);
        half = blockIdx.x & 1;
      }
      mb = t % num_m_blocks;
      nb = t / num_m_blocks;
    }
  }
};

template <int kEpi, bool kResident, bool kRepSfb>
__global__ void __launch_bounds__(kNumThreads, 1)
    nvfp4_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                      const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ CUtensorMap tmap_out, const uint8_t* __restrict__ a_sf,
                      const uint8_t* __restrict__ w_sf, const float* __restrict__ g_a,
                      const float* __restrict__ g_w, const float* __restrict__ alpha_in,
                      const uint16_t* __restrict__ bias, uint16_t* __restrict__ out, int m, int n,
                      int k, float* amax_out, uint64_t wait_limit,
                      const uint16_t* __restrict__ residual, const uint16_t* __restrict__ gate,
                      QuantOut qo) {
  using P = Plan<kEpi, kResident, kRepSfb>;
  constexpr int kStages = P::kStages;
  constexpr int kStageBytes = P::kStageBytes;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if ((smem_u32(smem) & 1023u) != 0) {  // the 128B-swizzled tiles need 1024-byte alignment
    if (threadIdx.x == 0) atomicOr(&g_device_error, kErrSmemAlign);
    return;
  }
  auto* bars = reinterpret_cast<Barriers<kStages>*>(smem + P::kBarrierOff);
  uint8_t* staging = smem + P::kStagingOff;
  uint16_t* gelu_tab = reinterpret_cast<uint16_t*>(smem + P::kTableOff);

  const int warp = warp_index_uniform();
  const int lane = threadIdx.x & 31;
  const int num_m_blocks = (m + BM - 1) / BM;
  const int num_n_blocks = n / BN;
  const int num_k_tiles = k / BK;
  const int64_t sf_tile_stride = static_cast<int64_t>(k / 64) * 512;  // bytes per 128-row block
  const uint64_t teardown_limit = wait_limit > kDefaultWaitLimit ? wait_limit : kDefaultWaitLimit;
  const TileSeq<kResident, kEpi != 1 && kEpi != 3> seq(num_m_blocks, num_n_blocks);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->acc_empty, kEpiWarps);
    mbar_init(&bars->teardown, 1);
    mbar_init(&bars->sfb_full, 1);
    mbar_init(&bars->sfb_free, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  // programmatic dependent launch: the next kernel may start its prologue; the roles
  // below wait for the previous kernel before they touch global memory
  if (threadIdx.x == 0) grid_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // (the whole warp runs the loop; one elected lane issues the copies)
    grid_dependency_wait();
    if (seq.count > 0) {
      bool sfb_armed = false;
      uint8_t* preload = P::kPreloadInStage ? smem + (kStages - 1) * kStageBytes : staging;
      if (kResident) {
        // the W scales of this CTA's N block, all K: two contiguous 128-row runs
        if (elect_one()) {
          mbar_arrive_expect_tx(&bars->sfb_full, static_cast<uint32_t>(2 * sf_tile_stride));
          bulk_load(preload, w_sf + (2 * seq.nb_fixed) * sf_tile_stride,
                    static_cast<uint32_t>(sf_tile_stride), &bars->sfb_full);
          bulk_load(preload + sf_tile_stride, w_sf + (2 * seq.nb_fixed + 1) * sf_tile_stride,
                    static_cast<uint32_t>(sf_tile_stride), &bars->sfb_full);
        }
        __syncwarp();
        sfb_armed = true;
      }
      uint32_t armed[kStages];
#pragma unroll
      for (int s = 0; s < kStages; ++s) armed[s] = 0;
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;  // K tiles loaded so far
      bool failed = false;
      for (int i = 0; i < seq.count && !failed && !warp_aborted(bars); ++i) {
        int mb, nb, half;
        seq.at(i, mb, nb, half);  // a half tile loads the whole W tile
        for (int kt = 0; kt < num_k_tiles; ++kt, ++issued) {
          if (P::kPreloadInStage && issued == kStages - 1 &&
              !warp_wait_bounded(&bars->sfb_free, 0, wait_limit)) {
            // the resident W scales still occupy the last stage's buffer
            warp_flag_error(bars, kErrWaitProducer);
            failed = true;
            break;
          }
          if (!warp_wait_bounded(&bars->empty[stage], phase ^ 1u, wait_limit)) {
            warp_flag_error(bars, kErrWaitProducer);
            break;
          }
          uint8_t* sa = smem + stage * kStageBytes;
          uint8_t* sb = sa + kABytes;
          uint8_t* ssfa = sb + kBBytes;
          uint64_t* full = &bars->full[stage];
          if (elect_one()) {
            mbar_arrive_expect_tx(full, kStageBytes);
            tma_load_2d(sa, &tmap_a, full, kt * BKB, mb * BM);
            tma_load_2d(sb, &tmap_b, full, kt * BKB, nb * BN);
            bulk_load(ssfa, a_sf + mb * sf_tile_stride + kt * 2048, kSfaBytes, full);
            if (kRepSfb) {
              // replicated layout: K tile kt of N block nb is 16 KB contiguous
              bulk_load(ssfa + kSfaBytes,
                        w_sf + (static_cast<int64_t>(nb) * (k / 64) + kt * 4) * (2 * 2048),
                        kSfbRepBytes, full);
            } else if (!kResident) {
              uint8_t* ssfb = ssfa + kSfaBytes;
              bulk_load(ssfb, w_sf + (2 * nb) * sf_tile_stride + kt * 2048, 2048, full);
              bulk_load(ssfb + 2048, w_sf + (2 * nb + 1) * sf_tile_stride + kt * 2048, 2048, full);
            }
          }
          __syncwarp();
          armed[stage] += 1;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // everything armed must have landed before shared memory goes away;
      // these waits keep the default limit even when a short one was requested
      for (int s = 0; s < kStages; ++s) {
        if (armed[s] > 0 &&
            !warp_wait_bounded(&bars->full[s], (armed[s] - 1) & 1u, teardown_limit)) {
          warp_flag_error(bars, kErrWaitTeardown);
        }
      }
      if (sfb_armed && !warp_wait_bounded(&bars->sfb_full, 0, teardown_limit))
        warp_flag_error(bars, kErrWaitTeardown);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // (the whole warp runs the loop; one elected lane issues the tcgen05 work,
    // always the same lane, so its commits cover its own copies and MMAs)
    if (seq.count > 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool issued_any = false;
      bool ok = true;
      const uint32_t acc = tmem;
      if (kResident) {
        if (!warp_wait_bounded(&bars->sfb_full, 0, wait_limit)) {
          warp_flag_error(bars, kErrWaitMma);
          ok = false;
        } else {
          tc_fence_after();
          const uint8_t* preload = P::kPreloadInStage ? smem + (kStages - 1) * kStageBytes : staging;
          if (elect_one()) {
            for (int s = 0; s < k / 64; ++s) {
              tmem_cp_32x128b_x4(tmem + kSfbCol + 8 * s,
                                 make_smem_desc(smem_u32(preload + 512 * s), 16, 128, 0));
              tmem_cp_32x128b_x4(tmem + kSfbCol + 8 * s + 4,
                                 make_smem_desc(smem_u32(preload + sf_tile_stride + 512 * s), 16,
                                                128, 0));
            }
            if (P::kPreloadInStage) tc_commit(&bars->sfb_free);  // the buffer may be refilled
          }
          __syncwarp();
          issued_any = true;
        }
      }
      for (int i = 0; ok && i < seq.count && !warp_aborted(bars); ++i) {
        int mb_unused, nb_unused, half;
        seq.at(i, mb_unused, nb_unused, half);
        // a half tile: N = 128 MMAs on W rows [128 * half, +128) of the stage and
        // the matching 4 of the 8 W-scale columns per K step
        const uint32_t idesc = half < 0 ? kIdesc : kIdescHalf;
        const uint32_t b_off = half > 0 ? static_cast<uint32_t>(kBBytes / 2) : 0u;
        const uint32_t sfb_off = half > 0 ? 4u : 0u;
        if (!warp_wait_bounded(&bars->acc_empty, (static_cast<uint32_t>(i) & 1u) ^ 1u,
                               wait_limit)) {
          warp_flag_error(bars, kErrWaitMma);
          break;
        }
        tc_fence_after();
        for (int kt = 0; kt < num_k_tiles; ++kt) {
          if (!warp_wait_bounded(&bars->full[stage], phase, wait_limit)) {
            warp_flag_error(bars, kErrWaitMma);
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* sa = smem + stage * kStageBytes;
          uint8_t* sb = sa + kABytes;
          uint8_t* ssfa = sb + kBBytes;
          const uint64_t adesc = make_smem_desc(smem_u32(sa), 16, 1024, 2);
          const uint64_t bdesc = make_smem_desc(smem_u32(sb) + b_off, 16, 1024, 2);
          if (elect_one()) {
            // scales: one 512-byte atom (32 rows x 16 B) per 64-deep K step
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              tmem_cp_32x128b_x4(tmem + kSfaCol + 4 * j,
                                 make_smem_desc(smem_u32(ssfa + 512 * j), 16, 128, 0));
              if (kRepSfb) {
                // row i of the 4 KB source: line i % 32 of the rows 0-127 atom
                // (first 2 KB) and of the rows 128-255 atom (LBO = 2 KB later)
                tmem_cp_128x256b(tmem + kSfbCol + 8 * j,
                                 make_smem_desc(smem_u32(ssfa + kSfaBytes + 4096 * j), 2048, 128, 0));
              } else if (!kResident) {
                uint8_t* ssfb = ssfa + kSfaBytes;
                tmem_cp_32x128b_x4(tmem + kSfbCol + 8 * j,
                                   make_smem_desc(smem_u32(ssfb + 512 * j), 16, 128, 0));
                tmem_cp_32x128b_x4(tmem + kSfbCol + 8 * j + 4,
                                   make_smem_desc(smem_u32(ssfb + 2048 + 512 * j), 16, 128, 0));
              }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t sfb = tmem + kSfbCol + 8 * (kResident ? kt * 4 + j : j) + sfb_off;
              mma_nvf4(acc, adesc + static_cast<uint64_t>(2 * j),
                       bdesc + static_cast<uint64_t>(2 * j), idesc, tmem + kSfaCol + 4 * j, sfb,
                       (kt > 0 || j > 0) ? 1u : 0u);
            }
            tc_commit(&bars->empty[stage]);
          }
          __syncwarp();
          issued_any = true;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (elect_one()) tc_commit(&bars->acc_full);
        __syncwarp();
      }
      if (warp_aborted(bars) && issued_any) {
        if (elect_one()) tc_commit(&bars->teardown);
        __syncwarp();
        if (!warp_wait_bounded(&bars->teardown, 0, teardown_limit))
          warp_flag_error(bars, kErrWaitTeardown);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Warp w reads TMEM lanes 32*(w%4).. (its quadrant) and columns
    // [64*q, 64*q+64), q = (w-2)/4.  Phase 1 pulls the accumulator slice into
    // registers, forms the mm_fp4 output bf16(alpha*acc) and frees TMEM for
    // the next tile; phase 2 adds the bias (and GELU) and stores.
    const int quad = warp & 3;
    const int quarter = (warp - 2) >> 2;
    const int col_base = quarter * 64;
    const int trow = quad * 32 + lane;
    if constexpr (P::kGelu) {
      gelu_table_init(gelu_tab, threadIdx.x - 64, kEpiThreads);
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
    }
    grid_dependency_wait();
    if (kEpi == 1 && qo.zero_word != nullptr && blockIdx.x == 0 && threadIdx.x == 64)
      *qo.zero_word = 0.0f;
    // kEpi 3: the intermediate's provisional encode scale and its loop invariants
    float gq = 0.0f, r6 = 0.0f, rgq = 0.0f;
    uint32_t qflags = 0;
    if constexpr (kEpi == 3) {
      // 2^-headroom_log2 as an exact power of two (headroom_log2 in [0, 30])
      gq = __fmul_rn(encode_scale(*qo.amax_hint), __int_as_float((127 - qo.headroom_log2) << 23));
      r6 = rcp_approx_ftz(6.0f);
      rgq = rcp_approx_ftz(gq);
      if (blockIdx.x == 0 && threadIdx.x == 64 && qo.g_used != nullptr) *qo.g_used = gq;
    }
    const uint32_t tab_base = smem_u32(gelu_tab);
    uint8_t* warp_staging = staging + (warp - 2) * kWarpStagingBytes;
    // alpha = 1 / (g_a * g_w): torch's reciprocal of the product, IEEE rounded
    const float alpha = alpha_in != nullptr ? *alpha_in : __frcp_rn(__fmul_rn(*g_a, *g_w));
    uint64_t alpha2;
    asm("mov.b64 %0, {%1, %1};" : "=l"(alpha2) : "f"(alpha));
    uint32_t amax2 = 0;  // max |h| of the low and high columns, bf16 magnitude bits
    for (int i = 0; i < seq.count; ++i) {
      if (!mbar_wait_bounded(&bars->acc_full, static_cast<uint32_t>(i) & 1u, wait_limit)) {
        flag_error(bars, kErrWaitEpilogue);
        break;
      }
      tc_fence_after();
      int mb, nb, half;
      seq.at(i, mb, nb, half);
      if (half >= 0 && quarter >= 2) {
        // a half tile has 128 accumulator columns: this warp's 64 are not part of it
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->acc_empty);
        continue;
      }
      uint32_t r[64];
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quad * 32) << 16) + col_base;
      tmem_ld_32x32b_x32(taddr + 0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
      tmem_ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_empty);
      // mm_fp4's output: bf16(alpha * acc), packed in pairs
      uint32_t y[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) y[j] = scale_pack_bf16x2(r[2 * j], r[2 * j + 1], alpha2);
      const int col0 = nb * BN + (half > 0 ? BN / 2 : 0) + col_base;
      if constexpr (kEpi == 3) {
        // GEMM1 quantizing its output: bias and GELU as kEpi 1, then each of the row's
        // four 16-column blocks is quantized with the provisional encode scale exactly as
        // the activation quantizer does it (quantize_block16); the 32 code bytes and the
        // four scale bytes (one 32-bit word of the 128x4 layout) are stored directly.
        const int row = mb * BM + trow;
        const bool real = row < m;
        const uint4* bias4 = reinterpret_cast<const uint4*>(bias + col0);
        uint32_t tile_max = 0, s8w = 0;
        uint32_t cw[8];
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) {
          uint32_t hw[8];
#pragma unroll
          for (int hq = 0; hq < 2; ++hq) {
            const int q = 2 * blk + hq;
            uint4 bv = make_uint4(0, 0, 0, 0);
            if (bias != nullptr) bv = __ldg(bias4 + q);
            const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              o[j] = y[4 * q + j];
              if (bias != nullptr) o[j] = add_bf16x2(o[j], bw[j]);
            }
            gelu_bf16x2_x4(o, tab_base, gelu_tab);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              tile_max = max_u16x2(tile_max, o[j] & 0x7FFF7FFFu);
              hw[4 * hq + j] = o[j];
            }
          }
          float sfval;
          uint32_t vbits;
          const uint32_t s8 = quantize_block16(hw, gq, r6, rgq, cw[2 * blk], cw[2 * blk + 1], &sfval,
                                               &vbits);
          s8w |= s8 << (8 * blk);
          if (real) {
            if (sfval > 448.0f) qflags |= kQuantSaturated;
            if (vbits >= 0x0080u && s8 == 0) qflags |= kQuantUnderflow;
          }
        }
        if (real) {
          amax2 = max_u16x2(amax2, tile_max);
          uint4* dst = reinterpret_cast<uint4*>(qo.codes + static_cast<int64_t>(row) * (n / 2) + col0 / 2);
          dst[0] = make_uint4(cw[0], cw[1], cw[2], cw[3]);
          dst[1] = make_uint4(cw[4], cw[5], cw[6], cw[7]);
        }
        // rows past m inside the last 128-row block get zero scales, as the quantizer's do
        const int64_t off = static_cast<int64_t>(row >> 7) * ((n / 64) * 512) + (col0 >> 6) * 512 +
                            (row & 31) * 16 + ((row & 127) >> 5) * 4;
        *reinterpret_cast<uint32_t*>(qo.sf + off) = real ? s8w : 0u;
      } else if constexpr (P::kStaged) {
        // GEMM1: bias, GELU and the amax on this thread's row, then the warp's
        // 32 x 64 block goes out in one tensor store from 128B-swizzled staging
        // (chunk c of row r at r*128 + ((c ^ (r & 7)) * 16), the tensor map's
        // swizzle), which clips rows past m.
        if (lane == 0) bulk_wait_group_read0();  // previous store has read the staging
        __syncwarp();
        const uint4* bias4 = reinterpret_cast<const uint4*>(bias + col0);
        uint32_t tile_max = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          uint4 bv = make_uint4(0, 0, 0, 0);
          if (bias != nullptr) bv = __ldg(bias4 + q);
          const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
          uint32_t o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            o[j] = y[4 * q + j];
            if (bias != nullptr) o[j] = add_bf16x2(o[j], bw[j]);
          }
          gelu_bf16x2_x4(o, tab_base, gelu_tab);
#pragma unroll
          for (int j = 0; j < 4; ++j) tile_max = max_u16x2(tile_max, o[j] & 0x7FFF7FFFu);
          *reinterpret_cast<uint4*>(warp_staging + lane * kStageRowBytes + ((q ^ (lane & 7)) * 16)) =
              make_uint4(o[0], o[1], o[2], o[3]);
        }
        if (mb * BM + trow < m) amax2 = max_u16x2(amax2, tile_max);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmap_out, warp_staging, col0, mb * BM + quad * 32);
          bulk_commit_group();
        }
      } else {
        const int row = mb * BM + trow;
        uint16_t* dst = out + static_cast<int64_t>(row) * n + col0;
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
          uint4 bv = make_uint4(0, 0, 0, 0);
          if (bias != nullptr) bv = __ldg(reinterpret_cast<const uint4*>(bias + col0 + c));
          const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
          uint32_t o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t w = y[c / 2 + j];
            if (bias != nullptr) w = add_bf16x2(w, bw[j]);
            o[j] = w;
          }
          if constexpr (kEpi == 2) {
            // gated residual: out = bf16(x + bf16(gate * y)), each a single bf16 rounding
            const uint4 gv = __ldg(reinterpret_cast<const uint4*>(gate + col0 + c));
            uint4 xv = make_uint4(0, 0, 0, 0);
            if (row < m)
              xv = __ldg(reinterpret_cast<const uint4*>(residual + static_cast<int64_t>(row) * n +
                                                        col0 + c));
            const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) o[j] = add_bf16x2(xw[j], mul_bf16x2(gw[j], o[j]));
          }
          if (row < m) {
            *reinterpret_cast<uint4*>(dst + c) = make_uint4(o[0], o[1], o[2], o[3]);
#pragma unroll
            for (int j = 0; j < 4; ++j) amax2 = bmax2(amax2, o[j] & 0x7FFF7FFFu);
          }
        }
      }
    }
    if ((kEpi == 0 || kEpi == 2) && amax_out != nullptr) {
      // max |out| (NaN ignored, as the amax kernel takes it), for the next layer's quantizer
      const uint32_t mag = max(amax2 & 0xFFFFu, amax2 >> 16);
      const uint32_t bits = __reduce_max_sync(0xFFFFFFFFu, mag << 16);
      if (lane == 0 && bits != 0) atomicMax(reinterpret_cast<unsigned int*>(amax_out), bits);
    }
    if (kEpi == 1 || kEpi == 3) {
      // the tensor stores must be complete before the CTA exits
      if (kEpi == 1 && lane == 0) bulk_wait_group0();
      const uint32_t mag = max(amax2 & 0xFFFFu, amax2 >> 16);
      const uint32_t bits = __reduce_max_sync(0xFFFFFFFFu, mag << 16);
      if (lane == 0 && bits != 0) atomicMax(reinterpret_cast<unsigned int*>(amax_out), bits);
      if (kEpi == 3) {
        const uint32_t f = __reduce_or_sync(0xFFFFFFFFu, qflags);
        if (lane == 0 && f != 0 && qo.flags != nullptr) atomicOr(qo.flags, f);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// ---------------------------------------------------------------- SM-pair GEMM
// nvfp4_gemm_pair_kernel: the FVQ_EPI_BF16 GEMM on clusters of two CTAs (the
// two SMs of a pair) and tcgen05.mma.cta_group::2: a 256 x 256 output tile per
// pair.  Each CTA loads its 128 rows of A, 128 of the tile's 256 W rows, its A
// scales and the W scales of all 256 rows (kRawSfb: the library layout, 4 KB
// per K tile, moved to TMEM with two 32x128b.warpx4 copies per K step;
// otherwise replicated four times, 16 KB, one 128x256b copy per K step).  The
// even CTA issues the scale copies and MMAs for both (one copy instruction
// fills both SMs' TMEM) and commits "stage free" and "accumulator full" to both
// CTAs' barriers; both epilogues report a drained accumulator to the even
// CTA.  All loads of both CTAs (codes, and the scales through 3-D tensor maps
// over their 512-byte atoms) count their bytes on the even CTA's stage
// barrier, which only the even CTA arms, so the MMA issuer needs no message
// from the odd CTA.  Rows per pair tile: 256, so the host uses it for
// m % 256 == 0.  The L2-to-SM traffic per K tile and CTA (38 KB with raw
// scales, 50 KB replicated) is what bounds this kernel.
constexpr int kPairBBytes = kBBytes / 2;  // 128 W rows per CTA
constexpr int kPairMaxStages = 6;

template <bool kRawSfb>
struct PairPlan {
  static constexpr int kStageBytes =
      kABytes + kPairBBytes + kSfaBytes + (kRawSfb ? kSfbBytes : kSfbRepBytes);  // 38 / 50 KB
  static constexpr int kStages = kRawSfb ? 5 : 4;
  static constexpr int kBarrierOff = kStages * kStageBytes;
  static constexpr int kSmemBytes = kBarrierOff + kBarrierBytes;
};
static_assert(PairPlan<true>::kSmemBytes <= 232448, "pair plan exceeds shared memory");
static_assert(PairPlan<false>::kSmemBytes <= 232448, "pair plan exceeds shared memory");
static_assert(PairPlan<true>::kStages <= kPairMaxStages && PairPlan<false>::kStages <= kPairMaxStages,
              "pair barrier arrays");
constexpr uint32_t kIdescPair = (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
                                (static_cast<uint32_t>(2 * BM >> 4) << 24);
// N = 128 pair tile (a 256 x 128 half of a tile, see PairSeq): 64 W rows per CTA
constexpr uint32_t kIdescPairHalf = (1u << 7) | (1u << 10) |
                                    (static_cast<uint32_t>(BN / 2 >> 3) << 17) |
                                    (static_cast<uint32_t>(2 * BM >> 4) << 24);
constexpr int kPairQuarterBBytes = kPairBBytes / 2;  // 64 W rows per CTA

// Tiles of one SM pair: tile t = pair + i * pairs, N block fastest, so that the pairs
// working at one time share few 256-row blocks of A (each is read from HBM once and then
// from L2 by the N blocks' pairs; with M fastest, an A larger than L2 -- H codes at 15360
// rows are 69 MB -- went to HBM once per N block).  When the tiles past the last full
// round number at most half the pairs, each of them is split into two 256 x 128 halves,
// one per pair, so that the last round takes about half as long (`half` is -1 for a
// whole tile, else 0 or 1).  Both CTAs of a pair compute the same sequence.
struct PairSeq {
  int count, full_rounds, num_n_blocks;
  bool split;
  __device__ PairSeq(int tiles, int n_blocks) : num_n_blocks(n_blocks) {
    const int pairs = gridDim.x / 2, pair = blockIdx.x / 2;
    count = pair < tiles ? (tiles - 1 - pair) / pairs + 1 : 0;
    const int rounds = tiles / pairs, rest = tiles - rounds * pairs;
    split = rest > 0 && 2 * rest <= pairs;
    full_rounds = rounds;
    if (split) count = rounds + (pair < 2 * rest ? 1 : 0);
  }
  __device__ void at(int i, int& mbp, int& nb, int& half) const {
    const int pairs = gridDim.x / 2, pair = blockIdx.x / 2;
    int t = pair + i * pairs;
    half = -1;
    if (split && i == full_rounds) {
      t = full_rounds * pairs + (pair >> 1);
      half = pair & 1;
    }
    nb = t % num_n_blocks;
    mbp = t / num_n_blocks;
  }
};

struct PairBarriers {
  uint64_t full[kPairMaxStages];    // even CTA: both CTAs' stage landed
  uint64_t empty[kPairMaxStages];   // the pair's MMAs on the stage completed
  uint64_t acc_full;                // the pair's accumulator is complete
  uint64_t acc_empty;               // even CTA: both epilogues drained their TMEM
  uint64_t teardown;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(PairBarriers) <= kBarrierBytes, "pair barrier area");

// kEpi 0: bf16(alpha*acc) + bias; kEpi 2 adds the gated residual of the DiT
// block, out = bf16(residual + bf16(gate * y)), as the one-SM kernel does.
template <int kEpi, bool kRawSfb>
__global__ void __launch_bounds__(kNumThreads, 1)
    nvfp4_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                           const __grid_constant__ CUtensorMap tmap_b_half,
                           const __grid_constant__ CUtensorMap tmap_b_quarter,
                           const __grid_constant__ CUtensorMap tmap_sfa,
                           const __grid_constant__ CUtensorMap tmap_sfb,
                           const float* __restrict__ g_a, const float* __restrict__ g_w,
                           const uint16_t* __restrict__ bias, uint16_t* __restrict__ out, int m,
                           int n, int k, uint64_t wait_limit, const uint16_t* __restrict__ residual,
                           const uint16_t* __restrict__ gate, float* amax_out) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicOr(&g_device_error, kErrSmemAlign);
    return;  // both CTAs see the same layout, so both return here
  }
  using P = PairPlan<kRawSfb>;
  constexpr int kPairStages = P::kStages;
  constexpr int kPairStageBytes = P::kStageBytes;
  auto* bars = reinterpret_cast<PairBarriers*>(smem + P::kBarrierOff);
  const int warp = warp_index_uniform();
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool even = rank == 0;
  // ragged m: the last pair tile may hold fewer than 256 rows; a CTA whose 128 rows lie
  // wholly past m loads the last valid row block instead (so every TMA box starts inside
  // A) and stores nothing
  const int num_m_pairs = (m + 2 * BM - 1) / (2 * BM);
  const int num_m_blocks = (m + BM - 1) / BM;
  const int num_n_blocks = n / BN;
  const PairSeq seq(num_m_pairs * num_n_blocks, num_n_blocks);  // same in both CTAs
  const int count = seq.count;
  const int num_k_tiles = k / BK;
  const uint64_t teardown_limit = wait_limit > kDefaultWaitLimit ? wait_limit : kDefaultWaitLimit;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->acc_empty, 2 * kEpiWarps);
    mbar_init(&bars->teardown, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b_half);
    prefetch_tmap(&tmap_b_quarter);
    prefetch_tmap(&tmap_sfa);
    prefetch_tmap(&tmap_sfb);
  }
  if (warp == 1) {
    tmem_alloc_pair(&bars->tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const auto even_addr = [&](const void* p) { return mapa_shared(smem_u32(p), 0); };
  const auto odd_addr = [&](const void* p) { return mapa_shared(smem_u32(p), 1); };
  if (threadIdx.x == 0) grid_launch_dependents();  // as in nvfp4_gemm_kernel

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    // (the whole warp runs the loop; one elected lane issues the copies)
    grid_dependency_wait();
    if (count > 0) {
      uint32_t armed[kPairStages];
#pragma unroll
      for (int s = 0; s < kPairStages; ++s) armed[s] = 0;
      int stage = 0;
      uint32_t phase = 0;
      for (int i = 0; i < count && !warp_aborted(bars); ++i) {
        int mbp, nb, half;
        seq.at(i, mbp, nb, half);
        const int a_block = min(2 * mbp + static_cast<int>(rank), num_m_blocks - 1);  // its rows
        // a half tile: this CTA's 64 of the half's 128 W rows, the same A and scale loads
        const uint32_t stage_tx =
            2u * static_cast<uint32_t>(half < 0 ? kPairStageBytes : kPairStageBytes - kPairQuarterBBytes);
        for (int kt = 0; kt < num_k_tiles; ++kt) {
          if (!warp_wait_cluster_bounded(&bars->empty[stage], phase ^ 1u, wait_limit)) {
            warp_flag_error(bars, kErrWaitProducer);
            break;
          }
          uint8_t* sa = smem + stage * kPairStageBytes;
          uint8_t* sb = sa + kABytes;
          uint8_t* ssfa = sb + kPairBBytes;
          uint8_t* ssfb = ssfa + kSfaBytes;
          const uint32_t bar = even_addr(&bars->full[stage]);
          if (elect_one()) {
            if (even) mbar_arrive_expect_tx(&bars->full[stage], stage_tx);
            tma_load_2d_pair(sa, &tmap_a, bar, kt * BKB, a_block * BM);
            if (half < 0)
              tma_load_2d_pair(sb, &tmap_b_half, bar, kt * BKB,
                               nb * BN + static_cast<int>(rank) * (BN / 2));
            else
              tma_load_2d_pair(sb, &tmap_b_quarter, bar, kt * BKB,
                               nb * BN + half * (BN / 2) + static_cast<int>(rank) * (BN / 4));
            // A scales: atoms 4kt..4kt+3 of 128-row block a_block; W scales: the
            // same atoms of 128-row blocks 2nb and 2nb+1 (raw), or the 32
            // replicated atoms of K steps 4kt..4kt+3 of N block nb
            tma_load_3d_pair(ssfa, &tmap_sfa, bar, 0, kt * 4, a_block);
            if (kRawSfb)
              tma_load_3d_pair(ssfb, &tmap_sfb, bar, 0, kt * 4, 2 * nb);
            else
              tma_load_3d_pair(ssfb, &tmap_sfb, bar, 0, 0, nb * (k / 64) + kt * 4);
          }
          __syncwarp();
          armed[stage] += 1;
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // the even CTA's stage barriers count both CTAs' loads; the odd CTA's land
      // before the even CTA's MMAs consume the stage, which the final cluster
      // barrier waits for
      for (int s = 0; even && s < kPairStages; ++s) {
        if (armed[s] > 0 &&
            !warp_wait_cluster_bounded(&bars->full[s], (armed[s] - 1) & 1u, teardown_limit))
          warp_flag_error(bars, kErrWaitTeardown);
      }
    }
  } else if (warp == 1) {
    if (count > 0 && even) {
      // ---------------------------------------------------------- MMA issuer (even CTA)
      // (the whole warp runs the loop; the same elected lane issues everything)
      int stage = 0;
      uint32_t phase = 0;
      bool issued_any = false;
      bool ok = true;
      for (int i = 0; ok && i < count && !warp_aborted(bars); ++i) {
        int mbp_unused, nb_unused, half;
        seq.at(i, mbp_unused, nb_unused, half);
        // a half tile: N = 128 MMAs on the first 64 W rows of each CTA's stage and the
        // half's 4 of the 8 W-scale columns per K step
        const uint32_t idesc = half < 0 ? kIdescPair : kIdescPairHalf;
        const uint32_t sfb_off = half > 0 ? 4u : 0u;
        if (!warp_wait_cluster_bounded(&bars->acc_empty, (static_cast<uint32_t>(i) & 1u) ^ 1u,
                                       wait_limit)) {
          warp_flag_error(bars, kErrWaitMma);
          break;
        }
        tc_fence_after();
        for (int kt = 0; kt < num_k_tiles; ++kt) {
          if (!warp_wait_cluster_bounded(&bars->full[stage], phase, wait_limit)) {
            warp_flag_error(bars, kErrWaitMma);
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* sa = smem + stage * kPairStageBytes;
          uint8_t* sb = sa + kABytes;
          uint8_t* ssfa = sb + kPairBBytes;
          uint8_t* ssfb = ssfa + kSfaBytes;
          const uint64_t adesc = make_smem_desc(smem_u32(sa), 16, 1024, 2);
          const uint64_t bdesc = make_smem_desc(smem_u32(sb), 16, 1024, 2);
          const uint32_t empty_odd = odd_addr(&bars->empty[stage]);
          if (elect_one()) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              tmem_cp_32x128b_x4_pair(tmem + kSfaCol + 4 * j,
                                      make_smem_desc(smem_u32(ssfa + 512 * j), 16, 128, 0));
              if (kRawSfb) {
                tmem_cp_32x128b_x4_pair(tmem + kSfbCol + 8 * j,
                                        make_smem_desc(smem_u32(ssfb + 512 * j), 16, 128, 0));
                tmem_cp_32x128b_x4_pair(tmem + kSfbCol + 8 * j + 4,
                                        make_smem_desc(smem_u32(ssfb + 2048 + 512 * j), 16, 128, 0));
              } else {
                tmem_cp_128x256b_pair(tmem + kSfbCol + 8 * j,
                                      make_smem_desc(smem_u32(ssfb + 4096 * j), 2048, 128, 0));
              }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              mma_nvf4_pair(tmem, adesc + static_cast<uint64_t>(2 * j),
                            bdesc + static_cast<uint64_t>(2 * j), idesc, tmem + kSfaCol + 4 * j,
                            tmem + kSfbCol + 8 * j + sfb_off, (kt > 0 || j > 0) ? 1u : 0u);
            }
            tc_commit_pair(smem_u32(&bars->empty[stage]));
            tc_commit_pair(empty_odd);
          }
          __syncwarp();
          issued_any = true;
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        const uint32_t acc_odd = odd_addr(&bars->acc_full);
        if (elect_one()) {
          tc_commit_pair(smem_u32(&bars->acc_full));
          tc_commit_pair(acc_odd);
        }
        __syncwarp();
      }
      if (warp_aborted(bars) && issued_any) {
        if (elect_one()) tc_commit_pair(smem_u32(&bars->teardown));
        __syncwarp();
        if (!warp_wait_bounded(&bars->teardown, 0, teardown_limit))
          warp_flag_error(bars, kErrWaitTeardown);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quad = warp & 3;
    const int quarter = (warp - 2) >> 2;
    const int col_base = quarter * 64;
    const int trow = quad * 32 + lane;
    grid_dependency_wait();
    const float alpha = __frcp_rn(__fmul_rn(*g_a, *g_w));
    uint64_t alpha2;
    asm("mov.b64 %0, {%1, %1};" : "=l"(alpha2) : "f"(alpha));
    const uint32_t acc_empty_addr = even_addr(&bars->acc_empty);
    uint32_t amax2 = 0;  // max |out| of the low and high columns (amax_out)
    for (int i = 0; i < count; ++i) {
      if (!mbar_wait_cluster_bounded(&bars->acc_full, static_cast<uint32_t>(i) & 1u, wait_limit)) {
        flag_error(bars, kErrWaitEpilogue);
        break;
      }
      tc_fence_after();
      int mbp, nb, half;
      seq.at(i, mbp, nb, half);
      if (half >= 0 && quarter >= 2) {
        // a half tile has 128 accumulator columns: this warp's 64 are not part of it
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acc_empty_addr);
        continue;
      }
      uint32_t r[64];
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quad * 32) << 16) + col_base;
      tmem_ld_32x32b_x32(taddr + 0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
      tmem_ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_addr);
      uint32_t y[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) y[j] = scale_pack_bf16x2(r[2 * j], r[2 * j + 1], alpha2);
      const int col0 = nb * BN + (half > 0 ? BN / 2 : 0) + col_base;
      const int row = mbp * 2 * BM + static_cast<int>(rank) * BM + trow;
      uint16_t* dst = out + static_cast<int64_t>(row) * n + col0;
#pragma unroll
      for (int c = 0; c < 64; c += 8) {
        uint4 bv = make_uint4(0, 0, 0, 0);
        if (bias != nullptr) bv = __ldg(reinterpret_cast<const uint4*>(bias + col0 + c));
        const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t w = y[c / 2 + j];
          if (bias != nullptr) w = add_bf16x2(w, bw[j]);
          o[j] = w;
        }
        if constexpr (kEpi == 2) {
          // gated residual: out = bf16(x + bf16(gate * y)), each a single bf16 rounding
          const uint4 gv = __ldg(reinterpret_cast<const uint4*>(gate + col0 + c));
          uint4 xv = make_uint4(0, 0, 0, 0);
          if (row < m)
            xv = __ldg(reinterpret_cast<const uint4*>(residual + static_cast<int64_t>(row) * n +
                                                      col0 + c));
          const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) o[j] = add_bf16x2(xw[j], mul_bf16x2(gw[j], o[j]));
        }
        if (row < m) {
          *reinterpret_cast<uint4*>(dst + c) = make_uint4(o[0], o[1], o[2], o[3]);
#pragma unroll
          for (int j = 0; j < 4; ++j) amax2 = bmax2(amax2, o[j] & 0x7FFF7FFFu);
        }
      }
    }
    if (amax_out != nullptr) {
      // max |out| (NaN ignored, as the amax kernel takes it), for the next layer's quantizer
      const uint32_t mag = max(amax2 & 0xFFFFu, amax2 >> 16);
      const uint32_t bits = __reduce_max_sync(0xFFFFFFFFu, mag << 16);
      if (lane == 0 && bits != 0) atomicMax(reinterpret_cast<unsigned int*>(amax_out), bits);
    }
  }

  tc_fence_before();
  cluster_sync();  // neither CTA leaves while the pair's MMAs or arrivals may touch it
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, kTmemCols);
}

// ---------------------------------------------------------------- FP8 GEMM
// fp8_gemm_kernel: E4M3 x E4M3 with fp32 accumulation (tcgen05.mma.kind::f8f6f4,
// K = 32 per MMA) and the row-wise scales of torch._scaled_mm (reference
// ffn_quantization.py:58-60), followed by the bias add of :68-69:
//   y[m, n] = bf16((acc[m, n] * sa[m]) * sw[n]),  then bf16(y + bias[n])
// kEpi 1 (the FFN's first linear) also applies GELU-tanh and records each
// row's max |h| (atomic max of its fp32 bits into row_amax[m]) for the per-row
// quantizer of the second linear.  CTA layout as in the NVFP4 kernel (warp 0
// TMA producer, warp 1 TMEM owner and MMA issuer, warps 2-17 epilogue); a
// stage holds the two code tiles of one 128-deep K tile and nothing else: the
// scales are per row and per column, applied in the epilogue.
constexpr int kF8BK = 128;                            // K elements (= bytes) per stage
constexpr uint32_t kF8TmemCols = 256;                 // the fp32 accumulator only
template <int kEpi>
struct F8Plan {
  static constexpr int kStageBytes = kABytes + kBBytes;  // 48 KB
  static constexpr int kStages = 3;
  static constexpr int kStagingOff = kStages * kStageBytes;
  static constexpr int kTableOff = kStagingOff + kStagingBytes;
  static constexpr int kBarrierOff = kTableOff + (kEpi == 1 ? kGeluTabBytes : 0);
  static constexpr int kSmemBytes = kBarrierOff + kBarrierBytes;
};
static_assert(F8Plan<0>::kSmemBytes <= 232448, "FP8 GEMM plan exceeds shared memory");
static_assert(F8Plan<1>::kSmemBytes <= 232448, "FP8 GEMM1 plan exceeds shared memory");
static_assert(kF8BK == BKB, "an FP8 K tile spans the same 128 bytes per row as an FP4 one");

// Instruction descriptor, kind::f8f6f4: fp32 accumulator (1 at bit 4), A and B
// E4M3 (format 0 at bits 7 and 10), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kIdescF8 = (1u << 4) | (static_cast<uint32_t>(BN >> 3) << 17) |
                              (static_cast<uint32_t>(BM >> 4) << 24);
constexpr uint32_t kIdescF8Half = (1u << 4) | (static_cast<uint32_t>(BN / 2 >> 3) << 17) |
                                  (static_cast<uint32_t>(BM >> 4) << 24);

// (lo, hi) * (sa, sa) * (sw_lo, sw_hi), two IEEE products per value (mul.rn.f32x2),
// rounded to a bf16x2 pair.
__device__ __forceinline__ uint32_t rowcol_scale_pack_bf16x2(uint32_t lo_bits, uint32_t hi_bits,
                                                             uint64_t sa2, float sw_lo,
                                                             float sw_hi) {
  uint64_t v, p, w, q;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "r"(lo_bits), "r"(hi_bits));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(p) : "l"(v), "l"(sa2));
  asm("mov.b64 %0, {%1, %2};" : "=l"(w) : "f"(sw_lo), "f"(sw_hi));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(q) : "l"(p), "l"(w));
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(q));
  return pack_bf16x2(lo, hi);
}

template <int kEpi>
__global__ void __launch_bounds__(kNumThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_b,
                    const __grid_constant__ CUtensorMap tmap_out, const float* __restrict__ sa_rows,
                    const float* __restrict__ sw_cols, const uint16_t* __restrict__ bias,
                    uint16_t* __restrict__ out, int m, int n, int k, uint32_t* row_amax,
                    uint64_t wait_limit) {
  using P = F8Plan<kEpi>;
  constexpr int kStages = P::kStages;
  constexpr int kStageBytes = P::kStageBytes;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicOr(&g_device_error, kErrSmemAlign);
    return;
  }
  auto* bars = reinterpret_cast<Barriers<kStages>*>(smem + P::kBarrierOff);
  uint8_t* staging = smem + P::kStagingOff;
  uint16_t* gelu_tab = reinterpret_cast<uint16_t*>(smem + P::kTableOff);

  const int warp = warp_index_uniform();
  const int lane = threadIdx.x & 31;
  const int num_m_blocks = (m + BM - 1) / BM;
  const int num_n_blocks = n / BN;
  const int num_k_tiles = k / kF8BK;
  const uint64_t teardown_limit = wait_limit > kDefaultWaitLimit ? wait_limit : kDefaultWaitLimit;
  const TileSeq<false, true> seq(num_m_blocks, num_n_blocks);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->acc_empty, kEpiWarps);
    mbar_init(&bars->teardown, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kF8TmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // (the whole warp runs the loop; one elected lane issues the copies)
    if (seq.count > 0) {
      uint32_t armed[kStages];
#pragma unroll
      for (int s = 0; s < kStages; ++s) armed[s] = 0;
      int stage = 0;
      uint32_t phase = 0;
      for (int i = 0; i < seq.count && !warp_aborted(bars); ++i) {
        int mb, nb, half;
        seq.at(i, mb, nb, half);  // a half tile loads the whole W tile
        for (int kt = 0; kt < num_k_tiles; ++kt) {
          if (!warp_wait_bounded(&bars->empty[stage], phase ^ 1u, wait_limit)) {
            warp_flag_error(bars, kErrWaitProducer);
            break;
          }
          uint8_t* sa = smem + stage * kStageBytes;
          uint8_t* sb = sa + kABytes;
          uint64_t* full = &bars->full[stage];
          if (elect_one()) {
            mbar_arrive_expect_tx(full, kStageBytes);
            tma_load_2d(sa, &tmap_a, full, kt * kF8BK, mb * BM);
            tma_load_2d(sb, &tmap_b, full, kt * kF8BK, nb * BN);
          }
          __syncwarp();
          armed[stage] += 1;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      for (int s = 0; s < kStages; ++s) {
        if (armed[s] > 0 &&
            !warp_wait_bounded(&bars->full[s], (armed[s] - 1) & 1u, teardown_limit)) {
          warp_flag_error(bars, kErrWaitTeardown);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // (the whole warp runs the loop; the same elected lane issues everything)
    if (seq.count > 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool issued_any = false;
      bool ok = true;
      for (int i = 0; ok && i < seq.count && !warp_aborted(bars); ++i) {
        int mb_unused, nb_unused, half;
        seq.at(i, mb_unused, nb_unused, half);
        const uint32_t idesc = half < 0 ? kIdescF8 : kIdescF8Half;
        const uint32_t b_off = half > 0 ? static_cast<uint32_t>(kBBytes / 2) : 0u;
        if (!warp_wait_bounded(&bars->acc_empty, (static_cast<uint32_t>(i) & 1u) ^ 1u,
                               wait_limit)) {
          warp_flag_error(bars, kErrWaitMma);
          break;
        }
        tc_fence_after();
        for (int kt = 0; kt < num_k_tiles; ++kt) {
          if (!warp_wait_bounded(&bars->full[stage], phase, wait_limit)) {
            warp_flag_error(bars, kErrWaitMma);
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* sa = smem + stage * kStageBytes;
          uint8_t* sb = sa + kABytes;
          const uint64_t adesc = make_smem_desc(smem_u32(sa), 16, 1024, 2);
          const uint64_t bdesc = make_smem_desc(smem_u32(sb) + b_off, 16, 1024, 2);
          if (elect_one()) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {  // 32-byte K steps inside the 128B swizzle atom
              mma_f8(tmem, adesc + static_cast<uint64_t>(2 * j),
                     bdesc + static_cast<uint64_t>(2 * j), idesc, (kt > 0 || j > 0) ? 1u : 0u);
            }
            tc_commit(&bars->empty[stage]);
          }
          __syncwarp();
          issued_any = true;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (elect_one()) tc_commit(&bars->acc_full);
        __syncwarp();
      }
      if (warp_aborted(bars) && issued_any) {
        if (elect_one()) tc_commit(&bars->teardown);
        __syncwarp();
        if (!warp_wait_bounded(&bars->teardown, 0, teardown_limit))
          warp_flag_error(bars, kErrWaitTeardown);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Warp w: TMEM lanes 32*(w%4).. and columns [64*q, 64*q+64), q = (w-2)/4,
    // as in the NVFP4 kernel.  The accumulator slice is pulled into registers
    // and TMEM released before any scaling, so the next tile's MMAs overlap it.
    const int quad = warp & 3;
    const int quarter = (warp - 2) >> 2;
    const int col_base = quarter * 64;
    const int trow = quad * 32 + lane;
    if constexpr (kEpi == 1) {
      gelu_table_init(gelu_tab, threadIdx.x - 64, kEpiThreads);
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
    }
    const uint32_t tab_base = smem_u32(gelu_tab);
    uint8_t* warp_staging = staging + (warp - 2) * kWarpStagingBytes;
    for (int i = 0; i < seq.count; ++i) {
      int mb, nb, half;
      seq.at(i, mb, nb, half);
      const int row = mb * BM + trow;
      const float sa = row < m ? __ldg(sa_rows + row) : 0.0f;
      if (!mbar_wait_bounded(&bars->acc_full, static_cast<uint32_t>(i) & 1u, wait_limit)) {
        flag_error(bars, kErrWaitEpilogue);
        break;
      }
      tc_fence_after();
      if (half >= 0 && quarter >= 2) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->acc_empty);
        continue;
      }
      uint32_t r[64];
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quad * 32) << 16) + col_base;
      tmem_ld_32x32b_x32(taddr + 0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
      tmem_ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_empty);
      uint64_t sa2;
      asm("mov.b64 %0, {%1, %1};" : "=l"(sa2) : "f"(sa));
      const int col0 = nb * BN + (half > 0 ? BN / 2 : 0) + col_base;
      const float4* sw4 = reinterpret_cast<const float4*>(sw_cols + col0);
      if (lane == 0) bulk_wait_group_read0();  // previous store has read the staging
      __syncwarp();
      const uint4* bias4 = reinterpret_cast<const uint4*>(bias + col0);
      uint32_t tile_max = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 s0 = __ldg(sw4 + 2 * q), s1 = __ldg(sw4 + 2 * q + 1);
        const float sw[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
        uint4 bv = make_uint4(0, 0, 0, 0);
        if (bias != nullptr) bv = __ldg(bias4 + q);
        const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          o[j] = rowcol_scale_pack_bf16x2(r[8 * q + 2 * j], r[8 * q + 2 * j + 1], sa2, sw[2 * j],
                                          sw[2 * j + 1]);
          if (bias != nullptr) o[j] = add_bf16x2(o[j], bw[j]);
        }
        if constexpr (kEpi == 1) {
          gelu_bf16x2_x4(o, tab_base, gelu_tab);
#pragma unroll
          for (int j = 0; j < 4; ++j) tile_max = max_u16x2(tile_max, o[j] & 0x7FFF7FFFu);
        }
        // 128B-swizzled staging (chunk c of row r at r*128 + ((c ^ (r & 7)) * 16)),
        // the output tensor map's swizzle
        *reinterpret_cast<uint4*>(warp_staging + lane * kStageRowBytes + ((q ^ (lane & 7)) * 16)) =
            make_uint4(o[0], o[1], o[2], o[3]);
      }
      if constexpr (kEpi == 1) {
        const uint32_t mag = max(tile_max & 0xFFFFu, tile_max >> 16);
        if (row < m && mag != 0) atomicMax(row_amax + row, mag << 16);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && mb * BM + quad * 32 < m) {
        tma_store_2d(&tmap_out, warp_staging, col0, mb * BM + quad * 32);
        bulk_commit_group();
      }
    }
    if (lane == 0) bulk_wait_group0();  // stores complete before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kF8TmemCols);
}

// ---------------------------------------------------------------- FP8 SM-pair GEMM
// fp8_gemm_pair_kernel: fp8_gemm_kernel on clusters of two CTAs (the two SMs
// of a pair) with tcgen05.mma.cta_group::2, M = 256 across the pair: one
// 256 x 256 output tile per pair.  Per 128-deep K tile each CTA loads its 128
// rows of A and 128 of the tile's 256 W rows (32 KB per SM instead of 48 KB:
// each W tile crosses from L2 once per pair), all counted on the even CTA's
// stage barrier, which only the even CTA arms.  The even CTA issues the MMAs
// and commits "stage free" and "accumulator full" to both CTAs' barriers;
// both CTAs run the epilogue on their own 128 accumulator rows and report a
// drained accumulator to the even CTA.  Rows past m (a last pair tile over
// the end of A) load as zeros and are not stored.
constexpr int kF8PairStageBytes = kABytes + kBBytes / 2;  // 32 KB
template <int kEpi>
struct F8PairPlan {
  static constexpr int kStages = kEpi == 0 ? 5 : 4;  // next to 64 KB of staging (+ GELU table)
  static constexpr int kStagingOff = kStages * kF8PairStageBytes;
  static constexpr int kTableOff = kStagingOff + kStagingBytes;
  static constexpr int kBarrierOff = kTableOff + (kEpi == 1 ? kGeluTabBytes : 0);
  static constexpr int kSmemBytes = kBarrierOff + kBarrierBytes;
};
static_assert(F8PairPlan<0>::kSmemBytes <= 232448, "FP8 pair plan exceeds shared memory");
static_assert(F8PairPlan<1>::kSmemBytes <= 232448, "FP8 pair GEMM1 plan exceeds shared memory");
constexpr uint32_t kIdescF8Pair = (1u << 4) | (static_cast<uint32_t>(BN >> 3) << 17) |
                                  (static_cast<uint32_t>(2 * BM >> 4) << 24);

template <int kStages>
struct F8PairBarriers {
  uint64_t full[kStages];    // even CTA: both CTAs' stage landed
  uint64_t empty[kStages];   // the pair's MMAs on the stage completed
  uint64_t acc_full;         // the pair's accumulator is complete
  uint64_t acc_empty;        // even CTA: both epilogues drained their TMEM
  uint64_t teardown;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(F8PairBarriers<6>) <= kBarrierBytes, "FP8 pair barrier area");

__device__ __forceinline__ void mma_f8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

template <int kEpi>
__global__ void __launch_bounds__(kNumThreads, 1)
    fp8_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                         const __grid_constant__ CUtensorMap tmap_b_half,
                         const __grid_constant__ CUtensorMap tmap_out,
                         const float* __restrict__ sa_rows, const float* __restrict__ sw_cols,
                         const uint16_t* __restrict__ bias, uint16_t* __restrict__ out, int m,
                         int n, int k, uint32_t* row_amax, uint64_t wait_limit) {
  using P = F8PairPlan<kEpi>;
  constexpr int kStages = P::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicOr(&g_device_error, kErrSmemAlign);
    return;  // both CTAs see the same layout, so both return here
  }
  auto* bars = reinterpret_cast<F8PairBarriers<kStages>*>(smem + P::kBarrierOff);
  uint8_t* staging = smem + P::kStagingOff;
  uint16_t* gelu_tab = reinterpret_cast<uint16_t*>(smem + P::kTableOff);
  const int warp = warp_index_uniform();
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool even = rank == 0;
  const int pairs = gridDim.x / 2, pair = blockIdx.x / 2;
  const int num_m_pairs = (m + 2 * BM - 1) / (2 * BM);
  const int num_n_blocks = n / BN;
  const int tiles = num_m_pairs * num_n_blocks;
  const int count = pair < tiles ? (tiles - 1 - pair) / pairs + 1 : 0;  // same in both CTAs
  const int num_k_tiles = k / kF8BK;
  const uint64_t teardown_limit = wait_limit > kDefaultWaitLimit ? wait_limit : kDefaultWaitLimit;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->acc_empty, 2 * kEpiWarps);
    mbar_init(&bars->teardown, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b_half);
  }
  if (warp == 1) {
    tmem_alloc_pair(&bars->tmem_base, kF8TmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const auto even_addr = [&](const void* p) { return mapa_shared(smem_u32(p), 0); };
  const auto odd_addr = [&](const void* p) { return mapa_shared(smem_u32(p), 1); };

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    // (the whole warp runs the loop; one elected lane issues the copies)
    if (count > 0) {
      uint32_t armed[kStages];
#pragma unroll
      for (int s = 0; s < kStages; ++s) armed[s] = 0;
      int stage = 0;
      uint32_t phase = 0;
      for (int i = 0; i < count && !warp_aborted(bars); ++i) {
        const int t = pair + i * pairs;
        const int nb = t % num_n_blocks, mbp = t / num_n_blocks;  // N block fastest (A reuse in L2)
        // this CTA's 128 rows; a block wholly past the last row loads the last
        // block instead (its rows are never stored), so every box starts inside A
        const int a_row = min((2 * mbp + static_cast<int>(rank)) * BM, ((m - 1) / BM) * BM);
        for (int kt = 0; kt < num_k_tiles; ++kt) {
          if (!warp_wait_cluster_bounded(&bars->empty[stage], phase ^ 1u, wait_limit)) {
            warp_flag_error(bars, kErrWaitProducer);
            break;
          }
          uint8_t* sa = smem + stage * kF8PairStageBytes;
          uint8_t* sb = sa + kABytes;
          const uint32_t bar = even_addr(&bars->full[stage]);
          if (elect_one()) {
            if (even) mbar_arrive_expect_tx(&bars->full[stage], 2 * kF8PairStageBytes);
            tma_load_2d_pair(sa, &tmap_a, bar, kt * kF8BK, a_row);
            tma_load_2d_pair(sb, &tmap_b_half, bar, kt * kF8BK,
                             nb * BN + static_cast<int>(rank) * (BN / 2));
          }
          __syncwarp();
          armed[stage] += 1;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // the even CTA's stage barriers count both CTAs' loads; the odd CTA's land
      // before the even CTA's MMAs consume the stage, which the final cluster
      // barrier waits for
      for (int s = 0; even && s < kStages; ++s) {
        if (armed[s] > 0 &&
            !warp_wait_cluster_bounded(&bars->full[s], (armed[s] - 1) & 1u, teardown_limit))
          warp_flag_error(bars, kErrWaitTeardown);
      }
    }
  } else if (warp == 1) {
    if (count > 0 && even) {
      // ---------------------------------------------------------- MMA issuer (even CTA)
      // (the whole warp runs the loop; the same elected lane issues everything)
      int stage = 0;
      uint32_t phase = 0;
      bool issued_any = false;
      bool ok = true;
      for (int i = 0; ok && i < count && !warp_aborted(bars); ++i) {
        if (!warp_wait_cluster_bounded(&bars->acc_empty, (static_cast<uint32_t>(i) & 1u) ^ 1u,
                                       wait_limit)) {
          warp_flag_error(bars, kErrWaitMma);
          break;
        }
        tc_fence_after();
        for (int kt = 0; kt < num_k_tiles; ++kt) {
          if (!warp_wait_cluster_bounded(&bars->full[stage], phase, wait_limit)) {
            warp_flag_error(bars, kErrWaitMma);
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* sa = smem + stage * kF8PairStageBytes;
          uint8_t* sb = sa + kABytes;
          const uint64_t adesc = make_smem_desc(smem_u32(sa), 16, 1024, 2);
          const uint64_t bdesc = make_smem_desc(smem_u32(sb), 16, 1024, 2);
          const uint32_t empty_odd = odd_addr(&bars->empty[stage]);
          if (elect_one()) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              mma_f8_pair(tmem, adesc + static_cast<uint64_t>(2 * j),
                          bdesc + static_cast<uint64_t>(2 * j), kIdescF8Pair,
                          (kt > 0 || j > 0) ? 1u : 0u);
            }
            tc_commit_pair(smem_u32(&bars->empty[stage]));
            tc_commit_pair(empty_odd);
          }
          __syncwarp();
          issued_any = true;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        const uint32_t acc_odd = odd_addr(&bars->acc_full);
        if (elect_one()) {
          tc_commit_pair(smem_u32(&bars->acc_full));
          tc_commit_pair(acc_odd);
        }
        __syncwarp();
      }
      if (warp_aborted(bars) && issued_any) {
        if (elect_one()) tc_commit_pair(smem_u32(&bars->teardown));
        __syncwarp();
        if (!warp_wait_bounded(&bars->teardown, 0, teardown_limit))
          warp_flag_error(bars, kErrWaitTeardown);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quad = warp & 3;
    const int quarter = (warp - 2) >> 2;
    const int col_base = quarter * 64;
    const int trow = quad * 32 + lane;
    if constexpr (kEpi == 1) {
      gelu_table_init(gelu_tab, threadIdx.x - 64, kEpiThreads);
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
    }
    const uint32_t tab_base = smem_u32(gelu_tab);
    uint8_t* warp_staging = staging + (warp - 2) * kWarpStagingBytes;
    const uint32_t acc_empty_addr = even_addr(&bars->acc_empty);
    for (int i = 0; i < count; ++i) {
      const int t = pair + i * pairs;
      const int nb = t % num_n_blocks, mbp = t / num_n_blocks;  // N block fastest (A reuse in L2)
      const int row0 = mbp * 2 * BM + static_cast<int>(rank) * BM;  // this CTA's first row
      const int row = row0 + trow;
      const float sa = row < m ? __ldg(sa_rows + row) : 0.0f;
      if (!mbar_wait_cluster_bounded(&bars->acc_full, static_cast<uint32_t>(i) & 1u, wait_limit)) {
        flag_error(bars, kErrWaitEpilogue);
        break;
      }
      tc_fence_after();
      uint32_t r[64];
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quad * 32) << 16) + col_base;
      tmem_ld_32x32b_x32(taddr + 0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
      tmem_ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_addr);
      uint64_t sa2;
      asm("mov.b64 %0, {%1, %1};" : "=l"(sa2) : "f"(sa));
      const int col0 = nb * BN + col_base;
      const float4* sw4 = reinterpret_cast<const float4*>(sw_cols + col0);
      if (lane == 0) bulk_wait_group_read0();  // previous store has read the staging
      __syncwarp();
      const uint4* bias4 = reinterpret_cast<const uint4*>(bias + col0);
      uint32_t tile_max = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 s0 = __ldg(sw4 + 2 * q), s1 = __ldg(sw4 + 2 * q + 1);
        const float sw[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
        uint4 bv = make_uint4(0, 0, 0, 0);
        if (bias != nullptr) bv = __ldg(bias4 + q);
        const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          o[j] = rowcol_scale_pack_bf16x2(r[8 * q + 2 * j], r[8 * q + 2 * j + 1], sa2, sw[2 * j],
                                          sw[2 * j + 1]);
          if (bias != nullptr) o[j] = add_bf16x2(o[j], bw[j]);
        }
        if constexpr (kEpi == 1) {
          gelu_bf16x2_x4(o, tab_base, gelu_tab);
#pragma unroll
          for (int j = 0; j < 4; ++j) tile_max = max_u16x2(tile_max, o[j] & 0x7FFF7FFFu);
        }
        // 128B-swizzled staging (chunk c of row r at r*128 + ((c ^ (r & 7)) * 16)),
        // the output tensor map's swizzle
        *reinterpret_cast<uint4*>(warp_staging + lane * kStageRowBytes + ((q ^ (lane & 7)) * 16)) =
            make_uint4(o[0], o[1], o[2], o[3]);
      }
      if constexpr (kEpi == 1) {
        const uint32_t mag = max(tile_max & 0xFFFFu, tile_max >> 16);
        if (row < m && mag != 0) atomicMax(row_amax + row, mag << 16);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && row0 + quad * 32 < m) {
        tma_store_2d(&tmap_out, warp_staging, col0, row0 + quad * 32);
        bulk_commit_group();
      }
    }
    if (lane == 0) bulk_wait_group0();  // stores complete before the CTA exits
  }

  tc_fence_before();
  cluster_sync();  // neither CTA leaves while the pair's MMAs or arrivals may touch it
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, kF8TmemCols);
}

// GELU of bf16 values through the epilogue's path (test support): values
// 2i and 2i+1 form one bf16x2 word, as in the epilogue; an odd last value
// goes through the single-value path.
__global__ void __launch_bounds__(256) gelu_probe_kernel(const uint16_t* in, uint16_t* out,
                                                         int64_t count) {
  __shared__ __align__(16) uint16_t tab[kGeluTabEntries];
  gelu_table_init(tab, threadIdx.x, blockDim.x);
  __syncthreads();
  const uint32_t tab_base = smem_u32(tab);
  // four words (eight values) per step through the epilogues' gelu_bf16x2_x4,
  // the tail of fewer than eight values one at a time
  const int64_t groups = count / 8;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < groups;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      w[j] = static_cast<uint32_t>(in[8 * i + 2 * j]) | (static_cast<uint32_t>(in[8 * i + 2 * j + 1]) << 16);
    gelu_bf16x2_x4(w, tab_base, tab);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      out[8 * i + 2 * j] = static_cast<uint16_t>(w[j] & 0xFFFFu);
      out[8 * i + 2 * j + 1] = static_cast<uint16_t>(w[j] >> 16);
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0)
    for (int64_t e = groups * 8; e < count; ++e) out[e] = static_cast<uint16_t>(gelu_bf16(in[e], tab));
}

// ---------------------------------------------------------------- host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

// 2-D map over a byte matrix [rows, row_bytes], box = box_rows x 128 bytes, 128B swizzle.
bool make_byte_map(CUtensorMap* map, const uint8_t* base, int64_t rows, int64_t row_bytes,
                   uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(BKB), box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// FP4 codes [rows, k/2 bytes]
bool make_code_map(CUtensorMap* map, const uint8_t* base, int64_t rows, int64_t k,
                   uint32_t box_rows) {
  return make_byte_map(map, base, rows, k / 2, box_rows);
}

// 2-D map over a bf16 output [rows, n], box = 32 rows x 64 columns (128 B), 128B swizzle.
bool make_out_map(CUtensorMap* map, const uint16_t* base, int64_t rows, int64_t n) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(n * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kStageRowBytes / 2), 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int kEpi, bool kResident, bool kRepSfb = false>
cudaError_t launch_gemm_t(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo,
                          const uint8_t* a_sf,
                          const uint8_t* w_sf, const float* g_a, const float* g_w,
                          const float* alpha, const uint16_t* bias, uint16_t* out, int m, int n,
                          int k, float* amax_out, uint64_t wait_limit, cudaStream_t st,
                          const uint16_t* residual = nullptr, const uint16_t* gate = nullptr,
                          const QuantOut& qo = QuantOut()) {
  static ContextCache attr_done;
  constexpr int kSmemBytes = Plan<kEpi, kResident, kRepSfb>::kSmemBytes;
  if (cudaError_t e = ensure_max_dynamic_smem(
          attr_done, reinterpret_cast<const void*>(nvfp4_gemm_kernel<kEpi, kResident, kRepSfb>),
          kSmemBytes))
    return e;
  const int tiles = ((m + BM - 1) / BM) * (n / BN);
  int grid = sm_count();
  if (grid > tiles) grid = tiles;
  // programmatic dependent launch (the kernel waits for its predecessor itself)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kNumThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, nvfp4_gemm_kernel<kEpi, kResident, kRepSfb>, ma, mb, mo, a_sf,
                            w_sf, g_a, g_w, alpha, bias, out, m, n, k, amax_out, wait_limit,
                            residual, gate, qo);
}

// 3-D maps over 512-byte scale atoms (128 x u32): A scales [blocks][k/64 atoms][128],
// box 4 atoms (one K tile); replicated W scales [n/256 * k/64][8 atoms][128], box
// 4 x 8 atoms (one K tile of one N block).
// 3-D maps over the 512-byte scale atoms (u32 elements): A scales as
// [row block][K step][atom], box = 4 K steps of one block; W scales raw the
// same way with a box of two blocks (the 256 rows of an N block), or, when
// `w_rep` is set, the replicated layout [N block * K step][8][atom] with a box
// of 4 K steps.
bool make_scale_maps(CUtensorMap* sfa, CUtensorMap* sfb, const uint8_t* a_sf, int64_t a_blocks,
                     const uint8_t* w_sf, bool w_rep, int64_t n, int64_t k) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return false;
  const cuuint64_t k64 = static_cast<cuuint64_t>(k / 64);
  cuuint32_t estr[3] = {1, 1, 1};
  cuuint64_t dims_a[3] = {128, k64, static_cast<cuuint64_t>(a_blocks)};
  cuuint64_t strides_a[2] = {512, k64 * 512};
  cuuint32_t box_a[3] = {128, 4, 1};
  CUresult r = enc(sfa, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t*>(a_sf), dims_a,
                   strides_a, box_a, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  if (!w_rep) {
    cuuint64_t dims_b[3] = {128, k64, static_cast<cuuint64_t>(n / 128)};
    cuuint64_t strides_b[2] = {512, k64 * 512};
    cuuint32_t box_b[3] = {128, 4, 2};
    r = enc(sfb, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t*>(w_sf), dims_b, strides_b,
            box_b, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
  }
  cuuint64_t dims_b[3] = {128, 8, static_cast<cuuint64_t>(n / BN) * k64};
  cuuint64_t strides_b[2] = {512, 4096};
  cuuint32_t box_b[3] = {128, 8, 4};
  r = enc(sfb, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t*>(w_sf), dims_b, strides_b,
          box_b, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int kEpi, bool kRawSfb>
cudaError_t launch_gemm_pair(const CUtensorMap& ma, const CUtensorMap& mb_half,
                             const CUtensorMap& mb_quarter,
                             const CUtensorMap& msfa, const CUtensorMap& msfb, const float* g_a,
                             const float* g_w,
                             const uint16_t* bias, uint16_t* out, int m, int n, int k,
                             uint64_t wait_limit, cudaStream_t st,
                             const uint16_t* residual = nullptr, const uint16_t* gate = nullptr,
                             float* amax_out = nullptr) {
  static ContextCache attr_done;
  if (cudaError_t e = ensure_max_dynamic_smem(
          attr_done, reinterpret_cast<const void*>(nvfp4_gemm_pair_kernel<kEpi, kRawSfb>),
          PairPlan<kRawSfb>::kSmemBytes))
    return e;
  const int tiles = ((m + 2 * BM - 1) / (2 * BM)) * (n / BN);
  int pairs = sm_count() / 2;
  if (pairs > 2 * tiles) pairs = 2 * tiles;  // up to two pairs per tile: halves (PairSeq)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  cfg.blockDim = dim3(kNumThreads);
  cfg.dynamicSmemBytes = PairPlan<kRawSfb>::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, nvfp4_gemm_pair_kernel<kEpi, kRawSfb>, ma, mb_half, mb_quarter,
                            msfa, msfb,
                            g_a, g_w, bias, out, m, n, k, wait_limit, residual, gate, amax_out);
}

template <int kEpi>
cudaError_t launch_fp8_gemm_t(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo,
                              const float* sa, const float* sw, const uint16_t* bias, uint16_t* out,
                              int m, int n, int k, uint32_t* row_amax, uint64_t wait_limit,
                              cudaStream_t st) {
  static ContextCache attr_done;
  constexpr int kSmemBytes = F8Plan<kEpi>::kSmemBytes;
  if (cudaError_t e = ensure_max_dynamic_smem(
          attr_done, reinterpret_cast<const void*>(fp8_gemm_kernel<kEpi>), kSmemBytes))
    return e;
  const int tiles = ((m + BM - 1) / BM) * (n / BN);
  int grid = sm_count();
  if (grid > tiles) grid = tiles;
  fp8_gemm_kernel<kEpi><<<grid, kNumThreads, kSmemBytes, st>>>(ma, mb, mo, sa, sw, bias, out, m, n,
                                                                k, row_amax, wait_limit);
  return cudaGetLastError();
}

template <int kEpi>
cudaError_t launch_fp8_gemm_pair_t(const CUtensorMap& ma, const CUtensorMap& mb_half,
                                   const CUtensorMap& mo, const float* sa, const float* sw,
                                   const uint16_t* bias, uint16_t* out, int m, int n, int k,
                                   uint32_t* row_amax, uint64_t wait_limit, cudaStream_t st) {
  static ContextCache attr_done;
  constexpr int kSmemBytes = F8PairPlan<kEpi>::kSmemBytes;
  if (cudaError_t e = ensure_max_dynamic_smem(
          attr_done, reinterpret_cast<const void*>(fp8_gemm_pair_kernel<kEpi>), kSmemBytes))
    return e;
  const int tiles = ((m + 2 * BM - 1) / (2 * BM)) * (n / BN);
  int pairs = sm_count() / 2;
  if (pairs > tiles) pairs = tiles;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  cfg.blockDim = dim3(kNumThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fp8_gemm_pair_kernel<kEpi>, ma, mb_half, mo, sa, sw, bias, out,
                            m, n, k, row_amax, wait_limit);
}

}  // namespace

// FP8 GEMMs on SM pairs (256 x 256 tiles): 0 never, 1 the plain-epilogue GEMMs only
// (the default: the GELU epilogue measured faster on one SM per tile, the plain one
// on pairs), 2 always.
static int g_fp8_pairing = 1;
void set_fp8_gemm_pairing(int mode) { g_fp8_pairing = mode; }

cudaError_t launch_fp8_gemm(const uint8_t* a, const float* sa, const uint8_t* w, const float* sw,
                            const uint16_t* bias, uint16_t* out, int64_t m, int64_t n, int64_t k,
                            int epilogue, uint32_t* row_amax, uint64_t wait_limit, cudaStream_t st,
                            const char** why) {
  alignas(64) CUtensorMap ma;
  alignas(64) CUtensorMap mb;
  if (!make_byte_map(&ma, a, m, k, BM) || !make_byte_map(&mb, w, n, k, BN)) {
    if (why) *why = "cuTensorMapEncodeTiled failed for the E4M3 operands";
    return cudaErrorInvalidValue;
  }
  alignas(64) CUtensorMap mo;
  std::memset(&mo, 0, sizeof(mo));
  const int mi = static_cast<int>(m), ni = static_cast<int>(n), ki = static_cast<int>(k);
  if (!make_out_map(&mo, out, m, n)) {
    if (why) *why = "cuTensorMapEncodeTiled failed for the output";
    return cudaErrorInvalidValue;
  }
  const bool pairs = g_fp8_pairing == 2 || (g_fp8_pairing == 1 && epilogue == 0);
  if (pairs && sm_count() >= 2) {
    alignas(64) CUtensorMap mb_half;
    if (!make_byte_map(&mb_half, w, n, k, BN / 2)) {
      if (why) *why = "cuTensorMapEncodeTiled failed for the SM-pair W map";
      return cudaErrorInvalidValue;
    }
    if (epilogue == 1)
      return launch_fp8_gemm_pair_t<1>(ma, mb_half, mo, sa, sw, bias, out, mi, ni, ki, row_amax,
                                       wait_limit, st);
    return launch_fp8_gemm_pair_t<0>(ma, mb_half, mo, sa, sw, bias, out, mi, ni, ki, nullptr,
                                     wait_limit, st);
  }
  if (epilogue == 1)
    return launch_fp8_gemm_t<1>(ma, mb, mo, sa, sw, bias, out, mi, ni, ki, row_amax, wait_limit, st);
  return launch_fp8_gemm_t<0>(ma, mb, mo, sa, sw, bias, out, mi, ni, ki, nullptr, wait_limit, st);
}

// GEMMs with replicated W scales and m % 256 == 0 run on SM pairs when enabled
// (off by default: measured at the one-SM kernel's speed, both clock-limited by
// the power cap under sustained tensor load).
static int g_pairing = 1;  // SM pairs with W scales in the library layout
void set_gemm_pairing(int mode) { g_pairing = mode; }
// Any m: a ragged last pair tile is handled in the kernel (see nvfp4_gemm_pair_kernel).
bool gemm_pairs(int64_t m, int epilogue) { return g_pairing != 0 && epilogue == 0 && m > 0; }
bool gemm_pairs_raw_scales(int64_t m) { return g_pairing == 1 && m > 0; }

cudaError_t launch_gemm(const uint8_t* a_codes, const uint8_t* a_sf, const float* g_a,
                        const uint8_t* w_codes, const uint8_t* w_sf, const float* g_w,
                        const float* alpha, const uint16_t* bias, uint16_t* out, int64_t m, int64_t n, int64_t k,
                        int epilogue, float* amax_out, uint64_t wait_limit, cudaStream_t st,
                        const char** why, const uint8_t* w_sf_rep, const uint16_t* residual,
                        const uint16_t* gate, const QuantOut* qo) {
  alignas(64) CUtensorMap ma;
  alignas(64) CUtensorMap mb;
  if (!make_code_map(&ma, a_codes, m, k, BM) || !make_code_map(&mb, w_codes, n, k, BN)) {
    if (why) *why = "cuTensorMapEncodeTiled failed for the code matrices";
    return cudaErrorInvalidValue;
  }
  alignas(64) CUtensorMap mo;
  std::memset(&mo, 0, sizeof(mo));
  if (epilogue == 1 && !make_out_map(&mo, out, m, n)) {
    if (why) *why = "cuTensorMapEncodeTiled failed for the output";
    return cudaErrorInvalidValue;
  }
  const int mi = static_cast<int>(m), ni = static_cast<int>(n), ki = static_cast<int>(k);
  if (epilogue == 3) {
    if (qo == nullptr || qo->codes == nullptr || qo->sf == nullptr || qo->amax_hint == nullptr ||
        amax_out == nullptr) {
      if (why) *why = "the quantizing epilogue needs codes, scales, an amax hint and amax_out";
      return cudaErrorInvalidValue;
    }
    const bool resident = (k / 64) <= kMaxResidentKSteps && (n / BN) <= sm_count();
    if (resident)
      return launch_gemm_t<3, true>(ma, mb, mo, a_sf, w_sf, g_a, g_w, alpha, bias, out, mi, ni, ki,
                                    amax_out, wait_limit, st, nullptr, nullptr, *qo);
    return launch_gemm_t<3, false>(ma, mb, mo, a_sf, w_sf, g_a, g_w, alpha, bias, out, mi, ni, ki,
                                   amax_out, wait_limit, st, nullptr, nullptr, *qo);
  }
  if (epilogue == 1) {
    // W scales stay in TMEM when they fit and every N block gets a CTA
    const bool resident = (k / 64) <= kMaxResidentKSteps && (n / BN) <= sm_count();
    QuantOut q;
    if (qo != nullptr) q.zero_word = qo->zero_word;
    if (resident)
      return launch_gemm_t<1, true>(ma, mb, mo, a_sf, w_sf, g_a, g_w, alpha, bias, out, mi, ni, ki,
                                    amax_out, wait_limit, st, nullptr, nullptr, q);
    return launch_gemm_t<1, false>(ma, mb, mo, a_sf, w_sf, g_a, g_w, alpha, bias, out, mi, ni, ki,
                                   amax_out, wait_limit, st, nullptr, nullptr, q);
  }
  if (epilogue == 2) {
    if (residual == nullptr || gate == nullptr) {
      if (why) *why = "the gated-residual epilogue needs the residual and the gate";
      return cudaErrorInvalidValue;
    }
    if (gemm_pairs_raw_scales(m) && alpha == nullptr && w_sf != nullptr) {
      alignas(64) CUtensorMap mb_half;
      alignas(64) CUtensorMap mb_quarter;
      alignas(64) CUtensorMap msfa;
      alignas(64) CUtensorMap msfb;
      if (!make_code_map(&mb_half, w_codes, n, k, BN / 2) ||
          !make_code_map(&mb_quarter, w_codes, n, k, BN / 4) ||
          !make_scale_maps(&msfa, &msfb, a_sf, (m + BM - 1) / BM, w_sf, false, n, k)) {
        if (why) *why = "cuTensorMapEncodeTiled failed for the SM-pair GEMM";
        return cudaErrorInvalidValue;
      }
      return launch_gemm_pair<2, true>(ma, mb_half, mb_quarter, msfa, msfb, g_a, g_w, bias, out, mi,
                                       ni, ki, wait_limit, st, residual, gate, amax_out);
    }
    if (w_sf_rep == nullptr) {
      if (why) *why = "the one-SM gated-residual epilogue needs replicated W scales";
      return cudaErrorInvalidValue;
    }
    return launch_gemm_t<2, false, true>(ma, mb, mo, a_sf, w_sf_rep, g_a, g_w, alpha, bias, out, mi,
                                         ni, ki, amax_out, wait_limit, st, residual, gate);
  }
  // SM pairs: mode 1 reads the W scales in the library layout, mode 2 the
  // replicated copy; each falls back to the other form when the caller has
  // only that one
  const bool have_raw = w_sf != nullptr, have_rep = w_sf_rep != nullptr;
  const bool pair_rep = have_rep && (g_pairing == 2 || !have_raw);
  if (gemm_pairs(m, epilogue) && alpha == nullptr && (have_raw || have_rep)) {
    alignas(64) CUtensorMap mb_half;
    alignas(64) CUtensorMap mb_quarter;
    alignas(64) CUtensorMap msfa;
    alignas(64) CUtensorMap msfb;
    if (!make_code_map(&mb_half, w_codes, n, k, BN / 2) ||
        !make_code_map(&mb_quarter, w_codes, n, k, BN / 4) ||
        !make_scale_maps(&msfa, &msfb, a_sf, (m + BM - 1) / BM, pair_rep ? w_sf_rep : w_sf, pair_rep,
                         n, k)) {
      if (why) *why = "cuTensorMapEncodeTiled failed for the SM-pair GEMM";
      return cudaErrorInvalidValue;
    }
    if (pair_rep)
      return launch_gemm_pair<0, false>(ma, mb_half, mb_quarter, msfa, msfb, g_a, g_w, bias, out, mi,
                                        ni, ki, wait_limit, st, nullptr, nullptr, amax_out);
    return launch_gemm_pair<0, true>(ma, mb_half, mb_quarter, msfa, msfb, g_a, g_w, bias, out, mi,
                                     ni, ki, wait_limit, st, nullptr, nullptr, amax_out);
  }
  if (w_sf_rep != nullptr)
    return launch_gemm_t<0, false, true>(ma, mb, mo, a_sf, w_sf_rep, g_a, g_w, alpha, bias, out, mi,
                                         ni, ki, amax_out, wait_limit, st);
  return launch_gemm_t<0, false>(ma, mb, mo, a_sf, w_sf, g_a, g_w, alpha, bias, out, mi, ni, ki,
                                 amax_out, wait_limit, st);
}

cudaError_t launch_gelu_probe(const uint16_t* in, uint16_t* out, int64_t count, cudaStream_t st) {
  if (count <= 0) return cudaSuccess;
  int64_t blocks = (count + 255) / 256;
  if (blocks > 1024) blocks = 1024;
  gelu_probe_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(in, out, count);
  return cudaGetLastError();
}

namespace {
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

struct CtxQuery {
  CtxGetCurrentFn get_current = nullptr;
  CtxGetIdFn get_id = nullptr;
};

const CtxQuery& ctx_query() {
  static CtxQuery q;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult r;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &r) == cudaSuccess &&
        r == cudaDriverEntryPointSuccess)
      q.get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &r) == cudaSuccess &&
        r == cudaDriverEntryPointSuccess)
      q.get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  return q;
}
}  // namespace

uint64_t current_context_id() {
  const CtxQuery& q = ctx_query();
  if (q.get_current == nullptr || q.get_id == nullptr) return 0;
  CUcontext c = nullptr;
  if (q.get_current(&c) != CUDA_SUCCESS || c == nullptr) return 0;
  unsigned long long id = 0;
  if (q.get_id(c, &id) != CUDA_SUCCESS) return 0;
  return static_cast<uint64_t>(id);
}

cudaError_t context_symbol_address(ContextCache& cache, const void* symbol, void** out) {
  uint64_t id = current_context_id();
  if (id != 0 && cache.get(id, out)) return cudaSuccess;
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, symbol);
  if (e != cudaSuccess) return e;
  if (p == nullptr) return cudaErrorInvalidSymbol;
  if (id == 0) id = current_context_id();  // the lookup itself made the primary context current
  if (id != 0) cache.put(id, p);
  *out = p;
  return cudaSuccess;
}

cudaError_t ensure_max_dynamic_smem(ContextCache& cache, const void* fn, int bytes) {
  void* done = nullptr;
  const uint64_t id = current_context_id();
  if (id != 0 && cache.get(id, &done)) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  const uint64_t id2 = id != 0 ? id : current_context_id();
  if (id2 != 0) cache.put(id2, reinterpret_cast<void*>(1));
  return cudaSuccess;
}

uint32_t* error_word_ptr() {
  static ContextCache cache;
  void* p = nullptr;
  if (context_symbol_address(cache, reinterpret_cast<const void*>(&g_device_error), &p) !=
      cudaSuccess)
    return nullptr;
  return static_cast<uint32_t*>(p);
}

cudaError_t set_error_word(uint32_t v, cudaStream_t st) {
  return cudaMemcpyToSymbolAsync(g_device_error, &v, sizeof(v), 0, cudaMemcpyHostToDevice, st);
}

cudaError_t read_error_word(uint32_t* v, cudaStream_t st) {
  cudaError_t e = cudaMemcpyFromSymbolAsync(v, g_device_error, sizeof(*v), 0,
                                            cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return e;
  return cudaStreamSynchronize(st);
}

}  // namespace fvq
