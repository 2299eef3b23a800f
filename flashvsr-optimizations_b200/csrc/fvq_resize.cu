// fvq_resize.cu -- Pillow-exact bicubic upscale of RGB frames, crop and bf16
// normalisation in one pass (reference pil_exact_gpu.py:30-150, called by
// chunked_input.py:111-113 as normalize_exact_gpu(resize_exact_gpu(frames))).
//
// Pillow's 8-bit resample (libImaging/Resample.c): per output position the
// bicubic taps (a = -0.5, support 2 when upscaling, at most 4 taps) are
// normalised by their sum in double and rounded to signed 22-bit fixed point;
// the horizontal pass accumulates 2^21 + sum(pixel * weight) in int32, shifts
// right by 22 and clips to a uint8 intermediate, and the vertical pass does the
// same on that intermediate.  The reference's normalisation maps each byte p to
// bf16(p / 255 * 2 - 1) evaluated in fp32.
//
// One CTA produces 32 output rows of one frame, across the whole crop:
//   1. the tap weights: horizontal ones for the crop's columns and vertical
//      ones for the tile's rows, computed in double with non-contracting
//      intrinsics (__dmul_rn / __dadd_rn ...) so each operation rounds as in
//      Pillow's C code; and the 256-entry normalisation table;
//   2. the input rows the tile needs (about 32 / scale + 4 of them) copied
//      into shared memory with 16-byte loads;
//   3. the horizontal pass for those rows, crop columns only, into a uint8
//      intermediate in shared memory -- it never reaches HBM;
//   4. the vertical pass, written as uint8 HWC rows (16 bytes per thread)
//      and/or as the normalised bf16 channel planes (8 values per thread).
// The work is HBM-bound on the outputs (4.5 MB of bytes and 8.9 MB of bf16 per
// 1664x896 frame); the intermediate and the coefficients stay on chip.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "fvq_internal.h"

namespace fvq {

namespace {

constexpr int kResizeThreads = 256;
constexpr int kTileRows = 32;     // output rows per CTA
constexpr int kPrecisionBits = 22;

// Pillow's bicubic_filter (a = -0.5), one IEEE double rounding per operation.
__device__ __forceinline__ double bicubic_tap(double x) {
  if (x < 0.0) x = -x;
  if (x < 1.0)
    return __dadd_rn(__dmul_rn(__dmul_rn(__dsub_rn(__dmul_rn(1.5, x), 2.5), x), x), 1.0);
  if (x < 2.0)
    return __dmul_rn(__dsub_rn(__dmul_rn(__dadd_rn(__dmul_rn(__dsub_rn(x, 5.0), x), 8.0), x), 4.0),
                     -0.5);
  return 0.0;
}

// precompute_coeffs + normalize_coeffs_8bpc for output position `pos` of an
// upscale in_size -> out_size: first tap index and four fixed-point weights
// (zero past the last tap).
__device__ void tap_weights(int pos, int in_size, int out_size, int* first, int4* w) {
  const double scale = __ddiv_rn(static_cast<double>(in_size), static_cast<double>(out_size));
  const double center = __dmul_rn(__dadd_rn(static_cast<double>(pos), 0.5), scale);
  int xmin = __double2int_rz(__dadd_rn(__dsub_rn(center, 2.0), 0.5));
  if (xmin < 0) xmin = 0;
  int xmax = __double2int_rz(__dadd_rn(__dadd_rn(center, 2.0), 0.5));
  if (xmax > in_size) xmax = in_size;
  xmax -= xmin;
  double k[4] = {0.0, 0.0, 0.0, 0.0};
  double ww = 0.0;
  for (int x = 0; x < xmax && x < 4; ++x) {
    // (x + xmin - center + 0.5): the integer sum first, as in Pillow
    k[x] = bicubic_tap(__dadd_rn(__dsub_rn(static_cast<double>(x + xmin), center), 0.5));
    ww = __dadd_rn(ww, k[x]);
  }
  int q[4] = {0, 0, 0, 0};
  for (int x = 0; x < xmax && x < 4; ++x) {
    const double kn = ww != 0.0 ? __ddiv_rn(k[x], ww) : k[x];
    const double v = __dmul_rn(kn, static_cast<double>(1 << kPrecisionBits));
    q[x] = kn < 0.0 ? __double2int_rz(__dadd_rn(-0.5, v)) : __double2int_rz(__dadd_rn(0.5, v));
  }
  *first = xmin;
  *w = make_int4(q[0], q[1], q[2], q[3]);
}

__device__ __forceinline__ uint32_t clip8(int acc) {
  const int v = acc >> kPrecisionBits;
  return static_cast<uint32_t>(v < 0 ? 0 : (v > 255 ? 255 : v));
}

struct ResizeGeom {
  int in_h, in_w, out_h, out_w;
  int crop_y, crop_x, crop_h, crop_w;
  int tile_w;       // crop columns per CTA (multiple of 16); the last tile may be narrower
                    // (a multiple of 8)
  int max_rows;     // input rows a 32-row tile can need
};

// Shared memory of one CTA: tap tables (first tap + 4 weights per column of the
// column tile and per row of the row tile), the bf16 table, the input rows, the
// uint8 intermediate.
struct ResizeSmem {
  int h_w, h_first, v_w, v_first, lut, run, temp, total;
  __host__ __device__ explicit ResizeSmem(const ResizeGeom& g) {
    h_w = 0;                                         // int4 [tile_w]
    v_w = h_w + g.tile_w * 16;                       // int4 [32]
    h_first = v_w + kTileRows * 16;                  // int [tile_w]
    v_first = h_first + (g.tile_w * 4 + 15) / 16 * 16;  // int [32]
    lut = v_first + kTileRows * 4;                   // u16 [256]
    run = lut + 512;                                 // input rows, packed, 16-byte skew slack
    temp = run + (g.max_rows * g.in_w * 3 + 32 + 15) / 16 * 16;
    total = temp + g.max_rows * g.tile_w * 3;        // intermediate rows, tile_w * 3 bytes each
  }
};

// Vertical pass to uint8 rows, kWords 32-bit words (4 bytes each) per item: 16-byte
// chunks when both the tile's and the output's row bytes are multiples of 16, else
// 8-byte chunks (crop_w % 8 == 0 keeps those aligned).
template <int kWords>
__device__ __forceinline__ void vertical_u8(const uint8_t* temp, int pitch, int rows, int n_rows,
                                            int r_lo, const int4* v_w, const int* v_first,
                                            uint8_t* dst_u8, int frame, int y0, int x0,
                                            const ResizeGeom& g) {
  constexpr int kBytes = 4 * kWords;
  const int chunks = pitch / kBytes;
  for (int item = threadIdx.x; item < rows * chunks; item += kResizeThreads) {
    const int yy = item / chunks, ch = item - yy * chunks;
    const int4 w = v_w[yy];
    const int f = v_first[yy] - r_lo;
    const uint32_t* ta = reinterpret_cast<const uint32_t*>(temp + f * pitch + ch * kBytes);
    const uint32_t* tb = reinterpret_cast<const uint32_t*>(temp + min(f + 1, n_rows - 1) * pitch + ch * kBytes);
    const uint32_t* tc = reinterpret_cast<const uint32_t*>(temp + min(f + 2, n_rows - 1) * pitch + ch * kBytes);
    const uint32_t* td = reinterpret_cast<const uint32_t*>(temp + min(f + 3, n_rows - 1) * pitch + ch * kBytes);
    uint32_t o[kWords];
#pragma unroll
    for (int q = 0; q < kWords; ++q) {
      const uint32_t wa = ta[q], wb = tb[q], wc = tc[q], wd = td[q];
      uint32_t packed = 0;
#pragma unroll
      for (int byte = 0; byte < 4; ++byte) {
        const int sh = byte * 8;
        int acc = 1 << (kPrecisionBits - 1);
        acc += static_cast<int>((wa >> sh) & 0xFF) * w.x;
        acc += static_cast<int>((wb >> sh) & 0xFF) * w.y;
        acc += static_cast<int>((wc >> sh) & 0xFF) * w.z;
        acc += static_cast<int>((wd >> sh) & 0xFF) * w.w;
        packed |= clip8(acc) << sh;
      }
      o[q] = packed;
    }
    uint8_t* dst = dst_u8 + ((static_cast<int64_t>(frame) * g.crop_h + y0 + yy) * g.crop_w + x0) * 3 +
                   ch * kBytes;
    if (kWords == 4)
      *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[kWords > 2 ? 2 : 0], o[kWords > 3 ? 3 : 0]);
    else
      *reinterpret_cast<uint2*>(dst) = make_uint2(o[0], o[1]);
  }
}

template <bool kU8, bool kBf16>
__global__ void __launch_bounds__(kResizeThreads) pil_resize_kernel(
    const uint8_t* __restrict__ src, ResizeGeom g, uint8_t* __restrict__ dst_u8,
    uint16_t* __restrict__ dst_bf16) {
  extern __shared__ __align__(16) uint8_t sm[];
  const ResizeSmem L(g);
  int4* h_w = reinterpret_cast<int4*>(sm + L.h_w);
  int4* v_w = reinterpret_cast<int4*>(sm + L.v_w);
  int* h_first = reinterpret_cast<int*>(sm + L.h_first);
  int* v_first = reinterpret_cast<int*>(sm + L.v_first);
  uint16_t* lut = reinterpret_cast<uint16_t*>(sm + L.lut);
  uint8_t* temp = sm + L.temp;

  const int frame = blockIdx.z;
  const int y0 = blockIdx.x * kTileRows;         // first crop row of the tile
  const int x0 = blockIdx.y * g.tile_w;          // first crop column of the tile
  const int rows = min(kTileRows, g.crop_h - y0);
  const int cols = min(g.tile_w, g.crop_w - x0);  // a multiple of 8
  const int pitch = cols * 3;                     // intermediate row bytes, a multiple of 8
  const int tid = threadIdx.x;

  // 1. tap weights and the normalisation table
  for (int i = tid; i < cols; i += kResizeThreads) {
    int f;
    int4 w;
    tap_weights(g.crop_x + x0 + i, g.in_w, g.out_w, &f, &w);
    h_first[i] = f;
    h_w[i] = w;
  }
  for (int i = tid; i < rows; i += kResizeThreads) {
    int f;
    int4 w;
    tap_weights(g.crop_y + y0 + i, g.in_h, g.out_h, &f, &w);
    v_first[i] = f;
    v_w[i] = w;
  }
  if (kBf16) {
    for (int p = tid; p < 256; p += kResizeThreads) {
      const float v = __fsub_rn(__fmul_rn(__fdiv_rn(static_cast<float>(p), 255.0f), 2.0f), 1.0f);
      lut[p] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
    }
  }
  __syncthreads();

  // 2. input rows [r_lo, r_hi] (taps past the image have weight 0), contiguous in
  //    global memory: copied as one run whose shared-memory origin has the same
  //    offset modulo 16 as the global start, so the 16-byte body loads land
  //    aligned; head and tail bytes one at a time, nothing outside the run read
  const int r_lo = v_first[0];
  const int r_hi = min(v_first[rows - 1] + 3, g.in_h - 1);
  const int n_rows = r_hi - r_lo + 1;
  const int row_bytes = g.in_w * 3;
  const uint8_t* base = src + (static_cast<int64_t>(frame) * g.in_h + r_lo) * row_bytes;
  uint8_t* in_rows = sm + L.run + (reinterpret_cast<uintptr_t>(base) & 15);
  {
    const int nbytes = n_rows * row_bytes;
    const int head = min(static_cast<int>((16 - (reinterpret_cast<uintptr_t>(base) & 15)) & 15),
                         nbytes);
    const int body = (nbytes - head) / 16;
    for (int i = tid; i < head; i += kResizeThreads) in_rows[i] = base[i];
    const uint4* g16 = reinterpret_cast<const uint4*>(base + head);
    uint4* s16 = reinterpret_cast<uint4*>(in_rows + head);
    for (int i = tid; i < body; i += kResizeThreads) s16[i] = __ldg(g16 + i);
    for (int i = head + body * 16 + tid; i < nbytes; i += kResizeThreads) in_rows[i] = base[i];
  }
  __syncthreads();

  // 3. horizontal pass: intermediate rows r_lo..r_hi of this column tile, one pixel per item
  for (int item = tid; item < n_rows * cols; item += kResizeThreads) {
    const int r = item / cols, x = item - r * cols;
    const int f = h_first[x];
    const int4 w = h_w[x];
    const uint8_t* p = in_rows + r * row_bytes;
    const int i0 = f * 3, i1 = min(f + 1, g.in_w - 1) * 3, i2 = min(f + 2, g.in_w - 1) * 3,
              i3 = min(f + 3, g.in_w - 1) * 3;
    uint8_t* t = temp + r * pitch + x * 3;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      int acc = 1 << (kPrecisionBits - 1);
      acc += static_cast<int>(p[i0 + c]) * w.x;
      acc += static_cast<int>(p[i1 + c]) * w.y;
      acc += static_cast<int>(p[i2 + c]) * w.z;
      acc += static_cast<int>(p[i3 + c]) * w.w;
      t[c] = static_cast<uint8_t>(clip8(acc));
    }
  }
  __syncthreads();

  // 4. vertical pass and outputs
  const int64_t plane = static_cast<int64_t>(g.crop_h) * g.crop_w;
  if (kU8) {
    // 16-byte stores need every output row start 16-byte aligned too (crop_w % 16 == 0)
    if (pitch % 16 == 0 && g.crop_w % 16 == 0)
      vertical_u8<4>(temp, pitch, rows, n_rows, r_lo, v_w, v_first, dst_u8, frame, y0, x0, g);
    else
      vertical_u8<2>(temp, pitch, rows, n_rows, r_lo, v_w, v_first, dst_u8, frame, y0, x0, g);
  }
  if (kBf16) {
    const int groups = cols / 8;  // 8 columns of one channel per item
    for (int item = tid; item < rows * 3 * groups; item += kResizeThreads) {
      const int yy = item / (3 * groups);
      const int rest = item - yy * 3 * groups;
      const int ch = rest / groups, gx = rest - ch * groups;
      const int4 w = v_w[yy];
      const int f = v_first[yy] - r_lo;
      const uint8_t* ta = temp + f * pitch;
      const uint8_t* tb = temp + min(f + 1, n_rows - 1) * pitch;
      const uint8_t* tc = temp + min(f + 2, n_rows - 1) * pitch;
      const uint8_t* td = temp + min(f + 3, n_rows - 1) * pitch;
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t pair = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int b = (gx * 8 + q * 2 + h) * 3 + ch;
          int acc = 1 << (kPrecisionBits - 1);
          acc += static_cast<int>(ta[b]) * w.x;
          acc += static_cast<int>(tb[b]) * w.y;
          acc += static_cast<int>(tc[b]) * w.z;
          acc += static_cast<int>(td[b]) * w.w;
          pair |= static_cast<uint32_t>(lut[clip8(acc)]) << (16 * h);
        }
        o[q] = pair;
      }
      uint16_t* dst = dst_bf16 + (static_cast<int64_t>(frame) * 3 + ch) * plane +
                      static_cast<int64_t>(y0 + yy) * g.crop_w + x0 + gx * 8;
      *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// The reference's normalize_exact_gpu on its own: uint8 [T, h, w, 3] with element
// strides (sb, sy, sx; channels adjacent) -> bf16 [T, 3, h, w], 8 columns per item.
__global__ void __launch_bounds__(kResizeThreads) pil_normalize_kernel(
    const uint8_t* __restrict__ src, int64_t frames, int h, int w, int64_t sb, int64_t sy,
    int64_t sx, uint16_t* __restrict__ dst) {
  __shared__ uint16_t lut[256];
  for (int p = threadIdx.x; p < 256; p += kResizeThreads) {
    const float v = __fsub_rn(__fmul_rn(__fdiv_rn(static_cast<float>(p), 255.0f), 2.0f), 1.0f);
    lut[p] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
  }
  __syncthreads();
  const int groups = w / 8;
  const int64_t items = frames * 3 * h * groups;
  for (int64_t it = blockIdx.x * static_cast<int64_t>(kResizeThreads) + threadIdx.x; it < items;
       it += static_cast<int64_t>(gridDim.x) * kResizeThreads) {
    const int gx = static_cast<int>(it % groups);
    const int64_t r = it / groups;
    const int y = static_cast<int>(r % h);
    const int64_t r2 = r / h;
    const int ch = static_cast<int>(r2 % 3);
    const int64_t t = r2 / 3;
    const uint8_t* p = src + t * sb + y * sy + static_cast<int64_t>(gx) * 8 * sx + ch;
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      o[q] = static_cast<uint32_t>(lut[__ldg(p + (2 * q) * sx)]) |
             (static_cast<uint32_t>(lut[__ldg(p + (2 * q + 1) * sx)]) << 16);
    *reinterpret_cast<uint4*>(dst + ((t * 3 + ch) * h + y) * static_cast<int64_t>(w) + gx * 8) =
        make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <bool kU8, bool kBf16>
cudaError_t launch_resize_t(const uint8_t* src, int64_t frames, const ResizeGeom& g, uint8_t* u8,
                            uint16_t* bf16, size_t smem, cudaStream_t st) {
  static ContextCache attr_done;
  if (cudaError_t e = ensure_max_dynamic_smem(
          attr_done, reinterpret_cast<const void*>(pil_resize_kernel<kU8, kBf16>), 227 * 1024))
    return e;
  const dim3 grid((g.crop_h + kTileRows - 1) / kTileRows, (g.crop_w + g.tile_w - 1) / g.tile_w,
                  static_cast<unsigned>(frames));
  pil_resize_kernel<kU8, kBf16><<<grid, kResizeThreads, smem, st>>>(src, g, u8, bf16);
  return cudaGetLastError();
}

}  // namespace

// Geometry arguments are checked by the C ABI (upscale, crop inside the output,
// crop_w % 8 == 0, frames < 65536); here the tiling and the shared-memory plan.
cudaError_t launch_pil_resize(const uint8_t* src, int64_t frames, int in_h, int in_w, int out_h,
                              int out_w, int crop_y, int crop_x, int crop_h, int crop_w,
                              uint8_t* dst_u8, uint16_t* dst_bf16, size_t* smem_needed,
                              cudaStream_t st) {
  ResizeGeom g;
  g.in_h = in_h;
  g.in_w = in_w;
  g.out_h = out_h;
  g.out_w = out_w;
  g.crop_y = crop_y;
  g.crop_x = crop_x;
  g.crop_h = crop_h;
  g.crop_w = crop_w;
  // columns per CTA: the crop in ceil(crop_w / 1024) tiles of equal width (multiples of 16)
  const int tiles = (crop_w + 1023) / 1024;
  g.tile_w = ((crop_w + tiles - 1) / tiles + 15) / 16 * 16;
  // rows a 32-row tile reads: its first taps span at most ceil(31 * in / out) + 1 rows, plus 3
  g.max_rows = static_cast<int>((static_cast<int64_t>(kTileRows) * in_h + out_h - 1) / out_h) + 5;
  if (g.max_rows > in_h) g.max_rows = in_h;
  const ResizeSmem L(g);
  const size_t smem = static_cast<size_t>(L.total);
  if (smem_needed) *smem_needed = smem;
  if (smem > static_cast<size_t>(220 * 1024)) return cudaErrorInvalidValue;
  if (frames <= 0) return cudaSuccess;
  if (dst_u8 && dst_bf16)
    return launch_resize_t<true, true>(src, frames, g, dst_u8, dst_bf16, smem, st);
  if (dst_u8) return launch_resize_t<true, false>(src, frames, g, dst_u8, nullptr, smem, st);
  return launch_resize_t<false, true>(src, frames, g, nullptr, dst_bf16, smem, st);
}

cudaError_t launch_pil_normalize(const uint8_t* src, int64_t frames, int h, int w, int64_t sb,
                                 int64_t sy, int64_t sx, uint16_t* dst, cudaStream_t st) {
  const int64_t items = frames * 3 * h * (w / 8);
  if (items <= 0) return cudaSuccess;
  int64_t blocks = (items + kResizeThreads - 1) / kResizeThreads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  pil_normalize_kernel<<<static_cast<unsigned>(blocks), kResizeThreads, 0, st>>>(src, frames, h, w,
                                                                                sb, sy, sx, dst);
  return cudaGetLastError();
}

}  // namespace fvq
