// fvq_noalloc.cu -- QuantLinear.forward for callers that cannot allocate.
//
// Some callers of this library cannot call cudaMalloc or any allocating
// routine at the point where they run the layer: code that lives inside a
// foreign runtime's memory pool or arena, plugins that are handed only input
// and output buffers, or callers that must not touch the allocator while
// other work is in flight.  fvq_nvfp4_linear needs a caller-supplied
// workspace (the amax pass's partials and counter, the global scale, and the
// activation's NVFP4 codes and scale factors).  fvq_nvfp4_linear_noalloc
// runs the same kernels with that workspace carved out of a fixed-size
// scratch array that is part of this library's device image instead.
//
// Limits and rules (also in include/fvq.h):
//   * the scratch is kNoAllocScratchBytes (16 MiB) per device, held by every
//     GPU that loads the library until the process exits;
//   * rows x in_features must fit it (fvq_nvfp4_linear_workspace_bytes);
//     larger calls are rejected with FVQ_EWORKSPACE and a message;
//   * the first call on a device resolves the array's device address with
//     cudaGetSymbolAddress (with that device current); make that first call
//     before any stream capture;
//   * every call shares the one array: calls that overlap on the GPU (other
//     streams, other host threads) race.  The amax arrival counter inside it
//     starts at zero (static device memory is zero-initialised) and every
//     call re-arms it; everything else is written before it is read.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/fvq.h"
#include "fvq_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[64] = {nullptr};

// Device address of the scratch array for the current device (set-up on first use).
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) return FVQ_ECUDA;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return FVQ_ECUDA;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return FVQ_OK;
}

}  // namespace

extern "C" {

size_t fvq_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int fvq_nvfp4_linear_noalloc(const uint16_t* x, int64_t rows, const fvq_linear* lin, uint16_t* y,
                             void* stream) {
  if (lin == nullptr) return fvq::report_error(FVQ_EINVAL, "fvq_nvfp4_linear_noalloc: lin is NULL");
  const size_t need = fvq_nvfp4_linear_workspace_bytes(rows, lin->in_features);
  if (need == 0)
    return fvq::report_error(FVQ_EINVAL, "fvq_nvfp4_linear_noalloc: rows and in_features must be > 0");
  if (need > kNoAllocScratchBytes)
    return fvq::report_error(
        FVQ_EWORKSPACE,
        "fvq_nvfp4_linear_noalloc: rows x in_features needs %zu bytes of scratch, more than the "
        "built-in %zu; call fvq_nvfp4_linear with a workspace instead",
        need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  if (noalloc_scratch(&scratch) != FVQ_OK)
    return fvq::report_error(FVQ_ECUDA,
                             "fvq_nvfp4_linear_noalloc: cudaGetSymbolAddress of the scratch failed");
  return fvq_nvfp4_linear(x, rows, lin, y, scratch, kNoAllocScratchBytes, stream);
}

}  // extern "C"
