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
//   * the first call in each CUDA context (the device's primary context, or a
//     caller's own driver-API context) resolves the array's device address with
//     cudaGetSymbolAddress, with that context current, and caches it under the
//     context's unique id, so a device reset or another context is looked up
//     again; make that first call before any stream capture;
//   * every call shares the one array: calls that overlap on the GPU (other
//     streams, other host threads) race.  The amax arrival counter inside it
//     starts at zero (static device memory is zero-initialised) and every
//     call re-arms it; everything else is written before it is read.
#include <cuda_runtime.h>

#include "../../include/fvq.h"
#include "fvq_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

fvq::ContextCache g_noalloc_addr;

// Device address of the scratch array in the calling thread's current CUDA context.
// The address belongs to the context (a device reset or a caller's own driver-API
// context loads the library's device image again, possibly elsewhere), so it is
// looked up with cudaGetSymbolAddress once per context and cached under the
// context's unique id.
int noalloc_scratch(void** out) {
  uint64_t ctx = fvq::current_context_id();
  if (ctx != 0 && g_noalloc_addr.get(ctx, out)) return FVQ_OK;
  void* ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress((void**)&ptr, g_noalloc_scratch);
  if (e != cudaSuccess || ptr == nullptr) return FVQ_ECUDA;
  if (ctx == 0) ctx = fvq::current_context_id();  // the lookup made the primary context current
  if (ctx != 0) g_noalloc_addr.put(ctx, ptr);
  *out = ptr;
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
