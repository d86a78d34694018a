// vw_static.cu -- the fixed device scratch of vw_sample_static, for callers that must not allocate device memory
// (an allocator-less host runtime, a process that owns all free memory through its own pool, a caller inside an
// allocation-free region).  The array lives in this file's own module, so a process that never calls
// vw_sample_static never loads it (with CUDA's default lazy module loading).

#include <cuda_runtime.h>

#include "vw_internal.h"

namespace vw {

static_assert(kStaticMaxVocab >= kRegElems * kThreads && (kStaticMaxVocab & (kStaticMaxVocab - 1)) == 0,
              "the per-CTA slice formula assumes a power-of-two vocabulary bound of at least one register row");
static_assert(kStaticScratchOffset % 256 == 0 && kStaticCtaStride % 256 == 0, "slices stay 256-byte aligned");

// Error word, deferred-list counters, deferred rows and the whole-row kernel's per-CTA slices (see vw_internal.h).
static __device__ __align__(256) char g_static_scratch[kStaticBytes];

cudaError_t static_scratch_address(char** ptr) {
    return cudaGetSymbolAddress(reinterpret_cast<void**>(ptr), g_static_scratch);
}

}  // namespace vw
