// gdn_mixer_prefill_noalloc: the chunked prefill with its scratch in a fixed
// device array of this library instead of a caller-provided workspace, so the
// call allocates nothing.
//
// The scratch is one file-scope __device__ array of GDN_STATIC_SCRATCH_BYTES.
// It belongs to this library's module: once the module is loaded on a device
// (at library load under CUDA_MODULE_LOADING=EAGER, at the first kernel launch
// under the default lazy loading) the array occupies that much device memory
// until the process exits, whether or not this entry is ever called.  Its
// address is looked up with cudaGetSymbolAddress on every call (cheap next to
// a prefill), so a context that was torn down and made again is handled.
//
// Every call on a device uses the same array: calls whose kernels can overlap
// on one device (different streams, or host threads without ordering between
// them) race on it and corrupt each other's results, so such calls must be
// serialised by the caller (one stream, or events).  What must start at zero
// is cleared by the call itself: the sequential kernel's state hand-off flags
// are zeroed by a cudaMemsetAsync in its launcher on every call, before the
// kernel runs (that memset is what makes reusing the array safe); everything
// else the kernels read is written earlier in the same call.
#include "gdn_kernels.cuh"

namespace gdn {
namespace {

__device__ __align__(256) unsigned char g_prefill_scratch[GDN_STATIC_SCRATCH_BYTES];

}  // namespace

cudaError_t static_prefill_scratch(void** addr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_prefill_scratch);
    if (e != cudaSuccess) return e;
    if (!p) return cudaErrorInvalidSymbol;
    *addr = p;
    return cudaSuccess;
}

}  // namespace gdn
