// gdn_mixer_prefill_noalloc: the two-kernel chunked prefill with its scratch
// in a fixed device array of this library instead of a caller-provided
// workspace, so the call allocates nothing.
//
// The scratch is one file-scope __device__ array of GDN_STATIC_SCRATCH_BYTES
// per device.  Its address is looked up once per device with
// cudaGetSymbolAddress (checked) and cached.  Every call on a device uses the
// same array: calls whose kernels can overlap on one device (different
// streams, or different host threads without ordering between them) race on
// it and corrupt each other's results, so such calls must be serialised by
// the caller (one stream, or events).  Nothing in the scratch needs to start
// at any value: the preparation kernel writes every byte the sequential
// kernel reads, before it reads it.
#include <mutex>

#include "gdn_kernels.cuh"

namespace gdn {
namespace {

__device__ __align__(256) unsigned char g_prefill_scratch[GDN_STATIC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
void* g_scratch_addr[MAX_DEVICES] = {nullptr};
std::mutex g_scratch_mu;

}  // namespace

cudaError_t static_prefill_scratch(void** addr) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= MAX_DEVICES) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_prefill_scratch);
        if (e != cudaSuccess) return e;
        if (!p) return cudaErrorInvalidSymbol;
        g_scratch_addr[dev] = p;
    }
    *addr = g_scratch_addr[dev];
    return cudaSuccess;
}

}  // namespace gdn
