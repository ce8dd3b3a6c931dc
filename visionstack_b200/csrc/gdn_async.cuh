// Bulk asynchronous copies (TMA engine, cp.async.bulk), mbarriers and the
// device error word used by the pipelined kernels (sm_100a inline PTX).
//
// Every wait on an mbarrier is bounded: after GDN_WAIT_LIMIT_NS of global
// time it gives up, records the reason in the device error word and returns
// false, so a kernel never spins forever.  No copy here uses cluster
// multicast: every source is this GPU's own global memory.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gdn_b200.h"  // GDN_DEVERR_* bits

#define GDN_WAIT_LIMIT_NS 1000000000ull  // 1 s

namespace gdn {

// Sticky per-device error word.  Each translation unit that includes this
// header has its own copy; it exposes a host reader (see gdn_kernels.cuh)
// that the C ABI combines in gdn_device_error().
static __device__ unsigned int g_device_error;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) accesses of the same memory.
// Programmatic dependent launch.  A kernel launched by launch_pdl may start while the
// previous kernel of its stream is still finishing (once every CTA of that kernel has called
// pdl_launch_dependents or exited); pdl_wait blocks until that kernel has completed and its
// memory operations are visible.  Launched any other way, both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for phase `parity` of the mbarrier; false after the limit.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, unsigned int err_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0u && global_timer_ns() - t0 > GDN_WAIT_LIMIT_NS) {
            atomicOr(&g_device_error, err_flag);
            return false;
        }
    }
}

// Invalidate an mbarrier (before it is initialised again for reuse).
__device__ __forceinline__ void mbar_inval(uint32_t bar) {
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

// A flag in global memory that another CTA of the same grid sets: wait (bounded) until it is
// non-zero, with acquire semantics at GPU scope; false (and GDN_DEVERR_HANDOFF_TIMEOUT) after
// the limit.
__device__ __forceinline__ bool wait_flag_bounded(const int* flag) {
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
        int v;
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if (v != 0) return true;
        if ((it & 63u) == 0u) {
            const uint64_t now = global_timer_ns();
            if (it == 0u) {
                t0 = now;
            } else if (now - t0 > GDN_WAIT_LIMIT_NS) {
                atomicOr(&g_device_error, GDN_DEVERR_HANDOFF_TIMEOUT);
                return false;
            }
        }
        __nanosleep(64);
    }
}
// Set a flag with release semantics at GPU scope (after this thread's writes and, through a
// prior block barrier and fences, its block's).
__device__ __forceinline__ void release_flag(int* flag) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(flag), "r"(1) : "memory");
}

// One bulk copy global -> shared of `bytes` (multiple of 16, both addresses
// 16-byte aligned), completing `bytes` of transaction count on `bar`.
__device__ __forceinline__ void bulk_load(uint32_t dst_smem, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst_smem),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// Tiled tensor copy global -> shared of one 3-D box of `tmap` at element
// coordinates (c0, c1, c2), completing its bytes on `bar`.  c0 * element size
// must be a multiple of 16 bytes; out-of-range rows are filled with zeros.
// Bring a kernel-parameter tensor map into the descriptor cache ahead of its first copy.
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst_smem, const void* tmap, int c0, int c1, int c2,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(dst_smem),
        "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
        : "memory");
}

// Tiled tensor copy shared -> global of one 3-D box of `tmap` at element
// coordinates (c0, c1, c2) (c0 * element size a multiple of 16 bytes, no
// negative coordinates), tracked by this thread's bulk-async group.
__device__ __forceinline__ void tma_store_3d(const void* tmap, uint32_t src_smem, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(tmap), "r"(c0),
        "r"(c1), "r"(c2), "r"(src_smem)
        : "memory");
}
// One bulk copy shared -> global of `bytes` (multiple of 16, both addresses
// 16-byte aligned), tracked by this thread's bulk-async group.
__device__ __forceinline__ void bulk_store(void* dst, uint32_t src_smem, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src_smem), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until every committed bulk store of this thread has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_group_read0() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until every committed bulk store of this thread has completed.
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

}  // namespace gdn
