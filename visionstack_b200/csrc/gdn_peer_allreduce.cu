// One-shot all-reduce (sum) of a small bf16 tensor across the GPUs of one
// node over NVLink peer memory: the exchange step of the value-head-sharded
// layers (the row-parallel out_proj / o_proj / down_proj partials, a few
// hundred KB per decode step), where a ring all-reduce is bound by its
// per-step latency rather than by bandwidth.
//
// Every rank holds one staging allocation, mapped into every other rank's
// address space by CUDA IPC (plain peer stores; no multicast):
//   data     bf16 [2][world][cap]    two slots (call parity) of every rank's partial
//   flags    int32 [world][nblocks]  flags[r][b] = last epoch rank r announced for block b
//   counters int32 [nblocks]         epochs of this rank's calls, per block
// Block b of a call owns elements [b * chunk, (b + 1) * chunk) and runs on
// its own: its epoch e = counters[b] + 1 (so a call captured in a CUDA graph
// advances on every replay).  It pushes the local partial's range into
// data[e & 1][rank] of every rank (posted stores over NVLink: nothing waits
// for a round trip), release-stores e into flags[rank][b] of every rank
// (ordered after the data on the same link), waits (bounded) until
// flags[r][b] >= e for every rank r, then sums the range of every rank's
// partial from its own memory in rank order 0..world-1 in fp32 (so every
// rank gets the same bits) and writes it to the output.  A slot is rewritten
// only two calls later, after every rank announced the call in between, which
// it does only after its reads of the earlier call: one flag exchange per
// call.  A wait that runs out sets GDN_DEVERR_PEER_TIMEOUT and the block
// returns; the group's epochs then disagree and the staging memory must be
// rebuilt.
#include <cuda_bf16.h>

#include "gdn_async.cuh"
#include "gdn_kernels.cuh"

namespace gdn {
namespace par {

constexpr int NT = 256;

__device__ __forceinline__ void st_release_sys(int* p, int v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(NT) peer_allreduce_kernel(const PeerAllReduceArgs a) {
    const int b = blockIdx.x, tid = threadIdx.x;
    const int epoch = a.counters[b] + 1;
    const long long slot_off = (long long)(epoch & 1) * a.world * a.cap;
    // 8-element (16-byte) units; n is a multiple of 8
    const long long units = a.n / 8, per = (units + a.nblocks - 1) / a.nblocks;
    const long long u0 = (long long)b * per < units ? (long long)b * per : units;
    const long long u1 = u0 + per < units ? u0 + per : units;
    const uint4* in = static_cast<const uint4*>(a.in);
    // this rank's partial into its row of the slot, on every rank
    const long long row_off = slot_off + (long long)a.rank * a.cap;
    for (long long u = u0 + tid; u < u1; u += NT) {
        const uint4 v = in[u];
        for (int r = 0; r < a.world; ++r) reinterpret_cast<uint4*>(a.data[r] + row_off)[u] = v;
    }
    __syncthreads();
    bool ok = true;
    if (tid < a.world) {
        // release at system scope: with the barrier above it orders every thread's pushed ranges
        // before the flag on the peer (a release is cumulative over what happens before it)
        st_release_sys(a.flags[tid] + a.rank * a.nblocks + b, epoch);
        const int* f = a.flags[a.rank] + tid * a.nblocks + b;
        if (ld_acquire_sys(f) < epoch) {
            const uint64_t t0 = global_timer_ns();
            for (uint32_t it = 1;; ++it) {
                if (ld_acquire_sys(f) >= epoch) break;
                if ((it & 63u) == 0u && global_timer_ns() - t0 > GDN_WAIT_LIMIT_NS) {
                    atomicOr(&g_device_error, GDN_DEVERR_PEER_TIMEOUT);
                    ok = false;
                    break;
                }
            }
        }
    }
    if (!__syncthreads_and(ok)) return;
    const uint16_t* own = a.data[a.rank] + slot_off;
    for (long long u = u0 + tid; u < u1; u += NT) {
        float acc[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = 0.f;
        for (int r = 0; r < a.world; ++r) {
            // .cv: fetched again on every call (the other GPUs rewrote it since the last one)
            const uint4 v = __ldcv(reinterpret_cast<const uint4*>(own + (long long)r * a.cap) + u);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                acc[2 * e] += __uint_as_float(w[e] << 16);
                acc[2 * e + 1] += __uint_as_float(w[e] & 0xFFFF0000u);
            }
        }
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const __nv_bfloat162 t = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
            o[e] = *reinterpret_cast<const uint32_t*>(&t);
        }
        static_cast<uint4*>(a.out)[u] = make_uint4(o[0], o[1], o[2], o[3]);
    }
    if (tid == 0) a.counters[b] = epoch;
}

}  // namespace par

cudaError_t launch_peer_allreduce(const PeerAllReduceArgs& a, cudaStream_t s) {
    par::peer_allreduce_kernel<<<a.nblocks, par::NT, 0, s>>>(a);
    return cudaGetLastError();
}

unsigned int peer_allreduce_device_error(bool clear) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
    if (clear && v) {
        const unsigned int zero = 0;
        cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
    }
    return v;
}

}  // namespace gdn
