// Acceptance of verified draft tokens on per-row state slots.
//
// After gdn_mixer_verify_slots has written the states after 1..T draft tokens
// of every row into the row's free slots, accepting `a` tokens of row b makes
// slot_table[b][a] the row's starting slot and returns the old starting slot
// to the free columns - a swap of two table entries.  This replaces the
// reference's per-step clone of every state (clone_and_expand) and its copy of
// the selected checkpoint (select_batch_item / extract_checkpoint,
// ShadowBoxer/models/qwen35/cache.py:131-244): the states themselves never
// move.
#include "gdn_async.cuh"
#include "gdn_kernels.cuh"

namespace gdn {
namespace {

__global__ void accept_slots_kernel(const int* __restrict__ accepted, int* __restrict__ table, int B, int n,
                                    int T) {
    pdl_launch_dependents();
    pdl_wait();  // the verify launch before this one reads the table
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const int a = accepted[b];
    if (a < 0 || a > T) {
        atomicOr(&g_device_error, GDN_DEVERR_BAD_SLOT);
        return;
    }
    if (a == 0) return;
    int* row = table + (size_t)b * n;
    const int cur = row[0];
    row[0] = row[a];
    row[a] = cur;
}

}  // namespace

cudaError_t launch_accept_slots(const int* accepted, int* table, int B, int n_slots, int T, cudaStream_t s) {
    const int threads = 128;
    return launch_pdl(accept_slots_kernel, dim3((B + threads - 1) / threads), dim3(threads), 0, s, accepted, table, B,
                      n_slots, T);
}

unsigned int slots_device_error(bool clear) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
    if (clear && v) {
        const unsigned int zero = 0;
        cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
    }
    return v;
}

}  // namespace gdn
