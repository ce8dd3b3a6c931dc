// Tensor-core self-test: one CTA computes D[128][N] = A * B with kind::tf32
// UMMA for each operand-layout combination the chunked prefill uses, so the
// shared-memory layouts, descriptors and tensor-memory handling of
// gdn_umma.cuh are checked against a host matmul before any model kernel
// relies on them.
//   mode 0: A K-major [128][128], B K-major [64][128]   (D = A B^T, N = 64)
//   mode 1: A K-major [128][128], B MN-major [128][128] (D = A B, K = 128)
//   mode 2: A K-major [128][64],  B MN-major [64][128]  (D = A B, K = 64)
//   mode 3: A MN-major [64][128] (stored k-major rows of A^T), B MN-major [64][128]
//   mode 4: A in tensor memory [128][128], B K-major [128][128] (D = A B^T, N = 128)
//   mode 5: A in tensor memory [128][64],  B K-major [64][64]   (D = A B^T, N = 64)
//   mode 6: A in tensor memory [128][64],  B MN-major [64][128] (D = A B, K = 64)
// and kind::f16 with bf16 operands (inputs rounded to bf16 on the device; A
// packed in pairs in tensor memory, B in the 16-bit 128-byte swizzle a TMA copy
// writes, in regions laid out like the sequential prefill kernel's [k;q] rows):
//   mode 7: A in tensor memory [128][128], B K-major [128][128] (D = A B^T, N = 128)
//   mode 8: A in tensor memory [128][64],  B MN-major [64][128] (D = A B, K = 64;
//           64-element mn atoms 16 KB apart)
// and kind::f16 with both bf16 operands in shared memory:
//   mode 9:  A K-major [128][128] (the [k;q] rows), B MN-major [128][64] (D = A B, N = 64)
//   mode 10: A MN-major [64][128] (k rows read as A^T, 64-element mn atoms 16 KB apart),
//            B MN-major [64][64] (D = A B, K = 64, N = 64)
// Inputs are plain row-major fp32 in global memory: A is [M][K] except for
// the MN-major A of modes 3 and 10 ([K][M]); B is [N][K] for K-major B and [K][N] for MN-major B.
#include <cuda_bf16.h>

#include "gdn_kernels.cuh"
#include "gdn_umma.cuh"

namespace gdn {

namespace {

struct SelfTestShape {
    int K, N, a_mn, b_mn, a_tmem, bf16;
};
constexpr uint32_t MN_ATOM16 = 16384;  // mode 8: stride between 64-element mn atoms

__host__ __device__ inline SelfTestShape selftest_shape(int mode) {
    switch (mode) {
        case 0: return {128, 64, 0, 0, 0, 0};
        case 1: return {128, 128, 0, 1, 0, 0};
        case 2: return {64, 128, 0, 1, 0, 0};
        case 3: return {64, 128, 1, 1, 0, 0};
        case 4: return {128, 128, 0, 0, 1, 0};
        case 5: return {64, 64, 0, 0, 1, 0};
        case 6: return {64, 128, 0, 1, 1, 0};
        case 7: return {128, 128, 0, 0, 1, 1};
        case 8: return {64, 128, 0, 1, 1, 1};
        case 9: return {128, 64, 0, 1, 0, 1};
        default: return {64, 64, 1, 1, 0, 1};
    }
}

__global__ void __launch_bounds__(128, 1) umma_selftest_kernel(int mode, const float* __restrict__ A,
                                                               const float* __restrict__ B, float* __restrict__ D) {
    extern __shared__ unsigned char raw[];
    const SelfTestShape sh = selftest_shape(mode);
    const int M = 128, K = sh.K, N = sh.N;
    const uint32_t raw_addr = smem_u32(raw);
    const uint32_t pad = ((raw_addr + 1023u) & ~1023u) - raw_addr;
    unsigned char* base = raw + pad;
    unsigned char* sA = base;                // M*K*4 bytes
    unsigned char* sB = base + 128 * 128 * 4;  // N*K*4 bytes
    uint64_t* bar = reinterpret_cast<uint64_t*>(base + 2 * 128 * 128 * 4);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(base + 2 * 128 * 128 * 4 + 8);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    for (int i = tid; i < M * K && !sh.a_tmem && sh.bf16; i += 128) {
        const __nv_bfloat16 v = __float2bfloat16_rn(A[i]);
        if (!sh.a_mn) {
            const int m = i / K, k = i % K;
            *reinterpret_cast<__nv_bfloat16*>(sA + umma::kmajor_off16(m, k, M)) = v;
        } else {
            const int k = i / M, m = i % M;
            *reinterpret_cast<__nv_bfloat16*>(sA + umma::mnmajor_off16(k, m, MN_ATOM16)) = v;
        }
    }
    for (int i = tid; i < M * K && !sh.a_tmem && !sh.bf16; i += 128) {
        if (!sh.a_mn) {
            const int m = i / K, k = i % K;
            *reinterpret_cast<float*>(sA + umma::kmajor_off(m, k, M)) = A[i];
        } else {
            const int k = i / M, m = i % M;
            *reinterpret_cast<float*>(sA + umma::mnmajor_off(k, m, K)) = A[i];
        }
    }
    for (int i = tid; i < N * K && sh.bf16; i += 128) {
        const __nv_bfloat16 v = __float2bfloat16_rn(B[i]);
        if (!sh.b_mn) {
            const int n = i / K, k = i % K;
            *reinterpret_cast<__nv_bfloat16*>(sB + umma::kmajor_off16(n, k, N)) = v;
        } else {
            const int k = i / N, n = i % N;
            *reinterpret_cast<__nv_bfloat16*>(sB + umma::mnmajor_off16(k, n, MN_ATOM16)) = v;
        }
    }
    for (int i = tid; i < N * K && !sh.bf16; i += 128) {
        if (!sh.b_mn) {
            const int n = i / K, k = i % K;
            *reinterpret_cast<float*>(sB + umma::kmajor_off(n, k, N)) = B[i];
        } else {
            const int k = i / N, n = i % N;
            *reinterpret_cast<float*>(sB + umma::mnmajor_off(k, n, K)) = B[i];
        }
    }
    fence_proxy_async_smem();
    if (tid == 0) {
        mbar_init(smem_u32(bar), 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        umma::tmem_alloc(smem_u32(tslot), 256);
        umma::tmem_relinquish();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tbase = *tslot;
    constexpr int A_COL = 128;  // A operand columns when A lives in tensor memory
    if (sh.a_tmem && sh.bf16) {
        // row m of A -> lane m, column A_COL + c holds the bf16 pair k = 2c, 2c + 1
        const int row = warp * 32 + lane;
        for (int c0 = 0; c0 < K / 2; c0 += 32) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const __nv_bfloat162 pr = __floats2bfloat162_rn(A[row * K + 2 * (c0 + j)], A[row * K + 2 * (c0 + j) + 1]);
                v[j] = __uint_as_float(*reinterpret_cast<const uint32_t*>(&pr));
            }
            umma::tmem_st32(umma::tmem_addr(tbase, warp * 32, A_COL + c0), v);
        }
        umma::tmem_wait_st();
    } else if (sh.a_tmem) {
        // row m of A -> lane m (warp w writes lanes 32w..32w+31), columns A_COL + k
        const int row = warp * 32 + lane;
        for (int c0 = 0; c0 < K; c0 += 32) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = A[row * K + c0 + j];
            umma::tmem_st32(umma::tmem_addr(tbase, warp * 32, A_COL + c0), v);
        }
        umma::tmem_wait_st();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();

    if (tid == 0 && sh.bf16) {
        const uint32_t idesc = umma::idesc_bf16(M, N, sh.a_mn, sh.b_mn);
        const uint64_t d0 = sh.b_mn ? umma::desc_mnmajor16_0(smem_u32(sB), MN_ATOM16) : umma::desc_kmajor0(smem_u32(sB));
        const uint64_t a0 = sh.a_mn ? umma::desc_mnmajor16_0(smem_u32(sA), MN_ATOM16) : umma::desc_kmajor0(smem_u32(sA));
        for (int kk = 0; kk < K / 16; ++kk) {
            const uint32_t step = sh.b_mn ? umma::mnmajor16_kstep(kk) : umma::kmajor_kstep(kk, N);
            if (sh.a_tmem) {
                umma::mma_bf16_ta(tbase, tbase + A_COL + kk * 8, umma::desc_add(d0, step), idesc, kk > 0 ? 1u : 0u);
            } else {
                const uint32_t astep = sh.a_mn ? umma::mnmajor16_kstep(kk) : umma::kmajor_kstep(kk, M);
                umma::mma_bf16(tbase, umma::desc_add(a0, astep), umma::desc_add(d0, step), idesc, kk > 0 ? 1u : 0u);
            }
        }
        umma::mma_commit(smem_u32(bar));
    } else if (tid == 0) {
        const uint32_t idesc = umma::idesc_tf32(M, N, sh.a_mn, sh.b_mn);
        for (int kk = 0; kk < K / 8; ++kk) {
            const uint64_t db = sh.b_mn ? umma::desc_mnmajor(smem_u32(sB), K, kk) : umma::desc_kmajor(smem_u32(sB), N, kk);
            if (sh.a_tmem) {
                umma::mma_tf32_ta(tbase, tbase + A_COL + kk * 8, db, idesc, kk > 0 ? 1u : 0u);
            } else {
                const uint64_t da =
                    sh.a_mn ? umma::desc_mnmajor(smem_u32(sA), K, kk) : umma::desc_kmajor(smem_u32(sA), M, kk);
                umma::mma_tf32(tbase, da, db, idesc, kk > 0 ? 1u : 0u);
            }
        }
        umma::mma_commit(smem_u32(bar));
    }
    const bool ok = mbar_wait_bounded(smem_u32(bar), 0, GDN_DEVERR_MMA_TIMEOUT);
    umma::fence_after_sync();
    if (ok) {
        for (int c0 = 0; c0 < N; c0 += 32) {
            float v[32];
            umma::tmem_ld32(umma::tmem_addr(tbase, warp * 32, c0), v);
            umma::tmem_wait_ld();
            const int row = warp * 32 + lane;
#pragma unroll
            for (int j = 0; j < 32; ++j) D[row * N + c0 + j] = v[j];
        }
    }
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tbase, 256);
}

// One thread runs one of the kernels' bounded waits on something that never arrives:
// kind 0 an mbarrier with no arrival (GDN_DEVERR_TMA_TIMEOUT after the limit), kind 1 the
// global flag flag[0] (GDN_DEVERR_HANDOFF_TIMEOUT unless flag[0] is already non-zero).
// flag[1] receives 1 when the wait succeeded, 2 when it gave up.
__global__ void __launch_bounds__(32, 1) expired_wait_kernel(int kind, int* flag) {
    __shared__ alignas(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    bool ok;
    if (kind == 0) {
        const uint32_t b = smem_u32(&bar);
        mbar_init(b, 1);
        fence_mbar_init();
        ok = mbar_wait_bounded(b, 0, GDN_DEVERR_TMA_TIMEOUT);
        mbar_inval(b);
    } else {
        ok = wait_flag_bounded(flag);
    }
    flag[1] = ok ? 1 : 2;
}

}  // namespace

cudaError_t launch_expired_wait_selftest(int kind, int* flag, cudaStream_t s) {
    expired_wait_kernel<<<1, 32, 0, s>>>(kind, flag);
    return cudaGetLastError();
}

cudaError_t launch_umma_selftest(int mode, const float* A, const float* B, float* D, cudaStream_t s) {
    const int bytes = 2 * 128 * 128 * 4 + 64 + 1024;
    cudaError_t e = cudaFuncSetAttribute(umma_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    umma_selftest_kernel<<<1, 128, bytes, s>>>(mode, A, B, D);
    return cudaGetLastError();
}

unsigned int umma_device_error(bool clear) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
    if (clear && v) {
        const unsigned int zero = 0;
        cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
    }
    return v;
}

}  // namespace gdn
