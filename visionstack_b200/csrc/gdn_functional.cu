// Stand-alone kernels behind two names of the reference's functional boundary
// that the fused token mixer otherwise computes inside its own kernels:
//
//  * the unit lower triangular solve (I + tril(U, -1))^-1 R of
//    _solve_unit_lower_triangular / _invert_unit_lower_triangular_block
//    (ShadowBoxer/models/qwen35/deltanet.py:93-162).  The reference builds the
//    inverse from 16x16 diagonal blocks by Neumann-series products and merges
//    them pairwise (T21 = -T22 U21 T11); here each right-hand-side column is
//    solved by forward substitution in fp32 (x_i = r_i - sum_{k<i} U_ik x_k),
//    the same linear map up to float rounding.  One thread per column, the
//    strictly lower triangle of U staged in shared memory;
//  * the gated RMSNorm of Qwen3_5RMSNormGated.forward
//    (ShadowBoxer/models/qwen35/config.py:136-143): h * rsqrt(mean(h^2) + eps),
//    rounded to the input dtype, times the weight (rounded again when both are
//    bf16, as torch's bf16 * bf16 product is), times SiLU(gate) in fp32,
//    rounded to the input dtype.  One warp per row.
#include <cuda_bf16.h>

#include "gdn_kernels.cuh"

namespace gdn {
namespace func {

constexpr int TRI_THREADS = 128;
constexpr int TRI_SMEM_MAX_N = 96;  // U staged in shared memory up to 96 x 96 (36 KB)

template <bool kSmem>
__global__ void __launch_bounds__(TRI_THREADS)
    trisolve_kernel(const float* __restrict__ ut, const float* __restrict__ rhs, float* __restrict__ out, int n,
                    int m) {
    extern __shared__ float sU[];
    const long long mat = blockIdx.x;
    const float* U = ut + mat * (long long)n * n;
    if (kSmem) {
        for (int i = threadIdx.x; i < n * n; i += TRI_THREADS) sU[i] = U[i];
        __syncthreads();
    }
    const int col = blockIdx.y * TRI_THREADS + threadIdx.x;
    if (col >= m) return;
    const float* R = rhs ? rhs + mat * (long long)n * m : nullptr;
    float* X = out + mat * (long long)n * m;
    for (int i = 0; i < n; ++i) {
        float acc = R ? R[(long long)i * m + col] : (i == col ? 1.0f : 0.0f);
        const float* row = kSmem ? sU + i * n : U + (long long)i * n;
        // two partial sums: a shorter dependency chain, same terms
        float a0 = 0.f, a1 = 0.f;
        int k = 0;
        for (; k + 1 < i; k += 2) {
            a0 = fmaf(row[k], X[(long long)k * m + col], a0);
            a1 = fmaf(row[k + 1], X[(long long)(k + 1) * m + col], a1);
        }
        if (k < i) a0 = fmaf(row[k], X[(long long)k * m + col], a0);
        X[(long long)i * m + col] = acc - (a0 + a1);
    }
}

template <typename T>
__device__ __forceinline__ float ld_f(const T* p, long long i);
template <>
__device__ __forceinline__ float ld_f<float>(const float* p, long long i) {
    return p[i];
}
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p, long long i) {
    return __bfloat162float(p[i]);
}

__device__ __forceinline__ float round_to(float x, int dtype) {
    return dtype == GDN_DTYPE_BF16 ? __bfloat162float(__float2bfloat16_rn(x)) : x;
}

// one warp per row; dims up to any size (strided over the lanes)
template <typename TX, typename TG, typename TW>
__global__ void __launch_bounds__(256)
    rms_norm_gated_kernel(const TX* __restrict__ x, const TG* __restrict__ gate, const TW* __restrict__ w,
                          TX* __restrict__ out, long long rows, int dim, float eps, int x_dtype, int round_prod) {
    const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const TX* xr = x + row * dim;
    const TG* gr = gate + row * dim;
    TX* orow = out + row * dim;
    float ss = 0.f;
    for (int j = lane; j < dim; j += 32) {
        const float h = ld_f<TX>(xr, j);
        ss = fmaf(h, h, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rstd = rsqrtf(ss / (float)dim + eps);
    for (int j = lane; j < dim; j += 32) {
        const float normed = round_to(ld_f<TX>(xr, j) * rstd, x_dtype);
        float scaled = ld_f<TW>(w, j) * normed;
        if (round_prod) scaled = round_to(scaled, GDN_DTYPE_BF16);
        const float g = ld_f<TG>(gr, j);
        const float gated = scaled * (g / (1.0f + expf(-g)));
        if constexpr (sizeof(TX) == 2)
            orow[j] = __float2bfloat16_rn(gated);
        else
            orow[j] = gated;
    }
}

template <typename TX, typename TG, typename TW>
cudaError_t launch_norm_t(const void* x, const void* gate, const void* w, void* out, long long rows, int dim,
                          float eps, int x_dtype, int round_prod, cudaStream_t s) {
    const long long grid = (rows + 7) / 8;
    rms_norm_gated_kernel<TX, TG, TW><<<(unsigned)grid, 256, 0, s>>>(
        static_cast<const TX*>(x), static_cast<const TG*>(gate), static_cast<const TW*>(w), static_cast<TX*>(out),
        rows, dim, eps, x_dtype, round_prod);
    return cudaGetLastError();
}

}  // namespace func

cudaError_t launch_trisolve(const float* ut, const float* rhs, float* out, long long batch, int n, int m,
                            cudaStream_t s) {
    const dim3 grid((unsigned)batch, (unsigned)((m + func::TRI_THREADS - 1) / func::TRI_THREADS));
    if (n <= func::TRI_SMEM_MAX_N) {
        func::trisolve_kernel<true><<<grid, func::TRI_THREADS, (size_t)n * n * sizeof(float), s>>>(ut, rhs, out, n,
                                                                                                  m);
    } else {
        func::trisolve_kernel<false><<<grid, func::TRI_THREADS, 0, s>>>(ut, rhs, out, n, m);
    }
    return cudaGetLastError();
}

cudaError_t launch_rms_norm_gated(const void* x, const void* gate, const void* w, void* out, long long rows, int dim,
                                  float eps, int x_dtype, int gate_dtype, int w_dtype, cudaStream_t s) {
    using bf = __nv_bfloat16;
    const int round_prod = (x_dtype == GDN_DTYPE_BF16 && w_dtype == GDN_DTYPE_BF16) ? 1 : 0;
    const bool xb = x_dtype == GDN_DTYPE_BF16, gb = gate_dtype == GDN_DTYPE_BF16, wb = w_dtype == GDN_DTYPE_BF16;
    if (xb) {
        if (gb) return wb ? func::launch_norm_t<bf, bf, bf>(x, gate, w, out, rows, dim, eps, x_dtype, round_prod, s)
                          : func::launch_norm_t<bf, bf, float>(x, gate, w, out, rows, dim, eps, x_dtype, round_prod, s);
        return wb ? func::launch_norm_t<bf, float, bf>(x, gate, w, out, rows, dim, eps, x_dtype, round_prod, s)
                  : func::launch_norm_t<bf, float, float>(x, gate, w, out, rows, dim, eps, x_dtype, round_prod, s);
    }
    if (gb) return wb ? func::launch_norm_t<float, bf, bf>(x, gate, w, out, rows, dim, eps, x_dtype, round_prod, s)
                      : func::launch_norm_t<float, bf, float>(x, gate, w, out, rows, dim, eps, x_dtype, round_prod, s);
    return wb ? func::launch_norm_t<float, float, bf>(x, gate, w, out, rows, dim, eps, x_dtype, round_prod, s)
              : func::launch_norm_t<float, float, float>(x, gate, w, out, rows, dim, eps, x_dtype, round_prod, s);
}

}  // namespace gdn
