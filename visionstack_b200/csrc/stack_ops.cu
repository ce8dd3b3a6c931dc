// Fused elementwise steps of the hybrid stack's layers around the token
// mixer, for bf16 activations: each replaces a chain of four or five PyTorch
// kernels (dtype copies, the weight offset, the norm, the residual add) that
// dominated the decode step's small-kernel time.
//
// * rms_norm_zc: the zero-centred RMSNorm of Qwen3_5RMSNorm (config.py:118-127):
//   y = bf16( x * rsqrt(mean(x^2) + eps) * (1 + w) ), all in fp32, optionally
//   after a residual add h = bf16(x + delta) (text.py:233-276: the residual
//   stream stays in the activation dtype), which is also written out.  A row
//   takes as many threads as it has 16-byte units (up to a whole 256-thread
//   block for the 2048-wide hidden rows, a warp for the 256-wide head rows),
//   its values held in registers between the sum of squares and the scaling;
//   rows may be strided (the per-head q / k norms read every other
//   256-element run of the query projection).
// * silu_mul: the gated MLP's act(gate) * up (text.py:215-230) with torch's
//   two roundings: bf16( bf16(silu(gate)) * up ).
#include <cuda_bf16.h>

#include "gdn_kernels.cuh"

namespace gdn {
namespace sops {

constexpr int NT = 256;

__device__ __forceinline__ void unpack8(const uint4 v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        f[2 * e] = __uint_as_float(w[e] << 16);
        f[2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
    }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 t = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
        w[e] = *reinterpret_cast<const uint32_t*>(&t);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// TPR threads per row (a power of two, 32..256), NT / TPR rows per block; each thread keeps its at
// most UPT 16-byte units of the row in registers between the sum of squares and the scaling.
constexpr int UPT = 8;
template <int TPR>
__global__ void __launch_bounds__(NT) rms_norm_zc_kernel(const RmsNormArgs a) {
    constexpr int RPB = NT / TPR, WPR = TPR / 32;
    __shared__ float part[NT / 32];
    const int r_in = threadIdx.x / TPR, t = threadIdx.x % TPR;
    const long long row = (long long)blockIdx.x * RPB + r_in;
    const bool live = row < a.rows;
    const int units = a.dim / 8;
    const long long rr = live ? row : 0;
    const uint4* x = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.x) + rr * a.x_stride);
    const uint4* d = a.delta ? reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.delta) +
                                                              rr * a.delta_stride)
                             : nullptr;
    uint4* res = a.res ? reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.res) + rr * a.res_stride) : nullptr;
    uint4 v[UPT];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < UPT; ++j) {
        const int u = t + j * TPR;
        if (!live || u >= units) continue;
        v[j] = x[u];
        float f[8];
        unpack8(v[j], f);
        if (d) {
            float g[8];
            unpack8(d[u], g);
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] += g[e];
            v[j] = pack8(f);  // the residual stream in bf16
            unpack8(v[j], f);
            res[u] = v[j];
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (WPR > 1) {
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
        __syncthreads();
        ss = 0.f;
#pragma unroll
        for (int w = 0; w < WPR; ++w) ss += part[r_in * WPR + w];
    }
    if (!live) return;
    const float r = rsqrtf(ss / (float)a.dim + a.eps);
    const uint4* w = static_cast<const uint4*>(a.w);
    uint4* out = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) + row * a.out_stride);
#pragma unroll
    for (int j = 0; j < UPT; ++j) {
        const int u = t + j * TPR;
        if (u >= units) continue;
        float f[8], g[8];
        unpack8(v[j], f);
        unpack8(w[u], g);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = (f[e] * r) * (1.0f + g[e]);
        out[u] = pack8(f);
    }
}

__global__ void __launch_bounds__(NT) silu_mul_kernel(const uint4* __restrict__ gate, const uint4* __restrict__ up,
                                                      uint4* __restrict__ out, long long units) {
    for (long long i = (long long)blockIdx.x * NT + threadIdx.x; i < units; i += (long long)gridDim.x * NT) {
        float g[8], u[8];
        unpack8(gate[i], g);
        unpack8(up[i], u);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float s = __bfloat162float(__float2bfloat16_rn(g[e] / (1.0f + expf(-g[e]))));
            g[e] = s * u[e];
        }
        out[i] = pack8(g);
    }
}

}  // namespace sops

cudaError_t launch_rms_norm_zc(const RmsNormArgs& a, cudaStream_t s) {
    // threads per row: the row's 16-byte units rounded up to a power of two, 32..256
    const int units = a.dim / 8;
    int tpr = 32;
    while (tpr < units && tpr < sops::NT) tpr *= 2;
    if ((units + tpr - 1) / tpr > sops::UPT) return cudaErrorInvalidValue;
    const long long rpb = sops::NT / tpr, blocks = (a.rows + rpb - 1) / rpb;
    switch (tpr) {
        case 32: sops::rms_norm_zc_kernel<32><<<(unsigned)blocks, sops::NT, 0, s>>>(a); break;
        case 64: sops::rms_norm_zc_kernel<64><<<(unsigned)blocks, sops::NT, 0, s>>>(a); break;
        case 128: sops::rms_norm_zc_kernel<128><<<(unsigned)blocks, sops::NT, 0, s>>>(a); break;
        default: sops::rms_norm_zc_kernel<256><<<(unsigned)blocks, sops::NT, 0, s>>>(a); break;
    }
    return cudaGetLastError();
}

cudaError_t launch_silu_mul(const void* gate, const void* up, void* out, long long n, cudaStream_t s) {
    const long long units = n / 8;
    long long blocks = (units + sops::NT - 1) / sops::NT;
    if (blocks > 148 * 16) blocks = 148 * 16;
    sops::silu_mul_kernel<<<(unsigned)blocks, sops::NT, 0, s>>>(static_cast<const uint4*>(gate),
                                                                 static_cast<const uint4*>(up),
                                                                 static_cast<uint4*>(out), units);
    return cudaGetLastError();
}

}  // namespace gdn
