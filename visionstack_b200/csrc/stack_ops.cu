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
// * qk_norm_rope: the gated attention's per-head q / k RMSNorm followed by the
//   partial rotary embedding (text.py:76-86, 140-156), one warp per (token,
//   head) row: the norm rounded to bf16, then for the first `rot` channels
//   bf16(bf16(x * cos) + bf16(rotate_half(x) * sin)) (rotate_half: the
//   partner half-range, negated in the first half; the partner's values come
//   by warp shuffle), written in the [B, heads, T, hd] layout the attention reads.
// * gate_out: attn.transpose(1, 2).reshape(B, T, H hd) * sigmoid(gate)
//   (text.py:204-209): bf16(o * bf16(sigmoid(g))) in the [B, T, H hd] layout.
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

__global__ void __launch_bounds__(NT) qk_norm_rope_kernel(const QkRopeArgs a) {
    const long long row = (long long)blockIdx.x * (NT / 32) + (threadIdx.x >> 5);
    const long long q_rows = (long long)a.B * a.T * a.H, k_rows = (long long)a.B * a.T * a.KVH;
    if (row >= q_rows + k_rows) return;
    const int lane = threadIdx.x & 31, units = a.hd / 8, half_u = a.rot / 16;
    const bool is_q = row < q_rows;
    const long long rr = is_q ? row : row - q_rows;
    const int heads = is_q ? a.H : a.KVH;
    const int h = (int)(rr % heads);
    const long long bt = rr / heads;  // b * T + t
    const int t = (int)(bt % a.T), b = (int)(bt / a.T);
    const __nv_bfloat16* src = is_q ? static_cast<const __nv_bfloat16*>(a.qg) + rr * (2 * a.hd)
                                    : static_cast<const __nv_bfloat16*>(a.k) + rr * a.hd;
    const uint4* w = static_cast<const uint4*>(is_q ? a.qw : a.kw);
    float f[8];
    float ss = 0.f;
    if (lane < units) {
        unpack8(reinterpret_cast<const uint4*>(src)[lane], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss / (float)a.hd + a.eps);
    uint4 y = make_uint4(0u, 0u, 0u, 0u);
    if (lane < units) {
        float g[8];
        unpack8(w[lane], g);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = (f[e] * r) * (1.0f + g[e]);
        y = pack8(f);  // the norm's output, rounded to bf16
    }
    // rotary: units below rot / 8 pair unit u with u +- rot / 16
    const int partner = lane < half_u ? lane + half_u : (lane < 2 * half_u ? lane - half_u : lane);
    uint4 pv;
    pv.x = __shfl_sync(0xffffffffu, y.x, partner);
    pv.y = __shfl_sync(0xffffffffu, y.y, partner);
    pv.z = __shfl_sync(0xffffffffu, y.z, partner);
    pv.w = __shfl_sync(0xffffffffu, y.w, partner);
    if (lane >= units) return;
    if (lane < 2 * half_u) {
        float x[8], p[8], c[8], sn[8];
        unpack8(y, x);
        unpack8(pv, p);
        const long long cs = ((long long)b * a.T + t) * a.rot + 8 * lane;
        unpack8(*reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.cos) + cs), c);
        unpack8(*reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.sin) + cs), sn);
        const float sign = lane < half_u ? -1.0f : 1.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float t1 = __bfloat162float(__float2bfloat16_rn(x[e] * c[e]));
            const float t2 = __bfloat162float(__float2bfloat16_rn((sign * p[e]) * sn[e]));
            x[e] = t1 + t2;
        }
        y = pack8(x);
    }
    __nv_bfloat16* dst = is_q ? static_cast<__nv_bfloat16*>(a.q_out) + (((long long)b * a.H + h) * a.T + t) * a.hd
                              : static_cast<__nv_bfloat16*>(a.k_out) + (((long long)b * a.KVH + h) * a.T + t) * a.hd;
    reinterpret_cast<uint4*>(dst)[lane] = y;
}

__global__ void __launch_bounds__(NT) gate_out_kernel(const GateOutArgs a) {
    const int units = a.hd / 8;
    const long long total = (long long)a.B * a.T * a.H * units;
    for (long long i = (long long)blockIdx.x * NT + threadIdx.x; i < total; i += (long long)gridDim.x * NT) {
        const int u = (int)(i % units);
        const long long rest = i / units;
        const int h = (int)(rest % a.H);
        const long long bt = rest / a.H;
        const int t = (int)(bt % a.T), b = (int)(bt / a.T);
        float o[8], g[8];
        unpack8(*reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.o) + b * a.o_sb + h * a.o_sh +
                                                t * a.o_st + 8 * u),
                o);
        unpack8(*reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.qg) + bt * (2LL * a.H * a.hd) +
                                                (long long)h * 2 * a.hd + a.hd + 8 * u),
                g);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] *= __bfloat162float(__float2bfloat16_rn(1.0f / (1.0f + expf(-g[e]))));
        reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) + bt * ((long long)a.H * a.hd) +
                                 (long long)h * a.hd)[u] = pack8(o);
    }
}

}  // namespace sops

cudaError_t launch_qk_norm_rope(const QkRopeArgs& a, cudaStream_t s) {
    const long long rows = (long long)a.B * a.T * (a.H + a.KVH);
    sops::qk_norm_rope_kernel<<<(unsigned)((rows + sops::NT / 32 - 1) / (sops::NT / 32)), sops::NT, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_gate_out(const GateOutArgs& a, cudaStream_t s) {
    const long long units = (long long)a.B * a.T * a.H * (a.hd / 8);
    long long blocks = (units + sops::NT - 1) / sops::NT;
    if (blocks > 148 * 16) blocks = 148 * 16;
    sops::gate_out_kernel<<<(unsigned)blocks, sops::NT, 0, s>>>(a);
    return cudaGetLastError();
}

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
