// Single-token grouped-query attention against a fixed-capacity KV buffer, for the decode steps
// of the hybrid stack's full-attention layers (ShadowBoxer/models/qwen35/text.py:160-212 with one
// query token): o = softmax(scale q K^T) V over the keys 0..pos, where pos is read on the device,
// so one captured launch serves every step.
//
// Split-KV in two kernels.  attn_split_kernel: one CTA per (key range, KV head, batch row); each
// warp walks blocks of 32 keys, a lane scoring one key against the G queries of the KV head
// (its key row read once, the queries from shared memory), an online softmax per query in the
// log2 domain, then the 32 keys' value rows accumulated with a lane holding HD/32 dims of all G
// outputs.  The warps' partial (max, sum, output) merge in shared memory into one partial per
// CTA.  attn_combine_kernel merges the key ranges and writes bf16.  HBM-bound: every key and
// value row is read once.
#include <cuda_bf16.h>
#include <math_constants.h>

#include "gdn_kernels.cuh"

namespace gdn {
namespace attn {

constexpr int NT = 256, NW = NT / 32, KB = 32;

template <int HD>
struct Row;  // HD/32 bf16 of a row per lane
template <>
struct Row<64> {
    using T = unsigned int;
};
template <>
struct Row<128> {
    using T = uint2;
};
template <>
struct Row<256> {
    using T = uint4;
};

// two bf16 packed in a word -> two floats (a bf16 is the upper half of its float)
__device__ __forceinline__ void unpack2(unsigned int w, float& a, float& b) {
    a = __uint_as_float(w << 16);
    b = __uint_as_float(w & 0xffff0000u);
}

template <int N>
__device__ __forceinline__ void unpack_row(const typename Row<N * 32>::T& r, float* f);
template <>
__device__ __forceinline__ void unpack_row<2>(const unsigned int& r, float* f) {
    unpack2(r, f[0], f[1]);
}
template <>
__device__ __forceinline__ void unpack_row<4>(const uint2& r, float* f) {
    unpack2(r.x, f[0], f[1]);
    unpack2(r.y, f[2], f[3]);
}
template <>
__device__ __forceinline__ void unpack_row<8>(const uint4& r, float* f) {
    unpack2(r.x, f[0], f[1]);
    unpack2(r.y, f[2], f[3]);
    unpack2(r.z, f[4], f[5]);
    unpack2(r.w, f[6], f[7]);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// shared memory of attn_split_kernel, in floats
template <int HD, int G>
struct Smem {
    static constexpr int Q = 0;                  // [G][HD] query * scale * log2(e)
    static constexpr int P = Q + G * HD;         // [NW][KB][G] probabilities of a warp's block
    static constexpr int ML = P + NW * KB * G;   // [NW][G][2] warp max / sum
    static constexpr int ACC = ML + NW * G * 2;  // [NW][G][HD] warp outputs
    static constexpr int FLOATS = ACC + NW * G * HD;
};

template <int HD, int G>
__global__ void __launch_bounds__(NT, 2) attn_split_kernel(const __nv_bfloat16* __restrict__ q,
                                                           const __nv_bfloat16* __restrict__ kbuf,
                                                           const __nv_bfloat16* __restrict__ vbuf,
                                                           const long long* __restrict__ pos, int cap, int span,
                                                           float qscale, float* __restrict__ part_o,
                                                           float* __restrict__ part_ml) {
    using SM = Smem<HD, G>;
    constexpr int DL = HD / 32;  // dims per lane
    extern __shared__ float sm[];
    const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int S = gridDim.x, KVH = gridDim.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long last = pos[0];
    const int n_valid = last < 0 ? 0 : (int)min((long long)cap, last + 1);
    const int k0 = s * span, k1 = min(k0 + span, n_valid);
    const size_t head = (size_t)b * KVH + h;
    float* po = part_o + ((head * S + s) * G) * HD;
    float* pml = part_ml + (head * S + s) * G * 2;

    if (k0 >= k1) {  // no keys in this range
        for (int i = threadIdx.x; i < G; i += NT) {
            pml[2 * i] = -CUDART_INF_F;
            pml[2 * i + 1] = 0.f;
        }
        return;
    }
    for (int i = threadIdx.x; i < G * HD; i += NT)
        sm[SM::Q + i] = __bfloat162float(q[head * G * HD + i]) * qscale;
    __syncthreads();

    const __nv_bfloat16* kh = kbuf + head * (size_t)cap * HD;
    const __nv_bfloat16* vh = vbuf + head * (size_t)cap * HD;
    float m[G], l[G], acc[G][DL];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -CUDART_INF_F;
        l[g] = 0.f;
#pragma unroll
        for (int i = 0; i < DL; ++i) acc[g][i] = 0.f;
    }
    float* sp = sm + SM::P + warp * KB * G;
    for (int blk = k0 + warp * KB; blk < k1; blk += NW * KB) {
        // scores of key blk + lane (log2 domain), -inf past the valid keys
        const int kk = blk + lane;
        float sc[G];
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g] = 0.f;
        if (kk < k1) {
            const uint4* kr = reinterpret_cast<const uint4*>(kh + (size_t)kk * HD);
#pragma unroll 4
            for (int c = 0; c < HD / 8; ++c) {
                float kf[8];
                unpack_row<8>(__ldg(kr + c), kf);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float4 qa = *reinterpret_cast<const float4*>(sm + SM::Q + g * HD + c * 8);
                    const float4 qb = *reinterpret_cast<const float4*>(sm + SM::Q + g * HD + c * 8 + 4);
                    float t = sc[g];
                    t = fmaf(qa.x, kf[0], t);
                    t = fmaf(qa.y, kf[1], t);
                    t = fmaf(qa.z, kf[2], t);
                    t = fmaf(qa.w, kf[3], t);
                    t = fmaf(qb.x, kf[4], t);
                    t = fmaf(qb.y, kf[5], t);
                    t = fmaf(qb.z, kf[6], t);
                    t = fmaf(qb.w, kf[7], t);
                    sc[g] = t;
                }
            }
        } else {
#pragma unroll
            for (int g = 0; g < G; ++g) sc[g] = -CUDART_INF_F;
        }
        // online softmax per query over this block (lane 0's key is always valid)
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float mn = fmaxf(m[g], warp_max(sc[g]));
            const float corr = exp2f(m[g] - mn);
            const float p = exp2f(sc[g] - mn);
            l[g] = l[g] * corr + warp_sum(p);
            m[g] = mn;
#pragma unroll
            for (int i = 0; i < DL; ++i) acc[g][i] *= corr;
            sp[lane * G + g] = p;
        }
        __syncwarp();
        const int nk = min(KB, k1 - blk);
        for (int j = 0; j < nk; ++j) {
            float vf[DL];
            unpack_row<DL>(__ldg(reinterpret_cast<const typename Row<HD>::T*>(vh + (size_t)(blk + j) * HD) + lane),
                           vf);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float p = sp[j * G + g];
#pragma unroll
                for (int i = 0; i < DL; ++i) acc[g][i] = fmaf(p, vf[i], acc[g][i]);
            }
        }
        __syncwarp();
    }

    // merge the warps: common max per query, then the scaled sums
    if (lane == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            sm[SM::ML + (warp * G + g) * 2] = m[g];
            sm[SM::ML + (warp * G + g) * 2 + 1] = l[g];
        }
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float M = -CUDART_INF_F;
        for (int w = 0; w < NW; ++w) M = fmaxf(M, sm[SM::ML + (w * G + g) * 2]);
        const float f = m[g] == -CUDART_INF_F ? 0.f : exp2f(m[g] - M);
#pragma unroll
        for (int i = 0; i < DL; ++i) sm[SM::ACC + (warp * G + g) * HD + lane * DL + i] = acc[g][i] * f;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < G * HD; e += NT) {
        float t = 0.f;
        for (int w = 0; w < NW; ++w) t += sm[SM::ACC + w * G * HD + e];
        po[e] = t;
    }
    if (threadIdx.x < G) {
        const int g = threadIdx.x;
        float M = -CUDART_INF_F;
        for (int w = 0; w < NW; ++w) M = fmaxf(M, sm[SM::ML + (w * G + g) * 2]);
        float L = 0.f;
        for (int w = 0; w < NW; ++w) {
            const float mw = sm[SM::ML + (w * G + g) * 2];
            if (mw != -CUDART_INF_F) L += sm[SM::ML + (w * G + g) * 2 + 1] * exp2f(mw - M);
        }
        pml[2 * g] = M;
        pml[2 * g + 1] = L;
    }
}

// one CTA per (query head, batch row): merge the key ranges, normalise, round to bf16.
// Query head hq = kv head * G + g; partials are [B][KVH][S][G][...].
template <int HD>
__global__ void __launch_bounds__(HD) attn_combine_kernel(const float* __restrict__ part_o,
                                                          const float* __restrict__ part_ml, int S, int G,
                                                          __nv_bfloat16* __restrict__ out) {
    const int hq = blockIdx.x, b = blockIdx.y, Hq = gridDim.x;
    const int d = threadIdx.x;
    const int h = hq / G, g = hq % G;
    const size_t base = ((size_t)b * (Hq / G) + h) * S;
    float M = -CUDART_INF_F;
    for (int s = 0; s < S; ++s) M = fmaxf(M, part_ml[((base + s) * G + g) * 2]);
    float L = 0.f, o = 0.f;
    if (M != -CUDART_INF_F) {
        for (int s = 0; s < S; ++s) {
            const float ms = part_ml[((base + s) * G + g) * 2];
            if (ms == -CUDART_INF_F) continue;
            const float f = exp2f(ms - M);
            L += part_ml[((base + s) * G + g) * 2 + 1] * f;
            o += part_o[((base + s) * G + g) * HD + d] * f;
        }
    }
    out[((size_t)b * Hq + hq) * HD + d] = __float2bfloat16_rn(L > 0.f ? o / L : 0.f);
}

template <int HD, int G>
cudaError_t launch_t(const AttnDecodeArgs& a, cudaStream_t st) {
    const int bytes = Smem<HD, G>::FLOATS * 4;
    cudaError_t e = cudaFuncSetAttribute(attn_split_kernel<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    attn_split_kernel<HD, G><<<dim3(a.splits, a.kv_heads, a.batch), NT, bytes, st>>>(
        static_cast<const __nv_bfloat16*>(a.q), static_cast<const __nv_bfloat16*>(a.k),
        static_cast<const __nv_bfloat16*>(a.v), a.pos, a.capacity, a.span, a.qscale, a.part_o, a.part_ml);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    attn_combine_kernel<HD><<<dim3(a.kv_heads * G, a.batch), HD, 0, st>>>(a.part_o, a.part_ml, a.splits, G,
                                                                        static_cast<__nv_bfloat16*>(a.out));
    return cudaGetLastError();
}

template <int HD>
cudaError_t launch_hd(const AttnDecodeArgs& a, cudaStream_t st) {
    switch (a.groups) {
        case 1: return launch_t<HD, 1>(a, st);
        case 2: return launch_t<HD, 2>(a, st);
        case 4: return launch_t<HD, 4>(a, st);
        case 8: return launch_t<HD, 8>(a, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace attn

cudaError_t launch_attn_decode(const AttnDecodeArgs& a, cudaStream_t st) {
    switch (a.head_dim) {
        case 64: return attn::launch_hd<64>(a, st);
        case 128: return attn::launch_hd<128>(a, st);
        case 256: return attn::launch_hd<256>(a, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace gdn
