// Single-token grouped-query attention against a fixed-capacity KV buffer, for the decode steps
// of the hybrid stack's full-attention layers (ShadowBoxer/models/qwen35/text.py:160-212 with one
// query token): o = softmax(scale q K^T) V over the keys 0..pos, where pos is read on the device,
// so one captured launch serves every step.
//
// Split-KV in two kernels.  attn_split_kernel: one CTA per (key range, KV head, batch row); each
// warp walks blocks of 32 keys: the block's key rows arrive in the warp's shared-memory stage by
// asynchronous 16-byte copies (one latency per block), a lane scores one key against the G
// queries of the KV head (the queries from shared memory, packed fp32x2 arithmetic), the value
// rows follow into the same stage while the online softmax per query runs (log2 domain), and a
// lane accumulates HD/32 dims of all G outputs over the block's value rows.  The warps' partial
// (max, sum, output) merge in shared memory into one partial per CTA.  attn_combine_kernel merges
// the key ranges and writes bf16.  HBM-bound: every key and value row is read once.
#include <cuda_bf16.h>
#include <math_constants.h>

#include "gdn_async.cuh"  // smem_u32
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

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Row r of a warp's stage holds HD bf16 as HD/8 chunks of 16 bytes; chunk c sits at position
// c ^ (r mod HD/8), so a lane per row (the scores) and a row per warp (the values) both read
// without bank conflicts.
template <int HD>
__device__ __forceinline__ uint32_t stage_off(int r, int byte_in_row) {
    constexpr int CH = HD / 8;
    const int c = byte_in_row >> 4;
    return (uint32_t)(r * HD * 2 + ((c ^ (r & (CH - 1))) << 4) + (byte_in_row & 15));
}

// rows blk .. blk+nk-1 of one head's [cap][HD] buffer into the warp's stage (asynchronous)
template <int HD>
__device__ __forceinline__ void stage_rows(uint32_t stage, const __nv_bfloat16* head, int blk, int nk, int lane) {
    constexpr int CH = HD / 8;
    for (int idx = lane; idx < nk * CH; idx += 32) {
        const int r = idx / CH, c = idx % CH;
        cp_async16(stage + stage_off<HD>(r, c * 16), head + (size_t)(blk + r) * HD + c * 8);
    }
    cp_async_commit();
}

// shared memory of attn_split_kernel, in bytes
template <int HD, int G>
struct Smem {
    static constexpr int GP = (G + 1) / 2;                  // query pairs
    static constexpr int STAGE = 0;                         // [NW][KB][HD] bf16 (then [NW][G][HD] f32)
    static constexpr int Q = STAGE + NW * KB * HD * 2;      // [GP][HD] float2: (q_2p[d], q_2p+1[d]) * scale * log2 e
    static constexpr int P = Q + GP * HD * 8;               // [NW][KB][G] f32 probabilities of a warp's block
    static constexpr int ML = P + NW * KB * G * 4;          // [NW][G][2] f32 warp max / sum
    static constexpr int BYTES = ML + NW * G * 2 * 4;
    static_assert(NW * G * HD * 4 <= NW * KB * HD * 2, "the merge area must fit in the stages");
};

template <int HD, int G>
__global__ void __launch_bounds__(NT, 1) attn_split_kernel(const __nv_bfloat16* __restrict__ q,
                                                           const __nv_bfloat16* __restrict__ kbuf,
                                                           const __nv_bfloat16* __restrict__ vbuf,
                                                           const long long* __restrict__ pos, int cap, int span,
                                                           float qscale, float* __restrict__ part_o,
                                                           float* __restrict__ part_ml) {
    using SM = Smem<HD, G>;
    constexpr int GP = SM::GP;
    constexpr int DL = HD / 32;  // value dims per lane
    extern __shared__ __align__(16) unsigned char smem[];
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
    float2* sq = reinterpret_cast<float2*>(smem + SM::Q);
    for (int i = threadIdx.x; i < GP * HD; i += NT) {
        const int pq = i / HD, d = i % HD;
        const float a = __bfloat162float(q[(head * G + 2 * pq) * HD + d]) * qscale;
        const float c = 2 * pq + 1 < G ? __bfloat162float(q[(head * G + 2 * pq + 1) * HD + d]) * qscale : 0.f;
        sq[i] = make_float2(a, c);
    }
    __syncthreads();

    const __nv_bfloat16* kh = kbuf + head * (size_t)cap * HD;
    const __nv_bfloat16* vh = vbuf + head * (size_t)cap * HD;
    const uint32_t stage = smem_u32(smem + SM::STAGE + warp * KB * HD * 2);
    const unsigned char* stage_p = smem + SM::STAGE + warp * KB * HD * 2;
    float* sp = reinterpret_cast<float*>(smem + SM::P) + warp * KB * G;
    float m[G], l[G];
    float2 acc[G][DL / 2];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -CUDART_INF_F;
        l[g] = 0.f;
#pragma unroll
        for (int i = 0; i < DL / 2; ++i) acc[g][i] = make_float2(0.f, 0.f);
    }
    for (int blk = k0 + warp * KB; blk < k1; blk += NW * KB) {
        const int nk = min(KB, k1 - blk);
        stage_rows<HD>(stage, kh, blk, nk, lane);
        cp_async_wait_all();
        __syncwarp();
        // scores of key blk + lane against every query (log2 domain), -inf past the valid keys
        float sc[G];
        if (lane < nk) {
            float2 s2[GP];
#pragma unroll
            for (int pq = 0; pq < GP; ++pq) s2[pq] = make_float2(0.f, 0.f);
#pragma unroll 2
            for (int c = 0; c < HD / 8; ++c) {
                const uint4 raw = *reinterpret_cast<const uint4*>(stage_p + stage_off<HD>(lane, c * 16));
                float kf[8];
                unpack_row<8>(raw, kf);
#pragma unroll
                for (int pq = 0; pq < GP; ++pq) {
#pragma unroll
                    for (int d2 = 0; d2 < 4; ++d2) {
                        const float4 qq = *reinterpret_cast<const float4*>(sq + pq * HD + c * 8 + 2 * d2);
                        s2[pq] = __ffma2_rn(make_float2(qq.x, qq.y), make_float2(kf[2 * d2], kf[2 * d2]), s2[pq]);
                        s2[pq] = __ffma2_rn(make_float2(qq.z, qq.w), make_float2(kf[2 * d2 + 1], kf[2 * d2 + 1]),
                                            s2[pq]);
                    }
                }
            }
#pragma unroll
            for (int g = 0; g < G; ++g) sc[g] = (g & 1) ? s2[g >> 1].y : s2[g >> 1].x;
        } else {
#pragma unroll
            for (int g = 0; g < G; ++g) sc[g] = -CUDART_INF_F;
        }
        __syncwarp();  // every lane is done with the key rows: the stage takes the value rows
        stage_rows<HD>(stage, vh, blk, nk, lane);
        // online softmax per query over this block (lane 0's key is always valid)
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float mn = fmaxf(m[g], warp_max(sc[g]));
            const float corr = exp2f(m[g] - mn);
            const float p = exp2f(sc[g] - mn);
            l[g] = l[g] * corr + warp_sum(p);
            m[g] = mn;
#pragma unroll
            for (int i = 0; i < DL / 2; ++i) acc[g][i] = __fmul2_rn(acc[g][i], make_float2(corr, corr));
            sp[lane * G + g] = p;
        }
        cp_async_wait_all();
        __syncwarp();
        for (int j = 0; j < nk; ++j) {
            float vf[DL];
            unpack_row<DL>(*reinterpret_cast<const typename Row<HD>::T*>(stage_p + stage_off<HD>(j, lane * DL * 2)),
                           vf);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float p = sp[j * G + g];
#pragma unroll
                for (int i = 0; i < DL / 2; ++i)
                    acc[g][i] = __ffma2_rn(make_float2(p, p), make_float2(vf[2 * i], vf[2 * i + 1]), acc[g][i]);
            }
        }
        __syncwarp();  // the stage and the probabilities are rewritten by the next block
    }

    // merge the warps (the merge area reuses the stages): common max per query, then the scaled sums
    float* sml = reinterpret_cast<float*>(smem + SM::ML);
    float* sacc = reinterpret_cast<float*>(smem + SM::STAGE);
    if (lane == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            sml[(warp * G + g) * 2] = m[g];
            sml[(warp * G + g) * 2 + 1] = l[g];
        }
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float M = -CUDART_INF_F;
        for (int w = 0; w < NW; ++w) M = fmaxf(M, sml[(w * G + g) * 2]);
        const float f = m[g] == -CUDART_INF_F ? 0.f : exp2f(m[g] - M);
#pragma unroll
        for (int i = 0; i < DL / 2; ++i) {
            sacc[(warp * G + g) * HD + lane * DL + 2 * i] = acc[g][i].x * f;
            sacc[(warp * G + g) * HD + lane * DL + 2 * i + 1] = acc[g][i].y * f;
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < G * HD; e += NT) {
        float t = 0.f;
        for (int w = 0; w < NW; ++w) t += sacc[w * G * HD + e];
        po[e] = t;
    }
    if (threadIdx.x < G) {
        const int g = threadIdx.x;
        float M = -CUDART_INF_F;
        for (int w = 0; w < NW; ++w) M = fmaxf(M, sml[(w * G + g) * 2]);
        float L = 0.f;
        for (int w = 0; w < NW; ++w) {
            const float mw = sml[(w * G + g) * 2];
            if (mw != -CUDART_INF_F) L += sml[(w * G + g) * 2 + 1] * exp2f(mw - M);
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
    const int bytes = Smem<HD, G>::BYTES;
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
