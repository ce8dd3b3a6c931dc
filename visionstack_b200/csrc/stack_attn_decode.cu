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

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t* r) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// d[16x8] += a[16x16] b[16x8], bf16 in, fp32 accumulate (warp-wide)
__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// shared memory of attn_split_kernel, in bytes
template <int HD, int G>
struct Smem {
    static constexpr int STAGE = 0;                     // [NW][KB][HD] bf16 (then [NW][G][HD] f32)
    static constexpr int PT = STAGE + NW * KB * HD * 2;  // [NW][8][KB] bf16: a warp's probabilities, query-major
    static constexpr int ML = PT + NW * 8 * KB * 2;      // [NW][8][2] f32 warp max / sum
    static constexpr int BYTES = ML + NW * 8 * 2 * 4;
    static_assert(NW * G * HD * 4 <= NW * KB * HD * 2, "the merge area must fit in the stages");
};

// Per warp and block of 32 keys, on the tensor cores (mma.sync m16n8k16, bf16 in, fp32 out):
// scores S[32 keys][8 queries] = K_blk Q^T (two 16-key tiles x HD/16 steps, K from the stage by
// ldmatrix, Q fragments held in registers; queries past G are zero), then
// O^T[HD][8] += V_blk^T P^T (HD/16 dim tiles x two 16-key steps, V transposed by ldmatrix.trans,
// P rounded to bf16 as the flash form of attention does).  Lane (g = lane / 4, t = lane % 4)
// holds scores of keys {g, g+8} (+16) for queries {2t, 2t+1} and outputs of dims {g, g+8} (+16i)
// for the same two queries, so the softmax state of a query lives in the lanes with its t.
template <int HD, int G>
__global__ void __launch_bounds__(NT, 1) attn_split_kernel(const __nv_bfloat16* __restrict__ q,
                                                           const __nv_bfloat16* __restrict__ kbuf,
                                                           const __nv_bfloat16* __restrict__ vbuf,
                                                           const long long* __restrict__ pos, int cap, int span,
                                                           float qscale, float* __restrict__ part_o,
                                                           float* __restrict__ part_ml) {
    using SM = Smem<HD, G>;
    constexpr int KS = HD / 16;  // 16-dim steps of the scores, 16-dim tiles of the outputs
    extern __shared__ __align__(16) unsigned char smem[];
    const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int S = gridDim.x, KVH = gridDim.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, tq = lane & 3;
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
    // Q fragments (B operand, k = dim, n = query): query gq, dims 16ks + 2tq + {0,1} and + 8
    uint32_t qf[KS][2];
    {
        const __nv_bfloat16* qrow = q + (head * G + gq) * HD;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            qf[ks][0] = gq < G ? __ldg(reinterpret_cast<const unsigned int*>(qrow + ks * 16 + 2 * tq)) : 0u;
            qf[ks][1] = gq < G ? __ldg(reinterpret_cast<const unsigned int*>(qrow + ks * 16 + 2 * tq + 8)) : 0u;
        }
    }

    const __nv_bfloat16* kh = kbuf + head * (size_t)cap * HD;
    const __nv_bfloat16* vh = vbuf + head * (size_t)cap * HD;
    const uint32_t stage = smem_u32(smem + SM::STAGE + warp * KB * HD * 2);
    unsigned char* stage_p = smem + SM::STAGE + warp * KB * HD * 2;
    __nv_bfloat16* spt = reinterpret_cast<__nv_bfloat16*>(smem + SM::PT) + warp * 8 * KB;
    const uint32_t spt_a = smem_u32(spt);
    float m[2] = {-CUDART_INF_F, -CUDART_INF_F}, l[2] = {0.f, 0.f};
    float acc[KS][4];
#pragma unroll
    for (int i = 0; i < KS; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

    for (int blk = k0 + warp * KB; blk < k1; blk += NW * KB) {
        const int nk = min(KB, k1 - blk);
        stage_rows<HD>(stage, kh, blk, nk, lane);
        cp_async_wait_all();
        __syncwarp();
        // scores: c[mt] = S[keys 16mt + gq (+8)][queries 2tq, 2tq+1]
        float c[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
            c[mt][0] = c[mt][1] = c[mt][2] = c[mt][3] = 0.f;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                uint32_t a[4];
                ldsm_x4(stage + stage_off<HD>(mt * 16 + (lane & 15), (ks * 2 + (lane >> 4)) * 16), a);
                mma16816(c[mt], a, qf[ks][0], qf[ks][1]);
            }
        }
        __syncwarp();  // every lane is done with the key rows: the stage takes the value rows
        stage_rows<HD>(stage, vh, blk, nk, lane);
        // online softmax (log2 domain) for queries 2tq + jj over the block's valid keys
        float corr[2];
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
            float sv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = (e >> 1) * 16 + gq + (e & 1) * 8;
                sv[e] = key < nk ? c[e >> 1][(e & 1) * 2 + jj] * qscale : -CUDART_INF_F;
            }
            float mx = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float mn = fmaxf(m[jj], mx);
            corr[jj] = exp2f(m[jj] - mn);
            float sum = 0.f;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float p = exp2f(sv[e] - mn);
                sum += p;
                const int key = (e >> 1) * 16 + gq + (e & 1) * 8;
                spt[(2 * tq + jj) * KB + key] = __float2bfloat16_rn(p);
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            sum += __shfl_xor_sync(0xffffffffu, sum, 8);
            sum += __shfl_xor_sync(0xffffffffu, sum, 16);
            l[jj] = l[jj] * corr[jj] + sum;
            m[jj] = mn;
        }
#pragma unroll
        for (int i = 0; i < KS; ++i) {
            acc[i][0] *= corr[0];
            acc[i][1] *= corr[1];
            acc[i][2] *= corr[0];
            acc[i][3] *= corr[1];
        }
        cp_async_wait_all();
        if (nk < KB) {  // rows past the valid keys: zero (their probabilities are 0; 0 x stale data)
            for (int idx = lane; idx < (KB - nk) * (HD / 8); idx += 32) {
                const int r = nk + idx / (HD / 8), cc = idx % (HD / 8);
                *reinterpret_cast<uint4*>(stage_p + stage_off<HD>(r, cc * 16)) = make_uint4(0u, 0u, 0u, 0u);
            }
        }
        __syncwarp();
        // P^T fragments (B operand, k = key, n = query): query gq, keys 16kk + 2tq + {0,1} and + 8
        uint32_t pb[2][2];
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            asm volatile("ld.shared.b32 %0, [%1];" : "=r"(pb[kk][0]) : "r"(spt_a + (gq * KB + kk * 16 + 2 * tq) * 2));
            asm volatile("ld.shared.b32 %0, [%1];" : "=r"(pb[kk][1]) : "r"(spt_a + (gq * KB + kk * 16 + 2 * tq + 8) * 2));
        }
        // outputs: acc[dt] = O[dims 16dt + gq (+8)][queries 2tq, 2tq+1]
#pragma unroll
        for (int dt = 0; dt < KS; ++dt) {
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
                uint32_t a[4];
                ldsm_x4_trans(stage + stage_off<HD>(kk * 16 + ((lane >> 4) << 3) + (lane & 7),
                                                    (dt * 2 + ((lane >> 3) & 1)) * 16), a);
                mma16816(acc[dt], a, pb[kk][0], pb[kk][1]);
            }
        }
        __syncwarp();  // the stage and the probabilities are rewritten by the next block
    }

    // merge the warps (the merge area reuses the stages): common max per query, then the scaled sums
    float* sml = reinterpret_cast<float*>(smem + SM::ML);
    float* sacc = reinterpret_cast<float*>(smem + SM::STAGE);
    if (gq == 0) {
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
            sml[(warp * 8 + 2 * tq + jj) * 2] = m[jj];
            sml[(warp * 8 + 2 * tq + jj) * 2 + 1] = l[jj];
        }
    }
    __syncthreads();
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
        const int n = 2 * tq + jj;
        if (n >= G) continue;
        float M = -CUDART_INF_F;
        for (int w = 0; w < NW; ++w) M = fmaxf(M, sml[(w * 8 + n) * 2]);
        const float f = m[jj] == -CUDART_INF_F ? 0.f : exp2f(m[jj] - M);
#pragma unroll
        for (int dt = 0; dt < KS; ++dt) {
            sacc[(warp * G + n) * HD + dt * 16 + gq] = acc[dt][jj] * f;
            sacc[(warp * G + n) * HD + dt * 16 + gq + 8] = acc[dt][2 + jj] * f;
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < G * HD; e += NT) {
        float t = 0.f;
        for (int w = 0; w < NW; ++w) t += sacc[w * G * HD + e];
        po[e] = t;
    }
    if (threadIdx.x < G) {
        const int n = threadIdx.x;
        float M = -CUDART_INF_F;
        for (int w = 0; w < NW; ++w) M = fmaxf(M, sml[(w * 8 + n) * 2]);
        float L = 0.f;
        for (int w = 0; w < NW; ++w) {
            const float mw = sml[(w * 8 + n) * 2];
            if (mw != -CUDART_INF_F) L += sml[(w * 8 + n) * 2 + 1] * exp2f(mw - M);
        }
        pml[2 * n] = M;
        pml[2 * n + 1] = L;
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
