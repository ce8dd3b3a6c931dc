// K3 (tensor-core form): chunked Gated DeltaNet prefill on tcgen05 (UMMA) tiles.
//
// One CTA owns one (batch row, value head) chain and walks its chunks of
// C = 64 tokens; the fp32 state S[128][128] stays in shared memory as the
// master copy (laid out as the MN-major B operand of the MMAs).  Per chunk,
// with Q, K the L2-normalised q (times dk^-1/2) and k rows, V the conv
// outputs, beta and gamma = cumsum(g) (deltanet.py:278-389, restated):
//
//   MMA-a  [K;Q] K^T      -> G = K K^T, P0 = Q K^T          (M128 N64  K128)
//   MMA-b  [K;Q] S        -> Y = K S,   O1 = Q S             (M128 N128 K128)
//   CUDA   A = tril(beta_i G_ij e^{g_i-g_j}, -1), P = P0 o e^{g_i-g_j} (j <= i),
//          T = (I + A)^-1 (blocked in-place inverse), Z = beta (V - e^g Y),
//          O1 <- e^g O1 (in tensor memory)
//   MMA-c  [T;P] Z        -> v_new = T Z                     (M128 N128 K64)
//   MMA-d  [T;P] v_new    -> O = e^g O1 + P v_new            (M128 N128 K64, accumulate)
//   MMA-e  K^T (e^{gC-g} v_new) -> S_delta                  (M128 N128 K64)
//   CUDA   gated RMSNorm of O rows -> output; S <- e^{gC} S + S_delta
//
// which is the reference's v_new = U - W S with U = T (beta V) and
// W = T (beta K e^g) (the same linear algebra, regrouped so every product is
// a tensor-core tile).  Operands are tf32 in 128-byte swizzled shared memory,
// accumulators fp32 in tensor memory (512 columns).  Sub-chunk checkpoints
// (deltanet.py:375-388) are computed on CUDA cores from the same v_new.
#include "gdn_async.cuh"
#include "gdn_common.cuh"
#include "gdn_conv_windows.cuh"
#include "gdn_kernels.cuh"
#include "gdn_tmap.h"
#include "gdn_umma.cuh"

namespace gdn {
namespace ptc {

constexpr int D = 128, C = 64, NT = 256;
// shared memory regions (bytes from the 1024-aligned base)
constexpr uint32_t R_S = 0;          // S master, MN-major [dk][dv], 64 KB
constexpr uint32_t R_KQ = 65536;     // [K;Q] K-major [128][dk] -> later [T;P] (32 KB) + v_new (32 KB)
constexpr uint32_t R_VN = R_KQ + 32768;
constexpr uint32_t R_VZ = 131072;    // V -> Z -> e^{gC-g} v_new, MN-major [tok][dv], 32 KB
constexpr uint32_t R_K = 163840;     // K as MN-major A operand [tok][dk], 32 KB
constexpr uint32_t R_Z = 196608;     // raw q/k/v rows of two 8-token sub-batches (12 KB), then z rows, bf16 [64][128]
constexpr uint32_t SUB = 8;          // tokens per conv sub-batch
constexpr uint32_t SUB_BYTES = SUB * 3 * 128 * 2;
constexpr uint32_t R_MISC = 212992;  // small vectors
constexpr int M_G = 0, M_B = 64, M_EG = 128, M_EF = 192, M_RQ = 256, M_RK = 320, M_NW = 384, M_F = 512,
              M_TMP = 576;           // floats
constexpr uint32_t R_BAR = R_MISC + (M_TMP + 1024) * 4;
constexpr uint32_t SMEM_BYTES = R_BAR + 64 + 1024;
// tensor memory columns
constexpr uint32_t T_YO = 0, T_G = 128, T_VN = 256, T_SD = 384, T_COLS = 512;

using TA = __nv_bfloat16;

__device__ __forceinline__ float& el(unsigned char* sm, uint32_t off) { return *reinterpret_cast<float*>(sm + off); }
__device__ __forceinline__ float4& el4(unsigned char* sm, uint32_t off) {
    return *reinterpret_cast<float4*>(sm + off);
}
// [T;P] / A element (row, col) of the K-major 128-row operand at R_KQ
__device__ __forceinline__ uint32_t tp_off(int row, int col) { return R_KQ + umma::kmajor_off(row, col, 128); }

__global__ void __launch_bounds__(NT, 1)
    prefill_tc_kernel(const MixParams p, const CkptList ck, const __grid_constant__ CUtensorMap tm_mixed,
                      const __grid_constant__ CUtensorMap tm_z) {
    extern __shared__ unsigned char raw[];
    const uint32_t raw_addr = smem_u32(raw);
    unsigned char* sm = raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const uint32_t sb = smem_u32(sm);
    float* misc = reinterpret_cast<float*>(sm + R_MISC);
    float* sG = misc + M_G;
    float* sB = misc + M_B;
    float* sEG = misc + M_EG;
    float* sEF = misc + M_EF;
    float* sRQ = misc + M_RQ;
    float* sRK = misc + M_RK;
    float* sNW = misc + M_NW;
    float* sF = misc + M_F;
    float* sTmp = misc + M_TMP;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + R_BAR);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + R_BAR + 32);
    const uint32_t mma_bar = smem_u32(&bars[0]), z_bar = smem_u32(&bars[1]);
    const uint32_t cbar[2] = {smem_u32(&bars[2]), smem_u32(&bars[3])};

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q4 = warp & 3, half = warp >> 2;
    const int bh = blockIdx.x;
    const int b = bh / p.Hv, h = bh - (bh / p.Hv) * p.Hv;
    const int rep = p.Hv / p.Hk, kh = h / rep;
    const int T = p.T, NC = (T + C - 1) / C;
    const int conv_dim = 2 * p.Hk * D + p.Hv * D;
    constexpr int L = 3;  // built for the 4-tap conv (checked by the launcher)
    const TA* cs_in = static_cast<const TA*>(p.cs_in);

    if (tid == 0) {
        mbar_init(mma_bar, 1);
        mbar_init(z_bar, 1);
        mbar_init(smem_u32(&bars[2]), 1);
        mbar_init(smem_u32(&bars[3]), 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        umma::tmem_alloc(smem_u32(tslot), T_COLS);
        umma::tmem_relinquish();
    }
    write_conv_windows<TA, D, D, NT>(p, ck, b, h, kh, rep);
    if (tid < D) sNW[tid] = Act<TA>::ldg(static_cast<const TA*>(p.normw) + tid);
    for (int idx = tid; idx < D * D / 4; idx += NT) {
        const int i = idx >> 5, j = (idx & 31) * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (p.S_in) v = __ldcs(reinterpret_cast<const float4*>(p.S_in + (size_t)bh * D * D + i * D + j));
        el4(sm, R_S + umma::mnmajor_off(i, j, D)) = v;
    }
    // conv channels of this thread (q, k of key head kh; v of value head h) and their history
    constexpr int NCH = 3 * D, CPT = (NCH + NT - 1) / NT;
    float hist[CPT][3], wt[CPT][4];
    {
        const TA* convw = static_cast<const TA*>(p.convw);
#pragma unroll
        for (int u = 0; u < CPT; ++u) {
            const int c = tid + u * NT;
            int gc = 0;
            if (c < D) gc = kh * D + c;
            else if (c < 2 * D) gc = p.Hk * D + kh * D + (c - D);
            else if (c < NCH) gc = 2 * p.Hk * D + h * D + (c - 2 * D);
#pragma unroll
            for (int j = 0; j < 4; ++j) wt[u][j] = 0.f;
#pragma unroll
            for (int j = 0; j < 3; ++j) hist[u][j] = 0.f;
            if (c < NCH) {
#pragma unroll
                for (int j = 0; j < 4; ++j) wt[u][j] = Act<TA>::ldg(convw + (size_t)gc * 4 + j);
                if (cs_in) {
#pragma unroll
                    for (int j = 0; j < L; ++j)
                        hist[u][j] = Act<TA>::ld(cs_in + ((size_t)b * conv_dim + gc) * L + (L - 1 - j));
                }
            }
        }
    }
    const float A_exp = -expf(p.A_log[h]);
    const float dtb = p.dt_bias[h];
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *tslot;
    const uint32_t idesc_a = umma::idesc_tf32(128, 64, 0, 0);
    const uint32_t idesc_b = umma::idesc_tf32(128, 128, 0, 1);
    const uint32_t idesc_e = umma::idesc_tf32(128, 128, 1, 1);

    uint32_t mma_phase = 0;
    int ck_i = 0;
    bool failed = false;
    int c_fail = 0;
    int sb_fail = -1;
    auto mma_wait = [&]() -> bool {
        const bool ok = mbar_wait_bounded(mma_bar, mma_phase & 1u, GDN_DEVERR_MMA_TIMEOUT);
        ++mma_phase;
        umma::fence_after_sync();
        return !__syncthreads_or(!ok);
    };

    for (int c = 0; c < NC; ++c) {
        const int t0 = c * C;
        // ---------------- conv: raw rows staged by bulk copies, 8 tokens at a time ----------------
        // sub-batch s of the chunk goes to buffer s & 1; the copy of s + 2 is
        // issued as soon as every thread has consumed s
        auto issue_sub = [&](int sbi) {
            // three [8 tokens][128 channels] boxes (q, k of key head kh; v of value head h)
            const int buf = sbi & 1;
            const uint32_t dst = sb + R_Z + buf * SUB_BYTES;
            mbar_arrive_expect_tx(cbar[buf], SUB_BYTES);
            const int tok = t0 + sbi * (int)SUB;
            tma_load_3d(dst, &tm_mixed, kh * D, tok, b, cbar[buf]);
            tma_load_3d(dst + SUB * D * 2, &tm_mixed, p.Hk * D + kh * D, tok, b, cbar[buf]);
            tma_load_3d(dst + 2 * SUB * D * 2, &tm_mixed, 2 * p.Hk * D + h * D, tok, b, cbar[buf]);
        };
        if (tid == 0) {
            fence_proxy_async_smem();
            issue_sub(0);
            issue_sub(1);
        }
        float raw_a = 0.f, raw_b = 0.f;  // gate inputs of token t0 + tid, in flight during the conv
        if (tid < C && t0 + tid < T) {
            const size_t ai = (size_t)b * p.as_b + (size_t)(t0 + tid) * p.as_t + h;
            raw_b = Act<TA>::ld(static_cast<const TA*>(p.b) + ai);
            raw_a = Act<TA>::ld(static_cast<const TA*>(p.a) + ai);
        }
        for (int sbi = 0; sbi < C / (int)SUB; ++sbi) {
            const int buf = sbi & 1;
            const bool ok = mbar_wait_bounded(cbar[buf], (uint32_t)(sbi >> 1) & 1u, GDN_DEVERR_TMA_TIMEOUT);
            if (!ok) {
                failed = true;
                sb_fail = sbi;
            }
            const TA* stage = reinterpret_cast<const TA*>(sm + R_Z + buf * SUB_BYTES);
#pragma unroll
            for (int u = 0; u < CPT; ++u) {
                const int ch = tid + u * NT;
                if (ch >= NCH) continue;
                const int seg = ch >> 7, ci = ch & 127;
                uint32_t o0, o1 = 0xFFFFFFFFu;  // destinations (row offsets added per token)
#pragma unroll
                for (int i = 0; i < (int)SUB; ++i) {
                    const int t = sbi * SUB + i, tg = t0 + t;
                    float val = 0.f;
                    if (tg < T) {
                        const float x = __bfloat162float(stage[(seg * SUB + i) * D + ci]);
                        const int valid = cs_in ? L : (tg < L ? tg : L);
                        const float cv = conv4_taps<TA>(x, hist[u][0], hist[u][1], hist[u][2], wt[u][0], wt[u][1],
                                                        wt[u][2], wt[u][3], valid);
                        val = Act<TA>::round(__fdividef(cv, 1.0f + __expf(-cv)));
                        hist[u][2] = hist[u][1];
                        hist[u][1] = hist[u][0];
                        hist[u][0] = x;
                    }
                    if (seg == 0) {
                        o0 = R_KQ + umma::kmajor_off(64 + t, ci, 128);
                    } else if (seg == 1) {
                        o0 = R_KQ + umma::kmajor_off(t, ci, 128);
                        o1 = R_K + umma::mnmajor_off(t, ci, C);
                    } else {
                        o0 = R_VZ + umma::mnmajor_off(t, ci, C);
                    }
                    el(sm, o0) = val;
                    if (seg == 1) el(sm, o1) = val;
                }
            }
            if (__syncthreads_or(failed)) {
                failed = true;
                break;
            }
            if (tid == 0 && sbi + 2 < C / (int)SUB) {
                fence_proxy_async_smem();
                issue_sub(sbi + 2);
            }
        }
        if (failed) {
            c_fail = -1;
            break;
        }
        // ---------------- z rows of the chunk: one [64][128] box into the freed staging area ----------------
        if (tid == 0) {
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(z_bar, (uint32_t)(C * D * sizeof(TA)));
            tma_load_3d(sb + R_Z, &tm_z, h * D, t0, b, z_bar);
        }
        if (tid < C) {
            float beta = 0.f, g = 0.f;
            if (t0 + tid < T) {
                beta = Act<TA>::round(sigmoid_f(raw_b));
                g = A_exp * softplus_f(raw_a + dtb);
            }
            sB[tid] = beta;
            sG[tid] = g;
        }
        __syncthreads();
        // ---------------- norms (warp per token), gamma (thread 0) ----------------
        for (int r = 0; r < C / 8; ++r) {
            const int t = warp + 8 * r;
            const float4 qv = el4(sm, R_KQ + umma::kmajor_off(64 + t, lane * 4, 128));
            const float4 kv = el4(sm, R_KQ + umma::kmajor_off(t, lane * 4, 128));
            float sq = qv.x * qv.x + qv.y * qv.y + qv.z * qv.z + qv.w * qv.w;
            float sk = kv.x * kv.x + kv.y * kv.y + kv.z * kv.z + kv.w * kv.w;
            sq = warp_sum(sq);
            sk = warp_sum(sk);
            if (lane == 0) {
                sRQ[t] = rsqrtf(sq + 1e-6f);
                sRK[t] = rsqrtf(sk + 1e-6f);
            }
        }
        if (tid == 0) {
            float acc = 0.f;
            for (int t = 0; t < C; ++t) {
                acc += sG[t];
                sG[t] = acc;
            }
        }
        __syncthreads();
        if (tid < C) {
            sEG[tid] = expf(sG[tid]);
            sEF[tid] = expf(sG[C - 1] - sG[tid]);
        }
        // scale q, k rows in place (q: (q * rq) * dk^-1/2, k: k * rk)
        for (int idx = tid; idx < 128 * 32; idx += NT) {
            const int r = idx >> 5, c4 = (idx & 31) * 4;
            float4& v = el4(sm, R_KQ + umma::kmajor_off(r, c4, 128));
            if (r < C) {
                const float s = sRK[r];
                v = umma::tf32_rna4(make_float4(v.x * s, v.y * s, v.z * s, v.w * s));
            } else {
                const float s = sRQ[r - C];
                v = umma::tf32_rna4(make_float4((v.x * s) * p.q_scale, (v.y * s) * p.q_scale, (v.z * s) * p.q_scale,
                                                (v.w * s) * p.q_scale));
            }
        }
        for (int idx = tid; idx < C * 32; idx += NT) {
            const int t = idx >> 5, d4 = (idx & 31) * 4;
            float4& v = el4(sm, R_K + umma::mnmajor_off(t, d4, C));
            const float s = sRK[t];
            v = umma::tf32_rna4(make_float4(v.x * s, v.y * s, v.z * s, v.w * s));
        }
        fence_proxy_async_smem();
        __syncthreads();
        // ---------------- MMA-a, MMA-b ----------------
        if (tid == 0) {
            umma::fence_after_sync();
            for (int kk = 0; kk < D / 8; ++kk)
                umma::mma_tf32(tmem + T_G, umma::desc_kmajor(sb + R_KQ, 128, kk), umma::desc_kmajor(sb + R_KQ, 128, kk),
                               idesc_a, kk > 0);
            for (int kk = 0; kk < D / 8; ++kk)
                umma::mma_tf32(tmem + T_YO, umma::desc_kmajor(sb + R_KQ, 128, kk), umma::desc_mnmajor(sb + R_S, D, kk),
                               idesc_b, kk > 0);
            umma::mma_commit(mma_bar);
        }
        if (!mma_wait()) {
            failed = true;
            c_fail = c;
            break;
        }
        // ---------------- A, P, Z, e^g O1 from tensor memory ----------------
        {
            const uint32_t lane_base = (uint32_t)(32 * q4) << 16;
            if (q4 < 2) {
                const int t = lane + 32 * q4;
                if (half == 0) {
                    const float bt = sB[t], gt = sG[t];
#pragma unroll
                    for (int c0 = 0; c0 < C; c0 += 32) {
                        float v[32];
                        umma::tmem_ld32(tmem + lane_base + T_G + c0, v);
                        umma::tmem_wait_ld();
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj) {
                            const int j = c0 + jj;
                            el(sm, tp_off(t, j)) = j < t ? (bt * v[jj]) * __expf(gt - sG[j]) : 0.f;
                        }
                    }
                } else {
                    const float bt = sB[t], et = sEG[t];
#pragma unroll
                    for (int c0 = 0; c0 < D; c0 += 32) {
                        float v[32];
                        umma::tmem_ld32(tmem + lane_base + T_YO + c0, v);
                        umma::tmem_wait_ld();
#pragma unroll
                        for (int jj = 0; jj < 32; jj += 4) {
                            float4& z = el4(sm, R_VZ + umma::mnmajor_off(t, c0 + jj, C));
                            z = umma::tf32_rna4(make_float4(bt * (z.x - et * v[jj]), bt * (z.y - et * v[jj + 1]),
                                                            bt * (z.z - et * v[jj + 2]), bt * (z.w - et * v[jj + 3])));
                        }
                    }
                }
            } else {
                const int t = lane + 32 * q4 - 64;
                if (half == 0) {
                    const float gt = sG[t];
#pragma unroll
                    for (int c0 = 0; c0 < C; c0 += 32) {
                        float v[32];
                        umma::tmem_ld32(tmem + lane_base + T_G + c0, v);
                        umma::tmem_wait_ld();
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj) {
                            const int j = c0 + jj;
                            el(sm, tp_off(64 + t, j)) = j <= t ? umma::tf32_rna(v[jj] * __expf(gt - sG[j])) : 0.f;
                        }
                    }
                } else {
                    const float et = sEG[t];
#pragma unroll
                    for (int c0 = 0; c0 < D; c0 += 32) {
                        float v[32];
                        umma::tmem_ld32(tmem + lane_base + T_YO + c0, v);
                        umma::tmem_wait_ld();
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj) v[jj] *= et;
                        umma::tmem_st32(tmem + lane_base + T_YO + c0, v);
                    }
                    umma::tmem_wait_st();
                }
            }
        }
        umma::fence_before_sync();
        __syncthreads();
        // ---------------- T = (I + A)^-1 in place (rows 0..63 of [T;P]) ----------------
        {
            float x[16];
            if (tid < 64) {
                const int base = (tid >> 4) * 16, cj = tid & 15;
#pragma unroll
                for (int r = 0; r < 16; ++r) {
                    float acc = r == cj ? 1.f : 0.f;
#pragma unroll
                    for (int cc = 0; cc < r; ++cc) acc = fmaf(-el(sm, tp_off(base + r, base + cc)), x[cc], acc);
                    x[r] = acc;
                }
            }
            __syncthreads();
            if (tid < 64) {
                const int base = (tid >> 4) * 16, cj = tid & 15;
#pragma unroll
                for (int r = 0; r < 16; ++r) el(sm, tp_off(base + r, base + cj)) = x[r];
            }
            __syncthreads();
            // 16 -> 32: T10 = -T11 (A10 T00) for the two 32x32 diagonal blocks
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int idx = tid + u * NT, pb = idx >> 8, r = (idx >> 4) & 15, jj = idx & 15;
                const int o = 32 * pb;
                float acc = 0.f;
#pragma unroll
                for (int cc = 0; cc < 16; ++cc)
                    acc = fmaf(el(sm, tp_off(o + 16 + r, o + cc)), el(sm, tp_off(o + cc, o + jj)), acc);
                sTmp[idx] = acc;
            }
            __syncthreads();
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int idx = tid + u * NT, pb = idx >> 8, r = (idx >> 4) & 15, jj = idx & 15;
                const int o = 32 * pb;
                float acc = 0.f;
#pragma unroll
                for (int cc = 0; cc < 16; ++cc)
                    acc = fmaf(el(sm, tp_off(o + 16 + r, o + 16 + cc)), sTmp[pb * 256 + cc * 16 + jj], acc);
                el(sm, tp_off(o + 16 + r, o + jj)) = -acc;
            }
            __syncthreads();
            // 32 -> 64
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int idx = tid + u * NT, r = idx >> 5, jj = idx & 31;
                float acc = 0.f;
#pragma unroll 8
                for (int cc = 0; cc < 32; ++cc)
                    acc = fmaf(el(sm, tp_off(32 + r, cc)), el(sm, tp_off(cc, jj)), acc);
                sTmp[idx] = acc;
            }
            __syncthreads();
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int idx = tid + u * NT, r = idx >> 5, jj = idx & 31;
                float acc = 0.f;
#pragma unroll 8
                for (int cc = 0; cc < 32; ++cc) acc = fmaf(el(sm, tp_off(32 + r, 32 + cc)), sTmp[cc * 32 + jj], acc);
                el(sm, tp_off(32 + r, jj)) = -acc;
            }
            __syncthreads();
            for (int idx = tid; idx < C * C; idx += NT) {
                float& x = el(sm, tp_off(idx >> 6, idx & 63));
                x = umma::tf32_rna(x);
            }
        }
        fence_proxy_async_smem();
        __syncthreads();
        // ---------------- MMA-c: v_new = T Z ----------------
        if (tid == 0) {
            umma::fence_after_sync();
            for (int kk = 0; kk < C / 8; ++kk)
                umma::mma_tf32(tmem + T_VN, umma::desc_kmajor(sb + R_KQ, 128, kk), umma::desc_mnmajor(sb + R_VZ, C, kk),
                               idesc_b, kk > 0);
            umma::mma_commit(mma_bar);
        }
        if (!mma_wait()) {
            failed = true;
            c_fail = c;
            break;
        }
        // ---------------- v_new and e^{gC-g} v_new to shared memory ----------------
        if (q4 < 2) {
            const int t = lane + 32 * q4;
            const uint32_t lane_base = (uint32_t)(32 * q4) << 16;
            const float ft = sEF[t];
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                const int c0 = 64 * half + 32 * cc;
                float v[32];
                umma::tmem_ld32(tmem + lane_base + T_VN + c0, v);
                umma::tmem_wait_ld();
#pragma unroll
                for (int jj = 0; jj < 32; jj += 4) {
                    const uint32_t o = umma::mnmajor_off(t, c0 + jj, C);
                    el4(sm, R_VN + o) = umma::tf32_rna4(make_float4(v[jj], v[jj + 1], v[jj + 2], v[jj + 3]));
                    el4(sm, R_VZ + o) =
                        umma::tf32_rna4(make_float4(v[jj] * ft, v[jj + 1] * ft, v[jj + 2] * ft, v[jj + 3] * ft));
                }
            }
        }
        fence_proxy_async_smem();
        umma::fence_before_sync();
        __syncthreads();
        // ---------------- MMA-d (O += P v_new), MMA-e (S_delta) ----------------
        if (tid == 0) {
            umma::fence_after_sync();
            for (int kk = 0; kk < C / 8; ++kk)
                umma::mma_tf32(tmem + T_YO, umma::desc_kmajor(sb + R_KQ, 128, kk), umma::desc_mnmajor(sb + R_VN, C, kk),
                               idesc_b, 1u);
            for (int kk = 0; kk < C / 8; ++kk)
                umma::mma_tf32(tmem + T_SD, umma::desc_mnmajor(sb + R_K, C, kk), umma::desc_mnmajor(sb + R_VZ, C, kk),
                               idesc_e, kk > 0);
            umma::mma_commit(mma_bar);
        }
        if (!mma_wait()) {
            failed = true;
            c_fail = c;
            break;
        }
        // ---------------- sub-chunk checkpoints (CUDA cores, before S changes) ----------------
        while (ck_i < ck.n && (ck.off[ck_i] - 1) / C == c && ck.off[ck_i] - t0 < C) {
            const int s_off = ck.off[ck_i] - t0;
            const float gs = sG[s_off - 1];
            if (tid < s_off) sF[tid] = expf(gs - sG[tid]);
            __syncthreads();
            const float es = expf(gs);
            float* dst = p.S_ckpt + ((size_t)ck.slot[ck_i] * p.B * p.Hv + bh) * (size_t)(D * D);
            for (int idx = tid; idx < D * D; idx += NT) {
                const int i = idx >> 7, j = idx & 127;
                float acc = 0.f;
                for (int t = 0; t < s_off; ++t)
                    acc = fmaf(el(sm, R_K + umma::mnmajor_off(t, i, C)) * sF[t], el(sm, R_VN + umma::mnmajor_off(t, j, C)),
                               acc);
                dst[idx] = fmaf(el(sm, R_S + umma::mnmajor_off(i, j, D)), es, acc);
            }
            __syncthreads();
            ++ck_i;
        }
        // ---------------- output rows (gated RMSNorm), warps 2,3,6,7 (lanes 64..127) ----------------
        // each of the two warps on a lane quarter takes half of the 128 columns;
        // the row sums of squares meet in shared memory
        const bool out_warp = q4 >= 2;
        const int ot = lane + 32 * q4 - 64, otg = t0 + ot;
        const uint32_t o_lane = (uint32_t)(32 * q4) << 16;
        if (out_warp) {
            float ss = 0.f;
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                float v[32];
                umma::tmem_ld32(tmem + o_lane + T_YO + 64 * half + 32 * cc, v);
                umma::tmem_wait_ld();
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) {
                    const float o = Act<TA>::round(v[jj]);
                    ss = fmaf(o, o, ss);
                }
            }
            sTmp[half * 64 + ot] = ss;
        }
        __syncthreads();
        if (out_warp) {
            const bool zok = mbar_wait_bounded(z_bar, (uint32_t)c & 1u, GDN_DEVERR_TMA_TIMEOUT);
            const float rstd = rsqrtf((sTmp[ot] + sTmp[64 + ot]) / (float)D + p.eps);
            TA* out = static_cast<TA*>(p.out) + ((size_t)b * T + otg) * (size_t)(p.Hv * D) + h * D;
            const TA* zr = reinterpret_cast<const TA*>(sm + R_Z) + ot * D;
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                const int c0 = 64 * half + 32 * cc;
                float v[32];
                umma::tmem_ld32(tmem + o_lane + T_YO + c0, v);
                umma::tmem_wait_ld();
                if (otg < T && zok) {
#pragma unroll
                    for (int jj = 0; jj < 32; jj += 8) {
                        uint4 zp = *reinterpret_cast<const uint4*>(zr + c0 + jj);
                        const __nv_bfloat16* zb = reinterpret_cast<const __nv_bfloat16*>(&zp);
                        __align__(16) __nv_bfloat16 ob[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const float o = Act<TA>::round(v[jj + e]);
                            const float y = Act<TA>::round(sNW[c0 + jj + e] * Act<TA>::round(o * rstd));
                            const float zz = __bfloat162float(zb[e]);
                            ob[e] = __float2bfloat16_rn(y * __fdividef(zz, 1.0f + __expf(-zz)));
                        }
                        *reinterpret_cast<uint4*>(out + c0 + jj) = *reinterpret_cast<const uint4*>(ob);
                    }
                }
            }
        }
        // ---------------- S <- e^{gC} S + S_delta; boundary checkpoints; final state ----------------
        {
            const int i = 32 * q4 + lane;
            const uint32_t lane_base = (uint32_t)(32 * q4) << 16;
            const float ec = sEG[C - 1];
            const bool last = c == NC - 1;
            int ck_b = ck_i;
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                const int c0 = 64 * half + 32 * cc;
                float v[32];
                umma::tmem_ld32(tmem + lane_base + T_SD + c0, v);
                umma::tmem_wait_ld();
#pragma unroll
                for (int jj = 0; jj < 32; jj += 4) {
                    float4& s = el4(sm, R_S + umma::mnmajor_off(i, c0 + jj, D));
                    float4 n;
                    n.x = fmaf(s.x, ec, v[jj]);
                    n.y = fmaf(s.y, ec, v[jj + 1]);
                    n.z = fmaf(s.z, ec, v[jj + 2]);
                    n.w = fmaf(s.w, ec, v[jj + 3]);
                    s = n;
                    for (int w = ck_b; w < ck.n && ck.off[w] - t0 == C; ++w)
                        if (p.S_ckpt)
                            __stcs(reinterpret_cast<float4*>(p.S_ckpt + ((size_t)ck.slot[w] * p.B * p.Hv + bh) *
                                                                            (size_t)(D * D) + i * D + c0 + jj), n);
                    if (last && p.S_out)
                        __stcs(reinterpret_cast<float4*>(p.S_out + (size_t)bh * D * D + i * D + c0 + jj), n);
                }
            }
            while (ck_b < ck.n && ck.off[ck_b] - t0 == C) ++ck_b;
            ck_i = ck_b;
        }
        umma::fence_before_sync();
        __syncthreads();
    }

    if (failed && tid == 0) {
        // let copies still in flight land before the CTA exits (bounded waits)
        if (c_fail >= 0) {
            mbar_wait_bounded(z_bar, (uint32_t)c_fail & 1u, GDN_DEVERR_TMA_TIMEOUT);
        } else if (sb_fail >= 0) {
            for (int sbi = sb_fail; sbi < sb_fail + 2 && sbi < C / (int)SUB; ++sbi)
                mbar_wait_bounded(cbar[sbi & 1], (uint32_t)(sbi >> 1) & 1u, GDN_DEVERR_TMA_TIMEOUT);
        }
    }
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tmem, T_COLS);
}

}  // namespace ptc

cudaError_t launch_prefill_tc(const MixParams& p, const CkptList& ck, int d, int dtype, cudaStream_t s,
                              bool* supported) {
    auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    *supported = dtype == GDN_DTYPE_BF16 && d == 128 && p.K == 4 && al(p.z) && al(p.mixed) && (p.zs_b % 8) == 0 &&
                 (p.zs_t % 8) == 0 && (p.ms_b % 8) == 0 && (p.ms_t % 8) == 0;
    if (!*supported) return cudaSuccess;
    const uint64_t conv_dim = 2ull * p.Hk * d + (uint64_t)p.Hv * d;
    CUtensorMap tm_mixed, tm_z;
    if (!encode_tmap_3d_bf16(&tm_mixed, p.mixed, conv_dim, (uint64_t)p.T, (uint64_t)p.B, (uint64_t)p.ms_t * 2,
                             (uint64_t)p.ms_b * 2, 128, ptc::SUB) ||
        !encode_tmap_3d_bf16(&tm_z, p.z, (uint64_t)p.Hv * d, (uint64_t)p.T, (uint64_t)p.B, (uint64_t)p.zs_t * 2,
                             (uint64_t)p.zs_b * 2, 128, ptc::C)) {
        *supported = false;  // no tensor maps: the CUDA-core kernel takes the call
        return cudaSuccess;
    }
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(ptc::prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)ptc::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    ptc::prefill_tc_kernel<<<p.B * p.Hv, ptc::NT, ptc::SMEM_BYTES, s>>>(p, ck, tm_mixed, tm_z);
    return cudaGetLastError();
}

unsigned int prefill_tc_device_error(bool clear) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
    if (clear && v) {
        const unsigned int zero = 0;
        cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
    }
    return v;
}

}  // namespace gdn
