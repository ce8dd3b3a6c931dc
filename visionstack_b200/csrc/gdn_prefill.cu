// K3: fused chunked Gated DeltaNet prefill (CUDA-core fp32 version).
//
// One CTA owns one (batch row, value head) and walks its chunks of C = 64
// tokens in order with the fp32 state S[d][d] resident in shared memory.  Per
// chunk (deltanet.py:278-389, restated):
//   inputs   conv + SiLU of the raw projections (history carried in registers
//            across chunks), q/k L2 norm, beta, g, gamma = cumsum(g)
//   A        = tril(diag(beta) K K^T o Gamma, -1),  Gamma_ij = e^{gamma_i - gamma_j}
//   [U | W]  = (I + A)^-1 [beta V | beta K e^gamma]   (forward substitution;
//            the reference builds the same inverse by block Neumann products,
//            deltanet.py:93-162)
//   v_new    = U - W S
//   O        = (Q e^gamma) S + (Q K^T o Gamma) v_new
//   S        = S e^{gamma_C} + (K e^{gamma_C - gamma})^T v_new
//   output   gated RMSNorm of O rows (config.py:136-143)
// Sub-chunk checkpoints (deltanet.py:375-388) are written from the same
// v_new.  Padded positions of the last chunk carry zero q/k/v/beta/g, as the
// reference's zero padding does (deltanet.py:288-296).
#include "gdn_common.cuh"
#include "gdn_kernels.cuh"
#include "gdn_conv_windows.cuh"

namespace gdn {

namespace prefill {

constexpr int C = 64;
constexpr int NT = 256;

template <int D>
struct Smem {
    static constexpr int QS = D + 4;      // padded row stride of Q / K
    static constexpr int XS = 2 * D + 4;  // row stride of X = [U | W]
    static constexpr int AS = C + 4;      // row stride of A / P
    static constexpr int S_OFF = 0;
    static constexpr int Q_OFF = S_OFF + D * D;
    static constexpr int K_OFF = Q_OFF + C * QS;
    static constexpr int X_OFF = K_OFF + C * QS;
    static constexpr int A_OFF = X_OFF + C * XS;
    static constexpr int G_OFF = A_OFF + C * AS;  // gamma
    static constexpr int B_OFF = G_OFF + C;       // beta
    static constexpr int E_OFF = B_OFF + C;       // e^gamma
    static constexpr int F_OFF = E_OFF + C;       // e^{gamma_C - gamma}
    static constexpr int R_OFF = F_OFF + C;       // per-token rq, rk (2*C)
    static constexpr int TOTAL = R_OFF + 2 * C;
    static constexpr size_t BYTES = (size_t)TOTAL * sizeof(float);
};

}  // namespace prefill

template <int D, typename TA, bool MIXER>
__global__ void __launch_bounds__(prefill::NT, 1) prefill_kernel(const MixParams p, const CkptList ck) {
    using namespace prefill;
    using SM = Smem<D>;
    constexpr int QS = SM::QS, XS = SM::XS, AS = SM::AS;
    constexpr int NCH = 3 * D;                       // q, k, v channels of this CTA
    constexpr int CPT = (NCH + NT - 1) / NT;         // channels per thread
    constexpr int JC = D / 16;                       // columns per thread (interleaved by 16)
    static_assert(D % 16 == 0 && 2 * D <= NT, "bad prefill tiling");

    extern __shared__ __align__(16) float smem[];
    float* sS = smem + SM::S_OFF;
    float* sQ = smem + SM::Q_OFF;
    float* sK = smem + SM::K_OFF;
    float* sX = smem + SM::X_OFF;
    float* sA = smem + SM::A_OFF;
    float* sG = smem + SM::G_OFF;
    float* sB = smem + SM::B_OFF;
    float* sE = smem + SM::E_OFF;
    float* sF = smem + SM::F_OFF;
    float* sR = smem + SM::R_OFF;

    const int bh = blockIdx.x;
    const int b = bh / p.Hv, h = bh - (bh / p.Hv) * p.Hv;
    const int rep = p.Hv / p.Hk;
    const int kh = h / rep;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int T = p.T;
    const int NC = (T + C - 1) / C;

    if (MIXER) write_conv_windows<TA, D, D, NT>(p, ck, b, h, kh, rep);

    // initial state
    const size_t sbase = (size_t)bh * D * D;
    for (int i = tid; i < D * D / 4; i += NT) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (p.S_in) v = __ldcs(reinterpret_cast<const float4*>(p.S_in + sbase) + i);
        reinterpret_cast<float4*>(sS)[i] = v;
    }

    // conv channels of this thread and their carried history (newest first)
    const int conv_dim = 2 * p.Hk * D + p.Hv * D;
    const int L = p.K - 1;
    const TA* mixed = static_cast<const TA*>(p.mixed);
    const TA* cs_in = static_cast<const TA*>(p.cs_in);
    float hist[CPT][3];
    float wt[CPT][4];
    int gch[CPT];
    if (MIXER) {
        const TA* convw = static_cast<const TA*>(p.convw);
#pragma unroll
        for (int u = 0; u < CPT; ++u) {
            const int c = tid + u * NT;
            int gc = 0;
            if (c < D) gc = kh * D + c;
            else if (c < 2 * D) gc = p.Hk * D + kh * D + (c - D);
            else if (c < NCH) gc = 2 * p.Hk * D + h * D + (c - 2 * D);
            gch[u] = gc;
#pragma unroll
            for (int j = 0; j < 4; ++j) wt[u][j] = 0.f;
#pragma unroll
            for (int j = 0; j < 3; ++j) hist[u][j] = 0.f;
            if (c < NCH) {
                for (int j = 0; j < p.K; ++j) wt[u][j] = Act<TA>::ldg(convw + (size_t)gc * p.K + j);
                if (cs_in)
                    for (int j = 0; j < L; ++j)
                        hist[u][j] = Act<TA>::ld(cs_in + ((size_t)b * conv_dim + gc) * L + (L - 1 - j));
            }
        }
    }

    int ck_i = 0;  // next checkpoint (sorted by offset)
    const float A_exp = MIXER ? -expf(p.A_log[h]) : 0.f;
    const float dtb = MIXER ? p.dt_bias[h] : 0.f;

    for (int c = 0; c < NC; ++c) {
        const int t0 = c * C;
        // ---------------- stage 1: inputs ----------------
        if (MIXER) {
#pragma unroll
            for (int u = 0; u < CPT; ++u) {
                const int ch = tid + u * NT;
                if (ch >= NCH) continue;
                float* dst = ch < D ? sQ + ch : (ch < 2 * D ? sK + (ch - D) : sX + (ch - 2 * D));
                const int ds = ch < 2 * D ? QS : XS;
                const TA* src = mixed + (size_t)b * p.ms_b + gch[u];
#pragma unroll 4
                for (int t = 0; t < C; ++t) {
                    const int tg = t0 + t;
                    float val = 0.f;
                    if (tg < T) {
                        const float x = Act<TA>::ld(src + (size_t)tg * p.ms_t);
                        const float win[4] = {x, hist[u][0], hist[u][1], hist[u][2]};
                        const int valid = cs_in ? L : (tg < L ? tg : L);
                        val = Act<TA>::round(silu_f(conv_taps<TA>(win, wt[u], p.K, valid)));
                        hist[u][2] = hist[u][1];
                        hist[u][1] = hist[u][0];
                        hist[u][0] = x;
                    }
                    dst[t * ds] = val;
                }
            }
            if (tid < C) {
                const int tg = t0 + tid;
                float beta = 0.f, g = 0.f;
                if (tg < T) {
                    const size_t ai = (size_t)b * p.as_b + (size_t)tg * p.as_t + h;
                    beta = Act<TA>::round(sigmoid_f(Act<TA>::ld(static_cast<const TA*>(p.b) + ai)));
                    g = A_exp * softplus_f(Act<TA>::ld(static_cast<const TA*>(p.a) + ai) + dtb);
                }
                sB[tid] = beta;
                sG[tid] = g;
            }
        } else {
            for (int i = tid; i < C * D; i += NT) {
                const int t = i / D, d = i - t * D;
                const int tg = t0 + t;
                float q = 0.f, k = 0.f, v = 0.f;
                if (tg < T) {
                    const size_t row = ((size_t)b * T + tg) * p.Hv + h;
                    q = Act<TA>::ld(static_cast<const TA*>(p.q) + row * D + d);
                    k = Act<TA>::ld(static_cast<const TA*>(p.k) + row * D + d);
                    v = Act<TA>::ld(static_cast<const TA*>(p.v) + row * D + d);
                }
                sQ[t * QS + d] = q;
                sK[t * QS + d] = k;
                sX[t * XS + d] = v;
            }
            if (tid < C) {
                const int tg = t0 + tid;
                float beta = 0.f, g = 0.f;
                if (tg < T) {
                    const size_t row = ((size_t)b * T + tg) * p.Hv + h;
                    beta = Act<TA>::ld(static_cast<const TA*>(p.beta) + row);
                    g = Act<TA>::ld(static_cast<const TA*>(p.g) + row);
                }
                sB[tid] = beta;
                sG[tid] = g;
            }
        }
        __syncthreads();

        // ---------------- stage 2: norms, gamma ----------------
        {
            const bool l2 = MIXER || p.use_l2;
            for (int t = warp; t < C; t += NT / 32) {
                float aq = 0.f, ak = 0.f;
                for (int d = lane; d < D; d += 32) {
                    const float q = sQ[t * QS + d], k = sK[t * QS + d];
                    aq = fmaf(q, q, aq);
                    ak = fmaf(k, k, ak);
                }
                aq = warp_sum(aq);
                ak = warp_sum(ak);
                const float rq = l2 ? rsqrtf(aq + 1e-6f) : 1.f;
                const float rk = l2 ? rsqrtf(ak + 1e-6f) : 1.f;
                for (int d = lane; d < D; d += 32) {
                    sQ[t * QS + d] = (sQ[t * QS + d] * rq) * p.q_scale;
                    sK[t * QS + d] = sK[t * QS + d] * rk;
                }
            }
            if (tid == 0) {
                float acc = 0.f;
                for (int t = 0; t < C; ++t) {
                    acc += sG[t];
                    sG[t] = acc;
                }
            }
        }
        __syncthreads();
        if (tid < C) {
            sE[tid] = expf(sG[tid]);
            sF[tid] = expf(sG[C - 1] - sG[tid]);
        }

        // ---------------- stage 3: A and R = [beta V | beta K e^gamma] ----------------
        {
            const int ti = tid & 15, tj = tid >> 4;
            float acc[4][4];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[r][q] = 0.f;
            for (int d = 0; d < D; d += 4) {
                float4 ki[4], kj[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) ki[r] = *reinterpret_cast<const float4*>(sK + (ti + 16 * r) * QS + d);
#pragma unroll
                for (int q = 0; q < 4; ++q) kj[q] = *reinterpret_cast<const float4*>(sK + (tj + 16 * q) * QS + d);
#pragma unroll
                for (int r = 0; r < 4; ++r)
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        acc[r][q] = fmaf(ki[r].x, kj[q].x, acc[r][q]);
                        acc[r][q] = fmaf(ki[r].y, kj[q].y, acc[r][q]);
                        acc[r][q] = fmaf(ki[r].z, kj[q].z, acc[r][q]);
                        acc[r][q] = fmaf(ki[r].w, kj[q].w, acc[r][q]);
                    }
            }
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int i = ti + 16 * r, j = tj + 16 * q;
                    sA[i * AS + j] = j < i ? (sB[i] * acc[r][q]) * expf(sG[i] - sG[j]) : 0.f;
                }
        }
        for (int i = tid; i < C * D; i += NT) {
            const int t = i / D, d = i - t * D;
            const float bt = sB[t];
            sX[t * XS + d] = sX[t * XS + d] * bt;
            sX[t * XS + D + d] = (sK[t * QS + d] * bt) * expf(sG[t]);
        }
        __syncthreads();

        // ---------------- stage 4: forward substitution, column per thread ----------------
        if (tid < 2 * D) {
            float x[C];
#pragma unroll
            for (int i = 0; i < C; ++i) x[i] = sX[i * XS + tid];
#pragma unroll
            for (int i = 1; i < C; ++i) {
                float acc = x[i];
#pragma unroll
                for (int j = 0; j < i; ++j) acc = fmaf(-sA[i * AS + j], x[j], acc);
                x[i] = acc;
            }
#pragma unroll
            for (int i = 0; i < C; ++i) sX[i * XS + tid] = x[i];
        }
        __syncthreads();

        // ---------------- stage 5: P, v_new = U - W S, Oq = Q S ----------------
        {
            const int ti = tid & 15, tj = tid >> 4;
            float acc[4][4];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[r][q] = 0.f;
            for (int d = 0; d < D; d += 4) {
                float4 qi[4], kj[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) qi[r] = *reinterpret_cast<const float4*>(sQ + (ti + 16 * r) * QS + d);
#pragma unroll
                for (int q = 0; q < 4; ++q) kj[q] = *reinterpret_cast<const float4*>(sK + (tj + 16 * q) * QS + d);
#pragma unroll
                for (int r = 0; r < 4; ++r)
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        acc[r][q] = fmaf(qi[r].x, kj[q].x, acc[r][q]);
                        acc[r][q] = fmaf(qi[r].y, kj[q].y, acc[r][q]);
                        acc[r][q] = fmaf(qi[r].z, kj[q].z, acc[r][q]);
                        acc[r][q] = fmaf(qi[r].w, kj[q].w, acc[r][q]);
                    }
            }
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int i = ti + 16 * r, j = tj + 16 * q;
                    sA[i * AS + j] = j <= i ? acc[r][q] * expf(sG[i] - sG[j]) : 0.f;
                }
        }
        const int ri = tid >> 4, cj = tid & 15;  // rows ri*4 + r, columns cj + 16 * q
        float oacc[4][JC];
        {
            float vacc[4][JC];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int q = 0; q < JC; ++q) {
                    oacc[r][q] = 0.f;
                    vacc[r][q] = 0.f;
                }
            for (int d = 0; d < D; ++d) {
                float wv[4], qv[4], sv[JC];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    wv[r] = sX[(ri * 4 + r) * XS + D + d];
                    qv[r] = sQ[(ri * 4 + r) * QS + d];
                }
#pragma unroll
                for (int q = 0; q < JC; ++q) sv[q] = sS[d * D + cj + 16 * q];
#pragma unroll
                for (int r = 0; r < 4; ++r)
#pragma unroll
                    for (int q = 0; q < JC; ++q) {
                        vacc[r][q] = fmaf(wv[r], sv[q], vacc[r][q]);
                        oacc[r][q] = fmaf(qv[r], sv[q], oacc[r][q]);
                    }
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float e = sE[ri * 4 + r];
#pragma unroll
                for (int q = 0; q < JC; ++q) {
                    float* u = sX + (ri * 4 + r) * XS + cj + 16 * q;
                    *u = *u - vacc[r][q];
                    oacc[r][q] *= e;
                }
            }
        }
        __syncthreads();

        // ---------------- stage 6: O = Oq + P v_new, output; state update ----------------
        {
            const int smax = ri * 4 + 3;
            for (int s = 0; s <= smax; ++s) {
                float pv[4], vv[JC];
#pragma unroll
                for (int r = 0; r < 4; ++r) pv[r] = sA[(ri * 4 + r) * AS + s];
#pragma unroll
                for (int q = 0; q < JC; ++q) vv[q] = sX[s * XS + cj + 16 * q];
#pragma unroll
                for (int r = 0; r < 4; ++r)
#pragma unroll
                    for (int q = 0; q < JC; ++q) oacc[r][q] = fmaf(pv[r], vv[q], oacc[r][q]);
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int t = ri * 4 + r, tg = t0 + t;
                if (MIXER) {
                    float part = 0.f;
#pragma unroll
                    for (int q = 0; q < JC; ++q) {
                        const float o = Act<TA>::round(oacc[r][q]);
                        part = fmaf(o, o, part);
                    }
                    part = half_warp_sum(part);
                    const float rstd = rsqrtf(part / (float)D + p.eps);
                    if (tg < T) {
                        const TA* normw = static_cast<const TA*>(p.normw);
                        const TA* z = static_cast<const TA*>(p.z);
                        TA* out = static_cast<TA*>(p.out) + ((size_t)b * T + tg) * (size_t)(p.Hv * D) + h * D;
                        const TA* zr = z + (size_t)b * p.zs_b + (size_t)tg * p.zs_t + h * D;
#pragma unroll
                        for (int q = 0; q < JC; ++q) {
                            const int j = cj + 16 * q;
                            const float o = Act<TA>::round(oacc[r][q]);
                            const float y = Act<TA>::round(Act<TA>::ldg(normw + j) * Act<TA>::round(o * rstd));
                            Act<TA>::st(out + j, y * silu_f(Act<TA>::ld(zr + j)));
                        }
                    }
                } else if (tg < T) {
                    TA* out = static_cast<TA*>(p.out) + (((size_t)b * T + tg) * p.Hv + h) * D;
#pragma unroll
                    for (int q = 0; q < JC; ++q) Act<TA>::st(out + cj + 16 * q, oacc[r][q]);
                }
            }
        }
        {
            // state rows ri + 16 r, columns cj + 16 q
            constexpr int RI = D / 16;
            // sub-chunk checkpoints of this chunk (s_off < C): S e^{gamma_{s-1}} + sum_{t<s} ...
            while (ck_i < ck.n && (ck.off[ck_i] - 1) / C == c && ck.off[ck_i] - t0 < C) {
                const int s_off = ck.off[ck_i] - t0;
                const float gs = sG[s_off - 1];
                float acc[RI][JC];
#pragma unroll
                for (int r = 0; r < RI; ++r)
#pragma unroll
                    for (int q = 0; q < JC; ++q) acc[r][q] = 0.f;
                for (int t = 0; t < s_off; ++t) {
                    const float f = expf(gs - sG[t]);
                    float kv[RI], vv[JC];
#pragma unroll
                    for (int r = 0; r < RI; ++r) kv[r] = sK[t * QS + ri + 16 * r] * f;
#pragma unroll
                    for (int q = 0; q < JC; ++q) vv[q] = sX[t * XS + cj + 16 * q];
#pragma unroll
                    for (int r = 0; r < RI; ++r)
#pragma unroll
                        for (int q = 0; q < JC; ++q) acc[r][q] = fmaf(kv[r], vv[q], acc[r][q]);
                }
                const float es = expf(gs);
                if (p.S_ckpt) {
                    float* dst = p.S_ckpt + (size_t)ck.slot[ck_i] * p.B * p.Hv * D * D + sbase;
#pragma unroll
                    for (int r = 0; r < RI; ++r)
#pragma unroll
                        for (int q = 0; q < JC; ++q) {
                            const int i = ri + 16 * r, j = cj + 16 * q;
                            dst[i * D + j] = fmaf(sS[i * D + j], es, acc[r][q]);
                        }
                }
                ++ck_i;
            }
            float acc[RI][JC];
#pragma unroll
            for (int r = 0; r < RI; ++r)
#pragma unroll
                for (int q = 0; q < JC; ++q) acc[r][q] = 0.f;
            for (int t = 0; t < C; ++t) {
                const float f = sF[t];
                float kv[RI], vv[JC];
#pragma unroll
                for (int r = 0; r < RI; ++r) kv[r] = sK[t * QS + ri + 16 * r] * f;
#pragma unroll
                for (int q = 0; q < JC; ++q) vv[q] = sX[t * XS + cj + 16 * q];
#pragma unroll
                for (int r = 0; r < RI; ++r)
#pragma unroll
                    for (int q = 0; q < JC; ++q) acc[r][q] = fmaf(kv[r], vv[q], acc[r][q]);
            }
            const float ec = sE[C - 1];
#pragma unroll
            for (int r = 0; r < RI; ++r)
#pragma unroll
                for (int q = 0; q < JC; ++q) {
                    const int i = ri + 16 * r, j = cj + 16 * q;
                    sS[i * D + j] = fmaf(sS[i * D + j], ec, acc[r][q]);
                }
            // chunk-boundary checkpoint (s_off == C)
            while (ck_i < ck.n && ck.off[ck_i] - t0 == C) {
                if (p.S_ckpt) {
                    float* dst = p.S_ckpt + (size_t)ck.slot[ck_i] * p.B * p.Hv * D * D + sbase;
#pragma unroll
                    for (int r = 0; r < RI; ++r)
#pragma unroll
                        for (int q = 0; q < JC; ++q) {
                            const int i = ri + 16 * r, j = cj + 16 * q;
                            dst[i * D + j] = sS[i * D + j];
                        }
                }
                ++ck_i;
            }
        }
        __syncthreads();
    }

    if (p.S_out) {
        for (int i = tid; i < D * D / 4; i += NT)
            __stcs(reinterpret_cast<float4*>(p.S_out + sbase) + i, reinterpret_cast<const float4*>(sS)[i]);
    }
}

template <int D, typename TA, bool MIXER>
static cudaError_t launch_one(const MixParams& p, const CkptList& ck, cudaStream_t s) {
    constexpr size_t bytes = prefill::Smem<D>::BYTES;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(prefill_kernel<D, TA, MIXER>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    prefill_kernel<D, TA, MIXER><<<p.B * p.Hv, prefill::NT, bytes, s>>>(p, ck);
    return cudaGetLastError();
}

template <typename TA, bool MIXER>
static cudaError_t dispatch_dims(const MixParams& p, const CkptList& ck, int d, cudaStream_t s, bool* ok) {
    *ok = true;
    if (d == 128) return launch_one<128, TA, MIXER>(p, ck, s);
    if (d == 64) return launch_one<64, TA, MIXER>(p, ck, s);
    if (d == 32) return launch_one<32, TA, MIXER>(p, ck, s);
    *ok = false;
    return cudaSuccess;
}

cudaError_t launch_prefill(const MixParams& p, const CkptList& ck, int d, int dtype, bool mixer, cudaStream_t s,
                           bool* supported) {
    if (dtype == GDN_DTYPE_BF16)
        return mixer ? dispatch_dims<__nv_bfloat16, true>(p, ck, d, s, supported)
                     : dispatch_dims<__nv_bfloat16, false>(p, ck, d, s, supported);
    return mixer ? dispatch_dims<float, true>(p, ck, d, s, supported)
                 : dispatch_dims<float, false>(p, ck, d, s, supported);
}

}  // namespace gdn
