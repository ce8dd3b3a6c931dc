// K1: fused token-by-token Gated DeltaNet step (decode, speculative verify).
//
// One CTA owns one (batch row, value head).  Its fp32 state tile
// S[dk][dv] is read from HBM once into registers (coalesced 128-bit loads:
// each warp streams whole rows), updated in registers for every token of the
// call, and written back once (in place when state_out == state_in).  Per
// token, everything between the input projections and out_proj is fused:
//   conv-state shift + depthwise causal conv + SiLU   (deltanet.py:41-90)
//   q/k L2 norm, q * dk^-1/2                          (deltanet.py:186-189)
//   beta = sigmoid(b), g = -exp(A_log) softplus(a+dt_bias)  (deltanet.py:516-517)
//   S <- a S;  u = beta (v - k S);  S <- S + k^T u;  o = q S (deltanet.py:210-221)
//   gated RMSNorm                                      (config.py:136-143)
// One read of S serves both k.S and q.S: o = a (q.S) + (q.k) u.
//
// The kernel is HBM-bound: per (b, h) it moves 2 * dk * dv * 4 bytes of state
// and a few KB of inputs.
#include "gdn_common.cuh"
#include "gdn_kernels.cuh"
#include "gdn_conv_windows.cuh"

namespace gdn {

template <int DK, int DV, int NT, typename TA, bool MIXER>
__global__ void __launch_bounds__(NT, (DK * DV >= 128 * 128) ? 2 : 4)
    decode_kernel(const MixParams p, const CkptList ck) {
    constexpr int CG = DV / 4;     // float4 column groups
    constexpr int RG = NT / CG;    // row groups
    constexpr int RPT = DK / RG;   // rows per thread
    constexpr int NW = NT / 32;
    static_assert(NT % CG == 0 && DK % RG == 0 && RPT >= 1, "bad decode tiling");

    const int bh = blockIdx.x;
    const int b = bh / p.Hv, h = bh - (bh / p.Hv) * p.Hv;
    const int rep = p.Hv / p.Hk;
    const int kh = h / rep;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int cg = tid % CG, rg = tid / CG;

    __shared__ __align__(16) float sq[DK];
    __shared__ __align__(16) float sk[DK];
    __shared__ __align__(16) float sv[DV];
    __shared__ __align__(16) float su[DV];
    __shared__ __align__(16) float so[DV];
    __shared__ __align__(16) float red[2][RG][DV];
    __shared__ float sc[8];
    __shared__ float snorm[NW];

    // 1. stream the state tile in (all loads issued before any use)
    const size_t sbase = (size_t)bh * DK * DV;
    float4 S[RPT];
    if (p.S_in) {
        const float4* src = reinterpret_cast<const float4*>(p.S_in + sbase);
#pragma unroll
        for (int r = 0; r < RPT; ++r) S[r] = __ldcs(src + (size_t)(r * RG + rg) * CG + cg);
    } else {
#pragma unroll
        for (int r = 0; r < RPT; ++r) S[r] = make_float4(0.f, 0.f, 0.f, 0.f);
    }

    if (MIXER) write_conv_windows<TA, DK, DV, NT>(p, ck, b, h, kh, rep);

    const int conv_dim = 2 * p.Hk * DK + p.Hv * DV;
    const int L = p.K - 1;
    const TA* mixed = static_cast<const TA*>(p.mixed);
    const TA* cs_in = static_cast<const TA*>(p.cs_in);

    int ck_i = 0;
    for (int t = 0; t < p.T; ++t) {
        // 2. inputs of token t: q, k (key head kh), v (value head h), gates
        if (MIXER) {
            const TA* convw = static_cast<const TA*>(p.convw);
            for (int c = tid; c < 2 * DK + DV; c += NT) {
                int gc;
                float* dst;
                if (c < DK) {
                    gc = kh * DK + c;
                    dst = sq + c;
                } else if (c < 2 * DK) {
                    gc = p.Hk * DK + kh * DK + (c - DK);
                    dst = sk + (c - DK);
                } else {
                    gc = 2 * p.Hk * DK + h * DV + (c - 2 * DK);
                    dst = sv + (c - 2 * DK);
                }
                float w[4], win[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    w[j] = 0.f;
                    win[j] = 0.f;
                }
                for (int j = 0; j < p.K; ++j) {
                    w[j] = Act<TA>::ldg(convw + (size_t)gc * p.K + j);
                    const int pos = t - j;
                    if (pos >= 0)
                        win[j] = Act<TA>::ld(mixed + (size_t)b * p.ms_b + (size_t)pos * p.ms_t + gc);
                    else if (cs_in)
                        win[j] = Act<TA>::ld(cs_in + ((size_t)b * conv_dim + gc) * L + (L + pos));
                }
                const int valid = cs_in ? L : t;
                *dst = Act<TA>::round(silu_f(conv_taps<TA>(win, w, p.K, valid)));
            }
            if (tid == 0) {
                const size_t ai = (size_t)b * p.as_b + (size_t)t * p.as_t + h;
                const float bb = Act<TA>::ld(static_cast<const TA*>(p.b) + ai);
                const float aa = Act<TA>::ld(static_cast<const TA*>(p.a) + ai);
                sc[0] = Act<TA>::round(sigmoid_f(bb));
                const float g = -expf(p.A_log[h]) * softplus_f(aa + p.dt_bias[h]);
                sc[1] = expf(g);
            }
        } else {
            const size_t row = ((size_t)b * p.T + t) * p.Hv + h;
            for (int c = tid; c < DK; c += NT) {
                sq[c] = Act<TA>::ld(static_cast<const TA*>(p.q) + row * DK + c);
                sk[c] = Act<TA>::ld(static_cast<const TA*>(p.k) + row * DK + c);
            }
            for (int c = tid; c < DV; c += NT) sv[c] = Act<TA>::ld(static_cast<const TA*>(p.v) + row * DV + c);
            if (tid == 0) {
                sc[0] = Act<TA>::ld(static_cast<const TA*>(p.beta) + row);
                sc[1] = expf(Act<TA>::ld(static_cast<const TA*>(p.g) + row));
            }
        }
        __syncthreads();

        // 3. |q|^2, |k|^2 and q.k of the raw conv outputs (one warp each)
        if (warp < 3) {
            float acc = 0.f;
            for (int i = lane; i < DK; i += 32) {
                const float x = warp == 1 ? sk[i] : sq[i];
                const float y = warp == 0 ? sq[i] : sk[i];
                acc = fmaf(x, y, acc);
            }
            acc = warp_sum(acc);
            if (lane == 0) sc[2 + warp] = acc;
        }
        __syncthreads();
        const bool l2 = MIXER || p.use_l2;
        const float rq = l2 ? rsqrtf(sc[2] + 1e-6f) : 1.0f;
        const float rk = l2 ? rsqrtf(sc[3] + 1e-6f) : 1.0f;
        const float beta = sc[0], alpha = sc[1];
        const float qk = sc[4] * rq * p.q_scale * rk;

        // 4. partial k.S and q.S over this thread's rows, reduced through smem
        float4 pk = make_float4(0.f, 0.f, 0.f, 0.f), pq = pk;
#pragma unroll
        for (int r = 0; r < RPT; ++r) {
            const int row = r * RG + rg;
            const float kv = sk[row] * rk;
            const float qv = (sq[row] * rq) * p.q_scale;
            pk.x = fmaf(kv, S[r].x, pk.x); pk.y = fmaf(kv, S[r].y, pk.y);
            pk.z = fmaf(kv, S[r].z, pk.z); pk.w = fmaf(kv, S[r].w, pk.w);
            pq.x = fmaf(qv, S[r].x, pq.x); pq.y = fmaf(qv, S[r].y, pq.y);
            pq.z = fmaf(qv, S[r].z, pq.z); pq.w = fmaf(qv, S[r].w, pq.w);
        }
        reinterpret_cast<float4*>(&red[0][rg][0])[cg] = pk;
        reinterpret_cast<float4*>(&red[1][rg][0])[cg] = pq;
        __syncthreads();
        for (int j = tid; j < DV; j += NT) {
            float ks = 0.f, qs = 0.f;
#pragma unroll
            for (int g = 0; g < RG; ++g) {
                ks += red[0][g][j];
                qs += red[1][g][j];
            }
            const float u = beta * (sv[j] - alpha * ks);
            su[j] = u;
            so[j] = fmaf(alpha, qs, qk * u);
        }
        __syncthreads();

        // 5. S <- alpha S + k u^T
        {
            const float4 u4 = reinterpret_cast<const float4*>(su)[cg];
#pragma unroll
            for (int r = 0; r < RPT; ++r) {
                const float kv = sk[r * RG + rg] * rk;
                S[r].x = fmaf(kv, u4.x, alpha * S[r].x);
                S[r].y = fmaf(kv, u4.y, alpha * S[r].y);
                S[r].z = fmaf(kv, u4.z, alpha * S[r].z);
                S[r].w = fmaf(kv, u4.w, alpha * S[r].w);
            }
        }
        // checkpoints after token t (sorted list; duplicates each get a copy)
        while (ck_i < ck.n && ck.off[ck_i] == t + 1) {
            if (p.S_ckpt) {
                float4* dst =
                    reinterpret_cast<float4*>(p.S_ckpt + (size_t)ck.slot[ck_i] * p.B * p.Hv * DK * DV + sbase);
#pragma unroll
                for (int r = 0; r < RPT; ++r) __stcs(dst + (size_t)(r * RG + rg) * CG + cg, S[r]);
            }
            ++ck_i;
        }

        // 6. output of token t
        if (MIXER) {
            // gated RMSNorm over dv: o rounded to the activation dtype first
            float part = 0.f;
            for (int j = tid; j < DV; j += NT) {
                const float o = Act<TA>::round(so[j]);
                part = fmaf(o, o, part);
            }
            part = warp_sum(part);
            if (lane == 0) snorm[warp] = part;
            __syncthreads();
            float ss = 0.f;
#pragma unroll
            for (int w = 0; w < NW; ++w) ss += snorm[w];
            const float rstd = rsqrtf(ss / (float)DV + p.eps);
            const TA* normw = static_cast<const TA*>(p.normw);
            const TA* z = static_cast<const TA*>(p.z);
            TA* out = static_cast<TA*>(p.out);
            for (int j = tid; j < DV; j += NT) {
                const float o = Act<TA>::round(so[j]);
                const float y = Act<TA>::round(Act<TA>::ldg(normw + j) * Act<TA>::round(o * rstd));
                const float zz = Act<TA>::ld(z + (size_t)b * p.zs_b + (size_t)t * p.zs_t + h * DV + j);
                Act<TA>::st(out + ((size_t)b * p.T + t) * (size_t)(p.Hv * DV) + h * DV + j, y * silu_f(zz));
            }
        } else {
            TA* out = static_cast<TA*>(p.out);
            const size_t row = ((size_t)b * p.T + t) * p.Hv + h;
            for (int j = tid; j < DV; j += NT) Act<TA>::st(out + row * DV + j, so[j]);
        }
        __syncthreads();
    }

    if (p.S_out) {
        float4* dst = reinterpret_cast<float4*>(p.S_out + sbase);
#pragma unroll
        for (int r = 0; r < RPT; ++r) __stcs(dst + (size_t)(r * RG + rg) * CG + cg, S[r]);
    }
}

template <int DK, int DV, typename TA, bool MIXER>
static cudaError_t launch_one(const MixParams& p, const CkptList& ck, cudaStream_t s) {
    constexpr int NT = 256;
    decode_kernel<DK, DV, NT, TA, MIXER><<<p.B * p.Hv, NT, 0, s>>>(p, ck);
    return cudaGetLastError();
}

template <typename TA, bool MIXER>
static cudaError_t dispatch_dims(const MixParams& p, const CkptList& ck, int dk, int dv, cudaStream_t s,
                                 bool* ok) {
    *ok = true;
    if (dk == 128 && dv == 128) return launch_one<128, 128, TA, MIXER>(p, ck, s);
    if (dk == 64 && dv == 64) return launch_one<64, 64, TA, MIXER>(p, ck, s);
    if (dk == 32 && dv == 32) return launch_one<32, 32, TA, MIXER>(p, ck, s);
    *ok = false;
    return cudaSuccess;
}

cudaError_t launch_decode(const MixParams& p, const CkptList& ck, int dk, int dv, int dtype, bool mixer,
                          cudaStream_t s, bool* supported) {
    if (dtype == GDN_DTYPE_BF16)
        return mixer ? dispatch_dims<__nv_bfloat16, true>(p, ck, dk, dv, s, supported)
                     : dispatch_dims<__nv_bfloat16, false>(p, ck, dk, dv, s, supported);
    return mixer ? dispatch_dims<float, true>(p, ck, dk, dv, s, supported)
                 : dispatch_dims<float, false>(p, ck, dk, dv, s, supported);
}

}  // namespace gdn
