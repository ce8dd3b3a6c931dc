// K2: parallel preparation pass of the two-kernel chunked prefill.
//
// One CTA per (batch row, key head kh, chunk of C = 64 tokens), every chunk at
// once: this is the part of the chunked algorithm (deltanet.py:266-343) that
// does not depend on the recurrent state, so it runs fully parallel and the
// sequential kernel (gdn_prefill_seq.cu) is left with the state-touching
// products only.  Per CTA:
//
//   1. raw q / k rows of key head kh and v rows of its `rep` value heads,
//      tokens t0-3 .. t0+63, arrive by tensor-map loads (the 3 extra rows are
//      the conv history; rows before the sequence start come from the conv
//      state, or are absent);
//   2. causal conv + SiLU (deltanet.py:41-90, per-tap rounding to the
//      activation dtype), written to the workspace in bf16 - exactly the
//      values the reference feeds to the delta rule;
//   3. L2-norm factors rq = (|q|^2 + 1e-6)^-1/2, rk likewise (config.py:114-115);
//   4. the raw [k;q] rows as a bf16 operand in swizzled shared memory and one
//      tcgen05 MMA (kind::f16; bf16 products are exact): G = k k^T, P0 = q k^T;
//   5. per value head h of the key head: beta = sigmoid(b) rounded,
//      g = -exp(A_log) softplus(a + dt_bias), gamma = cumsum(g)
//      (deltanet.py:516-517, 278-281); with the normalised rows K = k rk and
//      Q = q rq dk^-1/2 applied as row / column factors,
//      A = tril(beta_i K_i.K_j e^{gamma_i-gamma_j}, -1),
//      P = Q_i.K_j e^{gamma_i-gamma_j} (j <= i), T = (I + A)^-1 by forward
//      substitution in fp32 (the reference's triangular solve,
//      deltanet.py:93-162, restated);
//   6. T and P, rounded to tf32, are written as ready-made K-major 128-byte
//      swizzled operand images that the sequential kernel copies straight
//      into shared memory.
//
// Workspace (one call; sizes from gdn_prefill_workspace_bytes):
//   qkv   bf16 [B][NC*64][conv_dim]      conv + SiLU outputs (tokens >= T are 0)
//   nrm   fp32 [B][Hk][NC][2][64]        rq, rk
//   gate  fp32 [B][Hv][NC][2][64]        beta, gamma (within the chunk)
//   tp    fp32 [B][Hv][NC][2][64*64]     T image, P image
#include "gdn_async.cuh"
#include "gdn_common.cuh"
#include "gdn_kernels.cuh"
#include "gdn_prefill_ws.cuh"
#include "gdn_tmap.h"
#include "gdn_umma.cuh"

namespace gdn {
namespace pprep {

constexpr int D = 128, C = 64, NT = 256, HIST = 3, ROWS = C + HIST;
constexpr uint32_t GROUP_BYTES = ROWS * D * 2;  // raw rows of one 128-channel group, bf16
constexpr int MAX_REP = 4;
constexpr int A_STRIDE = 68;                     // floats per row of an A matrix (conflict-free row writes)
constexpr uint32_t A_BYTES = C * A_STRIDE * 4;
constexpr uint32_t IMG_BYTES = C * C * 4;        // one 64x64 tf32 operand image

__host__ __device__ constexpr uint32_t region0_bytes(int rep) {
    const uint32_t stage = (uint32_t)(2 + rep) * GROUP_BYTES;
    const uint32_t kq = 128u * D * 4u;
    // per value head: the A matrix (inverted in place into T) and one operand image (P, then T)
    const uint32_t am = (uint32_t)rep * (A_BYTES + IMG_BYTES);
    const uint32_t m = stage > kq ? stage : kq;
    return ((m > am ? m : am) + 1023u) & ~1023u;
}
// small vectors after region 0 (floats): rq[64], rk[64], then per value head r
// beta, gamma, e^gamma, e^-gamma [MAX_REP][64]
constexpr int V_RQ = 0, V_RK = 64, V_B = 128, V_G = V_B + 64 * MAX_REP, V_EG = V_G + 64 * MAX_REP,
              V_ENG = V_EG + 64 * MAX_REP, V_END = V_ENG + 64 * MAX_REP;
__host__ __device__ constexpr uint32_t smem_bytes(int rep) { return region0_bytes(rep) + V_END * 4 + 64 + 1024; }

using TA = __nv_bfloat16;

__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
    const __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&t);
}

// Round a pair of values to bf16 (one packed conversion) and back to float.
__device__ __forceinline__ void round2(float& a, float& b) {
    const uint32_t u = pack_bf2(a, b);
    a = bf_lo(u);
    b = bf_hi(u);
}
// Column j of the inverse of the unit lower triangular 32x32 block I + A
// (A strictly lower triangular, row stride A_STRIDE) by forward substitution:
// X[i][j] = [i == j] - sum_{k<i} A[i][k] X[k][j] (X[k][j] = 0 for k < j).
// Four partial sums (k mod 4) on packed fp32 pairs; x starts at zero and A is
// zero on and above its diagonal, so the products past k = i - 1 add exact zeros.
__device__ __forceinline__ void tri_inverse_block32(const float* A, int j, float (&x)[32]) {
#pragma unroll
    for (int i = 0; i < 32; ++i) x[i] = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        float2 s01 = make_float2(0.f, 0.f), s23 = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < i; k += 4) {
            const float4 a = *reinterpret_cast<const float4*>(A + i * A_STRIDE + k);
            s01 = __ffma2_rn(make_float2(a.x, a.y), make_float2(x[k], x[k + 1]), s01);
            s23 = __ffma2_rn(make_float2(a.z, a.w), make_float2(x[k + 2], x[k + 3]), s23);
        }
        x[i] = (i == j ? 1.f : 0.f) - ((s01.x + s01.y) + (s23.x + s23.y));
    }
}

// out[i][jb..jb+7] (+)= sign * sum_k L[i][k] R[k][jb..jb+7] over 32 k, row stride A_STRIDE
// (packed fp32 pairs).
__device__ __forceinline__ void block_row8(const float* L, const float* R, int i, int jb, float* out, float sign) {
    float2 acc[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[e] = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 32; k += 4) {
        const float4 a = *reinterpret_cast<const float4*>(L + i * A_STRIDE + k);
        const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const float4 r0 = *reinterpret_cast<const float4*>(R + (k + kk) * A_STRIDE + jb);
            const float4 r1 = *reinterpret_cast<const float4*>(R + (k + kk) * A_STRIDE + jb + 4);
            const float2 a2 = make_float2(av[kk], av[kk]);
            acc[0] = __ffma2_rn(a2, make_float2(r0.x, r0.y), acc[0]);
            acc[1] = __ffma2_rn(a2, make_float2(r0.z, r0.w), acc[1]);
            acc[2] = __ffma2_rn(a2, make_float2(r1.x, r1.y), acc[2]);
            acc[3] = __ffma2_rn(a2, make_float2(r1.z, r1.w), acc[3]);
        }
    }
    *reinterpret_cast<float4*>(out + i * A_STRIDE + jb) =
        make_float4(sign * acc[0].x, sign * acc[0].y, sign * acc[1].x, sign * acc[1].y);
    *reinterpret_cast<float4*>(out + i * A_STRIDE + jb + 4) =
        make_float4(sign * acc[2].x, sign * acc[2].y, sign * acc[3].x, sign * acc[3].y);
}

__global__ void __launch_bounds__(NT, 3)
    prefill_prep_kernel(const MixParams p, const PrefillWs ws, const __grid_constant__ CUtensorMap tm_mixed,
                        const __grid_constant__ CUtensorMap tm_qkv) {
    extern __shared__ unsigned char raw[];
    const uint32_t raw_addr = smem_u32(raw);
    unsigned char* sm = raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const int rep = p.Hv / p.Hk;
    const uint32_t R0 = region0_bytes(rep);
    float* vec = reinterpret_cast<float*>(sm + R0);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + R0 + V_END * 4);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + R0 + V_END * 4 + 16);
    const uint32_t bar_ld = smem_u32(&bars[0]), bar_mma = smem_u32(&bars[1]);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int NC = ws.nc;
    const int c = blockIdx.x % NC;
    const int bk = blockIdx.x / NC;
    const int kh = bk % p.Hk, b = bk / p.Hk;
    const int t0 = c * C;
    const int T = p.T;
    const int ngroups = 2 + rep;
    const int conv_dim = 2 * p.Hk * D + p.Hv * D;
    const TA* cs_in = static_cast<const TA*>(p.cs_in);

    if (tid == 0) {
        mbar_init(bar_ld, 1);
        mbar_init(bar_mma, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        umma::tmem_alloc(smem_u32(tslot), 64);
        umma::tmem_relinquish();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *tslot;

    // group g: 0 = q of kh, 1 = k of kh, 2 + r = v of value head kh*rep + r
    auto group_channel = [&](int g) -> int {
        return g == 0 ? kh * D : (g == 1 ? p.Hk * D + kh * D : 2 * p.Hk * D + (kh * rep + g - 2) * D);
    };
    if (tid == 0) {
        mbar_arrive_expect_tx(bar_ld, (uint32_t)ngroups * GROUP_BYTES);
        for (int g = 0; g < ngroups; ++g)
            tma_load_3d(smem_u32(sm + g * GROUP_BYTES), &tm_mixed, group_channel(g), t0 - HIST, b, bar_ld);
    }
    // gate inputs of every value head of this key head (threads 64r..64r+63 ->
    // value head r, one token each), loaded while the rows arrive
    const int g_r = tid >> 6, g_t = tid & 63;
    float raw_a = 0.f, raw_b = 0.f;
    if (g_r < rep && t0 + g_t < T) {
        const size_t ai = (size_t)b * p.as_b + (size_t)(t0 + g_t) * p.as_t + kh * rep + g_r;
        raw_a = Act<TA>::ld(static_cast<const TA*>(p.a) + ai);
        raw_b = Act<TA>::ld(static_cast<const TA*>(p.b) + ai);
    }
    const bool ld_ok = mbar_wait_bounded(bar_ld, 0, GDN_DEVERR_TMA_TIMEOUT);
    if (__syncthreads_or(!ld_ok)) {
        // the copies may still land: wait for them (bounded) before the CTA exits
        if (tid == 0) mbar_wait_bounded(bar_ld, 0, GDN_DEVERR_TMA_TIMEOUT);
        __syncthreads();
        if (warp == 0) umma::tmem_dealloc(tmem, 64);
        return;
    }

    // ---- conv + SiLU, in place: thread -> an adjacent channel pair of one group ----
    // Taps newest first with one bf16 rounding per tap (deltanet.py:66-80), on packed channel
    // pairs: the first tap is a bf16x2 multiply (the reference's rounded product), the others
    // bf16x2 fused multiply-adds.  The reference adds in fp32 and then rounds to bf16; the
    // product of two bf16 values and a bf16 accumulator always sum exactly in fp32 unless their
    // magnitudes differ by more than 2^8 (accumulator larger) or 2^16 (product larger), so the
    // two roundings agree except when such a sum also lands exactly on a bf16 tie.
    for (int pr = tid; pr < ngroups * (D / 2); pr += NT) {
        const int g = pr / (D / 2), ch = (pr % (D / 2)) * 2;
        const int gc = group_channel(g) + ch;
        unsigned char* gbase = sm + g * GROUP_BYTES;
        const TA* cw = static_cast<const TA*>(p.convw) + (size_t)gc * 4;
        __nv_bfloat162 w[4];  // tap j of both channels
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = __halves2bfloat162(cw[j], cw[4 + j]);
        // history x[-3..-1] of both channels, packed like the rows
        __nv_bfloat162 x1, x2, x3;
        if (c > 0) {
            x3 = *reinterpret_cast<const __nv_bfloat162*>(gbase + 0 * D * 2 + ch * 2);
            x2 = *reinterpret_cast<const __nv_bfloat162*>(gbase + 1 * D * 2 + ch * 2);
            x1 = *reinterpret_cast<const __nv_bfloat162*>(gbase + 2 * D * 2 + ch * 2);
        } else {
            const TA zero = __float2bfloat16_rn(0.f);
            const TA* sa = cs_in ? cs_in + ((size_t)b * conv_dim + gc) * HIST : nullptr;
            const TA* sb2 = cs_in ? cs_in + ((size_t)b * conv_dim + gc + 1) * HIST : nullptr;
            x3 = __halves2bfloat162(sa ? sa[0] : zero, sb2 ? sb2[0] : zero);
            x2 = __halves2bfloat162(sa ? sa[1] : zero, sb2 ? sb2[1] : zero);
            x1 = __halves2bfloat162(sa ? sa[2] : zero, sb2 ? sb2[2] : zero);
        }
        const bool full_window = cs_in != nullptr || c > 0;  // every token has 3 predecessors
        // 16 tokens at a time: every raw value of the group is loaded before any output is stored
        // (the outputs overwrite the same rows, so interleaved loads and stores would serialise)
        for (int tb = 0; tb < C; tb += 16) {
            __nv_bfloat162 xr[16];
#pragma unroll
            for (int j = 0; j < 16; ++j)
                xr[j] = *reinterpret_cast<const __nv_bfloat162*>(gbase + (tb + j + HIST) * D * 2 + ch * 2);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int t = tb + j;
                const __nv_bfloat162 x0 = xr[j];
                const int tg = t0 + t;
                uint32_t outv = 0u;
                if (tg < T) {
                    __nv_bfloat162 acc = __hmul2(x0, w[3]);
                    if (full_window || tg >= 1) acc = __hfma2(x1, w[2], acc);
                    if (full_window || tg >= 2) acc = __hfma2(x2, w[1], acc);
                    if (full_window || tg >= 3) acc = __hfma2(x3, w[0], acc);
                    const float ca = __low2float(acc), cb = __high2float(acc);
                    outv = pack_bf2(__fdividef(ca, 1.0f + __expf(-ca)), __fdividef(cb, 1.0f + __expf(-cb)));
                }
                x3 = x2;
                x2 = x1;
                x1 = x0;
                *reinterpret_cast<uint32_t*>(gbase + (t + HIST) * D * 2 + ch * 2) = outv;
            }
        }
    }
    // conv outputs (staging rows 3..66 of every group) to the workspace: one tensor store per group
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
        for (int g = 0; g < ngroups; ++g)
            tma_store_3d(&tm_qkv, smem_u32(sm + g * GROUP_BYTES + HIST * D * 2), group_channel(g), t0, b);
        bulk_commit_group();
    }
    __syncthreads();

    // ---- L2-norm factors of q and k: warp per token (8 tokens per warp, loads first) ----
    float* sRQ = vec + V_RQ;
    float* sRK = vec + V_RK;
    {
        constexpr int TPW = C / (NT / 32);  // tokens per warp
        float sq[TPW], sk[TPW];
#pragma unroll
        for (int i = 0; i < TPW; ++i) {
            const int t = warp + i * (NT / 32);
            const uint2 qv = *reinterpret_cast<const uint2*>(sm + 0 * GROUP_BYTES + (t + HIST) * D * 2 + lane * 8);
            const uint2 kv = *reinterpret_cast<const uint2*>(sm + 1 * GROUP_BYTES + (t + HIST) * D * 2 + lane * 8);
            const float q0 = bf_lo(qv.x), q1 = bf_hi(qv.x), q2 = bf_lo(qv.y), q3 = bf_hi(qv.y);
            const float k0 = bf_lo(kv.x), k1 = bf_hi(kv.x), k2 = bf_lo(kv.y), k3 = bf_hi(kv.y);
            sq[i] = q0 * q0 + q1 * q1 + q2 * q2 + q3 * q3;
            sk[i] = k0 * k0 + k1 * k1 + k2 * k2 + k3 * k3;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
            for (int i = 0; i < TPW; ++i) {
                sq[i] += __shfl_xor_sync(0xffffffffu, sq[i], o);
                sk[i] += __shfl_xor_sync(0xffffffffu, sk[i], o);
            }
        }
        if (lane < TPW) {
            // lane i publishes token warp + 8 i (register index by a select chain, no local memory)
            float a = sq[0], k = sk[0];
#pragma unroll
            for (int i = 1; i < TPW; ++i) {
                a = lane == i ? sq[i] : a;
                k = lane == i ? sk[i] : k;
            }
            const int t = warp + lane * (NT / 32);
            const float rq = rsqrtf(a + 1e-6f), rk = rsqrtf(k + 1e-6f);
            sRQ[t] = rq;
            sRK[t] = rk;
            float* nrm = ws.nrm + (((size_t)b * p.Hk + kh) * NC + c) * 128;
            nrm[t] = rq;
            nrm[64 + t] = rk;
        }
    }
    __syncthreads();

    // ---- [k;q] as a bf16 K-major operand (rows 0..63 k, 64..127 q: the exact conv outputs;
    //      the norm factors are applied to G and P0 afterwards) over the staging area ----
    if (tid == 0) bulk_wait_group_read0();  // the conv-output stores have read the staging rows
    uint4 kq_raw[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const int idx = tid + u * NT, r = idx >> 4, c8 = (idx & 15) * 8;
        const int g = r < C ? 1 : 0, t = r & 63;
        kq_raw[u] = *reinterpret_cast<const uint4*>(sm + g * GROUP_BYTES + (t + HIST) * D * 2 + c8 * 2);
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const int idx = tid + u * NT, r = idx >> 4, c8 = (idx & 15) * 8;
        *reinterpret_cast<uint4*>(sm + umma::kmajor_off16(r, c8, 128)) = kq_raw[u];
    }
    fence_proxy_async_smem();
    umma::fence_before_sync();
    __syncthreads();
    if (tid == 0) {
        umma::fence_after_sync();
        const uint64_t d0 = umma::desc_kmajor0(smem_u32(sm));
        const uint32_t idesc = umma::idesc_bf16(128, 64, 0, 0);
        for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t d = umma::desc_add(d0, umma::kmajor_kstep(kk, 128));
            umma::mma_bf16(tmem, d, d, idesc, kk > 0);  // [G; P0] = [k; q] k^T (raw rows)
        }
        umma::mma_commit(bar_mma);
    }

    // ---- gates and gamma while the MMA runs ----
    float* sB = vec + V_B;
    float* sG = vec + V_G;
    if (g_r < rep) {
        const int h = kh * rep + g_r;
        float beta = 0.f, g = 0.f;
        if (t0 + g_t < T) {
            beta = Act<TA>::round(sigmoid_f(raw_b));
            g = -expf(p.A_log[h]) * softplus_f(raw_a + p.dt_bias[h]);
        }
        sB[g_r * 64 + g_t] = beta;
        sG[g_r * 64 + g_t] = g;
    }
    __syncthreads();
    if (tid < rep) {
        // sequential cumsum (the reference's torch.cumsum over the chunk), in registers
        float4* gr = reinterpret_cast<float4*>(sG + tid * 64);
        float4 g4[C / 4];
#pragma unroll
        for (int i = 0; i < C / 4; ++i) g4[i] = gr[i];
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < C / 4; ++i) {
            acc += g4[i].x;
            g4[i].x = acc;
            acc += g4[i].y;
            g4[i].y = acc;
            acc += g4[i].z;
            g4[i].z = acc;
            acc += g4[i].w;
            g4[i].w = acc;
        }
#pragma unroll
        for (int i = 0; i < C / 4; ++i) gr[i] = g4[i];
    }
    __syncthreads();
    float* sEG = vec + V_EG;
    float* sENG = vec + V_ENG;
    for (int i = tid; i < rep * C; i += NT) {
        const int r = i / C, t = i % C;
        sEG[i] = expf(sG[i]);
        sENG[i] = expf(-sG[i]) * sRK[t];  // the column's norm factor rides on e^{-gamma_j}
        float* gate = ws.gate + (((size_t)b * p.Hv + kh * rep + r) * NC + c) * 128;
        gate[t] = sB[r * 64 + t];
        gate[64 + t] = sG[r * 64 + t];
    }

    const bool mma_ok = mbar_wait_bounded(bar_mma, 0, GDN_DEVERR_MMA_TIMEOUT);
    umma::fence_after_sync();
    if (__syncthreads_or(!mma_ok)) {
        if (tid == 0) {
            mbar_wait_bounded(bar_mma, 0, GDN_DEVERR_MMA_TIMEOUT);
            bulk_wait_group0();
        }
        umma::fence_before_sync();
        __syncthreads();
        if (warp == 0) umma::tmem_dealloc(tmem, 64);
        return;
    }

    // ---- A (shared memory) and P (operand image) per value head from G, P0 ----
    // 32 columns at a time; every shared-memory operand of a half is read into
    // registers before the half's stores, so loads never wait behind stores.
    {
        const int q4 = warp & 3;
        const uint32_t lane_base = (uint32_t)(32 * q4) << 16;
        const bool g_rows = q4 < 2;
        const int t = g_rows ? lane + 32 * q4 : lane + 32 * (q4 - 2);
        for (int r = warp >> 2; r < rep; r += 2) {
            const float* gr = sG + r * 64;
            const float gt = gr[t];
            // decay e^{gamma_t - gamma_j}: as e^{gamma_t} e^{-gamma_j} when neither factor can
            // leave the normal range (gamma >= -80 over the chunk), else one exp per pair; the
            // column's norm factor rk_j rides on it (G and P0 are products of the raw rows)
            const bool split = gr[C - 1] >= -80.f;
            const float egt = sEG[r * 64 + t];
            // row factor: beta_t rk_t for A, rq_t dk^-1/2 for P (q * rq * dk^-1/2), folded into
            // the decay while the tensor-memory load is in flight
            const float rowf = g_rows ? sB[r * 64 + t] * sRK[t] : sRQ[t] * p.q_scale;
            float* arow = reinterpret_cast<float*>(sm + r * A_BYTES) + t * A_STRIDE;
            unsigned char* img = sm + rep * A_BYTES + r * IMG_BYTES;
#pragma unroll 1
            for (int hf = 0; hf < 2; ++hf) {
                float v[32], dec[32];
                umma::tmem_ld32(tmem + lane_base + 32 * hf, v);
                if (split) {
                    const float4* e4 = reinterpret_cast<const float4*>(sENG + r * 64 + 32 * hf);
                    const float2 eg2 = make_float2(egt * rowf, egt * rowf);
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const float4 e = e4[q];
                        const float2 d01 = __fmul2_rn(eg2, make_float2(e.x, e.y));
                        const float2 d23 = __fmul2_rn(eg2, make_float2(e.z, e.w));
                        dec[4 * q] = d01.x;
                        dec[4 * q + 1] = d01.y;
                        dec[4 * q + 2] = d23.x;
                        dec[4 * q + 3] = d23.y;
                    }
                } else {
                    const float4* g4 = reinterpret_cast<const float4*>(gr + 32 * hf);
                    const float4* k4 = reinterpret_cast<const float4*>(sRK + 32 * hf);
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const float4 e = g4[q], rk = k4[q];
                        dec[4 * q] = __expf(gt - e.x) * (rowf * rk.x);
                        dec[4 * q + 1] = __expf(gt - e.y) * (rowf * rk.y);
                        dec[4 * q + 2] = __expf(gt - e.z) * (rowf * rk.z);
                        dec[4 * q + 3] = __expf(gt - e.w) * (rowf * rk.w);
                    }
                }
                umma::tmem_wait_ld();
#pragma unroll
                for (int jj = 0; jj < 32; jj += 4) {
                    const int j = 32 * hf + jj;
                    const float2 p01 = __fmul2_rn(make_float2(v[jj], v[jj + 1]), make_float2(dec[jj], dec[jj + 1]));
                    const float2 p23 =
                        __fmul2_rn(make_float2(v[jj + 2], v[jj + 3]), make_float2(dec[jj + 2], dec[jj + 3]));
                    if (g_rows) {
                        float4 a;
                        a.x = j + 0 < t ? p01.x : 0.f;
                        a.y = j + 1 < t ? p01.y : 0.f;
                        a.z = j + 2 < t ? p23.x : 0.f;
                        a.w = j + 3 < t ? p23.y : 0.f;
                        *reinterpret_cast<float4*>(arow + j) = a;
                    } else {
                        float4 a;
                        a.x = j + 0 <= t ? umma::tf32_rna(p01.x) : 0.f;
                        a.y = j + 1 <= t ? umma::tf32_rna(p01.y) : 0.f;
                        a.z = j + 2 <= t ? umma::tf32_rna(p23.x) : 0.f;
                        a.w = j + 3 <= t ? umma::tf32_rna(p23.y) : 0.f;
                        *reinterpret_cast<float4*>(img + umma::kmajor_off(t, j, C)) = a;
                    }
                }
            }
        }
    }
    fence_proxy_async_smem();
    umma::fence_before_sync();
    __syncthreads();
    if (tid == 0) {  // P images to the workspace
        for (int r = 0; r < rep; ++r)
            bulk_store(ws.tp + ((((size_t)b * p.Hv + kh * rep + r) * NC + c) * 2 + 1) * (C * C),
                       smem_u32(sm + rep * A_BYTES + r * IMG_BYTES), IMG_BYTES);
        bulk_commit_group();
    }

    // ---- T = (I + A)^-1 in 32x32 blocks (the doubling merge of deltanet.py:146-160) ----
    // In place over A: T11, T22 by forward substitution (one warp per block, lane = column,
    // written back after the block's rows are read), X = A21 T11 (parked in the zero upper-right
    // block), then T21 = -T22 X over the dead A21.
    float* Tall = reinterpret_cast<float*>(sm);  // A, then T, of value head r at Tall + r * C * A_STRIDE
    if (warp < 2 * rep) {
        const int r = warp >> 1, o = 32 * (warp & 1);
        const float* A = reinterpret_cast<const float*>(sm + r * A_BYTES) + o * A_STRIDE + o;
        float* Tr = Tall + r * C * A_STRIDE + o * A_STRIDE + o;
        float x[32];
        tri_inverse_block32(A, lane, x);
#pragma unroll
        for (int i = 0; i < 32; ++i) Tr[i * A_STRIDE + lane] = x[i];
    }
    __syncthreads();
    for (int u = tid; u < rep * 128; u += NT) {
        const int r = u >> 7, i = (u & 127) >> 2, jb = (u & 3) * 8;
        const float* A = reinterpret_cast<const float*>(sm + r * A_BYTES);
        float* Tr = Tall + r * C * A_STRIDE;
        block_row8(A + 32 * A_STRIDE, Tr, i, jb, Tr + 32, 1.f);  // X[i][jb..] = A21 T11
    }
    __syncthreads();
    for (int u = tid; u < rep * 128; u += NT) {
        const int r = u >> 7, i = (u & 127) >> 2, jb = (u & 3) * 8;
        float* Tr = Tall + r * C * A_STRIDE;
        block_row8(Tr + 32 * A_STRIDE + 32, Tr + 32, i, jb, Tr + 32 * A_STRIDE, -1.f);  // T21 = -T22 X
    }
    if (tid == 0) bulk_wait_group_read0();  // the P images are read: their space takes the T images
    __syncthreads();
    // T images (tf32, zero above the diagonal), then to the workspace
    for (int u = tid; u < rep * C * (C / 4); u += NT) {
        const int r = u / (C * C / 4), w = u % (C * C / 4), i = w >> 4, j = (w & 15) * 4;
        const float4 v = *reinterpret_cast<const float4*>(Tall + r * C * A_STRIDE + i * A_STRIDE + j);
        const float4 o = make_float4(j + 0 <= i ? umma::tf32_rna(v.x) : 0.f, j + 1 <= i ? umma::tf32_rna(v.y) : 0.f,
                                     j + 2 <= i ? umma::tf32_rna(v.z) : 0.f, j + 3 <= i ? umma::tf32_rna(v.w) : 0.f);
        *reinterpret_cast<float4*>(sm + rep * A_BYTES + r * IMG_BYTES + umma::kmajor_off(i, j, C)) = o;
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
        for (int r = 0; r < rep; ++r)
            bulk_store(ws.tp + (((size_t)b * p.Hv + kh * rep + r) * NC + c) * 2 * (C * C),
                       smem_u32(sm + rep * A_BYTES + r * IMG_BYTES), IMG_BYTES);
        bulk_commit_group();
    }
    if (tid == 0) bulk_wait_group0();  // conv-output stores complete before the CTA exits
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tmem, 64);
}

}  // namespace pprep

bool prefill_prep_supported(const MixParams& p, int d, int dtype) {
    const int rep = p.Hk > 0 ? p.Hv / p.Hk : 0;
    auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    return dtype == GDN_DTYPE_BF16 && d == 128 && p.K == 4 && (rep == 1 || rep == 2 || rep == 4) && al(p.mixed) &&
           (p.ms_b % 8) == 0 && (p.ms_t % 8) == 0 && al(p.z) && (p.zs_b % 8) == 0 && (p.zs_t % 8) == 0 &&
           al(p.out);
}

cudaError_t launch_prefill_prep(const MixParams& p, const PrefillWs& ws, cudaStream_t s) {
    const int rep = p.Hv / p.Hk;
    const uint64_t conv_dim = 2ull * p.Hk * 128 + (uint64_t)p.Hv * 128;
    CUtensorMap tm_mixed;
    if (!encode_tmap_3d_bf16(&tm_mixed, p.mixed, conv_dim, (uint64_t)p.T, (uint64_t)p.B, (uint64_t)p.ms_t * 2,
                             (uint64_t)p.ms_b * 2, 128, pprep::ROWS))
        return cudaErrorInvalidValue;
    CUtensorMap tm_qkv;
    if (!encode_tmap_3d_bf16(&tm_qkv, ws.qkv, conv_dim, (uint64_t)ws.tp_len, (uint64_t)p.B, conv_dim * 2,
                             conv_dim * 2 * (uint64_t)ws.tp_len, 128, pprep::C))
        return cudaErrorInvalidValue;
    const int bytes = (int)pprep::smem_bytes(rep);
    static int attr_bytes[64] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (attr_bytes[dev] < bytes) {
        e = cudaFuncSetAttribute(pprep::prefill_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        if (e != cudaSuccess) return e;
        attr_bytes[dev] = bytes;
    }
    const int grid = p.B * p.Hk * ws.nc;
    pprep::prefill_prep_kernel<<<grid, pprep::NT, bytes, s>>>(p, ws, tm_mixed, tm_qkv);
    return cudaGetLastError();
}

unsigned int prefill_prep_device_error(bool clear) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
    if (clear && v) {
        const unsigned int zero = 0;
        cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
    }
    return v;
}

}  // namespace gdn
