// K1 (streaming form): persistent, bulk-copy pipelined token-by-token Gated DeltaNet.
//
// Each CTA (one per SM) holds two independent consumer groups of 256 threads.
// A group walks (batch row, value head) tiles; each tile's inputs - the fp32
// state S[d][d] (one contiguous 64 KB block at d = 128), the raw projections
// of its q/k/v channels and z for every token, its conv-state and
// conv-weight rows - arrive in the group's shared-memory stage through bulk
// asynchronous copies (cp.async.bulk; the state and the small inputs complete
// on two mbarriers).  As soon as the group has moved the state into registers
// it issues the copy of its next tile's state, and after the conv the copies
// of the next tile's inputs, so those copies overlap the rest of the
// computation.  The two groups interleave, keeping two state
// tiles in flight per SM while the SMs do the conv / norm / delta-rule /
// gated-norm work.  The new state leaves from registers with streaming
// 128-bit stores (in place when state_out == state_in).
//
// With a slot table (gdn_mixer_verify_slots) the state and conv state of row b
// come from pool slot slot_table[b][0] and the state after token t goes to
// pool slot slot_table[b][t]: speculative-decode rollback becomes a swap of
// two table entries (gdn_slots.cu) instead of a copy.
//
// Math per token is that of decode_kernel (gdn_decode.cu): the reference's
// deltanet.py:41-90 (conv), :186-189 (L2 norm), :516-517 (gates),
// :210-221 (delta rule), config.py:136-143 (gated RMSNorm).
#include "gdn_async.cuh"
#include "gdn_common.cuh"
#include "gdn_kernels.cuh"

namespace gdn {
namespace dtma {

constexpr int GT = 256;     // threads per consumer group
constexpr int NG = 2;       // consumer groups per CTA
constexpr int NT = GT * NG;
constexpr int KC = 4;       // conv taps of the streaming kernel
constexpr int LC = KC - 1;  // conv-state length

template <int D, int TMAX, typename TA>
struct GroupLayout {
    static constexpr int ES = (int)sizeof(TA);
    static constexpr int CG = D / 4, RG = GT / CG;
    // stage: filled by bulk copies
    static constexpr int S_BYTES = D * D * 4;
    static constexpr int M_BYTES = TMAX * D * ES;  // one of q / k / v / z, all tokens
    static constexpr int OFF_S = 0;
    static constexpr int OFF_MQ = OFF_S + S_BYTES;
    static constexpr int OFF_MK = OFF_MQ + M_BYTES;
    static constexpr int OFF_MV = OFF_MK + M_BYTES;
    static constexpr int OFF_Z = OFF_MV + M_BYTES;
    static constexpr int OFF_CS = OFF_Z + M_BYTES;           // [3][D][LC]
    static constexpr int OFF_CW = OFF_CS + 3 * D * LC * ES;  // [3][D][KC]
    static constexpr int STAGE_END = OFF_CW + 3 * D * KC * ES;
    // work area: private to the group, valid while the stage refills
    static constexpr int OFF_CONV = (STAGE_END + 15) / 16 * 16;  // [TMAX][3D] f32 conv outputs q|k|v
    static constexpr int OFF_ZF = OFF_CONV + TMAX * 3 * D * 4;   // [TMAX][D] f32
    static constexpr int OFF_U = OFF_ZF + TMAX * D * 4;          // [D]
    static constexpr int OFF_O = OFF_U + D * 4;                  // [D]
    static constexpr int OFF_RED = OFF_O + D * 4;                // [2][RG][D]
    static constexpr int OFF_GATE = OFF_RED + 2 * RG * D * 4;    // [2][TMAX]
    static constexpr int OFF_BAR = (OFF_GATE + 2 * TMAX * 4 + 7) / 8 * 8;
    static constexpr int BYTES = (OFF_BAR + 16 + 127) / 128 * 128;  // two mbarriers: inputs, state
};

// Pool slot of column `col` of row b's slot table; -1 (and the error bit) when
// the entry is out of range, so a bad table is never followed.
__device__ __forceinline__ int row_slot(const MixParams& p, int b, int col) {
    const int s = __ldg(p.slot_table + (size_t)b * p.n_slots + col);
    if (s < 0 || s >= p.n_slots) {
        atomicOr(&g_device_error, GDN_DEVERR_BAD_SLOT);
        return -1;
    }
    return s;
}

// Output slot of checkpoint i of row b: the caller's index, or the pool slot.
__device__ __forceinline__ int ckpt_slot(const MixParams& p, const CkptList& ck, int i, int b) {
    return p.slot_table ? row_slot(p, b, ck.slot[i]) : ck.slot[i];
}

__device__ __forceinline__ void group_sync(int id) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(GT) : "memory");
}

__device__ __forceinline__ bool group_any(bool pred, int id) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}\n"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(GT)
        : "memory");
    return r != 0;
}

template <int D, int TMAX, typename TA>
__global__ void __launch_bounds__(NT, 1)
    decode_tma_kernel(const MixParams p, const CkptList ck, const int num_tiles) {
    using GL = GroupLayout<D, TMAX, TA>;
    constexpr int CG = GL::CG, RG = GL::RG, RPT = D / RG;
    static_assert(D % RG == 0 && RPT >= 4 && RPT % 4 == 0, "bad tiling");

    extern __shared__ __align__(128) unsigned char smem[];
    const int grp = threadIdx.x / GT, tid = threadIdx.x % GT, lane = tid & 31;
    const int bar_id = 1 + grp;  // named barrier of this group (0 is __syncthreads)
    unsigned char* gbase = smem + grp * GL::BYTES;
    float* cbuf = reinterpret_cast<float*>(gbase + GL::OFF_CONV);
    float* zbuf = reinterpret_cast<float*>(gbase + GL::OFF_ZF);
    float* su = reinterpret_cast<float*>(gbase + GL::OFF_U);
    float* so = reinterpret_cast<float*>(gbase + GL::OFF_O);
    float* red = reinterpret_cast<float*>(gbase + GL::OFF_RED);
    float* sgate = reinterpret_cast<float*>(gbase + GL::OFF_GATE);
    const uint32_t bar = smem_u32(gbase + GL::OFF_BAR), bar_s = bar + 8u;

    const int cg = tid % CG, rg = tid / CG;
    const int rep = p.Hv / p.Hk;
    const int T = p.T;
    const int conv_dim = 2 * p.Hk * D + p.Hv * D;
    const bool has_cs = p.cs_in != nullptr;
    const bool has_S = p.S_in != nullptr;
    const TA* gmixed = static_cast<const TA*>(p.mixed);
    const TA* gz = static_cast<const TA*>(p.z);

    if (tid == 0) {
        mbar_init(bar, 1);
        mbar_init(bar_s, 1);
        fence_mbar_init();
    }
    __syncthreads();

    // Thread 0 of the group issues the copies of one tile into the group's stage: the state
    // (on bar_s: it refills as soon as the state is in registers) and the small inputs (on bar:
    // they refill after the conv).
    auto start_slot = [&](int b) -> size_t {  // pool slot of the starting state (slot mode)
        if (!p.slot_table) return 0;
        const int s0 = row_slot(p, b, 0);
        return s0 < 0 ? 0 : (size_t)s0;
    };
    auto issue_state = [&](int tile) {
        const size_t slot0 = start_slot(tile / p.Hv);
        mbar_arrive_expect_tx(bar_s, (uint32_t)GL::S_BYTES);
        bulk_load(smem_u32(gbase + GL::OFF_S), p.S_in + (slot0 * p.B * p.Hv + tile) * D * D, GL::S_BYTES, bar_s);
    };
    auto issue = [&](int tile) {
        const int b = tile / p.Hv, h = tile - (tile / p.Hv) * p.Hv, kh = h / rep;
        const uint32_t mrow = D * sizeof(TA);
        const int c0 = kh * D, c1 = p.Hk * D + kh * D, c2 = 2 * p.Hk * D + h * D;
        const size_t slot0 = start_slot(b);
        uint32_t bytes = 4u * T * mrow + 3u * D * KC * sizeof(TA);
        if (has_cs) bytes += 3u * D * LC * sizeof(TA);
        mbar_arrive_expect_tx(bar, bytes);
        for (int t = 0; t < T; ++t) {
            const TA* row = gmixed + (size_t)b * p.ms_b + (size_t)t * p.ms_t;
            bulk_load(smem_u32(gbase + GL::OFF_MQ + t * mrow), row + c0, mrow, bar);
            bulk_load(smem_u32(gbase + GL::OFF_MK + t * mrow), row + c1, mrow, bar);
            bulk_load(smem_u32(gbase + GL::OFF_MV + t * mrow), row + c2, mrow, bar);
            bulk_load(smem_u32(gbase + GL::OFF_Z + t * mrow), gz + (size_t)b * p.zs_b + (size_t)t * p.zs_t + h * D,
                      mrow, bar);
        }
        const TA* cw = static_cast<const TA*>(p.convw);
        const int chans[3] = {c0, c1, c2};
#pragma unroll
        for (int g = 0; g < 3; ++g) {
            if (has_cs)
                bulk_load(smem_u32(gbase + GL::OFF_CS + g * D * LC * (int)sizeof(TA)),
                          static_cast<const TA*>(p.cs_in) + ((slot0 * p.B + b) * conv_dim + chans[g]) * LC,
                          D * LC * sizeof(TA), bar);
            bulk_load(smem_u32(gbase + GL::OFF_CW + g * D * KC * (int)sizeof(TA)), cw + (size_t)chans[g] * KC,
                      D * KC * sizeof(TA), bar);
        }
    };

    const int worker = blockIdx.x * NG + grp, nworkers = gridDim.x * NG;
    if (tid == 0 && worker < num_tiles) {
        if (has_S) issue_state(worker);
        issue(worker);
    }

    // gate inputs of the next tile are loaded one tile ahead into registers
    float na = 0.f, nb = 0.f;
    auto load_gates = [&](int tile) {
        if (tid < T && tile < num_tiles) {
            const int b = tile / p.Hv, h = tile - (tile / p.Hv) * p.Hv;
            const size_t ai = (size_t)b * p.as_b + (size_t)tid * p.as_t + h;
            na = Act<TA>::ld(static_cast<const TA*>(p.a) + ai);
            nb = Act<TA>::ld(static_cast<const TA*>(p.b) + ai);
        }
    };
    load_gates(worker);

    const TA* sMQ = reinterpret_cast<const TA*>(gbase + GL::OFF_MQ);
    const TA* sZ = reinterpret_cast<const TA*>(gbase + GL::OFF_Z);
    const TA* sCS = reinterpret_cast<const TA*>(gbase + GL::OFF_CS);
    const TA* sCW = reinterpret_cast<const TA*>(gbase + GL::OFF_CW);
    const float* sS = reinterpret_cast<const float*>(gbase + GL::OFF_S);

    uint32_t k = 0;
    bool failed = false;
    for (int tile = worker; tile < num_tiles; tile += nworkers, ++k) {
        const int b = tile / p.Hv, h = tile - (tile / p.Hv) * p.Hv, kh = h / rep;
        const float cur_a = na, cur_b = nb;
        load_gates(tile + nworkers);
        if (tid < T) {
            sgate[tid] = Act<TA>::round(sigmoid_f(cur_b));
            sgate[TMAX + tid] = expf(-expf(p.A_log[h]) * softplus_f(cur_a + p.dt_bias[h]));
        }

        const bool ok = (!has_S || mbar_wait_bounded(bar_s, k & 1u, GDN_DEVERR_TMA_TIMEOUT)) &&
                        mbar_wait_bounded(bar, k & 1u, GDN_DEVERR_TMA_TIMEOUT);

        // ---- consume the stage: state to registers, conv windows, conv of every token, z ----
        // The state is read before the group agrees on the waits (a thread whose wait gave up
        // reads stale, in-bounds data that is then discarded), so one barrier both agrees on
        // failure and releases the state region for the next tile's state.
        float4 S[RPT];  // rows rg*RPT .. +RPT-1, columns cg*4 .. cg*4+3
#pragma unroll
        for (int r = 0; r < RPT; ++r)
            S[r] = has_S ? *reinterpret_cast<const float4*>(sS + (rg * RPT + r) * D + cg * 4)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        if (group_any(!ok, bar_id)) {
            failed = true;
            break;
        }
        if (has_S && tid == 0 && tile + nworkers < num_tiles) {
            fence_proxy_async_smem();
            issue_state(tile + nworkers);
        }

        const bool own_qk = (h % rep) == 0;
        const int cbeg = own_qk ? 0 : 2 * D;
        {
            // conv windows (raw inputs, bit-exact copies): final state + checkpoints
            const int nwin = (p.cs_out ? 1 : 0) + (p.cs_ckpt ? ck.n : 0);
            for (int w = 0; w < nwin; ++w) {
                const bool fin = p.cs_out && w == 0;
                const int ci_idx = p.cs_out ? w - 1 : w;
                const int off = fin ? T : ck.off[ci_idx];
                const int slot = fin ? 0 : ckpt_slot(p, ck, ci_idx, b);
                if (slot < 0) continue;
                TA* dst = fin ? static_cast<TA*>(p.cs_out) + (size_t)b * conv_dim * LC
                              : static_cast<TA*>(p.cs_ckpt) + ((size_t)slot * p.B + b) * conv_dim * LC;
                for (int c = cbeg + tid; c < 3 * D; c += GT) {
                    const int g = c / D, ci = c % D;
                    const int gc = (g == 0 ? kh * D : (g == 1 ? p.Hk * D + kh * D : 2 * p.Hk * D + h * D)) + ci;
                    const TA* mg = sMQ + g * (GL::M_BYTES / (int)sizeof(TA));
#pragma unroll
                    for (int i = 0; i < LC; ++i) {
                        const int pos = off - LC + i;
                        TA val;
                        if (pos >= 0) val = mg[pos * D + ci];
                        else if (has_cs) val = sCS[(g * D + ci) * LC + (LC + pos)];
                        else val = TA(0.0f);
                        dst[(size_t)gc * LC + i] = val;
                    }
                }
            }
        }
        // conv + SiLU of every token, sliding a 4-tap window along the sequence;
        // indices past the conv channels copy z (balances the two phases)
        for (int c = tid; c < 3 * D + D; c += GT) {
            if (c >= 3 * D) {
                const int j = c - 3 * D;
                for (int t = 0; t < T; ++t) zbuf[t * D + j] = Act<TA>::ld(sZ + t * D + j);
                continue;
            }
            const int g = c / D, ci = c % D;
            const TA* mg = sMQ + g * (GL::M_BYTES / (int)sizeof(TA));
            float w[KC], win[KC];
#pragma unroll
            for (int j = 0; j < KC; ++j) w[j] = Act<TA>::ld(sCW + (g * D + ci) * KC + j);
            win[0] = 0.f;
#pragma unroll
            for (int j = 1; j < KC; ++j) win[j] = has_cs ? Act<TA>::ld(sCS + (g * D + ci) * LC + (LC - j)) : 0.f;
            for (int t = 0; t < T; ++t) {
                win[0] = Act<TA>::ld(mg + t * D + ci);
                cbuf[t * 3 * D + c] = Act<TA>::round(silu_f(conv_taps<TA>(win, w, KC, has_cs ? LC : t)));
#pragma unroll
                for (int j = KC - 1; j > 0; --j) win[j] = win[j - 1];
            }
        }
        group_sync(bar_id);  // stage consumed: refill it with this group's next tile
        if (tid == 0 && tile + nworkers < num_tiles) {
            fence_proxy_async_smem();
            issue(tile + nworkers);
        }

        int ck_i = 0;
        for (int t = 0; t < T; ++t) {
            const float* cq = cbuf + t * 3 * D;
            const float* ckk = cq + D;
            const float* cv = cq + 2 * D;
            // norms (every warp computes them; no barrier)
            float aq = 0.f, ak = 0.f, aqk = 0.f;
#pragma unroll
            for (int i = lane; i < D; i += 32) {
                const float q = cq[i], kk = ckk[i];
                aq = fmaf(q, q, aq);
                ak = fmaf(kk, kk, ak);
                aqk = fmaf(q, kk, aqk);
            }
            aq = warp_sum(aq);
            ak = warp_sum(ak);
            aqk = warp_sum(aqk);
            const float rq = rsqrtf(aq + 1e-6f), rk = rsqrtf(ak + 1e-6f);
            const float qk = aqk * rq * p.q_scale * rk;
            const float beta = sgate[t], alpha = sgate[TMAX + t];

            float kr[RPT], qr[RPT];
            const float2 rk2 = make_float2(rk, rk), rq2 = make_float2(rq, rq), qs2 = make_float2(p.q_scale, p.q_scale);
#pragma unroll
            for (int r4 = 0; r4 < RPT; r4 += 4) {
                const float4 k4 = *reinterpret_cast<const float4*>(ckk + rg * RPT + r4);
                const float4 q4 = *reinterpret_cast<const float4*>(cq + rg * RPT + r4);
                const float2 k01 = __fmul2_rn(make_float2(k4.x, k4.y), rk2), k23 = __fmul2_rn(make_float2(k4.z, k4.w), rk2);
                const float2 q01 = __fmul2_rn(__fmul2_rn(make_float2(q4.x, q4.y), rq2), qs2);
                const float2 q23 = __fmul2_rn(__fmul2_rn(make_float2(q4.z, q4.w), rq2), qs2);
                kr[r4] = k01.x; kr[r4 + 1] = k01.y; kr[r4 + 2] = k23.x; kr[r4 + 3] = k23.y;
                qr[r4] = q01.x; qr[r4 + 1] = q01.y; qr[r4 + 2] = q23.x; qr[r4 + 3] = q23.y;
            }
            // packed fp32 pairs: the same fused multiply-adds, two lanes per instruction
            float2 pk01 = make_float2(0.f, 0.f), pk23 = pk01, pq01 = pk01, pq23 = pk01;
#pragma unroll
            for (int r = 0; r < RPT; ++r) {
                const float2 kv = make_float2(kr[r], kr[r]), qv = make_float2(qr[r], qr[r]);
                const float2 s01 = make_float2(S[r].x, S[r].y), s23 = make_float2(S[r].z, S[r].w);
                pk01 = __ffma2_rn(kv, s01, pk01);
                pk23 = __ffma2_rn(kv, s23, pk23);
                pq01 = __ffma2_rn(qv, s01, pq01);
                pq23 = __ffma2_rn(qv, s23, pq23);
            }
            const float4 pk = make_float4(pk01.x, pk01.y, pk23.x, pk23.y);
            const float4 pq = make_float4(pq01.x, pq01.y, pq23.x, pq23.y);
            reinterpret_cast<float4*>(red + rg * D)[cg] = pk;
            reinterpret_cast<float4*>(red + (RG + rg) * D)[cg] = pq;
            group_sync(bar_id);
            // threads [0, D) reduce k.S into u; threads [D, 2D) reduce q.S into alpha q.S
            for (int jj = tid; jj < 2 * D; jj += GT) {
                const int j = jj % D, half = jj / D;
                float acc = 0.f;
#pragma unroll
                for (int g = 0; g < RG; ++g) acc += red[(half * RG + g) * D + j];
                if (half == 0) su[j] = beta * (cv[j] - alpha * acc);
                else so[j] = alpha * acc;
            }
            group_sync(bar_id);

            {
                const float4 u4 = reinterpret_cast<const float4*>(su)[cg];
                const float2 u01 = make_float2(u4.x, u4.y), u23 = make_float2(u4.z, u4.w);
                const float2 al = make_float2(alpha, alpha);
#pragma unroll
                for (int r = 0; r < RPT; ++r) {
                    const float2 kv = make_float2(kr[r], kr[r]);
                    const float2 s01 = __ffma2_rn(kv, u01, __fmul2_rn(al, make_float2(S[r].x, S[r].y)));
                    const float2 s23 = __ffma2_rn(kv, u23, __fmul2_rn(al, make_float2(S[r].z, S[r].w)));
                    S[r] = make_float4(s01.x, s01.y, s23.x, s23.y);
                }
            }
            while (ck_i < ck.n && ck.off[ck_i] == t + 1) {
                const int slot = p.S_ckpt ? ckpt_slot(p, ck, ck_i, b) : -1;
                if (slot >= 0) {
                    float4* dst = reinterpret_cast<float4*>(p.S_ckpt + ((size_t)slot * p.B * p.Hv + tile) *
                                                                           (size_t)(D * D));
#pragma unroll
                    for (int r = 0; r < RPT; ++r) __stcs(dst + (rg * RPT + r) * CG + cg, S[r]);
                }
                ++ck_i;
            }

            // gated RMSNorm of token t (sum of squares recomputed by every warp);
            // o = alpha q.S + (q.k) u
            float ss = 0.f;
#pragma unroll
            for (int j = lane; j < D; j += 32) {
                const float o = Act<TA>::round(fmaf(qk, su[j], so[j]));
                ss = fmaf(o, o, ss);
            }
            ss = warp_sum(ss);
            const float rstd = rsqrtf(ss / (float)D + p.eps);
            const TA* normw = static_cast<const TA*>(p.normw);
            TA* out = static_cast<TA*>(p.out) + ((size_t)b * T + t) * (size_t)(p.Hv * D) + h * D;
            for (int j = tid; j < D; j += GT) {
                const float o = Act<TA>::round(fmaf(qk, su[j], so[j]));
                const float y = Act<TA>::round(Act<TA>::ldg(normw + j) * Act<TA>::round(o * rstd));
                Act<TA>::st(out + j, y * silu_f(zbuf[t * D + j]));
            }
            // su / so / red are rewritten by the next token; after the last token the next
            // tile's first two barriers come before any thread writes them (or the gates)
            if (t + 1 < T) group_sync(bar_id);
        }

        if (p.S_out) {
            float4* dst = reinterpret_cast<float4*>(p.S_out + (size_t)tile * D * D);
#pragma unroll
            for (int r = 0; r < RPT; ++r) __stcs(dst + (rg * RPT + r) * CG + cg, S[r]);
        }
    }

    if (failed && tid == 0) {
        // the copies this group waited for may still land: wait for them (bounded) before exiting
        if (has_S) mbar_wait_bounded(bar_s, k & 1u, GDN_DEVERR_TMA_TIMEOUT);
        mbar_wait_bounded(bar, k & 1u, GDN_DEVERR_TMA_TIMEOUT);
    }
}

template <int D, int TMAX, typename TA>
cudaError_t launch_one(const MixParams& p, const CkptList& ck, cudaStream_t s) {
    constexpr int bytes = NG * GroupLayout<D, TMAX, TA>::BYTES;
    static_assert(bytes <= 232448, "shared memory budget");
    static bool attr_set[64] = {false};
    static int sm_count[64] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(decode_tma_kernel<D, TMAX, TA>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        if (e != cudaSuccess) return e;
        e = cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    const int tiles = p.B * p.Hv;
    int grid = (tiles + NG - 1) / NG;
    if (grid > sm_count[dev]) grid = sm_count[dev];
    decode_tma_kernel<D, TMAX, TA><<<grid, NT, bytes, s>>>(p, ck, tiles);
    return cudaGetLastError();
}

template <typename TA>
bool aligned_for_bulk(const MixParams& p, int d) {
    const long long es = sizeof(TA);
    auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    const long long conv_dim = 2LL * p.Hk * d + (long long)p.Hv * d;
    if (!al(p.mixed) || !al(p.z) || !al(p.convw) || (p.S_in && !al(p.S_in))) return false;
    if ((p.ms_b * es) % 16 || (p.ms_t * es) % 16 || (p.zs_b * es) % 16 || (p.zs_t * es) % 16) return false;
    if ((d * es) % 16 || (d * KC * es) % 16) return false;
    if (p.cs_in && (!al(p.cs_in) || (conv_dim * LC * es) % 16 || (d * LC * es) % 16)) return false;
    return true;
}

template <typename TA>
cudaError_t dispatch(const MixParams& p, const CkptList& ck, int d, cudaStream_t s, bool* ok) {
    constexpr bool bf = sizeof(TA) == 2;
    // bf16 takes any T <= 8; fp32 only the single-token step (its 8-token stages do not fit twice)
    *ok = aligned_for_bulk<TA>(p, d) && p.K == KC && (p.T == 1 || (bf && p.T <= 8)) && (d == 128 || d == 64);
    if (!*ok) return cudaSuccess;
    if (p.T == 1) return d == 128 ? launch_one<128, 1, TA>(p, ck, s) : launch_one<64, 1, TA>(p, ck, s);
    if constexpr (bf) return d == 128 ? launch_one<128, 8, TA>(p, ck, s) : launch_one<64, 8, TA>(p, ck, s);
    *ok = false;
    return cudaSuccess;
}

}  // namespace dtma

cudaError_t launch_decode_tma(const MixParams& p, const CkptList& ck, int d, int dtype, cudaStream_t s,
                              bool* supported) {
    if (dtype == GDN_DTYPE_BF16) return dtma::dispatch<__nv_bfloat16>(p, ck, d, s, supported);
    return dtma::dispatch<float>(p, ck, d, s, supported);
}

unsigned int decode_tma_device_error(bool clear) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
    if (clear && v) {
        const unsigned int zero = 0;
        cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
    }
    return v;
}

}  // namespace gdn
