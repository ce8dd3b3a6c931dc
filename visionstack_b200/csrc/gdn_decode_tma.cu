// K1 (streaming form): persistent, bulk-copy pipelined token-by-token Gated DeltaNet.
//
// Each CTA (one per SM) holds two independent consumer groups of 256 threads.
// A group walks (batch row, value head) tiles; each tile's inputs - the fp32
// state S[d][d] (one contiguous 64 KB block at d = 128), the raw projections
// of its q/k/v channels and z for every token, its conv-state and
// conv-weight rows - arrive in the group's shared-memory stage through bulk
// asynchronous copies (cp.async.bulk; the state and the small inputs complete
// on two mbarriers), issued by the lanes of the group's first warp.  The pool
// slots, gate inputs and decay constants of the next tile are looked up one
// tile ahead.  The two groups interleave, keeping two state tiles in flight
// per SM while the SMs do the conv / norm / delta-rule / gated-norm work.
//
// The state lives in registers and leaves with streaming 128-bit stores (in
// place when state_out == state_in).  An SM sustains only ~30 B/clk of such
// stores, so a multi-token call (speculative verify: a 64 KB checkpoint per
// token) is store-bound; its stores are therefore spread in quarters over the
// work that follows each update (the next token's norms, products and
// reduction, or the next tile's conv phase), instead of stalling every warp
// on the store queue at once.  The single-token step loads its next state as
// early as possible instead and stores its final state at the end of the tile.
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

#include <type_traits>

namespace gdn {
namespace dtma {

constexpr int GT = 256;     // threads per consumer group
constexpr int NG = 2;       // consumer groups per CTA
constexpr int NT = GT * NG;
constexpr int KC = 4;       // conv taps of the streaming kernel
constexpr int LC = KC - 1;  // conv-state length
// Checkpoints whose pool slots are looked up one tile ahead and kept in shared
// memory (slot mode); later ones look the table up where they are written.
constexpr int NCKS = 16;

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
    static constexpr int OFF_SLOT = OFF_GATE + 2 * TMAX * 4;     // [2][NCKS] checkpoint pool slots
    static constexpr int OFF_BAR = (OFF_SLOT + 2 * NCKS * 4 + 7) / 8 * 8;
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

    // Multi-token calls (TMAX > 1) defer the last token's state stores into the next tile's
    // conv phase, so its state is loaded after that phase; the single-token step loads the
    // next state first (its copy then starts earliest) and stores the final state at once.
    constexpr bool DEFER = TMAX > 1;

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
    // launched as a programmatic dependent: the next kernel may start as CTAs retire, and
    // nothing below touches global memory before the previous kernel has completed
    pdl_launch_dependents();
    pdl_wait();

    // Warp 0 of the group issues the copies of one tile into the group's stage: the state (on
    // bar_s, one copy by lane 0: it refills as soon as the state is in registers) and the small
    // inputs (on bar, spread over the lanes: they refill after the conv).  `slot0` is the pool
    // slot of the tile's starting state (0 without a slot table).
    auto issue_state = [&](int tile, size_t slot0) {
        mbar_arrive_expect_tx(bar_s, (uint32_t)GL::S_BYTES);
        bulk_load(smem_u32(gbase + GL::OFF_S), p.S_in + (slot0 * p.B * p.Hv + tile) * D * D, GL::S_BYTES, bar_s);
    };
    auto issue = [&](int tile, size_t slot0) {
        const int b = tile / p.Hv, h = tile - (tile / p.Hv) * p.Hv, kh = h / rep;
        constexpr uint32_t mrow = D * sizeof(TA);
        const int c0 = kh * D, c1 = p.Hk * D + kh * D, c2 = 2 * p.Hk * D + h * D;
        if (lane == 0) {
            uint32_t bytes = 4u * T * mrow + 3u * D * KC * sizeof(TA);
            if (has_cs) bytes += 3u * D * LC * sizeof(TA);
            mbar_arrive_expect_tx(bar, bytes);
        }
        __syncwarp();
        // copy i < 4T: token i / 4, stream i % 4 (q, k, v rows of the projections, z); then the
        // conv weights and the conv states of the three channel groups
        const int nrow = 4 * T;
        for (int i = lane; i < nrow + 6; i += 32) {
            if (i < nrow) {
                const int t = i >> 2, st = i & 3;
                const TA* src = st == 3 ? gz + (size_t)b * p.zs_b + (size_t)t * p.zs_t + h * D
                                        : gmixed + (size_t)b * p.ms_b + (size_t)t * p.ms_t +
                                              (st == 0 ? c0 : (st == 1 ? c1 : c2));
                bulk_load(smem_u32(gbase + GL::OFF_MQ + st * GL::M_BYTES + t * mrow), src, mrow, bar);
            } else {
                const int j = i - nrow, g = j % 3;
                const int ch = g == 0 ? c0 : (g == 1 ? c1 : c2);
                if (j < 3)
                    bulk_load(smem_u32(gbase + GL::OFF_CW + g * D * KC * (int)sizeof(TA)),
                              static_cast<const TA*>(p.convw) + (size_t)ch * KC, D * KC * sizeof(TA), bar);
                else if (has_cs)
                    bulk_load(smem_u32(gbase + GL::OFF_CS + g * D * LC * (int)sizeof(TA)),
                              static_cast<const TA*>(p.cs_in) + ((slot0 * p.B + b) * conv_dim + ch) * LC,
                              D * LC * sizeof(TA), bar);
            }
        }
    };
    auto start_slot = [&](int tile) -> int {  // pool slot of the tile's starting state (slot mode)
        if (!p.slot_table) return 0;
        const int s0 = row_slot(p, tile / p.Hv, 0);
        return s0 < 0 ? 0 : s0;
    };

    const int worker = blockIdx.x * NG + grp, nworkers = gridDim.x * NG;
    if (tid < 32 && worker < num_tiles) {
        const size_t s0 = (size_t)start_slot(worker);
        if (has_S && lane == 0) issue_state(worker, s0);
        issue(worker, s0);
    }

    // Looked up one tile ahead into registers: the gate inputs and decay constants of the next
    // tile's head, and in slot mode the pool slots of its starting state and of its checkpoints.
    float na = 0.f, nb = 0.f, nalog = 0.f, ndtb = 0.f;
    int nslot0 = 0, nck = -1;
    auto prefetch = [&](int tile) {
        if (tile >= num_tiles) return;
        const int b = tile / p.Hv, h = tile - (tile / p.Hv) * p.Hv;
        if (tid < T) {
            const size_t ai = (size_t)b * p.as_b + (size_t)tid * p.as_t + h;
            na = Act<TA>::ld(static_cast<const TA*>(p.a) + ai);
            nb = Act<TA>::ld(static_cast<const TA*>(p.b) + ai);
            nalog = p.A_log[h];
            ndtb = p.dt_bias[h];
        }
        if (p.slot_table) {
            if (tid < 32) nslot0 = start_slot(tile);
            if (tid < ck.n && tid < NCKS) nck = row_slot(p, b, ck.slot[tid]);
        }
    };
    prefetch(worker);
    static_assert(D <= GT, "one output column per thread");
    const float nw = tid < D ? Act<TA>::ldg(static_cast<const TA*>(p.normw) + tid) : 0.f;

    const TA* sMQ = reinterpret_cast<const TA*>(gbase + GL::OFF_MQ);
    const TA* sZ = reinterpret_cast<const TA*>(gbase + GL::OFF_Z);
    const TA* sCS = reinterpret_cast<const TA*>(gbase + GL::OFF_CS);
    const TA* sCW = reinterpret_cast<const TA*>(gbase + GL::OFF_CW);
    const float* sS = reinterpret_cast<const float*>(gbase + GL::OFF_S);

    // The state lives in registers: rows rg*RPT .. +RPT-1, columns cg*4 .. cg*4+3.  Its stores
    // (checkpoints, final state) are not issued in one burst after the update, which stalls
    // every warp on the store queue at the same moment, but in four quarters spread over the
    // work that follows: the end of the token's gated norm, then the next token's norms,
    // products and reduction, or for the last token of a tile the next tile's conv phase.
    // pend0 / pend1 are the destinations of the state held in S that are still owed a store
    // (null when none; the same for every thread of the group).
    float4 S[RPT];
    float4* pend0 = nullptr;
    float4* pend1 = nullptr;
    auto flush = [&](auto quarter) {
        constexpr int Q = decltype(quarter)::value, R0 = Q * (RPT / 4), R1 = R0 + RPT / 4;
        if (pend0 == nullptr) return;
#pragma unroll
        for (int r = R0; r < R1; ++r) {
            __stcs(pend0 + (rg * RPT + r) * CG + cg, S[r]);
            if (pend1) __stcs(pend1 + (rg * RPT + r) * CG + cg, S[r]);
        }
        if (Q == 3) pend0 = pend1 = nullptr;
    };
    auto owe = [&](float4* dst) {  // the state in S must also go to dst
        if (!pend0) pend0 = dst;
        else if (!pend1) pend1 = dst;
        else {
#pragma unroll
            for (int r = 0; r < RPT; ++r) __stcs(dst + (rg * RPT + r) * CG + cg, S[r]);
        }
    };
    using Q0 = std::integral_constant<int, 0>;
    using Q1 = std::integral_constant<int, 1>;
    using Q2 = std::integral_constant<int, 2>;
    using Q3 = std::integral_constant<int, 3>;

    uint32_t k = 0;
    bool failed = false;
    for (int tile = worker; tile < num_tiles; tile += nworkers, ++k) {
        const int b = tile / p.Hv, h = tile - (tile / p.Hv) * p.Hv, kh = h / rep;
        const float cur_a = na, cur_b = nb, cur_alog = nalog, cur_dtb = ndtb;
        const int cur_ck = nck;
        prefetch(tile + nworkers);
        if (tid < T) {
            sgate[tid] = Act<TA>::round(sigmoid_f(cur_b));
            sgate[TMAX + tid] = expf(-expf(cur_alog) * softplus_f(cur_a + cur_dtb));
        }
        // checkpoint slots of this tile, double-buffered by tile parity: the previous tile's last
        // readers may still be in its final token (no barrier ends a tile), and the group_any
        // barrier below publishes these before any reader of this tile
        int* sck = reinterpret_cast<int*>(gbase + GL::OFF_SLOT) + (k & 1u) * NCKS;
        if (p.slot_table && tid < ck.n && tid < NCKS) sck[tid] = cur_ck;
        auto ck_slot = [&](int i) -> int {  // output slot of checkpoint i of this tile
            if (!p.slot_table) return ck.slot[i];
            return i < NCKS ? sck[i] : row_slot(p, b, ck.slot[i]);
        };

        const bool ok = (!has_S || mbar_wait_bounded(bar_s, k & 1u, GDN_DEVERR_TMA_TIMEOUT)) &&
                        mbar_wait_bounded(bar, k & 1u, GDN_DEVERR_TMA_TIMEOUT);

        const bool own_qk = (h % rep) == 0;
        const int cbeg = own_qk ? 0 : 2 * D;
        // destination of window w: -1 the final conv state, else checkpoint w (null: bad slot)
        auto window_dst = [&](int w) -> TA* {
            if (w < 0) return static_cast<TA*>(p.cs_out) + (size_t)b * conv_dim * LC;
            const int slot = ck_slot(w);
            return slot < 0 ? nullptr : static_cast<TA*>(p.cs_ckpt) + ((size_t)slot * p.B + b) * conv_dim * LC;
        };
        // One conv window, one channel per thread: the single-token step writes only the final
        // conv state, and spreading its 3D channels over every thread beats fewer, wider stores.
        auto write_window_per_channel = [&](TA* dst, int off) {
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
        };
        // Conv windows (raw inputs, bit-exact copies) in one pass: the final conv state (offset T)
        // and the conv checkpoints.  A work item is (window, channel group, block of 8 channels):
        // it reads each tap's 8 channels with one 16-byte load (taps before the first token from
        // the conv state) and writes the block's [8][LC] span, contiguous in the conv state,
        // with 16-byte stores.
        auto write_windows = [&]() {
            constexpr int CB = 8, NB = D / CB;
            const int nwin = (p.cs_out ? 1 : 0) + (p.cs_ckpt ? ck.n : 0);
            const int g0 = cbeg / D, ng = 3 - g0;
            for (int it = tid; it < nwin * ng * NB; it += GT) {
                const int w = it / (ng * NB), rem = it - w * (ng * NB);
                const int g = g0 + rem / NB, ci0 = (rem % NB) * CB;
                const bool fin = p.cs_out && w == 0;
                const int ci_idx = p.cs_out ? w - 1 : w;
                TA* dst = window_dst(fin ? -1 : ci_idx);
                if (!dst) continue;
                const int off = fin ? T : ck.off[ci_idx];
                const int gch = g == 0 ? kh * D : (g == 1 ? p.Hk * D + kh * D : 2 * p.Hk * D + h * D);
                const TA* mg = sMQ + g * (GL::M_BYTES / (int)sizeof(TA));
                const TA* cs = sCS + (g * D + ci0) * LC;
                uint4* d4 = reinterpret_cast<uint4*>(dst + (size_t)(gch + ci0) * LC);
                if constexpr (sizeof(TA) == 2) {
                    uint32_t r[LC][4];  // tap i: channels ci0 .. ci0+7 as bf16 pairs
#pragma unroll
                    for (int i = 0; i < LC; ++i) {
                        const int pos = off - LC + i;
                        if (pos >= 0) {
                            const uint4 v = *reinterpret_cast<const uint4*>(mg + pos * D + ci0);
                            r[i][0] = v.x; r[i][1] = v.y; r[i][2] = v.z; r[i][3] = v.w;
                        } else {
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                const uint32_t lo = has_cs ? __bfloat16_as_ushort(cs[(2 * k) * LC + LC + pos]) : 0u;
                                const uint32_t hi = has_cs ? __bfloat16_as_ushort(cs[(2 * k + 1) * LC + LC + pos]) : 0u;
                                r[i][k] = lo | (hi << 16);
                            }
                        }
                    }
                    // (channel, tap) order: c0t0 c0t1 | c0t2 c1t0 | c1t1 c1t2 | c2t0 ...
                    uint32_t o[12];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        o[3 * k] = __byte_perm(r[0][k], r[1][k], 0x5410);
                        o[3 * k + 1] = __byte_perm(r[2][k], r[0][k], 0x7610);
                        o[3 * k + 2] = __byte_perm(r[1][k], r[2][k], 0x7632);
                    }
                    d4[0] = make_uint4(o[0], o[1], o[2], o[3]);
                    d4[1] = make_uint4(o[4], o[5], o[6], o[7]);
                    d4[2] = make_uint4(o[8], o[9], o[10], o[11]);
                } else {
                    float v[CB * LC];
#pragma unroll
                    for (int e = 0; e < CB * LC; ++e) {
                        const int c = e / LC, i = e % LC, pos = off - LC + i;
                        v[e] = pos >= 0 ? Act<TA>::ld(mg + pos * D + ci0 + c)
                                        : (has_cs ? Act<TA>::ld(cs + c * LC + LC + pos) : 0.f);
                    }
#pragma unroll
                    for (int q = 0; q < CB * LC / 4; ++q)
                        d4[q] = make_uint4(__float_as_uint(v[4 * q]), __float_as_uint(v[4 * q + 1]),
                                           __float_as_uint(v[4 * q + 2]), __float_as_uint(v[4 * q + 3]));
                }
            }
        };
        // conv + SiLU of channel c < 3D for every token, sliding a 4-tap window along the
        // sequence; c in [3D, 4D) copies z column c - 3D for every token
        auto conv_channel = [&](int c) {
            if (c >= 3 * D) {
                const int j = c - 3 * D;
                for (int t = 0; t < T; ++t) zbuf[t * D + j] = Act<TA>::ld(sZ + t * D + j);
                return;
            }
            const int g = c / D, ci = c % D;
            const TA* mg = sMQ + g * (GL::M_BYTES / (int)sizeof(TA));
            float w[KC], win[KC];  // win[j]: the input j tokens back
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
        };

        if constexpr (!DEFER) {
            // ---- consume the stage: state to registers, conv windows, conv of every token, z ----
            // The state is read before the group agrees on the waits (a thread whose wait gave up
            // reads stale, in-bounds data that is then discarded), so one barrier both agrees on
            // failure and releases the state region for the next tile's state.
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
                issue_state(tile + nworkers, (size_t)nslot0);
            }
            if (p.cs_out && !p.cs_ckpt) write_window_per_channel(window_dst(-1), T);
            else write_windows();
            for (int c = tid; c < 4 * D; c += GT) conv_channel(c);
            group_sync(bar_id);  // stage consumed: refill it with this group's next tile
            if (tid < 32 && tile + nworkers < num_tiles) {
                fence_proxy_async_smem();
                issue(tile + nworkers, (size_t)nslot0);
            }
        } else {
            // ---- conv windows and every token's conv while the previous tile's last state stores
            // drain, then the state (its registers are free once those stores are issued) ----
            if (group_any(!ok, bar_id)) {
                failed = true;
                break;
            }
            flush(Q1{});
            write_windows();
            flush(Q2{});
            for (int c = tid; c < 4 * D; c += GT) conv_channel(c);
            flush(Q3{});
#pragma unroll
            for (int r = 0; r < RPT; ++r)
                S[r] = has_S ? *reinterpret_cast<const float4*>(sS + (rg * RPT + r) * D + cg * 4)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
            group_sync(bar_id);  // stage consumed (inputs and state): refill it with this group's next tile
            if (tid < 32 && tile + nworkers < num_tiles) {
                fence_proxy_async_smem();
                if (has_S && lane == 0) issue_state(tile + nworkers, (size_t)nslot0);
                issue(tile + nworkers, (size_t)nslot0);
            }
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
            flush(Q1{});

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
            flush(Q2{});
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
            flush(Q3{});  // the state after the previous token is stored: S may change

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
                const int slot = p.S_ckpt ? ck_slot(ck_i) : -1;
                if (slot >= 0)
                    owe(reinterpret_cast<float4*>(p.S_ckpt + ((size_t)slot * p.B * p.Hv + tile) * (size_t)(D * D)));
                ++ck_i;
            }
            if (t + 1 == T && p.S_out) owe(reinterpret_cast<float4*>(p.S_out + (size_t)tile * D * D));

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
            if (tid < D) {
                const int j = tid;
                TA* out = static_cast<TA*>(p.out) + ((size_t)b * T + t) * (size_t)(p.Hv * D) + h * D;
                const float o = Act<TA>::round(fmaf(qk, su[j], so[j]));
                const float y = Act<TA>::round(nw * Act<TA>::round(o * rstd));
                Act<TA>::st(out + j, y * silu_f(zbuf[t * D + j]));
            }
            flush(Q0{});
            // su / so / red are rewritten by the next token; after the last token the next
            // tile's first two barriers come before any thread writes them (or the gates)
            if (t + 1 < T) group_sync(bar_id);
        }
        if constexpr (!DEFER) {  // the state is reloaded at the next tile's start
            flush(Q1{});
            flush(Q2{});
            flush(Q3{});
        }
    }
    if (!failed) {  // the last tile's final stores
        flush(Q1{});
        flush(Q2{});
        flush(Q3{});
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
    return launch_pdl(decode_tma_kernel<D, TMAX, TA>, dim3(grid), dim3(NT), bytes, s, p, ck, tiles);
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
    // conv windows leave in 16-byte chunks
    if ((p.cs_out || p.cs_ckpt) && ((conv_dim * LC * es) % 16 || (d * LC * es) % 16)) return false;
    if ((p.cs_out && !al(p.cs_out)) || (p.cs_ckpt && !al(p.cs_ckpt))) return false;
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
