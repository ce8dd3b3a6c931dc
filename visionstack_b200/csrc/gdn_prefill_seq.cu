// K3 (two-kernel form): the sequential inter-chunk pass of the chunked
// prefill, after gdn_prefill_prep.cu has produced every chunk's conv outputs,
// norm factors, gates and T / P operand images.
//
// One CTA per (batch row, value head) chain walks its chunks of C = 64 tokens.
// The state lives in tensor memory, TRANSPOSED: lane = value dim dv, column =
// key dim dk, so that it is directly the A operand of the next MMA (tcgen05
// reads A from tensor memory).  Two copies: the fp32 master and its tf32
// (round-to-nearest) operand copy.  Per chunk, with k, q the raw bf16 rows
// (exact as tf32 operands; the norm factors rk, rq and dk^-1/2 are applied per
// token outside the MMAs), V the v rows, beta and gamma = cumsum(g) of the
// chunk, T = (I + A)^-1 and P = (Q K^T) o e^{gamma_i - gamma_j} (j <= i) of the
// normalised rows:
//
//   MMA-b  [Y^T | O1^T] = S^T [k;q]^T                  (M128 N128 K128, A from TMEM)
//   CUDA   Z^T = beta (V - e^gamma rk Y)^T              (to TMEM)
//   MMA-c  v_new^T = Z^T T^T                            (M128 N64  K64,  A from TMEM)
//   CUDA   v_new^T and (e^{gamma_C - gamma} rk v_new)^T, tf32 (to TMEM)
//   MMA-d  D^T = v_new^T P^T                            (M128 N64  K64)
//   MMA-e  dS^T = (e^{gamma_C - gamma} rk v_new)^T k     (M128 N128 K64)
//   CUDA   S^T <- e^{gamma_C} S^T + dS^T (master and operand copy), boundary
//          checkpoints, final state
//   CUDA   output rows O = e^gamma rq dk^-1/2 O1 + D through the gated RMSNorm
//
// i.e. the reference's v_new = U - W S with U = T (beta V), W = T (beta K e^gamma)
// and O = (Q e^gamma) S + P v_new, S' = e^{gamma_C} S + (K e^{gamma_C-gamma})^T v_new
// (deltanet.py:323-389), regrouped and transposed.
//
// 16 warps in two roles.  Warpgroups 0-1 carry the state: the MMAs (warp 0
// issues them), Z, v_new, the state update.  Warpgroups 2-3 stage the next
// chunk's [k;q] and k operands (mbarriers b_done: MMA-b has read [k;q];
// staged: both operands ready), issue the input copies, and turn the previous
// chunk's O into output rows while the state path moves on: they copy O out
// of tensor memory as soon as MMA-d completes (mbarrier o_ready, a second
// commit of that MMA), release those columns (mbarrier o_free, which the next
// MMA-b waits for), then normalise and store.
#include "gdn_async.cuh"
#include "gdn_common.cuh"
#include "gdn_conv_windows.cuh"
#include "gdn_kernels.cuh"
#include "gdn_prefill_ws.cuh"
#include "gdn_tmap.h"
#include "gdn_umma.cuh"

namespace gdn {
namespace pseq {

constexpr int D = 128, C = 64, NT = 512, NMAIN = 256;
// shared memory (bytes from the 1024-aligned base)
// [k;q] rows of a chunk, two buffers (chunk parity): the bf16 rows as the
// 128-byte swizzled operand a TMA copy writes, 128 rows (k tokens 0..63, q
// tokens 64..127) by dk in two 64-element atoms 16 KB apart: K-major B of
// MMA-b, and its k rows MN-major B of MMA-e
constexpr uint32_t R_QK = 0, QK_BYTES = 32768;
constexpr uint32_t R_TP = 65536;    // T image, P image (16 KB each, tf32; B of MMA-c / MMA-d)
constexpr uint32_t R_VS = 98304;    // v rows bf16 [64][128]
constexpr uint32_t R_ZS = 114688;   // z rows (then the output rows)
constexpr uint32_t R_VEC = 131072;  // two buffers of rq[64] rk[64] beta[64] gamma[64] as loaded
constexpr uint32_t R_SCR = R_VEC + 2048;
// scratch floats: per chunk parity p, at S_V + 384 p, the per-token vectors beta, gamma,
// -e^gamma rk, e^{gamma_C - gamma} rk, e^gamma rq dk^-1/2 and the scalar e^{gamma_C}
constexpr int S_V = 0, S_F = 768, S_NW = 832, S_PART = 960, S_RSTD = 1216, S_END = 1280;
constexpr int V_B = 0, V_G = 64, V_EK = 128, V_EF = 192, V_EQ = 256, V_EC = 320;
constexpr uint32_t R_BAR = R_SCR + S_END * 4;
constexpr uint32_t SMEM_BYTES = R_BAR + 128 + 1024;
// tensor memory columns
constexpr uint32_t C_MS = 0, C_OP = 128, C_YO = 256, C_Z = 384, C_V = 448, T_COLS = 512;

using TA = __nv_bfloat16;

__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }
__device__ __forceinline__ float bf_at(const unsigned char* base, int idx) {
    return __uint_as_float((uint32_t)(*reinterpret_cast<const uint16_t*>(base + 2 * idx)) << 16);
}
__device__ __forceinline__ uint32_t bf2_bits(float a, float b) {
    const __nv_bfloat162 t = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&t);
}
// a pair of values rounded to bf16 (nearest, ties to even) with one packed
// conversion; the packed bits in *bits
__device__ __forceinline__ void round2_bf16(float& a, float& b, uint32_t* bits = nullptr) {
    const uint32_t u = bf2_bits(a, b);
    a = bf_lo(u);
    b = bf_hi(u);
    if (bits) *bits = u;
}
// round to 11 significant bits (tf32) on the fp32 pipe: Veltkamp's split with
// 2^13 + 1 (nearest); the explicitly rounded operators keep the compiler from
// contracting it into an fma
__device__ __forceinline__ float tf32_rn(float x) {
    const float t = __fmul_rn(x, 8193.0f);
    return __fsub_rn(t, __fsub_rn(t, x));
}
// packed fp32 pairs (one instruction for two lanes of arithmetic); a - b as fma(b, -1, a)
__device__ __forceinline__ float2 f2_sub(float2 a, float2 b) { return __ffma2_rn(b, make_float2(-1.f, -1.f), a); }
__device__ __forceinline__ float2 tf32_rn2(float2 x) {  // tf32_rn of both lanes
    const float2 t = __fmul2_rn(x, make_float2(8193.0f, 8193.0f));
    return f2_sub(t, f2_sub(t, x));
}

// 32 fp32 values as bf16 pairs hi + lo (hi = bf16(x), lo = bf16(x - hi); the
// difference is exact, so hi + lo is within 2^-17 of x relative), packed for a
// kind::f16 A operand: column j of each half holds elements 2j, 2j + 1.  The
// 32 columns at taddr: hi pairs in the first 16, lo pairs in the next 16.
__device__ __forceinline__ void store_split32(uint32_t taddr, const float (&x)[32]) {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {  // 8 pairs at a time
        uint32_t hi[8], lo[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float a = x[16 * hf + 2 * j], c = x[16 * hf + 2 * j + 1];
            const uint32_t u = bf2_bits(a, c);
            hi[j] = u;
            const float2 r = f2_sub(make_float2(a, c), make_float2(bf_lo(u), bf_hi(u)));
            lo[j] = bf2_bits(r.x, r.y);
        }
        umma::tmem_st8(taddr + 8 * hf, hi);
        umma::tmem_st8(taddr + 16 + 8 * hf, lo);
    }
}
// tensor-memory column of the hi (or lo) pairs of k-step kk (16 elements) of a
// split operand stored by store_split32 in 32-column blocks
__host__ __device__ constexpr uint32_t split_col(int kk, bool lo) {
    return (uint32_t)(32 * (kk >> 1) + 8 * (kk & 1) + (lo ? 16 : 0));
}

// named barriers: 1 and 5 = state warpgroups (256 threads; warps 1-7 may only
// arrive while warp 0 waits), 2 / 3 = output warpgroup 0 / 1 (128 threads
// each), 4 = both output warpgroups (256)
__device__ __forceinline__ void nb_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ bool nb_any(bool pred, int id, int n) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}\n"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void nb_arrive(int id, int n) { asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__global__ void __launch_bounds__(NT, 1)
    prefill_seq_kernel(const MixParams p, const CkptList ck, const PrefillWs ws,
                       const __grid_constant__ CUtensorMap tm_qk, const __grid_constant__ CUtensorMap tm_v,
                       const __grid_constant__ CUtensorMap tm_z, const __grid_constant__ CUtensorMap tm_out,
                       const int split) {
    extern __shared__ unsigned char raw[];
    const uint32_t raw_addr = smem_u32(raw);
    unsigned char* sm = raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const uint32_t sb = smem_u32(sm);
    float* scr = reinterpret_cast<float*>(sm + R_SCR);
    float* sF = scr + S_F;
    float* sNW = scr + S_NW;
    float* sPart = scr + S_PART;
    float* sRstd = scr + S_RSTD;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + R_BAR);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + R_BAR + 96);
    // input copies issued per barrier (q/k buffer 0, 1, v, T/P), for the drain at exit
    int* n_cp = reinterpret_cast<int*>(sm + R_BAR + 100);
    const uint32_t bar_qk0 = smem_u32(&bars[0]), bar_v = smem_u32(&bars[2]), bar_z = smem_u32(&bars[3]),
                   bar_tp = smem_u32(&bars[4]), bar_mma = smem_u32(&bars[5]), bar_ordy = smem_u32(&bars[6]),
                   bar_ofree = smem_u32(&bars[7]), bar_staged = smem_u32(&bars[8]), bar_o1 = smem_u32(&bars[9]);
    auto bar_qk = [&](int cc) { return bar_qk0 + 8u * (uint32_t)(cc & 1); };

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wg = warp >> 2, q4 = warp & 3;
    const bool main_grp = tid < NMAIN;
    const int dv = 32 * q4 + lane;  // this thread's tensor-memory lane
    const uint32_t lane_base = (uint32_t)(32 * q4) << 16;
    const int NCg = ws.nc;  // chunks of a chain
    const int chains = p.B * p.Hv;

    if (warp == 0) {
        umma::tmem_alloc(smem_u32(tslot), T_COLS);
        umma::tmem_relinquish();
    }
    if (tid == 0) {
        prefetch_tmap(&tm_qk);
        prefetch_tmap(&tm_v);
        prefetch_tmap(&tm_z);
        prefetch_tmap(&tm_out);
    }
    if (tid < D) sNW[tid] = Act<TA>::ldg(static_cast<const TA*>(p.normw) + tid);
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *tslot;

    // Split mode (more chains than CTAs): the chains' chunks laid end to end are cut into
    // gridDim.x equal runs of at least one chain each.  A run holds at most a chain's last
    // chunks (its tail), whole chains, and a chain's first chunks (its head); the CTA does the
    // head first and the tail last, so the head of a chain (at the previous CTA's start) is done
    // long before its tail begins.  The state crosses in hand-off slot k of the workspace
    // (between CTAs k and k + 1), released by a flag.  Otherwise one CTA takes one chain.
    long long lo = 0, hi = 0;
    int first = blockIdx.x, last = blockIdx.x;
    if (split) {
        const long long total = (long long)chains * NCg;
        const long long L = (total + gridDim.x - 1) / gridDim.x;
        lo = (long long)blockIdx.x * L;
        hi = lo + L < total ? lo + L : total;
        first = (int)(lo / NCg);
        last = (int)((hi - 1) / NCg);
    }
    auto piece_of = [&](int j, int& cs, int& ce) {
        if (!split) {
            cs = 0;
            ce = NCg;
            return;
        }
        const long long a0 = (long long)j * NCg;
        cs = (int)((lo > a0 ? lo : a0) - a0);
        ce = (int)((hi < a0 + NCg ? hi : a0 + NCg) - a0);
    };
    int cs_first, ce_first, cs_last, ce_last;
    piece_of(first, cs_first, ce_first);
    piece_of(last, cs_last, ce_last);
    const bool has_head = split && hi > lo && ce_last < NCg;  // the run ends inside chain `last`
    const bool has_tail = split && hi > lo && cs_first > 0 && !(has_head && first == last);
    const int npieces = split ? (hi > lo ? last - first + 1 : 0) : 1;
    bool cta_failed = false;
    for (int pi = 0; pi < npieces && !cta_failed; ++pi) {
    // time order: the head piece, the whole chains, the tail piece
    int chain = first;
    if (split) {
        const int k = pi - (has_head ? 1 : 0);  // index among the other pieces
        const int n_rest = npieces - (has_head ? 1 : 0);
        if (has_head && pi == 0) chain = last;
        else if (has_tail) chain = k < n_rest - 1 ? first + 1 + k : first;
        else chain = first + k;
    }
    int c_base, c_end;
    piece_of(chain, c_base, c_end);
    const int NC = c_end - c_base;                              // chunks of this piece
    const int in_slot = c_base > 0 ? (int)blockIdx.x - 1 : -1;  // state from the hand-off
    const int out_slot = c_end < NCg ? (int)blockIdx.x : -1;    // state to the hand-off
    const int bh = chain;
    const int b = bh / p.Hv, h = bh - (bh / p.Hv) * p.Hv;
    const int rep = p.Hv / p.Hk, kh = h / rep;

    if (tid == 0) {
        if (pi > 0)
            for (int i = 0; i < 10; ++i) mbar_inval(smem_u32(&bars[i]));
        for (int i = 0; i < 7; ++i) mbar_init(smem_u32(&bars[i]), 1);
        mbar_init(bar_o1, 1);
        mbar_init(bar_ofree, NT - NMAIN);
        mbar_init(bar_staged, NT - NMAIN);
        for (int i = 0; i < 4; ++i) n_cp[i] = 0;
        fence_mbar_init();
    }
    if (c_base == 0) write_conv_windows<TA, D, D, NT>(p, ck, b, h, kh, rep);
    bool hand_ok = true;
    if (in_slot >= 0 && tid == 0) hand_ok = wait_flag_bounded(ws.hflag + in_slot);
    umma::fence_before_sync();
    if (__syncthreads_or(!hand_ok)) {
        cta_failed = true;
        break;
    }
    umma::fence_after_sync();

    // initial state, transposed: lane dv, column dk (warpgroup wg: dk 32 wg .. 32 wg + 31);
    // its bf16 hi / lo operand in the same 32 columns of the operand region
    {
        const int c0 = 32 * wg;
        const float* src = in_slot >= 0 ? ws.hs + (size_t)in_slot * D * D
                                         : (p.S_in ? p.S_in + (size_t)bh * D * D : nullptr);
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = src ? __ldcg(src + (size_t)(c0 + j) * D + dv) : 0.f;
        umma::tmem_st32(tmem + lane_base + C_MS + c0, v);
        store_split32(tmem + lane_base + C_OP + c0, v);
        umma::tmem_wait_st();
    }

    const int v_ch = 2 * p.Hk * D + h * D;
    // Every input region is reloaded only after all readers of its previous copy are done and
    // that copy was seen complete by the issuing thread, so one copy per barrier is in flight.
    auto issue_qk = [&](int cc) {  // into buffer cc & 1
        const uint32_t dst = sb + R_QK + QK_BYTES * (uint32_t)(cc & 1), bar = bar_qk(cc);
        atomicAdd(&n_cp[cc & 1], 1);
        mbar_arrive_expect_tx(bar, 4u * 8192u + 1024u);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            tma_load_3d(dst + 16384u * j, &tm_qk, p.Hk * D + kh * D + 64 * j, (c_base + cc) * C, b, bar);  // k
            tma_load_3d(dst + 16384u * j + 8192u, &tm_qk, kh * D + 64 * j, (c_base + cc) * C, b, bar);     // q
        }
        const uint32_t vdst = sb + R_VEC + 1024u * (uint32_t)(cc & 1);
        bulk_load(vdst, ws.nrm + (((size_t)b * p.Hk + kh) * NCg + c_base + cc) * 128, 512, bar);
        bulk_load(vdst + 512, ws.gate + (((size_t)b * p.Hv + h) * NCg + c_base + cc) * 128, 512, bar);
    };
    auto issue_v = [&](int cc) {
        atomicAdd(&n_cp[2], 1);
        mbar_arrive_expect_tx(bar_v, (uint32_t)C * D * 2u);
        tma_load_3d(sb + R_VS, &tm_v, v_ch, (c_base + cc) * C, b, bar_v);
    };
    auto issue_z = [&](int cc) {
        mbar_arrive_expect_tx(bar_z, (uint32_t)C * D * 2u);
        tma_load_3d(sb + R_ZS, &tm_z, h * D, (c_base + cc) * C, b, bar_z);
    };
    auto issue_tp = [&](int cc) {
        atomicAdd(&n_cp[3], 1);
        mbar_arrive_expect_tx(bar_tp, 2u * C * C * 4u);
        bulk_load(sb + R_TP, ws.tp + (((size_t)b * p.Hv + h) * NCg + c_base + cc) * (2 * C * C), 2u * C * C * 4u,
                  bar_tp);
    };
    // z copies issued / waited for (output group)
    int n_z = 0, w_z = 0;
    if (tid == 0) {
        issue_qk(0);
        if (NC > 1) issue_qk(1);
        issue_v(0);
        issue_tp(0);
    }
    if (tid == NMAIN) {
        issue_z(0);
        n_z = 1;
    }
    umma::fence_before_sync();
    __syncthreads();

    // Input copies after the first ones: the output group's first thread issues v and T/P of
    // chunk c + 1 and the q/k rows of chunk c + 2 (into the buffer of chunk c) when MMA-d / MMA-e
    // of chunk c complete (o_ready: Z, step 5a and every MMA reading those regions are done).
    bool failed = false;
    if (main_grp) {
        // ======================= state path (warpgroups 0-1) =======================
        const uint32_t idesc_c = umma::idesc_tf32(128, 64, 0, 0);
        const uint32_t idesc_b = umma::idesc_bf16(128, 64, 0, 0);
        const uint32_t idesc_e = umma::idesc_bf16(128, 128, 0, 1);
        // B-operand descriptors at k-step 0 (the operand regions never move)
        const uint64_t d_t = umma::desc_kmajor0(sb + R_TP), d_p = umma::desc_kmajor0(sb + R_TP + C * C * 4);
        uint32_t mma_phase = 0;
        bool mma_pending = false;
        int ck_i = 0;  // first checkpoint past the piece's start (earlier ones belong to the head)
        while (ck_i < ck.n && ck.off[ck_i] <= c_base * C) ++ck_i;
        // A bounded wait that runs out marks this thread bad; the threads agree on it once per
        // chunk (the closing barrier) and leave together.  Until then a bad thread keeps going
        // on stale data: every address it touches is fixed by the chunk index, never by data.
        bool bad = false;
        auto mma_wait = [&]() {
            const bool ok = mbar_wait_bounded(bar_mma, mma_phase & 1u, GDN_DEVERR_MMA_TIMEOUT);
            ++mma_phase;
            umma::fence_after_sync();
            bad |= !ok;
            if (ok) mma_pending = false;
        };
        auto wait_phase = [&](uint32_t bar, int phase) {
            bad |= !mbar_wait_bounded(bar, (uint32_t)phase & 1u, GDN_DEVERR_TMA_TIMEOUT);
        };
        // the tensor-memory stores of all 256 threads before warp 0 issues the next MMA; the
        // other warps only arrive (they next wait for that MMA, so none can run a phase ahead)
        auto stores_to_warp0 = [&]() {
            umma::fence_before_sync();
            if (warp == 0)
                nb_sync(1, NMAIN);
            else
                nb_arrive(1, NMAIN);
        };
        for (int c = 0; c < NC; ++c) {
            const int t0 = (c_base + c) * C;
            float* sv = scr + S_V + 384 * (c & 1);
            const uint32_t r_qk = R_QK + QK_BYTES * (uint32_t)(c & 1);
            // ---------------- 2. MMA-b (after the output warps released O of the last chunk) ----------------
            // (warp 0 issues every MMA: elect.sync picks lane 0)
            if (warp == 0) {
                wait_phase(bar_qk(c), c >> 1);
                if (c > 0) bad |= !mbar_wait_bounded(bar_ofree, (uint32_t)(c - 1) & 1u, GDN_DEVERR_MMA_TIMEOUT);
                __syncwarp();
                umma::fence_after_sync();
                // Y^T (k rows) first, committed for the state path; then O1^T (q rows, for the
                // output warps), committed to o1_done, which MMA-e (it overwrites the state
                // operand columns) waits for; o_ready covers it too
                const uint64_t d_k = umma::desc_kmajor0(sb + r_qk), d_q = umma::desc_kmajor0(sb + r_qk + 8192);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma::mma_bf16_ta_elect(tmem + C_YO, tmem + C_OP + split_col(kk, false),
                                            umma::desc_add(d_k, umma::kmajor_kstep(kk, 128)), idesc_b, kk > 0);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma::mma_bf16_ta_elect(tmem + C_YO, tmem + C_OP + split_col(kk, true),
                                            umma::desc_add(d_k, umma::kmajor_kstep(kk, 128)), idesc_b, 1u);
                umma::mma_commit_elect(bar_mma);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma::mma_bf16_ta_elect(tmem + C_YO + 64, tmem + C_OP + split_col(kk, false),
                                            umma::desc_add(d_q, umma::kmajor_kstep(kk, 128)), idesc_b, kk > 0);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma::mma_bf16_ta_elect(tmem + C_YO + 64, tmem + C_OP + split_col(kk, true),
                                            umma::desc_add(d_q, umma::kmajor_kstep(kk, 128)), idesc_b, 1u);
                umma::mma_commit_elect(bar_o1);
                mma_pending = true;
            }
            mma_wait();
            wait_phase(bar_staged, c);  // the chunk's vectors (staged by the output warps)
            wait_phase(bar_v, c);
            // ---------------- 3. Z^T = beta (V - e^gamma rk Y)^T (warpgroup wg: tokens 32 wg ..) ----------------
            {
                float y[32];
                umma::tmem_ld32(tmem + lane_base + C_YO + 32 * wg, y);
                umma::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    const int t = 32 * wg + j;
                    const float2 vv = make_float2(bf_at(sm + R_VS, t * D + dv), bf_at(sm + R_VS, (t + 1) * D + dv));
                    const float2 nek = *reinterpret_cast<const float2*>(sv + V_EK + t);  // -e^gamma rk
                    const float2 be = *reinterpret_cast<const float2*>(sv + V_B + t);
                    const float2 r = tf32_rn2(__fmul2_rn(be, __ffma2_rn(nek, make_float2(y[j], y[j + 1]), vv)));
                    y[j] = r.x;
                    y[j + 1] = r.y;
                }
                umma::tmem_st32(tmem + lane_base + C_Z + 32 * wg, y);
                umma::tmem_wait_st();
            }
            stores_to_warp0();
            // ---------------- 4. MMA-c: v_new^T = Z^T T^T ----------------
            if (warp == 0) {
                wait_phase(bar_tp, c);
                __syncwarp();
                umma::fence_after_sync();
#pragma unroll
                for (int kk = 0; kk < C / 8; ++kk)
                    umma::mma_tf32_ta_elect(tmem + C_V, tmem + C_Z + kk * 8,
                                            umma::desc_add(d_t, umma::kmajor_kstep(kk, C)), idesc_c, kk > 0);
                umma::mma_commit_elect(bar_mma);
                mma_pending = true;
            }
            mma_wait();
            // ---------------- 5a. sub-chunk checkpoints (fp32 v_new, fp32 K, state before the update) ----------------
            // S_s = e^{gamma_{s-1}} S + sum_{t<s} e^{gamma_{s-1}-gamma_t} k_t^T v_new_t (deltanet.py:375-388)
            while (ck_i < ck.n && ck.off[ck_i] > t0 && ck.off[ck_i] - t0 < C) {
                const int s_off = ck.off[ck_i] - t0;
                const float* vec = reinterpret_cast<const float*>(sm + R_VEC + 1024u * (uint32_t)(c & 1));
                if (tid < C) sF[tid] = tid < s_off ? expf(sv[V_G + s_off - 1] - sv[V_G + tid]) : 0.f;
                nb_sync(1, NMAIN);
                const float es = expf(sv[V_G + s_off - 1]);
                float* dst = p.S_ckpt + ((size_t)ck.slot[ck_i] * p.B * p.Hv + bh) * (size_t)(D * D);
#pragma unroll 1
                for (int hb = 0; hb < 2; ++hb) {  // 32 key columns at a time
                    const int cb = 64 * wg + 32 * hb;
                    float m[32];
                    umma::tmem_ld32(tmem + lane_base + C_MS + cb, m);
                    umma::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j) m[j] *= es;
#pragma unroll 1
                    for (int th = 0; th < 2; ++th) {  // 32 tokens at a time
                        float wv[32];
                        umma::tmem_ld32(tmem + lane_base + C_V + 32 * th, wv);
                        umma::tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 32; ++j) wv[j] *= sF[32 * th + j] * vec[64 + 32 * th + j];  // decay, rk
                        // k row t = 32 th + j, key columns cb + 8 j8 .. + 7: one 16-byte unit of the
                        // swizzled rows (kmajor_off16 with t % 8 = j % 8 known at compile time)
                        const unsigned char* kb = sm + r_qk + 16384 * wg + 4096 * th;
                        const uint32_t hx0 = 64u * hb, hx1 = 64u - 64u * hb;
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const unsigned char* rowp = kb + (j >> 3) * 1024 + (j & 7) * 128 + ((j & 4) ? hx1 : hx0);
#pragma unroll
                            for (int j8 = 0; j8 < 4; ++j8) {  // 8 key columns per 16-byte swizzle unit
                                const uint4 k8 = *reinterpret_cast<const uint4*>(rowp + ((j8 ^ (j & 3)) << 4));
                                const uint32_t kw[4] = {k8.x, k8.y, k8.z, k8.w};
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    m[8 * j8 + 2 * e] = fmaf(wv[j], bf_lo(kw[e]), m[8 * j8 + 2 * e]);
                                    m[8 * j8 + 2 * e + 1] = fmaf(wv[j], bf_hi(kw[e]), m[8 * j8 + 2 * e + 1]);
                                }
                            }
                        }
                    }
#pragma unroll
                    for (int j = 0; j < 32; ++j) __stcs(dst + (size_t)(cb + j) * D + dv, m[j]);
                }
                nb_sync(1, NMAIN);
                ++ck_i;
            }
            // ---------------- 5b. (e^{gamma_C - gamma} rk v_new)^T as bf16 hi / lo ----------------
            {
                float w[32];
                umma::tmem_ld32(tmem + lane_base + C_V + 32 * wg, w);
                umma::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    const float2 r = __fmul2_rn(make_float2(w[j], w[j + 1]),
                                                *reinterpret_cast<const float2*>(sv + V_EF + 32 * wg + j));
                    w[j] = r.x;
                    w[j + 1] = r.y;
                }
                store_split32(tmem + lane_base + C_Z + 32 * wg, w);
                umma::tmem_wait_st();
            }
            stores_to_warp0();
            // ---------------- 6a. MMA-e: dS^T, into the operand columns (the state path waits for it) ----------------
            if (warp == 0) {
                wait_phase(bar_o1, c);
                __syncwarp();
                umma::fence_after_sync();
                const uint64_t d_km = umma::desc_mnmajor16_0(sb + r_qk, 16384);
#pragma unroll
                for (int kk = 0; kk < C / 16; ++kk)
                    umma::mma_bf16_ta_elect(tmem + C_OP, tmem + C_Z + split_col(kk, false),
                                            umma::desc_add(d_km, umma::mnmajor16_kstep(kk)), idesc_e, kk > 0);
#pragma unroll
                for (int kk = 0; kk < C / 16; ++kk)
                    umma::mma_bf16_ta_elect(tmem + C_OP, tmem + C_Z + split_col(kk, true),
                                            umma::desc_add(d_km, umma::mnmajor16_kstep(kk)), idesc_e, 1u);
                umma::mma_commit_elect(bar_mma);
                mma_pending = true;
            }
            // ---------------- 5c. v_new^T (tf32) for MMA-d while MMA-e runs ----------------
            {
                float v[32];
                umma::tmem_ld32(tmem + lane_base + C_V + 32 * wg, v);
                umma::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    const float2 r = tf32_rn2(make_float2(v[j], v[j + 1]));
                    v[j] = r.x;
                    v[j + 1] = r.y;
                }
                umma::tmem_st32(tmem + lane_base + C_V + 32 * wg, v);
                umma::tmem_wait_st();
            }
            // (a second barrier id: warps 1-7 reach this one without waiting on an MMA first)
            umma::fence_before_sync();
            if (warp == 0)
                nb_sync(5, NMAIN);
            else
                nb_arrive(5, NMAIN);
            // ---------------- 6b. MMA-d: D^T = v_new^T P^T (for the output warps) ----------------
            if (warp == 0) {
                umma::fence_after_sync();
#pragma unroll
                for (int kk = 0; kk < C / 8; ++kk)
                    umma::mma_tf32_ta_elect(tmem + C_YO, tmem + C_V + kk * 8,
                                            umma::desc_add(d_p, umma::kmajor_kstep(kk, C)), idesc_c, kk > 0);
                umma::mma_commit_elect(bar_ordy);  // O of this chunk is complete for the output warps
            }
            mma_wait();
            // ---------------- 7. state update (key columns 64 wg ..), checkpoints, final state ----------------
            // each thread reads dS^T from, and writes the new bf16 hi / lo operand into, the same
            // 32 columns of its own lane
            {
                const float ec = sv[V_EC];
                const bool last = c == NC - 1;
                float* const s_end = !last ? nullptr
                                     : out_slot >= 0 ? ws.hs + (size_t)out_slot * D * D
                                                     : (p.S_out ? p.S_out + (size_t)bh * D * D : nullptr);
#pragma unroll 1
                for (int c0 = 64 * wg; c0 < 64 * wg + 64; c0 += 32) {
                    float m[32], d[32];
                    umma::tmem_ld32(tmem + lane_base + C_MS + c0, m);
                    umma::tmem_ld32(tmem + lane_base + C_OP + c0, d);
                    umma::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        const float2 r = __ffma2_rn(make_float2(m[j], m[j + 1]), make_float2(ec, ec),
                                                    make_float2(d[j], d[j + 1]));
                        m[j] = r.x;
                        m[j + 1] = r.y;
                    }
                    umma::tmem_st32(tmem + lane_base + C_MS + c0, m);
                    store_split32(tmem + lane_base + C_OP + c0, m);
                    for (int w = ck_i; w < ck.n && ck.off[w] - t0 == C; ++w) {
                        float* dst = p.S_ckpt + ((size_t)ck.slot[w] * p.B * p.Hv + bh) * (size_t)(D * D);
#pragma unroll
                        for (int j = 0; j < 32; ++j) __stcs(dst + (size_t)(c0 + j) * D + dv, m[j]);
                    }
                    if (s_end) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) __stcg(s_end + (size_t)(c0 + j) * D + dv, m[j]);
                    }
                }
                umma::tmem_wait_st();
                if (last && out_slot >= 0) __threadfence();  // the hand-off state before its flag
            }
            while (ck_i < ck.n && ck.off[ck_i] - t0 == C) ++ck_i;
            umma::fence_before_sync();
            if (nb_any(bad, 1, NMAIN)) {
                failed = true;
                break;
            }
            umma::fence_after_sync();
            if (c == NC - 1 && out_slot >= 0 && tid == 0) release_flag(ws.hflag + out_slot);  // state written
        }
        if (tid == 0 && failed && mma_pending)  // an MMA in flight finishes (bounded) before the CTA exits
            mbar_wait_bounded(bar_mma, (mma_phase - 1) & 1u, GDN_DEVERR_MMA_TIMEOUT);
    } else {
        // ======================= per-token vectors and output rows (warpgroups 2-3) =======================
        const int owg = wg - 2, tw = 32 * owg;  // this warpgroup's tokens tw .. tw + 31
        const int otid = tid - NMAIN;
        const float nw = sNW[dv];
        // chunk cc's per-token vectors from its loaded rq, rk, beta, gamma: the norm factors
        // ride on the vectors, so the operand rows stay the exact bf16 values
        auto stage_vectors = [&](int cc) {
            const float* vec = reinterpret_cast<const float*>(sm + R_VEC + 1024u * (uint32_t)(cc & 1));
            float* sv = scr + S_V + 384 * (cc & 1);
            if (otid < C) {
                const float gC = vec[192 + C - 1], gt = vec[192 + otid], rk = vec[64 + otid];
                const float eg = expf(gt);
                sv[V_B + otid] = vec[128 + otid];
                sv[V_G + otid] = gt;
                sv[V_EK + otid] = -(eg * rk);
                sv[V_EF + otid] = expf(gC - gt) * rk;
                sv[V_EQ + otid] = eg * (vec[otid] * p.q_scale);
                if (otid == 0) sv[V_EC] = expf(gC);
            }
        };
        bool bad = false;
        bad |= !mbar_wait_bounded(bar_qk(0), 0u, GDN_DEVERR_TMA_TIMEOUT);
        stage_vectors(0);
        mbar_arrive(bar_staged);
        for (int c = 0; c < NC && !failed; ++c) {
            const int t0 = (c_base + c) * C;
            const float* sv = scr + S_V + 384 * (c & 1);
            bad |= !mbar_wait_bounded(bar_ordy, (uint32_t)c & 1u, GDN_DEVERR_MMA_TIMEOUT);
            umma::fence_after_sync();
            // O[t][dv] = e^{gamma_t} rq dk^-1/2 O1 + D
            float o[32];
            {
                float o1[32], dd[32];
                umma::tmem_ld32(tmem + lane_base + C_YO + 64 + tw, o1);
                umma::tmem_ld32(tmem + lane_base + C_YO + tw, dd);
                umma::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j) o[j] = fmaf(sv[V_EQ + tw + j], o1[j], dd[j]);
            }
            umma::fence_before_sync();
            mbar_arrive(bar_ofree);  // these tensor-memory columns may be overwritten now
            if (c + 1 < NC) {
                // the next chunk's vectors: after o_ready of this chunk the state path is done with
                // the previous chunk's (same parity), and it waits for these only in this chunk's
                // successor, so the staged phases never run two ahead of it
                bad |= !mbar_wait_bounded(bar_qk(c + 1), (uint32_t)((c + 1) >> 1) & 1u, GDN_DEVERR_TMA_TIMEOUT);
                stage_vectors(c + 1);
                mbar_arrive(bar_staged);
            }
            if (tid == NMAIN && !bad) {
                // MMA-c, MMA-d and MMA-e of chunk c are complete; the previous copy into each
                // region must also have been seen complete here before the next one is issued
                if (c + 1 < NC) {
                    const bool ok = mbar_wait_bounded(bar_v, (uint32_t)c & 1u, GDN_DEVERR_TMA_TIMEOUT) &&
                                    mbar_wait_bounded(bar_tp, (uint32_t)c & 1u, GDN_DEVERR_TMA_TIMEOUT);
                    bad |= !ok;
                    if (ok) {
                        issue_v(c + 1);
                        issue_tp(c + 1);
                    }
                }
                if (c + 2 < NC) {
                    const bool ok = mbar_wait_bounded(bar_qk(c), (uint32_t)(c >> 1) & 1u, GDN_DEVERR_TMA_TIMEOUT);
                    bad |= !ok;
                    if (ok) issue_qk(c + 2);
                }
            }
#pragma unroll
            for (int j = 0; j < 32; j += 2) round2_bf16(o[j], o[j + 1]);
            // per-token sums of squares over this warp's 32 lanes: halving exchange
            // that leaves token tw + lane in this lane
            float sq[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) sq[j] = o[j] * o[j];
#pragma unroll
            for (int st = 0; st < 5; ++st) {
                const int s = 16 >> st, half = 16 >> st;  // exchange distance = values kept after this step
                const bool up = (lane & s) != 0;
#pragma unroll
                for (int k = 0; k < half; ++k) {
                    const float send = up ? sq[k] : sq[k + half];
                    const float keep = up ? sq[k + half] : sq[k];
                    sq[k] = keep + __shfl_xor_sync(0xffffffffu, send, s);
                }
            }
            sPart[q4 * C + tw + lane] = sq[0];
            nb_sync(2 + owg, 128);
            if (q4 == 0) {
                const int t = tw + lane;
                const float ss = (sPart[t] + sPart[C + t]) + (sPart[2 * C + t] + sPart[3 * C + t]);
                sRstd[t] = rsqrtf(ss / (float)D + p.eps);
            }
            const bool zok = mbar_wait_bounded(bar_z, (uint32_t)w_z & 1u, GDN_DEVERR_TMA_TIMEOUT);
            w_z += zok;
            bad |= !zok;
            nb_sync(2 + owg, 128);
            // the rows are assembled in the z tile's place ([64 tokens][128] bf16) and leave by one
            // tensor store, so every z value is read before the tile is overwritten
            float y[32], zv[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                y[j] = o[j] * sRstd[tw + j];
                zv[j] = bf_at(sm + R_ZS, (tw + j) * D + dv);
            }
            nb_sync(4, NT - NMAIN);
            uint16_t* tile = reinterpret_cast<uint16_t*>(sm + R_ZS) + tw * D + dv;
#pragma unroll
            for (int j = 0; j < 32; j += 2) round2_bf16(y[j], y[j + 1]);
#pragma unroll
            for (int j = 0; j < 32; ++j) y[j] *= nw;
#pragma unroll
            for (int j = 0; j < 32; j += 2) round2_bf16(y[j], y[j + 1]);
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
                const float z0 = zv[j], z1 = zv[j + 1];
                float a0 = y[j] * __fdividef(z0, 1.0f + __expf(-z0));
                float a1 = y[j + 1] * __fdividef(z1, 1.0f + __expf(-z1));
                uint32_t bits;
                round2_bf16(a0, a1, &bits);
                tile[j * D] = (uint16_t)(bits & 0xFFFFu);
                tile[(j + 1) * D] = (uint16_t)(bits >> 16);
            }
            fence_proxy_async_smem();
            // the group agrees on a wait that ran out (any thread) once per chunk, before the store
            if (nb_any(bad, 4, NT - NMAIN)) {
                failed = true;
                break;
            }
            if (tid == NMAIN) {
                // rows past the sequence end fall outside the tensor map and are not written
                tma_store_3d(&tm_out, sb + R_ZS, h * D, t0, b);
                bulk_commit_group();
                if (c + 1 < NC) {
                    bulk_wait_group_read0();  // the tile is read: the next z rows may land there
                    issue_z(c + 1);
                    ++n_z;
                }
            }
        }
        if (tid == NMAIN) {
            if (failed)
                for (; w_z < n_z; ++w_z) mbar_wait_bounded(bar_z, (uint32_t)w_z & 1u, GDN_DEVERR_TMA_TIMEOUT);
            bulk_wait_group0();  // output rows written before the CTA exits
        }
    }
    umma::fence_before_sync();
    cta_failed = __syncthreads_or(failed);
    if (tid == 0) {
        // the last input copy into each region lands before the piece ends (bounded; every
        // earlier copy on the same barrier was seen complete before the next was issued)
        const uint32_t bar_cp[4] = {bar_qk0, bar_qk0 + 8u, bar_v, bar_tp};
        for (int i = 0; i < 4; ++i)
            if (n_cp[i] > 0) mbar_wait_bounded(bar_cp[i], (uint32_t)(n_cp[i] - 1) & 1u, GDN_DEVERR_TMA_TIMEOUT);
    }
    __syncthreads();
    }  // pieces
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tmem, T_COLS);
}

}  // namespace pseq

cudaError_t launch_prefill_seq(const MixParams& p, const CkptList& ck, const PrefillWs& ws, cudaStream_t s) {
    const uint64_t conv_dim = 2ull * p.Hk * 128 + (uint64_t)p.Hv * 128;
    CUtensorMap tm_qk, tm_v, tm_z, tm_out;
    if (!encode_tmap_3d_bf16(&tm_qk, ws.qkv, conv_dim, (uint64_t)ws.tp_len, (uint64_t)p.B, conv_dim * 2,
                             conv_dim * 2 * (uint64_t)ws.tp_len, 64, pseq::C, true) ||
        !encode_tmap_3d_bf16(&tm_v, ws.qkv, conv_dim, (uint64_t)ws.tp_len, (uint64_t)p.B, conv_dim * 2,
                             conv_dim * 2 * (uint64_t)ws.tp_len, 128, pseq::C) ||
        !encode_tmap_3d_bf16(&tm_z, p.z, (uint64_t)p.Hv * 128, (uint64_t)p.T, (uint64_t)p.B, (uint64_t)p.zs_t * 2,
                             (uint64_t)p.zs_b * 2, 128, pseq::C) ||
        !encode_tmap_3d_bf16(&tm_out, p.out, (uint64_t)p.Hv * 128, (uint64_t)p.T, (uint64_t)p.B,
                             (uint64_t)p.Hv * 128 * 2, (uint64_t)p.Hv * 128 * 2 * (uint64_t)p.T, 128, pseq::C))
        return cudaErrorInvalidValue;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(pseq::prefill_seq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)pseq::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    const int chains = p.B * p.Hv;
    if (ws.n_hs > 1 && chains > ws.n_hs) {
        // split mode: one CTA per SM, all resident at once (a cooperative launch guarantees it),
        // the chains cut into equal runs with state hand-offs between neighbouring CTAs
        e = cudaMemsetAsync(ws.hflag, 0, (size_t)ws.n_hs * sizeof(int), s);
        if (e != cudaSuccess) return e;
        int split = 1;
        void* kargs[] = {const_cast<MixParams*>(&p), const_cast<CkptList*>(&ck), const_cast<PrefillWs*>(&ws),
                         &tm_qk, &tm_v, &tm_z, &tm_out, &split};
        e = cudaLaunchCooperativeKernel((const void*)pseq::prefill_seq_kernel, dim3(ws.n_hs), dim3(pseq::NT), kargs,
                                        pseq::SMEM_BYTES, s);
        if (e == cudaSuccess) return cudaSuccess;
        (void)cudaGetLastError();  // not launchable as one resident wave here: one CTA per chain
    }
    pseq::prefill_seq_kernel<<<chains, pseq::NT, pseq::SMEM_BYTES, s>>>(p, ck, ws, tm_qk, tm_v, tm_z, tm_out, 0);
    return cudaGetLastError();
}

unsigned int prefill_seq_device_error(bool clear) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
    if (clear && v) {
        const unsigned int zero = 0;
        cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
    }
    return v;
}

}  // namespace gdn
