// Chunked prefill in ONE kernel: the sequential inter-chunk pass with the
// per-chunk preparation computed inside it, two chunks ahead, by a producer
// warpgroup pair.  Nothing round-trips through a workspace: the raw q / k / v
// projection rows arrive by tensor copies, are convolved in place in shared
// memory, and feed the tensor cores from there; T = (I + A)^-1 and the masked
// P = (Q K^T) o decay are built in shared memory next to them.
//
// Per chunk of C = 64 tokens (deltanet.py:266-389 restated; the reference's
// v_new = U - W S, O = (Q e^gamma) S + P v_new and
// S' = e^{gamma_C} S + (K e^{gamma_C - gamma})^T v_new, regrouped as
// v_new = T (beta (V - e^gamma K S)) and transposed so that the state is the
// tensor-memory A operand):
//
//   producer (warps 8-15), for chunk c + 2 while the state path runs chunk c:
//     raw q / k rows (tensor copies, 128-byte swizzle = the K-major operand
//     layout) -> causal conv + SiLU in place with the reference's per-tap bf16
//     rounding (deltanet.py:41-90) -> L2-norm factors rq, rk (config.py:114-115)
//     -> beta = sigmoid(b), g = -exp(A_log) softplus(a + dt_bias), gamma =
//     cumsum(g) (deltanet.py:516-517, 278-281) -> one tcgen05 MMA
//     [G; P0] = [k; q] k^T of the raw bf16 rows (exact products) into tensor
//     memory -> A = tril(beta_i rk_i rk_j G_ij e^{gamma_i - gamma_j}, -1) and
//     P = (rq_i dk^-1/2 rk_j P0_ij e^{gamma_i - gamma_j}) (j <= i) ->
//     T = (I + A)^-1 by 32 x 32 forward substitution merged by
//     T21 = -T22 (A21 T11) (the doubling of deltanet.py:146-160), both as
//     K-major tf32 operand images; and the v rows of chunk c + 1 (conv in place);
//   state path (warps 0-7): MMA-b [Y | O1]^T = S^T [k; q]^T (bf16 hi + lo state),
//     Z = beta (V - e^gamma rk Y), MMA-c v_new^T = Z^T T^T (tf32), MMA-e
//     dS^T = (e^{gamma_C - gamma} rk v_new)^T k (bf16 hi + lo), MMA-d
//     (P v_new)^T (tf32), S^T <- e^{gamma_C} S^T + dS^T, checkpoints;
//   output (warps 8-15 again, for chunk c): O = e^gamma rq dk^-1/2 O1 + P v_new
//     through the gated RMSNorm (config.py:136-143), stored by tensor copy.
//
// Tensor memory (512 columns): state master (fp32) 0-127, state operand
// (bf16 hi / lo) 128-255, [Y | O1] 256-383, Z / v_new split 384-447, v_new
// 448-511; between MMA-d of chunk c and MMA-c of chunk c + 1 the producer
// borrows columns 448-511 for [G; P0] of chunk c + 2.
//
// Chains: one CTA per (batch row, value head) chain, or, with more chains than
// SMs, one cooperative wave of one CTA per SM with the chains' chunks laid end
// to end and cut into equal runs; a chain's state crosses between CTAs through
// a hand-off slot and a release / acquire flag (bounded wait).
#include "gdn_async.cuh"
#include "gdn_common.cuh"
#include "gdn_conv_windows.cuh"
#include "gdn_kernels.cuh"
#include "gdn_tmap.h"
#include "gdn_umma.cuh"

namespace gdn {
namespace pfused {

constexpr int D = 128, C = 64, NT = 512, NMAIN = 256;
constexpr int NQK = 3, NTP = 2, NVB = 2;  // buffers: [k;q] rows, T|P images, v rows
// shared memory (bytes from the 1024-aligned base)
//   [k;q] rows of a chunk (bf16, 128-byte swizzle, the K-major operand layout): two 64-element
//   atoms 16 KB apart, each with the 64 k rows (8 KB) then the 64 q rows (8 KB)
constexpr uint32_t QK_BYTES = 32768, R_QK = 0;
constexpr uint32_t TP_BYTES = 32768, R_TP = R_QK + NQK * QK_BYTES;  // T image (A, then T), P image
constexpr uint32_t V_BYTES = 16384, R_V = R_TP + NTP * TP_BYTES;    // v rows bf16 [64][128]
constexpr uint32_t R_Z = R_V + NVB * V_BYTES;                        // z rows, then the output rows
constexpr uint32_t R_VEC = R_Z + 16384;                              // per-chunk vectors, NQK slots
// per-chunk vector slot (floats): rq, rk, beta, gamma, -e^gamma rk, e^{gamma_C - gamma} rk,
// e^gamma rq dk^-1/2, e^gamma, e^-gamma rk, e^{gamma_C}
constexpr int V_RQ = 0, V_RK = 64, V_B = 128, V_G = 192, V_EK = 256, V_EF = 320, V_EQ = 384, V_EG = 448,
              V_ENG = 512, V_EC = 576, VEC_FLOATS = 584;
// conv history: the 4 raw rows before a chunk (tokens t0-4 .. t0-1, 128-byte rows of one
// 64-channel atom): per [k;q] buffer q atom 0, q atom 1, k atom 0, k atom 1; per v buffer v
// atom 0, v atom 1
constexpr uint32_t HROWS = 4, HATOM = HROWS * 128;
constexpr uint32_t R_HIST = ((R_VEC + NQK * VEC_FLOATS * 4) + 1023u) & ~1023u;
constexpr uint32_t R_HQK = R_HIST, R_HV = R_HIST + NQK * 4 * HATOM;
constexpr uint32_t R_SCR = R_HV + NVB * 2 * HATOM;
// scratch floats: the gated-norm weight (as 128 bf16), the conv's norm partials (q / k x 2 atoms
// x 64 tokens), checkpoint decay
constexpr int S_PART = 128, S_F = 448, S_END = 512;
constexpr uint32_t R_BAR = R_SCR + S_END * 4;
constexpr int NBAR = 20;
constexpr uint32_t SMEM_BYTES = R_BAR + NBAR * 8 + 64 + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
// tensor memory columns
constexpr uint32_t C_MS = 0, C_OP = 128, C_YO = 256, C_Z = 384, C_V = 448, T_COLS = 512;
// barrier indices
constexpr int B_RAWQK = 0,   // 3: raw q/k rows of buffer i landed
    B_RAWV = 3,              // 2: raw v rows landed
    B_Z = 5,                 // z rows landed
    B_MMA = 6,               // state-path MMAs (3 commits per chunk)
    B_O1 = 7,                // O1 of the chunk complete
    B_ORDY = 8,              // MMA-d complete: O (O1 + P v_new) ready for the output warps
    B_GP = 9,                // [G; P0] MMA of the producer complete
    B_UNUSED = 10,
    B_KQ = 11,               // 3: conv'd [k;q] rows and vectors of buffer i ready (1 arrival)
    B_VR = 14,               // 2: conv'd v rows ready (1 arrival)
    B_APR = 16,              // 2: A (for T) and the P image of buffer i ready (1 arrival)
    B_GPFREE = 18;           // [G; P0] copied out of tensor memory (256 arrivals)

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
__device__ __forceinline__ __nv_bfloat162 as_bf2(uint32_t u) { return *reinterpret_cast<__nv_bfloat162*>(&u); }
__device__ __forceinline__ void round2_bf16(float& a, float& b, uint32_t* bits = nullptr) {
    const uint32_t u = bf2_bits(a, b);
    a = bf_lo(u);
    b = bf_hi(u);
    if (bits) *bits = u;
}
// a - b as one packed fma(b, -1, a)
__device__ __forceinline__ float2 f2_sub(float2 a, float2 b) { return __ffma2_rn(b, make_float2(-1.f, -1.f), a); }
// round both lanes to 11 significant bits (tf32, nearest) on the fp32 pipe (Veltkamp split
// with 2^13 + 1; explicitly rounded operators keep it from being contracted)
__device__ __forceinline__ float2 tf32_rn2(float2 x) {
    const float2 t = __fmul2_rn(x, make_float2(8193.0f, 8193.0f));
    return f2_sub(t, f2_sub(t, x));
}
// 32 fp32 values as bf16 pairs hi + lo (hi = bf16(x), lo = bf16(x - hi)), packed for a
// kind::f16 A operand: the 32 columns at taddr hold the hi pairs in the first 16, lo in the next
__device__ __forceinline__ void store_split32(uint32_t taddr, const float (&x)[32]) {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
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
__host__ __device__ constexpr uint32_t split_col(int kk, bool lo) {
    return (uint32_t)(32 * (kk >> 1) + 8 * (kk & 1) + (lo ? 16 : 0));
}
// named barriers: 1 / 5 = state warpgroups (256), 2 / 3 = producer warpgroup 0 / 1 (128 each),
// 4 = both producer warpgroups (256)
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
// byte offset of (row, channel) of one [64 rows][64 channels] bf16 block in the 128-byte
// swizzled layout (128-byte rows, 16-byte units XOR row % 8)
__device__ __forceinline__ uint32_t sw128(int row, int ch) {
    return (uint32_t)(row * 128 + ((((ch >> 3) ^ row) & 7) << 4) + ((ch & 7) << 1));
}
// byte offset of element (i, j) of a 64 x 64 fp32 matrix in the K-major 128-byte swizzled tf32
// operand image: 32-column atoms of 8 KB, 128-byte rows, 16-byte units XOR row % 8
__device__ __forceinline__ uint32_t img_off(int i, int j) {
    return (uint32_t)((j >> 5) * 8192 + i * 128 + ((((j & 31) >> 2) ^ (i & 7)) << 4) + ((j & 3) << 2));
}

// 2^x and 1/x on the special-function unit (PTX ex2.approx / rcp.approx, flush to zero)
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// SiLU of an fp32 pair, x / (1 + e^-x) with e^-x = 2^(-x log2(e)), on packed fp32x2 arithmetic
__device__ __forceinline__ float2 silu2(float2 x) {
    const float2 a = __fmul2_rn(x, make_float2(-1.4426950408889634f, -1.4426950408889634f));
    const float2 d = __fadd2_rn(make_float2(ex2_approx(a.x), ex2_approx(a.y)), make_float2(1.f, 1.f));
    return __fmul2_rn(x, make_float2(rcp_approx(d.x), rcp_approx(d.y)));
}
// conv + SiLU of one bf16 channel pair: taps newest first, one bf16 rounding per tap (the first
// a bf16 product, then fused multiply-adds: deltanet.py:66-80); SiLU in fp32, rounded to bf16
__device__ __forceinline__ uint32_t conv_silu_pair(__nv_bfloat162 x0, __nv_bfloat162 x1, __nv_bfloat162 x2,
                                                  __nv_bfloat162 x3, const __nv_bfloat162 (&w)[4]) {
    __nv_bfloat162 acc = __hmul2(x0, w[3]);
    acc = __hfma2(x1, w[2], acc);
    acc = __hfma2(x2, w[1], acc);
    acc = __hfma2(x3, w[0], acc);
    const float2 s = silu2(__bfloat1622float2(acc));
    return bf2_bits(s.x, s.y);
}
// conv + SiLU in place of 32 consecutive tokens of one q / k channel pair in a 128-byte swizzled
// 64-row block (o8[r]: byte offset of the pair in row r of each 8-row group), with the raw values
// of the three tokens before; sq[j] = sum of squares of the pair's two outputs of token j.
// Tokens at or past `nvalid` (kGuard) are outputs 0 (past the sequence end).
template <bool kGuard>
__device__ __forceinline__ void conv_qk32(unsigned char* base, const uint32_t (&o8)[8], uint32_t h1, uint32_t h2,
                                          uint32_t h3, const __nv_bfloat162 (&w)[4], int nvalid, float (&sq)[32]) {
    // 16 tokens at a time: every raw value of the group is loaded before any output is stored
    // (the stores go to the same rows, so loads and stores would otherwise serialise)
    __nv_bfloat162 x1 = as_bf2(h1), x2 = as_bf2(h2), x3 = as_bf2(h3);
#pragma unroll
    for (int g = 0; g < 32; g += 16) {
        uint32_t xr[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
            xr[j] = *reinterpret_cast<const uint32_t*>(base + ((g + j) >> 3) * 1024 + o8[(g + j) & 7]);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const __nv_bfloat162 x0 = as_bf2(xr[j]);
            const uint32_t o = (!kGuard || g + j < nvalid) ? conv_silu_pair(x0, x1, x2, x3, w) : 0u;
            *reinterpret_cast<uint32_t*>(base + ((g + j) >> 3) * 1024 + o8[(g + j) & 7]) = o;
            x3 = x2;
            x2 = x1;
            x1 = x0;
            const float2 f = make_float2(bf_lo(o), bf_hi(o));
            const float2 f2 = __fmul2_rn(f, f);
            sq[g + j] = f2.x + f2.y;
        }
    }
}
// the same for 16 tokens of one v channel pair in row-major [64][128] bf16 rows (base: the
// first token's cell)
template <bool kGuard>
__device__ __forceinline__ void conv_v16(unsigned char* base, uint32_t h1, uint32_t h2, uint32_t h3,
                                         const __nv_bfloat162 (&w)[4], int nvalid) {
    __nv_bfloat162 x1 = as_bf2(h1), x2 = as_bf2(h2), x3 = as_bf2(h3);
    uint32_t xr[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) xr[j] = *reinterpret_cast<const uint32_t*>(base + j * 256);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const __nv_bfloat162 x0 = as_bf2(xr[j]);
        *reinterpret_cast<uint32_t*>(base + j * 256) = (!kGuard || j < nvalid) ? conv_silu_pair(x0, x1, x2, x3, w) : 0u;
        x3 = x2;
        x2 = x1;
        x1 = x0;
    }
}
// A wait expected to be long (one role waiting for the other, or for a tensor copy): polls with
// a short sleep between tries so the waiting warps leave the issue slots to the working ones;
// bounded like mbar_wait_bounded.
__device__ __forceinline__ bool mbar_wait_patient(uint32_t bar, uint32_t parity, unsigned int err_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        __nanosleep(it < 16 ? 20 : 100);
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0u && global_timer_ns() - t0 > GDN_WAIT_LIMIT_NS) {
            atomicOr(&g_device_error, err_flag);
            return false;
        }
    }
}

// T = (I + A)^-1 of one chunk in place over A (the K-major operand image layout of img_off), by
// the 256 threads tix = 0..255 of a group that synchronises on named barrier bar_id, doubling up
// from the diagonal as the reference's block solve does (deltanet.py:112-162):
//   1. the four 16 x 16 diagonal blocks by forward substitution (two warps, a half-warp per
//      block, lane = column);
//   2. 16 -> 32: X = A21 T11 parked in the zero upper-right 16 x 16 of each 32 x 32 diagonal
//      block, then T21 = -T22 X over A21;
//   3. 32 -> 64: the same with the 32 x 32 blocks (X in the upper-right 32 x 32);
// then every element rounded to tf32 (nearest), zero above the diagonal (the parked products
// included), and fenced for the tensor cores.  The block products skip the known zeros of the
// triangular factors; every loop has a fixed trip count (predicated) so the loads pipeline.
__device__ __forceinline__ float4 ld_img4(const unsigned char* Tb, int i, int j) {
    return *reinterpret_cast<const float4*>(Tb + img_off(i, j));
}
__device__ __forceinline__ float2 ld_img2(const unsigned char* Tb, int i, int j) {
    return *reinterpret_cast<const float2*>(Tb + img_off(i, j));
}
__device__ __forceinline__ void build_t_image(unsigned char* Tb, int tix, int lane, int bar_id) {
    nb_sync(bar_id, 256);
    if (tix < 64) {  // 1. diagonal 16 x 16 blocks
        const int blk = (tix >> 4), o = 16 * blk, jl = lane & 15;
        float x[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) x[i] = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            float2 s01 = make_float2(0.f, 0.f), s23 = make_float2(0.f, 0.f);
#pragma unroll
            for (int k = 0; k < i; k += 4) {
                const float4 a = ld_img4(Tb, o + i, o + k);
                s01 = __ffma2_rn(make_float2(a.x, a.y), make_float2(x[k], x[k + 1]), s01);
                s23 = __ffma2_rn(make_float2(a.z, a.w), make_float2(x[k + 2], x[k + 3]), s23);
            }
            x[i] = (i == jl ? 1.f : 0.f) - ((s01.x + s01.y) + (s23.x + s23.y));
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) *reinterpret_cast<float*>(Tb + img_off(o + i, o + jl)) = x[i];
    }
    nb_sync(bar_id, 256);
    {  // 2. 16 -> 32 in both 32 x 32 diagonal blocks: item = (block, row r, two columns c2)
        const int o = 32 * (tix >> 7), r = (tix >> 3) & 15, c2 = (tix & 7) * 2;
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 16; ++k) {  // X[r][c2..] = A21[r][k] T11[k][c2..], T11[k][c] = 0 for k < c
            if (k >= c2) {
                const float a = *reinterpret_cast<const float*>(Tb + img_off(o + 16 + r, o + k));
                acc = __ffma2_rn(make_float2(a, a), ld_img2(Tb, o + k, o + c2), acc);
            }
        }
        *reinterpret_cast<float2*>(Tb + img_off(o + r, o + 16 + c2)) = acc;  // upper-right 16 x 16: free
        nb_sync(bar_id, 256);
        acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 16; ++k) {  // T21[r][c2..] = -T22[r][k] X[k][c2..], T22[r][k] = 0 for k > r
            if (k <= r) {
                const float a = *reinterpret_cast<const float*>(Tb + img_off(o + 16 + r, o + 16 + k));
                acc = __ffma2_rn(make_float2(a, a), ld_img2(Tb, o + k, o + 16 + c2), acc);
            }
        }
        *reinterpret_cast<float2*>(Tb + img_off(o + 16 + r, o + c2)) = make_float2(-acc.x, -acc.y);
    }
    nb_sync(bar_id, 256);
    const int bi = tix >> 3, jb = (tix & 7) * 4;
    {  // 3. X[bi][jb..] = A21[bi][:] T11[:][jb..] (T11[k][j] = 0 for k < j), into the upper-right 32 x 32
        float2 a01 = make_float2(0.f, 0.f), a23 = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 32; k += 4) {
            if (k >= jb) {
                const float4 a = ld_img4(Tb, 32 + bi, k);
                const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const float4 r = ld_img4(Tb, k + kk, jb);
                    a01 = __ffma2_rn(make_float2(av[kk], av[kk]), make_float2(r.x, r.y), a01);
                    a23 = __ffma2_rn(make_float2(av[kk], av[kk]), make_float2(r.z, r.w), a23);
                }
            }
        }
        *reinterpret_cast<float4*>(Tb + img_off(bi, 32 + jb)) = make_float4(a01.x, a01.y, a23.x, a23.y);
    }
    nb_sync(bar_id, 256);
    {  // T21[bi][jb..] = -T22[bi][:] X[:][jb..] (T22[i][k] = 0 for k > i), over A21
        float2 a01 = make_float2(0.f, 0.f), a23 = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 32; k += 4) {
            if (k <= bi) {
                const float4 a = ld_img4(Tb, 32 + bi, 32 + k);
                const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const float4 r = ld_img4(Tb, k + kk, 32 + jb);
                    a01 = __ffma2_rn(make_float2(av[kk], av[kk]), make_float2(r.x, r.y), a01);
                    a23 = __ffma2_rn(make_float2(av[kk], av[kk]), make_float2(r.z, r.w), a23);
                }
            }
        }
        *reinterpret_cast<float4*>(Tb + img_off(32 + bi, jb)) = make_float4(-a01.x, -a01.y, -a23.x, -a23.y);
    }
    nb_sync(bar_id, 256);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int idx = tix + 256 * e, i = idx >> 4, j = (idx & 15) * 4;
        float4* cell = reinterpret_cast<float4*>(Tb + img_off(i, j));
        const float4 v = *cell;
        *cell = make_float4(j + 0 <= i ? umma::tf32_rna(v.x) : 0.f, j + 1 <= i ? umma::tf32_rna(v.y) : 0.f,
                            j + 2 <= i ? umma::tf32_rna(v.z) : 0.f, j + 3 <= i ? umma::tf32_rna(v.w) : 0.f);
    }
    fence_proxy_async_smem();  // T is read by the tensor cores next
    nb_sync(bar_id, 256);
}

struct FusedMaps {
    CUtensorMap qk;    // raw mixed rows, box 64 channels x 64 tokens, 128-byte swizzle
    CUtensorMap v;     // raw mixed rows, box 128 channels x 64 tokens
    CUtensorMap hist;  // raw mixed rows, box 64 channels x 4 tokens
    CUtensorMap z;     // z rows, box 128 x 64
    CUtensorMap out;   // output rows, box 128 x 64
};

__global__ void __launch_bounds__(NT, 1)
    prefill_fused_kernel(const MixParams p, const CkptList ck, float* __restrict__ hs, int* __restrict__ hflag,
                         const __grid_constant__ FusedMaps maps, const int split) {
    extern __shared__ unsigned char raw[];
    const uint32_t raw_addr = smem_u32(raw);
    unsigned char* sm = raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const uint32_t sb = smem_u32(sm);
    float* scr = reinterpret_cast<float*>(sm + R_SCR);
    float* sPart = scr + S_PART;
    float* sF = scr + S_F;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + R_BAR);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + R_BAR + NBAR * 8);
    auto bar = [&](int i) { return smem_u32(&bars[i]); };
    auto vecs = [&](int cc) { return reinterpret_cast<float*>(sm + R_VEC) + VEC_FLOATS * (cc % NQK); };

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wg = warp >> 2, q4 = warp & 3;
    const bool main_grp = tid < NMAIN;
    const int dv = 32 * q4 + lane;  // this thread's tensor-memory lane
    const uint32_t lane_base = (uint32_t)(32 * q4) << 16;
    const int NCg = (p.T + C - 1) / C;  // chunks of a chain
    const int chains = p.B * p.Hv;
    const int conv_dim = 2 * p.Hk * D + p.Hv * D;

    if (warp == 0) {
        umma::tmem_alloc(smem_u32(tslot), T_COLS);
        umma::tmem_relinquish();
    }
    if (tid == 0) {
        prefetch_tmap(&maps.qk);
        prefetch_tmap(&maps.v);
        prefetch_tmap(&maps.hist);
        prefetch_tmap(&maps.z);
        prefetch_tmap(&maps.out);
    }
    if (tid < D) reinterpret_cast<TA*>(sm + R_SCR)[tid] = static_cast<const TA*>(p.normw)[tid];  // bf16
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *tslot;

    // Split mode (more chains than CTAs): the chains' chunks laid end to end are cut into
    // gridDim.x equal runs.  A run holds at most a chain's last chunks (its tail), whole chains
    // and a chain's first chunks (its head); the CTA does the head first and the tail last, so
    // the head of a chain (at the previous CTA's start) is done long before its tail begins.
    // The state crosses in hand-off slot k (between CTAs k and k + 1), released by a flag.
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
    const bool has_head = split && hi > lo && ce_last < NCg;
    const bool has_tail = split && hi > lo && cs_first > 0 && !(has_head && first == last);
    const int npieces = split ? (hi > lo ? last - first + 1 : 0) : 1;
    bool cta_failed = false;
    for (int pi = 0; pi < npieces && !cta_failed; ++pi) {
    int chain = first;
    if (split) {
        const int k = pi - (has_head ? 1 : 0);
        const int n_rest = npieces - (has_head ? 1 : 0);
        if (has_head && pi == 0) chain = last;
        else if (has_tail) chain = k < n_rest - 1 ? first + 1 + k : first;
        else chain = first + k;
    }
    int c_base, c_end;
    piece_of(chain, c_base, c_end);
    const int NC = c_end - c_base;
    const int in_slot = c_base > 0 ? (int)blockIdx.x - 1 : -1;
    const int out_slot = c_end < NCg ? (int)blockIdx.x : -1;
    const int bh = chain;
    const int b = bh / p.Hv, h = bh - (bh / p.Hv) * p.Hv;
    const int rep = p.Hv / p.Hk, kh = h / rep;

    if (tid == 0) {
        if (pi > 0)
            for (int i = 0; i < NBAR; ++i) mbar_inval(bar(i));
        // every producer thread arrives on gp_free; one thread on the others
        for (int i = 0; i < NBAR; ++i) mbar_init(bar(i), i == B_GPFREE ? NT - NMAIN : 1);
        fence_mbar_init();
    }
    if (c_base == 0) write_conv_windows<TA, D, D, NT>(p, ck, b, h, kh, rep);
    bool hand_ok = true;
    if (in_slot >= 0 && tid == 0) hand_ok = wait_flag_bounded(hflag + in_slot);
    umma::fence_before_sync();
    if (__syncthreads_or(!hand_ok)) {
        cta_failed = true;
        break;
    }
    umma::fence_after_sync();

    // initial state, transposed: lane dv, column dk (warpgroup wg of all four: dk 32 wg ..
    // 32 wg + 31) in the fp32 master, and its bf16 hi / lo operand in the same 32 columns of
    // the operand region
    {
        const int c0 = 32 * wg;
        const float* src = in_slot >= 0 ? hs + (size_t)in_slot * D * D
                                         : (p.S_in ? p.S_in + (size_t)bh * D * D : nullptr);
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = src ? __ldcg(src + (size_t)(c0 + j) * D + dv) : 0.f;
        umma::tmem_st32(tmem + lane_base + C_MS + c0, v);
        store_split32(tmem + lane_base + C_OP + c0, v);
        umma::tmem_wait_st();
    }
    const int v_ch = 2 * p.Hk * D + h * D;  // first v channel of this value head
    // input copies of chunk cc of the piece: raw [k;q] rows + their history into buffer cc % 3,
    // raw v rows + history into buffer cc % 2, z rows into the z tile
    auto issue_qk = [&](int cc) {
        const int t0 = (c_base + cc) * C;
        const uint32_t dst = sb + R_QK + QK_BYTES * (uint32_t)(cc % NQK), hb = sb + R_HQK + 4 * HATOM * (cc % NQK);
        const uint32_t br = bar(B_RAWQK + cc % NQK);
        mbar_arrive_expect_tx(br, QK_BYTES + 4 * HATOM);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            tma_load_3d(dst + 16384u * j, &maps.qk, p.Hk * D + kh * D + 64 * j, t0, b, br);          // k
            tma_load_3d(dst + 16384u * j + 8192u, &maps.qk, kh * D + 64 * j, t0, b, br);             // q
            tma_load_3d(hb + HATOM * j, &maps.hist, kh * D + 64 * j, t0 - (int)HROWS, b, br);        // q history
            tma_load_3d(hb + HATOM * (2 + j), &maps.hist, p.Hk * D + kh * D + 64 * j, t0 - (int)HROWS, b, br);
        }
    };
    auto issue_v = [&](int cc) {
        const int t0 = (c_base + cc) * C;
        const uint32_t br = bar(B_RAWV + cc % NVB), hb = sb + R_HV + 2 * HATOM * (cc % NVB);
        mbar_arrive_expect_tx(br, V_BYTES + 2 * HATOM);
        tma_load_3d(sb + R_V + V_BYTES * (uint32_t)(cc % NVB), &maps.v, v_ch, t0, b, br);
        tma_load_3d(hb, &maps.hist, v_ch, t0 - (int)HROWS, b, br);
        tma_load_3d(hb + HATOM, &maps.hist, v_ch + 64, t0 - (int)HROWS, b, br);
    };
    auto issue_z = [&](int cc) {
        mbar_arrive_expect_tx(bar(B_Z), (uint32_t)C * D * 2u);
        tma_load_3d(sb + R_Z, &maps.z, h * D, (c_base + cc) * C, b, bar(B_Z));
    };
    // every input copy is issued by one thread of the state path (warp 1, lane 0: warp 0 issues
    // the MMAs), which counts them for the drain at the piece's end
    constexpr int TMA_TID = 32;
    int n_rqk[NQK] = {0, 0, 0}, n_rv[NVB] = {0, 0}, n_z = 0;
    if (tid == TMA_TID) {
        for (int i = 0; i < NQK && i < NC; ++i) n_rqk[i] = 1;
        for (int i = 0; i < NVB && i < NC; ++i) n_rv[i] = 1;
        n_z = 1;
        issue_qk(0);
        if (NC > 1) issue_qk(1);
        if (NC > 2) issue_qk(2);
        issue_v(0);
        if (NC > 1) issue_v(1);
        issue_z(0);
    }
    umma::fence_before_sync();
    __syncthreads();
    bool failed = false;
    if (main_grp) {
        // ======================= state path (warpgroups 0-1) =======================
        const uint32_t idesc_c = umma::idesc_tf32(128, 64, 0, 0);
        const uint32_t idesc_b = umma::idesc_bf16(128, 64, 0, 0);
        const uint32_t idesc_e = umma::idesc_bf16(128, 128, 0, 1);
        uint32_t mma_phase = 0;
        bool mma_pending = false;
        int ck_i = 0;  // first checkpoint past the piece's start (earlier ones belong to the head)
        while (ck_i < ck.n && ck.off[ck_i] <= c_base * C) ++ck_i;
        // A bounded wait that runs out marks this thread bad; the threads agree on it once per
        // chunk and leave together.  Until then a bad thread keeps going on stale data: every
        // address it touches is fixed by the chunk index, never by data.
        bool bad = false;
        auto mma_wait = [&]() {  // patient: warps 1-7 wait here while warp 0 waits for the producer
            const bool ok = mbar_wait_patient(bar(B_MMA), mma_phase & 1u, GDN_DEVERR_MMA_TIMEOUT);
            ++mma_phase;
            umma::fence_after_sync();
            bad |= !ok;
            if (ok) mma_pending = false;
        };
        auto wait_phase = [&](uint32_t br, int phase) {  // signals of the producer warps
            bad |= !mbar_wait_patient(br, (uint32_t)phase & 1u, GDN_DEVERR_TMA_TIMEOUT);
        };
        auto stores_to_warp0 = [&]() {
            umma::fence_before_sync();
            if (warp == 0)
                nb_sync(1, NMAIN);
            else
                nb_arrive(1, NMAIN);
        };
        // output rows: token otok, channels 32 osg .. 32 osg + 31 as four 16-byte units, visited in
        // a per-lane rotated order (ounit[k]: byte offset in the row) so that a quarter-warp
        // touches 8 different bank groups
        const int otok = tid >> 2, osg = tid & 3;
        uint32_t ounit[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) ounit[k] = (uint32_t)(4 * osg + ((k + osg + (otok & 1)) & 3)) * 16u;
        int w_z = 0;  // z copies waited for
        // T of chunks 0 and 1 (later ones are built two chunks ahead at the end of each chunk)
        for (int cc = 0; cc < 2 && cc < NC; ++cc) {
            wait_phase(bar(B_APR + cc), 0);
            build_t_image(sm + R_TP + TP_BYTES * (uint32_t)cc, tid, lane, 1);
        }
        for (int c = 0; c < NC; ++c) {
            const int t0 = (c_base + c) * C;
            const float* sv = vecs(c);
            const uint32_t r_qk = R_QK + QK_BYTES * (uint32_t)(c % NQK);
            const uint32_t r_tp = R_TP + TP_BYTES * (uint32_t)(c % NTP);
            const unsigned char* vrows = sm + R_V + V_BYTES * (uint32_t)(c % NVB);
            // ---------------- MMA-b (this path read O of the last chunk out of [Y | O1] already) ----------------
            if (warp == 0) {
                wait_phase(bar(B_KQ + c % NQK), c / NQK);
                __syncwarp();
                umma::fence_after_sync();
                const uint64_t d_k = umma::desc_kmajor0(sb + r_qk), d_q = umma::desc_kmajor0(sb + r_qk + 8192);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma::mma_bf16_ta_elect(tmem + C_YO, tmem + C_OP + split_col(kk, false),
                                            umma::desc_add(d_k, umma::kmajor_kstep(kk, 128)), idesc_b, kk > 0);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma::mma_bf16_ta_elect(tmem + C_YO, tmem + C_OP + split_col(kk, true),
                                            umma::desc_add(d_k, umma::kmajor_kstep(kk, 128)), idesc_b, 1u);
                umma::mma_commit_elect(bar(B_MMA));
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma::mma_bf16_ta_elect(tmem + C_YO + 64, tmem + C_OP + split_col(kk, false),
                                            umma::desc_add(d_q, umma::kmajor_kstep(kk, 128)), idesc_b, kk > 0);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma::mma_bf16_ta_elect(tmem + C_YO + 64, tmem + C_OP + split_col(kk, true),
                                            umma::desc_add(d_q, umma::kmajor_kstep(kk, 128)), idesc_b, 1u);
                umma::mma_commit_elect(bar(B_O1));
                mma_pending = true;
            }
            mma_wait();
            wait_phase(bar(B_KQ + c % NQK), c / NQK);  // the chunk's vectors (every reader acquires them)
            wait_phase(bar(B_VR + c % NVB), c / NVB);  // the chunk's conv'd v rows
            const float ec = sv[V_EC];
            // ---------------- Z^T = beta (V - e^gamma rk Y)^T (warpgroup wg: tokens 32 wg ..) ----------------
            {
                float y[32];
                umma::tmem_ld32(tmem + lane_base + C_YO + 32 * wg, y);
                umma::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    const int t = 32 * wg + j;
                    const float2 vv = make_float2(bf_at(vrows, t * D + dv), bf_at(vrows, (t + 1) * D + dv));
                    const float2 nek = *reinterpret_cast<const float2*>(sv + V_EK + t);
                    const float2 be = *reinterpret_cast<const float2*>(sv + V_B + t);
                    const float2 r = tf32_rn2(__fmul2_rn(be, __ffma2_rn(nek, make_float2(y[j], y[j + 1]), vv)));
                    y[j] = r.x;
                    y[j + 1] = r.y;
                }
                umma::tmem_st32(tmem + lane_base + C_Z + 32 * wg, y);
                umma::tmem_wait_st();
            }
            stores_to_warp0();
            // ---------------- MMA-c: v_new^T = Z^T T^T (after the producer returned columns 448-511;
            //                  T of this chunk was built by this path two chunks ago) ----------------
            if (warp == 0) {
                const int gp = c + 1 < NC ? c + 1 : (c == 0 ? 0 : -1);
                if (gp >= 0) bad |= !mbar_wait_patient(bar(B_GPFREE), (uint32_t)gp & 1u, GDN_DEVERR_MMA_TIMEOUT);
                __syncwarp();
                umma::fence_after_sync();
                const uint64_t d_t = umma::desc_kmajor0(sb + r_tp);
#pragma unroll
                for (int kk = 0; kk < C / 8; ++kk)
                    umma::mma_tf32_ta_elect(tmem + C_V, tmem + C_Z + kk * 8,
                                            umma::desc_add(d_t, umma::kmajor_kstep(kk, C)), idesc_c, kk > 0);
                umma::mma_commit_elect(bar(B_MMA));
                mma_pending = true;
            }
            mma_wait();
            // ---------------- sub-chunk checkpoints (fp32 v_new, bf16 k rows, state before the update) ----------------
            // S_s = e^{gamma_{s-1}} S + sum_{t<s} e^{gamma_{s-1}-gamma_t} k_t^T v_new_t (deltanet.py:375-388)
            while (ck_i < ck.n && ck.off[ck_i] > t0 && ck.off[ck_i] - t0 < C) {
                const int s_off = ck.off[ck_i] - t0;
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
                        for (int j = 0; j < 32; ++j) wv[j] *= sF[32 * th + j] * sv[V_RK + 32 * th + j];
                        // k row t = 32 th + j, key columns cb + 8 j8 .. + 7: one 16-byte unit of the
                        // swizzled rows
                        const unsigned char* kb = sm + r_qk + 16384 * wg + 4096 * th;
                        const uint32_t hx0 = 64u * hb, hx1 = 64u - 64u * hb;
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const unsigned char* rowp = kb + (j >> 3) * 1024 + (j & 7) * 128 + ((j & 4) ? hx1 : hx0);
#pragma unroll
                            for (int j8 = 0; j8 < 4; ++j8) {
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
            // ---------------- (e^{gamma_C - gamma} rk v_new)^T as bf16 hi / lo ----------------
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
            // ---------------- MMA-e: dS^T into the operand columns (the state path waits for it) ----------------
            if (warp == 0) {
                wait_phase(bar(B_O1), c);
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
                umma::mma_commit_elect(bar(B_MMA));
                mma_pending = true;
            }
            // ---------------- v_new^T (tf32) for MMA-d while MMA-e runs ----------------
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
            umma::fence_before_sync();
            if (warp == 0)
                nb_sync(5, NMAIN);
            else
                nb_arrive(5, NMAIN);
            // ---------------- MMA-d: (P v_new)^T for the output warps ----------------
            if (warp == 0) {
                umma::fence_after_sync();
                const uint64_t d_p = umma::desc_kmajor0(sb + r_tp + 16384);
#pragma unroll
                for (int kk = 0; kk < C / 8; ++kk)
                    umma::mma_tf32_ta_elect(tmem + C_YO, tmem + C_V + kk * 8,
                                            umma::desc_add(d_p, umma::kmajor_kstep(kk, C)), idesc_c, kk > 0);
                umma::mma_commit_elect(bar(B_ORDY));
            }
            mma_wait();
            // ---------------- state update (key columns 64 wg ..), checkpoints, final state ----------------
            {
                const bool lastc = c == NC - 1;
                float* const s_end = !lastc ? nullptr
                                     : out_slot >= 0 ? hs + (size_t)out_slot * D * D
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
                if (lastc && out_slot >= 0) __threadfence();  // the hand-off state before its flag
            }
            while (ck_i < ck.n && ck.off[ck_i] - t0 == C) ++ck_i;
            // ---------------- output rows of chunk c through the gated RMSNorm (config.py:136-143) ----------------
            // O = e^gamma rq dk^-1/2 O1 + P v_new, rounded to bf16 (the reference's core output dtype),
            // staged token-major in the v buffer of chunk c (its v rows were consumed by Z)
            bad |= !mbar_wait_bounded(bar(B_ORDY), (uint32_t)c & 1u, GDN_DEVERR_MMA_TIMEOUT);
            umma::fence_after_sync();
            {
                float o1[32], dd[32];
                umma::tmem_ld32(tmem + lane_base + C_YO + 64 + 32 * wg, o1);
                umma::tmem_ld32(tmem + lane_base + C_YO + 32 * wg, dd);
                umma::tmem_wait_ld();
                const float* eqv = sv + V_EQ + 32 * wg;
                uint16_t* col = reinterpret_cast<uint16_t*>(sm + R_V + V_BYTES * (uint32_t)(c % NVB)) + 32 * wg * D + dv;
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    const uint32_t u = bf2_bits(fmaf(eqv[j], o1[j], dd[j]), fmaf(eqv[j + 1], o1[j + 1], dd[j + 1]));
                    col[j * D] = (uint16_t)(u & 0xFFFFu);
                    col[(j + 1) * D] = (uint16_t)(u >> 16);
                }
            }
            {
                const bool zok = mbar_wait_patient(bar(B_Z), (uint32_t)w_z & 1u, GDN_DEVERR_TMA_TIMEOUT);
                w_z += zok;
                bad |= !zok;
            }
            umma::fence_before_sync();
            nb_sync(1, NMAIN);  // O staged, and every read of [Y | O1] done: the next MMA-b may overwrite it
            umma::fence_after_sync();
            {  // each thread: one token's 32-channel segment; z read and the output written in place
                const unsigned char* ost = sm + R_V + V_BYTES * (uint32_t)(c % NVB) + otok * 256;
                unsigned char* zrow = sm + R_Z + otok * 256;
                uint4 ov[4], zw[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    ov[k] = *reinterpret_cast<const uint4*>(ost + ounit[k]);
                    zw[k] = *reinterpret_cast<const uint4*>(zrow + ounit[k]);
                }
                float2 acc = make_float2(0.f, 0.f);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t w4[4] = {ov[k].x, ov[k].y, ov[k].z, ov[k].w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = make_float2(bf_lo(w4[e]), bf_hi(w4[e]));
                        acc = __ffma2_rn(f, f, acc);
                    }
                }
                float ss = acc.x + acc.y;
                ss += __shfl_xor_sync(0xffffffffu, ss, 1);
                ss += __shfl_xor_sync(0xffffffffu, ss, 2);
                const float rstd = rsqrtf(ss / (float)D + p.eps);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    uint32_t w4[4] = {ov[k].x, ov[k].y, ov[k].z, ov[k].w};
                    const uint32_t z4[4] = {zw[k].x, zw[k].y, zw[k].z, zw[k].w};
                    const uint4 nw4 = *reinterpret_cast<const uint4*>(sm + R_SCR + ounit[k]);  // bf16 weights
                    const uint32_t nwk[4] = {nw4.x, nw4.y, nw4.z, nw4.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 y = __fmul2_rn(make_float2(bf_lo(w4[e]), bf_hi(w4[e])), make_float2(rstd, rstd));
                        // normed rounded to bf16, times the bf16 weight in one rounded bf16 product
                        const __nv_bfloat162 scaled = __hmul2(as_bf2(bf2_bits(y.x, y.y)), as_bf2(nwk[e]));
                        const float2 g = __fmul2_rn(__bfloat1622float2(scaled),
                                                    silu2(make_float2(bf_lo(z4[e]), bf_hi(z4[e]))));
                        w4[e] = bf2_bits(g.x, g.y);
                    }
                    *reinterpret_cast<uint4*>(zrow + ounit[k]) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                }
            }
            fence_proxy_async_smem();
            nb_sync(1, NMAIN);  // the output rows are complete; the staged O and z are read
            if (tid == TMA_TID && !bad) {
                // rows past the sequence end fall outside the tensor map and are not written
                tma_store_3d(&maps.out, sb + R_Z, h * D, t0, b);
                bulk_commit_group();
                // the buffers of chunk c are free (MMA-b, MMA-e, checkpoints and O staging done):
                // raw q / k rows of chunk c + 3 and raw v rows of chunk c + 2 land there
                if (c + 3 < NC) {
                    issue_qk(c + 3);
                    ++n_rqk[(c + 3) % NQK];
                }
                if (c + 2 < NC) {
                    issue_v(c + 2);
                    ++n_rv[(c + 2) % NVB];
                }
                if (c + 1 < NC) {
                    bulk_wait_group_read0();  // the tile is read: the next z rows may land there
                    issue_z(c + 1);
                    ++n_z;
                }
            }
            // ---------------- T of chunk c + 2 (its A and P come from the producer) ----------------
            if (c + 2 < NC) {
                wait_phase(bar(B_APR + (c + 2) % NTP), (c + 2) / NTP);
                build_t_image(sm + R_TP + TP_BYTES * (uint32_t)((c + 2) % NTP), tid, lane, 1);
            }
            umma::fence_before_sync();
            if (nb_any(bad, 1, NMAIN)) {
                failed = true;
                break;
            }
            umma::fence_after_sync();
            if (c == NC - 1 && out_slot >= 0 && tid == 0) release_flag(hflag + out_slot);  // state written
        }
        if (tid == 0 && failed && mma_pending)  // an MMA in flight finishes (bounded) before the CTA exits
            mbar_wait_bounded(bar(B_MMA), (mma_phase - 1) & 1u, GDN_DEVERR_MMA_TIMEOUT);
        if (tid == TMA_TID) {
            if (failed)
                for (; w_z < n_z; ++w_z) mbar_wait_bounded(bar(B_Z), (uint32_t)w_z & 1u, GDN_DEVERR_TMA_TIMEOUT);
            bulk_wait_group0();  // output rows written before the piece ends
            // the last copy into each buffer lands before the piece ends (bounded; every earlier one
            // on the same barrier was waited for before the next was issued)
            for (int i = 0; i < NQK; ++i)
                if (n_rqk[i] > 0)
                    mbar_wait_bounded(bar(B_RAWQK + i), (uint32_t)(n_rqk[i] - 1) & 1u, GDN_DEVERR_TMA_TIMEOUT);
            for (int i = 0; i < NVB; ++i)
                if (n_rv[i] > 0)
                    mbar_wait_bounded(bar(B_RAWV + i), (uint32_t)(n_rv[i] - 1) & 1u, GDN_DEVERR_TMA_TIMEOUT);
        }
    } else {
        // ================ producer and output rows (warpgroups 2-3, 256 threads) ================
        const int ptid = tid - NMAIN;
        const int owg = wg - 2, tw = 32 * owg;  // output tokens / [G; P0] columns tw .. tw + 31
        const TA* convw = static_cast<const TA*>(p.convw);
        const TA* cs_in = static_cast<const TA*>(p.cs_in);
        // this thread's q / k channel pair (conv of 32 tokens) and v channel pair (16 tokens)
        const int hf = ptid >> 7, pp = ptid & 127;
        const bool isk = pp >= 64;
        const int qch = 2 * (pp & 63), qatom = qch >> 6, qchl = qch & 63;
        const int gqk = (isk ? p.Hk * D : 0) + kh * D + qch;
        const int qt = ptid >> 6, vch = 2 * (ptid & 63);
        const int gv = v_ch + vch;
        uint32_t o8[8];  // byte offset of this thread's q / k pair in row r of an 8-row swizzle group
#pragma unroll
        for (int r = 0; r < 8; ++r) o8[r] = sw128(r, qchl);
        __nv_bfloat162 wqk[4], wvv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            wqk[j] = __halves2bfloat162(convw[(size_t)gqk * 4 + j], convw[(size_t)(gqk + 1) * 4 + j]);
            wvv[j] = __halves2bfloat162(convw[(size_t)gv * 4 + j], convw[(size_t)(gv + 1) * 4 + j]);
        }
        // raw history pair of channels (gc, gc + 1) at token tk < 0 of the chain: the conv state
        auto cs_pair = [&](int gc, int tk) -> uint32_t {
            if (!cs_in) return 0u;
            const TA* s = cs_in + ((size_t)b * conv_dim + gc) * 3 + (3 + tk);
            __nv_bfloat162 r = __halves2bfloat162(s[0], s[3]);
            return *reinterpret_cast<uint32_t*>(&r);
        };
        const float neg_a = -expf(p.A_log[h]), dt_b = p.dt_bias[h];  // g = neg_a softplus(a + dt_b)
        bool bad = false;
        bool gp_pending = false;
        int n_gp = 0;  // [G; P0] MMAs issued in this piece (thread 0)

        // --- conv + SiLU in place of the q / k rows of chunk cq and the v rows of chunk cv, norm
        //     factors, gates and per-token vectors of chunk cq; signals kq_ready(cq), v_ready(cv)
        auto prep = [&](int cq, int cv) {
            const int t0q = (c_base + cq) * C, t0v = (c_base + cv) * C;
            if (cq >= 0) bad |= !mbar_wait_patient(bar(B_RAWQK + cq % NQK), (uint32_t)(cq / NQK) & 1u,
                                                   GDN_DEVERR_TMA_TIMEOUT);
            if (cv >= 0) bad |= !mbar_wait_patient(bar(B_RAWV + cv % NVB), (uint32_t)(cv / NVB) & 1u,
                                                   GDN_DEVERR_TMA_TIMEOUT);
            float raw_a = 0.f, raw_b = 0.f;
            if (cq >= 0 && ptid < C && t0q + ptid < p.T) {
                const size_t ai = (size_t)b * p.as_b + (size_t)(t0q + ptid) * p.as_t + h;
                raw_a = Act<TA>::ld(static_cast<const TA*>(p.a) + ai);
                raw_b = Act<TA>::ld(static_cast<const TA*>(p.b) + ai);
            }
            unsigned char* qkb = sm + R_QK + QK_BYTES * (uint32_t)(cq % NQK) + qatom * 16384 + (isk ? 0 : 8192);
            unsigned char* vb = sm + R_V + V_BYTES * (uint32_t)(cv % NVB);
            // phase 1: the raw values of the three tokens before this thread's first token
            uint32_t q1 = 0u, q2 = 0u, q3 = 0u, v1 = 0u, v2 = 0u, v3 = 0u;
            if (cq >= 0) {
                if (hf == 1) {
                    q3 = *reinterpret_cast<const uint32_t*>(qkb + sw128(29, qchl));
                    q2 = *reinterpret_cast<const uint32_t*>(qkb + sw128(30, qchl));
                    q1 = *reinterpret_cast<const uint32_t*>(qkb + sw128(31, qchl));
                } else if (t0q > 0) {
                    const unsigned char* hb = sm + R_HQK + 4 * HATOM * (cq % NQK) + HATOM * ((isk ? 2 : 0) + qatom);
                    q3 = *reinterpret_cast<const uint32_t*>(hb + 1 * 128 + qchl * 2);
                    q2 = *reinterpret_cast<const uint32_t*>(hb + 2 * 128 + qchl * 2);
                    q1 = *reinterpret_cast<const uint32_t*>(hb + 3 * 128 + qchl * 2);
                } else {
                    q3 = cs_pair(gqk, -3);
                    q2 = cs_pair(gqk, -2);
                    q1 = cs_pair(gqk, -1);
                }
            }
            if (cv >= 0) {
                if (qt > 0) {
                    v3 = *reinterpret_cast<const uint32_t*>(vb + (16 * qt - 3) * 256 + vch * 2);
                    v2 = *reinterpret_cast<const uint32_t*>(vb + (16 * qt - 2) * 256 + vch * 2);
                    v1 = *reinterpret_cast<const uint32_t*>(vb + (16 * qt - 1) * 256 + vch * 2);
                } else if (t0v > 0) {
                    const unsigned char* hb = sm + R_HV + 2 * HATOM * (cv % NVB) + HATOM * (vch >> 6);
                    v3 = *reinterpret_cast<const uint32_t*>(hb + 1 * 128 + (vch & 63) * 2);
                    v2 = *reinterpret_cast<const uint32_t*>(hb + 2 * 128 + (vch & 63) * 2);
                    v1 = *reinterpret_cast<const uint32_t*>(hb + 3 * 128 + (vch & 63) * 2);
                } else {
                    v3 = cs_pair(gv, -3);
                    v2 = cs_pair(gv, -2);
                    v1 = cs_pair(gv, -1);
                }
            }
            nb_sync(4, NT - NMAIN);
            // phase 2: conv + SiLU in place; outputs of tokens past the sequence end are zero
            if (cq >= 0) {
                float sq[32];
                const int nval = p.T - (t0q + 32 * hf);
                if (nval >= 32)
                    conv_qk32<false>(qkb + 4096 * hf, o8, q1, q2, q3, wqk, nval, sq);
                else
                    conv_qk32<true>(qkb + 4096 * hf, o8, q1, q2, q3, wqk, nval, sq);
                // per-token sums over this warp's 64 channels: halving exchange that leaves token
                // 32 hf + lane in this lane
#pragma unroll
                for (int st = 0; st < 5; ++st) {
                    const int s = 16 >> st, half = 16 >> st;
                    const bool up = (lane & s) != 0;
#pragma unroll
                    for (int k = 0; k < half; ++k) {
                        const float send = up ? sq[k] : sq[k + half];
                        const float keep = up ? sq[k + half] : sq[k];
                        sq[k] = keep + __shfl_xor_sync(0xffffffffu, send, s);
                    }
                }
                sPart[(isk ? 128 : 0) + qatom * 64 + 32 * hf + lane] = sq[0];
            }
            if (cv >= 0) {
                const int nval = p.T - (t0v + 16 * qt);
                unsigned char* vcell = vb + 16 * qt * 256 + vch * 2;
                if (nval >= 16)
                    conv_v16<false>(vcell, v1, v2, v3, wvv, nval);
                else
                    conv_v16<true>(vcell, v1, v2, v3, wvv, nval);
            }
            fence_proxy_async_smem();  // the conv outputs are read by the tensor cores next
            nb_sync(4, NT - NMAIN);
            if (cv >= 0 && ptid == 0) mbar_arrive(bar(B_VR + cv % NVB));
            if (cq < 0) return;
            float* vv = vecs(cq);
            if (ptid < C) {
                const int t = ptid;
                const bool valid = t0q + t < p.T;
                vv[V_RQ + t] = rsqrtf((sPart[t] + sPart[64 + t]) + 1e-6f);
                vv[V_RK + t] = rsqrtf((sPart[128 + t] + sPart[192 + t]) + 1e-6f);
                vv[V_B + t] = valid ? Act<TA>::round(sigmoid_f(raw_b)) : 0.f;
                // gamma = cumsum(g) over the chunk (the reference's torch.cumsum): an inclusive scan
                // per warp by shuffles, then the second warp adds the first one's total
                float gs = valid ? neg_a * softplus_f(raw_a + dt_b) : 0.f;
#pragma unroll
                for (int d = 1; d < 32; d <<= 1) {
                    const float y = __shfl_up_sync(0xffffffffu, gs, d);
                    if (lane >= d) gs += y;
                }
                vv[V_G + t] = gs;
                nb_sync(6, C);
                if (t >= 32) vv[V_G + t] = gs + vv[V_G + 31];
                nb_sync(6, C);
                const float gt = vv[V_G + t], gC = vv[V_G + C - 1], rk = vv[V_RK + t];
                const float eg = expf(gt);
                vv[V_EG + t] = eg;
                vv[V_EK + t] = -(eg * rk);
                vv[V_EF + t] = expf(gC - gt) * rk;
                vv[V_EQ + t] = eg * (vv[V_RQ + t] * p.q_scale);
                vv[V_ENG + t] = expf(-gt) * rk;
                if (t == 0) vv[V_EC] = expf(gC);
            }
            nb_sync(4, NT - NMAIN);
            if (ptid == 0) mbar_arrive(bar(B_KQ + cq % NQK));
        };
        // --- [G; P0] = [k; q] k^T of chunk cc (raw conv outputs, exact bf16 products) into the
        //     borrowed tensor-memory columns; issued by thread 0
        auto issue_gp = [&](int cc) {
            if (ptid != 0) return;
            umma::fence_after_sync();
            const uint64_t d = umma::desc_kmajor0(sb + R_QK + QK_BYTES * (uint32_t)(cc % NQK));
            const uint32_t idesc = umma::idesc_bf16(128, 64, 0, 0);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                const uint64_t dk = umma::desc_add(d, umma::kmajor_kstep(kk, 128));
                umma::mma_bf16(tmem + C_V, dk, dk, idesc, kk > 0);
            }
            umma::mma_commit(bar(B_GP));
            gp_pending = true;
            ++n_gp;
        };
        // --- wait for [G; P0] of chunk cc, copy this thread's row segment out of tensor memory
        //     (lane dv: rows 0-63 = G, 64-127 = P0; columns tw .. tw + 31), give the columns back,
        //     and write A (lower triangle, fp32) and P (tf32, masked) of the chunk
        auto build_ap = [&](int cc) {
            const bool ok = mbar_wait_bounded(bar(B_GP), (uint32_t)cc & 1u, GDN_DEVERR_MMA_TIMEOUT);
            bad |= !ok;
            if (ok && ptid == 0) gp_pending = false;
            umma::fence_after_sync();
            float g[32];
            umma::tmem_ld32(tmem + lane_base + C_V + tw, g);
            umma::tmem_wait_ld();
            umma::fence_before_sync();
            mbar_arrive(bar(B_GPFREE));
            const float* vv = vecs(cc);
            const bool g_row = dv < C;
            const int t = dv & (C - 1);
            const float gt = vv[V_G + t];
            // decay e^{gamma_t - gamma_j}: as e^{gamma_t} e^{-gamma_j} when neither factor leaves
            // the normal range (gamma >= -80 over the chunk), else one exp per pair; the column
            // norm factor rk_j rides on it, the row factor is beta_t rk_t (A) or rq_t dk^-1/2 (P)
            const bool factored = vv[V_G + C - 1] >= -80.f;
            const float rowf = g_row ? vv[V_B + t] * vv[V_RK + t] : vv[V_RQ + t] * p.q_scale;
            const float erow = vv[V_EG + t] * rowf;
            unsigned char* dst = sm + R_TP + TP_BYTES * (uint32_t)(cc % NTP) + (g_row ? 0u : 16384u);
            // every value first (the column vectors read as 16-byte broadcasts), then the stores
            if (factored) {
                const float4* e4 = reinterpret_cast<const float4*>(vv + V_ENG + tw);
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 e = e4[q];
                    const float2 a = __fmul2_rn(make_float2(g[4 * q], g[4 * q + 1]),
                                                __fmul2_rn(make_float2(erow, erow), make_float2(e.x, e.y)));
                    const float2 b = __fmul2_rn(make_float2(g[4 * q + 2], g[4 * q + 3]),
                                                __fmul2_rn(make_float2(erow, erow), make_float2(e.z, e.w)));
                    g[4 * q] = a.x;
                    g[4 * q + 1] = a.y;
                    g[4 * q + 2] = b.x;
                    g[4 * q + 3] = b.y;
                }
            } else {
                const float4* g4 = reinterpret_cast<const float4*>(vv + V_G + tw);
                const float4* k4 = reinterpret_cast<const float4*>(vv + V_RK + tw);
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 gg = g4[q], rk = k4[q];
                    g[4 * q] *= __expf(gt - gg.x) * (rowf * rk.x);
                    g[4 * q + 1] *= __expf(gt - gg.y) * (rowf * rk.y);
                    g[4 * q + 2] *= __expf(gt - gg.z) * (rowf * rk.z);
                    g[4 * q + 3] *= __expf(gt - gg.w) * (rowf * rk.w);
                }
            }
#pragma unroll
            for (int jj = 0; jj < 32; jj += 4) {
                const int j = tw + jj;
                float val[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    val[e] = g_row ? (j + e < t ? g[jj + e] : 0.f) : (j + e <= t ? umma::tf32_rna(g[jj + e]) : 0.f);
                *reinterpret_cast<float4*>(dst + img_off(t, j)) = make_float4(val[0], val[1], val[2], val[3]);
            }
            fence_proxy_async_smem();  // P is read by MMA-d
            nb_sync(4, NT - NMAIN);    // every [G; P0] read and A / P write of the group is done
            if (ptid == 0) mbar_arrive(bar(B_APR + cc % NTP));
        };
        // ---- prologue: chunks 0 and 1 convolved, their A / P built ----
        prep(0, 0);
        if (NC > 1) prep(1, -1);
        issue_gp(0);
        build_ap(0);
        if (NC > 1) {
            issue_gp(1);
            build_ap(1);
        }
        if (nb_any(bad, 4, NT - NMAIN)) failed = true;
        for (int c = 0; c < NC && !failed; ++c) {
            // conv of the q / k rows of chunk c + 2 and the v rows of chunk c + 1, then [G; P0], A and
            // P of chunk c + 2 once MMA-d of chunk c has released the borrowed tensor-memory columns
            const int cq = c + 2 < NC ? c + 2 : -1, cv = c + 1 < NC ? c + 1 : -1;
            if (cq >= 0 || cv >= 0) prep(cq, cv);
            if (cq >= 0) {
                bad |= !mbar_wait_patient(bar(B_ORDY), (uint32_t)c & 1u, GDN_DEVERR_MMA_TIMEOUT);
                umma::fence_after_sync();
                issue_gp(cq);
                build_ap(cq);
            }
            if (nb_any(bad, 4, NT - NMAIN)) {
                failed = true;
                break;
            }
        }
        if (ptid == 0 && gp_pending)  // a [G; P0] MMA in flight finishes (bounded) before the piece ends
            mbar_wait_bounded(bar(B_GP), (uint32_t)(n_gp - 1) & 1u, GDN_DEVERR_MMA_TIMEOUT);
    }
    umma::fence_before_sync();
    cta_failed = __syncthreads_or(failed);
    }  // pieces
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tmem, T_COLS);
}

}  // namespace pfused

size_t prefill_fused_ws_layout(int n_hs, size_t off[2]) {
    off[0] = 0;
    off[1] = ((size_t)n_hs * 128 * 128 * 4 + 1023) & ~(size_t)1023;
    return (off[1] + (size_t)n_hs * 4 + 1023) & ~(size_t)1023;
}

cudaError_t launch_prefill_fused(const MixParams& p, const CkptList& ck, float* hs, int* hflag, int n_hs,
                                 cudaStream_t s) {
    const uint64_t conv_dim = 2ull * p.Hk * 128 + (uint64_t)p.Hv * 128;
    pfused::FusedMaps maps;
    const uint64_t T = (uint64_t)p.T, B = (uint64_t)p.B;
    if (!encode_tmap_3d_bf16(&maps.qk, p.mixed, conv_dim, T, B, (uint64_t)p.ms_t * 2, (uint64_t)p.ms_b * 2, 64,
                             pfused::C, true) ||
        !encode_tmap_3d_bf16(&maps.v, p.mixed, conv_dim, T, B, (uint64_t)p.ms_t * 2, (uint64_t)p.ms_b * 2, 128,
                             pfused::C) ||
        !encode_tmap_3d_bf16(&maps.hist, p.mixed, conv_dim, T, B, (uint64_t)p.ms_t * 2, (uint64_t)p.ms_b * 2, 64,
                             pfused::HROWS) ||
        !encode_tmap_3d_bf16(&maps.z, p.z, (uint64_t)p.Hv * 128, T, B, (uint64_t)p.zs_t * 2, (uint64_t)p.zs_b * 2,
                             128, pfused::C) ||
        !encode_tmap_3d_bf16(&maps.out, p.out, (uint64_t)p.Hv * 128, T, B, (uint64_t)p.Hv * 128 * 2,
                             (uint64_t)p.Hv * 128 * 2 * T, 128, pfused::C))
        return cudaErrorInvalidValue;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(pfused::prefill_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)pfused::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    const int chains = p.B * p.Hv;
    if (n_hs > 1 && chains > n_hs) {
        // split mode: one CTA per SM, all resident at once (a cooperative launch guarantees it),
        // the chains cut into equal runs with state hand-offs between neighbouring CTAs; the
        // hand-off flags start at zero on every call
        e = cudaMemsetAsync(hflag, 0, (size_t)n_hs * sizeof(int), s);
        if (e != cudaSuccess) return e;
        int split = 1;
        void* kargs[] = {const_cast<MixParams*>(&p), const_cast<CkptList*>(&ck), &hs, &hflag, &maps, &split};
        e = cudaLaunchCooperativeKernel((const void*)pfused::prefill_fused_kernel, dim3(n_hs), dim3(pfused::NT),
                                        kargs, pfused::SMEM_BYTES, s);
        if (e == cudaSuccess) return cudaSuccess;
        (void)cudaGetLastError();  // not launchable as one resident wave here: one CTA per chain
    }
    pfused::prefill_fused_kernel<<<chains, pfused::NT, pfused::SMEM_BYTES, s>>>(p, ck, hs, hflag, maps, 0);
    return cudaGetLastError();
}

unsigned int prefill_fused_device_error(bool clear) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
    if (clear && v) {
        const unsigned int zero = 0;
        cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
    }
    return v;
}

}  // namespace gdn
