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
// scratch floats: norm weight, partial sums (output-norm partials, or the conv's norm
// partials: q / k x 2 atoms x 64 tokens), rstd, checkpoint decay
constexpr int S_NW = 0, S_PART = 128, S_RSTD = 384, S_F = 448, S_END = 512;
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
    B_OFREE = 10,            // output warps copied O out of tensor memory (256 arrivals)
    B_KQ = 11,               // 3: conv'd [k;q] rows and vectors of buffer i ready (1 arrival)
    B_VR = 14,               // 2: conv'd v rows ready (1 arrival)
    B_TPR = 16,              // 2: T / P images ready (1 arrival)
    B_GPFREE = 18;           // [G; P0] copied out of tensor memory (1 arrival)

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

// conv + SiLU of one bf16 channel pair: taps newest first, one bf16 rounding per tap (the first
// a bf16 product, then fused multiply-adds: deltanet.py:66-80); SiLU in fp32, rounded to bf16
__device__ __forceinline__ uint32_t conv_silu_pair(__nv_bfloat162 x0, __nv_bfloat162 x1, __nv_bfloat162 x2,
                                                  __nv_bfloat162 x3, const __nv_bfloat162 (&w)[4]) {
    __nv_bfloat162 acc = __hmul2(x0, w[3]);
    acc = __hfma2(x1, w[2], acc);
    acc = __hfma2(x2, w[1], acc);
    acc = __hfma2(x3, w[0], acc);
    const float ca = __low2float(acc), cb = __high2float(acc);
    return bf2_bits(__fdividef(ca, 1.0f + __expf(-ca)), __fdividef(cb, 1.0f + __expf(-cb)));
}
__device__ __forceinline__ __nv_bfloat162 as_bf2(uint32_t u) { return *reinterpret_cast<__nv_bfloat162*>(&u); }
