// 5th-generation tensor core (tcgen05 / UMMA) helpers for sm_100a: tensor
// memory allocation, shared-memory matrix descriptors for 128-byte swizzled
// canonical layouts, the tf32 MMA, commit, and tensor-memory loads / stores.
//
// Operand layouts (fp32 / tf32 elements, 128-byte swizzle):
//  * K-major  [rows][k]  : the k axis is cut into 32-element (128-byte) atoms;
//    atom a holds every row's 128 bytes: byte(row, k) =
//      (k/32)*rows*128 + (row/8)*1024 + (row%8)*128 + ((k%32/4) ^ (row%8))*16 + (k%4)*4
//    descriptor: SBO = 1024 (8-row groups), LBO unused; one MMA k-step of 8
//    elements (32 bytes) advances the start address by 32 bytes inside an atom.
//    (canonical SWIZZLE_128B layout, 16-byte swizzle unit over 8-row groups)
//  * MN-major [k][mn]    : 32-bit operands use the SWIZZLE_128B_BASE32B layout
//    (the only MN-major layout the tf32 MMA accepts): the mn axis is cut into
//    32-element atoms, each atom holds every k row's 128 bytes, and the 32-byte
//    chunks of a row are swizzled over 4-row groups: byte(k, mn) =
//      (mn/32)*krows*128 + (k/4)*512 + (k%4)*128 + ((mn%32/8) ^ (k%4))*32 + (mn%8)*4
//    descriptor: LBO = krows*128 (next mn atom), SBO = 512 (next 4 k rows);
//    one MMA k-step of 8 rows advances the start address by 1024 bytes.
// Descriptor version 1, base offset 0: every operand region starts 1024-byte
// aligned.
//
// 16-bit (bf16) operands, 128-byte swizzle (the layout a TMA copy with
// CU_TENSOR_MAP_SWIZZLE_128B writes for a box 64 elements wide):
//  * K-major  [rows][k]  : atom = 64 k-elements (128 bytes) of every row:
//      byte(row, k) = (k/64)*rows*128 + (row/8)*1024 + (row%8)*128 +
//                     ((k%64/8) ^ (row%8))*16 + (k%8)*2
//    descriptor as for tf32 (SBO = 1024); one MMA k-step of 16 elements is
//    again 32 bytes inside an atom.
//  * MN-major [k][mn]    : the same bytes read the other way: atom = 64
//    mn-elements of 8 k rows; descriptor LBO = stride between 64-element mn
//    atoms, SBO = 1024 (next 8 k rows); a k-step of 16 rows is 2048 bytes.
//  * in tensor memory (A of kind::f16): row m = lane m, column c holds the
//    pair k = 2c (low half) and 2c + 1 (high half).
#pragma once

#include <stdint.h>

#include "gdn_async.cuh"

namespace gdn {
namespace umma {

__host__ __device__ constexpr uint32_t kmajor_off(int row, int k, int rows) {
    return (uint32_t)((k >> 5) * rows * 128 + (row >> 3) * 1024 + (row & 7) * 128 +
                      ((((k & 31) >> 2) ^ (row & 7)) << 4) + (k & 3) * 4);
}

__host__ __device__ constexpr uint32_t kmajor_off16(int row, int k, int rows) {
    return (uint32_t)((k >> 6) * rows * 128 + (row >> 3) * 1024 + (row & 7) * 128 +
                      ((((k & 63) >> 3) ^ (row & 7)) << 4) + (k & 7) * 2);
}
__host__ __device__ constexpr uint32_t mnmajor_off16(int k, int mn, uint32_t mn_atom_stride) {
    return (uint32_t)((mn >> 6) * mn_atom_stride + (k >> 3) * 1024 + (k & 7) * 128 +
                      ((((mn & 63) >> 3) ^ (k & 7)) << 4) + (mn & 7) * 2);
}

__host__ __device__ constexpr uint32_t mnmajor_off(int k, int mn, int krows) {
    return (uint32_t)((mn >> 5) * krows * 128 + (k >> 2) * 512 + (k & 3) * 128 +
                      ((((mn & 31) >> 3) ^ (k & 3)) << 5) + (mn & 7) * 4);
}

// Round an fp32 value to tf32 (10 explicit mantissa bits), nearest with ties
// away from zero.  The tensor core drops the low 13 bits of fp32 operands, so
// operands written through this rounding carry half the conversion error.
// Integer arithmetic on the bit pattern (add half of the dropped unit, clear
// the dropped bits; sign-magnitude makes the tie go away from zero): two ALU
// operations instead of a conversion-pipe instruction.  Same result as
// cvt.rna.tf32.f32 for every finite input.
__device__ __forceinline__ float tf32_rna(float x) {
    return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}
__device__ __forceinline__ float4 tf32_rna4(float4 v) {
    return make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
}

constexpr uint32_t LAYOUT_SW128 = 2;         // K-major operands
constexpr uint32_t LAYOUT_SW128_BASE32 = 1;  // MN-major 32-bit operands

// Shared-memory matrix descriptor, version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1u << 46;  // descriptor version (sm_100)
    d |= (uint64_t)(layout & 7u) << 61;
    return d;
}

// Descriptor of k-step kk (8 tf32 elements) of a K-major operand with `rows` rows.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t base, int rows, int kk) {
    return smem_desc(base + (uint32_t)((kk >> 2) * rows * 128 + (kk & 3) * 32), 16, 1024, LAYOUT_SW128);
}

// Descriptor of k-step kk (8 k rows) of an MN-major operand with `krows` k rows.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t base, int krows, int kk) {
    return smem_desc(base + (uint32_t)(kk * 1024), (uint32_t)(krows * 128), 512, LAYOUT_SW128_BASE32);
}

// Byte offset of k-step kk inside a K-major operand with `rows` rows, and of an
// MN-major operand: added (>> 4) to the descriptor's start-address field, so a
// loop over k-steps needs one descriptor and an add per step.
__host__ __device__ constexpr uint32_t kmajor_kstep(int kk, int rows) {
    return (uint32_t)((kk >> 2) * rows * 128 + (kk & 3) * 32);
}
__host__ __device__ constexpr uint32_t mnmajor_kstep(int kk) { return (uint32_t)(kk * 1024); }
// Descriptors of a K-major / MN-major operand at k-step 0 (start of a k loop).
__device__ __forceinline__ uint64_t desc_kmajor0(uint32_t base) { return smem_desc(base, 16, 1024, LAYOUT_SW128); }
__device__ __forceinline__ uint64_t desc_mnmajor0(uint32_t base, int krows) {
    return smem_desc(base, (uint32_t)(krows * 128), 512, LAYOUT_SW128_BASE32);
}
// desc0 advanced by `bytes` (the start address field is 16-byte units in the low 14 bits;
// operands here lie below 256 KB of shared memory, so the field cannot overflow).
__device__ __forceinline__ uint64_t desc_add(uint64_t desc0, uint32_t bytes) { return desc0 + (bytes >> 4); }

// MN-major 16-bit operand at k-step 0; a k-step (16 rows) adds 2048 bytes.
__device__ __forceinline__ uint64_t desc_mnmajor16_0(uint32_t base, uint32_t mn_atom_stride) {
    return smem_desc(base, mn_atom_stride, 1024, LAYOUT_SW128);
}
__host__ __device__ constexpr uint32_t mnmajor16_kstep(int kk) { return (uint32_t)(kk * 2048); }

// Instruction descriptor of kind::f16 with bf16 operands and fp32 accumulation.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int a_mn, int b_mn) {
    return (1u << 4)             // D format f32
           | (1u << 7)           // A format bf16
           | (1u << 10)          // B format bf16
           | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

// Instruction descriptor of kind::tf32 with fp32 accumulation.
// a_mn / b_mn: operand is MN-major (1) or K-major (0).
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N, int a_mn, int b_mn) {
    return (1u << 4)             // D format f32
           | (2u << 7)           // A format tf32
           | (2u << 10)          // B format tf32
           | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

// ---- tensor memory ----
// Allocation / deallocation are warp-wide (.sync.aligned): call from one full warp.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], issued by one thread.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 with bf16 operands, issued by one thread.
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]: A is read from tensor memory (row m of
// A = lane m, element k = column k for 32-bit operands; always K-major).
__device__ __forceinline__ void mma_tf32_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

// mma_tf32_ta issued from a whole converged warp: elect.sync picks one lane
// (the lowest active one, so the same lane on every call) to issue it.  The
// warp-uniform operands stay in uniform registers, which shortens the issue
// of short (N <= 64) MMAs; pair with mma_commit_elect.
__device__ __forceinline__ void mma_tf32_ta_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                  uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void mma_commit_elect(uint32_t bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(bar)
        : "memory");
}

// kind::f16 with bf16 operands, A from tensor memory (packed pairs), from one
// thread / from a converged warp through elect.sync.
__device__ __forceinline__ void mma_bf16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void mma_bf16_ta_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                  uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

// Arrive once on the mbarrier when every MMA issued so far by this thread completes.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// 32 consecutive fp32 columns of this thread's lane (32x32b shape, warp-wide).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

// 8 consecutive 32-bit columns of this thread's lane (32x32b shape, warp-wide).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
// 16 consecutive 32-bit columns of this thread's lane (32x32b shape, warp-wide).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// TMEM address of (lane, column): lane in bits 31..16, column in 15..0.
__device__ __forceinline__ uint32_t tmem_addr(uint32_t base, int lane, int col) {
    return base + ((uint32_t)lane << 16) + (uint32_t)col;
}

}  // namespace umma
}  // namespace gdn
