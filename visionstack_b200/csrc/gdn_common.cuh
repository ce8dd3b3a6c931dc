// Shared device helpers of the Gated DeltaNet kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

// Activation dtype traits.  The reference computes every elementwise op of a
// bf16 model in float and rounds the result to bf16 (PyTorch "opmath"); round()
// reproduces that rounding point, ld()/st() move one element.
template <typename T>
struct Act;

template <>
struct Act<float> {
    static __device__ __forceinline__ float ld(const float* p) { return *p; }
    static __device__ __forceinline__ float ldg(const float* p) { return __ldg(p); }
    static __device__ __forceinline__ void st(float* p, float x) { *p = x; }
    static __device__ __forceinline__ float round(float x) { return x; }
};

template <>
struct Act<__nv_bfloat16> {
    static __device__ __forceinline__ float ld(const __nv_bfloat16* p) { return __bfloat162float(*p); }
    static __device__ __forceinline__ float ldg(const __nv_bfloat16* p) { return __bfloat162float(__ldg(p)); }
    static __device__ __forceinline__ void st(__nv_bfloat16* p, float x) { *p = __float2bfloat16_rn(x); }
    static __device__ __forceinline__ float round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
};

// Nearest bf16 (ties to even) of a finite fp32 value, as fp32, in integer
// arithmetic (the same value as __float2bfloat16_rn, without the conversion
// pipe): add 0x7FFF plus the lowest kept bit, clear the low 16 bits.
__device__ __forceinline__ float bf16_round_alu(float x) {
    const uint32_t u = __float_as_uint(x);
    return __uint_as_float((u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u);
}
// The bf16 bit pattern of a value already rounded by bf16_round_alu.
__device__ __forceinline__ uint16_t bf16_bits(float rounded) { return (uint16_t)(__float_as_uint(rounded) >> 16); }

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }
// torch.nn.functional.softplus(beta=1, threshold=20)
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Sum over the 16 lanes that share (lane / 16).
__device__ __forceinline__ float half_warp_sum(float v) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Causal depthwise conv tap accumulation in the reference's order
// (deltanet.py:66-80): newest tap first, then older taps one at a time, with a
// rounding to the compute dtype after every tap.  win[j] is the raw input j
// positions back (win[0] = current token); taps with j > valid are absent
// (no previous conv state) and skipped, as the reference skips them.
template <typename TA>
__device__ __forceinline__ float conv_taps(const float* win, const float* w, int K, int valid) {
    float acc = Act<TA>::round(win[0] * w[K - 1]);
    for (int j = 1; j < K; ++j) {
        if (j > valid) break;
        acc = Act<TA>::round(fmaf(win[j], w[K - 1 - j], acc));
    }
    return acc;
}

// The same accumulation for the 4-tap conv with the window in registers
// (x0 = current token, x3 = three tokens back); `valid` as in conv_taps.
template <typename TA>
__device__ __forceinline__ float conv4_taps(float x0, float x1, float x2, float x3, float w0, float w1, float w2,
                                            float w3, int valid) {
    float acc = Act<TA>::round(x0 * w3);
    if (valid >= 1) acc = Act<TA>::round(fmaf(x1, w2, acc));
    if (valid >= 2) acc = Act<TA>::round(fmaf(x2, w1, acc));
    if (valid >= 3) acc = Act<TA>::round(fmaf(x3, w0, acc));
    return acc;
}

}  // namespace gdn
