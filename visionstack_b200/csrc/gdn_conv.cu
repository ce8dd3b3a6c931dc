// Stand-alone causal depthwise conv1d + SiLU in the reference's
// [batch, channels, seq_len] layout (functional boundary of
// _causal_conv1d_fn, deltanet.py:41-90).  One thread per (batch, channel)
// slides a kernel-wide window along the sequence; the new conv state is the
// raw input of the last kernel-1 positions (deltanet.py:24-38).
#include "gdn_common.cuh"
#include "gdn_kernels.cuh"

namespace gdn {

template <typename TA>
__global__ void conv1d_kernel(int B, int Cn, int T, int K, const TA* __restrict__ x, const TA* __restrict__ w,
                              const TA* __restrict__ st_in, TA* __restrict__ out, TA* __restrict__ st_out,
                              int apply_silu) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= B * Cn) return;
    const int L = K - 1;
    const TA* xr = x + (size_t)idx * T;
    float wt[4] = {0.f, 0.f, 0.f, 0.f};
    float hist[3] = {0.f, 0.f, 0.f};
    const int c = idx % Cn;
    for (int j = 0; j < K; ++j) wt[j] = Act<TA>::ldg(w + (size_t)c * K + j);
    if (st_in)
        for (int j = 0; j < L; ++j) hist[j] = Act<TA>::ld(st_in + (size_t)idx * L + (L - 1 - j));
    for (int t = 0; t < T; ++t) {
        const float xv = Act<TA>::ld(xr + t);
        const float win[4] = {xv, hist[0], hist[1], hist[2]};
        const int valid = st_in ? L : (t < L ? t : L);
        float acc = conv_taps<TA>(win, wt, K, valid);
        if (apply_silu) acc = Act<TA>::round(silu_f(acc));
        Act<TA>::st(out + (size_t)idx * T + t, acc);
        hist[2] = hist[1];
        hist[1] = hist[0];
        hist[0] = xv;
    }
    if (st_out) {
        for (int i = 0; i < L; ++i) {
            const int pos = T - L + i;
            TA v;
            if (pos >= 0) v = xr[pos];
            else if (st_in) v = st_in[(size_t)idx * L + (L + pos)];
            else v = TA(0.0f);
            st_out[(size_t)idx * L + i] = v;
        }
    }
}

cudaError_t launch_conv1d(int B, int Cn, int T, int K, int dtype, const void* x, const void* w, const void* state_in,
                          void* out, void* state_out, int silu, cudaStream_t s) {
    const int n = B * Cn, nt = 128, nb = (n + nt - 1) / nt;
    if (dtype == GDN_DTYPE_BF16) {
        using T16 = __nv_bfloat16;
        conv1d_kernel<T16><<<nb, nt, 0, s>>>(B, Cn, T, K, (const T16*)x, (const T16*)w, (const T16*)state_in,
                                             (T16*)out, (T16*)state_out, silu);
    } else {
        conv1d_kernel<float><<<nb, nt, 0, s>>>(B, Cn, T, K, (const float*)x, (const float*)w,
                                               (const float*)state_in, (float*)out, (float*)state_out, silu);
    }
    return cudaGetLastError();
}

}  // namespace gdn
