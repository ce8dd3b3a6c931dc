// Conv-window copies shared by the token-by-token and chunked kernels.
#pragma once

#include "gdn_common.cuh"
#include "gdn_kernels.cuh"

namespace gdn {

// Copy the raw conv windows (final conv state and conv checkpoints) of the
// channels this CTA owns.  value head h owns its dv value channels; the first
// value head of each GQA group also owns the q/k channels of its key head.
// Pure copies, bit-exact (deltanet.py:24-38, 479-487).
template <typename TA, int DK, int DV, int NT>
__device__ void write_conv_windows(const MixParams& p, const CkptList& ck, int b, int h, int kh, int rep) {
    const int L = p.K - 1;
    if (L <= 0) return;
    const int conv_dim = 2 * p.Hk * DK + p.Hv * DV;
    const bool own_qk = (h % rep) == 0;
    const int nch = (own_qk ? 2 * DK : 0) + DV;
    const TA* mixed = static_cast<const TA*>(p.mixed);
    const TA* cs_in = static_cast<const TA*>(p.cs_in);
    const size_t per_b = (size_t)conv_dim * L;
    for (int w = -1; w < ck.n; ++w) {
        int off;
        TA* dst;
        if (w < 0) {
            if (!p.cs_out) continue;
            off = p.T;
            dst = static_cast<TA*>(p.cs_out) + (size_t)b * per_b;
        } else {
            if (!p.cs_ckpt) break;
            off = ck.off[w];
            dst = static_cast<TA*>(p.cs_ckpt) + ((size_t)ck.slot[w] * p.B + b) * per_b;
        }
        for (int c = threadIdx.x; c < nch * L; c += NT) {
            const int ci = c / L, i = c - ci * L;
            int gc;
            if (own_qk) {
                gc = ci < DK ? kh * DK + ci
                             : (ci < 2 * DK ? p.Hk * DK + kh * DK + (ci - DK) : 2 * p.Hk * DK + h * DV + (ci - 2 * DK));
            } else {
                gc = 2 * p.Hk * DK + h * DV + ci;
            }
            const int pos = off - L + i;
            TA val;
            if (pos >= 0) {
                val = mixed[(size_t)b * p.ms_b + (size_t)pos * p.ms_t + gc];
            } else if (cs_in) {
                val = cs_in[((size_t)b * conv_dim + gc) * L + (L + pos)];
            } else {
                val = TA(0.0f);
            }
            dst[(size_t)gc * L + i] = val;
        }
    }
}

}  // namespace gdn
