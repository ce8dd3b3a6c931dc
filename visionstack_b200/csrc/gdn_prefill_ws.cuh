// Workspace of the two-kernel chunked prefill (gdn_prefill_prep.cu writes it,
// gdn_prefill_seq.cu reads it).  Every region starts 1024-byte aligned.
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace gdn {

struct PrefillWs {
    void* qkv;    // bf16 [B][tp_len][conv_dim]: conv + SiLU outputs (tokens >= T are 0)
    float* nrm;   // [B][Hk][nc][2][64]: rq, rk of each chunk's tokens
    float* gate;  // [B][Hv][nc][2][64]: beta, gamma (cumulative log decay within the chunk)
    float* tp;    // [B][Hv][nc][2][64*64]: T = (I + A)^-1 image, P image (tf32, K-major, swizzled)
    float* hs;    // [n_hs][d][d]: recurrent state handed between the sequential kernel's CTAs
    int* hflag;   // [n_hs]: hand-off flags (zeroed by the launcher every call)
    int n_hs;     // hand-off slots: 0, or the SM count when there are more chains than SMs
    int nc;       // chunks of 64 tokens
    int tp_len;   // nc * 64
};

// Byte offsets of the six regions for one call (n_hs hand-off slots); returns the total size.
inline size_t prefill_ws_layout(int B, int T, int Hk, int Hv, int d, int n_hs, size_t off[6]) {
    auto up = [](size_t x) { return (x + 1023) & ~(size_t)1023; };
    const size_t nc = (size_t)(T + 63) / 64, tp_len = nc * 64;
    const size_t conv_dim = 2 * (size_t)Hk * d + (size_t)Hv * d;
    off[0] = 0;
    off[1] = up(off[0] + (size_t)B * tp_len * conv_dim * 2);
    off[2] = up(off[1] + (size_t)B * Hk * nc * 128 * 4);
    off[3] = up(off[2] + (size_t)B * Hv * nc * 128 * 4);
    off[4] = up(off[3] + (size_t)B * Hv * nc * 2 * 64 * 64 * 4);
    off[5] = up(off[4] + (size_t)n_hs * d * d * 4);
    return up(off[5] + (size_t)n_hs * 4);
}

// Hand-off slots for `chains` (batch, value head) chains on a device with `sms` SMs: the
// sequential kernel splits chains across CTAs (one CTA per SM) only when there are more chains
// than SMs.
inline int prefill_handoff_slots(int chains, int sms) { return sms > 0 && chains > sms ? sms : 0; }

}  // namespace gdn
