// Kernel parameter blocks and launcher declarations of the Gated DeltaNet
// kernels.  The C ABI (gdn_capi.cu) validates arguments and fills these.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gdn_b200.h"
#include "gdn_prefill_ws.cuh"

namespace gdn {

// Checkpoints of one call, restricted to local offsets in 1..T and sorted by
// offset: slot[i] is the caller's checkpoint index (the output slot) of off[i].
struct CkptList {
    int n;
    int off[GDN_MAX_CHECKPOINTS];
    int slot[GDN_MAX_CHECKPOINTS];
};

struct MixParams {
    int B, T, Hk, Hv, K;
    float eps;      // gated-norm epsilon
    float q_scale;  // head_k_dim ** -0.5 rounded to float, as torch does
    int use_l2;     // split mode: apply the q/k L2 norm
    // fused-mixer inputs
    const void* mixed;
    long long ms_b, ms_t;
    const void* z;
    long long zs_b, zs_t;
    const void* a;
    const void* b;
    long long as_b, as_t;
    const void* convw;
    const float* A_log;
    const float* dt_bias;
    const void* normw;
    const void* cs_in;
    void* cs_out;
    // split-mode inputs ([B, T, H, d] / [B, T, H], contiguous)
    const void* q;
    const void* k;
    const void* v;
    const void* g;
    const void* beta;
    // state and outputs
    const float* S_in;
    float* S_out;
    void* out;
    float* S_ckpt;    // [n_slots, B, Hv, dk, dv]
    void* cs_ckpt;    // [n_slots, B, conv_dim, K-1]
    // Per-row state slots (gdn_mixer_verify_slots): when set, S_in / S_ckpt
    // and cs_in / cs_ckpt are the same pools [n_slots, B, ...]; row b reads
    // pool slot slot_table[b][0] and checkpoint i goes to pool slot
    // slot_table[b][ck.slot[i]].
    const int* slot_table;  // [B, n_slots]
    int n_slots;
};

// dtype: GDN_DTYPE_*; mixer: fused conv/gates/norm (true) or split q/k/v (false).
cudaError_t launch_decode(const MixParams& p, const CkptList& ck, int dk, int dv, int dtype, bool mixer,
                          cudaStream_t s, bool* supported);
cudaError_t launch_decode_tma(const MixParams& p, const CkptList& ck, int d, int dtype, cudaStream_t s,
                              bool* supported);
unsigned int decode_tma_device_error(bool clear);
cudaError_t launch_accept_slots(const int* accepted, int* table, int B, int n_slots, int T, cudaStream_t s);
unsigned int slots_device_error(bool clear);
cudaError_t launch_umma_selftest(int mode, const float* A, const float* B, float* D, cudaStream_t s);
unsigned int umma_device_error(bool clear);
cudaError_t launch_expired_wait_selftest(int kind, int* flag, cudaStream_t s);
// single-token grouped-query attention over a fixed-capacity KV buffer (stack_attn_decode.cu)
struct AttnDecodeArgs {
    const void* q;  // [batch][kv_heads * groups][head_dim] bf16
    const void* k;  // [batch][kv_heads][capacity][head_dim] bf16
    const void* v;
    void* out;              // like q
    const long long* pos;   // device: index of the last valid key
    int batch, kv_heads, groups, head_dim, capacity;
    int splits, span;       // key ranges of span keys (a multiple of 32)
    float qscale;           // softmax scale * log2(e)
    float* part_o;          // [batch][kv_heads][splits][groups][head_dim]
    float* part_ml;         // [batch][kv_heads][splits][groups][2]
};
cudaError_t launch_attn_decode(const AttnDecodeArgs& a, cudaStream_t st);
cudaError_t launch_prefill_tc(const MixParams& p, const CkptList& ck, int d, int dtype, cudaStream_t s,
                              bool* supported);
unsigned int prefill_tc_device_error(bool clear);
// two-kernel chunked prefill: parallel preparation pass, then the sequential pass
bool prefill_prep_supported(const MixParams& p, int d, int dtype);
cudaError_t launch_prefill_prep(const MixParams& p, const PrefillWs& ws, cudaStream_t s);
unsigned int prefill_prep_device_error(bool clear);
cudaError_t launch_prefill_seq(const MixParams& p, const CkptList& ck, const PrefillWs& ws, cudaStream_t s);
unsigned int prefill_seq_device_error(bool clear);
// single fused chunked prefill (gdn_prefill_fused.cu): workspace = n_hs hand-off states + flags
size_t prefill_fused_ws_layout(int n_hs, size_t off[2]);
cudaError_t launch_prefill_fused(const MixParams& p, const CkptList& ck, float* hs, int* hflag, int n_hs,
                                 cudaStream_t s);
unsigned int prefill_fused_device_error(bool clear);
// address of the fixed prefill scratch on the current device (looked up once per device)
cudaError_t static_prefill_scratch(void** addr);
// one-shot all-reduce over NVLink peer memory (gdn_peer_allreduce.cu)
constexpr int PEER_MAX_RANKS = 8;
struct PeerAllReduceArgs {
    const void* in;  // local partial, bf16 [n]
    void* out;       // sum, bf16 [n] (may be `in`)
    long long n;     // elements, a multiple of 8
    long long cap;   // elements per staging slot
    int rank, world, nblocks;
    uint16_t* data[PEER_MAX_RANKS];  // every rank's staging slots [2][world][cap] (peer-mapped)
    int* flags[PEER_MAX_RANKS];      // every rank's flags [world][nblocks] (peer-mapped)
    int* counters;                   // this rank's epochs [nblocks]
};
cudaError_t launch_peer_allreduce(const PeerAllReduceArgs& a, cudaStream_t s);
unsigned int peer_allreduce_device_error(bool clear);
// fused elementwise steps of the stack's layers (stack_ops.cu), bf16
struct RmsNormArgs {
    const void* x;       // [rows] x [dim], row stride x_stride elements
    long long x_stride;
    const void* delta;   // optional residual added first (row stride delta_stride); NULL: none
    long long delta_stride;
    void* res;           // with delta: bf16(x + delta), row stride res_stride
    long long res_stride;
    const void* w;       // [dim] zero-centred weight (the norm multiplies by 1 + w)
    void* out;           // [rows] x [dim], row stride out_stride
    long long out_stride;
    long long rows;
    int dim;
    float eps;
};
cudaError_t launch_rms_norm_zc(const RmsNormArgs& a, cudaStream_t s);
cudaError_t launch_silu_mul(const void* gate, const void* up, void* out, long long n, cudaStream_t s);
struct QkRopeArgs {
    const void* qg;   // [B][T][H][2 hd]: query (first hd) and gate of each head
    const void* k;    // [B][T][KVH][hd]
    const void* qw;   // [hd] zero-centred q-norm weight
    const void* kw;   // [hd] k-norm weight
    const void* cos;  // [B][T][rot]
    const void* sin;
    void* q_out;      // [B][H][T][hd]
    void* k_out;      // [B][KVH][T][hd]
    int B, T, H, KVH, hd, rot;
    float eps;
};
cudaError_t launch_qk_norm_rope(const QkRopeArgs& a, cudaStream_t s);
struct GateOutArgs {
    const void* o;                // attention output [B][H][T][hd], strides in elements (last dim contiguous)
    long long o_sb, o_sh, o_st;
    const void* qg;               // [B][T][H][2 hd] (the gate is the second hd of each head)
    void* out;                    // [B][T][H hd]
    int B, T, H, hd;
};
cudaError_t launch_gate_out(const GateOutArgs& a, cudaStream_t s);
cudaError_t launch_prefill(const MixParams& p, const CkptList& ck, int d, int dtype, bool mixer,
                           cudaStream_t s, bool* supported);
cudaError_t launch_conv1d(int B, int C, int T, int K, int dtype, const void* x, const void* w,
                          const void* state_in, void* out, void* state_out, int silu, cudaStream_t s);
// functional boundary (gdn_functional.cu): unit lower triangular solve and the gated RMSNorm
cudaError_t launch_trisolve(const float* ut, const float* rhs, float* out, long long batch, int n, int m,
                            cudaStream_t s);
cudaError_t launch_rms_norm_gated(const void* x, const void* gate, const void* w, void* out, long long rows, int dim,
                                  float eps, int x_dtype, int gate_dtype, int w_dtype, cudaStream_t s);

}  // namespace gdn
