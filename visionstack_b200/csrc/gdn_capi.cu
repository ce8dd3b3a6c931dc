// C ABI of the Gated DeltaNet kernels: host-side validation, checkpoint
// bookkeeping, dispatch.  Every entry returns an int32 status and never lets a
// bad argument reach the device.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <utility>
#include <vector>

#include "gdn_kernels.cuh"

namespace {

thread_local char g_err[512] = {0};

int32_t fail(int32_t code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

int32_t ok() {
    g_err[0] = '\0';
    return GDN_OK;
}

int32_t cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return ok();
    return fail(GDN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool aligned_elem(const void* p, int dtype) {
    const uintptr_t m = dtype == GDN_DTYPE_BF16 ? 1u : 3u;
    return (reinterpret_cast<uintptr_t>(p) & m) == 0;
}

// Keep offsets in 1..T, sort by offset (stable in the caller's slot order),
// reject duplicates (the reference keys checkpoints by position in a dict).
int32_t build_ckpts(int n, const int32_t* offsets, int T, gdn::CkptList* ck) {
    ck->n = 0;
    if (n < 0 || n > GDN_MAX_CHECKPOINTS)
        return fail(GDN_ERR_TOO_MANY_CHECKPOINTS, "num_checkpoints %d outside 0..%d", n, GDN_MAX_CHECKPOINTS);
    if (n > 0 && !offsets) return fail(GDN_ERR_INVALID_ARG, "checkpoint_offsets is NULL");
    std::vector<std::pair<int, int>> v;
    for (int i = 0; i < n; ++i)
        if (offsets[i] >= 1 && offsets[i] <= T) v.emplace_back(offsets[i], i);
    std::stable_sort(v.begin(), v.end(),
                     [](const std::pair<int, int>& a, const std::pair<int, int>& b) { return a.first < b.first; });
    for (size_t i = 1; i < v.size(); ++i)
        if (v[i].first == v[i - 1].first)
            return fail(GDN_ERR_INVALID_ARG, "duplicate checkpoint offset %d", v[i].first);
    ck->n = (int)v.size();
    for (size_t i = 0; i < v.size(); ++i) {
        ck->off[i] = v[i].first;
        ck->slot[i] = v[i].second;
    }
    return GDN_OK;
}

bool supported_head_dims(int dk, int dv) { return dk == dv && (dk == 32 || dk == 64 || dk == 128); }

int32_t validate_mixer(const gdn_mixer_args* a, gdn::MixParams* p, gdn::CkptList* ck) {
    if (!a) return fail(GDN_ERR_INVALID_ARG, "args is NULL");
    if (a->batch < 1 || a->seq_len < 1 || a->num_k_heads < 1 || a->num_v_heads < 1)
        return fail(GDN_ERR_INVALID_ARG, "batch, seq_len and head counts must be >= 1");
    if (a->num_v_heads % a->num_k_heads != 0)
        return fail(GDN_ERR_INVALID_ARG, "num_v_heads (%d) must be a multiple of num_k_heads (%d)", a->num_v_heads,
                    a->num_k_heads);
    if (!supported_head_dims(a->head_k_dim, a->head_v_dim))
        return fail(GDN_ERR_UNSUPPORTED, "head dims (%d, %d) not built: need dk == dv in {32, 64, 128}",
                    a->head_k_dim, a->head_v_dim);
    if (a->conv_kernel < 1 || a->conv_kernel > 4)
        return fail(GDN_ERR_UNSUPPORTED, "conv_kernel %d not in 1..4", a->conv_kernel);
    if (a->act_dtype != GDN_DTYPE_F32 && a->act_dtype != GDN_DTYPE_BF16)
        return fail(GDN_ERR_UNSUPPORTED, "act_dtype %d", a->act_dtype);
    if (!(a->norm_eps >= 0.0f)) return fail(GDN_ERR_INVALID_ARG, "norm_eps must be >= 0");
    if (a->flags & ~(GDN_FLAG_REGISTER_KERNEL | GDN_FLAG_CUDA_CORE_PREFILL | GDN_FLAG_PREP_IN_KERNEL_PREFILL))
        return fail(GDN_ERR_INVALID_ARG, "unknown flags 0x%x", a->flags);
    if (!a->mixed_qkv || !a->z || !a->a || !a->b || !a->conv_weight || !a->A_log || !a->dt_bias ||
        !a->norm_weight || !a->out)
        return fail(GDN_ERR_INVALID_ARG, "a required pointer is NULL");
    const int64_t dk = a->head_k_dim, dv = a->head_v_dim;
    const int64_t conv_dim = 2 * a->num_k_heads * dk + a->num_v_heads * dv;
    const int64_t vdim = a->num_v_heads * dv;
    const int64_t T = a->seq_len;
    if (a->mixed_stride_t < conv_dim || a->mixed_stride_b < (T - 1) * a->mixed_stride_t + conv_dim)
        return fail(GDN_ERR_INVALID_ARG, "mixed_qkv strides (%lld, %lld) too small for conv_dim %lld",
                    (long long)a->mixed_stride_b, (long long)a->mixed_stride_t, (long long)conv_dim);
    if (a->z_stride_t < vdim || a->z_stride_b < (T - 1) * a->z_stride_t + vdim)
        return fail(GDN_ERR_INVALID_ARG, "z strides too small");
    if (a->ab_stride_t < a->num_v_heads || a->ab_stride_b < (T - 1) * a->ab_stride_t + a->num_v_heads)
        return fail(GDN_ERR_INVALID_ARG, "a/b strides too small");
    const void* elem_ptrs[] = {a->mixed_qkv, a->z, a->a, a->b, a->conv_weight, a->norm_weight, a->out,
                               a->conv_state_in, a->conv_state_out, a->conv_checkpoints};
    for (const void* ptr : elem_ptrs)
        if (ptr && !aligned_elem(ptr, a->act_dtype)) return fail(GDN_ERR_ALIGNMENT, "misaligned activation pointer");
    const void* f4_ptrs[] = {a->state_in, a->state_out, a->state_checkpoints};
    for (const void* ptr : f4_ptrs)
        if (ptr && !aligned16(ptr)) return fail(GDN_ERR_ALIGNMENT, "state pointers must be 16-byte aligned");
    if (!aligned_elem(a->A_log, GDN_DTYPE_F32) || !aligned_elem(a->dt_bias, GDN_DTYPE_F32))
        return fail(GDN_ERR_ALIGNMENT, "A_log / dt_bias must be 4-byte aligned");
    if (a->conv_state_in && a->conv_state_in == a->conv_state_out)
        return fail(GDN_ERR_INVALID_ARG, "conv_state_out must not alias conv_state_in");
    int32_t st = build_ckpts(a->num_checkpoints, a->checkpoint_offsets, a->seq_len, ck);
    if (st != GDN_OK) return st;
    if (ck->n > 0 && (!a->state_checkpoints || !a->conv_checkpoints))
        return fail(GDN_ERR_INVALID_ARG, "checkpoints requested but state_checkpoints/conv_checkpoints is NULL");

    std::memset(p, 0, sizeof(*p));
    p->B = a->batch;
    p->T = a->seq_len;
    p->Hk = a->num_k_heads;
    p->Hv = a->num_v_heads;
    p->K = a->conv_kernel;
    p->eps = a->norm_eps;
    p->q_scale = (float)std::pow((double)dk, -0.5);
    p->use_l2 = 1;
    p->mixed = a->mixed_qkv;
    p->ms_b = a->mixed_stride_b;
    p->ms_t = a->mixed_stride_t;
    p->z = a->z;
    p->zs_b = a->z_stride_b;
    p->zs_t = a->z_stride_t;
    p->a = a->a;
    p->b = a->b;
    p->as_b = a->ab_stride_b;
    p->as_t = a->ab_stride_t;
    p->convw = a->conv_weight;
    p->A_log = a->A_log;
    p->dt_bias = a->dt_bias;
    p->normw = a->norm_weight;
    p->cs_in = a->conv_state_in;
    p->cs_out = a->conv_state_out;
    p->S_in = a->state_in;
    p->S_out = a->state_out;
    p->out = a->out;
    p->S_ckpt = a->state_checkpoints;
    p->cs_ckpt = a->conv_checkpoints;
    return GDN_OK;
}

}  // namespace

extern "C" {

int32_t gdn_version(void) { return GDN_ABI_VERSION; }

const char* gdn_last_error_string(void) { return g_err; }

int32_t gdn_mixer_decode(const gdn_mixer_args* args, void* stream) {
    gdn::CkptList ck;
    gdn::MixParams p;
    int32_t st = validate_mixer(args, &p, &ck);
    if (st != GDN_OK) return st;
    if (args->seq_len > GDN_MAX_DECODE_TOKENS)
        return fail(GDN_ERR_INVALID_ARG, "seq_len %d exceeds the token-by-token limit %d", args->seq_len,
                    GDN_MAX_DECODE_TOKENS);
    bool supported = false;
    cudaError_t e = cudaSuccess;
    if (!(args->flags & GDN_FLAG_REGISTER_KERNEL))
        e = gdn::launch_decode_tma(p, ck, args->head_k_dim, args->act_dtype, static_cast<cudaStream_t>(stream),
                                   &supported);
    if (!supported)
        e = gdn::launch_decode(p, ck, args->head_k_dim, args->head_v_dim, args->act_dtype, true,
                               static_cast<cudaStream_t>(stream), &supported);
    if (!supported) return fail(GDN_ERR_UNSUPPORTED, "no token-by-token kernel for these head dims");
    return cuda_status(e, "gdn_mixer_decode launch");
}

int32_t gdn_mixer_verify_slots(const gdn_mixer_args* args, const int32_t* slot_table, int32_t num_slots,
                               void* stream) {
    if (!args) return fail(GDN_ERR_INVALID_ARG, "args is NULL");
    if (!slot_table) return fail(GDN_ERR_INVALID_ARG, "slot_table is NULL");
    if ((reinterpret_cast<uintptr_t>(slot_table) & 3u) != 0) return fail(GDN_ERR_ALIGNMENT, "slot_table misaligned");
    if (args->seq_len < 1 || args->seq_len > GDN_MAX_DECODE_TOKENS)
        return fail(GDN_ERR_INVALID_ARG, "seq_len %d outside 1..%d", args->seq_len, GDN_MAX_DECODE_TOKENS);
    if (num_slots < args->seq_len + 1 || num_slots > GDN_MAX_DECODE_TOKENS + 1)
        return fail(GDN_ERR_INVALID_ARG, "num_slots %d outside seq_len + 1 (%d) .. %d", num_slots,
                    args->seq_len + 1, GDN_MAX_DECODE_TOKENS + 1);
    if (!args->state_in || !args->conv_state_in)
        return fail(GDN_ERR_INVALID_ARG, "state_in and conv_state_in (the slot pools) are required");
    if (args->state_out || args->conv_state_out || args->num_checkpoints || args->checkpoint_offsets ||
        args->state_checkpoints || args->conv_checkpoints)
        return fail(GDN_ERR_INVALID_ARG, "state_out, conv_state_out and checkpoint fields must be NULL / 0 "
                                         "with a slot table");
    if (args->flags & GDN_FLAG_REGISTER_KERNEL)
        return fail(GDN_ERR_UNSUPPORTED, "the slot table needs the pipelined kernel");
    gdn::CkptList ck;
    gdn::MixParams p;
    int32_t st = validate_mixer(args, &p, &ck);
    if (st != GDN_OK) return st;
    // every draft token is a checkpoint; checkpoint i (offset i + 1) goes to table column i + 1
    ck.n = args->seq_len;
    for (int i = 0; i < ck.n; ++i) {
        ck.off[i] = i + 1;
        ck.slot[i] = i + 1;
    }
    p.S_ckpt = const_cast<float*>(args->state_in);
    p.cs_ckpt = const_cast<void*>(args->conv_state_in);
    p.slot_table = slot_table;
    p.n_slots = num_slots;
    bool supported = false;
    cudaError_t e = gdn::launch_decode_tma(p, ck, args->head_k_dim, args->act_dtype,
                                           static_cast<cudaStream_t>(stream), &supported);
    if (!supported)
        return fail(GDN_ERR_UNSUPPORTED, "slot tables need 4-tap conv, head dim 64 or 128, 16-byte aligned inputs "
                                         "and bf16 activations (or seq_len 1)");
    return cuda_status(e, "gdn_mixer_verify_slots launch");
}

int32_t gdn_accept_slots(const int32_t* accepted, int32_t* slot_table, int32_t batch, int32_t num_slots,
                         int32_t seq_len, void* stream) {
    if (!accepted || !slot_table) return fail(GDN_ERR_INVALID_ARG, "a required pointer is NULL");
    if ((reinterpret_cast<uintptr_t>(accepted) & 3u) || (reinterpret_cast<uintptr_t>(slot_table) & 3u))
        return fail(GDN_ERR_ALIGNMENT, "accepted / slot_table misaligned");
    if (batch < 1) return fail(GDN_ERR_INVALID_ARG, "batch must be >= 1");
    if (seq_len < 1 || num_slots < seq_len + 1)
        return fail(GDN_ERR_INVALID_ARG, "need 1 <= seq_len < num_slots (got %d, %d)", seq_len, num_slots);
    return cuda_status(gdn::launch_accept_slots(accepted, slot_table, batch, num_slots, seq_len,
                                                static_cast<cudaStream_t>(stream)),
                       "gdn_accept_slots launch");
}

int32_t gdn_device_error(uint32_t* flags_out, int32_t clear) {
    if (!flags_out) return fail(GDN_ERR_INVALID_ARG, "flags_out is NULL");
    const unsigned int words[] = {gdn::decode_tma_device_error(clear != 0), gdn::umma_device_error(clear != 0),
                                  gdn::prefill_tc_device_error(clear != 0), gdn::slots_device_error(clear != 0),
                                  gdn::prefill_prep_device_error(clear != 0),
                                  gdn::prefill_seq_device_error(clear != 0),
                                  gdn::prefill_fused_device_error(clear != 0),
                                  gdn::peer_allreduce_device_error(clear != 0)};
    uint32_t all = 0;
    for (unsigned int w : words) {
        if (w == 0xFFFFFFFFu) return fail(GDN_ERR_CUDA, "could not read the device error word");
        all |= w;
    }
    *flags_out = all;
    return ok();
}

// Hand-off slots of the sequential prefill kernel on the current device (prefill_ws_layout).
static int handoff_slots(const gdn_mixer_args* args) {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    return gdn::prefill_handoff_slots(args->batch * args->num_v_heads, sms);
}

int64_t gdn_prefill_workspace_bytes(const gdn_mixer_args* args) {
    gdn::CkptList ck;
    gdn::MixParams p;
    const int32_t st = validate_mixer(args, &p, &ck);
    if (st != GDN_OK) return st;
    if ((args->flags & GDN_FLAG_CUDA_CORE_PREFILL) || !gdn::prefill_prep_supported(p, args->head_k_dim,
                                                                                 args->act_dtype))
        return 0;
    ok();
    if (!(args->flags & GDN_FLAG_PREP_IN_KERNEL_PREFILL)) {
        size_t off[6];
        return (int64_t)gdn::prefill_ws_layout(args->batch, args->seq_len, args->num_k_heads, args->num_v_heads,
                                               args->head_k_dim, handoff_slots(args), off);
    }
    const int n_hs = handoff_slots(args);
    size_t off[2];
    return n_hs > 0 ? (int64_t)gdn::prefill_fused_ws_layout(n_hs, off) : 0;
}

int32_t gdn_mixer_prefill_ws(const gdn_mixer_args* args, void* workspace, int64_t workspace_bytes, void* stream) {
    gdn::CkptList ck;
    gdn::MixParams p;
    int32_t st = validate_mixer(args, &p, &ck);
    if (st != GDN_OK) return st;
    if ((args->flags & GDN_FLAG_CUDA_CORE_PREFILL) || !gdn::prefill_prep_supported(p, args->head_k_dim,
                                                                                 args->act_dtype))
        return gdn_mixer_prefill(args, stream);  // needs no workspace
    if (args->flags & GDN_FLAG_PREP_IN_KERNEL_PREFILL) {
        // the single kernel: workspace only for the state hand-offs of split mode
        const int n_hs = handoff_slots(args);
        size_t off[2];
        const size_t need = n_hs > 0 ? gdn::prefill_fused_ws_layout(n_hs, off) : 0;
        if (need > 0) {
            if (!workspace || workspace_bytes < 0 || (size_t)workspace_bytes < need)
                return fail(GDN_ERR_INVALID_ARG, "workspace of %lld bytes needed (got %lld)", (long long)need,
                            (long long)workspace_bytes);
            if (!aligned16(workspace)) return fail(GDN_ERR_ALIGNMENT, "workspace must be 16-byte aligned");
        }
        unsigned char* base = static_cast<unsigned char*>(workspace);
        float* hs = need > 0 ? reinterpret_cast<float*>(base + off[0]) : nullptr;
        int* hflag = need > 0 ? reinterpret_cast<int*>(base + off[1]) : nullptr;
        const cudaError_t e =
            gdn::launch_prefill_fused(p, ck, hs, hflag, need > 0 ? n_hs : 0, static_cast<cudaStream_t>(stream));
        return cuda_status(e, "gdn_mixer_prefill_ws fused launch");
    }
    size_t off[6];
    const int n_hs = handoff_slots(args);
    const size_t need = gdn::prefill_ws_layout(args->batch, args->seq_len, args->num_k_heads, args->num_v_heads,
                                               args->head_k_dim, n_hs, off);
    if (!workspace || workspace_bytes < 0 || (size_t)workspace_bytes < need)
        return fail(GDN_ERR_INVALID_ARG, "workspace of %lld bytes needed (got %lld)", (long long)need,
                    (long long)workspace_bytes);
    if (!aligned16(workspace)) return fail(GDN_ERR_ALIGNMENT, "workspace must be 16-byte aligned");
    unsigned char* base = static_cast<unsigned char*>(workspace);
    gdn::PrefillWs ws;
    ws.qkv = base + off[0];
    ws.nrm = reinterpret_cast<float*>(base + off[1]);
    ws.gate = reinterpret_cast<float*>(base + off[2]);
    ws.tp = reinterpret_cast<float*>(base + off[3]);
    ws.hs = reinterpret_cast<float*>(base + off[4]);
    ws.hflag = reinterpret_cast<int*>(base + off[5]);
    ws.n_hs = n_hs;
    ws.nc = (args->seq_len + 63) / 64;
    ws.tp_len = ws.nc * 64;
    cudaError_t e = gdn::launch_prefill_prep(p, ws, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_status(e, "gdn_mixer_prefill_ws preparation launch");
    e = gdn::launch_prefill_seq(p, ck, ws, static_cast<cudaStream_t>(stream));
    return cuda_status(e, "gdn_mixer_prefill_ws sequential launch");
}

namespace {
// Key ranges of the decode attention: about four CTAs per SM of a 148-SM part, each range a
// multiple of 32 keys; a function of the shapes only, so the workspace size is too.
void attn_split(int32_t batch, int32_t kv_heads, int32_t capacity, int* splits, int* span) {
    const int kb = 32;
    const int pairs = std::max(1, batch * kv_heads);
    int S = std::max(1, (4 * 148 + pairs - 1) / pairs);
    S = std::min(S, (capacity + kb - 1) / kb);
    int sp = (capacity + S - 1) / S;
    sp = (sp + kb - 1) / kb * kb;
    *span = sp;
    *splits = (capacity + sp - 1) / sp;
}
int64_t attn_ws_bytes(int32_t batch, int32_t kv_heads, int32_t groups, int32_t head_dim, int32_t capacity,
                      int64_t* off_ml) {
    int S, sp;
    attn_split(batch, kv_heads, capacity, &S, &sp);
    const int64_t po = (int64_t)batch * kv_heads * S * groups * head_dim * 4;
    *off_ml = (po + 255) / 256 * 256;
    return *off_ml + (int64_t)batch * kv_heads * S * groups * 2 * 4;
}
bool attn_shape_ok(int32_t batch, int32_t kv_heads, int32_t groups, int32_t head_dim, int32_t capacity) {
    return batch > 0 && kv_heads > 0 && capacity > 0 && (groups == 1 || groups == 2 || groups == 4 || groups == 8) &&
           (head_dim == 64 || head_dim == 128 || head_dim == 256) &&
           (int64_t)batch * kv_heads * capacity * head_dim < (int64_t)1 << 40;
}
}  // namespace

int64_t gdn_attn_decode_workspace_bytes(int32_t batch, int32_t kv_heads, int32_t groups, int32_t head_dim,
                                        int32_t capacity) {
    if (!attn_shape_ok(batch, kv_heads, groups, head_dim, capacity))
        return fail(GDN_ERR_INVALID_ARG, "unsupported decode-attention shape");
    int64_t off;
    return attn_ws_bytes(batch, kv_heads, groups, head_dim, capacity, &off);
}

int32_t gdn_attn_decode(const void* q, const void* k_cache, const void* v_cache, const int64_t* pos, void* out,
                        int32_t batch, int32_t kv_heads, int32_t groups, int32_t head_dim, int32_t capacity,
                        float scale, void* workspace, int64_t workspace_bytes, void* stream) {
    if (!q || !k_cache || !v_cache || !pos || !out || !workspace)
        return fail(GDN_ERR_INVALID_ARG, "a required pointer is NULL");
    if (!attn_shape_ok(batch, kv_heads, groups, head_dim, capacity))
        return fail(GDN_ERR_INVALID_ARG, "unsupported decode-attention shape");
    const void* ptrs[] = {q, k_cache, v_cache, out, workspace};
    for (const void* p : ptrs)
        if (!aligned16(p)) return fail(GDN_ERR_ALIGNMENT, "pointers must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(pos) % 8) return fail(GDN_ERR_ALIGNMENT, "misaligned pos");
    int64_t off_ml;
    const int64_t need = attn_ws_bytes(batch, kv_heads, groups, head_dim, capacity, &off_ml);
    if (workspace_bytes < need) return fail(GDN_ERR_INVALID_ARG, "workspace too small (%lld < %lld)",
                                            (long long)workspace_bytes, (long long)need);
    gdn::AttnDecodeArgs a{};
    a.q = q;
    a.k = k_cache;
    a.v = v_cache;
    a.out = out;
    a.pos = reinterpret_cast<const long long*>(pos);
    a.batch = batch;
    a.kv_heads = kv_heads;
    a.groups = groups;
    a.head_dim = head_dim;
    a.capacity = capacity;
    attn_split(batch, kv_heads, capacity, &a.splits, &a.span);
    a.qscale = scale * 1.4426950408889634f;
    a.part_o = static_cast<float*>(workspace);
    a.part_ml = reinterpret_cast<float*>(static_cast<char*>(workspace) + off_ml);
    return cuda_status(gdn::launch_attn_decode(a, static_cast<cudaStream_t>(stream)), "gdn_attn_decode launch");
}

int32_t gdn_selftest_expired_wait(int32_t kind, int32_t* flag, void* stream) {
    if (kind < 0 || kind > 1) return fail(GDN_ERR_INVALID_ARG, "kind %d not in 0..1", kind);
    if (!flag) return fail(GDN_ERR_INVALID_ARG, "flag is NULL");
    if (reinterpret_cast<uintptr_t>(flag) % 4) return fail(GDN_ERR_ALIGNMENT, "misaligned flag");
    return cuda_status(gdn::launch_expired_wait_selftest(kind, flag, static_cast<cudaStream_t>(stream)),
                       "gdn_selftest_expired_wait launch");
}

int32_t gdn_selftest_umma(int32_t mode, const float* A, const float* B, float* D, void* stream) {
    if (mode < 0 || mode > 10) return fail(GDN_ERR_INVALID_ARG, "mode %d not in 0..10", mode);
    if (!A || !B || !D) return fail(GDN_ERR_INVALID_ARG, "a required pointer is NULL");
    const void* ptrs[] = {A, B, D};
    for (const void* ptr : ptrs)
        if (!aligned_elem(ptr, GDN_DTYPE_F32)) return fail(GDN_ERR_ALIGNMENT, "misaligned pointer");
    return cuda_status(gdn::launch_umma_selftest(mode, A, B, D, static_cast<cudaStream_t>(stream)),
                       "gdn_selftest_umma launch");
}

int32_t gdn_mixer_prefill(const gdn_mixer_args* args, void* stream) {
    gdn::CkptList ck;
    gdn::MixParams p;
    int32_t st = validate_mixer(args, &p, &ck);
    if (st != GDN_OK) return st;
    bool supported = false;
    cudaError_t e = cudaSuccess;
    if (!(args->flags & GDN_FLAG_CUDA_CORE_PREFILL))
        e = gdn::launch_prefill_tc(p, ck, args->head_k_dim, args->act_dtype, static_cast<cudaStream_t>(stream),
                                   &supported);
    if (!supported)
        e = gdn::launch_prefill(p, ck, args->head_k_dim, args->act_dtype, true, static_cast<cudaStream_t>(stream),
                                &supported);
    if (!supported) return fail(GDN_ERR_UNSUPPORTED, "no chunked kernel for these head dims");
    return cuda_status(e, "gdn_mixer_prefill launch");
}

int32_t gdn_delta_rule(int32_t batch, int32_t seq_len, int32_t num_heads, int32_t head_k_dim, int32_t head_v_dim,
                       int32_t in_dtype, const void* q, const void* k, const void* v, const void* g,
                       const void* beta, const float* state_in, float* state_out, void* out, int32_t use_qk_l2norm,
                       int32_t chunked, int32_t num_checkpoints, const int32_t* checkpoint_offsets,
                       float* state_checkpoints, void* stream) {
    if (batch < 1 || seq_len < 1 || num_heads < 1) return fail(GDN_ERR_INVALID_ARG, "sizes must be >= 1");
    if (!supported_head_dims(head_k_dim, head_v_dim))
        return fail(GDN_ERR_UNSUPPORTED, "head dims (%d, %d) not built: need dk == dv in {32, 64, 128}",
                    head_k_dim, head_v_dim);
    if (in_dtype != GDN_DTYPE_F32 && in_dtype != GDN_DTYPE_BF16)
        return fail(GDN_ERR_UNSUPPORTED, "in_dtype %d", in_dtype);
    if (!q || !k || !v || !g || !beta || !out) return fail(GDN_ERR_INVALID_ARG, "a required pointer is NULL");
    const void* elem_ptrs[] = {q, k, v, g, beta, out};
    for (const void* ptr : elem_ptrs)
        if (!aligned_elem(ptr, in_dtype)) return fail(GDN_ERR_ALIGNMENT, "misaligned input pointer");
    const void* f4_ptrs[] = {state_in, state_out, state_checkpoints};
    for (const void* ptr : f4_ptrs)
        if (ptr && !aligned16(ptr)) return fail(GDN_ERR_ALIGNMENT, "state pointers must be 16-byte aligned");
    gdn::CkptList ck;
    int32_t st = build_ckpts(num_checkpoints, checkpoint_offsets, seq_len, &ck);
    if (st != GDN_OK) return st;
    if (ck.n > 0 && !state_checkpoints)
        return fail(GDN_ERR_INVALID_ARG, "checkpoints requested but state_checkpoints is NULL");
    gdn::MixParams p;
    std::memset(&p, 0, sizeof(p));
    p.B = batch;
    p.T = seq_len;
    p.Hk = num_heads;
    p.Hv = num_heads;
    p.K = 1;
    p.q_scale = (float)std::pow((double)head_k_dim, -0.5);
    p.use_l2 = use_qk_l2norm ? 1 : 0;
    p.q = q;
    p.k = k;
    p.v = v;
    p.g = g;
    p.beta = beta;
    p.S_in = state_in;
    p.S_out = state_out;
    p.out = out;
    p.S_ckpt = state_checkpoints;
    bool supported = false;
    cudaError_t e;
    if (chunked)
        e = gdn::launch_prefill(p, ck, head_k_dim, in_dtype, false, static_cast<cudaStream_t>(stream), &supported);
    else
        e = gdn::launch_decode(p, ck, head_k_dim, head_v_dim, in_dtype, false, static_cast<cudaStream_t>(stream),
                               &supported);
    if (!supported) return fail(GDN_ERR_UNSUPPORTED, "no kernel for these head dims");
    return cuda_status(e, "gdn_delta_rule launch");
}

int32_t gdn_causal_conv1d(int32_t batch, int32_t channels, int32_t seq_len, int32_t kernel, int32_t dtype,
                          const void* x, const void* weight, const void* state_in, void* out, void* state_out,
                          int32_t apply_silu, void* stream) {
    if (batch < 1 || channels < 1 || seq_len < 1) return fail(GDN_ERR_INVALID_ARG, "sizes must be >= 1");
    if (kernel < 1 || kernel > 4) return fail(GDN_ERR_UNSUPPORTED, "kernel %d not in 1..4", kernel);
    if (dtype != GDN_DTYPE_F32 && dtype != GDN_DTYPE_BF16) return fail(GDN_ERR_UNSUPPORTED, "dtype %d", dtype);
    if (!x || !weight || !out) return fail(GDN_ERR_INVALID_ARG, "a required pointer is NULL");
    if ((int64_t)batch * channels > (int64_t)1 << 30) return fail(GDN_ERR_INVALID_ARG, "too many rows");
    const void* ptrs[] = {x, weight, state_in, out, state_out};
    for (const void* ptr : ptrs)
        if (ptr && !aligned_elem(ptr, dtype)) return fail(GDN_ERR_ALIGNMENT, "misaligned pointer");
    if (state_in && state_in == state_out) return fail(GDN_ERR_INVALID_ARG, "state_out must not alias state_in");
    cudaError_t e = gdn::launch_conv1d(batch, channels, seq_len, kernel, dtype, x, weight, state_in, out, state_out,
                                       apply_silu, static_cast<cudaStream_t>(stream));
    return cuda_status(e, "gdn_causal_conv1d launch");
}

int32_t gdn_solve_unit_lower_triangular(const float* ut, const float* rhs, float* out, int64_t batch, int32_t n,
                                        int32_t m, void* stream) {
    if (batch < 1 || n < 1 || m < 1) return fail(GDN_ERR_INVALID_ARG, "batch, n and m must be >= 1");
    if (batch > 0x7FFFFFFFll) return fail(GDN_ERR_INVALID_ARG, "batch %lld too large", (long long)batch);
    if (n > 4096 || m > (1 << 20)) return fail(GDN_ERR_INVALID_ARG, "n %d or m %d too large", n, m);
    if (!ut || !out) return fail(GDN_ERR_INVALID_ARG, "ut and out are required");
    if (!rhs && m != n) return fail(GDN_ERR_INVALID_ARG, "the inverse (rhs NULL) needs m == n");
    const void* ptrs[] = {ut, rhs, out};
    for (const void* ptr : ptrs)
        if (ptr && !aligned_elem(ptr, GDN_DTYPE_F32)) return fail(GDN_ERR_ALIGNMENT, "misaligned pointer");
    const int64_t n_out = batch * (int64_t)n * m, n_u = batch * (int64_t)n * n;
    auto overlaps = [](const float* a, int64_t na, const float* b, int64_t nb) {
        return a && b && a < b + nb && b < a + na;
    };
    if (overlaps(out, n_out, ut, n_u) || overlaps(out, n_out, rhs, n_out))
        return fail(GDN_ERR_INVALID_ARG, "out must not overlap ut or rhs");
    const cudaError_t e = gdn::launch_trisolve(ut, rhs, out, batch, n, m, static_cast<cudaStream_t>(stream));
    return cuda_status(e, "gdn_solve_unit_lower_triangular launch");
}

int32_t gdn_rms_norm_gated(const void* x, const void* gate, const void* weight, void* out, int64_t rows, int32_t dim,
                           float eps, int32_t x_dtype, int32_t gate_dtype, int32_t weight_dtype, void* stream) {
    if (rows < 1 || dim < 1) return fail(GDN_ERR_INVALID_ARG, "rows and dim must be >= 1");
    if (rows > ((int64_t)1 << 33)) return fail(GDN_ERR_INVALID_ARG, "too many rows");
    const int32_t dts[] = {x_dtype, gate_dtype, weight_dtype};
    for (int32_t d : dts)
        if (d != GDN_DTYPE_F32 && d != GDN_DTYPE_BF16) return fail(GDN_ERR_UNSUPPORTED, "dtype %d", d);
    if (!x || !gate || !weight || !out) return fail(GDN_ERR_INVALID_ARG, "a required pointer is NULL");
    if (!aligned_elem(x, x_dtype) || !aligned_elem(out, x_dtype) || !aligned_elem(gate, gate_dtype) ||
        !aligned_elem(weight, weight_dtype))
        return fail(GDN_ERR_ALIGNMENT, "misaligned pointer");
    if (!(eps >= 0.f)) return fail(GDN_ERR_INVALID_ARG, "eps must be >= 0");
    const cudaError_t e = gdn::launch_rms_norm_gated(x, gate, weight, out, rows, dim, eps, x_dtype, gate_dtype,
                                                     weight_dtype, static_cast<cudaStream_t>(stream));
    return cuda_status(e, "gdn_rms_norm_gated launch");
}

int32_t gdn_mixer_prefill_noalloc(const gdn_mixer_args* args, void* stream) {
    const int64_t need = gdn_prefill_workspace_bytes(args);
    if (need < 0) return (int32_t)need;  // invalid arguments, message already set
    if (need > GDN_STATIC_SCRATCH_BYTES)
        return fail(GDN_ERR_INVALID_ARG, "needs %lld bytes of scratch; the static scratch holds %lld",
                    (long long)need, (long long)GDN_STATIC_SCRATCH_BYTES);
    void* scratch = nullptr;
    if (need > 0) {
        const cudaError_t e = gdn::static_prefill_scratch(&scratch);
        if (e != cudaSuccess) return cuda_status(e, "address of the static prefill scratch");
    }
    return gdn_mixer_prefill_ws(args, scratch, need > 0 ? (int64_t)GDN_STATIC_SCRATCH_BYTES : 0, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// peer all-reduce: staging memory, IPC mappings, the call
// ---------------------------------------------------------------------------
namespace {
size_t up256(size_t x) { return (x + 255) & ~(size_t)255; }
// byte offsets of the flags and the epochs inside a staging allocation
void peer_layout(int world, int nblocks, int64_t cap, size_t* flags_off, size_t* counters_off, size_t* total) {
    *flags_off = up256((size_t)cap * world * 2 * 2);
    *counters_off = *flags_off + up256((size_t)world * nblocks * 4);
    *total = *counters_off + up256((size_t)nblocks * 4);
}
bool peer_shape_ok(int world, int nblocks, int64_t cap) {
    return world >= 1 && world <= GDN_PEER_MAX_RANKS && nblocks >= 1 && nblocks <= 1024 && cap >= 8 && cap % 8 == 0 &&
           cap <= (1ll << 34);
}
}  // namespace

int64_t gdn_peer_staging_bytes(int32_t world, int32_t nblocks, int64_t cap) {
    if (!peer_shape_ok(world, nblocks, cap))
        return fail(GDN_ERR_INVALID_ARG, "world 1..%d, nblocks 1..1024, cap a positive multiple of 8",
                    GDN_PEER_MAX_RANKS);
    size_t f, c, t;
    peer_layout(world, nblocks, cap, &f, &c, &t);
    ok();
    return (int64_t)t;
}

int32_t gdn_peer_staging_alloc(int64_t bytes, void** ptr_out) {
    if (!ptr_out || bytes <= 0) return fail(GDN_ERR_INVALID_ARG, "bytes must be positive and ptr_out non-NULL");
    *ptr_out = nullptr;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, (size_t)bytes);
    if (e != cudaSuccess) return cuda_status(e, "gdn_peer_staging_alloc cudaMalloc");
    e = cudaMemset(p, 0, (size_t)bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_status(e, "gdn_peer_staging_alloc cudaMemset");
    }
    *ptr_out = p;
    return ok();
}

int32_t gdn_peer_staging_free(void* ptr) {
    if (!ptr) return ok();
    return cuda_status(cudaFree(ptr), "gdn_peer_staging_free");
}

int32_t gdn_ipc_get_handle(const void* dev_ptr, void* handle_out) {
    static_assert(sizeof(cudaIpcMemHandle_t) == GDN_IPC_HANDLE_BYTES, "IPC handle size");
    if (!dev_ptr || !handle_out) return fail(GDN_ERR_INVALID_ARG, "a required pointer is NULL");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr));
    if (e != cudaSuccess) return cuda_status(e, "gdn_ipc_get_handle");
    memcpy(handle_out, &h, sizeof(h));
    return ok();
}

int32_t gdn_ipc_open_handle(const void* handle, void** dev_ptr_out) {
    if (!handle || !dev_ptr_out) return fail(GDN_ERR_INVALID_ARG, "a required pointer is NULL");
    *dev_ptr_out = nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return cuda_status(cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess), "gdn_ipc_open_handle");
}

int32_t gdn_ipc_close_handle(void* dev_ptr) {
    if (!dev_ptr) return ok();
    return cuda_status(cudaIpcCloseMemHandle(dev_ptr), "gdn_ipc_close_handle");
}

int32_t gdn_peer_allreduce_bf16(const gdn_peer_group* g, const void* in, void* out, int64_t n, void* stream) {
    if (!g || !in || !out) return fail(GDN_ERR_INVALID_ARG, "a required pointer is NULL");
    if (!peer_shape_ok(g->world, g->nblocks, g->cap) || g->rank < 0 || g->rank >= g->world)
        return fail(GDN_ERR_INVALID_ARG, "bad group: rank %d of %d, nblocks %d, cap %lld", g->rank, g->world,
                    g->nblocks, (long long)g->cap);
    if (n < 0 || n % 8 != 0 || n > g->cap)
        return fail(GDN_ERR_INVALID_ARG, "n = %lld must be a multiple of 8 and at most cap = %lld", (long long)n,
                    (long long)g->cap);
    if (!aligned16(in) || !aligned16(out)) return fail(GDN_ERR_ALIGNMENT, "in / out must be 16-byte aligned");
    for (int r = 0; r < g->world; ++r)
        if (!g->staging[r] || !aligned16(g->staging[r]))
            return fail(GDN_ERR_INVALID_ARG, "staging[%d] is NULL or misaligned", r);
    if (n == 0) return ok();
    size_t f, c, t;
    peer_layout(g->world, g->nblocks, g->cap, &f, &c, &t);
    gdn::PeerAllReduceArgs a;
    memset(&a, 0, sizeof(a));
    a.in = in;
    a.out = out;
    a.n = n;
    a.cap = g->cap;
    a.rank = g->rank;
    a.world = g->world;
    a.nblocks = g->nblocks;
    for (int r = 0; r < g->world; ++r) {
        unsigned char* base = static_cast<unsigned char*>(g->staging[r]);
        a.data[r] = reinterpret_cast<uint16_t*>(base);
        a.flags[r] = reinterpret_cast<int*>(base + f);
    }
    a.counters = reinterpret_cast<int*>(static_cast<unsigned char*>(g->staging[g->rank]) + c);
    return cuda_status(gdn::launch_peer_allreduce(a, static_cast<cudaStream_t>(stream)), "gdn_peer_allreduce_bf16");
}

// ---------------------------------------------------------------------------
// fused elementwise steps of the stack's layers
// ---------------------------------------------------------------------------
int32_t gdn_rms_norm_zc(const void* x, int64_t x_row_stride, const void* delta, int64_t delta_row_stride,
                        void* res_out, const void* weight, void* out, int64_t rows, int32_t dim, float eps,
                        void* stream) {
    if (!x || !weight || !out) return fail(GDN_ERR_INVALID_ARG, "a required pointer is NULL");
    if ((delta == nullptr) != (res_out == nullptr))
        return fail(GDN_ERR_INVALID_ARG, "delta and res_out are given together or not at all");
    if (rows < 0 || dim < 8 || dim > 16384 || dim % 8 != 0)
        return fail(GDN_ERR_INVALID_ARG, "rows >= 0, dim a multiple of 8 in 8..16384");
    if (rows > 0x7FFFFFFFll) return fail(GDN_ERR_INVALID_ARG, "rows = %lld: at most 2^31 - 1", (long long)rows);
    if (x_row_stride < dim || x_row_stride % 8 != 0 || (delta && (delta_row_stride < dim || delta_row_stride % 8 != 0)))
        return fail(GDN_ERR_INVALID_ARG, "row strides must be multiples of 8 of at least dim");
    const void* ptrs[] = {x, delta, res_out, weight, out};
    for (const void* p : ptrs)
        if (p && !aligned16(p)) return fail(GDN_ERR_ALIGNMENT, "pointers must be 16-byte aligned");
    if (rows == 0) return ok();
    gdn::RmsNormArgs a;
    a.x = x;
    a.x_stride = x_row_stride;
    a.delta = delta;
    a.delta_stride = delta_row_stride;
    a.res = res_out;
    a.res_stride = dim;
    a.w = weight;
    a.out = out;
    a.out_stride = dim;
    a.rows = rows;
    a.dim = dim;
    a.eps = eps;
    return cuda_status(gdn::launch_rms_norm_zc(a, static_cast<cudaStream_t>(stream)), "gdn_rms_norm_zc");
}

int32_t gdn_silu_mul(const void* gate, const void* up, void* out, int64_t n, void* stream) {
    if (!gate || !up || !out) return fail(GDN_ERR_INVALID_ARG, "a required pointer is NULL");
    if (n < 0 || n % 8 != 0) return fail(GDN_ERR_INVALID_ARG, "n = %lld must be a multiple of 8", (long long)n);
    if (!aligned16(gate) || !aligned16(up) || !aligned16(out))
        return fail(GDN_ERR_ALIGNMENT, "pointers must be 16-byte aligned");
    if (n == 0) return ok();
    return cuda_status(gdn::launch_silu_mul(gate, up, out, n, static_cast<cudaStream_t>(stream)), "gdn_silu_mul");
}

int32_t gdn_qk_norm_rope(const void* qg, const void* k, const void* q_weight, const void* k_weight, const void* cos,
                         const void* sin, void* q_out, void* k_out, int32_t batch, int32_t seq_len,
                         int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, int32_t rotary_dim, float eps,
                         void* stream) {
    const void* ptrs[] = {qg, k, q_weight, k_weight, cos, sin, q_out, k_out};
    for (const void* p : ptrs) {
        if (!p) return fail(GDN_ERR_INVALID_ARG, "a required pointer is NULL");
        if (!aligned16(p)) return fail(GDN_ERR_ALIGNMENT, "pointers must be 16-byte aligned");
    }
    if (batch < 0 || seq_len < 0 || num_heads < 1 || num_kv_heads < 1)
        return fail(GDN_ERR_INVALID_ARG, "bad sizes");
    if (head_dim < 8 || head_dim > 256 || head_dim % 8 != 0 || rotary_dim < 0 || rotary_dim % 16 != 0 ||
        rotary_dim > head_dim)
        return fail(GDN_ERR_UNSUPPORTED, "head_dim a multiple of 8 up to 256, rotary_dim a multiple of 16 up to it");
    if ((long long)batch * seq_len == 0) return ok();
    if ((long long)batch * seq_len * (num_heads + num_kv_heads) > 0x7FFFFFFFll * 8)
        return fail(GDN_ERR_INVALID_ARG, "too many (token, head) rows for one launch");
    gdn::QkRopeArgs a;
    a.qg = qg;
    a.k = k;
    a.qw = q_weight;
    a.kw = k_weight;
    a.cos = cos;
    a.sin = sin;
    a.q_out = q_out;
    a.k_out = k_out;
    a.B = batch;
    a.T = seq_len;
    a.H = num_heads;
    a.KVH = num_kv_heads;
    a.hd = head_dim;
    a.rot = rotary_dim;
    a.eps = eps;
    return cuda_status(gdn::launch_qk_norm_rope(a, static_cast<cudaStream_t>(stream)), "gdn_qk_norm_rope");
}

int32_t gdn_attn_gate_out(const void* o, int64_t o_stride_b, int64_t o_stride_h, int64_t o_stride_t, const void* qg,
                          void* out, int32_t batch, int32_t seq_len, int32_t num_heads, int32_t head_dim,
                          void* stream) {
    if (!o || !qg || !out) return fail(GDN_ERR_INVALID_ARG, "a required pointer is NULL");
    if (!aligned16(o) || !aligned16(qg) || !aligned16(out) || o_stride_b % 8 || o_stride_h % 8 || o_stride_t % 8)
        return fail(GDN_ERR_ALIGNMENT, "pointers 16-byte aligned, strides multiples of 8 elements");
    if (batch < 0 || seq_len < 0 || num_heads < 1 || head_dim < 8 || head_dim % 8 != 0)
        return fail(GDN_ERR_INVALID_ARG, "bad sizes");
    if ((long long)batch * seq_len == 0) return ok();
    gdn::GateOutArgs a;
    a.o = o;
    a.o_sb = o_stride_b;
    a.o_sh = o_stride_h;
    a.o_st = o_stride_t;
    a.qg = qg;
    a.out = out;
    a.B = batch;
    a.T = seq_len;
    a.H = num_heads;
    a.hd = head_dim;
    return cuda_status(gdn::launch_gate_out(a, static_cast<cudaStream_t>(stream)), "gdn_attn_gate_out");
}
