/*
 * gdn_b200.h - C ABI of the B200 (sm_100a) Gated DeltaNet token mixer.
 *
 * The token mixer is the part of the reference layer
 * `Qwen3_5GatedDeltaNet.forward` (ShadowBoxer/models/qwen35/deltanet.py:447-563)
 * between the four input projections and `out_proj`: causal depthwise conv1d
 * + SiLU, q/k L2 normalisation, the beta / decay gates, the gated delta rule
 * (token-by-token or chunked) and the output gated RMSNorm.  The projections
 * and `out_proj` stay library GEMMs in the host layer.
 *
 * Conventions
 *  - Every entry point returns an int32 status: GDN_OK (0) or a negative
 *    GDN_ERR_* code.  The message of the last failure on the calling thread is
 *    available from gdn_last_error_string().  (Same convention as the
 *    reference's native DLL, VizInjector/src/native/vizinjector_dll.h, bound
 *    with ctypes restype c_int32 and raised as RuntimeError by
 *    VizInjector/python/bindings.py:298-400.)
 *  - All tensor pointers are DEVICE pointers of the current CUDA device.
 *    `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *  - Arguments are validated on the host before any launch; nothing traps on
 *    the device.  Launch failures are reported as GDN_ERR_CUDA.
 *  - Activations, projection outputs, the conv weight, the conv state and the
 *    norm weight share one "activation dtype" (GDN_DTYPE_BF16 or
 *    GDN_DTYPE_F32); recurrent states are always float32
 *    [batch, num_v_heads, head_k_dim, head_v_dim] contiguous, as in the
 *    reference cache (ShadowBoxer/models/qwen35/cache.py:17-18).
 *  - GQA: value head h reads key head h / (num_v_heads / num_k_heads), the
 *    mapping of `repeat_interleave` at deltanet.py:520-523.
 */
#ifndef GDN_B200_H
#define GDN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_ABI_VERSION 1

#define GDN_OK 0
#define GDN_ERR_INVALID_ARG (-1)   /* null pointer, bad size or stride */
#define GDN_ERR_UNSUPPORTED (-2)   /* shape / dtype combination not built */
#define GDN_ERR_ALIGNMENT (-3)     /* pointer or stride misaligned */
#define GDN_ERR_CUDA (-4)          /* a CUDA runtime call or launch failed */
#define GDN_ERR_TOO_MANY_CHECKPOINTS (-5)

#define GDN_DTYPE_F32 0
#define GDN_DTYPE_BF16 1

/* gdn_mixer_args.flags: run the register-tile token-by-token kernel even
 * where the bulk-copy pipelined one applies, the CUDA-core chunked kernel even
 * where the tensor-core one applies, and (gdn_mixer_prefill_ws) the single
 * kernel that prepares each chunk in shared memory two chunks ahead of the
 * state pass instead of the two-kernel form with its preparation pass through
 * the workspace (same results up to float rounding).  The single kernel needs
 * a workspace only for state hand-offs (at most 64 KB per SM, whatever the
 * length); the two-kernel form is faster at the prefill benchmark's size. */
#define GDN_FLAG_REGISTER_KERNEL 1
#define GDN_FLAG_CUDA_CORE_PREFILL 2
#define GDN_FLAG_PREP_IN_KERNEL_PREFILL 4

/* Bits of the device error word (gdn_device_error). */
#define GDN_DEVERR_TMA_TIMEOUT 0x1u
#define GDN_DEVERR_MMA_TIMEOUT 0x2u
#define GDN_DEVERR_BAD_SLOT 0x4u   /* slot-table entry or accepted count out of range */
#define GDN_DEVERR_HANDOFF_TIMEOUT 0x8u  /* chunked prefill: a chain's state hand-off never arrived */
#define GDN_DEVERR_PEER_TIMEOUT 0x10u    /* peer all-reduce: another rank's flag never arrived */

/* Size of the library's fixed device scratch used by gdn_mixer_prefill_noalloc
 * (64 MiB per device: the two-kernel prefill's workspace for about 1.9k
 * tokens x 16 / 32 heads of 128; with GDN_FLAG_PREP_IN_KERNEL_PREFILL a call
 * needs at most one 64 KB state hand-off slot per SM, so every length fits). */
#define GDN_STATIC_SCRATCH_BYTES (64ll << 20)

/* Maximum number of state checkpoints one call can record. */
#define GDN_MAX_CHECKPOINTS 512
/* Longest sequence the token-by-token (decode / verify) entry accepts. */
#define GDN_MAX_DECODE_TOKENS 8

/*
 * Arguments of the fused token mixer (one layer, one call).
 *
 * Layout of the inputs (row-major, last dimension contiguous):
 *   mixed_qkv   [batch, seq_len, conv_dim]  channels ordered
 *               [q: Hk*dk | k: Hk*dk | v: Hv*dv], head-major (deltanet.py:508-514)
 *   z           [batch, seq_len, Hv*dv]
 *   a, b        [batch, seq_len, Hv]
 *   conv_weight [conv_dim, conv_kernel]
 *   A_log, dt_bias  [Hv] float32
 *   norm_weight [dv]
 * Outputs:
 *   out         [batch, seq_len, Hv*dv] gated-RMSNorm output (input of out_proj)
 *   conv_state_out [batch, conv_dim, conv_kernel-1]  raw inputs of the last
 *               conv_kernel-1 positions, oldest first (deltanet.py:24-38)
 *   state_out   [batch, Hv, dk, dv] float32
 * Checkpoints (deltanet.py:479-487, 223-226, 345-388): for each local offset
 * off = checkpoint_offsets[i] in 1..seq_len, slot i of state_checkpoints
 * ([num_checkpoints, batch, Hv, dk, dv] float32) receives the recurrent state
 * after `off` tokens and slot i of conv_checkpoints
 * ([num_checkpoints, batch, conv_dim, conv_kernel-1]) the conv state after
 * `off` tokens.  Offsets outside 1..seq_len are skipped.
 */
typedef struct gdn_mixer_args {
    int32_t batch;
    int32_t seq_len;
    int32_t num_k_heads;
    int32_t num_v_heads;
    int32_t head_k_dim;
    int32_t head_v_dim;
    int32_t conv_kernel;
    int32_t act_dtype;        /* GDN_DTYPE_* */
    float norm_eps;           /* rms_norm_eps of the gated norm */
    int32_t flags;            /* GDN_FLAG_* bits, 0 by default */

    const void* mixed_qkv;    /* required */
    int64_t mixed_stride_b;   /* elements between batch rows */
    int64_t mixed_stride_t;   /* elements between tokens */
    const void* z;            /* required */
    int64_t z_stride_b;
    int64_t z_stride_t;
    const void* a;            /* required */
    const void* b;            /* required */
    int64_t ab_stride_b;      /* shared by a and b */
    int64_t ab_stride_t;
    const void* conv_weight;  /* required */
    const float* A_log;       /* required */
    const float* dt_bias;     /* required */
    const void* norm_weight;  /* required */

    const void* conv_state_in;  /* NULL: zeros (no previous state) */
    void* conv_state_out;       /* NULL: not written; must not alias conv_state_in */
    const float* state_in;      /* NULL: zeros */
    float* state_out;           /* NULL: not written; may equal state_in (in-place) */
    void* out;                  /* required */

    int32_t num_checkpoints;            /* 0..GDN_MAX_CHECKPOINTS */
    int32_t reserved1;
    const int32_t* checkpoint_offsets;  /* HOST array of num_checkpoints local offsets */
    float* state_checkpoints;           /* device, may be NULL when num_checkpoints == 0 */
    void* conv_checkpoints;             /* device, may be NULL when num_checkpoints == 0 */
} gdn_mixer_args;

/* Library ABI version (GDN_ABI_VERSION). */
int32_t gdn_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* gdn_last_error_string(void);

/*
 * Token-by-token token mixer for 1 <= seq_len <= GDN_MAX_DECODE_TOKENS: the
 * single-token decode step and the speculative-decode verify step.
 * Replaces deltanet.py:479-561 on the branch where _chunk_gated_delta_rule
 * hands off to _recurrent_gated_delta_rule (deltanet.py:251-264, 165-233).
 * One launch: conv-state shift + conv + SiLU, L2 norms, gates, decay and
 * rank-1 delta update of the fp32 state (in place when state_out == state_in),
 * readout, gated RMSNorm, per-token checkpoints.  When the inputs are 16-byte
 * aligned (strides in multiples of 16 bytes) a persistent kernel streams the
 * per-(batch, head) tiles through a bulk-copy shared-memory pipeline;
 * otherwise a register-tile kernel runs.  Both compute the same thing.
 */
int32_t gdn_mixer_decode(const gdn_mixer_args* args, void* stream);

/*
 * Speculative-decode verify on per-row state slots: rollback without copies.
 *
 * The reference verifies a draft of T tokens on a cache cloned per candidate
 * (Qwen3_5HybridCache.clone_and_expand, ShadowBoxer/models/qwen35/cache.py:156-197)
 * that records a checkpoint after every draft token, then restores each row to
 * the checkpoint of its accepted length by copying it out of the checkpoint
 * dicts (select_batch_item / extract_checkpoint, cache.py:131-154, 199-244;
 * the loop in ShadowBoxer/models/qwen35/speculative.py:778-882).  Here each
 * batch row owns num_slots (>= seq_len + 1) state slots:
 *   args->state_in       state pool [num_slots, batch, Hv, dk, dv] float32
 *   args->conv_state_in  conv pool  [num_slots, batch, conv_dim, conv_kernel-1]
 *   slot_table           [batch, num_slots] int32 (device), a permutation of
 *                        0..num_slots-1 in every row
 * Row b starts from pool slot slot_table[b][0]; its recurrent and conv states
 * after t = 1..seq_len draft tokens go to pool slot slot_table[b][t].  The
 * starting slot is never written, so a fully rejected draft costs nothing.
 * args->state_out, conv_state_out, num_checkpoints and the checkpoint pointers
 * must be NULL / 0.  Everything else is as for gdn_mixer_decode.  Needs the
 * pipelined kernel's conditions (4-tap conv, head dim 64 or 128, 16-byte
 * aligned inputs, bf16 activations or seq_len 1), else GDN_ERR_UNSUPPORTED.
 * Table entries outside 0..num_slots-1 are never followed: the tile reads
 * slot 0 instead, skips the write and sets GDN_DEVERR_BAD_SLOT.
 */
int32_t gdn_mixer_verify_slots(const gdn_mixer_args* args, const int32_t* slot_table, int32_t num_slots,
                               void* stream);

/*
 * Accept accepted[b] (0..seq_len) draft tokens of row b after
 * gdn_mixer_verify_slots: swaps slot_table[b][0] and slot_table[b][accepted[b]],
 * so the row continues from its state after accepted[b] tokens (0 keeps the
 * state from before the draft; the old starting slot becomes free).  Device
 * int32 arrays, one small launch, no host synchronisation.  Counts outside
 * 0..seq_len leave the row unchanged and set GDN_DEVERR_BAD_SLOT.
 */
int32_t gdn_accept_slots(const int32_t* accepted, int32_t* slot_table, int32_t batch, int32_t num_slots,
                         int32_t seq_len, void* stream);

/*
 * Read (and optionally clear) the sticky device error word of the current
 * device: bounded waits inside the pipelined kernels that gave up set a
 * GDN_DEVERR_* bit instead of hanging.  Synchronises the device.  No
 * counterpart in the reference (it has no device code).
 */
int32_t gdn_device_error(uint32_t* flags_out, int32_t clear);

/*
 * Tensor-core self-test: D[128][N] = A * B with the 5th-generation tensor
 * core (tf32 in, fp32 out; modes 7..10 bf16 in) for operand-layout combination
 * `mode` (0..10, see gdn_umma_selftest.cu; modes 4..8 read A from tensor
 * memory, 9..10 both operands from shared memory), in plain
 * row-major fp32 device buffers.  Checks the shared-memory layouts,
 * descriptors and tensor-memory operands the chunked kernels rely on.  No
 * counterpart in the reference.
 */
int32_t gdn_selftest_umma(int32_t mode, const float* A, const float* B, float* D, void* stream);

/*
 * Failure-detection self-test: one thread runs one of the kernels' bounded
 * waits on something that never arrives, so that the wait gives up after
 * its limit (1 s) and the kernel returns.  kind 0 waits on an mbarrier with
 * no arrival (sets GDN_DEVERR_TMA_TIMEOUT); kind 1 waits on the device int
 * flag[0] (the chunked prefill's state hand-off wait; sets
 * GDN_DEVERR_HANDOFF_TIMEOUT unless flag[0] is already non-zero).  flag[1]
 * receives 1 when the wait succeeded and 2 when it gave up; the context
 * stays usable.  No counterpart in the reference.
 */
int32_t gdn_selftest_expired_wait(int32_t kind, int32_t* flag, void* stream);

/*
 * Decode attention of the hybrid stack's full-attention layers: one query
 * token per row against a fixed-capacity KV buffer, grouped-query
 * (text.py:160-212 with q_len 1; SDPA with enable_gqa).  q and out are
 * [batch][kv_heads * groups][head_dim] bf16 (query head h reads KV head
 * h / groups); k_cache and v_cache are [batch][kv_heads][capacity][head_dim]
 * bf16; keys 0..*pos attend (pos is read on the device, so a captured launch
 * serves every step; *pos >= capacity is clamped to the buffer).
 * out = softmax(scale q K^T) V in fp32, rounded to bf16.  groups in
 * {1, 2, 4, 8}, head_dim in {64, 128, 256}; pointers 16-byte aligned;
 * workspace of gdn_attn_decode_workspace_bytes (scratch).  No counterpart in
 * the reference's C code (the reference calls torch SDPA).
 */
int64_t gdn_attn_decode_workspace_bytes(int32_t batch, int32_t kv_heads, int32_t groups, int32_t head_dim,
                                        int32_t capacity);
int32_t gdn_attn_decode(const void* q, const void* k_cache, const void* v_cache, const int64_t* pos, void* out,
                        int32_t batch, int32_t kv_heads, int32_t groups, int32_t head_dim, int32_t capacity,
                        float scale, void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Chunked token mixer for any seq_len >= 1 (prefill).  Replaces
 * deltanet.py:479-561 on the _chunk_gated_delta_rule branch
 * (deltanet.py:266-407): the WY/UT intra-chunk solve and the sequential
 * inter-chunk state propagation, with conv, norms, gates and the gated RMSNorm
 * fused in.  Needs no workspace.  With bf16 activations, head dim 128 and
 * 16-byte aligned z rows the contractions run on the tensor cores (tcgen05,
 * tf32 operands, fp32 accumulation); otherwise a CUDA-core fp32 kernel runs.
 */
int32_t gdn_mixer_prefill(const gdn_mixer_args* args, void* stream);

/*
 * Device workspace, in bytes, that gdn_mixer_prefill_ws needs for these
 * arguments: 0 when the call takes a path without workspace, a negative
 * GDN_ERR_* code when the arguments are invalid.  At batch 8 x 8192 tokens,
 * 16 / 32 heads of 128 the default two-kernel form needs about 2.2 GB (the
 * conv outputs in bf16 plus a 32 KB pair of 64x64 tf32 matrices per chunk and
 * value head); when there are more (batch, value head) chains than the
 * current device has SMs both forms add one state-sized hand-off slot (64 KB)
 * and flag per SM, which is all that GDN_FLAG_PREP_IN_KERNEL_PREFILL needs
 * (about 9.7 MB on a 148-SM B200, whatever the length).  Ask with the device
 * current that will run the call.
 */
int64_t gdn_prefill_workspace_bytes(const gdn_mixer_args* args);

/*
 * Chunked token mixer (prefill) with a caller workspace, same arguments,
 * results and cache semantics as gdn_mixer_prefill.  By default two kernels:
 * a fully parallel preparation kernel (one CTA per batch row, key head and
 * chunk of 64 tokens) computes what does not depend on the recurrent state -
 * conv + SiLU, L2-norm factors, gates, and each chunk's (I + A)^-1 and masked
 * Q K^T (deltanet.py:266-343) - into `workspace`; the sequential kernel (one
 * CTA per batch row and value head, or one cooperative wave of one CTA per SM
 * when there are more chains than SMs) then carries the state through the
 * chunks (deltanet.py:345-389) with every state product on the tensor cores.
 * With GDN_FLAG_PREP_IN_KERNEL_PREFILL one kernel does both: producer warps
 * prepare each chunk in shared memory two chunks ahead of the state pass.
 * `workspace` (device, 16-byte aligned, at least gdn_prefill_workspace_bytes,
 * not overlapping any other argument; may be NULL when that is 0) is scratch:
 * the call clears what must start at zero and nothing in it survives the call.
 * Shapes neither form covers (activations other than bf16, head dims other
 * than 128, conv_kernel != 4, num_v_heads / num_k_heads not in {1, 2, 4},
 * misaligned inputs) or GDN_FLAG_CUDA_CORE_PREFILL run gdn_mixer_prefill
 * instead and ignore the workspace.
 */
int32_t gdn_mixer_prefill_ws(const gdn_mixer_args* args, void* workspace, int64_t workspace_bytes, void* stream);

/*
 * gdn_mixer_prefill_ws with the workspace taken from a fixed scratch array
 * of this library (GDN_STATIC_SCRATCH_BYTES per device, its address looked up
 * with cudaGetSymbolAddress on every call): the call allocates no device
 * memory, for callers that have no device allocator of their own (a C or FFI
 * host without PyTorch, which would otherwise need a cudaMalloc / cudaFree
 * pair - each synchronising the device - around every call).  Calls that need
 * more than GDN_STATIC_SCRATCH_BYTES of workspace (gdn_prefill_workspace_bytes)
 * are rejected with GDN_ERR_INVALID_ARG.  Every call on a device shares the
 * one scratch array: calls that can run at the same time on a device
 * (different streams, or host threads without ordering between them) race
 * on it and must be serialised by the caller.  The call clears what must
 * start at zero (the state hand-off flags, by an asynchronous memset on the
 * call's stream); the rest is written before it is read.  The array occupies
 * GDN_STATIC_SCRATCH_BYTES on every device where the library's module is
 * loaded (at library load with CUDA_MODULE_LOADING=EAGER, at its first kernel
 * launch with the default lazy loading), until the process exits, whether or
 * not this entry is called.  No counterpart in the reference (its PyTorch
 * path takes its temporaries from torch's allocator).
 */
int32_t gdn_mixer_prefill_noalloc(const gdn_mixer_args* args, void* stream);

/*
 * Stand-alone delta rule on already-split q/k/v, the functional boundary of
 * _recurrent_gated_delta_rule (deltanet.py:165-233) and
 * _chunk_gated_delta_rule (deltanet.py:236-407).
 *   q, k   [batch, seq_len, num_heads, dk]   (num_heads = value heads: the
 *          caller has already repeated GQA heads, as the reference does)
 *   v      [batch, seq_len, num_heads, dv]
 *   g, beta [batch, seq_len, num_heads]
 * in dtype `in_dtype` (contiguous).  `out` [batch, seq_len, num_heads, dv] is
 * written in `in_dtype`.  use_qk_l2norm != 0 applies the L2 norm of
 * config.py:114-115; q is always scaled by dk^-1/2.  `chunked` selects the
 * chunked algorithm (otherwise token by token, any seq_len).
 * Checkpoint offsets are local (absolute position - past_seen_tokens).
 */
int32_t gdn_delta_rule(int32_t batch, int32_t seq_len, int32_t num_heads, int32_t head_k_dim,
                       int32_t head_v_dim, int32_t in_dtype, const void* q, const void* k,
                       const void* v, const void* g, const void* beta, const float* state_in,
                       float* state_out, void* out, int32_t use_qk_l2norm, int32_t chunked,
                       int32_t num_checkpoints, const int32_t* checkpoint_offsets,
                       float* state_checkpoints, void* stream);

/*
 * Stand-alone causal depthwise conv1d + optional SiLU, the functional
 * boundary of _causal_conv1d_fn (deltanet.py:41-90), in the reference's
 * [batch, channels, seq_len] layout (contiguous).  Computes in the weight
 * dtype with one rounding per tap, as the reference does.
 *   x [batch, channels, seq_len], weight [channels, kernel],
 *   state_in [batch, channels, kernel-1] or NULL, out like x,
 *   state_out [batch, channels, kernel-1] or NULL.
 */
int32_t gdn_causal_conv1d(int32_t batch, int32_t channels, int32_t seq_len, int32_t kernel,
                          int32_t dtype, const void* x, const void* weight, const void* state_in,
                          void* out, void* state_out, int32_t apply_silu, void* stream);

/*
 * Unit lower triangular solve, the functional boundary of
 * _solve_unit_lower_triangular (deltanet.py:112-162) and, with rhs NULL,
 * _invert_unit_lower_triangular_block (deltanet.py:93-109):
 *   out[i] = (I + tril(ut[i], -1))^-1 rhs[i]       for i < batch
 * ut [batch, n, n] (its diagonal and upper triangle are ignored), rhs and out
 * [batch, n, m], float32, contiguous; rhs NULL means the identity (m == n).
 * fp32 forward substitution; same result as the reference's block-doubling
 * products up to float rounding.  out must not overlap ut or rhs.
 */
int32_t gdn_solve_unit_lower_triangular(const float* ut, const float* rhs, float* out, int64_t batch,
                                        int32_t n, int32_t m, void* stream);

/*
 * Gated RMSNorm over the last dimension, the math of
 * Qwen3_5RMSNormGated.forward (config.py:136-143):
 *   out = ((weight * round(x * rsqrt(mean(x^2) + eps))) * SiLU(gate)) rounded
 * to x's dtype, where round() is to x's dtype and the weight product is
 * rounded to bf16 when x and weight are both bf16 (torch's type promotion).
 * x, gate, out [rows, dim] contiguous (out in x's dtype), weight [dim].
 */
int32_t gdn_rms_norm_gated(const void* x, const void* gate, const void* weight, void* out, int64_t rows,
                           int32_t dim, float eps, int32_t x_dtype, int32_t gate_dtype,
                           int32_t weight_dtype, void* stream);

/*
 * One-shot all-reduce (sum) of a small bf16 tensor across the GPUs of one node
 * over NVLink peer memory, for the exchange step of the value-head-sharded
 * layers: the sum of the row-parallel out_proj partials after the token
 * mixer (and, in the sharded stack, of o_proj and down_proj), a few hundred
 * KB per decode step, where a ring all-reduce is bound by its latency.  No
 * counterpart in the reference (its engine runs on one GPU); it replaces the
 * NCCL all-reduce of that step for messages up to the staging capacity.
 *
 * Set-up, once per group (every rank, same arguments):
 *   1. gdn_peer_staging_bytes(world, nblocks, cap) bytes from
 *      gdn_peer_staging_alloc (cudaMalloc on the current device, zeroed;
 *      synchronous): two slots of every rank's partial (cap elements each),
 *      the flags and epochs;
 *   2. gdn_ipc_get_handle on it, the GDN_IPC_HANDLE_BYTES handles exchanged
 *      between the ranks (any host channel), gdn_ipc_open_handle on every
 *      other rank's handle: gdn_peer_group.staging[r] = rank r's allocation
 *      as mapped into this process (staging[rank] = the own pointer).
 * gdn_peer_allreduce_bf16 then sums `in` (n elements, n a multiple of 8,
 * n <= cap, 16-byte aligned; `out` may equal `in`) over the ranks into `out`,
 * on `stream`.  Every rank calls it the same number of times in the same
 * order (it can be captured in a CUDA graph: the call's epoch lives on the
 * device).  Every rank gets the same bits (fp32 sum in rank order, rounded to
 * bf16).  A rank that never arrives makes the others give up after 1 s with
 * GDN_DEVERR_PEER_TIMEOUT (gdn_device_error); the group must then be rebuilt.
 * Tear-down: gdn_ipc_close_handle on the opened mappings (after a barrier),
 * gdn_peer_staging_free on the own allocation.
 */
#define GDN_IPC_HANDLE_BYTES 64
#define GDN_PEER_MAX_RANKS 8
typedef struct gdn_peer_group {
    int32_t rank, world, nblocks; /* nblocks: thread blocks per call, 1..1024, the same on every rank */
    int64_t cap;                  /* elements per staging slot */
    void* staging[GDN_PEER_MAX_RANKS];
} gdn_peer_group;
int64_t gdn_peer_staging_bytes(int32_t world, int32_t nblocks, int64_t cap);
int32_t gdn_peer_staging_alloc(int64_t bytes, void** ptr_out);
int32_t gdn_peer_staging_free(void* ptr);
int32_t gdn_ipc_get_handle(const void* dev_ptr, void* handle_out);
int32_t gdn_ipc_open_handle(const void* handle, void** dev_ptr_out);
int32_t gdn_ipc_close_handle(void* dev_ptr);
int32_t gdn_peer_allreduce_bf16(const gdn_peer_group* group, const void* in, void* out, int64_t n, void* stream);

/*
 * Fused elementwise steps of the hybrid stack's layers (bf16 only), each one
 * launch in place of PyTorch's chain of dtype copies and elementwise kernels:
 *
 * gdn_rms_norm_zc: the zero-centred RMSNorm of Qwen3_5RMSNorm
 * (config.py:118-127), out = bf16(x * rsqrt(mean(x^2) + eps) * (1 + weight))
 * in fp32 per row of `dim` elements; with `delta` (and `res_out`) the residual
 * add of the decoder layer (text.py:233-276) comes first: res_out =
 * bf16(x + delta), normalised in its place.  x rows `x_row_stride` elements
 * apart (>= dim, a multiple of 8: strided rows such as the per-head q / k norms
 * are allowed), delta likewise; res_out and out contiguous [rows, dim];
 * pointers 16-byte aligned; dim a multiple of 8.  Outputs may alias inputs.
 *
 * gdn_silu_mul: the gated MLP's act(gate) * up (text.py:215-230) for SiLU,
 * with torch's roundings: out = bf16(bf16(silu(gate)) * up), n elements, a
 * multiple of 8, 16-byte aligned.
 */
int32_t gdn_rms_norm_zc(const void* x, int64_t x_row_stride, const void* delta, int64_t delta_row_stride,
                        void* res_out, const void* weight, void* out, int64_t rows, int32_t dim, float eps,
                        void* stream);
int32_t gdn_silu_mul(const void* gate, const void* up, void* out, int64_t n, void* stream);

/*
 * The gated attention's steps around its attention kernel (bf16 only):
 *
 * gdn_qk_norm_rope: the per-head q / k RMSNorm (Qwen3_5RMSNorm, config.py:
 * 118-127, weights q_weight / k_weight [head_dim]) followed by the partial
 * rotary embedding of text.py:76-86 with torch's roundings:
 * bf16(bf16(x * cos) + bf16(rotate_half(x) * sin)) on the first rotary_dim
 * channels, the rest passed through.  qg [batch, seq_len, num_heads,
 * 2 head_dim] is the q_proj output (query, then gate, per head), k
 * [batch, seq_len, num_kv_heads, head_dim] the k_proj output, cos / sin
 * [batch, seq_len, rotary_dim]; q_out [batch, num_heads, seq_len, head_dim]
 * and k_out [batch, num_kv_heads, seq_len, head_dim] are the layouts the
 * attention reads.  head_dim a multiple of 8 up to 256, rotary_dim a multiple
 * of 16 up to head_dim, everything contiguous and 16-byte aligned.
 *
 * gdn_attn_gate_out: out = attn.transpose(1, 2).reshape(batch, seq_len,
 * num_heads * head_dim) * sigmoid(gate) (text.py:204-209), i.e.
 * bf16(o * bf16(sigmoid(g))), with o [batch, num_heads, seq_len, head_dim]
 * given by its element strides (last dimension contiguous) and the gate read
 * from qg.
 */
int32_t gdn_qk_norm_rope(const void* qg, const void* k, const void* q_weight, const void* k_weight, const void* cos,
                         const void* sin, void* q_out, void* k_out, int32_t batch, int32_t seq_len,
                         int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, int32_t rotary_dim, float eps,
                         void* stream);
int32_t gdn_attn_gate_out(const void* o, int64_t o_stride_b, int64_t o_stride_h, int64_t o_stride_t, const void* qg,
                          void* out, int32_t batch, int32_t seq_len, int32_t num_heads, int32_t head_dim,
                          void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H */
