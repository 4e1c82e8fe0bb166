/*
 * aethermind_b200 -- C ABI of the B200-native Llama prefill/decode hot path.
 *
 * Two layers, both plain C (pointers, sizes, enums; no C++ or torch types):
 *
 *  1. amcu_* kernel launchers. Each is the CUDA drop-in for one CPU kernel (or
 *     one kernel the reference declares but has not written) of the reference
 *     engine's dispatch surface. Launchers are asynchronous on the given stream
 *     (a cudaStream_t passed as void*, NULL = legacy default stream), validate
 *     their arguments on the host and return an am_status_code. All tensor
 *     pointers are DEVICE pointers unless the field says otherwise. On failure
 *     amcu_last_error() returns a message for the calling thread.
 *
 *  2. am_* session API: the engine-level ABI the reference's product spec
 *     defines (runtime -> model -> session -> generate), run on one B200 (or
 *     one tensor-parallel rank of several). Host buffers in, host buffers out.
 *
 * Status codes, error objects and the argument-struct style are those of the
 * reference C ABI (include/c_api.h:55-88) and its SDK launchers
 * (include/aethermind/backend/cpu/kernels/rmsnorm/cpu_rmsnorm_kernel.h:13-53).
 */
#ifndef AETHERMIND_B200_H
#define AETHERMIND_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif
#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* Status and errors -- same numeric values as the reference's               */
/* am_status_code (include/c_api.h:55-74), so callers can share handling.     */
/* ------------------------------------------------------------------------ */
#ifndef AETHERMIND_C_API_H
typedef enum am_status_code {
    AM_STATUS_OK = 0,
    AM_STATUS_CANCELLED,
    AM_STATUS_UNKNOWN,
    AM_STATUS_INVALID_ARGUMENT,
    AM_STATUS_DEADLINE_EXCEEDED,
    AM_STATUS_NOT_FOUND,
    AM_STATUS_ALREADY_EXISTS,
    AM_STATUS_PERMISSION_DENIED,
    AM_STATUS_RESOURCE_EXHAUSTED,
    AM_STATUS_FAILED_PRECONDITION,
    AM_STATUS_ABORTED,
    AM_STATUS_OUT_OF_RANGE,
    AM_STATUS_UNIMPLEMENTED,
    AM_STATUS_INTERNAL,
    AM_STATUS_UNAVAILABLE,
    AM_STATUS_DATA_LOSS,
    AM_STATUS_OVERFLOW,
    AM_STATUS_UNAUTHENTICATED
} am_status_code;
typedef void* am_error_handle;
/* Replaces am_error_create/destroy/code/message (include/c_api.h:82-88). */
am_error_handle am_error_create(am_status_code code, const char* message);
void am_error_destroy(am_error_handle error);
am_status_code am_error_code(am_error_handle error);
const char* am_error_message(am_error_handle error);
#endif

/* Message of the last failing amcu_* / am_* call on this thread ("" if none). */
const char* amcu_last_error(void);
/* Library version string and the CUDA arch it was built for ("sm_100a"). */
const char* amcu_version(void);
/* Device error word of the current device: non-zero when a kernel's bounded
 * wait ran out (the kernel recorded a code and returned instead of hanging).
 * clear != 0 resets it. Synchronizes with the device. The library caches the
 * word's device address per device on first use: after cudaDeviceReset on a
 * device, kernels of this library and this call must not be used on it again
 * in the same process (the cached address belongs to the destroyed context). */
am_status_code amcu_device_error(int32_t* code, int32_t clear);

/* Element types (subset of the reference DataType used on the path). */
typedef enum amcu_dtype {
    AMCU_F32 = 0,
    AMCU_BF16 = 1,
    AMCU_F16 = 2,
    AMCU_I8 = 3,
    AMCU_I4 = 4, /* two values per byte */
    AMCU_I32 = 5,
    AMCU_I64 = 6,
    AMCU_U32 = 7
} amcu_dtype;

/* Weight formats (reference WeightFormat, include/aethermind/backend/kernel_selector.h:25-30). */
typedef enum amcu_weight_format {
    AMCU_WFMT_PLAIN = 0,   /* dense weights in the activation dtype, [N, K] row-major */
    AMCU_WFMT_INT8 = 2,    /* int8 per-output-channel symmetric, fp32 scale [N] */
    AMCU_WFMT_INT4 = 3     /* int4 group-wise symmetric, fp16 scale per (n, group of 128 along K) */
} amcu_weight_format;

/* ------------------------------------------------------------------------ */
/* Weight prepacking (replaces CpuWeightPrepacker::Pack,                      */
/* src/backend/cpu/cpu_weight_prepacker.cpp:88-119, a memcpy there).          */
/*                                                                            */
/* Canonical formats (what callers hand in):                                  */
/*   INT8: int8 q[N][K], float s[N]                                           */
/*   INT4: uint8 b[N][K/2] -- low nibble = even k, high nibble = odd k, two's */
/*         complement in [-8, 7]; uint16 (fp16 bits) s[N][K/128]             */
/*   PLAIN: act-dtype w[N][K]                                                 */
/* Device formats (what the GEMV/GEMM kernels read) are opaque; their sizes  */
/* come from amcu_packed_weight_bytes. Packing is exact: amcu_unpack_weight   */
/* returns the canonical bytes bit for bit.                                   */
/* ------------------------------------------------------------------------ */
typedef struct AmcuWeight {
    int32_t format;       /* amcu_weight_format */
    int32_t dtype;        /* PLAIN: element dtype (AMCU_F32 / AMCU_BF16) */
    int64_t n;            /* output features (rows) */
    int64_t k;            /* input features */
    int64_t group;        /* INT4 group size along K (128); ignored otherwise */
    const void* data;     /* device-format weights */
    const void* scales;   /* device-format scales (INT8; INT4 keeps them inside `data`, may be NULL) */
    int32_t gate_up_interleaved; /* 1: rows are [gate;up] interleaved by amcu_prepack_gate_up */
} AmcuWeight;

/* Bytes of the device-format weight / scale buffers (INT4: the scales are
 * part of the weight buffer and the scale buffer size is 0). */
int64_t amcu_packed_weight_bytes(int32_t format, int32_t dtype, int64_t n, int64_t k, int64_t group);
int64_t amcu_packed_scale_bytes(int32_t format, int64_t n, int64_t k, int64_t group);
/* canonical (device pointers) -> device format. */
am_status_code amcu_prepack_weight(int32_t format, int32_t dtype, int64_t n, int64_t k, int64_t group,
                                   const void* q_canonical, const void* s_canonical,
                                   void* q_packed, void* s_packed, void* stream);
/* canonical [n][k] part -> rows [row0, row0 + n) of a packed [n_total][k]
 * device weight (q_packed / s_packed point at the whole packed weight; row0 a
 * multiple of 16). Builds a fused weight (e.g. Q, K and V projections in one
 * [nq+2nkv][k] matrix) part by part, as the reference's loader fills one
 * fused tensor from several checkpoint tensors. */
am_status_code amcu_prepack_weight_rows(int32_t format, int32_t dtype, int64_t n, int64_t k, int64_t group,
                                        int64_t n_total, int64_t row0, const void* q_canonical,
                                        const void* s_canonical, void* q_packed, void* s_packed, void* stream);
/* device format -> canonical (for round-trip checks and checkpoint export). */
am_status_code amcu_unpack_weight(int32_t format, int32_t dtype, int64_t n, int64_t k, int64_t group,
                                  const void* q_packed, const void* s_packed,
                                  void* q_canonical, void* s_canonical, void* stream);
/* Fused gate/up weight for the SwiGLU MLP: packs gate[I][K] and up[I][K]
 * (canonical, same format) into one [2I][K] device weight whose GEMV/GEMM
 * epilogue emits silu(gate)*up directly. I must be a multiple of 8. */
am_status_code amcu_prepack_gate_up(int32_t format, int32_t dtype, int64_t inter, int64_t k, int64_t group,
                                    const void* gate_q, const void* gate_s,
                                    const void* up_q, const void* up_s,
                                    void* q_packed, void* s_packed, void* stream);

/* ------------------------------------------------------------------------ */
/* Synthetic weights: seeded integer-hash generators, bit-identical to the    */
/* CPU oracle's restatement; canonical formats as above.                      */
/* ------------------------------------------------------------------------ */
am_status_code amcu_synth_w4(uint64_t seed, uint64_t stream_id, int64_t n, int64_t k, float base_scale,
                             void* q_canonical, void* s_canonical, void* stream);
am_status_code amcu_synth_w8(uint64_t seed, uint64_t stream_id, int64_t n, int64_t k, float base_scale,
                             void* q_canonical, void* s_canonical, void* stream);
am_status_code amcu_synth_uniform_bf16(uint64_t seed, uint64_t stream_id, int64_t count, float amplitude,
                                       void* out, void* stream);

/* ------------------------------------------------------------------------ */
/* RMSNorm (+ optional fused residual add).                                   */
/* Replaces LaunchRmsNorm(const RmsNormArgs&)                                 */
/* (include/aethermind/backend/cpu/kernels/rmsnorm/cpu_rmsnorm_kernel.h:53)   */
/* and the Add that precedes it when residual != NULL                         */
/* (src/backend/cpu/kernels/add/add_scalar.cpp:56-65):                        */
/*   h = residual ? round(input + residual) : input ; residual_out <- h        */
/*   output = round(h * (mean(h^2) + eps)^-1/2 * weight)                      */
/* rows == 0 returns OK without touching memory (rmsnorm_entry.cpp:98-103).   */
/* ------------------------------------------------------------------------ */
typedef struct AmcuRmsNormArgs {
    const void* input;
    const void* weight;
    void* output;
    const void* residual;   /* optional */
    void* residual_out;     /* required when residual != NULL; may alias input */
    int64_t rows;
    int64_t hidden;
    int64_t input_row_stride;   /* elements; 0 = hidden */
    int64_t output_row_stride;  /* elements; 0 = hidden */
    float eps;
    int32_t dtype;              /* AMCU_F32 or AMCU_BF16 (input/output/weight) */
} AmcuRmsNormArgs;
am_status_code amcu_rmsnorm(const AmcuRmsNormArgs* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Linear: y[m, n] = sum_k x[m, k] * W[n, k]  (W [N=out, K=in], reference     */
/* LinearOp include/aethermind/operators/linear_op.h:87-91). No reference     */
/* kernel exists (LinearOp resolves NOT_FOUND); these are new.                */
/* ------------------------------------------------------------------------ */
typedef enum amcu_epilogue {
    AMCU_EPI_STORE = 0,        /* y = round(acc) */
    AMCU_EPI_RESIDUAL_ADD = 1, /* y = round(residual + round(acc)); residual may alias y */
    AMCU_EPI_SILU_MUL = 2      /* gate/up interleaved weight: y[m, i] = round(silu(round(g)) * round(u)) */
} amcu_epilogue;

/* Optional L2 prefetch hint: up to four byte ranges that the NEXT operation
 * on the stream will read (its weights and scales). The kernel asks the TMA
 * engine to pull them into L2 while it runs, spread over its CTAs, so the
 * next kernel finds its weights in L2 and HBM stays busy across kernel
 * boundaries. Pointers 16-byte aligned; sizes are rounded down to multiples
 * of 16; a NULL pointer or zero size is an unused slot. A hint never changes
 * results. (No counterpart in the reference, whose CPU kernels have no
 * device cache to fill.) */
typedef struct AmcuL2Prefetch {
    const void* ptr[4];
    uint64_t bytes[4];
} AmcuL2Prefetch;

typedef struct AmcuLinearArgs {
    const void* x;          /* [m, k] act dtype, row stride x_stride */
    AmcuWeight w;
    void* y;                /* [m, n] (SILU_MUL: [m, n/2]), row stride y_stride */
    const void* residual;   /* EPI_RESIDUAL_ADD only, row stride y_stride */
    int64_t m;
    int64_t x_stride;       /* elements; 0 = k */
    int64_t y_stride;       /* elements; 0 = n (or n/2 for SILU_MUL) */
    int32_t act_dtype;      /* AMCU_BF16 (quantized formats) or the plain weight dtype */
    int32_t epilogue;       /* amcu_epilogue */
    void* workspace;        /* device scratch (prefill GEMM); may be NULL for m <= 8 */
    size_t workspace_size;
    const void* norm_weight; /* optional: x is first RMS-normalized with this [k] weight
                                (the RMSNorm that precedes q/k/v and gate/up, fused) */
    float norm_eps;
    AmcuL2Prefetch l2_next;  /* optional: ranges the next operation reads */
    /* optional, tensor parallel, GEMV (m <= 8) with EPI_RESIDUAL_ADD only: the
     * ranks' partial products are summed over peer memory inside the GEMV's
     * epilogue, y = round(residual + round(sum over ranks of W_r x_r)), with no
     * separate all-reduce launch (areas, rank, world and wait_limit_us of
     * amcu_allreduce_oneshot_add are used; part, x and n are ignored). */
    const struct AmcuAllReduceArgs* peer_reduce;
} AmcuLinearArgs;
/* Dispatches on m: GEMV (m <= 8) or the tensor-core GEMM (m > 8). */
am_status_code amcu_linear(const AmcuLinearArgs* args, void* stream);
/* Bytes of workspace amcu_linear needs for these arguments (0 if none). */
size_t amcu_linear_workspace_bytes(const AmcuLinearArgs* args);
/* Decode GEMVs (m <= 8): W8 per-channel and W4 group-128. */
am_status_code amcu_gemv_w8(const AmcuLinearArgs* args, void* stream);
am_status_code amcu_gemv_w4g128(const AmcuLinearArgs* args, void* stream);
/* Prefill GEMMs (any m >= 1): dequant-to-bf16 tensor-core GEMM. */
am_status_code amcu_gemm_w8_prefill(const AmcuLinearArgs* args, void* stream);
am_status_code amcu_gemm_w4g128_prefill(const AmcuLinearArgs* args, void* stream);

/* ------------------------------------------------------------------------ */
/* RoPE + KV-cache write (replaces the RoPE and KVCacheUpdate nodes,          */
/* src/operators/rope_op.cpp:202-223, src/operators/kvcache_update_op.cpp).   */
/* Split-half rotation with inv_freq[i] = theta^(-2i/d) and angles in double  */
/* (reference RoPE design doc). Row r belongs to sequence b = r / rows_per_seq */
/* at position seq_pos[b] + r % rows_per_seq. q is rotated in place; k is     */
/* rotated and, with v, stored at cache[b][kv_head][pos][:]                   */
/* (layout of src/execution/kv_cache_view.cpp:41-75 with a leading slot axis).*/
/* ------------------------------------------------------------------------ */
typedef struct AmcuRopeKvArgs {
    void* q;                 /* [rows, n_q_heads * head_dim] (in place) */
    const void* k;           /* [rows, n_kv_heads * head_dim] */
    const void* v;           /* [rows, n_kv_heads * head_dim] */
    int64_t q_stride, k_stride, v_stride;   /* row strides in elements */
    void* k_cache;           /* this layer's K plane: [slots][n_kv][capacity][head_dim] */
    void* v_cache;
    int64_t slot_stride;     /* elements between slots (n_kv * capacity * head_dim if 0) */
    int64_t capacity;        /* max tokens per slot */
    const int32_t* seq_pos;  /* device [n_seq]: position of each sequence's first row */
    int64_t rows;
    int64_t rows_per_seq;
    int64_t n_q_heads, n_kv_heads, head_dim;
    double theta;
    int32_t dtype;           /* AMCU_F32 / AMCU_BF16 (activations and cache) */
    int32_t* status;         /* optional device word: set to AM_STATUS_OUT_OF_RANGE on a position >= capacity */
    const float* cos_sin;    /* optional table from amcu_rope_table (same values, no per-token trig) */
} AmcuRopeKvArgs;
am_status_code amcu_rope_kv_write(const AmcuRopeKvArgs* args, void* stream);
/* cos/sin table for positions [0, max_pos): table[pos][i] = (cos, sin) of
 * pos * theta^(-2i/head_dim), i < head_dim/2, computed in double and rounded
 * to float exactly as amcu_rope_kv_write does on the fly. 8*max_pos*(head_dim/2) bytes. */
am_status_code amcu_rope_table(double theta, int64_t head_dim, int64_t max_pos, float* table, void* stream);

/* ------------------------------------------------------------------------ */
/* GQA attention over the static KV cache (reference InferAttention,          */
/* src/operators/attention_op.cpp:65-169): causal scaled dot-product,         */
/* kv_head = q_head / (n_q/n_kv). Query row r of sequence b sits at position  */
/* seq_pos[b] + r % rows_per_seq and sees cache positions [0, that position]. */
/* Decode (rows_per_seq == 1): split-K over the sequence with a combine step; */
/* needs workspace (amcu_attention_workspace_bytes). Prefill: flash tiles.    */
/* ------------------------------------------------------------------------ */
typedef struct AmcuAttentionArgs {
    const void* q;           /* [rows, n_q_heads * head_dim] */
    int64_t q_stride;
    const void* k_cache;     /* [slots][n_kv][capacity][head_dim] */
    const void* v_cache;
    int64_t slot_stride;
    int64_t capacity;
    const int32_t* seq_pos;  /* device [n_seq] */
    void* out;               /* [rows, n_q_heads * head_dim] */
    int64_t out_stride;
    int64_t rows;
    int64_t rows_per_seq;
    int64_t n_q_heads, n_kv_heads, head_dim;
    int32_t dtype;           /* AMCU_F32 / AMCU_BF16 */
    int32_t num_splits;      /* decode only: 0 = choose from max_context */
    int64_t max_context;     /* upper bound on position+1 (sizes the split grid) */
    void* workspace;
    size_t workspace_size;
} AmcuAttentionArgs;
size_t amcu_attention_workspace_bytes(const AmcuAttentionArgs* args);
am_status_code amcu_attn_decode(const AmcuAttentionArgs* args, void* stream);
/* ------------------------------------------------------------------------ */
/* Persistent decode step (no single counterpart in the reference: it runs  */
/* every decoder layer of BuildLlamaDense -- attention RMSNorm, q/k/v        */
/* Linear, RoPE, KVCacheUpdate, Attention, o Linear + Add, MLP RMSNorm,      */
/* gate/up Linear + SiluMul, down Linear + Add -- for one decode step of a   */
/* batch-1, INT4 g128, bf16 model in one cooperative launch; one CTA per SM   */
/* streams its share of every layer's weights without pausing at the layer   */
/* or phase boundaries). hidden, inter and n_q*head_dim: multiples of 128,   */
/* at most 16384.                                                             */
/* ------------------------------------------------------------------------ */
typedef struct AmcuDecodeLayer {   /* one decoder layer, device pointers */
    const void* w_qkv;             /* INT4 [(nq + 2 nkv) * head_dim][hidden], device format */
    const void* w_o;               /* INT4 [hidden][nq * head_dim] */
    const void* w_gate_up;         /* INT4 [2 inter][hidden] from amcu_prepack_gate_up */
    const void* w_down;            /* INT4 [hidden][inter] */
    const void* attn_norm;         /* bf16 [hidden] */
    const void* mlp_norm;          /* bf16 [hidden] */
    void* k_cache;                 /* this layer's K plane [slots][nkv][capacity][head_dim] */
    void* v_cache;
} AmcuDecodeLayer;
typedef struct AmcuDecodeStackArgs {
    const AmcuDecodeLayer* layers; /* device array of n_layers descriptors */
    int64_t n_layers;
    int64_t batch;                 /* sequences: 1 */
    int64_t hidden, inter, n_q_heads, n_kv_heads, head_dim;
    void* x;                       /* [batch][hidden] bf16 residual stream, updated in place */
    void* qkv;                     /* [batch][(nq + 2 nkv) * head_dim] bf16 scratch */
    void* attn;                    /* unused (the attention output is merged inside the step) */
    void* act;                     /* [batch][inter] bf16 scratch */
    const int32_t* seq_pos;        /* [batch] position of each sequence's token */
    int64_t capacity, slot_stride; /* KV cache (slot_stride 0: n_kv * capacity * head_dim) */
    const float* cos_sin;          /* optional amcu_rope_table table */
    double theta;
    float rms_eps;
    int32_t* status;               /* optional: AM_STATUS_OUT_OF_RANGE on a position >= capacity */
    void* workspace;               /* amcu_decode_stack_workspace_bytes, 256-byte aligned, ZERO before the */
    size_t workspace_size;         /* first call (its counters reset themselves after every call) */
} AmcuDecodeStackArgs;
size_t amcu_decode_stack_workspace_bytes(const AmcuDecodeStackArgs* args);
am_status_code amcu_decode_stack(const AmcuDecodeStackArgs* args, void* stream);

/* Fused decode step: amcu_rope_kv_write(rope) then amcu_attn_decode(attn) in
 * one launch (bf16, one row per sequence; attn->q == rope->q, same caches and
 * positions). The rotated q is used on chip and NOT written back to rope->q;
 * the rotated k and v of the token are appended to the cache as
 * amcu_rope_kv_write does. No workspace: the split-K partials are merged
 * through distributed shared memory of a thread-block cluster. */
am_status_code amcu_attn_decode_rope(const AmcuRopeKvArgs* rope, const AmcuAttentionArgs* attn, void* stream);
am_status_code amcu_attn_prefill(const AmcuAttentionArgs* args, void* stream);
/* Decode attention that allocates nothing (no counterpart in the reference).
 * For callers that cannot allocate device memory while they run: a server
 * that reserves all of HBM at start-up and forbids later allocations, or a
 * latency-critical step where cudaMalloc's implicit synchronization is not
 * acceptable. Same kernels and result as amcu_attn_decode; the split-K
 * partials go to a 4 MiB scratch array built into the library (held on every
 * GPU that loads it, until exit) instead of args->workspace (ignored).
 * Sizes whose scratch (amcu_attention_workspace_bytes) exceeds 4 MiB are
 * rejected with AM_STATUS_INVALID_ARGUMENT. The first call on a device looks
 * up the scratch's device address; make that first call before any stream
 * capture. All calls share the one scratch: calls that overlap on the GPU
 * (e.g. on different streams) race and must be serialized by the caller.
 * The scratch address is cached per device for the life of the process:
 * do not call this after cudaDeviceReset on that device. */
am_status_code amcu_attn_decode_noalloc(const AmcuAttentionArgs* args, void* stream);

/* ------------------------------------------------------------------------ */
/* SiLU-Mul: out = round(silu(gate) * up), sign-branched fp32 SiLU            */
/* (src/graph/optimization/const_eval_silu_mul.cpp:18-33).                   */
/* ------------------------------------------------------------------------ */
am_status_code amcu_silu_mul(const void* gate, const void* up, void* out, int64_t count,
                             int32_t dtype, void* stream);
/* Residual add: out = round(a + b) (src/backend/cpu/kernels/add/add_scalar.cpp:56-65). */
am_status_code amcu_add(const void* a, const void* b, void* out, int64_t count, int32_t dtype,
                        void* stream);

/* ------------------------------------------------------------------------ */
/* Greedy argmax over the last axis (src/operators/argmax_op.cpp:6-45);      */
/* ties resolve to the lowest index. out_index: int64 [rows].                */
/* Optional out_gap: float [rows] = max - second max (near-tie detection).   */
/* ------------------------------------------------------------------------ */
am_status_code amcu_argmax(const void* logits, int64_t rows, int64_t vocab, int64_t row_stride,
                           int32_t dtype, int64_t* out_index, float* out_gap, void* stream);
/* Same result, split over many CTAs per row (for vocabularies of 10^5):
 * needs a device workspace of amcu_argmax_workspace_bytes(rows) bytes. */
size_t amcu_argmax_workspace_bytes(int64_t rows);
am_status_code amcu_argmax_ws(const void* logits, int64_t rows, int64_t vocab, int64_t row_stride,
                              int32_t dtype, int64_t* out_index, float* out_gap, void* workspace,
                              size_t workspace_size, void* stream);

/* ------------------------------------------------------------------------ */
/* Embedding gather (src/backend/cpu/kernels/embedding/embedding_entry.cpp:  */
/* 32-126). ids: int32/int64/uint32 [count]. table: act-dtype [vocab, hidden] */
/* or INT8 rows + fp32 row scales (tied int8 lm_head), dequantized to bf16.  */
/* A bad id leaves its row zero and, if status != NULL, sets *status (device) */
/* to AM_STATUS_OUT_OF_RANGE.                                                 */
/* ------------------------------------------------------------------------ */
typedef struct AmcuEmbeddingArgs {
    const void* ids;
    int32_t id_dtype;        /* AMCU_I32 / AMCU_I64 / AMCU_U32 */
    int64_t count;
    const void* table;
    const float* row_scales; /* non-NULL: table is int8 rows */
    int64_t vocab, hidden;
    void* out;               /* [count, hidden] */
    int32_t dtype;           /* output dtype AMCU_F32 / AMCU_BF16 */
    int32_t* status;
} AmcuEmbeddingArgs;
am_status_code amcu_embedding(const AmcuEmbeddingArgs* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Offline weight quantizer and dtype conversion (checkpoint loading). The    */
/* reference declares INT8 per-channel / INT4 group-wise weight-only formats */
/* (docs/products/aethermind_prd.md:216; QuantizationSpec,                    */
/* include/aethermind/graph/graph_types.h:123-138) but has no quantizer.      */
/* Symmetric absmax, written in the canonical formats above:                  */
/*   INT4: s = fp16(max|w| / 7) per (row, group of 128), q = clamp(rint(w/s), */
/*         -8, 7); INT8: s = max|w| / 127 per row, q = clamp(rint(w/s), ±127). */
/* w: device [n][k] in AMCU_F32 / AMCU_BF16 / AMCU_F16.                       */
/* ------------------------------------------------------------------------ */
am_status_code amcu_quantize_weight(int32_t format, const void* w, int32_t w_dtype, int64_t n, int64_t k,
                                    int64_t group, void* q, void* scales, void* stream);
/* dst[i] = src[i] converted (f32 / bf16 / f16 -> f32 / bf16, round to nearest even). */
am_status_code amcu_convert(const void* src, int32_t src_dtype, void* dst, int32_t dst_dtype, int64_t count,
                            void* stream);

/* ------------------------------------------------------------------------ */
/* One-shot all-reduce + residual add over peer memory (tensor-parallel      */
/* decode): x = round(x + round(sum over ranks of part_r)), bf16, n elements. */
/* Replaces the per-block NCCL all-reduce that tensor-parallel row splits     */
/* need after o_proj / down_proj; the reference engine runs on one device and */
/* has no collective (its LayerRunner, src/execution/layer_runner.cpp:24-93, */
/* would call it after those Linears).                                        */
/* areas[r]: rank r's exchange area as mapped in this process (own area       */
/* included; peers' through CUDA IPC), each amcu_allreduce_area_bytes()       */
/* bytes, zeroed before first use. The wait for the peers is bounded by       */
/* wait_limit_us (0: about 2 s); when it runs out the kernel records 0x401 in */
/* the device error word (amcu_device_error) and returns instead of hanging.  */
/* ------------------------------------------------------------------------ */
typedef struct AmcuAllReduceArgs {
    const void* part;      /* this rank's bf16 partial [n] */
    void* x;               /* bf16 residual [n], updated in place */
    int64_t n;             /* multiple of 8, at most 65536 */
    int32_t rank, world;   /* world in [2, 8] */
    void* areas[8];
    uint64_t wait_limit_us;
} AmcuAllReduceArgs;
size_t amcu_allreduce_area_bytes(void);
am_status_code amcu_allreduce_oneshot_add(const AmcuAllReduceArgs* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Session API (reference product spec: docs/products/aethermind_prd.md:     */
/* 296-320; the reference has not implemented it).                          */
/* ------------------------------------------------------------------------ */
typedef struct am_runtime_s* am_runtime_t;
typedef struct am_model_s* am_model_t;
typedef struct am_session_s* am_session_t;
typedef am_error_handle am_error_t;

typedef struct am_config_t {
    int32_t device_id;       /* CUDA device of this process */
    int32_t tp_rank;         /* tensor-parallel rank (0 for 1 GPU) */
    int32_t tp_size;         /* tensor-parallel world size (1 for 1 GPU) */
    const void* nccl_unique_id;  /* 128-byte ncclUniqueId shared by all ranks (tp_size > 1) */
} am_config_t;

typedef struct am_model_config_t {
    int64_t vocab, hidden, layers, n_q_heads, n_kv_heads, head_dim, inter;
    float rms_eps;
    double rope_theta;
    int32_t tied_embeddings;
    int32_t act_dtype;       /* AMCU_F32 (plain fp32 weights) or AMCU_BF16 */
    int32_t weight_format;   /* amcu_weight_format */
    int64_t group_size;      /* 128 for INT4 */
    int64_t max_seq;         /* static KV capacity per sequence */
    int64_t max_batch;       /* sequences per generate call (KV slots) */
} am_model_config_t;

typedef struct am_session_config_t {
    int64_t max_new_tokens;
    int32_t use_cuda_graph;  /* 1: decode steps replay a captured CUDA graph */
    int32_t unfused_attention; /* 1: decode RoPE and attention as two launches (default 0: one fused
                                  launch, amcu_attn_decode_rope, where the dtype has one) */
    int32_t persistent_decode; /* 1: all decoder layers of a bs <= 2 INT4 decode step in one persistent
                                  launch (amcu_decode_stack); default 0: one launch per op, faster today */
} am_session_config_t;

am_runtime_t am_runtime_create(const am_config_t* config);
void am_runtime_destroy(am_runtime_t runtime);

/* Weights from a Hugging Face Llama checkpoint directory (the reference's
 * ModelLoader::Load, src/model/model_loader.cpp:12-55): config.json plus
 * model.safetensors or model.safetensors.index.json and its shards; F32, BF16
 * or F16 tensors, quantized on the device at load time. am_model_load uses the
 * default options: INT4 g128 weights, bf16 activations, max_seq =
 * min(max_position_embeddings, 4096), max_batch 1. Errors: NOT_FOUND for a
 * missing directory or file, INVALID_ARGUMENT for a malformed config, header,
 * missing tensor or shape mismatch, UNIMPLEMENTED for rope scaling. */
typedef struct am_load_options_t {
    int32_t weight_format;   /* AMCU_WFMT_INT4 (0 = default), AMCU_WFMT_INT8 or AMCU_WFMT_PLAIN */
    int32_t act_dtype;       /* AMCU_BF16 (default) or AMCU_F32 (plain weights only) */
    int64_t max_seq;         /* 0: min(max_position_embeddings, 4096) */
    int64_t max_batch;       /* 0: 1 */
} am_load_options_t;
am_model_t am_model_load(am_runtime_t runtime, const char* path, am_error_t* error);
am_model_t am_model_load_ex(am_runtime_t runtime, const char* path, const am_load_options_t* options,
                            am_error_t* error);
/* Creates a model with device storage for every weight (uninitialised). */
am_model_t am_model_create(am_runtime_t runtime, const am_model_config_t* config, am_error_t* error);
/* Fills every weight from the seeded synthetic generator on the device. */
am_status_code am_model_init_synthetic(am_model_t model, uint64_t seed);
/* Sets one weight from HOST memory in canonical format. Names:
 * "embed" [vocab, hidden]; "final_norm" [hidden]; "lm_head" (untied);
 * "layers.<i>.{attn_norm,mlp_norm}" [hidden];
 * "layers.<i>.{wq,wk,wv,wo,wg,wu,wd}" -- data = q / plain weights, scales = scales.
 * For tp_size > 1 pass the FULL tensor; the rank keeps its shard. */
am_status_code am_model_set_weight(am_model_t model, const char* name, const void* data,
                                   const void* scales);
void am_model_unload(am_model_t model);

am_session_t am_session_create(am_model_t model, const am_session_config_t* config);
void am_session_destroy(am_session_t session);
/* Greedy generation for one sequence: prefill input_tokens, then decode until
 * output_capacity tokens (or the session's max_new_tokens). Host buffers. */
int am_session_generate(am_session_t session, const uint32_t* input_tokens, size_t input_len,
                        uint32_t* output_tokens, size_t output_capacity, size_t* output_len,
                        am_error_t* error);
/* Batched variant: batch sequences of equal prompt length, row-major
 * input [batch][input_len], output [batch][output_capacity]. */
int am_session_generate_batch(am_session_t session, const uint32_t* input_tokens, size_t batch,
                              size_t input_len, uint32_t* output_tokens, size_t output_capacity,
                              size_t* output_len, am_error_t* error);
/* Device-timed phases of the last generate call (CUDA events), in ms. */
am_status_code am_session_last_timing(am_session_t session, double* prefill_ms, double* decode_ms,
                                      int64_t* decode_steps);
/* Optional: logits top-1/top-2 gap per generated token of the last call
 * (host float [batch][n]) for near-tie diagnostics. */
am_status_code am_session_last_gaps(am_session_t session, float* gaps, size_t capacity);

/* Tensor parallelism: rank 0 creates the 128-byte NCCL unique id and shares it
 * with the other ranks (any transport) before am_runtime_create. */
am_status_code am_nccl_get_unique_id(void* out128);
/* One-shot all-reduce over peer memory for the decode steps (no counterpart
 * in the reference, whose engine runs on one device). After am_runtime_create
 * with tp_size > 1, every rank exports its exchange area as a 64-byte CUDA IPC
 * handle, the ranks share them (any transport), and each rank opens the
 * others' with the tp_size x 64 bytes in rank order. Sessions created
 * afterwards reduce the o/down partials of messages up to 65536 elements with
 * one kernel (sum + residual add) instead of NCCL + an add. Same node only. */
am_status_code am_runtime_peer_handle(am_runtime_t runtime, void* out64);
am_status_code am_runtime_open_peers(am_runtime_t runtime, const void* handles);
/* Message of the last failing am_* session call on this thread. */
const char* am_last_error(void);
/* Diagnostics: number of registered CUDA kernels, and the resolved kernel of
 * every step of a plan (phase 0 = prefill, 1 = decode) as text lines. */
int64_t am_debug_registry_size(void);
am_status_code am_debug_plan_steps(am_session_t session, int32_t phase, int64_t batch, int64_t rows_per_seq,
                                   char* buf, size_t capacity);
/* Kernel resolution through the CUDA backend's registry (no GPU needed):
 * op = reference OpType value, act/weight = amcu_dtype, format = reference
 * WeightFormat value (0 plain, 2 int8, 3 int4), phase 0 prefill / 1 decode /
 * 2 both. Writes the resolved kernel name; NOT_FOUND when none matches. */
am_status_code am_debug_resolve_kernel(int32_t op, int32_t act, int32_t weight, int32_t format, int32_t phase,
                                       char* name, size_t capacity);
/* KV layout offset (bytes) and bytes per plane exactly as the HBM KV manager
 * computes them (layout only, nothing is allocated). */
am_status_code am_debug_kv_offset(uint64_t layers, uint64_t kv_heads, uint64_t max_tokens, uint64_t head_dim,
                                  int32_t dtype, uint64_t slots, uint64_t layer, uint64_t kv_head, uint64_t pos,
                                  uint64_t dim, uint64_t slot, uint64_t* offset, uint64_t* bytes_per_plane);
/* Session reservation contract of the KV manager (capacity checks only). */
am_status_code am_debug_kv_reserve(uint64_t max_tokens, uint64_t prompt_len, uint64_t max_new);
/* The tensor-parallel block a rank keeps of a full [n, k] layer tensor
 * ("wq".."wd", norms, "embed", "lm_head"): out4 = {row0, rows, col0, cols},
 * the same rule the model uses when it shards weights (no reference
 * counterpart; the reference runs on one device). Host only. */
am_status_code am_debug_tp_shard(const char* tensor, int64_t n, int64_t k, int32_t rank, int32_t world,
                                 int64_t* out4);

#ifdef __cplusplus
}
#endif
#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#endif
