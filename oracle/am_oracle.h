/* CPU oracle for the Llama prefill/decode hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference engine's semantics for the ops the
 * reference declares but has no kernel for (Linear with W8/W4 dequant, RoPE,
 * KV-cache update, GQA causal attention, SiLU-Mul at runtime, argmax) plus a
 * full greedy Llama forward built from them. Each function cites the reference
 * file:line it follows (paths relative to the reference project root).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use
 * this library, and only as the checker / reported CPU baseline. The product
 * (aethermind_b200) never links or calls it.
 *
 * Parity pinning: RMSNorm, Embedding, Add and the SiLU-Mul arithmetic are
 * pinned against the reference's own compiled kernels (oracle/_ref) and the
 * golden values of its unit tests. Linear/dequant/RoPE/attention/argmax have
 * no executable reference and no golden vectors in the reference tests, so
 * they are restatements of the reference's written contracts ("parity
 * unpinned" beyond those contracts); the INT4 nibble order is this project's
 * canonical choice because the reference does not define one.
 */
#ifndef AM_ORACLE_H
#define AM_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar conversions (IEEE round-to-nearest-even) ---- */
float orc_bf16_round(float f);
uint16_t orc_f32_to_bf16(float f);
float orc_bf16_to_f32(uint16_t b);
uint16_t orc_f32_to_f16(float f);
float orc_f16_to_f32(uint16_t h);

/* ---- synthetic weights (integer hash; bit-identical to the device generator) ---- */
uint64_t orc_hash(uint64_t seed, uint64_t stream, uint64_t idx);
void orc_synth_w4(uint64_t seed, uint64_t stream, int64_t N, int64_t K, float base_scale,
                  uint8_t* packed, uint16_t* scales);
void orc_synth_w8(uint64_t seed, uint64_t stream, int64_t N, int64_t K, float base_scale,
                  int8_t* q, float* scales);
void orc_synth_uniform_bf16(uint64_t seed, uint64_t stream, int64_t n, float amplitude,
                            uint16_t* out);

/* ---- INT4 canonical packing ---- */
void orc_unpack_w4(const uint8_t* packed, int64_t N, int64_t K, int8_t* q);
void orc_pack_w4(const int8_t* q, int64_t N, int64_t K, uint8_t* packed);

/* ---- ops (float storage; act_bf16 = round results to bf16) ---- */
void orc_linear_f32(const float* x, const float* w, float* y, int64_t M, int64_t N, int64_t K,
                    int act_bf16);
void orc_linear_w8(const float* x, const int8_t* q, const float* s, float* y, int64_t M,
                   int64_t N, int64_t K, int act_bf16);
void orc_linear_w4(const float* x, const uint8_t* packed, const uint16_t* s, float* y, int64_t M,
                   int64_t N, int64_t K, int64_t group, int act_bf16);
void orc_rmsnorm(const float* x, const float* w, float* y, int64_t M, int64_t H, float eps,
                 int act_bf16);
void orc_rope(float* x, const int64_t* pos, int64_t M, int64_t nheads, int64_t d, double theta,
              int act_bf16);
void orc_silu_mul(const float* g, const float* u, float* y, int64_t n, int act_bf16);
void orc_add(const float* a, const float* b, float* y, int64_t n, int act_bf16);
int64_t orc_argmax(const float* v, int64_t n);
int orc_embedding(const int64_t* ids, int64_t M, const float* table, int64_t vocab, int64_t H,
                  float* out);
/* KV cache plane [nkv][cap][d] for one layer; writes rows [pos, pos+M). */
void orc_kv_write(float* kplane, float* vplane, const float* k, const float* v, int64_t M,
                  int64_t pos, int64_t nkv, int64_t cap, int64_t d);
/* causal GQA attention: query row i sits at position pos+i and sees [0, pos+i]. */
void orc_attention(const float* q, const float* kplane, const float* vplane, float* out,
                   int64_t M, int64_t pos, int64_t nq, int64_t nkv, int64_t cap, int64_t d,
                   int act_bf16);

/* ---- full model ---- */
typedef struct {
    int fmt;  /* 0 plain fp32, 1 int8 per-channel, 2 int4 group-wise */
    int64_t N, K, group;
    const float* w;      /* fmt 0: [N,K] */
    const int8_t* q8;    /* fmt 1: [N,K] */
    const float* s8;     /* fmt 1: [N] */
    const uint8_t* q4;   /* fmt 2: [N,K/2] */
    const uint16_t* s4;  /* fmt 2: [N,K/group] fp16 */
} orc_linear;

typedef struct {
    const float* attn_norm;
    const float* mlp_norm;
    orc_linear wq, wk, wv, wo, wg, wu, wd;
} orc_layer;

typedef struct {
    int64_t vocab, hidden, layers, nq, nkv, hd, inter, max_seq;
    float eps;
    double theta;
    int act_bf16;
    const float* embed;          /* [vocab, hidden] as float values, or NULL when tied-quantized */
    orc_linear lm_head;          /* for tied int8 models this is also the embedding source */
    const float* final_norm;
    const orc_layer* layer;      /* [layers] */
} orc_model;

/* Greedy generation for one sequence. Returns number of generated tokens. */
int64_t orc_generate(const orc_model* m, const int64_t* prompt, int64_t prompt_len,
                     int64_t max_new, int64_t* out_tokens, float* last_logits_out,
                     float* top2_gap_out);

/* Wall time (s) of the prefill and of the decode steps of the last orc_generate. */
void orc_last_timing(double* prefill_s, double* decode_s);

#ifdef __cplusplus
}
#endif
#endif
