/* CPU oracle for the Llama prefill/decode hot path -- TEST INFRASTRUCTURE ONLY.
 * See am_oracle.h for scope and the pinning status of each op. Reference
 * citations are file:line within the reference project. */
#include "am_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* conversions                                                         */
/* ------------------------------------------------------------------ */
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* BFloat16(float) RNE with quiet NaN (include/aethermind/dtypes/bfloat16.h:60). */
uint16_t orc_f32_to_bf16(float f) {
    uint32_t u = f2u(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
float orc_bf16_to_f32(uint16_t b) { return u2f(((uint32_t)b) << 16); }
float orc_bf16_round(float f) { return orc_bf16_to_f32(orc_f32_to_bf16(f)); }

/* IEEE binary16 decode. */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    if (exp == 0) {
        if (man == 0) return u2f(sign);
        float v = (float)man * (1.0f / 16777216.0f); /* man * 2^-24 */
        return sign ? -v : v;
    }
    if (exp == 31) return u2f(sign | 0x7f800000u | (man << 13));
    return u2f(sign | ((exp + 112u) << 23) | (man << 13));
}

/* IEEE binary16 encode, round to nearest even. */
uint16_t orc_f32_to_f16(float f) {
    uint32_t u = f2u(f);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
    if (a < 0x38800000u) {                                   /* subnormal / zero */
        /* value = a_float; subnormal step 2^-24 */
        float v = u2f(a);
        float scaled = v * 16777216.0f; /* exact: power-of-two scaling */
        /* round half to even */
        float fl = floorf(scaled);
        float diff = scaled - fl;
        uint32_t m = (uint32_t)fl;
        if (diff > 0.5f || (diff == 0.5f && (m & 1u))) m++;
        return (uint16_t)(sign | m);
    }
    uint32_t e = (a >> 23) - 112u, man = a & 0x7fffffu;
    uint32_t r = (e << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    return (uint16_t)(sign | r);
}

/* ------------------------------------------------------------------ */
/* synthetic weights                                                   */
/* ------------------------------------------------------------------ */
uint64_t orc_hash(uint64_t seed, uint64_t stream, uint64_t idx) {
    uint64_t z = seed * 0x9E3779B97F4A7C15ull + stream * 0xD1B54A32D192ED03ull +
                 idx * 0x94D049BB133111EBull + 0x632BE59BD9B4E019ull;
    z ^= z >> 30; z *= 0xBF58476D1CE4E5B9ull;
    z ^= z >> 27; z *= 0x94D049BB133111EBull;
    z ^= z >> 31;
    return z;
}

static inline float synth_scale(uint64_t h, float base) {
    float frac = (float)(uint32_t)(h >> 48) * (0.5f / 65536.0f); /* exact */
    return base * (0.75f + frac);
}

/* q[n,k] = nibble_{k%16}(hash(seed, 2*stream, (n*K+k)/16)) - 8; scale per
 * (n, g) = fp16(base * (0.75 + u16/2^17)). Canonical packing: byte (n, k/2)
 * holds even k in the low nibble, odd k in the high nibble, two's complement. */
void orc_synth_w4(uint64_t seed, uint64_t stream, int64_t N, int64_t K, float base,
                  uint8_t* packed, uint16_t* scales) {
    const int64_t G = K / 128;
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t k16 = 0; k16 < K / 16; ++k16) {
            uint64_t h = orc_hash(seed, 2 * stream, (uint64_t)(n * K / 16 + k16));
            for (int j = 0; j < 8; ++j) {
                int lo = (int)((h >> (8 * j)) & 15u) - 8;
                int hi = (int)((h >> (8 * j + 4)) & 15u) - 8;
                packed[n * (K / 2) + k16 * 8 + j] = (uint8_t)(((unsigned)lo & 15u) | (((unsigned)hi & 15u) << 4));
            }
        }
        for (int64_t g = 0; g < G; ++g)
            scales[n * G + g] = orc_f32_to_f16(synth_scale(orc_hash(seed, 2 * stream + 1, (uint64_t)(n * G + g)), base));
    }
}

/* q[n,k] = max(byte_{k%8}(hash(seed, 2*stream, (n*K+k)/8)) - 128, -127);
 * scale[n] = base * (0.75 + u16/2^17) in fp32. */
void orc_synth_w8(uint64_t seed, uint64_t stream, int64_t N, int64_t K, float base, int8_t* q,
                  float* scales) {
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t k8 = 0; k8 < K / 8; ++k8) {
            uint64_t h = orc_hash(seed, 2 * stream, (uint64_t)(n * K / 8 + k8));
            for (int j = 0; j < 8; ++j) {
                int v = (int)((h >> (8 * j)) & 255u) - 128;
                q[n * K + k8 * 8 + j] = (int8_t)(v < -127 ? -127 : v);
            }
        }
        scales[n] = synth_scale(orc_hash(seed, 2 * stream + 1, (uint64_t)n), base);
    }
}

/* out[i] = bf16((u24 * 2^-24 - 0.5) * amplitude), u24 = top 24 bits of hash. */
void orc_synth_uniform_bf16(uint64_t seed, uint64_t stream, int64_t n, float amp, uint16_t* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        uint64_t h = orc_hash(seed, 2 * stream, (uint64_t)i);
        float u = (float)(uint32_t)(h >> 40) * (1.0f / 16777216.0f) - 0.5f;
        out[i] = orc_f32_to_bf16(u * amp);
    }
}

void orc_unpack_w4(const uint8_t* packed, int64_t N, int64_t K, int8_t* q) {
    for (int64_t n = 0; n < N; ++n)
        for (int64_t k = 0; k < K; ++k) {
            uint8_t b = packed[n * (K / 2) + k / 2];
            int nib = (k & 1) ? (b >> 4) : (b & 15);
            q[n * K + k] = (int8_t)(nib >= 8 ? nib - 16 : nib);
        }
}

void orc_pack_w4(const int8_t* q, int64_t N, int64_t K, uint8_t* packed) {
    for (int64_t n = 0; n < N; ++n)
        for (int64_t k = 0; k < K; k += 2)
            packed[n * (K / 2) + k / 2] =
                    (uint8_t)(((unsigned)q[n * K + k] & 15u) | (((unsigned)q[n * K + k + 1] & 15u) << 4));
}

/* ------------------------------------------------------------------ */
/* ops                                                                 */
/* ------------------------------------------------------------------ */
static inline float out_round(float v, int bf) { return bf ? orc_bf16_round(v) : v; }

/* Linear: y[m,n] = sum_k x[m,k] * w[n,k], W row-major [N=out, K=in]
 * (include/aethermind/operators/linear_op.h:87-91; reference scalar loop in
 * docs/designs/kernel_dev/LinearOp算子设计与实现方案_v1.0.md:393-420).
 * fp32 models accumulate in double, bf16 models in fp32 (rounded once). */
void orc_linear_f32(const float* x, const float* w, float* y, int64_t M, int64_t N, int64_t K,
                    int bf) {
#pragma omp parallel for schedule(static) collapse(2)
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n) {
            double acc = 0.0;
            for (int64_t k = 0; k < K; ++k) acc += (double)x[m * K + k] * (double)w[n * K + k];
            y[m * N + n] = out_round((float)acc, bf);
        }
}

/* W8 per-output-channel symmetric (docs/products/aethermind_prd.md:216):
 * w[n,k] = q[n,k] * s[n]; the scale is applied once per output row. */
void orc_linear_w8(const float* x, const int8_t* q, const float* s, float* y, int64_t M, int64_t N,
                   int64_t K, int bf) {
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        const int8_t* row = q + n * K;
        for (int64_t m = 0; m < M; ++m) {
            const float* xr = x + m * K;
            float acc = 0.f;
            for (int64_t k = 0; k < K; ++k) acc += xr[k] * (float)row[k];
            y[m * N + n] = out_round(acc * s[n], bf);
        }
    }
}

/* W4 group-wise symmetric, group along K, fp16 scale per (n, group)
 * (docs/products/aethermind_prd.md:216, QuantizationSpec in
 * include/aethermind/graph/graph_types.h:123-138): per group the integer
 * products are summed in fp32, then scaled and accumulated. */
void orc_linear_w4(const float* x, const uint8_t* packed, const uint16_t* s, float* y, int64_t M,
                   int64_t N, int64_t K, int64_t group, int bf) {
    const int64_t G = K / group;
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        const uint8_t* row = packed + n * (K / 2);
        for (int64_t m = 0; m < M; ++m) {
            const float* xr = x + m * K;
            float acc = 0.f;
            for (int64_t g = 0; g < G; ++g) {
                float part = 0.f;
                for (int64_t k = g * group; k < (g + 1) * group; k += 2) {
                    uint8_t b = row[k / 2];
                    int lo = (b & 15), hi = (b >> 4);
                    lo = lo >= 8 ? lo - 16 : lo;
                    hi = hi >= 8 ? hi - 16 : hi;
                    part += xr[k] * (float)lo + xr[k + 1] * (float)hi;
                }
                acc += part * orc_f16_to_f32(s[n * G + g]);
            }
            y[m * N + n] = out_round(acc, bf);
        }
    }
}

/* RMSNorm: y = x * (mean(x^2) + eps)^-1/2 * w, double accumulation
 * (src/backend/cpu/kernels/rmsnorm/rmsnorm_fp32_scalar.cpp:10-31). */
void orc_rmsnorm(const float* x, const float* w, float* y, int64_t M, int64_t H, float eps, int bf) {
    for (int64_t m = 0; m < M; ++m) {
        double ss = 0.0;
        for (int64_t j = 0; j < H; ++j) ss += (double)x[m * H + j] * (double)x[m * H + j];
        double inv = 1.0 / sqrt(ss / (double)H + (double)eps);
        for (int64_t j = 0; j < H; ++j)
            y[m * H + j] = out_round((float)((double)x[m * H + j] * inv * (double)w[j]), bf);
    }
}

/* Split-half RoPE with angles in double
 * (docs/designs/kernel_dev/RoPEOp算子设计与实现方案_v1.0.md:588-620):
 * inv_freq[i] = 1/theta^(2i/d); cos/sin rounded to float; out computed in float. */
void orc_rope(float* x, const int64_t* pos, int64_t M, int64_t nheads, int64_t d, double theta,
              int bf) {
    const int64_t half = d / 2;
    float* c = (float*)malloc(sizeof(float) * half);
    float* s = (float*)malloc(sizeof(float) * half);
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t i = 0; i < half; ++i) {
            double inv = 1.0 / pow(theta, 2.0 * (double)i / (double)d);
            double ang = (double)pos[m] * inv;
            c[i] = (float)cos(ang);
            s[i] = (float)sin(ang);
        }
        for (int64_t h = 0; h < nheads; ++h) {
            float* v = x + (m * nheads + h) * d;
            for (int64_t i = 0; i < half; ++i) {
                float x1 = v[i], x2 = v[i + half];
                v[i] = out_round(x1 * c[i] - x2 * s[i], bf);
                v[i + half] = out_round(x2 * c[i] + x1 * s[i], bf);
            }
        }
    }
    free(c);
    free(s);
}

/* silu(g)*u, sign-branched, fp32, rounded once
 * (src/graph/optimization/const_eval_silu_mul.cpp:18-33). */
void orc_silu_mul(const float* g, const float* u, float* y, int64_t n, int bf) {
    for (int64_t i = 0; i < n; ++i) {
        float gv = g[i], si;
        if (gv >= 0.f) si = gv / (1.f + expf(-gv));
        else { float e = expf(gv); si = gv * e / (1.f + e); }
        y[i] = out_round(si * u[i], bf);
    }
}

/* Residual add: float add rounded once (src/backend/cpu/kernels/add/add_scalar.cpp:56-65). */
void orc_add(const float* a, const float* b, float* y, int64_t n, int bf) {
    for (int64_t i = 0; i < n; ++i) y[i] = out_round(a[i] + b[i], bf);
}

/* argmax over the last axis; ties resolve to the lowest index
 * (src/operators/argmax_op.cpp:6-45 leaves the tie rule open). */
int64_t orc_argmax(const float* v, int64_t n) {
    int64_t best = 0;
    for (int64_t i = 1; i < n; ++i)
        if (v[i] > v[best]) best = i;
    return best;
}

/* Embedding row gather with OutOfRange on a bad id
 * (src/backend/cpu/kernels/embedding/embedding_entry.cpp:114-123). Returns 11
 * (kOutOfRange) on a bad id, 0 on success. */
int orc_embedding(const int64_t* ids, int64_t M, const float* table, int64_t vocab, int64_t H,
                  float* out) {
    for (int64_t m = 0; m < M; ++m) {
        if (ids[m] < 0 || ids[m] >= vocab) return 11;
        memcpy(out + m * H, table + ids[m] * H, sizeof(float) * H);
    }
    return 0;
}

/* KV update: rows [pos, pos+M) of plane [nkv][cap][d]
 * (src/operators/kvcache_update_op.cpp:40-49, offsets kv_cache_view.cpp:41-75). */
void orc_kv_write(float* kp, float* vp, const float* k, const float* v, int64_t M, int64_t pos,
                  int64_t nkv, int64_t cap, int64_t d) {
    for (int64_t m = 0; m < M; ++m)
        for (int64_t h = 0; h < nkv; ++h) {
            memcpy(kp + (h * cap + pos + m) * d, k + (m * nkv + h) * d, sizeof(float) * d);
            memcpy(vp + (h * cap + pos + m) * d, v + (m * nkv + h) * d, sizeof(float) * d);
        }
}

/* Causal scaled dot-product GQA attention over the static cache
 * (src/operators/attention_op.cpp:65-147; kv_head = q_head / (nq/nkv),
 * divisibility at :26-30). Softmax in double. */
void orc_attention(const float* q, const float* kp, const float* vp, float* out, int64_t M,
                   int64_t pos, int64_t nq, int64_t nkv, int64_t cap, int64_t d, int bf) {
    const int64_t grp = nq / nkv;
    const double scale = 1.0 / sqrt((double)d);
#pragma omp parallel for schedule(static) collapse(2)
    for (int64_t m = 0; m < M; ++m)
        for (int64_t h = 0; h < nq; ++h) {
            const int64_t kvh = h / grp, L = pos + m + 1;
            const float* qv = q + (m * nq + h) * d;
            double* sc = (double*)malloc(sizeof(double) * L);
            double mx = -1e300;
            for (int64_t t = 0; t < L; ++t) {
                const float* kr = kp + (kvh * cap + t) * d;
                double dot = 0.0;
                for (int64_t i = 0; i < d; ++i) dot += (double)qv[i] * (double)kr[i];
                sc[t] = dot * scale;
                if (sc[t] > mx) mx = sc[t];
            }
            double den = 0.0;
            for (int64_t t = 0; t < L; ++t) { sc[t] = exp(sc[t] - mx); den += sc[t]; }
            for (int64_t i = 0; i < d; ++i) {
                double acc = 0.0;
                for (int64_t t = 0; t < L; ++t) acc += sc[t] * (double)vp[(kvh * cap + t) * d + i];
                out[(m * nq + h) * d + i] = out_round((float)(acc / den), bf);
            }
            free(sc);
        }
}

/* ------------------------------------------------------------------ */
/* full greedy Llama forward                                           */
/* ------------------------------------------------------------------ */
static void run_linear(const orc_linear* L, const float* x, float* y, int64_t M, int bf) {
    if (L->fmt == 0) orc_linear_f32(x, L->w, y, M, L->N, L->K, bf);
    else if (L->fmt == 1) orc_linear_w8(x, L->q8, L->s8, y, M, L->N, L->K, bf);
    else orc_linear_w4(x, L->q4, L->s4, y, M, L->N, L->K, L->group, bf);
}

/* Op order of ModelGraphBuilder::BuildLlamaDense
 * (src/model/model_graph_builder.cpp:133-419): Embedding -> L x [RMSNorm,
 * q/k/v Linear, RoPE, KVCacheUpdate, Attention, o Linear, Add, RMSNorm,
 * gate/up Linear, SiluMul, down Linear, Add] -> RMSNorm -> lm_head -> Argmax. */
static void forward_chunk(const orc_model* m, const int64_t* ids, int64_t M, int64_t pos,
                          float* kc, float* vc, float* logits) {
    const int bf = m->act_bf16;
    const int64_t H = m->hidden, d = m->hd, nq = m->nq, nkv = m->nkv, I = m->inter;
    const int64_t cap = m->max_seq;
    float* x = (float*)malloc(sizeof(float) * M * H);
    float* h = (float*)malloc(sizeof(float) * M * H);
    float* q = (float*)malloc(sizeof(float) * M * nq * d);
    float* k = (float*)malloc(sizeof(float) * M * nkv * d);
    float* v = (float*)malloc(sizeof(float) * M * nkv * d);
    float* a = (float*)malloc(sizeof(float) * M * nq * d);
    float* o = (float*)malloc(sizeof(float) * M * H);
    float* g = (float*)malloc(sizeof(float) * M * I);
    float* u = (float*)malloc(sizeof(float) * M * I);
    int64_t* posv = (int64_t*)malloc(sizeof(int64_t) * M);
    for (int64_t i = 0; i < M; ++i) posv[i] = pos + i;

    /* embedding: plain table, or int8 rows of the tied lm_head dequantized */
    for (int64_t i = 0; i < M; ++i) {
        if (m->embed) memcpy(x + i * H, m->embed + ids[i] * H, sizeof(float) * H);
        else {
            const orc_linear* L = &m->lm_head;
            for (int64_t j = 0; j < H; ++j)
                x[i * H + j] = out_round((float)L->q8[ids[i] * H + j] * L->s8[ids[i]], bf);
        }
    }
    const size_t plane = (size_t)nkv * cap * d;
    for (int64_t l = 0; l < m->layers; ++l) {
        const orc_layer* Ly = &m->layer[l];
        orc_rmsnorm(x, Ly->attn_norm, h, M, H, m->eps, bf);
        run_linear(&Ly->wq, h, q, M, bf);
        run_linear(&Ly->wk, h, k, M, bf);
        run_linear(&Ly->wv, h, v, M, bf);
        orc_rope(q, posv, M, nq, d, m->theta, bf);
        orc_rope(k, posv, M, nkv, d, m->theta, bf);
        orc_kv_write(kc + l * plane, vc + l * plane, k, v, M, pos, nkv, cap, d);
        orc_attention(q, kc + l * plane, vc + l * plane, a, M, pos, nq, nkv, cap, d, bf);
        run_linear(&Ly->wo, a, o, M, bf);
        orc_add(x, o, x, M * H, bf);
        orc_rmsnorm(x, Ly->mlp_norm, h, M, H, m->eps, bf);
        run_linear(&Ly->wg, h, g, M, bf);
        run_linear(&Ly->wu, h, u, M, bf);
        orc_silu_mul(g, u, g, M * I, bf);
        run_linear(&Ly->wd, g, o, M, bf);
        orc_add(x, o, x, M * H, bf);
    }
    /* only the last row feeds the lm_head */
    orc_rmsnorm(x + (M - 1) * H, m->final_norm, h, 1, H, m->eps, bf);
    run_linear(&m->lm_head, h, logits, 1, bf);
    free(x); free(h); free(q); free(k); free(v); free(a); free(o); free(g); free(u); free(posv);
}

#include <omp.h>
static double now_s(void) { return omp_get_wtime(); }
static double g_prefill_s = 0.0, g_decode_s = 0.0;
/* Wall time of the prefill and of the decode steps of the last orc_generate. */
void orc_last_timing(double* prefill_s, double* decode_s) {
    *prefill_s = g_prefill_s;
    *decode_s = g_decode_s;
}

int64_t orc_generate(const orc_model* m, const int64_t* prompt, int64_t P, int64_t max_new,
                     int64_t* out, float* last_logits, float* gaps) {
    const size_t plane = (size_t)m->nkv * m->max_seq * m->hd;
    float* kc = (float*)calloc(plane * m->layers, sizeof(float));
    float* vc = (float*)calloc(plane * m->layers, sizeof(float));
    float* logits = (float*)malloc(sizeof(float) * m->vocab);
    int64_t n = 0;
    if (P + max_new > m->max_seq) max_new = m->max_seq - P;
    double t0 = now_s();
    forward_chunk(m, prompt, P, 0, kc, vc, logits);
    g_prefill_s = now_s() - t0;
    t0 = now_s();
    for (n = 0; n < max_new; ++n) {
        int64_t t = orc_argmax(logits, m->vocab);
        if (gaps) {
            float second = -INFINITY;
            for (int64_t i = 0; i < m->vocab; ++i)
                if (i != t && logits[i] > second) second = logits[i];
            gaps[n] = logits[t] - second;
        }
        out[n] = t;
        if (n + 1 == max_new) break;
        forward_chunk(m, &out[n], 1, P + n, kc, vc, logits);
    }
    g_decode_s = now_s() - t0;
    if (last_logits) memcpy(last_logits, logits, sizeof(float) * m->vocab);
    free(kc); free(vc); free(logits);
    return max_new > 0 ? n + 1 : 0;
}
