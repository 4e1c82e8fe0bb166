// RMSNorm (+fused residual add), residual Add, SiLU-Mul, embedding gather,
// greedy argmax and the seeded synthetic-weight generators.
#include "../amcu_internal.h"
#include "common.cuh"

namespace amcu {

// ---------------------------------------------------------------------------
// RMSNorm. One CTA per row. Semantics of RmsNormKernel_CPU_FP32_Scalar
// (src/backend/cpu/kernels/rmsnorm/rmsnorm_fp32_scalar.cpp:10-31): the sum of
// squares is accumulated in fp32 here (the reference's AVX2 kernel does the
// same; its scalar kernel uses double) and the product x*inv_rms*w rounds once.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const T* __restrict__ in, const T* __restrict__ w,
                                                      T* __restrict__ out, const T* __restrict__ res,
                                                      T* res_out, int64_t hidden, int64_t in_stride,
                                                      int64_t out_stride, float eps) {
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.x;
    const T* x = in + row * in_stride;
    const T* r = res ? res + row * in_stride : nullptr;
    T* ro = res ? res_out + row * in_stride : nullptr;
    float ss = 0.f;
    for (int64_t j = threadIdx.x; j < hidden; j += blockDim.x) {
        float v = Act<T>::load(x[j]);
        if (r) {
            v = Act<T>::round(v + Act<T>::load(r[j]));
            ro[j] = Act<T>::store(v);
        }
        ss += v * v;
    }
    __shared__ float red[32];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = 1.0f / sqrtf(red[0] / (float)hidden + eps);
    const T* src = r ? ro : x;
    T* y = out + row * out_stride;
    for (int64_t j = threadIdx.x; j < hidden; j += blockDim.x) {
        const float v = Act<T>::load(src[j]);
        y[j] = Act<T>::store(v * inv * Act<T>::load(w[j]));
    }
}

// bf16 rows of at most 8 * 256 * CH elements (hidden % 8 == 0, 16-byte
// aligned rows): 16-byte loads, the row kept in registers between the sum of
// squares and the scaling; per element the same arithmetic as rmsnorm_kernel.
template <int CH>
__global__ void __launch_bounds__(256) rmsnorm_bf16_vec_kernel(const __nv_bfloat16* __restrict__ in,
                                                               const __nv_bfloat16* __restrict__ w,
                                                               __nv_bfloat16* __restrict__ out,
                                                               const __nv_bfloat16* __restrict__ res,
                                                               __nv_bfloat16* res_out, int64_t hidden, int64_t in_stride,
                                                               int64_t out_stride, float eps) {
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.x;
    const int nch = (int)(hidden / 8);
    const __nv_bfloat16* x = in + row * in_stride;
    float v[CH][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int j = threadIdx.x + c * blockDim.x;
        if (j >= nch) continue;
        uint4 u = ld_u4(x + j * 8);
        const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&u);
        if (res) {
            uint4 ru = ld_u4(res + row * in_stride + j * 8);
            const __nv_bfloat16* re = reinterpret_cast<const __nv_bfloat16*>(&ru);
            uint4 o;
            __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                v[c][e] = Act<__nv_bfloat16>::round(__bfloat162float(xe[e]) + __bfloat162float(re[e]));
                oe[e] = __float2bfloat16_rn(v[c][e]);
            }
            *reinterpret_cast<uint4*>(res_out + row * in_stride + j * 8) = o;
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) v[c][e] = __bfloat162float(xe[e]);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += v[c][e] * v[c][e];
    }
    __shared__ float red[32];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = 1.0f / sqrtf(red[0] / (float)hidden + eps);
    __nv_bfloat16* y = out + row * out_stride;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int j = threadIdx.x + c * blockDim.x;
        if (j >= nch) continue;
        uint4 wu = ld_u4(w + j * 8);
        const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wu);
        uint4 o;
        __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
        for (int e = 0; e < 8; ++e) oe[e] = __float2bfloat16_rn(v[c][e] * inv * __bfloat162float(we[e]));
        *reinterpret_cast<uint4*>(y + j * 8) = o;
    }
}

template <typename T>
__global__ void add_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ o, int64_t n) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        o[i] = Act<T>::store(Act<T>::load(a[i]) + Act<T>::load(b[i]));
}

template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ o, int64_t n) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        o[i] = Act<T>::store(silu_ref(Act<T>::load(g[i])) * Act<T>::load(u[i]));
}

// ---------------------------------------------------------------------------
// Embedding gather (src/backend/cpu/kernels/embedding/embedding_entry.cpp:114-123).
// ---------------------------------------------------------------------------
template <typename T, typename Id>
__global__ void embedding_kernel(const Id* __restrict__ ids, const void* __restrict__ table,
                                 const float* __restrict__ row_scales, int64_t vocab, int64_t hidden,
                                 T* __restrict__ out, int32_t* status) {
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.x;
    const int64_t id = (int64_t)ids[row];
    T* o = out + row * hidden;
    if (id < 0 || id >= vocab) {
        for (int64_t j = threadIdx.x; j < hidden; j += blockDim.x) o[j] = Act<T>::store(0.f);
        if (status && threadIdx.x == 0) atomicExch(status, (int32_t)AM_STATUS_OUT_OF_RANGE);
        return;
    }
    if (row_scales) {
        const int8_t* q = static_cast<const int8_t*>(table) + id * hidden;
        const float s = row_scales[id];
        for (int64_t j = threadIdx.x; j < hidden; j += blockDim.x) o[j] = Act<T>::store((float)q[j] * s);
    } else {
        const T* t = static_cast<const T*>(table) + id * hidden;
        for (int64_t j = threadIdx.x; j < hidden; j += blockDim.x) o[j] = t[j];
    }
}

// ---------------------------------------------------------------------------
// Greedy argmax, one CTA per row, ties -> lowest index; also reports the gap
// between the best and second-best logit for near-tie diagnostics.
// ---------------------------------------------------------------------------
struct Top2 {
    float v1;
    int64_t i1;
    float v2;
};
__device__ __forceinline__ bool better(float v, int64_t i, float bv, int64_t bi) {
    return v > bv || (v == bv && i < bi);
}
__device__ __forceinline__ Top2 merge_top2(Top2 a, Top2 b) {
    Top2 r;
    if (better(b.v1, b.i1, a.v1, a.i1)) {
        r.v1 = b.v1; r.i1 = b.i1; r.v2 = fmaxf(a.v1, b.v2);
    } else {
        r.v1 = a.v1; r.i1 = a.i1; r.v2 = fmaxf(a.v2, b.v1);
    }
    return r;
}
template <typename T>
__global__ void __launch_bounds__(1024) argmax_kernel(const T* __restrict__ logits, int64_t vocab, int64_t stride,
                                                      int64_t* __restrict__ out_idx, float* __restrict__ out_gap) {
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.x;
    const T* l = logits + row * stride;
    Top2 t{-INFINITY, INT64_MAX, -INFINITY};
    for (int64_t j = threadIdx.x; j < vocab; j += blockDim.x) {
        const float v = Act<T>::load(l[j]);
        if (better(v, j, t.v1, t.i1)) { t.v2 = t.v1; t.v1 = v; t.i1 = j; }
        else if (v > t.v2) t.v2 = v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Top2 u;
        u.v1 = __shfl_xor_sync(0xffffffffu, t.v1, o);
        u.i1 = __shfl_xor_sync(0xffffffffu, t.i1, o);
        u.v2 = __shfl_xor_sync(0xffffffffu, t.v2, o);
        t = merge_top2(t, u);
    }
    __shared__ Top2 red[32];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = t;
    __syncthreads();
    if (threadIdx.x == 0) {
        Top2 b = red[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) b = merge_top2(b, red[w]);
        out_idx[row] = b.i1 == INT64_MAX ? 0 : b.i1;
        if (out_gap) out_gap[row] = b.v1 - b.v2;
    }
}

// Two-phase argmax for long rows: `parts` CTAs per row each reduce a slice
// with 16-byte loads into a Top2 partial; one CTA per row merges them.
constexpr int kArgmaxParts = 64;
template <typename T>
__global__ void __launch_bounds__(256) argmax_partial_kernel(const T* __restrict__ logits, int64_t vocab,
                                                             int64_t stride, Top2* __restrict__ parts) {
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.y;
    const T* l = logits + row * stride;
    constexpr int V = 16 / sizeof(T);
    const int64_t nvec = vocab / V;
    const int64_t per = (nvec + gridDim.x - 1) / gridDim.x;
    const int64_t v0 = blockIdx.x * per, v1 = v0 + per < nvec ? v0 + per : nvec;
    Top2 t{-INFINITY, INT64_MAX, -INFINITY};
    auto consider = [&](float v, int64_t j) {
        if (better(v, j, t.v1, t.i1)) { t.v2 = t.v1; t.v1 = v; t.i1 = j; }
        else if (v > t.v2) t.v2 = v;
    };
    const bool aligned16 = (reinterpret_cast<uintptr_t>(l) & 15) == 0;
    if (aligned16) {
        for (int64_t vi = v0 + threadIdx.x; vi < v1; vi += blockDim.x) {
            const uint4 u = *reinterpret_cast<const uint4*>(l + vi * V);
            const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
            for (int j = 0; j < V; ++j) consider(Act<T>::load(e[j]), vi * V + j);
        }
    } else {
        for (int64_t j = v0 * V + threadIdx.x; j < v1 * V; j += blockDim.x) consider(Act<T>::load(l[j]), j);
    }
    if (blockIdx.x == gridDim.x - 1)  // ragged tail (vocab % V)
        for (int64_t j = nvec * V + threadIdx.x; j < vocab; j += blockDim.x) consider(Act<T>::load(l[j]), j);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Top2 u;
        u.v1 = __shfl_xor_sync(0xffffffffu, t.v1, o);
        u.i1 = __shfl_xor_sync(0xffffffffu, t.i1, o);
        u.v2 = __shfl_xor_sync(0xffffffffu, t.v2, o);
        t = merge_top2(t, u);
    }
    __shared__ Top2 red[8];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = t;
    __syncthreads();
    if (threadIdx.x == 0) {
        Top2 b = red[0];
        for (int w = 1; w < 8; ++w) b = merge_top2(b, red[w]);
        parts[row * gridDim.x + blockIdx.x] = b;
    }
}

__global__ void argmax_final_kernel(const Top2* __restrict__ parts, int nparts, int64_t* __restrict__ out_idx,
                                    float* __restrict__ out_gap) {
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.x;
    Top2 t{-INFINITY, INT64_MAX, -INFINITY};
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) t = merge_top2(t, parts[row * nparts + i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Top2 u;
        u.v1 = __shfl_xor_sync(0xffffffffu, t.v1, o);
        u.i1 = __shfl_xor_sync(0xffffffffu, t.i1, o);
        u.v2 = __shfl_xor_sync(0xffffffffu, t.v2, o);
        t = merge_top2(t, u);
    }
    if (threadIdx.x == 0) {
        out_idx[row] = t.i1 == INT64_MAX ? 0 : t.i1;
        if (out_gap) out_gap[row] = t.v1 - t.v2;
    }
}

// ---------------------------------------------------------------------------
// Synthetic weights: integer-hash generators; the fp32 arithmetic is exact
// except the final multiply and the fp16/bf16 conversion, all IEEE
// round-to-nearest-even, so the CPU oracle regenerates identical bits.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t synth_hash(uint64_t seed, uint64_t stream, uint64_t idx) {
    uint64_t z = seed * 0x9E3779B97F4A7C15ull + stream * 0xD1B54A32D192ED03ull + idx * 0x94D049BB133111EBull +
                 0x632BE59BD9B4E019ull;
    z ^= z >> 30;
    z *= 0xBF58476D1CE4E5B9ull;
    z ^= z >> 27;
    z *= 0x94D049BB133111EBull;
    z ^= z >> 31;
    return z;
}
__device__ __forceinline__ float synth_scale(uint64_t h, float base) {
    const float frac = __fmul_rn((float)(uint32_t)(h >> 48), 0.5f / 65536.0f);
    return __fmul_rn(base, __fadd_rn(0.75f, frac));
}

__global__ void synth_w4_kernel(uint64_t seed, uint64_t stream, int64_t N, int64_t K, float base,
                                uint8_t* __restrict__ packed, __half* __restrict__ scales) {
    const int64_t units = N * (K / 16), G = K / 128;
    for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units + N * G;
         u += (int64_t)gridDim.x * blockDim.x) {
        if (u < units) {
            const uint64_t h = synth_hash(seed, 2 * stream, (uint64_t)u);
            uint2 out;
            uint32_t w[2] = {0, 0};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t lo = (uint32_t)((h >> (8 * j)) & 15u);        // nibble value + 8 of q
                const uint32_t hi = (uint32_t)((h >> (8 * j + 4)) & 15u);
                const uint32_t byte = ((lo ^ 8u) & 15u) | (((hi ^ 8u) & 15u) << 4);
                w[j >> 2] |= byte << (8 * (j & 3));
            }
            out.x = w[0];
            out.y = w[1];
            // unit u covers row n = u / (K/16), k = (u % (K/16)) * 16 -> 8 bytes
            *reinterpret_cast<uint2*>(packed + u * 8) = out;
        } else {
            const int64_t s = u - units;
            scales[s] = __float2half_rn(synth_scale(synth_hash(seed, 2 * stream + 1, (uint64_t)s), base));
        }
    }
}

__global__ void synth_w8_kernel(uint64_t seed, uint64_t stream, int64_t N, int64_t K, float base,
                                int8_t* __restrict__ q, float* __restrict__ scales) {
    const int64_t units = N * (K / 8);
    for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units + N;
         u += (int64_t)gridDim.x * blockDim.x) {
        if (u < units) {
            const uint64_t h = synth_hash(seed, 2 * stream, (uint64_t)u);
            uint32_t w[2] = {0, 0};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                int v = (int)((h >> (8 * j)) & 255u) - 128;
                v = v < -127 ? -127 : v;
                w[j >> 2] |= ((uint32_t)(uint8_t)(int8_t)v) << (8 * (j & 3));
            }
            *reinterpret_cast<uint2*>(q + u * 8) = make_uint2(w[0], w[1]);
        } else {
            const int64_t n = u - units;
            scales[n] = synth_scale(synth_hash(seed, 2 * stream + 1, (uint64_t)n), base);
        }
    }
}

__global__ void synth_uniform_bf16_kernel(uint64_t seed, uint64_t stream, int64_t n, float amp,
                                          __nv_bfloat16* __restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint64_t h = synth_hash(seed, 2 * stream, (uint64_t)i);
        const float u = __fadd_rn(__fmul_rn((float)(uint32_t)(h >> 40), 1.0f / 16777216.0f), -0.5f);
        out[i] = __float2bfloat16_rn(__fmul_rn(u, amp));
    }
}

static int grid_for(int64_t n, int threads) {
    int64_t b = (n + threads - 1) / threads;
    const int64_t cap = (int64_t)num_sms() * 16;
    if (b > cap) b = cap;
    return (int)(b < 1 ? 1 : b);
}

}  // namespace amcu

using namespace amcu;

extern "C" {

am_status_code amcu_rmsnorm(const AmcuRmsNormArgs* a, void* stream) {
    clear_error();
    AMCU_REQUIRE(a != nullptr, "amcu_rmsnorm: null args");
    AMCU_REQUIRE(a->rows >= 0, "amcu_rmsnorm: requires non-negative rows");
    AMCU_REQUIRE(a->hidden > 0, "amcu_rmsnorm: requires positive hidden");
    if (a->rows == 0) return AM_STATUS_OK;
    AMCU_REQUIRE(a->input && a->weight && a->output, "amcu_rmsnorm: null data pointer");
    AMCU_REQUIRE(!a->residual || a->residual_out, "amcu_rmsnorm: residual requires residual_out");
    AMCU_REQUIRE(a->dtype == AMCU_F32 || a->dtype == AMCU_BF16, "amcu_rmsnorm: dtype must be f32 or bf16");
    const int64_t is = a->input_row_stride ? a->input_row_stride : a->hidden;
    const int64_t os = a->output_row_stride ? a->output_row_stride : a->hidden;
    AMCU_REQUIRE(is >= a->hidden && os >= a->hidden, "amcu_rmsnorm: row stride smaller than hidden");
    const int threads = a->hidden >= 1024 ? 256 : 128;
    if (a->dtype == AMCU_F32)
        launch_pdl(rmsnorm_kernel<float>, dim3((unsigned)a->rows), dim3(threads), 0, as_stream(stream), 
                (const float*)a->input, (const float*)a->weight, (float*)a->output, (const float*)a->residual,
                (float*)a->residual_out, a->hidden, is, os, a->eps);
    else if (a->hidden % 8 == 0 && a->hidden <= 8 * 256 * 4 && is % 8 == 0 && os % 8 == 0 &&
             aligned(a->input, 16) && aligned(a->weight, 16) && aligned(a->output, 16) &&
             (!a->residual || (aligned(a->residual, 16) && aligned(a->residual_out, 16))))
        launch_pdl(rmsnorm_bf16_vec_kernel<4>, dim3((unsigned)a->rows), dim3(256), 0, as_stream(stream),
                   (const __nv_bfloat16*)a->input, (const __nv_bfloat16*)a->weight, (__nv_bfloat16*)a->output,
                   (const __nv_bfloat16*)a->residual, (__nv_bfloat16*)a->residual_out, a->hidden, is, os, a->eps);
    else
        launch_pdl(rmsnorm_kernel<__nv_bfloat16>, dim3((unsigned)a->rows), dim3(threads), 0, as_stream(stream), 
                (const __nv_bfloat16*)a->input, (const __nv_bfloat16*)a->weight, (__nv_bfloat16*)a->output,
                (const __nv_bfloat16*)a->residual, (__nv_bfloat16*)a->residual_out, a->hidden, is, os, a->eps);
    return check_launch("amcu_rmsnorm");
}

am_status_code amcu_add(const void* x, const void* y, void* out, int64_t n, int32_t dtype, void* stream) {
    clear_error();
    AMCU_REQUIRE(n >= 0, "amcu_add: negative count");
    if (n == 0) return AM_STATUS_OK;
    AMCU_REQUIRE(x && y && out, "amcu_add: null pointer");
    AMCU_REQUIRE(dtype == AMCU_F32 || dtype == AMCU_BF16, "amcu_add: dtype must be f32 or bf16");
    if (dtype == AMCU_F32)
        launch_pdl(add_kernel<float>, dim3(grid_for(n, 256)), dim3(256), 0, as_stream(stream), (const float*)x, (const float*)y,
                                                                          (float*)out, n);
    else
        launch_pdl(add_kernel<__nv_bfloat16>, dim3(grid_for(n, 256)), dim3(256), 0, as_stream(stream), 
                (const __nv_bfloat16*)x, (const __nv_bfloat16*)y, (__nv_bfloat16*)out, n);
    return check_launch("amcu_add");
}

am_status_code amcu_silu_mul(const void* g, const void* u, void* out, int64_t n, int32_t dtype, void* stream) {
    clear_error();
    AMCU_REQUIRE(n >= 0, "amcu_silu_mul: negative count");
    if (n == 0) return AM_STATUS_OK;
    AMCU_REQUIRE(g && u && out, "amcu_silu_mul: null pointer");
    AMCU_REQUIRE(dtype == AMCU_F32 || dtype == AMCU_BF16, "amcu_silu_mul: dtype must be f32 or bf16");
    if (dtype == AMCU_F32)
        launch_pdl(silu_mul_kernel<float>, dim3(grid_for(n, 256)), dim3(256), 0, as_stream(stream), (const float*)g, (const float*)u,
                                                                               (float*)out, n);
    else
        launch_pdl(silu_mul_kernel<__nv_bfloat16>, dim3(grid_for(n, 256)), dim3(256), 0, as_stream(stream), 
                (const __nv_bfloat16*)g, (const __nv_bfloat16*)u, (__nv_bfloat16*)out, n);
    return check_launch("amcu_silu_mul");
}

am_status_code amcu_embedding(const AmcuEmbeddingArgs* a, void* stream) {
    clear_error();
    AMCU_REQUIRE(a != nullptr, "amcu_embedding: null args");
    AMCU_REQUIRE(a->count >= 0 && a->vocab > 0 && a->hidden > 0, "amcu_embedding: bad sizes");
    if (a->count == 0) return AM_STATUS_OK;
    AMCU_REQUIRE(a->ids && a->table && a->out, "amcu_embedding: null pointer");
    AMCU_REQUIRE(a->id_dtype == AMCU_I32 || a->id_dtype == AMCU_I64 || a->id_dtype == AMCU_U32,
                 "amcu_embedding: token ids must be int32, int64, or uint32");
    AMCU_REQUIRE(a->dtype == AMCU_F32 || a->dtype == AMCU_BF16, "amcu_embedding: dtype must be f32 or bf16");
    const dim3 grid((unsigned)a->count);
    cudaStream_t s = as_stream(stream);
#define AMCU_EMB(T, ID) \
    launch_pdl(embedding_kernel<T, ID>, grid, dim3(256), 0, s, (const ID*)a->ids, a->table, a->row_scales, a->vocab, a->hidden, (T*)a->out, a->status)
    if (a->dtype == AMCU_F32) {
        if (a->id_dtype == AMCU_I32) AMCU_EMB(float, int32_t);
        else if (a->id_dtype == AMCU_I64) AMCU_EMB(float, int64_t);
        else AMCU_EMB(float, uint32_t);
    } else {
        if (a->id_dtype == AMCU_I32) AMCU_EMB(__nv_bfloat16, int32_t);
        else if (a->id_dtype == AMCU_I64) AMCU_EMB(__nv_bfloat16, int64_t);
        else AMCU_EMB(__nv_bfloat16, uint32_t);
    }
#undef AMCU_EMB
    return check_launch("amcu_embedding");
}

am_status_code amcu_argmax(const void* logits, int64_t rows, int64_t vocab, int64_t stride, int32_t dtype,
                           int64_t* out_idx, float* out_gap, void* stream) {
    clear_error();
    AMCU_REQUIRE(rows >= 0 && vocab > 0, "amcu_argmax: bad sizes");
    if (rows == 0) return AM_STATUS_OK;
    AMCU_REQUIRE(logits && out_idx, "amcu_argmax: null pointer");
    if (stride == 0) stride = vocab;
    AMCU_REQUIRE(stride >= vocab, "amcu_argmax: row stride smaller than vocab");
    if (dtype == AMCU_F32)
        launch_pdl(argmax_kernel<float>, dim3((unsigned)rows), dim3(1024), 0, as_stream(stream), (const float*)logits, vocab, stride,
                                                                             out_idx, out_gap);
    else if (dtype == AMCU_BF16)
        launch_pdl(argmax_kernel<__nv_bfloat16>, dim3((unsigned)rows), dim3(1024), 0, as_stream(stream), 
                (const __nv_bfloat16*)logits, vocab, stride, out_idx, out_gap);
    else
        return set_error(AM_STATUS_INVALID_ARGUMENT, "amcu_argmax: dtype must be f32 or bf16");
    return check_launch("amcu_argmax");
}

size_t amcu_argmax_workspace_bytes(int64_t rows) {
    return rows > 0 ? (size_t)rows * kArgmaxParts * sizeof(Top2) : 0;
}

am_status_code amcu_argmax_ws(const void* logits, int64_t rows, int64_t vocab, int64_t stride, int32_t dtype,
                              int64_t* out_idx, float* out_gap, void* workspace, size_t workspace_size,
                              void* stream) {
    clear_error();
    AMCU_REQUIRE(rows >= 0 && vocab > 0, "amcu_argmax_ws: bad sizes");
    if (rows == 0) return AM_STATUS_OK;
    AMCU_REQUIRE(logits && out_idx, "amcu_argmax_ws: null pointer");
    if (stride == 0) stride = vocab;
    AMCU_REQUIRE(stride >= vocab, "amcu_argmax_ws: row stride smaller than vocab");
    AMCU_REQUIRE(workspace && workspace_size >= amcu_argmax_workspace_bytes(rows) && aligned(workspace, 16),
                 "amcu_argmax_ws: workspace of %zu bytes (16-byte aligned) required", amcu_argmax_workspace_bytes(rows));
    const dim3 grid(kArgmaxParts, (unsigned)rows);
    Top2* parts = static_cast<Top2*>(workspace);
    if (dtype == AMCU_F32)
        launch_pdl(argmax_partial_kernel<float>, grid, dim3(256), 0, as_stream(stream), (const float*)logits, vocab, stride, parts);
    else if (dtype == AMCU_BF16)
        launch_pdl(argmax_partial_kernel<__nv_bfloat16>, grid, dim3(256), 0, as_stream(stream), (const __nv_bfloat16*)logits, vocab,
                                                                                  stride, parts);
    else
        return set_error(AM_STATUS_INVALID_ARGUMENT, "amcu_argmax_ws: dtype must be f32 or bf16");
    launch_pdl(argmax_final_kernel, dim3((unsigned)rows), dim3(32), 0, as_stream(stream), parts, kArgmaxParts, out_idx, out_gap);
    return check_launch("amcu_argmax_ws");
}

am_status_code amcu_synth_w4(uint64_t seed, uint64_t sid, int64_t n, int64_t k, float base, void* q, void* s,
                             void* stream) {
    clear_error();
    AMCU_REQUIRE(n > 0 && k > 0 && k % 128 == 0, "amcu_synth_w4: k must be a positive multiple of 128");
    AMCU_REQUIRE(q && s && aligned(q, 8), "amcu_synth_w4: null or misaligned pointer");
    synth_w4_kernel<<<grid_for(n * (k / 16) + n * (k / 128), 256), 256, 0, as_stream(stream)>>>(
            seed, sid, n, k, base, (uint8_t*)q, (__half*)s);
    return check_launch("amcu_synth_w4");
}

am_status_code amcu_synth_w8(uint64_t seed, uint64_t sid, int64_t n, int64_t k, float base, void* q, void* s,
                             void* stream) {
    clear_error();
    AMCU_REQUIRE(n > 0 && k > 0 && k % 8 == 0, "amcu_synth_w8: k must be a positive multiple of 8");
    AMCU_REQUIRE(q && s && aligned(q, 8), "amcu_synth_w8: null or misaligned pointer");
    synth_w8_kernel<<<grid_for(n * (k / 8) + n, 256), 256, 0, as_stream(stream)>>>(seed, sid, n, k, base,
                                                                                   (int8_t*)q, (float*)s);
    return check_launch("amcu_synth_w8");
}

am_status_code amcu_synth_uniform_bf16(uint64_t seed, uint64_t sid, int64_t count, float amp, void* out,
                                       void* stream) {
    clear_error();
    AMCU_REQUIRE(count >= 0 && out, "amcu_synth_uniform_bf16: bad arguments");
    if (count == 0) return AM_STATUS_OK;
    synth_uniform_bf16_kernel<<<grid_for(count, 256), 256, 0, as_stream(stream)>>>(seed, sid, count, amp,
                                                                                   (__nv_bfloat16*)out);
    return check_launch("amcu_synth_uniform_bf16");
}

}  // extern "C"
