// Fused RoPE + KV-cache write.
//
// Semantics: split-half (HF Llama) rotary embedding of the reference RoPE
// design (docs/designs/kernel_dev/RoPEOp算子设计与实现方案_v1.0.md:588-620):
// inv_freq[i] = 1 / theta^(2i/d), angle = pos * inv_freq in double, cos/sin
// rounded to float, out[i] = x1*c - x2*s, out[i+d/2] = x2*c + x1*s in float
// (no fused multiply-add, so the result is the exact float expression).
// K (rotated) and V rows then go to cache[slot][kv_head][pos][:] -- the
// per-layer layout of KVCacheLayout::Offset (src/execution/kv_cache_view.cpp:41-75)
// with a leading slot axis for batched sequences.
#include "../amcu_internal.h"
#include "common.cuh"

namespace amcu {

template <typename T>
__global__ void __launch_bounds__(128) rope_kv_kernel(AmcuRopeKvArgs a) {
    const int64_t row = blockIdx.x;
    const int64_t b = row / a.rows_per_seq;
    const int64_t pos = (int64_t)a.seq_pos[b] + row % a.rows_per_seq;
    const int64_t d = a.head_dim, half = d / 2;
    if (pos < 0 || pos >= a.capacity) {
        if (a.status && threadIdx.x == 0) atomicExch(a.status, (int32_t)AM_STATUS_OUT_OF_RANGE);
        return;
    }
    extern __shared__ float cs[];  // [half] cos, [half] sin
    for (int64_t i = threadIdx.x; i < half; i += blockDim.x) {
        const double inv = 1.0 / pow(a.theta, 2.0 * (double)i / (double)d);
        const double ang = (double)pos * inv;
        cs[i] = (float)cos(ang);
        cs[half + i] = (float)sin(ang);
    }
    __syncthreads();
    T* q = static_cast<T*>(a.q) + row * a.q_stride;
    const T* k = static_cast<const T*>(a.k) + row * a.k_stride;
    const T* v = static_cast<const T*>(a.v) + row * a.v_stride;
    const int64_t slot_stride = a.slot_stride ? a.slot_stride : a.n_kv_heads * a.capacity * d;
    T* kc = static_cast<T*>(a.k_cache) + b * slot_stride + pos * d;
    T* vc = static_cast<T*>(a.v_cache) + b * slot_stride + pos * d;
    const int64_t nq = a.n_q_heads * half, nk = a.n_kv_heads * half;
    for (int64_t e = threadIdx.x; e < nq + nk; e += blockDim.x) {
        const bool is_q = e < nq;
        const int64_t ee = is_q ? e : e - nq;
        const int64_t h = ee / half, i = ee % half;
        const T* src = is_q ? q + h * d : k + h * d;
        const float x1 = Act<T>::load(src[i]), x2 = Act<T>::load(src[i + half]);
        const float c = cs[i], s = cs[half + i];
        const float o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
        const float o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
        if (is_q) {
            q[h * d + i] = Act<T>::store(o1);
            q[h * d + i + half] = Act<T>::store(o2);
        } else {
            T* dst = kc + h * a.capacity * d;
            dst[i] = Act<T>::store(o1);
            dst[i + half] = Act<T>::store(o2);
        }
    }
    for (int64_t e = threadIdx.x; e < a.n_kv_heads * d; e += blockDim.x) {
        const int64_t h = e / d, i = e % d;
        vc[h * a.capacity * d + i] = v[e];
    }
}

}  // namespace amcu

using namespace amcu;

extern "C" am_status_code amcu_rope_kv_write(const AmcuRopeKvArgs* a, void* stream) {
    clear_error();
    AMCU_REQUIRE(a != nullptr, "amcu_rope_kv_write: null args");
    AMCU_REQUIRE(a->rows >= 0, "amcu_rope_kv_write: negative rows");
    if (a->rows == 0) return AM_STATUS_OK;
    AMCU_REQUIRE(a->q && a->k && a->v && a->k_cache && a->v_cache && a->seq_pos, "amcu_rope_kv_write: null pointer");
    AMCU_REQUIRE(a->head_dim > 0 && a->head_dim % 2 == 0, "amcu_rope_kv_write: head_dim must be even");
    AMCU_REQUIRE(a->n_q_heads > 0 && a->n_kv_heads > 0 && a->n_q_heads % a->n_kv_heads == 0,
                 "amcu_rope_kv_write: n_q_heads must be a positive multiple of n_kv_heads");
    AMCU_REQUIRE(a->rows_per_seq > 0, "amcu_rope_kv_write: rows_per_seq must be positive");
    AMCU_REQUIRE(a->capacity > 0, "amcu_rope_kv_write: capacity must be positive");
    AMCU_REQUIRE(a->theta > 0.0, "amcu_rope_kv_write: theta must be positive");
    const size_t smem = sizeof(float) * a->head_dim;
    if (a->dtype == AMCU_F32)
        rope_kv_kernel<float><<<(unsigned)a->rows, 128, smem, as_stream(stream)>>>(*a);
    else if (a->dtype == AMCU_BF16)
        rope_kv_kernel<__nv_bfloat16><<<(unsigned)a->rows, 128, smem, as_stream(stream)>>>(*a);
    else
        return set_error(AM_STATUS_INVALID_ARGUMENT, "amcu_rope_kv_write: dtype must be f32 or bf16");
    return check_launch("amcu_rope_kv_write");
}
