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

__global__ void rope_table_kernel(double theta, int64_t d, int64_t max_pos, float2* table) {
    const int64_t half = d / 2;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < max_pos * half;
         e += (int64_t)gridDim.x * blockDim.x) {
        float c, s;
        rope_angle(theta, d, e / half, e % half, c, s);
        table[e] = make_float2(c, s);
    }
}

// One CTA per row; its threads walk the work items of all heads: heads
// [0, nq) are query heads (rotated in place), [nq, nq + nkv) key heads
// (rotated into the cache), the last nkv value heads (copied into the cache).
// A rotation item is two adjacent pairs (i, i + d/2), (i + 1, i + 1 + d/2),
// loaded and stored as two-element vectors; a value item is two elements.
template <typename T>
struct Pair2;
template <>
struct Pair2<float> {
    using V = float2;
    static __device__ __forceinline__ void get(const V& v, float& a, float& b) { a = v.x; b = v.y; }
    static __device__ __forceinline__ V make(float a, float b) { return make_float2(a, b); }
};
template <>
struct Pair2<__nv_bfloat16> {
    using V = __nv_bfloat162;
    static __device__ __forceinline__ void get(const V& v, float& a, float& b) {
        a = __low2float(v);
        b = __high2float(v);
    }
    static __device__ __forceinline__ V make(float a, float b) { return __floats2bfloat162_rn(a, b); }
};

template <typename T>
__global__ void __launch_bounds__(256) rope_kv_kernel(AmcuRopeKvArgs a) {
    using P2 = Pair2<T>;
    using V = typename P2::V;
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.x;
    const int64_t b = row / a.rows_per_seq;
    const int64_t pos = (int64_t)a.seq_pos[b] + row % a.rows_per_seq;
    const int64_t d = a.head_dim, half = d / 2, hp = half / 2;  // hp rotation items per head
    if (pos < 0 || pos >= a.capacity) {
        if (a.status && threadIdx.x == 0) atomicExch(a.status, (int32_t)AM_STATUS_OUT_OF_RANGE);
        return;
    }
    const int64_t slot_stride = a.slot_stride ? a.slot_stride : a.n_kv_heads * a.capacity * d;
    const int64_t nq = a.n_q_heads, nkv = a.n_kv_heads;
    const int64_t rot_items = (nq + nkv) * hp, items = rot_items + nkv * (d / 2);
    for (int64_t e = threadIdx.x; e < items; e += blockDim.x) {
        if (e >= rot_items) {  // value head: copy two elements
            const int64_t f = e - rot_items, h = f / (d / 2), c = 2 * (f % (d / 2));
            const V v = *reinterpret_cast<const V*>(static_cast<const T*>(a.v) + row * a.v_stride + h * d + c);
            *reinterpret_cast<V*>(static_cast<T*>(a.v_cache) + b * slot_stride + (h * a.capacity + pos) * d + c) = v;
            continue;
        }
        const int64_t head = e / hp, i = 2 * (e % hp);
        const bool is_q = head < nq;
        const T* src = is_q ? static_cast<const T*>(a.q) + row * a.q_stride + head * d
                            : static_cast<const T*>(a.k) + row * a.k_stride + (head - nq) * d;
        float x1[2], x2[2];
        P2::get(*reinterpret_cast<const V*>(src + i), x1[0], x1[1]);
        P2::get(*reinterpret_cast<const V*>(src + i + half), x2[0], x2[1]);
        float o1[2], o2[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            float c, sn;
            if (a.cos_sin) {
                const float2 cs = reinterpret_cast<const float2*>(a.cos_sin)[pos * half + i + j];
                c = cs.x;
                sn = cs.y;
            } else {
                rope_angle(a.theta, d, pos, i + j, c, sn);
            }
            o1[j] = __fsub_rn(__fmul_rn(x1[j], c), __fmul_rn(x2[j], sn));
            o2[j] = __fadd_rn(__fmul_rn(x2[j], c), __fmul_rn(x1[j], sn));
        }
        T* dst = is_q ? static_cast<T*>(a.q) + row * a.q_stride + head * d
                      : static_cast<T*>(a.k_cache) + b * slot_stride + ((head - nq) * a.capacity + pos) * d;
        *reinterpret_cast<V*>(dst + i) = P2::make(o1[0], o1[1]);
        *reinterpret_cast<V*>(dst + i + half) = P2::make(o2[0], o2[1]);
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
    AMCU_REQUIRE(a->head_dim % 4 == 0, "amcu_rope_kv_write: head_dim must be a multiple of 4");
    {
        const int64_t es = a->dtype == AMCU_F32 ? 8 : 4;  // bytes of a two-element vector
        const int64_t qs = a->q_stride, ks = a->k_stride, vs = a->v_stride;
        AMCU_REQUIRE(aligned(a->q, es) && aligned(a->k, es) && aligned(a->v, es) && aligned(a->k_cache, es) &&
                             aligned(a->v_cache, es) && qs % 2 == 0 && ks % 2 == 0 && vs % 2 == 0 &&
                             a->slot_stride % 2 == 0,
                     "amcu_rope_kv_write: rows must start on two-element boundaries");
    }
    const dim3 grid((unsigned)a->rows);
    if (a->dtype == AMCU_F32)
        launch_pdl(rope_kv_kernel<float>, grid, dim3(256), 0, as_stream(stream), *a);
    else if (a->dtype == AMCU_BF16)
        launch_pdl(rope_kv_kernel<__nv_bfloat16>, grid, dim3(256), 0, as_stream(stream), *a);
    else
        return set_error(AM_STATUS_INVALID_ARGUMENT, "amcu_rope_kv_write: dtype must be f32 or bf16");
    return check_launch("amcu_rope_kv_write");
}

extern "C" am_status_code amcu_rope_table(double theta, int64_t head_dim, int64_t max_pos, float* table, void* stream) {
    clear_error();
    AMCU_REQUIRE(table && head_dim > 0 && head_dim % 2 == 0 && max_pos > 0 && theta > 0.0,
                 "amcu_rope_table: bad arguments");
    AMCU_REQUIRE(aligned(table, 8), "amcu_rope_table: table must be 8-byte aligned");
    const int64_t n = max_pos * (head_dim / 2);
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    rope_table_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(theta, head_dim, max_pos,
                                                                       reinterpret_cast<float2*>(table));
    return check_launch("amcu_rope_table");
}
