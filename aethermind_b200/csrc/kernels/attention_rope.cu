// Fused decode step of the attention block: RoPE of q and k, the KV-cache
// append of this token, split-K attention over the cache and the merge of the
// splits, in one launch.
//
// Semantics: exactly amcu_rope_kv_write followed by amcu_attn_decode (the
// reference's RoPE, KVCacheUpdate and Attention nodes,
// src/operators/rope_op.cpp:202-223, src/operators/kvcache_update_op.cpp:142-158,
// src/operators/attention_op.cpp:151-169), except that the rotated q is not
// written back: it is rounded to bf16 as the in-place store would round it
// and used on chip.
//
// Layout of the work: one thread-block cluster per (sequence, kv head), its
// CTAs splitting the sequence [0, pos] into equal chunks of whole 8-key
// blocks. Every CTA rotates the GRP query heads itself; the CTA whose chunk
// holds `pos` also rotates k and appends k and v to the cache before reading
// its chunk. Each CTA merges its warps into a (max, sum, unnormalised output)
// partial in shared memory; after a cluster barrier every CTA combines a
// slice of the outputs by reading all partials through distributed shared
// memory, and a second barrier keeps the partials alive until all reads are
// done. No workspace, no second kernel.
#include <cooperative_groups.h>

#include <cstdlib>

#include "../amcu_internal.h"
#include "attn_decode.cuh"
#include "common.cuh"
#include "diag_timeline.cuh"

namespace cg = cooperative_groups;

namespace amcu {

// Warps per CTA of the fused kernel. 8 warps halve a CTA's key loop at
// context ~520 (2.3 against 3.6 us), but 16-CTA clusters of 256 threads
// become resident only as the q/k/v GEMV drains: the launch spans 14.6 us
// against 9.3 and the 8B decode runs 588 against 623 tok/s.
#ifndef AMCU_RA_WARPS
#define AMCU_RA_WARPS 4
#endif
constexpr int kRaWarps = AMCU_RA_WARPS;
constexpr int kRaThreads = kRaWarps * 32;
constexpr int kRaTargetCtas = 256;  // CTAs of one launch the cluster size aims at (batch 8, 8 kv heads: 4 per cluster)

struct RopeAttnParams {
    const __nv_bfloat16 *q, *k, *v;
    int64_t q_stride, k_stride, v_stride;
    __nv_bfloat16 *kc, *vc;
    int64_t slot_stride, capacity;
    const int32_t* seq_pos;
    int32_t* status;
    const float* cos_sin;
    double theta;
    __nv_bfloat16* out;
    int64_t out_stride;
    float scale_log2;
};

template <int GRP, int D, int CS>
__global__ void __launch_bounds__(kRaThreads) attn_rope_decode_kernel(RopeAttnParams p) {
    cg::cluster_group cluster = cg::this_cluster();
    DiagTl tl;
    tl.entry();
    const int rank = (int)cluster.block_rank();
    const int kvh = blockIdx.y;
    const int64_t row = blockIdx.z;  // one row per sequence
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Before the dependency wait: the position and the cache rows below it
    // were written by earlier decode steps, which have all completed by the
    // time this kernel can start (only the preceding q/k/v projection may
    // still be running).
    const int64_t pos = p.seq_pos[row];
    if (pos < 0 || pos >= p.capacity) {  // the whole cluster leaves together
        pdl_wait();
        if (rank == 0 && kvh == 0 && threadIdx.x == 0 && p.status) atomicExch(p.status, (int32_t)AM_STATUS_OUT_OF_RANGE);
        return;
    }
    const int64_t L = pos + 1;
    int64_t chunk = (L + CS - 1) / CS;
    chunk = (chunk + 7) / 8 * 8;
    const int64_t k_begin = (int64_t)rank * chunk;
    const int64_t k_end = k_begin + chunk < L ? k_begin + chunk : L;
    __nv_bfloat16* kbase = p.kc + row * p.slot_stride + (int64_t)kvh * p.capacity * D;
    __nv_bfloat16* vbase = p.vc + row * p.slot_stride + (int64_t)kvh * p.capacity * D;
    DecodeKeyLoop<GRP, D, kRaWarps> loop(kbase, vbase, k_begin, k_end, warp, lane);
    loop.load_first(pos);  // keys below pos are final

    pdl_wait();
    pdl_trigger();
    tl.waited();

    __shared__ __align__(16) float qs[GRP][D];
    __shared__ float sm_m[kRaWarps][GRP], sm_l[kRaWarps][GRP];
    __shared__ float sm_o[kRaWarps][GRP][D];
    __shared__ float pm[GRP], pl[GRP];
    __shared__ float po[GRP][D];

    rope_stage_q<GRP, D>(p.q + row * p.q_stride + (int64_t)kvh * GRP * D, pos, p.cos_sin, p.theta, p.scale_log2, qs,
                         threadIdx.x, kRaThreads);
    if (k_begin <= pos && pos < k_end)  // this CTA's chunk holds the new token: append it
        rope_append_kv<D>(p.k + row * p.k_stride + (int64_t)kvh * D, p.v + row * p.v_stride + (int64_t)kvh * D,
                          kbase + pos * D, vbase + pos * D, pos, p.cos_sin, p.theta, threadIdx.x, kRaThreads);
    __syncthreads();  // q staged; the appended row is visible to this CTA's reads
    if (threadIdx.x == 0) tl.mark2();

    DecodeWarpState<GRP, D> st;
    loop.run(qs, st);
    if (threadIdx.x == 0) tl.mark();
    decode_publish_warp<GRP, D>(st, warp, lane, sm_m, sm_l, sm_o);
    __syncthreads();
    for (int e = threadIdx.x; e < GRP * D; e += kRaThreads) {
        const int h = e / D, dd = e % D;
        float M, Ls, O;
        decode_merge_warps<GRP, D, kRaWarps>(h, dd, sm_m, sm_l, sm_o, M, Ls, O);
        po[h][dd] = O;
        if (dd == 0) {
            pm[h] = M;
            pl[h] = Ls;
        }
    }
    cluster.sync();  // every CTA's partial is complete

    // This CTA combines outputs [rank * per, (rank + 1) * per); all CS
    // partials of an element are fetched with independent loads. Once every
    // read of the other CTAs' shared memory is done the CTA arrives on the
    // cluster barrier, stores its outputs, and only then waits: the partials
    // stay alive until every CTA has read them, and the store overlaps the
    // barrier.
    constexpr int per = GRP * D / CS;
    constexpr int kIter = (per + kRaThreads - 1) / kRaThreads;
    float res[kIter];
#pragma unroll
    for (int it = 0; it < kIter; ++it) {
        const int j = threadIdx.x + it * kRaThreads;
        res[it] = 0.f;
        if (j >= per) continue;
        const int e = rank * per + j;
        const int h = e / D;
        float mr[CS], lr[CS], orr[CS];
#pragma unroll
        for (int r = 0; r < CS; ++r) {
            mr[r] = cluster.map_shared_rank(pm, r)[h];
            lr[r] = cluster.map_shared_rank(pl, r)[h];
            orr[r] = cluster.map_shared_rank(&po[0][0], r)[e];
        }
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < CS; ++r) M = fmaxf(M, mr[r]);
        float Ls = 0.f, O = 0.f;
#pragma unroll
        for (int r = 0; r < CS; ++r) {
            const float f = mr[r] == -INFINITY ? 0.f : exp2f(mr[r] - M);  // -inf: an empty chunk
            Ls += lr[r] * f;
            O += orr[r] * f;
        }
        res[it] = O / Ls;
    }
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
#pragma unroll
    for (int it = 0; it < kIter; ++it) {
        const int j = threadIdx.x + it * kRaThreads;
        if (j < per) p.out[row * p.out_stride + (int64_t)kvh * GRP * D + rank * per + j] = __float2bfloat16_rn(res[it]);
    }
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (threadIdx.x == 0) tl.done(2000u + CS);
}

template <int GRP, int D, int CS>
static cudaError_t launch_rope_attn(const RopeAttnParams& p, int64_t nkv, int64_t rows, cudaStream_t s) {
    constexpr int cs = CS;
    auto kern = attn_rope_decode_kernel<GRP, D, CS>;
    set_func_attr_once((const void*)kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)cs, (unsigned)nkv, (unsigned)rows);
    cfg.blockDim = dim3(kRaThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

// Cluster size: 16 CTAs per (sequence, kv head) where the device schedules
// clusters that large, else the portable 8.
template <int GRP, int D>
static int cluster_size() {
    static int cs = 0;
    if (cs == 0) {
        auto kern = attn_rope_decode_kernel<GRP, D, 16>;
        set_func_attr_once((const void*)kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(16, 1, 1);
        cfg.blockDim = dim3(kRaThreads);
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 16;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
        if (e != cudaSuccess) cudaGetLastError();
        cs = (e == cudaSuccess && n > 0) ? 16 : 8;
    }
    return cs;
}

// CTAs per cluster for `units` (sequence, kv head) pairs: 16 (8 where the
// device cannot schedule 16) for a batch-1 step, fewer as the batch grows so
// that a CTA keeps a useful share of the keys. 8B batch 8 (64 units) at
// context ~540, ms per decode step: 2.91 with 2 CTAs, 2.73 with 4, 3.09 with
// 8, 3.53 with 16. AMCU_ATTN_CS forces a size (power of two, 2..16).
template <int GRP, int D>
static int pick_cluster_size(int64_t units) {
    static const int forced = [] {
        const char* v = std::getenv("AMCU_ATTN_CS");
        return v ? std::atoi(v) : 0;
    }();
    const int maxcs = cluster_size<GRP, D>();
    int cs = forced > 0 ? forced : (int)(kRaTargetCtas / (units > 0 ? units : 1));
    int c = 2;
    while (c * 2 <= cs && c * 2 <= maxcs) c *= 2;
    return c;
}

template <int D>
static bool dispatch_rope_attn(const RopeAttnParams& p, int grp, int64_t nkv, int64_t rows, cudaStream_t s) {
    switch (grp) {
#define AMCU_RA(G)                                                                   \
    case G: {                                                                        \
        const int cs = pick_cluster_size<G, D>(nkv * rows);                          \
        const cudaError_t e = cs == 16 ? launch_rope_attn<G, D, 16>(p, nkv, rows, s) \
                              : cs == 8 ? launch_rope_attn<G, D, 8>(p, nkv, rows, s) \
                              : cs == 4 ? launch_rope_attn<G, D, 4>(p, nkv, rows, s) \
                                        : launch_rope_attn<G, D, 2>(p, nkv, rows, s); \
        (void)e;                                                                     \
        return true;                                                                 \
    }
        AMCU_RA(1)
        AMCU_RA(2)
        AMCU_RA(4)
        AMCU_RA(8)
#undef AMCU_RA
        default: return false;
    }
}

}  // namespace amcu

using namespace amcu;

extern "C" am_status_code amcu_attn_decode_rope(const AmcuRopeKvArgs* r, const AmcuAttentionArgs* a, void* stream) {
    clear_error();
    AMCU_REQUIRE(r && a, "amcu_attn_decode_rope: null args");
    AMCU_REQUIRE(r->rows == a->rows && r->rows >= 0, "amcu_attn_decode_rope: rope and attention rows differ");
    if (a->rows == 0) return AM_STATUS_OK;
    AMCU_REQUIRE(r->rows_per_seq == 1 && a->rows_per_seq == 1, "amcu_attn_decode_rope: decode takes one row per sequence");
    AMCU_REQUIRE(r->dtype == AMCU_BF16 && a->dtype == AMCU_BF16, "amcu_attn_decode_rope: bf16 only");
    AMCU_REQUIRE(r->n_q_heads == a->n_q_heads && r->n_kv_heads == a->n_kv_heads && r->head_dim == a->head_dim,
                 "amcu_attn_decode_rope: rope and attention head shapes differ");
    AMCU_REQUIRE(r->k_cache == a->k_cache && r->v_cache == a->v_cache && r->seq_pos == a->seq_pos &&
                         r->capacity == a->capacity,
                 "amcu_attn_decode_rope: rope and attention must name the same cache and positions");
    AMCU_REQUIRE(r->q == a->q, "amcu_attn_decode_rope: attention q must be the rope q");
    AMCU_REQUIRE(r->q && r->k && r->v && a->k_cache && a->v_cache && a->seq_pos && a->out,
                 "amcu_attn_decode_rope: null pointer");
    AMCU_REQUIRE(a->head_dim == 64 || a->head_dim == 128, "amcu_attn_decode_rope: head_dim must be 64 or 128");
    AMCU_REQUIRE(a->n_kv_heads > 0 && a->n_q_heads % a->n_kv_heads == 0,
                 "amcu_attn_decode_rope: n_q must be a multiple of n_kv");
    AMCU_REQUIRE(a->capacity > 0 && r->theta > 0.0, "amcu_attn_decode_rope: bad capacity or theta");
    AMCU_REQUIRE(aligned(a->k_cache, 16) && aligned(a->v_cache, 16), "amcu_attn_decode_rope: caches must be 16-byte aligned");
    RopeAttnParams p{};
    p.q = static_cast<const __nv_bfloat16*>(r->q);
    p.k = static_cast<const __nv_bfloat16*>(r->k);
    p.v = static_cast<const __nv_bfloat16*>(r->v);
    p.q_stride = r->q_stride ? r->q_stride : r->n_q_heads * r->head_dim;
    p.k_stride = r->k_stride ? r->k_stride : r->n_kv_heads * r->head_dim;
    p.v_stride = r->v_stride ? r->v_stride : r->n_kv_heads * r->head_dim;
    p.kc = static_cast<__nv_bfloat16*>(r->k_cache);
    p.vc = static_cast<__nv_bfloat16*>(r->v_cache);
    p.capacity = a->capacity;
    p.slot_stride = a->slot_stride ? a->slot_stride : a->n_kv_heads * a->capacity * a->head_dim;
    p.seq_pos = a->seq_pos;
    p.status = r->status;
    p.cos_sin = r->cos_sin;
    p.theta = r->theta;
    p.out = static_cast<__nv_bfloat16*>(a->out);
    p.out_stride = a->out_stride ? a->out_stride : a->n_q_heads * a->head_dim;
    p.scale_log2 = (float)(1.0 / sqrt((double)a->head_dim)) * kLog2e;
    const int grp = (int)(a->n_q_heads / a->n_kv_heads);
    const cudaStream_t s = as_stream(stream);
    const bool ok = a->head_dim == 128 ? dispatch_rope_attn<128>(p, grp, a->n_kv_heads, a->rows, s)
                                       : dispatch_rope_attn<64>(p, grp, a->n_kv_heads, a->rows, s);
    if (!ok) return set_error(AM_STATUS_INVALID_ARGUMENT, "amcu_attn_decode_rope: GQA group %d unsupported", grp);
    return check_launch("amcu_attn_decode_rope");
}

#ifdef AMCU_DIAG
// Diagnostics: the fused decode attention launch timeline (see diag_timeline.cuh).
extern "C" __attribute__((visibility("default"))) int amcu_diag_timeline_attn(void* out, int max) { return amcu::diag_timeline_take(out, max); }
#endif
