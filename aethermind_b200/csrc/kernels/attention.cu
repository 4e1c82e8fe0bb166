// GQA causal attention over the static KV cache.
//
// Semantics (src/operators/attention_op.cpp:65-147, causal per the reference's
// operator design): o = softmax(q k^T / sqrt(d)) v over cache positions
// [0, pos], kv_head = q_head / (n_q / n_kv).
//
// Split-K kernel: one CTA per (split, kv_head, query row). The CTA loads the
// GRP query heads that share the kv head once, so every K/V byte read from HBM
// serves all GRP heads. Four warps take 32-key blocks round-robin; in a block,
// lane j scores key j against all GRP heads (its K row is 2*d contiguous
// bytes), the warp does an online softmax, and then the warp accumulates
// P*V with lane l owning d/32 output dims (coalesced V rows). With one split
// the CTA normalises and stores the output directly; with several it writes
// (max, sum, unnormalised o) partials and a combine kernel merges them.
#include <mutex>

#include <cstdlib>

#include "../amcu_internal.h"
#include "attn_decode.cuh"
#include "common.cuh"

namespace amcu {

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&f)[8]);
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&f)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&f)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

struct AttnKParams {
    const void* q;
    int64_t q_stride;
    const void* kc;
    const void* vc;
    int64_t slot_stride, capacity;
    const int32_t* seq_pos;
    void* out;
    int64_t out_stride;
    int64_t rows_per_seq;
    int64_t nq, nkv;
    int nsplit;
    float* ws;  // [rows][nq][nsplit][D + 2]
    float scale_log2;
};

template <typename T, int GRP, int D>
__global__ void __launch_bounds__(kAttnThreads) attn_splitk_kernel(AttnKParams p) {
    pdl_wait();
    pdl_trigger();
    constexpr int NW = kAttnThreads / 32;
    constexpr int DL = D / 32;  // dims per lane in the P*V phase
    const int split = blockIdx.x, kvh = blockIdx.y;
    const int64_t row = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t b = row / p.rows_per_seq;
    const int64_t pos = (int64_t)p.seq_pos[b] + row % p.rows_per_seq;
    const int64_t L = pos + 1;
    int64_t chunk = (L + p.nsplit - 1) / p.nsplit;
    chunk = (chunk + 31) / 32 * 32;
    const int64_t k_begin = (int64_t)split * chunk;
    const int64_t k_end = k_begin + chunk < L ? k_begin + chunk : L;

    __shared__ __align__(16) float qs[GRP][D];
    __shared__ float sm_m[NW][GRP], sm_l[NW][GRP];
    __shared__ float sm_o[NW][GRP][D];
    const T* qrow = static_cast<const T*>(p.q) + row * p.q_stride + (int64_t)kvh * GRP * D;
    for (int i = threadIdx.x; i < GRP * D; i += kAttnThreads) qs[i / D][i % D] = Act<T>::load(qrow[i]);
    __syncthreads();

    const T* kbase = static_cast<const T*>(p.kc) + b * p.slot_stride + (int64_t)kvh * p.capacity * D;
    const T* vbase = static_cast<const T*>(p.vc) + b * p.slot_stride + (int64_t)kvh * p.capacity * D;

    float m[GRP], l[GRP], acc[GRP][DL];
#pragma unroll
    for (int h = 0; h < GRP; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int i = 0; i < DL; ++i) acc[h][i] = 0.f;
    }

    for (int64_t kb = k_begin + warp * 32; kb < k_end; kb += NW * 32) {
        const int64_t key = kb + lane;
        const bool valid = key < k_end;
        float s[GRP];
#pragma unroll
        for (int h = 0; h < GRP; ++h) s[h] = 0.f;
        if (valid) {
            const T* kr = kbase + key * D;
#pragma unroll 4
            for (int i = 0; i < D; i += 8) {
                float kf[8];
                load8<T>(kr + i, kf);
#pragma unroll
                for (int h = 0; h < GRP; ++h) {
                    const float4 q0 = *reinterpret_cast<const float4*>(&qs[h][i]);
                    const float4 q1 = *reinterpret_cast<const float4*>(&qs[h][i + 4]);
                    s[h] = fmaf(q0.x, kf[0], s[h]); s[h] = fmaf(q0.y, kf[1], s[h]);
                    s[h] = fmaf(q0.z, kf[2], s[h]); s[h] = fmaf(q0.w, kf[3], s[h]);
                    s[h] = fmaf(q1.x, kf[4], s[h]); s[h] = fmaf(q1.y, kf[5], s[h]);
                    s[h] = fmaf(q1.z, kf[6], s[h]); s[h] = fmaf(q1.w, kf[7], s[h]);
                }
            }
        }
        float pr[GRP];
#pragma unroll
        for (int h = 0; h < GRP; ++h) {
            const float sv = valid ? s[h] * p.scale_log2 : -INFINITY;
            const float bm = warp_max(sv);
            const float mn = fmaxf(m[h], bm);
            const float corr = exp2f(m[h] - mn);  // m = -inf first time -> 0
            pr[h] = valid ? exp2f(sv - mn) : 0.f;
            l[h] = l[h] * corr + warp_sum(pr[h]);
            m[h] = mn;
#pragma unroll
            for (int i = 0; i < DL; ++i) acc[h][i] *= corr;
        }
        const int nk = (int)(k_end - kb < 32 ? k_end - kb : 32);
        for (int j = 0; j < nk; ++j) {
            const T* vr = vbase + (kb + j) * D + lane * DL;
            float vf[DL];
#pragma unroll
            for (int i = 0; i < DL; ++i) vf[i] = Act<T>::load(vr[i]);
#pragma unroll
            for (int h = 0; h < GRP; ++h) {
                const float pj = __shfl_sync(0xffffffffu, pr[h], j);
#pragma unroll
                for (int i = 0; i < DL; ++i) acc[h][i] = fmaf(pj, vf[i], acc[h][i]);
            }
        }
    }

    // merge the warps
    if (lane == 0) {
#pragma unroll
        for (int h = 0; h < GRP; ++h) { sm_m[warp][h] = m[h]; sm_l[warp][h] = l[h]; }
    }
#pragma unroll
    for (int h = 0; h < GRP; ++h)
#pragma unroll
        for (int i = 0; i < DL; ++i) sm_o[warp][h][lane * DL + i] = acc[h][i];
    __syncthreads();
    for (int e = threadIdx.x; e < GRP * D; e += kAttnThreads) {
        const int h = e / D, dd = e % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, sm_m[w][h]);
        float Ls = 0.f, O = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                const float f = exp2f(sm_m[w][h] - M);
                Ls += sm_l[w][h] * f;
                O += sm_o[w][h][dd] * f;
            }
        }
        const int64_t qh = (int64_t)kvh * GRP + h;
        if (p.nsplit == 1) {
            T* o = static_cast<T*>(p.out) + row * p.out_stride + qh * D;
            o[dd] = Act<T>::store(O / Ls);
        } else {
            float* w = p.ws + ((row * p.nq + qh) * p.nsplit + split) * (D + 2);
            w[2 + dd] = O;
            if (dd == 0) { w[0] = M; w[1] = Ls; }
        }
    }
}


// Decode kernel (one query row per sequence, long context): the same split /
// combine structure, with a warp scoring 8 keys at a time (decode_keys_warp).
template <typename T, int GRP, int D>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(AttnKParams p) {
    pdl_wait();
    pdl_trigger();
    static_assert(sizeof(T) == 2, "bf16 only");
    const int split = blockIdx.x, kvh = blockIdx.y;
    const int64_t row = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t b = row / p.rows_per_seq;
    const int64_t pos = (int64_t)p.seq_pos[b] + row % p.rows_per_seq;
    const int64_t L = pos + 1;
    int64_t chunk = (L + p.nsplit - 1) / p.nsplit;
    chunk = (chunk + 7) / 8 * 8;
    const int64_t k_begin = (int64_t)split * chunk;
    const int64_t k_end = k_begin + chunk < L ? k_begin + chunk : L;

    __shared__ __align__(16) float qs[GRP][D];
    __shared__ float sm_m[kAttnWarps][GRP], sm_l[kAttnWarps][GRP];
    __shared__ float sm_o[kAttnWarps][GRP][D];
    const T* qrow = static_cast<const T*>(p.q) + row * p.q_stride + (int64_t)kvh * GRP * D;
    for (int i = threadIdx.x; i < GRP * D; i += kAttnThreads) qs[i / D][i % D] = Act<T>::load(qrow[i]) * p.scale_log2;
    __syncthreads();

    const T* kbase = static_cast<const T*>(p.kc) + b * p.slot_stride + (int64_t)kvh * p.capacity * D;
    const T* vbase = static_cast<const T*>(p.vc) + b * p.slot_stride + (int64_t)kvh * p.capacity * D;
    DecodeWarpState<GRP, D> st;
    decode_keys_warp<GRP, D, kAttnWarps>(kbase, vbase, k_begin, k_end, warp, lane, qs, st);
    decode_publish_warp<GRP, D>(st, warp, lane, sm_m, sm_l, sm_o);
    __syncthreads();
    for (int e = threadIdx.x; e < GRP * D; e += kAttnThreads) {
        const int h = e / D, dd = e % D;
        float M, Ls, O;
        decode_merge_warps<GRP, D, kAttnWarps>(h, dd, sm_m, sm_l, sm_o, M, Ls, O);
        const int64_t qh = (int64_t)kvh * GRP + h;
        if (p.nsplit == 1) {
            T* o = static_cast<T*>(p.out) + row * p.out_stride + qh * D;
            o[dd] = Act<T>::store(O / Ls);
        } else {
            float* w = p.ws + ((row * p.nq + qh) * p.nsplit + split) * (D + 2);
            w[2 + dd] = O;
            if (dd == 0) { w[0] = M; w[1] = Ls; }
        }
    }
}

// Merges the split partials of one (row, head): every split's (max, sum)
// is read in parallel, the weights exp2(m_s - M) go through shared memory,
// then each thread sums its output dim over the splits.
constexpr int kMaxSplits = 64;
template <typename T, int D>
__global__ void __launch_bounds__(D) attn_combine_kernel(AttnKParams p) {
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.x / p.nq, qh = blockIdx.x % p.nq;
    const float* w = p.ws + (row * p.nq + qh) * p.nsplit * (D + 2);
    __shared__ float f[kMaxSplits];
    __shared__ float red[D / 32];
    __shared__ float total;
    const int t = threadIdx.x;
    const float ms = t < p.nsplit ? w[t * (D + 2)] : -INFINITY;
    float M = warp_max(ms);
    if ((t & 31) == 0) red[t >> 5] = M;
    __syncthreads();
    M = red[0];
#pragma unroll
    for (int i = 1; i < D / 32; ++i) M = fmaxf(M, red[i]);
    __syncthreads();
    float fl = 0.f;
    if (t < p.nsplit) {
        const float fs = ms == -INFINITY ? 0.f : exp2f(ms - M);
        f[t] = fs;
        fl = fs * w[t * (D + 2) + 1];
    }
    fl = warp_sum(fl);
    if ((t & 31) == 0) red[t >> 5] = fl;
    __syncthreads();
    if (t == 0) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < D / 32; ++i) s += red[i];
        total = s;
    }
    __syncthreads();
    float O = 0.f;
    for (int s = 0; s < p.nsplit; ++s) O = fmaf(f[s], w[s * (D + 2) + 2 + t], O);
    static_cast<T*>(p.out)[row * p.out_stride + qh * D + t] = Act<T>::store(O / total);
}

template <typename T, int GRP, int D>
static void launch_attn(const AttnKParams& p, int64_t rows, cudaStream_t s) {
    const dim3 grid((unsigned)p.nsplit, (unsigned)p.nkv, (unsigned)rows);
    if constexpr (sizeof(T) == 2) {
        if (p.rows_per_seq == 1) launch_pdl(attn_decode_kernel<T, GRP, D>, grid, dim3(kAttnThreads), 0, s, p);
        else launch_pdl(attn_splitk_kernel<T, GRP, D>, grid, dim3(kAttnThreads), 0, s, p);
    } else {
        launch_pdl(attn_splitk_kernel<T, GRP, D>, grid, dim3(kAttnThreads), 0, s, p);
    }
    if (p.nsplit > 1) launch_pdl(attn_combine_kernel<T, D>, dim3((unsigned)(rows * p.nq)), dim3(D), 0, s, p);
}

template <typename T, int D>
static bool dispatch_grp(const AttnKParams& p, int grp, int64_t rows, cudaStream_t s) {
    switch (grp) {
        case 1: launch_attn<T, 1, D>(p, rows, s); return true;
        case 2: launch_attn<T, 2, D>(p, rows, s); return true;
        case 4: launch_attn<T, 4, D>(p, rows, s); return true;
        case 8: launch_attn<T, 8, D>(p, rows, s); return true;
        default: return false;
    }
}

}  // namespace amcu

namespace amcu {
bool launch_attn_prefill_flash(const AmcuAttentionArgs* a, cudaStream_t s);
}  // namespace amcu

using namespace amcu;

namespace {

int choose_splits(const AmcuAttentionArgs* a) {
    if (a->num_splits > 0) return a->num_splits;
    if (a->rows_per_seq > 1) return 1;
    const int64_t ctas = a->n_kv_heads * a->rows;
    int64_t by_len = (a->max_context + 31) / 32;
    int64_t by_sm = (4 * num_sms() + ctas - 1) / ctas;
    int64_t s = by_len < by_sm ? by_len : by_sm;
    if (s > kMaxSplits) s = kMaxSplits;
    return (int)(s < 1 ? 1 : s);
}

am_status_code validate_attn(const AmcuAttentionArgs* a, const char* who) {
    AMCU_REQUIRE(a != nullptr, "%s: null args", who);
    AMCU_REQUIRE(a->rows >= 0, "%s: negative rows", who);
    AMCU_REQUIRE(a->q && a->k_cache && a->v_cache && a->seq_pos && a->out, "%s: null pointer", who);
    AMCU_REQUIRE(a->n_kv_heads > 0 && a->n_q_heads % a->n_kv_heads == 0, "%s: n_q must be a multiple of n_kv", who);
    const int64_t grp = a->n_q_heads / a->n_kv_heads;
    AMCU_REQUIRE(grp == 1 || grp == 2 || grp == 4 || grp == 8, "%s: GQA group %lld unsupported", who, (long long)grp);
    AMCU_REQUIRE(a->head_dim == 64 || a->head_dim == 128, "%s: head_dim must be 64 or 128", who);
    AMCU_REQUIRE(a->dtype == AMCU_F32 || a->dtype == AMCU_BF16, "%s: dtype must be f32 or bf16", who);
    AMCU_REQUIRE(a->rows_per_seq > 0 && a->capacity > 0, "%s: bad rows_per_seq/capacity", who);
    AMCU_REQUIRE(a->num_splits >= 0 && a->num_splits <= kMaxSplits, "%s: num_splits must be in [0, %d]", who,
                 kMaxSplits);
    const int64_t elt = a->dtype == AMCU_F32 ? 4 : 2;
    AMCU_REQUIRE(aligned(a->q, 16) && aligned(a->k_cache, 16) && aligned(a->v_cache, 16),
                 "%s: q and caches must be 16-byte aligned", who);
    AMCU_REQUIRE(((a->q_stride ? a->q_stride : a->n_q_heads * a->head_dim) * elt) % 16 == 0,
                 "%s: q row stride must be a multiple of 16 bytes", who);
    return AM_STATUS_OK;
}

am_status_code run_attn(const AmcuAttentionArgs* a, int nsplit, cudaStream_t s) {
    AttnKParams p{};
    p.q = a->q;
    p.q_stride = a->q_stride ? a->q_stride : a->n_q_heads * a->head_dim;
    p.kc = a->k_cache;
    p.vc = a->v_cache;
    p.capacity = a->capacity;
    p.slot_stride = a->slot_stride ? a->slot_stride : a->n_kv_heads * a->capacity * a->head_dim;
    p.seq_pos = a->seq_pos;
    p.out = a->out;
    p.out_stride = a->out_stride ? a->out_stride : a->n_q_heads * a->head_dim;
    p.rows_per_seq = a->rows_per_seq;
    p.nq = a->n_q_heads;
    p.nkv = a->n_kv_heads;
    p.nsplit = nsplit;
    p.ws = static_cast<float*>(a->workspace);
    p.scale_log2 = (float)(1.0 / sqrt((double)a->head_dim)) * kLog2e;
    const int grp = (int)(a->n_q_heads / a->n_kv_heads);
    bool ok;
    if (a->dtype == AMCU_BF16)
        ok = a->head_dim == 128 ? dispatch_grp<__nv_bfloat16, 128>(p, grp, a->rows, s)
                                : dispatch_grp<__nv_bfloat16, 64>(p, grp, a->rows, s);
    else
        ok = a->head_dim == 128 ? dispatch_grp<float, 128>(p, grp, a->rows, s)
                                : dispatch_grp<float, 64>(p, grp, a->rows, s);
    if (!ok) return set_error(AM_STATUS_INVALID_ARGUMENT, "attention: unsupported GQA group");
    return check_launch("amcu_attention");
}

}  // namespace

extern "C" {

size_t amcu_attention_workspace_bytes(const AmcuAttentionArgs* a) {
    if (!a || a->rows <= 0) return 0;
    const int ns = choose_splits(a);
    if (ns <= 1) return 0;
    return (size_t)a->rows * a->n_q_heads * ns * (a->head_dim + 2) * sizeof(float);
}

am_status_code amcu_attn_decode(const AmcuAttentionArgs* a, void* stream) {
    clear_error();
    am_status_code st = validate_attn(a, "amcu_attn_decode");
    if (st != AM_STATUS_OK) return st;
    if (a->rows == 0) return AM_STATUS_OK;
    const int ns = choose_splits(a);
    if (ns > 1) {
        const size_t need = amcu_attention_workspace_bytes(a);
        AMCU_REQUIRE(a->workspace && a->workspace_size >= need,
                     "amcu_attn_decode: workspace of %zu bytes required", need);
    }
    return run_attn(a, ns, as_stream(stream));
}

am_status_code amcu_attn_prefill(const AmcuAttentionArgs* a, void* stream) {
    clear_error();
    am_status_code st = validate_attn(a, "amcu_attn_prefill");
    if (st != AM_STATUS_OK) return st;
    if (a->rows == 0) return AM_STATUS_OK;
    // bf16: the tensor-core flash kernel (attention_prefill.cu); fp32 and any
    // shape it does not take: one CTA per (row, kv head)
    static const bool flash = [] {
        const char* v = std::getenv("AMCU_ATTN_PREFILL_FLASH");
        return !(v && v[0] == '0');
    }();
    if (flash && launch_attn_prefill_flash(a, as_stream(stream))) return check_launch("amcu_attn_prefill");
    return run_attn(a, 1, as_stream(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free decode attention.
//
// Some callers cannot allocate device memory when they call into this
// library. Examples: a serving process that carves up HBM once at start-up
// and forbids allocations afterwards, or a latency-critical step in which
// cudaMalloc's implicit device synchronization is not acceptable. Such
// callers cannot provide the split-K workspace that amcu_attn_decode needs.
// amcu_attn_decode_noalloc runs the same kernels with a fixed scratch buffer
// that is compiled into the library instead.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes, so
// every GPU that loads this library holds it until the process exits. In
// host code the array's name only stands in for its device address. That
// address is looked up once per device with cudaGetSymbolAddress, while that
// device is current, on the first call made on that device.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;  // 4 MiB
static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[kNoAllocScratchBytes];

am_status_code noalloc_scratch(void** out) {
    static void* addr[64] = {};
    static std::mutex mu;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(AM_STATUS_INTERNAL, "cudaGetDevice failed: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return set_error(AM_STATUS_OUT_OF_RANGE, "device %d not supported", dev);
    std::lock_guard<std::mutex> lk(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            cudaGetLastError();
            return set_error(AM_STATUS_INTERNAL, "cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(e));
        }
        addr[dev] = p;
    }
    *out = addr[dev];
    return AM_STATUS_OK;
}

}  // namespace

extern "C" am_status_code amcu_attn_decode_noalloc(const AmcuAttentionArgs* a, void* stream) {
    clear_error();
    am_status_code st = validate_attn(a, "amcu_attn_decode_noalloc");
    if (st != AM_STATUS_OK) return st;
    if (a->rows == 0) return AM_STATUS_OK;
    const int ns = choose_splits(a);
    const size_t need = amcu_attention_workspace_bytes(a);
    if (need > kNoAllocScratchBytes)
        return set_error(AM_STATUS_INVALID_ARGUMENT,
                         "amcu_attn_decode_noalloc: these sizes need %zu bytes of split scratch; the built-in scratch "
                         "holds %zu (use fewer rows, heads or splits, or amcu_attn_decode with a workspace)",
                         need, kNoAllocScratchBytes);
    void* scratch = nullptr;
    st = noalloc_scratch(&scratch);
    if (st != AM_STATUS_OK) return st;
    // Every split writes all of its partial (max, sum, output) before the
    // combine reads it, so nothing in the scratch has to start at zero.
    AmcuAttentionArgs b = *a;
    b.workspace = scratch;
    b.workspace_size = kNoAllocScratchBytes;
    return run_attn(&b, ns, as_stream(stream));
}
