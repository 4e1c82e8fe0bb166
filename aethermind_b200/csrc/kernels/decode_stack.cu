// Persistent decode step: every decoder layer of a batch-1 INT4 decode step in
// one kernel.
//
// Semantics: for each layer, exactly the per-op plan's steps -- q/k/v GEMV
// with the fused attention RMSNorm, RoPE + KV append + attention, o GEMV +
// residual, gate/up GEMV with the fused MLP RMSNorm + SiLU-Mul, down GEMV +
// residual, in the reference's BuildLlamaDense order
// (src/model/model_graph_builder.cpp:324-419) with its rounding points: every
// op's output is rounded to bf16 once, RMSNorm's output too.
//
// Why one kernel: at batch 1 a layer streams ~115 MB of INT4 weights (8B
// shapes), about 17 us of HBM time, in five dependent GEMV/attention steps.
// Separate kernels pay a ramp-up and a drain per step. Here one CTA per SM
// stays resident for the whole step:
//   * warp 16 is the producer: it streams the CTA's share of every layer's
//     weights (q/k/v, o, gate/up, down, layer after layer) through a ring of
//     33 KB shared-memory stages with bulk copies, waiting only for free
//     stages -- never for the phases -- so the ring is full whenever the
//     consumers come back from a phase boundary or from attention;
//   * warps 0-15 are consumers. A GEMV phase stages its input row once per
//     CTA (one round of L2 loads: the row, and the norm weight or the
//     attention partials; RMSNorm factor and fp16 overflow guard from one
//     CTA-wide reduction), then consumes its contiguous run of weight rows, 2
//     pair records per warp per stage. The attention phase works on (kv head,
//     key split) units and writes unnormalised partials; the o GEMV's staging
//     merges them, so attention needs no extra round of global traffic.
// Phase boundaries are one monotonic arrival counter: a CTA arrives (release
// add) after its outputs are written and waits (acquire loads) for
// (phase + 1) x CTAs arrivals. The last CTA to leave the kernel resets the
// counter for the next step. Every wait is bounded: one that runs out records
// an error code in the device error word and stops waiting (the step's
// results are then invalid; the session reports DEADLINE_EXCEEDED).
// The kernel is launched cooperatively (all CTAs co-resident or no launch).
#include <cstdio>
#include <cstdlib>
#include <type_traits>
#include <vector>

#include "../amcu_internal.h"
#include "attn_decode.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "mma_int4.cuh"

namespace amcu {

constexpr int kDsConsumers = 16;
constexpr int kDsThreads = (kDsConsumers + 1) * 32;
constexpr int kDsCT = kDsConsumers * 32;                 // consumer threads
constexpr int kDsSU = 32;                                // pair records per ring stage
constexpr int kDsRecPerWarp = kDsSU / kDsConsumers;      // records per warp per stage
constexpr int kDsStageBytes = kDsSU * kW4PairBytes;
constexpr int kDsMaxK = 16384;                           // longest GEMV row (staged in registers)
constexpr int kDsCPT = kDsMaxK / 8 / kDsCT;              // 16-byte chunks per consumer thread
constexpr int kDsMaxSplits = 4;                          // attention key splits per kv head
constexpr int kDsKeysPerSplit = 128;
constexpr int32_t kErrDsBarrier = 0x301, kErrDsFull = 0x302, kErrDsEmpty = 0x303;
constexpr uint64_t kDsWaitNs = 2000000000ull;            // 2 s
constexpr int kBarC = 1;                                  // the consumers' named barrier

struct DsParams {
    const AmcuDecodeLayer* layers;
    int nlayers;
    __nv_bfloat16 *x, *qkv, *act;  // residual stream [H], q/k/v [qkv_n], act [I]
    int64_t H, I, nq, nkv;
    int64_t capacity;
    const int32_t* seq_pos;
    const float* cos_sin;
    double theta;
    float eps, scale_log2;
    float* attn_ws;           // [nkv][kDsMaxSplits][GRP][D + 2]: max, sum, unnormalised output
    unsigned int* sync;       // [0] arrivals, [32] exits (zero between launches)
    int stages;
    int rbmax;                // most row blocks a CTA owns in any GEMV phase
    int32_t *err, *status;
    unsigned long long* trace;  // AMCU_DIAG builds only: [cta][layer][kDsMarks] globaltimer stamps
};

// Diagnostics (AMCU_DIAG builds only; compiled out otherwise): phase stamps.
[[maybe_unused]] constexpr int kDsMarks = 28;
#ifdef AMCU_DIAG
__device__ __forceinline__ void ds_mark(const DsParams& p, int l, int idx) {
    if (p.trace && (threadIdx.x == 0 || threadIdx.x == kDsCT)) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        p.trace[((size_t)blockIdx.x * p.nlayers + l) * kDsMarks + idx] = t;
    }
}
#else
__device__ __forceinline__ void ds_mark(const DsParams&, int, int) {}
#endif

__device__ __forceinline__ uint64_t ds_clock_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* a) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_gpu(unsigned int* a, unsigned int v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}

// Row blocks [lo, hi) of an n-row weight that CTA c of `ctas` handles.
__device__ __forceinline__ void ds_range(int64_t n, int c, int ctas, int& lo, int& hi) {
    const int64_t nrb = n / 16;
    lo = (int)(nrb * c / ctas);
    hi = (int)(nrb * (c + 1) / ctas);
}

// Small per-CTA state of the consumers.
struct DsShared {
    float red[kDsConsumers][2];  // per-warp sum of squares, max magnitude
    float row_mul;               // staging multiplier (a power of two)
    int ok;                      // 0 once a wait ran out
    int ns;                      // attention splits this step
};

// The consumers' view of the ring.
struct DsRing {
    uint8_t* ring;
    uint64_t *full, *empty;
    int S, slot;
    uint32_t phase;
};

// The producer (warp 16, lane 0): requests every weight stage of the step in
// consumption order, each as soon as its ring slot is free (bounded waits).
template <int D>
__device__ __noinline__ void ds_produce(const DsParams& p, const DsRing& r) {
    const int G0 = (int)gridDim.x;
    const uint64_t pol = l2_policy_evict_first();  // weights are read once per step
    int slot = 0, issued = 0;
    uint32_t phase = 0;
    bool live = true;
    for (int l = 0; l < p.nlayers && live; ++l) {
        const AmcuDecodeLayer& ly = p.layers[l];
        const uint8_t* ws[4] = {static_cast<const uint8_t*>(ly.w_qkv), static_cast<const uint8_t*>(ly.w_o),
                                static_cast<const uint8_t*>(ly.w_gate_up), static_cast<const uint8_t*>(ly.w_down)};
        const int64_t ns[4] = {(p.nq + 2 * p.nkv) * D, p.H, 2 * p.I, p.H};
        const int64_t ks[4] = {p.H, p.nq * D, p.H, p.I};
        for (int ph = 0; ph < 4 && live; ++ph) {
            const int G = (int)(ks[ph] / 128);
            int lo, hi;
            ds_range(ns[ph], blockIdx.x, G0, lo, hi);
            const uint8_t* run = ws[ph] + (size_t)lo * G * kW4PairBytes;
            const int total = (hi - lo) * G;
            for (int st = 0; st * kDsSU < total; ++st, ++issued) {
                if (issued >= r.S && !mbar_wait(&r.empty[slot], phase ^ 1u)) {
                    record_device_error(p.err, kErrDsEmpty);
                    live = false;
                    break;
                }
                const int recs = total - st * kDsSU < kDsSU ? total - st * kDsSU : kDsSU;
#ifdef DS_NOSTREAM
                mbar_arrive(&r.full[slot]);  // diagnostics: no weight bytes (consumers read stale stages)
#else
                mbar_expect_tx(&r.full[slot], (uint32_t)(recs * kW4PairBytes));
                bulk_g2s_hint(r.ring + slot * kDsStageBytes, run + (size_t)st * kDsStageBytes,
                              (uint32_t)(recs * kW4PairBytes), &r.full[slot], pol);
#endif
                if (++slot == r.S) {
                    slot = 0;
                    phase ^= 1u;
                }
            }
            ds_mark(p, l, 15 + ph);  // every stage of this phase requested
        }
    }
    // the CTA's shared memory must outlive every copy still landing
    for (int i = issued > r.S ? issued - r.S : 0; i < issued; ++i)
        if (!mbar_wait(&r.full[i % r.S], (uint32_t)((i / r.S) & 1))) break;
}

// Phase boundary: every consumer thread's writes are done (named barrier),
// thread 0 arrives and waits for `target` arrivals, then all proceed.
#ifndef DS_POLL_NS
#define DS_POLL_NS 256
#endif
__device__ __forceinline__ void ds_sync(const DsParams& p, unsigned int target, DsShared* sh) {
    named_bar_sync(kBarC, kDsCT);
    if (threadIdx.x == 0) {
        __threadfence();
        red_release_gpu(p.sync, 1u);
        if (sh->ok) {
            const uint64_t t0 = ds_clock_ns();
            // polls back off: 148 CTAs spinning on one L2 line would slow
            // every other access that line's L2 slice serves
            while ((int)(ld_acquire_gpu(p.sync) - target) < 0) {
                __nanosleep(DS_POLL_NS);
                if (ds_clock_ns() - t0 > kDsWaitNs) {
                    record_device_error(p.err, kErrDsBarrier);
                    sh->ok = 0;
                    break;
                }
            }
        }
    }
    named_bar_sync(kBarC, kDsCT);
}

// L2 prefetch of a small read-only array (a norm weight) ahead of its use.
__device__ __forceinline__ void ds_prefetch_l2(const void* ptr, int64_t bytes) {
    if (blockIdx.x != 0 || ptr == nullptr) return;
    for (int64_t off = (int64_t)threadIdx.x * 128; off < bytes; off += (int64_t)kDsCT * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(static_cast<const char*>(ptr) + off));
}

struct DsSmem {
    int ring, bars, accs, sx, fw, un, total;
};
template <int GRP, int D>
__host__ __device__ inline DsSmem ds_smem(int64_t kmax, int64_t nq, int stages, int rbmax) {
    auto up = [](int64_t v) { return (int)((v + 127) / 128 * 128); };
    const int64_t xs = kmax * 2 + 16;
    const int64_t att = (int64_t)GRP * D * 4 + 2 * kDsConsumers * GRP * 4 + (int64_t)kDsConsumers * GRP * D * 4;
    DsSmem s;
    s.ring = 0;
    s.bars = stages * kDsStageBytes;
    s.accs = s.bars + up(2 * stages * 8);
    s.sx = s.accs + up((int64_t)rbmax * 16 * 8 * 4);       // [rbmax][16 rows][8 columns] fp32
    s.fw = s.sx + up(kmax / 128 * 8 * 4);                  // [G][8] group sums
    s.un = s.fw + up(nq * (kDsMaxSplits + 1) * 4);         // [nq][splits + 1] merge weights
    s.total = s.un + up(xs > att ? xs : att);
    return s;
}

// ---------------------------------------------------------------------------
// Staging: the input row of a GEMV phase into shared memory as fp16 (times
// 1/row_mul, an exact power of two that keeps it inside fp16's range), with
// the sums of every 128-column group for the INT4 offset removal.
//   MODE 0: y = round_bf16(x * inv * w), the RMSNorm of x (bf16 [k]) with
//           norm weight w, inv = (mean(x^2) + eps)^-1/2;
//   MODE 1: y = x;
//   MODE 2: y = the attention output, merged from the split partials:
//           round_bf16(sum_s o_s f_s / sum_s l_s f_s), f_s = 2^(m_s - max m).
// Chunk c (8 columns) of the row is handled by consumer thread c % 512, so a
// 128-column group is 16 consecutive lanes of one warp. Every CTA reduces the
// same values in the same order, so all CTAs stage the same row.
// ---------------------------------------------------------------------------
template <int MODE, int GRP, int D>
__device__ __noinline__ void ds_stage(const DsParams& p, const __nv_bfloat16* x, const __nv_bfloat16* w,
                                         int64_t k, uint8_t* xs, float* sx, float* fw, float* accs, int nacc,
                                         DsShared* sh) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int chunks = (int)(k / 8);
    for (int i = tid; i < nacc; i += kDsCT) accs[i] = 0.f;
    // pass 1: the row's values (bf16, packed) in registers, partial sum of
    // squares and largest magnitude
    uint4 v[kDsCPT];
    float ss = 0.f, amax = 0.f;
#pragma unroll
    for (int i = 0; i < kDsCPT; ++i) {
        const int c = tid + i * kDsCT;
        v[i] = make_uint4(0u, 0u, 0u, 0u);
        if (c < chunks) {
            if constexpr (MODE == 2) {
                // merge the splits of query head hq for dims [dd, dd + 8): every
                // load first (one round of L2 latency), then
                // round_bf16(sum_s o_s 2^(m_s - M) / sum_s l_s 2^(m_s - M))
                const int j0 = c * 8, hq = j0 / D, dd = j0 % D, kvh = hq / GRP, h = hq % GRP;
                const float* w0 = p.attn_ws + ((int64_t)kvh * kDsMaxSplits * GRP + h) * (D + 2);
                const int ns = sh->ns;
                float2 ml[kDsMaxSplits];
                float2 o[kDsMaxSplits][4];
#pragma unroll
                for (int sp = 0; sp < kDsMaxSplits; ++sp) {
                    const float* ws = w0 + (int64_t)sp * GRP * (D + 2);
                    ml[sp] = sp < ns ? __ldcg(reinterpret_cast<const float2*>(ws)) : make_float2(-INFINITY, 0.f);
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        o[sp][e] = sp < ns ? __ldcg(reinterpret_cast<const float2*>(ws + 2 + dd) + e)
                                           : make_float2(0.f, 0.f);
                }
                float M = -INFINITY;
#pragma unroll
                for (int sp = 0; sp < kDsMaxSplits; ++sp) M = fmaxf(M, ml[sp].x);
                float L = 0.f, out[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int sp = 0; sp < kDsMaxSplits; ++sp) {
                    const float f = ml[sp].x == -INFINITY ? 0.f : exp2f(ml[sp].x - M);  // -inf: empty split
                    L += ml[sp].y * f;
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        out[2 * e] += o[sp][e].x * f;
                        out[2 * e + 1] += o[sp][e].y * f;
                    }
                }
                uint32_t pk[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const __nv_bfloat162 b2 = __floats2bfloat162_rn(out[2 * e] / L, out[2 * e + 1] / L);
                    pk[e] = *reinterpret_cast<const uint32_t*>(&b2);
                    amax = fmaxf(amax, fmaxf(fabsf(__low2float(b2)), fabsf(__high2float(b2))));
                }
                v[i] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            } else {
                v[i] = __ldcg(reinterpret_cast<const uint4*>(x + (int64_t)c * 8));
                const uint32_t xw[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
                uint32_t ww[4] = {0u, 0u, 0u, 0u};
                if constexpr (MODE == 0) {
                    const uint4 wv = ld_u4(w + (int64_t)c * 8);
                    ww[0] = wv.x; ww[1] = wv.y; ww[2] = wv.z; ww[3] = wv.w;
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float a = __uint_as_float(xw[e] << 16), b = __uint_as_float(xw[e] & 0xffff0000u);
                    if constexpr (MODE == 0) {
                        ss += a * a + b * b;
                        // |x * w|: the normalized value is this times inv (before rounding)
                        amax = fmaxf(amax, fmaxf(fabsf(a * __uint_as_float(ww[e] << 16)),
                                                 fabsf(b * __uint_as_float(ww[e] & 0xffff0000u))));
                    } else {
                        amax = fmaxf(amax, fmaxf(fabsf(a), fabsf(b)));
                    }
                }
            }
        }
    }
    ss = warp_sum(ss);
    amax = warp_max(amax);
    if (lane == 0) {
        sh->red[warp][0] = ss;
        sh->red[warp][1] = amax;
    }
    named_bar_sync(kBarC, kDsCT);
    // every thread reduces the 16 warp partials in the same order
    float tss = 0.f, tmax = 0.f;
#pragma unroll
    for (int w8 = 0; w8 < kDsConsumers; ++w8) {
        tss += sh->red[w8][0];
        tmax = fmaxf(tmax, sh->red[w8][1]);
    }
    float inv = 1.f;
    if constexpr (MODE == 0) {
        inv = 1.0f / sqrtf(tss / (float)k + p.eps);
        tmax *= inv * 1.01f;  // covers the rounding of x * inv * w
    }
    // row_mul: a power of two with tmax / row_mul < 2^15 (fp16 staging stays finite)
    float mul = 1.f;
    if (tmax >= 32768.f) {
        const int e = (int)((__float_as_uint(tmax) >> 23) & 0xff) - 127 - 14;
        mul = __int_as_float((127 + (e > 0 ? e : 0)) << 23);
    }
    const float rmul = 1.0f / mul;  // exact
    if (tid == 0) sh->row_mul = mul;
    // pass 2: normalize, convert to fp16, group sums over 16 lanes
#pragma unroll
    for (int i = 0; i < kDsCPT; ++i) {
        const int c = tid + i * kDsCT;
        if (c < chunks) {  // chunks % 16 == 0: a group's 16 lanes are all active or all idle
            float y[8];
            const uint32_t xw[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
            if constexpr (MODE == 0) {
                const uint4 wv = ld_u4(w + (int64_t)c * 8);
                const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    y[2 * e] = Act<__nv_bfloat16>::round(__uint_as_float(xw[e] << 16) * inv *
                                                         __uint_as_float(ww[e] << 16));
                    y[2 * e + 1] = Act<__nv_bfloat16>::round(__uint_as_float(xw[e] & 0xffff0000u) * inv *
                                                             __uint_as_float(ww[e] & 0xffff0000u));
                }
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    y[2 * e] = __uint_as_float(xw[e] << 16);
                    y[2 * e + 1] = __uint_as_float(xw[e] & 0xffff0000u);
                }
            }
            uint32_t h[4];
            float sum = 0.f;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const __half2 hv = __floats2half2_rn(y[2 * e] * rmul, y[2 * e + 1] * rmul);
                sum += __low2float(hv) + __high2float(hv);
                h[e] = *reinterpret_cast<const uint32_t*>(&hv);
            }
            *reinterpret_cast<uint4*>(xs + (int64_t)c * 16) = make_uint4(h[0], h[1], h[2], h[3]);
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            sum += __shfl_xor_sync(0xffffffffu, sum, 8);
            if ((c & 15) == 0) sx[(c >> 4) * 8] = sum;
        }
    }
    named_bar_sync(kBarC, kDsCT);
}

// One GEMV phase of the consumers after staging: y = epilogue(W x) for this
// CTA's row blocks [lo, hi) of an INT4 [n][k] weight whose records the
// producer streams (row block after row block, K fastest, kDsSU per stage).
template <int EPI, int D>
__device__ __forceinline__ void ds_gemv(const DsParams& p, DsRing& r, int64_t k, int lo, int hi, const uint8_t* xs,
                                        const float* sx, float* accs, __nv_bfloat16* y, DsShared* sh) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int G = (int)(k / 128);
    const int total = (hi - lo) * G;
    const int nst = (total + kDsSU - 1) / kDsSU;
    const uint8_t* xr = xs + 32 * t;  // + 256 B per group
    uint8_t* const ring = r.ring;
    uint64_t* const empty = r.empty;
    const int S = r.S;
    int slot = r.slot;
    uint32_t phase = r.phase;
    bool live = sh->ok != 0;
    int cur = -1;
    float acc_lo = 0.f, acc_hi = 0.f;  // rows g and g+8, activation column 0 (t == 0 lanes)
    // record j * 16 + warp of every stage: its row block and group, advanced
    // by kDsSU records per stage without a division
    int rbj[kDsRecPerWarp], grj[kDsRecPerWarp];
#pragma unroll
    for (int j = 0; j < kDsRecPerWarp; ++j) {
        rbj[j] = (j * kDsConsumers + warp) / G;
        grj[j] = (j * kDsConsumers + warp) - rbj[j] * G;
    }
    for (int st = 0; st < nst; ++st) {
        if (live && !mbar_wait(&r.full[slot], phase)) {
            live = false;
            if (lane == 0) record_device_error(p.err, kErrDsFull);
        }
        const uint8_t* stage = ring + slot * kDsStageBytes;
        // both records' tiles first (independent MMA chains interleave)
        // both records' tiles first (independent MMA chains interleave)
        float part[kDsRecPerWarp][2][4];
        bool have[kDsRecPerWarp];
#pragma unroll
        for (int j = 0; j < kDsRecPerWarp; ++j) {
            have[j] = st * kDsSU + j * kDsConsumers + warp < total;
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int e = 0; e < 4; ++e) part[j][h][e] = 0.f;
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint4 wv[kDsRecPerWarp], x0[kDsRecPerWarp], x1[kDsRecPerWarp];
#pragma unroll
            for (int j = 0; j < kDsRecPerWarp; ++j) {
                const uint8_t* rec = stage + (j * kDsConsumers + warp) * kW4PairBytes;
                const uint8_t* xp = xr + grj[j] * 256 + h * 128;
                wv[j] = *reinterpret_cast<const uint4*>(rec + h * 512 + lane * 16);
                x0[j] = *reinterpret_cast<const uint4*>(xp);
                x1[j] = *reinterpret_cast<const uint4*>(xp + 16);
            }
            uint32_t a[kDsRecPerWarp][4];
#pragma unroll
            for (int j = 0; j < kDsRecPerWarp; ++j) unpack_w4_word_f16(wv[j].x, a[j]);
#pragma unroll
            for (int j = 0; j < kDsRecPerWarp; ++j) mma_f16_16816(part[j][h], a[j], x0[j].x, x0[j].y);
#pragma unroll
            for (int j = 0; j < kDsRecPerWarp; ++j) unpack_w4_word_f16(wv[j].y, a[j]);
#pragma unroll
            for (int j = 0; j < kDsRecPerWarp; ++j) mma_f16_16816(part[j][h], a[j], x0[j].z, x0[j].w);
#pragma unroll
            for (int j = 0; j < kDsRecPerWarp; ++j) unpack_w4_word_f16(wv[j].z, a[j]);
#pragma unroll
            for (int j = 0; j < kDsRecPerWarp; ++j) mma_f16_16816(part[j][h], a[j], x1[j].x, x1[j].y);
#pragma unroll
            for (int j = 0; j < kDsRecPerWarp; ++j) unpack_w4_word_f16(wv[j].w, a[j]);
#pragma unroll
            for (int j = 0; j < kDsRecPerWarp; ++j) mma_f16_16816(part[j][h], a[j], x1[j].z, x1[j].w);
        }
#pragma unroll
        for (int j = 0; j < kDsRecPerWarp; ++j) {
            if (have[j]) {
                if (rbj[j] != cur) {
                    if (cur >= 0 && t == 0) {
                        atomicAdd(accs + cur * 128 + g * 8, acc_lo);
                        atomicAdd(accs + cur * 128 + (g + 8) * 8, acc_hi);
                    }
                    acc_lo = acc_hi = 0.f;
                    cur = rbj[j];
                }
                // part[j][0] + part[j][1]: sum (1032 + q) x (rows g) and sum (1152 + 16 q) x
                // (rows g+8); MMA column 0 (lanes t == 0, c0 / c2) is the activation row
                const uint8_t* rec = stage + (j * kDsConsumers + warp) * kW4PairBytes;
                const float s2x = sx[grj[j] * 8];
                const uint32_t sv = *reinterpret_cast<const uint32_t*>(rec + 1024 + 4 * g);
                const __half2 s2 = *reinterpret_cast<const __half2*>(&sv);
                const float s_lo = __low2float(s2), s_hi = __high2float(s2) * 0.0625f;
                acc_lo = fmaf(fmaf(-1032.f, s2x, part[j][0][0] + part[j][1][0]), s_lo, acc_lo);
                acc_hi = fmaf(fmaf(-1152.f, s2x, part[j][0][2] + part[j][1][2]), s_hi, acc_hi);
            }
            grj[j] += kDsSU;
            while (grj[j] >= G) {
                grj[j] -= G;
                ++rbj[j];
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (++slot == S) {
            slot = 0;
            phase ^= 1;
        }
    }
    if (cur >= 0 && t == 0) {
        atomicAdd(accs + cur * 128 + g * 8, acc_lo);
        atomicAdd(accs + cur * 128 + (g + 8) * 8, acc_hi);
    }
    r.slot = slot;
    r.phase = phase;
    if (!live) sh->ok = 0;
    named_bar_sync(kBarC, kDsCT);
    // epilogue over (row block, weight row)
    const float rm = sh->row_mul;
    const int nloc = hi - lo;
    if constexpr (EPI == AMCU_EPI_SILU_MUL) {
        // rows 0-7 of a block are gate rows 8 rb .. 8 rb + 7, rows 8-15 the matching up rows
        for (int e = threadIdx.x; e < nloc * 8; e += kDsCT) {
            const int rr = e % 8, rl = e / 8;
            const float* a16 = accs + rl * 128;
            const float gt = Act<__nv_bfloat16>::round(a16[rr * 8] * rm);
            const float up = Act<__nv_bfloat16>::round(a16[(rr + 8) * 8] * rm);
            y[(int64_t)(lo + rl) * 8 + rr] = __float2bfloat16_rn(silu_ref(gt) * up);
        }
    } else {
        for (int e = threadIdx.x; e < nloc * 16; e += kDsCT) {
            const int rr = e % 16, rl = e / 16;
            const int64_t off = (int64_t)(lo + rl) * 16 + rr;
            float o = Act<__nv_bfloat16>::round(accs[rl * 128 + rr * 8] * rm);
            if constexpr (EPI == AMCU_EPI_RESIDUAL_ADD) o = o + __bfloat162float(__ldcg(y + off));  // y is the residual
            y[off] = __float2bfloat16_rn(o);
        }
    }
}

// One warp's share of a (kv head, key split) unit: blocks of 8 keys, spaced
// kDsConsumers * 8 apart. Lane 4k + q holds quarter q of key k's head_dim for
// the scores and output dims [lane * D/32, (lane + 1) * D/32) for P V. A
// step issues its K and V loads together (one round of memory latency) and
// keeps no second block in flight, so the loop fits the kernel's register
// budget without spilling. qs: the query heads times softmax_scale * log2(e).
template <int GRP, int D>
__device__ __forceinline__ void ds_key_loop(const __nv_bfloat16* kbase, const __nv_bfloat16* vbase, int64_t k_begin,
                                            int64_t k_end, int warp, int lane, const float (*qs)[D], float (&m)[GRP],
                                            float (&l)[GRP], float (&acc)[GRP][D / 32],
                                            unsigned long long* stamp = nullptr) {
    constexpr int DQ = D / 4, DL = D / 32;
    using VRaw = typename std::conditional<DL == 4, uint2, uint32_t>::type;
    const int kk = lane >> 2, qd = lane & 3;
#pragma unroll
    for (int h = 0; h < GRP; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int i = 0; i < DL; ++i) acc[h][i] = 0.f;
    }
    bool first = true;
    for (int64_t kb = k_begin + warp * 8; kb < k_end; kb += kDsConsumers * 8) {
#ifdef AMCU_DIAG
        if (stamp && first && lane == 0) stamp[0] = clock64();
#endif
        const int64_t key = kb + kk;
        const bool valid = key < k_end;
        uint4 kq[DQ / 8];
        VRaw vv[8];
#pragma unroll
        for (int i = 0; i < DQ / 8; ++i)
            kq[i] = valid ? *reinterpret_cast<const uint4*>(kbase + key * D + qd * DQ + i * 8) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int jj = 0; jj < 8; ++jj)
            vv[jj] = kb + jj < k_end ? *reinterpret_cast<const VRaw*>(vbase + (kb + jj) * D + lane * DL) : VRaw{};
        float sc[GRP];
#pragma unroll
        for (int h = 0; h < GRP; ++h) sc[h] = 0.f;
#pragma unroll
        for (int i = 0; i < DQ / 8; ++i) {
            const uint32_t w4[4] = {kq[i].x, kq[i].y, kq[i].z, kq[i].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float k0 = __uint_as_float(w4[e] << 16), k1 = __uint_as_float(w4[e] & 0xffff0000u);
                const int dd = qd * DQ + i * 8 + 2 * e;
#pragma unroll
                for (int h = 0; h < GRP; ++h) {
                    const float2 qq = *reinterpret_cast<const float2*>(&qs[h][dd]);
                    sc[h] = fmaf(qq.x, k0, fmaf(qq.y, k1, sc[h]));
                }
            }
        }
        float pr[GRP];
#ifdef AMCU_DIAG
        if (stamp && first && lane == 0) {
            stamp[1] = clock64() + ((unsigned long long)__float_as_uint(sc[0]) & 0);  // after the K loads' use
        }
#endif
#pragma unroll
        for (int h = 0; h < GRP; ++h) {
            sc[h] += __shfl_xor_sync(0xffffffffu, sc[h], 1);
            sc[h] += __shfl_xor_sync(0xffffffffu, sc[h], 2);
            const float sv = valid ? sc[h] : -INFINITY;
            float bm = fmaxf(sv, __shfl_xor_sync(0xffffffffu, sv, 4));
            bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 8));
            bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 16));
            const float mn = fmaxf(m[h], bm);
            const float corr = exp2f(m[h] - mn);
            pr[h] = valid ? exp2f(sv - mn) : 0.f;
            float bs = pr[h] + __shfl_xor_sync(0xffffffffu, pr[h], 4);
            bs += __shfl_xor_sync(0xffffffffu, bs, 8);
            bs += __shfl_xor_sync(0xffffffffu, bs, 16);
            l[h] = l[h] * corr + bs;
            m[h] = mn;
#pragma unroll
            for (int i = 0; i < DL; ++i) acc[h][i] *= corr;
        }
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
            float vf[DL];
            if constexpr (DL == 4) {
                const uint2 u = *reinterpret_cast<const uint2*>(&vv[jj]);
                vf[0] = __uint_as_float(u.x << 16); vf[1] = __uint_as_float(u.x & 0xffff0000u);
                vf[2] = __uint_as_float(u.y << 16); vf[3] = __uint_as_float(u.y & 0xffff0000u);
            } else {
                const uint32_t u = *reinterpret_cast<const uint32_t*>(&vv[jj]);
                vf[0] = __uint_as_float(u << 16); vf[1] = __uint_as_float(u & 0xffff0000u);
            }
#pragma unroll
            for (int h = 0; h < GRP; ++h) {
                const float pj = __shfl_sync(0xffffffffu, pr[h], 4 * jj);
#pragma unroll
                for (int i = 0; i < DL; ++i) acc[h][i] = fmaf(pj, vf[i], acc[h][i]);
            }
        }
#ifdef AMCU_DIAG
        if (stamp && first && lane == 0) {
            stamp[2] = clock64() + ((unsigned long long)__float_as_uint(acc[0][0]) & 0);
        }
#endif
        first = false;
    }
}

// L2 prefetch of the K (which == 0) or V rows [begin, min(end, pos)) of this
// CTA's attention units of a layer.
template <int D>
__device__ __forceinline__ void ds_prefetch_kv(const DsParams& p, const AmcuDecodeLayer& ly, int64_t pos, int ns,
                                               int which) {
    const int units = (int)p.nkv * ns;
    const int64_t Ltot = pos + 1;
    int64_t chunk = (Ltot + ns - 1) / ns;
    chunk = (chunk + 7) / 8 * 8;
    for (int un = blockIdx.x; un < units; un += gridDim.x) {
        const int kvh = un / ns, sp = un % ns;
        const int64_t b = (int64_t)sp * chunk;
        const int64_t e = b + chunk < pos ? b + chunk : pos;
        if (e <= b) continue;
        const __nv_bfloat16* base = static_cast<const __nv_bfloat16*>(which ? ly.v_cache : ly.k_cache) +
                                    (int64_t)kvh * p.capacity * D;
        for (int64_t r0 = b; r0 < e; r0 += 256) {  // pieces of at most 64 KB
            const int64_t r1 = r0 + 256 < e ? r0 + 256 : e;
            prefetch_l2_bulk(base + r0 * D, (uint32_t)((r1 - r0) * D * 2));
        }
    }
}

// Attention phase: units (kv head, key split) round-robin over the CTAs; each
// rotates its query heads, appends the new token's rotated k and v if its
// split holds the position, scores its keys and writes (max, sum,
// unnormalised output) per query head.
template <int GRP, int D>
__device__ __noinline__ void ds_attention(const DsParams& p, const AmcuDecodeLayer& ly, uint8_t* u, DsShared* sh,
                                          int64_t pos, int l) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float(*qs)[D] = reinterpret_cast<float(*)[D]>(u);
    float(*sm_m)[GRP] = reinterpret_cast<float(*)[GRP]>(u + GRP * D * 4);
    float(*sm_l)[GRP] = reinterpret_cast<float(*)[GRP]>(u + GRP * D * 4 + kDsConsumers * GRP * 4);
    float(*sm_o)[GRP][D] = reinterpret_cast<float(*)[GRP][D]>(u + GRP * D * 4 + 2 * kDsConsumers * GRP * 4);
    const int ns = sh->ns;
    const int units = (int)p.nkv * ns;
    const int64_t Ltot = pos + 1;
    int64_t chunk = (Ltot + ns - 1) / ns;
    chunk = (chunk + 7) / 8 * 8;
    for (int un = blockIdx.x; un < units; un += gridDim.x) {
        const int kvh = un / ns, sp = un % ns;
        const int64_t k_begin = (int64_t)sp * chunk;
        const int64_t k_end = k_begin + chunk < Ltot ? k_begin + chunk : Ltot;
        __nv_bfloat16* kbase = static_cast<__nv_bfloat16*>(ly.k_cache) + (int64_t)kvh * p.capacity * D;
        __nv_bfloat16* vbase = static_cast<__nv_bfloat16*>(ly.v_cache) + (int64_t)kvh * p.capacity * D;
        // rotate the query heads (cos/sin from the session's table, the same
        // values and rounding as the RoPE kernel) and, in the split that
        // holds the position, append the rotated k and the v of this token
        {
            constexpr int HALF = D / 2;
            const float2* cs = reinterpret_cast<const float2*>(p.cos_sin) + pos * HALF;
            const __nv_bfloat16* qrow = p.qkv + (int64_t)kvh * GRP * D;
            for (int i = threadIdx.x; i < GRP * HALF; i += kDsCT) {
                const int h = i / HALF, jj = i % HALF;
                const float2 c2 = cs[jj];
                const float x1 = __bfloat162float(__ldcg(qrow + h * D + jj));
                const float x2 = __bfloat162float(__ldcg(qrow + h * D + jj + HALF));
                qs[h][jj] = Act<__nv_bfloat16>::round(__fsub_rn(__fmul_rn(x1, c2.x), __fmul_rn(x2, c2.y))) *
                            p.scale_log2;
                qs[h][jj + HALF] = Act<__nv_bfloat16>::round(__fadd_rn(__fmul_rn(x2, c2.x), __fmul_rn(x1, c2.y))) *
                                   p.scale_log2;
            }
            if (k_begin <= pos && pos < k_end) {
                const __nv_bfloat16* krow = p.qkv + p.nq * D + (int64_t)kvh * D;
                const __nv_bfloat16* vrow = p.qkv + (p.nq + p.nkv) * D + (int64_t)kvh * D;
                __nv_bfloat16* kdst = kbase + pos * D;
                __nv_bfloat16* vdst = vbase + pos * D;
                for (int jj = threadIdx.x; jj < HALF; jj += kDsCT) {
                    const float2 c2 = cs[jj];
                    const float x1 = __bfloat162float(__ldcg(krow + jj)), x2 = __bfloat162float(__ldcg(krow + jj + HALF));
                    kdst[jj] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(x1, c2.x), __fmul_rn(x2, c2.y)));
                    kdst[jj + HALF] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(x2, c2.x), __fmul_rn(x1, c2.y)));
                }
                for (int jj = threadIdx.x; jj < D; jj += kDsCT) vdst[jj] = __ldcg(vrow + jj);
            }
        }
        named_bar_sync(kBarC, kDsCT);  // q staged; the appended row is visible to this CTA
        if (un == (int)blockIdx.x) ds_mark(p, l, 19);
        {
            DecodeWarpState<GRP, D> st;
            unsigned long long* stamp = nullptr;
#ifdef AMCU_DIAG
            if (p.trace && warp == 0 && un == (int)blockIdx.x)
                stamp = p.trace + ((size_t)blockIdx.x * p.nlayers + l) * kDsMarks + 22;
#endif
            ds_key_loop<GRP, D>(kbase, vbase, k_begin, k_end, warp, lane, qs, st.m, st.l, st.acc, stamp);
            decode_publish_warp<GRP, D>(st, warp, lane, sm_m, sm_l, sm_o);
        }
        named_bar_sync(kBarC, kDsCT);
        if (un == (int)blockIdx.x) ds_mark(p, l, 20);
        // partial per query head: [max, sum, unnormalised output] (D + 2 floats)
        float* w = p.attn_ws + ((int64_t)kvh * kDsMaxSplits + sp) * GRP * (D + 2);
        for (int e = threadIdx.x; e < GRP * D; e += kDsCT) {
            const int h = e / D, dd = e % D;
            float M, Ls, O;
            decode_merge_warps<GRP, D, kDsConsumers>(h, dd, sm_m, sm_l, sm_o, M, Ls, O);
            w[h * (D + 2) + 2 + dd] = O;
            if (dd == 0) {
                w[h * (D + 2)] = M;
                w[h * (D + 2) + 1] = Ls;
            }
        }
        named_bar_sync(kBarC, kDsCT);  // shared memory is reused by the next unit
        if (un == (int)blockIdx.x) ds_mark(p, l, 21);
    }
}

// 17 warps: one SM sub-partition holds 5 of them in its 16K registers, so a
// thread may use at most 96 (5 x 32 x 96 <= 16384).
template <int GRP, int D>
__global__ void __maxnreg__(96) decode_stack_kernel(DsParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ DsShared sh;
    const int64_t kmax = p.I > p.H ? p.I : p.H;
    const DsSmem L = ds_smem<GRP, D>(kmax, p.nq, p.stages, p.rbmax);
    DsRing r{smem + L.ring, reinterpret_cast<uint64_t*>(smem + L.bars),
             reinterpret_cast<uint64_t*>(smem + L.bars) + p.stages, p.stages, 0, 0u};
    const int64_t qkv_n = (p.nq + 2 * p.nkv) * D;
    const int G0 = (int)gridDim.x;
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&r.full[s], 1);
            mbar_init(&r.empty[s], kDsConsumers);
        }
        fence_mbar_init();
        sh.ok = 1;
    }
    __syncthreads();
    if (threadIdx.x >= kDsCT) {
        // weights depend on no earlier kernel: the stream starts before the dependency wait
        if (threadIdx.x == kDsCT) ds_produce<D>(p, r);
        return;
    }

    pdl_wait();
    const int64_t pos = p.seq_pos[0];
    const bool pos_ok = pos >= 0 && pos < p.capacity;
    if (threadIdx.x == 0) {
        int ns = (int)((pos + kDsKeysPerSplit) / kDsKeysPerSplit);
        const int cap = (int)(G0 / p.nkv) < kDsMaxSplits ? (int)(G0 / p.nkv) : kDsMaxSplits;
        sh.ns = ns < 1 ? 1 : (ns > cap ? cap : ns);
        if (!pos_ok && blockIdx.x == 0 && p.status) atomicExch(p.status, (int32_t)AM_STATUS_OUT_OF_RANGE);
    }
    named_bar_sync(kBarC, kDsCT);
    // the RoPE table row of this position serves every layer
    if (threadIdx.x == 0 && pos_ok) prefetch_l2_bulk(p.cos_sin + pos * D, (uint32_t)(D * 4));
    uint8_t* xs = smem + L.un;
    float* sx = reinterpret_cast<float*>(smem + L.sx);
    float* accs = reinterpret_cast<float*>(smem + L.accs);
    float* fw = reinterpret_cast<float*>(smem + L.fw);
    unsigned int q = 0;  // phases completed so far
    for (int l = 0; l < p.nlayers; ++l) {
        const AmcuDecodeLayer& ly = p.layers[l];
        int lo, hi;
        ds_mark(p, l, 0);
        // this CTA's attention units: pull their cached keys and values into L2
        // now (rows below pos are final), so the attention phase reads L2
        if (pos_ok && threadIdx.x < 2) ds_prefetch_kv<D>(p, ly, pos, sh.ns, threadIdx.x);
        // q/k/v = W_qkv RMSNorm(x)
        ds_range(qkv_n, blockIdx.x, G0, lo, hi);
        ds_stage<0, GRP, D>(p, p.x, static_cast<const __nv_bfloat16*>(ly.attn_norm), p.H, xs, sx, fw, accs,
                            (hi - lo) * 128, &sh);
        ds_mark(p, l, 1);
        ds_gemv<AMCU_EPI_STORE, D>(p, r, p.H, lo, hi, xs, sx, accs, p.qkv, &sh);
        ds_prefetch_l2(ly.mlp_norm, p.H * 2);
        ds_mark(p, l, 2);
        ds_sync(p, (++q) * G0, &sh);
        ds_mark(p, l, 3);
        // attention partials
        if (pos_ok) ds_attention<GRP, D>(p, ly, xs, &sh, pos, l);
        ds_mark(p, l, 4);
        ds_sync(p, (++q) * G0, &sh);
        ds_mark(p, l, 5);
        // x += W_o attention
        ds_range(p.H, blockIdx.x, G0, lo, hi);
        ds_stage<2, GRP, D>(p, nullptr, nullptr, p.nq * D, xs, sx, fw, accs, (hi - lo) * 128, &sh);
        ds_mark(p, l, 6);
        ds_gemv<AMCU_EPI_RESIDUAL_ADD, D>(p, r, p.nq * D, lo, hi, xs, sx, accs, p.x, &sh);
        ds_mark(p, l, 7);
        ds_sync(p, (++q) * G0, &sh);
        ds_mark(p, l, 8);
        // act = SiLU(W_gate RMSNorm(x)) * (W_up RMSNorm(x))
        ds_range(2 * p.I, blockIdx.x, G0, lo, hi);
        ds_stage<0, GRP, D>(p, p.x, static_cast<const __nv_bfloat16*>(ly.mlp_norm), p.H, xs, sx, fw, accs,
                            (hi - lo) * 128, &sh);
        ds_mark(p, l, 9);
        ds_gemv<AMCU_EPI_SILU_MUL, D>(p, r, p.H, lo, hi, xs, sx, accs, p.act, &sh);
        if (l + 1 < p.nlayers) ds_prefetch_l2(p.layers[l + 1].attn_norm, p.H * 2);
        ds_mark(p, l, 10);
        ds_sync(p, (++q) * G0, &sh);
        ds_mark(p, l, 11);
        // x += W_down act
        ds_range(p.H, blockIdx.x, G0, lo, hi);
        ds_stage<1, GRP, D>(p, p.act, nullptr, p.I, xs, sx, fw, accs, (hi - lo) * 128, &sh);
        ds_mark(p, l, 12);
        ds_gemv<AMCU_EPI_RESIDUAL_ADD, D>(p, r, p.I, lo, hi, xs, sx, accs, p.x, &sh);
        ds_mark(p, l, 13);
        if (l + 1 < p.nlayers) ds_sync(p, (++q) * G0, &sh);
        ds_mark(p, l, 14);
    }
    // leave: the last CTA out resets the counters for the next launch (every
    // other CTA has passed its last wait by then)
    named_bar_sync(kBarC, kDsCT);
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(p.sync + 32, 1u) == (unsigned int)G0 - 1) {
            atomicExch(p.sync, 0u);
            atomicExch(p.sync + 32, 0u);
        }
    }
    pdl_trigger();
}

template <int GRP, int D>
static am_status_code launch_stack(DsParams p, cudaStream_t s) {
    auto kern = decode_stack_kernel<GRP, D>;
    const int64_t kmax = p.I > p.H ? p.I : p.H;
    const int ctas = num_sms();
    {
        int64_t nmax = 2 * p.I > (p.nq + 2 * p.nkv) * D ? 2 * p.I : (p.nq + 2 * p.nkv) * D;
        if (p.H > nmax) nmax = p.H;
        p.rbmax = (int)((nmax / 16 + ctas - 1) / ctas);
    }
    int dev = 0, smem_max = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    smem_max -= (int)sizeof(DsShared) + 1024;
    // as many ring stages as still let one CTA reside on every SM
    int stages = 8, bytes = 0;
    for (; stages >= 3; --stages) {
        bytes = ds_smem<GRP, D>(kmax, p.nq, stages, p.rbmax).total;
        if (bytes > smem_max) continue;
        set_func_attr_once((const void*)kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max);
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kDsThreads, bytes) == cudaSuccess &&
            per_sm >= 1)
            break;
        cudaGetLastError();
    }
    if (stages < 3) {
        cudaFuncAttributes fa{};
        cudaFuncGetAttributes(&fa, kern);
        return set_error(AM_STATUS_INVALID_ARGUMENT,
                         "amcu_decode_stack: no CTA fits an SM (registers %d, max threads %d, static smem %zu, "
                         "dynamic smem %d)",
                         fa.numRegs, fa.maxThreadsPerBlock, fa.sharedSizeBytes, bytes);
    }
    p.stages = stages;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctas);
    cfg.blockDim = dim3(kDsThreads);
    cfg.dynamicSmemBytes = (size_t)bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(AM_STATUS_INTERNAL, "amcu_decode_stack launch: %s", cudaGetErrorString(e));
    }
#ifdef AMCU_DIAG
    if (p.trace) {
        // append this (eager, synchronised) step's stamps to the trace file
        const size_t n = (size_t)ctas * p.nlayers * kDsMarks;
        std::vector<unsigned long long> h(n);
        if (cudaStreamSynchronize(s) == cudaSuccess &&
            cudaMemcpy(h.data(), p.trace, n * 8, cudaMemcpyDeviceToHost) == cudaSuccess) {
            if (FILE* f = std::fopen(std::getenv("AMCU_DS_TRACE"), "ab")) {
                const int hdr[3] = {ctas, p.nlayers, kDsMarks};
                std::fwrite(hdr, sizeof(hdr), 1, f);
                std::fwrite(h.data(), 8, n, f);
                std::fclose(f);
            }
        }
    }
#endif
    return AM_STATUS_OK;
}

}  // namespace amcu

using namespace amcu;

extern "C" {

size_t amcu_decode_stack_workspace_bytes(const AmcuDecodeStackArgs* a) {
    if (!a || a->batch <= 0) return 0;
    const int64_t grp = a->n_q_heads / (a->n_kv_heads > 0 ? a->n_kv_heads : 1);
    const size_t ws = (size_t)a->n_kv_heads * kDsMaxSplits * grp * (a->head_dim + 2) * sizeof(float);
    return 256 + ws;
}

am_status_code amcu_decode_stack(const AmcuDecodeStackArgs* a, void* stream) {
    clear_error();
    AMCU_REQUIRE(a != nullptr, "amcu_decode_stack: null args");
    AMCU_REQUIRE(a->batch == 1, "amcu_decode_stack: batch must be 1");
    AMCU_REQUIRE(a->layers && a->n_layers > 0 && a->x && a->qkv && a->act && a->seq_pos && a->cos_sin,
                 "amcu_decode_stack: null pointer (the RoPE table cos_sin is required)");
    AMCU_REQUIRE(a->hidden % 128 == 0 && a->inter % 128 == 0 && (a->n_q_heads * a->head_dim) % 128 == 0,
                 "amcu_decode_stack: hidden, inter and n_q*head_dim must be multiples of 128");
    AMCU_REQUIRE(a->hidden <= kDsMaxK && a->inter <= kDsMaxK && a->n_q_heads * a->head_dim <= kDsMaxK,
                 "amcu_decode_stack: rows longer than %d columns are not supported", kDsMaxK);
    AMCU_REQUIRE(((a->n_q_heads + 2 * a->n_kv_heads) * a->head_dim) % 16 == 0, "amcu_decode_stack: bad q/k/v width");
    AMCU_REQUIRE(a->n_kv_heads > 0 && a->n_q_heads % a->n_kv_heads == 0, "amcu_decode_stack: n_q % n_kv != 0");
    AMCU_REQUIRE(a->n_q_heads <= kDsCT, "amcu_decode_stack: at most %d query heads", kDsCT);
    const size_t need = amcu_decode_stack_workspace_bytes(a);
    AMCU_REQUIRE(a->workspace && a->workspace_size >= need, "amcu_decode_stack: workspace of %zu bytes required", need);
    AMCU_REQUIRE(aligned(a->workspace, 256), "amcu_decode_stack: workspace must be 256-byte aligned");
    DsParams p{};
    p.layers = static_cast<const AmcuDecodeLayer*>(a->layers);
    p.nlayers = (int)a->n_layers;
    p.x = static_cast<__nv_bfloat16*>(a->x);
    p.qkv = static_cast<__nv_bfloat16*>(a->qkv);
    p.act = static_cast<__nv_bfloat16*>(a->act);
    p.H = a->hidden;
    p.I = a->inter;
    p.nq = a->n_q_heads;
    p.nkv = a->n_kv_heads;
    p.capacity = a->capacity;
    p.seq_pos = a->seq_pos;
    p.cos_sin = a->cos_sin;
    p.theta = a->theta;
    p.eps = a->rms_eps;
    p.scale_log2 = (float)(1.0 / sqrt((double)a->head_dim)) * kLog2e;
    uint8_t* w = static_cast<uint8_t*>(a->workspace);
    p.sync = reinterpret_cast<unsigned int*>(w);
    p.attn_ws = reinterpret_cast<float*>(w + 256);
    p.err = device_error_word();
    p.status = a->status;
    p.trace = nullptr;
#ifdef AMCU_DIAG
    if (std::getenv("AMCU_DS_TRACE")) {
        // diagnostics only (eager sessions): one stamp buffer, grown on demand
        static unsigned long long* buf = nullptr;
        static size_t cap = 0;
        const size_t n = (size_t)num_sms() * a->n_layers * kDsMarks;
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        cudaStreamIsCapturing(as_stream(stream), &cs);
        if (cs == cudaStreamCaptureStatusNone) {
            if (n > cap) {
                if (buf) cudaFree(buf);
                buf = nullptr;
                cap = 0;
                if (cudaMalloc(&buf, n * 8) == cudaSuccess) cap = n;
            }
            p.trace = buf;
            if (buf) cudaMemsetAsync(buf, 0, n * 8, as_stream(stream));
        }
    }
#endif
    const int grp = (int)(a->n_q_heads / a->n_kv_heads);
    const cudaStream_t s = as_stream(stream);
    if (a->head_dim == 128 && grp == 4) return launch_stack<4, 128>(p, s);
    if (a->head_dim == 128 && grp == 8) return launch_stack<8, 128>(p, s);
    if (a->head_dim == 64 && grp == 4) return launch_stack<4, 64>(p, s);
    return set_error(AM_STATUS_INVALID_ARGUMENT, "amcu_decode_stack: head_dim %lld with GQA group %d unsupported",
                     (long long)a->head_dim, grp);
}

}  // extern "C"
