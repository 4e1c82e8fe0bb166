// Persistent decode step: every decoder layer of a bs <= 2 INT4 decode step in
// one kernel.
//
// Semantics: for each layer, exactly the unfused plan's steps -- q/k/v GEMV
// with the fused attention RMSNorm, RoPE + KV append + attention, o GEMV +
// residual, gate/up GEMV with the fused MLP RMSNorm + SiLU-Mul, down GEMV +
// residual (the reference's BuildLlamaDense order, the same arithmetic and
// rounding points as gemv.cu and attention_rope.cu).
//
// Why one kernel: at bs = 1 every GEMV is a few microseconds of HBM
// streaming, and a kernel boundary costs a ramp-up (first weight bytes in
// flight, activations staged) and a drain (the last CTAs finishing) of the
// same order. Here one CTA per SM stays resident for the whole step:
//   * warp 16 is the producer: it streams the CTA's share of every layer's
//     weights (q/k/v, o, gate/up, down, layer after layer) through a ring of
//     16.5 KB shared-memory stages with bulk copies, waiting only for free
//     stages -- never for the phases -- so HBM keeps streaming while the
//     consumers wait at a grid barrier or run attention;
//   * warps 0-15 are consumers: a GEMV phase stages the activations (after a
//     grid barrier, since every CTA needs all of them), then consumes its row
//     blocks' stages, the 16 warps splitting each stage's 16 pair records;
//     the attention phase works on (sequence, kv head, split) units and the
//     last CTA to finish a (sequence, kv head) merges its splits.
// Grid barriers: a sense-reversing counter in global memory, one per phase
// (5 per layer). All waits are bounded: a wait that runs out records an
// error code in the device error word and the kernel runs on without
// waiting again (its results are then garbage, the host sees the code).
// The kernel is launched cooperatively (all CTAs co-resident or no launch).
#include <cooperative_groups.h>

#include <cstdio>
#include <cstdlib>
#include <vector>

#include "../amcu_internal.h"
#include "attn_decode.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "gemv_stage.cuh"
#include "mma_int4.cuh"

namespace amcu {

constexpr int kDsConsumers = 16;
constexpr int kDsThreads = (kDsConsumers + 1) * 32;
constexpr int kDsCT = kDsConsumers * 32;             // consumer threads
constexpr int kDsUnits = 16;                         // pair records per stage
constexpr int kDsStageBytes = kDsUnits * kW4PairBytes;
constexpr int kDsMaxRows = 2;                        // activation rows (sequences) per step
constexpr int kDsMaxSplits = 64;                     // attention splits per (sequence, kv head)
constexpr int32_t kErrDsBarrier = 0x301, kErrDsFull = 0x302, kErrDsEmpty = 0x303;
constexpr int kBarGemv = 1, kBarStage = 2, kBarAttn = 3;  // named barriers of the consumers

struct DsParams {
    const AmcuDecodeLayer* layers;
    int nlayers;
    __nv_bfloat16 *x, *qkv, *attn, *act;  // residual stream [B][H], q/k/v [B][qkv_n], attention [B][nq*D], act [B][I]
    int B;
    int64_t H, I, nq, nkv;
    int64_t capacity, slot_stride;
    const int32_t* seq_pos;
    const float* cos_sin;
    double theta;
    float eps, scale_log2;
    float* attn_ws;               // [B][nkv][ns][GRP][D + 2]
    int32_t* attn_cnt;            // [B][nkv] arrivals (zero between uses)
    unsigned int* bar;            // grid barrier words (zero between uses)
    int ns;                       // attention splits per (sequence, kv head)
    int stages;
    int32_t *err, *status;
    int rbmax;     // most row blocks a CTA owns in any GEMV phase
    int dbg_skip;  // diagnostics, AMCU_DIAG builds only (AMCU_DS_SKIP): bit 0 skips attention, bit 1 the grid barriers, bit 2 the weight stream (wrong results)
    unsigned long long* trace;  // diagnostics, AMCU_DIAG builds only (AMCU_DS_TRACE): [cta][layer][kDsMarks] globaltimer stamps, or null
};

constexpr int kDsMarks = 26;  // trace stamps per layer
#ifdef AMCU_DIAG
#define DS_SKIP(p) ((p).dbg_skip)
#define DS_TRACE(p) ((p).trace)
#else
#define DS_SKIP(p) 0
#define DS_TRACE(p) ((unsigned long long*)nullptr)
#endif

__device__ __forceinline__ void ds_mark(const DsParams& p, int l, int idx) {
    if (DS_TRACE(p) && threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        DS_TRACE(p)[((size_t)blockIdx.x * p.nlayers + l) * kDsMarks + idx] = t;
        if (idx == 0 || idx == 18)  // SM clock cycles beside the layer's first and last stamps
            DS_TRACE(p)[((size_t)blockIdx.x * p.nlayers + l) * kDsMarks + (idx == 0 ? 24 : 25)] = clock64();
    }
}

// Row blocks [lo, hi) of an n-row weight that CTA c of `ctas` handles.
__device__ __forceinline__ void ds_range(int64_t n, int c, int ctas, int& lo, int& hi) {
    const int64_t nrb = n / 16;
    lo = (int)(nrb * c / ctas);
    hi = (int)(nrb * (c + 1) / ctas);
}

__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* a) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
    return v;
}
__device__ __forceinline__ unsigned int atom_add_acq_rel_gpu(unsigned int* a, unsigned int v) {
    unsigned int old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(a), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void st_relaxed_gpu(unsigned int* a, unsigned int v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}

// Consumer-side grid barrier, two levels: after the consumer threads meet,
// thread 0 arrives (release) on its group's counter (CTA % kDsBarGroups,
// each counter in its own 128-byte line); the last arrival of a group
// arrives on the top counter, and the last arrival there resets it and bumps
// the generation word, on which everyone else spins with acquire loads
// (bounded). Counters return to zero before the generation moves.
constexpr int kDsBarGroups = 16;
constexpr int kDsBarWords = 32 * (2 + kDsBarGroups);  // gen, top, groups: one 128-byte line each
__device__ __forceinline__ void ds_grid_barrier(const DsParams& p, bool& ok) {
    if (DS_SKIP(p) & 2) return;
    named_bar_sync(kBarGemv, kDsCT);
    if (threadIdx.x == 0) {
        unsigned int* gen = p.bar;
        unsigned int* top = p.bar + 32;
        const int grp = blockIdx.x % kDsBarGroups;
        const int ngrp = (int)gridDim.x < kDsBarGroups ? (int)gridDim.x : kDsBarGroups;
        const unsigned int members = (gridDim.x - grp + kDsBarGroups - 1) / kDsBarGroups;
        unsigned int* cnt = p.bar + 64 + 32 * grp;
        const unsigned int g0 = ld_acquire_gpu(gen);
        bool released = false;
        if (atom_add_acq_rel_gpu(cnt, 1u) == members - 1) {
            st_relaxed_gpu(cnt, 0u);
            if (atom_add_acq_rel_gpu(top, 1u) == (unsigned int)ngrp - 1) {
                st_relaxed_gpu(top, 0u);
                atom_add_acq_rel_gpu(gen, 1u);
                released = true;
            }
        }
        if (!released && ok) {
            const long long t0 = clock64();
            while (ld_acquire_gpu(gen) == g0) {
                if (clock64() - t0 > kSpinLimitCycles) {
                    record_device_error(p.err, kErrDsBarrier);
                    ok = false;
                    break;
                }
            }
        }
    }
    named_bar_sync(kBarGemv, kDsCT);
}

// L2 prefetch of a small read-only array (a norm weight) a phase before its
// use, so the staging after the next grid barrier does not wait on HBM.
__device__ __forceinline__ void ds_prefetch_l2(const void* ptr, int64_t bytes) {
    if (blockIdx.x != 0 || ptr == nullptr) return;
    for (int64_t off = (int64_t)threadIdx.x * 128; off < bytes; off += (int64_t)kDsCT * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(static_cast<const char*>(ptr) + off));
}

struct DsSmem {
    int ring, bars, red, sx, un, total;
};
template <int GRP, int D>
__host__ __device__ inline DsSmem ds_smem(int64_t kmax, int stages, int rbmax) {
    auto up = [](int64_t v) { return (int)((v + 127) / 128 * 128); };
    const int64_t xs = kDsMaxRows * (kmax * 2 + 16);
    const int64_t att = (int64_t)GRP * D * 4 + 2 * kDsConsumers * GRP * 4 + (int64_t)kDsConsumers * GRP * D * 4 + 64;
    DsSmem s;
    s.ring = 0;
    s.bars = stages * kDsStageBytes;
    s.red = s.bars + up(2 * stages * 8);
    s.sx = s.red + up((int64_t)rbmax * 16 * 8 * 4);  // [rbmax][16 rows][8 activation rows] fp32
    s.un = s.sx + up(kmax / 128 * 8 * 4);
    s.total = s.un + up(xs > att ? xs : att);
    return s;
}

// The consumers' view of the ring.
struct DsRing {
    uint8_t* ring;
    uint64_t *full, *empty;
    int S, slot;
    uint32_t phase;
};

// One GEMV phase of the consumers: y = epilogue(x @ W^T) for this CTA's row
// blocks, W an INT4 [n][k] weight whose stages the producer streams.
template <int EPI>
__device__ __noinline__ void ds_gemv(const DsParams& p, DsRing& r, int64_t n, int64_t k, const __nv_bfloat16* x,
                        const __nv_bfloat16* norm_w, __nv_bfloat16* y, uint8_t* smem, const DsSmem& L,
                        StageShared* stsh, bool& ok, int l, int m0) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int M = p.B;
    const int xrow = (int)(k * 2 + 16);
    uint8_t* xs = smem + L.un;
    float* sx = reinterpret_cast<float*>(smem + L.sx);
    float* accs = reinterpret_cast<float*>(smem + L.red);
    {
        int lo0, hi0;
        ds_range(n, blockIdx.x, gridDim.x, lo0, hi0);
        for (int i = threadIdx.x; i < (hi0 - lo0) * 128; i += kDsCT) accs[i] = 0.f;  // staging's barriers publish this
    }
    {
        StageCtx sc{x, k, k, M, norm_w, p.eps, xs, xrow, sx, stsh, (int)threadIdx.x, kDsCT, kBarStage};
        stage_activations<true, true>(sc);
    }
    ds_mark(p, l, m0);
    const uint8_t* xr = xs + (g < M ? g : 0) * xrow + 32 * t;  // + 256 B per group
    const int per_row = (int)(k / 128) / kDsUnits;
    int lo, hi;
    ds_range(n, blockIdx.x, gridDim.x, lo, hi);
    // every warp adds its partial tile of a row block into accs[row block]
    // (shared-memory float atomics), so no warp waits for another until the
    // phase's row blocks are all consumed
    // The ring state and flags live in registers for the loop (the caller's
    // copies sit in local memory, which every asm memory clobber would reload).
    const uint8_t* const ring = r.ring + warp * kW4PairBytes;
    uint64_t* const full = r.full;
    uint64_t* const empty = r.empty;
    const int S = r.S;
    int slot = r.slot;
    uint32_t phase = r.phase;
    const bool stream = !(DS_SKIP(p) & 4);
    bool live = ok;
    for (int rb = lo; rb < hi; ++rb) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int j = 0; j < per_row; ++j) {
            if (live && stream && !mbar_wait(&full[slot], phase)) {
                live = false;
                if (lane == 0) record_device_error(p.err, kErrDsFull);
            }
            const uint8_t* rec = ring + slot * kDsStageBytes;
            const int grp = j * kDsUnits + warp;
            const uint8_t* xp = xr + grp * 256;
            float part[2][4];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
#pragma unroll
                for (int e = 0; e < 4; ++e) part[h][e] = 0.f;
                const uint4 x0 = *reinterpret_cast<const uint4*>(xp + h * 128);
                const uint4 x1 = *reinterpret_cast<const uint4*>(xp + h * 128 + 16);
                const uint4 wv = *reinterpret_cast<const uint4*>(rec + h * 512 + lane * 16);
                uint32_t a[4];
                unpack_w4_word_f16(wv.x, a);
                mma_f16_16816(part[h], a, x0.x, x0.y);
                unpack_w4_word_f16(wv.y, a);
                mma_f16_16816(part[h], a, x0.z, x0.w);
                unpack_w4_word_f16(wv.z, a);
                mma_f16_16816(part[h], a, x1.x, x1.y);
                unpack_w4_word_f16(wv.w, a);
                mma_f16_16816(part[h], a, x1.z, x1.w);
            }
            const float2 s2x = *reinterpret_cast<const float2*>(sx + grp * 8 + 2 * t);
            const uint32_t sv = *reinterpret_cast<const uint32_t*>(rec + 1024 + 4 * g);
            const __half2 s2 = *reinterpret_cast<const __half2*>(&sv);
            const float s_lo = __low2float(s2), s_hi = __high2float(s2) * 0.0625f;
            acc[0] = fmaf(fmaf(-1032.f, s2x.x, part[0][0] + part[1][0]), s_lo, acc[0]);
            acc[1] = fmaf(fmaf(-1032.f, s2x.y, part[0][1] + part[1][1]), s_lo, acc[1]);
            acc[2] = fmaf(fmaf(-1152.f, s2x.x, part[0][2] + part[1][2]), s_hi, acc[2]);
            acc[3] = fmaf(fmaf(-1152.f, s2x.y, part[0][3] + part[1][3]), s_hi, acc[3]);
            __syncwarp();
            if (lane == 0 && stream) mbar_arrive(&empty[slot]);
            if (++slot == S) {
                slot = 0;
                phase ^= 1;
            }
        }
        // lane (g, t): rows g and g+8 of the block, activation rows 2t and 2t+1
        float* a16 = accs + (rb - lo) * 128;
        atomicAdd(a16 + g * 8 + 2 * t, acc[0]);
        atomicAdd(a16 + g * 8 + 2 * t + 1, acc[1]);
        atomicAdd(a16 + (g + 8) * 8 + 2 * t, acc[2]);
        atomicAdd(a16 + (g + 8) * 8 + 2 * t + 1, acc[3]);
    }
    r.slot = slot;
    r.phase = phase;
    ok = live;
    named_bar_sync(kBarGemv, kDsCT);
    ds_mark(p, l, m0 + 1);
    // epilogue over (row block, weight row, activation row)
    const float* rmul = stsh->row_mul;
    const int nloc = hi - lo;
    if constexpr (EPI == AMCU_EPI_SILU_MUL) {
        // rows 0-7 of a block are gate rows 8 rb .. 8 rb + 7, rows 8-15 the matching up rows
        const int64_t ys = n / 2;
        for (int e = threadIdx.x; e < nloc * 8 * M; e += kDsCT) {
            const int m = e % M, rr = (e / M) % 8, rl = e / (M * 8);
            const float* a16 = accs + rl * 128;
            const float gt = Act<__nv_bfloat16>::round(a16[rr * 8 + m] * rmul[m]);
            const float up = Act<__nv_bfloat16>::round(a16[(rr + 8) * 8 + m] * rmul[m]);
            y[m * ys + (int64_t)(lo + rl) * 8 + rr] = __float2bfloat16_rn(silu_ref(gt) * up);
        }
    } else {
        for (int e = threadIdx.x; e < nloc * 16 * M; e += kDsCT) {
            const int m = e % M, rr = (e / M) % 16, rl = e / (M * 16);
            const int64_t off = m * n + (int64_t)(lo + rl) * 16 + rr;
            float o = Act<__nv_bfloat16>::round(accs[rl * 128 + rr * 8 + m] * rmul[m]);
            if constexpr (EPI == AMCU_EPI_RESIDUAL_ADD) o = o + __bfloat162float(y[off]);  // y is the residual
            y[off] = __float2bfloat16_rn(o);
        }
    }
}

// Attention phase: units (sequence b, kv head, split) round-robin over the
// CTAs; each writes a (max, sum, unnormalised output) partial, and the last
// CTA to finish a (b, kv head) merges its ns splits into p.attn.
template <int GRP, int D>
__device__ __noinline__ void ds_attention(const DsParams& p, const AmcuDecodeLayer& ly, uint8_t* smem, const DsSmem& L, bool& ok,
                                         int l) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t qkv_n = (p.nq + 2 * p.nkv) * D;
    uint8_t* u = smem + L.un;
    float(*qs)[D] = reinterpret_cast<float(*)[D]>(u);
    float(*sm_m)[GRP] = reinterpret_cast<float(*)[GRP]>(u + GRP * D * 4);
    float(*sm_l)[GRP] = reinterpret_cast<float(*)[GRP]>(u + GRP * D * 4 + kDsConsumers * GRP * 4);
    float(*sm_o)[GRP][D] = reinterpret_cast<float(*)[GRP][D]>(u + GRP * D * 4 + 2 * kDsConsumers * GRP * 4);
    int* last = reinterpret_cast<int*>(u + GRP * D * 4 + 2 * kDsConsumers * GRP * 4 + kDsConsumers * GRP * D * 4);
    const int units = p.B * (int)p.nkv * p.ns;
    for (int un = blockIdx.x; un < units; un += gridDim.x) {
        const int b = un / ((int)p.nkv * p.ns), kvh = (un / p.ns) % (int)p.nkv, sp = un % p.ns;
        const int64_t pos = p.seq_pos[b];
        if (pos < 0 || pos >= p.capacity) {
            if (kvh == 0 && sp == 0 && threadIdx.x == 0 && p.status) atomicExch(p.status, (int32_t)AM_STATUS_OUT_OF_RANGE);
            continue;
        }
        const int64_t Ltot = pos + 1;
        int64_t chunk = (Ltot + p.ns - 1) / p.ns;
        chunk = (chunk + 7) / 8 * 8;
        const int64_t k_begin = (int64_t)sp * chunk;
        const int64_t k_end = k_begin + chunk < Ltot ? k_begin + chunk : Ltot;
        __nv_bfloat16* kbase = static_cast<__nv_bfloat16*>(ly.k_cache) + b * p.slot_stride + (int64_t)kvh * p.capacity * D;
        __nv_bfloat16* vbase = static_cast<__nv_bfloat16*>(ly.v_cache) + b * p.slot_stride + (int64_t)kvh * p.capacity * D;
        const __nv_bfloat16* row = p.qkv + b * qkv_n;
        rope_stage_q<GRP, D, true>(row + (int64_t)kvh * GRP * D, pos, p.cos_sin, p.theta, p.scale_log2, qs, threadIdx.x, kDsCT);
        if (k_begin <= pos && pos < k_end)
            rope_append_kv<D, true>(row + p.nq * D + (int64_t)kvh * D, row + (p.nq + p.nkv) * D + (int64_t)kvh * D,
                              kbase + pos * D, vbase + pos * D, pos, p.cos_sin, p.theta, threadIdx.x, kDsCT);
        named_bar_sync(kBarAttn, kDsCT);  // q staged; the appended row is visible to this CTA
        if (un == blockIdx.x) ds_mark(p, l, 20);
        DecodeWarpState<GRP, D> st;
        DecodeKeyLoop<GRP, D, kDsConsumers> loop(kbase, vbase, k_begin, k_end, warp, lane);
        loop.run(qs, st);
        decode_publish_warp<GRP, D>(st, warp, lane, sm_m, sm_l, sm_o);
        named_bar_sync(kBarAttn, kDsCT);
        if (un == blockIdx.x) ds_mark(p, l, 21);
        float* w = p.attn_ws + (((int64_t)b * p.nkv + kvh) * p.ns + sp) * GRP * (D + 2);
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
        __threadfence();
        named_bar_sync(kBarAttn, kDsCT);
        if (threadIdx.x == 0) {
            int32_t* cnt = p.attn_cnt + (int64_t)b * p.nkv + kvh;
            *last = atomicAdd(cnt, 1) == p.ns - 1;
            if (*last) *cnt = 0;  // reset for the next layer (every arrival is in)
        }
        named_bar_sync(kBarAttn, kDsCT);
        if (un == blockIdx.x) ds_mark(p, l, 22);
        if (*last) {
            // merge the ns partials: every split's (max, sum) to shared memory
            // first (one round of loads), then each output element sums its ns
            // terms with independent loads
            __threadfence();
            const float* w0 = p.attn_ws + ((int64_t)b * p.nkv + kvh) * p.ns * GRP * (D + 2);
            float* fm = &sm_o[0][0][0];           // [ns][GRP] maxima, then weights exp2(m - M) (sm_o is free now)
            float* fs = fm + kDsMaxSplits * GRP;   // [ns][GRP] sums
            float* fl = fs + kDsMaxSplits * GRP;   // [GRP] total sums
            for (int i = threadIdx.x; i < p.ns * GRP; i += kDsCT) {
                fm[i] = __ldcg(w0 + i * (D + 2));
                fs[i] = __ldcg(w0 + i * (D + 2) + 1);
            }
            named_bar_sync(kBarAttn, kDsCT);
            if (threadIdx.x < GRP) {
                const int h = threadIdx.x;
                float M = -INFINITY;
                for (int s = 0; s < p.ns; ++s) M = fmaxf(M, fm[s * GRP + h]);
                float Ls = 0.f;
                for (int s = 0; s < p.ns; ++s) {
                    const float m = fm[s * GRP + h];
                    const float f = m == -INFINITY ? 0.f : exp2f(m - M);  // -inf: an empty split
                    Ls += fs[s * GRP + h] * f;
                    fm[s * GRP + h] = f;
                }
                fl[h] = Ls;
            }
            named_bar_sync(kBarAttn, kDsCT);
            for (int e = threadIdx.x; e < GRP * D; e += kDsCT) {
                const int h = e / D, dd = e % D;
                float O = 0.f;
#pragma unroll 8
                for (int s = 0; s < p.ns; ++s) O += __ldcg(w0 + (s * GRP + h) * (D + 2) + 2 + dd) * fm[s * GRP + h];
                p.attn[(int64_t)b * p.nq * D + ((int64_t)kvh * GRP + h) * D + dd] = __float2bfloat16_rn(O / fl[h]);
            }
        }
        named_bar_sync(kBarAttn, kDsCT);  // shared memory is reused by the next unit
        if (un == blockIdx.x) ds_mark(p, l, 23);
    }
    (void)ok;
}

template <int GRP, int D>
__global__ void __maxnreg__(96) decode_stack_kernel(DsParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ StageShared stsh;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t kmax = p.I > p.H ? p.I : p.H;
    const DsSmem L = ds_smem<GRP, D>(kmax, p.stages, p.rbmax);
    DsRing r{smem + L.ring, reinterpret_cast<uint64_t*>(smem + L.bars),
             reinterpret_cast<uint64_t*>(smem + L.bars) + p.stages, p.stages, 0, 0u};
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&r.full[s], 1);
            mbar_init(&r.empty[s], kDsConsumers);
        }
        fence_mbar_init();
    }
    __syncthreads();
    const int64_t qkv_n = (p.nq + 2 * p.nkv) * D;

    if (warp == kDsConsumers) {
        // ---- producer: the CTA's share of every layer's weights, in consumption order
        if (lane == 0 && !(DS_SKIP(p) & 4)) {
            int slot = 0;
            uint32_t phase = 0;
            int64_t i = 0;
            bool live = true;
            for (int l = 0; l < p.nlayers && live; ++l) {
                const AmcuDecodeLayer& ly = p.layers[l];
                const uint8_t* ws[4] = {static_cast<const uint8_t*>(ly.w_qkv), static_cast<const uint8_t*>(ly.w_o),
                                        static_cast<const uint8_t*>(ly.w_gate_up), static_cast<const uint8_t*>(ly.w_down)};
                const int64_t ns[4] = {qkv_n, p.H, 2 * p.I, p.H};
                const int64_t ks[4] = {p.H, p.nq * D, p.H, p.I};
                for (int ph = 0; ph < 4 && live; ++ph) {
                    const int per_row = (int)(ks[ph] / 128) / kDsUnits;
                    int lo, hi;
                    ds_range(ns[ph], blockIdx.x, gridDim.x, lo, hi);
                    const uint8_t* run = ws[ph] + (size_t)lo * (ks[ph] / 128) * kW4PairBytes;
                    for (int j = 0; j < (hi - lo) * per_row; ++j, ++i) {
                        if (i >= p.stages && !mbar_wait(&r.empty[slot], phase ^ 1u)) {
                            record_device_error(p.err, kErrDsEmpty);
                            live = false;
                            break;
                        }
                        mbar_expect_tx(&r.full[slot], kDsStageBytes);
                        bulk_g2s(r.ring + slot * kDsStageBytes, run + (size_t)j * kDsStageBytes, kDsStageBytes,
                                 &r.full[slot]);
                        if (++slot == p.stages) {
                            slot = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
        }
        return;
    }

    // ---- consumers
    pdl_wait();
    bool ok = true;
    for (int l = 0; l < p.nlayers; ++l) {
        const AmcuDecodeLayer& ly = p.layers[l];
        ds_mark(p, l, 0);
        if (l > 0) ds_grid_barrier(p, ok);  // the previous layer's residual stream is complete
        ds_mark(p, l, 1);
        ds_gemv<AMCU_EPI_STORE>(p, r, qkv_n, p.H, p.x, static_cast<const __nv_bfloat16*>(ly.attn_norm), p.qkv, smem, L,
                                &stsh, ok, l, 2);
        ds_mark(p, l, 4);
        ds_grid_barrier(p, ok);
        ds_mark(p, l, 5);
        if (!(DS_SKIP(p) & 1)) ds_attention<GRP, D>(p, ly, smem, L, ok, l);
        ds_mark(p, l, 6);
        ds_grid_barrier(p, ok);
        ds_mark(p, l, 7);
        ds_prefetch_l2(ly.mlp_norm, p.H * 2);
        ds_gemv<AMCU_EPI_RESIDUAL_ADD>(p, r, p.H, p.nq * D, p.attn, nullptr, p.x, smem, L, &stsh, ok, l, 8);
        ds_mark(p, l, 10);
        ds_grid_barrier(p, ok);
        ds_mark(p, l, 11);
        ds_gemv<AMCU_EPI_SILU_MUL>(p, r, 2 * p.I, p.H, p.x, static_cast<const __nv_bfloat16*>(ly.mlp_norm), p.act,
                                   smem, L, &stsh, ok, l, 12);
        ds_mark(p, l, 14);
        ds_grid_barrier(p, ok);
        ds_mark(p, l, 15);
        if (l + 1 < p.nlayers) ds_prefetch_l2(p.layers[l + 1].attn_norm, p.H * 2);
        ds_gemv<AMCU_EPI_RESIDUAL_ADD>(p, r, p.H, p.I, p.act, nullptr, p.x, smem, L, &stsh, ok, l, 16);
        ds_mark(p, l, 18);
    }
    pdl_trigger();
}

template <int GRP, int D>
static am_status_code launch_stack(DsParams p, cudaStream_t s) {
    auto kern = decode_stack_kernel<GRP, D>;
    const int64_t kmax = p.I > p.H ? p.I : p.H;
    {
        int64_t nmax = 2 * p.I > (p.nq + 2 * p.nkv) * D ? 2 * p.I : (p.nq + 2 * p.nkv) * D;
        if (p.H > nmax) nmax = p.H;
        const int ctas = num_sms();
        p.rbmax = (int)((nmax / 16 + ctas - 1) / ctas);
    }
    int dev = 0, smem_max = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    smem_max -= (int)sizeof(StageShared) + 1024;
    // as many ring stages as still let one CTA reside on every SM
    int stages = 12, bytes = 0;
    for (; stages >= 3; --stages) {
        bytes = ds_smem<GRP, D>(kmax, stages, p.rbmax).total;
        if (bytes > smem_max) continue;
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
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
                         fa.numRegs, fa.maxThreadsPerBlock, fa.sharedSizeBytes, ds_smem<GRP, D>(kmax, 3, p.rbmax).total);
    }
    p.stages = stages;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)num_sms());
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
        // diagnostics: append the stamps of this (eager, synchronised) step to the trace file
        const size_t n = (size_t)num_sms() * p.nlayers * kDsMarks;
        std::vector<unsigned long long> h(n);
        if (cudaStreamSynchronize(s) == cudaSuccess &&
            cudaMemcpy(h.data(), p.trace, n * 8, cudaMemcpyDeviceToHost) == cudaSuccess) {
            if (FILE* f = std::fopen(std::getenv("AMCU_DS_TRACE"), "ab")) {
                const int hdr[3] = {num_sms(), p.nlayers, kDsMarks};
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
    const size_t ws = (size_t)a->batch * a->n_kv_heads * kDsMaxSplits * grp * (a->head_dim + 2) * sizeof(float);
    const size_t cnt = (size_t)a->batch * a->n_kv_heads * sizeof(int32_t);
    return kDsBarWords * 4 + (cnt + 255) / 256 * 256 + ws;
}

am_status_code amcu_decode_stack(const AmcuDecodeStackArgs* a, void* stream) {
    clear_error();
    AMCU_REQUIRE(a != nullptr, "amcu_decode_stack: null args");
    AMCU_REQUIRE(a->batch >= 1 && a->batch <= kDsMaxRows, "amcu_decode_stack: batch must be 1..%d", kDsMaxRows);
    AMCU_REQUIRE(a->layers && a->n_layers > 0 && a->x && a->qkv && a->attn && a->act && a->seq_pos,
                 "amcu_decode_stack: null pointer");
    AMCU_REQUIRE(a->hidden % 2048 == 0 && a->inter % 2048 == 0 && (a->n_q_heads * a->head_dim) % 2048 == 0,
                 "amcu_decode_stack: hidden, inter and n_q*head_dim must be multiples of 2048");
    AMCU_REQUIRE(((a->n_q_heads + 2 * a->n_kv_heads) * a->head_dim) % 16 == 0, "amcu_decode_stack: bad q/k/v width");
    AMCU_REQUIRE(a->n_kv_heads > 0 && a->n_q_heads % a->n_kv_heads == 0, "amcu_decode_stack: n_q % n_kv != 0");
    const size_t need = amcu_decode_stack_workspace_bytes(a);
    AMCU_REQUIRE(a->workspace && a->workspace_size >= need, "amcu_decode_stack: workspace of %zu bytes required", need);
    AMCU_REQUIRE(aligned(a->workspace, 256), "amcu_decode_stack: workspace must be 256-byte aligned");
    DsParams p{};
    p.layers = static_cast<const AmcuDecodeLayer*>(a->layers);
    p.nlayers = (int)a->n_layers;
    p.x = static_cast<__nv_bfloat16*>(a->x);
    p.qkv = static_cast<__nv_bfloat16*>(a->qkv);
    p.attn = static_cast<__nv_bfloat16*>(a->attn);
    p.act = static_cast<__nv_bfloat16*>(a->act);
    p.B = (int)a->batch;
    p.H = a->hidden;
    p.I = a->inter;
    p.nq = a->n_q_heads;
    p.nkv = a->n_kv_heads;
    p.capacity = a->capacity;
    p.slot_stride = a->slot_stride ? a->slot_stride : a->n_kv_heads * a->capacity * a->head_dim;
    p.seq_pos = a->seq_pos;
    p.cos_sin = a->cos_sin;
    p.theta = a->theta;
    p.eps = a->rms_eps;
    p.scale_log2 = (float)(1.0 / sqrt((double)a->head_dim)) * kLog2e;
    uint8_t* w = static_cast<uint8_t*>(a->workspace);
    p.bar = reinterpret_cast<unsigned int*>(w);
    p.attn_cnt = reinterpret_cast<int32_t*>(w + kDsBarWords * 4);
    p.attn_ws = reinterpret_cast<float*>(w + kDsBarWords * 4 + ((size_t)a->batch * a->n_kv_heads * 4 + 255) / 256 * 256);
    // splits: about one (sequence, kv head, split) unit per SM
    int ns = (int)(num_sms() / (a->batch * a->n_kv_heads));
    p.ns = ns < 1 ? 1 : (ns > kDsMaxSplits ? kDsMaxSplits : ns);
    p.err = device_error_word();
    p.status = a->status;
    p.dbg_skip = 0;
    p.trace = nullptr;
#ifdef AMCU_DIAG
    static const int dbg = [] {
        const char* v = std::getenv("AMCU_DS_SKIP");
        return v ? std::atoi(v) : 0;
    }();
    p.dbg_skip = dbg;
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
