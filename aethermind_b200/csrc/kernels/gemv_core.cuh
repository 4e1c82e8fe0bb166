// Device building blocks of the decode GEMV kernel (gemv.cu), for any kernel
// that streams the tile16x64 weight format described there: the epilogues,
// the shared-memory carve-up, and the per-record and per-stage MMA loops.
#pragma once
#include "../amcu_internal.h"
#include "allreduce.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "mma_int4.cuh"

namespace amcu {

template <typename T>
__device__ __forceinline__ T epi_store(float v) { return Act<T>::store(v); }

__device__ __forceinline__ void st_release_sys_u32(uint32_t* a, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* a) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t gemv_clock_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
constexpr int32_t kErrGemvPeerWait = 0x402;
// The residual epilogue with the tensor-parallel sum over the ranks: its own
// kernel instantiation, so the single-GPU residual kernel keeps its code.
constexpr int kEpiResidualPeer = 3;

// Tensor-parallel o/down epilogue: y = round(residual + round(sum_r p_r)), the
// sum over the ranks' fp32 partials p_r of this row block, exchanged over peer
// memory by this warp alone (every rank's CTA owns the same row blocks):
//   1. e = epoch[rb] + 1; push this rank's partials into every peer's mailbox
//      (parity e & 1, slot of this rank), fence at system scope, release-store
//      e into each peer's flag of (this rank, rb);
//   2. wait (bounded) until every peer's flag of rb here is >= e;
//   3. sum the ranks' partials in rank order (the same order on every rank),
//      round, add the residual, store; epoch[rb] = e.
// Two parities suffice as in the one-shot all-reduce: a rank overwrites a
// parity only after its wait in the next call proved every peer finished
// reading it. Lane (g, t): rows g and g+8 of the block, activation rows 2t,
// 2t+1; the mailbox keeps [row][activation row < 8].
__device__ __forceinline__ void gemv_peer_sum_epilogue(const GemvParams& p, int64_t rb, int g, int t, const float (&acc)[4]) {
    const int lane = (g << 2) | t, rank = p.fuse.rank, world = p.fuse.world;
    uint8_t* own = p.fuse.area[rank];
    uint32_t* epochs = reinterpret_cast<uint32_t*>(own + ar_fuse_epochs_offset());
    const uint32_t e = epochs[rb] + 1;
    const int par = (int)(e & 1u);
    const int64_t n_lo = rb * 16 + g, n_hi = n_lo + 8;
    const int64_t i_lo = n_lo * 8 + 2 * t, i_hi = n_hi * 8 + 2 * t;
    const float2 v_lo = make_float2(acc[0], acc[1]), v_hi = make_float2(acc[2], acc[3]);
    for (int q = 0; q < world; ++q) {
        if (q == rank) continue;
        uint8_t* pa = p.fuse.area[q];
        *reinterpret_cast<float2*>(pa + ar_fuse_mail_offset(par, rank, i_lo)) = v_lo;
        *reinterpret_cast<float2*>(pa + ar_fuse_mail_offset(par, rank, i_hi)) = v_hi;
    }
    // the warp's stores precede lane 0's release (__syncwarp orders them), and
    // a release is cumulative: one release store per peer publishes them all
    __syncwarp();
    if (lane == 0)
        for (int q = 0; q < world; ++q)
            if (q != rank)
                st_release_sys_u32(reinterpret_cast<uint32_t*>(p.fuse.area[q] + ar_fuse_flags_offset()) +
                                           rank * kFuseMaxRb + rb,
                                   e);
    if (lane < world && lane != rank) {
        const uint32_t* f = reinterpret_cast<const uint32_t*>(own + ar_fuse_flags_offset()) + lane * kFuseMaxRb + rb;
        const uint64_t t0 = gemv_clock_ns();
        while ((int32_t)(ld_acquire_sys_u32(f) - e) < 0) {
            if (gemv_clock_ns() - t0 > p.fuse.wait_ns) {
                record_device_error(p.err, kErrGemvPeerWait);
                break;
            }
        }
    }
    __syncwarp();
    float2 s_lo = make_float2(0.f, 0.f), s_hi = make_float2(0.f, 0.f);
    for (int q = 0; q < world; ++q) {
        float2 a, b;
        if (q == rank) {
            a = v_lo;
            b = v_hi;
        } else {
            a = __ldcv(reinterpret_cast<const float2*>(own + ar_fuse_mail_offset(par, q, i_lo)));
            b = __ldcv(reinterpret_cast<const float2*>(own + ar_fuse_mail_offset(par, q, i_hi)));
        }
        s_lo.x += a.x; s_lo.y += a.y;
        s_hi.x += b.x; s_hi.y += b.y;
    }
    __nv_bfloat16* y = static_cast<__nv_bfloat16*>(p.y);
    const __nv_bfloat16* res = static_cast<const __nv_bfloat16*>(p.residual);
    const float v[4] = {s_lo.x, s_lo.y, s_hi.x, s_hi.y};
    const int ms[4] = {2 * t, 2 * t + 1, 2 * t, 2 * t + 1};
    const int64_t ns[4] = {n_lo, n_lo, n_hi, n_hi};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if (ms[i] < p.m) {
            const int64_t off = ms[i] * p.y_stride + ns[i];
            y[off] = __float2bfloat16_rn(Act<__nv_bfloat16>::round(v[i]) + __bfloat162float(res[off]));
        }
    }
    __syncwarp();
    if (lane == 0) epochs[rb] = e;
}

// rm0 / rm1: exact power-of-two multipliers of activation rows 2t and 2t+1
// (undo the staging's overflow guard).
template <int FMT, int EPI>
__device__ __forceinline__ void gemv_epilogue(const GemvParams& p, int64_t rb, int g, int t, float4 s4, float rm0,
                                              float rm1) {
    float acc[4] = {s4.x * rm0, s4.y * rm1, s4.z * rm0, s4.w * rm1};
    __nv_bfloat16* y = static_cast<__nv_bfloat16*>(p.y);
    const int m0 = 2 * t, m1 = 2 * t + 1;
    if constexpr (FMT == AMCU_WFMT_INT8) {
        // per-output-channel scale (device row order): rows rb*16+g and rb*16+g+8
        const float s_lo = static_cast<const float*>(p.scales)[rb * 16 + g];
        const float s_hi = static_cast<const float*>(p.scales)[rb * 16 + g + 8];
        acc[0] *= s_lo;
        acc[1] *= s_lo;
        acc[2] *= s_hi;
        acc[3] *= s_hi;
    }
    if constexpr (EPI == kEpiResidualPeer) {
        gemv_peer_sum_epilogue(p, rb, g, t, acc);
        return;
    }
    if constexpr (EPI == AMCU_EPI_SILU_MUL) {
        // c0/c1: gate row, c2/c3: up row of output column 8*rb + g.
        const int64_t col = rb * 8 + g;
        if (m0 < p.m) {
            float gt = Act<__nv_bfloat16>::round(acc[0]), up = Act<__nv_bfloat16>::round(acc[2]);
            y[m0 * p.y_stride + col] = epi_store<__nv_bfloat16>(silu_ref(gt) * up);
        }
        if (m1 < p.m) {
            float gt = Act<__nv_bfloat16>::round(acc[1]), up = Act<__nv_bfloat16>::round(acc[3]);
            y[m1 * p.y_stride + col] = epi_store<__nv_bfloat16>(silu_ref(gt) * up);
        }
    } else {
        const int64_t n_lo = rb * 16 + g, n_hi = n_lo + 8;
        const float v[4] = {acc[0], acc[1], acc[2], acc[3]};
        const int ms[4] = {m0, m1, m0, m1};
        const int64_t ns[4] = {n_lo, n_lo, n_hi, n_hi};
        const __nv_bfloat16* res = static_cast<const __nv_bfloat16*>(p.residual);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (ms[i] < p.m) {
                const int64_t off = ms[i] * p.y_stride + ns[i];
                float o = Act<__nv_bfloat16>::round(v[i]);
                if constexpr (EPI == AMCU_EPI_RESIDUAL_ADD) o = o + __bfloat162float(res[off]);
                y[off] = epi_store<__nv_bfloat16>(o);
            }
        }
    }
}

// L2 policy of the weight stream: each weight byte is read once per decode
// step, while the KV cache and the activations are read again soon, so the
// weights go first when L2 evicts.
#ifndef AMCU_GEMV_EVICT_FIRST
#define AMCU_GEMV_EVICT_FIRST 1
#endif
__device__ __forceinline__ uint64_t gemv_weight_policy() {
#if AMCU_GEMV_EVICT_FIRST
    return l2_policy_evict_first();
#else
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
    return pol;
#endif
}

constexpr int kXPad = 16;  // bytes of padding per staged activation row
#ifndef GEMV_MINB
#define GEMV_MINB 2
#endif
// CTAs per SM the launcher sizes the rings for.
#ifndef GEMV_CPS
#define GEMV_CPS 2
#endif

// Shared memory carve-up (bytes; every part 128-byte aligned).
struct GemvSmem {
    int red, sx, xs, ring, bars, total;
};
template <int FMT, int NC = kGemvConsumers>
__host__ __device__ inline GemvSmem gemv_smem(int m, int64_t k, int stage_bytes, int stages) {
    auto up = [](int64_t v) { return (int)((v + 127) / 128 * 128); };
    GemvSmem s;
    s.red = 0;
    s.sx = up(2 * NC * 32 * 16);
    s.xs = s.sx + up(FMT == AMCU_WFMT_INT4 ? (k / 128) * 8 * 4 : 0);
    s.ring = s.xs + up(m * (k * 2 + kXPad));
    s.bars = s.ring + stages * stage_bytes;
    s.total = s.bars + up(2 * stages * 8);
    return s;
}

// One 128-column group unit: `rec` is its record in the ring, `grp` its group
// within the row block, xrow_g this lane's activation bytes of group 0 (+256
// per group), sx the per-group activation sums (INT4). M1: one activation row
// (m = 1): output column 2t + 1 of the MMA tile is never stored, so its
// accumulators are not kept.
template <int FMT, bool M1>
__device__ __forceinline__ void gemv_unit(const uint8_t* rec, const uint8_t* xrow_g, const float* sx, int grp,
                                          int lane, int g, int t, float (&acc)[4]) {
    constexpr bool W4 = FMT == AMCU_WFMT_INT4;
    const uint8_t* xp = xrow_g + grp * 256;
    float part[2][4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int e = 0; e < 4; ++e) part[h][e] = 0.f;
        const uint4 x0 = *reinterpret_cast<const uint4*>(xp + h * 128);
        const uint4 x1 = *reinterpret_cast<const uint4*>(xp + h * 128 + 16);
        if constexpr (W4) {
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
        } else {
            const uint4 va = *reinterpret_cast<const uint4*>(rec + h * 1024 + lane * 32);
            const uint4 vb = *reinterpret_cast<const uint4*>(rec + h * 1024 + lane * 32 + 16);
            const uint32_t rg[4] = {va.x, va.y, va.z, va.w};
            const uint32_t rh[4] = {vb.x, vb.y, vb.z, vb.w};
            const uint32_t X[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                uint32_t a[4];
                unpack_w8_word(rg[jj], a[0], a[2]);
                unpack_w8_word(rh[jj], a[1], a[3]);
                mma_bf16_16816(part[h], a, X[2 * jj], X[2 * jj + 1]);
            }
        }
    }
    if constexpr (W4) {
        // part[0] + part[1] hold sum (1032 + q) x (rows g) and
        // sum (1152 + 16q) x (rows g+8) over the group's 128 columns
        const float2 s2x = *reinterpret_cast<const float2*>(sx + grp * 8 + 2 * t);
        const uint32_t sv = *reinterpret_cast<const uint32_t*>(rec + 1024 + 4 * g);
        const __half2 s2 = *reinterpret_cast<const __half2*>(&sv);
        const float s_lo = __low2float(s2), s_hi = __high2float(s2) * 0.0625f;
        acc[0] = fmaf(fmaf(-1032.f, s2x.x, part[0][0] + part[1][0]), s_lo, acc[0]);
        acc[2] = fmaf(fmaf(-1152.f, s2x.x, part[0][2] + part[1][2]), s_hi, acc[2]);
        if constexpr (!M1) {
            acc[1] = fmaf(fmaf(-1032.f, s2x.y, part[0][1] + part[1][1]), s_lo, acc[1]);
            acc[3] = fmaf(fmaf(-1152.f, s2x.y, part[0][3] + part[1][3]), s_hi, acc[3]);
        }
    } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
            if (!M1 || !(e & 1)) acc[e] += part[0][e] + part[1][e];
    }
}

// The `len` units of a stage (groups grp0.. of one row block): warp w takes
// units w, w + NC, ... Stages of 16 or 32 units get a fixed trip count, which
// lets the compiler overlap one unit's loads and unpack with the previous
// unit's MMA chain.
template <int FMT, bool M1, int NC = kGemvConsumers>
__device__ __forceinline__ void gemv_stage(const uint8_t* st, int len, const uint8_t* xrow_g, const float* sx,
                                           int grp0, int warp, int lane, int g, int t, float (&acc)[4]) {
    constexpr int UB = FMT == AMCU_WFMT_INT4 ? kW4PairBytes : 2048;
    if (len == 4 * NC) {
#pragma unroll
        for (int uu = 0; uu < 4; ++uu) {
            const int u = warp + uu * NC;
            gemv_unit<FMT, M1>(st + u * UB, xrow_g, sx, grp0 + u, lane, g, t, acc);
        }
    } else if (len == 2 * NC) {
#pragma unroll
        for (int uu = 0; uu < 2; ++uu) {
            const int u = warp + uu * NC;
            gemv_unit<FMT, M1>(st + u * UB, xrow_g, sx, grp0 + u, lane, g, t, acc);
        }
    } else {
        for (int u = warp; u < len; u += NC)
            gemv_unit<FMT, M1>(st + u * UB, xrow_g, sx, grp0 + u, lane, g, t, acc);
    }
}

}  // namespace amcu
