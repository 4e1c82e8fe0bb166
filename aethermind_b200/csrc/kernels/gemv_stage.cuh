// Activation staging shared by the GEMV kernels: the m <= 8 activation rows
// go to shared memory once per CTA, with the fused RMSNorm, and for INT4 as
// fp16 with per-128-column-group sums (and a power-of-two overflow guard).
#pragma once
#include "common.cuh"

namespace amcu {

struct StageShared {                    // small per-CTA state (shared memory)
    float row_mul[8];                   // epilogue multiplier per activation row (a power of two)
    float row_inv[8];                   // RMSNorm factor per row
    unsigned int row_amax[8];
    unsigned int row_big;               // bit m: row m needs a multiplier above 1 (fp16 overflow guard)
};

struct StageCtx {
    const __nv_bfloat16* x;  // [m][k] rows, stride x_stride
    int64_t x_stride;
    int64_t k;
    int m;
    const __nv_bfloat16* norm_w;  // optional fused RMSNorm weight [k]
    float eps;
    uint8_t* xs;   // [m][k] (+16 B per row) staging
    int xrow;      // bytes per staged row
    float* sx;     // [k / 128][8] group sums (INT4)
    StageShared* sh;
    int tid, nthreads, bar_id;  // the staging threads (a multiple of 32) and their named barrier
};

// Stages the activation rows: copy, RMSNorm factors (fused norm), then for
// INT4 one pass that normalizes, converts to fp16 and sums every 128-column
// group; INT8 keeps bf16. Ends with the staging threads synchronized. CG:
// read the activations around L1 (a persistent kernel reads buffers other
// SMs rewrote since its last read).
template <bool W4, bool CG = false>
__device__ __forceinline__ void stage_activations(const StageCtx& ctx) {
    auto ldx = [](const __nv_bfloat16* ptr) {
        if constexpr (CG) return __ldcg(reinterpret_cast<const uint4*>(ptr));
        else return ld_u4(ptr);
    };
    const int tid = ctx.tid, NT = ctx.nthreads, warp = tid >> 5, lane = tid & 31, nw = NT / 32;
    const int M = ctx.m, xrow = ctx.xrow, G = (int)(ctx.k / 128);
    uint8_t* xs = ctx.xs;
    float* sx = ctx.sx;
    float* row_mul = ctx.sh->row_mul;
    float* row_inv = ctx.sh->row_inv;
    unsigned int& row_big = ctx.sh->row_big;
    const int chunks = (int)(ctx.k / 8);  // 16-byte chunks per row
    const __nv_bfloat16* xg = ctx.x;
    const __nv_bfloat16* nwt = ctx.norm_w;
    if (tid < kGemvMaxM) row_mul[tid] = 1.f;
    if (tid == 0) row_big = 0u;
    for (int i = tid; i < M * chunks; i += NT) {
        const int m = i / chunks, c = i - m * chunks;
        *reinterpret_cast<uint4*>(xs + m * xrow + c * 16) = ldx(xg + m * ctx.x_stride + c * 8);
    }
    named_bar_sync(ctx.bar_id, NT);
    if (ctx.norm_w) {
        // row m's factor (mean(x^2) + eps)^-1/2, reduced by warp m % 8 in a
        // fixed order; y = round(x * factor * w) as the RMSNorm kernel computes it
        for (int m = warp; m < M; m += nw) {
            const uint8_t* xr = xs + m * xrow;
            float ss = 0.f;
            for (int c = lane; c < chunks; c += 32) {
                const uint4 v = *reinterpret_cast<const uint4*>(xr + c * 16);
                const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float a = __uint_as_float(w4[j] << 16), b = __uint_as_float(w4[j] & 0xffff0000u);
                    ss += a * a + b * b;
                }
            }
            ss = warp_sum(ss);
            if (lane == 0) row_inv[m] = 1.0f / sqrtf(ss / (float)ctx.k + ctx.eps);
        }
        named_bar_sync(ctx.bar_id, NT);
    }
    // normalized bf16 value of element pair j of a 16-byte chunk (a: x bits, w: norm weight bits)
    auto norm2 = [&](uint32_t a, uint32_t w, float inv, float& lo, float& hi) {
        lo = __uint_as_float(a << 16);
        hi = __uint_as_float(a & 0xffff0000u);
        if (ctx.norm_w) {
            lo = Act<__nv_bfloat16>::round(lo * inv * __uint_as_float(w << 16));
            hi = Act<__nv_bfloat16>::round(hi * inv * __uint_as_float(w & 0xffff0000u));
        }
    };
    if constexpr (W4) {
        // one thread per 16-column segment (8 per group): normalize, convert
        // to fp16 (times 1/row_mul), sum; the group sum is a shuffle over the
        // segment's 8 lanes
        auto convert_pass = [&](bool redo) {
            const int segs = G * 8 * M;
            for (int s0 = 0; s0 < segs; s0 += NT) {
                const int s = s0 + tid;
                float sum = 0.f;
                int m = 0, grp = 0;
                bool active = s < segs;
                if (active) {
                    m = s / (G * 8);
                    const int r = s - m * G * 8;
                    grp = r >> 3;
                    active = !redo || ((row_big >> m) & 1u);
                    if (active) {
                        const int c0 = grp * 16 + (r & 7) * 2;  // first 16-byte chunk of the segment
                        uint4* xp = reinterpret_cast<uint4*>(xs + m * xrow + c0 * 16);
                        uint4 v[2], wv[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
                        if (redo) {
                            v[0] = ldx(xg + m * ctx.x_stride + c0 * 8);
                            v[1] = ldx(xg + m * ctx.x_stride + c0 * 8 + 8);
                        } else {
                            v[0] = xp[0];
                            v[1] = xp[1];
                        }
                        if (ctx.norm_w) {
                            wv[0] = ld_u4(nwt + c0 * 8);
                            wv[1] = ld_u4(nwt + c0 * 8 + 8);
                        }
                        const float inv = ctx.norm_w ? row_inv[m] : 1.f, mul = 1.0f / row_mul[m];
                        const uint32_t a[8] = {v[0].x, v[0].y, v[0].z, v[0].w, v[1].x, v[1].y, v[1].z, v[1].w};
                        const uint32_t w[8] = {wv[0].x, wv[0].y, wv[0].z, wv[0].w, wv[1].x, wv[1].y, wv[1].z, wv[1].w};
                        uint32_t h[8];
                        float amax = 0.f;
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            float lo, hi;
                            norm2(a[j], w[j], inv, lo, hi);
                            amax = fmaxf(amax, fmaxf(fabsf(lo), fabsf(hi)));
                            const __half2 hv = __floats2half2_rn(lo * mul, hi * mul);
                            sum += __low2float(hv) + __high2float(hv);
                            h[j] = *reinterpret_cast<const uint32_t*>(&hv);
                        }
                        if (!redo && amax > 32768.f) atomicOr(&row_big, 1u << m);
                        xp[0] = make_uint4(h[0], h[1], h[2], h[3]);
                        xp[1] = make_uint4(h[4], h[5], h[6], h[7]);
                    }
                }
                sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                sum += __shfl_xor_sync(0xffffffffu, sum, 4);
                if (active && (s & 7) == 0) sx[grp * 8 + m] = sum;
            }
        };
        convert_pass(false);
        for (int i = tid; i < G * 8; i += NT)
            if ((i & 7) >= M) sx[i] = 0.f;  // rows without activations add nothing
        named_bar_sync(ctx.bar_id, NT);
        if (row_big != 0u) {
            // Rare: a row reaches 2^15, beyond what fp16 staging keeps. Find
            // its max, stage it again times 2^-e (exact) and let the epilogue
            // multiply by 2^e.
            unsigned int* row_amax = ctx.sh->row_amax;
            if (tid < kGemvMaxM) row_amax[tid] = 0u;
            named_bar_sync(ctx.bar_id, NT);
            for (int i = tid; i < M * chunks; i += NT) {
                const int m = i / chunks, c = i - m * chunks;
                if (!((row_big >> m) & 1u)) continue;
                const uint4 v = ldx(xg + m * ctx.x_stride + c * 8);
                const uint4 wv = ctx.norm_w ? ld_u4(nwt + c * 8) : make_uint4(0, 0, 0, 0);
                const uint32_t a[4] = {v.x, v.y, v.z, v.w}, w[4] = {wv.x, wv.y, wv.z, wv.w};
                float amax = 0.f;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float lo, hi;
                    norm2(a[j], w[j], ctx.norm_w ? row_inv[m] : 1.f, lo, hi);
                    amax = fmaxf(amax, fmaxf(fabsf(lo), fabsf(hi)));
                }
                atomicMax(&row_amax[m], __float_as_uint(amax));
            }
            named_bar_sync(ctx.bar_id, NT);
            if (tid < M && ((row_big >> tid) & 1u)) {
                // e = exponent(max) - 14 keeps the scaled max below 2^15
                const int e = (int)((row_amax[tid] >> 23) & 0xff) - 127 - 14;
                row_mul[tid] = __int_as_float((127 + (e > 0 ? e : 0)) << 23);
            }
            named_bar_sync(ctx.bar_id, NT);
            convert_pass(true);
            named_bar_sync(ctx.bar_id, NT);
        }
    } else if (ctx.norm_w) {
        for (int i = tid; i < M * chunks; i += NT) {
            const int m = i / chunks, c = i - m * chunks;
            uint4* xp = reinterpret_cast<uint4*>(xs + m * xrow + c * 16);
            const uint4 v = *xp, wv = ld_u4(nwt + c * 8);
            const uint32_t a[4] = {v.x, v.y, v.z, v.w}, w[4] = {wv.x, wv.y, wv.z, wv.w};
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float lo, hi;
                norm2(a[j], w[j], row_inv[m], lo, hi);
                __nv_bfloat162 h2 = __floats2bfloat162_rn(lo, hi);
                o[j] = *reinterpret_cast<uint32_t*>(&h2);
            }
            *xp = make_uint4(o[0], o[1], o[2], o[3]);
        }
        named_bar_sync(ctx.bar_id, NT);
    }
}

}  // namespace amcu
