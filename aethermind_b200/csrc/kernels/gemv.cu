// Weight-only dequant GEMV for decode (m <= 8) and the weight prepacker.
//
// Device weight format ("tile16x64", K-chunked stream): the [N, K] weight is
// cut into tiles of 16 output rows x 64 input columns. The tiles are stored in
// the chunk-major stream order of stream_geom() (gemv.cuh): the K tiles of a
// row block form kc chunks of tw tiles, and chunk w of every row block comes
// before chunk w + 1, so tile (rb, c) sits at stream index
// (c / tw * N/16 + rb) * tw + c % tw; tiles past K are zero. Inside a tile, lane L = 4g + t of a
// warp owns rows {g, g+8} x columns [16t, 16t+16): exactly the A-operand
// fragments of four m16n8k16 tensor-core MMAs in which MMA j contracts
// columns 16t+4j .. 16t+4j+3 of this lane (the MMA's k-slot -> column map is a
// free choice as long as the activation fragment uses the same one). One
// 16-byte (INT4) or 32-byte (INT8) coalesced load per lane per tile feeds the
// MMAs with no shuffles; the activations for the same columns are 32
// contiguous bytes per lane.
//   INT4 word j of lane L: nibble p at bits 4p, value +8 offset-binary is NOT
//        used: nibbles hold two's-complement q. p0,p4,p2,p6 = row g columns
//        +0,+1,+2,+3 and p1,p5,p3,p7 = row g+8 columns +0,+1,+2,+3, so
//        (word >> 4i) & 0x000F000F yields MMA register i directly.
//   INT8: 32 bytes per lane: row g columns [16t, 16t+16) then row g+8.
//   INT4 scales: per tile pair of the stream (one 128-column group) 16 fp16,
//        slot 2g = row g, 2g+1 = row g+8; zero for padding groups.
//   INT8 scales: fp32 [N] (device row order).
// Gate/up fusion: rows 0-7 of every tile are gate rows 8*rb..8*rb+7 and rows
// 8-15 the matching up rows, so one lane holds gate and up of the same output
// and the SiLU-Mul epilogue needs no data exchange.
#include "../amcu_internal.h"
#include "common.cuh"
#include "gemv.cuh"

namespace amcu {

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// INT4 word -> 4 bf16x2 MMA registers holding the exact integers q.
__device__ __forceinline__ void unpack_w4_word(uint32_t w, uint32_t (&a)[4]) {
    // (w >> 4i) & 0x000F000F selects two nibbles; XOR with 0x43084308 maps the
    // two's-complement nibble n to bf16 bits of 128 + (n ^ 8) = 136 + q
    // (exact: integers up to 256 are representable); subtracting 136 gives q.
    const uint32_t bias = 0x43084308u;  // bf16x2 (136, 136)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t v;
        const uint32_t s = w >> (4 * i);
        asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(v) : "r"(s), "r"(0x000F000Fu), "r"(bias));  // (a & b) ^ c
        __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&v);
        const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&bias);
        h = __hsub2(h, b);
        a[i] = *reinterpret_cast<uint32_t*>(&h);
    }
}

// Four int8 values -> two bf16x2 (bytes 0,1) and (bytes 2,3); exact.
__device__ __forceinline__ void unpack_w8_word(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t u = w ^ 0x80808080u;  // offset binary: q + 128
    float f[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t bits = __byte_perm(u, 0x4B000000u, 0x7650u + i);  // 0x4B0000bb = 2^23 + bb
        f[i] = __uint_as_float(bits) - 8388736.0f;                      // - (2^23 + 128)
    }
    __nv_bfloat162 p0 = __floats2bfloat162_rn(f[0], f[1]);
    __nv_bfloat162 p1 = __floats2bfloat162_rn(f[2], f[3]);
    lo = *reinterpret_cast<uint32_t*>(&p0);
    hi = *reinterpret_cast<uint32_t*>(&p1);
}

template <typename T>
__device__ __forceinline__ T epi_store(float v) { return Act<T>::store(v); }

template <int FMT, int EPI>
__device__ __forceinline__ void gemv_epilogue(const GemvParams& p, int64_t rb, int g, int t, float4 s4) {
    float acc[4] = {s4.x, s4.y, s4.z, s4.w};
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

// Streaming GEMV. A CTA has one warp per K chunk of the stream layout and
// owns `rb_per_cta` consecutive row blocks (16 output rows each). Warp w reads
// one contiguous stream -- chunk w of the CTA's row blocks -- with a register
// ring of kTwAlign tiles in flight: one coalesced 16-byte (INT4) or 32-byte
// (INT8) load per lane per tile, issued kTwAlign tiles ahead with plain pointer
// increments, no bounds checks (the stream's tail slack absorbs the last
// read-ahead). The activations (m <= 8 rows, bf16) are staged once per CTA in
// shared memory, zero-padded to the padded K.
//
// INT4 tiles are fed to the MMA as the exact bf16 integers 136 + q (one LOP3
// per register from the packed nibbles); the offset is removed after the MMA
// by subtracting 136 * sum(x) over each 128-column group, sums computed once
// per CTA into shared memory. Products (136 + q) * x are exact in fp32, so the
// correction costs only fp32 rounding.
//
// At the end of a row block the warps' 16 x 8 partial tiles meet in shared
// memory (double-buffered, one barrier) and one warp applies the epilogue.
constexpr int kXPad = 16;  // bytes of padding per staged activation row
#ifndef GEMV_MINB
#define GEMV_MINB 4
#endif
// Row blocks of its stream that a warp keeps requested into L2 ahead of the
// one it is reading (bulk L2 prefetch; 0 turns the prefetch off).
#ifndef GEMV_PW
#define GEMV_PW 2
#endif

// (q + 136) in bf16: (w >> 4i) & 0x000F000F selects two nibbles, XOR with
// 0x43084308 gives bf16 bits of 128 + (n ^ 8) = 136 + q (exact).
__device__ __forceinline__ void unpack_w4_word_biased(uint32_t w, uint32_t (&a)[4]) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
        asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(a[i]) : "r"(w >> (4 * i)), "r"(0x000F000Fu), "r"(0x43084308u));
}

template <int FMT>
__host__ __device__ constexpr int tile_bytes() { return FMT == AMCU_WFMT_INT4 ? 512 : 1024; }

template <int FMT, int EPI>
__global__ void __launch_bounds__(kGemvThreads, GEMV_MINB) gemv_tc_kernel(GemvParams p) {
    constexpr int TB = tile_bytes<FMT>();
    constexpr int NV = TB / 512;  // uint4 per lane per tile
    constexpr int D = kTwAlign;   // ring depth; tw is a multiple of it
    constexpr bool W4 = FMT == AMCU_WFMT_INT4;
    extern __shared__ __align__(16) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int nw = p.kc, tw = p.tw;
    const int kp = nw * tw * 64;  // padded K
    const int gp = kp / 128;      // padded groups (INT4)
    const int M = (int)p.m;
    const int xrow = kp * 2 + kXPad;
    float4* red = reinterpret_cast<float4*>(smem);                      // [2][nw][32]
    float* sx = reinterpret_cast<float*>(smem + 2 * nw * 32 * 16);      // [gp][8] (INT4)
    uint8_t* xs = smem + 2 * nw * 32 * 16 + (W4 ? gp * 8 * 4 : 0);      // [M][kp] bf16 (+pad)

    const int nrb = (int)(p.n / 16);
    const int rb0 = blockIdx.x * p.rb_per_cta;
    const int nr = (rb0 + p.rb_per_cta < nrb ? rb0 + p.rb_per_cta : nrb) - rb0;

    // this warp's stream: chunk `warp` of row blocks rb0 .. rb0 + nr
    const size_t s0 = ((size_t)warp * nrb + rb0) * tw;  // first tile
    const uint8_t* wbase = static_cast<const uint8_t*>(p.w) + s0 * TB;
    const uint8_t* sbase = static_cast<const uint8_t*>(p.scales) + s0 / 2 * 32;  // INT4: 32 B per tile pair
    auto prefetch_row = [&](int r) {
        if (GEMV_PW > 0 && lane == 0 && r < nr) {
            prefetch_l2_bulk(wbase + (size_t)r * tw * TB, (uint32_t)(tw * TB));
            if constexpr (W4) prefetch_l2_bulk(sbase + (size_t)r * tw / 2 * 32, (uint32_t)(tw / 2 * 32));
        }
    };
#pragma unroll
    for (int r = 0; r < GEMV_PW; ++r) prefetch_row(r);

    const uint8_t* wp = wbase + lane * 16 * NV;
    const uint8_t* sp = sbase + 4 * g;
    uint4 wbuf[D][NV];
    uint32_t sbuf[D / 2];
#pragma unroll
    for (int u = 0; u < D; ++u) {
#pragma unroll
        for (int v = 0; v < NV; ++v) wbuf[u][v] = ld_stream_u4(wp + u * TB + 16 * v);
        if (W4 && (u & 1) == 0) sbuf[u / 2] = __ldg(reinterpret_cast<const unsigned int*>(sp + (u / 2) * 32));
    }
    wp += D * TB;
    sp += (D / 2) * 32;

    // Weights do not depend on earlier kernels; the activations do.
    pdl_wait();
    pdl_trigger();

    // ---- stage activations [m][kp] (+16 B per row, zero beyond k) and, for INT4, per-group sums of x
    {
        const int chunks = kp / 8, real = (int)(p.k / 8);
        const __nv_bfloat16* xg = static_cast<const __nv_bfloat16*>(p.x);
        for (int i = threadIdx.x; i < M * chunks; i += blockDim.x) {
            const int m = i / chunks, c = i - m * chunks;
            *reinterpret_cast<uint4*>(xs + m * xrow + c * 16) =
                    c < real ? ld_u4(xg + m * p.x_stride + c * 8) : make_uint4(0, 0, 0, 0);
        }
    }
    __syncthreads();
    if (p.norm_w) {
        // fused RMSNorm of the staged rows: warp w owns rows w, w + nw, ... as
        // y = round(x * (mean(x^2) + eps)^-1/2 * w) (the RMSNorm kernel's formula)
        float* inv_s = reinterpret_cast<float*>(red);  // red is free until the first row-block end
        for (int m = warp; m < M; m += nw) {
            const uint8_t* xr = xs + m * xrow;
            float ss = 0.f;
            for (int c = lane; c < (int)(p.k / 8); c += 32) {
                const uint4 v = *reinterpret_cast<const uint4*>(xr + c * 16);
                const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float a = __uint_as_float(w4[j] << 16), b = __uint_as_float(w4[j] & 0xffff0000u);
                    ss += a * a + b * b;
                }
            }
            ss = warp_sum(ss);
            if (lane == 0) inv_s[m] = 1.0f / sqrtf(ss / (float)p.k + p.eps);
        }
        __syncthreads();
        const int chunks = (int)(p.k / 8);
        const __nv_bfloat16* nwt = static_cast<const __nv_bfloat16*>(p.norm_w);
        for (int i = threadIdx.x; i < M * chunks; i += blockDim.x) {
            const int m = i / chunks, c = i - m * chunks;
            uint4* xp = reinterpret_cast<uint4*>(xs + m * xrow + c * 16);
            const uint4 v = *xp, wv = ld_u4(nwt + c * 8);
            const float inv = inv_s[m];
            const uint32_t a[4] = {v.x, v.y, v.z, v.w}, b[4] = {wv.x, wv.y, wv.z, wv.w};
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float lo = __uint_as_float(a[j] << 16) * inv * __uint_as_float(b[j] << 16);
                const float hi = __uint_as_float(a[j] & 0xffff0000u) * inv * __uint_as_float(b[j] & 0xffff0000u);
                __nv_bfloat162 h2 = __floats2bfloat162_rn(lo, hi);
                o[j] = *reinterpret_cast<uint32_t*>(&h2);
            }
            *xp = make_uint4(o[0], o[1], o[2], o[3]);
        }
        __syncthreads();
    }
    if constexpr (W4) {
        const int segs = gp * 8 * M;  // 16-column segments, 8 per group
        for (int s0i = 0; s0i < segs; s0i += blockDim.x) {
            const int s = s0i + threadIdx.x;
            float sum = 0.f;
            int m = 0, grp = 0;
            if (s < segs) {
                m = s / (gp * 8);
                const int r = s - m * gp * 8;
                grp = r >> 3;
                const uint8_t* xp = xs + m * xrow + (grp * 128 + (r & 7) * 16) * 2;
                const uint4 a = *reinterpret_cast<const uint4*>(xp), b = *reinterpret_cast<const uint4*>(xp + 16);
                const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
                for (int j = 0; j < 8; ++j) sum += __uint_as_float(w[j] << 16) + __uint_as_float(w[j] & 0xffff0000u);
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            if (s < segs && (s & 7) == 0) sx[grp * 8 + m] = sum;
        }
        for (int i = threadIdx.x; i < gp * 8; i += blockDim.x)
            if ((i & 7) >= M) sx[i] = 0.f;  // rows without activations add nothing
        __syncthreads();
    }

    // Lanes whose activation row does not exist (g >= M) read row 0: they only
    // feed MMA output columns g >= M, which the epilogue never stores.
    const uint8_t* xw = xs + (g < M ? g : 0) * xrow + (warp * tw * 64 + 16 * t) * 2;  // + 128 B per tile
    const float* sxw = sx + (warp * tw / 2) * 8 + 2 * t;                               // + 8 floats per group
    int par = 0;
    for (int r = 0; r < nr; ++r, par ^= 1) {
        prefetch_row(r + GEMV_PW);
        const uint8_t* xp = xw;
        const float* sxp = sxw;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int j = 0; j < tw; j += D, xp += D * 128, sxp += (D / 2) * 8, wp += D * TB, sp += (D / 2) * 32) {
#pragma unroll
            for (int u = 0; u < D; u += 2) {
                float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint4 x0 = *reinterpret_cast<const uint4*>(xp + (u + h) * 128);
                    const uint4 x1 = *reinterpret_cast<const uint4*>(xp + (u + h) * 128 + 16);
                    const uint32_t X[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                    if constexpr (W4) {
                        const uint32_t words[4] = {wbuf[u + h][0].x, wbuf[u + h][0].y, wbuf[u + h][0].z,
                                                   wbuf[u + h][0].w};
#pragma unroll
                        for (int jj = 0; jj < 4; ++jj) {
                            uint32_t a[4];
                            unpack_w4_word_biased(words[jj], a);
                            mma_bf16_16816(part, a, X[2 * jj], X[2 * jj + 1]);
                        }
                    } else {
                        const uint32_t rg[4] = {wbuf[u + h][0].x, wbuf[u + h][0].y, wbuf[u + h][0].z,
                                                wbuf[u + h][0].w};
                        const uint32_t rh[4] = {wbuf[u + h][1].x, wbuf[u + h][1].y, wbuf[u + h][1].z,
                                                wbuf[u + h][1].w};
#pragma unroll
                        for (int jj = 0; jj < 4; ++jj) {
                            uint32_t a[4];
                            unpack_w8_word(rg[jj], a[0], a[2]);
                            unpack_w8_word(rh[jj], a[1], a[3]);
                            mma_bf16_16816(acc, a, X[2 * jj], X[2 * jj + 1]);
                        }
                    }
#pragma unroll
                    for (int v = 0; v < NV; ++v) wbuf[u + h][v] = ld_stream_u4(wp + (u + h) * TB + 16 * v);
                }
                if constexpr (W4) {
                    // part holds sum (136 + q) x over the group's 128 columns
                    const float2 s2x = *reinterpret_cast<const float2*>(sxp + (u / 2) * 8);
                    const __half2 s2 = *reinterpret_cast<const __half2*>(&sbuf[u / 2]);
                    const float s_lo = __low2float(s2), s_hi = __high2float(s2);
                    acc[0] = fmaf(fmaf(-136.f, s2x.x, part[0]), s_lo, acc[0]);
                    acc[1] = fmaf(fmaf(-136.f, s2x.y, part[1]), s_lo, acc[1]);
                    acc[2] = fmaf(fmaf(-136.f, s2x.x, part[2]), s_hi, acc[2]);
                    acc[3] = fmaf(fmaf(-136.f, s2x.y, part[3]), s_hi, acc[3]);
                    sbuf[u / 2] = __ldg(reinterpret_cast<const unsigned int*>(sp + (u / 2) * 32));
                }
            }
        }
        // row-block end: publish this warp's partial tile, meet the other
        // warps, and let one warp reduce and apply the epilogue
        red[(par * nw + warp) * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        named_bar_sync(1, nw * 32);
        const int rb = rb0 + r;
        if (warp == rb % nw) {
            float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int w = 0; w < nw; ++w) {
                const float4 v = red[(par * nw + w) * 32 + lane];
                s4.x += v.x; s4.y += v.y; s4.z += v.z; s4.w += v.w;
            }
            gemv_epilogue<FMT, EPI>(p, rb, g, t, s4);
        }
    }
}

template <int FMT>
static size_t gemv_smem_bytes(int64_t m, const StreamGeom& sg) {
    const int64_t kp = (int64_t)sg.kc * sg.tw * 64;
    return 2 * sg.kc * 32 * 16 + (FMT == AMCU_WFMT_INT4 ? (kp / 128) * 8 * 4 : 0) + m * (kp * 2 + kXPad);
}

// Plain fp32 weights (the fp32 tiny model): one thread per output, fp32 FMA.
template <typename T, int EPI>
__global__ void gemm_plain_kernel(GemvParams p) {
    pdl_wait();
    pdl_trigger();
    const int64_t n = blockIdx.x * 32 + (threadIdx.x & 31);
    const int64_t m = blockIdx.y * 8 + (threadIdx.x >> 5);
    const int64_t n_out = EPI == AMCU_EPI_SILU_MUL ? p.n / 2 : p.n;
    if (m >= p.m || n >= n_out) return;
    const T* x = static_cast<const T*>(p.x) + m * p.x_stride;
    const T* w = static_cast<const T*>(p.w);
    auto dot = [&](int64_t row) {
        const T* wr = w + row * p.k;
        float acc = 0.f;
        for (int64_t k = 0; k < p.k; ++k) acc = fmaf(Act<T>::load(x[k]), Act<T>::load(wr[k]), acc);
        return acc;
    };
    T* y = static_cast<T*>(p.y);
    if constexpr (EPI == AMCU_EPI_SILU_MUL) {
        // plain gate/up weight is [gate; up] stacked (2I rows)
        const float gt = Act<T>::round(dot(n)), up = Act<T>::round(dot(n + n_out));
        y[m * p.y_stride + n] = Act<T>::store(silu_ref(gt) * up);
    } else {
        float o = Act<T>::round(dot(n));
        if constexpr (EPI == AMCU_EPI_RESIDUAL_ADD)
            o = o + Act<T>::load(static_cast<const T*>(p.residual)[m * p.y_stride + n]);
        y[m * p.y_stride + n] = Act<T>::store(o);
    }
}

template <int FMT, int EPI>
static void launch_gemv_one(GemvParams p, cudaStream_t s) {
    constexpr int kMaxSmem = 200 * 1024;
    static int per_sm[9] = {};  // resident CTAs per SM by warps per CTA (one device per process on this path)
    const StreamGeom sg = stream_geom(p.k);
    if (per_sm[sg.kc] == 0) {
        cudaFuncSetAttribute(gemv_tc_kernel<FMT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
        int n = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_tc_kernel<FMT, EPI>, 32 * sg.kc,
                                                      gemv_smem_bytes<FMT>(1, sg));
        per_sm[sg.kc] = n > 0 ? n : 1;
    }
    const int64_t max_ctas = (int64_t)per_sm[sg.kc] * num_sms();
    const int64_t nrb = p.n / 16;
    p.kc = sg.kc;
    p.tw = sg.tw;
    p.rb_per_cta = (int)((nrb + max_ctas - 1) / max_ctas);
    const int64_t grid = (nrb + p.rb_per_cta - 1) / p.rb_per_cta;
    // The activation rows are staged in shared memory; when m rows of this K do
    // not fit, the rows go in slices (each slice streams W again).
    int64_t fit = p.m;
    while (fit > 1 && gemv_smem_bytes<FMT>(fit, sg) > (size_t)kMaxSmem) --fit;
    for (int64_t m0 = 0; m0 < p.m; m0 += fit) {
        GemvParams q = p;
        q.m = p.m - m0 < fit ? p.m - m0 : fit;
        q.x = static_cast<const __nv_bfloat16*>(p.x) + m0 * p.x_stride;
        q.y = static_cast<__nv_bfloat16*>(p.y) + m0 * p.y_stride;
        if (p.residual) q.residual = static_cast<const __nv_bfloat16*>(p.residual) + m0 * p.y_stride;
        launch_pdl(gemv_tc_kernel<FMT, EPI>, dim3((unsigned)grid), dim3(32 * sg.kc), gemv_smem_bytes<FMT>(q.m, sg),
                   s, q);
    }
}

template <int FMT>
static void launch_gemv_fmt(const GemvParams& p, int epi, cudaStream_t s) {
    switch (epi) {
        case AMCU_EPI_STORE: launch_gemv_one<FMT, AMCU_EPI_STORE>(p, s); break;
        case AMCU_EPI_RESIDUAL_ADD: launch_gemv_one<FMT, AMCU_EPI_RESIDUAL_ADD>(p, s); break;
        default: launch_gemv_one<FMT, AMCU_EPI_SILU_MUL>(p, s); break;
    }
}

void launch_gemv(const GemvParams& p, int fmt, int epi, cudaStream_t s) {
    if (fmt == AMCU_WFMT_INT4) launch_gemv_fmt<AMCU_WFMT_INT4>(p, epi, s);
    else launch_gemv_fmt<AMCU_WFMT_INT8>(p, epi, s);
}

void launch_gemm_plain(const GemvParams& p, int dtype, int epi, cudaStream_t s) {
    const int64_t n_out = epi == AMCU_EPI_SILU_MUL ? p.n / 2 : p.n;
    const dim3 grid((unsigned)ceil_div(n_out, 32), (unsigned)ceil_div(p.m, 8));
#define AMCU_PL(T, E) launch_pdl(gemm_plain_kernel<T, E>, grid, dim3(256), 0, s, p)
    if (dtype == AMCU_F32) {
        if (epi == AMCU_EPI_STORE) AMCU_PL(float, AMCU_EPI_STORE);
        else if (epi == AMCU_EPI_RESIDUAL_ADD) AMCU_PL(float, AMCU_EPI_RESIDUAL_ADD);
        else AMCU_PL(float, AMCU_EPI_SILU_MUL);
    } else {
        if (epi == AMCU_EPI_STORE) AMCU_PL(__nv_bfloat16, AMCU_EPI_STORE);
        else if (epi == AMCU_EPI_RESIDUAL_ADD) AMCU_PL(__nv_bfloat16, AMCU_EPI_RESIDUAL_ADD);
        else AMCU_PL(__nv_bfloat16, AMCU_EPI_SILU_MUL);
    }
#undef AMCU_PL
}

// ---------------------------------------------------------------------------
// Prepack / unpack between the canonical and the tile16x64 formats.
// ---------------------------------------------------------------------------
// Device row r -> (source, canonical row). With gate/up interleave, tile rows
// 0-7 come from gate rows 8*rb.., rows 8-15 from the matching up rows.
__device__ __forceinline__ int64_t src_row(int64_t r, bool il, int& which) {
    if (!il) { which = 0; return r; }
    const int64_t rb = r >> 4, rr = r & 15;
    which = rr >= 8;
    return rb * 8 + (rr & 7);
}

// Where the packers write: the source rows are row blocks [0, nrb) of a
// canonical matrix; they go to row blocks [rb0, rb0 + nrb) of a stream with
// nrb_total row blocks (a fused weight packs its parts one after another).
struct PackGeom {
    int64_t nrb, nrb_total, rb0;
    int kc, tw;
};
struct TilePos {
    int64_t rb, c;  // source row block and K tile (c >= K/64: padding)
    int64_t dst;    // stream tile index
};
// Tile `ti` of the part, counted chunk-major like the stream itself.
__device__ __forceinline__ TilePos part_tile(int64_t ti, const PackGeom& pg) {
    const int64_t cc = ti % pg.tw, rest = ti / pg.tw;
    const int64_t rb = rest % pg.nrb, w = rest / pg.nrb;
    return TilePos{rb, w * pg.tw + cc, (w * pg.nrb_total + pg.rb0 + rb) * pg.tw + cc};
}

// INT4: one thread per 32-bit device word of the part.
__global__ void pack_w4_kernel(const uint8_t* __restrict__ a, const uint8_t* __restrict__ b, bool il,
                               int64_t K, PackGeom pg, uint32_t* __restrict__ out, bool unpack,
                               uint8_t* __restrict__ canon_out) {
    const int64_t C = K / 64;
    const int64_t words = (int64_t)pg.kc * pg.nrb * pg.tw * 128;
    for (int64_t wi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; wi < words; wi += (int64_t)gridDim.x * blockDim.x) {
        const TilePos tp = part_tile(wi / 128, pg);  // 512 B per tile = 128 words
        const int in_tile = (int)(wi % 128);
        const int lane = in_tile >> 2, j = in_tile & 3;
        const int g = lane >> 2, t = lane & 3;
        const int64_t rb = tp.rb, c = tp.c;
        const int64_t col0 = c * 64 + 16 * t + 4 * j;
        uint32_t* dst = out + tp.dst * 128 + in_tile;
        // nibble p -> (row offset, column offset)
        const int prow[8] = {0, 8, 0, 8, 0, 8, 0, 8};
        const int pcol[8] = {0, 0, 2, 2, 1, 1, 3, 3};
        if (!unpack) {
            uint32_t word = 0;
            if (c < C) {
#pragma unroll
                for (int pp = 0; pp < 8; ++pp) {
                    int which;
                    const int64_t r = src_row(rb * 16 + g + prow[pp], il, which);
                    const uint8_t* src = which ? b : a;
                    const int64_t col = col0 + pcol[pp];
                    const uint8_t byte = src[r * (K / 2) + col / 2];
                    const uint32_t nib = (col & 1) ? (byte >> 4) : (byte & 15u);
                    word |= nib << (4 * pp);
                }
            }
            *dst = word;
        } else if (c < C) {
            const uint32_t word = *dst;
#pragma unroll
            for (int pp = 0; pp < 4; ++pp) {
                // nibbles pp and pp+4 hold columns col (even) and col+1 of one row
                const int64_t r = rb * 16 + g + prow[pp];
                const int64_t col = col0 + pcol[pp];
                const uint32_t lo = (word >> (4 * pp)) & 15u, hi = (word >> (4 * (pp + 4))) & 15u;
                canon_out[r * (K / 2) + col / 2] = (uint8_t)(lo | (hi << 4));
            }
        }
    }
}

// INT4 scales: canonical fp16 [N][G] -> per stream tile pair 16 halves, slot
// 2g = row g, 2g+1 = row g+8 (zero for padding groups).
__global__ void pack_s4_kernel(const __half* __restrict__ a, const __half* __restrict__ b, bool il, int64_t G,
                               PackGeom pg, __half* __restrict__ out, bool unpack) {
    const int64_t pairs = (int64_t)pg.kc * pg.nrb * (pg.tw / 2);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < pairs * 16;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int slot = (int)(i % 16);
        const TilePos tp = part_tile(i / 16 * 2, pg);  // first tile of the pair
        const int64_t grp = tp.c / 2;
        const int64_t r_dev = tp.rb * 16 + (slot >> 1) + ((slot & 1) ? 8 : 0);
        __half* dst = out + tp.dst / 2 * 16 + slot;
        if (!unpack) {
            if (grp < G) {
                int which;
                const int64_t r = src_row(r_dev, il, which);
                *dst = (which ? b : a)[r * G + grp];
            } else {
                *dst = __float2half(0.f);
            }
        } else if (grp < G) {
            const_cast<__half*>(a)[r_dev * G + grp] = *dst;
        }
    }
}

// INT8: one thread per 16-byte half-lane chunk of the part.
__global__ void pack_w8_kernel(const int8_t* __restrict__ a, const int8_t* __restrict__ b, bool il, int64_t K,
                               PackGeom pg, uint4* __restrict__ out, bool unpack) {
    const int64_t C = K / 64;
    const int64_t chunks = (int64_t)pg.kc * pg.nrb * pg.tw * 64;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < chunks; i += (int64_t)gridDim.x * blockDim.x) {
        const TilePos tp = part_tile(i / 64, pg);  // 1024 B per tile
        const int in_tile = (int)(i % 64);
        const int lane = in_tile >> 1, half = in_tile & 1;
        const int g = lane >> 2, t = lane & 3;
        const int64_t r_dev = tp.rb * 16 + g + (half ? 8 : 0);
        const int64_t col = tp.c * 64 + 16 * t;
        uint4* dst = out + tp.dst * 64 + in_tile;
        if (!unpack) {
            if (tp.c < C) {
                int which;
                const int64_t r = src_row(r_dev, il, which);
                *dst = *reinterpret_cast<const uint4*>((which ? b : a) + r * K + col);
            } else {
                *dst = make_uint4(0, 0, 0, 0);
            }
        } else if (tp.c < C) {
            *reinterpret_cast<uint4*>(const_cast<int8_t*>(a) + r_dev * K + col) = *dst;
        }
    }
}

__global__ void pack_s8_kernel(const float* __restrict__ a, const float* __restrict__ b, bool il, int64_t N,
                               float* __restrict__ out) {
    for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < N; r += (int64_t)gridDim.x * blockDim.x) {
        int which;
        const int64_t s = src_row(r, il, which);
        out[r] = (which ? b : a)[s];
    }
}

__global__ void copy_bytes_kernel(const uint8_t* __restrict__ a, const uint8_t* __restrict__ b, int64_t half_bytes,
                                  uint8_t* __restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < 2 * half_bytes; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = i < half_bytes ? a[i] : b[i - half_bytes];
}

}  // namespace amcu

using namespace amcu;

namespace {
int pack_grid(int64_t n) {
    int64_t b = (n + 255) / 256;
    if (b > 148 * 32) b = 148 * 32;
    return (int)(b < 1 ? 1 : b);
}
int plain_elt(int32_t dtype) { return dtype == AMCU_F32 ? 4 : 2; }

am_status_code check_weight_shape(int32_t format, int32_t dtype, int64_t n, int64_t k, int64_t group) {
    AMCU_REQUIRE(n > 0 && k > 0, "weight: n and k must be positive");
    if (format == AMCU_WFMT_PLAIN) {
        AMCU_REQUIRE(dtype == AMCU_F32 || dtype == AMCU_BF16, "plain weight dtype must be f32 or bf16");
        return AM_STATUS_OK;
    }
    AMCU_REQUIRE(format == AMCU_WFMT_INT8 || format == AMCU_WFMT_INT4, "unknown weight format %d", format);
    AMCU_REQUIRE(n % 16 == 0, "quantized weight: n (%lld) must be a multiple of 16", (long long)n);
    AMCU_REQUIRE(k % 64 == 0, "quantized weight: k (%lld) must be a multiple of 64", (long long)k);
    if (format == AMCU_WFMT_INT4) {
        AMCU_REQUIRE(group == 128, "int4 weight: only group size 128 is supported");
        AMCU_REQUIRE(k % 128 == 0, "int4 weight: k must be a multiple of 128");
    }
    return AM_STATUS_OK;
}

// Packs the canonical [n, k] part (qa/sa; with `il` the gate half, and qb/sb
// the up half) into rows [row0, row0 + n) of a packed [n_total, k] weight.
am_status_code prepack_impl(int32_t format, int32_t dtype, int64_t n, int64_t k, int64_t group, int64_t n_total,
                            int64_t row0, const void* qa, const void* sa, const void* qb, const void* sb, bool il,
                            void* qp, void* sp, cudaStream_t s) {
    (void)group;
    if (format == AMCU_WFMT_PLAIN) {
        uint8_t* dst = static_cast<uint8_t*>(qp) + row0 * k * plain_elt(dtype);
        if (!il) {
            cudaMemcpyAsync(dst, qa, (size_t)n * k * plain_elt(dtype), cudaMemcpyDeviceToDevice, s);
        } else {
            const int64_t hb = n / 2 * k * plain_elt(dtype);
            copy_bytes_kernel<<<pack_grid(2 * hb), 256, 0, s>>>((const uint8_t*)qa, (const uint8_t*)qb, hb, dst);
        }
        return check_launch("amcu_prepack_weight");
    }
    const StreamGeom sg = stream_geom(k);
    const PackGeom pg{n / 16, n_total / 16, row0 / 16, sg.kc, sg.tw};
    const int64_t stream_tiles = (int64_t)sg.kc * (n_total / 16) * sg.tw;
    const int64_t part_tiles = (int64_t)sg.kc * (n / 16) * sg.tw;
    if (format == AMCU_WFMT_INT4) {
        pack_w4_kernel<<<pack_grid(part_tiles * 128), 256, 0, s>>>((const uint8_t*)qa, (const uint8_t*)qb, il, k, pg,
                                                                   (uint32_t*)qp, false, nullptr);
        cudaMemsetAsync(static_cast<uint8_t*>(qp) + stream_tiles * 512, 0, kStreamPadBytes, s);
        pack_s4_kernel<<<pack_grid(part_tiles / 2 * 16), 256, 0, s>>>((const __half*)sa, (const __half*)sb, il,
                                                                      k / 128, pg, (__half*)sp, false);
        cudaMemsetAsync(static_cast<uint8_t*>(sp) + stream_tiles / 2 * 32, 0, kScalePadBytes, s);
    } else {
        pack_w8_kernel<<<pack_grid(part_tiles * 64), 256, 0, s>>>((const int8_t*)qa, (const int8_t*)qb, il, k, pg,
                                                                  (uint4*)qp, false);
        cudaMemsetAsync(static_cast<uint8_t*>(qp) + stream_tiles * 1024, 0, kStreamPadBytes, s);
        pack_s8_kernel<<<pack_grid(n), 256, 0, s>>>((const float*)sa, (const float*)sb, il, n,
                                                    static_cast<float*>(sp) + row0);
    }
    return check_launch("amcu_prepack_weight");
}
}  // namespace

extern "C" {

int64_t amcu_packed_weight_bytes(int32_t format, int32_t dtype, int64_t n, int64_t k, int64_t group) {
    (void)group;
    if (format == AMCU_WFMT_PLAIN) return n * k * plain_elt(dtype);
    const StreamGeom sg = stream_geom(k);
    const int64_t tiles = (int64_t)sg.kc * (n / 16) * sg.tw;
    return tiles * (format == AMCU_WFMT_INT8 ? 1024 : 512) + kStreamPadBytes;
}

int64_t amcu_packed_scale_bytes(int32_t format, int64_t n, int64_t k, int64_t group) {
    (void)group;
    if (format == AMCU_WFMT_INT8) return n * 4;
    if (format == AMCU_WFMT_INT4) {
        const StreamGeom sg = stream_geom(k);
        return (int64_t)sg.kc * (n / 16) * (sg.tw / 2) * 32 + kScalePadBytes;
    }
    return 0;
}

am_status_code amcu_prepack_weight(int32_t format, int32_t dtype, int64_t n, int64_t k, int64_t group,
                                   const void* q, const void* sc, void* qp, void* sp, void* stream) {
    clear_error();
    am_status_code st = check_weight_shape(format, dtype, n, k, group);
    if (st != AM_STATUS_OK) return st;
    AMCU_REQUIRE(q && qp, "amcu_prepack_weight: null pointer");
    AMCU_REQUIRE(format == AMCU_WFMT_PLAIN || (sc && sp), "amcu_prepack_weight: null scale pointer");
    AMCU_REQUIRE(aligned(qp, 16) && aligned(q, 16), "amcu_prepack_weight: weights must be 16-byte aligned");
    return prepack_impl(format, dtype, n, k, group, n, 0, q, sc, q, sc, false, qp, sp, as_stream(stream));
}

am_status_code amcu_prepack_weight_rows(int32_t format, int32_t dtype, int64_t n, int64_t k, int64_t group,
                                        int64_t n_total, int64_t row0, const void* q, const void* sc, void* qp,
                                        void* sp, void* stream) {
    clear_error();
    am_status_code st = check_weight_shape(format, dtype, n_total, k, group);
    if (st != AM_STATUS_OK) return st;
    st = check_weight_shape(format, dtype, n, k, group);
    if (st != AM_STATUS_OK) return st;
    AMCU_REQUIRE(row0 >= 0 && row0 % 16 == 0 && row0 + n <= n_total,
                 "amcu_prepack_weight_rows: rows [%lld, %lld) must lie in [0, %lld) and start on a 16-row boundary",
                 (long long)row0, (long long)(row0 + n), (long long)n_total);
    AMCU_REQUIRE(q && qp, "amcu_prepack_weight_rows: null pointer");
    AMCU_REQUIRE(format == AMCU_WFMT_PLAIN || (sc && sp), "amcu_prepack_weight_rows: null scale pointer");
    AMCU_REQUIRE(aligned(qp, 16) && aligned(q, 16), "amcu_prepack_weight_rows: weights must be 16-byte aligned");
    return prepack_impl(format, dtype, n, k, group, n_total, row0, q, sc, q, sc, false, qp, sp, as_stream(stream));
}

am_status_code amcu_prepack_gate_up(int32_t format, int32_t dtype, int64_t inter, int64_t k, int64_t group,
                                    const void* gq, const void* gs, const void* uq, const void* us, void* qp,
                                    void* sp, void* stream) {
    clear_error();
    AMCU_REQUIRE(inter > 0 && inter % 8 == 0, "amcu_prepack_gate_up: inter must be a positive multiple of 8");
    am_status_code st = check_weight_shape(format, dtype, 2 * inter, k, group);
    if (st != AM_STATUS_OK) return st;
    AMCU_REQUIRE(gq && uq && qp, "amcu_prepack_gate_up: null pointer");
    AMCU_REQUIRE(format == AMCU_WFMT_PLAIN || (gs && us && sp), "amcu_prepack_gate_up: null scale pointer");
    AMCU_REQUIRE(aligned(qp, 16) && aligned(gq, 16) && aligned(uq, 16), "amcu_prepack_gate_up: misaligned");
    return prepack_impl(format, dtype, 2 * inter, k, group, 2 * inter, 0, gq, gs, uq, us, true, qp, sp,
                        as_stream(stream));
}

am_status_code amcu_unpack_weight(int32_t format, int32_t dtype, int64_t n, int64_t k, int64_t group,
                                  const void* qp, const void* sp, void* q, void* sc, void* stream) {
    clear_error();
    am_status_code st = check_weight_shape(format, dtype, n, k, group);
    if (st != AM_STATUS_OK) return st;
    AMCU_REQUIRE(q && qp, "amcu_unpack_weight: null pointer");
    cudaStream_t s = as_stream(stream);
    if (format == AMCU_WFMT_PLAIN) {
        cudaMemcpyAsync(q, qp, (size_t)n * k * plain_elt(dtype), cudaMemcpyDeviceToDevice, s);
        return check_launch("amcu_unpack_weight");
    }
    const StreamGeom sg = stream_geom(k);
    const PackGeom pg{n / 16, n / 16, 0, sg.kc, sg.tw};
    const int64_t tiles = (int64_t)sg.kc * (n / 16) * sg.tw;
    if (format == AMCU_WFMT_INT4) {
        pack_w4_kernel<<<pack_grid(tiles * 128), 256, 0, s>>>(nullptr, nullptr, false, k, pg,
                                                              (uint32_t*)const_cast<void*>(qp), true, (uint8_t*)q);
        if (sc && sp)
            pack_s4_kernel<<<pack_grid(tiles / 2 * 16), 256, 0, s>>>((const __half*)sc, nullptr, false, k / 128, pg,
                                                                     (__half*)const_cast<void*>(sp), true);
    } else {
        pack_w8_kernel<<<pack_grid(tiles * 64), 256, 0, s>>>((const int8_t*)q, nullptr, false, k, pg,
                                                             (uint4*)const_cast<void*>(qp), true);
        if (sc && sp) cudaMemcpyAsync(sc, sp, (size_t)n * 4, cudaMemcpyDeviceToDevice, s);
    }
    return check_launch("amcu_unpack_weight");
}

}  // extern "C"
