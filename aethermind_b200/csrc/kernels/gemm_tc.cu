// Prefill dequant GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// y[m, n] = sum_k x[m, k] * w[n, k] for m > 8 rows (prefill), x bf16 and w
// the quantized device format of gemv.cu (INT4 pair records with inline group
// scales, or INT8 tiles with per-row scales).
//
// A CTA computes a 128 x 128 output tile, K in blocks of 128 (one INT4 scale
// group), through a ring of kStages shared-memory stages. Warp roles:
//   warps 0-7  dequantize: warp w turns the 16-row block w of the tile's
//              weights into bf16 (INT4: q * group scale, rounded once; INT8:
//              q exactly) written straight into the 128-byte-swizzled K-major
//              layout the MMA reads; afterwards the same warps are the
//              epilogue (TMEM -> registers -> bf16 outputs).
//   warp 8     TMA producer: the x tile, 128 rows x 128 columns, as two
//              128-byte-swizzled boxes per stage.
//   warp 9     MMA issuer: one elected thread issues tcgen05.mma
//              (kind::f16, bf16 x bf16 -> fp32, M = N = 128, K = 16) into a
//              128-column TMEM accumulator and commits each stage back to
//              the producers through an mbarrier; warp 9 also owns the TMEM
//              allocation.
// Every wait on an mbarrier is bounded: a wait that runs out records an
// error code in the device error word and the CTA finishes its control flow
// without waiting again (results are then garbage, and the host sees the
// code), so a fault of the pipeline cannot hang the GPU.
#include <cuda.h>

#include <cstdio>
#include <cstdlib>
#include <vector>

#include "../amcu_internal.h"
#include "common.cuh"
#include "gemm_tc.cuh"
#include "gemv.cuh"

namespace amcu {

constexpr int kTcBM = 128, kTcBN = 128, kTcBK = 128;
constexpr int kTcStages = 3;
constexpr int kTcDequantWarps = 8;
constexpr int kTcThreads = (kTcDequantWarps + 2) * 32;
constexpr int kTcTileBytes = kTcBM * kTcBK * 2;  // 32 KB per operand per stage (bf16)
constexpr int kTcWStage = kTcDequantWarps * kW4PairBytes;  // INT4 pair records of one stage (8 row blocks)
constexpr int kTcSmemBytes = 1024 + 2 * kTcStages * kTcTileBytes + (kTcStages + 2) * kTcBN * 4 + kTcStages * kTcWStage + 256;
constexpr int32_t kErrGemmTcWait = 0x201;

struct GemmTcKParams {
    const uint8_t* w;
    const float* scales;  // INT8 per-row scales
    __nv_bfloat16* y;
    const __nv_bfloat16* residual;
    int64_t m, n, k;
    int64_t y_stride;
    int32_t* err;
    unsigned long long* trace;  // diagnostics (AMCU_GEMM_TRACE): per CTA [16] cycle counters, or null
    int dbg;  // diagnostics (AMCU_GEMM_DBG, wrong results): bit 0 skips the dequant math, bit 1 the promotion, bit 2 the stores, bit 3 the epilogue's staging,
              // bit 4 the activation loads, bit 5 the record loads (swapped kernel)
};

// Diagnostics (AMCU_DIAG builds only; the default build compiles them out):
// ablation bits that skip parts of the work (wrong results, for timing
// studies) and per-CTA timers.
#ifdef AMCU_DIAG
#define TC_DBG(p) ((p).dbg)
#define TC_TRACE(p) ((p).trace)
#else
#define TC_DBG(p) 0
#define TC_TRACE(p) ((unsigned long long*)nullptr)
#endif

// Diagnostics: a globaltimer stamp into slot `slot` of this CTA's counters.
__device__ __forceinline__ void tc_stamp(const GemmTcKParams& p, int slot) {
    if (!TC_TRACE(p)) return;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    p.trace[((size_t)blockIdx.y * gridDim.x + blockIdx.x) * 16 + slot] = t;
}

// Diagnostics: cycles spent in a wait or a phase, summed per CTA and role.
struct TcClock {
    long long t0 = 0;
    __device__ __forceinline__ void start(const GemmTcKParams& p) {
        if (TC_TRACE(p)) t0 = clock64();
    }
    __device__ __forceinline__ void stop(const GemmTcKParams& p, int slot) {
        if (TC_TRACE(p)) atomicAdd(TC_TRACE(p) + ((size_t)blockIdx.y * gridDim.x + blockIdx.x) * 16 + slot,
                               (unsigned long long)(clock64() - t0));
    }
};

// ---- tcgen05 / TMA helpers (inline PTX) ----
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major operand in the 128-byte
// swizzle layout: rows of 128 bytes, 8-row atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t tc_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);  // start address
    d |= (uint64_t)1 << 16;                    // leading byte offset (unused when swizzled)
    d |= (uint64_t)(1024 >> 4) << 32;          // stride byte offset: next 8-row atom
    d |= (uint64_t)1 << 46;                    // descriptor version
    d |= (uint64_t)2 << 61;                    // 128-byte swizzle
    return d;
}

// Instruction descriptor: kind::f16, D fp32, A and B bf16, both K-major, M x N.
__host__ __device__ constexpr uint32_t tc_idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
            " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
            : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
                    smem_u32(dst)),
            "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
            : "memory");
}
// 32 lanes x 32 consecutive columns of 32-bit TMEM cells -> 32 registers per thread.
__device__ __forceinline__ void tc_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
              "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
              "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
              "=r"(r[30]), "=r"(r[31])
            : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Byte offset of 16-byte chunk c (0..15 over the 128 K columns) of row r in
// a 128 x 128 bf16 operand tile: two 64-column halves of 16 KB, each rows of
// 128 bytes with the 16-byte chunks XOR-swizzled by row % 8.
__device__ __forceinline__ uint32_t sw128_offset(int r, int c) {
    return (uint32_t)((c >> 3) * 16384 + (r >> 3) * 1024 + (r & 7) * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// Eight bf16 of (q * s) from eight two's-complement nibbles given in order.
__device__ __forceinline__ uint4 dequant8_w4(const uint32_t (&nib)[8], float s) {
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float a = (__uint_as_float(0x4B000000u | (nib[2 * i] ^ 8u)) - 8388616.0f) * s;
        const float b = (__uint_as_float(0x4B000000u | (nib[2 * i + 1] ^ 8u)) - 8388616.0f) * s;
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        o[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}
// Eight bf16 holding eight int8 exactly.
__device__ __forceinline__ uint4 dequant8_w8(uint2 v) {
    const uint32_t w[2] = {v.x, v.y};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint32_t u = w[i] ^ 0x80808080u;
        float f[4];
#pragma unroll
        for (int b = 0; b < 4; ++b)
            f[b] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650u + b)) - 8388736.0f;
        __nv_bfloat162 p0 = __floats2bfloat162_rn(f[0], f[1]), p1 = __floats2bfloat162_rn(f[2], f[3]);
        o[2 * i] = *reinterpret_cast<uint32_t*>(&p0);
        o[2 * i + 1] = *reinterpret_cast<uint32_t*>(&p1);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// Warp `wb`'s 16 rows x 128 columns of the weight tile for K block kb, in
// bf16, into the swizzled stage B. Rows beyond n are zero.
template <int FMT>
__device__ __forceinline__ void dequant_rows(const GemmTcKParams& p, int64_t rb, int kb, int wb, int lane,
                                             uint8_t* B) {
    const int g = lane >> 2, t = lane & 3;
    const int r0 = wb * 16 + g, r1 = r0 + 8;  // rows of the tile this lane fills
    if (rb * 16 >= p.n) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            *reinterpret_cast<uint4*>(B + sw128_offset(r0, 4 * t + c)) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(B + sw128_offset(r1, 4 * t + c)) = make_uint4(0, 0, 0, 0);
        }
        return;
    }
    if constexpr (FMT == AMCU_WFMT_INT4) {
        const int64_t G = p.k / 128;
        const uint8_t* rec = p.w + ((size_t)rb * G + kb) * kW4PairBytes;
        const uint32_t sv = __ldg(reinterpret_cast<const unsigned int*>(rec + 1024 + 4 * g));
        const __half2 s2 = *reinterpret_cast<const __half2*>(&sv);
        const float s_lo = __low2float(s2), s_hi = __high2float(s2);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint4 wv = __ldg(reinterpret_cast<const uint4*>(rec + h * 512 + lane * 16));
            const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
            // word j: columns 16t+4j .. +3; nibbles p0,p4,p2,p6 row g and p1,p5,p3,p7 row g+8
            uint32_t lo[16], hi[16];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                // nibble p at bits 4p: row g columns +0..+3 are p0, p4, p2, p6; row g+8 p1, p5, p3, p7
                lo[4 * j + 0] = (w[j] >> 0) & 15u;
                lo[4 * j + 1] = (w[j] >> 16) & 15u;
                lo[4 * j + 2] = (w[j] >> 8) & 15u;
                lo[4 * j + 3] = (w[j] >> 24) & 15u;
                hi[4 * j + 0] = (w[j] >> 4) & 15u;
                hi[4 * j + 1] = (w[j] >> 20) & 15u;
                hi[4 * j + 2] = (w[j] >> 12) & 15u;
                hi[4 * j + 3] = (w[j] >> 28) & 15u;
            }
            // columns h*64 + 16t + [0, 8) and [8, 16): chunks 8h + 2t and 8h + 2t + 1
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t a[8], b[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    a[e] = lo[8 * c + e];
                    b[e] = hi[8 * c + e];
                }
                *reinterpret_cast<uint4*>(B + sw128_offset(r0, 8 * h + 2 * t + c)) = dequant8_w4(a, s_lo);
                *reinterpret_cast<uint4*>(B + sw128_offset(r1, 8 * h + 2 * t + c)) = dequant8_w4(b, s_hi);
            }
        }
    } else {
        const int64_t C = p.k / 64;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint8_t* tile = p.w + ((size_t)rb * C + 2 * kb + h) * 1024;
            // 32 bytes per lane: row g columns [16t, 16t+16) then row g+8
            const uint4 va = __ldg(reinterpret_cast<const uint4*>(tile + lane * 32));
            const uint4 vb = __ldg(reinterpret_cast<const uint4*>(tile + lane * 32 + 16));
            *reinterpret_cast<uint4*>(B + sw128_offset(r0, 8 * h + 2 * t)) = dequant8_w8(make_uint2(va.x, va.y));
            *reinterpret_cast<uint4*>(B + sw128_offset(r0, 8 * h + 2 * t + 1)) = dequant8_w8(make_uint2(va.z, va.w));
            *reinterpret_cast<uint4*>(B + sw128_offset(r1, 8 * h + 2 * t)) = dequant8_w8(make_uint2(vb.x, vb.y));
            *reinterpret_cast<uint4*>(B + sw128_offset(r1, 8 * h + 2 * t + 1)) = dequant8_w8(make_uint2(vb.z, vb.w));
        }
    }
}

// INT4, exact: warp wb's 16 rows x 128 columns (pair record `rec`, staged in
// shared memory by the TMA warp) as the exact bf16 integers q
// (one LOP3 + one bf16x2 subtract per two weights; word layout as in gemv.cu:
// (w >> 4i) & 0x000F000F is register i, i = 0/2 row g and 1/3 row g+8), and
// the rows' group scales as fp32 into scl[row]. Rows beyond n are zero.
__device__ __forceinline__ void dequant_rows_w4_exact(const GemmTcKParams& p, int64_t rb, const uint8_t* rec, int wb,
                                                      int lane, uint8_t* B, float* scl) {
    const int g = lane >> 2, t = lane & 3;
    const int r0 = wb * 16 + g, r1 = r0 + 8;
    if (rb * 16 >= p.n) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            *reinterpret_cast<uint4*>(B + sw128_offset(r0, 4 * t + c)) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(B + sw128_offset(r1, 4 * t + c)) = make_uint4(0, 0, 0, 0);
        }
        if (t == 0) {
            scl[r0] = 0.f;
            scl[r1] = 0.f;
        }
        return;
    }
    if (t == 0) {
        const uint32_t sv = *reinterpret_cast<const uint32_t*>(rec + 1024 + 4 * g);
        const __half2 s2 = *reinterpret_cast<const __half2*>(&sv);
        scl[r0] = __low2float(s2);
        scl[r1] = __high2float(s2);
    }
    const __nv_bfloat162 bias = __floats2bfloat162_rn(136.f, 136.f);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint4 wv = *reinterpret_cast<const uint4*>(rec + h * 512 + lane * 16);
        const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t reg[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                uint32_t v;
                asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(v) : "r"(w[j] >> (4 * i)), "r"(0x000F000Fu), "r"(0x43084308u));
                __nv_bfloat162 b = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&v), bias);
                reg[j][i] = *reinterpret_cast<uint32_t*>(&b);
            }
        // row g: columns 16t + [0, 8) from words 0-1 (registers 0, 2), [8, 16) from words 2-3
        *reinterpret_cast<uint4*>(B + sw128_offset(r0, 8 * h + 2 * t)) = make_uint4(reg[0][0], reg[0][2], reg[1][0], reg[1][2]);
        *reinterpret_cast<uint4*>(B + sw128_offset(r0, 8 * h + 2 * t + 1)) = make_uint4(reg[2][0], reg[2][2], reg[3][0], reg[3][2]);
        *reinterpret_cast<uint4*>(B + sw128_offset(r1, 8 * h + 2 * t)) = make_uint4(reg[0][1], reg[0][3], reg[1][1], reg[1][3]);
        *reinterpret_cast<uint4*>(B + sw128_offset(r1, 8 * h + 2 * t + 1)) = make_uint4(reg[2][1], reg[2][3], reg[3][1], reg[3][3]);
    }
}

// Stores / epilogue of one thread's 32 accumulated columns col0 .. col0 + 31
// of output row `row` (values already scaled to the weight's units).
template <int FMT, int EPI>
__device__ __forceinline__ void tc_store32(const GemmTcKParams& p, int row, int64_t n0, int col0, const float (&v)[32]) {
    if constexpr (EPI == AMCU_EPI_SILU_MUL) {
        // columns in 16-groups: 8 gate then the matching 8 up rows of the weight
#pragma unroll
        for (int gq = 0; gq < 2; ++gq) {
            const int64_t nb = n0 + col0 + gq * 16;  // first weight row of the group
            if (nb >= p.n) break;
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
                float r2[2];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    float gt = v[gq * 16 + e + u], up = v[gq * 16 + 8 + e + u];
                    if constexpr (FMT == AMCU_WFMT_INT8) {
                        gt *= p.scales[nb + e + u];
                        up *= p.scales[nb + 8 + e + u];
                    }
                    gt = Act<__nv_bfloat16>::round(gt);
                    up = Act<__nv_bfloat16>::round(up);
                    r2[u] = silu_ref(gt) * up;
                }
                __nv_bfloat162 h2 = __floats2bfloat162_rn(r2[0], r2[1]);
                o[e / 2] = *reinterpret_cast<uint32_t*>(&h2);
            }
            *reinterpret_cast<uint4*>(p.y + (int64_t)row * p.y_stride + nb / 2) = make_uint4(o[0], o[1], o[2], o[3]);
        }
    } else {
#pragma unroll
        for (int e8 = 0; e8 < 32; e8 += 8) {
            const int64_t nc = n0 + col0 + e8;
            if (nc >= p.n) break;
            uint4 res = make_uint4(0, 0, 0, 0);
            if constexpr (EPI == AMCU_EPI_RESIDUAL_ADD)
                res = *reinterpret_cast<const uint4*>(p.residual + (int64_t)row * p.y_stride + nc);
            const uint32_t rw[4] = {res.x, res.y, res.z, res.w};
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
                float r2[2];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    float a = v[e8 + e + u];
                    if constexpr (FMT == AMCU_WFMT_INT8) a *= p.scales[nc + e + u];
                    a = Act<__nv_bfloat16>::round(a);
                    if constexpr (EPI == AMCU_EPI_RESIDUAL_ADD)
                        a += __uint_as_float(u == 0 ? rw[e / 2] << 16 : rw[e / 2] & 0xffff0000u);
                    r2[u] = a;
                }
                __nv_bfloat162 h2 = __floats2bfloat162_rn(r2[0], r2[1]);
                o[e / 2] = *reinterpret_cast<uint32_t*>(&h2);
            }
            *reinterpret_cast<uint4*>(p.y + (int64_t)row * p.y_stride + nc) = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

// INT4 keeps every 128-column group's product exact: the MMAs of one K block
// accumulate sum q * x in a fresh TMEM buffer (two buffers, 256 columns), and
// the dequant warps fold it into registers with the group scale (acc += s *
// partial) while the tensor cores work on the next block -- the reference's
// order of operations (sum over groups of scale * integer dot product) up to
// fp32 rounding. INT8 (one per-row scale) accumulates all of K in TMEM and
// scales in the epilogue.
template <int FMT, int EPI>
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmx,
                                                                 GemmTcKParams p) {
    constexpr bool W4 = FMT == AMCU_WFMT_INT4;
    constexpr int kTmemCols = W4 ? 2 * kTcBN : kTcBN;
    constexpr int kScl = kTcStages + 2;  // scale ring: entry kb % kScl is rewritten only after promotion(kb)
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* As = smem;                             // [kTcStages][32 KB]
    uint8_t* Bs = smem + kTcStages * kTcTileBytes;  // [kTcStages][32 KB]
    float* scl = reinterpret_cast<float*>(Bs + kTcStages * kTcTileBytes);  // [kScl][128]
    uint8_t* Ws = reinterpret_cast<uint8_t*>(scl + kScl * kTcBN);        // [kTcStages][8 records] (INT4)
    uint64_t* full_a = reinterpret_cast<uint64_t*>(Ws + (W4 ? kTcStages * kTcWStage : 0));
    uint64_t* full_b = full_a + kTcStages;
    uint64_t* empty = full_b + kTcStages;
    uint64_t* tfull = empty + kTcStages;  // [2] accumulator buffer ready
    uint64_t* tempty = tfull + 2;         // [2] accumulator buffer read out
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kTcBM;
    const int64_t n0 = (int64_t)blockIdx.y * kTcBN;
    const int KB = (int)(p.k / kTcBK);

    if (warp == kTcDequantWarps + 1) {
        if (lane == 0) {
            for (int s = 0; s < kTcStages; ++s) {
                mbar_init(&full_a[s], 1);
                mbar_init(&full_b[s], kTcDequantWarps);
                mbar_init(&empty[s], 1);
            }
            for (int b = 0; b < 2; ++b) {
                mbar_init(&tfull[b], 1);
                mbar_init(&tempty[b], kTcDequantWarps);
            }
            fence_mbar_init();
        }
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = *tmem_slot;
    bool ok = true;
    TcClock whole;
    if (threadIdx.x == 0) whole.start(p);

    if (warp == kTcDequantWarps) {
        // ---- TMA producer: x tiles (the activations come from the previous kernel)
        pdl_wait();
        if (lane == 0) {
            for (int kb = 0; kb < KB; ++kb) {
                const int s = kb % kTcStages;
                if (kb >= kTcStages && ok && !mbar_wait(&empty[s], ((kb / kTcStages) & 1) ^ 1)) {
                    ok = false;
                    record_device_error(p.err, kErrGemmTcWait);
                }
                if (!ok) break;
                uint32_t bytes = kTcTileBytes;
                int nrec = 0;
                if constexpr (W4) {
                    // the 8 row blocks' pair records of this K block (rows beyond n: none)
                    const int64_t rem = (p.n - n0) / 16;
                    nrec = rem < kTcDequantWarps ? (int)rem : kTcDequantWarps;
                    bytes += (uint32_t)(nrec * kW4PairBytes);
                }
                mbar_expect_tx(&full_a[s], bytes);
                uint8_t* dst = As + s * kTcTileBytes;
                tma_load_2d(dst, &tmx, kb * kTcBK, m0, &full_a[s]);
                tma_load_2d(dst + kTcTileBytes / 2, &tmx, kb * kTcBK + 64, m0, &full_a[s]);
                if constexpr (W4) {
                    const int64_t G = p.k / 128;
                    for (int w = 0; w < nrec; ++w)
                        bulk_g2s(Ws + s * kTcWStage + w * kW4PairBytes,
                                 p.w + ((size_t)(n0 / 16 + w) * G + kb) * kW4PairBytes, kW4PairBytes, &full_a[s]);
                }
            }
        }
    } else if (warp == kTcDequantWarps + 1) {
        // ---- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = tc_idesc_bf16(kTcBM, kTcBN);
            for (int kb = 0; kb < KB; ++kb) {
                const int s = kb % kTcStages;
                const uint32_t par = (kb / kTcStages) & 1;
                TcClock ck;
                ck.start(p);
                if (ok && !mbar_wait(&full_a[s], par)) ok = false;
                ck.stop(p, 0);  // 0: MMA waits for the TMA stage
                ck.start(p);
                if (ok && !mbar_wait(&full_b[s], par)) ok = false;
                ck.stop(p, 1);  // 1: MMA waits for the dequantized weights
                ck.start(p);
                if (W4 && ok && kb >= 2 && !mbar_wait(&tempty[kb & 1], ((kb >> 1) & 1) ^ 1)) ok = false;
                ck.stop(p, 2);  // 2: MMA waits for a free accumulator buffer
                if (!ok) {
                    record_device_error(p.err, kErrGemmTcWait);
                    break;
                }
                tc_fence_after();
                const uint32_t a0 = smem_u32(As + s * kTcTileBytes), b0 = smem_u32(Bs + s * kTcTileBytes);
                const uint32_t d = W4 ? taddr + (uint32_t)((kb & 1) * kTcBN) : taddr;
#pragma unroll
                for (int j = 0; j < kTcBK / 16; ++j) {
                    // K step j: half j / 4 of the tile, 32 bytes per step inside the swizzled rows
                    const uint32_t off = (uint32_t)((j >> 2) * (kTcTileBytes / 2) + (j & 3) * 32);
                    tc_mma(d, tc_desc_sw128(a0 + off), tc_desc_sw128(b0 + off), idesc, W4 ? (j != 0) : ((kb | j) != 0));
                }
                tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
                if (W4) tc_commit(&tfull[kb & 1]);
            }
            if (!W4) tc_commit(&tfull[0]);  // all MMAs done: the accumulator is final
        }
    } else {
        // ---- dequant warps (weights do not depend on the previous kernel) and epilogue
        const int64_t rb = n0 / 16 + warp;
        const int quarter = warp & 3, half = warp >> 2;
        const int row = m0 + quarter * 32 + lane;  // TMEM lane of this thread = tile row
        auto produce = [&](int kb) {
            TcClock ck;
            if (warp == 0 && lane == 0) ck.start(p);
            const int s = kb % kTcStages;
            if constexpr (W4) {
                // the TMA warp staged this stage's records after the stage was released
                if (ok && !mbar_wait(&full_a[s], (kb / kTcStages) & 1)) {
                    ok = false;
                    if (lane == 0) record_device_error(p.err, kErrGemmTcWait);
                }
            } else if (kb >= kTcStages && ok && !mbar_wait(&empty[s], ((kb / kTcStages) & 1) ^ 1)) {
                ok = false;
                if (lane == 0) record_device_error(p.err, kErrGemmTcWait);
            }
            if (!ok) return;
            if (!(TC_DBG(p) & 1)) {
                if constexpr (W4)
                    dequant_rows_w4_exact(p, rb, Ws + s * kTcWStage + warp * kW4PairBytes, warp, lane,
                                          Bs + s * kTcTileBytes, scl + (kb % kScl) * kTcBN);
                else dequant_rows<FMT>(p, rb, kb, warp, lane, Bs + s * kTcTileBytes);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
            __syncwarp();
            if (lane == 0) mbar_arrive(&full_b[s]);
            if (warp == 0 && lane == 0) ck.stop(p, 3);  // 3: dequant warp 0 producing a stage
        };
        float acc[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) acc[i] = 0.f;
        if constexpr (W4) {
            for (int kb = 0; kb < kTcStages && kb < KB; ++kb) produce(kb);
            for (int kb = 0; kb < KB; ++kb) {
                TcClock ck;
                if (warp == 0 && lane == 0) ck.start(p);
                if (ok && !mbar_wait(&tfull[kb & 1], (kb >> 1) & 1)) {
                    ok = false;
                    if (lane == 0) record_device_error(p.err, kErrGemmTcWait);
                }
                if (warp == 0 && lane == 0) ck.stop(p, 4);  // 4: dequant warp 0 waits for the MMAs
                if (warp == 0 && lane == 0) ck.start(p);
                tc_fence_after();
                const float* sc = scl + (kb % kScl) * kTcBN + half * 64;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    if (TC_DBG(p) & 2) break;
                    uint32_t r[32];
                    tc_ld_32x32b_x32(taddr + (uint32_t)((kb & 1) * kTcBN) + ((uint32_t)(quarter * 32) << 16) +
                                             (uint32_t)(half * 64 + c * 32),
                                     r);
#pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        const float4 s4 = *reinterpret_cast<const float4*>(sc + c * 32 + i);
                        acc[c * 32 + i + 0] = fmaf(s4.x, __uint_as_float(r[i + 0]), acc[c * 32 + i + 0]);
                        acc[c * 32 + i + 1] = fmaf(s4.y, __uint_as_float(r[i + 1]), acc[c * 32 + i + 1]);
                        acc[c * 32 + i + 2] = fmaf(s4.z, __uint_as_float(r[i + 2]), acc[c * 32 + i + 2]);
                        acc[c * 32 + i + 3] = fmaf(s4.w, __uint_as_float(r[i + 3]), acc[c * 32 + i + 3]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[kb & 1]);
                if (warp == 0 && lane == 0) ck.stop(p, 5);  // 5: dequant warp 0 promoting
                if (kb + kTcStages < KB) produce(kb + kTcStages);
            }
        } else {
            for (int kb = 0; kb < KB; ++kb) produce(kb);
            if (ok && !mbar_wait(&tfull[0], 0)) {
                ok = false;
                if (lane == 0) record_device_error(p.err, kErrGemmTcWait);
            }
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t r[32];
                tc_ld_32x32b_x32(taddr + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(half * 64 + c * 32), r);
#pragma unroll
                for (int i = 0; i < 32; ++i) acc[c * 32 + i] = __uint_as_float(r[i]);
            }
        }
        // ---- epilogue: this thread's row, columns half * 64 .. + 63
        TcClock cke;
        if (warp == 0 && lane == 0) cke.start(p);
        pdl_wait();
        if (row < p.m && ok && !(TC_DBG(p) & 4)) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = acc[c * 32 + i];
                tc_store32<FMT, EPI>(p, row, n0, half * 64 + c * 32, v);
            }
        }
        pdl_trigger();
        if (warp == 0 && lane == 0) cke.stop(p, 7);  // 7: epilogue
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) whole.stop(p, 6);  // 6: CTA main body
    if (warp == kTcDequantWarps + 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(kTmemCols) : "memory");
    }
}


// ---------------------------------------------------------------------------
// INT4 with the operands swapped: out^T = W x^T. The dequantized weights are
// the MMA's A operand and go from registers straight into tensor memory
// (tcgen05.st), the activations are B (TMA, 128-byte swizzle). Shared memory
// then carries only the activation tiles (written by TMA, read once by the
// tensor cores) and the pair records, about half the bytes per FLOP of the
// kernel above, whose bf16 weight tiles are written and read through shared
// memory. A CTA computes 128 weight rows x 128 tokens.
//
// Tensor memory (512 columns): D0 [0, 128) and D1 [128, 256) hold the
// partial sums of one K block (one scale group) each, A stage s at
// [256 + 64 s, +64) holds 128 weight rows x 128 K as bf16 pairs.
//
// Warps 0-7: warp w dequantizes weight rows 32 (w % 4) .. +31 (its TMEM lane
// quarter), K half w / 4 of every block, then folds the partial sums of the
// same rows, token half w / 4, into registers with each row's group scale,
// and finally stores those outputs. Warp 8: TMA of the activation tile and
// the 8 pair records per stage. Warp 9: TMEM owner and MMA issuer.
constexpr int kSwStages = 4;   // shared-memory activation stages
constexpr int kSwWStages = 8;  // shared-memory pair-record stages (their own producer warp runs ahead)
constexpr int kSwAStages = 4;  // TMEM weight stages (64 columns each, after the 256 accumulator columns)
constexpr int kSwXBytes = kTcBN * kTcBK * 2;  // activation tile: 128 tokens x 128 K
constexpr int kSwDqWarps = 16;                // dequant / promotion / epilogue warps
constexpr int kSwThreads = (kSwDqWarps + 3) * 32;  // + activation TMA warp, MMA warp, record warp
constexpr int kSwSmemBytes = 1024 + kSwStages * kSwXBytes + kSwWStages * kTcWStage + (kSwAStages + 2) * kTcBM * 4 + 512;

__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
            " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
            "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(acc)
            : "memory");
}
__device__ __forceinline__ void tc_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
            "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
            "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
            "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
            "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
            "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
            : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tc_st_32x32b_x16_nowait(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
            "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
            "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
            : "memory");
}
__device__ __forceinline__ void tc_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
            "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
            "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
            : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

template <int EPI>
__global__ void __launch_bounds__(kSwThreads, 1) gemm_w4_swap_kernel(const __grid_constant__ CUtensorMap tmx,
                                                                      GemmTcKParams p) {
    constexpr int S = kSwStages, SA = kSwAStages, SW = kSwWStages;
    static_assert(S == SA, "one release per K block frees the activation stage and the TMEM weight stage");
    constexpr int kScl = SA + 2;  // scale ring: entry kb % kScl is rewritten only after promotion(kb)
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* Xs = smem;                                                  // [S][32 KB] activations
    uint8_t* Ws = smem + S * kSwXBytes;                                  // [SW][8 pair records]
    float* scl = reinterpret_cast<float*>(Ws + SW * kTcWStage);          // [kScl][128] row scales
    uint64_t* full = reinterpret_cast<uint64_t*>(scl + kScl * kTcBM);    // [S] activation stage landed (TMA)
    uint64_t* fulla = full + S;                                          // [SA] weights of TMEM stage in place
    uint64_t* empty = fulla + SA;                                        // [S] MMAs of the activation stage done
    uint64_t* fullw = empty + S;                                         // [SW] record stage landed
    uint64_t* wempty = fullw + SW;                                       // [SW] record stage read by the dequant warps
    uint64_t* tempty = wempty + SW;                                      // [2] partial sums folded
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    int* dq_fail = reinterpret_cast<int*>(tmem_slot + 1);  // a dequant-side wait ran out

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) tc_stamp(p, 9);  // CTA start
    const int m0 = blockIdx.x * kTcBN;                 // first token
    const int64_t n0 = (int64_t)blockIdx.y * kTcBM;    // first weight row
    const int KB = (int)(p.k / kTcBK);

    if (warp == kSwDqWarps + 1) {
        if (lane == 0) {
            for (int s = 0; s < S; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], 1);
            }
            for (int s = 0; s < SA; ++s) mbar_init(&fulla[s], kSwDqWarps);
            *dq_fail = 0;
            for (int s = 0; s < SW; ++s) {
                mbar_init(&fullw[s], 1);
                mbar_init(&wempty[s], kSwDqWarps);
            }
            for (int b = 0; b < 2; ++b) {
                mbar_init(&tempty[b], kSwDqWarps);
            }
            fence_mbar_init();
        }
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = *tmem_slot;
    bool ok = true;
    TcClock whole;
    if (threadIdx.x == 0) whole.start(p);

    if (warp == kSwDqWarps) {
        // ---- TMA producer of the activation tiles (they come from the previous kernel)
        pdl_wait();
        if (lane == 0) {
            for (int kb = 0; kb < KB; ++kb) {
                const int s = kb % S;
                if (kb >= S && ok && !mbar_wait(&empty[s], ((kb / S) & 1) ^ 1)) {
                    ok = false;
                    record_device_error(p.err, kErrGemmTcWait);
                }
                if (!ok) break;
                if (TC_DBG(p) & 16) {  // diagnostics: no activation loads
                    mbar_arrive(&full[s]);
                    continue;
                }
                mbar_expect_tx(&full[s], (uint32_t)kSwXBytes);
                uint8_t* dst = Xs + s * kSwXBytes;
                tma_load_2d(dst, &tmx, kb * kTcBK, m0, &full[s]);
                tma_load_2d(dst + kSwXBytes / 2, &tmx, kb * kTcBK + 64, m0, &full[s]);
            }
        }
    } else if (warp == kSwDqWarps + 2) {
        // ---- producer of the pair records (weights: no dependence on the previous kernel)
        if (lane == 0) {
            const int64_t rem = (p.n - n0) / 16;
            const int nrec = rem < kTcBM / 16 ? (int)rem : kTcBM / 16;
            const int64_t G = p.k / 128;
            for (int kb = 0; kb < KB; ++kb) {
                const int s = kb % SW;
                if (kb >= SW && ok && !mbar_wait(&wempty[s], ((kb / SW) & 1) ^ 1)) {
                    ok = false;
                    record_device_error(p.err, kErrGemmTcWait);
                }
                if (!ok) break;
                if (TC_DBG(p) & 32) {  // diagnostics: no record loads
                    mbar_arrive(&fullw[s]);
                    continue;
                }
                mbar_expect_tx(&fullw[s], (uint32_t)(nrec * kW4PairBytes));
                for (int w = 0; w < nrec; ++w)
                    bulk_g2s(Ws + s * kTcWStage + w * kW4PairBytes, p.w + ((size_t)(n0 / 16 + w) * G + kb) * kW4PairBytes,
                             kW4PairBytes, &fullw[s]);
            }
        }
    } else if (warp == kSwDqWarps + 1) {
        // ---- MMA issuer: D[kb & 1] = W_tile(kb) x X_tile(kb)^T over the block's 8 K steps
        if (lane == 0) {
            constexpr uint32_t idesc = tc_idesc_bf16(kTcBM, kTcBN);
            for (int kb = 0; kb < KB; ++kb) {
                const int s = kb % S;
                const uint32_t par = (kb / S) & 1;
                TcClock ck;
                ck.start(p);
                if (ok && !mbar_wait(&full[s], par)) ok = false;
                ck.stop(p, 0);
                ck.start(p);
                if (ok && !mbar_wait(&fulla[kb % SA], (kb / SA) & 1)) ok = false;
                ck.stop(p, 1);
                ck.start(p);
                if (ok && kb >= 2 && !mbar_wait(&tempty[kb & 1], ((kb >> 1) & 1) ^ 1)) ok = false;
                ck.stop(p, 2);
                if (kb == 0) tc_stamp(p, 8);
                if (!ok) {
                    record_device_error(p.err, kErrGemmTcWait);
                    break;
                }
                tc_fence_after();
                const uint32_t b0 = smem_u32(Xs + s * kSwXBytes);
                const uint32_t d = taddr + (uint32_t)((kb & 1) * kTcBN);
                const uint32_t a = taddr + 256u + (uint32_t)(64 * (kb % SA));
#pragma unroll
                for (int j = 0; j < kTcBK / 16; ++j) {
                    // K step j: 16 bf16 = 8 TMEM columns of A; 32 bytes per step in the swizzled B rows
                    const uint32_t off = (uint32_t)((j >> 2) * (kSwXBytes / 2) + (j & 3) * 32);
                    tc_mma_ts(d, a + (uint32_t)(8 * j), tc_desc_sw128(b0 + off), idesc, j != 0);
                }
                if (kb == KB - 1) tc_stamp(p, 10);  // last MMAs issued
                // one commit: the block's MMAs are done, so the activation stage
                // and the TMEM weight stage are free and its partial sums ready
                // (a second commit per block measured 1.7% slower)
                tc_commit(&empty[s]);
            }
        }
    } else {
        // ---- dequant / promotion / epilogue warps: warp w serves TMEM lane
        // quarter q = w % 4 (weight rows 32 q .. +31, one per lane) and part
        // pt = w / 4: K columns 32 pt .. +31 of every block when producing,
        // tokens 32 pt .. +31 when promoting and storing
        const int q = warp & 3, pt = warp >> 2;
        const int r = q * 32 + lane;  // weight row in the tile = TMEM lane
        const int blk = r >> 4, rr = r & 15, g = rr & 7, hi = rr >> 3;
        const int64_t rb = n0 / 16 + blk;
        const bool valid = rb * 16 < p.n;
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        int pending = -1;  // stage whose TMEM store is issued but not yet published
        // completes the TMEM store of the last produced stage and hands it to the MMA warp
        auto publish = [&]() {
            if (pending < 0) return;
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&fulla[pending % SA]);
            pending = -1;
        };
        auto dq_wait = [&](uint64_t* b1, uint32_t par1, uint64_t* b2, uint32_t par2) {
            if (ok && (!mbar_wait(b1, par1) || (b2 && !mbar_wait(b2, par2)))) {
                ok = false;
                if (lane == 0) record_device_error(p.err, kErrGemmTcWait);
            }
        };
        auto produce = [&](int kb) {
            TcClock ck;
            if (warp == 0 && lane == 0) ck.start(p);
            const int sw = kb % SW, sa = kb % SA;
            dq_wait(&fullw[sw], (kb / SW) & 1, kb >= SA ? &empty[sa] : nullptr, ((kb / SA) & 1) ^ 1);
            if (!ok) return;
            publish();
            const uint8_t* rec = Ws + sw * kTcWStage + blk * kW4PairBytes;
            uint32_t v[16];
            if (valid && !(TC_DBG(p) & 1)) {
                if (pt == 0)
                    scl[(kb % kScl) * kTcBM + r] =
                            __half2float(reinterpret_cast<const __half*>(rec + 1024)[2 * g + hi]);
                // Rows g and g+8 of the 16-row block share the 64 bytes at 64 g of
                // tile pt / 2 (K columns 64 (pt / 2) .. +63); word 4t + j covers
                // columns 16t + 4j .. +3 as nibbles p0 p4 p2 p6 (row g) / p1 p5 p3 p7
                // (row g+8). Part pt takes the 32 bytes of its 32 columns.
                const uint4* src = reinterpret_cast<const uint4*>(rec + (pt >> 1) * 512 + g * 64 + (pt & 1) * 32);
                const uint4 wa = src[0], wb = src[1];
                const uint32_t w8[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
                const __nv_bfloat162 bias = __floats2bfloat162_rn(136.f, 136.f);
                const uint32_t sh = 4u * (uint32_t)hi;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    uint32_t lo2, hi2;
                    asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(lo2) : "r"(w8[j] >> sh), "r"(0x000F000Fu), "r"(0x43084308u));
                    asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(hi2) : "r"(w8[j] >> (sh + 8)), "r"(0x000F000Fu), "r"(0x43084308u));
                    __nv_bfloat162 b0 = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&lo2), bias);
                    __nv_bfloat162 b1 = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&hi2), bias);
                    v[2 * j] = *reinterpret_cast<uint32_t*>(&b0);
                    v[2 * j + 1] = *reinterpret_cast<uint32_t*>(&b1);
                }
            } else {
                if (pt == 0) scl[(kb % kScl) * kTcBM + r] = 0.f;
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] = 0u;
            }
            tc_st_32x32b_x16_nowait(taddr + lane_base + 256u + (uint32_t)(64 * sa + 16 * pt), v);
            __syncwarp();
            if (lane == 0) mbar_arrive(&wempty[sw]);  // records read (the scale went to scl)
            pending = kb;
            if (warp == 0 && lane == 0) ck.stop(p, 3);
        };
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.f;
        for (int kb = 0; kb < SA && kb < KB; ++kb) produce(kb);
        publish();
        for (int kb = 0; kb < KB; ++kb) {
            TcClock ck;
            if (warp == 0 && lane == 0) ck.start(p);
            // partial sums of block kb ready: its MMAs completed (the commit on
            // empty[kb % S]). That phase cannot be overtaken: block kb + S
            // needs buffer kb & 1 back, i.e. every warp past promotion kb + 2.
            dq_wait(&empty[kb % S], (kb / S) & 1, nullptr, 0);
            if (warp == 0 && lane == 0) ck.stop(p, 4);
            if (warp == 0 && lane == 0) ck.start(p);
            tc_fence_after();
            const float sc = scl[(kb % kScl) * kTcBM + r];
            if (!(TC_DBG(p) & 2)) {
                uint32_t t32[32];
                tc_ld_32x32b_x32(taddr + lane_base + (uint32_t)((kb & 1) * kTcBN + 32 * pt), t32);
#pragma unroll
                for (int i = 0; i < 32; ++i) acc[i] = fmaf(sc, __uint_as_float(t32[i]), acc[i]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[kb & 1]);
            if (warp == 0 && lane == 0) ck.stop(p, 5);
            if (kb + SA < KB) produce(kb + SA);
            if (kb + 1 + SA >= KB) publish();  // nothing produced after this one
        }
        publish();
        if (warp == 0 && lane == 0) tc_stamp(p, 11);  // last promotion done
        // ---- epilogue: the tile goes through shared memory (the first activation
        // stage, idle now: every MMA has completed) as [128 tokens][128 or 64
        // columns] bf16, then out with 16-byte row stores
        TcClock cke;
        if (warp == 0 && lane == 0) cke.start(p);
        constexpr bool SILU = EPI == AMCU_EPI_SILU_MUL;
        constexpr int OC = SILU ? kTcBM / 2 : kTcBM;  // output columns of the tile
        __nv_bfloat16* T = reinterpret_cast<__nv_bfloat16*>(Xs);
        const int tb = 32 * pt;  // this thread's first token in the tile
        if (TC_DBG(p) & 8) {
        } else if constexpr (SILU) {
            // rows 0-7 of a 16-row block are gate rows, 8-15 the matching up
            // rows: lanes g and g+8 swap one value per token pair, so each
            // computes one of the two outputs
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
                const float send = hi ? acc[i] : acc[i + 1];
                const float recv = __shfl_xor_sync(0xffffffffu, send, 8);
                const float gt = hi ? recv : acc[i], up = hi ? acc[i + 1] : recv;
                T[(tb + i + hi) * OC + blk * 8 + g] =
                        __float2bfloat16_rn(silu_ref(Act<__nv_bfloat16>::round(gt)) * Act<__nv_bfloat16>::round(up));
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) T[(tb + i) * OC + r] = __float2bfloat16_rn(Act<__nv_bfloat16>::round(acc[i]));
        }
        named_bar_sync(1, kSwDqWarps * 32);
        pdl_wait();
        if (ok && !(TC_DBG(p) & 4)) {
            const int64_t c0 = SILU ? n0 / 2 : n0;          // first output column of the tile
            const int64_t cend = SILU ? p.n / 2 : p.n;
            constexpr int CH = OC / 8;                      // 16-byte chunks per token row
            for (int e = threadIdx.x; e < kTcBN * CH; e += kSwDqWarps * 32) {
                const int tr = e / CH, ch = e % CH;
                const int64_t col = c0 + ch * 8;
                if (m0 + tr >= p.m || col >= cend) continue;
                uint4 v = *reinterpret_cast<const uint4*>(T + tr * OC + ch * 8);
                const int64_t off = (int64_t)(m0 + tr) * p.y_stride + col;
                if constexpr (EPI == AMCU_EPI_RESIDUAL_ADD) {
                    const uint4 rv = *reinterpret_cast<const uint4*>(p.residual + off);
                    uint32_t a4[4] = {v.x, v.y, v.z, v.w};
                    const uint32_t r4[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float lo = __uint_as_float(a4[j] << 16) + __uint_as_float(r4[j] << 16);
                        const float hi2 = __uint_as_float(a4[j] & 0xffff0000u) + __uint_as_float(r4[j] & 0xffff0000u);
                        __nv_bfloat162 h2 = __floats2bfloat162_rn(lo, hi2);
                        a4[j] = *reinterpret_cast<uint32_t*>(&h2);
                    }
                    v = make_uint4(a4[0], a4[1], a4[2], a4[3]);
                }
                *reinterpret_cast<uint4*>(p.y + off) = v;
            }
        }
        if (warp == 0 && lane == 0) cke.stop(p, 7);
        if (warp == 0 && lane == 0) tc_stamp(p, 12);  // epilogue done
        pdl_trigger();
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) whole.stop(p, 6);
    if (warp == kSwDqWarps + 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(512) : "memory");
    }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// dependency on a particular driver library name).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        else
            cudaGetLastError();
    }
    return fn;
}

bool gemm_tc_supported(const GemmTcParams& p, int fmt) {
    if (fmt != AMCU_WFMT_INT4 && fmt != AMCU_WFMT_INT8) return false;
    if (p.k % kTcBK != 0 || p.n % 16 != 0) return false;
    if ((p.x_stride * 2) % 16 != 0 || (reinterpret_cast<uintptr_t>(p.x) & 15) != 0) return false;
    if ((reinterpret_cast<uintptr_t>(p.y) & 15) != 0 || (p.y_stride * 2) % 16 != 0) return false;
    if (p.residual && (reinterpret_cast<uintptr_t>(p.residual) & 15) != 0) return false;
    if (p.m > 0x7fffffff || p.k > 0x7fffffff) return false;
    return encode_tiled() != nullptr;
}
size_t gemm_tc_workspace_bytes(const GemmTcParams&, int) { return 0; }

#ifdef AMCU_DIAG
static int gemm_dbg() {
    static const int v = [] {
        const char* e = std::getenv("AMCU_GEMM_DBG");
        return e ? std::atoi(e) : 0;
    }();
    return v;
}

// Diagnostics (AMCU_GEMM_TRACE=file, eager runs only): per-CTA cycle counters
// of one launch, appended to the file when the launch has finished.
struct TcTrace {
    unsigned long long* buf = nullptr;
    size_t n = 0;
    dim3 grid;
    cudaStream_t s;
    TcTrace(dim3 g, cudaStream_t st) : grid(g), s(st) {
        static const char* path = std::getenv("AMCU_GEMM_TRACE");
        if (!path) return;
        n = (size_t)g.x * g.y * 16;
        if (cudaMalloc(&buf, n * 8) != cudaSuccess || cudaMemsetAsync(buf, 0, n * 8, s) != cudaSuccess) buf = nullptr;
    }
    ~TcTrace() {
        if (!buf) return;
        std::vector<unsigned long long> h(n);
        if (cudaStreamSynchronize(s) == cudaSuccess && cudaMemcpy(h.data(), buf, n * 8, cudaMemcpyDeviceToHost) == cudaSuccess)
            if (FILE* f = std::fopen(std::getenv("AMCU_GEMM_TRACE"), "ab")) {
                const int hdr[2] = {(int)grid.x, (int)grid.y};
                std::fwrite(hdr, sizeof(hdr), 1, f);
                std::fwrite(h.data(), 8, n, f);
                std::fclose(f);
            }
        cudaFree(buf);
    }
};
#else
static int gemm_dbg() { return 0; }
struct TcTrace {
    unsigned long long* buf = nullptr;
    TcTrace(dim3, cudaStream_t) {}
};
#endif

template <int FMT, int EPI>
static am_status_code launch_tc(const GemmTcParams& g, const CUtensorMap& map, cudaStream_t s) {
    auto kern = gemm_tc_kernel<FMT, EPI>;
    set_func_attr_once((const void*)kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmemBytes);
    GemmTcKParams p{};
    p.w = static_cast<const uint8_t*>(g.w);
    p.scales = static_cast<const float*>(g.scales);
    p.y = static_cast<__nv_bfloat16*>(g.y);
    p.residual = static_cast<const __nv_bfloat16*>(g.residual);
    p.m = g.m;
    p.n = g.n;
    p.k = g.k;
    p.y_stride = g.y_stride;
    p.err = device_error_word();
    p.dbg = gemm_dbg();
    const dim3 grid((unsigned)((g.m + kTcBM - 1) / kTcBM), (unsigned)((g.n + kTcBN - 1) / kTcBN));
    TcTrace tr(grid, s);
    p.trace = tr.buf;
    launch_pdl(kern, grid, dim3(kTcThreads), (size_t)kTcSmemBytes, s, map, p);
    return AM_STATUS_OK;
}

template <int EPI>
static am_status_code launch_swap(const GemmTcParams& g, const CUtensorMap& map, cudaStream_t s) {
    auto kern = gemm_w4_swap_kernel<EPI>;
    set_func_attr_once((const void*)kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSwSmemBytes);
    GemmTcKParams p{};
    p.w = static_cast<const uint8_t*>(g.w);
    p.y = static_cast<__nv_bfloat16*>(g.y);
    p.residual = static_cast<const __nv_bfloat16*>(g.residual);
    p.m = g.m;
    p.n = g.n;
    p.k = g.k;
    p.y_stride = g.y_stride;
    p.err = device_error_word();
    p.dbg = gemm_dbg();
    const dim3 grid((unsigned)((g.m + kTcBN - 1) / kTcBN), (unsigned)((g.n + kTcBM - 1) / kTcBM));
    TcTrace tr(grid, s);
    p.trace = tr.buf;
    launch_pdl(kern, grid, dim3(kSwThreads), (size_t)kSwSmemBytes, s, map, p);
    return AM_STATUS_OK;
}

am_status_code launch_gemm_tc(const GemmTcParams& g, int fmt, int epi, cudaStream_t s) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return set_error(AM_STATUS_UNAVAILABLE, "cuTensorMapEncodeTiled unavailable");
    // x as a 2-D bf16 tensor [m rows][k columns], boxes of 64 columns x 128 rows, 128-byte swizzle
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)g.k, (cuuint64_t)g.m};
    const cuuint64_t strides[1] = {(cuuint64_t)g.x_stride * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)kTcBM};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(g.x), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(AM_STATUS_INTERNAL, "cuTensorMapEncodeTiled failed (%d)", (int)r);
#define AMCU_TC(F, E) return launch_tc<F, E>(g, map, s)
    static const bool swap = [] {
        const char* v = std::getenv("AMCU_GEMM_SWAP");
        return !(v && v[0] == '0');
    }();
    if (fmt == AMCU_WFMT_INT4 && swap) {
        if (epi == AMCU_EPI_STORE) return launch_swap<AMCU_EPI_STORE>(g, map, s);
        if (epi == AMCU_EPI_RESIDUAL_ADD) return launch_swap<AMCU_EPI_RESIDUAL_ADD>(g, map, s);
        return launch_swap<AMCU_EPI_SILU_MUL>(g, map, s);
    }
    if (fmt == AMCU_WFMT_INT4) {
        if (epi == AMCU_EPI_STORE) AMCU_TC(AMCU_WFMT_INT4, AMCU_EPI_STORE);
        if (epi == AMCU_EPI_RESIDUAL_ADD) AMCU_TC(AMCU_WFMT_INT4, AMCU_EPI_RESIDUAL_ADD);
        AMCU_TC(AMCU_WFMT_INT4, AMCU_EPI_SILU_MUL);
    }
    if (epi == AMCU_EPI_STORE) AMCU_TC(AMCU_WFMT_INT8, AMCU_EPI_STORE);
    if (epi == AMCU_EPI_RESIDUAL_ADD) AMCU_TC(AMCU_WFMT_INT8, AMCU_EPI_RESIDUAL_ADD);
    AMCU_TC(AMCU_WFMT_INT8, AMCU_EPI_SILU_MUL);
#undef AMCU_TC
}

}  // namespace amcu
