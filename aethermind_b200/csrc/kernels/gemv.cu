// Weight-only dequant GEMV for decode (m <= 8) and the weight prepacker.
//
// Device weight format ("tile16x64"): the [N, K] weight is cut into tiles of
// 16 output rows x 64 input columns, stored row block after row block with K
// fastest. Inside a tile, lane L = 4g + t of a warp owns rows {g, g+8} x
// columns [16t, 16t+16): exactly the A-operand fragments of four m16n8k16
// tensor-core MMAs in which MMA j contracts columns 16t+4j .. 16t+4j+3 of this
// lane (the MMA's k-slot -> column map is a free choice as long as the
// activation fragment uses the same one). One 16-byte (INT4) or 32-byte
// (INT8) conflict-free load per lane per tile feeds the MMAs with no
// shuffles; the activations for the same columns are 32 contiguous bytes per
// lane.
//   INT4: the two tiles of a 128-column group and the group's 16 row scales
//        form one 1056-byte pair record (tile 2p, tile 2p+1, 16 fp16 scales
//        with slot 2g = row g, 2g+1 = row g+8), so one bulk copy brings
//        weights and scales together; record (rb, p) at (rb * K/128 + p) *
//        1056. Word j of lane L: nibble p at bits 4p holds two's-complement
//        q; p0,p4,p2,p6 = row g columns +0,+1,+2,+3 and p1,p5,p3,p7 = row g+8
//        columns +0,+1,+2,+3, so (word >> 4i) & 0x000F000F yields MMA
//        register i directly.
//   INT8: 1024-byte tiles, tile (rb, c) at (rb * K/64 + c) * 1024; 32 bytes
//        per lane: row g columns [16t, 16t+16) then row g+8. Scales: fp32 [N]
//        (device row order) in their own buffer.
// Gate/up fusion: rows 0-7 of every tile are gate rows 8*rb..8*rb+7 and rows
// 8-15 the matching up rows, so one lane holds gate and up of the same output
// and the SiLU-Mul epilogue needs no data exchange.
#include <cooperative_groups.h>

#include "../amcu_internal.h"
#include <cstdlib>

#include "allreduce.cuh"
#include "diag_timeline.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "gemv_core.cuh"
#include "gemv_stage.cuh"
#include "mma_int4.cuh"

namespace cg = cooperative_groups;

namespace amcu {

// Streaming GEMV. A CTA of 8 consumer warps and 1 producer warp owns
// `rb_per_cta` consecutive row blocks (16 output rows each), one contiguous
// run of the packed weight. The producer streams that run through a ring of
// `stages` shared-memory stages with bulk copies (TMA engine) of 8-33 KB --
// copies that small stop being able to keep HBM busy -- completing on one
// mbarrier per stage; the consumers release a stage on a second mbarrier. The first stages are
// requested before the kernel waits for its predecessor. In a stage the
// consumer warps split the 128-column groups (INT4 pair records, INT8 tile
// pairs) and read their tiles with one conflict-free shared load per lane per
// tile. The activations (m <= 8 rows, bf16) are staged once per CTA in shared
// memory.
//
// INT4 tiles go to fp16 MMAs as exact integers with an offset: one LOP3
// selects two nibbles and ORs in the fp16 exponent of 1024, giving 1032 + q
// for nibbles in bits 0-3 of each half (rows g) and 1152 + 16q for nibbles in
// bits 4-7 (rows g+8), so a 32-bit word costs four LOP3 and one shift. The
// offsets are removed after the MMA with the per-group sums of x (computed
// once per CTA) and the 16 is folded into the row's scale. The activations
// are staged as fp16 for this: converting bf16 to fp16 is exact in fp16's
// normal range, and a row whose magnitude would overflow fp16 is staged
// multiplied by an exact power of two that the epilogue takes back out.
// Products (offset + q) * x are exact in fp32, so the offsets cost only fp32
// rounding.
//
// At the end of a row block the warps' 16 x 8 partial tiles meet in shared
// memory (double-buffered, one barrier) and one warp applies the epilogue.
//
// The grid covers the CTA slots of all SMs only as far as whole row blocks
// allow (e.g. 256 CTAs for 1792 row blocks on 296 slots). Dealing the groups
// to all 296 slots in equal ranges cut inside row blocks (a split-K with a
// last-arriver combine) measured slower, 17.4 against 13.3 us for the 8B
// gate/up: the free slots let the next kernel's CTAs start early under PDL and
// fetch their weights while this one finishes, which outweighs the balance.
template <int FMT, int EPI, bool M1, int NC>
__global__ void __launch_bounds__((NC + 1) * 32, NC == kGemvConsumers ? GEMV_MINB : 1) gemv_tc_kernel(GemvParams p) {
    DiagTl tl;
    tl.entry();
    constexpr bool W4 = FMT == AMCU_WFMT_INT4;
    constexpr int UB = W4 ? kW4PairBytes : 2048;  // bytes per 128-column group unit
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int S = p.stages, SU = p.stage_units;  // stages; group units per stage
    const int SBY = SU * UB;                     // bytes per stage
    const int G = (int)(p.k / 128);              // group units per row block
    const int M = (int)p.m;
    const int xrow = (int)(p.k * 2 + kXPad);
    const GemvSmem L = gemv_smem<FMT, NC>(M, p.k, SBY, S);
    float4* red = reinterpret_cast<float4*>(smem + L.red);  // [2][consumers][32]
    float* sx = reinterpret_cast<float*>(smem + L.sx);      // [G][8] (INT4)
    uint8_t* xs = smem + L.xs;                              // [M][k] bf16 (+pad)
    uint8_t* ring = smem + L.ring;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
    uint64_t* empty = full + S;

    // row blocks rb0 .. rb0 + nr - 1, per_row stages of SU units each (SU divides G)
    const int nrb = (int)(p.n / 16);
    const int rb0 = blockIdx.x * p.rb_per_cta;
    const int nr = (rb0 + p.rb_per_cta < nrb ? rb0 + p.rb_per_cta : nrb) - rb0;
    const int per_row = G / SU;
    const int total = nr * per_row;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NC);
        }
        fence_mbar_init();
        l2_prefetch_share(p.l2_next);
    }
    __syncthreads();

    if (warp == NC) {
        // ---- producer: weights do not depend on earlier kernels, so the ring
        // fills while the previous kernel finishes.
        if (lane == 0) {
            int slot = 0;
            uint32_t phase = 0;
            const uint8_t* run = static_cast<const uint8_t*>(p.w) + (size_t)rb0 * G * UB;
            const uint64_t pol = gemv_weight_policy();
            for (int i = 0; i < total; ++i) {
                if (i >= S && !mbar_wait(&empty[slot], phase ^ 1u)) {
                    record_device_error(p.err, kErrGemvEmptyWait);
                    break;
                }
                mbar_expect_tx(&full[slot], SBY);
                bulk_g2s_hint(ring + slot * SBY, run + (size_t)i * SBY, SBY, &full[slot], pol);
                if (++slot == S) {
                    slot = 0;
                    phase ^= 1;
                }
            }
        }
        return;
    }

    __shared__ StageShared stsh;
    pdl_wait();
    pdl_trigger();
    tl.waited();

    // ---- stage the activations (fused RMSNorm; INT4: fp16 + group sums)
    {
        StageCtx sc{static_cast<const __nv_bfloat16*>(p.x), p.x_stride, p.k, M,
                    static_cast<const __nv_bfloat16*>(p.norm_w), p.eps, xs, xrow, sx, &stsh,
                    (int)threadIdx.x, NC * 32, 2};
        stage_activations<W4>(sc);
    }
    if (threadIdx.x == 0) tl.mark2();  // staged
    const float* row_mul = stsh.row_mul;
    constexpr int NT = NC * 32;
    const float rm0 = 2 * t < M ? row_mul[2 * t] : 1.f, rm1 = 2 * t + 1 < M ? row_mul[2 * t + 1] : 1.f;

    // Lanes whose activation row does not exist (g >= M) read row 0: they only
    // feed MMA output columns g >= M, which the epilogue never stores.
    const uint8_t* xrow_g = xs + (g < M ? g : 0) * xrow + 32 * t;  // + 256 B per group unit
    int slot = 0;
    uint32_t phase = 0;
    bool ok = true;  // false once a wait ran out: keep the control flow, skip further waits
    int fail_i = -1;
    int par = 0;
    float acc[4];
    // one stage: wait for it, run its units, release it
    auto stage = [&](int i, int grp0, int len) {
        if (ok && !mbar_wait(&full[slot], phase)) {
            ok = false;
            fail_i = i;
            if (lane == 0) record_device_error(p.err, kErrGemvFullWait);
        }
        gemv_stage<FMT, M1, NC>(ring + slot * SBY, len, xrow_g, sx, grp0, warp, lane, g, t, acc);
        __syncwarp();  // every lane has read the stage
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (++slot == S) {
            slot = 0;
            phase ^= 1;
        }
    };
    // row-block end: publish this warp's partial tile, meet the other warps,
    // and let one warp reduce and apply the epilogue
    auto finish = [&](int rb) {
        red[(par * NC + warp) * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        named_bar_sync(1, NT);
        if (warp == rb % NC) {
            float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int w = 0; w < NC; ++w) {
                const float4 v = red[(par * NC + w) * 32 + lane];
                s4.x += v.x; s4.y += v.y; s4.z += v.z; s4.w += v.w;
            }
            gemv_epilogue<FMT, EPI>(p, rb, g, t, s4, rm0, rm1);
        }
        par ^= 1;
    };
    for (int r = 0; r < nr; ++r) {
        acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
        for (int j = 0; j < per_row; ++j) stage(r * per_row + j, j * SU, SU);
        finish(rb0 + r);
    }
    if (threadIdx.x == 0) tl.mark();  // every row block done (thread 0's view)
    if (fail_i >= 0 && warp == 0 && lane == 0) {
        // A wait ran out: stages fail_i .. total - 1 may still be landing.
        // Give them a bounded chance before the CTA's shared memory goes away.
        for (int k = fail_i; k < total; ++k)
            if (!mbar_wait(&full[k % S], (uint32_t)(k / S) & 1u)) {
                record_device_error(p.err, kErrGemvDrain);
                break;
            }
    }
    AMCU_DIAG_TL(named_bar_sync(1, NT); if (threadIdx.x == 0) tl.done(1000u + 10u * EPI + (NC == kGemvConsumers ? 0u : 1u));)
}

// K split over a 2-CTA thread-block cluster, for activation rows too long to
// stage whole in one CTA (e.g. 8 rows of K = 14336: 229 KB of fp16). Cluster
// c owns row blocks [c * rb_per_cta, ...); CTA rank r of the cluster stages
// columns [r K/2, (r + 1) K/2) of every activation row and streams the
// matching half of each row block's groups, with the same unit, stage and
// staging code as gemv_tc_kernel. At a row block's end rank 1's reducing warp
// stores its partial tile (already multiplied by its rows' overflow-guard
// factors) into rank 0's shared memory and arrives on a rank-0 mbarrier (one
// per row block of the cluster, used once); rank 0's warp waits for it
// (bounded), adds the halves in rank order and applies the epilogue. The
// weight is streamed once, where row slices would stream it once per slice.
constexpr int kKs2MaxRb = 16;  // row blocks per cluster at most (partial slots)
constexpr int32_t kErrGemvClusterWait = 0x104;

__device__ __forceinline__ bool mbar_wait_acq_cluster(uint64_t* bar, uint32_t parity) {
    const long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile(
                "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
                " selp.u32 %0, 1, 0, p;\n}"
                : "=r"(ok)
                : "r"(smem_u32(bar)), "r"(parity)
                : "memory");
        if (ok) return true;
        if (clock64() - t0 > kSpinLimitCycles) return false;
    }
}

template <int FMT, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemvThreadsWide, 1) gemv_ks2_kernel(GemvParams p) {
    constexpr bool W4 = FMT == AMCU_WFMT_INT4;
    constexpr int UB = W4 ? kW4PairBytes : 2048;
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int S = p.stages, SU = p.stage_units;
    const int SBY = SU * UB;
    const int G = (int)(p.k / 128), GH = G / 2;  // groups of a row block; of this CTA's half
    const int64_t kh = (int64_t)GH * 128;
    const int M = (int)p.m;
    const int xrow = (int)(kh * 2 + kXPad);
    const GemvSmem L = gemv_smem<FMT, kGemvConsumersWide>(M, kh, SBY, S);
    float4* red = reinterpret_cast<float4*>(smem + L.red);
    float* sx = reinterpret_cast<float*>(smem + L.sx);
    uint8_t* xs = smem + L.xs;
    uint8_t* ring = smem + L.ring;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
    uint64_t* empty = full + S;
    __shared__ __align__(16) float4 peer_part[kKs2MaxRb][32];  // rank 0: rank 1's partial per row block
    __shared__ __align__(8) uint64_t peer_bar[kKs2MaxRb];

    const int nrb = (int)(p.n / 16);
    const int rb0 = (int)(blockIdx.x / 2) * p.rb_per_cta;
    const int nr = (rb0 + p.rb_per_cta < nrb ? rb0 + p.rb_per_cta : nrb) - rb0;
    const int per_row = GH / SU;
    const int total = nr * per_row;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kGemvConsumersWide);
        }
        for (int r = 0; r < kKs2MaxRb; ++r) mbar_init(&peer_bar[r], 1);
        fence_mbar_init();
        l2_prefetch_share(p.l2_next);
    }
    cluster.sync();  // rank 0's barriers exist before rank 1 can arrive on them

    if (warp == kGemvConsumersWide) {
        // this warp stays resident until the final cluster barrier: it lets
        // the next kernel launch like the consumers do
        pdl_trigger();
        if (lane == 0) {
            int slot = 0;
            uint32_t phase = 0;
            for (int i = 0; i < total; ++i) {
                if (i >= S && !mbar_wait(&empty[slot], phase ^ 1u)) {
                    record_device_error(p.err, kErrGemvEmptyWait);
                    break;
                }
                const int r = i / per_row, j = i - r * per_row;
                const uint8_t* src = static_cast<const uint8_t*>(p.w) +
                                     ((size_t)(rb0 + r) * G + (size_t)rank * GH + (size_t)j * SU) * UB;
                mbar_expect_tx(&full[slot], SBY);
                bulk_g2s_hint(ring + slot * SBY, src, SBY, &full[slot], gemv_weight_policy());
                if (++slot == S) {
                    slot = 0;
                    phase ^= 1;
                }
            }
        }
    } else {
        pdl_wait();
        pdl_trigger();
        __shared__ StageShared stsh;
        {
            StageCtx sc{static_cast<const __nv_bfloat16*>(p.x) + (int64_t)rank * kh, p.x_stride, kh, M, nullptr,
                        p.eps, xs, xrow, sx, &stsh, (int)threadIdx.x, kGemvConsumersWide * 32, 2};
            stage_activations<W4>(sc);
        }
        const float rm0 = 2 * t < M ? stsh.row_mul[2 * t] : 1.f, rm1 = 2 * t + 1 < M ? stsh.row_mul[2 * t + 1] : 1.f;
        const uint8_t* xrow_g = xs + (g < M ? g : 0) * xrow + 32 * t;
        float4* peer0 = cluster.map_shared_rank(&peer_part[0][0], 0);  // rank 0's slots
        uint32_t peer_bar0 = 0;  // shared::cluster address of rank 0's barrier 0
        asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(peer_bar0) : "r"(smem_u32(&peer_bar[0])));
        int slot = 0;
        uint32_t phase = 0;
        bool ok = true;
        int fail_i = -1, par = 0;
        float acc[4];
        for (int r = 0; r < nr; ++r) {
            acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
            for (int j = 0; j < per_row; ++j) {
                const int i = r * per_row + j;
                if (ok && !mbar_wait(&full[slot], phase)) {
                    ok = false;
                    fail_i = i;
                    if (lane == 0) record_device_error(p.err, kErrGemvFullWait);
                }
                gemv_stage<FMT, false, kGemvConsumersWide>(ring + slot * SBY, SU, xrow_g, sx, j * SU, warp, lane, g, t, acc);
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
                if (++slot == S) {
                    slot = 0;
                    phase ^= 1;
                }
            }
            red[(par * kGemvConsumersWide + warp) * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
            named_bar_sync(1, kGemvConsumersWide * 32);
            if (warp == r % kGemvConsumersWide) {
                float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int w = 0; w < kGemvConsumersWide; ++w) {
                    const float4 v = red[(par * kGemvConsumersWide + w) * 32 + lane];
                    s4.x += v.x; s4.y += v.y; s4.z += v.z; s4.w += v.w;
                }
                // this half's rows at their true scale (the guards may differ per half)
                s4.x *= rm0; s4.y *= rm1; s4.z *= rm0; s4.w *= rm1;
                if (rank == 1) {
                    peer0[r * 32 + lane] = s4;
                    __syncwarp();  // the warp's stores precede lane 0's release
                    if (lane == 0)
                        asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                                             peer_bar0 + (uint32_t)(r * sizeof(uint64_t)))
                                     : "memory");
                } else {
                    if (!mbar_wait_acq_cluster(&peer_bar[r], 0)) {
                        if (lane == 0) record_device_error(p.err, kErrGemvClusterWait);
                    }
                    const float4 o = peer_part[r][lane];
                    s4.x += o.x; s4.y += o.y; s4.z += o.z; s4.w += o.w;
                    gemv_epilogue<FMT, EPI>(p, rb0 + r, g, t, s4, 1.f, 1.f);
                }
            }
            par ^= 1;
        }
        if (fail_i >= 0 && warp == 0 && lane == 0)
            for (int k = fail_i; k < total; ++k)
                if (!mbar_wait(&full[k % S], (uint32_t)(k / S) & 1u)) {
                    record_device_error(p.err, kErrGemvDrain);
                    break;
                }
    }
    cluster.sync();  // rank 1's stores into rank 0 are done before either CTA leaves
}

template <int FMT>
static int stage_units(int64_t k, int cap_w4 = 0) {
    // group units per stage: the largest divisor of k/128 up to a cap (INT4:
    // 32 pair records = 33 KB, so a consumer warp takes 4 records between two
    // ring waits -- measured 2.8% faster decode than 16; INT8: 8 tile pairs =
    // 16 KB)
#ifndef GEMV_W4_SU_CAP
#define GEMV_W4_SU_CAP 32
#endif
    const int G = (int)(k / 128), cap = FMT == AMCU_WFMT_INT4 ? (cap_w4 > 0 ? cap_w4 : GEMV_W4_SU_CAP) : 8;
    int best = 1;
    for (int d = 1; d <= cap; ++d)
        if (G % d == 0) best = d;
    return best;
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
static void launch_gemv_variant(const GemvParams& q, int64_t grid, size_t smem, bool wide, cudaStream_t s) {
    constexpr int kMaxSmem = 224 * 1024;
    auto go = [&](auto kern, int nc) {
        set_func_attr_once((const void*)kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
        launch_pdl(kern, dim3((unsigned)grid), dim3((nc + 1) * 32), smem, s, q);
    };
    if (wide) {
        if (q.m == 1) go(gemv_tc_kernel<FMT, EPI, true, kGemvConsumersWide>, kGemvConsumersWide);
        else go(gemv_tc_kernel<FMT, EPI, false, kGemvConsumersWide>, kGemvConsumersWide);
    } else {
        if (q.m == 1) go(gemv_tc_kernel<FMT, EPI, true, kGemvConsumers>, kGemvConsumers);
        else go(gemv_tc_kernel<FMT, EPI, false, kGemvConsumers>, kGemvConsumers);
    }
}

// The 2-CTA K split (gemv_ks2_kernel) when the activation rows do not fit one
// CTA whole but their halves do; false when it does not apply.
template <int FMT, int EPI>
static bool launch_gemv_ks2(GemvParams p, cudaStream_t s) {
    if constexpr (EPI == kEpiResidualPeer) {
        return false;
    } else {
        constexpr int kMaxSmem = 224 * 1024;
        constexpr int kStatic = kKs2MaxRb * 32 * 16 + kKs2MaxRb * 8 + 1024;  // peer slots, barriers, staging state
        constexpr int UB = FMT == AMCU_WFMT_INT4 ? kW4PairBytes : 2048;
        const int64_t G = p.k / 128;
        if (G % 2 != 0 || p.norm_w != nullptr || p.m > kGemvMaxM) return false;
        const int64_t kh = G / 2 * 128;
        int su = 0, stages = 0;
        for (int cap : {0, 16, 8}) {
            su = stage_units<FMT>(kh, cap);
            stages = 8;
            while (stages > 2 && gemv_smem<FMT, kGemvConsumersWide>((int)p.m, kh, su * UB, stages).total + kStatic > kMaxSmem) --stages;
            if (gemv_smem<FMT, kGemvConsumersWide>((int)p.m, kh, su * UB, stages).total + kStatic <= kMaxSmem) break;
            stages = 0;
        }
        if (stages == 0) return false;
        const int64_t nrb = p.n / 16, clusters = num_sms() / 2;
        const int64_t per = (nrb + clusters - 1) / clusters;
        if (per > kKs2MaxRb) return false;
        p.stages = stages;
        p.stage_units = su;
        p.rb_per_cta = (int)per;
        const int64_t grid = 2 * ((nrb + per - 1) / per);
        const size_t smem = (size_t)gemv_smem<FMT, kGemvConsumersWide>((int)p.m, kh, su * UB, stages).total;
        // the largest dynamic size any call can ask for (set once per device)
        set_func_attr_once((const void*)gemv_ks2_kernel<FMT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kMaxSmem - kStatic);
        launch_pdl(gemv_ks2_kernel<FMT, EPI>, dim3((unsigned)grid), dim3(kGemvThreadsWide), smem, s, p);
        return true;
    }
}

template <int FMT, int EPI>
static void launch_gemv_one(GemvParams p, cudaStream_t s) {
    constexpr int kMaxSmem = 224 * 1024;
    const int smem_sm = smem_per_sm();
    constexpr int UB = FMT == AMCU_WFMT_INT4 ? kW4PairBytes : 2048;
    const int per_cta2 = smem_sm / GEMV_CPS - 2048;  // GEMV_CPS CTAs per SM (room for the per-CTA reserve)
    const int per_cta1 = kMaxSmem;                  // one CTA per SM
    // The activation rows are staged in shared memory; when the m rows of this
    // K do not fit beside a ring of two 16-record stages, they go in equal
    // slices (each slice streams W again).
    int64_t fit = p.m;
    while (fit > 1 && gemv_smem<FMT>((int)fit, p.k, stage_units<FMT>(p.k, 16) * UB, 2).total > per_cta1) --fit;
    if (fit < p.m && launch_gemv_ks2<FMT, EPI>(p, s)) return;  // halves of K instead of row slices
    {
        const int64_t slices = (p.m + fit - 1) / fit;
        fit = (p.m + slices - 1) / slices;
    }
    // Ring geometry for a slice of `rows`: GEMV_CPS (2) CTAs per SM, 16
    // consumer warps, while two full stages (32 INT4 records, the largest
    // divisor of k/128 up to 32) fit beside the staged rows; otherwise one CTA
    // per SM with a deeper ring (2..8 stages), because the two-CTA ring would
    // be two shallow stages and leave too few bytes in flight (8 rows: q/k/v
    // 12.1 -> 10.2 us, o 10.3 -> 8.9, gate/up 20.9 -> 19.6; the 70B down
    // projection, 57 KB of staged row: 32.4 -> 29.8; every shape that keeps
    // two full stages is faster with two CTAs). The grid is sized for the CTAs
    // resident at once, so no CTA waits for a second wave.
    auto plan = [&](int rows, int& su, int& stages, int& per_sm, bool& wide) {
        su = stage_units<FMT>(p.k);
        wide = false;
        // AMCU_GEMV_WIDE=1 forces one CTA of 16 consumer warps per SM for
        // every shape (a measurement switch: 8B batch-1 decode 545 against
        // 581 tok/s with the two-CTA geometry)
        static const bool force_wide = [] {
            const char* v = std::getenv("AMCU_GEMV_WIDE");
            return v && v[0] == '1';
        }();
        if (!force_wide && gemv_smem<FMT>(rows, p.k, su * UB, 2).total <= per_cta2) {
            stages = 8;
            while (stages > 2 && gemv_smem<FMT>(rows, p.k, su * UB, stages).total > per_cta2) --stages;
            per_sm = smem_sm / (gemv_smem<FMT>(rows, p.k, su * UB, stages).total + 1024);
            return;
        }
        if (gemv_smem<FMT, kGemvConsumersWide>(rows, p.k, su * UB, 2).total > per_cta1) su = stage_units<FMT>(p.k, 16);
        stages = 8;
        while (stages > 2 && gemv_smem<FMT, kGemvConsumersWide>(rows, p.k, su * UB, stages).total > per_cta1) --stages;
        per_sm = 1;
        wide = true;
    };
    const int64_t nrb = p.n / 16;
    for (int64_t m0 = 0; m0 < p.m; m0 += fit) {
        GemvParams q = p;
        q.m = p.m - m0 < fit ? p.m - m0 : fit;
        int su = 0, stages = 0, per_sm = 1;
        bool wide = false;
        plan((int)q.m, su, stages, per_sm, wide);
#ifdef GEMV_GRID_CPS
        if (per_sm > GEMV_GRID_CPS) per_sm = GEMV_GRID_CPS;
#endif
        q.stages = stages;
        q.stage_units = su;
        const int64_t max_ctas = (int64_t)(per_sm > 0 ? per_sm : 1) * num_sms();
        q.rb_per_cta = (int)((nrb + max_ctas - 1) / max_ctas);
        const int64_t grid = (nrb + q.rb_per_cta - 1) / q.rb_per_cta;
        q.x = static_cast<const __nv_bfloat16*>(p.x) + m0 * p.x_stride;
        q.y = static_cast<__nv_bfloat16*>(p.y) + m0 * p.y_stride;
        if (p.residual) q.residual = static_cast<const __nv_bfloat16*>(p.residual) + m0 * p.y_stride;
        // one CTA per SM: 16 consumer warps share its staged rows (the
        // unpack + MMA rate of 8 warps is about half of an SM's HBM share)
        const size_t smem = (size_t)(wide ? gemv_smem<FMT, kGemvConsumersWide>((int)q.m, p.k, su * UB, stages).total
                                          : gemv_smem<FMT>((int)q.m, p.k, su * UB, stages).total);
        launch_gemv_variant<FMT, EPI>(q, grid, smem, wide, s);
    }
}

template <int FMT>
static void launch_gemv_fmt(const GemvParams& p, int epi, cudaStream_t s) {
    switch (epi) {
        case AMCU_EPI_STORE: launch_gemv_one<FMT, AMCU_EPI_STORE>(p, s); break;
        case AMCU_EPI_RESIDUAL_ADD:
            if (p.fuse.world > 1) launch_gemv_one<FMT, kEpiResidualPeer>(p, s);
            else launch_gemv_one<FMT, AMCU_EPI_RESIDUAL_ADD>(p, s);
            break;
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

// INT4: one thread per 32-bit word of a tile or of a pair record's scales.
// Rows of the source part go to row blocks [rb0, rb0 + N/16) of the packed
// weight (a fused weight packs its parts one after another).
__global__ void pack_w4_kernel(const uint8_t* __restrict__ a, const uint8_t* __restrict__ b, const __half* sa,
                               const __half* sb, bool il, int64_t N, int64_t K, int64_t rb0,
                               uint32_t* __restrict__ out, bool unpack, uint8_t* __restrict__ canon_out,
                               __half* __restrict__ canon_s) {
    const int64_t G = K / 128;
    constexpr int kWords = kW4PairBytes / 4;  // 264: 2 x 128 tile words + 8 scale words
    const int64_t total = N / 16 * G * kWords;
    for (int64_t wi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; wi < total;
         wi += (int64_t)gridDim.x * blockDim.x) {
        const int64_t rec = wi / kWords;  // (row block, group) of the part
        const int in_rec = (int)(wi % kWords);
        const int64_t rb = rec / G, grp = rec % G;
        uint32_t* dst = out + ((rb0 + rb) * G + grp) * kWords + in_rec;
        if (in_rec >= 256) {  // scales: word s holds slots 2s, 2s+1 = rows s, s+8
            const int gg = in_rec - 256;
            const int64_t rlo = rb * 16 + gg, rhi = rlo + 8;
            if (!unpack) {
                int wl, wh;
                const int64_t slo = src_row(rlo, il, wl), shi = src_row(rhi, il, wh);
                const __half hl = (wl ? sb : sa)[slo * G + grp], hh = (wh ? sb : sa)[shi * G + grp];
                *dst = (uint32_t)__half_as_ushort(hl) | ((uint32_t)__half_as_ushort(hh) << 16);
            } else if (canon_s) {
                const uint32_t v = *dst;
                canon_s[rlo * G + grp] = __ushort_as_half((unsigned short)(v & 0xffffu));
                canon_s[rhi * G + grp] = __ushort_as_half((unsigned short)(v >> 16));
            }
            continue;
        }
        const int h = in_rec >> 7, in_tile = in_rec & 127;
        const int lane = in_tile >> 2, j = in_tile & 3;
        const int g = lane >> 2, t = lane & 3;
        const int64_t col0 = grp * 128 + h * 64 + 16 * t + 4 * j;
        // nibble p -> (row offset, column offset)
        const int prow[8] = {0, 8, 0, 8, 0, 8, 0, 8};
        const int pcol[8] = {0, 0, 2, 2, 1, 1, 3, 3};
        if (!unpack) {
            uint32_t word = 0;
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
            *dst = word;
        } else {
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

// INT8: one thread per 16-byte half-lane chunk.
__global__ void pack_w8_kernel(const int8_t* __restrict__ a, const int8_t* __restrict__ b, bool il, int64_t N,
                               int64_t K, int64_t rb0, uint4* __restrict__ out, bool unpack) {
    const int64_t chunks = N * K / 16;
    const int64_t C = K / 64;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < chunks; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t tile = i / 64;  // 1024 B per tile
        const int in_tile = (int)(i % 64);
        const int lane = in_tile >> 1, half = in_tile & 1;
        const int g = lane >> 2, t = lane & 3;
        const int64_t rb = tile / C, c = tile % C;
        const int64_t r_dev = rb * 16 + g + (half ? 8 : 0);
        const int64_t col = c * 64 + 16 * t;
        uint4* dst = out + ((rb0 + rb) * C + c) * 64 + in_tile;
        if (!unpack) {
            int which;
            const int64_t r = src_row(r_dev, il, which);
            *dst = *reinterpret_cast<const uint4*>((which ? b : a) + r * K + col);
        } else {
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
    (void)n_total;
    if (format == AMCU_WFMT_PLAIN) {
        uint8_t* dst = static_cast<uint8_t*>(qp) + row0 * k * plain_elt(dtype);
        if (!il) {
            cudaMemcpyAsync(dst, qa, (size_t)n * k * plain_elt(dtype), cudaMemcpyDeviceToDevice, s);
        } else {
            const int64_t hb = n / 2 * k * plain_elt(dtype);
            copy_bytes_kernel<<<pack_grid(2 * hb), 256, 0, s>>>((const uint8_t*)qa, (const uint8_t*)qb, hb, dst);
        }
    } else if (format == AMCU_WFMT_INT4) {
        const int64_t words = n / 16 * (k / 128) * (kW4PairBytes / 4);
        pack_w4_kernel<<<pack_grid(words), 256, 0, s>>>((const uint8_t*)qa, (const uint8_t*)qb, (const __half*)sa,
                                                        (const __half*)sb, il, n, k, row0 / 16, (uint32_t*)qp, false,
                                                        nullptr, nullptr);
    } else {
        pack_w8_kernel<<<pack_grid(n * k / 16), 256, 0, s>>>((const int8_t*)qa, (const int8_t*)qb, il, n, k, row0 / 16,
                                                            (uint4*)qp, false);
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
    if (format == AMCU_WFMT_INT8) return n * k;
    return n / 16 * (k / 128) * kW4PairBytes;  // weights and scales together
}

int64_t amcu_packed_scale_bytes(int32_t format, int64_t n, int64_t k, int64_t group) {
    (void)k;
    (void)group;
    if (format == AMCU_WFMT_INT8) return n * 4;
    return 0;  // INT4 scales live inside the packed weight
}

am_status_code amcu_prepack_weight(int32_t format, int32_t dtype, int64_t n, int64_t k, int64_t group,
                                   const void* q, const void* sc, void* qp, void* sp, void* stream) {
    clear_error();
    am_status_code st = check_weight_shape(format, dtype, n, k, group);
    if (st != AM_STATUS_OK) return st;
    AMCU_REQUIRE(q && qp, "amcu_prepack_weight: null pointer");
    AMCU_REQUIRE(format == AMCU_WFMT_PLAIN || sc, "amcu_prepack_weight: null scale pointer");
    AMCU_REQUIRE(format != AMCU_WFMT_INT8 || sp, "amcu_prepack_weight: null packed scale pointer");
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
    AMCU_REQUIRE(format == AMCU_WFMT_PLAIN || sc, "amcu_prepack_weight_rows: null scale pointer");
    AMCU_REQUIRE(format != AMCU_WFMT_INT8 || sp, "amcu_prepack_weight_rows: null packed scale pointer");
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
    AMCU_REQUIRE(format == AMCU_WFMT_PLAIN || (gs && us), "amcu_prepack_gate_up: null scale pointer");
    AMCU_REQUIRE(format != AMCU_WFMT_INT8 || sp, "amcu_prepack_gate_up: null packed scale pointer");
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
    } else if (format == AMCU_WFMT_INT4) {
        (void)sp;
        pack_w4_kernel<<<pack_grid(n / 16 * (k / 128) * (kW4PairBytes / 4)), 256, 0, s>>>(
                nullptr, nullptr, nullptr, nullptr, false, n, k, 0, (uint32_t*)const_cast<void*>(qp), true,
                (uint8_t*)q, (__half*)sc);
    } else {
        pack_w8_kernel<<<pack_grid(n * k / 16), 256, 0, s>>>((const int8_t*)q, nullptr, false, n, k, 0,
                                                            (uint4*)const_cast<void*>(qp), true);
        if (sc && sp) cudaMemcpyAsync(sc, sp, (size_t)n * 4, cudaMemcpyDeviceToDevice, s);
    }
    return check_launch("amcu_unpack_weight");
}

}  // extern "C"

#ifdef AMCU_DIAG
// Diagnostics: the GEMV launch timeline (see diag_timeline.cuh).
extern "C" __attribute__((visibility("default"))) int amcu_diag_timeline_gemv(void* out, int max) { return amcu::diag_timeline_take(out, max); }
#endif
