// Host-visible launch interface of the GEMV / GEMM kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "aethermind_b200.h"

namespace amcu {

constexpr int kGemvConsumers = 8;                     // consumer warps per GEMV CTA
constexpr int kGemvThreads = (kGemvConsumers + 1) * 32;  // + one producer warp
constexpr int kGemvConsumersWide = 16;               // consumer warps of a one-CTA-per-SM GEMV
constexpr int kGemvThreadsWide = (kGemvConsumersWide + 1) * 32;
constexpr int kGemvMaxM = 8;
constexpr int kW4PairBytes = 2 * 512 + 32;  // INT4 pair record: two tiles + 16 fp16 scales

struct GemvParams {
    const void* x;
    const void* w;
    const void* scales;  // INT8 only (INT4 scales live in the pair records)
    void* y;
    const void* residual;
    int64_t m, n, k;
    int64_t x_stride, y_stride;
    int32_t* err;        // device error word for bounded waits
    const void* norm_w;  // optional fused RMSNorm weight [k] (bf16)
    float eps;
    int rb_per_cta;      // set by the launcher
    int stages;          // shared-memory ring stages (set by the launcher)
    int stage_units;     // 128-column group units per stage (set by the launcher)
    AmcuL2Prefetch l2_next;  // ranges the next operation reads (hint)
    // Tensor-parallel RESIDUAL_ADD: partials summed over the ranks in the
    // epilogue (world 0 = off); every rank's exchange area as mapped here.
    struct {
        uint8_t* area[8];
        int rank, world;
        uint64_t wait_ns;
    } fuse;
};

// Quantized (INT4 / INT8 tile16x64) GEMV, m <= kGemvMaxM, bf16 activations.
void launch_gemv(const GemvParams& p, int fmt, int epi, cudaStream_t s);
// Plain weights in the activation dtype, any m.
void launch_gemm_plain(const GemvParams& p, int dtype, int epi, cudaStream_t s);

}  // namespace amcu
