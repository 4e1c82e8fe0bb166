// Host-visible launch interface of the GEMV / GEMM kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace amcu {

constexpr int kGemvThreads = 256;
constexpr int kGemvMaxM = 8;

struct GemvParams {
    const void* x;
    const void* w;
    const void* scales;
    void* y;
    const void* residual;
    int64_t m, n, k;
    int64_t x_stride, y_stride;
    int32_t* err;     // device error word for bounded waits
    const void* norm_w;  // optional fused RMSNorm weight [k] (bf16)
    float eps;
    int rb_per_cta;   // set by the launcher
};

// Quantized (INT4 / INT8 tile16x64) GEMV, m <= kGemvMaxM, bf16 activations.
void launch_gemv(const GemvParams& p, int fmt, int epi, cudaStream_t s);
// Plain weights in the activation dtype, any m.
void launch_gemm_plain(const GemvParams& p, int dtype, int epi, cudaStream_t s);

}  // namespace amcu
