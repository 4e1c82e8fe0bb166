// Prefill dequant GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "aethermind_b200.h"

namespace amcu {

struct GemmTcParams {
    const void* x;
    const void* w;
    const void* scales;
    void* y;
    const void* residual;
    int64_t m, n, k;
    int64_t x_stride, y_stride;
    void* workspace;
    size_t workspace_size;
};

bool gemm_tc_supported(const GemmTcParams& p, int fmt);
size_t gemm_tc_workspace_bytes(const GemmTcParams& p, int fmt);
am_status_code launch_gemm_tc(const GemmTcParams& p, int fmt, int epi, cudaStream_t s);

}  // namespace amcu
