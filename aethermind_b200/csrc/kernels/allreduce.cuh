// One-shot all-reduce + residual add over peer memory (tensor-parallel decode).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace amcu {

constexpr int kArMaxRanks = 8;
constexpr int kArChunk = 4096;                        // elements per CTA (fixed ranges)
constexpr int kArMaxCtas = 16;
constexpr int64_t kArMaxElems = (int64_t)kArChunk * kArMaxCtas;  // largest one-shot message

struct ArParams {
    const void* part;               // this rank's bf16 partial [n]
    void* x;                        // bf16 residual [n], updated in place
    int64_t n;
    int rank, world;
    uint8_t* area[kArMaxRanks];     // every rank's exchange area as mapped in this process (own included)
    int32_t* err;
    uint64_t wait_ns;               // bound of the wait for the peers' chunks (0: about 2 s)
};

// The GEMV epilogue's all-reduce (decode o/down over peer memory): fp32
// partials of up to kFuseMaxVals outputs (n rows x m <= 8 activation rows),
// one flag and epoch per row block. Placed after the one-shot region of the
// same exchange area.
constexpr int64_t kFuseMaxVals = (int64_t)16384 * 8;
constexpr int kFuseMaxRb = 1024;
__host__ __device__ inline size_t ar_fuse_base() {
    return (size_t)2 * kArMaxRanks * kArMaxElems * 2 + (size_t)kArMaxRanks * kArMaxCtas * 4 + (size_t)kArMaxCtas * 4;
}
__host__ __device__ inline size_t ar_fuse_mail_offset(int parity, int src, int64_t i) {
    return ar_fuse_base() + (((size_t)parity * kArMaxRanks + src) * kFuseMaxVals + (size_t)i) * 4;
}
__host__ __device__ inline size_t ar_fuse_flags_offset() {
    return ar_fuse_base() + (size_t)2 * kArMaxRanks * kFuseMaxVals * 4;
}
__host__ __device__ inline size_t ar_fuse_epochs_offset() {
    return ar_fuse_flags_offset() + (size_t)kArMaxRanks * kFuseMaxRb * 4;
}
size_t ar_area_bytes();
bool ar_oneshot_supported(int64_t n, int world);
void launch_ar_oneshot_add(const ArParams& p, cudaStream_t s);

}  // namespace amcu
