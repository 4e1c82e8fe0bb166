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

size_t ar_area_bytes();
bool ar_oneshot_supported(int64_t n, int world);
void launch_ar_oneshot_add(const ArParams& p, cudaStream_t s);

}  // namespace amcu
