#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace amcu {
// out[b][counter] = next[b]; seq_pos[b] = set_pos (>= 0) or seq_pos[b] + 1; ++counter.
void launch_advance(const int64_t* next, const float* gap, int64_t* out, float* gaps_out, int64_t out_cap,
                    int32_t* seq_pos, int32_t* counter, int64_t batch, int32_t set_pos, cudaStream_t s);
}  // namespace amcu
