// Device-side bookkeeping of the greedy decode loop, so a captured decode step
// can be replayed without any host round trip: after the argmax of step i the
// chosen token of every sequence is appended to the output buffer, its logit
// gap is recorded, and the sequence position advances.
#include "../amcu_internal.h"
#include "common.cuh"
#include "decode_state.cuh"

namespace amcu {

__global__ void advance_kernel(const int64_t* __restrict__ next, const float* __restrict__ gap, int64_t* out,
                               float* gaps_out, int64_t out_cap, int32_t* seq_pos, int32_t* counter,
                               int64_t batch, int32_t set_pos) {
    pdl_wait();
    pdl_trigger();
    const int idx = *counter;
    for (int64_t b = threadIdx.x; b < batch; b += blockDim.x) {
        if (idx < out_cap) {
            out[b * out_cap + idx] = next[b];
            if (gaps_out && gap) gaps_out[b * out_cap + idx] = gap[b];
        }
        seq_pos[b] = set_pos >= 0 ? set_pos : seq_pos[b] + 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) *counter = idx + 1;
}

void launch_advance(const int64_t* next, const float* gap, int64_t* out, float* gaps_out, int64_t out_cap,
                    int32_t* seq_pos, int32_t* counter, int64_t batch, int32_t set_pos, cudaStream_t s) {
    launch_pdl(advance_kernel, dim3(1), dim3(256), 0, s, next, gap, out, gaps_out, out_cap, seq_pos, counter, batch, set_pos);
}

}  // namespace amcu
