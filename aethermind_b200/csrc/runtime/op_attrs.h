// Per-op attribute PODs carried in KernelContext::attrs (the reference passes
// e.g. RMSNorm eps the same way, src/operators/rmsnorm_op.cpp:26-27).
#pragma once
#include <cstdint>

namespace aethermind {

struct RmsNormAttrs {
    float eps;
};
struct LinearAttrs {
    int32_t epilogue;                  // amcu_epilogue
    const void* norm_weight = nullptr;  // fused RMSNorm of the input (decode GEMV)
    float norm_eps = 0.f;
    const AmcuAllReduceArgs* peer_reduce = nullptr;  // tensor-parallel o/down: ranks summed in the epilogue
};
struct RopeKvAttrs {
    double theta;
    int64_t rows_per_seq, capacity, slot_stride, n_q, n_kv, head_dim;
    const int32_t* seq_pos;
    int32_t* status;
    const float* cos_sin = nullptr;  // precomputed table (amcu_rope_table)
};
struct AttentionAttrs {
    int64_t rows_per_seq, capacity, slot_stride, n_q, n_kv, head_dim, max_context;
    const int32_t* seq_pos;
    int32_t num_splits;
};
struct RopeAttentionAttrs {
    RopeKvAttrs rope;
    AttentionAttrs attn;
};
struct EmbeddingAttrs {
    const float* row_scales;
    int32_t* status;
};
struct ArgmaxAttrs {
    float* gap_out;
};

}  // namespace aethermind
