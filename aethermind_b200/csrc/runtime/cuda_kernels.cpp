// CUDA kernel registrations: one AM_REGISTER_KERNEL per (op, selector), each a
// thin KernelFunc over the amcu_* C ABI plus the KernelParamsBuilder that turns
// the step's tensor views into the launcher's argument struct (the pattern of
// src/backend/cpu/kernels/rmsnorm/rmsnorm_entry.cpp:146-227).
//
// Fused steps of the Llama plan (reference op -> registered CUDA op):
//   Add + RMSNorm          -> kRmsNorm with a residual input
//   q/k/v Linear           -> one kLinear over the concatenated [q;k;v] weight
//   RoPE + KVCacheUpdate   -> kRoPE (rotates q, writes rotated k and v to the cache)
//   RoPE + KVCacheUpdate + Attention (decode, bf16)
//                          -> kRoPEAttention (one launch, rotated q stays on chip)
//   every decoder layer of a bs <= 2 INT4 decode step
//                          -> kDecodeStack (one persistent cooperative launch)
//   o Linear + Add         -> kLinear with the residual-add epilogue
//   gate/up Linear+SiluMul -> kLinear over the interleaved gate/up weight (SiLU-Mul epilogue)
//   down Linear + Add      -> kLinear with the residual-add epilogue
#include <cstring>
#include <new>

#include "runtime/dispatch.h"
#include "runtime/op_attrs.h"

namespace aethermind {
namespace {

cudaStream_t S(const KernelContext& c) { return c.stream ? c.stream->handle() : nullptr; }
Status FromAm(am_status_code c) { return Status::FromAm(c, amcu_last_error()); }

int32_t AmDtype(DType d) {
    switch (d) {
        case DType::kF32: return AMCU_F32;
        case DType::kBF16: return AMCU_BF16;
        case DType::kI32: return AMCU_I32;
        case DType::kI64: return AMCU_I64;
        case DType::kU32: return AMCU_U32;
        default: return -1;
    }
}

template <typename A>
const A* Attrs(std::span<const std::byte> attrs) {
    return attrs.size() >= sizeof(A) ? reinterpret_cast<const A*>(attrs.data()) : nullptr;
}

// ---- RMSNorm ----
Status BuildRmsNorm(std::span<const TensorView> in, std::span<const MutableTensorView> out,
                    std::span<const std::byte> attrs, const void*, void* buf) noexcept {
    if (in.size() < 2 || out.empty()) return Status::InvalidArgument("RmsNorm expects (x, w[, residual]) -> (y[, h])");
    const auto* at = Attrs<RmsNormAttrs>(attrs);
    if (!at) return Status::InvalidArgument("RmsNorm attrs missing");
    auto* a = new (buf) AmcuRmsNormArgs{};
    a->input = in[0].data;
    a->weight = in[1].data;
    a->output = out[0].mutable_data();
    a->rows = in[0].dim(0);
    a->hidden = in[0].dim(1);
    a->input_row_stride = in[0].strides[0];
    a->output_row_stride = out[0].strides[0];
    a->eps = at->eps;
    a->dtype = AmDtype(in[0].dtype);
    if (in.size() > 2) {
        if (out.size() < 2) return Status::InvalidArgument("RmsNorm with residual needs a residual output");
        a->residual = in[2].data;
        a->residual_out = out[1].mutable_data();
    }
    return Status::Ok();
}
Status RmsNormFn(const KernelContext& c) noexcept {
    return FromAm(amcu_rmsnorm(static_cast<const AmcuRmsNormArgs*>(c.kernel_params), S(c)));
}

// ---- Linear ----
Status BuildLinear(std::span<const TensorView> in, std::span<const MutableTensorView> out,
                   std::span<const std::byte> attrs, const void* packed, void* buf) noexcept {
    if (in.empty() || out.empty() || !packed) return Status::InvalidArgument("Linear expects x, packed weight -> y");
    const auto* at = Attrs<LinearAttrs>(attrs);
    auto* a = new (buf) AmcuLinearArgs{};
    a->x = in[0].data;
    a->w = *static_cast<const AmcuWeight*>(packed);
    a->y = out[0].mutable_data();
    a->m = in[0].dim(0);
    a->x_stride = in[0].strides[0];
    a->y_stride = out[0].strides[0];
    a->act_dtype = AmDtype(in[0].dtype);
    a->epilogue = at ? at->epilogue : AMCU_EPI_STORE;
    if (at) {
        a->norm_weight = at->norm_weight;
        a->norm_eps = at->norm_eps;
        a->peer_reduce = at->peer_reduce;
    }
    if (in.size() > 1) a->residual = in[1].data;
    return Status::Ok();
}
Status LinearFn(const KernelContext& c) noexcept {
    AmcuLinearArgs a = *static_cast<const AmcuLinearArgs*>(c.kernel_params);
    a.workspace = c.workspace_binding.data;
    a.workspace_size = c.workspace_binding.size;
    return FromAm(amcu_linear(&a, S(c)));
}
Status GemvW4Fn(const KernelContext& c) noexcept {
    return FromAm(amcu_gemv_w4g128(static_cast<const AmcuLinearArgs*>(c.kernel_params), S(c)));
}
Status GemvW8Fn(const KernelContext& c) noexcept {
    return FromAm(amcu_gemv_w8(static_cast<const AmcuLinearArgs*>(c.kernel_params), S(c)));
}
Status GemmW4Fn(const KernelContext& c) noexcept {
    AmcuLinearArgs a = *static_cast<const AmcuLinearArgs*>(c.kernel_params);
    a.workspace = c.workspace_binding.data;
    a.workspace_size = c.workspace_binding.size;
    return FromAm(amcu_gemm_w4g128_prefill(&a, S(c)));
}
Status GemmW8Fn(const KernelContext& c) noexcept {
    AmcuLinearArgs a = *static_cast<const AmcuLinearArgs*>(c.kernel_params);
    a.workspace = c.workspace_binding.data;
    a.workspace_size = c.workspace_binding.size;
    return FromAm(amcu_gemm_w8_prefill(&a, S(c)));
}

// ---- RoPE + KV write ----
Status BuildRopeKv(std::span<const TensorView> in, std::span<const MutableTensorView> out,
                   std::span<const std::byte> attrs, const void*, void* buf) noexcept {
    if (in.size() < 3 || out.size() < 3) return Status::InvalidArgument("RoPE expects (q, k, v) -> (q, k_cache, v_cache)");
    const auto* at = Attrs<RopeKvAttrs>(attrs);
    if (!at) return Status::InvalidArgument("RoPE attrs missing");
    auto* a = new (buf) AmcuRopeKvArgs{};
    a->q = out[0].mutable_data();
    a->k = in[1].data;
    a->v = in[2].data;
    a->q_stride = in[0].strides[0];
    a->k_stride = in[1].strides[0];
    a->v_stride = in[2].strides[0];
    a->k_cache = out[1].mutable_data();
    a->v_cache = out[2].mutable_data();
    a->slot_stride = at->slot_stride;
    a->capacity = at->capacity;
    a->seq_pos = at->seq_pos;
    a->rows = in[0].dim(0);
    a->rows_per_seq = at->rows_per_seq;
    a->n_q_heads = at->n_q;
    a->n_kv_heads = at->n_kv;
    a->head_dim = at->head_dim;
    a->theta = at->theta;
    a->dtype = AmDtype(in[0].dtype);
    a->status = at->status;
    a->cos_sin = at->cos_sin;
    return Status::Ok();
}
Status RopeKvFn(const KernelContext& c) noexcept {
    return FromAm(amcu_rope_kv_write(static_cast<const AmcuRopeKvArgs*>(c.kernel_params), S(c)));
}

// ---- Attention ----
Status BuildAttention(std::span<const TensorView> in, std::span<const MutableTensorView> out,
                      std::span<const std::byte> attrs, const void*, void* buf) noexcept {
    if (in.size() < 3 || out.empty()) return Status::InvalidArgument("Attention expects (q, k_cache, v_cache) -> o");
    const auto* at = Attrs<AttentionAttrs>(attrs);
    if (!at) return Status::InvalidArgument("Attention attrs missing");
    auto* a = new (buf) AmcuAttentionArgs{};
    a->q = in[0].data;
    a->q_stride = in[0].strides[0];
    a->k_cache = in[1].data;
    a->v_cache = in[2].data;
    a->slot_stride = at->slot_stride;
    a->capacity = at->capacity;
    a->seq_pos = at->seq_pos;
    a->out = out[0].mutable_data();
    a->out_stride = out[0].strides[0];
    a->rows = in[0].dim(0);
    a->rows_per_seq = at->rows_per_seq;
    a->n_q_heads = at->n_q;
    a->n_kv_heads = at->n_kv;
    a->head_dim = at->head_dim;
    a->dtype = AmDtype(in[0].dtype);
    a->num_splits = at->num_splits;
    a->max_context = at->max_context;
    return Status::Ok();
}
Status AttnDecodeFn(const KernelContext& c) noexcept {
    AmcuAttentionArgs a = *static_cast<const AmcuAttentionArgs*>(c.kernel_params);
    a.workspace = c.workspace_binding.data;
    a.workspace_size = c.workspace_binding.size;
    return FromAm(amcu_attn_decode(&a, S(c)));
}
Status AttnPrefillFn(const KernelContext& c) noexcept {
    AmcuAttentionArgs a = *static_cast<const AmcuAttentionArgs*>(c.kernel_params);
    a.workspace = c.workspace_binding.data;
    a.workspace_size = c.workspace_binding.size;
    return FromAm(amcu_attn_prefill(&a, S(c)));
}

// ---- fused decode RoPE + KV append + attention ----
struct RopeAttnArgs {
    AmcuRopeKvArgs rope;
    AmcuAttentionArgs attn;
};
// in: (q, k, v, k_cache, v_cache); out: (o, k_cache, v_cache)
Status BuildRopeAttention(std::span<const TensorView> in, std::span<const MutableTensorView> out,
                          std::span<const std::byte> attrs, const void*, void* buf) noexcept {
    if (in.size() < 5 || out.size() < 3)
        return Status::InvalidArgument("RoPEAttention expects (q, k, v, k_cache, v_cache) -> (o, k_cache, v_cache)");
    const auto* at = Attrs<RopeAttentionAttrs>(attrs);
    if (!at) return Status::InvalidArgument("RoPEAttention attrs missing");
    auto* a = new (buf) RopeAttnArgs{};
    AmcuRopeKvArgs& r = a->rope;
    r.q = const_cast<void*>(in[0].data);
    r.k = in[1].data;
    r.v = in[2].data;
    r.q_stride = in[0].strides[0];
    r.k_stride = in[1].strides[0];
    r.v_stride = in[2].strides[0];
    r.k_cache = out[1].mutable_data();
    r.v_cache = out[2].mutable_data();
    r.slot_stride = at->rope.slot_stride;
    r.capacity = at->rope.capacity;
    r.seq_pos = at->rope.seq_pos;
    r.rows = in[0].dim(0);
    r.rows_per_seq = at->rope.rows_per_seq;
    r.n_q_heads = at->rope.n_q;
    r.n_kv_heads = at->rope.n_kv;
    r.head_dim = at->rope.head_dim;
    r.theta = at->rope.theta;
    r.dtype = AmDtype(in[0].dtype);
    r.status = at->rope.status;
    r.cos_sin = at->rope.cos_sin;
    AmcuAttentionArgs& t = a->attn;
    t.q = in[0].data;
    t.q_stride = in[0].strides[0];
    t.k_cache = out[1].mutable_data();
    t.v_cache = out[2].mutable_data();
    t.slot_stride = at->attn.slot_stride;
    t.capacity = at->attn.capacity;
    t.seq_pos = at->attn.seq_pos;
    t.out = out[0].mutable_data();
    t.out_stride = out[0].strides[0];
    t.rows = in[0].dim(0);
    t.rows_per_seq = at->attn.rows_per_seq;
    t.n_q_heads = at->attn.n_q;
    t.n_kv_heads = at->attn.n_kv;
    t.head_dim = at->attn.head_dim;
    t.dtype = AmDtype(in[0].dtype);
    t.max_context = at->attn.max_context;
    return Status::Ok();
}
Status RopeAttnFn(const KernelContext& c) noexcept {
    const auto* a = static_cast<const RopeAttnArgs*>(c.kernel_params);
    return FromAm(amcu_attn_decode_rope(&a->rope, &a->attn, S(c)));
}

// ---- persistent decode step (attrs: the complete AmcuDecodeStackArgs) ----
Status BuildDecodeStack(std::span<const TensorView>, std::span<const MutableTensorView>,
                        std::span<const std::byte> attrs, const void*, void* buf) noexcept {
    if (attrs.size() != sizeof(AmcuDecodeStackArgs)) return Status::InvalidArgument("DecodeStack attrs missing");
    std::memcpy(buf, attrs.data(), sizeof(AmcuDecodeStackArgs));
    return Status::Ok();
}
Status DecodeStackFn(const KernelContext& c) noexcept {
    return FromAm(amcu_decode_stack(static_cast<const AmcuDecodeStackArgs*>(c.kernel_params), S(c)));
}

// ---- elementwise ----
struct BinaryArgs {
    const void* a;
    const void* b;
    void* out;
    int64_t count;
    int32_t dtype;
};
Status BuildBinary(std::span<const TensorView> in, std::span<const MutableTensorView> out,
                   std::span<const std::byte>, const void*, void* buf) noexcept {
    if (in.size() < 2 || out.empty()) return Status::InvalidArgument("binary op expects (a, b) -> out");
    int64_t n = 1;
    for (int i = 0; i < in[0].ndim; ++i) n *= in[0].shape[i];
    new (buf) BinaryArgs{in[0].data, in[1].data, out[0].mutable_data(), n, AmDtype(in[0].dtype)};
    return Status::Ok();
}
Status SiluMulFn(const KernelContext& c) noexcept {
    auto* a = static_cast<const BinaryArgs*>(c.kernel_params);
    return FromAm(amcu_silu_mul(a->a, a->b, a->out, a->count, a->dtype, S(c)));
}
Status AddFn(const KernelContext& c) noexcept {
    auto* a = static_cast<const BinaryArgs*>(c.kernel_params);
    return FromAm(amcu_add(a->a, a->b, a->out, a->count, a->dtype, S(c)));
}

// ---- Embedding ----
Status BuildEmbedding(std::span<const TensorView> in, std::span<const MutableTensorView> out,
                      std::span<const std::byte> attrs, const void*, void* buf) noexcept {
    if (in.size() < 2 || out.empty()) return Status::InvalidArgument("Embedding expects (ids, table) -> out");
    const auto* at = Attrs<EmbeddingAttrs>(attrs);
    auto* a = new (buf) AmcuEmbeddingArgs{};
    a->ids = in[0].data;
    a->id_dtype = AmDtype(in[0].dtype);
    a->count = in[0].dim(0);
    a->table = in[1].data;
    a->vocab = in[1].dim(0);
    a->hidden = in[1].dim(1);
    a->out = out[0].mutable_data();
    a->dtype = AmDtype(out[0].dtype);
    if (at) {
        a->row_scales = at->row_scales;
        a->status = at->status;
    }
    return Status::Ok();
}
Status EmbeddingFn(const KernelContext& c) noexcept {
    return FromAm(amcu_embedding(static_cast<const AmcuEmbeddingArgs*>(c.kernel_params), S(c)));
}

// ---- Argmax ----
struct ArgmaxArgs {
    const void* logits;
    int64_t rows, vocab, stride;
    int32_t dtype;
    int64_t* out;
    float* gap;
};
Status BuildArgmax(std::span<const TensorView> in, std::span<const MutableTensorView> out,
                   std::span<const std::byte> attrs, const void*, void* buf) noexcept {
    if (in.empty() || out.empty()) return Status::InvalidArgument("Argmax expects logits -> index");
    const auto* at = Attrs<ArgmaxAttrs>(attrs);
    new (buf) ArgmaxArgs{in[0].data, in[0].dim(0), in[0].dim(1), in[0].strides[0], AmDtype(in[0].dtype),
                         static_cast<int64_t*>(out[0].mutable_data()), at ? at->gap_out : nullptr};
    return Status::Ok();
}
Status ArgmaxFn(const KernelContext& c) noexcept {
    auto* a = static_cast<const ArgmaxArgs*>(c.kernel_params);
    if (c.workspace_binding.data)
        return FromAm(amcu_argmax_ws(a->logits, a->rows, a->vocab, a->stride, a->dtype, a->out, a->gap,
                                     c.workspace_binding.data, c.workspace_binding.size, S(c)));
    return FromAm(amcu_argmax(a->logits, a->rows, a->vocab, a->stride, a->dtype, a->out, a->gap, S(c)));
}

constexpr DeviceType kCU = DeviceType::kCUDA;

}  // namespace

// Registrations ------------------------------------------------------------
#define AM_SEL(act, wdt, fmt, phase) \
    KernelSelector { kCU, DType::act, DType::wdt, WeightFormat::fmt, IsaLevel::kScalar, ExecPhase::phase }

AM_REGISTER_KERNEL(RmsNorm_CUDA_F32, KernelDescriptor{OpType::kRmsNorm, AM_SEL(kF32, kF32, kPlain, kBoth), RmsNormFn,
                                                      "RmsNorm_CUDA_F32", 0, BuildRmsNorm, sizeof(AmcuRmsNormArgs)})
AM_REGISTER_KERNEL(RmsNorm_CUDA_BF16, KernelDescriptor{OpType::kRmsNorm, AM_SEL(kBF16, kBF16, kPlain, kBoth), RmsNormFn,
                                                       "RmsNorm_CUDA_BF16", 0, BuildRmsNorm, sizeof(AmcuRmsNormArgs)})

AM_REGISTER_KERNEL(Linear_CUDA_F32_Plain, KernelDescriptor{OpType::kLinear, AM_SEL(kF32, kF32, kPlain, kBoth), LinearFn,
                                                           "Linear_CUDA_F32_Plain", 0, BuildLinear, sizeof(AmcuLinearArgs)})
AM_REGISTER_KERNEL(Linear_CUDA_BF16_Plain, KernelDescriptor{OpType::kLinear, AM_SEL(kBF16, kBF16, kPlain, kBoth), LinearFn,
                                                            "Linear_CUDA_BF16_Plain", 0, BuildLinear, sizeof(AmcuLinearArgs)})
AM_REGISTER_KERNEL(Linear_CUDA_W4_Decode, KernelDescriptor{OpType::kLinear, AM_SEL(kBF16, kI4, kQuantizedInt4, kDecode),
                                                           GemvW4Fn, "GemvW4G128_CUDA_Decode", 1, BuildLinear,
                                                           sizeof(AmcuLinearArgs)})
AM_REGISTER_KERNEL(Linear_CUDA_W4_Prefill, KernelDescriptor{OpType::kLinear, AM_SEL(kBF16, kI4, kQuantizedInt4, kPrefill),
                                                            GemmW4Fn, "GemmW4G128_CUDA_Prefill", 1, BuildLinear,
                                                            sizeof(AmcuLinearArgs)})
AM_REGISTER_KERNEL(Linear_CUDA_W8_Decode, KernelDescriptor{OpType::kLinear, AM_SEL(kBF16, kI8, kQuantizedInt8, kDecode),
                                                           GemvW8Fn, "GemvW8_CUDA_Decode", 1, BuildLinear,
                                                           sizeof(AmcuLinearArgs)})
AM_REGISTER_KERNEL(Linear_CUDA_W8_Prefill, KernelDescriptor{OpType::kLinear, AM_SEL(kBF16, kI8, kQuantizedInt8, kPrefill),
                                                            GemmW8Fn, "GemmW8_CUDA_Prefill", 1, BuildLinear,
                                                            sizeof(AmcuLinearArgs)})

AM_REGISTER_KERNEL(RoPEKV_CUDA_F32, KernelDescriptor{OpType::kRoPE, AM_SEL(kF32, kF32, kPlain, kBoth), RopeKvFn,
                                                     "RoPEKVWrite_CUDA_F32", 0, BuildRopeKv, sizeof(AmcuRopeKvArgs)})
AM_REGISTER_KERNEL(RoPEKV_CUDA_BF16, KernelDescriptor{OpType::kRoPE, AM_SEL(kBF16, kBF16, kPlain, kBoth), RopeKvFn,
                                                      "RoPEKVWrite_CUDA_BF16", 0, BuildRopeKv, sizeof(AmcuRopeKvArgs)})

AM_REGISTER_KERNEL(Attn_CUDA_F32_Decode, KernelDescriptor{OpType::kAttention, AM_SEL(kF32, kF32, kPlain, kDecode),
                                                          AttnDecodeFn, "AttnDecodeSplitK_CUDA_F32", 0, BuildAttention,
                                                          sizeof(AmcuAttentionArgs)})
AM_REGISTER_KERNEL(Attn_CUDA_BF16_Decode, KernelDescriptor{OpType::kAttention, AM_SEL(kBF16, kBF16, kPlain, kDecode),
                                                           AttnDecodeFn, "AttnDecodeSplitK_CUDA_BF16", 0, BuildAttention,
                                                           sizeof(AmcuAttentionArgs)})
AM_REGISTER_KERNEL(Attn_CUDA_F32_Prefill, KernelDescriptor{OpType::kAttention, AM_SEL(kF32, kF32, kPlain, kPrefill),
                                                           AttnPrefillFn, "AttnPrefill_CUDA_F32", 0, BuildAttention,
                                                           sizeof(AmcuAttentionArgs)})
AM_REGISTER_KERNEL(Attn_CUDA_BF16_Prefill, KernelDescriptor{OpType::kAttention, AM_SEL(kBF16, kBF16, kPlain, kPrefill),
                                                            AttnPrefillFn, "AttnPrefill_CUDA_BF16", 0, BuildAttention,
                                                            sizeof(AmcuAttentionArgs)})

AM_REGISTER_KERNEL(RoPEAttn_CUDA_BF16_Decode,
                   KernelDescriptor{OpType::kRoPEAttention, AM_SEL(kBF16, kBF16, kPlain, kDecode), RopeAttnFn,
                                    "RoPEAttnDecodeCluster_CUDA_BF16", 0, BuildRopeAttention, sizeof(RopeAttnArgs)})

AM_REGISTER_KERNEL(DecodeStack_CUDA_W4,
                   KernelDescriptor{OpType::kDecodeStack, AM_SEL(kBF16, kI4, kQuantizedInt4, kDecode), DecodeStackFn,
                                    "DecodeStackPersistent_CUDA_W4", 0, BuildDecodeStack, sizeof(AmcuDecodeStackArgs)})

AM_REGISTER_KERNEL(SiluMul_CUDA_F32, KernelDescriptor{OpType::kSiluMul, AM_SEL(kF32, kF32, kPlain, kBoth), SiluMulFn,
                                                      "SiluMul_CUDA_F32", 0, BuildBinary, sizeof(BinaryArgs)})
AM_REGISTER_KERNEL(SiluMul_CUDA_BF16, KernelDescriptor{OpType::kSiluMul, AM_SEL(kBF16, kBF16, kPlain, kBoth), SiluMulFn,
                                                       "SiluMul_CUDA_BF16", 0, BuildBinary, sizeof(BinaryArgs)})
AM_REGISTER_KERNEL(Add_CUDA_F32, KernelDescriptor{OpType::kAdd, AM_SEL(kF32, kF32, kPlain, kBoth), AddFn, "Add_CUDA_F32",
                                                  0, BuildBinary, sizeof(BinaryArgs)})
AM_REGISTER_KERNEL(Add_CUDA_BF16, KernelDescriptor{OpType::kAdd, AM_SEL(kBF16, kBF16, kPlain, kBoth), AddFn,
                                                   "Add_CUDA_BF16", 0, BuildBinary, sizeof(BinaryArgs)})

AM_REGISTER_KERNEL(Embedding_CUDA_F32, KernelDescriptor{OpType::kEmbedding, AM_SEL(kF32, kF32, kPlain, kBoth),
                                                        EmbeddingFn, "Embedding_CUDA_F32", 0, BuildEmbedding,
                                                        sizeof(AmcuEmbeddingArgs)})
AM_REGISTER_KERNEL(Embedding_CUDA_BF16, KernelDescriptor{OpType::kEmbedding, AM_SEL(kBF16, kBF16, kPlain, kBoth),
                                                         EmbeddingFn, "Embedding_CUDA_BF16", 0, BuildEmbedding,
                                                         sizeof(AmcuEmbeddingArgs)})
AM_REGISTER_KERNEL(Embedding_CUDA_BF16_I8Rows,
                   KernelDescriptor{OpType::kEmbedding, AM_SEL(kBF16, kI8, kQuantizedInt8, kBoth), EmbeddingFn,
                                    "Embedding_CUDA_BF16_Int8Rows", 0, BuildEmbedding, sizeof(AmcuEmbeddingArgs)})

AM_REGISTER_KERNEL(Argmax_CUDA_F32, KernelDescriptor{OpType::kArgmax, AM_SEL(kF32, kF32, kPlain, kBoth), ArgmaxFn,
                                                     "Argmax_CUDA_F32", 0, BuildArgmax, sizeof(ArgmaxArgs)})
AM_REGISTER_KERNEL(Argmax_CUDA_BF16, KernelDescriptor{OpType::kArgmax, AM_SEL(kBF16, kBF16, kPlain, kBoth), ArgmaxFn,
                                                      "Argmax_CUDA_BF16", 0, BuildArgmax, sizeof(ArgmaxArgs)})

}  // namespace aethermind
