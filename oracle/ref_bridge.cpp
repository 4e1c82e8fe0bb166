// Test infrastructure only: a ctypes-callable bridge onto the reference
// engine's OWN compiled CPU kernels (libam_ref.so, built from the reference
// sources by oracle/Makefile). It adds no arithmetic of its own; each function
// packs plain pointers into the reference's argument structs and calls the
// reference entry point named in its comment. Nothing in the product links it.
#include "aethermind/backend/cpu/kernels/add/cpu_add_kernel.h"
#include "aethermind/backend/cpu/kernels/rmsnorm/cpu_rmsnorm_kernel.h"
#include "aethermind/backend/kernel_context.h"
#include "aethermind/dtypes/bfloat16.h"
#include "aethermind/execution/kv_cache_manager.h"
#include "aethermind/execution/kv_cache_view.h"
#include "aethermind/operators/op_params.h"
#include "backend/cpu/kernels/embedding/embedding_internal.h"
#include "backend/cpu/kernels/rmsnorm/rmsnorm_internal.h"
#include "graph/optimization/const_eval_internal.h"

#include <cstdint>
#include <cstring>

using namespace aethermind;

namespace {
DataType DtypeFromCode(int code) {
    // 0 = fp32, 1 = bf16
    return code == 1 ? DataType::BFloat(16) : DataType::Float32();
}
}  // namespace

extern "C" {

// LaunchRmsNorm (src/backend/cpu/kernels/rmsnorm/rmsnorm_api.cpp:9-39): picks
// the AVX2 kernel for unit column strides. force_scalar calls
// RmsNormKernel_CPU_FP32_Scalar (rmsnorm_fp32_scalar.cpp:37-63) directly.
int refb_rmsnorm_f32(const float* in, const float* w, float* out, int64_t rows,
                     int64_t hidden, int64_t in_row_stride, int64_t out_row_stride,
                     float eps, int force_scalar) {
    if (force_scalar) {
        cpu::detail::RmsNormFp32KernelArgs a;
        a.input = in;
        a.weight = w;
        a.output = out;
        a.seq_len = rows;
        a.hidden_size = hidden;
        a.input_row_stride = in_row_stride;
        a.input_col_stride = 1;
        a.weight_stride = 1;
        a.output_row_stride = out_row_stride;
        a.output_col_stride = 1;
        a.eps = eps;
        return static_cast<int>(cpu::detail::RmsNormKernel_CPU_FP32_Scalar(a).code());
    }
    RmsNormArgs a;
    a.input = in;
    a.weight = w;
    a.output = out;
    a.seq_len = rows;
    a.hidden_size = hidden;
    a.input_row_stride = in_row_stride;
    a.output_row_stride = out_row_stride;
    a.eps = eps;
    a.dtype = DataType::Float32();
    return static_cast<int>(LaunchRmsNorm(a).code());
}

// LaunchAdd (src/backend/cpu/kernels/add/add_api.cpp) -> AddKernel_Scalar.
int refb_add(const void* lhs, const void* rhs, void* out, int64_t numel, int dtype_code) {
    AddArgs a;
    a.lhs_data = lhs;
    a.rhs_data = rhs;
    a.output_data = out;
    a.numel = numel;
    a.dtype = DtypeFromCode(dtype_code);
    return static_cast<int>(LaunchAdd(a).code());
}

// SiluMul constant evaluator (src/graph/optimization/const_eval_silu_mul.cpp:18-33),
// the only executable SiLU-Mul arithmetic in the reference.
int refb_silu_mul(const void* gate, const void* up, void* out, int64_t numel, int dtype_code) {
    const DataType dt = DtypeFromCode(dtype_code);
    int64_t shape[1] = {numel};
    int64_t strides[1] = {1};
    TensorView ins[2] = {TensorView{gate, dt, shape, strides}, TensorView{up, dt, shape, strides}};
    MutableTensorView outs[1] = {MutableTensorView{out, dt, shape, strides}};
    OpParams params{SiluMulParams{}};
    return static_cast<int>(
            detail::GetSiluMulConstEvaluator().Evaluate(ins, outs, params).code());
}

// EmbeddingKernel (src/backend/cpu/kernels/embedding/embedding_entry.cpp:32-126).
// id_dtype: 0 = int32, 1 = int64, 2 = uint32.
int refb_embedding_f32(const void* ids, int64_t n_ids, int id_dtype, const float* weight,
                       int64_t vocab, int64_t hidden, float* out) {
    const DataType idt = id_dtype == 0 ? DataType::Int(32)
                         : id_dtype == 1 ? DataType::Int(64)
                                         : DataType::UInt(32);
    int64_t id_shape[1] = {n_ids};
    int64_t id_strides[1] = {1};
    int64_t w_shape[2] = {vocab, hidden};
    int64_t w_strides[2] = {hidden, 1};
    int64_t o_shape[2] = {n_ids, hidden};
    int64_t o_strides[2] = {hidden, 1};
    cpu::detail::EmbeddingParams p{
            .token_ids = TensorView{ids, idt, id_shape, id_strides},
            .weight = TensorView{weight, DataType::Float32(), w_shape, w_strides},
            .output = MutableTensorView{out, DataType::Float32(), o_shape, o_strides},
    };
    KernelContext ctx{};
    ctx.device_type = DeviceType::kCPU;
    ctx.kernel_params = &p;
    return static_cast<int>(cpu::detail::EmbeddingKernel(ctx).code());
}

// KVCacheLayout::Offset (src/execution/kv_cache_view.cpp:41-75) with strides set
// up exactly as KVCacheManager::Init does (src/execution/kv_cache_manager.cpp:74-78).
int refb_kv_offset(uint64_t layers, uint64_t heads, uint64_t max_tokens, uint64_t head_dim,
                   int dtype_code, uint64_t l, uint64_t h, uint64_t p, uint64_t d,
                   uint64_t* offset_out, uint64_t* bytes_per_plane_out) {
    KVCacheManager mgr;
    Status st = mgr.Init(layers, heads, max_tokens, head_dim, DtypeFromCode(dtype_code));
    if (!st.ok()) return static_cast<int>(st.code());
    auto off = mgr.layout().Offset(l, h, p, d);
    if (!off.ok()) return static_cast<int>(off.status().code());
    *offset_out = off.value();
    *bytes_per_plane_out = mgr.layout().BytesPerPlane().value();
    return 0;
}

// KVCacheManager session contract (kv_cache_manager.cpp:99-155): reserve with
// (prompt_len, max_new) and report the status code, for boundary tests.
int refb_kv_reserve(uint64_t max_tokens, uint64_t prompt_len, uint64_t max_new) {
    KVCacheManager mgr;
    Status st = mgr.Init(1, 1, max_tokens, 8, DataType::Float32());
    if (!st.ok()) return static_cast<int>(st.code());
    auto v = mgr.ReserveForSession(prompt_len, max_new);
    return static_cast<int>(v.ok() ? StatusCode::kOk : v.status().code());
}

// BFloat16(float) conversion (include/aethermind/dtypes/bfloat16.h:60): RNE.
uint16_t refb_bf16_from_f32(float f) {
    BFloat16 b(f);
    return b.x;
}

}  // extern "C"
