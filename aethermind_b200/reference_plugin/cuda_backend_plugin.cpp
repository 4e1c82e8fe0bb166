// CUDA backend plugin for the reference engine (fengjiran/AetherMind),
// written against its public headers and calling this library's C ABI.
//
// This is the file a maintainer of the reference adds to make its Executor run
// on B200: it registers CUDA kernels in the reference's own KernelRegistry with
// AM_REGISTER_KERNEL (include/aethermind/backend/kernel_static_registration.h:15-22)
// under KernelSelector{.device_type = kCUDA, ...}, and exposes a Backend
// (include/aethermind/backend/backend.h:14-28) through a BackendFactory
// (include/aethermind/backend/backend_factory.h:12-17) that
// RuntimeBuilder::RegisterBackendFactory (include/aethermind/runtime/runtime_builder.h:22-24)
// accepts. Plans whose nodes carry device_type = kCUDA then resolve these
// kernels in ExecutionPlanBuilder::Build and run them from LayerRunner::RunStep,
// with no change to the reference's operators, planner or executor.
//
// Each kernel is the reference's KernelFunc signature
// (include/aethermind/backend/kernel_types.h:21) around one amcu_* launcher:
//   * a KernelParamsBuilder (kernel_types.h:41-43) placement-news a small POD
//     of device pointers, shapes and strides from the step's TensorViews into
//     the caller's 512-byte params buffer;
//   * the KernelFunc reads it, the op's attrs (RMSNorm: eps, as RmsNormOp::Prepare
//     stores it, src/operators/rmsnorm_op.cpp:26-27) and the stream, and launches.
// Tensors bound to these steps are DEVICE pointers. The reference's LayerRunner
// passes no stream (src/execution/layer_runner.cpp:13), so a null
// KernelContext::stream means the CUDA legacy default stream; a caller that
// owns a stream passes a CudaStream. Kernels are asynchronous: a caller
// synchronizes the stream before reading outputs, and a fault surfaces there.
#include <cuda_runtime.h>

#include <cstring>
#include <memory>
#include <new>
#include <span>

#include "aethermind/backend/backend.h"
#include "aethermind/backend/backend_factory.h"
#include "aethermind/backend/kernel_context.h"
#include "aethermind/backend/kernel_descriptor.h"
#include "aethermind/backend/kernel_registry.h"
#include "aethermind/backend/kernel_static_registration.h"
#include "aethermind/backend/stream.h"
#include "aethermind/base/tensor_view.h"

#include "aethermind_b200.h"

namespace aethermind_b200_plugin {

using namespace aethermind;

// A reference Stream carrying a CUDA stream.
class CudaStream final : public Stream {
public:
    explicit CudaStream(cudaStream_t s) noexcept : stream_(s) {}
    cudaStream_t native() const noexcept { return stream_; }

private:
    cudaStream_t stream_;
};

inline void* NativeStream(const KernelContext& ctx) noexcept {
    if (auto* cs = dynamic_cast<CudaStream*>(ctx.stream)) return cs->native();
    return nullptr;  // the legacy default stream
}

inline Status FromAm(am_status_code code) {
    if (code == AM_STATUS_OK) return Status::Ok();
    const char* msg = amcu_last_error();
    switch (code) {
        case AM_STATUS_INVALID_ARGUMENT: return Status::InvalidArgument(msg);
        case AM_STATUS_OUT_OF_RANGE: return Status::OutOfRange(msg);
        case AM_STATUS_UNIMPLEMENTED: return Status::Unimplemented(msg);
        case AM_STATUS_NOT_FOUND: return Status::NotFound(msg);
        default: return Status::Internal(msg);
    }
}

inline bool ToAmcuDtype(const DataType& t, int32_t& out) noexcept {
    if (t == DataType::Float32()) { out = AMCU_F32; return true; }
    if (t == DataType::BFloat(16)) { out = AMCU_BF16; return true; }
    return false;
}

// ---- RMSNorm: [rows, hidden] (last dim contiguous) x weight [hidden] ----
struct RmsNormCudaParams {
    const void* input;
    const void* weight;
    void* output;
    int64_t rows, hidden, in_stride, out_stride;
    int32_t dtype;
};

Status BuildRmsNormParams(std::span<const TensorView> in, std::span<const MutableTensorView> out,
                          void* buffer) noexcept {
    if (in.size() != 2 || out.size() != 1) return Status::InvalidArgument("RmsNorm CUDA: 2 inputs, 1 output");
    const TensorView& x = in[0];
    const TensorView& w = in[1];
    const MutableTensorView& y = out[0];
    if (x.rank() < 1 || w.rank() != 1 || y.rank() != x.rank())
        return Status::InvalidArgument("RmsNorm CUDA: input [..., hidden], weight [hidden]");
    const int32_t r = x.rank();
    const int64_t hidden = x.dim(r - 1);
    if (w.dim(0) != hidden || y.dim(r - 1) != hidden) return Status::InvalidArgument("RmsNorm CUDA: hidden mismatch");
    if (x.stride(r - 1) != 1 || y.stride(r - 1) != 1 || w.stride(0) != 1)
        return Status::InvalidArgument("RmsNorm CUDA: the last dim must be contiguous");
    int32_t dt = 0;
    if (!ToAmcuDtype(x.dtype(), dt) || x.dtype() != w.dtype() || x.dtype() != y.dtype())
        return Status::InvalidArgument("RmsNorm CUDA: f32 or bf16, one dtype for input, weight and output");
    int64_t rows = 1;
    for (int32_t i = 0; i + 1 < r; ++i) rows *= x.dim(i);
    auto* p = new (buffer) RmsNormCudaParams{};
    p->input = x.data();
    p->weight = w.data();
    p->output = y.data();
    p->rows = rows;
    p->hidden = hidden;
    p->in_stride = r >= 2 ? x.stride(r - 2) : hidden;
    p->out_stride = r >= 2 ? y.stride(r - 2) : hidden;
    p->dtype = dt;
    return Status::Ok();
}

Status RmsNormCudaKernel(const KernelContext& ctx) noexcept {
    const auto* p = static_cast<const RmsNormCudaParams*>(ctx.kernel_params);
    if (p == nullptr) return Status::InvalidArgument("RmsNorm CUDA: kernel params missing");
    float eps = 0.f;
    if (ctx.attrs.size() != sizeof(float)) return Status::InvalidArgument("RmsNorm CUDA: eps attr missing");
    std::memcpy(&eps, ctx.attrs.data(), sizeof(float));
    if (p->rows == 0) return Status::Ok();  // empty input: nothing to touch (rmsnorm_entry.cpp:98-103)
    AmcuRmsNormArgs a{};
    a.input = p->input;
    a.weight = p->weight;
    a.output = p->output;
    a.rows = p->rows;
    a.hidden = p->hidden;
    a.input_row_stride = p->in_stride;
    a.output_row_stride = p->out_stride;
    a.eps = eps;
    a.dtype = p->dtype;
    return FromAm(amcu_rmsnorm(&a, NativeStream(ctx)));
}

// ---- Add: two same-shape contiguous tensors ----
struct AddCudaParams {
    const void* a;
    const void* b;
    void* out;
    int64_t count;
    int32_t dtype;
};

Status BuildAddParams(std::span<const TensorView> in, std::span<const MutableTensorView> out, void* buffer) noexcept {
    if (in.size() != 2 || out.size() != 1) return Status::InvalidArgument("Add CUDA: 2 inputs, 1 output");
    const TensorView& a = in[0];
    const TensorView& b = in[1];
    const MutableTensorView& y = out[0];
    if (!a.is_contiguous() || !b.is_contiguous() || !y.is_contiguous() || a.numel() != b.numel() ||
        a.numel() != y.numel())
        return Status::InvalidArgument("Add CUDA: contiguous tensors of one shape (no broadcast)");
    int32_t dt = 0;
    if (!ToAmcuDtype(a.dtype(), dt) || a.dtype() != b.dtype() || a.dtype() != y.dtype())
        return Status::InvalidArgument("Add CUDA: f32 or bf16, one dtype");
    new (buffer) AddCudaParams{a.data(), b.data(), y.data(), a.numel(), dt};
    return Status::Ok();
}

Status AddCudaKernel(const KernelContext& ctx) noexcept {
    const auto* p = static_cast<const AddCudaParams*>(ctx.kernel_params);
    if (p == nullptr) return Status::InvalidArgument("Add CUDA: kernel params missing");
    if (p->count == 0) return Status::Ok();
    return FromAm(amcu_add(p->a, p->b, p->out, p->count, p->dtype, NativeStream(ctx)));
}

inline KernelSelector CudaSel(DataType t) {
    return KernelSelector{.device_type = DeviceType::kCUDA, .act_dtype = t, .weight_dtype = t,
                          .weight_format = WeightFormat::kPlain, .isa = IsaLevel::kScalar,
                          .phase = ExecPhase::kBoth};
}

// ---- the backend: resolves kCUDA selectors in the reference's registry ----
class CudaBackend final : public Backend {
public:
    CudaBackend() {
        // the registry is frozen by the first backend built (as CpuBackend does)
        (void)KernelRegistry::Global().Freeze();
    }
    DeviceType device_type() const noexcept override { return DeviceType::kCUDA; }
    const BackendCapabilities& capabilities() const noexcept override { return caps_; }
    KernelFunc ResolveKernel(OpType op, const KernelSelector& sel) const noexcept override {
        if (sel.device_type != DeviceType::kCUDA) return nullptr;
        const auto d = KernelRegistry::Global().Resolve(op, sel);
        return d.ok() ? (*d)->kernel_func : nullptr;
    }
    StatusOr<ResolvedKernel> ResolveKernelInfo(OpType op, const KernelSelector& sel) const noexcept override {
        if (sel.device_type != DeviceType::kCUDA)
            return Status::InvalidArgument("the CUDA backend resolves kCUDA selectors only");
        const auto d = KernelRegistry::Global().Resolve(op, sel);
        if (!d.ok()) return d.status();
        return ResolvedKernel{.op_type = op,
                              .fn = (*d)->kernel_func,
                              .attrs = {},
                              .debug_name = (*d)->name.c_str(),
                              .params_builder = (*d)->params_builder,
                              .params_size = (*d)->params_size};
    }
    const KernelRegistry* TryGetKernelRegistryForDebug() const noexcept override { return &KernelRegistry::Global(); }

private:
    BackendCapabilities caps_{};
};

class CudaBackendFactory final : public BackendFactory {
public:
    DeviceType device_type() const noexcept override { return DeviceType::kCUDA; }
    std::unique_ptr<Backend> Create() const override { return std::make_unique<CudaBackend>(); }
};

}  // namespace aethermind_b200_plugin

// Static registration into the reference's global registry (runs when this
// library is loaded, before any backend freezes the registry). The macro
// expects to expand inside namespace aethermind, as the reference's own
// kernel files use it.
namespace aethermind {
AM_REGISTER_KERNEL(AmcuRmsNormF32,
                   ::aethermind::KernelDescriptor{
                           .op_type = ::aethermind::OpType::kRmsNorm,
                           .selector = ::aethermind_b200_plugin::CudaSel(::aethermind::DataType::Float32()),
                           .kernel_func = &::aethermind_b200_plugin::RmsNormCudaKernel,
                           .name = "aethermind_b200::rmsnorm_cuda_f32",
                           .priority = 0,
                           .params_builder = &::aethermind_b200_plugin::BuildRmsNormParams,
                           .params_size = sizeof(::aethermind_b200_plugin::RmsNormCudaParams)})
AM_REGISTER_KERNEL(AmcuRmsNormBF16,
                   ::aethermind::KernelDescriptor{
                           .op_type = ::aethermind::OpType::kRmsNorm,
                           .selector = ::aethermind_b200_plugin::CudaSel(::aethermind::DataType::BFloat(16)),
                           .kernel_func = &::aethermind_b200_plugin::RmsNormCudaKernel,
                           .name = "aethermind_b200::rmsnorm_cuda_bf16",
                           .priority = 0,
                           .params_builder = &::aethermind_b200_plugin::BuildRmsNormParams,
                           .params_size = sizeof(::aethermind_b200_plugin::RmsNormCudaParams)})
AM_REGISTER_KERNEL(AmcuAddF32,
                   ::aethermind::KernelDescriptor{
                           .op_type = ::aethermind::OpType::kAdd,
                           .selector = ::aethermind_b200_plugin::CudaSel(::aethermind::DataType::Float32()),
                           .kernel_func = &::aethermind_b200_plugin::AddCudaKernel,
                           .name = "aethermind_b200::add_cuda_f32",
                           .priority = 0,
                           .params_builder = &::aethermind_b200_plugin::BuildAddParams,
                           .params_size = sizeof(::aethermind_b200_plugin::AddCudaParams)})
AM_REGISTER_KERNEL(AmcuAddBF16,
                   ::aethermind::KernelDescriptor{
                           .op_type = ::aethermind::OpType::kAdd,
                           .selector = ::aethermind_b200_plugin::CudaSel(::aethermind::DataType::BFloat(16)),
                           .kernel_func = &::aethermind_b200_plugin::AddCudaKernel,
                           .name = "aethermind_b200::add_cuda_bf16",
                           .priority = 0,
                           .params_builder = &::aethermind_b200_plugin::BuildAddParams,
                           .params_size = sizeof(::aethermind_b200_plugin::AddCudaParams)})
}  // namespace aethermind

// The factory a host hands to RuntimeBuilder::RegisterBackendFactory(kCUDA, ...).
extern "C" __attribute__((visibility("default"))) void* aethermind_b200_make_cuda_backend_factory() {
    return new aethermind_b200_plugin::CudaBackendFactory();
}
