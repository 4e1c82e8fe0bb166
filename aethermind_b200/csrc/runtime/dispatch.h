// Kernel dispatch surface of the CUDA backend.
//
// Mirrors the reference engine's plugin ABI so a CUDA kernel registers and
// resolves exactly like a CPU one:
//   OpType                       include/aethermind/operators/op_type.h:22-40
//   KernelSelector/SelectorMatches include/aethermind/backend/kernel_selector.h:41-71
//   KernelFunc/KernelParamsBuilder include/aethermind/backend/kernel_types.h:21-51
//   KernelContext                include/aethermind/backend/kernel_context.h:14-22
//   KernelDescriptor + validation include/aethermind/backend/kernel_descriptor.h:12-57
//   KernelRegistry               include/aethermind/backend/kernel_registry.h:40-77
//   AM_REGISTER_KERNEL           include/aethermind/backend/kernel_static_registration.h:15-22
// Registration happens at static-init time inside this library; the first
// backend constructed freezes the registry, after which Resolve is lock-free.
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <mutex>
#include <span>
#include <string>
#include <vector>

#include "runtime/status.h"

namespace aethermind {

enum class OpType : uint16_t {
    kUnknown = 0,
    kEmbedding,
    kRmsNorm,
    kLinear,
    kMatMul,
    kRoPE,
    kAttention,
    kSilu,
    kSiluMul,
    kElementwiseMul,
    kKVCacheUpdate,
    kAdd,
    kSoftmax,
    kArgmax,
    kReshape,
    kPermute,
    kReorder,
    kRoPEAttention,  // fused decode step: RoPE + KVCacheUpdate + Attention
    kDecodeStack,    // persistent decode step: every decoder layer in one launch
};
const char* ToString(OpType op) noexcept;

// Same type and values as the reference's DeviceType (include/aethermind/base/device.h:23-28).
enum class DeviceType : uint8_t { kCPU = 0, kCUDA, kCANN, kUndefined };

// The element types used on the path. The reference's DataType is a DLPack-style
// (code, bits, lanes) triple; this engine only needs these, and the reference
// plugin (reference_plugin/cuda_backend_plugin.cpp) converts at the boundary.
enum class DType : uint8_t { kUndefined = 0, kF32, kBF16, kF16, kI8, kI4, kI32, kI64, kU32 };

enum class IsaLevel : uint8_t { kScalar = 0, kAVX2, kAVX512, kAMX };
enum class ExecPhase : uint8_t { kPrefill = 0, kDecode, kBoth };
enum class WeightFormat : uint8_t { kPlain = 0, kPacked, kQuantizedInt8, kQuantizedInt4 };

inline bool PhaseMatches(ExecPhase candidate, ExecPhase request) noexcept {
    return candidate == request || candidate == ExecPhase::kBoth;
}

struct KernelSelector {
    DeviceType device_type = DeviceType::kUndefined;
    DType act_dtype = DType::kUndefined;
    DType weight_dtype = DType::kUndefined;
    WeightFormat weight_format = WeightFormat::kPlain;
    IsaLevel isa = IsaLevel::kScalar;
    ExecPhase phase = ExecPhase::kBoth;
    friend bool operator==(const KernelSelector&, const KernelSelector&) = default;
};

// Exact device/dtypes/format, phase equal-or-Both, isa <= request.
inline bool SelectorMatches(const KernelSelector& c, const KernelSelector& r) noexcept {
    return c.device_type == r.device_type && c.act_dtype == r.act_dtype && c.weight_dtype == r.weight_dtype &&
           c.weight_format == r.weight_format && PhaseMatches(c.phase, r.phase) && c.isa <= r.isa;
}
std::string ToString(const KernelSelector& s);

// A borrowed device tensor (pointer, dtype, up to 4 dims, strides in elements).
struct TensorView {
    const void* data = nullptr;
    DType dtype = DType::kUndefined;
    int ndim = 0;
    int64_t shape[4] = {0, 0, 0, 0};
    int64_t strides[4] = {0, 0, 0, 0};
    int64_t dim(int i) const { return shape[i]; }
    bool is_valid() const { return dtype != DType::kUndefined && ndim > 0; }
};
struct MutableTensorView : TensorView {
    void* mutable_data() const { return const_cast<void*>(data); }
};
TensorView MakeView(const void* p, DType dt, std::initializer_list<int64_t> shape);
MutableTensorView MakeMutableView(void* p, DType dt, std::initializer_list<int64_t> shape);

// Stream carrying a cudaStream_t (the reference's Stream is an empty CPU
// placeholder, include/aethermind/backend/stream.h:6-14).
class Stream {
public:
    explicit Stream(cudaStream_t s = nullptr) : s_(s) {}
    cudaStream_t handle() const { return s_; }

private:
    cudaStream_t s_;
};

class WorkspaceArena;
struct WorkspaceBinding {
    void* data = nullptr;
    size_t size = 0;
};

struct KernelContext {
    DeviceType device_type = DeviceType::kUndefined;
    Stream* stream = nullptr;
    WorkspaceArena* workspace = nullptr;
    WorkspaceBinding workspace_binding{};
    const void* packed_weights = nullptr;
    const void* kernel_params = nullptr;
    std::span<const std::byte> attrs{};
};

using KernelFunc = Status (*)(const KernelContext&) noexcept;
using KernelParamsBuilder = Status (*)(std::span<const TensorView> inputs,
                                       std::span<const MutableTensorView> outputs,
                                       std::span<const std::byte> attrs, const void* packed_weights,
                                       void* params_buffer) noexcept;
inline constexpr size_t kMaxKernelParamsSize = 512;

struct KernelDescriptor {
    OpType op_type = OpType::kUnknown;
    KernelSelector selector{};
    KernelFunc kernel_func = nullptr;
    std::string name{};
    int priority = 0;  // higher wins; first registered wins a tie
    KernelParamsBuilder params_builder = nullptr;
    size_t params_size = 0;
};
Status ValidateKernelDescriptor(const KernelDescriptor& d) noexcept;

struct ResolvedKernel {
    OpType op_type = OpType::kUnknown;
    KernelFunc fn = nullptr;
    const char* debug_name = nullptr;
    KernelParamsBuilder params_builder = nullptr;
    size_t params_size = 0;
};

class KernelRegistry {
public:
    static KernelRegistry& Global();
    Status Register(const KernelDescriptor& d);
    void Freeze() noexcept;
    bool frozen() const noexcept { return frozen_.load(std::memory_order_acquire); }
    StatusOr<ResolvedKernel> Resolve(OpType op, const KernelSelector& request) const noexcept;
    std::vector<std::string> DebugDump() const;
    size_t size() const;

private:
    mutable std::mutex mu_;
    std::vector<KernelDescriptor> kernels_;
    std::atomic<bool> frozen_{false};
};

// Backend (include/aethermind/backend/backend.h:14-28).
class Backend {
public:
    virtual ~Backend() = default;
    virtual DeviceType device_type() const noexcept = 0;
    virtual StatusOr<ResolvedKernel> ResolveKernelInfo(OpType op, const KernelSelector& s) const noexcept = 0;
    virtual const KernelRegistry* TryGetKernelRegistryForDebug() const noexcept = 0;
};

class CudaBackend final : public Backend {
public:
    explicit CudaBackend(int device_id);
    DeviceType device_type() const noexcept override { return DeviceType::kCUDA; }
    StatusOr<ResolvedKernel> ResolveKernelInfo(OpType op, const KernelSelector& s) const noexcept override;
    const KernelRegistry* TryGetKernelRegistryForDebug() const noexcept override { return &KernelRegistry::Global(); }
    int device_id() const { return device_id_; }
    int num_sms() const { return num_sms_; }

private:
    int device_id_;
    int num_sms_ = 148;
};

namespace kernel_registration_detail {
bool RegisterOrDie(const KernelDescriptor& d);
}

}  // namespace aethermind

#define AM_REGISTER_KERNEL(unique_name, ...)                                                              \
    namespace {                                                                                           \
    [[maybe_unused]] static const bool _am_kernel_reg_##unique_name =                                     \
            ::aethermind::kernel_registration_detail::RegisterOrDie(__VA_ARGS__);                          \
    }
