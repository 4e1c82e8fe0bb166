// KernelRegistry / CudaBackend implementation (contract of
// src/backend/kernel_registry.cpp:30-112 and src/backend/cpu/cpu_backend.cpp:7-65).
#include "runtime/dispatch.h"

#include <cstdio>
#include <cstdlib>

namespace aethermind {

std::string Status::ToString() const {
    static const char* names[] = {"OK", "Cancelled", "Unknown", "InvalidArgument", "DeadlineExceeded",
                                  "NotFound", "AlreadyExists", "PermissionDenied", "ResourceExhausted",
                                  "FailedPrecondition", "Aborted", "OutOfRange", "Unimplemented",
                                  "Internal", "Unavailable", "DataLoss", "Overflow", "Unauthenticated"};
    const int c = static_cast<int>(code_);
    return std::string(c < 18 ? names[c] : "?") + (msg_.empty() ? "" : ": " + msg_);
}

const char* ToString(OpType op) noexcept {
    switch (op) {
        case OpType::kEmbedding: return "Embedding";
        case OpType::kRmsNorm: return "RmsNorm";
        case OpType::kLinear: return "Linear";
        case OpType::kMatMul: return "MatMul";
        case OpType::kRoPE: return "RoPE";
        case OpType::kAttention: return "Attention";
        case OpType::kSilu: return "Silu";
        case OpType::kSiluMul: return "SiluMul";
        case OpType::kElementwiseMul: return "ElementwiseMul";
        case OpType::kKVCacheUpdate: return "KVCacheUpdate";
        case OpType::kAdd: return "Add";
        case OpType::kSoftmax: return "Softmax";
        case OpType::kArgmax: return "Argmax";
        case OpType::kReshape: return "Reshape";
        case OpType::kPermute: return "Permute";
        case OpType::kReorder: return "Reorder";
        case OpType::kRoPEAttention: return "RoPEAttention";
        case OpType::kDecodeStack: return "DecodeStack";
        default: return "Unknown";
    }
}

std::string ToString(const KernelSelector& s) {
    char buf[160];
    snprintf(buf, sizeof(buf), "{device=%d act=%d weight=%d format=%d isa=%d phase=%d}", (int)s.device_type,
             (int)s.act_dtype, (int)s.weight_dtype, (int)s.weight_format, (int)s.isa, (int)s.phase);
    return buf;
}

static void fill_contiguous(TensorView& v, std::initializer_list<int64_t> shape) {
    v.ndim = (int)shape.size();
    int i = 0;
    for (int64_t d : shape) v.shape[i++] = d;
    int64_t st = 1;
    for (int j = v.ndim - 1; j >= 0; --j) {
        v.strides[j] = st;
        st *= v.shape[j];
    }
}

TensorView MakeView(const void* p, DType dt, std::initializer_list<int64_t> shape) {
    TensorView v;
    v.data = p;
    v.dtype = dt;
    fill_contiguous(v, shape);
    return v;
}

MutableTensorView MakeMutableView(void* p, DType dt, std::initializer_list<int64_t> shape) {
    MutableTensorView v;
    v.data = p;
    v.dtype = dt;
    fill_contiguous(v, shape);
    return v;
}

Status ValidateKernelDescriptor(const KernelDescriptor& d) noexcept {
    if (d.op_type == OpType::kUnknown) return Status::InvalidArgument("Kernel descriptor op_type cannot be kUnknown");
    if (d.kernel_func == nullptr) return Status::InvalidArgument("Kernel descriptor function cannot be null");
    if (d.name.empty()) return Status::InvalidArgument("Kernel descriptor name cannot be empty");
    if (d.selector.device_type == DeviceType::kUndefined)
        return Status::InvalidArgument("Kernel descriptor device_type cannot be kUndefined");
    if (d.params_builder != nullptr) {
        if (d.params_size == 0) return Status::InvalidArgument("params_size must be > 0 when params_builder is set");
        if (d.params_size > kMaxKernelParamsSize)
            return Status::InvalidArgument("params_size exceeds kMaxKernelParamsSize");
    }
    return Status::Ok();
}

KernelRegistry& KernelRegistry::Global() {
    static KernelRegistry r;
    return r;
}

Status KernelRegistry::Register(const KernelDescriptor& d) {
    AM_RETURN_IF_ERROR(ValidateKernelDescriptor(d));
    std::lock_guard<std::mutex> lk(mu_);
    if (frozen_.load(std::memory_order_acquire))
        return Status::FailedPrecondition("KernelRegistry is frozen; register kernels before the first backend");
    for (const auto& k : kernels_)
        if (k.op_type == d.op_type && k.selector == d.selector)
            return Status::AlreadyExists("duplicate kernel for " + std::string(ToString(d.op_type)) + " " +
                                         ToString(d.selector));
    kernels_.push_back(d);
    return Status::Ok();
}

void KernelRegistry::Freeze() noexcept { frozen_.store(true, std::memory_order_release); }

StatusOr<ResolvedKernel> KernelRegistry::Resolve(OpType op, const KernelSelector& req) const noexcept {
    if (!frozen()) return Status::FailedPrecondition("KernelRegistry must be frozen before Resolve");
    const KernelDescriptor* best = nullptr;
    for (const auto& k : kernels_) {
        if (k.op_type != op || !SelectorMatches(k.selector, req)) continue;
        if (best == nullptr || k.priority > best->priority) best = &k;
    }
    if (best == nullptr)
        return Status::NotFound(std::string("no CUDA kernel for ") + ToString(op) + " " + ToString(req));
    ResolvedKernel r;
    r.op_type = op;
    r.fn = best->kernel_func;
    r.debug_name = best->name.c_str();
    r.params_builder = best->params_builder;
    r.params_size = best->params_size;
    return r;
}

std::vector<std::string> KernelRegistry::DebugDump() const {
    std::lock_guard<std::mutex> lk(mu_);
    std::vector<std::string> out;
    for (const auto& k : kernels_)
        out.push_back(std::string(ToString(k.op_type)) + " " + k.name + " " + ToString(k.selector) +
                      " prio=" + std::to_string(k.priority));
    return out;
}

size_t KernelRegistry::size() const {
    std::lock_guard<std::mutex> lk(mu_);
    return kernels_.size();
}

CudaBackend::CudaBackend(int device_id) : device_id_(device_id) {
    KernelRegistry::Global().Freeze();  // first backend freezes (src/backend/cpu/cpu_backend.cpp:7-10)
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device_id) == cudaSuccess && n > 0) num_sms_ = n;
}

StatusOr<ResolvedKernel> CudaBackend::ResolveKernelInfo(OpType op, const KernelSelector& s) const noexcept {
    if (s.device_type != DeviceType::kCUDA)
        return Status::InvalidArgument("CudaBackend only resolves kCUDA selectors");
    return KernelRegistry::Global().Resolve(op, s);
}

namespace kernel_registration_detail {
bool RegisterOrDie(const KernelDescriptor& d) {
    Status st = KernelRegistry::Global().Register(d);
    if (!st.ok()) {
        fprintf(stderr, "Kernel registration failed: %s\n", st.ToString().c_str());
        std::abort();
    }
    return true;
}
}  // namespace kernel_registration_detail

}  // namespace aethermind
