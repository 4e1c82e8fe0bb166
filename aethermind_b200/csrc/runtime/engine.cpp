// Allocator, workspace arena, KV cache manager/view, LayerRunner and the NCCL
// communicator of the CUDA backend.
#include "runtime/engine.h"

#include <cuda_runtime.h>

#include "amcu_internal.h"
#include "kernels/allreduce.cuh"

#include <dlfcn.h>

#include <cstdlib>
#include <cstring>

namespace aethermind {

size_t DTypeBytes(DType d) {
    switch (d) {
        case DType::kF32: case DType::kI32: case DType::kU32: return 4;
        case DType::kBF16: case DType::kF16: return 2;
        case DType::kI8: return 1;
        case DType::kI64: return 8;
        default: return 0;
    }
}

// ---------------------------------------------------------------- memory ---
DeviceBuffer& DeviceBuffer::operator=(DeviceBuffer&& o) noexcept {
    if (this != &o) {
        if (ptr_) cudaFree(ptr_);
        ptr_ = o.ptr_;
        size_ = o.size_;
        o.ptr_ = nullptr;
        o.size_ = 0;
    }
    return *this;
}
DeviceBuffer::~DeviceBuffer() {
    if (ptr_) cudaFree(ptr_);
}

StatusOr<DeviceBuffer> CudaAllocator::Allocate(size_t bytes) {
    if (bytes == 0) bytes = 256;
    bytes = (bytes + 255) / 256 * 256;
    void* p = nullptr;
    cudaSetDevice(device_);
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return Status::ResourceExhausted(std::string("cudaMalloc(") + std::to_string(bytes) +
                                         ") failed: " + cudaGetErrorString(e));
    }
    allocated_ += bytes;
    return DeviceBuffer(p, bytes);
}

Status WorkspaceArena::Reserve(CudaAllocator& alloc, size_t bytes) {
    if (bytes <= buf_.size()) return Status::Ok();
    auto b = alloc.Allocate(bytes);
    if (!b.ok()) return b.status();
    buf_ = std::move(b.value());
    return Status::Ok();
}

StatusOr<WorkspaceBinding> WorkspaceArena::Bind(size_t offset, size_t size) const {
    if (size == 0) return WorkspaceBinding{};
    if (offset + size < offset || offset + size > buf_.size())
        return Status::OutOfRange("workspace binding exceeds the arena capacity");
    return WorkspaceBinding{buf_.as<char>() + offset, size};
}

// -------------------------------------------------------------- KV cache ---
Status KVCacheLayout::Validate() const {
    if (num_layers == 0 || num_kv_heads == 0 || max_tokens == 0 || head_dim == 0 || num_slots == 0)
        return Status::InvalidArgument("KV layout dimensions must be positive");
    if (elt_bytes == 0) return Status::InvalidArgument("KV layout dtype must be initialized");
    return Status::Ok();
}

StatusOr<size_t> KVCacheLayout::Offset(size_t l, size_t h, size_t p, size_t d, size_t slot) const {
    AM_RETURN_IF_ERROR(Validate());
    if (l >= num_layers) return Status::OutOfRange("layer index out of range");
    if (h >= num_kv_heads) return Status::OutOfRange("kv_head index out of range");
    if (p >= max_tokens) return Status::OutOfRange("seq_pos index out of range");
    if (d >= head_dim) return Status::OutOfRange("dim index out of range");
    if (slot >= num_slots) return Status::OutOfRange("slot index out of range");
    return l * layer_stride + slot * slot_stride + h * head_stride + p * token_stride + d * elt_bytes;
}

StatusOr<size_t> KVCacheLayout::BytesPerPlane() const {
    AM_RETURN_IF_ERROR(Validate());
    return num_layers * layer_stride;
}

bool KVCacheView::valid() const {
    return layout_ && k_ && v_ && k_->is_initialized() && slot_ && slot_->in_use && slot_->generation == generation_;
}

Status KVCacheView::ValidateWrite(size_t layer, size_t h, size_t pos, size_t count) const {
    if (!valid()) return Status::FailedPrecondition("KVCacheView is invalid or stale");
    if (layer >= layout_->num_layers || h >= layout_->num_kv_heads)
        return Status::OutOfRange("KV write layer/head out of range");
    if (pos + count < pos || pos + count > slot_->capacity_tokens)
        return Status::OutOfRange("KV write exceeds the session capacity");
    return Status::Ok();
}

Status KVCacheView::ValidateRead(size_t layer, size_t h, size_t begin, size_t end) const {
    if (!valid()) return Status::FailedPrecondition("KVCacheView is invalid or stale");
    if (layer >= layout_->num_layers || h >= layout_->num_kv_heads)
        return Status::OutOfRange("KV read layer/head out of range");
    if (begin > end || end > slot_->current_pos) return Status::OutOfRange("KV read beyond committed tokens");
    return Status::Ok();
}

StatusOr<void*> KVCacheView::MutableKeyData(size_t layer, size_t h, size_t pos, size_t slot) {
    AM_RETURN_IF_ERROR(ValidateWrite(layer, h, pos, 1));
    auto off = layout_->Offset(layer, h, pos, 0, slot);
    if (!off.ok()) return off.status();
    return static_cast<void*>(k_->as<char>() + off.value());
}

StatusOr<void*> KVCacheView::MutableValueData(size_t layer, size_t h, size_t pos, size_t slot) {
    AM_RETURN_IF_ERROR(ValidateWrite(layer, h, pos, 1));
    auto off = layout_->Offset(layer, h, pos, 0, slot);
    if (!off.ok()) return off.status();
    return static_cast<void*>(v_->as<char>() + off.value());
}

Status KVCacheView::CommitUntil(size_t new_pos) {
    if (!valid()) return Status::FailedPrecondition("KVCacheView is invalid or stale");
    if (new_pos < slot_->current_pos || new_pos > slot_->capacity_tokens)
        return Status::OutOfRange("CommitUntil outside [current_pos, capacity]");
    slot_->current_pos = new_pos;
    return Status::Ok();
}

Status KVCacheManager::InitLayoutOnly(size_t L, size_t H, size_t T, size_t D, DType dt, size_t slots) {
    layout_ = {};
    slot_ = {};
    initialized_ = false;
    layout_.num_layers = L;
    layout_.num_kv_heads = H;
    layout_.max_tokens = T;
    layout_.head_dim = D;
    layout_.num_slots = slots;
    layout_.elt_bytes = DTypeBytes(dt);
    AM_RETURN_IF_ERROR(layout_.Validate());
    layout_.token_stride = D * layout_.elt_bytes;
    layout_.head_stride = T * layout_.token_stride;
    layout_.slot_stride = H * layout_.head_stride;
    layout_.layer_stride = slots * layout_.slot_stride;
    total_bytes_ = 2 * L * layout_.layer_stride;
    initialized_ = true;
    return Status::Ok();
}

Status KVCacheManager::Init(CudaAllocator& alloc, size_t L, size_t H, size_t T, size_t D, DType dt, size_t slots) {
    AM_RETURN_IF_ERROR(InitLayoutOnly(L, H, T, D, dt, slots));
    initialized_ = false;
    const size_t plane = L * layout_.layer_stride;
    auto kb = alloc.Allocate(plane);
    if (!kb.ok()) return kb.status();
    auto vb = alloc.Allocate(plane);
    if (!vb.ok()) return vb.status();
    k_ = std::move(kb.value());
    v_ = std::move(vb.value());
    // Zero both planes and wait: the engine runs on its own non-blocking stream,
    // which does not order against the legacy stream a plain cudaMemset uses.
    cudaMemset(k_.data(), 0, plane);
    cudaMemset(v_.data(), 0, plane);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return Status::Internal(std::string("KV cache init: ") + cudaGetErrorString(e));
    total_bytes_ = 2 * plane;
    initialized_ = true;
    return Status::Ok();
}

StatusOr<KVCacheView> KVCacheManager::ReserveForSession(size_t prompt_len, size_t max_new) {
    if (!initialized_) return Status::FailedPrecondition("the KV cache has not been set up (call Init first)");
    if (slot_.in_use) return Status::FailedPrecondition("a session already holds the KV cache; release it before reserving again");
    const size_t req = prompt_len + max_new;
    if (req < prompt_len) return Status::Overflow("prompt_len + max_new does not fit in size_t");
    if (req == 0) return Status::InvalidArgument("a KV reservation needs prompt_len + max_new >= 1");
    if (req > layout_.max_tokens) return Status::OutOfRange("prompt_len + max_new is larger than the KV cache's max_tokens");
    ++slot_.generation;
    slot_.in_use = true;
    slot_.capacity_tokens = req;
    slot_.prompt_len = prompt_len;
    slot_.current_pos = prompt_len;
    return KVCacheView(&layout_, &k_, &v_, &slot_);
}

Status KVCacheManager::ResetSession(KVCacheView& view) {
    if (!initialized_) return Status::FailedPrecondition("the KV cache has not been set up (call Init first)");
    if (!view.valid()) return Status::FailedPrecondition("this KV view was released or belongs to an older reservation (reset)");
    slot_.current_pos = slot_.prompt_len;
    return Status::Ok();
}

Status KVCacheManager::ReleaseSession(KVCacheView& view) {
    if (!initialized_) return Status::FailedPrecondition("the KV cache has not been set up (call Init first)");
    if (!view.valid()) return Status::FailedPrecondition("this KV view was released or belongs to an older reservation (release)");
    slot_.in_use = false;
    slot_.capacity_tokens = slot_.prompt_len = slot_.current_pos = 0;
    ++slot_.generation;
    view.Invalidate();
    return Status::Ok();
}

// ---------------------------------------------------------------- runner ---
Status LayerRunner::RunStep(const ExecutionPlan& plan, size_t i, Stream& stream, WorkspaceArena* ws,
                            const KVCacheView* kv) const {
    const ExecutionStep& st = plan.steps[i];
    // State-alias check (src/execution/layer_runner.cpp:69-93).
    if (st.kv_alias && (kv == nullptr || !kv->valid()))
        return Status::FailedPrecondition("step '" + st.label + "' needs a valid KV cache view");
    if (st.host_fn) return st.host_fn(st.host_ctx, stream.handle());
    KernelContext ctx;
    ctx.device_type = DeviceType::kCUDA;
    ctx.stream = &stream;
    ctx.workspace = ws;
    if (st.workspace_size > 0) {
        if (ws == nullptr) return Status::FailedPrecondition("step '" + st.label + "' needs a workspace");
        auto b = ws->Bind(st.workspace_offset, st.workspace_size);
        if (!b.ok()) return b.status();
        ctx.workspace_binding = b.value();
    }
    ctx.packed_weights = st.packed_weights;
    ctx.kernel_params = st.params.data();
    ctx.attrs = std::span<const std::byte>(st.attrs.data(), st.attrs.size());
    Status s = st.kernel.fn(ctx);
    if (!s.ok()) return Status(s.code(), "step " + std::to_string(i) + " (" + st.label + "): " + s.message());
    return s;
}

// AM_STEP_CHECK=1: synchronize after every step and report the first step
// whose kernel failed (diagnostics; never inside a stream capture).
static bool StepCheckEnabled() {
    static const bool on = [] {
        const char* e = getenv("AM_STEP_CHECK");
        return e && e[0] == '1';
    }();
    return on;
}

Status LayerRunner::Run(const ExecutionPlan& plan, Stream& stream, WorkspaceArena* ws, const KVCacheView* kv) const {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    const bool check = StepCheckEnabled() && cudaStreamIsCapturing(stream.handle(), &cap) == cudaSuccess &&
                       cap == cudaStreamCaptureStatusNone;
    for (size_t i = 0; i < plan.steps.size(); ++i) {
        AM_RETURN_IF_ERROR(RunStep(plan, i, stream, ws, kv));
        if (check) {
            cudaError_t e = cudaStreamSynchronize(stream.handle());
            if (e == cudaSuccess) e = cudaGetLastError();
            if (e != cudaSuccess)
                return Status::Internal("step " + std::to_string(i) + " (" + plan.steps[i].label +
                                        "): " + cudaGetErrorString(e));
        }
    }
    return Status::Ok();
}

// ------------------------------------------------------------------ NCCL ---
namespace {
using ncclResult_t = int;
struct NcclApi {
    ncclResult_t (*GetUniqueId)(void*) = nullptr;
    ncclResult_t (*CommInitRank)(void**, int, std::array<char, 128>, int) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, int, int, void*, cudaStream_t) = nullptr;
    ncclResult_t (*CommDestroy)(void*) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    bool loaded = false;
};
NcclApi& nccl() {
    static NcclApi api;
    if (!api.loaded) {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (h) {
            api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
            api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
            api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(dlsym(h, "ncclAllReduce"));
            api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
            api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
        }
        api.loaded = true;
    }
    return api;
}
constexpr int kNcclFloat32 = 7, kNcclBfloat16 = 9, kNcclSum = 0;
Status NcclStatus(ncclResult_t r, const char* what) {
    if (r == 0) return Status::Ok();
    const char* m = nccl().GetErrorString ? nccl().GetErrorString(r) : "?";
    return Status::Internal(std::string(what) + ": " + m);
}
}  // namespace

Status NcclGetUniqueId(void* out) {
    if (!nccl().GetUniqueId) return Status::Unavailable("libnccl.so.2 could not be loaded");
    return NcclStatus(nccl().GetUniqueId(out), "ncclGetUniqueId");
}

Status Communicator::Init(int rank, int world, const void* uid) {
    rank_ = rank;
    world_ = world;
    if (world <= 1) return Status::Ok();
    if (!nccl().CommInitRank) return Status::Unavailable("libnccl.so.2 could not be loaded");
    if (!uid) return Status::InvalidArgument("tp_size > 1 requires an nccl_unique_id");
    std::array<char, 128> id;
    std::memcpy(id.data(), uid, 128);
    return NcclStatus(nccl().CommInitRank(&comm_, world, id, rank), "ncclCommInitRank");
}

Communicator::~Communicator() {
    if (comm_ && nccl().CommDestroy) nccl().CommDestroy(comm_);
    for (int r = 0; r < world_ && r < 8; ++r)
        if (peers_[r] && peers_[r] != area_) cudaIpcCloseMemHandle(peers_[r]);
    if (area_) cudaFree(area_);
}

Status Communicator::PeerHandle(void* out64) {
    if (world_ <= 1) return Status::InvalidArgument("peer exchange needs tp_size > 1");
    if (world_ > amcu::kArMaxRanks) return Status::InvalidArgument("peer exchange supports at most 8 ranks");
    if (!area_) {
        const size_t bytes = amcu::ar_area_bytes();
        if (cudaMalloc(&area_, bytes) != cudaSuccess) {
            area_ = nullptr;
            cudaGetLastError();
            return Status::ResourceExhausted("peer exchange area");
        }
        if (cudaMemset(area_, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess)
            return Status::Internal("peer exchange area: memset failed");
    }
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, area_) != cudaSuccess) {
        cudaGetLastError();
        return Status::Unavailable("cudaIpcGetMemHandle failed");
    }
    static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
    std::memcpy(out64, &h, 64);
    return Status::Ok();
}

Status Communicator::OpenPeers(const void* handles) {
    if (!area_) return Status::FailedPrecondition("call am_runtime_peer_handle first");
    if (peers_open_) return Status::Ok();
    for (int r = 0; r < world_; ++r) {
        if (r == rank_) {
            peers_[r] = area_;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const char*>(handles) + 64 * r, 64);
        if (cudaIpcOpenMemHandle(&peers_[r], h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            peers_[r] = nullptr;
            cudaGetLastError();
            return Status::Unavailable("cudaIpcOpenMemHandle failed for rank " + std::to_string(r));
        }
    }
    peers_open_ = true;
    peer_args_ = AmcuAllReduceArgs{};
    peer_args_.rank = rank_;
    peer_args_.world = world_;
    for (int r = 0; r < world_; ++r) peer_args_.areas[r] = peers_[r];
    peer_args_.wait_limit_us = wait_ns_ / 1000;
    return Status::Ok();
}

bool Communicator::OneShotReady(int64_t n) const { return peers_open_ && amcu::ar_oneshot_supported(n, world_); }

Status Communicator::AllReduceAddBf16(const void* part, void* x, int64_t n, cudaStream_t s) {
    amcu::ArParams p{};
    p.part = part;
    p.x = x;
    p.n = n;
    p.rank = rank_;
    p.world = world_;
    for (int r = 0; r < world_; ++r) p.area[r] = static_cast<uint8_t*>(peers_[r]);
    p.err = amcu::device_error_word();
    p.wait_ns = wait_ns_;
    amcu::launch_ar_oneshot_add(p, s);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? Status::Ok() : Status::Internal(std::string("one-shot all-reduce: ") + cudaGetErrorString(e));
}

Status Communicator::AllReduceSumBf16(void* buf, size_t n, cudaStream_t s) {
    if (world_ <= 1) return Status::Ok();
    return NcclStatus(nccl().AllReduce(buf, buf, n, kNcclBfloat16, kNcclSum, comm_, s), "ncclAllReduce");
}

Status Communicator::AllReduceSumF32(void* buf, size_t n, cudaStream_t s) {
    if (world_ <= 1) return Status::Ok();
    return NcclStatus(nccl().AllReduce(buf, buf, n, kNcclFloat32, kNcclSum, comm_, s), "ncclAllReduce");
}

}  // namespace aethermind
