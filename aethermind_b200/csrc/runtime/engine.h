// Host runtime of the CUDA backend: device allocator, workspace arena, static
// KV-cache manager, execution plan / LayerRunner / Executor, tensor-parallel
// communicator, and the Llama model + session that drive them.
#pragma once
#include <cuda_runtime.h>

#include <array>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "runtime/dispatch.h"
#include "runtime/op_attrs.h"

namespace aethermind {

size_t DTypeBytes(DType d);

// ---------------------------------------------------------------------------
// Memory: CUDA allocator (replaces the aborting stub of
// src/memory/cuda_allocator.cpp:6-11) and an owning device buffer.
// ---------------------------------------------------------------------------
class DeviceBuffer {
public:
    DeviceBuffer() = default;
    DeviceBuffer(void* p, size_t n) : ptr_(p), size_(n) {}
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    DeviceBuffer(DeviceBuffer&& o) noexcept : ptr_(o.ptr_), size_(o.size_) { o.ptr_ = nullptr; o.size_ = 0; }
    DeviceBuffer& operator=(DeviceBuffer&& o) noexcept;
    ~DeviceBuffer();
    void* data() const { return ptr_; }
    size_t size() const { return size_; }
    template <typename T> T* as() const { return static_cast<T*>(ptr_); }
    bool is_initialized() const { return ptr_ != nullptr; }

private:
    void* ptr_ = nullptr;
    size_t size_ = 0;
};

class CudaAllocator {
public:
    explicit CudaAllocator(int device) : device_(device) {}
    // 256-byte aligned device memory; ResourceExhausted on OOM.
    StatusOr<DeviceBuffer> Allocate(size_t bytes);
    size_t allocated_bytes() const { return allocated_; }

private:
    int device_;
    size_t allocated_ = 0;
};

// Device workspace arena with the offset semantics of CpuWorkspaceArena::Bind
// (src/backend/cpu/cpu_workspace_arena.cpp:10-30): a binding is a slice valid
// for one step.
class WorkspaceArena {
public:
    Status Reserve(CudaAllocator& alloc, size_t bytes);
    StatusOr<WorkspaceBinding> Bind(size_t offset, size_t size) const;
    size_t capacity() const { return buf_.size(); }

private:
    DeviceBuffer buf_;
};

// ---------------------------------------------------------------------------
// Static KV cache (include/aethermind/execution/kv_cache_view.h:11-106,
// src/execution/kv_cache_manager.cpp:49-160) in HBM, with a slot axis so a
// batch of sequences shares one manager. Per layer the plane is
// [slot][kv_head][pos][dim]; slot 0 reproduces the reference offsets.
// ---------------------------------------------------------------------------
struct KVCacheLayout {
    size_t num_layers = 0, num_slots = 1, num_kv_heads = 0, max_tokens = 0, head_dim = 0;
    size_t elt_bytes = 0;
    size_t token_stride = 0, head_stride = 0, slot_stride = 0, layer_stride = 0;  // bytes
    Status Validate() const;
    StatusOr<size_t> Offset(size_t layer, size_t kv_head, size_t pos, size_t dim, size_t slot = 0) const;
    StatusOr<size_t> BytesPerPlane() const;
};

struct SessionKVSlot {
    uint64_t generation = 0;
    bool in_use = false;
    size_t capacity_tokens = 0, prompt_len = 0, current_pos = 0;
};

class KVCacheView {
public:
    KVCacheView() = default;
    KVCacheView(const KVCacheLayout* l, DeviceBuffer* k, DeviceBuffer* v, SessionKVSlot* s)
        : layout_(l), k_(k), v_(v), slot_(s), generation_(s ? s->generation : 0) {}
    bool valid() const;
    size_t current_pos() const { return valid() ? slot_->current_pos : 0; }
    size_t token_capacity() const { return valid() ? slot_->capacity_tokens : 0; }
    Status ValidateWrite(size_t layer, size_t kv_head, size_t pos, size_t count) const;
    Status ValidateRead(size_t layer, size_t kv_head, size_t begin, size_t end) const;
    StatusOr<void*> MutableKeyData(size_t layer, size_t kv_head, size_t pos, size_t slot = 0);
    StatusOr<void*> MutableValueData(size_t layer, size_t kv_head, size_t pos, size_t slot = 0);
    Status CommitUntil(size_t new_pos);
    void Invalidate() { slot_ = nullptr; }

private:
    const KVCacheLayout* layout_ = nullptr;
    DeviceBuffer* k_ = nullptr;
    DeviceBuffer* v_ = nullptr;
    SessionKVSlot* slot_ = nullptr;
    uint64_t generation_ = 0;
};

class KVCacheManager {
public:
    Status Init(CudaAllocator& alloc, size_t num_layers, size_t num_kv_heads, size_t max_tokens, size_t head_dim,
                DType kv_dtype, size_t num_slots = 1);
    // Layout and session bookkeeping only, no device storage (host-logic tests).
    Status InitLayoutOnly(size_t num_layers, size_t num_kv_heads, size_t max_tokens, size_t head_dim,
                          DType kv_dtype, size_t num_slots = 1);
    StatusOr<KVCacheView> ReserveForSession(size_t prompt_len, size_t max_new_tokens);
    Status ResetSession(KVCacheView& view);
    Status ReleaseSession(KVCacheView& view);
    const KVCacheLayout& layout() const { return layout_; }
    size_t capacity_tokens() const { return layout_.max_tokens; }
    size_t total_bytes() const { return total_bytes_; }
    bool is_initialized() const { return initialized_; }
    void* key_plane(size_t layer) const { return k_.as<char>() + layer * layout_.layer_stride; }
    void* value_plane(size_t layer) const { return v_.as<char>() + layer * layout_.layer_stride; }

private:
    KVCacheLayout layout_{};
    DeviceBuffer k_, v_;
    SessionKVSlot slot_{};
    size_t total_bytes_ = 0;
    bool initialized_ = false;
};

// ---------------------------------------------------------------------------
// Execution plan (include/aethermind/execution/execution_plan.h:16-25) and the
// per-step runner (src/execution/layer_runner.cpp:24-67). Kernels are resolved
// and their params built once, at plan-build time; running a step is one
// indirect call with no lookup and no allocation.
// ---------------------------------------------------------------------------
struct ExecutionStep {
    OpType op = OpType::kUnknown;
    ResolvedKernel kernel{};
    alignas(16) std::array<std::byte, kMaxKernelParamsSize> params{};
    std::vector<std::byte> attrs;
    const void* packed_weights = nullptr;
    size_t workspace_offset = 0, workspace_size = 0;
    bool kv_alias = false;  // reads/writes the KV cache
    std::string label;
    // Non-registry steps (collectives, decode bookkeeping): called instead of
    // the kernel when set.
    Status (*host_fn)(void* ctx, cudaStream_t s) noexcept = nullptr;
    void* host_ctx = nullptr;
};

struct ExecutionPlan {
    ExecPhase phase = ExecPhase::kBoth;
    std::vector<ExecutionStep> steps;
    size_t workspace_bytes = 0;
    // Contexts of this plan's host steps (ExecutionStep::host_ctx points into
    // them): they live exactly as long as the plan.
    std::vector<std::shared_ptr<void>> host_ctx_owned;
};

class LayerRunner {
public:
    Status Run(const ExecutionPlan& plan, Stream& stream, WorkspaceArena* ws, const KVCacheView* kv) const;
    Status RunStep(const ExecutionPlan& plan, size_t i, Stream& stream, WorkspaceArena* ws,
                   const KVCacheView* kv) const;
};

class Executor {
public:
    Status Execute(const ExecutionPlan& plan, Stream& stream, WorkspaceArena* ws, const KVCacheView* kv) const {
        return runner_.Run(plan, stream, ws, kv);
    }

private:
    LayerRunner runner_;
};

// ---------------------------------------------------------------------------
// Tensor-parallel communicator over NCCL (loaded at run time).
// ---------------------------------------------------------------------------
class Communicator {
public:
    ~Communicator();
    Status Init(int rank, int world, const void* unique_id);
    Status AllReduceSumBf16(void* buf, size_t count, cudaStream_t s);
    Status AllReduceSumF32(void* buf, size_t count, cudaStream_t s);
    int rank() const { return rank_; }
    int world() const { return world_; }
    bool active() const { return comm_ != nullptr; }

    // One-shot all-reduce over peer memory (no NCCL): this rank's exchange
    // area is exported as a CUDA IPC handle, the peers' areas are opened from
    // theirs; then x += sum of the ranks' partials runs as one kernel.
    Status PeerHandle(void* out64);
    Status OpenPeers(const void* handles);  // world x 64 bytes, rank order
    bool OneShotReady(int64_t n) const;
    Status AllReduceAddBf16(const void* part, void* x, int64_t n, cudaStream_t s);
    // Bound of the one-shot all-reduce's wait for the peers (0: about 2 s).
    void set_wait_ns(uint64_t ns) { wait_ns_ = ns; }
    // The peer areas for a GEMV whose epilogue sums the ranks' partials
    // (AmcuLinearArgs::peer_reduce); null until OpenPeers succeeded.
    const AmcuAllReduceArgs* PeerReduceArgs() const { return peers_open_ ? &peer_args_ : nullptr; }

private:
    void* comm_ = nullptr;
    int rank_ = 0, world_ = 1;
    void* area_ = nullptr;          // this rank's exchange area
    void* peers_[8] = {};           // every rank's area as mapped here
    bool peers_open_ = false;
    uint64_t wait_ns_ = 0;
    AmcuAllReduceArgs peer_args_{};
};
Status NcclGetUniqueId(void* out128);

}  // namespace aethermind
