// Llama model, session and the am_* session C ABI.
//
// The per-layer op order is that of ModelGraphBuilder::BuildLlamaDense
// (src/model/model_graph_builder.cpp:133-419) with the fusions listed in
// cuda_kernels.cpp. A plan is built once per (phase, batch, rows-per-sequence):
// every kernel is resolved through the CudaBackend and its params are baked, so
// running it is a loop of indirect calls. The decode plan plus the decode
// bookkeeping kernel is captured once into a CUDA graph and replayed per token;
// all loop state (current token, positions, output buffer) lives in HBM, so a
// whole generation needs one host->device copy in and one device->host copy out.
//
// Tensor parallelism (tp_size > 1): q/k/v and gate/up are split by output rows
// (heads / intermediate columns), o and down by input columns; each rank holds
// n_kv/tp KV heads of the cache. o and down write partial sums that one NCCL
// all-reduce per block combines before the residual add.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "amcu_internal.h"
#include "kernels/decode_state.cuh"
#include "runtime/engine.h"
#include "runtime/hf_checkpoint.h"

namespace aethermind {
namespace {

thread_local std::string g_err;
am_status_code Fail(const Status& s) {
    g_err = s.ToString();
    return s.am_code();
}

Status CudaOk(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return Status::Ok();
    cudaGetLastError();
    return Status::Internal(std::string(what) + ": " + cudaGetErrorString(e));
}
#define AM_CUDA(call) AM_RETURN_IF_ERROR(CudaOk((call), #call))

DType FromAmDtype(int32_t d) {
    switch (d) {
        case AMCU_F32: return DType::kF32;
        case AMCU_BF16: return DType::kBF16;
        default: return DType::kUndefined;
    }
}

struct LinearWeight {
    AmcuWeight w{};
    DeviceBuffer q, s;
};

}  // namespace
}  // namespace aethermind

struct am_runtime_s {
    int device = 0;
    int tp_rank = 0, tp_size = 1;
    std::unique_ptr<aethermind::CudaAllocator> alloc;
    std::unique_ptr<aethermind::CudaBackend> backend;
    aethermind::Communicator comm;
    cudaStream_t stream = nullptr;
};

struct am_model_s {
    am_runtime_s* rt = nullptr;
    am_model_config_t cfg{};
    int64_t nq_l = 0, nkv_l = 0, inter_l = 0, qkv_n = 0;
    aethermind::DType act = aethermind::DType::kUndefined;
    aethermind::DeviceBuffer embed, embed_scales, final_norm;
    aethermind::LinearWeight lm_head;
    struct Layer {
        aethermind::DeviceBuffer attn_norm, mlp_norm;
        aethermind::LinearWeight qkv, o, gu, d;
        aethermind::DeviceBuffer gate_q, gate_s;  // canonical gate staged until "wu" arrives
    };
    std::vector<Layer> layers;
};

namespace aethermind {
namespace {

// Host -> device copy ordered on the engine's stream and complete on return.
// (A plain cudaMemcpy from pageable memory may return before its DMA lands,
// and the engine's non-blocking stream is not ordered after it.)
cudaError_t UploadSync(am_model_s* m, void* dst, const void* src, size_t bytes) {
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, m->rt->stream);
    if (e != cudaSuccess) return e;
    return cudaStreamSynchronize(m->rt->stream);
}

int64_t WeightBytes(const am_model_config_t& c, int64_t n, int64_t k) {
    return amcu_packed_weight_bytes(c.weight_format, c.act_dtype, n, k, c.group_size);
}
int64_t ScaleBytes(const am_model_config_t& c, int64_t n, int64_t k) {
    return amcu_packed_scale_bytes(c.weight_format, n, k, c.group_size);
}

Status AllocLinear(am_model_s* m, LinearWeight& lw, int64_t n, int64_t k, bool gate_up) {
    const auto& c = m->cfg;
    auto q = m->rt->alloc->Allocate(WeightBytes(c, n, k));
    if (!q.ok()) return q.status();
    lw.q = std::move(q.value());
    if (ScaleBytes(c, n, k) > 0) {  // INT8; INT4 scales live inside the packed weight
        auto s = m->rt->alloc->Allocate(ScaleBytes(c, n, k));
        if (!s.ok()) return s.status();
        lw.s = std::move(s.value());
    }
    lw.w.format = c.weight_format;
    lw.w.dtype = c.act_dtype;
    lw.w.n = n;
    lw.w.k = k;
    lw.w.group = c.group_size;
    lw.w.data = lw.q.data();
    lw.w.scales = lw.s.data();
    lw.w.gate_up_interleaved = gate_up ? 1 : 0;
    return Status::Ok();
}

Status AllocVec(am_model_s* m, DeviceBuffer& b, size_t bytes) {
    auto r = m->rt->alloc->Allocate(bytes);
    if (!r.ok()) return r.status();
    b = std::move(r.value());
    return Status::Ok();
}

// Canonical per-row byte counts (weights, scales).
size_t RowBytes(const am_model_config_t& c, int64_t k) {
    if (c.weight_format == AMCU_WFMT_INT4) return k / 2;
    if (c.weight_format == AMCU_WFMT_INT8) return k;
    return k * (c.act_dtype == AMCU_F32 ? 4 : 2);
}
size_t ScaleRowBytes(const am_model_config_t& c, int64_t k) {
    if (c.weight_format == AMCU_WFMT_INT4) return (k / c.group_size) * 2;
    if (c.weight_format == AMCU_WFMT_INT8) return 4;
    return 0;
}

// A canonical matrix resident on the device (full or already sharded).
struct Canon {
    DeviceBuffer q, s;
    int64_t n = 0, k = 0;
};

// Copies rows [r0, r0+nr) x columns [c0, c0+nc) of a canonical matrix that is
// on the device (src) into a new compact canonical matrix.
Status SliceCanon(am_model_s* m, const Canon& src, int64_t r0, int64_t nr, int64_t c0, int64_t nc, Canon& dst) {
    const auto& c = m->cfg;
    cudaStream_t s = m->rt->stream;
    dst.n = nr;
    dst.k = nc;
    AM_RETURN_IF_ERROR(AllocVec(m, dst.q, RowBytes(c, nc) * nr));
    const size_t sp = RowBytes(c, src.k), dp = RowBytes(c, nc);
    const size_t off = RowBytes(c, c0);  // c0 multiple of the group size -> whole bytes
    AM_CUDA(cudaMemcpy2DAsync(dst.q.data(), dp, src.q.as<char>() + r0 * sp + off, sp, dp, nr,
                              cudaMemcpyDeviceToDevice, s));
    if (c.weight_format != AMCU_WFMT_PLAIN) {
        AM_RETURN_IF_ERROR(AllocVec(m, dst.s, ScaleRowBytes(c, nc) * nr));
        const size_t ssp = ScaleRowBytes(c, src.k), sdp = ScaleRowBytes(c, nc);
        const size_t soff = c.weight_format == AMCU_WFMT_INT4 ? (c0 / c.group_size) * 2 : 0;
        AM_CUDA(cudaMemcpy2DAsync(dst.s.data(), sdp, src.s.as<char>() + r0 * ssp + soff, ssp, sdp, nr,
                                  cudaMemcpyDeviceToDevice, s));
    }
    return CudaOk(cudaStreamSynchronize(s), "shard copy");  // src may be freed next
}

// Prepacks a canonical matrix into rows [row0, row0 + n) of a device weight.
Status PackInto(am_model_s* m, LinearWeight& lw, int64_t row0, const Canon& cn) {
    const auto& c = m->cfg;
    am_status_code st = amcu_prepack_weight_rows(c.weight_format, c.act_dtype, cn.n, cn.k, c.group_size, lw.w.n,
                                                 row0, cn.q.data(), cn.s.data(), lw.q.data(), lw.s.data(),
                                                 m->rt->stream);
    AM_RETURN_IF_ERROR(Status::FromAm(st, amcu_last_error()));
    // The canonical staging buffers are freed by the caller right after this;
    // the copy on the engine's non-blocking stream must have read them first.
    return CudaOk(cudaStreamSynchronize(m->rt->stream), "prepack");
}

enum class Split { kNone, kRows, kCols };

// This rank's block of an [n, k] tensor under a split: rows [r0, r0 + nr) x
// columns [c0, c0 + nc). Rows: column-parallel (q/k/v by heads, gate/up by
// intermediate columns); columns: row-parallel (o, down), at boundaries that
// stay multiples of 128 when the shapes are (checked at model creation).
void ShardRange(Split sp, int64_t n, int64_t k, int r, int w, int64_t& r0, int64_t& nr, int64_t& c0, int64_t& nc) {
    r0 = 0, nr = n, c0 = 0, nc = k;
    if (w <= 1 || sp == Split::kNone) return;
    if (sp == Split::kRows) {
        nr = n / w;
        r0 = r * nr;
    } else {
        nc = k / w;
        c0 = r * nc;
    }
}

// Full canonical tensor (device) -> this rank's shard.
Status Shard(am_model_s* m, Canon& full, Split sp, int64_t unit, Canon& out) {
    const int r = m->rt->tp_rank, w = m->rt->tp_size;
    (void)unit;
    if (w == 1 || sp == Split::kNone) {
        out = std::move(full);
        return Status::Ok();
    }
    int64_t r0, nr, c0, nc;
    ShardRange(sp, full.n, full.k, r, w, r0, nr, c0, nc);
    return SliceCanon(m, full, r0, nr, c0, nc, out);
}

Status UploadCanon(am_model_s* m, int64_t n, int64_t k, const void* hq, const void* hs, Canon& out) {
    const auto& c = m->cfg;
    out.n = n;
    out.k = k;
    AM_RETURN_IF_ERROR(AllocVec(m, out.q, RowBytes(c, k) * n));
    AM_CUDA(UploadSync(m, out.q.data(), hq, RowBytes(c, k) * n));
    if (c.weight_format != AMCU_WFMT_PLAIN) {
        if (!hs) return Status::InvalidArgument("quantized weight needs scales");
        AM_RETURN_IF_ERROR(AllocVec(m, out.s, ScaleRowBytes(c, k) * n));
        AM_CUDA(UploadSync(m, out.s.data(), hs, ScaleRowBytes(c, k) * n));
    }
    return Status::Ok();
}

constexpr float kW4Base = 0.02f / 4.6098f;   // std of uniform ints in [-8, 7]
constexpr float kW8Base = 0.02f / 73.61f;    // std of uniform ints in [-127, 127]
constexpr float kEmbedAmp = 0.0692820f;      // uniform(-a/2, a/2) with std 0.02

Status SynthCanon(am_model_s* m, uint64_t seed, uint64_t stream_id, int64_t n, int64_t k, Canon& out) {
    const auto& c = m->cfg;
    out.n = n;
    out.k = k;
    AM_RETURN_IF_ERROR(AllocVec(m, out.q, RowBytes(c, k) * n));
    am_status_code st;
    if (c.weight_format == AMCU_WFMT_INT4) {
        AM_RETURN_IF_ERROR(AllocVec(m, out.s, ScaleRowBytes(c, k) * n));
        st = amcu_synth_w4(seed, stream_id, n, k, kW4Base, out.q.data(), out.s.data(), m->rt->stream);
    } else if (c.weight_format == AMCU_WFMT_INT8) {
        AM_RETURN_IF_ERROR(AllocVec(m, out.s, ScaleRowBytes(c, k) * n));
        st = amcu_synth_w8(seed, stream_id, n, k, kW8Base, out.q.data(), out.s.data(), m->rt->stream);
    } else if (c.act_dtype == AMCU_BF16) {
        st = amcu_synth_uniform_bf16(seed, stream_id, n * k, kEmbedAmp, out.q.data(), m->rt->stream);
    } else {
        return Status::Unimplemented("synthetic weights for plain fp32 models are not generated on device");
    }
    return Status::FromAm(st, amcu_last_error());
}

// Which fused weight / row offset a per-matrix name maps to.
struct Target {
    LinearWeight* lw = nullptr;
    int64_t row0 = 0;
    int64_t n_full = 0, k_full = 0;
    Split split = Split::kNone;
    int kind = 0;  // 0 plain, 1 gate (staged), 2 up (pack with staged gate)
};

Status ResolveTarget(am_model_s* m, int layer, const std::string& t, Target& tg) {
    const auto& c = m->cfg;
    auto& L = m->layers[layer];
    const int64_t d = c.head_dim;
    if (t == "wq") tg = {&L.qkv, 0, c.n_q_heads * d, c.hidden, Split::kRows, 0};
    else if (t == "wk") tg = {&L.qkv, m->nq_l * d, c.n_kv_heads * d, c.hidden, Split::kRows, 0};
    else if (t == "wv") tg = {&L.qkv, (m->nq_l + m->nkv_l) * d, c.n_kv_heads * d, c.hidden, Split::kRows, 0};
    else if (t == "wo") tg = {&L.o, 0, c.hidden, c.n_q_heads * d, Split::kCols, 0};
    else if (t == "wg") tg = {&L.gu, 0, c.inter, c.hidden, Split::kRows, 1};
    else if (t == "wu") tg = {&L.gu, 0, c.inter, c.hidden, Split::kRows, 2};
    else if (t == "wd") tg = {&L.d, 0, c.hidden, c.inter, Split::kCols, 0};
    else return Status::NotFound("unknown layer tensor '" + t + "'");
    return Status::Ok();
}

Status StoreLinear(am_model_s* m, int layer, Target& tg, Canon& shard) {
    const auto& c = m->cfg;
    if (tg.kind == 0) return PackInto(m, *tg.lw, tg.row0, shard);
    auto& L = m->layers[layer];
    if (tg.kind == 1) {
        L.gate_q = std::move(shard.q);
        L.gate_s = std::move(shard.s);
        return Status::Ok();
    }
    if (!L.gate_q.is_initialized()) return Status::FailedPrecondition("set 'wg' before 'wu'");
    am_status_code st = amcu_prepack_gate_up(c.weight_format, c.act_dtype, shard.n, shard.k, c.group_size,
                                             L.gate_q.data(), L.gate_s.data(), shard.q.data(), shard.s.data(),
                                             tg.lw->q.data(), tg.lw->s.data(), m->rt->stream);
    AM_RETURN_IF_ERROR(Status::FromAm(st, amcu_last_error()));
    AM_CUDA(cudaStreamSynchronize(m->rt->stream));
    L.gate_q = DeviceBuffer();
    L.gate_s = DeviceBuffer();
    return Status::Ok();
}

// ------------------------------------------------------------------ session

struct AllReduceCtx {
    Communicator* comm;
    void* buf;
    size_t count;
};
Status AllReduceStep(void* ctx, cudaStream_t s) noexcept {
    auto* a = static_cast<AllReduceCtx*>(ctx);
    return a->comm->AllReduceSumBf16(a->buf, a->count, s);
}
// x += all-reduce(partial) in one kernel over peer memory
struct PeerAllReduceCtx {
    Communicator* comm;
    const void* part;
    void* x;
    int64_t count;
};
Status PeerAllReduceAddStep(void* ctx, cudaStream_t s) noexcept {
    auto* a = static_cast<PeerAllReduceCtx*>(ctx);
    return a->comm->AllReduceAddBf16(a->part, a->x, a->count, s);
}

}  // namespace
}  // namespace aethermind

struct am_session_s {
    am_model_s* m = nullptr;
    am_session_config_t cfg{};
    aethermind::KVCacheManager kv;
    aethermind::WorkspaceArena ws;
    aethermind::Executor exec;
    aethermind::DeviceBuffer tokens, next_tok, seq_pos, counter, out_tokens, gaps, gap_tmp, status;
    aethermind::DeviceBuffer x, h, qkv, attn, act, part, hlast, logits;
    aethermind::DeviceBuffer rope_table;  // [max_seq][head_dim/2] (cos, sin)
    // persistent decode step: per-layer descriptor table and its workspace
    // (zeroed once; its counters reset themselves after every launch)
    aethermind::DeviceBuffer stack_layers, stack_ws;
    bool graph_unsupported = false;  // decode plan could not be captured: eager decode
    int64_t rows_cap = 0, out_cap = 0;
    // plans
    aethermind::ExecutionPlan prefill, decode;
    int64_t prefill_B = -1, prefill_R = -1, decode_B = -1;
    cudaGraphExec_t graph = nullptr;
    int64_t graph_B = -1;
    void* pinned = nullptr;
    size_t pinned_bytes = 0;
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
    double last_prefill_ms = 0, last_decode_ms = 0;
    int64_t last_steps = 0, last_B = 0, last_N = 0;
    std::vector<float> last_gaps;
};

namespace aethermind {
namespace {

Status EnsureRows(am_session_s* s, int64_t rows) {
    if (rows <= s->rows_cap) return Status::Ok();
    auto* m = s->m;
    const auto& c = m->cfg;
    const size_t e = DTypeBytes(m->act);
    auto& A = *m->rt->alloc;
    auto get = [&](DeviceBuffer& b, size_t bytes) -> Status {
        auto r = A.Allocate(bytes);
        if (!r.ok()) return r.status();
        b = std::move(r.value());
        return Status::Ok();
    };
    AM_RETURN_IF_ERROR(get(s->tokens, rows * 8));
    AM_RETURN_IF_ERROR(get(s->x, rows * c.hidden * e));
    AM_RETURN_IF_ERROR(get(s->h, rows * c.hidden * e));
    AM_RETURN_IF_ERROR(get(s->qkv, rows * m->qkv_n * e));
    AM_RETURN_IF_ERROR(get(s->attn, rows * m->nq_l * c.head_dim * e));
    AM_RETURN_IF_ERROR(get(s->act, rows * m->inter_l * e));
    AM_RETURN_IF_ERROR(get(s->part, rows * c.hidden * e));
    s->rows_cap = rows;
    s->prefill_B = -1;  // buffers moved: plans must be rebuilt
    s->decode_B = -1;
    if (s->graph) {
        cudaGraphExecDestroy(s->graph);
        s->graph = nullptr;
        s->graph_B = -1;
    }
    return Status::Ok();
}

struct PlanBuilder {
    am_session_s* s;
    am_model_s* m;
    ExecutionPlan* plan;
    ExecPhase phase;

    KernelSelector Sel(DType act, DType wdt, WeightFormat f) const {
        return KernelSelector{DeviceType::kCUDA, act, wdt, f, IsaLevel::kScalar, phase};
    }
    template <typename A>
    Status Add(OpType op, const KernelSelector& sel, std::initializer_list<TensorView> in,
               std::initializer_list<MutableTensorView> out, const A* attrs, const void* packed,
               const std::string& label, bool kv = false) {
        auto r = m->rt->backend->ResolveKernelInfo(op, sel);
        if (!r.ok()) return r.status();
        ExecutionStep st;
        st.op = op;
        st.kernel = r.value();
        st.label = label;
        st.kv_alias = kv;
        st.packed_weights = packed;
        if (attrs) {
            st.attrs.resize(sizeof(A));
            std::memcpy(st.attrs.data(), attrs, sizeof(A));
        }
        std::vector<TensorView> iv(in);
        std::vector<MutableTensorView> ov(out);
        AM_RETURN_IF_ERROR(st.kernel.params_builder(iv, ov, std::span<const std::byte>(st.attrs.data(), st.attrs.size()),
                                                    packed, st.params.data()));
        // workspace needs
        if (op == OpType::kLinear) {
            st.workspace_size = amcu_linear_workspace_bytes(reinterpret_cast<const AmcuLinearArgs*>(st.params.data()));
        } else if (op == OpType::kArgmax) {
            st.workspace_size = amcu_argmax_workspace_bytes(in.begin()->dim(0));  // one partial set per row
        } else if (op == OpType::kAttention && phase == ExecPhase::kDecode) {
            st.workspace_size =
                    amcu_attention_workspace_bytes(reinterpret_cast<const AmcuAttentionArgs*>(st.params.data()));
        }
        if (st.workspace_size > plan->workspace_bytes) plan->workspace_bytes = st.workspace_size;
        plan->steps.push_back(std::move(st));
        return Status::Ok();
    }
};

TensorView View2(const void* p, DType dt, int64_t rows, int64_t cols, int64_t stride) {
    TensorView v = MakeView(p, dt, {rows, cols});
    v.strides[0] = stride;
    return v;
}
MutableTensorView MView2(void* p, DType dt, int64_t rows, int64_t cols, int64_t stride) {
    MutableTensorView v = MakeMutableView(p, dt, {rows, cols});
    v.strides[0] = stride;
    return v;
}

// Weight prefetch across kernel boundaries (off unless AMCU_L2_HINTS asks):
// a quantized Linear step can ask for the next Linear step's weights and
// scales to be pulled into L2 while it runs (the last step of the plan asks
// for the first one's, which the next decode step reads), and for the one
// after that too when the next weight is small. Measured on the 8B batch-1
// decode step, the hints cost more than they save: the prefetch traffic
// (67 MB asked for by each q/k/v projection) competes with the latency-bound
// loads of the kernels in between. Per-launch timeline, us per layer:
// q/k/v 9.5 -> 7.6, o 6.4 -> 5.5, down 13.7 -> 12.8 without hints; decode
// 581 -> 624 tok/s, batch 8 3004 -> 3249, 70B 90.2 -> 96.8, 1B 1530 -> 1505.
void SetL2Hints(ExecutionPlan& plan) {
    constexpr uint64_t kMaxRange = 64ull << 20;   // L2 is 126 MB
    constexpr uint64_t kSmallWeight = 16ull << 20;
    std::vector<size_t> lin;
    for (size_t i = 0; i < plan.steps.size(); ++i) {
        const auto* w = static_cast<const AmcuWeight*>(plan.steps[i].packed_weights);
        if (plan.steps[i].op == OpType::kLinear && w && w->format != AMCU_WFMT_PLAIN) lin.push_back(i);
    }
    // AMCU_L2_HINTS: 0 (default) = no hints, 1 = the next weight only,
    // 2 = the next weight and, after a small one, the one after it
    static const int mode = [] {
        const char* v = std::getenv("AMCU_L2_HINTS");
        return v ? std::atoi(v) : 0;
    }();
    if (lin.size() < 2 || mode == 0) return;
    auto weight_of = [&](size_t j) { return static_cast<const AmcuWeight*>(plan.steps[lin[j % lin.size()]].packed_weights); };
    auto wbytes = [](const AmcuWeight* w) {
        return (uint64_t)amcu_packed_weight_bytes(w->format, w->dtype, w->n, w->k, w->group);
    };
    for (size_t j = 0; j < lin.size(); ++j) {
        AmcuL2Prefetch h{};
        int slot = 0;
        for (size_t ahead = 1; ahead <= 2 && slot + 2 <= 4; ++ahead) {
            const AmcuWeight* w = weight_of(j + ahead);
            const uint64_t b = wbytes(w);
            h.ptr[slot] = w->data;
            h.bytes[slot++] = b < kMaxRange ? b : kMaxRange;
            h.ptr[slot] = w->scales;
            h.bytes[slot++] = (uint64_t)amcu_packed_scale_bytes(w->format, w->n, w->k, w->group);
            if (b >= kSmallWeight || mode == 1) break;
        }
        reinterpret_cast<AmcuLinearArgs*>(plan.steps[lin[j]].params.data())->l2_next = h;
    }
}

Status BuildPlan(am_session_s* s, ExecPhase phase, int64_t B, int64_t R, ExecutionPlan& plan) {
    am_model_s* m = s->m;
    const auto& c = m->cfg;
    const DType A = m->act;
    const int64_t M = B * R, H = c.hidden, d = c.head_dim;
    const size_t e = DTypeBytes(A);
    plan = ExecutionPlan{};
    plan.phase = phase;
    PlanBuilder pb{s, m, &plan, phase};
    const WeightFormat wf = c.weight_format == AMCU_WFMT_INT4   ? WeightFormat::kQuantizedInt4
                            : c.weight_format == AMCU_WFMT_INT8 ? WeightFormat::kQuantizedInt8
                                                                 : WeightFormat::kPlain;
    const DType wdt = wf == WeightFormat::kQuantizedInt4 ? DType::kI4 : wf == WeightFormat::kQuantizedInt8 ? DType::kI8 : A;
    const KernelSelector lin = pb.Sel(A, wdt, wf);
    const KernelSelector act = pb.Sel(A, A, WeightFormat::kPlain);
    const bool tp = m->rt->tp_size > 1;
    // Decode GEMVs (m <= 8) stage their activations anyway: the RMSNorm in
    // front of q/k/v and gate/up runs there instead of as its own kernel.
    const bool fuse_norm = phase == ExecPhase::kDecode && wf != WeightFormat::kPlain && M <= 8;
    // decode attention blocks (one row per sequence, any batch) as one fused
    // RoPE + attention launch where a kernel for it is registered (bf16) and
    // the session does not ask for the unfused steps
    const bool fuse_attn = phase == ExecPhase::kDecode && R == 1 && s->cfg.unfused_attention == 0 &&
                           m->rt->backend->ResolveKernelInfo(OpType::kRoPEAttention, act).ok();
    // Embedding
    {
        const bool tied_i8 = c.tied_embeddings && wf == WeightFormat::kQuantizedInt8;
        EmbeddingAttrs ea{tied_i8 ? m->embed_scales.as<float>() : nullptr, s->status.as<int32_t>()};
        TensorView ids = MakeView(phase == ExecPhase::kPrefill ? s->tokens.data() : s->next_tok.data(), DType::kI64, {M});
        TensorView table = MakeView(m->embed.data(), tied_i8 ? DType::kI8 : A, {c.vocab, H});
        AM_RETURN_IF_ERROR(pb.Add(OpType::kEmbedding, tied_i8 ? pb.Sel(A, DType::kI8, WeightFormat::kQuantizedInt8) : act,
                                  {ids, table}, {MView2(s->x.data(), A, M, H, H)}, &ea, nullptr, "embedding"));
    }
    RmsNormAttrs na{c.rms_eps};
    // Decode of a batch-1 INT4 model on one GPU: every decoder layer in one
    // persistent launch (amcu_decode_stack), when the session asks for it.
    const KernelSelector stack_sel = pb.Sel(A, DType::kI4, WeightFormat::kQuantizedInt4);
    const bool use_stack = phase == ExecPhase::kDecode && R == 1 && B == 1 && !tp &&
                           wf == WeightFormat::kQuantizedInt4 && A == DType::kBF16 &&
                           s->cfg.persistent_decode != 0 && c.hidden <= 16384 && m->inter_l <= 16384 &&
                           m->nq_l * d <= 16384 && m->rt->backend->ResolveKernelInfo(OpType::kDecodeStack, stack_sel).ok();
    if (use_stack) {
        std::vector<AmcuDecodeLayer> tab(c.layers);
        for (int64_t l = 0; l < c.layers; ++l) {
            auto& L = m->layers[l];
            tab[l] = AmcuDecodeLayer{L.qkv.w.data, L.o.w.data, L.gu.w.data, L.d.w.data, L.attn_norm.data(),
                                     L.mlp_norm.data(), s->kv.key_plane(l), s->kv.value_plane(l)};
        }
        if (!s->stack_layers.is_initialized() || s->stack_layers.size() < tab.size() * sizeof(AmcuDecodeLayer))
            AM_RETURN_IF_ERROR(AllocVec(m, s->stack_layers, tab.size() * sizeof(AmcuDecodeLayer)));
        AM_CUDA(UploadSync(m, s->stack_layers.data(), tab.data(), tab.size() * sizeof(AmcuDecodeLayer)));
        AmcuDecodeStackArgs a{};
        a.layers = static_cast<const AmcuDecodeLayer*>(s->stack_layers.data());
        a.n_layers = c.layers;
        a.batch = B;
        a.hidden = H;
        a.inter = m->inter_l;
        a.n_q_heads = m->nq_l;
        a.n_kv_heads = m->nkv_l;
        a.head_dim = d;
        a.x = s->x.data();
        a.qkv = s->qkv.data();
        a.attn = s->attn.data();
        a.act = s->act.data();
        a.seq_pos = s->seq_pos.as<int32_t>();
        a.capacity = (int64_t)s->kv.layout().max_tokens;
        a.slot_stride = (int64_t)(s->kv.layout().slot_stride / e);
        a.cos_sin = s->rope_table.as<float>();
        a.theta = c.rope_theta;
        a.rms_eps = c.rms_eps;
        a.status = s->status.as<int32_t>();
        const size_t wsb = amcu_decode_stack_workspace_bytes(&a);
        if (!s->stack_ws.is_initialized() || s->stack_ws.size() < wsb) {
            AM_RETURN_IF_ERROR(AllocVec(m, s->stack_ws, wsb));
            AM_CUDA(cudaMemsetAsync(s->stack_ws.data(), 0, wsb, m->rt->stream));
            AM_CUDA(cudaStreamSynchronize(m->rt->stream));
        }
        a.workspace = s->stack_ws.data();
        a.workspace_size = s->stack_ws.size();
        AM_RETURN_IF_ERROR(pb.Add(OpType::kDecodeStack, stack_sel, {}, {}, &a, nullptr, "decoder_layers (persistent)", true));
    }
    for (int64_t l = 0; l < (use_stack ? 0 : c.layers); ++l) {
        auto& L = m->layers[l];
        const std::string p = "layer" + std::to_string(l) + ".";
        LinearAttrs store{AMCU_EPI_STORE};
        if (fuse_norm) {  // attn_norm folded into the q/k/v GEMV's activation staging
            LinearAttrs qa{AMCU_EPI_STORE, L.attn_norm.data(), c.rms_eps};
            AM_RETURN_IF_ERROR(pb.Add(OpType::kLinear, lin, {View2(s->x.data(), A, M, H, H)},
                                      {MView2(s->qkv.data(), A, M, m->qkv_n, m->qkv_n)}, &qa, &L.qkv.w,
                                      p + "attn_norm+qkv_proj"));
        } else {
            AM_RETURN_IF_ERROR(pb.Add(OpType::kRmsNorm, act,
                                      {View2(s->x.data(), A, M, H, H), MakeView(L.attn_norm.data(), A, {H})},
                                      {MView2(s->h.data(), A, M, H, H)}, &na, nullptr, p + "attn_norm"));
            AM_RETURN_IF_ERROR(pb.Add(OpType::kLinear, lin, {View2(s->h.data(), A, M, H, H)},
                                      {MView2(s->qkv.data(), A, M, m->qkv_n, m->qkv_n)}, &store, &L.qkv.w,
                                      p + "qkv_proj"));
        }
        const int64_t qn = m->nq_l * d, kn = m->nkv_l * d;
        char* qkv = s->qkv.as<char>();
        RopeKvAttrs ra{c.rope_theta, R, (int64_t)s->kv.layout().max_tokens,
                       (int64_t)(s->kv.layout().slot_stride / e), m->nq_l, m->nkv_l, d, s->seq_pos.as<int32_t>(),
                       s->status.as<int32_t>(), s->rope_table.as<float>()};
        TensorView q = View2(qkv, A, M, qn, m->qkv_n), k = View2(qkv + qn * e, A, M, kn, m->qkv_n),
                   v = View2(qkv + (qn + kn) * e, A, M, kn, m->qkv_n);
        MutableTensorView qo = MView2(qkv, A, M, qn, m->qkv_n);
        MutableTensorView kc = MakeMutableView(s->kv.key_plane(l), A, {(int64_t)s->kv.layout().num_slots, m->nkv_l,
                                                                      (int64_t)s->kv.layout().max_tokens, d});
        MutableTensorView vc = MakeMutableView(s->kv.value_plane(l), A, {(int64_t)s->kv.layout().num_slots, m->nkv_l,
                                                                        (int64_t)s->kv.layout().max_tokens, d});
        AttentionAttrs aa{R, (int64_t)s->kv.layout().max_tokens, (int64_t)(s->kv.layout().slot_stride / e), m->nq_l,
                          m->nkv_l, d, c.max_seq, s->seq_pos.as<int32_t>(), 0};
        if (fuse_attn) {  // RoPE + KV append + attention in one launch
            RopeAttentionAttrs fa{ra, aa};
            TensorView kcv = MakeView(kc.data, A, {(int64_t)s->kv.layout().num_slots, m->nkv_l,
                                                   (int64_t)s->kv.layout().max_tokens, d});
            TensorView vcv = MakeView(vc.data, A, {(int64_t)s->kv.layout().num_slots, m->nkv_l,
                                                   (int64_t)s->kv.layout().max_tokens, d});
            AM_RETURN_IF_ERROR(pb.Add(OpType::kRoPEAttention, act, {q, k, v, kcv, vcv},
                                      {MView2(s->attn.data(), A, M, qn, qn), kc, vc}, &fa, nullptr,
                                      p + "rope_kv_write+attention", true));
        } else {
            AM_RETURN_IF_ERROR(
                    pb.Add(OpType::kRoPE, act, {q, k, v}, {qo, kc, vc}, &ra, nullptr, p + "rope_kv_write", true));
            AM_RETURN_IF_ERROR(pb.Add(OpType::kAttention, act, {q, kc, vc}, {MView2(s->attn.data(), A, M, qn, qn)},
                                      &aa, nullptr, p + "attention", true));
        }
        auto residual_block = [&](LinearWeight& W, const TensorView& in, const std::string& name) -> Status {
            if (!tp) {
                LinearAttrs res{AMCU_EPI_RESIDUAL_ADD};
                return pb.Add(OpType::kLinear, lin, {in, View2(s->x.data(), A, M, H, H)}, {MView2(s->x.data(), A, M, H, H)},
                              &res, &W.w, p + name);
            }
            // decode GEMV on 2 ranks: the partials are summed over peer memory
            // in the GEMV's own epilogue, residual added there (one launch).
            // On 2 B200s the 8B decode step measured 1.937 ms/token fused,
            // 1.941 with the one-shot kernel, 2.035 with NCCL. From 3 ranks the
            // separate one-shot kernel: each row block's wait for every peer
            // holds its CTA in step with the slowest rank, which on 4 B200s
            // cost 2.59 ms/token against 1.71 with the one-shot kernel (2.07
            // with NCCL). AMCU_TP_FUSED_ALLREDUCE=0 / =1 forces either way.
            static const int fused_env = [] {
                const char* v = std::getenv("AMCU_TP_FUSED_ALLREDUCE");
                return v ? (v[0] == '0' ? 0 : 1) : -1;
            }();
            const bool fused_ok = fused_env == 1 || (fused_env < 0 && m->rt->tp_size <= 2);
            if (fused_ok && phase == ExecPhase::kDecode && M <= 8 && wf != WeightFormat::kPlain && A == DType::kBF16 &&
                m->rt->comm.PeerReduceArgs() != nullptr && H * 8 <= 16384 * 8) {
                LinearAttrs res{AMCU_EPI_RESIDUAL_ADD};
                res.peer_reduce = m->rt->comm.PeerReduceArgs();
                return pb.Add(OpType::kLinear, lin, {in, View2(s->x.data(), A, M, H, H)},
                              {MView2(s->x.data(), A, M, H, H)}, &res, &W.w, p + name + "+allreduce(peer)");
            }
            AM_RETURN_IF_ERROR(pb.Add(OpType::kLinear, lin, {in}, {MView2(s->part.data(), A, M, H, H)}, &store, &W.w,
                                      p + name + "_partial"));
            if (A == DType::kBF16 && m->rt->comm.OneShotReady(M * H)) {
                auto pctx = std::make_shared<PeerAllReduceCtx>(
                        PeerAllReduceCtx{&m->rt->comm, s->part.data(), s->x.data(), M * H});
                ExecutionStep st;
                st.label = p + name + "_allreduce_residual(peer)";
                st.host_fn = PeerAllReduceAddStep;
                st.host_ctx = pctx.get();
                plan.steps.push_back(std::move(st));
                plan.host_ctx_owned.push_back(std::move(pctx));
                return Status::Ok();
            }
            auto ctx = std::make_shared<AllReduceCtx>(AllReduceCtx{&m->rt->comm, s->part.data(), (size_t)(M * H)});
            ExecutionStep st;
            st.label = p + name + "_allreduce";
            st.host_fn = AllReduceStep;
            st.host_ctx = ctx.get();
            plan.steps.push_back(std::move(st));
            plan.host_ctx_owned.push_back(std::move(ctx));
            return pb.Add(OpType::kAdd, act, {View2(s->x.data(), A, M, H, H), View2(s->part.data(), A, M, H, H)},
                          {MView2(s->x.data(), A, M, H, H)}, (const int*)nullptr, nullptr, p + name + "_residual");
        };
        AM_RETURN_IF_ERROR(residual_block(L.o, View2(s->attn.data(), A, M, qn, qn), "o_proj"));
        if (fuse_norm) {  // mlp_norm folded into the gate/up GEMV's activation staging
            LinearAttrs silu{AMCU_EPI_SILU_MUL, L.mlp_norm.data(), c.rms_eps};
            AM_RETURN_IF_ERROR(pb.Add(OpType::kLinear, lin, {View2(s->x.data(), A, M, H, H)},
                                      {MView2(s->act.data(), A, M, m->inter_l, m->inter_l)}, &silu, &L.gu.w,
                                      p + "mlp_norm+gate_up_silu"));
        } else {
            AM_RETURN_IF_ERROR(pb.Add(OpType::kRmsNorm, act,
                                      {View2(s->x.data(), A, M, H, H), MakeView(L.mlp_norm.data(), A, {H})},
                                      {MView2(s->h.data(), A, M, H, H)}, &na, nullptr, p + "mlp_norm"));
            LinearAttrs silu{AMCU_EPI_SILU_MUL};
            AM_RETURN_IF_ERROR(pb.Add(OpType::kLinear, lin, {View2(s->h.data(), A, M, H, H)},
                                      {MView2(s->act.data(), A, M, m->inter_l, m->inter_l)}, &silu, &L.gu.w,
                                      p + "gate_up_silu"));
        }
        AM_RETURN_IF_ERROR(residual_block(L.d, View2(s->act.data(), A, M, m->inter_l, m->inter_l), "down_proj"));
    }
    // final norm on the last row of every sequence
    AM_RETURN_IF_ERROR(pb.Add(OpType::kRmsNorm, act,
                              {View2(s->x.as<char>() + (R - 1) * H * e, A, B, H, R * H), MakeView(m->final_norm.data(), A, {H})},
                              {MView2(s->hlast.data(), A, B, H, H)}, &na, nullptr, "final_norm"));
    LinearAttrs store{AMCU_EPI_STORE};
    AM_RETURN_IF_ERROR(pb.Add(OpType::kLinear, lin, {View2(s->hlast.data(), A, B, H, H)},
                              {MView2(s->logits.data(), A, B, c.vocab, c.vocab)}, &store, &m->lm_head.w, "lm_head"));
    ArgmaxAttrs ga{s->gap_tmp.as<float>()};
    AM_RETURN_IF_ERROR(pb.Add(OpType::kArgmax, act, {View2(s->logits.data(), A, B, c.vocab, c.vocab)},
                              {MakeMutableView(s->next_tok.data(), DType::kI64, {B})}, &ga, nullptr, "argmax"));
    SetL2Hints(plan);
    return Status::Ok();
}

Status EnsureWorkspace(am_session_s* s, const ExecutionPlan& p) {
    return s->ws.Reserve(*s->m->rt->alloc, p.workspace_bytes);
}

Status RunAdvance(am_session_s* s, int64_t B, int32_t set_pos, cudaStream_t st) {
    amcu::launch_advance(s->next_tok.as<int64_t>(), s->gap_tmp.as<float>(), s->out_tokens.as<int64_t>(),
                         s->gaps.as<float>(), s->out_cap, s->seq_pos.as<int32_t>(), s->counter.as<int32_t>(), B,
                         set_pos, st);
    return CudaOk(cudaGetLastError(), "decode advance");
}

Status Generate(am_session_s* s, const uint32_t* in, int64_t B, int64_t P, int64_t N, std::vector<int64_t>& out) {
    am_model_s* m = s->m;
    const auto& c = m->cfg;
    cudaStream_t st = m->rt->stream;
    if (B < 1 || B > c.max_batch) return Status::InvalidArgument("batch must be in [1, max_batch]");
    if (P < 1) return Status::InvalidArgument("input_len must be at least 1");
    if (N < 1) return Status::InvalidArgument("output capacity must be at least 1");
    for (int64_t i = 0; i < B * P; ++i)
        if (in[i] >= (uint32_t)c.vocab) return Status::OutOfRange("input token id out of range");
    auto view = s->kv.ReserveForSession(P, N);
    if (!view.ok()) return view.status();
    KVCacheView kv = view.value();
    struct Release {
        am_session_s* s;
        KVCacheView* v;
        ~Release() { s->kv.ReleaseSession(*v); }
    } rel{s, &kv};

    AM_RETURN_IF_ERROR(EnsureRows(s, B * P));
    if (s->out_cap < N) {
        auto o = m->rt->alloc->Allocate(c.max_batch * N * 8);
        if (!o.ok()) return o.status();
        s->out_tokens = std::move(o.value());
        auto g = m->rt->alloc->Allocate(c.max_batch * N * 4);
        if (!g.ok()) return g.status();
        s->gaps = std::move(g.value());
        s->out_cap = N;
        s->decode_B = -1;
        if (s->graph) { cudaGraphExecDestroy(s->graph); s->graph = nullptr; s->graph_B = -1; }
    }
    if (s->prefill_B != B || s->prefill_R != P) {
        AM_RETURN_IF_ERROR(BuildPlan(s, ExecPhase::kPrefill, B, P, s->prefill));
        s->prefill_B = B;
        s->prefill_R = P;
    }
    if (s->decode_B != B) {
        AM_RETURN_IF_ERROR(BuildPlan(s, ExecPhase::kDecode, B, 1, s->decode));
        s->decode_B = B;
        if (s->graph) { cudaGraphExecDestroy(s->graph); s->graph = nullptr; s->graph_B = -1; }
    }
    AM_RETURN_IF_ERROR(EnsureWorkspace(s, s->prefill));
    AM_RETURN_IF_ERROR(EnsureWorkspace(s, s->decode));

    // stage the prompt (pinned host -> device)
    // pinned staging: prompt [B*P] int64 | tokens [max_batch*out_cap] int64 |
    // gaps [max_batch*out_cap] float | status int32
    const size_t need = B * P * 8 + c.max_batch * s->out_cap * 12 + 16;
    if (s->pinned_bytes < need) {
        if (s->pinned) cudaFreeHost(s->pinned);
        AM_CUDA(cudaMallocHost(&s->pinned, need));
        s->pinned_bytes = need;
    }
    int64_t* hp = static_cast<int64_t*>(s->pinned);
    for (int64_t i = 0; i < B * P; ++i) hp[i] = in[i];
    Stream stream(st);
    AM_CUDA(cudaMemcpyAsync(s->tokens.data(), hp, B * P * 8, cudaMemcpyHostToDevice, st));
    AM_CUDA(cudaMemsetAsync(s->seq_pos.data(), 0, c.max_batch * 4, st));
    AM_CUDA(cudaMemsetAsync(s->counter.data(), 0, 4, st));
    AM_CUDA(cudaMemsetAsync(s->status.data(), 0, 4, st));
    AM_CUDA(cudaEventRecord(s->ev[0], st));
    struct NvtxRange {  // named ranges for profilers (am_prefill / am_decode)
        explicit NvtxRange(const char* n) { nvtxRangePushA(n); }
        ~NvtxRange() { nvtxRangePop(); }
    };
    std::unique_ptr<NvtxRange> range = std::make_unique<NvtxRange>("am_prefill");
    AM_RETURN_IF_ERROR(s->exec.Execute(s->prefill, stream, &s->ws, &kv));
    AM_RETURN_IF_ERROR(RunAdvance(s, B, (int32_t)P, st));
    AM_CUDA(cudaEventRecord(s->ev[1], st));
    // Finish the eagerly launched prefill before the decode loop starts: the
    // decode graph (captured below on first use) reads the positions and the
    // token counter the prefill's last kernel wrote.
    AM_CUDA(cudaStreamSynchronize(st));

    bool use_graph = s->cfg.use_cuda_graph != 0 && !s->graph_unsupported;
    range.reset();
    range = std::make_unique<NvtxRange>("am_decode");
    for (int64_t i = 1; i < N; ++i) {
        if (use_graph && s->graph_B == B) {
            AM_CUDA(cudaGraphLaunch(s->graph, st));
            continue;
        }
        // Eager decode step. The first one also loads every decode kernel's
        // module (CUDA loads modules lazily, on first launch), so nothing is
        // loaded while the decode graph is being captured below.
        AM_RETURN_IF_ERROR(s->exec.Execute(s->decode, stream, &s->ws, &kv));
        AM_RETURN_IF_ERROR(RunAdvance(s, B, -1, st));
        if (use_graph && i + 1 < N) {
            AM_CUDA(cudaStreamSynchronize(st));
            cudaGraph_t g = nullptr;
            AM_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            Status cs = s->exec.Execute(s->decode, stream, &s->ws, &kv);
            if (cs.ok()) cs = RunAdvance(s, B, -1, st);
            cudaError_t ce = cudaStreamEndCapture(st, &g);
            cudaGraphExec_t ge = nullptr;
            cudaError_t ie = cudaErrorInvalidValue;
            if (cs.ok() && ce == cudaSuccess) ie = cudaGraphInstantiate(&ge, g, 0);
            if (g) cudaGraphDestroy(g);
            if (!cs.ok() || ce != cudaSuccess || ie != cudaSuccess) {
                // A step of this plan cannot be captured: this session decodes
                // eagerly from now on (the captured steps never ran).
                cudaGetLastError();
                s->graph_unsupported = true;
                use_graph = false;
                continue;
            }
            s->graph = ge;
            s->graph_B = B;
            AM_CUDA(cudaGraphUpload(ge, st));
        }
    }
    AM_CUDA(cudaEventRecord(s->ev[2], st));
    range.reset();
    int64_t* ho = hp + B * P;
    float* hg = reinterpret_cast<float*>(ho + c.max_batch * s->out_cap);
    AM_CUDA(cudaMemcpyAsync(ho, s->out_tokens.data(), B * s->out_cap * 8, cudaMemcpyDeviceToHost, st));
    AM_CUDA(cudaMemcpyAsync(hg, s->gaps.data(), B * s->out_cap * 4, cudaMemcpyDeviceToHost, st));
    int32_t status_h = 0;
    int32_t* hstatus = reinterpret_cast<int32_t*>(hg + c.max_batch * s->out_cap);
    AM_CUDA(cudaMemcpyAsync(hstatus, s->status.data(), 4, cudaMemcpyDeviceToHost, st));
    // The device error word collects the codes of bounded waits that ran out
    // (a tensor-parallel peer that never arrived, a stalled copy): the kernel
    // that gave up skipped its wait, so the tokens of this call cannot be
    // trusted. Read it with the results and clear it for the next call.
    int32_t* dev_err = amcu::device_error_word();
    if (!dev_err) return Status::Internal("device error word unavailable");
    hstatus[1] = 0;
    AM_CUDA(cudaMemcpyAsync(hstatus + 1, dev_err, 4, cudaMemcpyDeviceToHost, st));
    AM_CUDA(cudaStreamSynchronize(st));
    status_h = hstatus[0];
    if (hstatus[1] != 0) {
        const int32_t code = hstatus[1];
        AM_CUDA(cudaMemsetAsync(dev_err, 0, 4, st));
        AM_CUDA(cudaStreamSynchronize(st));
        char msg[160];
        std::snprintf(msg, sizeof msg,
                      "a kernel's bounded wait ran out (device error code 0x%x); the generated tokens are invalid",
                      (unsigned)code);
        return Status::DeadlineExceeded(msg);
    }
    if (status_h != 0) return Status(static_cast<StatusCode>(status_h), "device reported an out-of-range index");
    AM_RETURN_IF_ERROR(kv.CommitUntil(P + N - 1));
    out.resize(B * N);
    s->last_gaps.resize(B * N);
    for (int64_t b = 0; b < B; ++b)
        for (int64_t i = 0; i < N; ++i) {
            out[b * N + i] = ho[b * s->out_cap + i];
            s->last_gaps[b * N + i] = hg[b * s->out_cap + i];
        }
    float ms0 = 0, ms1 = 0;
    cudaEventElapsedTime(&ms0, s->ev[0], s->ev[1]);
    cudaEventElapsedTime(&ms1, s->ev[1], s->ev[2]);
    s->last_prefill_ms = ms0;
    s->last_decode_ms = ms1;
    s->last_steps = N - 1;
    s->last_B = B;
    s->last_N = N;
    return Status::Ok();
}

// ---- checkpoint loading (am_model_load) ----

int32_t AmcuDtypeOf(hf::TensorDtype t) {
    return t == hf::TensorDtype::kF32 ? AMCU_F32 : t == hf::TensorDtype::kBF16 ? AMCU_BF16 : AMCU_F16;
}

Status CheckShape(const std::string& name, const hf::TensorInfo& t, std::vector<int64_t> want) {
    if (t.shape != want) {
        std::string got, exp;
        for (int64_t d : t.shape) got += std::to_string(d) + ",";
        for (int64_t d : want) exp += std::to_string(d) + ",";
        return Status::InvalidArgument("tensor '" + name + "' has shape [" + got + "], expected [" + exp + "]");
    }
    return Status::Ok();
}

// The raw checkpoint tensor on the device (its own dtype).
Status UploadRaw(am_model_s* m, const hf::TensorInfo& t, DeviceBuffer& out) {
    AM_RETURN_IF_ERROR(AllocVec(m, out, t.bytes));
    return CudaOk(UploadSync(m, out.data(), t.data, t.bytes), "checkpoint upload");
}

// A raw [n][k] tensor -> a canonical device matrix of the model's format:
// quantized (INT4 / INT8) or converted to the activation dtype (plain).
Status CanonFromRaw(am_model_s* m, const hf::TensorInfo& t, const DeviceBuffer& raw, int64_t n, int64_t k, Canon& out) {
    const auto& c = m->cfg;
    cudaStream_t st = m->rt->stream;
    out.n = n;
    out.k = k;
    AM_RETURN_IF_ERROR(AllocVec(m, out.q, RowBytes(c, k) * n));
    if (c.weight_format == AMCU_WFMT_PLAIN) {
        AM_RETURN_IF_ERROR(Status::FromAm(amcu_convert(raw.data(), AmcuDtypeOf(t.dtype), out.q.data(), c.act_dtype,
                                                       n * k, st),
                                          amcu_last_error()));
    } else {
        AM_RETURN_IF_ERROR(AllocVec(m, out.s, ScaleRowBytes(c, k) * n));
        AM_RETURN_IF_ERROR(Status::FromAm(amcu_quantize_weight(c.weight_format, raw.data(), AmcuDtypeOf(t.dtype), n, k,
                                                               c.group_size, out.q.data(), out.s.data(), st),
                                          amcu_last_error()));
    }
    return CudaOk(cudaStreamSynchronize(st), "quantize");
}

Status ConvertInto(am_model_s* m, const hf::TensorInfo& t, DeviceBuffer& dst, int64_t count) {
    DeviceBuffer raw;
    AM_RETURN_IF_ERROR(UploadRaw(m, t, raw));
    AM_RETURN_IF_ERROR(Status::FromAm(amcu_convert(raw.data(), AmcuDtypeOf(t.dtype), dst.data(), m->cfg.act_dtype,
                                                   count, m->rt->stream),
                                      amcu_last_error()));
    return CudaOk(cudaStreamSynchronize(m->rt->stream), "convert");
}

// Every tensor of the checkpoint into the model (names as the reference's
// HF weight resolver reads them, src/model/formats/hf/hf_weight_resolver.cpp).
Status LoadCheckpoint(am_model_s* m, const hf::Checkpoint& ck, bool tied_in_file) {
    const auto& c = m->cfg;
    const int64_t H = c.hidden, d = c.head_dim;
    auto get = [&](const std::string& name, std::vector<int64_t> shape) -> StatusOr<const hf::TensorInfo*> {
        auto t = ck.Get(name);
        if (!t.ok()) return t.status();
        AM_RETURN_IF_ERROR(CheckShape(name, *t.value(), std::move(shape)));
        return t.value();
    };
    // embedding (and the tied lm_head)
    {
        auto e = get("model.embed_tokens.weight", {c.vocab, H});
        if (!e.ok()) return e.status();
        const hf::TensorInfo& et = *e.value();
        DeviceBuffer raw;
        AM_RETURN_IF_ERROR(UploadRaw(m, et, raw));
        if (c.tied_embeddings && c.weight_format == AMCU_WFMT_INT8) {
            // one INT8 matrix serves both: dequantized rows for the embedding
            Canon full;
            AM_RETURN_IF_ERROR(CanonFromRaw(m, et, raw, c.vocab, H, full));
            AM_CUDA(cudaMemcpyAsync(m->embed.data(), full.q.data(), c.vocab * H, cudaMemcpyDeviceToDevice, m->rt->stream));
            AM_CUDA(cudaMemcpyAsync(m->embed_scales.data(), full.s.data(), c.vocab * 4, cudaMemcpyDeviceToDevice,
                                    m->rt->stream));
            AM_RETURN_IF_ERROR(PackInto(m, m->lm_head, 0, full));
        } else {
            AM_RETURN_IF_ERROR(Status::FromAm(amcu_convert(raw.data(), AmcuDtypeOf(et.dtype), m->embed.data(), c.act_dtype,
                                                           c.vocab * H, m->rt->stream),
                                              amcu_last_error()));
            AM_CUDA(cudaStreamSynchronize(m->rt->stream));
            if (tied_in_file) {  // plain tied, or an INT4 model that keeps its own quantized lm_head copy
                Canon head;
                AM_RETURN_IF_ERROR(CanonFromRaw(m, et, raw, c.vocab, H, head));
                AM_RETURN_IF_ERROR(PackInto(m, m->lm_head, 0, head));
            }
        }
    }
    if (!tied_in_file) {
        auto h = get("lm_head.weight", {c.vocab, H});
        if (!h.ok()) return h.status();
        DeviceBuffer raw;
        AM_RETURN_IF_ERROR(UploadRaw(m, *h.value(), raw));
        Canon head;
        AM_RETURN_IF_ERROR(CanonFromRaw(m, *h.value(), raw, c.vocab, H, head));
        AM_RETURN_IF_ERROR(PackInto(m, m->lm_head, 0, head));
    }
    {
        auto fnorm = get("model.norm.weight", {H});
        if (!fnorm.ok()) return fnorm.status();
        AM_RETURN_IF_ERROR(ConvertInto(m, *fnorm.value(), m->final_norm, H));
    }
    const char* hf_names[7] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                               "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"};
    const char* names[7] = {"wq", "wk", "wv", "wo", "wg", "wu", "wd"};
    for (int64_t l = 0; l < c.layers; ++l) {
        const std::string pre = "model.layers." + std::to_string(l) + ".";
        auto in = get(pre + "input_layernorm.weight", {H});
        if (!in.ok()) return in.status();
        AM_RETURN_IF_ERROR(ConvertInto(m, *in.value(), m->layers[l].attn_norm, H));
        auto post = get(pre + "post_attention_layernorm.weight", {H});
        if (!post.ok()) return post.status();
        AM_RETURN_IF_ERROR(ConvertInto(m, *post.value(), m->layers[l].mlp_norm, H));
        for (int t = 0; t < 7; ++t) {
            Target tg;
            AM_RETURN_IF_ERROR(ResolveTarget(m, (int)l, names[t], tg));
            auto w = get(pre + hf_names[t] + ".weight", {tg.n_full, tg.k_full});
            if (!w.ok()) return w.status();
            DeviceBuffer raw;
            AM_RETURN_IF_ERROR(UploadRaw(m, *w.value(), raw));
            Canon full, shard;
            AM_RETURN_IF_ERROR(CanonFromRaw(m, *w.value(), raw, tg.n_full, tg.k_full, full));
            AM_RETURN_IF_ERROR(Shard(m, full, tg.split, 0, shard));
            AM_RETURN_IF_ERROR(StoreLinear(m, (int)l, tg, shard));
        }
        (void)d;
    }
    return CudaOk(cudaDeviceSynchronize(), "checkpoint load");
}

}  // namespace
}  // namespace aethermind

using namespace aethermind;

extern "C" {

am_runtime_t am_runtime_create(const am_config_t* cfg) {
    auto* rt = new am_runtime_s();
    if (cfg) {
        rt->device = cfg->device_id;
        rt->tp_rank = cfg->tp_rank;
        rt->tp_size = cfg->tp_size > 0 ? cfg->tp_size : 1;
    }
    if (cudaSetDevice(rt->device) != cudaSuccess) {
        g_err = "cudaSetDevice failed";
        delete rt;
        return nullptr;
    }
    rt->alloc = std::make_unique<CudaAllocator>(rt->device);
    rt->backend = std::make_unique<CudaBackend>(rt->device);
    cudaStreamCreateWithFlags(&rt->stream, cudaStreamNonBlocking);
    if (rt->tp_size > 1) {
        Status s = rt->comm.Init(rt->tp_rank, rt->tp_size, cfg->nccl_unique_id);
        if (!s.ok()) {
            g_err = s.ToString();
            cudaStreamDestroy(rt->stream);
            delete rt;
            return nullptr;
        }
    }
    return rt;
}

void am_runtime_destroy(am_runtime_t rt) {
    if (!rt) return;
    if (rt->stream) cudaStreamDestroy(rt->stream);
    delete rt;
}

am_status_code am_runtime_peer_handle(am_runtime_t rt, void* out64) {
    if (!rt || !out64) return Fail(Status::InvalidArgument("am_runtime_peer_handle: null argument"));
    Status s = rt->comm.PeerHandle(out64);
    return s.ok() ? AM_STATUS_OK : Fail(s);
}

am_status_code am_runtime_open_peers(am_runtime_t rt, const void* handles) {
    if (!rt || !handles) return Fail(Status::InvalidArgument("am_runtime_open_peers: null argument"));
    if (cudaSetDevice(rt->device) != cudaSuccess) return Fail(Status::Internal("cudaSetDevice failed"));
    Status s = rt->comm.OpenPeers(handles);
    return s.ok() ? AM_STATUS_OK : Fail(s);
}

am_status_code am_nccl_get_unique_id(void* out128) {
    Status s = NcclGetUniqueId(out128);
    return s.ok() ? AM_STATUS_OK : Fail(s);
}

const char* am_last_error(void) { return g_err.c_str(); }

am_model_t am_model_create(am_runtime_t rt, const am_model_config_t* cfg, am_error_t* error) {
    auto fail = [&](const Status& s) -> am_model_t {
        g_err = s.ToString();
        if (error) *error = am_error_create(s.am_code(), s.message().c_str());
        return nullptr;
    };
    if (!rt || !cfg) return fail(Status::InvalidArgument("null runtime or config"));
    const auto& c = *cfg;
    const int tp = rt->tp_size;
    if (c.vocab <= 0 || c.hidden <= 0 || c.layers <= 0 || c.n_q_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim <= 0 ||
        c.inter <= 0 || c.max_seq <= 0 || c.max_batch <= 0)
        return fail(Status::InvalidArgument("model dimensions must be positive"));
    if (c.n_q_heads * c.head_dim != c.hidden)
        return fail(Status::InvalidArgument("n_q_heads * head_dim must equal hidden"));
    if (c.n_q_heads % c.n_kv_heads != 0) return fail(Status::InvalidArgument("n_q_heads must be a multiple of n_kv_heads"));
    if (c.n_kv_heads % tp != 0 || c.inter % tp != 0)
        return fail(Status::InvalidArgument("n_kv_heads and inter must be divisible by tp_size"));
    if (FromAmDtype(c.act_dtype) == DType::kUndefined) return fail(Status::InvalidArgument("act dtype must be f32/bf16"));
    if (c.weight_format != AMCU_WFMT_PLAIN && c.act_dtype != AMCU_BF16)
        return fail(Status::InvalidArgument("quantized weights need bf16 activations"));
    if (c.weight_format == AMCU_WFMT_INT4 && c.group_size != 128)
        return fail(Status::InvalidArgument("int4 weights need group_size 128"));
    if (c.tied_embeddings && c.weight_format == AMCU_WFMT_INT4)
        return fail(Status::Unimplemented("tied embeddings are supported for plain and int8 weights"));
    auto* m = new am_model_s();
    m->rt = rt;
    m->cfg = c;
    m->act = FromAmDtype(c.act_dtype);
    m->nq_l = c.n_q_heads / tp;
    m->nkv_l = c.n_kv_heads / tp;
    m->inter_l = c.inter / tp;
    m->qkv_n = (m->nq_l + 2 * m->nkv_l) * c.head_dim;
    const size_t e = DTypeBytes(m->act);
    auto chk = [&](Status s) {
        if (!s.ok()) throw s;
    };
    try {
        if (c.weight_format != AMCU_WFMT_PLAIN) {
            const int64_t kmul = c.weight_format == AMCU_WFMT_INT4 ? 128 : 64;
            if (m->qkv_n % 16 || c.hidden % 16 || (2 * m->inter_l) % 16 || c.vocab % 16 || c.hidden % kmul ||
                (m->nq_l * c.head_dim) % kmul || m->inter_l % kmul)
                throw Status::InvalidArgument("quantized shapes need N % 16 == 0 and K % " + std::to_string(kmul) +
                                              " == 0 per rank");
        }
        if (c.tied_embeddings && c.weight_format == AMCU_WFMT_INT8) {
            chk(AllocVec(m, m->embed, c.vocab * c.hidden));
            chk(AllocVec(m, m->embed_scales, c.vocab * 4));
        } else {
            chk(AllocVec(m, m->embed, c.vocab * c.hidden * e));
        }
        chk(AllocVec(m, m->final_norm, c.hidden * e));
        chk(AllocLinear(m, m->lm_head, c.vocab, c.hidden, false));
        m->layers.resize(c.layers);
        for (auto& L : m->layers) {
            chk(AllocVec(m, L.attn_norm, c.hidden * e));
            chk(AllocVec(m, L.mlp_norm, c.hidden * e));
            chk(AllocLinear(m, L.qkv, m->qkv_n, c.hidden, false));
            chk(AllocLinear(m, L.o, c.hidden, m->nq_l * c.head_dim, false));
            chk(AllocLinear(m, L.gu, 2 * m->inter_l, c.hidden, true));
            chk(AllocLinear(m, L.d, c.hidden, m->inter_l, false));
        }
    } catch (const Status& s) {
        delete m;
        return fail(s);
    }
    return m;
}

am_model_t am_model_load_ex(am_runtime_t rt, const char* path, const am_load_options_t* opt, am_error_t* error) {
    auto fail = [&](const Status& s) -> am_model_t {
        g_err = s.ToString();
        if (error) *error = am_error_create(s.am_code(), s.message().c_str());
        return nullptr;
    };
    if (!rt || !path) return fail(Status::InvalidArgument("am_model_load: null runtime or path"));
    auto ck = hf::Checkpoint::Open(path);
    if (!ck.ok()) return fail(ck.status());
    const hf::LlamaConfig& hc = ck.value()->config();
    am_load_options_t o{};
    if (opt) o = *opt;
    am_model_config_t mc{};
    mc.vocab = hc.vocab;
    mc.hidden = hc.hidden;
    mc.layers = hc.layers;
    mc.n_q_heads = hc.n_q_heads;
    mc.n_kv_heads = hc.n_kv_heads;
    mc.head_dim = hc.head_dim;
    mc.inter = hc.inter;
    mc.rms_eps = hc.rms_eps;
    mc.rope_theta = hc.rope_theta;
    mc.weight_format = o.weight_format ? o.weight_format : AMCU_WFMT_INT4;
    mc.act_dtype = o.act_dtype ? o.act_dtype : AMCU_BF16;
    mc.group_size = 128;
    mc.max_seq = o.max_seq > 0 ? o.max_seq : (hc.max_position_embeddings < 4096 ? hc.max_position_embeddings : 4096);
    mc.max_batch = o.max_batch > 0 ? o.max_batch : 1;
    // a checkpoint without lm_head.weight ties it to the embedding
    const bool tied_in_file = hc.tied_embeddings || !ck.value()->Has("lm_head.weight");
    // INT4 keeps a quantized copy of a tied lm_head next to the bf16 embedding
    mc.tied_embeddings = tied_in_file && mc.weight_format != AMCU_WFMT_INT4;
    am_error_t cerr = nullptr;
    am_model_t m = am_model_create(rt, &mc, &cerr);
    if (!m) {
        Status s(static_cast<StatusCode>(cerr ? am_error_code(cerr) : AM_STATUS_INTERNAL),
                 std::string("am_model_load: ") + (cerr ? am_error_message(cerr) : "model create failed"));
        if (cerr) am_error_destroy(cerr);
        return fail(s);
    }
    Status st;
    try {
        st = LoadCheckpoint(m, *ck.value(), tied_in_file);
    } catch (const Status& s) {
        st = s;
    }
    if (!st.ok()) {
        am_model_unload(m);
        return fail(st);
    }
    return m;
}

am_model_t am_model_load(am_runtime_t rt, const char* path, am_error_t* error) {
    return am_model_load_ex(rt, path, nullptr, error);
}

void am_model_unload(am_model_t m) { delete m; }

static Status FillOnes(am_model_s* m, DeviceBuffer& b, int64_t n) {
    std::vector<char> host(n * DTypeBytes(m->act));
    if (m->act == DType::kF32) {
        float* f = reinterpret_cast<float*>(host.data());
        for (int64_t i = 0; i < n; ++i) f[i] = 1.f;
    } else {
        uint16_t* u = reinterpret_cast<uint16_t*>(host.data());
        for (int64_t i = 0; i < n; ++i) u[i] = 0x3F80;  // bf16 1.0
    }
    return CudaOk(UploadSync(m, b.data(), host.data(), host.size()), "norm upload");
}

am_status_code am_model_init_synthetic(am_model_t m, uint64_t seed) {
    if (!m) return Fail(Status::InvalidArgument("null model"));
    const auto& c = m->cfg;
    try {
        auto chk = [&](Status s) {
            if (!s.ok()) throw s;
        };
        cudaStream_t st = m->rt->stream;
        // embedding / lm_head
        if (c.tied_embeddings && c.weight_format == AMCU_WFMT_INT8) {
            Canon full;
            chk(SynthCanon(m, seed, 1, c.vocab, c.hidden, full));
            chk(CudaOk(cudaMemcpyAsync(m->embed.data(), full.q.data(), c.vocab * c.hidden, cudaMemcpyDeviceToDevice, st), "embed"));
            chk(CudaOk(cudaMemcpyAsync(m->embed_scales.data(), full.s.data(), c.vocab * 4, cudaMemcpyDeviceToDevice, st), "embed"));
            chk(PackInto(m, m->lm_head, 0, full));
        } else {
            if (m->act != DType::kBF16) throw Status::Unimplemented("synthetic init needs bf16 activations");
            chk(Status::FromAm(amcu_synth_uniform_bf16(seed, 1, c.vocab * c.hidden, kEmbedAmp, m->embed.data(), st),
                               amcu_last_error()));
            Canon head;
            chk(SynthCanon(m, seed, 2, c.vocab, c.hidden, head));
            chk(PackInto(m, m->lm_head, 0, head));
        }
        chk(FillOnes(m, m->final_norm, c.hidden));
        const char* names[7] = {"wq", "wk", "wv", "wo", "wg", "wu", "wd"};
        for (int64_t l = 0; l < c.layers; ++l) {
            chk(FillOnes(m, m->layers[l].attn_norm, c.hidden));
            chk(FillOnes(m, m->layers[l].mlp_norm, c.hidden));
            for (int t = 0; t < 7; ++t) {
                Target tg;
                chk(ResolveTarget(m, (int)l, names[t], tg));
                Canon full, shard;
                chk(SynthCanon(m, seed, 16 + (uint64_t)l * 8 + t, tg.n_full, tg.k_full, full));
                chk(Shard(m, full, tg.split, 0, shard));
                chk(StoreLinear(m, (int)l, tg, shard));
                chk(CudaOk(cudaStreamSynchronize(st), "synth"));
            }
        }
        chk(CudaOk(cudaStreamSynchronize(st), "synthetic init"));
    } catch (const Status& s) {
        return Fail(s);
    }
    return AM_STATUS_OK;
}

am_status_code am_model_set_weight(am_model_t m, const char* name_c, const void* data, const void* scales) {
    if (!m || !name_c || !data) return Fail(Status::InvalidArgument("null argument"));
    const auto& c = m->cfg;
    const std::string name(name_c);
    const size_t e = DTypeBytes(m->act);
    try {
        auto chk = [&](Status s) {
            if (!s.ok()) throw s;
        };
        if (name == "embed") {
            if (c.tied_embeddings && c.weight_format == AMCU_WFMT_INT8)
                throw Status::InvalidArgument("tied int8 model: set 'lm_head' (it also feeds the embedding)");
            chk(CudaOk(UploadSync(m, m->embed.data(), data, c.vocab * c.hidden * e), "embed"));
            if (c.tied_embeddings) {  // tied plain: the lm_head is the same matrix
                Canon full;
                chk(UploadCanon(m, c.vocab, c.hidden, data, scales, full));
                chk(PackInto(m, m->lm_head, 0, full));
            }
        } else if (name == "lm_head") {
            Canon full;
            chk(UploadCanon(m, c.vocab, c.hidden, data, scales, full));
            if (c.tied_embeddings && c.weight_format == AMCU_WFMT_INT8) {
                chk(CudaOk(UploadSync(m, m->embed.data(), data, c.vocab * c.hidden), "embed"));
                chk(CudaOk(UploadSync(m, m->embed_scales.data(), scales, c.vocab * 4), "embed"));
            }
            chk(PackInto(m, m->lm_head, 0, full));
        } else if (name == "final_norm") {
            chk(CudaOk(UploadSync(m, m->final_norm.data(), data, c.hidden * e), "norm"));
        } else if (name.rfind("layers.", 0) == 0) {
            const size_t dot = name.find('.', 7);
            if (dot == std::string::npos) throw Status::NotFound("bad weight name " + name);
            const int l = std::stoi(name.substr(7, dot - 7));
            if (l < 0 || l >= c.layers) throw Status::OutOfRange("layer index out of range");
            const std::string t = name.substr(dot + 1);
            auto& L = m->layers[l];
            if (t == "attn_norm" || t == "mlp_norm") {
                chk(CudaOk(UploadSync(m, (t == "attn_norm" ? L.attn_norm : L.mlp_norm).data(), data, c.hidden * e), "norm"));
            } else {
                Target tg;
                chk(ResolveTarget(m, l, t, tg));
                Canon full, shard;
                chk(UploadCanon(m, tg.n_full, tg.k_full, data, scales, full));
                chk(Shard(m, full, tg.split, 0, shard));
                chk(StoreLinear(m, l, tg, shard));
            }
        } else {
            throw Status::NotFound("unknown weight name " + name);
        }
        chk(CudaOk(cudaStreamSynchronize(m->rt->stream), "set_weight"));
        chk(CudaOk(cudaDeviceSynchronize(), "set_weight"));
    } catch (const Status& s) {
        return Fail(s);
    } catch (const std::exception& ex) {
        return Fail(Status::InvalidArgument(ex.what()));
    }
    return AM_STATUS_OK;
}

am_session_t am_session_create(am_model_t m, const am_session_config_t* cfg) {
    if (!m) return nullptr;
    auto* s = new am_session_s();
    s->m = m;
    if (cfg) s->cfg = *cfg;
    else s->cfg.use_cuda_graph = 1;
    const auto& c = m->cfg;
    auto& A = *m->rt->alloc;
    Status st = s->kv.Init(A, c.layers, m->nkv_l, c.max_seq, c.head_dim, m->act, c.max_batch);
    auto get = [&](DeviceBuffer& b, size_t bytes) {
        if (!st.ok()) return;
        auto r = A.Allocate(bytes);
        if (!r.ok()) { st = r.status(); return; }
        b = std::move(r.value());
    };
    get(s->next_tok, c.max_batch * 8);
    get(s->seq_pos, c.max_batch * 4);
    get(s->counter, 16);
    get(s->gap_tmp, c.max_batch * 4);
    get(s->status, 16);
    get(s->hlast, c.max_batch * c.hidden * DTypeBytes(m->act));
    get(s->logits, c.max_batch * c.vocab * DTypeBytes(m->act));
    get(s->rope_table, c.max_seq * (c.head_dim / 2) * 8);
    if (st.ok())
        st = Status::FromAm(amcu_rope_table(c.rope_theta, c.head_dim, c.max_seq, s->rope_table.as<float>(),
                                            m->rt->stream),
                            amcu_last_error());
    if (st.ok()) st = CudaOk(cudaStreamSynchronize(m->rt->stream), "rope table");
    if (!st.ok()) {
        g_err = st.ToString();
        delete s;
        return nullptr;
    }
    for (auto& e : s->ev) cudaEventCreate(&e);
    return s;
}

void am_session_destroy(am_session_t s) {
    if (!s) return;
    if (s->graph) cudaGraphExecDestroy(s->graph);
    if (s->pinned) cudaFreeHost(s->pinned);
    for (auto& e : s->ev)
        if (e) cudaEventDestroy(e);
    delete s;
}

int am_session_generate_batch(am_session_t s, const uint32_t* in, size_t batch, size_t in_len, uint32_t* out,
                              size_t cap, size_t* out_len, am_error_t* error) {
    auto fail = [&](const Status& st) {
        g_err = st.ToString();
        if (error) *error = am_error_create(st.am_code(), st.message().c_str());
        return (int)st.am_code();
    };
    if (!s || !in || !out) return fail(Status::InvalidArgument("null argument"));
    int64_t N = (int64_t)cap;
    if (s->cfg.max_new_tokens > 0 && N > s->cfg.max_new_tokens) N = s->cfg.max_new_tokens;
    std::vector<int64_t> toks;
    Status st = Generate(s, in, (int64_t)batch, (int64_t)in_len, N, toks);
    if (!st.ok()) return fail(st);
    for (size_t b = 0; b < batch; ++b)
        for (int64_t i = 0; i < N; ++i) out[b * cap + i] = (uint32_t)toks[b * N + i];
    if (out_len) *out_len = (size_t)N;
    return AM_STATUS_OK;
}

int am_session_generate(am_session_t s, const uint32_t* in, size_t in_len, uint32_t* out, size_t cap,
                        size_t* out_len, am_error_t* error) {
    return am_session_generate_batch(s, in, 1, in_len, out, cap, out_len, error);
}

am_status_code am_session_last_timing(am_session_t s, double* prefill_ms, double* decode_ms, int64_t* steps) {
    if (!s) return Fail(Status::InvalidArgument("null session"));
    if (prefill_ms) *prefill_ms = s->last_prefill_ms;
    if (decode_ms) *decode_ms = s->last_decode_ms;
    if (steps) *steps = s->last_steps;
    return AM_STATUS_OK;
}

am_status_code am_session_last_gaps(am_session_t s, float* gaps, size_t capacity) {
    if (!s || !gaps) return Fail(Status::InvalidArgument("null argument"));
    const size_t n = s->last_gaps.size() < capacity ? s->last_gaps.size() : capacity;
    std::memcpy(gaps, s->last_gaps.data(), n * sizeof(float));
    return AM_STATUS_OK;
}

// Debug / test hooks (not part of the reference surface).
int64_t am_debug_registry_size(void) { return (int64_t)KernelRegistry::Global().size(); }
am_status_code am_debug_plan_steps(am_session_t s, int32_t phase, int64_t batch, int64_t rows_per_seq, char* buf,
                                   size_t cap) {
    if (!s || !buf) return Fail(Status::InvalidArgument("null argument"));
    ExecutionPlan p;
    Status st = EnsureRows(s, batch * rows_per_seq);
    if (st.ok()) st = BuildPlan(s, phase == 0 ? ExecPhase::kPrefill : ExecPhase::kDecode, batch, rows_per_seq, p);
    if (!st.ok()) return Fail(st);
    std::string out;
    for (auto& step : p.steps)
        out += step.label + " " + (step.host_fn ? std::string("<host>") : std::string(step.kernel.debug_name)) + "\n";
    s->prefill_B = s->decode_B = -1;
    std::snprintf(buf, cap, "%s", out.c_str());
    return AM_STATUS_OK;
}

am_status_code am_debug_resolve_kernel(int32_t op, int32_t act, int32_t weight, int32_t format, int32_t phase,
                                       char* name, size_t cap) {
    static CudaBackend* backend = new CudaBackend(0);  // constructing a backend freezes the registry
    auto dt = [](int32_t d) {
        switch (d) {
            case AMCU_F32: return DType::kF32;
            case AMCU_BF16: return DType::kBF16;
            case AMCU_I8: return DType::kI8;
            case AMCU_I4: return DType::kI4;
            default: return DType::kUndefined;
        }
    };
    KernelSelector sel{DeviceType::kCUDA, dt(act), dt(weight), static_cast<WeightFormat>(format), IsaLevel::kScalar,
                       static_cast<ExecPhase>(phase)};
    auto r = backend->ResolveKernelInfo(static_cast<OpType>(op), sel);
    if (!r.ok()) return Fail(r.status());
    if (name && cap) std::snprintf(name, cap, "%s", r.value().debug_name);
    return AM_STATUS_OK;
}

am_status_code am_debug_kv_offset(uint64_t layers, uint64_t heads, uint64_t max_tokens, uint64_t head_dim,
                                  int32_t dtype, uint64_t slots, uint64_t l, uint64_t h, uint64_t p, uint64_t d,
                                  uint64_t slot, uint64_t* offset, uint64_t* bytes_per_plane) {
    KVCacheManager mgr;
    Status st = mgr.InitLayoutOnly(layers, heads, max_tokens, head_dim, FromAmDtype(dtype), slots);
    if (!st.ok()) return Fail(st);
    auto off = mgr.layout().Offset(l, h, p, d, slot);
    if (!off.ok()) return Fail(off.status());
    if (offset) *offset = off.value();
    if (bytes_per_plane) *bytes_per_plane = mgr.layout().BytesPerPlane().value();
    return AM_STATUS_OK;
}

am_status_code am_debug_tp_shard(const char* tensor, int64_t n, int64_t k, int32_t rank, int32_t world,
                                 int64_t* out4) {
    if (!tensor || !out4 || world < 1 || rank < 0 || rank >= world)
        return Fail(Status::InvalidArgument("am_debug_tp_shard: bad arguments"));
    const std::string t(tensor);
    Split sp;
    if (t == "wq" || t == "wk" || t == "wv" || t == "wg" || t == "wu") sp = Split::kRows;
    else if (t == "wo" || t == "wd") sp = Split::kCols;
    else if (t == "embed" || t == "lm_head" || t == "attn_norm" || t == "mlp_norm" || t == "final_norm") sp = Split::kNone;
    else return Fail(Status::NotFound("am_debug_tp_shard: unknown tensor " + t));
    ShardRange(sp, n, k, rank, world, out4[0], out4[1], out4[2], out4[3]);
    return AM_STATUS_OK;
}

am_status_code am_debug_kv_reserve(uint64_t max_tokens, uint64_t prompt_len, uint64_t max_new) {
    KVCacheManager mgr;
    Status st = mgr.InitLayoutOnly(1, 1, max_tokens, 8, DType::kF32, 1);
    if (!st.ok()) return Fail(st);
    auto v = mgr.ReserveForSession(prompt_len, max_new);
    if (!v.ok()) return Fail(v.status());
    // a second reservation while the first is active must fail (single active session)
    auto v2 = mgr.ReserveForSession(prompt_len, max_new);
    if (v2.ok()) return Fail(Status::Internal("second reservation unexpectedly succeeded"));
    return AM_STATUS_OK;
}

}  // extern "C"
