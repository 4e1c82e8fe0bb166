// C-ABI entry points of the Linear family: argument validation and the
// m-based dispatch between the decode GEMV and the prefill GEMM.
#include "../amcu_internal.h"
#include "allreduce.cuh"
#include "gemm_tc.cuh"
#include "gemv.cuh"

using namespace amcu;

namespace {

am_status_code validate_linear(const AmcuLinearArgs* a, const char* who) {
    AMCU_REQUIRE(a != nullptr, "%s: null args", who);
    const AmcuWeight& w = a->w;
    AMCU_REQUIRE(a->m >= 0, "%s: negative m", who);
    AMCU_REQUIRE(w.n > 0 && w.k > 0, "%s: weight n and k must be positive", who);
    AMCU_REQUIRE(a->x && a->y && w.data, "%s: null pointer", who);
    AMCU_REQUIRE(a->epilogue >= AMCU_EPI_STORE && a->epilogue <= AMCU_EPI_SILU_MUL, "%s: bad epilogue", who);
    AMCU_REQUIRE(a->epilogue != AMCU_EPI_RESIDUAL_ADD || a->residual, "%s: residual epilogue needs residual", who);
    AMCU_REQUIRE(!a->norm_weight || w.format != AMCU_WFMT_PLAIN,
                 "%s: the fused RMSNorm is available for quantized weights", who);
    AMCU_REQUIRE(!a->norm_weight || aligned(a->norm_weight, 16), "%s: norm weight must be 16-byte aligned", who);
    AMCU_REQUIRE(a->epilogue != AMCU_EPI_SILU_MUL || w.gate_up_interleaved || w.format == AMCU_WFMT_PLAIN,
                 "%s: SILU_MUL epilogue needs a weight from amcu_prepack_gate_up", who);
    if (w.format == AMCU_WFMT_PLAIN) {
        AMCU_REQUIRE(a->act_dtype == w.dtype, "%s: plain weights must match the activation dtype", who);
        AMCU_REQUIRE(a->act_dtype == AMCU_F32 || a->act_dtype == AMCU_BF16, "%s: act dtype must be f32/bf16", who);
    } else {
        AMCU_REQUIRE(w.format == AMCU_WFMT_INT8 || w.format == AMCU_WFMT_INT4, "%s: unknown weight format", who);
        AMCU_REQUIRE(a->act_dtype == AMCU_BF16, "%s: quantized weights take bf16 activations", who);
        AMCU_REQUIRE(w.format != AMCU_WFMT_INT8 || w.scales, "%s: null scales", who);
        AMCU_REQUIRE(w.n % 16 == 0 && w.k % 64 == 0, "%s: n %% 16 and k %% 64 must be 0", who);
        AMCU_REQUIRE(w.format != AMCU_WFMT_INT4 || (w.group == 128 && w.k % 128 == 0),
                     "%s: int4 needs group 128 and k %% 128 == 0", who);
        AMCU_REQUIRE(aligned(a->x, 16) && aligned(w.data, 16), "%s: x and weights must be 16-byte aligned", who);
        const int64_t xs = a->x_stride ? a->x_stride : w.k;
        AMCU_REQUIRE(xs % 8 == 0, "%s: x row stride must be a multiple of 8 elements", who);
    }
    if (const AmcuAllReduceArgs* pr = a->peer_reduce) {
        AMCU_REQUIRE(a->epilogue == AMCU_EPI_RESIDUAL_ADD && w.format != AMCU_WFMT_PLAIN && a->m <= kGemvMaxM,
                     "%s: peer_reduce needs a quantized GEMV (m <= %d) with the residual epilogue", who, kGemvMaxM);
        AMCU_REQUIRE(pr->world >= 2 && pr->world <= kArMaxRanks && pr->rank >= 0 && pr->rank < pr->world,
                     "%s: peer_reduce rank/world out of range", who);
        AMCU_REQUIRE(w.n * kGemvMaxM <= kFuseMaxVals && w.n / 16 <= kFuseMaxRb,
                     "%s: peer_reduce supports at most %lld output rows", who, (long long)(kFuseMaxVals / kGemvMaxM));
        for (int r = 0; r < pr->world; ++r)
            AMCU_REQUIRE(pr->areas[r] != nullptr, "%s: peer_reduce area %d missing", who, r);
    }
    return AM_STATUS_OK;
}

GemvParams make_params(const AmcuLinearArgs* a) {
    GemvParams p{};
    p.x = a->x;
    p.w = a->w.data;
    p.scales = a->w.scales;
    p.y = a->y;
    p.residual = a->residual;
    p.m = a->m;
    p.n = a->w.n;
    p.k = a->w.k;
    p.x_stride = a->x_stride ? a->x_stride : a->w.k;
    p.y_stride = a->y_stride ? a->y_stride : (a->epilogue == AMCU_EPI_SILU_MUL ? a->w.n / 2 : a->w.n);
    p.err = device_error_word();
    p.norm_w = a->norm_weight;
    p.eps = a->norm_eps;
    p.l2_next = a->l2_next;
    if (const AmcuAllReduceArgs* pr = a->peer_reduce) {
        for (int r = 0; r < pr->world; ++r) p.fuse.area[r] = static_cast<uint8_t*>(pr->areas[r]);
        p.fuse.rank = pr->rank;
        p.fuse.world = pr->world;
        p.fuse.wait_ns = pr->wait_limit_us ? pr->wait_limit_us * 1000ull : 2000000000ull;
    }
    return p;
}

am_status_code run_gemv(const AmcuLinearArgs* a, cudaStream_t s) {
    GemvParams p = make_params(a);
    // Rows beyond kGemvMaxM are processed in slices (each slice re-reads W).
    const int64_t elt = 2;
    for (int64_t m0 = 0; m0 < a->m; m0 += kGemvMaxM) {
        GemvParams q = p;
        q.m = a->m - m0 < kGemvMaxM ? a->m - m0 : kGemvMaxM;
        q.x = static_cast<const char*>(p.x) + m0 * p.x_stride * elt;
        q.y = static_cast<char*>(p.y) + m0 * p.y_stride * elt;
        if (p.residual) q.residual = static_cast<const char*>(p.residual) + m0 * p.y_stride * elt;
        launch_gemv(q, a->w.format, a->epilogue, s);
    }
    return check_launch("amcu_gemv");
}

am_status_code run_gemm(const AmcuLinearArgs* a, cudaStream_t s) {
    AMCU_REQUIRE(a->peer_reduce == nullptr, "amcu_linear: peer_reduce is for the decode GEMV (m <= %d)", kGemvMaxM);
    if (a->w.format == AMCU_WFMT_PLAIN) {
        launch_gemm_plain(make_params(a), a->act_dtype, a->epilogue, s);
        return check_launch("amcu_gemm_plain");
    }
    GemmTcParams g{};
    const GemvParams p = make_params(a);
    g.x = p.x; g.w = p.w; g.scales = p.scales; g.y = p.y; g.residual = p.residual;
    g.m = p.m; g.n = p.n; g.k = p.k; g.x_stride = p.x_stride; g.y_stride = p.y_stride;
    g.workspace = a->workspace;
    g.workspace_size = a->workspace_size;
    if (!a->norm_weight && gemm_tc_supported(g, a->w.format)) {
        am_status_code st = launch_gemm_tc(g, a->w.format, a->epilogue, s);
        if (st != AM_STATUS_OK) return st;
        return check_launch("amcu_gemm_tc");
    }
    return run_gemv(a, s);
}

}  // namespace

extern "C" {

size_t amcu_linear_workspace_bytes(const AmcuLinearArgs* a) {
    if (!a || a->w.format == AMCU_WFMT_PLAIN || a->m <= kGemvMaxM) return 0;
    GemmTcParams g{};
    g.m = a->m; g.n = a->w.n; g.k = a->w.k;
    return gemm_tc_workspace_bytes(g, a->w.format);
}

am_status_code amcu_linear(const AmcuLinearArgs* a, void* stream) {
    clear_error();
    am_status_code st = validate_linear(a, "amcu_linear");
    if (st != AM_STATUS_OK) return st;
    if (a->m == 0) return AM_STATUS_OK;
    if (a->w.format != AMCU_WFMT_PLAIN && a->m <= kGemvMaxM) return run_gemv(a, as_stream(stream));
    return run_gemm(a, as_stream(stream));
}

am_status_code amcu_gemv_w8(const AmcuLinearArgs* a, void* stream) {
    clear_error();
    am_status_code st = validate_linear(a, "amcu_gemv_w8");
    if (st != AM_STATUS_OK) return st;
    AMCU_REQUIRE(a->w.format == AMCU_WFMT_INT8, "amcu_gemv_w8: weight format must be INT8");
    AMCU_REQUIRE(a->m <= kGemvMaxM, "amcu_gemv_w8: m must be <= %d", kGemvMaxM);
    if (a->m == 0) return AM_STATUS_OK;
    return run_gemv(a, as_stream(stream));
}

am_status_code amcu_gemv_w4g128(const AmcuLinearArgs* a, void* stream) {
    clear_error();
    am_status_code st = validate_linear(a, "amcu_gemv_w4g128");
    if (st != AM_STATUS_OK) return st;
    AMCU_REQUIRE(a->w.format == AMCU_WFMT_INT4, "amcu_gemv_w4g128: weight format must be INT4");
    AMCU_REQUIRE(a->m <= kGemvMaxM, "amcu_gemv_w4g128: m must be <= %d", kGemvMaxM);
    if (a->m == 0) return AM_STATUS_OK;
    return run_gemv(a, as_stream(stream));
}

am_status_code amcu_gemm_w8_prefill(const AmcuLinearArgs* a, void* stream) {
    clear_error();
    am_status_code st = validate_linear(a, "amcu_gemm_w8_prefill");
    if (st != AM_STATUS_OK) return st;
    AMCU_REQUIRE(a->w.format == AMCU_WFMT_INT8, "amcu_gemm_w8_prefill: weight format must be INT8");
    if (a->m == 0) return AM_STATUS_OK;
    return run_gemm(a, as_stream(stream));
}

am_status_code amcu_gemm_w4g128_prefill(const AmcuLinearArgs* a, void* stream) {
    clear_error();
    am_status_code st = validate_linear(a, "amcu_gemm_w4g128_prefill");
    if (st != AM_STATUS_OK) return st;
    AMCU_REQUIRE(a->w.format == AMCU_WFMT_INT4, "amcu_gemm_w4g128_prefill: weight format must be INT4");
    if (a->m == 0) return AM_STATUS_OK;
    return run_gemm(a, as_stream(stream));
}

}  // extern "C"
