// Decode-attention building blocks shared by the split-K kernel and the fused
// RoPE + attention kernel: one warp scores 8 keys per step against the GRP
// query heads of a kv head and keeps an online softmax.
#pragma once
#include <type_traits>

#include "common.cuh"

namespace amcu {

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr float kLog2e = 1.4426950408889634f;

// Per-warp running softmax state: max m (log2 domain), sum l, and the
// unnormalised output; lane l owns output dims [l * D/32, (l+1) * D/32).
template <int GRP, int D>
struct DecodeWarpState {
    float m[GRP], l[GRP], acc[GRP][D / 32];
};

// Keys [k_begin, k_end) of one (row, kv head), blocks of 8 keys round-robin
// over the CTA's NW warps. qs holds the GRP query heads scaled by
// softmax_scale * log2(e). Lane 4k+q holds quarter q of key k's head_dim:
// four 16-byte K loads per lane, a two-shuffle reduction, one online-softmax
// update per 8-key block, then P*V with lane l owning head_dim/32 output dims
// of every head (V rows read coalesced). The next block's K and V are loaded
// while the current one is scored, so each warp keeps two blocks in flight;
// the first block can be loaded early (load_first) by a caller that knows the
// keys are final before the query is.
template <int GRP, int D, int NW>
struct DecodeKeyLoop {
    static constexpr int DQ = D / 4;   // dims per lane in the QK phase
    static constexpr int DL = D / 32;  // dims per lane in the PV phase
    using VRaw = typename std::conditional<DL == 4, uint2, uint32_t>::type;
    const __nv_bfloat16 *kbase, *vbase;
    int64_t k_begin, k_end;
    int warp, lane;
    uint4 kv4[DQ / 8];
    VRaw vr[8];
    bool first_loaded = false;

    __device__ __forceinline__ DecodeKeyLoop(const __nv_bfloat16* kb, const __nv_bfloat16* vb, int64_t b, int64_t e,
                                             int w, int l)
        : kbase(kb), vbase(vb), k_begin(b), k_end(e), warp(w), lane(l) {}

    __device__ __forceinline__ void load_block(int64_t kb) {
        const int kk = lane >> 2, qd = lane & 3;
        const int64_t key = kb + kk;
#pragma unroll
        for (int i = 0; i < DQ / 8; ++i)
            kv4[i] = key < k_end ? *reinterpret_cast<const uint4*>(kbase + key * D + qd * DQ + i * 8)
                                 : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (kb + j < k_end) vr[j] = *reinterpret_cast<const VRaw*>(vbase + (kb + j) * D + lane * DL);
            else vr[j] = VRaw{};
        }
    }
    // Loads this warp's first block now if all its keys are below `final_end`.
    __device__ __forceinline__ void load_first(int64_t final_end) {
        const int64_t kb = k_begin + warp * 8;
        const int64_t last = kb + 8 < k_end ? kb + 8 : k_end;
        if (kb < k_end && last <= final_end) {
            load_block(kb);
            first_loaded = true;
        }
    }

    __device__ __forceinline__ void run(const float (*qs)[D], DecodeWarpState<GRP, D>& st) {
        const int kk = lane >> 2, qd = lane & 3;
#pragma unroll
        for (int h = 0; h < GRP; ++h) {
            st.m[h] = -INFINITY;
            st.l[h] = 0.f;
#pragma unroll
            for (int i = 0; i < DL; ++i) st.acc[h][i] = 0.f;
        }
        int64_t kb = k_begin + warp * 8;
        if (kb < k_end && !first_loaded) load_block(kb);
        for (; kb < k_end; kb += NW * 8) {
            const int64_t key = kb + kk;
            const bool valid = key < k_end;
            uint4 ck[DQ / 8];
            VRaw cv[8];
#pragma unroll
            for (int i = 0; i < DQ / 8; ++i) ck[i] = kv4[i];
#pragma unroll
            for (int j = 0; j < 8; ++j) cv[j] = vr[j];
            if (kb + NW * 8 < k_end) load_block(kb + NW * 8);  // next block in flight
            float vf[8][DL];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if constexpr (DL == 4) {
                    const uint2 u = *reinterpret_cast<const uint2*>(&cv[j]);
                    vf[j][0] = __uint_as_float(u.x << 16); vf[j][1] = __uint_as_float(u.x & 0xffff0000u);
                    vf[j][2] = __uint_as_float(u.y << 16); vf[j][3] = __uint_as_float(u.y & 0xffff0000u);
                } else {
                    const uint32_t u = *reinterpret_cast<const uint32_t*>(&cv[j]);
                    vf[j][0] = __uint_as_float(u << 16); vf[j][1] = __uint_as_float(u & 0xffff0000u);
                }
            }
            float s[GRP];
#pragma unroll
            for (int h = 0; h < GRP; ++h) s[h] = 0.f;
#pragma unroll
            for (int i = 0; i < DQ / 8; ++i) {
                const uint32_t w4[4] = {ck[i].x, ck[i].y, ck[i].z, ck[i].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float k0 = __uint_as_float(w4[e] << 16), k1 = __uint_as_float(w4[e] & 0xffff0000u);
                    const int dd = qd * DQ + i * 8 + 2 * e;
#pragma unroll
                    for (int h = 0; h < GRP; ++h) {
                        const float2 qq = *reinterpret_cast<const float2*>(&qs[h][dd]);
                        s[h] = fmaf(qq.x, k0, fmaf(qq.y, k1, s[h]));
                    }
                }
            }
            float pr[GRP];
#pragma unroll
            for (int h = 0; h < GRP; ++h) {
                s[h] += __shfl_xor_sync(0xffffffffu, s[h], 1);
                s[h] += __shfl_xor_sync(0xffffffffu, s[h], 2);
                const float sv = valid ? s[h] : -INFINITY;
                float bm = fmaxf(sv, __shfl_xor_sync(0xffffffffu, sv, 4));
                bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 8));
                bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 16));
                const float mn = fmaxf(st.m[h], bm);
                const float corr = exp2f(st.m[h] - mn);
                pr[h] = valid ? exp2f(sv - mn) : 0.f;
                float bs = pr[h] + __shfl_xor_sync(0xffffffffu, pr[h], 4);
                bs += __shfl_xor_sync(0xffffffffu, bs, 8);
                bs += __shfl_xor_sync(0xffffffffu, bs, 16);
                st.l[h] = st.l[h] * corr + bs;
                st.m[h] = mn;
#pragma unroll
                for (int i = 0; i < DL; ++i) st.acc[h][i] *= corr;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
#pragma unroll
                for (int h = 0; h < GRP; ++h) {
                    const float pj = __shfl_sync(0xffffffffu, pr[h], 4 * j);
#pragma unroll
                    for (int i = 0; i < DL; ++i) st.acc[h][i] = fmaf(pj, vf[j][i], st.acc[h][i]);
                }
            }
        }
    }
};

template <int GRP, int D, int NW>
__device__ __forceinline__ void decode_keys_warp(const __nv_bfloat16* kbase, const __nv_bfloat16* vbase,
                                                 int64_t k_begin, int64_t k_end, int warp, int lane,
                                                 const float (*qs)[D], DecodeWarpState<GRP, D>& st) {
    DecodeKeyLoop<GRP, D, NW> loop(kbase, vbase, k_begin, k_end, warp, lane);
    loop.run(qs, st);
}

// Publishes the warp states (sm_m/sm_l per warp, sm_o per warp) for a
// CTA-level merge.
template <int GRP, int D>
__device__ __forceinline__ void decode_publish_warp(const DecodeWarpState<GRP, D>& st, int warp, int lane,
                                                    float (*sm_m)[GRP], float (*sm_l)[GRP], float (*sm_o)[GRP][D]) {
    constexpr int DL = D / 32;
    if (lane == 0) {
#pragma unroll
        for (int h = 0; h < GRP; ++h) {
            sm_m[warp][h] = st.m[h];
            sm_l[warp][h] = st.l[h];
        }
    }
#pragma unroll
    for (int h = 0; h < GRP; ++h)
#pragma unroll
        for (int i = 0; i < DL; ++i) sm_o[warp][h][lane * DL + i] = st.acc[h][i];
}

// Merges the published warp states of element e = (head h, dim dd): returns
// the CTA's max M, sum Ls and unnormalised output O for it.
template <int GRP, int D, int NW>
__device__ __forceinline__ void decode_merge_warps(int h, int dd, const float (*sm_m)[GRP], const float (*sm_l)[GRP],
                                                   const float (*sm_o)[GRP][D], float& M, float& Ls, float& O) {
    M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, sm_m[w][h]);
    Ls = 0.f;
    O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float f = exp2f(sm_m[w][h] - M);
            Ls += sm_l[w][h] * f;
            O += sm_o[w][h][dd] * f;
        }
    }
}

// cos/sin of RoPE pair i at position pos: the session table when given, else
// the double-precision formula (the same values).
template <int D>
__device__ __forceinline__ void rope_cs(const float* cos_sin, double theta, int64_t pos, int i, float& c, float& s) {
    if (cos_sin) {
        const float2 v = reinterpret_cast<const float2*>(cos_sin)[pos * (D / 2) + i];
        c = v.x;
        s = v.y;
    } else {
        rope_angle(theta, D, pos, i, c, s);
    }
}

// The GRP query heads at qrow, rotated at pos, rounded to bf16 as the
// in-place RoPE store rounds them, times scale_log2, into qs. Threads
// tid = 0 .. nthreads - 1 share the work.
template <int GRP, int D, bool CG = false>
__device__ __forceinline__ void rope_stage_q(const __nv_bfloat16* qrow, int64_t pos, const float* cos_sin, double theta,
                                             float scale_log2, float (*qs)[D], int tid, int nthreads) {
    constexpr int HALF = D / 2;
    auto ld = [](const __nv_bfloat16* ptr) {
        if constexpr (CG) return __ldcg(ptr);
        else return *ptr;
    };
    for (int i = tid; i < GRP * HALF; i += nthreads) {
        const int h = i / HALF, j = i % HALF;
        float c, s;
        rope_cs<D>(cos_sin, theta, pos, j, c, s);
        const float x1 = __bfloat162float(ld(qrow + h * D + j)), x2 = __bfloat162float(ld(qrow + h * D + j + HALF));
        const float o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
        const float o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
        qs[h][j] = Act<__nv_bfloat16>::round(o1) * scale_log2;
        qs[h][j + HALF] = Act<__nv_bfloat16>::round(o2) * scale_log2;
    }
}

// Appends one token of one kv head: k rotated at pos into kdst, v copied.
template <int D, bool CG = false>
__device__ __forceinline__ void rope_append_kv(const __nv_bfloat16* krow, const __nv_bfloat16* vrow,
                                               __nv_bfloat16* kdst, __nv_bfloat16* vdst, int64_t pos,
                                               const float* cos_sin, double theta, int tid, int nthreads) {
    constexpr int HALF = D / 2;
    auto ld = [](const __nv_bfloat16* ptr) {
        if constexpr (CG) return __ldcg(ptr);
        else return *ptr;
    };
    for (int j = tid; j < HALF; j += nthreads) {
        float c, s;
        rope_cs<D>(cos_sin, theta, pos, j, c, s);
        const float x1 = __bfloat162float(ld(krow + j)), x2 = __bfloat162float(ld(krow + j + HALF));
        kdst[j] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)));
        kdst[j + HALF] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s)));
    }
    for (int j = tid; j < D; j += nthreads) vdst[j] = ld(vrow + j);
}

}  // namespace amcu
