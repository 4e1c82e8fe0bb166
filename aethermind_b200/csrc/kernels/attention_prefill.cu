// Causal GQA prefill attention on the tensor cores (bf16), flash style.
//
// out[row, h, :] = softmax(q[row, h, :] . K[0 .. pos]^T / sqrt(d)) . V[0 .. pos]
// for the rows of a prompt (row i of sequence b sits at position
// seq_pos[b] + i; keys come from the static cache, already holding this
// prompt's rows), the Attention node of the reference
// (src/operators/attention_op.cpp:65-147: causal, GQA head map
// kv_head = q_head / (n_q / n_kv)).
//
// A CTA takes 64 query rows of one q head; each of its 4 warps owns 16 rows.
// Key tiles of 64 rows go through shared memory in two stages (cp.async: the
// next tile loads while this one is used), K and V both row-major with rows
// padded to 16 bytes apart modulo 128, so the ldmatrix fragment loads (K
// plain, V transposed) hit distinct banks. Per tile a warp
// computes S = Q K^T with mma.sync m16n8k16 (bf16 in, fp32 out), masks the
// keys past each row's position, updates the running max / sum (online
// softmax in base 2, fp32), and accumulates O += P V with P converted to bf16
// straight from the S accumulators (their C-fragment layout is the A-fragment
// layout of the next MMA). The output is O / sum, rounded once to bf16.
#include "../amcu_internal.h"
#include "common.cuh"
#include "mma_int4.cuh"

namespace amcu {

constexpr int kFpBM = 64;  // query rows per CTA
constexpr int kFpBN = 64;  // keys per tile
constexpr int kFpThreads = 128;
constexpr float kFpLog2e = 1.4426950408889634f;

struct FpParams {
    const __nv_bfloat16* q;
    int64_t q_stride;
    const __nv_bfloat16* kc;
    const __nv_bfloat16* vc;
    int64_t slot_stride, capacity;
    const int32_t* seq_pos;
    __nv_bfloat16* out;
    int64_t out_stride;
    int64_t R;    // rows per sequence
    int64_t nq;   // query heads
    int grp;      // query heads per kv head
    float scale_log2;
};

__device__ __forceinline__ uint32_t ld_b32(const __nv_bfloat16* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
// 16-byte global -> shared copy; src_bytes 0 fills the 16 bytes with zeros
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int D>
constexpr int fp_smem_bytes() { return 2 * 2 * kFpBN * (D + 8) * 2; }  // [K, V][2 stages][64 keys][D + 8]

template <int D>
__global__ void __launch_bounds__(kFpThreads) attn_prefill_flash_kernel(FpParams p) {
    constexpr int KS = D / 16;     // k-steps of S = Q K^T
    constexpr int DT = D / 8;      // n-tiles of O
    constexpr int ST = D + 8;      // K / V row stride in shared memory (elements): 16 B apart mod 128 B,
                                   // so the 8 rows of an ldmatrix hit distinct banks
    constexpr int TILE = kFpBN * ST;
    extern __shared__ __align__(16) __nv_bfloat16 fp_smem[];
    __nv_bfloat16* Ks = fp_smem;              // [2][64][ST]
    __nv_bfloat16* Vs = fp_smem + 2 * TILE;   // [2][64][ST]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int64_t b = blockIdx.z, h = blockIdx.y;
    const int64_t kvh = h / p.grp;
    // the longest causal row blocks first (they need the most key tiles)
    const int64_t i0 = (int64_t)(gridDim.x - 1 - blockIdx.x) * kFpBM;
    pdl_wait();
    pdl_trigger();
    const int64_t p0 = p.seq_pos[b];
    const int64_t last = (i0 + kFpBM < p.R ? i0 + kFpBM : p.R) - 1;  // last valid row of the CTA
    int64_t L = p0 + last + 1;                                       // keys this CTA needs
    if (L > p.capacity) L = p.capacity;

    const __nv_bfloat16* kbase = p.kc + b * p.slot_stride + kvh * p.capacity * D;
    const __nv_bfloat16* vbase = p.vc + b * p.slot_stride + kvh * p.capacity * D;
    const int ntiles = (int)((L + kFpBN - 1) / kFpBN);
    // keys k0 .. k0 + 63 of K and V into stage st (zeros past L)
    auto load_tile = [&](int kt, int st) {
        const int64_t k0 = (int64_t)kt * kFpBN;
        for (int e = threadIdx.x; e < kFpBN * (D / 8); e += kFpThreads) {
            const int kr = e / (D / 8), c8 = e % (D / 8);
            const int64_t key = k0 + kr;
            const bool in = key < L;
            const int64_t off = (in ? key : 0) * D + c8 * 8;
            cp_async16(Ks + st * TILE + kr * ST + c8 * 8, kbase + off, in ? 16u : 0u);
            cp_async16(Vs + st * TILE + kr * ST + c8 * 8, vbase + off, in ? 16u : 0u);
        }
        cp_async_commit();
    };
    if (ntiles > 0) load_tile(0, 0);

    // this lane's two rows (g and g+8 of the warp's 16) and their positions
    const int64_t ra = i0 + warp * 16 + g, rb = ra + 8;
    const int64_t pa = p0 + ra, pb = p0 + rb;
    const __nv_bfloat16* qa_row = p.q + (b * p.R + (ra < p.R ? ra : 0)) * p.q_stride + h * D;
    const __nv_bfloat16* qb_row = p.q + (b * p.R + (rb < p.R ? rb : 0)) * p.q_stride + h * D;
    uint32_t qf[KS][4];
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
        qf[ks][0] = ra < p.R ? ld_b32(qa_row + 16 * ks + 2 * t) : 0u;
        qf[ks][1] = rb < p.R ? ld_b32(qb_row + 16 * ks + 2 * t) : 0u;
        qf[ks][2] = ra < p.R ? ld_b32(qa_row + 16 * ks + 2 * t + 8) : 0u;
        qf[ks][3] = rb < p.R ? ld_b32(qb_row + 16 * ks + 2 * t + 8) : 0u;
    }
    float o[DT][4];
#pragma unroll
    for (int i = 0; i < DT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float ma = -INFINITY, mb = -INFINITY, la = 0.f, lb = 0.f;

    // ldmatrix lane roles: lane l addresses row l % 8 of matrix l / 8
    const int lm = lane >> 3, lr = lane & 7;
    for (int kt = 0; kt < ntiles; ++kt) {
        const int st = kt & 1;
        if (kt + 1 < ntiles) {
            load_tile(kt + 1, st ^ 1);  // that stage was last read in iteration kt - 1
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();  // tile kt is in shared memory for every thread
        const __nv_bfloat16* Kt = Ks + st * TILE;
        const __nv_bfloat16* Vt = Vs + st * TILE;
        const int64_t k0 = (int64_t)kt * kFpBN;
        // ---- S = Q K^T for this warp's 16 rows x 64 keys. B[k = d][n = key] =
        // K[key][d]: one ldmatrix.x4 gives n-tile nt's fragments of k-steps
        // ks and ks + 1 (matrices: d 16ks, 16ks+8, 16ks+16, 16ks+24)
        float s[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
            for (int ks = 0; ks < KS; ks += 2) {
                uint32_t kf[4];
                ldsm_x4(kf, Kt + (nt * 8 + lr) * ST + 16 * ks + 8 * lm);
                mma_bf16_16816(s[nt], qf[ks], kf[0], kf[1]);
                mma_bf16_16816(s[nt], qf[ks + 1], kf[2], kf[3]);
            }
        }
        // ---- causal mask, scale, running max
        float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const int64_t key = k0 + nt * 8 + 2 * t;
            s[nt][0] = key <= pa ? s[nt][0] * p.scale_log2 : -INFINITY;
            s[nt][1] = key + 1 <= pa ? s[nt][1] * p.scale_log2 : -INFINITY;
            s[nt][2] = key <= pb ? s[nt][2] * p.scale_log2 : -INFINITY;
            s[nt][3] = key + 1 <= pb ? s[nt][3] * p.scale_log2 : -INFINITY;
            mxa = fmaxf(mxa, fmaxf(s[nt][0], s[nt][1]));
            mxb = fmaxf(mxb, fmaxf(s[nt][2], s[nt][3]));
        }
        mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
        mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
        mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
        mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
        const float na = fmaxf(ma, mxa), nb = fmaxf(mb, mxb);
        // a row with every key so far masked keeps max -inf: use 0 as the
        // reference so exp2 gives 0, not NaN
        const float ra_ref = na == -INFINITY ? 0.f : na, rb_ref = nb == -INFINITY ? 0.f : nb;
        const float ca = exp2f(ma - ra_ref), cb = exp2f(mb - rb_ref);
        ma = na;
        mb = nb;
        la *= ca;
        lb *= cb;
#pragma unroll
        for (int i = 0; i < DT; ++i) {
            o[i][0] *= ca;
            o[i][1] *= ca;
            o[i][2] *= cb;
            o[i][3] *= cb;
        }
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            s[nt][0] = exp2f(s[nt][0] - ra_ref);
            s[nt][1] = exp2f(s[nt][1] - ra_ref);
            s[nt][2] = exp2f(s[nt][2] - rb_ref);
            s[nt][3] = exp2f(s[nt][3] - rb_ref);
            la += s[nt][0] + s[nt][1];
            lb += s[nt][2] + s[nt][3];
        }
        // ---- O += P V, k-step kk covers keys 16 kk .. +15 (n-tiles 2kk, 2kk+1
        // of S). B[k = key][n = d] = V[key][d]: one ldmatrix.x4.trans gives the
        // fragments of d-tiles dt and dt + 1 (matrices: keys +0 / +8 x d 8dt / 8dt+8)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const uint32_t pf[4] = {pack_bf16(s[2 * kk][0], s[2 * kk][1]), pack_bf16(s[2 * kk][2], s[2 * kk][3]),
                                    pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]),
                                    pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
            for (int dt = 0; dt < DT; dt += 2) {
                uint32_t vf[4];
                ldsm_x4_trans(vf, Vt + (kk * 16 + 8 * (lm & 1) + lr) * ST + 8 * (dt + (lm >> 1)));
                mma_bf16_16816(o[dt], pf, vf[0], vf[1]);
                mma_bf16_16816(o[dt + 1], pf, vf[2], vf[3]);
            }
        }
        __syncthreads();  // every warp is done with stage st before it is refilled
    }
    // ---- normalise and store
    la += __shfl_xor_sync(0xffffffffu, la, 1);
    la += __shfl_xor_sync(0xffffffffu, la, 2);
    lb += __shfl_xor_sync(0xffffffffu, lb, 1);
    lb += __shfl_xor_sync(0xffffffffu, lb, 2);
    const float ia = la > 0.f ? 1.f / la : 0.f, ib = lb > 0.f ? 1.f / lb : 0.f;
    if (ra < p.R) {
        __nv_bfloat16* orow = p.out + (b * p.R + ra) * p.out_stride + h * D + 2 * t;
#pragma unroll
        for (int dt = 0; dt < DT; ++dt)
            *reinterpret_cast<uint32_t*>(orow + dt * 8) = pack_bf16(o[dt][0] * ia, o[dt][1] * ia);
    }
    if (rb < p.R) {
        __nv_bfloat16* orow = p.out + (b * p.R + rb) * p.out_stride + h * D + 2 * t;
#pragma unroll
        for (int dt = 0; dt < DT; ++dt)
            *reinterpret_cast<uint32_t*>(orow + dt * 8) = pack_bf16(o[dt][2] * ib, o[dt][3] * ib);
    }
}

// Launches the tensor-core prefill attention; false when the shape is not
// one it handles (bf16, head_dim 64 or 128, rows a multiple of rows_per_seq).
bool launch_attn_prefill_flash(const AmcuAttentionArgs* a, cudaStream_t s) {
    if (a->dtype != AMCU_BF16 || (a->head_dim != 64 && a->head_dim != 128)) return false;
    if (a->rows % a->rows_per_seq != 0) return false;
    const int64_t qs = a->q_stride ? a->q_stride : a->n_q_heads * a->head_dim;
    const int64_t os = a->out_stride ? a->out_stride : a->n_q_heads * a->head_dim;
    if (qs % 2 != 0 || os % 2 != 0 || !aligned(a->out, 4)) return false;
    const int64_t slot = a->slot_stride ? a->slot_stride : a->n_kv_heads * a->capacity * a->head_dim;
    if (!aligned(a->k_cache, 16) || !aligned(a->v_cache, 16) || slot % 8 != 0) return false;  // 16-byte copies
    FpParams p{};
    p.q = static_cast<const __nv_bfloat16*>(a->q);
    p.q_stride = qs;
    p.kc = static_cast<const __nv_bfloat16*>(a->k_cache);
    p.vc = static_cast<const __nv_bfloat16*>(a->v_cache);
    p.capacity = a->capacity;
    p.slot_stride = a->slot_stride ? a->slot_stride : a->n_kv_heads * a->capacity * a->head_dim;
    p.seq_pos = a->seq_pos;
    p.out = static_cast<__nv_bfloat16*>(a->out);
    p.out_stride = os;
    p.R = a->rows_per_seq;
    p.nq = a->n_q_heads;
    p.grp = (int)(a->n_q_heads / a->n_kv_heads);
    p.scale_log2 = (float)(1.0 / sqrt((double)a->head_dim)) * kFpLog2e;
    const dim3 grid((unsigned)((p.R + kFpBM - 1) / kFpBM), (unsigned)a->n_q_heads, (unsigned)(a->rows / p.R));
    if (a->head_dim == 128) {
        set_func_attr_once((const void*)attn_prefill_flash_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           fp_smem_bytes<128>());
        launch_pdl(attn_prefill_flash_kernel<128>, grid, dim3(kFpThreads), fp_smem_bytes<128>(), s, p);
    } else {
        set_func_attr_once((const void*)attn_prefill_flash_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           fp_smem_bytes<64>());
        launch_pdl(attn_prefill_flash_kernel<64>, grid, dim3(kFpThreads), fp_smem_bytes<64>(), s, p);
    }
    return true;
}

}  // namespace amcu
