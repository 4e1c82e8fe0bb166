// Shared device helpers for the sm_100a kernels of the Llama hot path.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "aethermind_b200.h"

namespace amcu {

constexpr int kNumSMs = 148;  // B200: 2 dies x 74 SMs

// Activation storage types. `load`/`store` convert to/from the fp32 compute type
// with a single round-to-nearest-even on store, matching the reference's
// "compute in fp32, round once to the storage dtype" rule.
template <typename T> struct Act;
template <> struct Act<float> {
    static __device__ __forceinline__ float load(float v) { return v; }
    static __device__ __forceinline__ float store(float v) { return v; }
    static __device__ __forceinline__ float round(float v) { return v; }
};
template <> struct Act<__nv_bfloat16> {
    static __device__ __forceinline__ float load(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 store(float v) { return __float2bfloat16_rn(v); }
    static __device__ __forceinline__ float round(float v) {
        return __bfloat162float(__float2bfloat16_rn(v));
    }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Streaming 128-bit global load that bypasses L1 allocation (weights are read
// exactly once per step).
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint4 ld_u4(const void* p) {
    return *reinterpret_cast<const uint4*>(p);
}

// RoPE angle of pair i at position pos: inv_freq = 1 / theta^(2i/d) and the
// angle in double, cos/sin rounded to float.
__device__ __forceinline__ void rope_angle(double theta, int64_t d, int64_t pos, int64_t i, float& c, float& s) {
    const double inv = 1.0 / pow(theta, 2.0 * (double)i / (double)d);
    const double ang = (double)pos * inv;
    c = (float)cos(ang);
    s = (float)sin(ang);
}

// SiLU with the sign branch of the reference's const evaluator.
__device__ __forceinline__ float silu_ref(float g) {
    if (g >= 0.f) return g / (1.f + expf(-g));
    const float e = expf(g);
    return g * e / (1.f + e);
}

// ---------------------------------------------------------------------------
// Device error word (one int32 per device, host side: amcu::device_error_word()):
// a kernel whose bounded wait runs out records a code there and returns
// instead of hanging; the host reads and clears it with amcu_device_error().
// ---------------------------------------------------------------------------
constexpr long long kSpinLimitCycles = 4000000000LL;  // ~2 s at 1.9 GHz
constexpr int32_t kErrGemvFullWait = 0x101, kErrGemvEmptyWait = 0x102, kErrGemvDrain = 0x103;

__device__ __forceinline__ void record_device_error(int32_t* word, int32_t code) {
    if (word) atomicCAS(word, 0, code);
}

// ---- mbarrier + bulk-copy (TMA engine) helpers ----
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
    return ok != 0;
}
// Non-blocking test of the phase with the given parity.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
            "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
    return ok != 0;
}
// Bounded wait for the phase with the given parity; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kSpinLimitCycles) return false;
    return true;
}
// An L2 policy that evicts these lines first: for data read exactly once
// (streamed weights), so it does not push out what is read again soon.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// Global -> shared bulk copy with an L2 cache policy, completing on `bar`.
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
    asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
                    "r"(smem_u32(dst)),
            "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
            : "memory");
}
// Global -> shared bulk copy completing on `bar` (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ uint4 lds_u4(const void* p) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "r"(smem_u32(p)));
    return r;
}
__device__ __forceinline__ uint32_t lds_u32(const void* p) {
    uint32_t r;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(r) : "r"(smem_u32(p)));
    return r;
}
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---- programmatic dependent launch (PDL) ----
// Kernels of the decode/prefill path are launched with programmatic stream
// serialization (launch_pdl), so a kernel's CTAs may start while the kernel
// before it on the stream is still running. Every such kernel calls pdl_wait()
// before it reads or writes anything the earlier kernels produce or consume;
// work that depends on nothing (weight prefetch) goes before it. pdl_wait
// returns once all earlier kernels have completed and their writes are
// visible, so chains stay ordered transitively. pdl_trigger() lets the next
// kernel's CTAs be scheduled; without it they start at this kernel's exit.
// Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Asks the TMA engine to pull [p, p + bytes) into L2 (no completion to wait
// on). p 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// This CTA's share of an L2 prefetch hint: the ranges are split evenly over
// the grid's CTAs (4 KB granules) and thread 0 requests its share in pieces
// of at most 64 KB.
__device__ __forceinline__ void l2_prefetch_share(const AmcuL2Prefetch& pf) {
    if (threadIdx.x != 0) return;
    const uint64_t nb = (uint64_t)gridDim.x * gridDim.y * gridDim.z;
    const uint64_t b = blockIdx.x + (uint64_t)gridDim.x * (blockIdx.y + (uint64_t)gridDim.y * blockIdx.z);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const uint64_t bytes = pf.bytes[r] & ~(uint64_t)15;
        if (pf.ptr[r] == nullptr || bytes == 0) continue;
        const uint64_t per = ((bytes + nb - 1) / nb + 4095) & ~(uint64_t)4095;
        const uint64_t begin = b * per;
        const uint64_t end = begin + per < bytes ? begin + per : bytes;
        for (uint64_t off = begin; off < end; off += 65536) {
            const uint64_t n = end - off < 65536 ? end - off : 65536;
            prefetch_l2_bulk(static_cast<const uint8_t*>(pf.ptr[r]) + off, (uint32_t)n);
        }
    }
}

// Orderable 32-bit key of a float (total order matching float <, NaN last).
__device__ __forceinline__ uint32_t float_order_key(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

}  // namespace amcu
