// Shared device helpers for the sm_100a kernels of the Llama hot path.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

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

// SiLU with the sign branch of the reference's const evaluator.
__device__ __forceinline__ float silu_ref(float g) {
    if (g >= 0.f) return g / (1.f + expf(-g));
    const float e = expf(g);
    return g * e / (1.f + e);
}

// Orderable 32-bit key of a float (total order matching float <, NaN last).
__device__ __forceinline__ uint32_t float_order_key(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

}  // namespace amcu
