// Offline weight quantizer and dtype conversion for checkpoint loading.
//
// The reference declares INT8 per-channel and INT4 group-wise weight-only
// quantization (docs/products/aethermind_prd.md:216, QuantizationSpec in
// include/aethermind/graph/graph_types.h:123-138) but ships no quantizer; this
// is the symmetric absmax recipe, written into the canonical formats the
// prepacker takes (include/aethermind_b200.h):
//   INT4, group g along K: s = fp16(max|w| / 7) per (row, group),
//        q = clamp(rint(w / s), -8, 7) (round half to even), two values per
//        byte, low nibble = even k;
//   INT8, per output row:  s = max|w| / 127 (fp32), q = clamp(rint(w / s), -127, 127).
// A group or row of zeros gets s = 0 and q = 0. The division is the correctly
// rounded fp32 one, so a CPU restatement gives the same bytes.
#include "../amcu_internal.h"
#include "common.cuh"

namespace amcu {

__device__ __forceinline__ float load_as_float(const void* p, int dtype, int64_t i) {
    if (dtype == AMCU_F32) return static_cast<const float*>(p)[i];
    if (dtype == AMCU_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(static_cast<const __half*>(p)[i]);
}

// One warp per (row, group of 128); lane l holds columns 4l .. 4l + 3.
__global__ void quantize_w4_kernel(const void* w, int dtype, int64_t n, int64_t k, uint8_t* q, uint16_t* s) {
    const int lane = threadIdx.x & 31;
    const int64_t unit = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int64_t G = k / 128;
    if (unit >= n * G) return;
    const int64_t row = unit / G, grp = unit % G;
    const int64_t base = row * k + grp * 128 + lane * 4;
    float v[4], amax = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[i] = load_as_float(w, dtype, base + i);
        amax = fmaxf(amax, fabsf(v[i]));
    }
    amax = warp_max(amax);
    const __half sh = __float2half_rn(__fdiv_rn(amax, 7.0f));
    const float sc = __half2float(sh);
    uint8_t nib[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float r = sc > 0.f ? rintf(__fdiv_rn(v[i], sc)) : 0.f;
        r = fminf(fmaxf(r, -8.f), 7.f);
        nib[i] = (uint8_t)((int)r & 0xF);
    }
    uint8_t* qr = q + row * (k / 2) + grp * 64 + lane * 2;
    qr[0] = (uint8_t)(nib[0] | (nib[1] << 4));
    qr[1] = (uint8_t)(nib[2] | (nib[3] << 4));
    if (lane == 0) s[row * G + grp] = *reinterpret_cast<const uint16_t*>(&sh);
}

// One 256-thread block per row.
__global__ void quantize_w8_kernel(const void* w, int dtype, int64_t n, int64_t k, int8_t* q, float* s) {
    __shared__ float red[8];
    const int64_t row = blockIdx.x;
    const int tid = threadIdx.x;
    float amax = 0.f;
    for (int64_t c = tid; c < k; c += blockDim.x) amax = fmaxf(amax, fabsf(load_as_float(w, dtype, row * k + c)));
    amax = warp_max(amax);
    if ((tid & 31) == 0) red[tid >> 5] = amax;
    __syncthreads();
    float m = 0.f;
    for (int i = 0; i < (int)(blockDim.x / 32); ++i) m = fmaxf(m, red[i]);
    const float sc = __fdiv_rn(m, 127.0f);
    for (int64_t c = tid; c < k; c += blockDim.x) {
        float r = sc > 0.f ? rintf(__fdiv_rn(load_as_float(w, dtype, row * k + c), sc)) : 0.f;
        r = fminf(fmaxf(r, -127.f), 127.f);
        q[row * k + c] = (int8_t)r;
    }
    if (tid == 0) s[row] = sc;
}

__global__ void convert_kernel(const void* src, int sdt, void* dst, int ddt, int64_t count) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = load_as_float(src, sdt, i);
        if (ddt == AMCU_F32) static_cast<float*>(dst)[i] = v;
        else static_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(v);
    }
}

}  // namespace amcu

using namespace amcu;

extern "C" am_status_code amcu_quantize_weight(int32_t format, const void* w, int32_t w_dtype, int64_t n, int64_t k,
                                               int64_t group, void* q, void* scales, void* stream) {
    AMCU_REQUIRE(w && q && scales, "amcu_quantize_weight: null pointer");
    AMCU_REQUIRE(w_dtype == AMCU_F32 || w_dtype == AMCU_BF16 || w_dtype == AMCU_F16,
                 "amcu_quantize_weight: source dtype must be f32, bf16 or f16");
    AMCU_REQUIRE(n > 0 && k > 0, "amcu_quantize_weight: n and k must be positive");
    cudaStream_t s = as_stream(stream);
    if (format == AMCU_WFMT_INT4) {
        AMCU_REQUIRE(group == 128 && k % 128 == 0, "amcu_quantize_weight: int4 needs group 128 and k %% 128 == 0");
        const int64_t units = n * (k / 128);
        quantize_w4_kernel<<<(unsigned)ceil_div(units, 8), 256, 0, s>>>(w, w_dtype, n, k, static_cast<uint8_t*>(q),
                                                                        static_cast<uint16_t*>(scales));
    } else if (format == AMCU_WFMT_INT8) {
        quantize_w8_kernel<<<(unsigned)n, 256, 0, s>>>(w, w_dtype, n, k, static_cast<int8_t*>(q),
                                                       static_cast<float*>(scales));
    } else {
        return set_error(AM_STATUS_INVALID_ARGUMENT, "amcu_quantize_weight: format must be INT4 or INT8");
    }
    return check_launch("amcu_quantize_weight");
}

extern "C" am_status_code amcu_convert(const void* src, int32_t src_dtype, void* dst, int32_t dst_dtype, int64_t count,
                                       void* stream) {
    AMCU_REQUIRE(src && dst, "amcu_convert: null pointer");
    AMCU_REQUIRE(src_dtype == AMCU_F32 || src_dtype == AMCU_BF16 || src_dtype == AMCU_F16,
                 "amcu_convert: source dtype must be f32, bf16 or f16");
    AMCU_REQUIRE(dst_dtype == AMCU_F32 || dst_dtype == AMCU_BF16, "amcu_convert: destination dtype must be f32 or bf16");
    if (count <= 0) return AM_STATUS_OK;
    const unsigned blocks = (unsigned)(ceil_div(count, 256) < 4096 ? ceil_div(count, 256) : 4096);
    convert_kernel<<<blocks, 256, 0, as_stream(stream)>>>(src, src_dtype, dst, dst_dtype, count);
    return check_launch("amcu_convert");
}
