// Tensor-core helpers of the quantized GEMVs: legacy mma.sync fragments
// (m16n8k16, fp32 accumulate) and the nibble / byte unpacks that feed them
// from the tile16x64 layout (gemv.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace amcu {

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Four int8 values -> two bf16x2 (bytes 0,1) and (bytes 2,3); exact.
__device__ __forceinline__ void unpack_w8_word(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t u = w ^ 0x80808080u;  // offset binary: q + 128
    float f[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t bits = __byte_perm(u, 0x4B000000u, 0x7650u + i);  // 0x4B0000bb = 2^23 + bb
        f[i] = __uint_as_float(bits) - 8388736.0f;                      // - (2^23 + 128)
    }
    __nv_bfloat162 p0 = __floats2bfloat162_rn(f[0], f[1]);
    __nv_bfloat162 p1 = __floats2bfloat162_rn(f[2], f[3]);
    lo = *reinterpret_cast<uint32_t*>(&p0);
    hi = *reinterpret_cast<uint32_t*>(&p1);
}

// INT4 word -> fp16 MMA registers: a0/a2 = 1032 + q (bits 0-3, 8-11 of each
// half: rows g), a1/a3 = 1152 + 16q (bits 4-7, 12-15: rows g+8). (w & mask)
// ^ c flips the nibble's sign bit (n ^ 8 = q + 8) and sets exponent 1024.
__device__ __forceinline__ void unpack_w4_word_f16(uint32_t w, uint32_t (&a)[4]) {
    const uint32_t w8 = w >> 8;
    asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(a[0]) : "r"(w), "r"(0x000F000Fu), "r"(0x64086408u));
    asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(a[1]) : "r"(w), "r"(0x00F000F0u), "r"(0x64806480u));
    asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(a[2]) : "r"(w8), "r"(0x000F000Fu), "r"(0x64086408u));
    asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(a[3]) : "r"(w8), "r"(0x00F000F0u), "r"(0x64806480u));
}

}  // namespace amcu
