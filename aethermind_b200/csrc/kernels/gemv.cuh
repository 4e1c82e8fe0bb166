// Host-visible launch interface of the GEMV / GEMM kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace amcu {

constexpr int kGemvThreads = 256;  // upper bound: a CTA has one warp per K chunk (<= 8)
constexpr int kGemvMaxM = 8;

// K-chunked stream layout of quantized weights. The K tiles (64 columns) of
// a row block are split into `kc` chunks of `tw` tiles (tw a multiple of
// kTwAlign, the tail zero-padded); the packed weight is stored chunk-major:
// tile (rb, c) sits at stream index (c / tw * nrb + rb) * tw + c % tw. One
// GEMV warp owns one chunk, so its tiles for consecutive row blocks form one
// contiguous stream. kc (1..8) is chosen for the least padding, ties going to
// more chunks. kStreamPadBytes of slack after the stream absorb the ring's
// read-ahead past a warp's last tile.
constexpr int kTwAlign = 4;
constexpr int64_t kStreamPadBytes = 16384;
constexpr int64_t kScalePadBytes = 256;
struct StreamGeom {
    int kc;  // chunks = warps per CTA
    int tw;  // tiles per chunk and row block
};
inline __host__ __device__ StreamGeom stream_geom(int64_t k) {
    const int64_t c = k / 64;
    StreamGeom best{1, (int)((c + kTwAlign - 1) / kTwAlign * kTwAlign)};
    int64_t best_tiles = best.tw;
    for (int kc = 2; kc <= 8; ++kc) {
        int64_t tw = (c + kc - 1) / kc;
        tw = (tw + kTwAlign - 1) / kTwAlign * kTwAlign;
        if (kc * tw <= best_tiles) {
            best = StreamGeom{kc, (int)tw};
            best_tiles = kc * tw;
        }
    }
    return best;
}

struct GemvParams {
    const void* x;
    const void* w;
    const void* scales;
    void* y;
    const void* residual;
    int64_t m, n, k;
    int64_t x_stride, y_stride;
    int32_t* err;     // device error word for bounded waits
    const void* norm_w;  // optional fused RMSNorm weight [k] (bf16)
    float eps;
    int rb_per_cta;   // set by the launcher
    int kc, tw;       // stream geometry (set by the launcher)
};

// Quantized (INT4 / INT8 tile16x64) GEMV, m <= kGemvMaxM, bf16 activations.
void launch_gemv(const GemvParams& p, int fmt, int epi, cudaStream_t s);
// Plain weights in the activation dtype, any m.
void launch_gemm_plain(const GemvParams& p, int dtype, int epi, cudaStream_t s);

}  // namespace amcu
