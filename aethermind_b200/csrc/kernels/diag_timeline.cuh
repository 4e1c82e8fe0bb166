// Diagnostics (AMCU_DIAG builds only; the default build compiles all of this
// out): a per-CTA launch timeline. Every instrumented CTA appends one record
// with its SM, the globaltimer at entry, when its dependency wait returned,
// up to two marks in between (fields pad, pad2) and when its work was done. Each
// translation unit that includes this header keeps its own log (file-scope
// device arrays); its amcu_diag_timeline_*
// export copies the log out and resets it. The host merges the logs by time:
// a dependent kernel's CTAs finish after every CTA of the kernel before it,
// so records sorted by finish time fall into one group per launch.
#pragma once
#include <stdint.h>

namespace amcu {

struct DiagTlRec {
    uint32_t tag, cta, smid, grid;
    unsigned long long t_entry, t_wait, t_done, pad, pad2, pad3, pad4, pad5;
};

#ifdef AMCU_DIAG
constexpr int kDiagTlMax = 1 << 18;
static __device__ DiagTlRec g_diag_tl[kDiagTlMax];
static __device__ unsigned int g_diag_tl_n;

__device__ __forceinline__ unsigned long long diag_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
struct DiagTl {
    unsigned long long t_entry = 0, t_wait = 0, t_mark = 0, t_mark2 = 0;
    __device__ __forceinline__ void entry() { t_entry = diag_now(); }
    __device__ __forceinline__ void mark() { t_mark = diag_now(); }
    __device__ __forceinline__ void mark2() { t_mark2 = diag_now(); }
    __device__ __forceinline__ void waited() { t_wait = diag_now(); }
    __device__ __forceinline__ void done(uint32_t tag) {
        const unsigned int i = atomicAdd(&g_diag_tl_n, 1u);
        if (i >= (unsigned)kDiagTlMax) return;
        unsigned int sm;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
        DiagTlRec r;
        r.tag = tag;
        r.cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
        r.smid = sm;
        r.grid = gridDim.x * gridDim.y * gridDim.z;
        r.t_entry = t_entry;
        r.t_wait = t_wait;
        r.t_done = diag_now();
        r.pad = t_mark;
        r.pad2 = t_mark2;
        r.pad3 = r.pad4 = r.pad5 = 0;
        g_diag_tl[i] = r;
    }
};
// Host side: copy up to `max` records into `out`, reset the log; returns the
// number of records written (or -1 on a CUDA error).
static inline int diag_timeline_take(void* out, int max) {
    unsigned int n = 0;
    if (cudaMemcpyFromSymbol(&n, g_diag_tl_n, sizeof(n)) != cudaSuccess) return -1;
    if (n > (unsigned)kDiagTlMax) n = kDiagTlMax;
    if ((int)n > max) n = (unsigned)max;
    if (n && cudaMemcpyFromSymbol(out, g_diag_tl, n * sizeof(DiagTlRec)) != cudaSuccess) return -1;
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_diag_tl_n, &zero, sizeof(zero)) != cudaSuccess) return -1;
    return (int)n;
}
#define AMCU_DIAG_TL(x) x
#else
struct DiagTl {
    __device__ __forceinline__ void entry() {}
    __device__ __forceinline__ void waited() {}
    __device__ __forceinline__ void mark() {}
    __device__ __forceinline__ void mark2() {}
    __device__ __forceinline__ void done(uint32_t) {}
};
#define AMCU_DIAG_TL(x)
#endif

}  // namespace amcu
