// One-shot all-reduce + residual add over peer memory (tensor-parallel decode).
//
// Every rank owns one device area (cudaMalloc, shared with the other ranks of
// the box through CUDA IPC):
//   mailbox [2 parities][kArMaxRanks sources][kArMaxElems] bf16
//   flags   [kArMaxRanks sources][kArMaxCtas] u32   (written by the peers)
//   epochs  [kArMaxCtas] u32                        (this rank only)
// A call sums the ranks' bf16 partials of n elements and adds the result to
// the residual x in place: x = bf16(x + bf16(sum_r partial_r)), the order of
// the single-GPU residual epilogue (rounded projection, then the add).
//
// CTA c owns the fixed element range [c kArChunk, (c+1) kArChunk) -- the same
// range whatever n is, so the epoch and parity of a range never mix calls of
// different sizes -- and runs its own protocol, so no grid-wide
// synchronisation is needed:
//   1. e = epochs[c] + 1, parity e & 1;
//   2. store the local chunk into mailbox[parity][rank] of every peer (NVLink
//      stores), fence at system scope, then release-store e into each peer's
//      flags[rank][c];
//   3. wait (bounded) until flags[p][c] >= e here for every peer p, with
//      acquire loads;
//   4. sum the local partial and the peers' chunks from the local mailbox,
//      add the residual, store x; epochs[c] = e.
// The area also holds the region of the GEMV-epilogue all-reduce
// (allreduce.cuh, ar_fuse_*), which follows the same protocol per row block.
// Two parities suffice: a rank writes parity (e+1) & 1 only after finishing
// call e, and cannot start call e+2 before every peer has written call e+1,
// i.e. finished reading parity e & 1.
#include "../amcu_internal.h"
#include "allreduce.cuh"
#include "common.cuh"

namespace amcu {

constexpr int32_t kErrArWait = 0x401;
constexpr int kArThreads = 256;
constexpr uint64_t kArDefaultWaitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__host__ __device__ inline size_t ar_mailbox_offset(int parity, int src, int64_t i) {
    return (((size_t)parity * kArMaxRanks + src) * kArMaxElems + (size_t)i) * 2;
}
__host__ __device__ constexpr size_t ar_flags_offset() { return (size_t)2 * kArMaxRanks * kArMaxElems * 2; }
__host__ __device__ constexpr size_t ar_epochs_offset() { return ar_flags_offset() + (size_t)kArMaxRanks * kArMaxCtas * 4; }
size_t ar_area_bytes() { return ar_fuse_epochs_offset() + (size_t)kFuseMaxRb * 4; }

__global__ void __launch_bounds__(kArThreads) ar_oneshot_add_kernel(ArParams p) {
    const int c = blockIdx.x, tid = threadIdx.x;
    const int64_t lo = (int64_t)c * kArChunk;
    const int64_t hi = lo + kArChunk < p.n ? lo + kArChunk : p.n;
    uint8_t* own = p.area[p.rank];
    uint32_t* epochs = reinterpret_cast<uint32_t*>(own + ar_epochs_offset());
    pdl_wait();
    const uint32_t e = epochs[c] + 1;
    const int par = (int)(e & 1);
    // 2. push the local chunk to every peer
    for (int64_t v = lo / 8 + tid; v < hi / 8; v += kArThreads) {
        const uint4 d = reinterpret_cast<const uint4*>(p.part)[v];
        for (int q = 0; q < p.world; ++q)
            if (q != p.rank) *reinterpret_cast<uint4*>(p.area[q] + ar_mailbox_offset(par, p.rank, v * 8)) = d;
    }
    __threadfence_system();
    __syncthreads();
    if (tid < p.world && tid != p.rank)
        st_release_sys(reinterpret_cast<uint32_t*>(p.area[tid] + ar_flags_offset()) + p.rank * kArMaxCtas + c, e);
    // 3. wait for the peers' chunks
    if (tid < p.world && tid != p.rank) {
        const uint32_t* f = reinterpret_cast<const uint32_t*>(own + ar_flags_offset()) + tid * kArMaxCtas + c;
        const uint64_t t0 = globaltimer_ns();
        const uint64_t lim = p.wait_ns ? p.wait_ns : kArDefaultWaitNs;
        while ((int32_t)(ld_acquire_sys(f) - e) < 0) {
            if (globaltimer_ns() - t0 > lim) {
                record_device_error(p.err, kErrArWait);
                break;
            }
        }
    }
    __syncthreads();
    // 4. sum + residual
    for (int64_t v = lo / 8 + tid; v < hi / 8; v += kArThreads) {
        const uint4 d = reinterpret_cast<const uint4*>(p.part)[v];
        float s[8];
        const uint32_t dw[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            s[2 * j] = __uint_as_float(dw[j] << 16);
            s[2 * j + 1] = __uint_as_float(dw[j] & 0xffff0000u);
        }
        for (int q = 0; q < p.world; ++q) {
            if (q == p.rank) continue;
            const uint4 o = *reinterpret_cast<const uint4*>(own + ar_mailbox_offset(par, q, v * 8));
            const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                s[2 * j] += __uint_as_float(ow[j] << 16);
                s[2 * j + 1] += __uint_as_float(ow[j] & 0xffff0000u);
            }
        }
        const uint4 xr = reinterpret_cast<const uint4*>(p.x)[v];
        const uint32_t xw[4] = {xr.x, xr.y, xr.z, xr.w};
        uint32_t out[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float a = __bfloat162float(__float2bfloat16_rn(s[2 * j])) + __uint_as_float(xw[j] << 16);
            const float b = __bfloat162float(__float2bfloat16_rn(s[2 * j + 1])) + __uint_as_float(xw[j] & 0xffff0000u);
            __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
            out[j] = *reinterpret_cast<uint32_t*>(&h);
        }
        reinterpret_cast<uint4*>(p.x)[v] = make_uint4(out[0], out[1], out[2], out[3]);
    }
    __syncthreads();
    if (tid == 0) epochs[c] = e;
    pdl_trigger();
}

bool ar_oneshot_supported(int64_t n, int world) {
    return world >= 2 && world <= kArMaxRanks && n > 0 && n <= kArMaxElems && n % 8 == 0;
}

void launch_ar_oneshot_add(const ArParams& p, cudaStream_t s) {
    const int64_t g = (p.n + kArChunk - 1) / kArChunk;  // <= kArMaxCtas (n <= kArMaxElems)
    launch_pdl(ar_oneshot_add_kernel, dim3((unsigned)g), dim3(kArThreads), 0, s, p);
}

}  // namespace amcu

using namespace amcu;

extern "C" size_t amcu_allreduce_area_bytes(void) { return ar_area_bytes(); }

extern "C" am_status_code amcu_allreduce_oneshot_add(const AmcuAllReduceArgs* a, void* stream) {
    AMCU_REQUIRE(a != nullptr, "amcu_allreduce_oneshot_add: null args");
    AMCU_REQUIRE(a->world >= 2 && a->world <= kArMaxRanks, "amcu_allreduce_oneshot_add: world must be in [2, %d]",
                 kArMaxRanks);
    AMCU_REQUIRE(a->rank >= 0 && a->rank < a->world, "amcu_allreduce_oneshot_add: rank out of range");
    AMCU_REQUIRE(ar_oneshot_supported(a->n, a->world),
                 "amcu_allreduce_oneshot_add: n must be a positive multiple of 8 up to %lld",
                 (long long)kArMaxElems);
    AMCU_REQUIRE(a->part && a->x && aligned(a->part, 16) && aligned(a->x, 16),
                 "amcu_allreduce_oneshot_add: part and x must be 16-byte aligned device pointers");
    ArParams p{};
    p.part = a->part;
    p.x = a->x;
    p.n = a->n;
    p.rank = a->rank;
    p.world = a->world;
    for (int r = 0; r < a->world; ++r) {
        AMCU_REQUIRE(a->areas[r] && aligned(a->areas[r], 16), "amcu_allreduce_oneshot_add: area %d missing", r);
        p.area[r] = static_cast<uint8_t*>(a->areas[r]);
    }
    p.err = device_error_word();
    p.wait_ns = a->wait_limit_us * 1000ull;
    launch_ar_oneshot_add(p, as_stream(stream));
    return check_launch("amcu_allreduce_oneshot_add");
}
