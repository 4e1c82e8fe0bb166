// Internal host-side helpers shared by the C-ABI translation units.
#pragma once
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "aethermind_b200.h"

namespace amcu {

// Records a printf-style message for amcu_last_error() and returns `code`.
am_status_code set_error(am_status_code code, const char* fmt, ...);
void clear_error();

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// Maps a CUDA error from a launch to a Status (launch-time errors only;
// asynchronous faults surface at the caller's next synchronisation).
inline am_status_code check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(AM_STATUS_INTERNAL, "%s: %s", what, cudaGetErrorString(e));
    return AM_STATUS_OK;
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

int num_sms();

// Whether kernels of the hot path are launched with programmatic stream
// serialization (on unless the environment sets AMCU_PDL=0; read once).
bool pdl_enabled();

// Launches `kernel` on `s` with the programmatic-stream-serialization
// attribute when pdl_enabled(). The kernel must call pdl_wait() before it
// touches memory that earlier kernels on the stream write or read. Launch
// errors are left for check_launch() (cudaGetLastError).
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
// cudaFuncSetAttribute(func, attr, value) once per (device, function,
// attribute) on the current device: function attributes are per device, so a
// process that runs on several devices sets them on each (thread-safe).
void set_func_attr_once(const void* func, cudaFuncAttribute attr, int value);
// Shared memory per SM of the current device (cached per device).
int smem_per_sm();

// Per-device int32 error word that kernels with bounded waits write on timeout
// (allocated on first use on the current device; nullptr if that fails).
int32_t* device_error_word();

}  // namespace amcu

#define AMCU_REQUIRE(cond, ...)                                        \
    do {                                                               \
        if (!(cond)) return ::amcu::set_error(AM_STATUS_INVALID_ARGUMENT, __VA_ARGS__); \
    } while (0)
