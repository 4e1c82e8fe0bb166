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
// Per-device int32 error word that kernels with bounded waits write on timeout
// (allocated on first use on the current device; nullptr if that fails).
int32_t* device_error_word();

}  // namespace amcu

#define AMCU_REQUIRE(cond, ...)                                        \
    do {                                                               \
        if (!(cond)) return ::amcu::set_error(AM_STATUS_INVALID_ARGUMENT, __VA_ARGS__); \
    } while (0)
