// Error objects, per-thread last-error message and device queries of the C ABI.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <tuple>

#include <dlfcn.h>
#include <execinfo.h>
#include <signal.h>
#include <unistd.h>
#include <string>

#include "amcu_internal.h"

namespace amcu {

namespace {
thread_local std::string g_last_error;
}

am_status_code set_error(am_status_code code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

void clear_error() { g_last_error.clear(); }

int num_sms() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    return n;
}

bool pdl_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("AMCU_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

void set_func_attr_once(const void* func, cudaFuncAttribute attr, int value) {
    static std::mutex mu;
    static std::set<std::tuple<int, const void*, int>> done;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return;
    std::lock_guard<std::mutex> lk(mu);
    if (done.insert({dev, func, (int)attr}).second) cudaFuncSetAttribute(func, attr, value);
}

int smem_per_sm() {
    static int per_dev[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 228 * 1024;
    if (per_dev[dev] == 0) {  // benign race: every writer stores the same value
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
        per_dev[dev] = v > 0 ? v : 228 * 1024;
    }
    return per_dev[dev];
}

int32_t* device_error_word() {
    static int32_t* words[64] = {};
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!words[dev]) {
        void* p = nullptr;
        if (cudaMalloc(&p, 256) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        cudaMemset(p, 0, 256);
        cudaDeviceSynchronize();
        words[dev] = static_cast<int32_t*>(p);
    }
    return words[dev];
}

}  // namespace amcu

namespace {
// Error object of the reference C ABI (src/c_api_error.cpp:14-41): a status
// code plus an owned message.
struct ErrorObject {
    am_status_code code;
    std::string message;
};
}  // namespace

extern "C" {

const char* amcu_last_error(void) { return amcu::g_last_error.c_str(); }

am_status_code amcu_device_error(int32_t* code, int32_t clear) {
    int32_t* w = amcu::device_error_word();
    if (!w) return amcu::set_error(AM_STATUS_INTERNAL, "device error word unavailable");
    int32_t v = 0;
    if (cudaMemcpy(&v, w, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return amcu::set_error(AM_STATUS_INTERNAL, "reading the device error word failed");
    if (clear && v != 0) {
        cudaMemset(w, 0, 4);
        cudaDeviceSynchronize();
    }
    if (code) *code = v;
    return AM_STATUS_OK;
}

const char* amcu_version(void) { return "aethermind_b200 0.1 (sm_100a)"; }

am_error_handle am_error_create(am_status_code code, const char* message) {
    return new ErrorObject{code, message ? message : ""};
}

void am_error_destroy(am_error_handle e) { delete static_cast<ErrorObject*>(e); }

am_status_code am_error_code(am_error_handle e) {
    return e ? static_cast<ErrorObject*>(e)->code : AM_STATUS_OK;
}

const char* am_error_message(am_error_handle e) {
    return e ? static_cast<ErrorObject*>(e)->message.c_str() : "";
}

}  // extern "C"

// Diagnostics: with AM_SEGV_TRACE=1 in the environment, a crash of the host
// process prints the faulting call stack (module and offset of every frame)
// to stderr before the default action runs.
namespace {
void segv_trace(int sig) {
    void* frames[64];
    const int n = backtrace(frames, 64);
    char line[512];
    for (int i = 0; i < n; ++i) {
        Dl_info info{};
        if (dladdr(frames[i], &info) && info.dli_fname) {
            const int len = snprintf(line, sizeof line, "am-segv #%d %s+0x%lx %s\n", i, info.dli_fname,
                                     (unsigned long)((char*)frames[i] - (char*)info.dli_fbase),
                                     info.dli_sname ? info.dli_sname : "");
            if (len > 0) (void)!write(2, line, (size_t)len < sizeof line ? (size_t)len : sizeof line - 1);
        }
    }
    signal(sig, SIG_DFL);
    raise(sig);
}
struct SegvTraceInstaller {
    SegvTraceInstaller() {
        const char* v = std::getenv("AM_SEGV_TRACE");
        if (v && v[0] == '1') signal(SIGSEGV, segv_trace);
    }
} g_segv_trace_installer;
}  // namespace

