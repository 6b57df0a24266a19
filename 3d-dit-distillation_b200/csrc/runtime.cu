// Library-wide runtime pieces of the C ABI: version, error strings, launch
// accounting.  The device error word lives with the kernels that set it
// (attention.cu).
#include <atomic>
#include <cstdio>

#include "common.cuh"

namespace vdit {

static std::atomic<long long> g_launches{0};

void count_launches(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

static thread_local char g_last_error[256] = "";

void record_cuda_error(cudaError_t e) {
    snprintf(g_last_error, sizeof(g_last_error), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
}

}  // namespace vdit

extern "C" const char* vdit_last_cuda_error(void) { return vdit::g_last_error; }

extern "C" const char* vdit_version(void) { return "vdit 0.1 (sm_100a)"; }

extern "C" const char* vdit_error_string(int code) {
    switch (code) {
        case VDIT_OK: return "ok";
        case VDIT_ERR_ARG: return "invalid argument (shape, size or null pointer)";
        case VDIT_ERR_ALIGN: return "pointer or stride not 16-byte aligned";
        case VDIT_ERR_LAUNCH: return "CUDA launch failed";
        case VDIT_ERR_UNSUPPORTED: return "unsupported head_dim or width";
        case VDIT_ERR_WORKSPACE: return "workspace missing or too small";
        case VDIT_ERR_DRIVER: return "CUDA driver entry point failed";
        case VDIT_ERR_TOO_LARGE: return "size exceeds the fixed scratch of the no-alloc entry point";
        default: return "unknown error";
    }
}

extern "C" long long vdit_launch_count(void) { return vdit::g_launches.load(std::memory_order_relaxed); }

