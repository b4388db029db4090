// status.cu -- rk_status strings and the per-thread last-error text.
#include <cstdio>
#include <string>

#include "status.h"

namespace rk {
namespace {
thread_local std::string g_last;
}
rk_status fail(rk_status s, const char* what) {
    g_last = what ? what : "";
    return s;
}
rk_status fail_cuda_err(rk_status s, const char* what, cudaError_t e) {
    g_last = std::string(what ? what : "") + ": " + cudaGetErrorString(e);
    return s;
}
rk_status fail_cuda(rk_status s, const char* what) { return fail_cuda_err(s, what, cudaGetLastError()); }
}  // namespace rk

extern "C" const char* rk_last_error(void) { return rk::g_last.c_str(); }

extern "C" const char* rk_status_string(rk_status s) {
    switch (s) {
        case RK_OK: return "ok";
        case RK_ERR_CANNOT_IMPLEMENT: return "cannot implement";
        case RK_ERR_WORKSPACE: return "workspace too small";
        case RK_ERR_INIT: return "initialisation failed";
        case RK_ERR_LAUNCH: return "kernel launch failed";
        case RK_ERR_CUDA: return "CUDA error";
        case RK_ERR_WEIGHTS: return "bad weight file";
        case RK_ERR_DEVICE_TIMEOUT: return "device wait timed out";
        case RK_ERR_OOM: return "out of device memory";
        case RK_ERR_STATE: return "invalid call order";
        default: return "unknown status";
    }
}
