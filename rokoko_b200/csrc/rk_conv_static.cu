// rk_conv_static.cu -- rk_conv1d_fprop_static: the conv seam for callers that
// must not allocate device memory, and rk_conv1d_static_check, which reads its
// device error word.
//
// Some callers cannot call cudaMalloc at the point where they need a
// convolution:
//   * hosts whose device memory is handed out by their own pool or caching
//     allocator, which a library must not bypass or fragment;
//   * streaming / real-time threads that cannot block on the allocator
//     (cudaMalloc and cudaFree may synchronise the device);
//   * plugin hosts that grant a fixed device-memory budget when the plugin
//     is loaded.
// For them this entry point runs the same tcgen05 convolution as
// rk_conv1d_fprop, with its scratch (operand planes, packed weights and the
// device error word) in one file-scope device array of RK_CONV_STATIC_SCRATCH_BYTES.
// The array exists on every GPU that loads this library, for the lifetime of
// the process.
//
// Set-up: the first call on a device (and the first after that device's
// context was destroyed and re-created) resolves the array's device address
// with cudaGetSymbolAddress (host code cannot use the array's name as a device
// address) while that device is current, caches it with the context it belongs
// to, and sets the conv kernels' attributes on that device; make that first
// call before any stream capture.  No call allocates or frees device memory.
// Every call reuses the same array and leaves its contents behind; the error
// word is cleared by each call and every other scratch byte a call reads is
// written by that call first.  Calls that can overlap on the GPU (different
// streams, or different host threads, on one device) race on the array and
// must be serialised by the caller.
#include <cuda.h>

#include <mutex>

#include "../../include/rk_b200.h"
#include "status.h"

namespace {

static __device__ __align__(256) unsigned char g_conv_scratch[RK_CONV_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
struct Cached {
    void* ptr = nullptr;
    CUcontext ctx = nullptr;  // the context the address belongs to
};
Cached g_cache[kMaxDevices];

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

CUcontext current_context() {
    static CtxGetCurrentFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<CtxGetCurrentFn>(p);
    }();
    CUcontext c = nullptr;
    if (fn) fn(&c);
    return c;
}

// Device address of g_conv_scratch on the current device (resolved once per
// device and context; resolving also sets the conv kernels' attributes there).
rk_status scratch_address(void** out, const char* who) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return rk::fail_cuda_err(RK_ERR_CUDA, who, e);
    if (dev < 0 || dev >= kMaxDevices) return rk::fail(RK_ERR_CANNOT_IMPLEMENT, "device index above 63");
    const CUcontext ctx = current_context();
    std::lock_guard<std::mutex> g(g_mu);
    Cached& c = g_cache[dev];
    if (!c.ptr || c.ctx != ctx) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_conv_scratch);
        if (e != cudaSuccess || !p) return rk::fail_cuda_err(RK_ERR_INIT, "cudaGetSymbolAddress", e);
        const rk_status s = rk::conv_seam_init_device();
        if (s != RK_OK) return s;
        c.ptr = p;
        c.ctx = current_context();  // the symbol lookup made the device's context current
    }
    *out = c.ptr;
    return RK_OK;
}

}  // namespace

extern "C" rk_status rk_conv1d_fprop_static(const float* x, const float* w, const float* bias, float* y,
                                            const float* residual, int C_in, int C_out, int T_in, int K, int stride,
                                            int padding, int dilation, int precision, void* stream) {
    const size_t need = rk_conv1d_workspace_size(C_in, C_out, T_in, K, stride, padding, dilation, precision);
    if (need == 0) return rk::fail(RK_ERR_CANNOT_IMPLEMENT, "rk_conv1d_fprop_static: unsupported arguments");
    if (need > (size_t)RK_CONV_STATIC_SCRATCH_BYTES)
        return rk::fail(RK_ERR_WORKSPACE,
                        "rk_conv1d_fprop_static: this convolution needs more scratch than the fixed "
                        "RK_CONV_STATIC_SCRATCH_BYTES (32 MiB) array; use rk_conv1d_fprop with a caller workspace");
    void* ws = nullptr;
    const rk_status s = scratch_address(&ws, "rk_conv1d_fprop_static");
    if (s != RK_OK) return s;
    return rk_conv1d_fprop(x, w, bias, y, residual, ws, RK_CONV_STATIC_SCRATCH_BYTES, C_in, C_out, T_in, K, stride,
                           padding, dilation, precision, stream);
}

extern "C" rk_status rk_conv1d_static_check(void* stream) {
    void* ws = nullptr;
    const rk_status s = scratch_address(&ws, "rk_conv1d_static_check");
    if (s != RK_OK) return s;
    return rk_conv1d_check(ws, stream);
}
