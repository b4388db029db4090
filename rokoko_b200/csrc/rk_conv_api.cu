// rk_conv_api.cu -- the stateless C-ABI conv seam, the drop-in for the
// reference's cutlass_conv1d_fprop[_f16] (src/cutlass_conv.cu:239-313,
// src/cutlass_conv_f16.cu:216-273) and cutlass_conv1d_workspace_bytes
// (src/cutlass_conv.cu:319-330).
//
// Entry points:
//   rk_conv1d_fprop      FP32 operands, precision chosen by argument
//   rk_conv1d_fprop_f32  cutlass_conv1d_fprop's exact argument list (FP32
//                        operands, FP32 semantics: split-bf16 products)
//   rk_conv1d_fprop_f16  cutlass_conv1d_fprop_f16's exact argument list (half
//                        x and w, FP32 bias / residual / y, fp16 products with
//                        FP32 accumulation)
//
// Workspace layout (256-byte aligned slabs):
//   [0, 256)          device error word (uint32) + padding
//   activation planes  rows x Cp 16-bit, hi then lo (split)
//   weight planes      C_out (padded to a multiple of 128) x taps x Cp 16-bit, hi then lo (split)
//   split-K scratch    FP32 partial accumulators, only for launches with few output tiles
#include <cuda_fp16.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/rk_b200.h"
#include "conv_tc.cuh"
#include "pack.cuh"
#include "status.h"

namespace {

struct ConvPlan {
    int T_out, taps, Cp, rows, tap_off[rk::CONV_MAX_TAPS];
    size_t act_plane, w_plane, scratch, total;
};

size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

bool plan_conv(int C_in, int C_out, int T_in, int K, int stride, int pad, int dil, int precision, ConvPlan& p) {
    if (C_in < 1 || C_out < 1 || T_in < 1 || K < 1 || stride < 1 || dil < 1 || pad < 0) return false;
    if (stride > 1 && dil != 1) return false;
    p.T_out = (T_in + 2 * pad - dil * (K - 1) - 1) / stride + 1;
    if (p.T_out < 1) return false;
    if (stride == 1) {
        p.taps = K;
        p.Cp = (C_in + 63) / 64 * 64;
        p.rows = T_in;
        for (int k = 0; k < K && k < rk::CONV_MAX_TAPS; k++) p.tap_off[k] = k * dil - pad;
    } else {
        p.taps = (K + stride - 1) / stride;
        p.Cp = (stride * C_in + 63) / 64 * 64;
        p.rows = p.T_out + p.taps - 1;
        for (int j = 0; j < p.taps && j < rk::CONV_MAX_TAPS; j++) p.tap_off[j] = j;
    }
    if (p.taps > rk::CONV_MAX_TAPS) return false;
    const int planes = precision == RK_PRECISION_FP32 ? 2 : 1;
    p.act_plane = al256((size_t)p.rows * p.Cp * 2);
    p.w_plane = al256((size_t)rk::conv_tc_weight_rows(C_out) * p.taps * p.Cp * 2);
    // launches with fewer 64-row x 128-channel tiles than a B200 has SMs may split their
    // reduction over up to 8 CTAs (the kernel's limit)
    const long tiles = (long)((p.T_out + 63) / 64) * ((C_out + 127) / 128);
    p.scratch = tiles < 148 ? al256((size_t)8 * p.T_out * C_out * 4) : 0;
    p.total = 256 + planes * (p.act_plane + p.w_plane) + p.scratch;
    return true;
}

int grid_for(long n) {
    const long b = (n + 255) / 256;
    return (int)(b < 148 * 16 ? (b > 0 ? b : 1) : 148 * 16);
}

// half activations [T_in][C_in] -> fp16 plane [rows][Cp], same super-row
// gather as pack_act (dst[q][r*C_in + c] = x[q*stride - pad + r][c], r < stride)
__global__ void pack_half_act_kernel(const __half* __restrict__ x, int T_in, int C_in, int rows, int Cp, int stride,
                                     int pad, __half* __restrict__ out) {
    const long total = (long)rows * Cp;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int q = (int)(i / Cp), cd = (int)(i - (long)q * Cp);
        const int r = cd / C_in, c = cd - r * C_in;
        __half v = __float2half_rn(0.0f);
        if (r < stride) {
            const int row = q * stride - pad + r;
            if (row >= 0 && row < T_in) v = x[(long)row * C_in + c];
        }
        out[i] = v;
    }
}

// half weights [C_out][K][C_in] (NHWC) -> fp16 plane [C_out][taps][Cp] (the layout of pack_weights_nhwc)
__global__ void pack_half_w_kernel(const __half* __restrict__ w, int C_out, int K, int C_in, int stride, int taps,
                                   int Cp, __half* __restrict__ out) {
    const long total = (long)C_out * taps * Cp;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int cd = (int)(i % Cp);
        const long t2 = i / Cp;
        const int j = (int)(t2 % taps), co = (int)(t2 / taps);
        const int r = cd / C_in, ci = cd - r * C_in;
        const int k = j * stride + r;
        out[i] = (r < stride && k < K) ? w[((long)co * K + k) * C_in + ci] : __float2half_rn(0.0f);
    }
}

// The kernels' shared-memory attributes are per device (they hold for every
// host thread), so they are set once per device for the whole process.
std::mutex g_init_mu;
bool g_init_done[64] = {};

// Operands: FP32 (x_half == false) or half (x_half == true; FP16 semantics only).
rk_status conv_fprop(const void* x, const void* w, bool half_in, const float* bias, float* y, const float* residual,
                     void* workspace, size_t workspace_bytes, int C_in, int C_out, int T_in, int K, int stride,
                     int padding, int dilation, int precision, void* stream_, const char* who) {
    cudaStream_t st = (cudaStream_t)stream_;
    ConvPlan p;
    const std::string nm(who);
    if (!x || !w || !y || (precision != RK_PRECISION_FP32 && precision != RK_PRECISION_FP16) ||
        (half_in && precision != RK_PRECISION_FP16) ||
        !plan_conv(C_in, C_out, T_in, K, stride, padding, dilation, precision, p))
        return rk::fail(RK_ERR_CANNOT_IMPLEMENT, (nm + ": unsupported arguments").c_str());
    if (!workspace || workspace_bytes < p.total || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return rk::fail(RK_ERR_WORKSPACE, (nm + ": workspace too small or not 256-byte aligned").c_str());
    rk_status s = rk::conv_seam_init_device();
    if (s != RK_OK) return s;
    const bool split = precision == RK_PRECISION_FP32;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    uint32_t* err = reinterpret_cast<uint32_t*>(ws);
    uint8_t* a_hi = ws + 256;
    uint8_t* a_lo = a_hi + p.act_plane;
    uint8_t* w_hi = a_hi + (split ? 2 : 1) * p.act_plane;
    uint8_t* w_lo = w_hi + p.w_plane;
    uint8_t* scratch = w_hi + (split ? 2 : 1) * p.w_plane;
    // the error word reports on this call only
    if (cudaMemsetAsync(err, 0, 4, st) != cudaSuccess) return rk::fail_cuda(RK_ERR_CUDA, "memset");

    if (half_in) {
        pack_half_act_kernel<<<grid_for((long)p.rows * p.Cp), 256, 0, st>>>(
            static_cast<const __half*>(x), T_in, C_in, p.rows, p.Cp, stride, stride > 1 ? padding : 0,
            reinterpret_cast<__half*>(a_hi));
        if (cudaGetLastError() != cudaSuccess) return rk::fail_cuda(RK_ERR_LAUNCH, "pack_half_act");
        pack_half_w_kernel<<<grid_for((long)C_out * p.taps * p.Cp), 256, 0, st>>>(
            static_cast<const __half*>(w), C_out, K, C_in, stride, p.taps, p.Cp, reinterpret_cast<__half*>(w_hi));
        if (cudaGetLastError() != cudaSuccess) return rk::fail_cuda(RK_ERR_LAUNCH, "pack_half_w");
    } else {
        rk::PackArgs pa{};
        pa.x = static_cast<const float*>(x); pa.ldx = C_in; pa.rows_src = T_in; pa.C = C_in; pa.rows_dst = p.rows;
        pa.Cp = p.Cp; pa.hi = a_hi; pa.lo = a_lo; pa.sr_stride = stride; pa.sr_pad = stride > 1 ? padding : 0;
        if (rk::pack_act(pa, split, st) != cudaSuccess) return rk::fail_cuda(RK_ERR_LAUNCH, "pack_act");
        if (rk::pack_weights_nhwc(static_cast<const float*>(w), C_out, K, C_in, stride, w_hi, w_lo, split, st) !=
            cudaSuccess)
            return rk::fail_cuda(RK_ERR_LAUNCH, "pack_weights");
    }
    // weight rows beyond C_out (padding up to the 128-row tile) only feed
    // accumulator rows the epilogue never stores
    rk::ConvOperands ops;
    ops.act_hi = a_hi;
    ops.act_lo = split ? a_lo : nullptr;
    ops.act_rows = (uint64_t)p.rows;
    ops.act_cp = (uint64_t)p.Cp;
    const uint64_t wcols = (uint64_t)p.taps * p.Cp, wrows = (uint64_t)rk::conv_tc_weight_rows(C_out);
    if (!rk::make_tmap_k64(&ops.w_hi, w_hi, split, wcols, wrows, wcols, rk::CONV_W_ROWS) ||
        (split && !rk::make_tmap_k64(&ops.w_lo, w_lo, true, wcols, wrows, wcols, rk::CONV_W_ROWS)))
        return rk::fail(RK_ERR_INIT, (nm + ": tensor map encoding failed").c_str());
    if (!split) ops.w_lo = ops.w_hi;
    ops.scratch = p.scratch ? reinterpret_cast<float*>(scratch) : nullptr;
    ops.scratch_bytes = p.scratch;

    rk::ConvArgs a{};
    a.M = p.T_out; a.C_out = C_out; a.kblocks = p.Cp / 64; a.taps = p.taps;
    for (int k = 0; k < p.taps; k++) a.tap_off[k] = p.tap_off[k];
    a.a_off = 0; a.b_phase_rows = 0; a.T_out = p.T_out; a.o_min = 0; a.o_stride = 1; a.o_off = 0; a.o_phase_step = 0;
    a.y = y; a.ldy = C_out;
    a.bias = residual ? nullptr : bias;
    a.res = residual; a.ldres = C_out; a.res_shift = 0;
    a.acc_in = nullptr; a.ldacc = 0; a.alpha = 1.0f;
    a.stats = nullptr; a.stats_ld = 0; a.stats_parts = 0; a.dup_src_row = -1;
    a.err = err;
    if (rk::conv_tc_launch(ops, a, split, 1, st) != cudaSuccess)
        return rk::fail_cuda(RK_ERR_LAUNCH, (nm + ": conv_tc").c_str());
    return RK_OK;
}

}  // namespace

namespace rk {
rk_status conv_seam_init_device() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail_cuda_err(RK_ERR_CUDA, "cudaGetDevice", e);
    if (dev < 0 || dev >= 64) return fail(RK_ERR_CANNOT_IMPLEMENT, "device index above 63");
    std::lock_guard<std::mutex> g(g_init_mu);
    if (!g_init_done[dev]) {
        if ((e = conv_tc_init()) != cudaSuccess) return fail_cuda_err(RK_ERR_INIT, "conv_tc_init", e);
        g_init_done[dev] = true;
    }
    return RK_OK;
}
}  // namespace rk

extern "C" size_t rk_conv1d_workspace_size(int C_in, int C_out, int T_in, int K, int stride, int padding,
                                           int dilation, int precision) {
    ConvPlan p;
    if (precision != RK_PRECISION_FP32 && precision != RK_PRECISION_FP16) return 0;
    if (!plan_conv(C_in, C_out, T_in, K, stride, padding, dilation, precision, p)) return 0;
    return p.total;
}

extern "C" size_t rk_conv1d_workspace_bytes(int C_in, int C_out, int T_in, int K, int stride, int padding,
                                            int dilation) {
    // the FP32 path needs the larger workspace (two operand planes), so this size serves both seams
    return rk_conv1d_workspace_size(C_in, C_out, T_in, K, stride, padding, dilation, RK_PRECISION_FP32);
}

extern "C" rk_status rk_conv1d_fprop(const float* x, const float* w, const float* bias, float* y,
                                     const float* residual, void* workspace, size_t workspace_bytes, int C_in,
                                     int C_out, int T_in, int K, int stride, int padding, int dilation,
                                     int precision, void* stream) {
    return conv_fprop(x, w, false, bias, y, residual, workspace, workspace_bytes, C_in, C_out, T_in, K, stride,
                      padding, dilation, precision, stream, "rk_conv1d_fprop");
}

extern "C" rk_status rk_conv1d_fprop_f32(const float* x, const float* w, const float* bias, float* y,
                                         const float* residual, float* workspace, size_t workspace_bytes, int C_in,
                                         int C_out, int T_in, int K, int stride, int padding, int dilation,
                                         void* stream) {
    return conv_fprop(x, w, false, bias, y, residual, workspace, workspace_bytes, C_in, C_out, T_in, K, stride,
                      padding, dilation, RK_PRECISION_FP32, stream, "rk_conv1d_fprop_f32");
}

extern "C" rk_status rk_conv1d_fprop_f16(const void* x, const void* w, const float* bias, float* y,
                                         const float* residual, float* workspace, size_t workspace_bytes, int C_in,
                                         int C_out, int T_in, int K, int stride, int padding, int dilation,
                                         void* stream) {
    return conv_fprop(x, w, true, bias, y, residual, workspace, workspace_bytes, C_in, C_out, T_in, K, stride,
                      padding, dilation, RK_PRECISION_FP16, stream, "rk_conv1d_fprop_f16");
}

extern "C" rk_status rk_conv1d_check(void* workspace, void* stream_) {
    uint32_t e = 0;
    cudaStream_t st = (cudaStream_t)stream_;
    if (!workspace) return rk::fail(RK_ERR_CANNOT_IMPLEMENT, "rk_conv1d_check: null workspace");
    if (cudaMemcpyAsync(&e, workspace, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return rk::fail_cuda(RK_ERR_CUDA, "rk_conv1d_check");
    if (e) {
        if (cudaMemsetAsync(workspace, 0, 4, st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess)
            return rk::fail_cuda(RK_ERR_CUDA, "rk_conv1d_check: clearing the error word");
        char buf[96];
        snprintf(buf, sizeof buf, "device wait timed out (code %u)", e);
        return rk::fail(RK_ERR_DEVICE_TIMEOUT, buf);
    }
    return RK_OK;
}
