// rk_conv_api.cu -- the stateless C-ABI conv seam (rk_conv1d_fprop), the
// drop-in for the reference's cutlass_conv1d_fprop[_f16]
// (src/cutlass_conv.cu:239-313, src/cutlass_conv_f16.cu:216-273).
//
// Workspace layout (256-byte aligned slabs):
//   [0, 256)          device error word (uint32) + padding
//   activation planes  rows x Cp 16-bit, hi then lo (split)
//   weight planes      C_out (padded to a multiple of 128) x taps x Cp 16-bit, hi then lo (split)
//   split-K scratch    FP32 partial accumulators, only for launches with few output tiles
#include <cstdio>
#include <cstring>
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

}  // namespace

extern "C" size_t rk_conv1d_workspace_size(int C_in, int C_out, int T_in, int K, int stride, int padding,
                                           int dilation, int precision) {
    ConvPlan p;
    if (!plan_conv(C_in, C_out, T_in, K, stride, padding, dilation, precision, p)) return 0;
    return p.total;
}

extern "C" rk_status rk_conv1d_fprop(const float* x, const float* w, const float* bias, float* y,
                                     const float* residual, void* workspace, size_t workspace_bytes, int C_in,
                                     int C_out, int T_in, int K, int stride, int padding, int dilation,
                                     int precision, void* stream_) {
    cudaStream_t st = (cudaStream_t)stream_;
    ConvPlan p;
    if (!x || !w || !y || (precision != RK_PRECISION_FP32 && precision != RK_PRECISION_FP16) ||
        !plan_conv(C_in, C_out, T_in, K, stride, padding, dilation, precision, p))
        return rk::fail(RK_ERR_CANNOT_IMPLEMENT, "rk_conv1d_fprop: unsupported arguments");
    if (!workspace || workspace_bytes < p.total || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return rk::fail(RK_ERR_WORKSPACE, "rk_conv1d_fprop: workspace too small or not 256-byte aligned");
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

    rk::PackArgs pa{};
    pa.x = x; pa.ldx = C_in; pa.rows_src = T_in; pa.C = C_in; pa.rows_dst = p.rows; pa.Cp = p.Cp;
    pa.hi = a_hi; pa.lo = a_lo; pa.sr_stride = stride; pa.sr_pad = stride > 1 ? padding : 0;
    if (rk::pack_act(pa, split, st) != cudaSuccess) return rk::fail_cuda(RK_ERR_LAUNCH, "pack_act");
    if (rk::pack_weights_nhwc(w, C_out, K, C_in, stride, w_hi, w_lo, split, st) != cudaSuccess)
        return rk::fail_cuda(RK_ERR_LAUNCH, "pack_weights");

    static thread_local int init_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (init_dev != dev) {
        if (rk::conv_tc_init() != cudaSuccess) return rk::fail_cuda(RK_ERR_INIT, "conv_tc_init");
        init_dev = dev;
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
        return rk::fail(RK_ERR_INIT, "rk_conv1d_fprop: tensor map encoding failed");
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
    if (rk::conv_tc_launch(ops, a, split, 1, st) != cudaSuccess) return rk::fail_cuda(RK_ERR_LAUNCH, "conv_tc");
    return RK_OK;
}

extern "C" rk_status rk_conv1d_check(void* workspace, void* stream_) {
    uint32_t e = 0;
    cudaStream_t st = (cudaStream_t)stream_;
    if (cudaMemcpyAsync(&e, workspace, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return rk::fail_cuda(RK_ERR_CUDA, "rk_conv1d_check");
    if (e) {
        cudaMemsetAsync(workspace, 0, 4, st);
        char buf[96];
        snprintf(buf, sizeof buf, "device wait timed out (code %u)", e);
        return rk::fail(RK_ERR_DEVICE_TIMEOUT, buf);
    }
    return RK_OK;
}
