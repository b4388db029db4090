// exec.h -- launch helpers shared by the forward passes (decode.cu, infer.cu):
// conv / operand-pack / AdaIN-coefficient launches with status tracking, the
// AdainResBlk1d block, and stage capture for rk_record_stages.
#pragma once
#include <cuda_runtime.h>

#include "../../include/rk_b200.h"
#include "model.h"
#include "ops.cuh"
#include "status.h"

namespace rk {

// Timeline mark (rk_profile with RK_PROFILE_TIMELINE): records an event on `st`
// after the launch just enqueued; a no-op otherwise.
void tl_mark(rk_ctx* c, cudaStream_t st, const char* name);

struct Run {
    rk_ctx* c;
    cudaStream_t st;
    bool split;  // FP32 semantics
    rk_status status = RK_OK;

    bool ok() const { return status == RK_OK; }
    void check_launch(const char* what) {
        c->launches++;
        tl_mark(c, st, what);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess && status == RK_OK) status = fail_cuda_err(RK_ERR_LAUNCH, what, e);
    }
    void merge(const Run& o) { if (status == RK_OK) status = o.status; }
};

// conv launch description (defaults: plain stride-1 conv, bias on)
struct ConvCall {
    const ConvW* w = nullptr;
    const Operand* op = nullptr;
    int rows_in = 0;        // rows of the operand planes
    bool split = true;
    int M = 0, T_out = 0;
    int dil = 1, pad = 0;   // tap_off[k] = k*dil - pad (phases == 1)
    int a_off = 0;
    int o_stride = 1, o_off = 0, o_phase_step = 0;
    float* y = nullptr;
    int ldy = 0;
    const float* res = nullptr;
    int ldres = 0, res_shift = 0;
    const float* acc_in = nullptr;
    int ldacc = 0;
    float alpha = 1.0f;
    float* stats = nullptr;
    int stats_ld = 0;
    int dup_src_row = -1;
    int o_min = 0;          // first valid output row
    int act = 0;            // 1: GELU after bias
    bool use_bias = true;
    bool no_splitk = false; // never split the reduction (summation order independent of M)
    const int* part_rows = nullptr;  // segmented rows: valid rows per 64-row part (ConvArgs::part_rows)
};

int stats_parts_for(const ConvCall& cc);
void conv(Run& r, const ConvCall& cc);
void pack(Run& r, const float* x, int ldx, int rows, int C, const Operand& op, int Cp, bool split,
          const float* coef = nullptr, const float* snake = nullptr, float slope = 0.f, bool lrelu = false,
          int sr_stride = 1, int sr_pad = 0, int rows_dst = -1, SegRows sr = SegRows{}, int coef_stride = 0);
void coef(Run& r, const float* stats, int parts, int ld, int col0, const AdaINW& n, int T, const StyleFC& fc,
          Lane& ln);
void record(Run& r, const char* name, const float* d, size_t n);
void record_cols(Run& r, const char* name, const float* d, int rows, int ld, int C);
void resblk1d(Run& r, const ResBlk1dW& b, const float* x, int ldx, const float* stats_x, int parts_x, int ldsx,
              int T, float* y, int ldy, float* stats_y, int ldsy, const StyleFC& fc);
void resblock1(Run& r, Lane& ln, const ResBlock1W& rb, const float* x0, const float* sx0, int parts0, int T,
               float* out, const StyleFC& fc);

}  // namespace rk
