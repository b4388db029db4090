// seg.h -- several utterances in one tensor: the segmented frame layout and
// the AdainResBlk1d block over it (per-utterance InstanceNorm).
//
// Utterance u's n_u rows (n_u = its L_b, a multiple of 32) start at off[u], a
// multiple of 64, with at least one gap row after it (the K = 3 convs'
// padding); R rows in all.  A x2 upsample doubles every offset and length.
// A 64-row part never holds two utterances, so the InstanceNorm partials that
// conv epilogues write per part belong to one utterance each; per-part valid-row
// counts make the epilogues skip gap rows, AdaIN coefficients are computed per
// utterance, and the operand packs write gap rows as zeros.
#pragma once
#include <vector>

#include "exec.h"
#include "ops.cuh"

namespace rk {

struct FrameLayout {
    int B = 0, R = 0;
    std::vector<int> off, len;
    // device tables: SegRows + AdaSegs of the base and of the x2 layout
    SegRows sr1, sr2;
    AdaSegs as1, as2;
};

// Host side: offsets for lengths Lb, and the device tables' contents
// ([seg1 P | rows1 P | seg2 2P | rows2 2P | p0 B | np B | T B | p0_2 B | np_2 B | T_2 B], P = R / 64).
std::vector<int> frame_layout_host(const std::vector<int>& Lb, FrameLayout& L);
// Points the layout's tables at their device copy `d`; g_stride = floats between
// two utterances' style-FC outputs (the AdaIN gamma / beta).
void frame_layout_device(const int* d, int g_stride, FrameLayout& L);

// Buffers of resblk1d_seg: operand planes, shortcut output, conv1 output,
// per-utterance coefficients, conv1 statistics; fc = the utterances'
// style-FC outputs ([B][fc_stride], gamma at + AdaINW::fc_off).
struct SegWS {
    Operand op;
    float *sc = nullptr, *r1 = nullptr, *coef = nullptr, *stats_a = nullptr;
    const float* fc = nullptr;
    int fc_stride = 0;
};

// AdainResBlk1d (src/rokoko.cpp:583-643) over the segmented rows of a batch.
// x [R_in][ldx] (in_x2: the x2 layout) with partials stats_x over all parts of
// its layout (row pitch ldsx); y [R_out][ldy] (x2 when in_x2 or upsampling),
// partials stats_y (nullable, pitch ldsy).
void resblk1d_seg(Run& r, const SegWS& ws, const ResBlk1dW& b, const FrameLayout& L, bool in_x2, const float* x,
                  int ldx, const float* stats_x, int ldsx, float* y, int ldy, float* stats_y, int ldsy);

}  // namespace rk
