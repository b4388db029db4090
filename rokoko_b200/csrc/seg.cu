// seg.cu -- the segmented frame layout (several utterances in one tensor) and
// AdainResBlk1d over it with per-utterance InstanceNorm; used by the batched
// F0 / N chains (infer.cu) and the batched decoder blocks (decode_batch.cu).
#include <algorithm>
#include <cmath>

#include "seg.h"

namespace rk {

// Frames of a batch in the segmented layout the F0 / N chains run on:
// utterance u's L_b frames start at off[u], a multiple of 64, with at least one
// zero-operand gap row after it (the K = 3 convs' padding), R rows in all.
// After the x2 upsample of the chains every offset and length doubles.  Parts
// (64 rows) never straddle two utterances, so the InstanceNorm partials the
// conv epilogues write per part belong to one utterance each.
std::vector<int> frame_layout_host(const std::vector<int>& Lb, FrameLayout& L) {
    const int B = (int)Lb.size();
    L.B = B;
    L.off.resize(B);
    L.len = Lb;
    int o = 0;
    for (int b = 0; b < B; b++) {
        L.off[b] = o;
        o = (o + Lb[b] + 1 + 63) / 64 * 64;
    }
    L.R = (L.off[B - 1] + Lb[B - 1] + 63) / 64 * 64;
    const int P = L.R / 64;
    // [seg1 P | rows1 P | seg2 2P | rows2 2P | p0 B | np B | T B | p0_2 B | np_2 B | T_2 B]
    std::vector<int> h((size_t)6 * P + 6 * B, 0);
    int* seg1 = h.data();
    int* rows1 = seg1 + P;
    int* seg2 = rows1 + P;
    int* rows2 = seg2 + 2 * P;
    int* ab = rows2 + 2 * P;
    for (int p = 0; p < P; p++) seg1[p] = -1;
    for (int p = 0; p < 2 * P; p++) seg2[p] = -1;
    for (int b = 0; b < B; b++) {
        const int p0 = L.off[b] / 64, np = (Lb[b] + 63) / 64;
        for (int p = p0; p < p0 + np; p++) {
            seg1[p] = b;
            rows1[p] = std::min(64, L.off[b] + Lb[b] - 64 * p);
            const int v2 = 2 * rows1[p];
            seg2[2 * p] = b;
            rows2[2 * p] = std::min(64, v2);
            if (v2 > 64) { seg2[2 * p + 1] = b; rows2[2 * p + 1] = v2 - 64; }
        }
        ab[b] = p0; ab[B + b] = np; ab[2 * B + b] = Lb[b];
        ab[3 * B + b] = 2 * p0; ab[4 * B + b] = (2 * Lb[b] + 63) / 64; ab[5 * B + b] = 2 * Lb[b];
    }
    return h;
}

void frame_layout_device(const int* d, int g_stride, FrameLayout& L) {
    const int P = L.R / 64, B = L.B;
    L.sr1 = SegRows{d, d + P};
    L.sr2 = SegRows{d + 2 * P, d + 4 * P};
    const int* ab = d + 6 * P;
    L.as1 = AdaSegs{ab, ab + B, ab + 2 * B, B, g_stride};
    L.as2 = AdaSegs{ab + 3 * B, ab + 4 * B, ab + 5 * B, B, g_stride};
}

void resblk1d_seg(Run& r, const SegWS& ws, const ResBlk1dW& b, const FrameLayout& L, bool in_x2, const float* x,
                  int ldx, const float* stats_x, int ldsx, float* y, int ldy, float* stats_y, int ldsy) {
    const bool sp = r.split;
    const bool out_x2 = in_x2 || b.upsample;
    const int Rin = in_x2 ? 2 * L.R : L.R, Ro = out_x2 ? 2 * L.R : L.R;
    const SegRows& sri = in_x2 ? L.sr2 : L.sr1;
    const SegRows& sro = out_x2 ? L.sr2 : L.sr1;
    const AdaSegs& asi = in_x2 ? L.as2 : L.as1;
    const AdaSegs& aso = out_x2 ? L.as2 : L.as1;
    const int parts_in = Rin / 64, parts_out = Ro / 64;
    const float* res = x;
    int ldres = ldx, shift = 0;
    if (b.shortcut) {  // 1x1 conv at the input rows (the nearest upsample commutes with it)
        pack(r, x, ldx, Rin, b.din, ws.op, b.conv1x1.Cp, sp);
        ConvCall cs;
        cs.w = &b.conv1x1; cs.op = &ws.op; cs.rows_in = Rin; cs.split = sp; cs.M = Rin; cs.T_out = Rin;
        cs.y = ws.sc; cs.ldy = b.dout; cs.use_bias = false; cs.no_splitk = true; cs.part_rows = sri.part_rows;
        conv(r, cs);
        res = ws.sc; ldres = b.dout; shift = b.upsample ? 1 : 0;
    }
    auto coefs = [&](const float* stats, int parts, int ld, const AdaINW& n, const AdaSegs& as) {
        if (!r.ok()) return;
        AdaSegs a = as;
        a.g_stride = ws.fc_stride;
        adain_coef(stats, parts, ld, 0, n.C, 0, ws.fc + n.fc_off, ws.fc + n.fc_off + n.C, n.norm_w, n.norm_b, ws.coef,
                   r.st, a);
        r.check_launch("adain_coef");
    };
    coefs(stats_x, parts_in, ldsx, b.norm1, asi);
    if (b.upsample) {
        if (!r.ok()) return;
        dw_upsample_pack(x, ldx, Rin, b.din, ws.coef, ws.coef + b.din, 0.2f, b.pool_w, b.pool_b, ws.op.hi, ws.op.lo,
                         b.conv1.Cp, sp, r.st, sri, 2 * b.din);
        r.check_launch("dw_upsample_pack");
    } else {
        pack(r, x, ldx, Rin, b.din, ws.op, b.conv1.Cp, sp, ws.coef, nullptr, 0.2f, true, 1, 0, -1, sri, 2 * b.din);
    }
    ConvCall c1;
    c1.w = &b.conv1; c1.op = &ws.op; c1.rows_in = Ro; c1.split = sp; c1.M = Ro; c1.T_out = Ro; c1.pad = 1;
    c1.y = ws.r1; c1.ldy = b.dout; c1.stats = ws.stats_a; c1.stats_ld = b.dout; c1.no_splitk = true;
    c1.part_rows = sro.part_rows;
    conv(r, c1);
    coefs(ws.stats_a, parts_out, b.dout, b.norm2, aso);
    pack(r, ws.r1, b.dout, Ro, b.dout, ws.op, b.conv2.Cp, sp, ws.coef, nullptr, 0.2f, true, 1, 0, -1, sro,
         2 * b.dout);
    ConvCall c2;
    c2.w = &b.conv2; c2.op = &ws.op; c2.rows_in = Ro; c2.split = sp; c2.M = Ro; c2.T_out = Ro; c2.pad = 1;
    c2.y = y; c2.ldy = ldy; c2.res = res; c2.ldres = ldres; c2.res_shift = shift;
    c2.alpha = 1.0f / sqrtf(2.0f);
    c2.stats = stats_y; c2.stats_ld = ldsy ? ldsy : ldy; c2.no_splitk = true; c2.part_rows = sro.part_rows;
    conv(r, c2);
}

}  // namespace rk
