// decode_batch.cu -- rk_decode over a batch of pending utterances: the decoder
// blocks (src/rokoko.cpp:915-990: F0 / N downsample, concat, asr_res, encode +
// four decode blocks) of every utterance in one pass over their segmented
// frames (seg.h), so that each of the ~60 launches has the rows of the whole
// batch instead of one utterance's L, then the generator of each utterance as
// its cached CUDA graph (decode.cu, generator-only variant).
//
// Reduction order: no conv launch here splits its reduction and every
// InstanceNorm partial covers rows of one utterance, so an utterance's bits do
// not depend on the batch it is decoded in (rk_infer decodes a batch of one).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "decode.h"
#include "exec.h"
#include "model.h"
#include "ops.cuh"
#include "seg.h"
#include "status.h"

namespace rk {

namespace {

size_t al(size_t x) { return (x + 255) & ~size_t(255); }

rk_status ensure_dws(rk_ctx* c, int R, int B) {
    DecBatchWS& w = c->dws;
    if (w.cap_R >= R && w.cap_B >= B) return RK_OK;
    R = std::max(R, w.cap_R);
    B = std::max(B, w.cap_B);
    if (!w.allocs.empty()) {
        cudaStreamSynchronize(c->stream);
        for (void* p : w.allocs) cudaFree(p);
        w.allocs.clear();
    }
    const size_t r = (size_t)R, P = r / 64;
    const size_t st = 2 * (P + 8) * 1090, st2 = 2 * (2 * P + 8) * 1024;
    const size_t plane = 2 * r * 1152 * 2;  // decode[3] conv1: 2R rows of the 1090 (-> 1152) channels
    struct Req { void** p; size_t bytes; };
    std::vector<Req> reqs = {
        {(void**)&w.asr, r * 512 * 4}, {(void**)&w.f0, 2 * r * 4}, {(void**)&w.n, 2 * r * 4},
        {(void**)&w.style, (size_t)B * 128 * 4}, {(void**)&w.fc, (size_t)B * c->dec.fc.rows * 4},
        {(void**)&w.f0d, r * 4}, {(void**)&w.nd, r * 4}, {(void**)&w.cat514, r * 514 * 4},
        {(void**)&w.asr_res, r * 64 * 4}, {(void**)&w.gx, 2 * r * 512 * 4},
        {(void**)&w.in1090[0], r * 1090 * 4}, {(void**)&w.in1090[1], r * 1090 * 4},
        {(void**)&w.in1090[2], r * 1090 * 4}, {(void**)&w.in1090[3], r * 1090 * 4},
        {(void**)&w.stats_cat, st * 4}, {(void**)&w.stats_in[0], st * 4}, {(void**)&w.stats_in[1], st * 4},
        {(void**)&w.stats_in[2], st * 4}, {(void**)&w.stats_in[3], st * 4},
        {(void**)&w.sc, r * 1024 * 4}, {(void**)&w.r1, r * 1024 * 4}, {(void**)&w.coef, (size_t)B * 2 * 1152 * 4},
        {(void**)&w.stats_a, st2 * 4}, {(void**)&w.layout, (6 * P + 6 * (size_t)B) * 4},
        {&w.op.hi, plane}, {&w.op.lo, plane},
    };
    size_t total = 0;
    for (auto& q : reqs) total += al(q.bytes);
    char* base = nullptr;
    if (cudaMalloc(&base, total) != cudaSuccess) {
        cudaGetLastError();
        w.cap_R = w.cap_B = 0;
        return fail(RK_ERR_OOM, "batched decoder workspace allocation");
    }
    w.allocs.push_back(base);
    size_t off = 0;
    for (auto& q : reqs) { *q.p = base + off; off += al(q.bytes); }
    w.op.plane_bytes = plane;
    w.cap_R = R;
    w.cap_B = B;
    return RK_OK;
}

// decoder blocks of the batch -> dws.gx [2R][512] (x2 layout)
rk_status enqueue_decoder_blocks(rk_ctx* c, const FrameLayout& L) {
    const DecoderW& d = c->dec;
    DecBatchWS& w = c->dws;
    const bool sp = c->precision == RK_PRECISION_FP32;
    Run r{c, c->stream, sp};
    const int R = L.R, P = R / 64, B = L.B;
    style_fc_batch(d.fc.w, d.fc.b, w.style, 128, B, w.fc, d.fc.rows, r.st);
    r.check_launch("style_fc");
    f0n_down_seg(w.f0, w.n, d.f0_conv_w, d.f0_conv_b, d.n_conv_w, d.n_conv_b, w.f0d, w.nd, R, L.sr1, L.as1, r.st);
    r.check_launch("f0n_down");
    concat_cols(w.cat514, 514, 0, R, w.asr, 512, 512, nullptr, 0, 0, w.f0d, w.nd, r.st);
    r.check_launch("concat514");
    col_stats(w.cat514, 514, 0, 514, R, STATS_ROWS, w.stats_cat, r.st, L.sr1.part_rows);
    r.check_launch("col_stats");
    {  // asr_res: Conv1d 512 -> 64 (K1), FP32 semantics in both precisions
        pack(r, w.asr, 512, R, 512, w.op, d.asr_res.Cp, true);
        ConvCall ca;
        ca.w = &d.asr_res; ca.op = &w.op; ca.rows_in = R; ca.split = true; ca.M = R; ca.T_out = R;
        ca.y = w.asr_res; ca.ldy = 64; ca.no_splitk = true; ca.part_rows = L.sr1.part_rows;
        conv(r, ca);
    }
    for (int i = 0; i < 4; i++) {  // side channels of the decode-block inputs: [x | asr_res | F0d | Nd]
        concat_cols(w.in1090[i], 1090, 1024, R, w.asr_res, 64, 64, nullptr, 0, 0, w.f0d, w.nd, r.st);
        r.check_launch("concat_side");
        col_stats(w.in1090[i], 1090, 1024, 66, R, STATS_ROWS, w.stats_in[i], r.st, L.sr1.part_rows);
        r.check_launch("col_stats");
    }
    SegWS ws;
    ws.op = w.op; ws.sc = w.sc; ws.r1 = w.r1; ws.coef = w.coef; ws.stats_a = w.stats_a;
    ws.fc = w.fc; ws.fc_stride = d.fc.rows;  // the acoustic-style FCs of every utterance
    (void)P;
    resblk1d_seg(r, ws, d.encode, L, false, w.cat514, 514, w.stats_cat, 514, w.in1090[0], 1090, w.stats_in[0], 1090);
    for (int bi = 0; bi < 3; bi++)
        resblk1d_seg(r, ws, d.decode[bi], L, false, w.in1090[bi], 1090, w.stats_in[bi], 1090, w.in1090[bi + 1], 1090,
                     w.stats_in[bi + 1], 1090);
    resblk1d_seg(r, ws, d.decode[3], L, false, w.in1090[3], 1090, w.stats_in[3], 1090, w.gx, 512, nullptr, 0);
    return r.status;
}

}  // namespace

void free_decode_batch_ws(rk_ctx* c) {
    for (void* p : c->dws.allocs) cudaFree(p);
    c->dws = DecBatchWS{};
}

rk_status decode_batch(rk_ctx* c, const PendingRef* p, int n, float* const* pcm) {
    if (n < 1) return RK_OK;
    std::vector<int> Lb(n);
    int Lbmax = 0;
    for (int i = 0; i < n; i++) { Lb[i] = p[i].L_b; Lbmax = std::max(Lbmax, p[i].L_b); }
    FrameLayout lay;
    const std::vector<int> tables = frame_layout_host(Lb, lay);
    rk_status s = ensure_dws(c, lay.R, n);
    if (!s) s = ensure_decode_ws(c, Lbmax);
    if (s) return s;
    DecBatchWS& w = c->dws;
    cudaStream_t st = c->stream;
    // pageable source: the copy completes before the call returns
    if (cudaMemcpyAsync(w.layout, tables.data(), tables.size() * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return fail_cuda(RK_ERR_CUDA, "rk_decode: layout upload");
    frame_layout_device(w.layout, c->dec.fc.rows, lay);
    for (int i = 0; i < n; i++) {  // inputs into the segmented frames
        const size_t o = (size_t)lay.off[i];
        if (cudaMemcpyAsync(w.asr + o * 512, p[i].asr, (size_t)Lb[i] * 512 * 4, cudaMemcpyDeviceToDevice, st) !=
                cudaSuccess ||
            cudaMemcpyAsync(w.f0 + 2 * o, p[i].f0, (size_t)2 * Lb[i] * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(w.n + 2 * o, p[i].n, (size_t)2 * Lb[i] * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(w.style + (size_t)i * 128, p[i].style, 128 * 4, cudaMemcpyDeviceToDevice, st) !=
                cudaSuccess)
            return fail_cuda(RK_ERR_CUDA, "rk_decode: decoder inputs");
    }
    s = enqueue_decoder_blocks(c, lay);
    if (s) return s;
    DecodeWS& ws = c->ws;
    for (int i = 0; i < n; i++) {  // the generator of each utterance (its graph reads ws.gx / f0 / style)
        const size_t o = (size_t)lay.off[i];
        if (cudaMemcpyAsync(ws.gx, w.gx + 2 * o * 512, (size_t)2 * Lb[i] * 512 * 4, cudaMemcpyDeviceToDevice, st) !=
                cudaSuccess ||
            cudaMemcpyAsync(ws.f0, p[i].f0, (size_t)2 * Lb[i] * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(ws.style, p[i].style, 128 * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
            return fail_cuda(RK_ERR_CUDA, "rk_decode: generator inputs");
        s = enqueue_decode(c, Lb[i], /*gen_only*/ true);
        if (s) return s;
        const size_t ns = (size_t)600 * p[i].L;
        if (pcm && pcm[i] && cudaMemcpyAsync(pcm[i], ws.audio, ns * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
            return fail_cuda(RK_ERR_CUDA, "rk_decode: pcm download");
    }
    return RK_OK;
}

}  // namespace rk
