// infer.cu -- the full forward for one utterance (rokoko_infer,
// src/rokoko.cpp:829-1297): ALBERT, text encoder, duration encoder and
// durations, duration -> alignment, shared LSTM, F0 / N prediction, then the
// decode phase (decode.cu).
//
// Every linear layer and conv runs on the tcgen05 conv kernel (a Linear is a
// K = 1 conv); row LayerNorms / AdaLayerNorm / attention / LSTM recurrence are
// the kernels of front_ops.cu and lstm.cu.  The only host <-> device sync
// inside is the read-back of the predicted durations (the reference reads L,
// src/rokoko.cpp:790-793), needed to size the decode.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "decode.h"
#include "exec.h"
#include "front_ops.cuh"
#include "infer.h"
#include "ops.cuh"

namespace rk {

namespace {

size_t al(size_t x) { return (x + 255) & ~size_t(255); }

OpPlanes planes(const Operand& o, int Cp) { return OpPlanes{o.hi, o.lo, Cp}; }

void lstm(Run& r, const LstmW& l, const Operand& op, int T, float* out) {
    FrontWS& f = r.c->fws;
    ConvCall cg;
    cg.w = &l.wih; cg.op = &op; cg.rows_in = T; cg.split = r.split; cg.M = T; cg.T_out = T;
    cg.y = f.ig; cg.ldy = 2048;
    conv(r, cg);
    if (!r.ok()) return;
    cudaError_t e = bilstm_recurrence(f.ig, l.whh, T, out, r.c->err, r.st);
    r.c->launches++;
    if (e != cudaSuccess) r.status = fail_cuda_err(RK_ERR_LAUNCH, "bilstm", e);
}

void linear(Run& r, const ConvW& w, const Operand& op, int T, float* y, int act = 0) {
    ConvCall cc;
    cc.w = &w; cc.op = &op; cc.rows_in = T; cc.split = r.split; cc.M = T; cc.T_out = T;
    cc.y = y; cc.ldy = w.C_out;
    cc.act = act;
    conv(r, cc);
}

}  // namespace

void free_front_ws(rk_ctx* c) {
    for (void* p : c->fws.allocs) cudaFree(p);
    for (void* p : c->fws.frame_allocs) cudaFree(p);
    c->fws = FrontWS{};
}

namespace {
struct Req { void** p; size_t bytes; };
char* alloc_group(std::vector<Req>& reqs, size_t extra, std::vector<void*>& owner) {
    size_t total = extra;
    for (auto& q : reqs) total += al(q.bytes);
    char* base = nullptr;
    if (cudaMalloc(&base, total) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    owner.push_back(base);
    size_t off = 0;
    for (auto& q : reqs) { *q.p = base + off; off += al(q.bytes); }
    return base + off;
}
}  // namespace

// Token-sized buffers (max_tokens rows), allocated once.
rk_status ensure_front_tokens(rk_ctx* c) {
    FrontWS& f = c->fws;
    if (!f.allocs.empty()) return RK_OK;
    const size_t T = (size_t)c->max_tokens;
    std::vector<Req> reqs = {
        {(void**)&f.tok, T * 4}, {(void**)&f.style, 256 * 4}, {(void**)&f.dur_i, T * 4}, {(void**)&f.dur_use, T * 4},
        {(void**)&f.dur_f, T * 4}, {(void**)&f.emb, T * 128 * 4}, {(void**)&f.h, T * 768 * 4},
        {(void**)&f.qkv, T * 2304 * 4}, {(void**)&f.ctx, T * 768 * 4}, {(void**)&f.tmp, T * 768 * 4},
        {(void**)&f.ffmid, T * 2048 * 4}, {(void**)&f.d_en, T * 512 * 4}, {(void**)&f.te, T * 512 * 4},
        {(void**)&f.tbuf, T * 512 * 4}, {(void**)&f.cat, T * 640 * 4}, {(void**)&f.lstm_out, T * 512 * 4},
        {(void**)&f.proj, T * 50 * 4},
    };
    if (!alloc_group(reqs, 0, f.allocs)) return fail(RK_ERR_OOM, "front workspace allocation");
    return RK_OK;
}

// Frame-sized buffers for up to L_b frames (grow on demand; contents are not
// carried across a growth).
rk_status ensure_front_frames(rk_ctx* c, int L_b) {
    FrontWS& f = c->fws;
    if (f.cap_L >= L_b) return RK_OK;
    for (void* p : f.frame_allocs) cudaFree(p);
    f.frame_allocs.clear();
    const size_t L = (size_t)L_b, rows = std::max((size_t)c->max_tokens, L);
    std::vector<Req> reqs = {
        {(void**)&f.ig, rows * 2048 * 4}, {(void**)&f.en, L * 640 * 4}, {(void**)&f.shared, L * 512 * 4},
        {(void**)&f.x1, L * 512 * 4}, {(void**)&f.x2, 2 * L * 256 * 4}, {(void**)&f.x3, 2 * L * 256 * 4},
        {(void**)&f.stats, 2 * ((2 * L + STATS_ROWS - 1) / STATS_ROWS + 8) * 512 * 4},
        {(void**)&f.stats2, 2 * ((2 * L + STATS_ROWS - 1) / STATS_ROWS + 8) * 512 * 4},
    };
    const size_t plane = al(std::max((size_t)c->max_tokens * 2048, L * 640) * 2);
    char* rest = alloc_group(reqs, 2 * plane, f.frame_allocs);
    if (!rest) return fail(RK_ERR_OOM, "front frame workspace allocation");
    f.op.hi = rest;
    f.op.lo = rest + plane;
    f.op.plane_bytes = plane;
    f.cap_L = L_b;
    return RK_OK;
}

// Encode phase up to the durations (src/rokoko.cpp:872-916); inputs in fws.tok / fws.style.
rk_status enqueue_encode(rk_ctx* c, int T) {
    FrontW& F = c->front;
    FrontWS& f = c->fws;
    const bool sp = c->precision == RK_PRECISION_FP32;
    Run r{c, c->stream, sp};
    const float* s_pr = f.style + 128;  // ref_s[128:256] prosody style
    style_fc(F.fc.w, F.fc.b, s_pr, F.fc.out, F.fc.rows, r.st);
    r.check_launch("style_fc");
    // ---- ALBERT (src/rokoko.cpp:335-408)
    embed_ln(f.tok, T, F.word, F.pos, F.type, F.emb_ln_w, F.emb_ln_b, f.emb, planes(f.op, F.proj.Cp), sp, r.st);
    r.check_launch("embed_ln");
    linear(r, F.proj, f.op, T, f.h);
    pack(r, f.h, 768, T, 768, f.op, F.qkv.Cp, sp);
    for (int layer = 0; layer < 12 && r.ok(); layer++) {
        linear(r, F.qkv, f.op, T, f.qkv);
        attention(f.qkv, T, f.ctx, r.st);
        r.check_launch("attention");
        pack(r, f.ctx, 768, T, 768, f.op, F.dense.Cp, sp);
        linear(r, F.dense, f.op, T, f.tmp);
        res_ln(f.h, f.tmp, T, F.attn_ln_w, F.attn_ln_b, planes(f.op, F.ffn.Cp), sp, r.st);
        r.check_launch("res_ln");
        linear(r, F.ffn, f.op, T, f.ffmid, /*gelu*/ 1);
        pack(r, f.ffmid, 2048, T, 2048, f.op, F.ffn_out.Cp, sp);
        linear(r, F.ffn_out, f.op, T, f.tmp);
        res_ln(f.h, f.tmp, T, F.ffn_ln_w, F.ffn_ln_b, planes(f.op, F.qkv.Cp), sp, r.st);
        r.check_launch("res_ln");
    }
    record(r, "bert", f.h, (size_t)T * 768);
    linear(r, F.bert_enc, f.op, T, f.d_en);  // operand of the last res_ln is h
    record(r, "d_en", f.d_en, (size_t)T * 512);
    // ---- text encoder (src/rokoko.cpp:421-478)
    gather_rows(f.tok, T, F.te_embed, 512, f.te, planes(f.op, F.te_conv[0].Cp), sp, r.st);
    r.check_launch("gather_rows");
    for (int i = 0; i < 3 && r.ok(); i++) {
        ConvCall cc;
        cc.w = &F.te_conv[i]; cc.op = &f.op; cc.rows_in = T; cc.split = sp; cc.M = T; cc.T_out = T; cc.pad = 2;
        cc.y = f.tbuf; cc.ldy = 512;
        conv(r, cc);
        ln_lrelu(f.tbuf, T, F.te_ln_g[i], F.te_ln_b[i], f.te, planes(f.op, i < 2 ? F.te_conv[i + 1].Cp : 512), sp,
                 r.st);
        r.check_launch("ln_lrelu");
    }
    lstm(r, F.te_lstm, f.op, T, f.te);
    record(r, "text_enc", f.te, (size_t)T * 512);
    // ---- duration encoder (src/rokoko.cpp:884-897): cat = [x | s_pr]
    adaln_concat(f.d_en, T, nullptr, nullptr, s_pr, f.cat, planes(f.op, 640), sp, r.st);
    r.check_launch("adaln_concat");
    for (int i = 0; i < 3 && r.ok(); i++) {
        lstm(r, F.dur_lstm[i], f.op, T, f.lstm_out);
        const float* gm = F.fc.out + F.aln_off[i];
        adaln_concat(f.lstm_out, T, gm, gm + 512, s_pr, f.cat, planes(f.op, 640), sp, r.st);
        r.check_launch("adaln_concat");
    }
    record(r, "dur_enc", f.cat, (size_t)T * 640);
    // ---- durations (src/rokoko.cpp:899-905)
    lstm(r, F.dur_final, f.op, T, f.lstm_out);
    pack(r, f.lstm_out, 512, T, 512, f.op, F.dur_proj.Cp, sp);
    linear(r, F.dur_proj, f.op, T, f.proj);
    durations(f.proj, T, f.dur_f, f.dur_i, r.st);
    r.check_launch("durations");
    record(r, "dur_float", f.dur_f, (size_t)T);
    return r.status;
}

// Alignment, shared LSTM and F0 / N prediction (src/rokoko.cpp:848-913) for
// durations fws.dur_use; writes the decoder inputs ws.asr / ws.f0 / ws.n / ws.style.
rk_status enqueue_predict(rk_ctx* c, int T, int L_b) {
    FrontW& F = c->front;
    FrontWS& f = c->fws;
    DecodeWS& w = c->ws;
    const bool sp = c->precision == RK_PRECISION_FP32;
    Run r{c, c->stream, sp};
    align_gather(f.dur_use, T, L_b, f.cat, f.te, f.en, w.asr, planes(f.op, 640), sp, r.st);
    r.check_launch("align_gather");
    lstm(r, F.shared, f.op, L_b, f.shared);
    record(r, "shared", f.shared, (size_t)L_b * 512);
    record(r, "asr_aligned", w.asr, (size_t)L_b * 512);
    const int parts = conv_tc_stats_parts(L_b, 1);
    col_stats(f.shared, 512, 0, 512, L_b, STATS_ROWS, f.stats, r.st);
    r.check_launch("col_stats");
    for (int chain = 0; chain < 2 && r.ok(); chain++) {
        const ResBlk1dW* b = chain == 0 ? F.f0 : F.nn;
        resblk1d(r, b[0], f.shared, 512, f.stats, parts, 512, L_b, f.x1, 512, f.stats2, 512, F.fc);
        resblk1d(r, b[1], f.x1, 512, f.stats2, parts, 512, L_b, f.x2, 256, f.stats, 256, F.fc);
        resblk1d(r, b[2], f.x2, 256, f.stats, conv_tc_stats_parts(2 * L_b, 1), 256, 2 * L_b, f.x3, 256, nullptr, 0, F.fc);
        rowdot(f.x3, 2 * L_b, 256, chain == 0 ? F.f0_proj_w : F.n_proj_w, chain == 0 ? F.f0_proj_b : F.n_proj_b,
               chain == 0 ? w.f0 : w.n, r.st);
        r.check_launch("rowdot");
        if (chain == 0) {  // the N chain reuses the statistics buffer of `shared`
            col_stats(f.shared, 512, 0, 512, L_b, STATS_ROWS, f.stats, r.st);
            r.check_launch("col_stats");
        }
    }
    record(r, "f0_pred", w.f0, (size_t)2 * L_b);
    record(r, "n_pred", w.n, (size_t)2 * L_b);
    if (cudaMemcpyAsync(w.style, f.style, 128 * 4, cudaMemcpyDeviceToDevice, r.st) != cudaSuccess)
        return fail_cuda(RK_ERR_CUDA, "style copy");
    return r.status;
}

}  // namespace rk
