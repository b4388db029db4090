// infer.cu -- the front half of rokoko_infer (src/rokoko.cpp:829-914,
// src/rokoko_f16.cpp:688-914) for a whole batch of utterances at once:
// ALBERT, text encoder, duration encoder and durations, duration -> alignment
// and the shared LSTM, then each utterance's F0 / N prediction.
//
// The reference runs one utterance per call (src/weights.h:402-405) and reads
// its predicted durations back once per utterance (src/rokoko_f16.cpp:790-793).
// Here every launch of the token phase covers all utterances of the batch:
// the linear layers and convs run on the tcgen05 conv kernel over the rows of
// every utterance (segmented layout, front_ops.cuh), attention runs per
// (utterance, head) inside one launch, and each BiLSTM is one persistent
// launch over all utterances and both directions.  The host reads the
// durations of the whole batch back once, sizes the frames, and the frame
// phase (alignment, shared LSTM) is again one launch per layer for the batch.
// The F0 / N chains (InstanceNorm over each utterance's own frames) run per
// utterance as a CUDA graph keyed by the frame bucket L_b.
//
// Reduction order: front-half conv launches never split their reduction
// (split-K would make the summation order depend on the batch's row count),
// so every utterance's activations are bit-identical whether it is encoded
// alone or in a batch.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "decode.h"
#include "exec.h"
#include "front_ops.cuh"
#include "infer.h"
#include "ops.cuh"
#include "seg.h"

namespace rk {

namespace {

size_t al(size_t x) { return (x + 255) & ~size_t(255); }

OpPlanes planes(const Operand& o, int Cp) { return OpPlanes{o.hi, o.lo, Cp}; }

// a K = 1 conv (Linear) over `rows` rows, no split-K
void linear(Run& r, const ConvW& w, const Operand& op, int rows, float* y, int act = 0) {
    ConvCall cc;
    cc.w = &w; cc.op = &op; cc.rows_in = rows; cc.split = r.split; cc.M = rows; cc.T_out = rows;
    cc.y = y; cc.ldy = w.C_out;
    cc.act = act;
    cc.no_splitk = true;
    conv(r, cc);
}

void lstm(Run& r, const LstmW& l, const Operand& op, int rows, SegMeta seq, float* out) {
    FrontWS& f = r.c->fws;
    ConvCall cg;
    cg.w = &l.wih; cg.op = &op; cg.rows_in = rows; cg.split = r.split; cg.M = rows; cg.T_out = rows;
    cg.y = f.ig; cg.ldy = 2048;
    cg.no_splitk = true;
    conv(r, cg);
    if (!r.ok()) return;
    cudaError_t e = bilstm_recurrence(f.ig, l.whh, seq, bilstm_group(seq.n), out, r.st);
    r.check_launch("bilstm");
    if (e != cudaSuccess && r.ok()) r.status = fail_cuda_err(RK_ERR_LAUNCH, "bilstm", e);
}

struct Req {
    void** p;
    size_t bytes;
};

// one cudaMalloc for a group of buffers (256-byte aligned slices); frees the group's previous allocation
rk_status alloc_group(rk_ctx* c, std::vector<Req> reqs, std::vector<void*>& owner, const char* what) {
    if (!owner.empty()) {
        cudaDeviceSynchronize();  // queued work (either stream of the context) may still use the old buffers
        for (void* p : owner) cudaFree(p);
        owner.clear();
    }
    size_t total = 0;
    for (auto& q : reqs) total += al(q.bytes);
    char* base = nullptr;
    if (cudaMalloc(&base, total) != cudaSuccess) {
        cudaGetLastError();
        return fail(RK_ERR_OOM, what);
    }
    owner.push_back(base);
    size_t off = 0;
    for (auto& q : reqs) { *q.p = base + off; off += al(q.bytes); }
    return RK_OK;
}

rk_status ensure_rows(rk_ctx* c, int R, int B) {
    FrontWS& f = c->fws;
    if (f.cap_R >= R && f.cap_B >= B) return RK_OK;
    R = std::max(R, f.cap_R);
    B = std::max(B, f.cap_B);
    const size_t r = (size_t)R;
    std::vector<Req> reqs = {
        {(void**)&f.meta, (4 * r + 4 * (size_t)B) * 4}, {(void**)&f.dur_i, r * 4}, {(void**)&f.style, B * 256 * 4},
        {(void**)&f.fc, (size_t)B * c->front.fc.rows * 4}, {(void**)&f.dur_f, r * 4}, {(void**)&f.emb, r * 128 * 4},
        {(void**)&f.h, r * 768 * 4}, {(void**)&f.qkv, r * 2304 * 4}, {(void**)&f.ctx, r * 768 * 4},
        {(void**)&f.tmp, r * 768 * 4}, {(void**)&f.ffmid, r * 2048 * 4}, {(void**)&f.d_en, r * 512 * 4},
        {(void**)&f.te, r * 512 * 4}, {(void**)&f.tbuf, r * 512 * 4}, {(void**)&f.cat, r * 640 * 4},
        {(void**)&f.lstm_out, r * 512 * 4}, {(void**)&f.proj, r * 50 * 4},
    };
    rk_status s = alloc_group(c, reqs, f.row_allocs, "front workspace allocation (token rows)");
    if (s) { f.cap_R = f.cap_B = 0; return s; }
    f.cap_R = R;
    f.cap_B = B;
    return RK_OK;
}

// LSTM input gates for `rows` rows and operand planes of `plane_bytes` each
rk_status ensure_ig_op(rk_ctx* c, size_t rows, size_t plane_bytes) {
    FrontWS& f = c->fws;
    if (f.cap_ig >= rows && f.cap_op >= plane_bytes) return RK_OK;
    rows = std::max(rows, f.cap_ig);
    plane_bytes = al(std::max(plane_bytes, f.cap_op));
    std::vector<void*>& owner = f.ig_allocs;
    std::vector<Req> reqs = {{(void**)&f.ig, rows * 2048 * 4}, {&f.op.hi, plane_bytes}, {&f.op.lo, plane_bytes}};
    rk_status s = alloc_group(c, reqs, owner, "front workspace allocation (gates / operands)");
    if (s) { f.cap_ig = f.cap_op = 0; return s; }
    f.cap_ig = rows;
    f.cap_op = plane_bytes;
    f.op.plane_bytes = plane_bytes;
    return RK_OK;
}

rk_status ensure_frames(rk_ctx* c, int F) {
    FrontWS& f = c->fws;
    if (f.cap_F >= F) return RK_OK;
    const size_t n = (size_t)F;
    std::vector<Req> reqs = {{(void**)&f.en, n * 640 * 4}, {(void**)&f.shared_all, n * 512 * 4},
                             {(void**)&f.frame_tok, n * 4}};
    rk_status s = alloc_group(c, reqs, f.frame_allocs, "front workspace allocation (frames)");
    if (s) { f.cap_F = 0; return s; }
    f.cap_F = F;
    return RK_OK;
}

// the batched F0 / N chains: R frame rows (x2 after the upsample), B utterances
rk_status ensure_pred(rk_ctx* c, int R, int B) {
    FrontWS& f = c->fws;
    if (f.cap_Rp >= R && f.cap_Bp >= B) return RK_OK;
    R = std::max(R, f.cap_Rp);
    B = std::max(B, f.cap_Bp);
    const size_t r = (size_t)R;
    const size_t st = 2 * (2 * r / 64 + 8) * 512 * 4;
    const size_t plane = 2 * r * 512 * 2;
    std::vector<Req> reqs = {
        {(void**)&f.x1, r * 512 * 4}, {(void**)&f.x2, 2 * r * 256 * 4}, {(void**)&f.x3, 2 * r * 256 * 4},
        {(void**)&f.r1, r * 512 * 4}, {(void**)&f.sc, r * 256 * 4}, {(void**)&f.coef, (size_t)B * 2 * 512 * 4},
        {(void**)&f.stats, st}, {(void**)&f.stats2, st}, {(void**)&f.stats_a, st},
        {(void**)&f.layout, (6 * r / 64 + 6 * (size_t)B) * 4}, {&f.op_p.hi, plane}, {&f.op_p.lo, plane},
    };
    rk_status s = alloc_group(c, reqs, f.pred_allocs, "front workspace allocation (predictor)");
    if (s) { f.cap_Rp = f.cap_Bp = 0; return s; }
    f.op_p.plane_bytes = plane;
    f.cap_Rp = R;
    f.cap_Bp = B;
    return RK_OK;
}

rk_status ensure_stage(rk_ctx* c, size_t bytes) {
    if (c->h_stage_bytes >= bytes) return RK_OK;
    if (c->h_stage) {
        cudaDeviceSynchronize();  // no upload out of the old buffer may still be queued
        cudaFreeHost(c->h_stage);
        c->h_stage = nullptr;
        c->h_stage_bytes = 0;
    }
    bytes = std::max(bytes, (size_t)1 << 20);
    if (cudaHostAlloc(&c->h_stage, bytes, cudaHostAllocPortable) != cudaSuccess) {
        cudaGetLastError();
        return fail(RK_ERR_OOM, "pinned staging buffer");
    }
    c->h_stage_bytes = bytes;
    return RK_OK;
}

// stash memory for pending utterances (chunks kept for reuse until rk_destroy)
float* stash_alloc(rk_ctx* c, size_t bytes) {
    bytes = al(bytes);
    for (auto& ch : c->stash)
        if (ch.pool == c->stash_pool && ch.bytes - ch.used >= bytes) {
            float* p = reinterpret_cast<float*>(ch.base + ch.used);
            ch.used += bytes;
            return p;
        }
    const size_t sz = std::max(bytes, (size_t)256 << 20);
    char* base = nullptr;
    if (cudaMalloc(&base, sz) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    c->stash.push_back({base, sz, bytes, c->stash_pool});
    return reinterpret_cast<float*>(base);
}

// ---------------------------------------------------------------- token phase
// ALBERT (src/rokoko.cpp:335-408), text encoder (:421-478), duration encoder
// (:884-897) and durations (:899-905) for every utterance of the batch.
rk_status enqueue_token_phase(rk_ctx* c, RowMeta m, SegMeta seg, int B) {
    FrontW& F = c->front;
    FrontWS& f = c->fws;
    const bool sp = c->precision == RK_PRECISION_FP32;
    Run r{c, c->fst, sp};
    const int R = m.R;
    // prosody-style FCs of every utterance (AdaLayerNorm gamma / beta of the duration encoder)
    style_fc_batch(F.fc.w, F.fc.b, f.style + 128, 256, B, f.fc, F.fc.rows, r.st);
    r.check_launch("style_fc");
    // ---- ALBERT
    embed_ln(m, F.word, F.pos, F.type, F.emb_ln_w, F.emb_ln_b, f.emb, planes(f.op, F.proj.Cp), sp, r.st);
    r.check_launch("embed_ln");
    linear(r, F.proj, f.op, R, f.h);
    pack(r, f.h, 768, R, 768, f.op, F.qkv.Cp, sp);
    for (int layer = 0; layer < 12 && r.ok(); layer++) {
        linear(r, F.qkv, f.op, R, f.qkv);
        {   // FP32 semantics in both precisions: the reference's FP16 build also keeps the
            // attention GEMMs on FP32 data (src/rokoko_f16.cpp:227-244)
            const cudaError_t e = attention_tc(f.qkv, seg, f.ctx, true, c->err, r.st);
            r.check_launch("attention_tc");
            if (e != cudaSuccess && r.ok()) r.status = fail_cuda_err(RK_ERR_LAUNCH, "attention_tc", e);
        }
        pack(r, f.ctx, 768, R, 768, f.op, F.dense.Cp, sp);
        linear(r, F.dense, f.op, R, f.tmp);
        res_ln(f.h, f.tmp, m, F.attn_ln_w, F.attn_ln_b, planes(f.op, F.ffn.Cp), sp, r.st);
        r.check_launch("res_ln");
        linear(r, F.ffn, f.op, R, f.ffmid, /*gelu*/ 1);
        pack(r, f.ffmid, 2048, R, 2048, f.op, F.ffn_out.Cp, sp);
        linear(r, F.ffn_out, f.op, R, f.tmp);
        res_ln(f.h, f.tmp, m, F.ffn_ln_w, F.ffn_ln_b, planes(f.op, F.qkv.Cp), sp, r.st);
        r.check_launch("res_ln");
    }
    record(r, "bert", f.h, (size_t)c->fws.len0 * 768);
    linear(r, F.bert_enc, f.op, R, f.d_en);  // operand of the last res_ln is h
    record(r, "d_en", f.d_en, (size_t)c->fws.len0 * 512);
    // ---- text encoder
    gather_rows(m, F.te_embed, 512, f.te, planes(f.op, F.te_conv[0].Cp), sp, r.st);
    r.check_launch("gather_rows");
    for (int i = 0; i < 3 && r.ok(); i++) {
        ConvCall cc;
        cc.w = &F.te_conv[i]; cc.op = &f.op; cc.rows_in = R; cc.split = sp; cc.M = R; cc.T_out = R; cc.pad = 2;
        cc.y = f.tbuf; cc.ldy = 512;
        cc.no_splitk = true;
        conv(r, cc);
        ln_lrelu(f.tbuf, m, F.te_ln_g[i], F.te_ln_b[i], f.te, planes(f.op, i < 2 ? F.te_conv[i + 1].Cp : 512), sp,
                 r.st);
        r.check_launch("ln_lrelu");
    }
    lstm(r, F.te_lstm, f.op, R, seg, f.te);
    record(r, "text_enc", f.te, (size_t)c->fws.len0 * 512);
    // ---- duration encoder: cat = [x | s_pr]
    const float* s_pr = f.style + 128;
    adaln_concat(f.d_en, m, f.fc, F.fc.rows, -1, s_pr, 256, f.cat, planes(f.op, 640), sp, r.st);
    r.check_launch("adaln_concat");
    for (int i = 0; i < 3 && r.ok(); i++) {
        lstm(r, F.dur_lstm[i], f.op, R, seg, f.lstm_out);
        adaln_concat(f.lstm_out, m, f.fc, F.fc.rows, F.aln_off[i], s_pr, 256, f.cat, planes(f.op, 640), sp, r.st);
        r.check_launch("adaln_concat");
    }
    record(r, "dur_enc", f.cat, (size_t)c->fws.len0 * 640);
    // ---- durations
    lstm(r, F.dur_final, f.op, R, seg, f.lstm_out);
    pack(r, f.lstm_out, 512, R, 512, f.op, F.dur_proj.Cp, sp);
    linear(r, F.dur_proj, f.op, R, f.proj);
    durations(f.proj, m, f.dur_f, f.dur_i, r.st);
    r.check_launch("durations");
    record(r, "dur_float", f.dur_f, (size_t)c->fws.len0);
    return r.status;
}

// ---------------------------------------------------------------- frame phase
// alignment and the shared LSTM for every utterance (src/rokoko.cpp:848-871)
rk_status enqueue_frame_phase(rk_ctx* c, const int* dur_use, SegMeta tok, SegMeta frames, int F, float* asr_out) {
    FrontW& Fw = c->front;
    FrontWS& f = c->fws;
    const bool sp = c->precision == RK_PRECISION_FP32;
    Run r{c, c->fst, sp};
    align_gather(dur_use, tok, frames, f.cat, f.te, f.en, asr_out, f.frame_tok, planes(f.op, 640), sp, r.st);
    r.check_launch("align_gather");
    lstm(r, Fw.shared, f.op, F, frames, f.shared_all);
    return r.status;
}

// ---------------------------------------------------------------- predictor
// F0 / N chains of every utterance of the batch (src/rokoko.cpp:876-913) from
// fws.shared_all (the shared LSTM's output in the segmented frame layout) ->
// f0 / n [2R] in the x2 layout.
rk_status enqueue_predict_batch(rk_ctx* c, const FrameLayout& L, float* f0, float* n) {
    FrontW& F = c->front;
    FrontWS& f = c->fws;
    const bool sp = c->precision == RK_PRECISION_FP32;
    Run r{c, c->fst, sp};
    SegWS ws;
    ws.op = f.op_p; ws.sc = f.sc; ws.r1 = f.r1; ws.coef = f.coef; ws.stats_a = f.stats_a;
    ws.fc = f.fc; ws.fc_stride = F.fc.rows;  // the prosody-style FCs of the token phase
    for (int chain = 0; chain < 2 && r.ok(); chain++) {
        col_stats(f.shared_all, 512, 0, 512, L.R, STATS_ROWS, f.stats, r.st, L.sr1.part_rows);
        r.check_launch("col_stats");
        const ResBlk1dW* b = chain == 0 ? F.f0 : F.nn;
        resblk1d_seg(r, ws, b[0], L, false, f.shared_all, 512, f.stats, 512, f.x1, 512, f.stats2, 512);
        resblk1d_seg(r, ws, b[1], L, false, f.x1, 512, f.stats2, 512, f.x2, 256, f.stats, 256);
        resblk1d_seg(r, ws, b[2], L, true, f.x2, 256, f.stats, 256, f.x3, 256, nullptr, 0);
        rowdot(f.x3, 2 * L.R, 256, chain == 0 ? F.f0_proj_w : F.n_proj_w, chain == 0 ? F.f0_proj_b : F.n_proj_b,
               chain == 0 ? f0 : n, r.st);
        r.check_launch("rowdot");
    }
    return r.status;
}

}  // namespace

void free_front_ws(rk_ctx* c) {
    FrontWS& f = c->fws;
    for (void* p : f.row_allocs) cudaFree(p);
    for (void* p : f.frame_allocs) cudaFree(p);
    for (void* p : f.pred_allocs) cudaFree(p);
    for (void* p : f.ig_allocs) cudaFree(p);
    c->fws = FrontWS{};
    for (auto& ch : c->stash) cudaFree(ch.base);
    c->stash.clear();
    if (c->h_stage) cudaFreeHost(c->h_stage);
    c->h_stage = nullptr;
    c->h_stage_bytes = 0;
    for (int i = 0; i < 2; i++) {
        if (c->h_pcm[i]) cudaFreeHost(c->h_pcm[i]);
        c->h_pcm[i] = nullptr;
        c->h_pcm_cap[i] = 0;
    }
}

void stash_reset(rk_ctx* c, int pool) {
    for (auto& ch : c->stash)
        if (ch.pool == pool) ch.used = 0;
}

rk_status encode_batch(rk_ctx* c, const int32_t* tokens, const int32_t* T_per, int B, const float* style,
                       const int32_t* dur_override, int32_t* dur_out, int32_t* L_out, const char* who) {
    const std::string w(who);
    auto bad = [&](const char* m) { return fail(RK_ERR_CANNOT_IMPLEMENT, (w + ": " + m).c_str()); };
    if (!tokens || !T_per || !style || B < 1) return bad("null argument or empty batch");
    if (!c->loaded) return fail(RK_ERR_STATE, (w + ": no weights loaded").c_str());
    if (!c->has_front)
        return fail(RK_ERR_WEIGHTS, (w + ": weight file has no front half (ALBERT / predictor)").c_str());
    // ---- validate and lay out the token rows
    std::vector<int> off(B), len(B);
    int R = 0, Tmax = 0;
    size_t n_tok = 0;
    for (int b = 0; b < B; b++) {
        const int T = T_per[b];
        if (T < 1 || T > c->max_tokens) return bad("T out of range");
        off[b] = R;
        len[b] = T;
        R += T + SEG_GAP;
        Tmax = std::max(Tmax, T);
        n_tok += (size_t)T;
    }
    for (size_t i = 0; i < n_tok; i++)
        if (tokens[i] < 0 || tokens[i] >= 178) return bad("token id out of range");
    if (dur_override)
        for (size_t i = 0; i < n_tok; i++)
            if (dur_override[i] < 0 || dur_override[i] > 4096) return bad("duration override out of range");
    rk_status s = ensure_rows(c, R, B);
    if (!s) s = ensure_ig_op(c, (size_t)R, (size_t)R * 2048 * 2);
    // metadata ints: tok[R] pos[R] utt[R] seg_off[B] seg_len[B], then the styles
    const size_t n_meta = 3 * (size_t)R + 2 * (size_t)B;
    if (!s) s = ensure_stage(c, std::max(n_meta * 4 + (size_t)B * 256 * 4, (size_t)R * 4 * 2 + 4 * (size_t)B * 4));
    if (s) return s;
    FrontWS& f = c->fws;
    // the previous batch's last uploads out of the staging buffer must be done before it is rewritten
    if (c->ev_stage && cudaEventSynchronize(c->ev_stage) != cudaSuccess)
        return fail_cuda(RK_ERR_CUDA, (w + ": staging buffer").c_str());
    int* hm = static_cast<int*>(c->h_stage);
    int* h_tok = hm;
    int* h_pos = hm + R;
    int* h_utt = hm + 2 * R;
    {
        size_t k = 0;
        for (int b = 0; b < B; b++) {
            for (int t = 0; t < len[b]; t++, k++) {
                h_tok[off[b] + t] = tokens[k];
                h_pos[off[b] + t] = t;
                h_utt[off[b] + t] = b;
            }
            for (int g = 0; g < SEG_GAP; g++) {
                h_tok[off[b] + len[b] + g] = 0;
                h_pos[off[b] + len[b] + g] = -1;
                h_utt[off[b] + len[b] + g] = -1;
            }
        }
    }
    std::memcpy(hm + 3 * R, off.data(), (size_t)B * 4);
    std::memcpy(hm + 3 * R + B, len.data(), (size_t)B * 4);
    float* h_style = reinterpret_cast<float*>(hm + n_meta);
    std::memcpy(h_style, style, (size_t)B * 256 * 4);
    cudaStream_t st = c->fst;
    if (c->record) c->stages.clear();
    f.len0 = len[0];
    if (cudaMemcpyAsync(f.meta, hm, n_meta * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(f.style, h_style, (size_t)B * 256 * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return fail_cuda(RK_ERR_CUDA, (w + ": input upload").c_str());
    RowMeta m{f.meta, f.meta + R, f.meta + 2 * R, R};
    SegMeta seg{f.meta + 3 * R, f.meta + 3 * R + B, B, Tmax};
    s = enqueue_token_phase(c, m, seg, B);
    if (s) { cudaStreamSynchronize(st); return s; }
    // ---- predicted durations of the batch -> host (one read-back per batch)
    int* h_dur = hm;
    if (cudaMemcpyAsync(h_dur, f.dur_i, (size_t)R * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return fail_cuda(RK_ERR_CUDA, (w + ": duration read-back").c_str());
    const int bucket = c->l_bucket > 1 ? c->l_bucket : 1;
    std::vector<int> L(B), Lb(B);
    std::vector<int> use((size_t)R, 0);  // durations used (override or predicted), segmented layout
    int Lbmax = 0;
    {
        size_t k = 0;
        for (int b = 0; b < B; b++) {
            long long sum = 0;
            for (int t = 0; t < len[b]; t++, k++) {
                const int pred = h_dur[off[b] + t];
                const int u = dur_override ? dur_override[k] : pred;
                if (dur_out) dur_out[k] = pred;
                use[off[b] + t] = u;
                sum += u;
            }
            if (sum < 1 || sum > 64 * 1024) return bad("total duration out of range");
            L[b] = (int)sum;
            Lb[b] = (int)((sum + bucket - 1) / bucket * bucket);  // src/rokoko.cpp:797-802
            Lbmax = std::max(Lbmax, Lb[b]);
            if (L_out) L_out[b] = L[b];
        }
    }
    // segmented frame layout of the batch (64-aligned utterances, gap rows between)
    FrameLayout lay;
    const std::vector<int> tables = frame_layout_host(Lb, lay);
    const int F = lay.R;
    s = ensure_frames(c, F);
    if (!s) s = ensure_ig_op(c, (size_t)F, (size_t)F * 640 * 2);
    if (!s) s = ensure_pred(c, F, B);
    if (!s) s = ensure_decode_ws(c, Lbmax);
    if (!s) s = ensure_stage(c, (size_t)R * 4 * 2 + 2 * (size_t)B * 4 + tables.size() * 4);
    if (s) return s;
    hm = static_cast<int*>(c->h_stage);  // may have moved in ensure_stage: the durations were consumed
    // stash of the batch's decoder inputs: asr [F][512], f0 / n [2F], style [B][128]
    float* st_asr = stash_alloc(c, (size_t)F * 512 * 4);
    float* st_f0 = st_asr ? stash_alloc(c, (size_t)2 * F * 4) : nullptr;
    float* st_n = st_f0 ? stash_alloc(c, (size_t)2 * F * 4) : nullptr;
    float* st_style = st_n ? stash_alloc(c, (size_t)B * 128 * 4) : nullptr;
    if (!st_style) return fail(RK_ERR_OOM, (w + ": pending-utterance stash").c_str());
    int* h_use = hm + R;
    std::memcpy(h_use, use.data(), (size_t)R * 4);
    int* h_fseg = hm + 2 * R;
    std::memcpy(h_fseg, lay.off.data(), (size_t)B * 4);
    std::memcpy(h_fseg + B, Lb.data(), (size_t)B * 4);
    int* h_tab = h_fseg + 2 * B;
    std::memcpy(h_tab, tables.data(), tables.size() * 4);
    // dur_use goes where tok[] was (the token phase is done with it), frame segments after utt[]
    int* d_fseg = f.meta + 2 * R;
    if (cudaMemcpyAsync(f.meta, h_use, (size_t)R * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(d_fseg, h_fseg, (size_t)2 * B * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(f.layout, h_tab, tables.size() * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return fail_cuda(RK_ERR_CUDA, (w + ": duration upload").c_str());
    if ((!c->ev_stage && cudaEventCreateWithFlags(&c->ev_stage, cudaEventDisableTiming) != cudaSuccess) ||
        cudaEventRecord(c->ev_stage, st) != cudaSuccess)
        return fail_cuda(RK_ERR_CUDA, (w + ": staging event").c_str());
    frame_layout_device(f.layout, c->front.fc.rows, lay);
    SegMeta frames{d_fseg, d_fseg + B, B, Lbmax};
    s = enqueue_frame_phase(c, f.meta, seg, frames, F, st_asr);
    if (s) { cudaStreamSynchronize(st); return s; }
    {
        Run r{c, st, c->precision == RK_PRECISION_FP32};
        if (c->record) {
            std::vector<int> ft((size_t)Lb[0]);
            cudaStreamSynchronize(st);
            if (cudaMemcpy(ft.data(), f.frame_tok, (size_t)Lb[0] * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
                return fail_cuda(RK_ERR_CUDA, "stage copy");
            auto& sr = c->stages["frame_token"];
            sr.data.assign(ft.begin(), ft.end());
        }
        record(r, "shared", f.shared_all, (size_t)Lb[0] * 512);
        record(r, "asr_aligned", st_asr, (size_t)Lb[0] * 512);
        if (r.status) return r.status;
    }
    // ---- F0 / N chains of the whole batch, straight into the stash (x2 layout)
    s = enqueue_predict_batch(c, lay, st_f0, st_n);
    if (s) { cudaStreamSynchronize(st); return s; }
    {
        Run r{c, st, c->precision == RK_PRECISION_FP32};
        record(r, "f0_pred", st_f0, (size_t)2 * Lb[0]);
        record(r, "n_pred", st_n, (size_t)2 * Lb[0]);
        if (r.status) return r.status;
    }
    if (cudaMemcpy2DAsync(st_style, 128 * 4, f.style, 256 * 4, 128 * 4, B, cudaMemcpyDeviceToDevice, st) !=
        cudaSuccess)
        return fail_cuda(RK_ERR_CUDA, (w + ": style stash").c_str());
    std::vector<int> foff = lay.off;
    for (int b = 0; b < B; b++)
        c->pending.push_back({L[b], Lb[b], st_asr + (size_t)foff[b] * 512, st_f0 + (size_t)2 * foff[b],
                              st_n + (size_t)2 * foff[b], st_style + (size_t)b * 128});
    return RK_OK;
}

}  // namespace rk
