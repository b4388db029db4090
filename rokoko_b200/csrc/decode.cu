// decode.cu -- decoder + generator forward (the decode phase of rokoko_infer,
// src/rokoko.cpp:915-1290) on the tcgen05 conv and the bandwidth kernels.
//
// Dataflow per AdaIN'd conv: the producing conv's epilogue writes FP32 output
// plus per-channel partial sums -> adain_coef turns them into scale/shift ->
// pack_act applies AdaIN (+ Snake or LeakyReLU) and writes the next conv's
// 16-bit operand planes -> next conv.  Residual adds, bias, the reflection pad
// of ups[1], the `x += source` merge and the 1/sqrt(2) of AdainResBlk1d are
// folded into conv epilogues; the resblock average + LeakyReLU into the
// operand pack of the next conv.
//
// Concurrency (all joined back to the context stream, so the whole decode is
// one CUDA graph):
//   side stream : SineGen -> STFT -> noise_convs[0] -> noise_res[0] -> noise_convs[1] -> noise_res[1]
//                 (depends only on F0; overlaps the decoder blocks)
//   main stream : decoder blocks, ups[i], resblock 3i, average + pack
//   lanes 1, 2  : resblocks 3i+1, 3i+2 (independent of resblock 3i)
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>

#include "decode.h"
#include "exec.h"
#include "model.h"
#include "ops.cuh"
#include "pack.cuh"
#include "status.h"

namespace rk {



int stats_parts_for(const ConvCall& cc) { return conv_tc_stats_parts(cc.M, cc.w->phases); }

void tl_mark(rk_ctx* c, cudaStream_t st, const char* name) {
    if (!c->profile || !(c->prof_mode & RK_PROFILE_TIMELINE)) return;
    const size_t i = c->tl_meta.size();
    if (c->tl_events.size() <= i) {
        cudaEvent_t e;
        if (cudaEventCreate(&e) != cudaSuccess) { cudaGetLastError(); return; }
        c->tl_events.push_back(e);
    }
    int sid = 0;
    if (st == c->side) sid = 1;
    else if (st == c->rb[0]) sid = 2;
    else if (st == c->rb[1]) sid = 3;
    // external: inside a stream capture the record becomes an event node of the graph
    if (cudaEventRecordWithFlags(c->tl_events[i], st, cudaEventRecordExternal) != cudaSuccess) {
        cudaGetLastError();
        return;
    }
    c->tl_meta.push_back({sid, name});
}

void conv(Run& r, const ConvCall& cc) {
    if (!r.ok()) return;
    const ConvW& w = *cc.w;
    ConvOperands ops;
    if ((size_t)cc.rows_in * w.Cp * 2 > cc.op->plane_bytes) {
        r.status = fail(RK_ERR_WORKSPACE, "conv operand larger than its planes");
        return;
    }
    int toff[CONV_MAX_TAPS];
    for (int k = 0; k < w.taps; k++) toff[k] = w.phases > 1 ? -k : (w.stride > 1 ? k : k * cc.dil - cc.pad);
    ops.act_hi = cc.op->hi;
    ops.act_lo = cc.split ? cc.op->lo : nullptr;
    ops.act_rows = (uint64_t)cc.rows_in;
    ops.act_cp = (uint64_t)w.Cp;
    ops.w_hi = w.tm_hi;
    ops.w_lo = w.tm_lo;
    if (!cc.no_splitk) {  // the split-K scratch of this stream
        const cudaStream_t sts[4] = {r.c->stream, r.c->side, r.c->rb[0], r.c->rb[1]};
        for (int i = 0; i < 4; i++)
            if (r.st == sts[i]) { ops.scratch = r.c->splitk[i]; ops.scratch_bytes = rk_ctx::kSplitKBytes; }
    }
    ConvArgs a{};
    a.M = cc.M;
    a.C_out = w.C_out;
    a.kblocks = w.Cp / 64;
    a.taps = w.taps;
    for (int k = 0; k < w.taps; k++) a.tap_off[k] = toff[k];
    a.a_off = cc.a_off;
    a.b_phase_rows = w.phases > 1 ? w.C_out : 0;
    a.T_out = cc.T_out;
    a.o_min = cc.o_min;
    a.o_stride = cc.o_stride; a.o_off = cc.o_off; a.o_phase_step = cc.o_phase_step;
    a.y = cc.y; a.ldy = cc.ldy;
    a.bias = cc.use_bias ? w.bias : nullptr;
    a.res = cc.res; a.ldres = cc.ldres; a.res_shift = cc.res_shift;
    a.acc_in = cc.acc_in; a.ldacc = cc.ldacc;
    a.alpha = cc.alpha;
    a.act = cc.act;
    a.stats = cc.stats;
    a.stats_ld = cc.stats_ld ? cc.stats_ld : w.C_out;
    a.stats_parts = stats_parts_for(cc);
    a.dup_src_row = cc.dup_src_row;
    a.part_rows = cc.part_rows;
    a.err = r.c->err;
    rk_ctx* c = r.c;
    cudaEvent_t e1 = nullptr;
    if (c->profile && (c->prof_mode & RK_PROFILE_CONV)) {
        while (c->prof_events.size() < c->prof_used + 2) {
            cudaEvent_t evt;
            if (cudaEventCreate(&evt) != cudaSuccess) { r.status = fail_cuda(RK_ERR_CUDA, "profile event"); return; }
            c->prof_events.push_back(evt);
        }
        cudaEvent_t e0 = c->prof_events[c->prof_used];
        e1 = c->prof_events[c->prof_used + 1];
        c->prof_used += 2;
        // algorithmic FLOPs: 2 C_in C_out K T_out (ConvTranspose1d: x T_in)
        const double rows = w.phases > 1 ? (double)cc.rows_in : (double)cc.T_out;
        c->prof_flops.push_back(2.0 * w.C_in * w.C_out * w.K * rows);
        // external: inside a stream capture the record becomes an event node of the graph
        cudaEventRecordWithFlags(e0, r.st, cudaEventRecordExternal);
    }
    int nk = 0;
    cudaError_t e = conv_tc_launch(ops, a, cc.split, w.phases, r.st, &nk);
    if (e1) cudaEventRecordWithFlags(e1, r.st, cudaEventRecordExternal);
    r.c->launches += nk;
    if (c->profile && (c->prof_mode & RK_PROFILE_TIMELINE)) {
        // "conv C_in>C_out K d T_out [convT T_in] [res]": the shape a reader needs for the
        // conv's FLOPs and bytes (res: a residual tensor is read)
        char nm[96];
        int n = snprintf(nm, sizeof nm, "conv %d>%d K%d d%d T%d", w.C_in, w.C_out, w.K, cc.dil, cc.T_out);
        auto room = [&]() { n = n < 0 ? 0 : std::min(n, (int)sizeof nm - 1); return sizeof nm - (size_t)n; };
        if (w.phases > 1) { const size_t left = room(); n += snprintf(nm + n, left, " convT %d", cc.rows_in); }
        if (cc.res) { const size_t left = room(); snprintf(nm + n, left, " res"); }
        tl_mark(c, r.st, nm);
    }
    if (e != cudaSuccess) r.status = fail_cuda_err(RK_ERR_LAUNCH, "conv_tc", e);
}

void pack(Run& r, const float* x, int ldx, int rows, int C, const Operand& op, int Cp, bool split,
          const float* coef, const float* snake, float slope, bool lrelu, int sr_stride, int sr_pad, int rows_dst,
          SegRows sr, int coef_stride) {
    if (!r.ok()) return;
    PackArgs a{};
    a.part_seg = sr.part_seg;
    a.part_rows = sr.part_rows;
    a.coef_stride = coef_stride;
    a.x = x; a.ldx = ldx; a.rows_src = rows; a.C = C;
    a.rows_dst = rows_dst >= 0 ? rows_dst : rows;
    a.Cp = Cp; a.hi = op.hi; a.lo = op.lo;
    a.sr_stride = sr_stride; a.sr_pad = sr_pad;
    if (coef) { a.scale = coef; a.shift = coef + C; }
    a.snake = snake; a.slope = slope; a.lrelu = lrelu ? 1 : 0;
    if ((size_t)a.rows_dst * Cp * 2 > op.plane_bytes) {
        r.status = fail(RK_ERR_WORKSPACE, "operand plane too small");
        return;
    }
    cudaError_t e = pack_act(a, split, r.st);
    r.c->launches++;
    if (r.c->profile && (r.c->prof_mode & RK_PROFILE_TIMELINE)) {
        // "<kind> C R Cp Rd [split]": source channels and rows, operand columns and rows
        char nm[96];
        snprintf(nm, sizeof nm, "%s C%d R%d Cp%d Rd%d%s", coef ? (snake ? "pack_adain_snake" : "pack_adain_lrelu") : "pack",
                 C, rows, Cp, a.rows_dst, split ? " split" : "");
        tl_mark(r.c, r.st, nm);
    }
    if (e != cudaSuccess) r.status = fail_cuda_err(RK_ERR_LAUNCH, "pack_act", e);
}

void coef(Run& r, const float* stats, int parts, int ld, int col0, const AdaINW& n, int T, const StyleFC& fc,
          Lane& ln) {
    if (!r.ok()) return;
    adain_coef(stats, parts, ld, col0, n.C, T, fc.out + n.fc_off, fc.out + n.fc_off + n.C, n.norm_w, n.norm_b,
               ln.coef, r.st);
    r.check_launch("adain_coef");
}

// Stage capture (rk_record_stages): synchronous copies, never inside a graph.
void record(Run& r, const char* name, const float* d, size_t n) {
    if (!r.c->record || !r.ok()) return;
    auto& s = r.c->stages[name];
    s.data.resize(n);
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(s.data.data(), d, n * 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) r.status = fail_cuda_err(RK_ERR_CUDA, "stage copy", e);
}

// record the first C columns of a [rows][ld] buffer
void record_cols(Run& r, const char* name, const float* d, int rows, int ld, int C) {
    if (!r.c->record || !r.ok()) return;
    std::vector<float> full((size_t)rows * ld);
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(full.data(), d, full.size() * 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) { r.status = fail_cuda_err(RK_ERR_CUDA, "stage copy", e); return; }
    auto& s = r.c->stages[name];
    s.data.resize((size_t)rows * C);
    for (int t = 0; t < rows; t++) std::memcpy(&s.data[(size_t)t * C], &full[(size_t)t * ld], C * 4);
}

// AdainResBlk1d (src/rokoko.cpp:583-643) on the main lane.  x [T][ldx] (din
// channels) with partials stats_x (parts_x, pitch ldsx); y [T_out][ldy];
// stats_y (optional) partials of y with pitch ldsy.
void resblk1d(Run& r, const ResBlk1dW& b, const float* x, int ldx, const float* stats_x, int parts_x, int ldsx,
              int T, float* y, int ldy, float* stats_y, int ldsy, const StyleFC& fc) {
    DecodeWS& w = r.c->ws;
    Lane& ln = w.lane[0];
    const int To = b.upsample ? 2 * T : T;
    const bool sp = r.split;
    // shortcut: 1x1 conv at T rows (nearest upsample commutes with it), on
    // resblock lane 1 beside the main branch (it only needs x); joined before conv2
    const float* res = x;
    int ldres = ldx, shift = 0;
    const bool serial = r.c->profile && (r.c->prof_mode & RK_PROFILE_SERIAL);
    Run rs{r.c, serial ? r.st : r.c->rb[0], sp};
    if (b.shortcut) {
        if (!r.ok()) return;
        if (rs.st != r.st && (cudaEventRecord(r.c->ev_sc[0], r.st) != cudaSuccess ||
                              cudaStreamWaitEvent(rs.st, r.c->ev_sc[0], 0) != cudaSuccess)) {
            r.status = fail_cuda(RK_ERR_CUDA, "shortcut fork");
            return;
        }
        pack(rs, x, ldx, T, b.din, w.op_b, b.conv1x1.Cp, sp);
        ConvCall cs;
        cs.w = &b.conv1x1; cs.op = &w.op_b; cs.rows_in = T; cs.split = sp; cs.M = T; cs.T_out = T;
        cs.y = w.enc_sc; cs.ldy = b.dout; cs.use_bias = false;
        conv(rs, cs);
        res = w.enc_sc; ldres = b.dout; shift = b.upsample ? 1 : 0;
    }
    // norm1 -> LeakyReLU(0.2) [-> depthwise ConvTranspose upsample] -> operand
    coef(r, stats_x, parts_x, ldsx, 0, b.norm1, T, fc, ln);
    if (b.upsample) {
        if (!r.ok()) return;
        dw_upsample_pack(x, ldx, T, b.din, ln.coef, ln.coef + b.din, 0.2f, b.pool_w, b.pool_b, ln.op.hi, ln.op.lo,
                         b.conv1.Cp, sp, r.st);
        r.check_launch("dw_upsample_pack");
    } else {
        pack(r, x, ldx, T, b.din, ln.op, b.conv1.Cp, sp, ln.coef, nullptr, 0.2f, true);
    }
    ConvCall c1;
    c1.w = &b.conv1; c1.op = &ln.op; c1.rows_in = To; c1.split = sp; c1.M = To; c1.T_out = To; c1.pad = 1;
    c1.y = w.enc_r1; c1.ldy = b.dout; c1.stats = ln.stats_a; c1.stats_ld = b.dout;
    conv(r, c1);
    coef(r, ln.stats_a, stats_parts_for(c1), b.dout, 0, b.norm2, To, fc, ln);
    pack(r, w.enc_r1, b.dout, To, b.dout, ln.op, b.conv2.Cp, sp, ln.coef, nullptr, 0.2f, true);
    if (b.shortcut) {
        r.merge(rs);
        if (rs.st != r.st && r.ok() &&
            (cudaEventRecord(r.c->ev_sc[1], rs.st) != cudaSuccess ||
             cudaStreamWaitEvent(r.st, r.c->ev_sc[1], 0) != cudaSuccess))
            r.status = fail_cuda(RK_ERR_CUDA, "shortcut join");
    }
    // conv2 + shortcut + bias, times 1/sqrt(2)
    ConvCall c2;
    c2.w = &b.conv2; c2.op = &ln.op; c2.rows_in = To; c2.split = sp; c2.M = To; c2.T_out = To; c2.pad = 1;
    c2.y = y; c2.ldy = ldy; c2.res = res; c2.ldres = ldres; c2.res_shift = shift;
    c2.alpha = 1.0f / sqrtf(2.0f);
    c2.stats = stats_y; c2.stats_ld = ldsy;
    conv(r, c2);
}

// AdaINResBlock1 (src/rokoko.cpp:775-801) on lane `ln`: x0 [T][C] with
// partials sx0 (parts0 parts); dilation steps 0 and 1 (d = 1, 3) write
// ln.xa / ln.xb (with partials), step 2 (d = 5) writes `out`.
void resblock1(Run& r, Lane& ln, const ResBlock1W& rb, const float* x0, const float* sx0, int parts0, int T,
               float* out, const StyleFC& fc) {
    const int C = rb.C, K = rb.K;
    const int dil[3] = {1, 3, 5};
    const float* x = x0;
    const float* sx = sx0;
    const int parts = conv_tc_stats_parts(T, 1);
    int px = parts0;
    float* nxt[2] = {ln.xa, ln.xb};
    float* nst[2] = {ln.stats_b, ln.stats_c};
    for (int j = 0; j < 3; j++) {
        coef(r, sx, px, C, 0, rb.adain1[j], T, fc, ln);
        pack(r, x, C, T, C, ln.op, rb.convs1[j].Cp, r.split, ln.coef, rb.alpha1[j]);
        ConvCall c1;
        c1.w = &rb.convs1[j]; c1.op = &ln.op; c1.rows_in = T; c1.split = r.split; c1.M = T; c1.T_out = T;
        c1.dil = dil[j]; c1.pad = (K * dil[j] - dil[j]) / 2;
        c1.y = ln.co; c1.ldy = C; c1.stats = ln.stats_a; c1.stats_ld = C;
        conv(r, c1);
        coef(r, ln.stats_a, parts, C, 0, rb.adain2[j], T, fc, ln);
        pack(r, ln.co, C, T, C, ln.op, rb.convs2[j].Cp, r.split, ln.coef, rb.alpha2[j]);
        ConvCall c2;
        c2.w = &rb.convs2[j]; c2.op = &ln.op; c2.rows_in = T; c2.split = r.split; c2.M = T; c2.T_out = T;
        c2.pad = (K - 1) / 2;
        c2.res = x; c2.ldres = C;
        c2.y = j < 2 ? nxt[j] : out; c2.ldy = C;
        if (j < 2) { c2.stats = nst[j]; c2.stats_ld = C; }
        conv(r, c2);
        if (j < 2) { x = nxt[j]; sx = nst[j]; px = parts; }
    }
}

namespace {

bool ev(cudaError_t e) { return e == cudaSuccess; }

}  // namespace

// ---------------------------------------------------------------- workspace
static size_t al(size_t x) { return (x + 255) & ~size_t(255); }

void free_decode_ws(rk_ctx* c) {
    // a decode may still be in flight (streaming calls grow the workspace while one runs)
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second.exec);
    c->graphs.clear();
    for (void* p : c->ws.allocs) cudaFree(p);
    c->ws = DecodeWS{};
}

rk_status ensure_decode_ws(rk_ctx* c, int L) {
    if (c->ws.cap_L >= L) return RK_OK;
    free_decode_ws(c);
    DecodeWS& w = c->ws;
    const size_t L2 = 2 * (size_t)L, T1 = 20 * (size_t)L, T2 = 120 * (size_t)L + 1, TA = 600 * (size_t)L;
    const size_t gen = std::max(T1 * 256, T2 * 128);
    const size_t dec = L2 * 1024;
    const size_t parts = (T2 + STATS_ROWS - 1) / STATS_ROWS + 16;
    const size_t stats = 2 * parts * 1090;
    const size_t plane = std::max({T2 * 128, T1 * 256, L2 * 1152, L2 * 512}) * 2;
    struct Req { float** p; size_t n; };
    std::vector<Req> reqs = {
        {&w.asr, (size_t)L * 512}, {&w.f0, L2}, {&w.n, L2}, {&w.style, 128},
        {&w.f0d, (size_t)L}, {&w.nd, (size_t)L}, {&w.cat514, (size_t)L * 514}, {&w.asr_res, (size_t)L * 64},
        {&w.in1090[0], (size_t)L * 1090}, {&w.in1090[1], (size_t)L * 1090}, {&w.in1090[2], (size_t)L * 1090},
        {&w.in1090[3], (size_t)L * 1090}, {&w.enc_r1, dec}, {&w.enc_sc, dec},
        {&w.stats_cat514, stats}, {&w.stats_in[0], stats}, {&w.stats_in[1], stats}, {&w.stats_in[2], stats},
        {&w.stats_in[3], stats},
        {&w.gx, L2 * 512}, {&w.phase_low, L2 * 9}, {&w.har_src, TA}, {&w.har, T2 * 22},
        {&w.src, gen}, {&w.src2[0], T1 * 256}, {&w.src2[1], T2 * 128}, {&w.stats_src, stats},
        {&w.u, gen}, {&w.stats_u, stats}, {&w.avg, gen},
        {&w.post, T2 * 22}, {&w.frames, T2 * 20}, {&w.audio, TA},
    };
    Lane* lanes[4] = {&w.lane[0], &w.lane[1], &w.lane[2], &w.noise};
    for (Lane* ln : lanes) {
        reqs.push_back({&ln->xa, gen});
        reqs.push_back({&ln->xb, gen});
        reqs.push_back({&ln->co, gen});
        reqs.push_back({&ln->out, gen});
        reqs.push_back({&ln->stats_a, stats});
        reqs.push_back({&ln->stats_b, stats});
        reqs.push_back({&ln->stats_c, stats});
        reqs.push_back({&ln->coef, 2 * 1152});
    }
    size_t total = 0;
    for (auto& q : reqs) total += al(q.n * 4);
    std::vector<std::pair<Operand*, size_t>> ops = {{&w.op_b, al(plane)}, {&w.op_har0, al((T1 + 2) * 192 * 2)},
                                                    {&w.op_har1, al(T2 * 64 * 2)}};
    for (Lane* ln : lanes) ops.push_back({&ln->op, al(plane)});
    for (auto& o : ops) total += 2 * o.second;
    char* base = nullptr;
    if (cudaMalloc(&base, total) != cudaSuccess) {
        cudaGetLastError();
        return fail(RK_ERR_OOM, "decode workspace allocation");
    }
    w.allocs.push_back(base);
    size_t off = 0;
    for (auto& q : reqs) { *q.p = reinterpret_cast<float*>(base + off); off += al(q.n * 4); }
    for (auto& o : ops) {
        o.first->hi = base + off; off += o.second;
        o.first->lo = base + off; off += o.second;
        o.first->plane_bytes = o.second;
    }
    w.lane[0].st = c->stream;
    w.lane[1].st = c->rb[0];
    w.lane[2].st = c->rb[1];
    w.noise.st = c->side;
    w.cap_L = L;
    return RK_OK;
}

// ---------------------------------------------------------------- forward
// Inputs already in ws.asr [L][512], ws.f0 [2L], ws.n [2L], ws.style [128].
// gen_only: the decoder blocks ran elsewhere (the batched pass of rk_decode) and
// their output is already in ws.gx [2L][512]; the graph starts at the generator.
static rk_status enqueue_decode_body(rk_ctx* c, int L, bool gen_only) {
    DecodeWS& w = c->ws;
    const DecoderW& d = c->dec;
    const int L2 = 2 * L, T1 = 20 * L, T2 = 120 * L + 1, TA = 600 * L;
    const bool sp = c->precision == RK_PRECISION_FP32;
    // RK_PROFILE_SERIAL: every lane on the context stream
    const bool serial = c->profile && (c->prof_mode & RK_PROFILE_SERIAL);
    const cudaStream_t side = serial ? c->stream : c->side;
    const cudaStream_t lane1 = serial ? c->stream : c->rb[0], lane2 = serial ? c->stream : c->rb[1];
    Run r{c, c->stream, sp};
    Run s{c, side, sp};
    tl_mark(c, c->stream, "start");

    // style FCs first (the noise branch needs them too)
    style_fc(d.fc.w, d.fc.b, w.style, d.fc.out, d.fc.rows, r.st);
    r.check_launch("style_fc");
    if (!ev(cudaEventRecord(c->ev_fork, r.st)) || !ev(cudaStreamWaitEvent(side, c->ev_fork, 0)))
        return fail_cuda(RK_ERR_CUDA, "fork");

    // ---- side stream: SineGen -> STFT -> noise branches (depend on F0 only)
    sinegen_phase(w.f0, L2, w.phase_low, s.st);
    s.check_launch("sinegen_phase");
    sinegen_source(w.phase_low, w.f0, d.source_w, d.source_b, w.har_src, L2, s.st);
    s.check_launch("sinegen_source");
    stft(w.har_src, TA, w.har, T2, s.st);
    s.check_launch("stft");
    pack(s, w.har, 22, T2, 22, w.op_har0, d.noise_convs[0].Cp, sp, nullptr, nullptr, 0.f, false, 6, 3,
         T1 + d.noise_convs[0].taps - 1);
    pack(s, w.har, 22, T2, 22, w.op_har1, d.noise_convs[1].Cp, sp);
    for (int i = 0; i < 2; i++) {
        const int Co = i == 0 ? 256 : 128;
        const int Tn = i == 0 ? T1 : T2;
        ConvCall cn;
        cn.w = &d.noise_convs[i]; cn.split = sp; cn.y = w.src; cn.ldy = Co; cn.stats = w.stats_src; cn.stats_ld = Co;
        cn.M = Tn; cn.T_out = Tn;
        if (i == 0) { cn.op = &w.op_har0; cn.rows_in = T1 + d.noise_convs[0].taps - 1; }
        else { cn.op = &w.op_har1; cn.rows_in = T2; }
        conv(s, cn);
        resblock1(s, w.noise, d.noise_res[i], w.src, w.stats_src, stats_parts_for(cn), Tn, w.src2[i], d.fc);
        if (!ev(cudaEventRecord(c->ev_src[i], s.st))) return fail_cuda(RK_ERR_CUDA, "noise event");
    }
    if (!s.ok()) return s.status;

    // ---- decoder blocks (src/rokoko.cpp:921-990) on the main stream
    if (!gen_only) {
    f0n_down(w.f0, w.n, d.f0_conv_w, d.f0_conv_b, d.n_conv_w, d.n_conv_b, w.f0d, w.nd, L, r.st);
    r.check_launch("f0n_down");
    concat_cols(w.cat514, 514, 0, L, w.asr, 512, 512, nullptr, 0, 0, w.f0d, w.nd, r.st);
    r.check_launch("concat514");
    col_stats(w.cat514, 514, 0, 514, L, STATS_ROWS, w.stats_cat514, r.st);
    r.check_launch("col_stats");
    {  // asr_res: Conv1d 512 -> 64 (K1), FP32 semantics in both precisions
        pack(r, w.asr, 512, L, 512, w.op_b, d.asr_res.Cp, true);
        ConvCall ca;
        ca.w = &d.asr_res; ca.op = &w.op_b; ca.rows_in = L; ca.split = true; ca.M = L; ca.T_out = L;
        ca.y = w.asr_res; ca.ldy = 64;
        conv(r, ca);
    }
    const int parts_L = conv_tc_stats_parts(L, 1);
    for (int i = 0; i < 4; i++) {  // side channels of the decode-block inputs: [x | asr_res | F0d | Nd]
        concat_cols(w.in1090[i], 1090, 1024, L, w.asr_res, 64, 64, nullptr, 0, 0, w.f0d, w.nd, r.st);
        r.check_launch("concat_side");
        col_stats(w.in1090[i], 1090, 1024, 66, L, STATS_ROWS, w.stats_in[i], r.st);
        r.check_launch("col_stats");
    }
    resblk1d(r, d.encode, w.cat514, 514, w.stats_cat514, parts_L, 514, L, w.in1090[0], 1090, w.stats_in[0], 1090,
             d.fc);
    record_cols(r, "dec_encode", w.in1090[0], L, 1090, 1024);
    record(r, "asr_res", w.asr_res, (size_t)L * 64);
    for (int bi = 0; bi < 3; bi++)
        resblk1d(r, d.decode[bi], w.in1090[bi], 1090, w.stats_in[bi], parts_L, 1090, L, w.in1090[bi + 1], 1090,
                 w.stats_in[bi + 1], 1090, d.fc);
    resblk1d(r, d.decode[3], w.in1090[3], 1090, w.stats_in[3], parts_L, 1090, L, w.gx, 512, nullptr, 0, d.fc);
    record(r, "dec_decode3", w.gx, (size_t)L2 * 512);
    }
    // LeakyReLU(0.1) -> ups[0] operand
    pack(r, w.gx, 512, L2, 512, w.op_b, d.ups[0].Cp, sp, nullptr, nullptr, 0.1f, true);
    if (!r.ok()) return r.status;

    // ---- generator (src/rokoko.cpp:1030-1150)
    int Tl = L2;
    const int ur[2] = {10, 6}, ukk[2] = {20, 12};
    for (int i = 0; i < 2; i++) {
        const int Co = i == 0 ? 256 : 128;
        const int s_ = ur[i], p = (ukk[i] - ur[i]) / 2;
        const int Tu = (Tl - 1) * s_ - 2 * p + ukk[i] + (i == 1 ? 1 : 0);
        if (!ev(cudaStreamWaitEvent(r.st, c->ev_src[i], 0))) return fail_cuda(RK_ERR_CUDA, "join noise");
        record(r, i == 0 ? "gen0_src" : "gen1_src", w.src2[i], (size_t)Tu * Co);
        if (i == 0) {
            record(r, "har_source", w.har_src, TA);
            record(r, "har", w.har, (size_t)T2 * 22);
        }
        // ups: polyphase ConvTranspose1d + bias + noise source; stage 1 adds the
        // reflection pad (1, 0): convT row t -> row t + 1, row 0 = convT row 1
        ConvCall cu;
        cu.w = &d.ups[i]; cu.op = &w.op_b; cu.rows_in = Tl; cu.split = sp;
        const int shift = i == 1 ? 1 : 0;
        cu.M = Tl + 1; cu.T_out = Tu;  // q in [0, Tl]; out_row = q*s + r - p + shift
        cu.o_stride = s_; cu.o_off = -p + shift; cu.o_phase_step = 1;
        cu.y = w.u; cu.ldy = Co; cu.res = w.src2[i]; cu.ldres = Co;
        cu.stats = w.stats_u; cu.stats_ld = Co;
        cu.dup_src_row = i == 1 ? 2 : -1;
        cu.o_min = shift;  // row 0 of the padded output is only the duplicate
        conv(r, cu);
        const int parts_u = stats_parts_for(cu);
        record(r, i == 0 ? "gen0_ups" : "gen1_ups", w.u, (size_t)Tu * Co);
        // the three resblocks run concurrently on lanes 0, 1, 2
        if (!ev(cudaEventRecord(c->ev_u, r.st)) || !ev(cudaStreamWaitEvent(lane1, c->ev_u, 0)) ||
            !ev(cudaStreamWaitEvent(lane2, c->ev_u, 0)))
            return fail_cuda(RK_ERR_CUDA, "fork resblocks");
        Run lr[3] = {r, Run{c, lane1, sp}, Run{c, lane2, sp}};
        for (int j = 0; j < 3; j++)
            resblock1(lr[j], w.lane[j], d.resblocks[i * 3 + j], w.u, w.stats_u, parts_u, Tu, w.lane[j].out, d.fc);
        r = lr[0];
        r.merge(lr[1]);
        r.merge(lr[2]);
        for (int j = 0; j < 2; j++)
            if (!ev(cudaEventRecord(c->ev_rb[j], lr[j + 1].st)) || !ev(cudaStreamWaitEvent(r.st, c->ev_rb[j], 0)))
                return fail_cuda(RK_ERR_CUDA, "join resblocks");
        if (!r.ok()) return r.status;
        // ((rb0 + rb1) + rb2) / 3 -> LeakyReLU(0.1) -> ups[1] operand, or LeakyReLU(0.01) -> conv_post operand
        const ConvW& nextw = i == 0 ? d.ups[1] : d.conv_post;
        const Operand& nop = i == 0 ? w.op_b : w.lane[0].op;
        cudaError_t e = pack_avg3(w.lane[0].out, w.lane[1].out, w.lane[2].out, Tu, Co, nextw.Cp,
                                  i == 0 ? 0.1f : 0.01f, nop.hi, nop.lo, sp, c->record ? w.avg : nullptr, r.st);
        c->launches++;
        tl_mark(c, r.st, "pack_avg3");
        if (e != cudaSuccess) return fail_cuda_err(RK_ERR_LAUNCH, "pack_avg3", e);
        record(r, i == 0 ? "gen0_out" : "gen1_out", w.avg, (size_t)Tu * Co);
        Tl = Tu;
    }
    // conv_post (128 -> 22, K7, p3) -> iSTFT
    ConvCall cp;
    cp.w = &d.conv_post; cp.op = &w.lane[0].op; cp.rows_in = Tl; cp.split = sp; cp.M = Tl; cp.T_out = Tl;
    cp.pad = 3;
    cp.y = w.post; cp.ldy = 22;
    conv(r, cp);
    record(r, "conv_post", w.post, (size_t)Tl * 22);
    if (!r.ok()) return r.status;
    istft(w.post, T2, w.frames, w.audio, TA, r.st);
    r.check_launch("istft");
    c->launches++;  // istft is two kernels
    return r.status;
}

// One CUDA graph per L.  Stage recording runs the same launch sequence eagerly;
// a profiled decode (RK_PROFILE_CONV and / or RK_PROFILE_TIMELINE, optionally
// RK_PROFILE_SERIAL) is captured into its own graph whose timing events are
// event nodes, so that each replay re-records them.
rk_status enqueue_decode(rk_ctx* c, int L, bool gen_only) {
    const bool prof_graph = c->profile && (c->prof_mode & (RK_PROFILE_CONV | RK_PROFILE_TIMELINE));
    if (c->record || (c->profile && !prof_graph) || !c->use_graphs) return enqueue_decode_body(c, L, gen_only);
    const std::pair<int, int> key{L, (prof_graph ? c->prof_mode : 0) | (gen_only ? 0x100 : 0)};
    auto it = c->graphs.find(key);
    if (it == c->graphs.end()) {
        const long long before = c->launches;
        // conv timing events of a profiling capture start at the front of the pool
        const size_t used0 = c->prof_used;
        std::vector<double> flops0;
        std::vector<rk_ctx::TlMark> marks0;
        if (prof_graph) { flops0.swap(c->prof_flops); c->prof_used = 0; marks0.swap(c->tl_meta); }
        if (cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
            return fail_cuda(RK_ERR_CUDA, "graph capture begin");
        rk_status s = enqueue_decode_body(c, L, gen_only);
        cudaGraph_t g = nullptr;
        cudaError_t e = cudaStreamEndCapture(c->stream, &g);
        rk_ctx::GraphRec rec;
        if (prof_graph) {
            rec.prof_events = c->prof_used;
            rec.prof_flops.swap(c->prof_flops);
            rec.tl_marks.swap(c->tl_meta);
            c->prof_used = used0;
            c->prof_flops.swap(flops0);
            c->tl_meta.swap(marks0);
        }
        if (s != RK_OK) { if (g) cudaGraphDestroy(g); cudaGetLastError(); return s; }
        if (e != cudaSuccess) return fail_cuda_err(RK_ERR_CUDA, "graph capture end", e);
        e = cudaGraphInstantiateWithFlags(&rec.exec, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) return fail_cuda_err(RK_ERR_CUDA, "graph instantiate", e);
        rec.launches = c->launches - before;
        c->launches = before;
        it = c->graphs.emplace(key, std::move(rec)).first;
    }
    if (prof_graph) {
        // the replay re-records the graph's event pairs: earlier pairs must have been read
        if (c->prof_used != 0 || !c->tl_meta.empty())
            return fail(RK_ERR_STATE, "rk_profile_read / rk_profile_timeline must follow each profiled decode");
        c->prof_used = it->second.prof_events;
        c->prof_flops = it->second.prof_flops;
        c->tl_meta = it->second.tl_marks;
    }
    cudaError_t e = cudaGraphLaunch(it->second.exec, c->stream);
    if (e != cudaSuccess) return fail_cuda_err(RK_ERR_LAUNCH, "graph launch", e);
    c->launches += it->second.launches;
    return RK_OK;
}

}  // namespace rk
