// api.cu -- rk_ctx lifecycle and the model-level C-ABI entry points.
//
// rk_decode_features* = the decode phase of rokoko_infer (src/rokoko.cpp:915-1290)
// on caller-given features; rk_infer adds the front half (src/rokoko.cpp:829-914).
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/rk_b200.h"
#include "decode.h"
#include "g2p.h"
#include "infer.h"
#include "model.h"
#include "status.h"
#include "weights.h"

using namespace rk;

namespace {

rk_status check_device_error(rk_ctx* c) {
    uint32_t e = 0;
    cudaError_t ce = cudaMemcpyAsync(&e, c->err, 4, cudaMemcpyDeviceToHost, c->stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(c->stream);
    if (ce != cudaSuccess) return fail_cuda_err(RK_ERR_CUDA, "device sync", ce);
    if (e) {
        cudaMemsetAsync(c->err, 0, 4, c->stream);
        std::string m = "a device-side wait gave up (code " + std::to_string(e) + ")";
        return fail(RK_ERR_DEVICE_TIMEOUT, m.c_str());
    }
    return RK_OK;
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" rk_status rk_create(int device, const rk_options* opts, rk_ctx** out) {
    if (!out) return fail(RK_ERR_CANNOT_IMPLEMENT, "rk_create: null out");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        return fail(RK_ERR_CUDA, "rk_create: no such CUDA device");
    }
    DeviceGuard g(device);
    rk_ctx* c = new rk_ctx();
    c->device = device;
    if (opts) {
        c->precision = opts->precision;
        if (opts->max_tokens > 0) c->max_tokens = opts->max_tokens;
        if (opts->l_bucket > 0) c->l_bucket = opts->l_bucket;
    }
    if (c->precision != RK_PRECISION_FP32 && c->precision != RK_PRECISION_FP16) {
        delete c;
        return fail(RK_ERR_CANNOT_IMPLEMENT, "rk_create: unknown precision");
    }
    if (c->max_tokens > 512) {
        delete c;
        return fail(RK_ERR_CANNOT_IMPLEMENT, "rk_create: max_tokens above 512 (ALBERT position table)");
    }
    bool ok = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&c->enc, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&c->rb[0], cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&c->rb[1], cudaStreamNonBlocking) == cudaSuccess;
    cudaEvent_t* evs[] = {&c->ev_fork, &c->ev_join, &c->ev_src[0], &c->ev_src[1], &c->ev_u, &c->ev_rb[0], &c->ev_rb[1],
                          &c->ev_sc[0], &c->ev_sc[1]};
    for (cudaEvent_t* e : evs) ok = ok && cudaEventCreateWithFlags(e, cudaEventDisableTiming) == cudaSuccess;
    ok = ok && cudaMalloc(&c->err, 256) == cudaSuccess && cudaMemset(c->err, 0, 256) == cudaSuccess;
    c->fst = c->stream;
    if (!ok) {
        rk_status s = fail_cuda(RK_ERR_CUDA, "rk_create");
        rk_destroy(c);
        return s;
    }
    *out = c;
    return RK_OK;
}

extern "C" void rk_destroy(rk_ctx* c) {
    if (!c) return;
    DeviceGuard g(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->side) cudaStreamSynchronize(c->side);
    c->pending.clear();
    free_decode_ws(c);
    free_decode_batch_ws(c);
    free_front_ws(c);
    free_weights(c);
    free_g2p(c);
    for (cudaEvent_t e : c->prof_events) cudaEventDestroy(e);
    for (cudaEvent_t e : c->tl_events) cudaEventDestroy(e);
    for (cudaEvent_t e : {c->ev_chunk, c->ev_enc[0], c->ev_enc[1], c->ev_stage})
        if (e) cudaEventDestroy(e);
    if (c->err) cudaFree(c->err);
    cudaEvent_t evs[] = {c->ev_fork, c->ev_join, c->ev_src[0], c->ev_src[1], c->ev_u, c->ev_rb[0], c->ev_rb[1],
                         c->ev_sc[0], c->ev_sc[1]};
    for (cudaEvent_t e : evs)
        if (e) cudaEventDestroy(e);
    for (cudaStream_t s : c->rb)
        if (s) { cudaStreamSynchronize(s); cudaStreamDestroy(s); }
    if (c->enc) { cudaStreamSynchronize(c->enc); cudaStreamDestroy(c->enc); }
    if (c->side) cudaStreamDestroy(c->side);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

extern "C" rk_status rk_load_weights_koko(rk_ctx* c, const void* blob, size_t bytes) {
    if (!c || !blob) return fail(RK_ERR_CANNOT_IMPLEMENT, "rk_load_weights_koko: null argument");
    DeviceGuard g(c->device);
    return load_weights(c, blob, bytes);
}

namespace {
rk_status decode_common(rk_ctx* c, int L) {
    if (!c->loaded) return fail(RK_ERR_STATE, "no weights loaded");
    if (L < 1 || L > 64 * 1024) return fail(RK_ERR_CANNOT_IMPLEMENT, "L out of range");
    return ensure_decode_ws(c, L);
}
}  // namespace

extern "C" rk_status rk_decode_features(rk_ctx* c, const float* asr, const float* f0, const float* n,
                                        const float* style128, int L, float* pcm) {
    if (!c || !asr || !f0 || !n || !style128 || !pcm) return fail(RK_ERR_CANNOT_IMPLEMENT, "null argument");
    DeviceGuard g(c->device);
    rk_status s = decode_common(c, L);
    if (s) return s;
    DecodeWS& w = c->ws;
    cudaStream_t st = c->stream;
    if (cudaMemcpyAsync(w.asr, asr, (size_t)L * 512 * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(w.f0, f0, (size_t)2 * L * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(w.n, n, (size_t)2 * L * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(w.style, style128, 128 * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return fail_cuda(RK_ERR_CUDA, "input upload");
    if (c->record) c->stages.clear();
    s = enqueue_decode(c, L);
    if (s) { cudaStreamSynchronize(st); cudaStreamSynchronize(c->side); return s; }
    if (cudaMemcpyAsync(pcm, w.audio, (size_t)600 * L * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return fail_cuda(RK_ERR_CUDA, "pcm download");
    return check_device_error(c);
}

extern "C" rk_status rk_decode_features_device(rk_ctx* c, const float* d_asr, const float* d_f0, const float* d_n,
                                               const float* d_style128, int L, float* d_pcm) {
    if (!c || !d_asr || !d_f0 || !d_n || !d_style128 || !d_pcm)
        return fail(RK_ERR_CANNOT_IMPLEMENT, "null argument");
    DeviceGuard g(c->device);
    rk_status s = decode_common(c, L);
    if (s) return s;
    DecodeWS& w = c->ws;
    cudaStream_t st = c->stream;
    if (cudaMemcpyAsync(w.asr, d_asr, (size_t)L * 512 * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(w.f0, d_f0, (size_t)2 * L * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(w.n, d_n, (size_t)2 * L * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(w.style, d_style128, 128 * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return fail_cuda(RK_ERR_CUDA, "input copy");
    s = enqueue_decode(c, L);
    if (s) return s;
    if (cudaMemcpyAsync(d_pcm, w.audio, (size_t)600 * L * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return fail_cuda(RK_ERR_CUDA, "pcm copy");
    return RK_OK;
}

extern "C" rk_status rk_record_stages(rk_ctx* c, int on) {
    if (!c) return fail(RK_ERR_CANNOT_IMPLEMENT, "null ctx");
    c->record = on != 0;
    c->stages.clear();
    return RK_OK;
}

extern "C" rk_status rk_get_stage(rk_ctx* c, const char* name, float* dst, size_t cap, size_t* count) {
    if (!c || !name) return fail(RK_ERR_CANNOT_IMPLEMENT, "null argument");
    auto it = c->stages.find(name);
    if (count) *count = it == c->stages.end() ? 0 : it->second.data.size();
    if (it != c->stages.end() && dst)
        std::memcpy(dst, it->second.data.data(), sizeof(float) * std::min(cap, it->second.data.size()));
    return RK_OK;
}

extern "C" rk_status rk_kernel_count(rk_ctx* c, long long* count, int reset) {
    if (!c) return fail(RK_ERR_CANNOT_IMPLEMENT, "null ctx");
    if (count) *count = c->launches;
    if (reset) c->launches = 0;
    return RK_OK;
}

extern "C" void* rk_stream(rk_ctx* c) { return c ? (void*)c->stream : nullptr; }

extern "C" rk_status rk_profile(rk_ctx* c, int on) {
    if (!c) return fail(RK_ERR_CANNOT_IMPLEMENT, "null ctx");
    if (on & ~(RK_PROFILE_CONV | RK_PROFILE_SERIAL | RK_PROFILE_TIMELINE))
        return fail(RK_ERR_CANNOT_IMPLEMENT, "rk_profile: unknown mode bits");
    c->profile = on != 0;
    c->prof_mode = on;
    c->tl_meta.clear();
    c->prof_used = 0;
    c->prof_flops.clear();
    c->prof_ms_acc = 0.0;
    c->prof_flops_acc = 0.0;
    c->prof_launches_acc = 0;
    return RK_OK;
}

extern "C" rk_status rk_profile_read(rk_ctx* c, double* conv_ms, double* conv_flops, long long* conv_launches) {
    if (!c) return fail(RK_ERR_CANNOT_IMPLEMENT, "null ctx");
    DeviceGuard g(c->device);
    if (cudaStreamSynchronize(c->stream) != cudaSuccess) return fail_cuda(RK_ERR_CUDA, "rk_profile_read sync");
    for (size_t i = 0; i + 1 < c->prof_used; i += 2) {
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, c->prof_events[i], c->prof_events[i + 1]) != cudaSuccess)
            return fail_cuda(RK_ERR_CUDA, "rk_profile_read elapsed");
        c->prof_ms_acc += ms;
        c->prof_flops_acc += c->prof_flops[i / 2];
        c->prof_launches_acc++;
    }
    c->prof_used = 0;
    c->prof_flops.clear();
    if (conv_ms) *conv_ms = c->prof_ms_acc;
    if (conv_flops) *conv_flops = c->prof_flops_acc;
    if (conv_launches) *conv_launches = c->prof_launches_acc;
    return RK_OK;
}

extern "C" rk_status rk_profile_timeline(rk_ctx* c, char* buf, size_t cap, size_t* len) {
    if (!c) return fail(RK_ERR_CANNOT_IMPLEMENT, "null ctx");
    DeviceGuard g(c->device);
    if (cudaDeviceSynchronize() != cudaSuccess) return fail_cuda(RK_ERR_CUDA, "rk_profile_timeline sync");
    std::string out;
    size_t base = 0;
    for (size_t i = 0; i < c->tl_meta.size(); i++) {
        if (c->tl_meta[i].name == "start") base = i;
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, c->tl_events[base], c->tl_events[i]) != cudaSuccess)
            return fail_cuda(RK_ERR_CUDA, "rk_profile_timeline elapsed");
        char line[160];
        snprintf(line, sizeof line, "%d\t%s\t%.4f\n", c->tl_meta[i].stream, c->tl_meta[i].name.c_str(), ms);
        out += line;
    }
    if (len) *len = out.size() + 1;
    if (buf && cap) {
        c->tl_meta.clear();
        const size_t n = out.size() < cap - 1 ? out.size() : cap - 1;
        memcpy(buf, out.data(), n);
        buf[n] = 0;
    }
    return RK_OK;
}

// Reference decode-arena size (src/rokoko_common.h:160-229), kept for API
// compatibility with callers that size their own arenas from it.
extern "C" size_t rk_compute_decode_bytes(int T, int L) {
    const size_t L2 = 2 * (size_t)L, TA = L2 * 300, hf = TA / 5 + 1;
    auto a = [](size_t off, size_t bytes) { return ((off + 255) & ~size_t(255)) + bytes; };
    size_t off = 0;
    off = a(off, 128 * 11 * hf * 4);
    off = a(off, (size_t)T * L * 4);
    off = a(off, (size_t)L * 640 * 4);
    off = a(off, (size_t)L * 512 * 4);
    off = a(off, 512 * L2 * 4);
    off = a(off, 512 * L2 * 4);
    off = a(off, 2048 * 4);
    off = a(off, L2 * 4);
    off = a(off, L2 * 4);
    off = a(off, (size_t)L * 512 * 4);
    off = a(off, (size_t)L * 4);
    off = a(off, (size_t)L * 4);
    off = a(off, (size_t)L * 514 * 4);
    off = a(off, 1090 * L2 * 4);
    off = a(off, 1090 * L2 * 4);
    off = a(off, 4 * 1090 * 4);
    off = a(off, (size_t)L * 1024 * 4);
    off = a(off, (size_t)L * 64 * 4);
    off = a(off, L2 * 1090 * 4);
    for (int i = 0; i < 3; i++) off = a(off, (size_t)L * 1024 * 4);
    off = a(off, L2 * 512 * 4);
    off = a(off, 22 * hf * 4);
    size_t sg = off;
    sg = a(sg, L2 * 9 * 4);
    sg = a(sg, TA * 4);
    sg = a(sg, 9 * 4);
    off = a(off, hf * 22 * 4);
    const size_t pool_end = a(off, 5 * 128 * hf * 4);
    off = sg > pool_end ? sg : pool_end;
    off = a(off, 512 * 4);
    off = a(off, TA * 4);
    return off;
}

namespace {

// Decoder + generator for pending utterances [first, first + n): the decoder
// blocks of up to kDecodeBatch of them per pass (decode_batch.cu), then each
// one's generator graph; PCM (600 L samples each) to pcm[i] (host, may be null).
constexpr int kDecodeBatch = 64;

rk_status decode_entries(rk_ctx* c, size_t first, int n, float* const* pcm) {
    for (int b0 = 0; b0 < n; b0 += kDecodeBatch) {
        const int nb = std::min(kDecodeBatch, n - b0);
        std::vector<PendingRef> refs(nb);
        for (int i = 0; i < nb; i++) {
            const rk_ctx::Pending& p = c->pending[first + b0 + i];
            refs[i] = PendingRef{p.L, p.L_b, p.asr, p.f0, p.n, p.style};
        }
        rk_status s = decode_batch(c, refs.data(), nb, pcm ? pcm + b0 : nullptr);
        if (s) return s;
    }
    return RK_OK;
}

void drop_pending(rk_ctx* c, size_t keep) {
    c->pending.resize(std::min(keep, c->pending.size()));
    if (c->pending.empty()) stash_reset(c, 0);
}

}  // namespace

extern "C" rk_status rk_infer(rk_ctx* c, const int32_t* tokens, int T, const float* style256,
                              const int32_t* dur_override, int32_t* dur_out, int* L_out, float* pcm,
                              size_t pcm_capacity, size_t* n_samples) {
    if (!c) return fail(RK_ERR_CANNOT_IMPLEMENT, "rk_infer: null argument");
    DeviceGuard g(c->device);
    const size_t before = c->pending.size();
    int32_t Tv = T, L = 0;
    rk_status s = encode_batch(c, tokens, &Tv, 1, style256, dur_override, dur_out, &L, "rk_infer");
    if (s) { cudaStreamSynchronize(c->stream); drop_pending(c, before); return s; }
    if (L_out) *L_out = L;
    const size_t n = std::min((size_t)600 * (size_t)L, pcm_capacity);
    std::vector<float> tmp;
    float* dst = pcm;
    if (pcm && n < (size_t)600 * L) { tmp.resize((size_t)600 * L); dst = tmp.data(); }
    s = decode_entries(c, c->pending.size() - 1, 1, &dst);
    if (!s) s = check_device_error(c);
    else cudaStreamSynchronize(c->stream);
    drop_pending(c, before);
    if (s) return s;
    if (pcm && dst != pcm) std::memcpy(pcm, dst, n * 4);
    if (n_samples) *n_samples = pcm ? n : 0;
    return RK_OK;
}

// ------------------------------------------------------------------ batched
// rk_encode runs the front half of B utterances in one pass (encode_batch)
// and keeps each one's decoder inputs (aligned features, F0, N, acoustic
// style) in the context's stash; rk_decode then runs the decoder for every
// pending utterance in order.

extern "C" rk_status rk_encode(rk_ctx* c, const int32_t* tokens, const int32_t* T_per_utt, int B,
                               const float* style, const int32_t* dur_override, int32_t* dur_out, int32_t* L_out) {
    if (!c || !tokens || !T_per_utt || !style || B < 1) return fail(RK_ERR_CANNOT_IMPLEMENT, "rk_encode: bad argument");
    DeviceGuard g(c->device);
    const size_t before = c->pending.size();
    rk_status s = encode_batch(c, tokens, T_per_utt, B, style, dur_override, dur_out, L_out, "rk_encode");
    if (!s) s = check_device_error(c);
    else cudaStreamSynchronize(c->stream);
    if (s) drop_pending(c, before);
    return s;
}

extern "C" rk_status rk_decode(rk_ctx* c, float* pcm, size_t pcm_capacity, size_t* n_samples, int* B_out) {
    if (!c) return fail(RK_ERR_CANNOT_IMPLEMENT, "rk_decode: null context");
    DeviceGuard g(c->device);
    const int B = (int)c->pending.size();
    if (B_out) *B_out = B;
    size_t need = 0;
    for (auto& p : c->pending) need += (size_t)600 * p.L;
    if (pcm && pcm_capacity < need) return fail(RK_ERR_WORKSPACE, "rk_decode: pcm buffer smaller than 600 * sum(L)");
    std::vector<float*> dst((size_t)B, nullptr);
    size_t off = 0;
    for (int b = 0; b < B; b++) {
        const size_t n = (size_t)600 * c->pending[b].L;
        if (pcm) dst[b] = pcm + off;
        if (n_samples) n_samples[b] = pcm ? n : 0;
        off += n;
    }
    rk_status s = decode_entries(c, 0, B, dst.data());
    cudaStreamSynchronize(c->stream);
    drop_pending(c, 0);
    return s ? s : check_device_error(c);
}

// ------------------------------------------------------------------ streaming
// rk_synthesize_stream: the utterances in chunks of `chunk`; chunk k's decodes
// are enqueued on the decode streams, then chunk k + 1's front half runs on
// the context's second stream (ctx->enc) while they execute, and the PCM of
// chunk k is handed to the callback utterance by utterance once it is in host
// memory.  Reference: TtsPipeline::synthesize_streaming (src/rokoko.h:298-360),
// which runs its chunks one after the other.

namespace {

struct FrontStream {  // the front half on ctx->enc for the scope of a streaming call
    rk_ctx* c;
    explicit FrontStream(rk_ctx* c_) : c(c_) { c->fst = c->enc; }
    ~FrontStream() { c->fst = c->stream; c->stash_pool = 0; }
};

rk_status ensure_pcm(rk_ctx* c, int i, size_t n) {
    if (c->h_pcm_cap[i] >= n) return RK_OK;
    if (c->h_pcm[i]) cudaFreeHost(c->h_pcm[i]);
    c->h_pcm[i] = nullptr;
    c->h_pcm_cap[i] = 0;
    n = std::max(n, (size_t)1 << 20);
    if (cudaHostAlloc(reinterpret_cast<void**>(&c->h_pcm[i]), n * 4, cudaHostAllocPortable) != cudaSuccess) {
        cudaGetLastError();
        return fail(RK_ERR_OOM, "rk_synthesize_stream: pinned PCM buffer");
    }
    c->h_pcm_cap[i] = n;
    return RK_OK;
}

}  // namespace

extern "C" rk_status rk_synthesize_stream(rk_ctx* c, const int32_t* tokens, const int32_t* T_per_utt, int B,
                                          const float* style, const int32_t* dur_override, int chunk,
                                          rk_pcm_fn on_pcm, void* user) {
    if (!c || !tokens || !T_per_utt || !style || B < 1 || chunk < 1 || !on_pcm)
        return fail(RK_ERR_CANNOT_IMPLEMENT, "rk_synthesize_stream: bad argument");
    if (!c->pending.empty())
        return fail(RK_ERR_STATE, "rk_synthesize_stream: utterances from rk_encode are still pending (rk_decode first)");
    DeviceGuard g(c->device);
    for (cudaEvent_t* e : {&c->ev_chunk, &c->ev_enc[0], &c->ev_enc[1]})
        if (!*e && cudaEventCreateWithFlags(e, cudaEventDisableTiming) != cudaSuccess)
            return fail_cuda(RK_ERR_CUDA, "rk_synthesize_stream: event");
    FrontStream fs(c);
    const int n_chunks = (B + chunk - 1) / chunk;
    std::vector<size_t> tok_off((size_t)B + 1, 0);
    for (int b = 0; b < B; b++) {
        if (T_per_utt[b] < 1) return fail(RK_ERR_CANNOT_IMPLEMENT, "rk_synthesize_stream: T out of range");
        tok_off[b + 1] = tok_off[b] + (size_t)T_per_utt[b];
    }
    auto encode_chunk = [&](int k) {
        const int b0 = k * chunk, nb = std::min(chunk, B - b0);
        c->stash_pool = 1 + (k & 1);
        stash_reset(c, c->stash_pool);  // chunk k - 2 of this pool has been decoded and handed out
        rk_status s = encode_batch(c, tokens + tok_off[b0], T_per_utt + b0, nb, style + (size_t)b0 * 256,
                                   dur_override ? dur_override + tok_off[b0] : nullptr, nullptr, nullptr,
                                   "rk_synthesize_stream");
        // encode_batch returns with the chunk's frame phase and F0 / N chains still queued on `enc`:
        // its decodes (on the context stream) wait for them
        if (!s && cudaEventRecord(c->ev_enc[k & 1], c->enc) != cudaSuccess)
            s = fail_cuda(RK_ERR_CUDA, "rk_synthesize_stream: event record");
        return s;
    };
    auto abort_all = [&](rk_status s) {
        cudaDeviceSynchronize();
        c->pending.clear();
        stash_reset(c, 1);
        stash_reset(c, 2);
        return s;
    };
    rk_status s = encode_chunk(0);
    if (s) return abort_all(s);
    for (int k = 0; k < n_chunks; k++) {
        const int b0 = k * chunk, nb = std::min(chunk, B - b0);
        // chunk k's entries are the first nb pending ones
        size_t total = 0;
        for (int i = 0; i < nb; i++) total += (size_t)600 * c->pending[i].L;
        const int pb = k & 1;
        if ((s = ensure_pcm(c, pb, total))) return abort_all(s);
        if (cudaStreamWaitEvent(c->stream, c->ev_enc[k & 1], 0) != cudaSuccess)
            return abort_all(fail_cuda(RK_ERR_CUDA, "rk_synthesize_stream: event wait"));
        std::vector<size_t> n_of(nb), at(nb);
        std::vector<float*> dst(nb);
        size_t off = 0;
        for (int i = 0; i < nb; i++) {
            at[i] = off;
            n_of[i] = (size_t)600 * c->pending[i].L;
            dst[i] = c->h_pcm[pb] + off;
            off += n_of[i];
        }
        if ((s = decode_entries(c, 0, nb, dst.data()))) return abort_all(s);
        if (cudaEventRecord(c->ev_chunk, c->stream) != cudaSuccess)
            return abort_all(fail_cuda(RK_ERR_CUDA, "rk_synthesize_stream: event record"));
        // the next chunk's front half overlaps this chunk's decode (its own stream, its own buffers)
        if (k + 1 < n_chunks && (s = encode_chunk(k + 1))) return abort_all(s);
        if (cudaEventSynchronize(c->ev_chunk) != cudaSuccess)
            return abort_all(fail_cuda(RK_ERR_CUDA, "rk_synthesize_stream: decode"));
        if ((s = check_device_error(c))) return abort_all(s);
        c->pending.erase(c->pending.begin(), c->pending.begin() + nb);
        for (int i = 0; i < nb; i++)
            if (!on_pcm(user, b0 + i, c->h_pcm[pb] + at[i], n_of[i])) return abort_all(RK_OK);  // caller stopped
    }
    return RK_OK;
}
