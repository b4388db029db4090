// rokoko_compat.cpp -- the reference's C++ model seam (include/rokoko/weights.h)
// implemented on the C ABI of librokoko_b200.so: Weights::load ->
// rk_create + rk_load_weights_koko, rokoko_infer -> rk_infer (predicted
// durations, L bucketed by 32 as src/rokoko_f16.cpp:797-802 does); and the
// reference's phonemizer class (include/rokoko/g2p.h): G2PModelCuda::load ->
// rk_create + rk_g2p_load, infer -> rk_g2p_infer; and its IPA helpers
// (include/rokoko/tokens.h) on rk_ipa_to_tokens / rk_ipa_chunks.
#include "weights.h"
#include "g2p.h"
#include "tokens.h"

#include <cstdio>
#include <cstring>
#include <fstream>
#include <iostream>
#include <iterator>
#include <stdexcept>

#include "../rk_b200.h"

static_assert(sizeof(int) == sizeof(int32_t), "token ids are passed through as int32");

namespace rokoko {

namespace {

[[noreturn]] void raise(const std::string& what, rk_status s) {
    throw std::runtime_error(what + ": " + rk_status_string(s) + ": " + rk_last_error());
}

}  // namespace

void GpuArena::init(size_t bytes) {
    if (cudaMalloc(&base, bytes) != cudaSuccess) {
        cudaGetLastError();
        throw std::runtime_error("GpuArena::init: cudaMalloc failed");
    }
    capacity = bytes;
    offset = 0;
}

void GpuArena::destroy() {
    if (base) cudaFree(base);
    base = nullptr;
    capacity = 0;
    offset = 0;
}

void* GpuArena::alloc(size_t bytes) {
    const size_t aligned = (offset + 255) & ~size_t(255);
    if (aligned + bytes > capacity) throw std::runtime_error("GpuArena: out of arena memory");
    offset = aligned + bytes;
    return base + aligned;
}

Weights Weights::load(const std::string& path, cudaStream_t stream) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("Weights::load: cannot open " + path);
    std::vector<char> blob((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    if (blob.size() < 16) throw std::runtime_error("Weights::load: " + path + " is not a KOKO file");
    uint32_t version = 0;
    std::memcpy(&version, blob.data() + 4, 4);
    Weights w;
    w.version = (int)version;
    if (cudaGetDevice(&w.device) != cudaSuccess) {
        cudaGetLastError();
        throw std::runtime_error("Weights::load: no CUDA device");
    }
    if (stream && cudaStreamSynchronize(stream) != cudaSuccess) {
        cudaGetLastError();
        throw std::runtime_error("Weights::load: stream synchronisation failed");
    }
    rk_options o{version == 2 ? RK_PRECISION_FP16 : RK_PRECISION_FP32, 0, 0};
    rk_status s = rk_create(w.device, &o, &w.ctx);
    if (s) raise("Weights::load: rk_create", s);
    s = rk_load_weights_koko(w.ctx, blob.data(), blob.size());
    if (s) {
        rk_destroy(w.ctx);
        w.ctx = nullptr;
        raise("Weights::load: " + path, s);
    }
    return w;
}

void Weights::free() {
    if (ctx) rk_destroy(ctx);
    ctx = nullptr;
}

size_t compute_decode_bytes(int T, int L) { return rk_compute_decode_bytes(T, L); }

std::vector<float> rokoko_infer(const Weights& w, const int* token_ids, int T, const float* style_vec,
                                cudaStream_t stream, GpuArena& /*arena*/, GpuArena& /*decode_arena*/,
                                float* /*d_workspace*/, size_t /*workspace_bytes*/) {
    if (!w.ctx) throw std::runtime_error("rokoko_infer: weights not loaded");
    // work the caller queued on its stream comes first
    if (stream && cudaStreamSynchronize(stream) != cudaSuccess) {
        cudaGetLastError();
        throw std::runtime_error("rokoko_infer: stream synchronisation failed");
    }
    // front half (L known after the duration read-back), then the decoder into a buffer of 600 L samples
    const int32_t Tv = T;
    int32_t L = 0;
    rk_status s = rk_encode(w.ctx, reinterpret_cast<const int32_t*>(token_ids), &Tv, 1, style_vec, nullptr, nullptr,
                            &L);
    if (s) raise("rokoko_infer: front half", s);
    std::vector<float> pcm((size_t)600 * L);
    size_t n = 0;
    int B = 0;
    s = rk_decode(w.ctx, pcm.data(), pcm.size(), &n, &B);
    if (s) raise("rokoko_infer: decoder", s);
    pcm.resize(n);
    return pcm;
}

void precompute_weight_norms(Weights&, cudaStream_t) {}

void write_wav_to_(std::ostream& f, const float* audio, int n_samples, int sample_rate) {
    auto u32 = [&](uint32_t v) { f.write(reinterpret_cast<const char*>(&v), 4); };
    auto u16 = [&](uint16_t v) { f.write(reinterpret_cast<const char*>(&v), 2); };
    const uint32_t data = (uint32_t)n_samples * 2;
    f.write("RIFF", 4); u32(36 + data); f.write("WAVE", 4);
    f.write("fmt ", 4); u32(16); u16(1); u16(1); u32((uint32_t)sample_rate); u32((uint32_t)sample_rate * 2);
    u16(2); u16(16);
    f.write("data", 4); u32(data);
    for (int i = 0; i < n_samples; i++) {
        float v = audio[i] < -1.f ? -1.f : (audio[i] > 1.f ? 1.f : audio[i]);
        u16((uint16_t)(int16_t)(v * 32767.0f));
    }
}

bool write_wav(const std::string& path, const float* audio, int n_samples, int sample_rate) {
    if (path == "-") {
        write_wav_to_(std::cout, audio, n_samples, sample_rate);
        return (bool)std::cout;
    }
    std::ofstream f(path, std::ios::binary);
    if (!f) return false;
    write_wav_to_(f, audio, n_samples, sample_rate);
    return (bool)f;
}

// ------------------------------------------------------------------ G2PModelCuda

bool G2PModelCuda::load(const char* path, cudaStream_t stream) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    std::vector<char> blob((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    if (stream) cudaStreamSynchronize(stream);
    if (!ctx_) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return false;
        rk_options o{};
        o.precision = RK_PRECISION_FP32;
        if (rk_create(dev, &o, &ctx_) != RK_OK) {
            ctx_ = nullptr;
            return false;
        }
    }
    if (rk_g2p_load(ctx_, blob.data(), blob.size()) != RK_OK) {
        std::fprintf(stderr, "g2p: %s\n", rk_last_error());
        return loaded_;  // a model loaded before stays in place
    }
    loaded_ = true;
    return true;
}

std::vector<std::string> G2PModelCuda::infer_batch(const std::vector<std::string>& texts,
                                                   cudaStream_t stream) const {
    std::vector<std::string> res(texts.size());
    if (!loaded_ || texts.empty()) return res;
    if (stream) cudaStreamSynchronize(stream);
    const int n = (int)texts.size();
    std::vector<const char*> ptr(n);
    std::vector<size_t> len(n), out_len(n);
    size_t cap = 16;
    for (int i = 0; i < n; i++) {
        ptr[i] = texts[i].data();
        len[i] = texts[i].size();
        cap += 12 * texts[i].size();  // up to 3 phones of <= 4 bytes per input byte
    }
    std::vector<char> out(cap);
    rk_status s = rk_g2p_infer(ctx_, ptr.data(), len.data(), n, out.data(), out.size(), out_len.data());
    if (s == RK_ERR_WORKSPACE) {
        size_t need = 16;
        for (size_t l : out_len) need += l;
        out.resize(need);
        s = rk_g2p_infer(ctx_, ptr.data(), len.data(), n, out.data(), out.size(), out_len.data());
    }
    if (s != RK_OK) raise("G2PModelCuda::infer", s);
    size_t off = 0;
    for (int i = 0; i < n; i++) {
        res[i].assign(out.data() + off, out_len[i]);
        off += out_len[i];
    }
    return res;
}

std::string G2PModelCuda::infer(const std::string& text, cudaStream_t stream) const {
    if (!loaded_) return "";
    return infer_batch({text}, stream)[0];
}

void G2PModelCuda::free() {
    if (ctx_) rk_destroy(ctx_);
    ctx_ = nullptr;
    loaded_ = false;
}

size_t G2PModelCuda::param_bytes() const { return ctx_ ? rk_g2p_param_bytes(ctx_) : 0; }

// ------------------------------------------------------------------ IPA -> tokens

std::vector<int32_t> to_tokens(const std::string& phonemes) {
    size_t n = 0;
    rk_status s = rk_ipa_to_tokens(phonemes.data(), phonemes.size(), nullptr, 0, &n);
    if (s != RK_OK) raise("to_tokens", s);
    std::vector<int32_t> ids(n);
    s = rk_ipa_to_tokens(phonemes.data(), phonemes.size(), ids.data(), ids.size(), &n);
    if (s != RK_OK) raise("to_tokens", s);
    return ids;
}

std::vector<Chunk> chunk_ipa(const std::string& ipa) {
    size_t n = 0;
    rk_status s = rk_ipa_chunks(ipa.data(), ipa.size(), nullptr, 0, &n);
    if (s != RK_OK) raise("chunk_ipa", s);
    std::vector<size_t> ends(n);
    s = rk_ipa_chunks(ipa.data(), ipa.size(), ends.data(), ends.size(), &n);
    if (s != RK_OK) raise("chunk_ipa", s);
    std::vector<Chunk> out;
    size_t start = 0;
    for (size_t e : ends) {
        Chunk c;
        c.phonemes = ipa.substr(start, e - start);
        c.tokens = to_tokens(c.phonemes);
        out.push_back(std::move(c));
        start = e;
    }
    return out;
}

}  // namespace rokoko

