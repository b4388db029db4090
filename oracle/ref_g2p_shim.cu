// oracle/ref_g2p_shim.cu -- C-ABI wrapper of the reference's own neural
// phonemizer (rokoko::G2PModelCuda, src/g2p.h, with its CUTLASS GEMMs from
// src/cutlass_gemm.cu), compiled from the reference checkout into oracle/_ref/
// only.  TEST INFRASTRUCTURE: tests/golden/make_g2p_golden.py runs it on a
// B200 to record the reference's outputs for a seeded G2P3 file; nothing in
// the product links or loads it.
//
// Only the reference's first, uncaptured run per input length is used: a
// second call with the same length would capture a CUDA graph
// (src/g2p.h:846-859), so the shim refuses repeated lengths.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <set>
#include <string>
#include <unordered_map>
#include <vector>

#include <cuda_runtime.h>

// g2p.h logs through the vlog macro of src/weights.h
#define vlog(...) \
    do {          \
    } while (0)
// the per-frame argmax and logits live in the model's private workspace
#define private public
#include "g2p.h"
#undef private

namespace {

struct Holder {
    rokoko::G2PModelCuda model;
    cudaStream_t stream = nullptr;
    std::set<int> seen;
};

int count_codepoints(const char* s, size_t n) {  // the lead-byte rule of src/g2p.h:682-694
    const uint8_t* p = (const uint8_t*)s;
    const uint8_t* end = p + n;
    int T = 0;
    while (p < end) {
        int len = *p < 0x80 ? 1 : (*p & 0xE0) == 0xC0 ? 2 : (*p & 0xF0) == 0xE0 ? 3 : 4;
        p += len;
        if (p > end) p = end;
        T++;
    }
    return T;
}

}  // namespace

extern "C" {

void* ref_g2p_load(const char* path) {
    Holder* h = new Holder;
    if (cudaStreamCreate(&h->stream) != cudaSuccess || !h->model.load(path, h->stream)) {
        if (h->stream) cudaStreamDestroy(h->stream);
        delete h;
        return nullptr;
    }
    return h;
}

void ref_g2p_free(void* p) {
    Holder* h = static_cast<Holder*>(p);
    h->model.free();
    cudaStreamDestroy(h->stream);
    delete h;
}

// Runs the reference's infer() once for a new input length.  Writes the UTF-8
// phones (returns their length), the per-frame argmax [T*up] into best and the
// logits [T*up][n_phones] into logits (either may be null).  Returns -2 for a
// repeated length, -1 when a buffer is short.
long ref_g2p_infer(void* p, const char* text, size_t n, char* out, size_t cap, int32_t* best, size_t best_cap,
                   float* logits, size_t logits_cap) {
    Holder* h = static_cast<Holder*>(p);
    const int T = count_codepoints(text, n);
    if (T > 0 && !h->seen.insert(T).second) return -2;
    const std::string r = h->model.infer(std::string(text, n), h->stream);
    if (r.size() > cap) return -1;
    std::memcpy(out, r.data(), r.size());
    const rokoko::G2PModelCuda& m = h->model;
    if (T > 0 && T <= m.max_pos_) {
        // the workspace slices of infer() (src/g2p.h:700-740), in order, 256-byte aligned
        const int d = m.d_, hh = m.heads_, ff = m.ff_, up = m.up_, np_ = m.n_phones_, Tu = T * up;
        uintptr_t w = (uintptr_t)m.workspace_;
        auto take = [&](size_t bytes) {
            w = (w + 255) & ~(uintptr_t)255;
            const uintptr_t at = w;
            w += bytes;
            return at;
        };
        take((size_t)T * 4);                    // ids
        take((size_t)T * d * 4);                // X
        take((size_t)T * 3 * d * 4);            // QKV
        take((size_t)hh * T * T * 4);           // scores
        take((size_t)T * d * 4);                // attn_out
        take((size_t)T * d * 4);                // normed
        take((size_t)T * 2 * ff * 4);           // ffn_out
        take((size_t)T * d * up * 4);           // X_up_proj
        take((size_t)Tu * d * 4);               // X_up
        const uintptr_t lg = take((size_t)Tu * np_ * 4);
        const uintptr_t am = take((size_t)Tu * 4);
        if (best) {
            if ((size_t)Tu > best_cap) return -1;
            cudaMemcpy(best, (const void*)am, (size_t)Tu * 4, cudaMemcpyDeviceToHost);
        }
        if (logits) {
            if ((size_t)Tu * np_ > logits_cap) return -1;
            // the reference adds the head bias inside its argmax kernel, not to the stored logits
            cudaMemcpy(logits, (const void*)lg, (size_t)Tu * np_ * 4, cudaMemcpyDeviceToHost);
        }
    }
    return (long)r.size();
}

}  // extern "C"
