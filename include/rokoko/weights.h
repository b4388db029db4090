// weights.h -- source-compatible replacement for the reference's model seam,
// the declarations a caller of rokoko_infer compiles against
// (LokalOptima/rokoko src/weights.h:45-86 GpuArena, :372-384 Weights::load /
// free, :398-416 compute_decode_bytes, rokoko_infer, write_wav,
// precompute_weight_norms).  Code written against the reference's weights.h
// compiles unchanged with -I include/rokoko and links against
// librokoko_compat.so + librokoko_b200.so, which run the B200 kernels through
// the C ABI in ../rk_b200.h.
//
// Differences a caller can observe:
//   * Weights holds an rk_ctx instead of ~700 device pointers; Weights::load
//     picks the precision from the file (KOKO v1: FP32 semantics, v2: FP16
//     weights), as the reference picks it by which binary reads the file.
//   * rokoko_infer keeps its workspace inside the context: the arenas and the
//     workspace are accepted and left unused (a caller that sized them with
//     compute_decode_bytes keeps working), and `stream` is synchronised with the
//     context's stream before the call (work the caller queued there is visible).
//   * Errors throw std::runtime_error (rk_last_error's text) where the reference
//     prints and exits (src/weights.h:29-37).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <ostream>
#include <string>
#include <vector>

struct rk_ctx;

namespace rokoko {

// 256-byte-aligned bump allocator with the reference's interface (src/weights.h:45-86).
struct GpuArena {
    char* base = nullptr;
    size_t capacity = 0;
    size_t offset = 0;

    void init(size_t bytes);
    void destroy();
    void reset() { offset = 0; }
    void* alloc(size_t bytes);
    template <typename T>
    T* alloc(size_t count) {
        return static_cast<T*>(alloc(count * sizeof(T)));
    }
    size_t save() const { return offset; }
    void restore(size_t saved) { offset = saved; }
};

struct Weights {
    rk_ctx* ctx = nullptr;  // one B200 context holding the packed weights
    int version = 0;        // KOKO file version (1: fp32, 2: pre-baked fp16)
    int device = 0;

    // Reads a KOKO v1 or v2 file and uploads it to the current CUDA device.
    static Weights load(const std::string& path, cudaStream_t stream = nullptr);
    void free();
};

// Exact decode-arena bytes of the reference for T tokens and L frames.
size_t compute_decode_bytes(int T, int L);

// Phoneme token ids (host, incl. BOS = EOS = 0) + style vector (host [256]) -> PCM.
std::vector<float> rokoko_infer(const Weights& w, const int* token_ids, int T, const float* style_vec,
                                cudaStream_t stream, GpuArena& arena, GpuArena& decode_arena, float* d_workspace,
                                size_t workspace_bytes);

// Weight norms are folded into the packed weights when the file is loaded: a no-op kept for callers.
void precompute_weight_norms(Weights& w, cudaStream_t stream);

// 16-bit PCM WAV; path "-" writes to stdout.
bool write_wav(const std::string& path, const float* audio, int n_samples, int sample_rate);
void write_wav_to_(std::ostream& f, const float* audio, int n_samples, int sample_rate);

}  // namespace rokoko
