// g2p.h -- source-compatible replacement for the reference's neural
// phonemizer class (LokalOptima/rokoko src/g2p.h:374-430 G2PModelCuda: load,
// infer, free, loaded, param_bytes).  Code written against the reference's
// class compiles unchanged with -I include/rokoko and links against
// librokoko_compat.so + librokoko_b200.so, which run the model on the B200
// kernels through the C ABI in ../rk_b200.h (rk_g2p_*).
//
// Differences a caller can observe:
//   * the model lives in an rk_ctx of its own on the current CUDA device;
//     `stream` is synchronised before the model runs (work the caller queued
//     there is visible), and infer() returns after the result is on the host,
//     as the reference's does;
//   * infer_batch() phonemizes many texts in one device pass (not in the
//     reference);
//   * the computation has FP32 semantics (split-bf16 tensor-core products,
//     FP32 accumulate) where the reference uses TF32 GEMMs, so a frame whose
//     two best phones are within TF32 rounding of each other may resolve
//     differently.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <string>
#include <vector>

struct rk_ctx;

namespace rokoko {

struct G2PModelCuda {
    bool load(const char* path, cudaStream_t stream);
    std::string infer(const std::string& text, cudaStream_t stream) const;
    std::vector<std::string> infer_batch(const std::vector<std::string>& texts, cudaStream_t stream) const;
    void free();

    bool loaded() const { return loaded_; }
    size_t param_bytes() const;

    G2PModelCuda() = default;
    G2PModelCuda(const G2PModelCuda&) = delete;
    G2PModelCuda& operator=(const G2PModelCuda&) = delete;
    ~G2PModelCuda() { free(); }

private:
    rk_ctx* ctx_ = nullptr;
    bool loaded_ = false;
};

}  // namespace rokoko
