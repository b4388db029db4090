// weights.h -- KOKO file parsing and the weight loader entry points.
#pragma once
#include <cstdint>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/rk_b200.h"

struct rk_ctx;

namespace rk {

struct WeightError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

struct KTensor {
    std::string dtype;
    std::vector<int> shape;
    const uint8_t* data = nullptr;
    size_t bytes = 0;
};

// Parsed view of a KOKO blob (no copies; points into the caller's bytes).
struct KokoFile {
    uint32_t version = 0;
    std::unordered_map<std::string, KTensor> tensors;
    bool parse(const uint8_t* blob, size_t n, std::string& err);
    const KTensor* find(const std::string& name) const;
    std::vector<float> f32(const std::string& name) const;  // fp32 or fp16 -> float
};

// Host image of the packed weights: 256-byte aligned slices; put() returns the
// slice's offset tagged as a pointer (relocated when the image is uploaded).
struct Image {
    std::vector<uint8_t> bytes;
    void* put(const void* h, size_t n);
};

// KOKO v1 / v2 (packed on the host, uploaded as one image) or v3 (the image itself).
rk_status load_weights(rk_ctx* c, const void* blob, size_t bytes);
void free_weights(rk_ctx* c);

}  // namespace rk
