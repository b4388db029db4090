// tokens.h -- the reference's IPA -> model-input helpers (LokalOptima/rokoko
// src/rokoko.h:141-221: to_tokens, chunk_ipa, Chunk, MAX_IPA_CHARS) with the
// same signatures, implemented in librokoko_compat.so on rk_ipa_to_tokens /
// rk_ipa_chunks (../rk_b200.h).  The reference defines them inline in
// rokoko.h beside its server pipeline; a caller that only needs the text side
// includes this header instead.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace rokoko {

static constexpr int MAX_IPA_CHARS = 510;

struct Chunk {
    std::string phonemes;
    std::vector<int32_t> tokens;
};

std::vector<int32_t> to_tokens(const std::string& phonemes);
std::vector<Chunk> chunk_ipa(const std::string& ipa);

}  // namespace rokoko
