// g2p.h -- the neural phonemizer's weights and workspace inside an rk_ctx.
//
// Model (rokoko::G2PModelCuda, src/g2p.h:374-430): char embedding ->
// n_layers x (RMSNorm -> RoPE multi-head attention -> residual -> RMSNorm ->
// SwiGLU FFN -> residual) -> 3x upsample linear -> phone head -> CTC.
#pragma once
#include <cstdint>
#include <unordered_map>
#include <vector>

#include "model.h"

namespace rk {

struct G2PLayerW {
    float* n1 = nullptr;   // RMSNorm weights [d]
    float* n2 = nullptr;
    ConvW qkv;             // d -> 3d, bias
    ConvW out;             // d -> d, bias (residual in the epilogue)
    ConvW gate_up;         // d -> 2 ff: rows [gate | up], bias
    ConvW down;            // ff -> d, bias (residual in the epilogue)
};

struct G2PW {
    int d = 0, heads = 0, n_layers = 0, ff = 0, up = 0, n_chars = 0, n_phones = 0;
    float* emb = nullptr;        // [n_chars][d]
    float* rope_cos = nullptr;   // [2048][d / heads / 2]
    float* rope_sin = nullptr;
    std::vector<G2PLayerW> layers;
    ConvW upw;                   // d -> up d, bias: row t -> rows t up .. t up + up - 1
    ConvW head;                  // d -> n_phones, bias
    std::unordered_map<uint32_t, int> char2id;
    std::unordered_map<int, uint32_t> id2phone;
    void* base = nullptr;        // the one device allocation of the weights
    size_t bytes = 0;            // parameter bytes as the reference counts them (FP32)
};

struct G2PWS {
    int cap_R = 0, cap_n = 0;
    std::vector<void*> allocs;
    int32_t* meta = nullptr;     // ids [R] | pos [R] | seg off [n] | seg len [n]
    float* x = nullptr;          // [R][d] residual stream
    float* qkv = nullptr;        // [R][3d]
    float* ctx = nullptr;        // [R][d] attention output
    float* gu = nullptr;         // [R][2 ff] gate | up
    float* xu = nullptr;         // [R][up d] == [R up][d]
    float* logits = nullptr;     // [R up][n_phones]
    int32_t* best = nullptr;     // [R up] per-frame argmax
    Operand op;                  // 16-bit operand planes of the next linear
    void* h_stage = nullptr;     // pinned host staging (meta up, best down)
    size_t h_stage_bytes = 0;
    std::vector<int32_t> last_best;  // the last call's per-frame ids (rk_g2p_frames)
};

constexpr int G2P_MAX_POS = 2048;  // src/g2p.h:416 max_pos_: longest input in characters

struct G2PState {  // rk_ctx::g2p once rk_g2p_load succeeded
    G2PW w;
    G2PWS ws;
};

void free_g2p(rk_ctx* c);

}  // namespace rk
