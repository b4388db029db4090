// model.h -- device-side model state of one rk_ctx: packed weights, the
// decode workspace and the launch helpers shared by the forward passes.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <map>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/rk_b200.h"
#include "conv_tc.cuh"

namespace rk {

// A conv / linear weight packed for conv_tc: planes [phases*C_out][taps*Cp].
struct ConvW {
    int C_in = 0, C_out = 0, K = 0;     // logical shape
    int taps = 0, Cp = 0, phases = 1;   // packed shape
    int stride = 1;                     // >1: super-row layout (stride s, dilation 1)
    void* hi = nullptr;                 // bf16 (split) or fp16
    void* lo = nullptr;                 // bf16 lo plane (split only)
    float* bias = nullptr;              // [C_out] or null
    bool split = true;                  // planes are bf16 hi + lo (else one fp16 plane)
    CUtensorMap tm_hi{}, tm_lo{};
};

// AdaIN / InstanceNorm parameters: norm weight/bias and the row offset of its
// style-FC output (gamma = fc[off .. off+C), beta = fc[off+C .. off+2C)).
struct AdaINW {
    int C = 0;
    float* norm_w = nullptr;
    float* norm_b = nullptr;
    int fc_off = -1;  // row offset into the style-FC output of its group
};

struct ResBlk1dW {  // AdainResBlk1d
    int din = 0, dout = 0;
    bool shortcut = false, upsample = false;
    ConvW conv1, conv2, conv1x1;
    AdaINW norm1, norm2;
    float* pool_w = nullptr;  // depthwise ConvTranspose1d [din][3]
    float* pool_b = nullptr;
};

struct ResBlock1W {  // AdaINResBlock1
    int C = 0, K = 0;
    ConvW convs1[3], convs2[3];
    AdaINW adain1[3], adain2[3];
    float* alpha1[3] = {nullptr, nullptr, nullptr};
    float* alpha2[3] = {nullptr, nullptr, nullptr};
};

struct StyleFC {  // all style FCs driven by one half of the style vector
    int rows = 0;
    float* w = nullptr;  // [rows][128]
    float* b = nullptr;  // [rows]
    float* out = nullptr;  // [rows]
};

struct DecoderW {
    float* f0_conv_w = nullptr;  // [3]
    float* f0_conv_b = nullptr;
    float* n_conv_w = nullptr;
    float* n_conv_b = nullptr;
    ConvW asr_res;               // 512 -> 64, K=1
    ResBlk1dW encode, decode[4];
    ConvW ups[2];                // polyphase ConvTranspose1d
    ConvW noise_convs[2];        // [0]: super-row stride 6; [1]: K=1
    ResBlock1W noise_res[2], resblocks[6];
    ConvW conv_post;
    float* source_w = nullptr;   // m_source.l_linear [9]
    float* source_b = nullptr;   // [1]
    StyleFC fc;                  // acoustic-style FCs (decoder + generator)
};

struct LstmW {  // one bidirectional LSTM (src/weights.h:242-250)
    int in = 0;
    ConvW wih;              // [2048][in]: forward rows 0..1023, reverse 1024..2047; bias = bih + bhh
    float* whh = nullptr;   // [2][1024][256] recurrent weights (FP16-rounded values in FP16 semantics)
};

struct FrontW {  // ALBERT, text encoder and prosody predictor
    float *word = nullptr, *pos = nullptr, *type = nullptr, *emb_ln_w = nullptr, *emb_ln_b = nullptr;
    ConvW proj, qkv, dense, ffn, ffn_out, bert_enc;
    float *attn_ln_w = nullptr, *attn_ln_b = nullptr, *ffn_ln_w = nullptr, *ffn_ln_b = nullptr;
    float* te_embed = nullptr;  // [178][512]
    ConvW te_conv[3];
    float *te_ln_g[3] = {}, *te_ln_b[3] = {};
    LstmW te_lstm, dur_lstm[3], dur_final, shared;
    int aln_off[3] = {-1, -1, -1};  // AdaLayerNorm fc rows in the prosody style-FC group
    ConvW dur_proj;
    ResBlk1dW f0[3], nn[3];
    float *f0_proj_w = nullptr, *f0_proj_b = nullptr, *n_proj_w = nullptr, *n_proj_b = nullptr;
    StyleFC fc;  // prosody-style FCs (predictor)
};

struct Buf {  // device allocation tracked for the arena
    void* p = nullptr;
    size_t bytes = 0;
};

// Operand planes for conv_tc.
struct Operand {
    void* hi = nullptr;
    void* lo = nullptr;
    size_t plane_bytes = 0;  // capacity of one plane
};

// Buffers of one concurrent lane (one stream) of AdaINResBlock1 work.
struct Lane {
    cudaStream_t st = nullptr;
    float *xa = nullptr, *xb = nullptr, *co = nullptr, *out = nullptr;  // [T][C] fp32
    float *stats_a = nullptr, *stats_b = nullptr, *stats_c = nullptr;   // conv partials
    float* coef = nullptr;                                               // [2][C]
    Operand op;
};

// Workspace for one decode of up to `cap_L` frames.
struct DecodeWS {
    int cap_L = 0;
    std::vector<void*> allocs;
    // inputs
    float *asr = nullptr, *f0 = nullptr, *n = nullptr, *style = nullptr;
    // decoder
    float *f0d = nullptr, *nd = nullptr, *cat514 = nullptr, *asr_res = nullptr;
    float *in1090[4] = {nullptr, nullptr, nullptr, nullptr};
    float *enc_r1 = nullptr, *enc_sc = nullptr;
    float *stats_cat514 = nullptr, *stats_in[4] = {nullptr, nullptr, nullptr, nullptr};
    // generator
    float *gx = nullptr;                          // decoder output [2L][512]
    float *phase_low = nullptr, *har_src = nullptr, *har = nullptr;
    float *src = nullptr, *src2[2] = {nullptr, nullptr}, *stats_src = nullptr;
    float *u = nullptr, *stats_u = nullptr;
    float *avg = nullptr;                         // resblock average (only when recording)
    float *post = nullptr, *frames = nullptr, *audio = nullptr;
    Lane lane[3];                                 // resblocks j = 0, 1, 2 (lane 0 also runs the decoder)
    Lane noise;                                   // noise branch (side stream)
    Operand op_b;                                 // decoder shortcut operand / ups operand
    Operand op_har0, op_har1;
};

// Front-half workspace.  Three groups, each grown on demand:
//   rows    token rows of a batch in the segmented layout (front_ops.cuh):
//           cap_R rows, cap_B utterances;
//   frames  decoder frames of a batch in the segmented frame layout (utterance
//           b's L_b frames at a 64-aligned offset, gap rows between): cap_F
//           rows, plus the LSTM input-gate and operand buffers sized for both
//           row and frame phases;
//   pred    the batch's F0 / N chains over the same frames (and their x2
//           upsampled layout).
struct FrontWS {
    int cap_R = 0, cap_B = 0;
    std::vector<void*> row_allocs;
    int* meta = nullptr;  // tok[R] | pos[R] | utt[R] | seg_off[B] | seg_len[B] | dur_use[R] | f_off[B] | f_len[B]
    int* dur_i = nullptr;
    float *style = nullptr, *fc = nullptr, *dur_f = nullptr, *emb = nullptr, *h = nullptr, *qkv = nullptr,
          *ctx = nullptr, *tmp = nullptr, *ffmid = nullptr, *d_en = nullptr, *te = nullptr, *tbuf = nullptr,
          *cat = nullptr, *lstm_out = nullptr, *proj = nullptr;
    int cap_F = 0;
    std::vector<void*> frame_allocs;
    float *en = nullptr, *shared_all = nullptr;
    int* frame_tok = nullptr;
    size_t cap_ig = 0, cap_op = 0;  // rows of ig; bytes of one operand plane
    std::vector<void*> ig_allocs;
    float* ig = nullptr;            // [rows][2048] LSTM input gates
    Operand op;
    int len0 = 0;                   // token count of the batch's first utterance (stage capture)
    // the batched F0 / N chains over the segmented frame rows (capacity cap_Rp rows, cap_Bp utterances)
    int cap_Rp = 0, cap_Bp = 0;
    std::vector<void*> pred_allocs;
    float *x1 = nullptr, *x2 = nullptr, *x3 = nullptr, *r1 = nullptr, *sc = nullptr, *coef = nullptr,
          *stats = nullptr, *stats2 = nullptr, *stats_a = nullptr;
    int* layout = nullptr;  // segment tables of the frame layout (device)
    Operand op_p;
};

// The decoder blocks of a batch of pending utterances over their segmented
// frames (capacity cap_R rows, cap_B utterances); see seg.h.
struct DecBatchWS {
    int cap_R = 0, cap_B = 0;
    std::vector<void*> allocs;
    float *asr = nullptr, *f0 = nullptr, *n = nullptr, *style = nullptr, *fc = nullptr, *f0d = nullptr,
          *nd = nullptr, *cat514 = nullptr, *asr_res = nullptr, *gx = nullptr;
    float* in1090[4] = {nullptr, nullptr, nullptr, nullptr};
    float *stats_cat = nullptr, *stats_in[4] = {nullptr, nullptr, nullptr, nullptr};
    float *sc = nullptr, *r1 = nullptr, *coef = nullptr, *stats_a = nullptr;
    int* layout = nullptr;
    Operand op;
};

struct StageRec {  // captured stage activations (rk_record_stages)
    std::vector<float> data;
};

}  // namespace rk

namespace rk {
struct G2PState;  // g2p.h: the neural phonemizer of a context
}

// one timeline mark: the stream index and the launch name
struct TlMarkRec {
    int stream;
    std::string name;
};

struct rk_ctx {
    int device = 0;
    int precision = RK_PRECISION_FP32;
    int l_bucket = 32;
    int max_tokens = 512;
    cudaStream_t stream = nullptr;
    cudaStream_t side = nullptr;  // SineGen / STFT / noise branch
    cudaStream_t enc = nullptr;   // front half while a streaming call decodes the previous chunk
    cudaStream_t fst = nullptr;   // the stream the front half is enqueued on (stream or enc)
    cudaStream_t rb[2] = {nullptr, nullptr};  // resblock lanes 1 and 2
    // fork/join events: fork (main -> side), src[i] (side -> main, noise branch i
    // done), u (main -> resblock lanes), rb[j] (resblock lane j -> main)
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr, ev_src[2] = {nullptr, nullptr}, ev_u = nullptr,
                ev_rb[2] = {nullptr, nullptr};
    // AdainResBlk1d shortcut branch fork / join (main <-> resblock lane 1)
    cudaEvent_t ev_sc[2] = {nullptr, nullptr};
    bool use_graphs = true;
    uint32_t* err = nullptr;      // device error word
    // split-K scratch of the conv launcher, one per stream (main, side, rb[0], rb[1]):
    // convs that may run concurrently never share one
    static constexpr size_t kSplitKBytes = 16u << 20;
    float* splitk[4] = {nullptr, nullptr, nullptr, nullptr};
    bool loaded = false;
    std::vector<void*> weight_allocs;
    // the packed weights: one device allocation holding the whole weight image
    void* weights_base = nullptr;
    size_t weights_bytes = 0;
    rk::DecoderW dec;
    rk::FrontW front;
    bool has_front = false;
    rk::DecodeWS ws;
    rk::FrontWS fws;
    rk::DecBatchWS dws;
    bool record = false;
    std::map<std::string, rk::StageRec> stages;
    long long launches = 0;
    // decode graphs keyed by (L, profiling mode): the executable, the kernel
    // count it replays, and (profiling variant) the conv timing events it records
    struct GraphRec {
        cudaGraphExec_t exec = nullptr;
        long long launches = 0;
        size_t prof_events = 0;
        std::vector<double> prof_flops;
        std::vector<struct TlMarkRec> tl_marks;
    };
    std::map<std::pair<int, int>, GraphRec> graphs;
    // profiling (rk_profile): mode bits RK_PROFILE_*; event pairs around each conv launch
    bool profile = false;
    int prof_mode = 0;
    // timeline (RK_PROFILE_TIMELINE): one event after every launch, with its stream and name;
    // event 0 of a decode is the "start" mark on the context stream
    std::vector<cudaEvent_t> tl_events;
    using TlMark = TlMarkRec;
    std::vector<TlMark> tl_meta;
    std::vector<cudaEvent_t> prof_events;  // pool, 2 per launch
    size_t prof_used = 0;
    std::vector<double> prof_flops;        // algorithmic FLOPs of each timed launch
    double prof_ms_acc = 0.0, prof_flops_acc = 0.0;
    long long prof_launches_acc = 0;
    // utterances encoded by rk_encode and not yet decoded: their decoder inputs
    // (asr [L_b][512], f0 / n [2 L_b], style [128]) live in the stash chunks
    struct Pending {
        int L, L_b;
        float *asr, *f0, *n, *style;
    };
    std::vector<Pending> pending;
    struct StashChunk {
        char* base;
        size_t bytes, used;
        int pool;  // 0: rk_encode / rk_infer; 1, 2: alternate chunks of a streaming call
    };
    std::vector<StashChunk> stash;
    int stash_pool = 0;  // pool the next encode allocates from
    // pinned PCM of the chunks of a streaming call (double-buffered)
    float* h_pcm[2] = {nullptr, nullptr};
    size_t h_pcm_cap[2] = {0, 0};
    cudaEvent_t ev_chunk = nullptr;
    cudaEvent_t ev_enc[2] = {nullptr, nullptr};  // a streaming chunk's front half is done (on `enc`)
    // pinned host staging for the batch metadata upload and the duration read-back
    void* h_stage = nullptr;
    size_t h_stage_bytes = 0;
    cudaEvent_t ev_stage = nullptr;  // the last uploads out of h_stage are done
    // the neural phonemizer (rk_g2p_load), independent of the TTS weights
    rk::G2PState* g2p = nullptr;
};
