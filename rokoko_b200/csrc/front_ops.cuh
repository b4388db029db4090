// front_ops.cuh -- front-half row kernels, attention, durations, alignment and
// the BiLSTM recurrence, over a batch of utterances.
//
// Token rows of a batch use a segmented layout: utterance b occupies rows
// [off_b, off_b + T_b) and is followed by SEG_GAP zero rows, so the K = 5
// text-encoder convolutions (padding 2) see zeros past each utterance's ends
// exactly as a single-utterance conv does.  Every row kernel writes zeros to
// the gap rows of its outputs and operand planes.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace rk {

constexpr int SEG_GAP = 2;  // zero rows after every utterance (text-encoder conv K 5, padding 2)

struct OpPlanes {  // destination operand planes [rows][Cp] (bf16 hi/lo or fp16 hi)
    void* hi;
    void* lo;
    int Cp;
};

// Per-row metadata of the segmented layout (device arrays of R entries).
struct RowMeta {
    const int* tok;  // token id (0 in gap rows)
    const int* pos;  // position within the utterance, -1 in gap rows
    const int* utt;  // utterance index, -1 in gap rows
    int R;
};

// Per-utterance segments (device arrays of n entries): rows [off, off + len).
struct SegMeta {
    const int* off;
    const int* len;
    int n;
    int max_len;
};

void embed_ln(RowMeta m, const float* word, const float* pos, const float* type, const float* g, const float* b,
              float* out, OpPlanes op, bool split, cudaStream_t st);
void res_ln(float* h, const float* a, RowMeta m, const float* g, const float* b, OpPlanes op, bool split,
            cudaStream_t st);
void ln_lrelu(const float* x, RowMeta m, const float* g, const float* b, float* out, OpPlanes op, bool split,
              cudaStream_t st);
// cat[r] = [x[r] (AdaLN'd with utterance u's gamma / beta when gamma_off >= 0) | style row u]:
// gamma = fc + u*fc_stride + gamma_off, beta = gamma + 512, style = style + u*style_stride.
void adaln_concat(const float* x, RowMeta m, const float* fc, int fc_stride, int gamma_off, const float* style,
                  int style_stride, float* cat, OpPlanes op, bool split, cudaStream_t st);
// Scaled dot-product attention (12 heads of 64, no mask) within every segment,
// on the tensor cores (attention_tc.cu): qkv [rows][2304] = [Q | K | V],
// ctx [rows][768]; split = FP32 semantics (split-bf16 products), else fp16.
// heads of 64 dimensions; QKV rows [3 * 64 heads], output rows [64 heads]
cudaError_t attention_tc(const float* qkv, SegMeta s, float* ctx, bool split, uint32_t* err, cudaStream_t st,
                         int heads = 12);
cudaError_t attention_tc_init();
void durations(const float* proj, RowMeta m, float* dur_f, int* dur_i, cudaStream_t st);
// Duration -> alignment for every utterance: a block-wide scan of its durations
// dur[tok.off .. +tok.len) gives token t's first frame; frame l < L of the
// utterance copies token row t(l) (cat -> en and its operand planes, te -> asr),
// frames [L, frames.len) are zero.  frame_tok[frames.off + l] = t(l) or -1.
void align_gather(const int* dur, SegMeta tok, SegMeta frames, const float* cat, const float* te, float* en,
                  float* asr, int* frame_tok, OpPlanes op, bool split, cudaStream_t st);
void rowdot(const float* x, int T, int C, const float* w, const float* b, float* y, cudaStream_t st);
void gather_rows(RowMeta m, const float* table, int D, float* out, OpPlanes op, bool split, cudaStream_t st);

// Bidirectional LSTM recurrence (src/rokoko.cpp:484-550, src/kernels.cu:976-997)
// for every sequence of `seq` at once, given precomputed input gates
// ig [rows][2048] (forward 0..1023 | reverse 1024..2047, bias included) and
// Whh [2][1024][256]: out[rows][512] = [h_fwd | h_rev] for the sequences' rows.
// One 8-CTA cluster per (group of up to `group` sequences, direction).
cudaError_t bilstm_recurrence(const float* ig, const float* whh, SegMeta seq, int group, float* out,
                              cudaStream_t st);
// Sequences per cluster for n sequences: enough to keep every cluster resident at once.
int bilstm_group(int n);
cudaError_t bilstm_init();

}  // namespace rk
