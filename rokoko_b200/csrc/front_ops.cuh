// front_ops.cuh -- front-half row kernels, attention, durations, alignment.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace rk {

struct OpPlanes {  // destination operand planes [rows][Cp] (bf16 hi/lo or fp16 hi)
    void* hi;
    void* lo;
    int Cp;
};

void embed_ln(const int* tok, int T, const float* word, const float* pos, const float* type, const float* g,
              const float* b, float* out, OpPlanes op, bool split, cudaStream_t st);
void res_ln(float* h, const float* a, int T, const float* g, const float* b, OpPlanes op, bool split,
            cudaStream_t st);
void ln_lrelu(const float* x, int T, const float* g, const float* b, float* out, OpPlanes op, bool split,
              cudaStream_t st);
void adaln_concat(const float* x, int T, const float* gamma, const float* beta, const float* style, float* cat,
                  OpPlanes op, bool split, cudaStream_t st);
void attention(const float* qkv, int T, float* ctx, cudaStream_t st);
void durations(const float* proj, int T, float* dur_f, int* dur_i, cudaStream_t st);
void align_gather(const int* dur, int T, int L_b, const float* cat, const float* te, float* en, float* asr,
                  OpPlanes op, bool split, cudaStream_t st);
void rowdot(const float* x, int T, int C, const float* w, const float* b, float* y, cudaStream_t st);
void gather_rows(const int* tok, int T, const float* table, int D, float* out, OpPlanes op, bool split,
                 cudaStream_t st);

// Bidirectional LSTM recurrence (src/rokoko.cpp:484-550, src/kernels.cu:976-997)
// given precomputed input gates ig [T][2048] (forward 0..1023 | reverse
// 1024..2047, bias included) and Whh [2][1024][256]: out [T][512] = [h_fwd | h_rev].
cudaError_t bilstm_recurrence(const float* ig, const float* whh, int T, float* out, uint32_t* err, cudaStream_t st);
cudaError_t bilstm_init();

}  // namespace rk
