// ops.cuh -- bandwidth-bound kernels of the decoder / generator path.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace rk {

// Segmented rows (several utterances in one tensor): 64-row parts, part p of
// segment part_seg[p] (-1: a part of gap rows only) whose first part_rows[p]
// rows are valid; the others are gap rows between utterances.
struct SegRows {
    const int* part_seg = nullptr;
    const int* part_rows = nullptr;
};

// Segments of an AdaIN: segment u owns parts [p0[u], p0[u] + np[u]) of T[u]
// valid rows; its gamma / beta sit g_stride floats after segment u - 1's.
struct AdaSegs {
    const int* p0 = nullptr;
    const int* np = nullptr;
    const int* T = nullptr;
    int n = 0;
    int g_stride = 0;
};

// out[r] = W[r,:] . s + b[r]  for all style-FC rows of one style half.
void style_fc(const float* W, const float* b, const float* s, float* out, int rows, cudaStream_t st);
// The same for B style vectors s + u*s_stride: out[u*rows + r] (bit-identical per utterance).
void style_fc_batch(const float* W, const float* b, const float* s, int s_stride, int B, float* out, int rows,
                    cudaStream_t st);

// AdaIN coefficients from per-part column sums: stats[p*ld + c] (sums) and
// stats[(parts+p)*ld + c] (squares), c in [col0, col0+C).
//   mean = S/T, var = Q/T - mean^2, inv = 1/sqrt(var + 1e-5)
//   scale = (1+gamma) w inv;  shift = (1+gamma)(b - w mean inv) + beta
// written to coef[0..C) (scale) and coef[C..2C) (shift).
// With seg.p0 set: one coefficient set per segment, coef[u][2C] (scale then shift).
void adain_coef(const float* stats, int parts, int ld, int col0, int C, int T, const float* gamma,
                const float* beta, const float* norm_w, const float* norm_b, float* coef, cudaStream_t st,
                AdaSegs seg = AdaSegs{});

// Column sums / squares of x[T, ld] columns [col0, col0+ncols) over row blocks
// of `rows_per_part`, written as stats[p*ld + c] / stats[(parts+p)*ld + c].
// part_rows (nullable; rows_per_part 64): only the first part_rows[p] rows of part p are summed.
void col_stats(const float* x, int ld, int col0, int ncols, int T, int rows_per_part, float* stats,
               cudaStream_t st, const int* part_rows = nullptr);

// F0/N downsample Conv1d(1,1,K3,s2,p1) for both curves: y[t] = sum_k w[k] x[2t-1+k] + b.
void f0n_down(const float* f0, const float* n, const float* wf, const float* bf, const float* wn,
              const float* bn, float* f0d, float* nd, int L, cudaStream_t st);

// The same over the segmented rows of a batch (base layout R rows; F0 / N in the x2 layout).
void f0n_down_seg(const float* f0, const float* n, const float* wf, const float* bf, const float* wn,
                  const float* bn, float* f0d, float* nd, int R, SegRows sr, AdaSegs as, cudaStream_t st);

// dst[t, :] = [a[t, 0:ca] | b[t, 0:cb] | c[t] | d[t]] into columns [col0, ...) of a row of length ld.
void concat_cols(float* dst, int ld, int col0, int T, const float* a, int lda, int ca, const float* b, int ldb,
                 int cb, const float* c, const float* d, cudaStream_t st);

// AdainResBlk1d upsample path: a = lrelu(scale*x + shift, slope), then the
// depthwise ConvTranspose1d (K3, s2, p1, op1) with pool weights w[C][3] + b,
// written as conv operand planes [2T][Cp] (split bf16 or fp16).
// With sr set: x is a segmented layout, gap rows stay zero, coefficients per
// segment at scale + u * cstride (shift likewise).
void dw_upsample_pack(const float* x, int ldx, int T, int C, const float* scale, const float* shift, float slope,
                      const float* w, const float* b, void* hi, void* lo, int Cp, bool split, cudaStream_t st,
                      SegRows sr = SegRows{}, int cstride = 0);

// SineGen (phase scan, then per-sample source), STFT and iSTFT.
void sinegen_phase(const float* f0, int L2, float* phase_low, cudaStream_t st);
void sinegen_source(const float* phase_low, const float* f0, const float* lw, const float* lb, float* out, int L2,
                    cudaStream_t st);
void stft(const float* x, int T, float* har, int T2, cudaStream_t st);
void istft(const float* post, int T2, float* frames, float* y, int T_audio, cudaStream_t st);
// host-computed twiddles / window (double -> float once), uploaded to constant memory
cudaError_t upload_twiddles();

}  // namespace rk
