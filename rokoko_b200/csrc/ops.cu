// ops.cu -- bandwidth-bound kernels of the decoder / generator.
//
// Reference semantics (src/kernels.cu):
//   AdaIN statistics + affine     :413-504  (here: stats come from the conv
//                                   epilogue; this file turns them into
//                                   per-channel scale/shift)
//   depthwise ConvTranspose1d     :557-594  (fused with AdaIN + LeakyReLU and the
//                                   operand cast of the next conv)
//   strided conv F0/N down        :712-746
//   SineGen phase / source        :1337-1452
//   STFT / iSTFT                  :819-970  (twiddle tables, gather-form
//                                   overlap-add without atomics)
// Float operations that must match the CPU restatement bit-for-bit (SineGen
// phases, STFT sums) use explicit __fadd_rn / __fmul_rn so the compiler cannot
// contract them into FMAs.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cmath>

#include "ops.cuh"

namespace rk {

namespace {

__constant__ float c_cos[11][20];
__constant__ float c_sin[11][20];
__constant__ float c_win[20];

int nblocks(long work, int threads, int cap = 148 * 16) {
    long b = (work + threads - 1) / threads;
    if (b > cap) b = cap;
    return (int)(b < 1 ? 1 : b);
}

// segment of row r of a segmented layout, -1 for a gap row
__device__ __forceinline__ int seg_of_row(const SegRows& sr, int r) {
    const int p = r >> 6;
    return (r & 63) < sr.part_rows[p] ? sr.part_seg[p] : -1;
}

// element counts for which a 32-bit grid-stride index cannot overflow
bool small_index(long total) { return total < (1L << 31) - 148L * 16 * 1024; }

// one warp per (style-FC row, utterance blockIdx.y)
__global__ void style_fc_kernel(const float* __restrict__ W, const float* __restrict__ b,
                                const float* __restrict__ s_all, int s_stride, float* __restrict__ out_all,
                                int rows) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float* s = s_all + (size_t)blockIdx.y * s_stride;
    float* out = out_all + (size_t)blockIdx.y * rows;
    const float* w = W + (size_t)warp * 128;
    float acc = 0.f;
#pragma unroll
    for (int k = lane; k < 128; k += 32) acc += w[k] * s[k];
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) out[warp] = acc + b[warp];
}

// AdaIN coefficients from the InstanceNorm partials: block = 8 channels x 128
// part slices; slice y sums parts y, y + 128, ... in double (eight loads of
// each kind in flight together), then a fixed-order halving tree over the
// slices.  mean = S / T, var = Q / T - mean^2 (biased, the reference's
// single-pass form), scale = (1 + gamma) w / sqrt(var + 1e-5),
// shift = (1 + gamma)(b - w mean / sqrt(var + eps)) + beta.
// Segmented form (seg != null): blockIdx.y = segment u, which owns parts
// [seg.p0[u], seg.p0[u] + seg.np[u]) of rows seg.T[u]; its gamma / beta are
// offset by u * seg.g_stride and its coefficients by u * 2C; the squares of the
// statistics sit `parts` (all parts of the array) after the sums.
__global__ void __launch_bounds__(1024) adain_coef_kernel(const float* __restrict__ stats, int parts, int ld,
                                                          int col0, int C, int T, const float* __restrict__ gamma,
                                                          const float* __restrict__ beta,
                                                          const float* __restrict__ nw,
                                                          const float* __restrict__ nb, float* __restrict__ coef,
                                                          AdaSegs seg) {
    __shared__ double sh_s[128][8], sh_q[128][8];
    const int cx = threadIdx.x, py = threadIdx.y;
    const int c = blockIdx.x * 8 + cx;
    int pbase = 0, np = parts;
    if (seg.p0) {
        const int u = blockIdx.y;
        pbase = seg.p0[u];
        np = seg.np[u];
        T = seg.T[u];
        gamma += (size_t)u * seg.g_stride;
        beta += (size_t)u * seg.g_stride;
        coef += (size_t)u * 2 * C;
    }
    double s = 0.0, q = 0.0;
    if (c < C && np > 0) {
        // eight parts per slice in flight at once: addresses clamped to the last
        // part, the sums predicated (parts ascending, as a serial loop would add them)
        for (int p0 = py; p0 < np; p0 += 8 * 128) {
            float sv[8], qv[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int pc = pbase + min(p0 + u * 128, np - 1);
                sv[u] = stats[(size_t)pc * ld + col0 + c];
                qv[u] = stats[(size_t)(parts + pc) * ld + col0 + c];
            }
#pragma unroll
            for (int u = 0; u < 8; u++)
                if (p0 + u * 128 < np) {
                    s += sv[u];
                    q += qv[u];
                }
        }
    }
    sh_s[py][cx] = s;
    sh_q[py][cx] = q;
    __syncthreads();
    for (int o = 64; o >= 1; o >>= 1) {
        if (py < o) {
            sh_s[py][cx] += sh_s[py + o][cx];
            sh_q[py][cx] += sh_q[py + o][cx];
        }
        __syncthreads();
    }
    if (py != 0 || c >= C || T < 1) return;
    const double mean_d = sh_s[0][cx] / T;
    const double var_d = sh_q[0][cx] / T - mean_d * mean_d;
    const float mean = (float)mean_d;
    const float inv_std = (float)(1.0 / sqrt(var_d + 1e-5));
    const float g = 1.0f + gamma[c];
    coef[c] = g * nw[c] * inv_std;
    coef[C + c] = g * (nb[c] - nw[c] * mean * inv_std) + beta[c];
}

// Column sum / sum-of-squares partials per part of rows_per_part rows.  Block
// = 32 columns x 8 row slices; slice y sums rows y, y + 8, ... of the part
// (loads independent and in flight together), then slice 0 adds the eight
// slice sums in order.
__global__ void __launch_bounds__(256) col_stats_kernel(const float* __restrict__ x, int ld, int col0, int ncols,
                                                        int T, int rows_per_part, int parts,
                                                        float* __restrict__ stats, const int* __restrict__ part_rows) {
    __shared__ float sh_s[8][32], sh_q[8][32];
    const int cx = threadIdx.x, sy = threadIdx.y;
    const int c = blockIdx.x * 32 + cx;
    const int p = blockIdx.y;
    const int r0 = p * rows_per_part;
    const int r1 = part_rows ? r0 + part_rows[p] : min(T, r0 + rows_per_part);
    float s = 0.f, q = 0.f;
    if (c < ncols) {
#pragma unroll 4
        for (int r = r0 + sy; r < r1; r += 8) {
            const float v = x[(size_t)r * ld + col0 + c];
            s += v;
            q += v * v;
        }
    }
    sh_s[sy][cx] = s;
    sh_q[sy][cx] = q;
    __syncthreads();
    if (sy != 0 || c >= ncols) return;
    float ts = 0.f, tq = 0.f;
#pragma unroll
    for (int k = 0; k < 8; k++) { ts += sh_s[k][cx]; tq += sh_q[k][cx]; }
    stats[(size_t)p * ld + col0 + c] = ts;
    stats[(size_t)(parts + p) * ld + col0 + c] = tq;
}

__global__ void f0n_down_kernel(const float* __restrict__ f0, const float* __restrict__ n,
                                const float* __restrict__ wf, const float* __restrict__ bf,
                                const float* __restrict__ wn, const float* __restrict__ bn, float* f0d, float* nd,
                                int L) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= L) return;
    float a = 0.f, b = 0.f;
    for (int k = 0; k < 3; k++) {
        const int ti = 2 * t - 1 + k;
        if (ti >= 0 && ti < 2 * L) {
            a += wf[k] * f0[ti];
            b += wn[k] * n[ti];
        }
    }
    f0d[t] = a + bf[0];
    nd[t] = b + bn[0];
}

// Segmented form over the rows of a batch: row r of utterance u (base layout,
// offset off_u = 64 * p0[u]) reads F0 / N at x2 rows [2 off_u, 2 off_u + 2 n_u);
// gap rows are written as zeros.
__global__ void f0n_down_seg_kernel(const float* __restrict__ f0, const float* __restrict__ n,
                                    const float* __restrict__ wf, const float* __restrict__ bf,
                                    const float* __restrict__ wn, const float* __restrict__ bn, float* f0d,
                                    float* nd, int R, SegRows sr, AdaSegs as) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= R) return;
    const int u = seg_of_row(sr, r);
    if (u < 0) { f0d[r] = 0.f; nd[r] = 0.f; return; }
    const int off = 64 * as.p0[u], len = as.T[u];
    const int t = r - off;
    float a = 0.f, b = 0.f;
    for (int k = 0; k < 3; k++) {
        const int ti = 2 * t - 1 + k;
        if (ti >= 0 && ti < 2 * len) {
            a += wf[k] * f0[2 * off + ti];
            b += wn[k] * n[2 * off + ti];
        }
    }
    f0d[r] = a + bf[0];
    nd[r] = b + bn[0];
}

// I = int when the element count leaves room for the grid stride below 2^31
// (32-bit division), long otherwise.
template <typename I>
__global__ void concat_cols_kernel(float* dst, int ld, int col0, int T, const float* a, int lda, int ca,
                                   const float* b, int ldb, int cb, const float* c, const float* d) {
    const int W = ca + cb + (c ? 1 : 0) + (d ? 1 : 0);
    const I total = (I)T * W;
    for (I i = (I)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (I)gridDim.x * blockDim.x) {
        const int t = (int)(i / W), j = (int)(i - (I)t * W);
        float v;
        if (j < ca) v = a[(size_t)t * lda + j];
        else if (j < ca + cb) v = b[(size_t)t * ldb + (j - ca)];
        else if (c && j == ca + cb) v = c[t];
        else v = d[t];
        dst[(size_t)t * ld + col0 + j] = v;
    }
}

// Segmented form (sr.part_seg != null): the input rows are a segmented layout
// (SegRows); an output row belongs to its input row's segment, gap rows are
// written as zeros, inputs outside the row's segment count as zeros (the
// utterance's own boundary), and the AdaIN coefficients of segment u sit at
// scale + u * cstride.

template <bool SPLIT, typename I>
__global__ void dw_upsample_pack_kernel(const float* __restrict__ x, int ldx, int T, int C,
                                        const float* __restrict__ scale, const float* __restrict__ shift,
                                        float slope, const float* __restrict__ w, const float* __restrict__ bias,
                                        void* hi, void* lo, int Cp, SegRows sr, int cstride) {
    const int To = 2 * T;
    const I total = (I)To * Cp;
    for (I i = (I)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (I)gridDim.x * blockDim.x) {
        const int t = (int)(i / Cp), c = (int)(i - (I)t * Cp);
        float v = 0.f;
        const int u = sr.part_seg ? seg_of_row(sr, t >> 1) : 0;
        if (c < C && u >= 0) {
            const float sc = scale[(size_t)u * cstride + c], sh = shift[(size_t)u * cstride + c];
            float acc = 0.f;
            for (int k = 0; k < 3; k++) {
                const int tu = t + 1 - k;
                if (tu >= 0 && (tu & 1) == 0 && (tu >> 1) < T && (!sr.part_seg || seg_of_row(sr, tu >> 1) == u)) {
                    float a = sc * x[(size_t)(tu >> 1) * ldx + c] + sh;
                    a = a > 0.f ? a : slope * a;
                    acc += w[c * 3 + k] * a;
                }
            }
            v = acc + bias[c];
        }
        if (SPLIT) {
            const __nv_bfloat16 h = __float2bfloat16_rn(v);
            static_cast<__nv_bfloat16*>(hi)[i] = h;
            static_cast<__nv_bfloat16*>(lo)[i] = __float2bfloat16_rn(v - __bfloat162float(h));
        } else {
            static_cast<__half*>(hi)[i] = __float2half_rn(v);
        }
    }
}

// Per-frame phase increments of the 9 harmonics (src/kernels.cu:1337-1384):
// the increments of a chunk of frames are computed by the whole block (they do
// not depend on one another) and staged in shared memory; one thread per
// harmonic then runs the cumulative sum serially, in the reference's order, so
// the phase is bit-identical to a one-thread scan.
__global__ void __launch_bounds__(1024) sinegen_phase_kernel(const float* __restrict__ f0, int L2,
                                                             const float* __restrict__ rand_ini,
                                                             float* __restrict__ phase_low) {
    constexpr int CH = 1024;  // frames per chunk
    __shared__ float vs[9][CH];
    const int T_audio = L2 * 300;
    const float scale = __fmul_rn(__fmul_rn(2.0f, 3.14159265358979323846f), 300.0f);
    float run = 0.f;  // carried across chunks by threads 0..8
    for (int t0 = 0; t0 < L2; t0 += CH) {
        const int n = min(CH, L2 - t0);
        for (int i = threadIdx.x; i < 9 * n; i += blockDim.x) {
            const int h = i / n, tt = i - h * n;
            const int t = t0 + tt;
            const float ri = rand_ini[h];
            float src = __fsub_rn(__fdiv_rn(__fmul_rn(__fadd_rn((float)t, 0.5f), (float)T_audio), (float)L2), 0.5f);
            src = fmaxf(0.0f, fminf(src, (float)(T_audio - 1)));
            const int lo = (int)src;
            const int hi = min(lo + 1, T_audio - 1);
            const float frac = __fsub_rn(src, (float)lo);
            float rad_lo = fmodf(__fdiv_rn(__fmul_rn(f0[lo / 300], (float)(h + 1)), 24000.0f), 1.0f);
            float rad_hi = fmodf(__fdiv_rn(__fmul_rn(f0[hi / 300], (float)(h + 1)), 24000.0f), 1.0f);
            if (rad_lo < 0.0f) rad_lo = __fadd_rn(rad_lo, 1.0f);
            if (rad_hi < 0.0f) rad_hi = __fadd_rn(rad_hi, 1.0f);
            if (lo == 0) rad_lo = __fadd_rn(rad_lo, ri);
            if (hi == 0) rad_hi = __fadd_rn(rad_hi, ri);
            vs[h][tt] = __fadd_rn(__fmul_rn(__fsub_rn(1.0f, frac), rad_lo), __fmul_rn(frac, rad_hi));
        }
        __syncthreads();
        if (threadIdx.x < 9) {
            const int h = threadIdx.x;
#pragma unroll 8
            for (int tt = 0; tt < n; tt++) {
                const int t = t0 + tt;
                run = t == 0 ? vs[h][tt] : __fadd_rn(run, vs[h][tt]);
                phase_low[t * 9 + h] = __fmul_rn(run, scale);
            }
        }
        __syncthreads();
    }
}

__global__ void sinegen_source_kernel(const float* __restrict__ phase_low, const float* __restrict__ f0,
                                      const float* __restrict__ lw, const float* __restrict__ lb,
                                      float* __restrict__ out, int L2, int T_audio) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T_audio) return;
    float src = __fsub_rn(__fdiv_rn(__fmul_rn(__fadd_rn((float)t, 0.5f), (float)L2), (float)T_audio), 0.5f);
    src = fmaxf(0.0f, fminf(src, (float)(L2 - 1)));
    const int lo = (int)src;
    const int hi = min(lo + 1, L2 - 1);
    const float frac = __fsub_rn(src, (float)lo);
    const float f0v = f0[t / 300];
    const float uv = (f0v > 10.0f) ? 1.0f : 0.0f;
    const float namp = __fadd_rn(__fmul_rn(uv, 0.003f), __fmul_rn(__fsub_rn(1.0f, uv), 0.1f / 3.0f));
    float sum = lb[0];
    for (int h = 0; h < 9; h++) {
        const float ph = __fadd_rn(__fmul_rn(__fsub_rn(1.0f, frac), phase_low[lo * 9 + h]),
                                   __fmul_rn(frac, phase_low[hi * 9 + h]));
        const float sine = __fmul_rn(sinf(ph), 0.1f);
        uint32_t hs = (uint32_t)t * 2654435761u + (uint32_t)h * 340573321u + 42u;
        hs ^= hs >> 16; hs *= 0x85ebca6bu;
        hs ^= hs >> 13; hs *= 0xc2b2ae35u; hs ^= hs >> 16;
        const float u1 = __fdiv_rn((float)((hs & 0xFFFFFFu) + 1u), 16777217.0f);
        hs = hs * 1664525u + 1013904223u;
        const float u2 = __fdiv_rn((float)(hs & 0xFFFFFFu), 16777216.0f);
        const float nz = __fmul_rn(__fmul_rn(sqrtf(__fmul_rn(-2.0f, logf(u1))),
                                             cosf(__fmul_rn(__fmul_rn(2.0f, 3.14159265358979323846f), u2))),
                                   namp);
        const float val = __fadd_rn(__fmul_rn(sine, uv), nz);
        sum = __fadd_rn(sum, __fmul_rn(val, lw[h]));
    }
    out[t] = tanhf(sum);
}

// One thread per frame.  The DFT is evaluated in symmetric / antisymmetric
// pairs (n, 20-n) with exactly mirrored window and twiddles:
//   re = xw0 c0 + xw10 c10 + sum_{n=1..9} (xw[n] + xw[20-n]) c[n]
//   im = -sum_{n=1..9} (xw[n] - xw[20-n]) s[n]
// so analytically real bins (k = 0, 10, all bins of the symmetric frame 0)
// are exactly real; a zero imaginary part is taken as +0.
__global__ void stft_kernel(const float* __restrict__ x, int T, float* __restrict__ har, int T2) {
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    if (f >= T2) return;
    float xw[20];
#pragma unroll
    for (int n = 0; n < 20; n++) {
        int i = f * 5 + n - 10;
        if (i < 0) i = -i;
        else if (i >= T) i = 2 * T - 2 - i;
        xw[n] = __fmul_rn(x[i], c_win[n]);
    }
    float sp[10], dm[10];
#pragma unroll
    for (int n = 1; n < 10; n++) { sp[n] = __fadd_rn(xw[n], xw[20 - n]); dm[n] = __fsub_rn(xw[n], xw[20 - n]); }
#pragma unroll 1
    for (int k = 0; k < 11; k++) {
        float re = __fadd_rn(__fmul_rn(xw[0], c_cos[k][0]), __fmul_rn(xw[10], c_cos[k][10]));
        float im = 0.f;
#pragma unroll
        for (int n = 1; n < 10; n++) {
            re = __fadd_rn(re, __fmul_rn(sp[n], c_cos[k][n]));
            im = __fsub_rn(im, __fmul_rn(dm[n], c_sin[k][n]));
        }
        im = __fadd_rn(im, 0.0f);  // -0 -> +0
        har[(size_t)f * 22 + k] = sqrtf(__fadd_rn(__fmul_rn(re, re), __fmul_rn(im, im)));
        har[(size_t)f * 22 + 11 + k] = atan2f(im, re);
    }
}

// iSTFT part 1: per frame, spec = exp(c[0:11]), phase = sin(c[11:22]),
// inverse real DFT (bins 0 and 10 weight 1, others 2) / 20, times the window.
__global__ void istft_frames_kernel(const float* __restrict__ post, int T2, float* __restrict__ fr) {
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    if (f >= T2) return;
    float re[11], im[11];
#pragma unroll
    for (int k = 0; k < 11; k++) {
        const float mag = expf(post[(size_t)f * 22 + k]);
        const float ph = sinf(post[(size_t)f * 22 + 11 + k]);
        re[k] = __fmul_rn(mag, cosf(ph));
        im[k] = __fmul_rn(mag, sinf(ph));
    }
#pragma unroll 4
    for (int n = 0; n < 20; n++) {
        float v = 0.f;
#pragma unroll
        for (int k = 0; k < 11; k++) {
            const float contrib = __fsub_rn(__fmul_rn(re[k], c_cos[k][n]), __fmul_rn(im[k], c_sin[k][n]));
            v = __fadd_rn(v, (k == 0 || k == 10) ? contrib : __fmul_rn(2.0f, contrib));
        }
        fr[(size_t)f * 20 + n] = __fmul_rn(__fmul_rn(v, 0.05f), c_win[n]);
    }
}

// iSTFT part 2: gather-form overlap-add (each sample sums <= 4 frames in
// ascending frame order), window-square normalisation, centre pad stripped.
__global__ void istft_ola_kernel(const float* __restrict__ fr, int T2, float* __restrict__ y, int T_audio) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T_audio) return;
    const int u = t + 10;
    float acc = 0.f, ws = 0.f;
    const int f_hi = min(u / 5, T2 - 1);
    for (int f = max(0, (u - 15) / 5); f <= f_hi; f++) {
        const int n = u - 5 * f;
        if (n < 0 || n >= 20) continue;
        acc = __fadd_rn(acc, fr[(size_t)f * 20 + n]);
        ws = __fadd_rn(ws, __fmul_rn(c_win[n], c_win[n]));
    }
    y[t] = (ws > 1e-8f) ? __fdiv_rn(acc, ws) : 0.0f;
}

}  // namespace

void style_fc(const float* W, const float* b, const float* s, float* out, int rows, cudaStream_t st) {
    style_fc_kernel<<<(rows * 32 + 255) / 256, 256, 0, st>>>(W, b, s, 0, out, rows);
}

void style_fc_batch(const float* W, const float* b, const float* s, int s_stride, int B, float* out, int rows,
                    cudaStream_t st) {
    style_fc_kernel<<<dim3((rows * 32 + 255) / 256, B), 256, 0, st>>>(W, b, s, s_stride, out, rows);
}

void adain_coef(const float* stats, int parts, int ld, int col0, int C, int T, const float* gamma,
                const float* beta, const float* nw, const float* nb, float* coef, cudaStream_t st, AdaSegs seg) {
    adain_coef_kernel<<<dim3((C + 7) / 8, seg.p0 ? seg.n : 1), dim3(8, 128), 0, st>>>(
        stats, parts, ld, col0, C, T, gamma, beta, nw, nb, coef, seg);
}

void col_stats(const float* x, int ld, int col0, int ncols, int T, int rows_per_part, float* stats,
               cudaStream_t st, const int* part_rows) {
    const int parts = (T + rows_per_part - 1) / rows_per_part;
    dim3 grid((ncols + 31) / 32, parts);
    col_stats_kernel<<<grid, dim3(32, 8), 0, st>>>(x, ld, col0, ncols, T, rows_per_part, parts, stats, part_rows);
}

void f0n_down_seg(const float* f0, const float* n, const float* wf, const float* bf, const float* wn,
                  const float* bn, float* f0d, float* nd, int R, SegRows sr, AdaSegs as, cudaStream_t st) {
    f0n_down_seg_kernel<<<(R + 255) / 256, 256, 0, st>>>(f0, n, wf, bf, wn, bn, f0d, nd, R, sr, as);
}

void f0n_down(const float* f0, const float* n, const float* wf, const float* bf, const float* wn, const float* bn,
              float* f0d, float* nd, int L, cudaStream_t st) {
    f0n_down_kernel<<<(L + 255) / 256, 256, 0, st>>>(f0, n, wf, bf, wn, bn, f0d, nd, L);
}

void concat_cols(float* dst, int ld, int col0, int T, const float* a, int lda, int ca, const float* b, int ldb,
                 int cb, const float* c, const float* d, cudaStream_t st) {
    const long total = (long)T * (ca + cb + 2);
    if (small_index(total))
        concat_cols_kernel<int><<<nblocks(total, 256), 256, 0, st>>>(dst, ld, col0, T, a, lda, ca, b, ldb, cb, c, d);
    else
        concat_cols_kernel<long><<<nblocks(total, 256), 256, 0, st>>>(dst, ld, col0, T, a, lda, ca, b, ldb, cb, c, d);
}

void dw_upsample_pack(const float* x, int ldx, int T, int C, const float* scale, const float* shift, float slope,
                      const float* w, const float* b, void* hi, void* lo, int Cp, bool split, cudaStream_t st,
                      SegRows sr, int cstride) {
    const long total = (long)2 * T * Cp;
    const int g = nblocks(total, 256);
    if (small_index(total)) {
        if (split) dw_upsample_pack_kernel<true, int><<<g, 256, 0, st>>>(x, ldx, T, C, scale, shift, slope, w, b, hi, lo, Cp, sr, cstride);
        else dw_upsample_pack_kernel<false, int><<<g, 256, 0, st>>>(x, ldx, T, C, scale, shift, slope, w, b, hi, lo, Cp, sr, cstride);
    } else {
        if (split) dw_upsample_pack_kernel<true, long><<<g, 256, 0, st>>>(x, ldx, T, C, scale, shift, slope, w, b, hi, lo, Cp, sr, cstride);
        else dw_upsample_pack_kernel<false, long><<<g, 256, 0, st>>>(x, ldx, T, C, scale, shift, slope, w, b, hi, lo, Cp, sr, cstride);
    }
}

namespace {
__device__ float d_rand_ini[9];
constexpr int kMaxDevices = 64;
float* g_rand_ini_ptr[kMaxDevices] = {};  // per-device address of d_rand_ini (set by upload_twiddles)
int cur_dev() {
    int d = 0;
    cudaGetDevice(&d);
    return d < kMaxDevices ? d : 0;
}
}

void sinegen_phase(const float* f0, int L2, float* phase_low, cudaStream_t st) {
    sinegen_phase_kernel<<<1, 1024, 0, st>>>(f0, L2, g_rand_ini_ptr[cur_dev()], phase_low);
}

void sinegen_source(const float* phase_low, const float* f0, const float* lw, const float* lb, float* out, int L2,
                    cudaStream_t st) {
    const int T_audio = L2 * 300;
    sinegen_source_kernel<<<(T_audio + 255) / 256, 256, 0, st>>>(phase_low, f0, lw, lb, out, L2, T_audio);
}

void stft(const float* x, int T, float* har, int T2, cudaStream_t st) {
    stft_kernel<<<(T2 + 127) / 128, 128, 0, st>>>(x, T, har, T2);
}

void istft(const float* post, int T2, float* frames, float* y, int T_audio, cudaStream_t st) {
    istft_frames_kernel<<<(T2 + 127) / 128, 128, 0, st>>>(post, T2, frames);
    istft_ola_kernel<<<(T_audio + 255) / 256, 256, 0, st>>>(frames, T2, y, T_audio);
}

}  // namespace rk

#include <random>

namespace rk {
// Twiddles, window and SineGen's rand_ini, computed once on the host:
// angles 2*pi*r/20 evaluated in double for r <= 10, mirrored exactly for
// r > 10 and rounded to float (quarter angles exact), periodic Hann window
// mirrored the same way; rand_ini from mt19937(42) +
// uniform_real_distribution<float>(0, 1) for harmonics 1..8 (src/rokoko.cpp:958-967).
cudaError_t upload_twiddles() {
    float cs[11][20], sn[11][20], win[20], ri[9];
    double cr[20], sr[20], wn[20];
    for (int r = 0; r <= 10; r++) {
        cr[r] = std::cos(2.0 * M_PI * r / 20.0);
        sr[r] = std::sin(2.0 * M_PI * r / 20.0);
        wn[r] = 0.5 * (1.0 - cr[r]);
    }
    cr[0] = 1; sr[0] = 0; cr[5] = 0; sr[5] = 1; cr[10] = -1; sr[10] = 0;
    wn[0] = 0; wn[10] = 1; wn[5] = 0.5;
    for (int r = 11; r < 20; r++) { cr[r] = cr[20 - r]; sr[r] = -sr[20 - r]; wn[r] = wn[20 - r]; }
    for (int n = 0; n < 20; n++) win[n] = (float)wn[n];
    for (int k = 0; k < 11; k++)
        for (int n = 0; n < 20; n++) {
            const int r = (k * n) % 20;
            cs[k][n] = (float)cr[r];
            sn[k][n] = (float)sr[r];
        }
    std::mt19937 rng(42);
    std::uniform_real_distribution<float> uni(0.0f, 1.0f);
    ri[0] = 0.f;
    for (int h = 1; h < 9; h++) ri[h] = uni(rng);
    cudaError_t e;
    if ((e = cudaMemcpyToSymbol(c_cos, cs, sizeof cs)) != cudaSuccess) return e;
    if ((e = cudaMemcpyToSymbol(c_sin, sn, sizeof sn)) != cudaSuccess) return e;
    if ((e = cudaMemcpyToSymbol(c_win, win, sizeof win)) != cudaSuccess) return e;
    if ((e = cudaMemcpyToSymbol(d_rand_ini, ri, sizeof ri)) != cudaSuccess) return e;
    return cudaGetSymbolAddress(reinterpret_cast<void**>(&g_rand_ini_ptr[cur_dev()]), d_rand_ini);
}
}  // namespace rk
