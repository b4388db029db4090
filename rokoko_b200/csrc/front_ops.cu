// front_ops.cu -- bandwidth / latency kernels of the front half (ALBERT, text
// encoder, prosody predictor) and the duration -> alignment expansion.
//
// Reference semantics (src/kernels.cu): embeddings + LayerNorm :15-95,
// residual LayerNorm :102-144, softmax :189-225, channel LayerNorm :364-404,
// AdaLayerNorm :513-548, sigmoid-sum :643-662, round/clamp durations
// :1457-1479, alignment :1484-1505 (here an index gather instead of a dense 0/1
// matrix and two GEMMs, src/rokoko.cpp:850-863, 916-919).
// Row kernels use one warp per row with the two-pass mean / variance of the
// reference, and write the next GEMM's 16-bit operand planes directly.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "front_ops.cuh"

namespace rk {

namespace {

__device__ __forceinline__ void put_op(void* hi, void* lo, size_t i, float v, bool split) {
    if (split) {
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        static_cast<__nv_bfloat16*>(hi)[i] = h;
        static_cast<__nv_bfloat16*>(lo)[i] = __float2bfloat16_rn(v - __bfloat162float(h));
    } else {
        static_cast<__half*>(hi)[i] = __float2half_rn(v);
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// two-pass row statistics over D values held VPL per lane (D = 32 * VPL)
template <int VPL>
__device__ __forceinline__ void row_stats(const float (&v)[VPL], int D, float& mean, float& inv, float eps) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; i++) s += v[i];
    mean = warp_sum(s) / D;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; i++) { const float d = v[i] - mean; q += d * d; }
    inv = rsqrtf(warp_sum(q) / D + eps);
}

__global__ void embed_ln_kernel(const int* __restrict__ tok, int T, const float* __restrict__ word,
                                const float* __restrict__ pos, const float* __restrict__ type,
                                const float* __restrict__ g, const float* __restrict__ b, float* __restrict__ out,
                                OpPlanes op, bool split) {
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= T) return;
    constexpr int D = 128, VPL = 4;
    float v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int d = lane + 32 * i;
        v[i] = (word[(size_t)tok[t] * D + d] + pos[(size_t)t * D + d]) + type[d];
    }
    float mean, inv;
    row_stats<VPL>(v, D, mean, inv, 1e-12f);
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int d = lane + 32 * i;
        const float y = (v[i] - mean) * inv * g[d] + b[d];
        out[(size_t)t * D + d] = y;
        put_op(op.hi, op.lo, (size_t)t * op.Cp + d, y, split);
    }
}

// h = LN(h + a) (eps 1e-12), D = 768; also the next GEMM's operand
__global__ void res_ln_kernel(float* __restrict__ h, const float* __restrict__ a, int T,
                              const float* __restrict__ g, const float* __restrict__ b, OpPlanes op, bool split) {
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= T) return;
    constexpr int D = 768, VPL = 24;
    float v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const size_t o = (size_t)t * D + lane + 32 * i;
        v[i] = h[o] + a[o];
    }
    float mean, inv;
    row_stats<VPL>(v, D, mean, inv, 1e-12f);
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int d = lane + 32 * i;
        const float y = (v[i] - mean) * inv * g[d] + b[d];
        h[(size_t)t * D + d] = y;
        put_op(op.hi, op.lo, (size_t)t * op.Cp + d, y, split);
    }
}

// text encoder: y = LeakyReLU(LN_channels(x) * gamma + beta, 0.2), D = 512
__global__ void ln_lrelu_kernel(const float* __restrict__ x, int T, const float* __restrict__ g,
                                const float* __restrict__ b, float* __restrict__ out, OpPlanes op, bool split) {
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= T) return;
    constexpr int D = 512, VPL = 16;
    float v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; i++) v[i] = x[(size_t)t * D + lane + 32 * i];
    float mean, inv;
    row_stats<VPL>(v, D, mean, inv, 1e-5f);
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int d = lane + 32 * i;
        float y = (v[i] - mean) * inv * g[d] + b[d];
        y = y > 0.f ? y : 0.2f * y;
        out[(size_t)t * D + d] = y;
        put_op(op.hi, op.lo, (size_t)t * op.Cp + d, y, split);
    }
}

// cat[t] = [x[t] (AdaLN'd when gamma != null) | style]  (D = 512 + 128)
__global__ void adaln_concat_kernel(const float* __restrict__ x, int T, const float* __restrict__ gamma,
                                    const float* __restrict__ beta, const float* __restrict__ style,
                                    float* __restrict__ cat, OpPlanes op, bool split) {
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= T) return;
    constexpr int D = 512, VPL = 16;
    float v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; i++) v[i] = x[(size_t)t * D + lane + 32 * i];
    if (gamma) {
        float mean, inv;
        row_stats<VPL>(v, D, mean, inv, 1e-5f);
#pragma unroll
        for (int i = 0; i < VPL; i++) {
            const int d = lane + 32 * i;
            v[i] = (1.0f + gamma[d]) * ((v[i] - mean) * inv) + beta[d];
        }
    }
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int d = lane + 32 * i;
        cat[(size_t)t * 640 + d] = v[i];
        put_op(op.hi, op.lo, (size_t)t * op.Cp + d, v[i], split);
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int d = lane + 32 * i;
        cat[(size_t)t * 640 + 512 + d] = style[d];
        put_op(op.hi, op.lo, (size_t)t * op.Cp + 512 + d, style[d], split);
    }
}

// Scaled dot-product attention without mask, FP32 (src/rokoko.cpp:363-384):
// S = Q K^T * 0.125, softmax over keys, O = P V.  Block = 8 warps = 8 query
// rows of one head; keys / values staged through shared memory in chunks.
constexpr int ATT_ROWS = 8, ATT_CHUNK = 64, ATT_MAXT = 512;
__global__ void attention_kernel(const float* __restrict__ qkv, int T, float* __restrict__ ctx) {
    __shared__ float kv[ATT_CHUNK][65];
    __shared__ float sc[ATT_ROWS][ATT_MAXT];
    __shared__ float qs[ATT_ROWS][64];
    const int head = blockIdx.y, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i = blockIdx.x * ATT_ROWS + w;
    const bool row_ok = i < T;
    if (row_ok) {
        qs[w][lane] = qkv[(size_t)i * 2304 + head * 64 + lane];
        qs[w][lane + 32] = qkv[(size_t)i * 2304 + head * 64 + lane + 32];
    }
    // scores
    for (int j0 = 0; j0 < T; j0 += ATT_CHUNK) {
        const int nj = min(ATT_CHUNK, T - j0);
        __syncthreads();
        for (int e = threadIdx.x; e < nj * 64; e += blockDim.x) {
            const int j = e >> 6, d = e & 63;
            kv[j][d] = qkv[(size_t)(j0 + j) * 2304 + 768 + head * 64 + d];
        }
        __syncthreads();
        if (row_ok)
            for (int j = lane; j < nj; j += 32) {
                float acc = 0.f;
#pragma unroll 16
                for (int d = 0; d < 64; d++) acc += qs[w][d] * kv[j][d];
                sc[w][j0 + j] = acc * 0.125f;
            }
    }
    // softmax over the row (max-subtracted exp, times 1/sum)
    float inv = 0.f;
    if (row_ok) {
        float mx = -1e30f;
        for (int j = lane; j < T; j += 32) mx = fmaxf(mx, sc[w][j]);
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float s = 0.f;
        for (int j = lane; j < T; j += 32) {
            const float e = expf(sc[w][j] - mx);
            sc[w][j] = e;
            s += e;
        }
        inv = 1.0f / warp_sum(s);
    }
    // O = P V
    float o0 = 0.f, o1 = 0.f;
    for (int j0 = 0; j0 < T; j0 += ATT_CHUNK) {
        const int nj = min(ATT_CHUNK, T - j0);
        __syncthreads();
        for (int e = threadIdx.x; e < nj * 64; e += blockDim.x) {
            const int j = e >> 6, d = e & 63;
            kv[j][d] = qkv[(size_t)(j0 + j) * 2304 + 1536 + head * 64 + d];
        }
        __syncthreads();
        if (row_ok)
            for (int j = 0; j < nj; j++) {
                const float p = sc[w][j0 + j] * inv;
                o0 += p * kv[j][lane];
                o1 += p * kv[j][lane + 32];
            }
    }
    if (row_ok) {
        ctx[(size_t)i * 768 + head * 64 + lane] = o0;
        ctx[(size_t)i * 768 + head * 64 + lane + 32] = o1;
    }
}

// dur[t] = sum_50 sigmoid(proj[t]); int = max(1, round-half-even(dur))
__global__ void durations_kernel(const float* __restrict__ proj, int T, float* __restrict__ dur_f,
                                 int* __restrict__ dur_i) {
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= T) return;
    float s = 0.f;
    for (int d = lane; d < 50; d += 32) s += 1.0f / (1.0f + expf(-proj[(size_t)t * 50 + d]));
    s = warp_sum(s);
    if (lane == 0) {
        dur_f[t] = s;
        dur_i[t] = max(1, __float2int_rn(s));
    }
}

// Alignment as an index gather: frame l of token t(l) where token t covers
// frames [sum_{i<t} d_i, sum_{i<=t} d_i).  en[l] = cat[t(l)] (640, also as the
// shared LSTM's operand), asr[l] = te[t(l)] (512); frames >= L are zero.
__global__ void align_gather_kernel(const int* __restrict__ dur, int T, int L_b, const float* __restrict__ cat,
                                    const float* __restrict__ te, float* __restrict__ en, float* __restrict__ asr,
                                    OpPlanes op, bool split) {
    __shared__ int start[ATT_MAXT + 1];
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int t = 0; t < T; t++) { start[t] = acc; acc += dur[t]; }
        start[T] = acc;
    }
    __syncthreads();
    const int L = start[T];
    for (int l = blockIdx.x; l < L_b; l += gridDim.x) {
        int tok = -1;
        if (l < L) {  // binary search: largest t with start[t] <= l
            int lo = 0, hi = T - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (start[mid] <= l) lo = mid; else hi = mid - 1;
            }
            tok = lo;
        }
        for (int d = threadIdx.x; d < 640; d += blockDim.x) {
            const float v = tok >= 0 ? cat[(size_t)tok * 640 + d] : 0.f;
            en[(size_t)l * 640 + d] = v;
            put_op(op.hi, op.lo, (size_t)l * op.Cp + d, v, split);
            if (d < 512) asr[(size_t)l * 512 + d] = tok >= 0 ? te[(size_t)tok * 512 + d] : 0.f;
        }
    }
}

// y[t] = w . x[t] + b (Conv1d 256 -> 1, K = 1, FP32 weights: src/kernels.cu:286-320)
__global__ void rowdot_kernel(const float* __restrict__ x, int T, int C, const float* __restrict__ w,
                              const float* __restrict__ b, float* __restrict__ y) {
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= T) return;
    float s = 0.f;
    for (int c = lane; c < C; c += 32) s += w[c] * x[(size_t)t * C + c];
    s = warp_sum(s);
    if (lane == 0) y[t] = s + b[0];
}

__global__ void gather_rows_kernel(const int* __restrict__ tok, int T, const float* __restrict__ table, int D,
                                   float* __restrict__ out, OpPlanes op, bool split) {
    const int t = blockIdx.x;
    if (t >= T) return;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        const float v = table[(size_t)tok[t] * D + d];
        out[(size_t)t * D + d] = v;
        put_op(op.hi, op.lo, (size_t)t * op.Cp + d, v, split);
    }
}

int rows_grid(int T) { return (T + 7) / 8; }

}  // namespace

void embed_ln(const int* tok, int T, const float* word, const float* pos, const float* type, const float* g,
              const float* b, float* out, OpPlanes op, bool split, cudaStream_t st) {
    embed_ln_kernel<<<rows_grid(T), 256, 0, st>>>(tok, T, word, pos, type, g, b, out, op, split);
}
void res_ln(float* h, const float* a, int T, const float* g, const float* b, OpPlanes op, bool split,
            cudaStream_t st) {
    res_ln_kernel<<<rows_grid(T), 256, 0, st>>>(h, a, T, g, b, op, split);
}
void ln_lrelu(const float* x, int T, const float* g, const float* b, float* out, OpPlanes op, bool split,
              cudaStream_t st) {
    ln_lrelu_kernel<<<rows_grid(T), 256, 0, st>>>(x, T, g, b, out, op, split);
}
void adaln_concat(const float* x, int T, const float* gamma, const float* beta, const float* style, float* cat,
                  OpPlanes op, bool split, cudaStream_t st) {
    adaln_concat_kernel<<<rows_grid(T), 256, 0, st>>>(x, T, gamma, beta, style, cat, op, split);
}
void attention(const float* qkv, int T, float* ctx, cudaStream_t st) {
    attention_kernel<<<dim3((T + ATT_ROWS - 1) / ATT_ROWS, 12), 32 * ATT_ROWS, 0, st>>>(qkv, T, ctx);
}
void durations(const float* proj, int T, float* dur_f, int* dur_i, cudaStream_t st) {
    durations_kernel<<<rows_grid(T), 256, 0, st>>>(proj, T, dur_f, dur_i);
}
void align_gather(const int* dur, int T, int L_b, const float* cat, const float* te, float* en, float* asr,
                  OpPlanes op, bool split, cudaStream_t st) {
    align_gather_kernel<<<148 * 2, 256, 0, st>>>(dur, T, L_b, cat, te, en, asr, op, split);
}
void rowdot(const float* x, int T, int C, const float* w, const float* b, float* y, cudaStream_t st) {
    rowdot_kernel<<<rows_grid(T), 256, 0, st>>>(x, T, C, w, b, y);
}
void gather_rows(const int* tok, int T, const float* table, int D, float* out, OpPlanes op, bool split,
                 cudaStream_t st) {
    gather_rows_kernel<<<T, 256, 0, st>>>(tok, T, table, D, out, op, split);
}

}  // namespace rk
