// front_ops.cu -- bandwidth / latency kernels of the front half (ALBERT, text
// encoder, prosody predictor) and the duration -> alignment expansion, over
// every utterance of a batch at once (segmented row layout, front_ops.cuh).
//
// Reference semantics (src/kernels.cu): embeddings + LayerNorm :15-95,
// residual LayerNorm :102-144, channel LayerNorm :364-404,
// AdaLayerNorm :513-548, sigmoid-sum :643-662, round/clamp durations
// :1457-1479, alignment :1484-1505 (here a scan + index gather instead of a
// dense 0/1 matrix and two GEMMs, src/rokoko.cpp:850-863, 916-919).
// Row kernels use one warp per row with the two-pass mean / variance of the
// reference, and write the next GEMM's 16-bit operand planes directly.  The
// arithmetic of a row does not depend on the batch it is in, so an utterance
// gives the same bits alone or batched.
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

// zeros for a gap row: the FP32 output row (length D, pitch ldo) and the operand columns [0, Cp)
__device__ __forceinline__ void zero_row(float* out, int ldo, int D, int r, OpPlanes op, bool split, int lane) {
    for (int d = lane; d < D; d += 32)
        if (out) out[(size_t)r * ldo + d] = 0.f;
    for (int d = lane; d < op.Cp; d += 32) put_op(op.hi, op.lo, (size_t)r * op.Cp + d, 0.f, split);
}

__global__ void embed_ln_kernel(RowMeta m, const float* __restrict__ word, const float* __restrict__ pos,
                                const float* __restrict__ type, const float* __restrict__ g,
                                const float* __restrict__ b, float* __restrict__ out, OpPlanes op, bool split) {
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= m.R) return;
    constexpr int D = 128, VPL = 4;
    const int p = m.pos[r];
    if (p < 0) { zero_row(out, D, D, r, op, split, lane); return; }
    const int tk = m.tok[r];
    float v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int d = lane + 32 * i;
        v[i] = (word[(size_t)tk * D + d] + pos[(size_t)p * D + d]) + type[d];
    }
    float mean, inv;
    row_stats<VPL>(v, D, mean, inv, 1e-12f);
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int d = lane + 32 * i;
        const float y = (v[i] - mean) * inv * g[d] + b[d];
        out[(size_t)r * D + d] = y;
        put_op(op.hi, op.lo, (size_t)r * op.Cp + d, y, split);
    }
}

// h = LN(h + a) (eps 1e-12), D = 768; also the next GEMM's operand
__global__ void res_ln_kernel(float* __restrict__ h, const float* __restrict__ a, RowMeta m,
                              const float* __restrict__ g, const float* __restrict__ b, OpPlanes op, bool split) {
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= m.R) return;
    constexpr int D = 768, VPL = 24;
    if (m.pos[r] < 0) { zero_row(h, D, D, r, op, split, lane); return; }
    float v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const size_t o = (size_t)r * D + lane + 32 * i;
        v[i] = h[o] + a[o];
    }
    float mean, inv;
    row_stats<VPL>(v, D, mean, inv, 1e-12f);
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int d = lane + 32 * i;
        const float y = (v[i] - mean) * inv * g[d] + b[d];
        h[(size_t)r * D + d] = y;
        put_op(op.hi, op.lo, (size_t)r * op.Cp + d, y, split);
    }
}

// text encoder: y = LeakyReLU(LN_channels(x) * gamma + beta, 0.2), D = 512
__global__ void ln_lrelu_kernel(const float* __restrict__ x, RowMeta m, const float* __restrict__ g,
                                const float* __restrict__ b, float* __restrict__ out, OpPlanes op, bool split) {
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= m.R) return;
    constexpr int D = 512, VPL = 16;
    if (m.pos[r] < 0) { zero_row(out, D, D, r, op, split, lane); return; }
    float v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; i++) v[i] = x[(size_t)r * D + lane + 32 * i];
    float mean, inv;
    row_stats<VPL>(v, D, mean, inv, 1e-5f);
#pragma unroll
    for (int i = 0; i < VPL; i++) {
        const int d = lane + 32 * i;
        float y = (v[i] - mean) * inv * g[d] + b[d];
        y = y > 0.f ? y : 0.2f * y;
        out[(size_t)r * D + d] = y;
        put_op(op.hi, op.lo, (size_t)r * op.Cp + d, y, split);
    }
}

// cat[r] = [x[r] (AdaLN'd when gamma_off >= 0) | style]  (D = 512 + 128)
__global__ void adaln_concat_kernel(const float* __restrict__ x, RowMeta m, const float* __restrict__ fc,
                                    int fc_stride, int gamma_off, const float* __restrict__ style, int style_stride,
                                    float* __restrict__ cat, OpPlanes op, bool split) {
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= m.R) return;
    constexpr int D = 512, VPL = 16;
    const int u = m.utt[r];
    if (u < 0) { zero_row(cat, 640, 640, r, op, split, lane); return; }
    float v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; i++) v[i] = x[(size_t)r * D + lane + 32 * i];
    if (gamma_off >= 0) {
        const float* gamma = fc + (size_t)u * fc_stride + gamma_off;
        const float* beta = gamma + 512;
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
        cat[(size_t)r * 640 + d] = v[i];
        put_op(op.hi, op.lo, (size_t)r * op.Cp + d, v[i], split);
    }
    const float* s = style + (size_t)u * style_stride;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int d = lane + 32 * i;
        cat[(size_t)r * 640 + 512 + d] = s[d];
        put_op(op.hi, op.lo, (size_t)r * op.Cp + 512 + d, s[d], split);
    }
}

// dur[r] = sum_50 sigmoid(proj[r]); int = max(1, round-half-even(dur)); gap rows 0
__global__ void durations_kernel(const float* __restrict__ proj, RowMeta m, float* __restrict__ dur_f,
                                 int* __restrict__ dur_i) {
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= m.R) return;
    if (m.pos[r] < 0) {
        if (lane == 0) { dur_f[r] = 0.f; dur_i[r] = 0; }
        return;
    }
    float s = 0.f;
    for (int d = lane; d < 50; d += 32) s += 1.0f / (1.0f + expf(-proj[(size_t)r * 50 + d]));
    s = warp_sum(s);
    if (lane == 0) {
        dur_f[r] = s;
        dur_i[r] = max(1, __float2int_rn(s));
    }
}

// One block per (frame chunk, utterance): the block scans the utterance's
// durations (exclusive prefix sums in shared memory, integer so exact), then
// its frames find their token by binary search.
constexpr int ALIGN_THREADS = 256;
__global__ void __launch_bounds__(ALIGN_THREADS) align_gather_kernel(
    const int* __restrict__ dur, SegMeta tok, SegMeta frames, const float* __restrict__ cat,
    const float* __restrict__ te, float* __restrict__ en, float* __restrict__ asr, int* __restrict__ frame_tok,
    OpPlanes op, bool split) {
    __shared__ int start[512 + 1];
    __shared__ int warp_tot[ALIGN_THREADS / 32];
    const int u = blockIdx.y;
    const int T = tok.len[u], toff = tok.off[u];
    const int Lb = frames.len[u], foff = frames.off[u];
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    // thread i holds durations 2i and 2i + 1 (T <= 512 = 2 x 256)
    const int a = 2 * tid < T ? dur[toff + 2 * tid] : 0;
    const int b = 2 * tid + 1 < T ? dur[toff + 2 * tid + 1] : 0;
    int incl = a + b;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) warp_tot[wid] = incl;
    __syncthreads();
    int before = 0;
    for (int k = 0; k < wid; k++) before += warp_tot[k];
    const int excl = before + incl - (a + b);
    if (2 * tid < T) start[2 * tid] = excl;
    if (2 * tid + 1 < T) start[2 * tid + 1] = excl + a;
    if (tid == ALIGN_THREADS - 1) start[T] = before + incl;  // total L (zeros past T add nothing)
    __syncthreads();
    const int L = start[T];
    for (int l = blockIdx.x; l < Lb; l += gridDim.x) {
        int t = -1;
        if (l < L) {  // largest t with start[t] <= l
            int lo = 0, hi = T - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (start[mid] <= l) lo = mid; else hi = mid - 1;
            }
            t = lo;
        }
        const size_t f = (size_t)foff + l;
        if (tid == 0) frame_tok[f] = t;
        for (int d = tid; d < 640; d += ALIGN_THREADS) {
            const float v = t >= 0 ? cat[(size_t)(toff + t) * 640 + d] : 0.f;
            en[f * 640 + d] = v;
            put_op(op.hi, op.lo, f * op.Cp + d, v, split);
            if (d < 512) asr[f * 512 + d] = t >= 0 ? te[(size_t)(toff + t) * 512 + d] : 0.f;
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

__global__ void gather_rows_kernel(RowMeta m, const float* __restrict__ table, int D, float* __restrict__ out,
                                   OpPlanes op, bool split) {
    const int r = blockIdx.x;
    if (r >= m.R) return;
    const bool gap = m.pos[r] < 0;
    const int tk = m.tok[r];
    for (int d = threadIdx.x; d < op.Cp; d += blockDim.x) {
        const float v = (!gap && d < D) ? table[(size_t)tk * D + d] : 0.f;
        if (d < D) out[(size_t)r * D + d] = v;
        put_op(op.hi, op.lo, (size_t)r * op.Cp + d, v, split);
    }
}

int rows_grid(int R) { return (R + 7) / 8; }

}  // namespace

void embed_ln(RowMeta m, const float* word, const float* pos, const float* type, const float* g, const float* b,
              float* out, OpPlanes op, bool split, cudaStream_t st) {
    embed_ln_kernel<<<rows_grid(m.R), 256, 0, st>>>(m, word, pos, type, g, b, out, op, split);
}
void res_ln(float* h, const float* a, RowMeta m, const float* g, const float* b, OpPlanes op, bool split,
            cudaStream_t st) {
    res_ln_kernel<<<rows_grid(m.R), 256, 0, st>>>(h, a, m, g, b, op, split);
}
void ln_lrelu(const float* x, RowMeta m, const float* g, const float* b, float* out, OpPlanes op, bool split,
              cudaStream_t st) {
    ln_lrelu_kernel<<<rows_grid(m.R), 256, 0, st>>>(x, m, g, b, out, op, split);
}
void adaln_concat(const float* x, RowMeta m, const float* fc, int fc_stride, int gamma_off, const float* style,
                  int style_stride, float* cat, OpPlanes op, bool split, cudaStream_t st) {
    adaln_concat_kernel<<<rows_grid(m.R), 256, 0, st>>>(x, m, fc, fc_stride, gamma_off, style, style_stride, cat, op,
                                                         split);
}
void durations(const float* proj, RowMeta m, float* dur_f, int* dur_i, cudaStream_t st) {
    durations_kernel<<<rows_grid(m.R), 256, 0, st>>>(proj, m, dur_f, dur_i);
}
void align_gather(const int* dur, SegMeta tok, SegMeta frames, const float* cat, const float* te, float* en,
                  float* asr, int* frame_tok, OpPlanes op, bool split, cudaStream_t st) {
    // frame chunks per utterance: about two waves of blocks over the whole batch
    int chunks = (148 * 4 + frames.n - 1) / frames.n;
    if (chunks > frames.max_len) chunks = frames.max_len;
    if (chunks < 1) chunks = 1;
    align_gather_kernel<<<dim3(chunks, frames.n), ALIGN_THREADS, 0, st>>>(dur, tok, frames, cat, te, en, asr,
                                                                         frame_tok, op, split);
}
void rowdot(const float* x, int T, int C, const float* w, const float* b, float* y, cudaStream_t st) {
    rowdot_kernel<<<rows_grid(T), 256, 0, st>>>(x, T, C, w, b, y);
}
void gather_rows(RowMeta m, const float* table, int D, float* out, OpPlanes op, bool split, cudaStream_t st) {
    gather_rows_kernel<<<m.R, 256, 0, st>>>(m, table, D, out, op, split);
}

}  // namespace rk
