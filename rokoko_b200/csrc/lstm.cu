// lstm.cu -- persistent bidirectional LSTM recurrence for many sequences at
// once, on thread-block clusters.
//
// The reference runs each timestep as two launches per direction (a GEMV
// Whh h and a gates kernel, src/rokoko.cpp:484-550, src/kernels.cu:976-1045),
// ~4 T graph nodes per BiLSTM and one utterance at a time.  Here one launch
// runs the whole recurrence of every sequence of a batch: one cluster of 8
// CTAs per (group of up to MAX_GROUP sequences, direction); CTA r owns hidden
// units [32r, 32r+32), i.e. 128 gate rows (i, f, g, o of its units) x 256 of
// Whh, resident in shared memory (128 KB) for all steps and shared by the
// group's sequences.  Per step every CTA computes its 128 gate
// pre-activations of each sequence from that sequence's full h_{t-1}, updates
// its 32 cells per sequence, and broadcasts the new h values into every CTA's
// shared memory (DSMEM); a hardware cluster barrier (release/acquire)
// separates the steps.  No spin-waits.  Sequences of a group may differ in
// length: the group runs max(len) steps and a sequence stops writing after
// its own length (the reverse direction starts at each sequence's own end).
// A sequence's arithmetic (the order of every product and sum) does not
// depend on the group it is in, so a batched utterance gives the same bits as
// the same utterance alone.
#include <cooperative_groups.h>

#include "front_ops.cuh"

namespace cg = cooperative_groups;

namespace rk {

namespace {

constexpr int CTAS = 8, H = 256, ROWS = 128, MAX_GROUP = 8;
constexpr size_t LSTM_SMEM =
    (size_t)(64 * ROWS * 4 + 2 * MAX_GROUP * H + 2 * MAX_GROUP * ROWS + MAX_GROUP * ROWS) * sizeof(float);

__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

template <int G>
__global__ void __cluster_dims__(CTAS, 1, 1) __launch_bounds__(256, 1)
    bilstm_kernel(const float* __restrict__ ig, const float* __restrict__ whh, SegMeta seq, float* __restrict__ out) {
    extern __shared__ float4 sm4[];
    float4* W = sm4;                                          // [64 k4][128 rows] of 4 consecutive k
    float* hbuf = reinterpret_cast<float*>(sm4 + 64 * ROWS);  // [2][G][256]
    float* part = hbuf + 2 * MAX_GROUP * H;                   // [2 halves][G][128] half dot products
    float* gsh = part + 2 * MAX_GROUP * ROWS;                 // [G][128] gate pre-activations
    cg::cluster_group cluster = cg::this_cluster();
    const int r = (int)cluster.block_rank();
    const int cl = blockIdx.x / CTAS;
    const int dir = cl & 1, grp = cl >> 1;
    const int first = grp * G;
    const int ng = min(G, seq.n - first);
    const int tid = threadIdx.x;
    int my_off[G], my_len[G], steps = 0;
#pragma unroll
    for (int s = 0; s < G; s++) {
        my_off[s] = s < ng ? seq.off[first + s] : 0;
        my_len[s] = s < ng ? seq.len[first + s] : 0;
        steps = max(steps, my_len[s]);
    }
    // local row lr = q*32 + u  <->  global gate row q*256 + 32r + u
    for (int e = tid; e < ROWS * 64; e += blockDim.x) {
        const int lr = e / 64, k4 = e % 64;
        const int grow = (lr / 32) * H + r * 32 + (lr % 32);
        const float4 v = *reinterpret_cast<const float4*>(whh + ((size_t)dir * 1024 + grow) * H + 4 * k4);
        W[k4 * ROWS + lr] = v;
    }
    for (int k = tid; k < 2 * G * H; k += blockDim.x) hbuf[k] = 0.f;
    float c = 0.f;  // cell of (sequence tid / 32, unit tid % 32) for tid < 32 G
    cluster.sync();
    const int lr = tid & (ROWS - 1), half = tid >> 7;
    const int grow = (lr / 32) * H + r * 32 + (lr % 32);
    for (int step = 0; step < steps; step++) {
        const float* hcur = hbuf + (step & 1) * G * H;
        float acc[G];
#pragma unroll
        for (int s = 0; s < G; s++) acc[s] = 0.f;
#pragma unroll 4
        for (int k4 = half * 32; k4 < half * 32 + 32; k4++) {
            const float4 w = W[k4 * ROWS + lr];
#pragma unroll
            for (int s = 0; s < G; s++) {
                const float4 h = reinterpret_cast<const float4*>(hcur + s * H)[k4];
                acc[s] += w.x * h.x;
                acc[s] += w.y * h.y;
                acc[s] += w.z * h.z;
                acc[s] += w.w * h.w;
            }
        }
#pragma unroll
        for (int s = 0; s < G; s++) part[(half * G + s) * ROWS + lr] = acc[s];
        __syncthreads();
        if (half == 0) {
#pragma unroll
            for (int s = 0; s < G; s++)
                if (step < my_len[s]) {
                    const int t = dir ? my_len[s] - 1 - step : step;
                    gsh[s * ROWS + lr] = ig[(size_t)(my_off[s] + t) * 2048 + dir * 1024 + grow] +
                                         (part[s * ROWS + lr] + part[(G + s) * ROWS + lr]);
                }
        }
        __syncthreads();
        if (tid < 32 * G) {
            const int s = tid >> 5, u = tid & 31;
            if (step < my_len[s]) {
                const float* g = gsh + s * ROWS;
                const float ii = sigm(g[u]);
                const float ff = sigm(g[32 + u]);
                const float gg = tanhf(g[64 + u]);
                const float oo = sigm(g[96 + u]);
                c = ff * c + ii * gg;
                const float h = oo * tanhf(c);
                const int t = dir ? my_len[s] - 1 - step : step;
                out[(size_t)(my_off[s] + t) * 512 + dir * H + r * 32 + u] = h;
                float* slot = hbuf + ((step + 1) & 1) * G * H + s * H + r * 32 + u;
#pragma unroll
                for (int dst = 0; dst < CTAS; dst++) *cluster.map_shared_rank(slot, dst) = h;
            }
        }
        cluster.sync();
    }
}

template <int G>
cudaError_t launch_g(const float* ig, const float* whh, SegMeta seq, float* out, cudaStream_t st) {
    const int groups = (seq.n + G - 1) / G;
    bilstm_kernel<G><<<2 * groups * CTAS, 256, LSTM_SMEM, st>>>(ig, whh, seq, out);
    return cudaGetLastError();
}

}  // namespace

cudaError_t bilstm_init() {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(bilstm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)LSTM_SMEM)) ||
        (e = cudaFuncSetAttribute(bilstm_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)LSTM_SMEM)) ||
        (e = cudaFuncSetAttribute(bilstm_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)LSTM_SMEM)) ||
        (e = cudaFuncSetAttribute(bilstm_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)LSTM_SMEM)))
        return e;
    return cudaSuccess;
}

int bilstm_group(int n) {
    // 148 SMs hold 18 eight-CTA clusters (one CTA per SM: 128 KB of weights each);
    // two directions per group
    const int clusters = 148 / CTAS;
    for (int g = 1; g < MAX_GROUP; g *= 2)
        if (2 * ((n + g - 1) / g) <= clusters) return g;
    return MAX_GROUP;
}

cudaError_t bilstm_recurrence(const float* ig, const float* whh, SegMeta seq, int group, float* out,
                              cudaStream_t st) {
    if (seq.n < 1 || seq.max_len < 1) return cudaSuccess;
    switch (group) {
        case 1: return launch_g<1>(ig, whh, seq, out, st);
        case 2: return launch_g<2>(ig, whh, seq, out, st);
        case 4: return launch_g<4>(ig, whh, seq, out, st);
        default: return launch_g<8>(ig, whh, seq, out, st);
    }
}

}  // namespace rk
