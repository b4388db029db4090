// lstm.cu -- persistent bidirectional LSTM recurrence on thread-block clusters.
//
// The reference runs each timestep as two launches per direction (a GEMV
// Whh h and a gates kernel, src/rokoko.cpp:484-550, src/kernels.cu:976-1045),
// ~4 T graph nodes per BiLSTM.  Here one launch runs the whole recurrence:
// one cluster of 8 CTAs per direction; CTA r owns hidden units [32r, 32r+32),
// i.e. 128 gate rows (i, f, g, o of its units) x 256 of Whh, resident in shared
// memory (128 KB) for all steps.  Per step every CTA computes its 128 gate
// pre-activations from the full h_{t-1}, updates its 32 cells, and broadcasts
// its 32 new h values into every CTA's shared memory (DSMEM); a hardware
// cluster barrier (release/acquire) separates the steps.  No spin-waits.
#include <cooperative_groups.h>

#include "front_ops.cuh"

namespace cg = cooperative_groups;

namespace rk {

namespace {

constexpr int CTAS = 8, H = 256, ROWS = 128;
constexpr size_t LSTM_SMEM = (size_t)(64 * ROWS * 4 + 2 * H + 2 * ROWS + ROWS) * sizeof(float);

__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

__global__ void __cluster_dims__(CTAS, 1, 1) __launch_bounds__(256, 1)
    bilstm_kernel(const float* __restrict__ ig, const float* __restrict__ whh, int T, float* __restrict__ out) {
    extern __shared__ float4 sm4[];
    float4* W = sm4;                                     // [64 k4][128 rows] of 4 consecutive k
    float* hbuf = reinterpret_cast<float*>(sm4 + 64 * ROWS);  // [2][256]
    float* part = hbuf + 2 * H;                          // [2][128] half dot products
    float* g = part + 2 * ROWS;                          // [128] gate pre-activations
    cg::cluster_group cluster = cg::this_cluster();
    const int r = (int)cluster.block_rank();
    const int dir = blockIdx.x / CTAS;
    const int tid = threadIdx.x;
    // local row lr = q*32 + u  <->  global gate row q*256 + 32r + u
    for (int e = tid; e < ROWS * 64; e += blockDim.x) {
        const int lr = e / 64, k4 = e % 64;
        const int grow = (lr / 32) * H + r * 32 + (lr % 32);
        const float4 v = *reinterpret_cast<const float4*>(whh + ((size_t)dir * 1024 + grow) * H + 4 * k4);
        W[k4 * ROWS + lr] = v;
    }
    for (int k = tid; k < 2 * H; k += blockDim.x) hbuf[k] = 0.f;
    float c = 0.f;
    cluster.sync();
    const int lr = tid & (ROWS - 1), half = tid >> 7;
    const int grow = (lr / 32) * H + r * 32 + (lr % 32);
    for (int step = 0; step < T; step++) {
        const int t = dir ? T - 1 - step : step;
        const float4* hc = reinterpret_cast<const float4*>(hbuf + (step & 1) * H);
        float acc = 0.f;
#pragma unroll 8
        for (int k4 = half * 32; k4 < half * 32 + 32; k4++) {
            const float4 w = W[k4 * ROWS + lr];
            const float4 h = hc[k4];
            acc += w.x * h.x;
            acc += w.y * h.y;
            acc += w.z * h.z;
            acc += w.w * h.w;
        }
        part[half * ROWS + lr] = acc;
        __syncthreads();
        if (half == 0) g[lr] = ig[(size_t)t * 2048 + dir * 1024 + grow] + (part[lr] + part[ROWS + lr]);
        __syncthreads();
        if (tid < 32) {
            const int u = tid;
            const float ii = sigm(g[u]);
            const float ff = sigm(g[32 + u]);
            const float gg = tanhf(g[64 + u]);
            const float oo = sigm(g[96 + u]);
            c = ff * c + ii * gg;
            const float h = oo * tanhf(c);
            out[(size_t)t * 512 + dir * H + r * 32 + u] = h;
            float* slot = hbuf + ((step + 1) & 1) * H + r * 32 + u;
#pragma unroll
            for (int dst = 0; dst < CTAS; dst++) *cluster.map_shared_rank(slot, dst) = h;
        }
        cluster.sync();
    }
}

}  // namespace

cudaError_t bilstm_init() {
    return cudaFuncSetAttribute(bilstm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)LSTM_SMEM);
}

cudaError_t bilstm_recurrence(const float* ig, const float* whh, int T, float* out, uint32_t*, cudaStream_t st) {
    if (T < 1) return cudaSuccess;
    bilstm_kernel<<<2 * CTAS, 256, LSTM_SMEM, st>>>(ig, whh, T, out);
    return cudaGetLastError();
}

}  // namespace rk
