// attention_tc.cu -- multi-head self-attention on the tensor cores (tcgen05 / TMEM).
//
// ALBERT (src/rokoko_f16.cpp:227-244: batched GEMM Q K^T, softmax kernel
// src/kernels.cu:189-225, batched GEMM P V; src/rokoko.cpp:363-384) and the
// neural phonemizer (src/g2p.h:772-790): S = Q K^T / 8 per head of 64
// dimensions, softmax over the keys (no mask), O = P V, for every sequence of
// a batch (segments of the row layout).  QKV rows hold [Q | K | V] of `heads`
// heads each ([rows][3 * 64 heads]); the output rows are [rows][64 heads].
//
// One CTA of 128 threads per (128-query tile, head, sequence):
//   1. Q [128 x 64] and, in chunks of 64 keys, K [64 x 64] are converted from
//      the FP32 QKV rows into 16-bit planes in shared memory (the 128-byte
//      swizzled K-major layout the MMA reads; FP32 semantics keep bf16 hi and
//      lo planes and issue hi*hi + hi*lo + lo*hi), and one elected thread
//      issues S[:, 64c .. 64c+64) = Q K_c^T into TMEM (M = 128 queries,
//      N = 64 keys, K = 64 dims), chunks double-buffered behind mbarriers.
//   2. Thread i owns query row i = TMEM lane i: it reads its scores straight
//      from TMEM (tcgen05.ld), takes the row maximum, then per key chunk
//      computes e = exp(s / 8 - max) (0 past the sequence's keys), adds it to
//      the row sum and writes the row of E_c into shared memory; V_c is
//      written transposed (dims x keys) beside it; the elected thread issues
//      O += E_c V_c into TMEM.
//   3. O row / sum -> output.
// Up to 512 keys the scores of all keys sit in TMEM at once and O takes the
// columns of chunk 0 once they are read.  Longer sequences run in key blocks
// of 448 (seven chunks; O in columns 448..511): per block the running row
// maximum is raised to the block's and O and the row sum are rescaled by
// exp(old max - new max) before the block's E V products (online softmax).
// The scores never leave the SM.  Every wait is bounded (ptx.cuh): a timeout
// records an error code in the context's error word and the CTA finishes
// without writing (the host reports RK_ERR_DEVICE_TIMEOUT).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "front_ops.cuh"
#include "ptx.cuh"

namespace rk {

namespace {

constexpr int QT = 128;   // queries per CTA (the MMA M)
constexpr int KC = 64;    // keys per chunk (the S MMA N, the O MMA K)
constexpr int HD = 64;    // head dim
constexpr uint32_t ROWB = 128;  // bytes per 64-element 16-bit row

// NBUF buffers of the K, E and V tiles: 2 lets the next chunk's conversion run
// beside the current chunk's MMA; 1 halves their shared memory (split-bf16:
// 96 KB instead of 160 KB), so that two CTAs share an SM.
template <bool SPLIT, int NBUF>
struct AttCfg {
    static constexpr int NPL = SPLIT ? 2 : 1;
    static constexpr uint32_t Q_PLANE = QT * ROWB;    // 16 KB
    static constexpr uint32_t K_PLANE = KC * ROWB;    // 8 KB
    static constexpr uint32_t E_PLANE = QT * ROWB;    // 16 KB
    static constexpr uint32_t V_PLANE = HD * ROWB;    // 8 KB
    static constexpr uint32_t Q_OFF = 0;
    static constexpr uint32_t K_OFF = Q_OFF + NPL * Q_PLANE;
    static constexpr uint32_t E_OFF = K_OFF + NBUF * NPL * K_PLANE;
    static constexpr uint32_t V_OFF = E_OFF + NBUF * NPL * E_PLANE;
    static constexpr uint32_t BYTES = V_OFF + NBUF * NPL * V_PLANE;
};

// byte offset of 16-bit element (r, k) of a [rows][64] tile in the 128-byte swizzle
__device__ __forceinline__ uint32_t sw_off(int r, int k) {
    return (uint32_t)r * ROWB + ((((uint32_t)k >> 3) ^ ((uint32_t)r & 7u)) << 4) + (((uint32_t)k & 7u) << 1);
}

// 8 FP32 values -> one 16-byte chunk of the hi plane (and the lo plane when split)
template <bool SPLIT>
__device__ __forceinline__ void put8(uint8_t* hi, uint8_t* lo, uint32_t off, const float (&v)[8]) {
    if (SPLIT) {
        __align__(16) __nv_bfloat16 h[8], l[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            h[j] = __float2bfloat16_rn(v[j]);
            l[j] = __float2bfloat16_rn(v[j] - __bfloat162float(h[j]));
        }
        *reinterpret_cast<uint4*>(hi + off) = *reinterpret_cast<uint4*>(h);
        *reinterpret_cast<uint4*>(lo + off) = *reinterpret_cast<uint4*>(l);
    } else {
        __align__(16) __half h[8];
#pragma unroll
        for (int j = 0; j < 8; j++) h[j] = __float2half_rn(v[j]);
        *reinterpret_cast<uint4*>(hi + off) = *reinterpret_cast<uint4*>(h);
    }
}

__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// D (+)= A B^T over one 64-wide K block: 4 MMAs of K = 16 (x3 products when split)
template <bool SPLIT>
__device__ __forceinline__ void mma_block(uint32_t d_tmem, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi,
                                          uint32_t b_lo, uint32_t idesc, bool accumulate) {
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
        const uint64_t ah = sw128_kmajor_desc(a_hi + kk * 32, 0), bh = sw128_kmajor_desc(b_hi + kk * 32, 0);
        umma_f16(d_tmem, ah, bh, idesc, (accumulate || kk > 0) ? 1u : 0u);
        if (SPLIT) {
            umma_f16(d_tmem, ah, sw128_kmajor_desc(b_lo + kk * 32, 0), idesc, 1u);
            umma_f16(d_tmem, sw128_kmajor_desc(a_lo + kk * 32, 0), bh, idesc, 1u);
        }
    }
}

constexpr int BLOCK_CHUNKS = 7;      // key chunks per block beyond 512 keys
constexpr uint32_t O_COL_BLOCKED = 448;  // O's TMEM columns when the keys run in blocks

template <bool SPLIT, int NBUF>
__global__ void __launch_bounds__(128) attention_tc_kernel(const float* __restrict__ qkv_all, SegMeta s,
                                                           float* __restrict__ ctx_all, int hid, uint32_t* err) {
    using C = AttCfg<SPLIT, NBUF>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t s_bar[2], pv_bar[2], fin_bar;
    __shared__ uint32_t tmem_base_sh;

    const int T = s.len[blockIdx.z];
    const int q0 = blockIdx.x * QT;
    if (q0 >= T) return;  // uniform over the CTA
    const int head = blockIdx.y;
    const int ld = 3 * hid;  // QKV row pitch
    const float* qkv = qkv_all + (size_t)s.off[blockIdx.z] * ld;
    const int tid = threadIdx.x, warp = tid >> 5;
    const int nch = (T + KC - 1) / KC;
    const bool single = nch * KC <= 512;  // every key's score in TMEM at once
    const int bch = single ? nch : BLOCK_CHUNKS;
    const uint32_t o_col = single ? 0u : O_COL_BLOCKED;
    uint32_t ncols = 64;
    while ((int)ncols < (single ? nch * KC : 512)) ncols <<= 1;

    if (tid == 0) {
        for (int i = 0; i < 2; i++) { mbar_init(&s_bar[i], 1); mbar_init(&pv_bar[i], 1); }
        mbar_init(&fin_bar, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&tmem_base_sh, ncols);
        tmem_relinquish();
    }
    // ---- Q tile: thread t = query row q0 + t (zeros past T)
    {
        uint8_t* qh = smem + C::Q_OFF;
        uint8_t* ql = qh + C::Q_PLANE;
        const int q = q0 + tid;
        const float* src = qkv + (size_t)q * ld + head * HD;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            float v[8];
            if (q < T) {
                const float4 a = reinterpret_cast<const float4*>(src + 8 * j)[0];
                const float4 b = reinterpret_cast<const float4*>(src + 8 * j)[1];
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) v[i] = 0.f;
            }
            put8<SPLIT>(qh, ql, sw_off(tid, 8 * j), v);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;
    const uint32_t idesc = umma_idesc_f16(QT, KC, SPLIT);
    const uint32_t q_hi = smem_u32(smem + C::Q_OFF), q_lo = q_hi + C::Q_PLANE;
    bool ok = true;

    const uint32_t row_tmem = tmem + ((uint32_t)(warp * 32) << 16);
    float mx = -3.0e38f, sum = 0.f;
    int gs = 0, gp = 0;        // S and E V chunks issued so far (mbarrier phases)
    uint32_t fin_n = 0;        // uses of fin_bar so far
    for (int c0 = 0; c0 < nch && ok; c0 += bch) {
        const int c1 = min(nch, c0 + bch);
        // ---- phase S: scores of the block's key chunks into TMEM columns [64 (c - c0), +64)
        for (int c = c0; c < c1; c++, gs++) {
            const int buf = gs % NBUF;  // the S MMA that last read this K buffer must be done
            if (gs >= NBUF && !mbar_wait(&s_bar[buf], ((gs - NBUF) / NBUF) & 1, err, RK_DEV_TIMEOUT_FULL)) ok = false;
            if (!__syncthreads_and(ok)) break;
            uint8_t* kh = smem + C::K_OFF + buf * C::NPL * C::K_PLANE;
            uint8_t* kl = kh + C::K_PLANE;
            {   // key row t >> 1, dims [32 (t & 1), +32)
                const int kr = tid >> 1, half = tid & 1;
                const int key = c * KC + kr;
                const float* src = qkv + (size_t)key * ld + hid + head * HD + 32 * half;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    float v[8];
                    if (key < T) {
                        const float4 a = reinterpret_cast<const float4*>(src + 8 * j)[0];
                        const float4 b = reinterpret_cast<const float4*>(src + 8 * j)[1];
                        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
                    } else {
#pragma unroll
                        for (int i = 0; i < 8; i++) v[i] = 0.f;
                    }
                    put8<SPLIT>(kh, kl, sw_off(kr, 32 * half + 8 * j), v);
                }
            }
            fence_async_smem();
            tc_fence_before();
            __syncthreads();
            if (tid == 0) {
                tc_fence_after();
                const uint32_t k_hi = smem_u32(kh), k_lo = k_hi + C::K_PLANE;
                mma_block<SPLIT>(tmem + (uint32_t)((c - c0) * KC), q_hi, q_lo, k_hi, k_lo, idesc, false);
                umma_commit(&s_bar[buf]);
            }
        }
        // the block's scores (and every earlier E V product) have landed
        if (tid == 0 && ok) umma_commit(&fin_bar);
        if (ok && !mbar_wait(&fin_bar, fin_n & 1u, err, RK_DEV_TIMEOUT_ACC)) ok = false;
        fin_n++;
        ok = __syncthreads_and(ok);
        tc_fence_after();
        if (!ok) break;
        // ---- pass A: row maximum of the scaled scores over the block's keys
        float bmx = mx;
        for (int c = c0; c < c1; c++) {
#pragma unroll
            for (int h = 0; h < 2; h++) {
                float v[32];
                tmem_ld32(row_tmem + (uint32_t)((c - c0) * KC + 32 * h), v);
#pragma unroll
                for (int j = 0; j < 32; j++)
                    if (c * KC + 32 * h + j < T) bmx = fmaxf(bmx, v[j] * 0.125f);
            }
        }
        if (c0 > 0) {
            // online softmax: O and the row sum so far to the new maximum (alpha = 1 when the
            // block does not raise it).  The condition is uniform over the CTA: tcgen05.ld / st
            // are .sync.aligned, every lane of a warp must execute them together.
            const float alpha = expf(mx - bmx);
            sum *= alpha;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                float v[32];
                tmem_ld32(row_tmem + o_col + (uint32_t)(32 * h), v);
#pragma unroll
                for (int j = 0; j < 32; j++) v[j] *= alpha;
                tmem_st32(row_tmem + o_col + (uint32_t)(32 * h), v);
            }
        }
        mx = bmx;
        // ---- pass B: e = exp(s / 8 - max) chunk by chunk, O += E_c V_c
        for (int c = c0; c < c1; c++, gp++) {
            const int buf = gp % NBUF;  // the E V MMA that last read these buffers must be done
            if (gp >= NBUF && !mbar_wait(&pv_bar[buf], ((gp - NBUF) / NBUF) & 1, err, RK_DEV_TIMEOUT_FULL)) ok = false;
            if (!__syncthreads_and(ok)) break;
            uint8_t* eh = smem + C::E_OFF + buf * C::NPL * C::E_PLANE;
            uint8_t* el = eh + C::E_PLANE;
            uint8_t* vh = smem + C::V_OFF + buf * C::NPL * C::V_PLANE;
            uint8_t* vl = vh + C::V_PLANE;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                float v[32];
                tmem_ld32(row_tmem + (uint32_t)((c - c0) * KC + 32 * h), v);
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    const float e = (c * KC + 32 * h + j < T) ? expf(v[j] * 0.125f - mx) : 0.f;
                    sum += e;
                    v[j] = e;
                }
#pragma unroll
                for (int g = 0; g < 4; g++) {
                    float w[8];
#pragma unroll
                    for (int i = 0; i < 8; i++) w[i] = v[8 * g + i];
                    put8<SPLIT>(eh, el, sw_off(tid, 32 * h + 8 * g), w);
                }
            }
            {   // V_c transposed: thread t -> dim t & 63, keys 32 (t >> 6) .. +32 in chunks of 8
                const int d = tid & 63, kh0 = (tid >> 6) * 32;
#pragma unroll
                for (int g = 0; g < 4; g++) {
                    float w[8];
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int key = c * KC + kh0 + 8 * g + i;
                        w[i] = key < T ? qkv[(size_t)key * ld + 2 * hid + head * HD + d] : 0.f;
                    }
                    put8<SPLIT>(vh, vl, sw_off(d, kh0 + 8 * g), w);
                }
            }
            fence_async_smem();
            tc_fence_before();
            __syncthreads();
            if (tid == 0) {
                tc_fence_after();
                const uint32_t e_hi = smem_u32(eh), e_lo = e_hi + C::E_PLANE;
                const uint32_t v_hi = smem_u32(vh), v_lo = v_hi + C::V_PLANE;
                mma_block<SPLIT>(tmem + o_col, e_hi, e_lo, v_hi, v_lo, idesc, gp > 0);
                umma_commit(&pv_bar[buf]);
            }
        }
    }
    if (tid == 0 && ok) umma_commit(&fin_bar);
    if (ok && !mbar_wait(&fin_bar, fin_n & 1u, err, RK_DEV_TIMEOUT_ACC)) ok = false;
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (ok) {
        // ---- O / sum -> ctx (row q0 + t, columns head*64 ..)
        const int q = q0 + tid;
        const float inv = 1.0f / sum;
        float* dst = ctx_all + ((size_t)s.off[blockIdx.z] + q) * hid + head * HD;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            float v[32];
            tmem_ld32(row_tmem + o_col + (uint32_t)(32 * h), v);
            if (q < T) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4*>(dst + 32 * h + j) =
                        make_float4(v[j] * inv, v[j + 1] * inv, v[j + 2] * inv, v[j + 3] * inv);
            }
        }
    }
    // every MMA this CTA issued has completed once its commits land; drain before freeing TMEM
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, ncols);
    }
}

template <bool SPLIT, int NBUF>
constexpr size_t att_smem() {
    return AttCfg<SPLIT, NBUF>::BYTES + 1024;
}

template <bool SPLIT, int NBUF>
cudaError_t att_attr() {
    return cudaFuncSetAttribute(attention_tc_kernel<SPLIT, NBUF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)att_smem<SPLIT, NBUF>());
}

template <bool SPLIT, int NBUF>
void att_launch(dim3 grid, const float* qkv, SegMeta s, float* ctx, int hid, uint32_t* err, cudaStream_t st) {
    attention_tc_kernel<SPLIT, NBUF><<<grid, 128, att_smem<SPLIT, NBUF>(), st>>>(qkv, s, ctx, hid, err);
}

}  // namespace

cudaError_t attention_tc_init() {
    cudaError_t e;
    if ((e = att_attr<true, 1>()) || (e = att_attr<true, 2>()) || (e = att_attr<false, 1>()) ||
        (e = att_attr<false, 2>()))
        return e;
    return cudaSuccess;
}

cudaError_t attention_tc(const float* qkv, SegMeta s, float* ctx, bool split, uint32_t* err, cudaStream_t st,
                         int heads) {
    if (heads < 1 || s.n < 1 || s.max_len < 1) return heads < 1 ? cudaErrorInvalidValue : cudaSuccess;
    const dim3 grid((s.max_len + QT - 1) / QT, heads, s.n);
    const int hid = heads * HD;
    // up to 512 keys (every key's scores in TMEM at once): single K / E / V buffers, two CTAs per
    // SM; longer sequences (key blocks with online rescaling) keep two buffers.  The arithmetic
    // is the same either way.
    const bool single = s.max_len <= 512;
    if (split) single ? att_launch<true, 1>(grid, qkv, s, ctx, hid, err, st)
                      : att_launch<true, 2>(grid, qkv, s, ctx, hid, err, st);
    else single ? att_launch<false, 1>(grid, qkv, s, ctx, hid, err, st)
                : att_launch<false, 2>(grid, qkv, s, ctx, hid, err, st);
    return cudaGetLastError();
}

}  // namespace rk
