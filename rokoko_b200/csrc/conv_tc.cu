// conv_tc.cu -- tcgen05 / TMEM implicit-GEMM Conv1d for sm_100a.
//
// Replaces the reference's CUTLASS-2.x Sm80 implicit-GEMM convolutions
// (src/cutlass_conv.cu:239-313, src/cutlass_conv_f16.cu:216-273), its
// im2col + GEMM fallback (src/rokoko.cpp:286-302) and the GEMM + atomic col2im
// ConvTranspose1d (src/rokoko.cpp:308-329, src/kernels.cu:1141-1173).
//
// CTA = 6 warps, one 128-row x NB-column output tile, two CTAs per SM:
//   warp 0   TMA producer.  Per 64-channel block it loads ONE activation tile
//            of H = 128 + halo rows (halo = max tap offset - min tap offset;
//            TMA zero-fills rows outside [0, T_in), i.e. the padding), and per
//            (channel block, tap) one weight tile.
//   warp 1   owns TMEM; one elected thread issues tcgen05.mma (M=128, N=NB,
//            K=16 each, 4 per 64-channel block, x3 in split mode).  Tap k
//            reuses the activation tile through a descriptor whose start is
//            shifted by (tap_off[k] - min_off) rows, so the activations cross
//            L2 -> SMEM once per channel block instead of once per tap.
//   warps 2-5 epilogue: tcgen05.ld 32 columns, transpose through shared memory
//            and process the tile as coalesced float4 row segments: bias,
//            residual, accumulate, scale, store, plus per-channel sum and
//            sum-of-squares partials for the next InstanceNorm.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "conv_tc.cuh"
#include "ptx.cuh"

namespace rk {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int MAX_HPAD = 184;       // halo tile rows (128 + halo <= 178, padded to 8)
constexpr int STAGE_PAD = 36;       // epilogue staging row pitch (floats)

template <int NB, bool SPLIT>
struct Cfg {
    static constexpr int NPL = SPLIT ? 2 : 1;
    static constexpr uint32_t B_BYTES = NB * BK * 2;          // one plane
    static constexpr uint32_t B_STAGE = NPL * B_BYTES;
    // budget: two CTAs per SM (<= ~113 KB each)
    static constexpr int B_STAGES = SPLIT ? 2 : 4;
    static constexpr uint32_t TMEM_COLS = NB < 32 ? 32 : NB;
    static constexpr size_t smem_bytes(int H_pad) {
        return 1024 + (size_t)NPL * H_pad * 128 + (size_t)B_STAGES * B_STAGE;
    }
    static constexpr size_t SMEM_MAX = 1024 + (size_t)NPL * MAX_HPAD * 128 + (size_t)B_STAGES * B_STAGE;
};

// gelu_new: 0.5 v (1 + tanh(0.7978845608 (v + 0.044715 v^3)))
__device__ __forceinline__ float gelu_tanh(float v) {
    const float inner = 0.7978845608028654f * (v + 0.044715f * v * v * v);
    return 0.5f * v * (1.0f + tanhf(inner));
}

template <int NB, bool SPLIT>
__global__ void __launch_bounds__(192, 2)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmA_hi, const __grid_constant__ CUtensorMap tmA_lo,
                   const __grid_constant__ CUtensorMap tmB_hi, const __grid_constant__ CUtensorMap tmB_lo,
                   const __grid_constant__ ConvArgs args) {
    using C = Cfg<NB, SPLIT>;
    constexpr int BS = C::B_STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t a_full, a_empty, acc_bar;
    __shared__ __align__(8) uint64_t b_full[BS], b_empty[BS];
    __shared__ uint32_t tmem_base_sh;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tile = blockIdx.x, n_tile = blockIdx.y, phase = blockIdx.z;
    const int m0 = m_tile * BM, n0 = n_tile * NB;
    const int H_pad = args.h_pad;
    const uint32_t a_plane = (uint32_t)H_pad * 128;
    uint8_t* a_buf = smem;                                   // [plane][H_pad rows][128 B]
    uint8_t* b_buf = smem + C::NPL * a_plane;                // [stage][plane][NB rows][128 B]
    const int KB = args.kblocks, TAPS = args.taps;

    if (warp == 0 && lane == 0) {
        mbar_init(&a_full, 1);
        mbar_init(&a_empty, 1);
        mbar_init(&acc_bar, 1);
        for (int s = 0; s < BS; s++) { mbar_init(&b_full[s], 1); mbar_init(&b_empty[s], 1); }
        fence_mbar_init();
        tma_prefetch_desc(&tmA_hi);
        tma_prefetch_desc(&tmB_hi);
        if (SPLIT) { tma_prefetch_desc(&tmA_lo); tma_prefetch_desc(&tmB_lo); }
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            const int brow = phase * args.b_phase_rows + n0;
            const int arow = m0 + args.a_off + args.min_off;
            int bit = 0;
            bool alive = true;
            for (int kb = 0; kb < KB && alive; kb++) {
                // the single activation buffer is free once every MMA of the previous block completed
                if (!mbar_wait(&a_empty, ((uint32_t)kb & 1u) ^ 1u, args.err, RK_DEV_TIMEOUT_EMPTY)) break;
                mbar_arrive_expect_tx(&a_full, C::NPL * a_plane);
                tma_load_2d(a_buf, &tmA_hi, &a_full, kb * BK, arow);
                if (SPLIT) tma_load_2d(a_buf + a_plane, &tmA_lo, &a_full, kb * BK, arow);
                for (int tap = 0; tap < TAPS; tap++, bit++) {
                    const int s = bit % BS;
                    const uint32_t round = (uint32_t)(bit / BS);
                    if (!mbar_wait(&b_empty[s], (round & 1u) ^ 1u, args.err, RK_DEV_TIMEOUT_EMPTY)) {
                        alive = false;
                        break;
                    }
                    uint8_t* sb = b_buf + (size_t)s * C::B_STAGE;
                    mbar_arrive_expect_tx(&b_full[s], C::B_STAGE);
                    const int bx = (tap * KB + kb) * BK;
                    tma_load_2d(sb, &tmB_hi, &b_full[s], bx, brow);
                    if (SPLIT) tma_load_2d(sb + C::B_BYTES, &tmB_lo, &b_full[s], bx, brow);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(BM, NB, SPLIT);
            const uint32_t a_hi = smem_u32(a_buf), a_lo = a_hi + a_plane;
            int bit = 0;
            bool alive = true;
            for (int kb = 0; kb < KB && alive; kb++) {
                if (!mbar_wait(&a_full, (uint32_t)kb & 1u, args.err, RK_DEV_TIMEOUT_FULL)) break;
                tc_fence_after();
                for (int tap = 0; tap < TAPS; tap++, bit++) {
                    const int s = bit % BS;
                    const uint32_t round = (uint32_t)(bit / BS);
                    if (!mbar_wait(&b_full[s], round & 1u, args.err, RK_DEV_TIMEOUT_FULL)) {
                        alive = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t shift = (uint32_t)(args.tap_off[tap] - args.min_off) * 128u;
                    const uint32_t b_hi = smem_u32(b_buf + (size_t)s * C::B_STAGE), b_lo = b_hi + C::B_BYTES;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; kk++) {
                        const uint64_t dah = sw128_kmajor_desc(a_hi + shift + kk * 32, args.desc_mode);
                        const uint64_t dbh = sw128_kmajor_desc(b_hi + kk * 32, 0);
                        umma_f16(tmem, dah, dbh, idesc, (kb > 0 || tap > 0 || kk > 0) ? 1u : 0u);
                        if (SPLIT) {
                            umma_f16(tmem, dah, sw128_kmajor_desc(b_lo + kk * 32, 0), idesc, 1u);
                            umma_f16(tmem, sw128_kmajor_desc(a_lo + shift + kk * 32, args.desc_mode), dbh, idesc,
                                     1u);
                        }
                    }
                    umma_commit(&b_empty[s]);
                }
                umma_commit(&a_empty);
            }
            umma_commit(&acc_bar);
            // every MMA this thread issued has completed once acc_bar flips
            mbar_wait(&acc_bar, 0, args.err, RK_DEV_TIMEOUT_DRAIN);
        }
    } else {
        // ------------------------------------------------ epilogue (warps 2..5)
        const int wq = warp & 3;  // TMEM lane quarter this warp may access
        const bool ok = mbar_wait(&acc_bar, 0, args.err, RK_DEV_TIMEOUT_ACC);
        tc_fence_after();
        // every MMA has completed, so the operand buffers are free: stage through them
        float* stg = reinterpret_cast<float*>(smem) + (size_t)wq * 32 * STAGE_PAD;
        float* red = reinterpret_cast<float*>(smem) + 4 * 32 * STAGE_PAD;  // [2][4][NB]
        const bool want_stats = args.stats != nullptr;
        const int cg = lane & 7;        // 4-column group within the 32-column chunk
        const int rsub = lane >> 3;     // row within a group of 4
#pragma unroll 1
        for (int c = 0; c < NB / 32; c++) {
            float v[32];
            tmem_ld32(tmem + ((uint32_t)(wq * 32) << 16) + (uint32_t)(c * 32), v);
#pragma unroll
            for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<float4*>(stg + lane * STAGE_PAD + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            __syncwarp();
            const int co = n0 + c * 32 + cg * 4;
            const int ncol = min(4, args.C_out - co);
            float4 bias4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (args.bias && ncol > 0) {
                bias4.x = args.bias[co];
                if (ncol > 1) bias4.y = args.bias[co + 1];
                if (ncol > 2) bias4.z = args.bias[co + 2];
                if (ncol > 3) bias4.w = args.bias[co + 3];
            }
            float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f), q4 = s4;
#pragma unroll 2
            for (int i = 0; i < 8; i++) {
                const int r = i * 4 + rsub;
                const int m = m0 + wq * 32 + r;
                const int out_row = m * args.o_stride + args.o_off + phase * args.o_phase_step;
                const bool valid = ok && m < args.M && out_row >= args.o_min && out_row < args.T_out && ncol > 0;
                if (!valid) continue;
                const float4 a = *reinterpret_cast<const float4*>(stg + r * STAGE_PAD + cg * 4);
                const bool vec = ncol == 4;
                // main row, then (reflection pad) the duplicate written to row 0
                for (int pass = 0; pass < 2; pass++) {
                    int orow = out_row, rrow = out_row >> args.res_shift;
                    if (pass == 1) {
                        if (out_row != args.dup_src_row) break;
                        orow = 0;
                        rrow = 0;
                    }
                    float4 o = a;
                    if (args.res) {
                        const float* rp = args.res + (size_t)rrow * args.ldres + co;
                        if (vec && (args.ldres & 3) == 0) {
                            const float4 r4 = *reinterpret_cast<const float4*>(rp);
                            o.x += r4.x; o.y += r4.y; o.z += r4.z; o.w += r4.w;
                        } else {
                            o.x += rp[0];
                            if (ncol > 1) o.y += rp[1];
                            if (ncol > 2) o.z += rp[2];
                            if (ncol > 3) o.w += rp[3];
                        }
                    }
                    o.x += bias4.x; o.y += bias4.y; o.z += bias4.z; o.w += bias4.w;
                    if (args.act == 1) {
                        o.x = gelu_tanh(o.x); o.y = gelu_tanh(o.y); o.z = gelu_tanh(o.z); o.w = gelu_tanh(o.w);
                    }
                    if (args.acc_in) {
                        const float* ap = args.acc_in + (size_t)orow * args.ldacc + co;
                        o.x = ap[0] + o.x;
                        if (ncol > 1) o.y = ap[1] + o.y;
                        if (ncol > 2) o.z = ap[2] + o.z;
                        if (ncol > 3) o.w = ap[3] + o.w;
                    }
                    o.x *= args.alpha; o.y *= args.alpha; o.z *= args.alpha; o.w *= args.alpha;
                    float* yp = args.y + (size_t)orow * args.ldy + co;
                    if (vec && (args.ldy & 3) == 0) {
                        *reinterpret_cast<float4*>(yp) = o;
                    } else {
                        yp[0] = o.x;
                        if (ncol > 1) yp[1] = o.y;
                        if (ncol > 2) yp[2] = o.z;
                        if (ncol > 3) yp[3] = o.w;
                    }
                    if (ncol < 4) { o.w = 0.f; if (ncol < 3) o.z = 0.f; if (ncol < 2) o.y = 0.f; }
                    s4.x += o.x; s4.y += o.y; s4.z += o.z; s4.w += o.w;
                    q4.x += o.x * o.x; q4.y += o.y * o.y; q4.z += o.z * o.z; q4.w += o.w * o.w;
                }
            }
            if (want_stats) {
#pragma unroll
                for (int off = 8; off <= 16; off <<= 1) {
                    s4.x += __shfl_xor_sync(0xffffffffu, s4.x, off);
                    s4.y += __shfl_xor_sync(0xffffffffu, s4.y, off);
                    s4.z += __shfl_xor_sync(0xffffffffu, s4.z, off);
                    s4.w += __shfl_xor_sync(0xffffffffu, s4.w, off);
                    q4.x += __shfl_xor_sync(0xffffffffu, q4.x, off);
                    q4.y += __shfl_xor_sync(0xffffffffu, q4.y, off);
                    q4.z += __shfl_xor_sync(0xffffffffu, q4.z, off);
                    q4.w += __shfl_xor_sync(0xffffffffu, q4.w, off);
                }
                if (rsub == 0) {
                    float* rs = red + (size_t)wq * NB + c * 32 + cg * 4;
                    float* rq = red + (size_t)(4 + wq) * NB + c * 32 + cg * 4;
                    rs[0] = s4.x; rs[1] = s4.y; rs[2] = s4.z; rs[3] = s4.w;
                    rq[0] = q4.x; rq[1] = q4.y; rq[2] = q4.z; rq[3] = q4.w;
                }
            }
            __syncwarp();
        }
        if (want_stats) {
            asm volatile("bar.sync 1, 128;" ::: "memory");
            const int part = blockIdx.z * gridDim.x + blockIdx.x;
            for (int col = threadIdx.x - 64; col < NB; col += 128) {
                const int co = n0 + col;
                if (co < args.C_out) {
                    const float s = (red[0 * NB + col] + red[1 * NB + col]) + (red[2 * NB + col] + red[3 * NB + col]);
                    const float q = (red[4 * NB + col] + red[5 * NB + col]) + (red[6 * NB + col] + red[7 * NB + col]);
                    args.stats[(size_t)part * args.stats_ld + co] = s;
                    args.stats[(size_t)(args.stats_parts + part) * args.stats_ld + co] = q;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

template <int NB, bool SPLIT>
cudaError_t set_attr() {
    return cudaFuncSetAttribute(conv_tc_kernel<NB, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)Cfg<NB, SPLIT>::SMEM_MAX);
}

template <int NB, bool SPLIT>
cudaError_t launch_inst(const ConvOperands& ops, const ConvArgs& a, int n_phases, cudaStream_t stream) {
    using C = Cfg<NB, SPLIT>;
    const size_t smem = C::smem_bytes(a.h_pad);
    if (smem > C::SMEM_MAX) return cudaErrorInvalidValue;
    dim3 grid((a.M + BM - 1) / BM, (a.C_out + NB - 1) / NB, n_phases);
    conv_tc_kernel<NB, SPLIT><<<grid, 192, smem, stream>>>(ops.a_hi, SPLIT ? ops.a_lo : ops.a_hi, ops.b_hi,
                                                            SPLIT ? ops.b_lo : ops.b_hi, a);
    return cudaGetLastError();
}

}  // namespace

bool make_tmap_k64(CUtensorMap* m, const void* base, bool bf16, uint64_t cols, uint64_t rows, uint64_t ld,
                   uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * 2) & 15) || box_rows > 256 || box_rows == 0) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

cudaError_t conv_tc_init() {
    cudaError_t e;
    if ((e = set_attr<128, true>()) || (e = set_attr<128, false>()) || (e = set_attr<64, true>()) ||
        (e = set_attr<64, false>()) || (e = set_attr<32, true>()) || (e = set_attr<32, false>()))
        return e;
    return cudaSuccess;
}

int conv_tc_ntile(int C_out) {
    if (C_out > 64) return 128;
    if (C_out > 32) return 64;
    return 32;
}

int conv_tc_halo_rows(const int* tap_off, int taps) {
    int lo = tap_off[0], hi = tap_off[0];
    for (int k = 1; k < taps; k++) {
        lo = tap_off[k] < lo ? tap_off[k] : lo;
        hi = tap_off[k] > hi ? tap_off[k] : hi;
    }
    const int h = BM + hi - lo;
    return (h + 7) / 8 * 8;
}

cudaError_t conv_tc_launch(const ConvOperands& ops, const ConvArgs& a_in, bool split, int n_phases,
                           cudaStream_t stream) {
    if (a_in.taps < 1 || a_in.taps > CONV_MAX_TAPS || a_in.kblocks < 1 || a_in.M < 1) return cudaErrorInvalidValue;
    ConvArgs a = a_in;
    int lo = a.tap_off[0];
    for (int k = 1; k < a.taps; k++) lo = a.tap_off[k] < lo ? a.tap_off[k] : lo;
    a.min_off = lo;
    a.h_pad = conv_tc_halo_rows(a.tap_off, a.taps);
    if (a.h_pad > MAX_HPAD) return cudaErrorInvalidValue;
    // Row-shifted descriptor starts use base offset 0: the 128-byte swizzle phase
    // follows the absolute shared-memory address (checked on B200 against the
    // float64 convolution for shifts that are not multiples of 8 rows).
    a.desc_mode = 0;
    switch (conv_tc_ntile(a.C_out)) {
        case 128: return split ? launch_inst<128, true>(ops, a, n_phases, stream)
                               : launch_inst<128, false>(ops, a, n_phases, stream);
        case 64: return split ? launch_inst<64, true>(ops, a, n_phases, stream)
                              : launch_inst<64, false>(ops, a, n_phases, stream);
        default: return split ? launch_inst<32, true>(ops, a, n_phases, stream)
                              : launch_inst<32, false>(ops, a, n_phases, stream);
    }
}

}  // namespace rk
