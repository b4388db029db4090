// conv_tc.cu -- tcgen05 / TMEM implicit-GEMM Conv1d for sm_100a.
//
// Replaces the reference's CUTLASS-2.x Sm80 implicit-GEMM convolutions
// (src/cutlass_conv.cu:239-313, src/cutlass_conv_f16.cu:216-273), its
// im2col + GEMM fallback (src/rokoko.cpp:286-302) and the GEMM + atomic col2im
// ConvTranspose1d (src/rokoko.cpp:308-329, src/kernels.cu:1141-1173).
//
// CTA = 6 warps, one 128-row x NB-column output tile:
//   warp 0   TMA producer: per (tap, 64-channel block) one A tile per plane at
//            row offset m0 + a_off + tap_off[tap] (TMA zero-fills rows outside
//            [0, T_in), which is the convolution's zero padding) and one B tile
//            per plane.
//   warp 1   owns TMEM; one elected thread issues tcgen05.mma (M=128, N=NB,
//            K=16 per instruction, 4 per 64-channel block; three per step in
//            split mode) and tcgen05.commit to release smem stages.
//   warps 2-5 epilogue: tcgen05.ld 32 columns at a time, fused bias /
//            residual / accumulate / scale, fp32 store, and per-channel
//            sum / sum-of-squares over the tile's rows (warp transpose-reduce,
//            then across the four warps) for the next InstanceNorm.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "conv_tc.cuh"
#include "ptx.cuh"

namespace rk {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;

template <int NB, bool SPLIT>
struct Cfg {
    static constexpr int NPL = SPLIT ? 2 : 1;
    static constexpr uint32_t A_BYTES = BM * BK * 2;
    static constexpr uint32_t B_BYTES = NB * BK * 2;
    static constexpr uint32_t STAGE_BYTES = NPL * (A_BYTES + B_BYTES);
    static constexpr int STAGES_RAW = (192 * 1024) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
    static constexpr uint32_t TMEM_COLS = NB < 32 ? 32 : NB;
    static constexpr size_t SMEM = (size_t)STAGES * STAGE_BYTES + 1024;
};

// Butterfly transpose-reduction: on entry every lane holds 32 column values of
// its own row; on exit v[0] of lane l is the sum over the warp's 32 rows of
// column l.  31 shuffles per 32 columns.
__device__ __forceinline__ float warp_col_sums(float (&v)[32], int lane) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < off; i++) {
            float send = upper ? v[i] : v[i + off];
            float keep = upper ? v[i + off] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
    return v[0];
}

template <int NB, bool SPLIT>
__global__ void __launch_bounds__(192, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmA_hi, const __grid_constant__ CUtensorMap tmA_lo,
                   const __grid_constant__ CUtensorMap tmB_hi, const __grid_constant__ CUtensorMap tmB_lo,
                   const __grid_constant__ ConvArgs args) {
    using C = Cfg<NB, SPLIT>;
    constexpr int STAGES = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t full_bar[STAGES];
    __shared__ __align__(8) uint64_t empty_bar[STAGES];
    __shared__ __align__(8) uint64_t acc_bar;
    __shared__ uint32_t tmem_base_sh;
    __shared__ float red_s[4][NB];
    __shared__ float red_q[4][NB];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tile = blockIdx.x, n_tile = blockIdx.y, phase = blockIdx.z;
    const int m0 = m_tile * BM, n0 = n_tile * NB;
    const int num_k = args.taps * args.kblocks;

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < STAGES; s++) { mbar_init(&full_bar[s], 1); mbar_init(&empty_bar[s], 1); }
        mbar_init(&acc_bar, 1);
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
            const int arow0 = m0 + args.a_off;
            for (int it = 0; it < num_k; it++) {
                const int s = it % STAGES;
                const uint32_t round = (uint32_t)(it / STAGES);
                if (!mbar_wait(&empty_bar[s], (round & 1u) ^ 1u, args.err, RK_DEV_TIMEOUT_EMPTY)) break;
                const int tap = it / args.kblocks, cb = it - tap * args.kblocks;
                uint8_t* st = smem + (size_t)s * C::STAGE_BYTES;
                mbar_arrive_expect_tx(&full_bar[s], C::STAGE_BYTES);
                const int ay = arow0 + args.tap_off[tap];
                tma_load_2d(st, &tmA_hi, &full_bar[s], cb * BK, ay);
                if (SPLIT) tma_load_2d(st + C::A_BYTES, &tmA_lo, &full_bar[s], cb * BK, ay);
                const int bx = (tap * args.kblocks + cb) * BK;
                uint8_t* sb = st + C::NPL * C::A_BYTES;
                tma_load_2d(sb, &tmB_hi, &full_bar[s], bx, brow);
                if (SPLIT) tma_load_2d(sb + C::B_BYTES, &tmB_lo, &full_bar[s], bx, brow);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(BM, NB, SPLIT);
            for (int it = 0; it < num_k; it++) {
                const int s = it % STAGES;
                const uint32_t round = (uint32_t)(it / STAGES);
                if (!mbar_wait(&full_bar[s], round & 1u, args.err, RK_DEV_TIMEOUT_FULL)) break;
                tc_fence_after();
                const uint32_t a_hi = smem_u32(smem + (size_t)s * C::STAGE_BYTES);
                const uint32_t a_lo = a_hi + C::A_BYTES;
                const uint32_t b_hi = a_hi + C::NPL * C::A_BYTES;
                const uint32_t b_lo = b_hi + C::B_BYTES;
#pragma unroll
                for (int kk = 0; kk < BK / 16; kk++) {
                    const uint64_t dah = sw128_kmajor_desc(a_hi + kk * 32);
                    const uint64_t dbh = sw128_kmajor_desc(b_hi + kk * 32);
                    umma_f16(tmem, dah, dbh, idesc, (it > 0 || kk > 0) ? 1u : 0u);
                    if (SPLIT) {
                        umma_f16(tmem, dah, sw128_kmajor_desc(b_lo + kk * 32), idesc, 1u);
                        umma_f16(tmem, sw128_kmajor_desc(a_lo + kk * 32), dbh, idesc, 1u);
                    }
                }
                umma_commit(&empty_bar[s]);
            }
            umma_commit(&acc_bar);
            // every MMA this thread issued has completed once acc_bar flips
            mbar_wait(&acc_bar, 0, args.err, RK_DEV_TIMEOUT_DRAIN);
        }
    } else {
        // ------------------------------------------------ epilogue (warps 2..5)
        const int wq = warp & 3;  // TMEM lane quarter this warp may access
        const int row = wq * 32 + lane;
        const int m = m0 + row;
        const bool ok = mbar_wait(&acc_bar, 0, args.err, RK_DEV_TIMEOUT_ACC);
        tc_fence_after();
        const int out_row = m * args.o_stride + args.o_off + phase * args.o_phase_step;
        const bool valid = ok && m < args.M && out_row >= 0 && out_row < args.T_out;
        const bool dup = valid && out_row == args.dup_src_row;
        const bool want_stats = args.stats != nullptr;
#pragma unroll 1
        for (int c = 0; c < NB / 32; c++) {
            float v[32];
            tmem_ld32(tmem + ((uint32_t)(wq * 32) << 16) + (uint32_t)(c * 32), v);
            const int co0 = n0 + c * 32;
            const int ncol = min(32, args.C_out - co0);
            float s[32], q[32];
#pragma unroll
            for (int j = 0; j < 32; j++) { s[j] = 0.f; q[j] = 0.f; }
            if (valid) {
                const float* rp = args.res ? args.res + (size_t)(out_row >> args.res_shift) * args.ldres + co0 : nullptr;
                const float* ap = args.acc_in ? args.acc_in + (size_t)out_row * args.ldacc + co0 : nullptr;
                float* yp = args.y + (size_t)out_row * args.ldy + co0;
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    if (j < ncol) {
                        float o = v[j];
                        if (rp) o += rp[j];
                        if (args.bias) o += args.bias[co0 + j];
                        if (ap) o = ap[j] + o;
                        o *= args.alpha;
                        yp[j] = o;
                        s[j] = o;
                        q[j] = o * o;
                    }
                }
                if (dup) {
                    const float* r0 = args.res ? args.res + co0 : nullptr;
                    const float* a0 = args.acc_in ? args.acc_in + co0 : nullptr;
                    float* y0 = args.y + co0;
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        if (j < ncol) {
                            float o = v[j];
                            if (r0) o += r0[j];
                            if (args.bias) o += args.bias[co0 + j];
                            if (a0) o = a0[j] + o;
                            o *= args.alpha;
                            y0[j] = o;
                            s[j] += o;
                            q[j] += o * o;
                        }
                    }
                }
            }
            if (want_stats) {
                const float cs = warp_col_sums(s, lane);
                const float cq = warp_col_sums(q, lane);
                red_s[wq][c * 32 + lane] = cs;
                red_q[wq][c * 32 + lane] = cq;
            }
        }
        if (want_stats) {
            asm volatile("bar.sync 1, 128;" ::: "memory");
            const int part = blockIdx.z * gridDim.x + blockIdx.x;
            for (int col = threadIdx.x - 64; col < NB; col += 128) {
                const int co = n0 + col;
                if (co < args.C_out) {
                    const float s = (red_s[0][col] + red_s[1][col]) + (red_s[2][col] + red_s[3][col]);
                    const float q = (red_q[0][col] + red_q[1][col]) + (red_q[2][col] + red_q[3][col]);
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
cudaError_t launch_inst(const ConvOperands& ops, const ConvArgs& a, int n_phases, cudaStream_t stream) {
    using C = Cfg<NB, SPLIT>;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(conv_tc_kernel<NB, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)C::SMEM);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    dim3 grid((a.M + BM - 1) / BM, (a.C_out + NB - 1) / NB, n_phases);
    conv_tc_kernel<NB, SPLIT><<<grid, 192, C::SMEM, stream>>>(ops.a_hi, SPLIT ? ops.a_lo : ops.a_hi, ops.b_hi,
                                                               SPLIT ? ops.b_lo : ops.b_hi, a);
    return cudaGetLastError();
}

}  // namespace

bool make_tmap_k64(CUtensorMap* m, const void* base, bool bf16, uint64_t cols, uint64_t rows, uint64_t ld,
                   uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * 2) & 15) || box_rows > 256) return false;
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

int conv_tc_ntile(int C_out) {
    if (C_out % 256 == 0) return 256;
    if (C_out > 64) return 128;
    if (C_out > 32) return 64;
    return 32;
}

cudaError_t conv_tc_launch(const ConvOperands& ops, const ConvArgs& a, bool split, int n_phases,
                           cudaStream_t stream) {
    if (a.taps < 1 || a.taps > CONV_MAX_TAPS || a.kblocks < 1 || a.M < 1) return cudaErrorInvalidValue;
    switch (conv_tc_ntile(a.C_out)) {
        case 256: return split ? launch_inst<256, true>(ops, a, n_phases, stream)
                               : launch_inst<256, false>(ops, a, n_phases, stream);
        case 128: return split ? launch_inst<128, true>(ops, a, n_phases, stream)
                               : launch_inst<128, false>(ops, a, n_phases, stream);
        case 64: return split ? launch_inst<64, true>(ops, a, n_phases, stream)
                              : launch_inst<64, false>(ops, a, n_phases, stream);
        default: return split ? launch_inst<32, true>(ops, a, n_phases, stream)
                              : launch_inst<32, false>(ops, a, n_phases, stream);
    }
}

}  // namespace rk
