// conv_tc.cu -- tcgen05 / TMEM implicit-GEMM Conv1d for sm_100a.
//
// Replaces the reference's CUTLASS-2.x Sm80 implicit-GEMM convolutions
// (src/cutlass_conv.cu:239-313, src/cutlass_conv_f16.cu:216-273), its
// im2col + GEMM fallback (src/rokoko.cpp:286-302) and the GEMM + atomic col2im
// ConvTranspose1d (src/rokoko.cpp:308-329, src/kernels.cu:1141-1173).
//
// Orientation: the weights are the MMA's M = 128 side (output channels) and
// the activations the N side (BN = 64, 128, 192 or 256 time rows), so one weight
// tile streamed from L2 feeds BN rows of output; at BN = 256 the tensor pipe
// runs near its peak with a two-deep weight ring (measured on B200: the same
// stream at N = 128 saturates the L2 -> SMEM path first).
//
// Persistent kernel: grid = min(tiles, SMs), one CTA per SM; CTA b runs tiles
// b, b + grid, ... (time fastest, so neighbouring CTAs share the weight tile in
// L2).  10 warps, specialised:
//   warp 0   TMA producer.  Per tile and 64-channel block it loads ONE
//            activation tile of BN + halo rows (two boxes; halo = max tap
//            offset - min tap offset; TMA zero-fills rows outside [0, T_in),
//            i.e. the padding) into a 2-deep ring, and per (channel block, tap)
//            one 128-row weight tile into a 2..8-deep ring.
//   warp 1   owns TMEM (two accumulators of BN columns); one elected thread
//            issues tcgen05.mma (M=128, N=BN, K=16; 4 per 64-channel block, x3
//            in split mode).  Tap k reads the activation tile through a
//            descriptor whose start is shifted by (tap_off[k] - min_off) rows,
//            so activations cross L2 -> SMEM once per channel block.
//   warps 2-9 epilogue of the previous tile while the MMAs of the next one run:
//            warp w reads TMEM lanes 32(w%4).. = output channels (two warps per
//            lane quarter split the tile's row pairs), tcgen05.ld
//            brings 32 time rows per thread, and every row is stored as 32
//            consecutive channels (one 128-byte segment per warp): bias,
//            residual, accumulate, scale, store, plus per-channel sum and
//            sum-of-squares partials (64-row parts) for the next InstanceNorm.
// Every wait is bounded (ptx.cuh); a timeout records an error code and the
// roles drain and return, so a protocol fault is an error status, not a hang.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "conv_tc.cuh"
#include "ptx.cuh"

namespace rk {

namespace {

constexpr int BK = 64;
constexpr int X_STAGES = 2;
constexpr int MAX_W_STAGES = 8;
constexpr size_t SMEM_LIMIT = 227 * 1024 - 1024;  // dynamic bytes; leaves room for the static barriers
constexpr int MAX_K_SPLIT = 8;

template <int BN, bool SPLIT>
struct Cfg {
    static constexpr int NPL = SPLIT ? 2 : 1;
    static constexpr uint32_t W_PLANE = CONV_W_ROWS * BK * 2;   // 16 KB
    static constexpr uint32_t W_STAGE = NPL * W_PLANE;
    static size_t x_stage(int box) { return (size_t)NPL * 2 * box * 128; }
    static size_t fixed_bytes(int box) { return 1024 + X_STAGES * x_stage(box); }
    static int w_stages(int box) {
        if (fixed_bytes(box) >= SMEM_LIMIT) return 0;
        const int n = (int)((SMEM_LIMIT - fixed_bytes(box)) / W_STAGE);
        return n > MAX_W_STAGES ? MAX_W_STAGES : n;
    }
    static size_t smem_bytes(int box, int ws) { return fixed_bytes(box) + (size_t)ws * W_STAGE; }
    // TMEM: two accumulators of BN columns, ACC_STRIDE apart; the allocation is a power of two
    static constexpr uint32_t TMEM_ALLOC = 2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512);
    static constexpr uint32_t ACC_STRIDE = TMEM_ALLOC / 2;
};

// gelu_new: 0.5 v (1 + tanh(0.7978845608 (v + 0.044715 v^3)))
__device__ __forceinline__ float gelu_tanh(float v) {
    const float inner = 0.7978845608028654f * (v + 0.044715f * v * v * v);
    return 0.5f * v * (1.0f + tanhf(inner));
}

struct Tiles {
    int tiles_t, tiles_c, n_phases, n_tiles;
    __device__ void decode(int t, int& t_tile, int& c_tile, int& phase, int& ks) const {
        const int per = tiles_t * tiles_c * n_phases;
        ks = t / per;
        int rem = t - ks * per;
        phase = rem / (tiles_t * tiles_c);
        rem -= phase * tiles_t * tiles_c;
        c_tile = rem / tiles_t;
        t_tile = rem - c_tile * tiles_t;
    }
};

// The epilogue's FP32 reads of a tile (residual and accumulator-input rows,
// whole rows when the channel pitch equals C_out, so that the range is
// contiguous) are prefetched into L2 when the tile's loads are issued: the
// reads then hit L2 during the epilogue instead of all CTAs' epilogues pulling
// them from HBM at once after their MMAs.  Plain row layout only (o_stride 1, no
// row shift); every prefetched byte lies inside the rows [o_min, T_out).
__device__ __forceinline__ void prefetch_rows(const float* base, int ld, int r0, int r1) {
    if (!base || r1 <= r0) return;
    const char* p = reinterpret_cast<const char*>(base + (size_t)r0 * ld);
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uintptr_t a16 = (a + 15) & ~uintptr_t(15);
    const uintptr_t end = (a + (size_t)(r1 - r0) * ld * 4) & ~uintptr_t(15);
    for (uintptr_t q = a16; q < end; q += 32768) {
        const uintptr_t n = end - q < 32768 ? end - q : 32768;
        l2_prefetch_bulk(reinterpret_cast<const void*>(q), (uint32_t)n);
    }
}

__device__ __forceinline__ void prefetch_epilogue_rows(const ConvArgs& a, int t_tile, int phase, int BN) {
    if (a.o_stride != 1 || a.res_shift != 0 || a.part_out) return;
    const int m0 = t_tile * BN;
    const int rows = min(BN, a.M - m0);
    int r0 = m0 + a.o_off + phase * a.o_phase_step, r1 = r0 + rows;
    r0 = max(r0, a.o_min);
    r1 = min(r1, a.T_out);
    if (a.res && a.ldres == a.C_out) prefetch_rows(a.res, a.ldres, r0, r1);
    if (a.acc_in && a.ldacc == a.C_out) prefetch_rows(a.acc_in, a.ldacc, r0, r1);
}

template <int BN, bool SPLIT>
__global__ void __launch_bounds__(320, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmX_hi, const __grid_constant__ CUtensorMap tmX_lo,
                   const __grid_constant__ CUtensorMap tmW_hi, const __grid_constant__ CUtensorMap tmW_lo,
                   const __grid_constant__ ConvArgs args, int n_phases, int WS) {
    using C = Cfg<BN, SPLIT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t x_full[X_STAGES], x_empty[X_STAGES];
    __shared__ __align__(8) uint64_t w_full[MAX_W_STAGES], w_empty[MAX_W_STAGES];
    __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], drain_bar;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int epi_dead;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int box = args.act_box;
    const uint32_t x_plane = (uint32_t)(2 * box) * 128;
    const uint32_t x_stage = C::NPL * x_plane;
    uint8_t* x_buf = smem;                                       // [stage][plane][2*box rows][128 B]
    uint8_t* w_buf = smem + (size_t)X_STAGES * x_stage;          // [stage][plane][128 rows][128 B]
    const int KB = args.kblocks, TAPS = args.taps;
    const int S = args.k_split > 1 ? args.k_split : 1;
    Tiles g;
    g.tiles_t = (args.M + BN - 1) / BN;
    g.tiles_c = (args.C_out + CONV_W_ROWS - 1) / CONV_W_ROWS;
    g.n_phases = n_phases;
    g.n_tiles = g.tiles_t * g.tiles_c * n_phases * S;

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < X_STAGES; s++) { mbar_init(&x_full[s], 1); mbar_init(&x_empty[s], 1); }
        for (int s = 0; s < WS; s++) { mbar_init(&w_full[s], 1); mbar_init(&w_empty[s], 1); }
        for (int s = 0; s < 2; s++) { mbar_init(&acc_full[s], 1); mbar_init(&acc_empty[s], 8); }
        mbar_init(&drain_bar, 1);
        epi_dead = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmX_hi);
        tma_prefetch_desc(&tmW_hi);
        if (SPLIT) { tma_prefetch_desc(&tmX_lo); tma_prefetch_desc(&tmW_lo); }
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base_sh, C::TMEM_ALLOC);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t xi = 0, wi = 0;
            bool alive = true;
            for (int t = blockIdx.x; t < g.n_tiles && alive; t += gridDim.x) {
                int t_tile, c_tile, phase, ks;
                g.decode(t, t_tile, c_tile, phase, ks);
                const int wrow = phase * args.b_phase_rows + c_tile * CONV_W_ROWS;
                const int xrow = t_tile * BN + args.a_off + args.min_off;
                if (ks == S - 1) prefetch_epilogue_rows(args, t_tile, phase, BN);
                const int kb1 = (ks + 1) * KB / S;
                for (int kb = ks * KB / S; kb < kb1 && alive; kb++, xi++) {
                    const uint32_t sx = xi % X_STAGES, rx = xi / X_STAGES;
                    if (!mbar_wait(&x_empty[sx], (rx & 1u) ^ 1u, args.err, RK_DEV_TIMEOUT_EMPTY)) { alive = false; break; }
                    uint8_t* xb = x_buf + (size_t)sx * x_stage;
                    mbar_arrive_expect_tx(&x_full[sx], x_stage);
                    tma_load_2d(xb, &tmX_hi, &x_full[sx], kb * BK, xrow);
                    tma_load_2d(xb + (size_t)box * 128, &tmX_hi, &x_full[sx], kb * BK, xrow + box);
                    if (SPLIT) {
                        tma_load_2d(xb + x_plane, &tmX_lo, &x_full[sx], kb * BK, xrow);
                        tma_load_2d(xb + x_plane + (size_t)box * 128, &tmX_lo, &x_full[sx], kb * BK, xrow + box);
                    }
                    for (int tap = 0; tap < TAPS; tap++, wi++) {
                        const uint32_t sw = wi % (uint32_t)WS, rw = wi / (uint32_t)WS;
                        if (!mbar_wait(&w_empty[sw], (rw & 1u) ^ 1u, args.err, RK_DEV_TIMEOUT_EMPTY)) {
                            alive = false;
                            break;
                        }
                        uint8_t* wb = w_buf + (size_t)sw * C::W_STAGE;
                        mbar_arrive_expect_tx(&w_full[sw], C::W_STAGE);
                        const int wx = (tap * KB + kb) * BK;
                        tma_load_2d(wb, &tmW_hi, &w_full[sw], wx, wrow);
                        if (SPLIT) tma_load_2d(wb + C::W_PLANE, &tmW_lo, &w_full[sw], wx, wrow);
                    }
                }
            }
            // the last copy issued into each stage has landed (instant unless a consumer gave up)
            for (uint32_t k = xi > (uint32_t)X_STAGES ? xi - X_STAGES : 0u; k < xi; k++)
                mbar_wait(&x_full[k % X_STAGES], (k / X_STAGES) & 1u, args.err, RK_DEV_TIMEOUT_DRAIN);
            for (uint32_t k = wi > (uint32_t)WS ? wi - WS : 0u; k < wi; k++)
                mbar_wait(&w_full[k % WS], (k / WS) & 1u, args.err, RK_DEV_TIMEOUT_DRAIN);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(CONV_W_ROWS, BN, SPLIT);
            uint32_t xi = 0, wi = 0, tl = 0;
            bool alive = true;
            for (int t = blockIdx.x; t < g.n_tiles && alive; t += gridDim.x, tl++) {
                int t_tile, c_tile, phase, ks;
                g.decode(t, t_tile, c_tile, phase, ks);
                const int kb0 = ks * KB / S, kb1 = (ks + 1) * KB / S;
                const uint32_t acc = tl & 1u, ru = tl >> 1;
                if (!mbar_wait(&acc_empty[acc], (ru & 1u) ^ 1u, args.err, RK_DEV_TIMEOUT_EMPTY)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + acc * C::ACC_STRIDE;
                for (int kb = kb0; kb < kb1 && alive; kb++, xi++) {
                    const uint32_t sx = xi % X_STAGES, rx = xi / X_STAGES;
                    if (!mbar_wait(&x_full[sx], rx & 1u, args.err, RK_DEV_TIMEOUT_FULL)) { alive = false; break; }
                    tc_fence_after();
                    const uint32_t x_hi = smem_u32(x_buf + (size_t)sx * x_stage), x_lo = x_hi + x_plane;
                    for (int tap = 0; tap < TAPS; tap++, wi++) {
                        const uint32_t sw = wi % (uint32_t)WS, rw = wi / (uint32_t)WS;
                        if (!mbar_wait(&w_full[sw], rw & 1u, args.err, RK_DEV_TIMEOUT_FULL)) {
                            alive = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t shift = (uint32_t)(args.tap_off[tap] - args.min_off) * 128u;
                        const uint32_t w_hi = smem_u32(w_buf + (size_t)sw * C::W_STAGE), w_lo = w_hi + C::W_PLANE;
#pragma unroll
                        for (int kk = 0; kk < BK / 16; kk++) {
                            const uint64_t dwh = sw128_kmajor_desc(w_hi + kk * 32, 0);
                            const uint64_t dxh = sw128_kmajor_desc(x_hi + shift + kk * 32, args.desc_mode);
                            umma_f16(d_tmem, dwh, dxh, idesc, (kb > kb0 || tap > 0 || kk > 0) ? 1u : 0u);
                            if (SPLIT) {
                                umma_f16(d_tmem, dwh, sw128_kmajor_desc(x_lo + shift + kk * 32, args.desc_mode),
                                         idesc, 1u);
                                umma_f16(d_tmem, sw128_kmajor_desc(w_lo + kk * 32, 0), dxh, idesc, 1u);
                            }
                        }
                        umma_commit(&w_empty[sw]);
                    }
                    umma_commit(&x_empty[sx]);
                }
                umma_commit(&acc_full[acc]);
            }
            // drain: every MMA this thread issued has completed once this commit lands
            umma_commit(&drain_bar);
            mbar_wait(&drain_bar, 0, args.err, RK_DEV_TIMEOUT_DRAIN);
            tc_fence_before();
        }
    } else {
        // ------------------------------------------------ epilogue (warps 2..9)
        // TMEM lane quarter = warp % 4 (the hardware rule); the two warps of a
        // quarter split the tile's 64-row pairs of chunks between them.
        const int wq = warp & 3;
        const int half = (warp - 2) >> 2;
        const bool want_stats = args.stats != nullptr;
        const int parts_per_phase = (args.M + STATS_ROWS - 1) / STATS_ROWS;
        uint32_t tl = 0;
        for (int t = blockIdx.x; t < g.n_tiles; t += gridDim.x, tl++) {
            int t_tile, c_tile, phase, ks;
            g.decode(t, t_tile, c_tile, phase, ks);
            const int m0 = t_tile * BN;
            const int co = c_tile * CONV_W_ROWS + wq * 32 + lane;
            const bool co_ok = co < args.C_out;
            const float bias_v = (args.bias && co_ok) ? args.bias[co] : 0.0f;
            const uint32_t acc = tl & 1u, ru = tl >> 1;
            const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[acc], ru & 1u, args.err, RK_DEV_TIMEOUT_ACC));
            tc_fence_after();
            if (!ok && lane == 0) epi_dead = 1;
            const uint32_t s_tmem = tmem + acc * C::ACC_STRIDE + ((uint32_t)(wq * 32) << 16);
            // Common case, branch-free so the 32 rows of a chunk interleave: plain
            // residual (no row shift), no activation, no accumulator input, no
            // duplicated row in the pair, and every row of the pair inside the output.
            const bool fast_conv = co_ok && !args.act && !args.acc_in && args.res_shift == 0;
            if (args.part_out) {
                // split-K: raw accumulators of this reduction slice, rows by m
                float* po = args.part_out + ((size_t)(ks * n_phases + phase) * args.M) * args.C_out + co;
#pragma unroll 1
                for (int c = half * 2; c < (ok ? BN / 32 : 0); c += (c & 1) ? 3 : 1) {
                    float v[32];
                    tmem_ld32(s_tmem + (uint32_t)(c * 32), v);
                    const int mc = m0 + c * 32;
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        if (mc + j < args.M && co_ok) po[(size_t)(mc + j) * args.C_out] = v[j];
                }
            }
            const int n_pairs = (ok && !args.part_out) ? min(BN / 64, (args.M - m0 + 63) / 64) : 0;
#pragma unroll 1
            for (int pp = half; pp < n_pairs; pp += 2) {
                float s = 0.f, q = 0.f;
                const int mp = m0 + pp * 64;
                const int orow_p = mp * args.o_stride + args.o_off + phase * args.o_phase_step;
                const int orow_last = orow_p + 63 * args.o_stride;
                // warp-uniform: tcgen05.ld below is a .sync.aligned instruction, so every lane
                // of the warp must take the same path (lanes past C_out take the general one)
                // the reflection-pad duplicate row, if this pair holds it, takes the general path
                const bool has_dup = args.dup_src_row >= orow_p && args.dup_src_row <= orow_last &&
                                     (args.dup_src_row - orow_p) % args.o_stride == 0;
                const int pvalid = args.part_rows ? args.part_rows[mp >> 6] : 64;  // valid rows of this part
                const bool fast = __all_sync(0xffffffffu, fast_conv && !has_dup && mp + 63 < args.M &&
                                                              orow_p >= args.o_min && orow_last < args.T_out &&
                                                              pvalid == 64);
                if (fast) {
                    // residual rows of both chunks in flight before the accumulator reads
                    const size_t rstep = (size_t)args.o_stride * args.ldres, ystep = (size_t)args.o_stride * args.ldy;
                    float rv[64];
                    if (args.res) {
                        const float* rp = args.res + (size_t)orow_p * args.ldres + co;
#pragma unroll
                        for (int j = 0; j < 64; j++) rv[j] = rp[j * rstep];
                    } else {
#pragma unroll
                        for (int j = 0; j < 64; j++) rv[j] = 0.f;
                    }
                    float* yp = args.y + (size_t)orow_p * args.ldy + co;
#pragma unroll
                    for (int cc = 0; cc < 2; cc++) {
                        float v[32];
                        tmem_ld32(s_tmem + (uint32_t)((2 * pp + cc) * 32), v);
#pragma unroll
                        for (int j = 0; j < 32; j++) {
                            float o = v[j];
                            if (args.res) o += rv[cc * 32 + j];
                            o += bias_v;
                            o *= args.alpha;
                            yp[(cc * 32 + j) * ystep] = o;
                            s += o;
                            q += o * o;
                        }
                    }
                } else {
                    // General path (partial chunks, row-shifted residual, GELU, accumulator
                    // input, the reflection-pad duplicate): one TMEM column per valid row, a
                    // rolled loop so that the rarely executed code stays small.  Row validity
                    // is warp-uniform, so every lane takes the same tcgen05.ld.
#pragma unroll 1
                    for (int j = 0; j < 64; j++) {
                        const int m = mp + j;
                        const int orow = orow_p + j * args.o_stride;
                        if (m >= args.M || orow < args.o_min || orow >= args.T_out || j >= pvalid) continue;
                        const float acc = tmem_ld1(s_tmem + (uint32_t)(2 * pp * 32 + j));
                        if (!co_ok) continue;
                        for (int pass = 0; pass < 2; pass++) {
                            // pass 1: reflection pad (1, 0), the accumulator of dup_src_row also
                            // goes to row 0 with residual / accumulator row 0
                            if (pass == 1 && orow != args.dup_src_row) break;
                            const int orw = pass ? 0 : orow;
                            const int rrow = pass ? 0 : (orow >> args.res_shift);
                            float o = acc;
                            if (args.res) o += args.res[(size_t)rrow * args.ldres + co];
                            o += bias_v;
                            if (args.act == 1) o = gelu_tanh(o);
                            if (args.acc_in) o = args.acc_in[(size_t)orw * args.ldacc + co] + o;
                            o *= args.alpha;
                            args.y[(size_t)orw * args.ldy + co] = o;
                            s += o;
                            q += o * o;
                        }
                    }
                }
                if (want_stats && mp < args.M && co_ok) {
                    const int part = phase * parts_per_phase + mp / STATS_ROWS;
                    args.stats[(size_t)part * args.stats_ld + co] = s;
                    args.stats[(size_t)(args.stats_parts + part) * args.stats_ld + co] = q;
                }
            }
            // this warp's share of the accumulator has been read: hand it back
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
            // all eight epilogue warps meet here every tile, whatever happened above
            asm volatile("bar.sync 1, 256;" ::: "memory");
            if (epi_dead) break;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_ALLOC);
    }
}

// Split-K second stage: one block per (32 channels, 64-row part); thread
// (x, y) owns channel x and rows y*8 .. y*8+7 of the part.  256-thread blocks
// leave room for every row's and slice's load in flight at once.  Sums the k_split
// raw accumulators in slice order, applies the same epilogue as the conv kernel
// (residual, bias, activation, accumulator input, scale, reflection-pad
// duplicate) and writes the part's statistics, combined over y in a fixed order.
template <int KS>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const __grid_constant__ ConvArgs a, int n_phases) {
    __shared__ float red_s[8][32], red_q[8][32];
    const int cx = threadIdx.x, ry = threadIdx.y;
    const int co = blockIdx.x * 32 + cx;
    const int ppp = (a.M + STATS_ROWS - 1) / STATS_ROWS;
    const int phase = blockIdx.y / ppp, p = blockIdx.y - phase * ppp;
    const bool co_ok = co < a.C_out;
    const size_t slice = (size_t)n_phases * a.M * a.C_out;
    const float bias_v = (a.bias && co_ok) ? a.bias[co] : 0.0f;
    float s = 0.f, q = 0.f;
    const int m0 = p * STATS_ROWS + ry * 8;
    // every row's and slice's load in flight before the ordered sums: addresses are
    // clamped into the slice (rows past M and channels past C_out are discarded below)
    const int co_c = co_ok ? co : a.C_out - 1;
    float pv[KS][8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int m_c = m0 + i < a.M ? m0 + i : a.M - 1;
        const float* src = a.part_out + ((size_t)phase * a.M + m_c) * a.C_out + co_c;
#pragma unroll
        for (int k = 0; k < KS; k++) pv[k][i] = src[k * slice];
    }
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        float acc = pv[0][i];
#pragma unroll
        for (int k = 1; k < KS; k++) acc += pv[k][i];
        v[i] = acc;
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int m = m0 + i;
        const int orow = m * a.o_stride + a.o_off + phase * a.o_phase_step;
        if (!co_ok || m >= a.M || orow < a.o_min || orow >= a.T_out) continue;
        if (a.part_rows && (m & 63) >= a.part_rows[m >> 6]) continue;  // gap row between utterances
        for (int pass = 0; pass < 2; pass++) {
            int orw = orow, rrow = orow >> a.res_shift;
            if (pass == 1) {
                if (orow != a.dup_src_row) break;
                orw = 0;
                rrow = 0;
            }
            float o = v[i];
            if (a.res) o += a.res[(size_t)rrow * a.ldres + co];
            o += bias_v;
            if (a.act == 1) o = gelu_tanh(o);
            if (a.acc_in) o = a.acc_in[(size_t)orw * a.ldacc + co] + o;
            o *= a.alpha;
            a.y[(size_t)orw * a.ldy + co] = o;
            s += o;
            q += o * o;
        }
    }
    if (!a.stats) return;
    red_s[ry][cx] = s;
    red_q[ry][cx] = q;
    __syncthreads();
    if (ry == 0 && co_ok) {
        float ts = 0.f, tq = 0.f;
#pragma unroll
        for (int k = 0; k < 8; k++) { ts += red_s[k][cx]; tq += red_q[k][cx]; }
        const int part = phase * ppp + p;
        a.stats[(size_t)part * a.stats_ld + co] = ts;
        a.stats[(size_t)(a.stats_parts + part) * a.stats_ld + co] = tq;
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

template <int BN, bool SPLIT>
cudaError_t set_attr() {
    return cudaFuncSetAttribute(conv_tc_kernel<BN, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)SMEM_LIMIT);
}

// SM count of the current device (cached per device).
int sm_count() {
    static int cache[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

// Activation box rows for a BN-row tile: the tile (BN + halo rows) is loaded
// as two boxes of this many rows (a TMA box is at most 256 rows).
int act_box_rows(int BN, int halo) {
    const int half = (BN + halo + 1) / 2;
    return (half + 7) / 8 * 8;
}

template <int BN, bool SPLIT>
cudaError_t launch_inst(const ConvOperands& ops, ConvArgs a, int halo, int n_phases, cudaStream_t stream,
                        int* kernels) {
    using C = Cfg<BN, SPLIT>;
    a.act_box = act_box_rows(BN, halo);
    const int ws = C::w_stages(a.act_box);
    if (ws < 2 || a.act_box > 256) return cudaErrorInvalidValue;
    CUtensorMap x_hi, x_lo;
    if (!make_tmap_k64(&x_hi, ops.act_hi, SPLIT, ops.act_cp, ops.act_rows, ops.act_cp, a.act_box) ||
        (SPLIT && !make_tmap_k64(&x_lo, ops.act_lo, true, ops.act_cp, ops.act_rows, ops.act_cp, a.act_box)))
        return cudaErrorInvalidValue;
    if (!SPLIT) x_lo = x_hi;
    const size_t smem = C::smem_bytes(a.act_box, ws);
    const int tiles = ((a.M + BN - 1) / BN) * ((a.C_out + CONV_W_ROWS - 1) / CONV_W_ROWS) * n_phases;
    const int ks = a.k_split;
    a.part_out = ks > 1 ? ops.scratch : nullptr;
    const int work = tiles * ks;
    const int grid = work < sm_count() ? work : sm_count();
    conv_tc_kernel<BN, SPLIT><<<grid, 320, smem, stream>>>(x_hi, x_lo, ops.w_hi, SPLIT ? ops.w_lo : ops.w_hi, a,
                                                            n_phases, ws);
    cudaError_t e = cudaGetLastError();
    if (kernels) *kernels = ks > 1 ? 2 : 1;
    if (e != cudaSuccess || ks == 1) return e;
    dim3 rg((a.C_out + 31) / 32, conv_tc_stats_parts(a.M, n_phases));
    const dim3 rb(32, 8);
    switch (ks) {
        case 2: splitk_reduce_kernel<2><<<rg, rb, 0, stream>>>(a, n_phases); break;
        case 3: splitk_reduce_kernel<3><<<rg, rb, 0, stream>>>(a, n_phases); break;
        case 4: splitk_reduce_kernel<4><<<rg, rb, 0, stream>>>(a, n_phases); break;
        case 5: splitk_reduce_kernel<5><<<rg, rb, 0, stream>>>(a, n_phases); break;
        case 6: splitk_reduce_kernel<6><<<rg, rb, 0, stream>>>(a, n_phases); break;
        case 7: splitk_reduce_kernel<7><<<rg, rb, 0, stream>>>(a, n_phases); break;
        default: splitk_reduce_kernel<MAX_K_SPLIT><<<rg, rb, 0, stream>>>(a, n_phases); break;
    }
    return cudaGetLastError();
}

// Time tile BN and split-K factor for a launch.  Estimated time = waves of
// work units x time of one unit, where a unit is one (tile, reduction slice)
// and its time is its MMA work over the tile's sustained tensor rate (a weight
// tile streamed from L2 feeds BN rows: measured on B200 about full rate at
// BN = 256, 70 % at 128, 40 % at 64), plus the split-K second pass (partials
// written and read once at about 4 TB/s).  Only BN whose activation ring fits
// in shared memory are considered.  Long launches (M >= 4096 rows: the
// generator's resblocks, which run three at a time on concurrent streams)
// minimise SM-time instead of waves: the partial last wave of one launch is
// filled by CTAs of the others (measured on the config-1 decode graph: BN =
// 256 for these launches, 2.53 -> 2.40 ms).
void pick_tiling(const ConvArgs& a, int n_phases, int halo, bool split, const ConvOperands& ops, int* bn_out,
                 int* ks_out) {
    const int ctiles = (a.C_out + CONV_W_ROWS - 1) / CONV_W_ROWS * n_phases;
    const int sms = sm_count();
    const int cands[4] = {256, 192, 128, 64};
    const double eff[4] = {1.0, 0.9, 0.7, 0.4};
    // rows x (64-channel block) x tap per us at full tensor rate: 12 (split) or 4
    // MMAs of 128 x 256 x 16 per 256 rows, ~128 clocks each at ~1.9 GHz
    const double tc_rows_per_us = split ? 316.0 : 948.0;
    const size_t slice_bytes = (size_t)n_phases * a.M * a.C_out * sizeof(float);
    double best = 1e30;
    *bn_out = 0;
    *ks_out = 1;
    const bool sm_time = a.M >= 4096;
    for (int i = 0; i < 4; i++) {
        const int bn = cands[i];
        const int box = act_box_rows(bn, halo);
        const int ws = split ? Cfg<256, true>::w_stages(box) : Cfg<256, false>::w_stages(box);
        if (ws < 2 || box > 256) continue;
        const int tiles = (a.M + bn - 1) / bn * ctiles;
        int kmax = 1;
        if (ops.scratch && a.kblocks >= 4 && !sm_time) {
            kmax = a.kblocks / 2 < MAX_K_SPLIT ? a.kblocks / 2 : MAX_K_SPLIT;
            while (kmax > 1 && (size_t)kmax * slice_bytes > ops.scratch_bytes) kmax--;
        }
        for (int ks = 1; ks <= kmax; ks++) {
            const int units = tiles * ks;
            const double waves = sm_time ? (double)units / sms : (double)((units + sms - 1) / sms);
            const double unit_us = (double)bn * a.taps * ((a.kblocks + ks - 1) / ks) / (tc_rows_per_us * eff[i]);
            double t = waves * unit_us;
            if (ks > 1) t += 2.0 * ks * slice_bytes / 4.0e6 + 3.0;  // second pass + its launch
            if (t < best * 0.97) {
                best = t;
                *bn_out = bn;
                *ks_out = ks;
            }
        }
    }
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
    if ((e = set_attr<256, true>()) || (e = set_attr<256, false>()) || (e = set_attr<192, true>()) ||
        (e = set_attr<192, false>()) || (e = set_attr<128, true>()) || (e = set_attr<128, false>()) ||
        (e = set_attr<64, true>()) || (e = set_attr<64, false>()))
        return e;
    return cudaSuccess;
}

cudaError_t conv_tc_launch(const ConvOperands& ops, const ConvArgs& a_in, bool split, int n_phases,
                           cudaStream_t stream, int* kernels) {
    if (kernels) *kernels = 0;
    if (a_in.taps < 1 || a_in.taps > CONV_MAX_TAPS || a_in.kblocks < 1 || a_in.M < 1 || n_phases < 1 ||
        !ops.act_hi || (split && !ops.act_lo) || ops.act_cp != (uint64_t)a_in.kblocks * 64)
        return cudaErrorInvalidValue;
    if (a_in.stats && a_in.stats_parts != conv_tc_stats_parts(a_in.M, n_phases)) return cudaErrorInvalidValue;
    ConvArgs a = a_in;
    a.k_split = 1;
    a.part_out = nullptr;
    int lo = a.tap_off[0], hi = a.tap_off[0];
    for (int k = 1; k < a.taps; k++) {
        lo = a.tap_off[k] < lo ? a.tap_off[k] : lo;
        hi = a.tap_off[k] > hi ? a.tap_off[k] : hi;
    }
    a.min_off = lo;
    // Row-shifted descriptor starts use base offset 0: the 128-byte swizzle phase
    // follows the absolute shared-memory address (checked on B200 against the
    // float64 convolution for shifts that are not multiples of 8 rows).
    a.desc_mode = 0;
    const int halo = hi - lo;
    int bn = 0;
    pick_tiling(a, n_phases, halo, split, ops, &bn, &a.k_split);
    switch (bn) {
        case 256: return split ? launch_inst<256, true>(ops, a, halo, n_phases, stream, kernels)
                               : launch_inst<256, false>(ops, a, halo, n_phases, stream, kernels);
        case 192: return split ? launch_inst<192, true>(ops, a, halo, n_phases, stream, kernels)
                               : launch_inst<192, false>(ops, a, halo, n_phases, stream, kernels);
        case 128: return split ? launch_inst<128, true>(ops, a, halo, n_phases, stream, kernels)
                               : launch_inst<128, false>(ops, a, halo, n_phases, stream, kernels);
        case 64: return split ? launch_inst<64, true>(ops, a, halo, n_phases, stream, kernels)
                              : launch_inst<64, false>(ops, a, halo, n_phases, stream, kernels);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace rk
