// conv_tc.cuh -- host interface of the tcgen05 implicit-GEMM Conv1d kernel.
//
// One kernel covers every dense contraction of the decoder/generator:
//   Conv1d (any K, dilation; stride 1)      out_row = m,             in_row = m + tap_off[k]
//   ConvTranspose1d as s polyphase convs   out_row = q*s + r - p,   in_row = q - j   (phase r)
//   Linear / 1x1 conv                       K = 1
// GEMM view (transposed, so that the wide dimension feeds the N side of the
// MMA): D[c_out][m] = sum over (tap, c_in) W[c_out][tap, c_in] * X[m + tap_off][c_in]
// with M = 128 output channels per tile and N = BN time rows (64, 128, 192 or 256).
// Activations are [T, Cp] channels-last 16-bit planes (Cp = C_in rounded up to
// 64, zero padded); weights are [rows, taps*Cp] with rows = phases*C_out
// rounded up to a multiple of 128.  FP32 semantics use three bf16 products per
// step (hi*hi + hi*lo + lo*hi, "split" mode); FP16-weight semantics use one
// fp16 product.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace rk {

constexpr int CONV_MAX_TAPS = 16;
constexpr int CONV_W_ROWS = 128;   // weight rows per tile (the MMA M); weight planes are padded to a multiple
constexpr int STATS_ROWS = 64;     // rows per InstanceNorm partial ("part") everywhere in the library

struct ConvArgs {
    int M;              // GEMM rows (time) per phase
    int C_out;          // output channels (the last channel tile may be partial)
    int kblocks;        // Cp / 64
    int taps;
    int tap_off[CONV_MAX_TAPS];
    int a_off;          // in_row = m + a_off + tap_off[k]
    int b_phase_rows;   // weight-row offset between phases (= C_out), 0 when one phase
    int T_out;          // valid output rows are [o_min, T_out)
    int o_min;
    int o_stride, o_off, o_phase_step;  // out_row = m*o_stride + o_off + phase*o_phase_step
    float* y;
    int ldy;
    const float* bias;  // [C_out] or null
    const float* res;   // residual rows res[(out_row >> res_shift) * ldres + c] or null
    int ldres, res_shift;
    const float* acc_in;  // y = acc_in + v or null
    int ldacc;
    float alpha;          // final scale
    int act;              // 0: none, 1: tanh-GELU after bias (ALBERT FFN, src/kernels.cu:151-158)
    float* stats;         // per-part column sums, or null: part p = phase*ceil(M/64) + m/64 covers 64 rows;
                          //   sums at stats[p*stats_ld + c], squares at stats[(stats_parts + p)*stats_ld + c]
    int stats_ld;         // row pitch of the partials (>= C_out; wider for channel-concatenated inputs)
    int stats_parts;      // ceil(M / 64) * phases
    int dup_src_row;      // >= 0: the accumulator of out_row == dup_src_row is also written to row 0
                          // (with residual row 0): reflection pad (1, 0) of the ConvTranspose output
    const int* part_rows; // segmented rows (one phase only): rows [64p, 64p + part_rows[p]) of each 64-row
                          //   part are valid; the others (gaps between utterances) are neither stored nor
                          //   counted in the statistics; null = every row < M is valid
    uint32_t* err;        // device error word
    // filled by conv_tc_launch
    int k_split;          // > 1: the reduction is split over k_split CTAs per tile (see conv_tc_launch)
    float* part_out;      // split-K raw accumulators [k_split][phases*M][C_out]
    int min_off;          // smallest tap offset (the activation tile starts there)
    int act_box;          // activation TMA box rows; the tile is two boxes
    int desc_mode;        // shared-memory descriptor base-offset convention for row-shifted starts
};

// Operands of one launch: the activation planes (the launcher encodes their
// tensor maps) and the weights' pre-encoded maps (box 64 x 128).
struct ConvOperands {
    const void* act_hi = nullptr;
    const void* act_lo = nullptr;   // split mode only
    uint64_t act_rows = 0;          // rows of the activation planes (reads beyond are zero: padding)
    uint64_t act_cp = 0;            // Cp (columns = row pitch, elements)
    CUtensorMap w_hi, w_lo;         // w_lo unused in fp16 mode
    // Optional split-K scratch (device, FP32).  When a launch has too few output
    // tiles to fill the GPU and a long reduction, the reduction is split across
    // CTAs that write raw partial accumulators here, and a second kernel sums
    // them in a fixed order and applies the epilogue.  Launches that may run
    // concurrently must not share a scratch buffer.
    float* scratch = nullptr;
    size_t scratch_bytes = 0;
};

// Encodes a 2-D K-major tile map (box 64 x box_rows, 128B swizzle) over a
// 16-bit matrix with `rows` rows of `cols` elements and `ld` elements per row.
bool make_tmap_k64(CUtensorMap* m, const void* base, bool bf16, uint64_t cols, uint64_t rows, uint64_t ld,
                   uint32_t box_rows);

// Weight-plane rows to allocate for `rows` = phases * C_out (a multiple of CONV_W_ROWS).
inline int conv_tc_weight_rows(int rows) { return (rows + CONV_W_ROWS - 1) / CONV_W_ROWS * CONV_W_ROWS; }

// Number of InstanceNorm partials a launch writes: ceil(M / 64) * phases.
inline int conv_tc_stats_parts(int M, int n_phases) { return (M + STATS_ROWS - 1) / STATS_ROWS * n_phases; }

// Launch; split = three-pass bf16 mode.  n_phases = polyphase count.
// Enqueues one kernel, or two (split-K partials, then the ordered reduction
// and epilogue) when ops.scratch is set and the launch has few tiles.
// `kernels` (nullable) receives the number of kernels enqueued.
cudaError_t conv_tc_launch(const ConvOperands& ops, const ConvArgs& a, bool split, int n_phases,
                           cudaStream_t stream, int* kernels = nullptr);

// Sets the kernels' dynamic shared-memory limits on the current device (call
// once per device before the first launch, outside any stream capture).
cudaError_t conv_tc_init();

}  // namespace rk
