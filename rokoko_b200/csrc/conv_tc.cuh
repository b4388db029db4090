// conv_tc.cuh -- host interface of the tcgen05 implicit-GEMM Conv1d kernel.
//
// One kernel covers every dense contraction of the decoder/generator:
//   Conv1d (any K, dilation; stride 1)      out_row = m,             in_row = m + tap_off[k]
//   ConvTranspose1d as s polyphase convs   out_row = q*s + r - p,   in_row = q - j   (grid.z = phase r)
//   Linear / 1x1 conv                       K = 1
// GEMM view: M = time rows, N = output channels, reduction = taps x input
// channels.  Activations are [T, Cp] channels-last 16-bit planes (Cp = C_in
// rounded up to 64, zero padded); weights are [phases*C_out, taps*Cp].
// FP32 semantics use three bf16 products per step (hi*hi + hi*lo + lo*hi,
// "split" mode); FP16-weight semantics use one fp16 product.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace rk {

constexpr int CONV_MAX_TAPS = 16;

struct ConvArgs {
    int M;              // GEMM rows per phase
    int C_out;          // output channels (the last N tile may be partial)
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
    float* stats;         // per-CTA partial column sums, or null: part p = blockIdx.z*gridDim.x + blockIdx.x
                          //   sums at stats[p*stats_ld + c], squares at stats[(stats_parts + p)*stats_ld + c]
    int stats_ld;         // row pitch of the partials (>= C_out; wider for channel-concatenated inputs)
    int stats_parts;      // gridDim.x * gridDim.z
    int dup_src_row;      // >= 0: the accumulator of out_row == dup_src_row is also written to row 0
                          // (with residual row 0): reflection pad (1, 0) of the ConvTranspose output
    uint32_t* err;        // device error word
    // filled by conv_tc_launch
    int min_off;          // smallest tap offset (the halo tile starts there)
    int h_pad;            // halo tile rows: 128 + max_off - min_off, rounded up to 8
    int desc_mode;        // shared-memory descriptor base-offset convention for row-shifted starts
};

struct ConvOperands {
    CUtensorMap a_hi, a_lo, b_hi, b_lo;  // a_lo/b_lo unused in fp16 mode
};

// Encodes a 2-D K-major tile map (box 64 x box_rows, 128B swizzle) over a
// 16-bit matrix with `rows` rows of `cols` elements and `ld` elements per row.
bool make_tmap_k64(CUtensorMap* m, const void* base, bool bf16, uint64_t cols, uint64_t rows, uint64_t ld,
                   uint32_t box_rows);

// Rows of the activation tile the kernel loads per 64-channel block (the TMA
// box height of the activation tensor map): 128 + (max - min tap offset),
// rounded up to a multiple of 8.
int conv_tc_halo_rows(const int* tap_off, int taps);

// Launch; split = three-pass bf16 mode.  n_phases = grid.z.
cudaError_t conv_tc_launch(const ConvOperands& ops, const ConvArgs& a, bool split, int n_phases,
                           cudaStream_t stream);

// Sets the kernels' dynamic shared-memory limits on the current device (call
// once per device before the first launch, outside any stream capture).
cudaError_t conv_tc_init();

// N tile the launcher uses for a given C_out (32, 64 or 128).
int conv_tc_ntile(int C_out);

}  // namespace rk
