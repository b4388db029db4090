// pack.cuh -- operand producers for the tcgen05 conv: FP32 activations or
// weights -> 16-bit K-major planes (split bf16 hi/lo, or fp16), with optional
// fused per-channel affine (AdaIN), Snake and LeakyReLU on the way.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace rk {

struct PackArgs {
    const float* x;   // source rows
    int ldx;          // floats per source row
    int rows_src;     // valid source rows (rows outside read as 0)
    int C;            // channels taken from each source row
    int rows_dst;     // destination rows to write
    int Cp;           // destination row length (multiple of 64), zero padded
    void* hi;         // bf16 hi plane (split) or fp16 plane
    void* lo;         // bf16 lo plane (split only)
    // super-row gather (strided conv): dst[q][r*C + c] = f(src[q*sr_stride - sr_pad + r][c]) for r < sr_stride
    int sr_stride;    // 1 = plain copy
    int sr_pad;
    const float* scale;   // per-channel affine y = scale*x + shift (nullable)
    const float* shift;
    const float* snake;   // Snake alpha per channel (nullable)
    float slope;          // LeakyReLU slope
    int lrelu;            // apply LeakyReLU
    // segmented rows (sr_stride 1 only): destination row q of part q/64 is valid
    // when q % 64 < part_rows[q/64] and then uses the scale / shift of segment
    // part_seg[q/64] (at + seg * coef_stride); other rows are written as zeros
    const int* part_seg;
    const int* part_rows;
    int coef_stride;
};

// split = bf16 hi/lo; otherwise one fp16 plane.
cudaError_t pack_act(const PackArgs& a, bool split, cudaStream_t st);

// Weights [C_out][K][C_in] fp32 (NHWC, the reference's cutlass_reshape_weights
// layout) -> planes [C_out][taps'][Cp'] where a strided conv is re-expressed
// over super-rows: taps' = ceil(K/stride), Cp' = round_up(stride*C_in, 64).
cudaError_t pack_weights_nhwc(const float* w, int C_out, int K, int C_in, int stride, void* hi, void* lo,
                              bool split, cudaStream_t st);

// Average of the three generator resblocks followed by LeakyReLU, written as
// the next conv's operand:  v = ((x0 + x1) + x2) * (1/3);  v = lrelu(v, slope).
// The reference does memset + 3 adds + scale + a separate LeakyReLU
// (src/rokoko.cpp:1096-1116, 1253).  f32_out (nullable) also receives the
// average before the LeakyReLU.
cudaError_t pack_avg3(const float* x0, const float* x1, const float* x2, int T, int C, int Cp, float slope, void* hi,
                      void* lo, bool split, float* f32_out, cudaStream_t st);

}  // namespace rk
