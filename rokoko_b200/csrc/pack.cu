// pack.cu -- FP32 -> 16-bit operand planes for the tcgen05 conv.
//
// The reference casts every activation to FP16 in a separate kernel before
// each FP16 conv/GEMM (cast_f32_to_f16[_pad], src/kernels.cu:1048-1058,
// 1283-1302) and applies AdaIN / Snake / LeakyReLU in yet other passes
// (src/kernels.cu:443-504, 170-183).  Here one pass reads the FP32 tensor and
// writes the conv's operand directly, channel-padded to a multiple of 64.
// Split mode writes hi = bf16(v) and lo = bf16(v - hi), so that
// hi*Whi + hi*Wlo + lo*Whi reproduces an FP32 product to ~2^-16 relative.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "pack.cuh"

namespace rk {

namespace {

// sin(x) for the Snake activation: Cody-Waite reduction of x to r in [-pi, pi]
// with 2 pi split as C1 + C2 (C1 = 6.28125 has 8 significant bits, so k * C1
// is exact for |k| < 2^15 and the first reduction step is exact), then the
// hardware sine on the reduced argument (documented maximum absolute error
// 2^-21.41 on [-pi, pi]).  Total absolute error stays below 1e-6 for |x| < 1e4,
// an order of magnitude under the 2^-16 relative precision of the bf16 hi + lo
// operand the result is packed into; beyond that range the library sinf is used.
__device__ __forceinline__ float snake_sin(float x) {
    if (fabsf(x) >= 1.0e4f) return sinf(x);
    const float k = rintf(x * 0.15915494309189535f);
    float r = fmaf(-k, 6.28125f, x);
    r = fmaf(-k, 1.9353071795864769e-3f, r);
    return __sinf(r);
}

// 1/alpha of the Snake term x + sin^2(alpha x) / alpha: the hardware
// reciprocal (at most 1 ulp from the rounded quotient), far inside the 2^-16
// relative precision of the packed operand, in one instruction instead of a
// correctly rounded division per element.
__device__ __forceinline__ float snake_inv(float al) { return __fdividef(1.0f, al); }

__device__ __forceinline__ float act_transform(float v, int c, const PackArgs& a, int seg) {
    if (a.scale) v = a.scale[(size_t)seg * a.coef_stride + c] * v + a.shift[(size_t)seg * a.coef_stride + c];
    if (a.snake) {
        const float al = a.snake[c];
        const float s = snake_sin(al * v);
        v = fmaf(s * s, snake_inv(al), v);
    }
    if (a.lrelu) v = v > 0.0f ? v : a.slope * v;
    return v;
}

// one thread = 8 consecutive destination channels of one destination row
// I = int when the group count leaves room for the grid stride below 2^31.
template <bool SPLIT, typename I>
__global__ void pack_act_kernel(PackArgs a) {
    const int groups = a.Cp >> 3;
    const I total = (I)a.rows_dst * groups;
    for (I idx = (I)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (I)gridDim.x * blockDim.x) {
        const int q = (int)(idx / groups);
        const int g = (int)(idx - (I)q * groups);
        int seg = 0;
        if (a.part_seg) seg = (q & 63) < a.part_rows[q >> 6] ? a.part_seg[q >> 6] : -1;
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int cd = g * 8 + j;          // destination channel
            const int r = cd / a.C;            // sub-row within the super-row
            const int c = cd - r * a.C;        // source channel
            float x = 0.0f;
            if (r < a.sr_stride && seg >= 0) {
                const int row = q * a.sr_stride - a.sr_pad + r;
                if (row >= 0 && row < a.rows_src) x = act_transform(a.x[(long)row * a.ldx + c], c, a, seg);
            }
            v[j] = x;
        }
        if (SPLIT) {
            __align__(16) __nv_bfloat16 h[8], l[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                h[j] = __float2bfloat16_rn(v[j]);
                l[j] = __float2bfloat16_rn(v[j] - __bfloat162float(h[j]));
            }
            reinterpret_cast<uint4*>(a.hi)[idx] = *reinterpret_cast<uint4*>(h);
            reinterpret_cast<uint4*>(a.lo)[idx] = *reinterpret_cast<uint4*>(l);
        } else {
            __align__(16) __half h[8];
#pragma unroll
            for (int j = 0; j < 8; j++) h[j] = __float2half_rn(v[j]);
            reinterpret_cast<uint4*>(a.hi)[idx] = *reinterpret_cast<uint4*>(h);
        }
    }
}

// Fast path: plain rows (no super-row gather), C a multiple of 8, every
// per-channel table 16-byte aligned, fewer than 2^31 groups.  One thread = 8
// channels of one row: two float4 loads of the row and of each per-channel
// table, one 16-byte store per plane.
__device__ __forceinline__ void load8(const float* p, int c, float (&v)[8]) {
    const float4 a = reinterpret_cast<const float4*>(p + c)[0], b = reinterpret_cast<const float4*>(p + c)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

template <bool SPLIT>
__global__ void pack_act_vec_kernel(PackArgs a) {
    const int groups = a.Cp >> 3, cgroups = a.C >> 3;
    const int total = a.rows_dst * groups;
    // (q, g) = divmod(idx, groups), advanced by the grid stride without a division per item
    const int stride = gridDim.x * blockDim.x, dq = stride / groups, dg = stride - dq * groups;
    int idx = blockIdx.x * blockDim.x + threadIdx.x;
    int q = idx / groups, g = idx - q * groups;
    for (; idx < total; idx += stride, q += dq, g += dg) {
        if (g >= groups) { g -= groups; q++; }
        int seg = 0;
        if (a.part_seg) seg = (q & 63) < a.part_rows[q >> 6] ? a.part_seg[q >> 6] : -1;
        float v[8];
        if (g < cgroups && q < a.rows_src && seg >= 0) {
            load8(a.x + (size_t)q * a.ldx, g * 8, v);
            if (a.scale) {
                float sc[8], sh[8];
                load8(a.scale + (size_t)seg * a.coef_stride, g * 8, sc);
                load8(a.shift + (size_t)seg * a.coef_stride, g * 8, sh);
#pragma unroll
                for (int j = 0; j < 8; j++) v[j] = sc[j] * v[j] + sh[j];
            }
            if (a.snake) {
                float al[8];
                load8(a.snake, g * 8, al);
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const float sn = snake_sin(al[j] * v[j]);
                    v[j] = fmaf(sn * sn, snake_inv(al[j]), v[j]);
                }
            }
            if (a.lrelu) {
#pragma unroll
                for (int j = 0; j < 8; j++) v[j] = v[j] > 0.0f ? v[j] : a.slope * v[j];
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; j++) v[j] = 0.0f;
        }
        if (SPLIT) {
            __align__(16) __nv_bfloat16 h[8], l[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                h[j] = __float2bfloat16_rn(v[j]);
                l[j] = __float2bfloat16_rn(v[j] - __bfloat162float(h[j]));
            }
            reinterpret_cast<uint4*>(a.hi)[idx] = *reinterpret_cast<uint4*>(h);
            reinterpret_cast<uint4*>(a.lo)[idx] = *reinterpret_cast<uint4*>(l);
        } else {
            __align__(16) __half h[8];
#pragma unroll
            for (int j = 0; j < 8; j++) h[j] = __float2half_rn(v[j]);
            reinterpret_cast<uint4*>(a.hi)[idx] = *reinterpret_cast<uint4*>(h);
        }
    }
}

template <bool SPLIT>
__global__ void pack_w_kernel(const float* w, int C_out, int K, int C_in, int stride, int taps, int Cp, void* hi,
                              void* lo) {
    const long total = (long)C_out * taps * Cp;
    for (long idx = (long)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (long)gridDim.x * blockDim.x) {
        const int cd = (int)(idx % Cp);
        const long t2 = idx / Cp;
        const int j = (int)(t2 % taps);
        const int co = (int)(t2 / taps);
        const int r = cd / C_in, ci = cd - r * C_in;
        const int k = j * stride + r;
        float v = 0.0f;
        if (r < stride && k < K) v = w[((long)co * K + k) * C_in + ci];
        if (SPLIT) {
            __nv_bfloat16 h = __float2bfloat16_rn(v);
            reinterpret_cast<__nv_bfloat16*>(hi)[idx] = h;
            reinterpret_cast<__nv_bfloat16*>(lo)[idx] = __float2bfloat16_rn(v - __bfloat162float(h));
        } else {
            reinterpret_cast<__half*>(hi)[idx] = __float2half_rn(v);
        }
    }
}

template <bool SPLIT>
__global__ void pack_avg3_kernel(const float* __restrict__ x0, const float* __restrict__ x1,
                                 const float* __restrict__ x2, int T, int C, int Cp, float slope, void* hi, void* lo,
                                 float* f32_out) {
    const int groups = Cp >> 3;
    const long total = (long)T * groups;
    const float third = 1.0f / 3.0f;
    for (long idx = (long)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (long)gridDim.x * blockDim.x) {
        const int t = (int)(idx / groups);
        const int g = (int)(idx - (long)t * groups);
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int c = g * 8 + j;
            float a = 0.f;
            if (c < C) {
                const size_t o = (size_t)t * C + c;
                a = ((x0[o] + x1[o]) + x2[o]) * third;
                if (f32_out) f32_out[o] = a;
                a = a > 0.f ? a : slope * a;
            }
            v[j] = a;
        }
        if (SPLIT) {
            __align__(16) __nv_bfloat16 h[8], l[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                h[j] = __float2bfloat16_rn(v[j]);
                l[j] = __float2bfloat16_rn(v[j] - __bfloat162float(h[j]));
            }
            reinterpret_cast<uint4*>(hi)[idx] = *reinterpret_cast<uint4*>(h);
            reinterpret_cast<uint4*>(lo)[idx] = *reinterpret_cast<uint4*>(l);
        } else {
            __align__(16) __half h[8];
#pragma unroll
            for (int j = 0; j < 8; j++) h[j] = __float2half_rn(v[j]);
            reinterpret_cast<uint4*>(hi)[idx] = *reinterpret_cast<uint4*>(h);
        }
    }
}

// pack_avg3 fast path: C a multiple of 8, every tensor 16-byte aligned, fewer
// than 2^31 groups; float4 loads and stores, 32-bit indexing.
template <bool SPLIT>
__global__ void pack_avg3_vec_kernel(const float* __restrict__ x0, const float* __restrict__ x1,
                                     const float* __restrict__ x2, int T, int C, int Cp, float slope, void* hi,
                                     void* lo, float* f32_out) {
    const int groups = Cp >> 3, cgroups = C >> 3;
    const int total = T * groups;
    const float third = 1.0f / 3.0f;
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
        const int t = idx / groups;
        const int g = idx - t * groups;
        float v[8];
        if (g < cgroups) {
            const size_t o = (size_t)t * C + g * 8;
            float a0[8], a1[8], a2[8];
            load8(x0 + o, 0, a0);
            load8(x1 + o, 0, a1);
            load8(x2 + o, 0, a2);
#pragma unroll
            for (int j = 0; j < 8; j++) v[j] = ((a0[j] + a1[j]) + a2[j]) * third;
            if (f32_out) {
                reinterpret_cast<float4*>(f32_out + o)[0] = make_float4(v[0], v[1], v[2], v[3]);
                reinterpret_cast<float4*>(f32_out + o)[1] = make_float4(v[4], v[5], v[6], v[7]);
            }
#pragma unroll
            for (int j = 0; j < 8; j++) v[j] = v[j] > 0.f ? v[j] : slope * v[j];
        } else {
#pragma unroll
            for (int j = 0; j < 8; j++) v[j] = 0.0f;
        }
        if (SPLIT) {
            __align__(16) __nv_bfloat16 h[8], l[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                h[j] = __float2bfloat16_rn(v[j]);
                l[j] = __float2bfloat16_rn(v[j] - __bfloat162float(h[j]));
            }
            reinterpret_cast<uint4*>(hi)[idx] = *reinterpret_cast<uint4*>(h);
            reinterpret_cast<uint4*>(lo)[idx] = *reinterpret_cast<uint4*>(l);
        } else {
            __align__(16) __half h[8];
#pragma unroll
            for (int j = 0; j < 8; j++) h[j] = __float2half_rn(v[j]);
            reinterpret_cast<uint4*>(hi)[idx] = *reinterpret_cast<uint4*>(h);
        }
    }
}

int grid_for(long work, int threads) {
    long b = (work + threads - 1) / threads;
    if (b > 148L * 16) b = 148L * 16;
    return (int)(b < 1 ? 1 : b);
}

}  // namespace

cudaError_t pack_act(const PackArgs& a, bool split, cudaStream_t st) {
    if ((a.Cp & 63) || a.sr_stride < 1 || (a.part_seg && (a.sr_stride != 1 || !a.part_rows)) ||
        (a.part_seg && a.scale && (a.coef_stride & 3)))
        return cudaErrorInvalidValue;
    const long total = (long)a.rows_dst * (a.Cp >> 3);
    if (total == 0) return cudaSuccess;
    auto al16 = [](const float* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const bool vec = a.sr_stride == 1 && a.sr_pad == 0 && (a.C & 7) == 0 && (a.ldx & 3) == 0 && al16(a.x) &&
                     al16(a.scale) && al16(a.shift) && al16(a.snake) && total < (1L << 31) - 148L * 16 * 256;
    if (vec) {
        if (split) pack_act_vec_kernel<true><<<grid_for(total, 256), 256, 0, st>>>(a);
        else pack_act_vec_kernel<false><<<grid_for(total, 256), 256, 0, st>>>(a);
    } else {
        const bool small = total < (1L << 31) - 148L * 16 * 256;
        if (split && small) pack_act_kernel<true, int><<<grid_for(total, 256), 256, 0, st>>>(a);
        else if (split) pack_act_kernel<true, long><<<grid_for(total, 256), 256, 0, st>>>(a);
        else if (small) pack_act_kernel<false, int><<<grid_for(total, 256), 256, 0, st>>>(a);
        else pack_act_kernel<false, long><<<grid_for(total, 256), 256, 0, st>>>(a);
    }
    return cudaGetLastError();
}

cudaError_t pack_avg3(const float* x0, const float* x1, const float* x2, int T, int C, int Cp, float slope, void* hi,
                      void* lo, bool split, float* f32_out, cudaStream_t st) {
    if (Cp & 63) return cudaErrorInvalidValue;
    const long total = (long)T * (Cp >> 3);
    auto al16 = [](const float* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const bool vec = (C & 7) == 0 && al16(x0) && al16(x1) && al16(x2) && al16(f32_out) &&
                     total < (1L << 31) - 148L * 16 * 256;
    if (vec) {
        if (split) pack_avg3_vec_kernel<true><<<grid_for(total, 256), 256, 0, st>>>(x0, x1, x2, T, C, Cp, slope, hi, lo, f32_out);
        else pack_avg3_vec_kernel<false><<<grid_for(total, 256), 256, 0, st>>>(x0, x1, x2, T, C, Cp, slope, hi, lo, f32_out);
    } else {
        if (split) pack_avg3_kernel<true><<<grid_for(total, 256), 256, 0, st>>>(x0, x1, x2, T, C, Cp, slope, hi, lo, f32_out);
        else pack_avg3_kernel<false><<<grid_for(total, 256), 256, 0, st>>>(x0, x1, x2, T, C, Cp, slope, hi, lo, f32_out);
    }
    return cudaGetLastError();
}

cudaError_t pack_weights_nhwc(const float* w, int C_out, int K, int C_in, int stride, void* hi, void* lo,
                              bool split, cudaStream_t st) {
    const int taps = (K + stride - 1) / stride;
    const int Cp = (stride * C_in + 63) / 64 * 64;
    const long total = (long)C_out * taps * Cp;
    if (split) pack_w_kernel<true><<<grid_for(total, 256), 256, 0, st>>>(w, C_out, K, C_in, stride, taps, Cp, hi, lo);
    else pack_w_kernel<false><<<grid_for(total, 256), 256, 0, st>>>(w, C_out, K, C_in, stride, taps, Cp, hi, lo);
    return cudaGetLastError();
}

}  // namespace rk
