// ref_shim.cu -- test infrastructure, not product code.
//
// A C-ABI shim over the reference's own CUDA kernel launchers (declared in the
// reference's src/kernels.h, compiled from src/kernels.cu where it lies; see
// oracle/Makefile target `ref`).  Each entry takes HOST arrays, copies them to
// the device, runs one reference launcher on the default stream, copies the
// result back and frees everything, so that a Python script can call the
// reference through ctypes and record golden input/output vectors
// (tests/golden/make_golden.py).  Nothing in the product links this file.
//
// Return value: 0, or the cudaError_t of the first failing call.
#include <cuda_runtime.h>

#include <vector>

#include "kernels.h"

namespace {

struct Dev {
    std::vector<void*> ptrs;
    cudaError_t err = cudaSuccess;
    template <class T>
    T* in(const T* h, size_t n) {
        T* d = out<T>(n);
        if (d && n && err == cudaSuccess) err = cudaMemcpy(d, h, n * sizeof(T), cudaMemcpyHostToDevice);
        return d;
    }
    template <class T>
    T* out(size_t n) {
        void* d = nullptr;
        if (err == cudaSuccess) err = cudaMalloc(&d, (n ? n : 1) * sizeof(T));
        if (d) {
            ptrs.push_back(d);
            if (err == cudaSuccess) err = cudaMemset(d, 0, (n ? n : 1) * sizeof(T));
        }
        return (T*)d;
    }
    template <class T>
    void back(T* h, const T* d, size_t n) {
        if (err == cudaSuccess) err = cudaDeviceSynchronize();
        if (err == cudaSuccess) err = cudaGetLastError();
        if (err == cudaSuccess && n) err = cudaMemcpy(h, d, n * sizeof(T), cudaMemcpyDeviceToHost);
    }
    ~Dev() {
        for (void* p : ptrs) cudaFree(p);
    }
};

}  // namespace

extern "C" {

// SineGen: sinegen_phase_f32 + sinegen_source_f32 (src/kernels.h:302-318),
// called as src/rokoko.cpp:1149-1151 does.
int ref_sinegen(const float* f0, int L2, const float* rand_ini, const float* lw, const float* lb, unsigned seed,
                float* phase_low, float* har_source) {
    Dev d;
    const int T_audio = L2 * 300;
    float* df0 = d.in(f0, L2);
    float* dri = d.in(rand_ini, 9);
    float* dlw = d.in(lw, 9);
    float* dlb = d.in(lb, 1);
    float* dph = d.out<float>((size_t)L2 * 9);
    float* dsrc = d.out<float>(T_audio);
    if (d.err) return d.err;
    rokoko::sinegen_phase_f32(df0, dri, dph, L2, 0);
    rokoko::sinegen_source_f32(dph, df0, dlw, dlb, dsrc, L2, T_audio, seed, 0);
    d.back(phase_low, dph, (size_t)L2 * 9);
    d.back(har_source, dsrc, T_audio);
    return d.err;
}

// stft_f32 (src/kernels.h:212-214): mag, phase [11, frames], frames = T/hop + 1.
int ref_stft(const float* x, int T, int n_fft, int hop, float* mag, float* phase) {
    Dev d;
    const int frames = T / hop + 1, nb = n_fft / 2 + 1;
    float* dx = d.in(x, T);
    float* dm = d.out<float>((size_t)nb * frames);
    float* dp = d.out<float>((size_t)nb * frames);
    if (d.err) return d.err;
    rokoko::stft_f32(dx, dm, dp, T, n_fft, hop, 0);
    d.back(mag, dm, (size_t)nb * frames);
    d.back(phase, dp, (size_t)nb * frames);
    return d.err;
}

// istft_f32 (src/kernels.h:222-224): mag (already exp'd), phase (already sin'd) [11, frames].
int ref_istft(const float* mag, const float* phase, int frames, int n_fft, int hop, int T, float* y) {
    Dev d;
    const int nb = n_fft / 2 + 1;
    float* dm = d.in(mag, (size_t)nb * frames);
    float* dp = d.in(phase, (size_t)nb * frames);
    float* dy = d.out<float>(T);
    if (d.err) return d.err;
    rokoko::istft_f32(dm, dp, dy, frames, n_fft, hop, T, 0);
    d.back(y, dy, T);
    return d.err;
}

// exp_f32 / sin_f32 (src/kernels.h:199-204).
int ref_exp_sin(const float* x, int n, float* ex, float* sn) {
    Dev d;
    float* dx = d.in(x, n);
    float* de = d.out<float>(n);
    float* ds = d.out<float>(n);
    if (d.err) return d.err;
    rokoko::exp_f32(dx, de, n, 0);
    rokoko::sin_f32(dx, ds, n, 0);
    d.back(ex, de, n);
    d.back(sn, ds, n);
    return d.err;
}

// instance_norm_style_affine_f32 (src/kernels.h:118-124); snake_alpha may be null.
int ref_adain(const float* x, int T, int C, const float* norm_w, const float* norm_b, const float* gamma,
              const float* beta, const float* snake_alpha, float* y) {
    Dev d;
    float* dx = d.in(x, (size_t)T * C);
    float* dw = d.in(norm_w, C);
    float* db = d.in(norm_b, C);
    float* dg = d.in(gamma, C);
    float* dbe = d.in(beta, C);
    float* da = snake_alpha ? d.in(snake_alpha, C) : nullptr;
    float* dws = d.out<float>((size_t)2 * C);
    float* dy = d.out<float>((size_t)T * C);
    if (d.err) return d.err;
    rokoko::instance_norm_style_affine_f32(dx, dw, db, dg, dbe, dy, dws, C, T, 1e-5f, 0, da);
    d.back(y, dy, (size_t)T * C);
    return d.err;
}

// layer_norm_f32 (src/kernels.h:43-44) and ada_layer_norm_f32 (src/kernels.h:131-133).
int ref_layer_norm(const float* x, int N, int D, const float* gamma, const float* beta, float eps, int ada,
                   float* y) {
    Dev d;
    float* dx = d.in(x, (size_t)N * D);
    float* dg = d.in(gamma, D);
    float* db = d.in(beta, D);
    float* dy = d.out<float>((size_t)N * D);
    if (d.err) return d.err;
    if (ada)
        rokoko::ada_layer_norm_f32(dx, dg, db, dy, N, D, eps, 0);
    else
        rokoko::layer_norm_f32(dx, dg, db, dy, N, D, eps, 0);
    d.back(y, dy, (size_t)N * D);
    return d.err;
}

// round_clamp_durations_f32 + build_alignment_f32 (src/kernels.h:320-328):
// float durations -> int durations, L, and the [T, L] alignment (L <= max_L).
int ref_durations_alignment(const float* dur, int T, int max_L, int* int_dur, int* L_out, float* align) {
    Dev d;
    float* dd = d.in(dur, T);
    int* di = d.out<int>(T);
    int* dL = d.out<int>(1);
    if (d.err) return d.err;
    rokoko::round_clamp_durations_f32(dd, di, dL, T, 0);
    d.back(int_dur, di, T);
    d.back(L_out, dL, 1);
    if (d.err) return d.err;
    const int L = *L_out;
    if (L < 0 || L > max_L) return -1;
    float* da = d.out<float>((size_t)T * L);
    if (d.err) return d.err;
    rokoko::build_alignment_f32(di, da, T, L, 0);
    d.back(align, da, (size_t)T * L);
    return d.err;
}

// sigmoid_sum_f32 (src/kernels.h:161-162): the duration head's sum of sigmoids.
int ref_sigmoid_sum(const float* x, int N, int D, float* y) {
    Dev d;
    float* dx = d.in(x, (size_t)N * D);
    float* dy = d.out<float>(N);
    if (d.err) return d.err;
    rokoko::sigmoid_sum_f32(dx, dy, N, D, 0);
    d.back(y, dy, N);
    return d.err;
}

// lstm_gates_f32 (src/kernels.h:230-232): one step of gate activations.
int ref_lstm_gates(const float* gates, const float* c_prev, int H, float* c_out, float* h_out) {
    Dev d;
    float* dg = d.in(gates, (size_t)4 * H);
    float* dc = d.in(c_prev, H);
    float* dh = d.out<float>(H);
    if (d.err) return d.err;
    rokoko::lstm_gates_f32(dg, dc, dc, dh, H, 0);
    d.back(c_out, dc, H);
    d.back(h_out, dh, H);
    return d.err;
}

// conv1d_general_f32 (src/kernels.h:183-186): x [T_in, C_in], w [C_out, C_in, K].
int ref_conv1d(const float* x, const float* w, const float* bias, int C_in, int C_out, int T_in, int K, int stride,
               int pad, int dil, float* y) {
    Dev d;
    const int T_out = (T_in + 2 * pad - dil * (K - 1) - 1) / stride + 1;
    float* dx = d.in(x, (size_t)T_in * C_in);
    float* dw = d.in(w, (size_t)C_out * C_in * K);
    float* db = bias ? d.in(bias, C_out) : nullptr;
    float* dy = d.out<float>((size_t)T_out * C_out);
    if (d.err) return d.err;
    rokoko::conv1d_general_f32(dx, dw, db, dy, C_in, C_out, T_in, K, stride, pad, dil, 0);
    d.back(y, dy, (size_t)T_out * C_out);
    return d.err;
}

// conv_transpose1d_depthwise_f32 (src/kernels.h:140-143).
int ref_convT_depthwise(const float* x, const float* w, const float* bias, int C, int T_in, int K, int stride,
                        int pad, int out_pad, float* y) {
    Dev d;
    const int T_out = (T_in - 1) * stride - 2 * pad + K + out_pad;
    float* dx = d.in(x, (size_t)T_in * C);
    float* dw = d.in(w, (size_t)C * K);
    float* db = d.in(bias, C);
    float* dy = d.out<float>((size_t)T_out * C);
    if (d.err) return d.err;
    rokoko::conv_transpose1d_depthwise_f32(dx, dw, db, dy, C, T_in, K, stride, pad, out_pad, 0);
    d.back(y, dy, (size_t)T_out * C);
    return d.err;
}

// weight_norm_f32 (src/kernels.h:100-101).
int ref_weight_norm(const float* g, const float* v, int C_out, int fan_in, float* w) {
    Dev d;
    float* dg = d.in(g, C_out);
    float* dv = d.in(v, (size_t)C_out * fan_in);
    float* dw = d.out<float>((size_t)C_out * fan_in);
    if (d.err) return d.err;
    rokoko::weight_norm_f32(dg, dv, dw, C_out, fan_in, 0);
    d.back(w, dw, (size_t)C_out * fan_in);
    return d.err;
}

// reflection_pad_1d_f32 (src/kernels.h:192-194).
int ref_reflection_pad(const float* x, int C, int T, int pl, int pr, float* y) {
    Dev d;
    float* dx = d.in(x, (size_t)T * C);
    float* dy = d.out<float>((size_t)(T + pl + pr) * C);
    if (d.err) return d.err;
    rokoko::reflection_pad_1d_f32(dx, dy, C, T, pl, pr, 0);
    d.back(y, dy, (size_t)(T + pl + pr) * C);
    return d.err;
}

// gelu_f32 / leaky_relu_f32 (src/kernels.h:59-65).
int ref_gelu_lrelu(const float* x, int n, float slope, float* g, float* l) {
    Dev d;
    float* dx = d.in(x, n);
    float* dg = d.out<float>(n);
    float* dl = d.out<float>(n);
    if (d.err) return d.err;
    rokoko::gelu_f32(dx, dg, n, 0);
    rokoko::leaky_relu_f32(dx, dl, n, slope, 0);
    d.back(g, dg, n);
    d.back(l, dl, n);
    return d.err;
}

// softmax_f32 (src/kernels.h:71): rows of D.
int ref_softmax(const float* x, int N, int D, float* y) {
    Dev d;
    float* dx = d.in(x, (size_t)N * D);
    float* dy = d.out<float>((size_t)N * D);
    if (d.err) return d.err;
    rokoko::softmax_f32(dx, dy, N, D, 0);
    d.back(y, dy, (size_t)N * D);
    return d.err;
}

}  // extern "C"
