"""Records golden input/output vectors from the reference's own CUDA kernels.

Runs on a machine with a B200 and the shim library built by
`make -C oracle ref` (oracle/_ref/libref_kernels.so: the reference's
src/kernels.cu compiled where it lies, behind oracle/ref_shim.cu).  Every
input is generated here from a fixed numpy seed; each reference launcher is
called once through ctypes and its output is stored beside its inputs in
ref_kernels.npz, which tests/test_golden.py compares against the CPU oracle.

    python tests/golden/make_golden.py OUT_DIR
"""
from __future__ import annotations

import ctypes
import json
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

F = ctypes.POINTER(ctypes.c_float)
I = ctypes.POINTER(ctypes.c_int)


def fp(a):
    return None if a is None else a.ctypes.data_as(F)


def ip(a):
    return a.ctypes.data_as(I)


def f32(a):
    return np.ascontiguousarray(a, np.float32)


def main(out_dir: str) -> None:
    import oracle  # only for rand_ini (the reference's host-side mt19937(42) draw, restated)
    so = os.path.join(ROOT, "oracle", "_ref", "libref_kernels.so")
    R = ctypes.CDLL(so)
    for name in ("ref_sinegen", "ref_stft", "ref_istft", "ref_exp_sin", "ref_adain", "ref_layer_norm",
                 "ref_durations_alignment", "ref_sigmoid_sum", "ref_lstm_gates", "ref_conv1d",
                 "ref_convT_depthwise", "ref_weight_norm", "ref_gelu_lrelu", "ref_softmax"):
        getattr(R, name).restype = ctypes.c_int
    R.ref_layer_norm.argtypes = [F, ctypes.c_int, ctypes.c_int, F, F, ctypes.c_float, ctypes.c_int, F]
    R.ref_gelu_lrelu.argtypes = [F, ctypes.c_int, ctypes.c_float, F, F]
    R.ref_sinegen.argtypes = [F, ctypes.c_int, F, F, F, ctypes.c_uint, F, F]

    def ok(rc, what):
        if rc != 0:
            raise RuntimeError(f"{what}: error {rc}")

    rng = np.random.default_rng(20240601)
    g = {}

    # ---- SineGen (seed 42 noise, rand_ini from mt19937(42)) ----
    L2 = 24
    t = np.arange(L2)
    f0 = 140 + 60 * np.sin(t / 3.0) + rng.normal(0, 5, L2)
    f0[3:6] = 0.0      # unvoiced
    f0[10] = 7.5       # below the 10 Hz voicing threshold
    f0[17] = 10.0      # exactly at the threshold (unvoiced: f0 > 10 is voiced)
    f0 = f32(f0)
    ri = f32(oracle.rand_ini())
    lw = f32(rng.normal(0, 0.4, 9))
    lb = f32([0.05])
    ph = np.empty(L2 * 9, np.float32)
    src = np.empty(L2 * 300, np.float32)
    ok(R.ref_sinegen(fp(f0), L2, fp(ri), fp(lw), fp(lb), 42, fp(ph), fp(src)), "sinegen")
    g.update(sg_f0=f0, sg_rand_ini=ri, sg_lw=lw, sg_lb=lb, sg_phase_low=ph, sg_har_source=src)

    # ---- STFT of that source (n_fft 20, hop 5) ----
    T = src.shape[0]
    frames = T // 5 + 1
    mag = np.empty((11, frames), np.float32)
    pha = np.empty((11, frames), np.float32)
    ok(R.ref_stft(fp(src), T, 20, 5, fp(mag), fp(pha)), "stft")
    g.update(stft_x=src, stft_mag=mag, stft_phase=pha)

    # ---- exp / sin + iSTFT on generator-style input c [frames, 22] ----
    nf = 97
    c = f32(rng.normal(0, 0.7, (nf, 22)))
    ct = f32(c.T)  # reference layout [22, frames]
    ex = np.empty(ct.size, np.float32)
    sn = np.empty(ct.size, np.float32)
    ok(R.ref_exp_sin(fp(ct), ct.size, fp(ex), fp(sn)), "exp_sin")
    ex = ex.reshape(22, nf)[:11].copy()
    sn = sn.reshape(22, nf)[11:].copy()
    Ta = (nf - 1) * 5
    y = np.empty(Ta, np.float32)
    ok(R.ref_istft(fp(ex), fp(sn), nf, 20, 5, Ta, fp(y)), "istft")
    g.update(istft_c=c, istft_y=y)

    # ---- AdaIN (InstanceNorm + style affine, optional Snake) ----
    for i, (T_, C_, snake) in enumerate([(37, 64, False), (300, 128, True), (5, 514, False), (1, 8, False)]):
        x = f32(rng.normal(0.3, 1.5, (T_, C_)))
        nw = f32(rng.normal(1, 0.1, C_))
        nb = f32(rng.normal(0, 0.1, C_))
        gm = f32(rng.normal(0, 0.2, C_))
        bt = f32(rng.normal(0, 0.2, C_))
        al = f32(rng.uniform(0.5, 1.5, C_)) if snake else None
        yv = np.empty_like(x)
        ok(R.ref_adain(fp(x), T_, C_, fp(nw), fp(nb), fp(gm), fp(bt), fp(al), fp(yv)), "adain")
        g.update({f"adain{i}_x": x, f"adain{i}_nw": nw, f"adain{i}_nb": nb, f"adain{i}_gamma": gm,
                  f"adain{i}_beta": bt, f"adain{i}_y": yv})
        if snake:
            g[f"adain{i}_alpha"] = al

    # ---- LayerNorm and AdaLayerNorm ----
    for i, (N, D, eps, ada) in enumerate([(9, 768, 1e-12, 0), (7, 512, 1e-5, 1), (3, 128, 1e-12, 0)]):
        x = f32(rng.normal(0.1, 2.0, (N, D)))
        gm = f32(rng.normal(1 if not ada else 0, 0.2, D))
        bt = f32(rng.normal(0, 0.2, D))
        yv = np.empty_like(x)
        ok(R.ref_layer_norm(fp(x), N, D, fp(gm), fp(bt), eps, ada, fp(yv)), "layer_norm")
        g.update({f"ln{i}_x": x, f"ln{i}_gamma": gm, f"ln{i}_beta": bt, f"ln{i}_y": yv,
                  f"ln{i}_meta": np.array([eps, ada], np.float64)})

    # ---- duration head: sigmoid sum, round half-even + clamp, alignment ----
    logits = f32(rng.normal(-0.5, 2.0, (23, 50)))
    ss = np.empty(23, np.float32)
    ok(R.ref_sigmoid_sum(fp(logits), 23, 50, fp(ss)), "sigmoid_sum")
    g.update(dur_logits=logits, dur_sigsum=ss)
    dur = f32([0.2, 0.5, 1.5, 2.5, 3.5, 7.49, 12.51, 0.0, 1.0, 4.5, 5.5, 2.4999, 30.7] +
              list(rng.uniform(0.3, 9.7, 10)))
    idur = np.empty(dur.size, np.int32)
    Lo = np.zeros(1, np.int32)
    align = np.empty((dur.size, 4096), np.float32)
    ok(R.ref_durations_alignment(fp(dur), dur.size, 4096, ip(idur), ip(Lo), fp(align)), "durations")
    L = int(Lo[0])
    align = align.reshape(-1)[: dur.size * L].reshape(dur.size, L).copy()
    g.update(dur_float=dur, dur_int=idur, dur_L=np.array([L], np.int32), dur_align=align)

    # ---- LSTM gate step ----
    H = 256
    gates = f32(rng.normal(0, 2.0, 4 * H))
    cp = f32(rng.normal(0, 1.0, H))
    co = np.empty(H, np.float32)
    ho = np.empty(H, np.float32)
    ok(R.ref_lstm_gates(fp(gates), fp(cp), H, fp(co), fp(ho)), "lstm_gates")
    g.update(lstm_gates=gates, lstm_c_prev=cp, lstm_c=co, lstm_h=ho)

    # ---- generic Conv1d (naive reference kernel) ----
    for i, (Ci, Co, T_, K, s, p, d, bias) in enumerate([
            (8, 6, 37, 7, 1, 9, 3, True),     # dilated resblock tap pattern
            (22, 16, 61, 12, 6, 3, 1, True),  # noise_convs.0 geometry (K 12, stride 6, pad 3)
            (5, 4, 10, 1, 1, 0, 1, False),    # 1x1 shortcut, no bias
            (1, 1, 20, 3, 2, 1, 1, True)]):   # F0 / N downsample
        x = f32(rng.normal(0, 1, (T_, Ci)))
        w = f32(rng.normal(0, 1 / np.sqrt(Ci * K), (Co, Ci, K)))
        b = f32(rng.normal(0, 0.1, Co)) if bias else None
        To = (T_ + 2 * p - d * (K - 1) - 1) // s + 1
        yv = np.empty((To, Co), np.float32)
        ok(R.ref_conv1d(fp(x), fp(w), fp(b), Ci, Co, T_, K, s, p, d, fp(yv)), "conv1d")
        g.update({f"conv{i}_x": x, f"conv{i}_w": w, f"conv{i}_y": yv,
                  f"conv{i}_geom": np.array([s, p, d], np.int32)})
        if bias:
            g[f"conv{i}_b"] = b

    # ---- depthwise ConvTranspose1d K3 s2 p1 op1 ----
    C_, T_ = 8, 19
    x = f32(rng.normal(0, 1, (T_, C_)))
    w = f32(rng.normal(0, 0.5, (C_, 3)))
    b = f32(rng.normal(0, 0.1, C_))
    yv = np.empty((2 * T_, C_), np.float32)
    ok(R.ref_convT_depthwise(fp(x), fp(w), fp(b), C_, T_, 3, 2, 1, 1, fp(yv)), "convT")
    g.update(convT_x=x, convT_w=w, convT_b=b, convT_y=yv)

    # ---- weight norm ----
    gv = f32(rng.uniform(0.2, 2.0, 6))
    v = f32(rng.normal(0, 1, (6, 8, 7)))
    wv = np.empty_like(v)
    ok(R.ref_weight_norm(fp(gv), fp(v), 6, 56, fp(wv)), "weight_norm")
    g.update(wn_g=gv, wn_v=v, wn_w=wv)

    # ---- GELU (tanh form) / LeakyReLU ----
    x = f32(np.concatenate([np.linspace(-8, 8, 1601), rng.normal(0, 3, 399)]))
    ge = np.empty_like(x)
    lr = np.empty_like(x)
    ok(R.ref_gelu_lrelu(fp(x), x.size, 0.2, fp(ge), fp(lr)), "gelu")
    g.update(act_x=x, act_gelu=ge, act_lrelu02=lr)

    # ---- softmax rows ----
    for i, (N, D) in enumerate([(5, 33), (4, 1), (2, 512)]):
        x = f32(rng.normal(0, 3, (N, D)))
        yv = np.empty_like(x)
        ok(R.ref_softmax(fp(x), N, D, fp(yv)), "softmax")
        g.update({f"sm{i}_x": x, f"sm{i}_y": yv})

    os.makedirs(out_dir, exist_ok=True)
    np.savez_compressed(os.path.join(out_dir, "ref_kernels.npz"), **g)
    try:
        gpu = subprocess.run(["nvidia-smi", "--query-gpu=name,driver_version", "--format=csv,noheader", "-i", "0"],
                             capture_output=True, text=True).stdout.strip()
    except OSError:
        gpu = "unknown"
    nvcc = subprocess.run(["nvcc", "--version"], capture_output=True, text=True).stdout.strip().splitlines()[-1]
    with open(os.path.join(out_dir, "ref_kernels.json"), "w") as f:
        json.dump({"source": "reference src/kernels.cu via oracle/ref_shim.cu", "gpu": gpu, "nvcc": nvcc,
                   "arrays": len(g), "generator": "tests/golden/make_golden.py"}, f, indent=1)
    print(f"wrote {len(g)} arrays to {out_dir}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(ROOT, "tests", "golden"))
