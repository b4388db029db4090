"""Command-line front-end (the reference's CLI is src/main.cu:56-345; its text
front-end, G2P and downloads are outside this library's scope).

    python -m rokoko_b200.cli decode [--L 400] [--seed 0] [--repeat 1] [-o out.wav] [--weights koko.bin]
        decoder + generator on seeded config-1 features (asr / F0 / N / style)
    python -m rokoko_b200.cli conv --cin 128 --cout 128 --T 48001 --K 7 --dil 3 [--fp16] [--repeat 3]
        one tcgen05 conv through rk_conv1d_fprop on random device data (microbenchmark / profiling)
    python -m rokoko_b200.cli synth --tokens 0,50,83,...,0 [--voice voice.bin] [--row N] [-o out.wav]
        full forward (rokoko_infer) on token ids; --voice is a raw float32 [rows, 256] voice pack
        (src/main.cu:46, src/rokoko.h:327-340: style row = min(T-2, rows-1))

Without --weights a seeded random-init KOKO v1 file is generated in memory.
WAV output is 16-bit PCM at 24 kHz (write_wav_to_, src/rokoko_common.h:62-99).
"""
from __future__ import annotations

import argparse
import struct
import sys
import time

import numpy as np


def write_wav(path: str, audio: np.ndarray, sr: int = 24000) -> None:
    pcm = np.clip(audio, -1.0, 1.0)
    pcm = (pcm * 32767.0).astype("<i2").tobytes()
    hdr = b"RIFF" + struct.pack("<I", 36 + len(pcm)) + b"WAVEfmt " + struct.pack("<IHHIIHH", 16, 1, 1, sr, sr * 2,
                                                                                 2, 16) + b"data" + struct.pack("<I", len(pcm))
    out = sys.stdout.buffer if path == "-" else open(path, "wb")
    out.write(hdr + pcm)
    if path != "-":
        out.close()


def _weights(path: str | None) -> bytes:
    from . import koko
    if path:
        with open(path, "rb") as f:
            return f.read()
    return koko.random_v1_blob(0)


def _conv_bench(a) -> int:
    import torch

    from . import lib
    L = lib.load()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(a.T, a.cin, device=dev, generator=g)
    w = torch.randn(a.cout, a.K, a.cin, device=dev, generator=g) * (a.cin * a.K) ** -0.5
    b = torch.randn(a.cout, device=dev, generator=g)
    pad = a.dil * (a.K - 1) // 2
    T_out = a.T + 2 * pad - a.dil * (a.K - 1)
    y = torch.empty(T_out, a.cout, device=dev)
    r = torch.randn(T_out, a.cout, device=dev, generator=g) if a.residual else None
    prec = lib.RK_PRECISION_FP16 if a.fp16 else lib.RK_PRECISION_FP32
    nbytes = L.rk_conv1d_workspace_size(a.cin, a.cout, a.T, a.K, 1, pad, a.dil, prec)
    ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)
    wp = (ws.data_ptr() + 255) // 256 * 256
    st = torch.cuda.current_stream().cuda_stream
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * a.repeat)]
    for i in range(a.repeat):
        ev[2 * i].record()
        lib.check(L.rk_conv1d_fprop(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(),
                                    r.data_ptr() if r is not None else None, wp, nbytes, a.cin, a.cout, a.T, a.K,
                                    1, pad, a.dil, prec, st), "rk_conv1d_fprop")
        ev[2 * i + 1].record()
    lib.check(L.rk_conv1d_check(wp, st), "rk_conv1d_check")
    ms = min(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(a.repeat))
    fl = 2.0 * a.cin * a.cout * a.K * T_out
    print(f"conv C_in={a.cin} C_out={a.cout} T={a.T} K={a.K} dil={a.dil}: {ms * 1e3:.1f} us incl. operand packing, "
          f"{fl / ms / 1e9:.1f} TFLOP/s algorithmic", file=sys.stderr)
    return 0


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="rokoko_b200")
    sub = p.add_subparsers(dest="cmd", required=True)
    d = sub.add_parser("decode")
    d.add_argument("--L", type=int, default=400)
    d.add_argument("--seed", type=int, default=0)
    d.add_argument("--repeat", type=int, default=1)
    d.add_argument("--fp16", action="store_true")
    d.add_argument("--weights")
    d.add_argument("-o", "--output")
    cv = sub.add_parser("conv")
    cv.add_argument("--cin", type=int, default=128)
    cv.add_argument("--cout", type=int, default=128)
    cv.add_argument("--T", type=int, default=48001)
    cv.add_argument("--K", type=int, default=7)
    cv.add_argument("--dil", type=int, default=1)
    cv.add_argument("--residual", action="store_true")
    cv.add_argument("--fp16", action="store_true")
    cv.add_argument("--repeat", type=int, default=3)
    s = sub.add_parser("synth")
    s.add_argument("--tokens", required=True)
    s.add_argument("--voice")
    s.add_argument("--row", type=int, default=None)
    s.add_argument("--fp16", action="store_true")
    s.add_argument("--weights")
    s.add_argument("-o", "--output")
    a = p.parse_args(argv)

    if a.cmd == "conv":
        return _conv_bench(a)
    from . import configs
    from .context import FP16, FP32, Context
    blob = _weights(a.weights)
    ctx = Context(0, FP16 if a.fp16 else FP32)
    ctx.load_weights(blob)
    if a.cmd == "decode":
        c = configs.config1(seed=a.seed, L=a.L)
        t0 = time.perf_counter()
        for _ in range(a.repeat):
            pcm = ctx.decode_features(c.asr, c.f0, c.n, c.style)
        dt = (time.perf_counter() - t0) / a.repeat
        print(f"decode L={a.L}: {pcm.shape[0] / 24000:.2f} s audio in {dt * 1e3:.2f} ms "
              f"({pcm.shape[0] / 24000 / dt:.0f}x real time)", file=sys.stderr)
    else:
        tok = np.array([int(x) for x in a.tokens.split(",")], np.int32)
        if a.voice:
            v = np.fromfile(a.voice, np.float32).reshape(-1, 256)
            row = a.row if a.row is not None else min(max(tok.shape[0] - 2, 0), v.shape[0] - 1)
            style = v[row]
        else:
            style = configs.config0().style
        pcm, dur, L = ctx.infer(tok, style)
        print(f"synth T={tok.shape[0]}: L={L} frames, {pcm.shape[0] / 24000:.2f} s audio", file=sys.stderr)
    if a.output:
        write_wav(a.output, pcm)
    ctx.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
