"""Command-line front-end (the reference's CLI is src/main.cu:56-345; its text
normalizer, voice management and downloads are outside this library's scope).

    python -m rokoko_b200.cli decode [--L 400] [--seed 0] [--repeat 1] [-o out.wav] [--weights koko.bin]
        decoder + generator on seeded config-1 features (asr / F0 / N / style)
    python -m rokoko_b200.cli synth (--tokens 0,50,83,...,0 | --ipa "həlˈoʊ" | --text "hello" [--g2p g2p.bin])
                                    [--voice voice.bin] [--row N] [-o out.wav]
        full forward (rokoko_infer) on token ids, on IPA (chunk_ipa + to_tokens, src/rokoko.h:141-221,
        each chunk synthesised and the PCM concatenated), or on text through the neural phonemizer
        first (no text normalisation: the text goes to the phonemizer as given); --voice is a raw
        float32 [rows, 256] voice pack (src/main.cu:46, src/rokoko.h:327-340: style row =
        min(T-2, rows-1) per chunk)

Without --weights a seeded random-init KOKO v1 file is generated in memory, and without
--g2p a seeded random-init G2P3 model (rokoko_b200.g2pfile.random_blob).
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
    s = sub.add_parser("synth")
    src = s.add_mutually_exclusive_group(required=True)
    src.add_argument("--tokens")
    src.add_argument("--ipa")
    src.add_argument("--text")
    s.add_argument("--g2p")
    s.add_argument("--voice")
    s.add_argument("--row", type=int, default=None)
    s.add_argument("--fp16", action="store_true")
    s.add_argument("--weights")
    s.add_argument("-o", "--output")
    a = p.parse_args(argv)

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
        if a.tokens:
            chunks = [np.array([int(x) for x in a.tokens.split(",")], np.int32)]
        else:
            from . import tokens as tk
            ipa = a.ipa
            if a.text is not None:
                from . import g2pfile
                from .g2p import G2PModel
                g = G2PModel(ctx=ctx)
                ok = g.load(a.g2p) if a.g2p else g.load_bytes(g2pfile.random_blob(0))
                if not ok:
                    print(f"failed to load the G2P model {a.g2p}", file=sys.stderr)
                    return 1
                ipa = g.infer(a.text)
                g.free()
                print(f"g2p: {ipa}", file=sys.stderr)
            chunks = [ids for _, ids in tk.chunk_ipa(ipa)]
        v = np.fromfile(a.voice, np.float32).reshape(-1, 256) if a.voice else None
        pcms = []
        for tok in chunks:
            if v is not None:
                row = a.row if a.row is not None else min(max(tok.shape[0] - 2, 0), v.shape[0] - 1)
                style = v[row]
            else:
                style = configs.config0().style
            pcm, dur, L = ctx.infer(tok, style)
            pcms.append(pcm)
            print(f"synth T={tok.shape[0]}: L={L} frames, {pcm.shape[0] / 24000:.2f} s audio", file=sys.stderr)
        pcm = np.concatenate(pcms) if pcms else np.zeros(0, np.float32)
    if a.output:
        write_wav(a.output, pcm)
    ctx.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
