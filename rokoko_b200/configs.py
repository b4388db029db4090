"""Seeded synthetic inputs for the benchmark configurations.

Config 0: one utterance, 64 phoneme ids U[1,177] wrapped in BOS/EOS = 0
          (rokoko's to_tokens convention, src/rokoko.h:141-154), style 256 ~ N(0, 0.1)
          (ref_s[0:128] decoder, [128:256] predictor), durations overridden by U[2,8].
Config 1: decoder/generator only: asr [400, 512] ~ N(0, 1) (frames x channels),
          F0 [800] a 200 Hz +-50 Hz seeded random walk, N [800] ~ N(0, 0.1),
          style [128] ~ N(0, 0.1).  L = 400 frames -> 240,000 samples = 10.0 s.
Config 2: 16 utterances, T in U[32,256] (+BOS/EOS), durations U[2,8], FP16 weights.
Config 3: one 510-token utterance (+BOS/EOS), durations U[3,10], FP16 weights.
Config 4: 1024 utterances, T ~ truncated N(120, 60) clipped to [16,510], durations U[2,8],
          a style vector per utterance, FP16 weights.
No public dataset is involved; every array comes from numpy's PCG64 with a fixed seed.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class Utterance:
    tokens: np.ndarray      # int32 [T] incl. BOS/EOS
    style: np.ndarray       # float32 [256]
    durations: np.ndarray   # int32 [T] (override)


@dataclass
class DecoderFeatures:
    asr: np.ndarray         # float32 [L, 512]
    f0: np.ndarray          # float32 [2L]
    n: np.ndarray           # float32 [2L]
    style: np.ndarray       # float32 [128] (acoustic half)


def _utt(rng, n_phon: int, dlo: int, dhi: int) -> Utterance:
    tok = np.concatenate([[0], rng.integers(1, 178, n_phon), [0]]).astype(np.int32)
    style = (rng.standard_normal(256) * 0.1).astype(np.float32)
    dur = rng.integers(dlo, dhi + 1, tok.shape[0]).astype(np.int32)
    return Utterance(tok, style, dur)


def config0(seed: int = 0, n_phon: int = 64) -> Utterance:
    return _utt(np.random.default_rng(1000 + seed), n_phon, 2, 8)


def f0_walk(rng, n: int, center: float = 200.0, spread: float = 50.0, step: float = 5.0) -> np.ndarray:
    f = np.empty(n, np.float64)
    v = center
    for i in range(n):
        v = float(np.clip(v + rng.normal(0.0, step), center - spread, center + spread))
        f[i] = v
    return f.astype(np.float32)


def config1(seed: int = 0, L: int = 400) -> DecoderFeatures:
    rng = np.random.default_rng(2000 + seed)
    asr = rng.standard_normal((L, 512)).astype(np.float32)
    f0 = f0_walk(rng, 2 * L)
    n = (rng.standard_normal(2 * L) * 0.1).astype(np.float32)
    style = (rng.standard_normal(128) * 0.1).astype(np.float32)
    return DecoderFeatures(asr, f0, n, style)


def config2(seed: int = 0, batch: int = 16) -> list[Utterance]:
    rng = np.random.default_rng(3000 + seed)
    return [_utt(rng, int(rng.integers(32, 257)), 2, 8) for _ in range(batch)]


def config3(seed: int = 0) -> Utterance:
    return _utt(np.random.default_rng(4000 + seed), 510, 3, 10)


def config4(seed: int = 0, count: int = 1024) -> list[Utterance]:
    rng = np.random.default_rng(5000 + seed)
    out = []
    for _ in range(count):
        while True:
            t = rng.normal(120.0, 60.0)
            if 16 <= t <= 510:
                break
        out.append(_utt(rng, int(round(t)), 2, 8))
    return out


def audio_seconds_decoder(L: int) -> float:
    return 600 * L / 24000.0
