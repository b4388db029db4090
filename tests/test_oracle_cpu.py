"""CPU oracle self-checks (no GPU): determinism, STFT/iSTFT properties,
SineGen invariants, and a small end-to-end decode."""
import numpy as np
import pytest

import oracle


def test_stft_exact_real_bins_and_frame0():
    rng = np.random.default_rng(0)
    x = rng.standard_normal(1000).astype(np.float32) * 0.1
    har = oracle.stft(x)
    ph = har[:, 11:]
    # bins 0 and 10 are real: phase exactly 0 or pi
    assert np.all(np.isin(ph[:, 0], [0.0, np.float32(np.pi)]))
    assert np.all(np.isin(ph[:, 10], [0.0, np.float32(np.pi)]))
    # frame 0 is symmetric after reflect padding: every bin real
    assert np.all(np.isin(ph[0], [0.0, np.float32(np.pi)]))
    assert har.shape == (201, 22)


def test_stft_istft_match_torch_float64():
    # an independent pin of the STFT / iSTFT restatement: torch.stft / torch.istft
    # in float64 with the reference's parameters (n_fft 20, hop 5, periodic Hann,
    # center=True, reflect padding; src/kernels.cu stft / istft kernels)
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(1)
    w = torch.hann_window(20, periodic=True, dtype=torch.float64)
    x = (rng.standard_normal(1000) * 0.1).astype(np.float32)
    har = oracle.stft(x)
    S = torch.stft(torch.tensor(x, dtype=torch.float64), n_fft=20, hop_length=5, win_length=20, window=w,
                   center=True, pad_mode="reflect", return_complex=True).numpy().T
    assert np.abs(np.abs(S) - har[:, :11]).max() <= 1e-6
    big = np.abs(S) > 1e-3  # phase is ill-conditioned for tiny bins
    dphi = np.angle(np.exp(1j * (np.angle(S) - har[:, 11:])))
    assert np.abs(dphi[big]).max() <= 1e-4
    T2 = 41
    c = (rng.standard_normal((T2, 22)) * 0.5).astype(np.float32)
    y = oracle.istft(c, (T2 - 1) * 5)
    X = np.exp(c[:, :11].astype(np.float64)) * np.exp(1j * np.sin(c[:, 11:].astype(np.float64)))
    yt = torch.istft(torch.tensor(X.T), n_fft=20, hop_length=5, win_length=20, window=w, center=True,
                     length=(T2 - 1) * 5).numpy()
    assert np.linalg.norm(y - yt) / np.linalg.norm(yt) <= 1e-6


def test_sinegen_deterministic_and_bounded():
    f0 = np.full(40, 200.0, np.float32)
    lw = np.full(9, 0.1, np.float32)
    lb = np.zeros(1, np.float32)
    ph1, s1 = oracle.sinegen(f0, lw, lb)
    ph2, s2 = oracle.sinegen(f0, lw, lb)
    assert np.array_equal(s1, s2) and np.array_equal(ph1, ph2)
    assert np.all(np.abs(s1) < 1.0)
    # phases increase monotonically for a constant positive F0
    assert np.all(np.diff(ph1[:, 0]) > 0)
    # rand_ini from mt19937(42): first harmonic fixed at 0
    ri = oracle.rand_ini()
    assert ri[0] == 0.0 and np.all((ri[1:] >= 0) & (ri[1:] < 1))


@pytest.mark.slow
def test_small_decode_deterministic(v1_blob):
    from rokoko_b200 import configs
    oracle.set_threads(4)
    m = oracle.Oracle(v1_blob)
    c = configs.config1(seed=11, L=8)
    a = m.decode_features(c.asr, c.f0, c.n, c.style)
    b = m.decode_features(c.asr, c.f0, c.n, c.style)
    assert a.shape == (4800,) and np.isfinite(a).all()
    assert np.array_equal(a, b)
