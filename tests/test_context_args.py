"""Argument checks of the Python front-end (no GPU): arrays whose sizes do not
match what the C ABI reads through the pointer are rejected before any call
into librokoko_b200.so."""
import numpy as np
import pytest

from rokoko_b200 import configs
from rokoko_b200.context import Context


class _NoCalls:
    """Stands in for the loaded library: any attribute access is a failure."""

    def __getattr__(self, name):
        raise AssertionError(f"C ABI reached: {name}")


def _ctx():
    c = object.__new__(Context)
    c._L = _NoCalls()
    c.h = None  # close() is a no-op
    return c


def test_decode_features_rejects_mis_sized_inputs():
    ctx = _ctx()
    c = configs.config1(seed=0, L=8)
    with pytest.raises(ValueError, match="asr"):
        ctx.decode_features(c.asr[:, :256], c.f0, c.n, c.style)
    with pytest.raises(ValueError, match="asr"):
        ctx.decode_features(c.asr.reshape(-1), c.f0, c.n, c.style)
    with pytest.raises(ValueError, match="f0"):
        ctx.decode_features(c.asr, c.f0[:-1], c.n, c.style)
    with pytest.raises(ValueError, match="n"):
        ctx.decode_features(c.asr, c.f0, np.zeros(3, np.float32), c.style)
    with pytest.raises(ValueError, match="style"):
        ctx.decode_features(c.asr, c.f0, c.n, np.zeros(256, np.float32))


def test_infer_rejects_mis_sized_inputs():
    ctx = _ctx()
    u = configs.config0(seed=1, n_phon=10)
    with pytest.raises(ValueError, match="style"):
        ctx.infer(u.tokens, u.style[:128], u.durations)
    with pytest.raises(ValueError, match="dur_override"):
        ctx.infer(u.tokens, u.style, u.durations[:-1])
    with pytest.raises(ValueError, match="tokens"):
        ctx.infer(u.tokens.reshape(1, -1), u.style, u.durations)


def test_encode_rejects_mis_sized_inputs():
    ctx = _ctx()
    good = configs.config0(seed=2, n_phon=8)
    bad_dur = configs.Utterance(good.tokens, good.style, good.durations[:-1])
    with pytest.raises(ValueError, match="durations"):
        ctx.encode([good, bad_dur])
    bad_style = configs.Utterance(good.tokens, good.style[:100], good.durations)
    with pytest.raises(ValueError, match="style"):
        ctx.encode([bad_style])
