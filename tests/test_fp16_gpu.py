"""FP16-weights path (the reference's rokoko.fp16 binary, src/rokoko_f16.cpp)
on the B200 vs the CPU oracle in its FP16 mode.

The library loads the KOKO v2 file written by rokoko_b200.convert_v2 (byte-
identical to the reference converter's output); the oracle reads the v1 file
and rounds the same weights to FP16.  Bars: durations, L and sample counts
exact; waveform relative L2 <= 1e-2 (FP16 weights, FP32 accumulate).
Shapes: config 2 (16 utterances, T in [32, 256] + BOS/EOS, durations U[2,8]),
config 3 (510 tokens + BOS/EOS, durations U[3,10], about 3300 frames) and the
config-1 decoder features.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-2


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def v2_blob(v1_blob):
    from rokoko_b200 import convert_v2
    return convert_v2.convert_blob(v1_blob)


@pytest.fixture(scope="module")
def oracle16(v1_blob):
    import oracle
    oracle.set_threads(max(1, os.cpu_count() or 1))
    m = oracle.Oracle(v1_blob, fp16=True)
    yield m
    m.close()


@pytest.fixture(scope="module")
def ctx_v2(v2_blob):
    from rokoko_b200.context import FP16, Context
    ctx = Context(0, FP16)
    ctx.load_weights(v2_blob)
    yield ctx
    ctx.close()


@pytest.mark.parametrize("L", [37, 400])
def test_decode_features_fp16(ctx_v2, oracle16, L):
    from rokoko_b200 import configs
    c = configs.config1(seed=L, L=L)
    pcm = ctx_v2.decode_features(c.asr, c.f0, c.n, c.style)
    ref = oracle16.decode_features(c.asr, c.f0, c.n, c.style)
    assert pcm.shape == ref.shape == (600 * L,)
    r = rel_l2(pcm, ref)
    print(f"L={L}: {r:.3e}")
    assert r <= TOL


def test_v2_file_matches_v1_file_in_fp16(ctx_v2, v1_blob):
    # the v2 file bakes weight norm in FP32 numpy and rounds to FP16; loading the
    # v1 file in FP16 mode bakes it in double: the two differ by FP16 rounding of
    # a few weights only
    from rokoko_b200 import configs
    from rokoko_b200.context import FP16, Context
    c = configs.config1(seed=5, L=64)
    with Context(0, FP16) as ctx_v1:
        ctx_v1.load_weights(v1_blob)
        a = ctx_v1.decode_features(c.asr, c.f0, c.n, c.style)
    b = ctx_v2.decode_features(c.asr, c.f0, c.n, c.style)
    assert rel_l2(b, a) <= 2e-3


def test_config2_batch_fp16(ctx_v2, oracle16):
    """Config 2: the 16 utterances go through rk_encode as one batch (length-
    sorted, as the shard plan orders a bucket) and rk_decode; every one is
    checked against the B = 1 oracle: predicted durations and L exact, sample
    count 600 L, waveform relative L2 <= 1e-2."""
    from rokoko_b200 import configs
    batch = configs.config2(seed=2)
    order = sorted(range(len(batch)), key=lambda i: batch[i].tokens.shape[0])
    durs, Ls = ctx_v2.encode([batch[i] for i in order])
    pcms = ctx_v2.decode(Ls)
    worst = 0.0
    for k, i in enumerate(order):
        u = batch[i]
        ref, ref_dur, ref_L, _ = oracle16.infer(u.tokens, u.style, u.durations, bucket=32)
        assert np.array_equal(durs[k], ref_dur), i
        assert Ls[k] == ref_L == int(u.durations.sum())
        assert pcms[k].shape == ref.shape == (600 * Ls[k],)
        r = rel_l2(pcms[k], ref)
        worst = max(worst, r)
        print(f"T={u.tokens.shape[0]} L={Ls[k]}: {r:.3e}")
        assert r <= TOL, (i, r)
    print(f"config 2: 16 utterances, worst rel L2 {worst:.3e}")


def test_predicted_durations_fp16(ctx_v2, oracle16):
    """Config-0 shape (64 phonemes, T = 66) with the durations the model
    predicts (no override): integer durations and L bit-exact against the
    FP16-mode oracle, alignment indices exact, waveform within 1e-2."""
    from rokoko_b200 import configs
    u = configs.config0(seed=64, n_phon=64)
    ctx_v2.record(True)
    try:
        pcm, dur, L = ctx_v2.infer(u.tokens, u.style, None)
        ft = ctx_v2.stage("frame_token")
    finally:
        ctx_v2.record(False)
    oracle16.record(True)
    ref, ref_dur, ref_L, _ = oracle16.infer(u.tokens, u.style, None, bucket=32)
    ref_ft = oracle16.stage("frame_token")
    oracle16.record(False)
    assert np.array_equal(dur, ref_dur), (dur, ref_dur)
    assert L == ref_L == int(dur.sum())
    assert np.array_equal(ft, ref_ft)
    assert pcm.shape == ref.shape == (600 * L,)
    r = rel_l2(pcm, ref)
    print(f"T=66 predicted durations: L={L}, rel L2 {r:.3e}")
    assert r <= TOL


def test_config3_long_utterance_fp16(ctx_v2, oracle16):
    from rokoko_b200 import configs
    u = configs.config3(seed=3)
    assert u.tokens.shape[0] == 512
    ctx_v2.record(True)
    try:
        pcm, dur, L = ctx_v2.infer(u.tokens, u.style, u.durations)
        ft = ctx_v2.stage("frame_token")
    finally:
        ctx_v2.record(False)
    oracle16.record(True)
    ref, ref_dur, ref_L, _ = oracle16.infer(u.tokens, u.style, u.durations, bucket=32)
    ref_ft = oracle16.stage("frame_token")
    oracle16.record(False)
    assert np.array_equal(dur, ref_dur) and L == ref_L == int(u.durations.sum())
    assert np.array_equal(ft, ref_ft), "alignment indices differ"
    assert pcm.shape == ref.shape == (600 * L,)
    r = rel_l2(pcm, ref)
    print(f"config 3: L={L}, {pcm.shape[0] / 24000:.1f} s audio, rel L2 {r:.3e}")
    assert r <= TOL
