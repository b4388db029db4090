"""Decoder + generator (config 1 path) on the B200 vs the CPU FP32 oracle.

Bar: waveform relative L2 <= 1e-3 (FP32 semantics: three-pass split-bf16
tensor-core products, FP32 accumulate), with per-stage activation checks;
sample counts bit-exact.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

STAGES = [  # name, relative-L2 tolerance
    ("dec_encode", 1e-4),
    ("asr_res", 1e-5),
    ("dec_decode3", 2e-4),
    ("har_source", 1e-5),
    ("har", 2e-5),
    ("gen0_src", 3e-4),
    ("gen0_ups", 3e-4),
    ("gen0_out", 5e-4),
    ("gen1_src", 5e-4),
    ("gen1_ups", 5e-4),
    ("gen1_out", 8e-4),
    ("conv_post", 1e-3),
]


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def oracle_model(v1_blob):
    import oracle
    oracle.set_threads(8)
    m = oracle.Oracle(v1_blob)
    m.record(True)
    return m


@pytest.fixture(scope="module")
def gpu_ctx(v1_blob):
    from rokoko_b200.context import Context, FP32
    ctx = Context(0, FP32)
    ctx.load_weights(v1_blob)
    ctx.record(True)
    yield ctx
    ctx.close()


@pytest.mark.parametrize("L", [37, 400])
def test_decode_features_fp32(gpu_ctx, oracle_model, L):
    from rokoko_b200 import configs
    c = configs.config1(seed=L, L=L)
    ref = oracle_model.decode_features(c.asr, c.f0, c.n, c.style)
    pcm = gpu_ctx.decode_features(c.asr, c.f0, c.n, c.style)
    assert pcm.shape == ref.shape == (600 * L,)
    assert np.isfinite(pcm).all()
    report = []
    for name, tol in STAGES:
        g, o = gpu_ctx.stage(name), oracle_model.stage(name)
        assert g is not None and o is not None, name
        assert g.shape == o.shape, (name, g.shape, o.shape)
        report.append((name, rel_l2(g, o), tol))
    wav = rel_l2(pcm, ref)
    msg = "\n".join(f"{n}: {r:.3e} (tol {t:.0e})" for n, r, t in report) + f"\naudio: {wav:.3e}"
    print(msg)
    for n, r, t in report:
        assert r <= t, msg
    assert wav <= 1e-3, msg
