"""Config 4 (the box-throughput workload) through the path boxbench times: a
seeded 32-utterance slice of the 1024 utterances, ordered by the shard plan,
run through rk_encode + rk_decode in batches on two rk_ctx driven by two host
threads (rokoko_b200.boxbench.run_share), FP16 weights (KOKO v2).  Every
utterance is checked against the B = 1 FP16-mode oracle: L and the sample
count exact, waveform relative L2 <= 1e-2."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-2


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_config4_slice_two_contexts(v1_blob):
    import oracle
    from rokoko_b200 import boxbench, configs, convert_v2, shard
    from rokoko_b200.context import FP16, Context
    utts = configs.config4(seed=0, count=1024)[:32]
    items = shard.units(utts)
    order = shard.plan(items, 1)[0]
    v2 = convert_v2.convert_blob(v1_blob)
    ctxs = [Context(0, FP16), Context(0, FP16)]
    try:
        for c in ctxs:
            c.load_weights(v2)
        out = dict(boxbench.run_share(ctxs, utts, order, 8))
    finally:
        for c in ctxs:
            c.close()
    assert sorted(out) == list(range(len(utts)))
    oracle.set_threads(max(1, os.cpu_count() or 1))
    orc = oracle.Oracle(v1_blob, fp16=True)
    worst = 0.0
    try:
        for i, u in enumerate(utts):
            L = int(u.durations.sum())
            ref, _, ref_L, _ = orc.infer(u.tokens, u.style, u.durations, bucket=32)
            assert ref_L == L and out[i].shape == ref.shape == (600 * L,), i
            r = rel_l2(out[i], ref)
            worst = max(worst, r)
            assert r <= TOL, (i, r)
    finally:
        orc.close()
    print(f"config-4 slice: {len(utts)} utterances, worst rel L2 {worst:.3e}")
