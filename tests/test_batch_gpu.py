"""Batched entry points (rk_encode + rk_decode) on the B200: every utterance
of a batch comes out bit-identical to its own rk_infer call (the kernels are
deterministic), and the batch holds utterances of different lengths (so of
different decoder-frame buckets)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_encode_decode_batch_matches_single_utterance_infer(v1_blob):
    from rokoko_b200 import configs
    from rokoko_b200.context import FP32, Context
    batch = [configs.config0(seed=s, n_phon=n) for s, n in ((1, 12), (2, 30), (3, 7))]
    with Context(0, FP32) as ctx:
        ctx.load_weights(v1_blob)
        durs, Ls = ctx.encode(batch)
        pcms = ctx.decode(Ls)
        assert len(pcms) == len(batch)
        for u, d, L, pcm in zip(batch, durs, Ls, pcms):
            ref, ref_dur, ref_L = ctx.infer(u.tokens, u.style, u.durations)
            assert L == ref_L == int(u.durations.sum())
            assert np.array_equal(d, ref_dur)
            assert pcm.shape == ref.shape == (600 * L,)
            assert np.array_equal(pcm, ref)
        # nothing pending after rk_decode
        assert ctx.decode([]) == []
