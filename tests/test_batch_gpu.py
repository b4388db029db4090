"""Batched entry points (rk_encode + rk_decode) on the B200: every utterance
of a batch comes out bit-identical to its own rk_infer call (the front half's
arithmetic per utterance does not depend on the batch: no split reductions,
per-sequence LSTM sums in a fixed order), and the batch holds utterances of
different lengths (so of different decoder-frame buckets)."""
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


def test_two_contexts_on_two_threads_match_one_context(v1_blob):
    """Two rk_ctx on one GPU, each driven by its own host thread at the same
    time (the box-throughput setup of rokoko_b200.boxbench), produce PCM
    bit-identical to one context running the same batches alone."""
    import threading

    from rokoko_b200 import configs
    from rokoko_b200.context import FP32, Context
    batches = [[configs.config0(seed=10 + 3 * b + k, n_phon=6 + 5 * k) for k in range(3)] for b in range(4)]
    with Context(0, FP32) as ctx:
        ctx.load_weights(v1_blob)
        ref = [ctx.decode(ctx.encode(bt)[1]) for bt in batches]
    ctxs = [Context(0, FP32), Context(0, FP32)]
    try:
        for c in ctxs:
            c.load_weights(v1_blob)
        out = [None] * len(batches)
        errors = []

        def worker(c):
            try:
                for b in range(c, len(batches), 2):
                    out[b] = ctxs[c].decode(ctxs[c].encode(batches[b])[1])
            except BaseException as e:
                errors.append(e)

        th = [threading.Thread(target=worker, args=(c,)) for c in range(2)]
        for t in th:
            t.start()
        for t in th:
            t.join()
        assert not errors, errors
        for b in range(len(batches)):
            assert len(out[b]) == len(ref[b])
            for p, r in zip(out[b], ref[b]):
                assert np.array_equal(p, r)
    finally:
        for c in ctxs:
            c.close()


@pytest.mark.parametrize("overrides", [True, False])
def test_large_batch_fp16_bit_identical_to_single(v1_blob, overrides):
    """40 utterances of different lengths in one rk_encode (the BiLSTM kernel
    then packs eight sequences per cluster): every utterance's durations, L and
    PCM equal its own rk_infer call bit for bit, with the durations given and
    with the durations the model predicts."""
    from rokoko_b200 import configs, convert_v2
    from rokoko_b200.context import FP16, Context
    batch = [configs.config0(seed=100 + k, n_phon=3 + (k * 7) % 29) for k in range(40)]
    v2 = convert_v2.convert_blob(v1_blob)
    with Context(0, FP16) as ctx:
        ctx.load_weights(v2)
        durs, Ls = ctx.encode(batch, overrides=overrides)
        pcms = ctx.decode(Ls)
        assert len(pcms) == len(batch)
        for u, d, L, pcm in zip(batch, durs, Ls, pcms):
            ref, ref_dur, ref_L = ctx.infer(u.tokens, u.style, u.durations if overrides else None)
            assert L == ref_L
            assert np.array_equal(d, ref_dur)
            assert np.array_equal(pcm, ref)
