"""Streaming synthesis (rk_synthesize_stream; the reference's
TtsPipeline::synthesize_streaming, src/rokoko.h:298-360): the utterances are
handed to the callback in order, each bit-identical to its own rk_infer call
(the chunk's front half runs on a second stream beside the previous chunk's
decode, with its own buffers); returning False from the callback stops the
call cleanly and the context stays usable."""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_stream_matches_infer_and_stops(v1_blob):
    from rokoko_b200 import configs, convert_v2
    from rokoko_b200.context import FP16, Context
    utts = configs.config4(seed=3, count=24)
    v2 = convert_v2.convert_blob(v1_blob)
    with Context(0, FP16) as ctx:
        ctx.load_weights(v2)
        got = []
        t0 = time.perf_counter()
        first = []

        def on_pcm(i, pcm):
            if not first:
                first.append(time.perf_counter() - t0)
            got.append((i, pcm))
            return True

        ctx.synthesize_stream(utts, on_pcm, chunk=5)
        total = time.perf_counter() - t0
        assert [i for i, _ in got] == list(range(len(utts)))
        for (i, pcm), u in zip(got, utts):
            ref, _, L = ctx.infer(u.tokens, u.style, u.durations)
            assert L == int(u.durations.sum()) and pcm.shape == ref.shape
            assert np.array_equal(pcm, ref), i
        audio = sum(p.shape[0] for _, p in got) / 24000.0
        print(f"stream: {len(utts)} utterances, first audio after {first[0] * 1e3:.0f} ms, "
              f"{audio / total:.0f} audio-s/s on one context")
        # the caller stops after the third utterance: nothing is pending afterwards
        seen = []
        ctx.synthesize_stream(utts, lambda i, p: seen.append(i) or len(seen) < 3, chunk=4)
        assert seen == [0, 1, 2]
        assert ctx.decode([]) == []
        # predicted durations stream the same way as rk_infer without override
        got2 = []
        ctx.synthesize_stream(utts[:6], lambda i, p: got2.append(p) or True, chunk=4, overrides=False)
        for p, u in zip(got2, utts[:6]):
            ref, _, _ = ctx.infer(u.tokens, u.style)
            assert np.array_equal(p, ref)
