"""Text -> PCM on the B200: the phonemizer (rk_g2p_infer), the IPA chunking and
token conversion (rk_ipa_chunks / rk_ipa_to_tokens) and rokoko_infer per chunk,
as the reference's pipeline composes them (src/rokoko.h:301-345; no text
normalisation here), checked against the CPU oracle on the same tokens, and the
CLI's --text / --ipa paths."""
import os
import subprocess
import sys
import tempfile

import numpy as np
import pytest

import oracle
from rokoko_b200 import g2pfile, tokens

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_text_chunks_to_pcm(v1_blob):
    from rokoko_b200.context import FP32, Context
    from rokoko_b200.g2p import G2PModel
    text = "the quick brown fox jumps over the lazy dog. " * 14  # > 510 phones: several chunks
    rng = np.random.default_rng(2)
    style = (0.1 * rng.standard_normal(256)).astype(np.float32)
    orc = oracle.Oracle(v1_blob)
    with Context(0, FP32) as ctx:
        ctx.load_weights(v1_blob)
        g = G2PModel(ctx=ctx)
        assert g.load_bytes(g2pfile.random_blob(0))
        ipa = g.infer(text)
        chunks = tokens.chunk_ipa(ipa)
        assert len(chunks) >= 2 and "".join(p for p, _ in chunks) == ipa
        for piece, ids in chunks:
            assert ids[0] == 0 and ids[-1] == 0 and 2 <= ids.size <= 512
        for piece, ids in chunks[:1]:  # the oracle on the first chunk
            dur = rng.integers(2, 5, size=ids.size).astype(np.int32)
            pcm, d, L = ctx.infer(ids, style, dur)
            ref, ref_d, ref_L, _ = orc.infer(ids, style, dur)
            assert L == ref_L and np.array_equal(d, ref_d)
            rel = float(np.linalg.norm(pcm.astype(np.float64) - ref) / np.linalg.norm(ref))
            assert rel <= 1e-3, rel
    orc.close()


def test_cli_text_and_ipa():
    with tempfile.TemporaryDirectory() as d:
        for args in (["--text", "hello world."], ["--ipa", "həlˈoʊ wˈɜːld."]):
            out = os.path.join(d, "o.wav")
            subprocess.run([sys.executable, "-m", "rokoko_b200.cli", "synth", *args, "-o", out], check=True,
                           cwd=ROOT, timeout=600, capture_output=True)
            assert os.path.getsize(out) > 44
