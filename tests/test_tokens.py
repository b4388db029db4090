"""IPA -> model input (rk_ipa_to_tokens / rk_ipa_chunks; rokoko::to_tokens /
chunk_ipa, src/rokoko.h:141-221) against the reference's own outputs
(tests/golden/ipa_tokens.json, recorded by tests/golden/make_ipa_tokens.py from
the reference's header).  Host code: runs on the CPU."""
import json
import os
import subprocess
import tempfile

import numpy as np
import pytest

from rokoko_b200 import lib, tokens

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(ROOT, "tests", "golden", "ipa_tokens.json")) as f:
        return json.load(f)["cases"]


def test_chunks_and_tokens_match_reference(golden):
    assert len(golden) >= 20
    for case in golden:
        got = tokens.chunk_ipa(case["ipa"])
        assert [len(p.encode("utf-8")) for p, _ in got] == [c["bytes"] for c in case["chunks"]], case["ipa"][:40]
        for (_, ids), c in zip(got, case["chunks"]):
            assert ids.dtype == np.int32 and ids.tolist() == c["tokens"]


def test_to_tokens_basics():
    assert tokens.to_tokens("").tolist() == [0, 0]
    # space 16, '.' 4, 'a' 43; code points outside the vocabulary are dropped
    assert tokens.to_tokens("a .X").tolist() == [0, 43, 16, 4, 0]
    assert tokens.to_tokens("ˈ").tolist() == [0, 156, 0]


def test_short_buffers_report_sizes():
    import ctypes
    L = lib.load()
    n = ctypes.c_size_t(0)
    ids = (ctypes.c_int32 * 2)()
    assert L.rk_ipa_to_tokens(b"abc", 3, ids, 2, ctypes.byref(n)) == lib.RK_ERR_WORKSPACE and n.value == 5
    ends = (ctypes.c_size_t * 1)()
    s = ("x" * 1021).encode()
    assert L.rk_ipa_chunks(s, len(s), ends, 1, ctypes.byref(n)) == lib.RK_ERR_WORKSPACE and n.value == 3


def test_cpp_caller_matches_reference(golden):
    from test_cpp_compat import _compile_src
    with tempfile.TemporaryDirectory() as d:
        exe = _compile_src(d, "tokens_main")
        text = "\n".join(c["ipa"] for c in golden) + "\n"
        out = subprocess.run([exe], input=text.encode("utf-8"), check=True, capture_output=True,
                             timeout=120).stdout.decode()
    for line, case in zip(out.splitlines(), golden):
        parts = line.split(" | ")
        assert int(parts[0]) == len(case["chunks"])
        for p, c in zip(parts[1:], case["chunks"]):
            v = [int(x) for x in p.split()]
            assert v[0] == c["bytes"] and v[2:2 + v[1]] == c["tokens"]
