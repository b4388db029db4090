"""rk_compute_decode_bytes equals the reference's compute_decode_bytes
(src/rokoko_common.h:160-229), the arena size callers of rokoko_infer
allocate.  The reference's own values come from compiling its header
(tests/golden/make_decode_bytes.py) over a grid of token counts T and frame
counts L; when RK_REFERENCE_DIR names a reference checkout the header is also
compiled and compared live.  Host arithmetic only: no GPU."""
import json
import os

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _fixture():
    with open(os.path.join(HERE, "golden", "decode_bytes.json")) as f:
        return json.load(f)["rows"]


def test_matches_reference_sizes(rk_lib):
    rows = _fixture()
    assert len(rows) >= 60
    bad = [(T, L, ref, rk_lib.rk_compute_decode_bytes(T, L)) for T, L, ref in rows
           if rk_lib.rk_compute_decode_bytes(T, L) != ref]
    assert not bad, bad[:5]


@pytest.mark.skipif(not os.environ.get("RK_REFERENCE_DIR"), reason="RK_REFERENCE_DIR not set")
def test_matches_reference_header_live(rk_lib):
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_decode_bytes",
                                                  os.path.join(HERE, "golden", "make_decode_bytes.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    for T, L, ref in mod.sizes(os.environ["RK_REFERENCE_DIR"]):
        assert rk_lib.rk_compute_decode_bytes(T, L) == ref, (T, L)
