"""bench.py's host-side helpers on synthetic inputs (no GPU): the per-shape conv
and operand-pack tables built from a serial timeline, the interleaved step order,
and the seeded phonemizer texts."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
from rokoko_b200 import g2pfile  # noqa: E402


def _timeline():
    # (stream, name, end ms): each launch's time is the gap to the previous mark
    return [(0, "start", 0.0), (0, "pack_adain_snake C128 R48001 Cp128 Rd48001 split", 0.016),
            (0, "conv 128>128 K11 d1 T48001", 0.056), (0, "conv 128>128 K11 d3 T48001 res", 0.096),
            (0, "conv 256>128 K12 d1 T48001 convT 8001", 0.16), (0, "adain_coef", 0.167),
            (0, "conv 512>256 K20 d1 T8000 convT", 0.2)]  # a label without input rows is skipped


def test_conv_shapes_rows():
    rows = bench.conv_shapes(_timeline(), 1679.4, 6532.2)
    by = {r["shape"]: r for r in rows}
    assert set(by) == {"128>128 K11 T48001", "128>128 K11 T48001 res", "256>128 K12 T48001 convT"}
    r = by["128>128 K11 T48001"]
    flops = 2 * 128 * 128 * 11 * 48001
    assert r["launches"] == 1 and abs(r["ms"] - 0.04) < 1e-9
    assert abs(r["tflops"] - flops / 0.04e-3 / 1e12) < 0.1
    # FP32 semantics: P_eff = burst / 3; K = 11 at C = 128 is above the ridge, so tensor-bound
    assert r["bound"] == "tensor" and abs(r["bound_tflops"] - 1679.4 / 3) < 0.1
    # the residual read lowers the intensity of the same shape
    assert by["128>128 K11 T48001 res"]["flop_per_byte"] < r["flop_per_byte"]
    # ConvTranspose counts input rows
    t = by["256>128 K12 T48001 convT"]
    assert abs(t["tflops"] - 2 * 256 * 128 * 12 * 8001 / 0.064e-3 / 1e12) < 0.1


def test_pack_shapes_rows():
    rows = bench.pack_shapes(_timeline(), 6532.2)
    assert len(rows) == 1
    r = rows[0]
    by = 48001 * 128 * 4 + 48001 * 128 * 2 * 2
    assert r["shape"] == "pack_adain_snake C128 R48001 split" and r["launches"] == 1
    assert abs(r["gb_s"] - by / 0.016e-3 / 1e9) < 0.1
    assert abs(r["frac_of_hbm"] - r["gb_s"] / 6532.2) < 1e-3


def test_interleaved_order_is_a_permutation():
    for n in (1, 2, 7, 32, 100):
        o = bench.interleaved(n)
        assert sorted(o) == list(range(n))
    assert bench.interleaved(32) == bench.interleaved(32)


def test_g2p_texts_are_seeded_ascii():
    a, b = g2pfile.random_texts(50, seed=3), g2pfile.random_texts(50, seed=3)
    assert a == b and a != g2pfile.random_texts(50, seed=4)
    assert all(1 <= len(t) <= 510 and all(32 <= ord(ch) < 127 for ch in t) for t in a)
    assert 90 < sum(map(len, a)) / len(a) < 150
