"""rokoko_b200.convert_v2 against the reference's own converter
(scripts/convert_v2.py), recorded for the seed-0 random-init v1 file in
tests/golden/v2_seed0.json by tests/golden/make_v2_digest.py."""
import hashlib
import json
import os

import numpy as np
import pytest

from rokoko_b200 import convert_v2, koko

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "v2_seed0.json")


@pytest.fixture(scope="module")
def v2_blob(v1_blob):
    return convert_v2.convert_blob(v1_blob)


def test_v2_bytes_identical_to_reference_converter(v2_blob):
    ref = json.load(open(GOLDEN))
    _, tensors = koko.parse(v2_blob)
    mine = [[n, str(a.dtype), list(a.shape), hashlib.sha256(a.tobytes()).hexdigest()[:16]]
            for n, a in tensors.items()]
    # tensor by tensor first, for a readable failure
    assert [m[0] for m in mine] == [r[0] for r in ref["tensors"]]
    for m, r in zip(mine, ref["tensors"]):
        assert m == r, (m, r)
    assert len(v2_blob) == ref["bytes"] == 163390976  # the reference FP16 binary's expected size
    assert hashlib.sha256(v2_blob).hexdigest() == ref["sha256"]


def test_v2_layout_rules(v2_blob):
    _, t = koko.parse(v2_blob)
    # NHWC [C_out, K, C_in], FP16
    w = t["decoder.generator.resblocks.3.convs1.0.weight_v.nhwc_f16"]
    assert w.dtype == np.float16 and w.shape == (128, 3, 128)
    # C_in = 22 padded to 24 with zeros
    p = t["decoder.generator.noise_convs.0.weight.nhwc_f16_pad24"]
    assert p.shape == (256, 12, 24) and not p[:, :, 22:].any()
    # 514 -> 1024: C_in % 8 != 0 -> padded copy
    assert "decoder.encode.conv1.weight_v.nhwc_f16_pad520" in t
    # LSTM combined biases are FP32 sums
    assert t["predictor.shared.bias_combined_rev"].dtype == np.float32
    # conv_post keeps a plain FP16 copy (C_out = 22 is not a multiple of 4)
    assert t["decoder.generator.conv_post.weight_v.f16"].shape == (22, 128, 7)
