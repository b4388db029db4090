"""KOKO v3, the B200-layout weight file (rk_convert_koko_b200): conversion on
the host, and on a GPU a context that loads the v3 file decodes bit for bit
what a context that loads the v1 / v2 file does (the v3 file is the same
packed image the v1 / v2 loader builds), with both load times measured."""
import struct
import time

import numpy as np
import pytest


@pytest.fixture(scope="module")
def blobs(v1_blob):
    from rokoko_b200 import convert_b200, convert_v2, lib
    v2 = convert_v2.convert_blob(v1_blob)
    return {
        "v1": v1_blob, "v2": v2,
        "v3_fp32": convert_b200.convert(v1_blob, lib.RK_PRECISION_FP32),
        "v3_fp16": convert_b200.convert(v2, lib.RK_PRECISION_FP16),
    }


def test_v3_header_and_sizes(blobs):
    for k in ("v3_fp32", "v3_fp16"):
        magic, version, dlen = struct.unpack("<IIQ", blobs[k][:16])
        assert magic == 0x4F4B4F4B and version == 3 and dlen > 0
        prec, has_front = struct.unpack("<II", blobs[k][16:24])
        assert has_front == 1 and prec == (0 if k == "v3_fp32" else 1)
    # split planes (hi + lo) are two bf16 copies: the FP32 image is larger than the FP16 one
    assert len(blobs["v3_fp32"]) > len(blobs["v3_fp16"]) > 0


def test_v3_conversion_rejects_mismatches(blobs):
    from rokoko_b200 import convert_b200, lib
    with pytest.raises(lib.RkError):
        convert_b200.convert(blobs["v2"], lib.RK_PRECISION_FP32)  # v2 holds FP16 weights
    with pytest.raises(lib.RkError):
        convert_b200.convert(b"KOKO" + bytes(12), lib.RK_PRECISION_FP32)


@pytest.mark.gpu
@pytest.mark.parametrize("prec_name", ["fp32", "fp16"])
def test_v3_load_is_bit_identical(blobs, prec_name):
    from rokoko_b200 import configs, lib
    from rokoko_b200.context import FP16, FP32, Context
    prec = FP32 if prec_name == "fp32" else FP16
    src = blobs["v1"] if prec == FP32 else blobs["v2"]
    v3 = blobs["v3_" + prec_name]
    c1 = configs.config1(seed=4, L=64)
    u = configs.config0(seed=8, n_phon=20)
    outs, times = [], []
    for blob in (src, v3):
        with Context(0, prec) as ctx:
            ctx.load_weights(blob)  # warm the allocator / kernel attributes once
            t0 = time.perf_counter()
            ctx.load_weights(blob)
            times.append(time.perf_counter() - t0)
            pcm = ctx.decode_features(c1.asr, c1.f0, c1.n, c1.style)
            pcm2, dur, L = ctx.infer(u.tokens, u.style)
            outs.append((pcm, pcm2, dur, L))
    (a1, a2, ad, aL), (b1, b2, bd, bL) = outs
    assert np.array_equal(a1, b1) and np.array_equal(a2, b2) and np.array_equal(ad, bd) and aL == bL
    print(f"{prec_name}: load v1/v2 {times[0]:.3f} s, v3 {times[1]:.3f} s")
    # the wrong precision is refused with a clear error
    with Context(0, FP16 if prec == FP32 else FP32) as ctx:
        with pytest.raises(lib.RkError, match="v3"):
            ctx.load_weights(v3)
