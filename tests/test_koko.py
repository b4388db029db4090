"""KOKO weight-file format (src/weights.cpp:35-50, 500-564): the random-init
writer produces the reference's exact tensor inventory and file size."""
import numpy as np

from rokoko_b200 import koko


def test_inventory_matches_reference_file_size():
    specs = koko.model_tensor_specs()
    assert len(specs) == 688
    names = [s.name for s in specs]
    assert len(set(names)) == len(names)
    blob = koko.random_v1_blob(0)
    # the reference's FP32 binary expects exactly this many bytes (default_weights_size)
    assert len(blob) == 327296512


def test_roundtrip_and_weight_norm_identity():
    t = koko.random_tensors(1)
    blob = koko.serialize(list(t.items()))
    ver, back = koko.parse(blob)
    assert ver == 1 and set(back) == set(t)
    for n in ("decoder.generator.resblocks.3.convs1.0.weight_v", "bert.embeddings.LayerNorm.weight"):
        assert np.array_equal(back[n], t[n])
    # g = ||v|| per output row, so the materialised weight-norm weight equals v
    v = t["decoder.generator.ups.0.weight_v"]
    g = t["decoder.generator.ups.0.weight_g"].reshape(-1)
    nrm = np.sqrt((v.astype(np.float64).reshape(v.shape[0], -1) ** 2).sum(1))
    assert np.allclose(g, nrm, rtol=1e-6)


def test_parse_rejects_bad_magic():
    import pytest
    with pytest.raises(ValueError):
        koko.parse(b"\x00" * 64)
