"""KOKO v1 (FP32) -> v2 (pre-baked FP16) weight-file converter.

Restates the reference's scripts/convert_v2.py (`convert`, :111-349) so that a
user of this package can produce the file its FP16 path loads
(src/weights.cpp:320-494 `assign_v2_fp16_pointers`) without the reference
tree.  The output is byte-identical to the reference script's on the same
input (tests/test_convert_v2.py pins it against a digest recorded from the
reference script).

What the v2 file holds, per tensor family (the file's tensor order is part of
the format, because offsets follow it; it is reproduced exactly):

* weight norm baked in: every `.weight_v` with a `.weight_g` becomes
  g * v / max(||v||, 1e-12), the norm over all dims but 0, in FP32
  (convert_v2.py:87-92, 116-120);
* FP32 tensors kept as they are (embeddings, norms, biases, small convs);
* `<name>.f16`: an FP16 copy of a GEMM weight (linear layers, LSTM matrices,
  AdaIN FCs, ConvTranspose weights, conv_post);
* `<name>.nhwc_f16`: a conv weight [C_out, C_in, K] transposed to
  [C_out, K, C_in] in FP16 when C_in % 8 == 0 and C_out % 4 == 0;
  `<name>.nhwc_f16_pad<N>` with C_in zero-padded up to N = ceil8(C_in) when only
  C_in is misaligned; nothing when C_out % 4 != 0 (convert_v2.py:135-146);
* `<prefix>.bias_combined_fwd|rev` = bias_ih + bias_hh per LSTM direction, FP32.

    python -m rokoko_b200.convert_v2 --weights weights.bin -o weights.fp16.bin
"""
from __future__ import annotations

import argparse
import sys

import numpy as np

from . import koko

# Geometry of the convolutions that get NHWC copies: (C_out, C_in, K).
_F0N_BLOCKS = ((512, 512, False, False), (512, 256, True, True), (256, 256, False, False))
_DEC_BLOCKS = ((1090, 1024), (1090, 1024), (1090, 1024), (1090, 512))
_RESBLOCKS = ((256, 3), (256, 7), (256, 11), (128, 3), (128, 7), (128, 11))
_NOISE_RES = ((256, 7), (128, 11))


def bake_weight_norm(g: np.ndarray, v: np.ndarray) -> np.ndarray:
    """g * v / max(||v||_2, 1e-12) over all dims but 0, evaluated in FP32 with
    numpy's own norm (the same reduction the reference script uses)."""
    rows = v.shape[0]
    flat = v.reshape(rows, -1)
    nrm = np.linalg.norm(flat, axis=1, keepdims=True).clip(min=1e-12)
    return (g.reshape(rows, 1) * flat / nrm).reshape(v.shape).astype(np.float32)


class _Plan:
    """Collects (name, array) entries in file order."""

    def __init__(self, t: dict[str, np.ndarray]):
        self.t = t
        self.entries: list[tuple[str, np.ndarray]] = []

    def fp32(self, *names: str) -> None:
        for n in names:
            if n in self.t:
                self.entries.append((n, self.t[n]))

    def half(self, *names: str) -> None:
        for n in names:
            if n in self.t:
                self.entries.append((n + ".f16", self.t[n].astype(np.float16)))

    def nhwc(self, name: str, c_out: int, c_in: int, k: int) -> None:
        v = self.t.get(name)
        if v is None or c_out % 4:
            return
        w = np.ascontiguousarray(v.reshape(c_out, c_in, k).transpose(0, 2, 1))  # [C_out, K, C_in]
        if c_in % 8 == 0:
            self.entries.append((name + ".nhwc_f16", w.astype(np.float16)))
            return
        c_pad = (c_in + 7) // 8 * 8
        wp = np.zeros((c_out, k, c_pad), w.dtype)
        wp[:, :, :c_in] = w
        self.entries.append((f"{name}.nhwc_f16_pad{c_pad}", wp.astype(np.float16)))

    def lstm(self, prefix: str) -> None:
        self.half(*(prefix + s for s in (".weight_ih_l0", ".weight_hh_l0", ".weight_ih_l0_reverse",
                                         ".weight_hh_l0_reverse")))
        for d, sfx in (("fwd", ""), ("rev", "_reverse")):
            bi, bh = self.t.get(f"{prefix}.bias_ih_l0{sfx}"), self.t.get(f"{prefix}.bias_hh_l0{sfx}")
            if bi is not None and bh is not None:
                self.entries.append((f"{prefix}.bias_combined_{d}", (bi + bh).astype(np.float32)))

    def adain_pair(self, p1: str, p2: str) -> None:
        """Two AdaIN1d layers: FP32 norm weight / bias / FC bias of each, then FP16 FC weights."""
        for p in (p1, p2):
            self.fp32(p + ".norm.weight", p + ".norm.bias", p + ".fc.bias")
        self.half(p1 + ".fc.weight", p2 + ".fc.weight")

    def resblk1d(self, p: str, c_in: int, c_out: int, shortcut: bool, upsample: bool) -> None:
        """AdainResBlk1d: conv biases, NHWC conv weights, AdaINs, optional 1x1 shortcut and pool."""
        self.fp32(p + ".conv1.bias", p + ".conv2.bias")
        self.nhwc(p + ".conv1.weight_v", c_out, c_in, 3)
        self.nhwc(p + ".conv2.weight_v", c_out, c_out, 3)
        self.adain_pair(p + ".norm1", p + ".norm2")
        if shortcut:
            self.nhwc(p + ".conv1x1.weight_v", c_out, c_in, 1)
        if upsample:
            self.fp32(p + ".pool.weight_v", p + ".pool.bias")

    def resblock1(self, p: str, c: int, k: int) -> None:
        """AdaINResBlock1: per round j, both convs, then both AdaINs, then the Snake alphas."""
        for j in range(3):
            for grp in ("convs1", "convs2"):
                self.fp32(f"{p}.{grp}.{j}.bias")
                self.nhwc(f"{p}.{grp}.{j}.weight_v", c, c, k)
            for grp in ("adain1", "adain2"):
                q = f"{p}.{grp}.{j}"
                self.fp32(q + ".norm.weight", q + ".norm.bias", q + ".fc.bias")
                self.half(q + ".fc.weight")
            self.fp32(f"{p}.alpha1.{j}", f"{p}.alpha2.{j}")


def convert(tensors: dict[str, np.ndarray]) -> list[tuple[str, np.ndarray]]:
    """v1 tensors -> v2 entries in file order.  `tensors` is not modified."""
    t = dict(tensors)
    for gname in [n for n in t if n.endswith(".weight_g")]:
        vname = gname[: -len(".weight_g")] + ".weight_v"
        if vname in t:
            t[vname] = bake_weight_norm(t[gname], t[vname])
    P = _Plan(t)

    # ALBERT: embeddings FP32; projections FP16 with FP32 biases and norms
    P.fp32(*(f"bert.embeddings.{n}" for n in ("word_embeddings.weight", "position_embeddings.weight",
                                              "token_type_embeddings.weight", "LayerNorm.weight",
                                              "LayerNorm.bias")))
    P.fp32("bert.encoder.embedding_hidden_mapping_in.bias")
    P.half("bert.encoder.embedding_hidden_mapping_in.weight")
    a = "bert.encoder.albert_layer_groups.0.albert_layers.0"
    for lin in (".attention.query", ".attention.key", ".attention.value", ".attention.dense"):
        P.fp32(a + lin + ".bias")
        P.half(a + lin + ".weight")
    P.fp32(a + ".attention.LayerNorm.weight", a + ".attention.LayerNorm.bias")
    for lin in (".ffn", ".ffn_output"):
        P.fp32(a + lin + ".bias")
        P.half(a + lin + ".weight")
    P.fp32(a + ".full_layer_layer_norm.weight", a + ".full_layer_layer_norm.bias")
    P.fp32("bert_encoder.bias")
    P.half("bert_encoder.weight")

    # text encoder
    P.fp32("text_encoder.embedding.weight")
    for i in range(3):
        c = f"text_encoder.cnn.{i}"
        P.fp32(c + ".0.bias", c + ".1.gamma", c + ".1.beta")
        P.nhwc(c + ".0.weight_v", 512, 512, 5)
    P.lstm("text_encoder.lstm")

    # prosody predictor
    for i in range(3):
        P.lstm(f"predictor.text_encoder.lstms.{2 * i}")
        P.fp32(f"predictor.text_encoder.lstms.{2 * i + 1}.fc.bias")
        P.half(f"predictor.text_encoder.lstms.{2 * i + 1}.fc.weight")
    P.lstm("predictor.lstm")
    P.fp32("predictor.duration_proj.linear_layer.bias")
    P.half("predictor.duration_proj.linear_layer.weight")
    P.lstm("predictor.shared")
    for chain in ("predictor.F0", "predictor.N"):
        for i, (c_in, c_out, shortcut, upsample) in enumerate(_F0N_BLOCKS):
            P.resblk1d(f"{chain}.{i}", c_in, c_out, shortcut, upsample)
    P.fp32("predictor.F0_proj.weight", "predictor.F0_proj.bias", "predictor.N_proj.weight", "predictor.N_proj.bias")

    # decoder
    P.fp32("decoder.F0_conv.weight_v", "decoder.F0_conv.bias", "decoder.N_conv.weight_v", "decoder.N_conv.bias")
    P.fp32("decoder.asr_res.0.weight_v", "decoder.asr_res.0.bias")
    P.resblk1d("decoder.encode", 514, 1024, True, False)
    for i, (c_in, c_out) in enumerate(_DEC_BLOCKS):
        P.resblk1d(f"decoder.decode.{i}", c_in, c_out, True, i == 3)

    # generator
    g = "decoder.generator"
    for i in range(2):
        P.fp32(f"{g}.ups.{i}.bias")
        P.half(f"{g}.ups.{i}.weight_v")
    P.fp32(f"{g}.noise_convs.0.bias")
    P.nhwc(f"{g}.noise_convs.0.weight", 256, 22, 12)
    P.fp32(f"{g}.noise_convs.1.bias")
    P.nhwc(f"{g}.noise_convs.1.weight", 128, 22, 1)
    for i, (c, k) in enumerate(_RESBLOCKS):
        P.resblock1(f"{g}.resblocks.{i}", c, k)
    for i, (c, k) in enumerate(_NOISE_RES):
        P.resblock1(f"{g}.noise_res.{i}", c, k)
    P.fp32(f"{g}.conv_post.bias")
    P.half(f"{g}.conv_post.weight_v")
    P.fp32(f"{g}.m_source.l_linear.weight", f"{g}.m_source.l_linear.bias")
    return P.entries


def convert_blob(v1_blob: bytes) -> bytes:
    """KOKO v1 bytes -> KOKO v2 bytes."""
    version, tensors = koko.parse(v1_blob)
    if version != 1:
        raise ValueError(f"expected a KOKO v1 file, got version {version}")
    return koko.serialize(convert(tensors), version=2)


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="rokoko_b200.convert_v2", description="KOKO v1 (FP32) -> v2 (FP16) weights")
    p.add_argument("--weights", required=True, help="KOKO v1 file")
    p.add_argument("-o", "--output", required=True)
    a = p.parse_args(argv)
    with open(a.weights, "rb") as f:
        out = convert_blob(f.read())
    with open(a.output, "wb") as f:
        f.write(out)
    print(f"{a.output}: {len(out)} bytes", file=sys.stderr)
    return 0


if __name__ == "__main__":
    sys.exit(main())
