"""KOKO weight-file format: tensor inventory, random-init writer, reader.

The on-disk layout is the one rokoko's loader parses (src/weights.cpp:35-50
`parse_header`, :500-564 `Weights::prefetch`; writer side
scripts/convert_v2.py:54-81 `write_koko_v2`):

    u32 magic 0x4F4B4F4B ("KOKO") | u32 version (1 = fp32, 2 = pre-baked fp16)
    u64 header_len | header text: one line per tensor
        "<name> <offset> <size_bytes> <dtype fp32|fp16> <dim0> <dim1> ..."
    zero pad to align(16 + header_len, 4096) = data start
    tensor data; every tensor starts 256-byte aligned (offsets relative to data start)

Tensor names and shapes follow the reference's name->pointer binding
(src/weights.cpp:57-314) and the converter's view of the same tensors
(scripts/convert_v2.py:208-347).  `model_tensor_specs()` lists every tensor the
hot path reads plus `bert.pooler` (loaded, unused, src/weights.cpp:102-103).

Random initialisation follows the benchmark recipe: linear/conv/embedding
weights ~ N(0, 0.02); weight-norm g = ||v|| (so the materialised weight equals
v); LayerNorm / InstanceNorm gamma = 1, beta = 0; Snake alpha = 1; all biases 0.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np

KOKO_MAGIC = 0x4F4B4F4B
HEADER_ALIGN = 4096
TENSOR_ALIGN = 256

# kinds drive the random initialiser
LINEAR, BIAS, ONES, ZEROS, WEIGHT_G, EMBED = "linear", "bias", "ones", "zeros", "weight_g", "embed"


@dataclass(frozen=True)
class Spec:
    name: str
    shape: tuple
    kind: str


def _bilstm(prefix: str, inp: int, hid: int = 256):
    out = []
    for sfx in ("", "_reverse"):
        out += [
            Spec(f"{prefix}.weight_ih_l0{sfx}", (4 * hid, inp), LINEAR),
            Spec(f"{prefix}.weight_hh_l0{sfx}", (4 * hid, hid), LINEAR),
            Spec(f"{prefix}.bias_ih_l0{sfx}", (4 * hid,), BIAS),
            Spec(f"{prefix}.bias_hh_l0{sfx}", (4 * hid,), BIAS),
        ]
    return out


def _wn_conv(prefix: str, cout: int, cin: int, k: int, bias: bool = True):
    out = [Spec(f"{prefix}.weight_g", (cout, 1, 1), WEIGHT_G),
           Spec(f"{prefix}.weight_v", (cout, cin, k), LINEAR)]
    if bias:
        out.append(Spec(f"{prefix}.bias", (cout,), BIAS))
    return out


def _adain1d(prefix: str, c: int, style: int = 128):
    return [Spec(f"{prefix}.norm.weight", (c,), ONES),
            Spec(f"{prefix}.norm.bias", (c,), ZEROS),
            Spec(f"{prefix}.fc.weight", (2 * c, style), LINEAR),
            Spec(f"{prefix}.fc.bias", (2 * c,), BIAS)]


def _adain_resblk1d(prefix: str, din: int, dout: int, shortcut: bool, upsample: bool):
    """AdainResBlk1d (src/weights.cpp:164-186)."""
    out = _wn_conv(f"{prefix}.conv1", dout, din, 3) + _wn_conv(f"{prefix}.conv2", dout, dout, 3)
    out += _adain1d(f"{prefix}.norm1", din) + _adain1d(f"{prefix}.norm2", dout)
    if shortcut:
        out += _wn_conv(f"{prefix}.conv1x1", dout, din, 1, bias=False)
    if upsample:
        out += _wn_conv(f"{prefix}.pool", din, 1, 3)
    return out


def _adain_resblock1(prefix: str, c: int, k: int):
    """AdaINResBlock1 (src/weights.cpp:226-245)."""
    out = []
    for j in range(3):
        out += _wn_conv(f"{prefix}.convs1.{j}", c, c, k)
        out += _wn_conv(f"{prefix}.convs2.{j}", c, c, k)
        out += _adain1d(f"{prefix}.adain1.{j}", c)
        out += _adain1d(f"{prefix}.adain2.{j}", c)
        out += [Spec(f"{prefix}.alpha1.{j}", (1, c, 1), ONES),
                Spec(f"{prefix}.alpha2.{j}", (1, c, 1), ONES)]
    return out


def model_tensor_specs() -> list[Spec]:
    s: list[Spec] = []
    # ALBERT (src/weights.cpp:67-104)
    s += [Spec("bert.embeddings.word_embeddings.weight", (178, 128), EMBED),
          Spec("bert.embeddings.position_embeddings.weight", (512, 128), EMBED),
          Spec("bert.embeddings.token_type_embeddings.weight", (2, 128), EMBED),
          Spec("bert.embeddings.LayerNorm.weight", (128,), ONES),
          Spec("bert.embeddings.LayerNorm.bias", (128,), ZEROS),
          Spec("bert.encoder.embedding_hidden_mapping_in.weight", (768, 128), LINEAR),
          Spec("bert.encoder.embedding_hidden_mapping_in.bias", (768,), BIAS)]
    a = "bert.encoder.albert_layer_groups.0.albert_layers.0"
    for n in ("query", "key", "value", "dense"):
        s += [Spec(f"{a}.attention.{n}.weight", (768, 768), LINEAR),
              Spec(f"{a}.attention.{n}.bias", (768,), BIAS)]
    s += [Spec(f"{a}.attention.LayerNorm.weight", (768,), ONES),
          Spec(f"{a}.attention.LayerNorm.bias", (768,), ZEROS),
          Spec(f"{a}.ffn.weight", (2048, 768), LINEAR), Spec(f"{a}.ffn.bias", (2048,), BIAS),
          Spec(f"{a}.ffn_output.weight", (768, 2048), LINEAR), Spec(f"{a}.ffn_output.bias", (768,), BIAS),
          Spec(f"{a}.full_layer_layer_norm.weight", (768,), ONES),
          Spec(f"{a}.full_layer_layer_norm.bias", (768,), ZEROS),
          Spec("bert.pooler.weight", (768, 768), LINEAR), Spec("bert.pooler.bias", (768,), BIAS),
          Spec("bert_encoder.weight", (512, 768), LINEAR), Spec("bert_encoder.bias", (512,), BIAS)]
    # text encoder (src/weights.cpp:115-134)
    s.append(Spec("text_encoder.embedding.weight", (178, 512), EMBED))
    for i in range(3):
        s += _wn_conv(f"text_encoder.cnn.{i}.0", 512, 512, 5)
        s += [Spec(f"text_encoder.cnn.{i}.1.gamma", (512,), ONES),
              Spec(f"text_encoder.cnn.{i}.1.beta", (512,), ZEROS)]
    s += _bilstm("text_encoder.lstm", 512)
    # predictor (src/weights.cpp:188-223)
    for i in range(3):
        s += _bilstm(f"predictor.text_encoder.lstms.{2 * i}", 640)
        s += [Spec(f"predictor.text_encoder.lstms.{2 * i + 1}.fc.weight", (1024, 128), LINEAR),
              Spec(f"predictor.text_encoder.lstms.{2 * i + 1}.fc.bias", (1024,), BIAS)]
    s += _bilstm("predictor.lstm", 640)
    s += [Spec("predictor.duration_proj.linear_layer.weight", (50, 512), LINEAR),
          Spec("predictor.duration_proj.linear_layer.bias", (50,), BIAS)]
    s += _bilstm("predictor.shared", 640)
    for chain in ("F0", "N"):
        s += _adain_resblk1d(f"predictor.{chain}.0", 512, 512, False, False)
        s += _adain_resblk1d(f"predictor.{chain}.1", 512, 256, True, True)
        s += _adain_resblk1d(f"predictor.{chain}.2", 256, 256, False, False)
        s += [Spec(f"predictor.{chain}_proj.weight", (1, 256, 1), LINEAR),
              Spec(f"predictor.{chain}_proj.bias", (1,), BIAS)]
    # decoder (src/weights.cpp:230-262)
    s += _wn_conv("decoder.F0_conv", 1, 1, 3) + _wn_conv("decoder.N_conv", 1, 1, 3)
    s += _wn_conv("decoder.asr_res.0", 64, 512, 1)
    s += _adain_resblk1d("decoder.encode", 514, 1024, True, False)
    for i in range(4):
        s += _adain_resblk1d(f"decoder.decode.{i}", 1090, 1024 if i < 3 else 512, True, i == 3)
    # generator (src/weights.cpp:264-313)
    g = "decoder.generator"
    s += [Spec(f"{g}.m_source.l_linear.weight", (1, 9), LINEAR),
          Spec(f"{g}.m_source.l_linear.bias", (1,), BIAS)]
    s += [Spec(f"{g}.ups.0.weight_g", (512, 1, 1), WEIGHT_G),
          Spec(f"{g}.ups.0.weight_v", (512, 256, 20), LINEAR), Spec(f"{g}.ups.0.bias", (256,), BIAS),
          Spec(f"{g}.ups.1.weight_g", (256, 1, 1), WEIGHT_G),
          Spec(f"{g}.ups.1.weight_v", (256, 128, 12), LINEAR), Spec(f"{g}.ups.1.bias", (128,), BIAS)]
    s += [Spec(f"{g}.noise_convs.0.weight", (256, 22, 12), LINEAR), Spec(f"{g}.noise_convs.0.bias", (256,), BIAS),
          Spec(f"{g}.noise_convs.1.weight", (128, 22, 1), LINEAR), Spec(f"{g}.noise_convs.1.bias", (128,), BIAS)]
    s += _adain_resblock1(f"{g}.noise_res.0", 256, 7) + _adain_resblock1(f"{g}.noise_res.1", 128, 11)
    for i, (c, k) in enumerate([(256, 3), (256, 7), (256, 11), (128, 3), (128, 7), (128, 11)]):
        s += _adain_resblock1(f"{g}.resblocks.{i}", c, k)
    s += _wn_conv(f"{g}.conv_post", 22, 128, 7)
    return s


def random_tensors(seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """Seeded random-init weights (see module docstring for the recipe)."""
    rng = np.random.default_rng(seed)
    specs = model_tensor_specs()
    out: dict[str, np.ndarray] = {}
    for sp in specs:
        if sp.kind in (LINEAR, EMBED):
            out[sp.name] = (rng.standard_normal(sp.shape, dtype=np.float32) * np.float32(std)).astype(np.float32)
        elif sp.kind == ONES:
            out[sp.name] = np.ones(sp.shape, np.float32)
        elif sp.kind in (BIAS, ZEROS):
            out[sp.name] = np.zeros(sp.shape, np.float32)
    # weight_g = ||weight_v|| per output row (dim 0), computed in float64
    for sp in specs:
        if sp.kind == WEIGHT_G:
            v = out[sp.name[: -len("weight_g")] + "weight_v"]
            nrm = np.sqrt((v.astype(np.float64).reshape(v.shape[0], -1) ** 2).sum(axis=1))
            out[sp.name] = nrm.astype(np.float32).reshape(sp.shape)
    return {sp.name: out[sp.name] for sp in specs}


def serialize(entries: list[tuple[str, np.ndarray]], version: int = 1) -> bytes:
    """KOKO bytes for `entries` (fp32 or fp16 arrays, in the order given)."""
    lines, offset, blobs = [], 0, []
    for name, arr in entries:
        arr = np.ascontiguousarray(arr)
        dt = {np.dtype(np.float32): "fp32", np.dtype(np.float16): "fp16"}[arr.dtype]
        lines.append(f"{name} {offset} {arr.nbytes} {dt} " + " ".join(str(d) for d in arr.shape))
        blobs.append((offset, arr.tobytes()))
        offset = (offset + arr.nbytes + TENSOR_ALIGN - 1) // TENSOR_ALIGN * TENSOR_ALIGN
    header = "\n".join(lines).encode()
    data_start = (16 + len(header) + HEADER_ALIGN - 1) // HEADER_ALIGN * HEADER_ALIGN
    buf = bytearray(data_start + offset)
    struct.pack_into("<IIQ", buf, 0, KOKO_MAGIC, version, len(header))
    buf[16:16 + len(header)] = header
    for off, b in blobs:
        buf[data_start + off: data_start + off + len(b)] = b
    return bytes(buf)


def random_v1_blob(seed: int = 0) -> bytes:
    return serialize(list(random_tensors(seed).items()), version=1)


def parse(blob: bytes) -> tuple[int, dict[str, np.ndarray]]:
    """Parse KOKO bytes -> (version, {name: array}).  Mirrors src/weights.cpp:500-564."""
    magic, version, hlen = struct.unpack_from("<IIQ", blob, 0)
    if magic != KOKO_MAGIC:
        raise ValueError("bad KOKO magic")
    if version not in (1, 2):
        raise ValueError(f"unsupported KOKO version {version}")
    header = blob[16:16 + hlen].decode()
    data_start = (16 + hlen + HEADER_ALIGN - 1) // HEADER_ALIGN * HEADER_ALIGN
    out = {}
    for line in header.strip().split("\n"):
        p = line.split()
        name, off, size, dt = p[0], int(p[1]), int(p[2]), p[3]
        shape = tuple(int(x) for x in p[4:])
        ndt = np.float32 if dt == "fp32" else np.float16
        out[name] = np.frombuffer(blob, ndt, size // np.dtype(ndt).itemsize, data_start + off).reshape(shape)
    return version, out
