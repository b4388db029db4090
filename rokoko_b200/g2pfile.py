"""G2P3 model file: format, fixed vocabularies, seeded random-init writer, reader.

The layout is the one rokoko's neural phonemizer loads
(`G2PModelCuda::load_from_file_`, src/g2p.h:441-540):

    "G2P3" | u32 hdr[10] = d, heads, n_layers, ff, up, n_chars, n_phones, 0, 0, flags
    u32 n_char_entries | n x (u32 codepoint, u32 id)      char -> input id
    u32 n_phone_entries | n x (u32 codepoint, u32 id)     output id -> phone
    f32 weights, in this order (PyTorch Linear layout [out][in]):
        char_emb [n_chars][d]
        per layer: n1_w [d], qkv_w [3d][d], qkv_b [3d], out_w [d][d], out_b [d],
                   n2_w [d], gate_w [ff][d], gate_b [ff], up_w [ff][d], up_b [ff],
                   down_w [d][ff], down_b [d]
        up_w [up*d][d], up_b [up*d], head_w [n_phones][d], head_b [n_phones]

flags: bit 0 RoPE, bit 1 QK-norm, bit 2 conv module, bit 3 RMSNorm.  The
reference loader accepts only RoPE + RMSNorm without QK-norm / conv module
(flags 9, src/g2p.h:464-471); so does this framework.

Vocabularies.  Input: the 95 printable ASCII characters (space .. '~') map to
ids 1 .. 95, id 0 = PAD (every other character); n_chars = 96.  Output: id 0 =
CTC blank, ids 1 .. 77 = 77 phone symbols (the 26 lowercase letters and the
51 IPA-extension code points U+0250 .. U+0282); n_phones = 78.  These are the
sizes of the model the reference ships (fixed ASCII charset, 77 IPA phones);
its trained weights are not available here, so `random_blob` writes a seeded
random initialisation with the reference model's shape (d 256, 4 heads of 64,
8 layers, SwiGLU ff 1024, 3x upsample).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np

MAGIC = b"G2P3"
FLAG_ROPE, FLAG_QK_NORM, FLAG_CONV, FLAG_RMSNORM = 1, 2, 4, 8
MAX_POS = 2048  # the reference's max_pos_ (src/g2p.h:425): longest input in characters

CHAR_CODEPOINTS = list(range(32, 127))                                # ids 1 .. 95
PHONE_CODEPOINTS = list(range(ord("a"), ord("z") + 1)) + list(range(0x250, 0x283))  # ids 1 .. 77


@dataclass
class G2PConfig:
    d: int = 256
    heads: int = 4
    n_layers: int = 8
    ff: int = 1024
    up: int = 3
    n_chars: int = len(CHAR_CODEPOINTS) + 1
    n_phones: int = len(PHONE_CODEPOINTS) + 1
    flags: int = FLAG_ROPE | FLAG_RMSNORM


def tensor_specs(cfg: G2PConfig) -> list[tuple[str, tuple]]:
    """(name, shape) of every weight in file order."""
    d, ff = cfg.d, cfg.ff
    out = [("char_emb", (cfg.n_chars, d))]
    for i in range(cfg.n_layers):
        p = f"layers.{i}."
        out += [(p + "n1_w", (d,)), (p + "qkv_w", (3 * d, d)), (p + "qkv_b", (3 * d,)),
                (p + "out_w", (d, d)), (p + "out_b", (d,)), (p + "n2_w", (d,)),
                (p + "gate_w", (ff, d)), (p + "gate_b", (ff,)), (p + "up_w", (ff, d)), (p + "up_b", (ff,)),
                (p + "down_w", (d, ff)), (p + "down_b", (d,))]
    out += [("up_w", (cfg.up * d, d)), ("up_b", (cfg.up * d,)),
            ("head_w", (cfg.n_phones, d)), ("head_b", (cfg.n_phones,))]
    return out


def random_weights(cfg: G2PConfig, seed: int = 0) -> dict[str, np.ndarray]:
    """Seeded initialisation: embeddings N(0, 1); Linear weights N(0, 1/in) (unit-variance
    outputs); biases N(0, 0.02); RMSNorm weights 1 + N(0, 0.1); the head N(0, 4/in), so
    that the per-frame argmax has clear margins."""
    rng = np.random.default_rng(seed)
    w = {}
    for name, shape in tensor_specs(cfg):
        leaf = name.rsplit(".", 1)[-1]
        if name == "char_emb":
            a = rng.standard_normal(shape)
        elif leaf.endswith("_b"):
            a = 0.02 * rng.standard_normal(shape)
        elif leaf in ("n1_w", "n2_w"):
            a = 1.0 + 0.1 * rng.standard_normal(shape)
        elif name == "head_w":
            a = rng.standard_normal(shape) * (2.0 / np.sqrt(shape[1]))
        else:
            a = rng.standard_normal(shape) / np.sqrt(shape[1])
        w[name] = a.astype(np.float32)
    return w


def serialize(cfg: G2PConfig, weights: dict[str, np.ndarray]) -> bytes:
    hdr = [cfg.d, cfg.heads, cfg.n_layers, cfg.ff, cfg.up, cfg.n_chars, cfg.n_phones, 0, 0, cfg.flags]
    out = [MAGIC, struct.pack("<10I", *hdr)]
    out.append(struct.pack("<I", len(CHAR_CODEPOINTS)))
    out += [struct.pack("<2I", cp, i + 1) for i, cp in enumerate(CHAR_CODEPOINTS)]
    out.append(struct.pack("<I", len(PHONE_CODEPOINTS)))
    out += [struct.pack("<2I", cp, i + 1) for i, cp in enumerate(PHONE_CODEPOINTS)]
    for name, shape in tensor_specs(cfg):
        a = np.ascontiguousarray(weights[name], dtype="<f4")
        if a.shape != shape:
            raise ValueError(f"{name}: shape {a.shape}, expected {shape}")
        out.append(a.tobytes())
    return b"".join(out)


def random_blob(seed: int = 0, cfg: G2PConfig | None = None) -> bytes:
    cfg = cfg or G2PConfig()
    return serialize(cfg, random_weights(cfg, seed))


def parse(blob: bytes) -> tuple[G2PConfig, dict[int, int], dict[int, int], dict[str, np.ndarray]]:
    """(config, char codepoint -> id, phone id -> codepoint, weights) of a G2P3 blob."""
    if blob[:4] != MAGIC:
        raise ValueError("not a G2P3 file")
    hdr = struct.unpack_from("<10I", blob, 4)
    cfg = G2PConfig(d=hdr[0], heads=hdr[1], n_layers=hdr[2], ff=hdr[3], up=hdr[4], n_chars=hdr[5],
                    n_phones=hdr[6], flags=hdr[9])
    off = 44
    (n,) = struct.unpack_from("<I", blob, off)
    off += 4
    chars = {}
    for _ in range(n):
        cp, i = struct.unpack_from("<2I", blob, off)
        chars[cp] = i
        off += 8
    (n,) = struct.unpack_from("<I", blob, off)
    off += 4
    phones = {}
    for _ in range(n):
        cp, i = struct.unpack_from("<2I", blob, off)
        phones[i] = cp
        off += 8
    w = {}
    for name, shape in tensor_specs(cfg):
        cnt = int(np.prod(shape))
        w[name] = np.frombuffer(blob, dtype="<f4", count=cnt, offset=off).reshape(shape)
        off += 4 * cnt
    if off != len(blob):
        raise ValueError(f"G2P3 size mismatch: {off} bytes parsed of {len(blob)}")
    return cfg, chars, phones, w


def random_texts(n: int, seed: int = 0, mean: float = 121.0, sd: float = 60.0, lo: int = 1,
                 hi: int = 510) -> list[str]:
    """Seeded synthetic sentences: lengths ~ truncated N(mean, sd) (the reference's G2P
    corpus averages 121 characters per sentence), words of 1-10 lowercase letters with
    an occasional capital, digit or punctuation mark, separated by spaces."""
    rng = np.random.default_rng(seed)
    letters = "abcdefghijklmnopqrstuvwxyz"
    extra = "ABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789,.;:!?'-\""
    out = []
    for _ in range(n):
        L = int(np.clip(round(rng.normal(mean, sd)), lo, hi))
        s = []
        while len(s) < L:
            w = rng.integers(1, 11)
            for _ in range(w):
                s.append(extra[rng.integers(len(extra))] if rng.random() < 0.08 else letters[rng.integers(26)])
            s.append(" ")
        out.append("".join(s[:L]))
    return out
