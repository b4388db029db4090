"""IPA -> model input: the host side of rokoko's to_tokens / chunk_ipa
(src/rokoko.h:141-221) on the library's rk_ipa_* entry points.

    from rokoko_b200 import tokens
    ids = tokens.to_tokens("həlˈoʊ wˈɜːld.")        # int32 [BOS, ..., EOS]
    for piece, ids in tokens.chunk_ipa(long_ipa):     # <= 510 code points each
        ...

With the phonemizer (rokoko_b200.g2p) this is the text side of the path:
text -> G2PModel.infer -> chunk_ipa -> Context.infer / encode per chunk.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import lib

MAX_IPA_CHARS = 510


def to_tokens(ipa: str) -> np.ndarray:
    L = lib.load()
    b = ipa.encode("utf-8")
    n = ctypes.c_size_t(0)
    lib.check(L.rk_ipa_to_tokens(b, len(b), None, 0, ctypes.byref(n)), "rk_ipa_to_tokens")
    out = np.zeros(n.value, np.int32)
    lib.check(L.rk_ipa_to_tokens(b, len(b), out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), out.size,
                                 ctypes.byref(n)), "rk_ipa_to_tokens")
    return out


def chunk_bounds(ipa: bytes) -> list[int]:
    """End byte offsets of the chunks of UTF-8 IPA bytes."""
    L = lib.load()
    n = ctypes.c_size_t(0)
    lib.check(L.rk_ipa_chunks(ipa, len(ipa), None, 0, ctypes.byref(n)), "rk_ipa_chunks")
    ends = (ctypes.c_size_t * max(n.value, 1))()
    lib.check(L.rk_ipa_chunks(ipa, len(ipa), ends, n.value, ctypes.byref(n)), "rk_ipa_chunks")
    return list(ends[: n.value])


def chunk_ipa(ipa: str) -> list[tuple[str, np.ndarray]]:
    """(piece, token ids) per chunk, as the reference's chunk_ipa."""
    b = ipa.encode("utf-8")
    out, start = [], 0
    for end in chunk_bounds(b):
        piece = b[start:end].decode("utf-8", errors="surrogateescape")
        out.append((piece, to_tokens(piece)))
        start = end
    return out
