"""Record the reference's own phonemizer outputs -> tests/golden/ref_g2p.json.

    make -C oracle ref-g2p REF_DIR=<reference checkout> CUTLASS_DIR=<cutlass include dir>   # here
    python tests/golden/make_g2p_golden.py                                                  # on a B200

Loads oracle/_ref/libref_g2p.so (the reference's rokoko::G2PModelCuda,
src/g2p.h, with its CUTLASS GEMMs, behind oracle/ref_g2p_shim.cu) on the
seeded G2P3 file rokoko_b200.g2pfile.random_blob(0), runs its infer() once per
input and stores, per input: the text, the reference's UTF-8 phones, its
per-frame argmax ids and the top-2 margin of its logits per frame (head bias
added).  Inputs: seeded synthetic sentences of distinct lengths (the
reference captures a CUDA graph on the second call of a length, which the
shim refuses), non-ASCII text, 600 characters, the 2048-character maximum,
2049 characters and the empty string (both give "").
"""
from __future__ import annotations

import base64
import ctypes
import json
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from rokoko_b200 import g2pfile  # noqa: E402

OUT = os.path.join(ROOT, "tests", "golden", "ref_g2p.json")


def cases() -> list[str]:
    texts, seen = [], set()
    for t in g2pfile.random_texts(60, seed=7, mean=110, sd=70, lo=2, hi=500):
        if len(t) not in seen and len(texts) < 36:
            seen.add(len(t))
            texts.append(t)
    extra = ["naïve café, 12 € — ok", "Hello, World! 123", "a",
             g2pfile.random_texts(1, seed=11, mean=600, sd=0, lo=600, hi=600)[0],
             g2pfile.random_texts(1, seed=12, mean=2048, sd=0, lo=2048, hi=2048)[0],
             g2pfile.random_texts(1, seed=13, mean=2049, sd=0, lo=2049, hi=2049)[0], ""]
    return texts + extra


def main() -> int:
    lib = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref_g2p.so"))
    lib.ref_g2p_load.restype = ctypes.c_void_p
    lib.ref_g2p_load.argtypes = [ctypes.c_char_p]
    lib.ref_g2p_free.argtypes = [ctypes.c_void_p]
    lib.ref_g2p_infer.restype = ctypes.c_long
    lib.ref_g2p_infer.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p,
                                  ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                  ctypes.c_size_t]
    blob = g2pfile.random_blob(0)
    cfg, _, _, w = g2pfile.parse(blob)
    with tempfile.NamedTemporaryFile(suffix=".bin", delete=False) as f:
        f.write(blob)
        path = f.name
    h = lib.ref_g2p_load(path.encode())
    os.unlink(path)
    if not h:
        print("reference G2P load failed", file=sys.stderr)
        return 1
    out = []
    lens = set()
    for text in cases():
        b = text.encode("utf-8")
        T = len(text)
        if T in lens and T > 0:
            raise RuntimeError(f"repeated length {T}")
        lens.add(T)
        rows = max(T, 1) * cfg.up
        best = np.zeros(rows, np.int32)
        logits = np.zeros(rows * cfg.n_phones, np.float32)
        buf = ctypes.create_string_buffer(4 * rows + 16)
        n = lib.ref_g2p_infer(h, b, len(b), buf, len(buf), best.ctypes.data, best.size, logits.ctypes.data,
                              logits.size)
        if n < 0:
            raise RuntimeError(f"ref_g2p_infer returned {n} for length {T}")
        rec = {"text": text, "out": buf.raw[:n].decode("utf-8")}
        if 0 < T <= g2pfile.MAX_POS:
            lg = logits.reshape(rows, cfg.n_phones)[: T * cfg.up] + w["head_b"][None, :]
            top = np.sort(lg, axis=1)
            rec["best"] = base64.b64encode(best[: T * cfg.up].astype(np.uint8).tobytes()).decode()
            rec["margin"] = base64.b64encode((top[:, -1] - top[:, -2]).astype(np.float16).tobytes()).decode()
        out.append(rec)
    lib.ref_g2p_free(h)
    with open(OUT, "w") as f:
        json.dump({"model": "rokoko_b200.g2pfile.random_blob(0)", "source": "reference src/g2p.h infer() on B200",
                   "cases": out}, f, indent=0, ensure_ascii=False)
    print(f"wrote {OUT}: {len(out)} cases")
    return 0


if __name__ == "__main__":
    sys.exit(main())
