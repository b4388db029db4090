"""Records what the reference's own v1 -> v2 weight converter produces for the
seed-0 random-init KOKO v1 file, so tests/test_convert_v2.py can hold
rokoko_b200.convert_v2 to it byte for byte.

Needs the reference checkout (its scripts/convert_v2.py is imported and run
through its own parse_koko / convert / write_koko_v2); run it where that tree
exists.  Writes tests/golden/v2_seed0.json: file size, SHA-256 and the
(name, dtype, shape, SHA-256) of every tensor, in file order.

    python tests/golden/make_v2_digest.py [REFERENCE_DIR]
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)


def main(ref_dir: str) -> None:
    from rokoko_b200 import koko
    spec = importlib.util.spec_from_file_location("ref_convert_v2", os.path.join(ref_dir, "scripts", "convert_v2.py"))
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    scratch = os.path.join(HERE, ".scratch")
    os.makedirs(scratch, exist_ok=True)
    try:
        src = os.path.join(scratch, "v1_seed0.bin")
        dst = os.path.join(scratch, "v2_seed0.bin")
        with open(src, "wb") as f:
            f.write(koko.random_v1_blob(0))
        ref.write_koko_v2(dst, ref.convert(ref.parse_koko(src)))
        with open(dst, "rb") as f:
            blob = f.read()
    finally:
        shutil.rmtree(scratch, ignore_errors=True)
    _, tensors = koko.parse(blob)
    rec = {
        "generator": "tests/golden/make_v2_digest.py (reference scripts/convert_v2.py on koko.random_v1_blob(0))",
        "bytes": len(blob),
        "sha256": hashlib.sha256(blob).hexdigest(),
        "tensors": [[n, str(a.dtype), list(a.shape), hashlib.sha256(a.tobytes()).hexdigest()[:16]]
                    for n, a in tensors.items()],
    }
    with open(os.path.join(HERE, "v2_seed0.json"), "w") as f:
        json.dump(rec, f, indent=0)
    print(f"{len(rec['tensors'])} tensors, {rec['bytes']} bytes, sha256 {rec['sha256']}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_v2_digest.py <reference checkout>")
    main(sys.argv[1])
