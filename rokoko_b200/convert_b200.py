"""KOKO v1 / v2 -> KOKO v3, the B200-layout weight file.

    python -m rokoko_b200.convert_b200 weights.bin weights.b200.bin [--fp16]

v3 holds the weights exactly as librokoko_b200 packs them for the tcgen05
kernels (rk_convert_koko_b200 in include/rk_b200.h): loading it is one device
allocation and one copy instead of the per-tensor weight norm, transposes,
polyphase split and 16-bit conversion.  --fp16 packs for RK_PRECISION_FP16
contexts (fp16 planes; a v2 input needs it); without it, split-bf16 planes for
RK_PRECISION_FP32.  Runs on the host; no GPU is needed.
"""
from __future__ import annotations

import argparse
import ctypes
import sys

from . import lib


def convert(blob: bytes, precision: int) -> bytes:
    L = lib.load()
    src = (ctypes.c_char * len(blob)).from_buffer_copy(blob)
    n = ctypes.c_size_t(0)
    lib.check(L.rk_convert_koko_b200(src, len(blob), precision, None, 0, ctypes.byref(n)), "rk_convert_koko_b200")
    out = (ctypes.c_char * n.value)()
    lib.check(L.rk_convert_koko_b200(src, len(blob), precision, out, n.value, ctypes.byref(n)),
              "rk_convert_koko_b200")
    return bytes(out)


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="rokoko_b200.convert_b200")
    p.add_argument("src")
    p.add_argument("dst")
    p.add_argument("--fp16", action="store_true")
    a = p.parse_args(argv)
    with open(a.src, "rb") as f:
        blob = f.read()
    out = convert(blob, lib.RK_PRECISION_FP16 if a.fp16 else lib.RK_PRECISION_FP32)
    with open(a.dst, "wb") as f:
        f.write(out)
    print(f"{a.dst}: {len(out)} bytes", file=sys.stderr)
    return 0


if __name__ == "__main__":
    sys.exit(main())
