"""Records the reference's decode-arena size, compute_decode_bytes(T, L)
(src/rokoko_common.h:160-229 of LokalOptima/rokoko), over a grid of (T, L)
into decode_bytes.json beside this script.

    python tests/golden/make_decode_bytes.py <reference checkout>

The function is header-only host code: a three-line C++ program that includes
the reference's src/rokoko_common.h is compiled with g++ in a temporary
directory (the header pulls in CUDA's headers, nothing is linked) and prints
the sizes.  tests/test_decode_bytes.py holds rk_compute_decode_bytes to them.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
GRID_T = [3, 18, 66, 130, 258, 512]
GRID_L = [1, 7, 32, 100, 352, 400, 416, 1000, 1664, 3328, 4096]

PROGRAM = r'''
#include "rokoko_common.h"
#include <cstdio>
int main() {
    const int Ts[] = {%s};
    const int Ls[] = {%s};
    for (int T : Ts)
        for (int L : Ls) printf("%%d %%d %%zu\n", T, L, rokoko::compute_decode_bytes(T, L));
    return 0;
}
'''


def sizes(reference: str) -> list[list[int]]:
    src = os.path.join(reference, "src")
    cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    with tempfile.TemporaryDirectory() as d:
        cpp = os.path.join(d, "decode_bytes.cpp")
        exe = os.path.join(d, "decode_bytes")
        with open(cpp, "w") as f:
            f.write(PROGRAM % (", ".join(map(str, GRID_T)), ", ".join(map(str, GRID_L))))
        subprocess.run(["g++", "-std=c++17", "-O1", "-I", src, "-I", cuda_inc, cpp, "-o", exe], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    return [[int(x) for x in line.split()] for line in out.splitlines() if line.strip()]


def main(reference: str) -> None:
    rows = sizes(reference)
    with open(os.path.join(HERE, "decode_bytes.json"), "w") as f:
        json.dump({"source": "rokoko::compute_decode_bytes, src/rokoko_common.h:160-229",
                   "rows": rows}, f)
        f.write("\n")
    print(f"{len(rows)} sizes written")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_decode_bytes.py <reference checkout>")
    main(sys.argv[1])
