"""Records the reference's IPA -> token conversion and chunking
(rokoko::to_tokens / chunk_ipa, src/rokoko.h:141-221 of LokalOptima/rokoko)
for seeded IPA strings into ipa_tokens.json beside this script.

    python tests/golden/make_ipa_tokens.py <reference checkout>

The functions are header-only host code: a short program that includes the
reference's src/rokoko.h is compiled with nvcc (the header pulls in CUDA
headers and the phonemizer's kernels; nothing of them runs) in a temporary
directory, reads one IPA string per line and prints, per chunk, its byte
length and token ids.  tests/test_tokens.py holds rk_ipa_to_tokens /
rk_ipa_chunks to them.
"""
from __future__ import annotations

import json
import os
import random
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))

PROGRAM = r'''
#include "rokoko.h"
#include <cstdio>
#include <iostream>
int main() {
    std::string line;
    while (std::getline(std::cin, line)) {
        auto chunks = rokoko::chunk_ipa(line);
        printf("%zu", chunks.size());
        for (auto& c : chunks) {
            printf(" | %zu %zu", c.phonemes.size(), c.tokens.size());
            for (int t : c.tokens) printf(" %d", t);
        }
        printf("\n");
    }
    return 0;
}
'''

# symbols of the Kokoro vocabulary and a few outside it (dropped by to_tokens)
IPA = ("abcdefhijklmnopqrstuvwxyz" "AIOQSTWY" "ɑɐɒæβɔɕçɖðʤəɚɛɜɟɡɥɨɪʝɯɰŋɳɲɴøɸθœɹɾɻʁɽʂʃʈʧʊʋʌɣɤχʎʒʔ"
       "ˈˌːʰʲ↓→↗↘ᵻ" "̃ʣʥʦʨᵝꭧᵊ")
OUTSIDE = "XZ0123456789ɫ★é"
MARKS = ".!?,:;"


def _string(rng: random.Random, n: int, marks: bool, spaces: bool, outside: float) -> str:
    s = []
    while len(s) < n:
        r = rng.random()
        if marks and r < 0.03:
            s.append(rng.choice(MARKS))
        elif spaces and r < 0.18:
            s.append(" ")
        elif r < 0.18 + outside:
            s.append(rng.choice(OUTSIDE))
        else:
            s.append(rng.choice(IPA))
    return "".join(s[:n])


def cases() -> list[str]:
    rng = random.Random(20261202)
    out = ["", "a", "həlˈoʊ wˈɜːld.", "ˈ" * 510, "ɑ" * 511, "x" * 1021]
    for n in (5, 60, 200, 509, 510, 511, 512, 700, 1100, 1600, 2600):
        out.append(_string(rng, n, True, True, 0.02))
    for n in (600, 1300):
        out.append(_string(rng, n, False, True, 0.0))   # no sentence or clause marks: split at spaces
        out.append(_string(rng, n, False, False, 0.0))  # none at all: hard split at 510 code points
    # a sentence mark right at the 510th code point, and one just past it
    base = _string(rng, 700, False, True, 0.0)
    out.append(base[:509] + "." + base[510:])
    out.append(base[:510] + "!" + base[511:])
    out.append(base[:300] + "," + base[301:])
    return out


def run(reference: str, inputs: list[str]) -> list[list]:
    src = os.path.join(reference, "src")
    with tempfile.TemporaryDirectory() as d:
        cu = os.path.join(d, "ipa_tokens.cu")
        exe = os.path.join(d, "ipa_tokens")
        with open(cu, "w") as f:
            f.write(PROGRAM)
        nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
        subprocess.run([nvcc, "-std=c++17", "-O1", "-ccbin", "/usr/bin/g++", "-I", src, cu, "-o", exe], check=True,
                       capture_output=True)
        text = "\n".join(inputs) + "\n"
        out = subprocess.run([exe], input=text.encode("utf-8"), check=True, capture_output=True).stdout.decode()
    rows = []
    for line in out.splitlines():
        parts = line.split(" | ")
        chunks = []
        for p in parts[1:]:
            v = [int(x) for x in p.split()]
            chunks.append({"bytes": v[0], "tokens": v[2:2 + v[1]]})
        assert len(chunks) == int(parts[0])
        rows.append(chunks)
    assert len(rows) == len(inputs)
    return rows


def main(reference: str) -> None:
    inputs = cases()
    rows = run(reference, inputs)
    with open(os.path.join(HERE, "ipa_tokens.json"), "w") as f:
        json.dump({"source": "rokoko::chunk_ipa / to_tokens, src/rokoko.h:141-221",
                   "cases": [{"ipa": s, "chunks": c} for s, c in zip(inputs, rows)]}, f, ensure_ascii=False)
        f.write("\n")
    print(f"{len(inputs)} cases written")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_ipa_tokens.py <reference checkout>")
    main(sys.argv[1])
