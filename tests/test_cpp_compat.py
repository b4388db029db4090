"""The reference's C++ model seam (rokoko::Weights / GpuArena / rokoko_infer /
precompute_weight_norms / compute_decode_bytes / write_wav, its src/weights.h)
implemented by librokoko_compat.so over the C ABI.  tests/cpp/rokoko_infer_main.cpp
is a caller written against that seam; it is compiled here with g++ against
include/rokoko/weights.h and, on a GPU, must produce exactly the PCM that
rk_infer gives for the same tokens and style (the same kernels underneath)."""
import os
import subprocess
import tempfile

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "rokoko_b200")
CUDA = "/usr/local/cuda"


def _compile_src(out_dir: str, name: str) -> str:
    """g++ tests/cpp/<name>.cpp against include/rokoko and the compat library."""
    exe = os.path.join(out_dir, name)
    cmd = ["/usr/bin/g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include", "rokoko"),
           "-I", os.path.join(CUDA, "include"), os.path.join(ROOT, "tests", "cpp", name + ".cpp"),
           "-o", exe, "-L", PKG, "-lrokoko_compat", "-lrokoko_b200", "-L", os.path.join(CUDA, "lib64"),
           "-lcudart_static", "-ldl", "-lpthread", "-lrt", f"-Wl,-rpath,{PKG}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def _compile(out_dir: str) -> str:
    return _compile_src(out_dir, "rokoko_infer_main")


def test_compat_library_exports_the_reference_seam():
    lib = os.path.join(PKG, "librokoko_compat.so")
    assert os.path.exists(lib), "run python -m rokoko_b200.build"
    syms = subprocess.run(["nm", "-DC", lib], check=True, capture_output=True, text=True).stdout
    for name in ("rokoko::rokoko_infer(rokoko::Weights const&, int const*, int, float const*, CUstream_st*, "
                 "rokoko::GpuArena&, rokoko::GpuArena&, float*, unsigned long)",
                 "rokoko::Weights::load(", "rokoko::precompute_weight_norms(rokoko::Weights&, CUstream_st*)",
                 "rokoko::compute_decode_bytes(int, int)", "rokoko::write_wav("):
        assert name in syms, name
    with tempfile.TemporaryDirectory() as d:
        assert os.path.exists(_compile(d))


@pytest.mark.gpu
def test_cpp_rokoko_infer_matches_rk_infer(v1_blob):
    from rokoko_b200 import configs, convert_v2
    from rokoko_b200.context import FP16, FP32, Context
    u = configs.config0(seed=21, n_phon=24)
    with tempfile.TemporaryDirectory() as d:
        exe = _compile(d)
        tok, sty = os.path.join(d, "tok.i32"), os.path.join(d, "style.f32")
        u.tokens.astype(np.int32).tofile(tok)
        u.style.astype(np.float32).tofile(sty)
        for blob, prec in ((v1_blob, FP32), (convert_v2.convert_blob(v1_blob), FP16)):
            wpath, out, wav = os.path.join(d, "w.bin"), os.path.join(d, "pcm.f32"), os.path.join(d, "out.wav")
            with open(wpath, "wb") as f:
                f.write(blob)
            subprocess.run([exe, wpath, tok, sty, out, wav], check=True, timeout=600)
            pcm = np.fromfile(out, np.float32)
            with Context(0, prec) as ctx:
                ctx.load_weights(blob)
                ref, _, L = ctx.infer(u.tokens, u.style)
            assert pcm.shape == ref.shape == (600 * L,)
            assert np.array_equal(pcm, ref)
            assert os.path.getsize(wav) == 44 + 2 * pcm.shape[0]
