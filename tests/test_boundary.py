"""The C-ABI library loads and exports every entry point include/rk_b200.h
declares (no compute calls: this runs without a GPU)."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "rk_b200.h")).read()
    return sorted(set(re.findall(r"RK_API\s+[\w\s\*]+?\b(rk_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    for must in ("rk_create", "rk_destroy", "rk_load_weights_koko", "rk_infer", "rk_decode_features",
                 "rk_conv1d_fprop", "rk_conv1d_workspace_size", "rk_compute_decode_bytes"):
        assert must in names


def test_library_exports_every_declared_symbol(rk_lib):
    from rokoko_b200 import lib
    exported = set(lib.exported_symbols())
    missing = [n for n in declared_symbols() if n not in exported]
    # every declared name must also have a ctypes signature
    sig = {n for n, _, _ in lib.SIGNATURES}
    assert not [n for n in declared_symbols() if n not in sig], "signature table incomplete"
    assert not missing, missing


def test_status_strings_and_sizes_without_gpu(rk_lib):
    assert rk_lib.rk_status_string(0) == b"ok"
    assert rk_lib.rk_status_string(-2) == b"workspace too small"
    # pure host arithmetic: the reference's decode-arena formula (src/rokoko_common.h:160-229)
    assert rk_lib.rk_compute_decode_bytes(66, 352) > 0
    # workspace planning for the conv seam (host only)
    assert rk_lib.rk_conv1d_workspace_size(128, 128, 1000, 3, 1, 1, 1, 0) > 0
    assert rk_lib.rk_conv1d_workspace_size(128, 128, 1000, 3, 2, 1, 2, 0) == 0  # stride with dilation unsupported
