"""tcgen05 implicit-GEMM conv (rk_conv1d_fprop) vs a float64 torch conv1d.

Tolerances: split-bf16 (FP32 semantics) relative L2 <= 2e-5; fp16 mode
compares against the float64 conv of the fp16-rounded operands, <= 2e-5.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

CASES = [
    # C_in, C_out, T_in, K, stride, pad, dil, residual
    (128, 128, 1000, 3, 1, 1, 1, False),
    (128, 128, 777, 11, 1, 25, 5, True),
    (256, 256, 300, 7, 1, 9, 3, False),
    (514, 1024, 400, 3, 1, 1, 1, False),
    (1090, 512, 130, 3, 1, 1, 1, True),
    (22, 256, 4801, 12, 6, 3, 1, False),
    (128, 22, 901, 7, 1, 3, 1, False),
    (512, 64, 400, 1, 1, 0, 1, False),
    (22, 128, 333, 1, 1, 0, 1, False),
    (768, 2048, 66, 1, 1, 0, 1, False),
    # more tiles than SMs: each persistent CTA runs several tiles through both accumulators
    (128, 128, 48001, 7, 1, 9, 3, True),
    (128, 128, 100000, 3, 1, 1, 1, False),
    # long launches (256-row tiles where the ring fits): widest halo (K 11, dilation 5),
    # partial last tiles, bias and residual epilogues
    (128, 128, 48001, 11, 1, 25, 5, False),
    (256, 256, 8000, 11, 1, 25, 5, True),
    (256, 256, 5000, 3, 1, 1, 1, False),
    (128, 128, 4104, 7, 1, 3, 1, True),
]


def _run(rk_lib, C_in, C_out, T_in, K, stride, pad, dil, residual, precision):
    from rokoko_b200 import lib
    g = torch.Generator().manual_seed(C_in * 7 + K)
    x = torch.randn(T_in, C_in, generator=g)
    w = torch.randn(C_out, C_in, K, generator=g) * (1.0 / np.sqrt(C_in * K))
    b = torch.randn(C_out, generator=g)
    T_out = (T_in + 2 * pad - dil * (K - 1) - 1) // stride + 1
    r = torch.randn(T_out, C_out, generator=g) if residual else None
    if precision == lib.RK_PRECISION_FP16:
        xq, wq = x.half().double(), w.half().double()
    else:
        xq, wq = x.double(), w.double()
    ref = torch.nn.functional.conv1d(xq.t()[None], wq, None, stride, pad, dil)[0].t()
    ref = ref + (r.double() if residual else b.double())
    dev = torch.device("cuda:0")
    xd = x.to(dev).contiguous()
    wd = w.permute(0, 2, 1).contiguous().to(dev)  # NHWC [C_out, K, C_in]
    bd = b.to(dev)
    rd = r.to(dev).contiguous() if residual else None
    yd = torch.full((T_out, C_out), float("nan"), device=dev)
    ws_bytes = rk_lib.rk_conv1d_workspace_size(C_in, C_out, T_in, K, stride, pad, dil, precision)
    assert ws_bytes > 0
    ws = torch.empty(ws_bytes + 256, dtype=torch.uint8, device=dev)
    ws_ptr = (ws.data_ptr() + 255) // 256 * 256
    st = torch.cuda.current_stream().cuda_stream
    rc = rk_lib.rk_conv1d_fprop(xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), yd.data_ptr(),
                                rd.data_ptr() if residual else None, ws_ptr, ws_bytes, C_in, C_out, T_in, K,
                                stride, pad, dil, precision, st)
    lib.check(rc, "rk_conv1d_fprop")
    lib.check(rk_lib.rk_conv1d_check(ws_ptr, st), "rk_conv1d_check")
    y = yd.double().cpu()
    rel = float((y - ref).norm() / ref.norm())
    return rel, y, ref


@pytest.mark.parametrize("case", CASES, ids=[f"ci{c[0]}_co{c[1]}_t{c[2]}_k{c[3]}_s{c[4]}_d{c[6]}" for c in CASES])
@pytest.mark.parametrize("precision", [0, 1], ids=["split", "fp16"])
def test_conv_matches_fp64(rk_lib, case, precision):
    rel, y, ref = _run(rk_lib, *case, precision)
    assert np.isfinite(y.numpy()).all()
    assert rel < 2e-5, rel


SEAM_CASES = [
    # C_in, C_out, T_in, K, stride, pad, dil, residual: shapes of the reference's callers
    (128, 128, 4801, 7, 1, 9, 3, True),
    (22, 256, 4801, 12, 6, 3, 1, False),
    (520, 1024, 130, 3, 1, 1, 1, False),   # C_in % 8 == 0 as the reference's fp16 path requires
]


@pytest.mark.parametrize("case", SEAM_CASES, ids=[f"ci{c[0]}_co{c[1]}_k{c[3]}_s{c[4]}" for c in SEAM_CASES])
def test_reference_signature_seams(rk_lib, case):
    """rk_conv1d_fprop_f32 / _f16 take cutlass_conv1d_fprop[_f16]'s argument
    list (no precision argument; half x and w for _f16).  _f32 is the same
    kernel sequence as rk_conv1d_fprop in FP32 semantics, so the outputs are
    bit-identical; _f16 is checked against the float64 conv of the half
    operands (fp16 products are exact in FP32, the sum is FP32)."""
    from rokoko_b200 import lib
    C_in, C_out, T_in, K, stride, pad, dil, residual = case
    g = torch.Generator().manual_seed(C_in + 31 * K)
    x = torch.randn(T_in, C_in, generator=g)
    w = torch.randn(C_out, C_in, K, generator=g) * (1.0 / np.sqrt(C_in * K))
    b = torch.randn(C_out, generator=g)
    T_out = (T_in + 2 * pad - dil * (K - 1) - 1) // stride + 1
    r = torch.randn(T_out, C_out, generator=g) if residual else None
    dev = torch.device("cuda:0")
    st = torch.cuda.current_stream().cuda_stream
    xd, wd, bd = x.to(dev), w.permute(0, 2, 1).contiguous().to(dev), b.to(dev)
    rd = r.to(dev) if residual else None
    rp = rd.data_ptr() if residual else None
    need = rk_lib.rk_conv1d_workspace_bytes(C_in, C_out, T_in, K, stride, pad, dil)
    assert need >= rk_lib.rk_conv1d_workspace_size(C_in, C_out, T_in, K, stride, pad, dil, 1) > 0
    ws = torch.empty(need + 256, dtype=torch.uint8, device=dev)
    wp = (ws.data_ptr() + 255) // 256 * 256
    y_a = torch.full((T_out, C_out), float("nan"), device=dev)
    y_b = torch.full((T_out, C_out), float("nan"), device=dev)
    lib.check(rk_lib.rk_conv1d_fprop(xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), y_a.data_ptr(), rp, wp, need,
                                     C_in, C_out, T_in, K, stride, pad, dil, lib.RK_PRECISION_FP32, st),
              "rk_conv1d_fprop")
    lib.check(rk_lib.rk_conv1d_fprop_f32(xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), y_b.data_ptr(), rp, wp, need,
                                         C_in, C_out, T_in, K, stride, pad, dil, st), "rk_conv1d_fprop_f32")
    lib.check(rk_lib.rk_conv1d_check(wp, st), "rk_conv1d_check")
    assert torch.equal(y_a, y_b)
    # fp16 seam: half operands in device memory
    xh, wh = xd.half(), wd.half()
    y_h = torch.full((T_out, C_out), float("nan"), device=dev)
    lib.check(rk_lib.rk_conv1d_fprop_f16(xh.data_ptr(), wh.data_ptr(), bd.data_ptr(), y_h.data_ptr(), rp, wp, need,
                                         C_in, C_out, T_in, K, stride, pad, dil, st), "rk_conv1d_fprop_f16")
    lib.check(rk_lib.rk_conv1d_check(wp, st), "rk_conv1d_check")
    ref = torch.nn.functional.conv1d(x.half().double().t()[None], w.half().double(), None, stride, pad, dil)[0].t()
    ref = ref + (r.double() if residual else b.double())
    y = y_h.double().cpu()
    rel = float((y - ref).norm() / ref.norm())
    assert rel < 2e-5, rel
