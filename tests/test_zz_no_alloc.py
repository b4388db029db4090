"""rk_conv1d_fprop_static: the convolution entry point that allocates nothing.

It serves callers that cannot allocate device memory where they need a
convolution (a host whose device memory comes from its own pool, a thread that
must not block on the allocator, a fixed plugin budget).  Its scratch lives in
one library-owned device array, so these tests check that (1) two calls in a
row through the C ABI give the same result as rk_conv1d_fprop with a
caller-provided workspace (the same kernels with the same tiling, so bit for
bit, which is inside the 2e-5 tolerance of the other conv tests), and that
rk_conv1d_static_check then reports a clean error word, and (2) a shape larger
than the array is rejected with RK_ERR_WORKSPACE without touching the output.

This file is named so that pytest collects it last.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

TOL = 2e-5  # relative L2, as in tests/test_conv_gpu.py


def _conv_inputs(seed, C_in, C_out, T_in, K, residual):
    g = torch.Generator().manual_seed(seed)
    dev = torch.device("cuda:0")
    x = torch.randn(T_in, C_in, generator=g).to(dev)
    w = (torch.randn(C_out, K, C_in, generator=g) * (1.0 / np.sqrt(C_in * K))).to(dev)  # NHWC
    b = torch.randn(C_out, generator=g).to(dev)
    r = torch.randn(T_in, C_out, generator=g).to(dev) if residual else None
    return x, w, b, r


def test_static_scratch_matches_workspace_entry(rk_lib):
    from rokoko_b200 import lib
    dev = torch.device("cuda:0")
    st = torch.cuda.current_stream().cuda_stream
    cases = [  # C_in, C_out, T_in, K, dil, precision, residual (pad keeps T_out = T_in)
        (128, 128, 4000, 7, 3, lib.RK_PRECISION_FP32, True),
        (256, 128, 2500, 3, 1, lib.RK_PRECISION_FP16, False),
    ]
    for seed, (C_in, C_out, T_in, K, dil, prec, res) in enumerate(cases):  # two calls in a row
        pad = dil * (K - 1) // 2
        x, w, b, r = _conv_inputs(seed, C_in, C_out, T_in, K, res)
        need = rk_lib.rk_conv1d_workspace_size(C_in, C_out, T_in, K, 1, pad, dil, prec)
        assert 0 < need <= lib.RK_CONV_STATIC_SCRATCH_BYTES
        ws = torch.empty(need + 256, dtype=torch.uint8, device=dev)
        wp = (ws.data_ptr() + 255) // 256 * 256
        y_ws = torch.full((T_in, C_out), float("nan"), device=dev)
        y_st = torch.full((T_in, C_out), float("nan"), device=dev)
        rp = r.data_ptr() if r is not None else None
        lib.check(rk_lib.rk_conv1d_fprop(x.data_ptr(), w.data_ptr(), b.data_ptr(), y_ws.data_ptr(), rp, wp, need,
                                         C_in, C_out, T_in, K, 1, pad, dil, prec, st), "rk_conv1d_fprop")
        lib.check(rk_lib.rk_conv1d_fprop_static(x.data_ptr(), w.data_ptr(), b.data_ptr(), y_st.data_ptr(), rp,
                                                C_in, C_out, T_in, K, 1, pad, dil, prec, st),
                  "rk_conv1d_fprop_static")
        torch.cuda.synchronize()
        lib.check(rk_lib.rk_conv1d_static_check(st), "rk_conv1d_static_check")
        lib.check(rk_lib.rk_conv1d_check(wp, st), "rk_conv1d_check")
        a, e = y_st.double().cpu(), y_ws.double().cpu()
        assert torch.isfinite(a).all()
        rel = float((a - e).norm() / e.norm())
        assert rel <= TOL, (seed, rel)
        assert torch.equal(y_st, y_ws), seed


def test_static_scratch_rejects_oversize(rk_lib):
    from rokoko_b200 import lib
    dev = torch.device("cuda:0")
    C, T, K = 128, 200000, 3  # about 100 MB of split-bf16 operand planes
    assert rk_lib.rk_conv1d_workspace_size(C, C, T, K, 1, 1, 1, lib.RK_PRECISION_FP32) > \
        lib.RK_CONV_STATIC_SCRATCH_BYTES
    x = torch.zeros(T, C, device=dev)
    w = torch.zeros(C, K, C, device=dev)
    y = torch.full((T, C), 7.0, device=dev)
    rc = rk_lib.rk_conv1d_fprop_static(x.data_ptr(), w.data_ptr(), None, y.data_ptr(), None, C, C, T, K, 1, 1, 1,
                                       lib.RK_PRECISION_FP32, torch.cuda.current_stream().cuda_stream)
    assert rc == lib.RK_ERR_WORKSPACE
    assert b"RK_CONV_STATIC_SCRATCH_BYTES" in rk_lib.rk_last_error()
    torch.cuda.synchronize()
    assert bool((y == 7.0).all())


def test_error_word_is_reported_and_cleared(rk_lib):
    """The conv error word (the first 4 bytes of a workspace, and of the static
    scratch array that rk_conv1d_static_check reads the same way): a code that a
    bounded device wait left there is reported once as RK_ERR_DEVICE_TIMEOUT and
    cleared.  The code is planted by the test (no wait is made to run out)."""
    from rokoko_b200 import lib
    dev = torch.device("cuda:0")
    st = torch.cuda.current_stream().cuda_stream
    ws = torch.zeros(256, dtype=torch.int32, device=dev)
    ws[0] = 2  # RK_DEV_TIMEOUT_EMPTY
    torch.cuda.synchronize()
    assert rk_lib.rk_conv1d_check(ws.data_ptr(), st) == lib.RK_ERR_DEVICE_TIMEOUT
    assert int(ws[0].item()) == 0
    assert rk_lib.rk_conv1d_check(ws.data_ptr(), st) == lib.RK_OK
    assert rk_lib.rk_conv1d_static_check(st) == lib.RK_OK
