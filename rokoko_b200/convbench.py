"""Micro-benchmark of the stateless conv seam (rk_conv1d_fprop) on one shape.

    python -m rokoko_b200.convbench --cin 128 --cout 128 --T 48001 --K 7 --dil 3 [--residual] [--fp16] [--repeat 3]

Runs the tcgen05 convolution through the C ABI on seeded random device data
(weights NHWC [C_out, K, C_in], padding dil*(K-1)/2) `repeat` times and prints
the best CUDA-event time per call (operand packing included) and the
algorithmic TFLOP/s (2 C_in C_out K T_out).  It is the command the conv ncu
captures under profiles/ run.
"""
from __future__ import annotations

import argparse
import sys


def _conv_bench(a) -> int:
    import torch

    from . import lib
    L = lib.load()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(a.T, a.cin, device=dev, generator=g)
    w = torch.randn(a.cout, a.K, a.cin, device=dev, generator=g) * (a.cin * a.K) ** -0.5
    b = torch.randn(a.cout, device=dev, generator=g)
    pad = a.dil * (a.K - 1) // 2
    T_out = a.T + 2 * pad - a.dil * (a.K - 1)
    y = torch.empty(T_out, a.cout, device=dev)
    r = torch.randn(T_out, a.cout, device=dev, generator=g) if a.residual else None
    prec = lib.RK_PRECISION_FP16 if a.fp16 else lib.RK_PRECISION_FP32
    nbytes = L.rk_conv1d_workspace_size(a.cin, a.cout, a.T, a.K, 1, pad, a.dil, prec)
    ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)
    wp = (ws.data_ptr() + 255) // 256 * 256
    st = torch.cuda.current_stream().cuda_stream
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * a.repeat)]
    for i in range(a.repeat):
        ev[2 * i].record()
        lib.check(L.rk_conv1d_fprop(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(),
                                    r.data_ptr() if r is not None else None, wp, nbytes, a.cin, a.cout, a.T, a.K,
                                    1, pad, a.dil, prec, st), "rk_conv1d_fprop")
        ev[2 * i + 1].record()
    lib.check(L.rk_conv1d_check(wp, st), "rk_conv1d_check")
    ms = min(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(a.repeat))
    fl = 2.0 * a.cin * a.cout * a.K * T_out
    print(f"conv C_in={a.cin} C_out={a.cout} T={a.T} K={a.K} dil={a.dil}: {ms * 1e3:.1f} us incl. operand packing, "
          f"{fl / ms / 1e9:.1f} TFLOP/s algorithmic", file=sys.stderr)
    return 0


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="rokoko_b200.convbench")
    p.add_argument("--cin", type=int, default=128)
    p.add_argument("--cout", type=int, default=128)
    p.add_argument("--T", type=int, default=48001)
    p.add_argument("--K", type=int, default=7)
    p.add_argument("--dil", type=int, default=1)
    p.add_argument("--residual", action="store_true")
    p.add_argument("--fp16", action="store_true")
    p.add_argument("--repeat", type=int, default=3)
    return _conv_bench(p.parse_args(argv))


if __name__ == "__main__":
    sys.exit(main())
