"""Backward benchmark of ComplexConv2d: the data gradient and the weight
gradient that ``forward()``'s autograd node runs, timed with one CUDA-event
pair around ``iters`` back-to-back calls after ``warmup`` calls (the
methodology of benchmark_conv2d.py).  Effective TFLOP/s count 8*N*P*Q*K*C*R*S
per gradient (the forward's flops); frac is of the dense TF32 peak
(measured bf16 cuBLAS / 2).  The reference has no backward (its README lists
it as absent), so there is no reference column.

    python cutlass-complex-conv_b200/benchmarks/benchmark_backward.py [--batch 64] [--only wgrad]
    python .../benchmark_backward.py --batch 8 --only wgrad --iters 2 --warmup 1   # ncu-sized
"""

import argparse
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import torch  # noqa: E402

from complex_conv2d import ComplexConv2d, _C  # noqa: E402

LAYERS = {
    "56": (128, 128, 56, 3, 1, 1),     # 128->128 @ 56x56, 3x3, s1 p1
    "s2": (64, 128, 112, 3, 2, 1),     # 3x3 stride-2 64->128 @ 112x112
    "1x1": (256, 1024, 28, 1, 1, 0),   # 1x1 256->1024 @ 28x28
}


def peak_tflops():
    path = os.path.join(os.path.dirname(os.path.dirname(HERE)), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f)["bf16_tflops"] / 2.0
    except (OSError, KeyError, ValueError):
        return 1590.0 / 2.0


def time_calls(fn, iters, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters / 1e3


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--layer", choices=sorted(LAYERS), default="56")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--only", choices=["dgrad", "wgrad"], default=None)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    args = ap.parse_args()
    c, k, hw, r, st, pd = LAYERS[args.layer]
    n = args.batch
    torch.manual_seed(0)
    layer = ComplexConv2d(c, k, r, st, pd).cuda()
    x = torch.complex(torch.randn(n, c, hw, hw), torch.randn(n, c, hw, hw)).cuda()
    with torch.no_grad():
        y = layer(x)
    dy = torch.complex(torch.randn(y.shape), torch.randn(y.shape)).cuda()
    p, q = y.shape[2], y.shape[3]
    flops = 8 * n * p * q * k * c * r * r
    peak = peak_tflops()
    runs = {"dgrad": lambda: layer._data_grad(dy, hw, hw),
            "wgrad": lambda: _C.wgrad_complex(x, dy, r, r, st, st, pd, pd)}
    for name, fn in runs.items():
        if args.only and name != args.only:
            continue
        t = time_calls(fn, args.iters, args.warmup)
        tf = flops / t / 1e12
        print(f"{args.layer} b{n} {name}: {t * 1e6:.1f} us  {tf:.0f} TFLOP/s  {tf / peak:.3f} of "
              f"the TF32 peak", flush=True)


if __name__ == "__main__":
    main()
