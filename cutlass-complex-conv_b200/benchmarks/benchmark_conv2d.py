"""Per-shape benchmark table, the methodology of the reference harness
(benchmarks/benchmark_conv2d.py:36-53,82-178 of cutlass-complex-conv):
warmup, then one CUDA-event pair around ``iters`` back-to-back calls, for the
GPU four-real-Conv2d baseline (cuDNN), ``forward()`` and ``forward_planar()``,
after a correctness gate (allclose 1e-3 against the four-conv baseline).

Adds, per case: effective TFLOP/s, the fraction of the dense TF32 peak
(measured bf16 cuBLAS / 2), algorithmic GB/s, and a CUDA-graph replay of
``forward_planar`` (launch overhead removed) for the launch-bound batch-1
shapes.

    python cutlass-complex-conv_b200/benchmarks/benchmark_conv2d.py [--cases a,b] [--json]
    python .../benchmark_conv2d.py --cases b64_128_128_56 --only planar --iters 1 --warmup 1
    python .../benchmark_conv2d.py --cases b64_128_128_56 --only forward --iters 2 --warmup 1
"""

import argparse
import json
import os
import sys
from dataclasses import dataclass

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import torch  # noqa: E402
import torch.nn as nn  # noqa: E402

from complex_conv2d import ComplexConv2d  # noqa: E402


@dataclass(frozen=True)
class BenchmarkCase:
    name: str
    n: int
    c: int
    h: int
    w: int
    k: int
    r: int
    s: int
    stride: int = 1
    padding: int = 1
    input_std: float = 1.0

    @property
    def pq(self):
        p = (self.h + 2 * self.padding - self.r) // self.stride + 1
        q = (self.w + 2 * self.padding - self.s) // self.stride + 1
        return p, q

    @property
    def flops(self):
        p, q = self.pq
        return 8 * self.n * p * q * self.k * self.c * self.r * self.s

    @property
    def alg_bytes(self):
        p, q = self.pq
        return 8 * (self.n * self.h * self.w * self.c + self.k * self.r * self.s * self.c
                    + self.n * p * q * self.k)


CASES = [
    # The reference's DEFAULT_CASES (benchmark_conv2d.py:27-33): batch 1, 3x3, s1 p1.
    BenchmarkCase("conv_32_32", 1, 32, 32, 32, 32, 3, 3),
    BenchmarkCase("b1_32_64_56", 1, 32, 56, 56, 64, 3, 3),
    BenchmarkCase("b1_64_128_28", 1, 64, 28, 28, 128, 3, 3),
    BenchmarkCase("b1_128_256_14", 1, 128, 14, 14, 256, 3, 3),
    BenchmarkCase("b1_256_512_7", 1, 256, 7, 7, 512, 3, 3),
    # Batched configs of the north star.
    BenchmarkCase("b64_128_128_56", 64, 128, 56, 56, 128, 3, 3),
    BenchmarkCase("b32_s2_64_128_112", 32, 64, 112, 112, 128, 3, 3, 2, 1),
    BenchmarkCase("b32_1x1_256_1024_28", 32, 256, 28, 28, 1024, 1, 1, 1, 0),
    BenchmarkCase("b32_64_64_320", 32, 64, 320, 320, 64, 3, 3, 1, 1, 0.1),
]
# Not in the default run: one GPU's share of the MRI config at 4 GPUs (a
# profiling-sized case of the same kernel).
EXTRA_CASES = [
    BenchmarkCase("b8_64_64_320", 8, 64, 320, 320, 64, 3, 3, 1, 1, 0.1),
]


class FourConv(nn.Module):
    """GPU four-real-Conv2d baseline (benchmarks/baseline.py:5-45)."""

    def __init__(self, case):
        super().__init__()
        kw = dict(stride=case.stride, padding=case.padding, bias=False)
        self.conv_real = nn.Conv2d(case.c, case.k, (case.r, case.s), **kw)
        self.conv_imag = nn.Conv2d(case.c, case.k, (case.r, case.s), **kw)

    def forward(self, x):
        return ((self.conv_real(x.real) - self.conv_imag(x.imag)).to(torch.complex64)
                + 1j * (self.conv_real(x.imag) + self.conv_imag(x.real)).to(torch.complex64))


def benchmark_cuda(fn, warmup, iters):
    with torch.no_grad():
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(iters):
            fn()
        end.record()
        torch.cuda.synchronize()
    return start.elapsed_time(end) / iters


def benchmark_graph(fn, warmup, iters):
    """Replay ``fn`` captured in a CUDA graph (launch overhead removed)."""
    with torch.no_grad():
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return benchmark_cuda(g.replay, warmup, iters)


def tf32_peak():
    try:
        with open(os.path.join(os.path.dirname(os.path.dirname(HERE)), "MEASURED_PEAKS.json")) as f:
            return json.load(f)["bf16_tflops"] / 2.0
    except Exception:
        return 1590.0 / 2.0


def run_case(case, device, warmup, iters, only, precision):
    torch.manual_seed(0)
    base = FourConv(case).to(device).eval()
    mod = ComplexConv2d(case.c, case.k, (case.r, case.s), stride=case.stride,
                        padding=case.padding, device=device, precision=precision).eval()
    with torch.no_grad():
        mod.weight_real.copy_(base.conv_real.weight)
        mod.weight_imag.copy_(base.conv_imag.weight)
    g = torch.Generator(device=device).manual_seed(0)
    x = torch.complex(torch.randn(case.n, case.c, case.h, case.w, generator=g, device=device),
                      torch.randn(case.n, case.c, case.h, case.w, generator=g, device=device))
    x = x * case.input_std
    xr = x.real.permute(0, 2, 3, 1).contiguous()
    xi = x.imag.permute(0, 2, 3, 1).contiguous()
    res = {"case": case.name, "gflop": case.flops / 1e9}
    if only in ("all", "planar"):
        res["planar_ms"] = benchmark_cuda(lambda: mod.forward_planar(xr, xi), warmup, iters)
    if only == "planar":
        return res
    with torch.no_grad():
        y_ref = base(x)
        y = mod(x)
    err = (y - y_ref).abs().max().item()
    close = torch.allclose(y, y_ref, atol=1e-3 * max(1.0, case.input_std * 10), rtol=1e-3)
    if not close:
        raise RuntimeError(f"{case.name}: correctness check failed (max_error={err:.3e})")
    res["max_error"] = err
    if only == "forward":
        res["forward_ms"] = benchmark_cuda(lambda: mod(x), warmup, iters)
        res["tflops_forward"] = case.flops / (res["forward_ms"] * 1e-3) / 1e12
        return res
    res["baseline_ms"] = benchmark_cuda(lambda: base(x), warmup, iters)
    res["forward_ms"] = benchmark_cuda(lambda: mod(x), warmup, iters)
    if case.n == 1:
        res["planar_graph_ms"] = benchmark_graph(lambda: mod.forward_planar(xr, xi), warmup, iters)
        res["forward_graph_ms"] = benchmark_graph(lambda: mod(x), warmup, iters)
    peak = tf32_peak()
    best = min(v for k2, v in res.items() if k2.endswith("_ms") and k2 != "baseline_ms")
    res["tflops_planar"] = case.flops / (res["planar_ms"] * 1e-3) / 1e12
    res["tflops_forward"] = case.flops / (res["forward_ms"] * 1e-3) / 1e12
    res["frac_tf32_peak_best"] = case.flops / (best * 1e-3) / 1e12 / peak
    res["gbs_forward"] = case.alg_bytes / (res["forward_ms"] * 1e-3) / 1e9
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--warmup", type=int, default=30)
    ap.add_argument("--iters", type=int, default=200)
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--cases", default="all")
    ap.add_argument("--only", choices=["all", "planar", "forward"], default="all")
    ap.add_argument("--precision", default="tf32")
    ap.add_argument("--json", action="store_true")
    args = ap.parse_args()
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is required to run this benchmark")
    cases = (CASES if args.cases == "all"
             else [c for c in CASES + EXTRA_CASES if c.name in args.cases.split(",")])
    print("PyTorch :", torch.__version__, "| GPU:", torch.cuda.get_device_name(args.device),
          "| TF32 peak (measured bf16/2):", tf32_peak(), "TFLOP/s")
    for case in cases:
        it = args.iters if case.flops < 20e9 else max(1, args.iters // 10)
        res = run_case(case, torch.device(args.device), args.warmup, it, args.only, args.precision)
        if args.json:
            print(json.dumps(res), flush=True)
        else:
            print("  ".join(f"{k}={v:.4g}" if isinstance(v, float) else f"{k}={v}"
                            for k, v in res.items()), flush=True)


if __name__ == "__main__":
    main()
