"""Benchmark of the B200 complex Conv2d forward (one JSON line on rank 0).

Workload (default): BASELINE configs[2], the batched compute-bound layer
    batch 64, Cin = Cout = 128, 56x56, 3x3, stride 1, pad 1, complex64,
    inputs iid N(0,1) per part, weights U(+-1/sqrt(1152)).
The global batch of 64 is split across ranks (one process per GPU, weights
replicated, no collective on the data path): strong scaling.

A step is one ``ComplexConv2d.forward`` call (complex64 NCHW in, complex64
NCHW out) over the rank's batch slice.  ``value`` is the whole-job effective
TFLOP/s (8 flops per complex MAC) with inputs resident in HBM; each rank's
input (>= 25 MB per GPU at 8 GPUs, 205 MB at 1 GPU) and output stream through
L2 every step.  ``e2e`` times the public host-buffer call
``ComplexConv2d.forward_host`` (the same forward, with every step's input
copied in from pinned host memory and its output copied back, chunks of images
pipelined over the two copy directions); ``e2e.serial_ms_per_step`` is the
plain copy-in, ``forward``, copy-out sequence for comparison.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME] [--precision tf32|3xtf32]

``--impl reference`` times the reference's four-real-Conv2d path
(benchmarks/baseline.py:5-45) on the host CPU, restated in oracle/, on a
bounded sample of the same workload (rank 0 only).
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.join(ROOT, "cutlass-complex-conv_b200")
for _p in (ROOT, PKG_ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "complex-conv ms/call & effective TFLOP/s (8·MACs) vs TF32 peak, 1/2/4/8 GPU"
UNIT = "TFLOP/s"

# name: (N, C, H, W, K, R, S, stride, pad, input_std)
WORKLOADS = {
    "b64_128_128_56": (64, 128, 56, 56, 128, 3, 3, 1, 1, 1.0),
    "b32_s2_64_128_112": (32, 64, 112, 112, 128, 3, 3, 2, 1, 1.0),
    "b32_1x1_256_1024_28": (32, 256, 28, 28, 1024, 1, 1, 1, 0, 1.0),
    "b32_64_64_320": (32, 64, 320, 320, 64, 3, 3, 1, 1, 0.1),
    "b1_32_64_56": (1, 32, 56, 56, 64, 3, 3, 1, 1, 1.0),
    "b1_64_128_28": (1, 64, 28, 28, 128, 3, 3, 1, 1, 1.0),
    "b1_128_256_14": (1, 128, 14, 14, 256, 3, 3, 1, 1, 1.0),
    "b1_256_512_7": (1, 256, 7, 7, 512, 3, 3, 1, 1, 1.0),
}
DEFAULT_WORKLOAD = "b64_128_128_56"


def out_hw(h, w, r, s, stride, pad):
    return (h + 2 * pad - r) // stride + 1, (w + 2 * pad - s) // stride + 1


def workload_flops(n, c, h, w, k, r, s, stride, pad):
    p, q = out_hw(h, w, r, s, stride, pad)
    return 8 * n * p * q * k * c * r * s


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                "source": "fallback"}


def profiled_traffic(kernel, workload):
    """DRAM bytes per launch from a committed ncu summary, if one exists."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_{workload}.txt")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.idx = device_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="ccv_clocks_", suffix=".csv")
            os.close(fd)
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"],
                    "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.close()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 8:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                except ValueError:
                    continue
                for nm, v in zip(names, parts[4:8]):
                    if v.lower().startswith("active"):
                        reasons.add(nm)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ distributed
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_pg(world, backend, device=None):
    import datetime
    import torch.distributed as dist
    if world > 1 and not dist.is_initialized():
        kw = {"device_id": device} if device is not None else {}
        # Keep library banners (e.g. NCCL's version line) off stdout, which
        # carries only the JSON result line.
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=120), **kw)
            dist.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)


def max_over_ranks(value, world, device):
    from complex_conv2d.distributed import max_over_ranks as _max
    return _max(value, device) if world > 1 else value


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ------------------------------------------------------------------ CPU baseline
def cpu_baseline(wl, budget_s=12.0):
    """The reference's four-conv path (restated in oracle/) on host cores, fp32,
    on a bounded sample: single images of the workload's layer."""
    import oracle
    n, c, h, w, k, r, s, st, pd, std = wl
    case = oracle.ConvCase(1, c, h, w, k, r, s, st, st, pd, pd)
    threads = torch.get_num_threads()
    t1, _ = oracle.time_cpu_four_conv(case, iters=1, warmup=1)
    iters = max(1, min(200, int(budget_s / max(t1, 1e-4))))
    dt, threads = oracle.time_cpu_four_conv(case, iters=iters, warmup=0)
    tflops = case.flops / dt / 1e12
    return {"value": tflops, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{iters} single-image calls (batch 1 of the workload layer), fp32, "
                      f"{dt * 1e3:.2f} ms/call, os.cpu_count()={os.cpu_count()}"}, dt


def run_reference(args, wl):
    world, rank, local = dist_setup()
    if rank != 0:
        return 0
    import oracle
    n, c, h, w, k, r, s, st, pd, std = wl
    case = oracle.ConvCase(1, c, h, w, k, r, s, st, st, pd, pd)
    x, wr, wi = oracle.make_inputs(case, input_std=std)
    with torch.no_grad():
        for _ in range(args.warmup):
            oracle.four_conv(x, wr, wi, (st, st), (pd, pd), dtype=torch.float32)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            oracle.four_conv(x, wr, wi, (st, st), (pd, pd), dtype=torch.float32)
        dt = (time.perf_counter() - t0) / max(args.steps, 1)
    value = case.flops / dt / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "sample": "batch 1 of the workload layer per step",
                   "global_batch": n, "c": c, "h": h, "w": w, "k": k, "r": r, "s": s,
                   "stride": st, "pad": pd},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"{args.steps} single-image four-conv calls, fp32 CPU torch"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ our arm
def run_ours(args, wl):
    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    init_pg(world, "nccl", dev)
    from complex_conv2d import ComplexConv2d

    from complex_conv2d.distributed import batch_shard
    n, c, h, w, k, r, s, st, pd, std = wl
    _, nb = batch_shard(n, world, rank)
    if nb == 0:
        raise SystemExit(f"global batch {n} leaves rank {rank} of {world} without images")
    p, q = out_hw(h, w, r, s, st, pd)
    flops_rank = workload_flops(nb, c, h, w, k, r, s, st, pd)
    flops_total = workload_flops(n, c, h, w, k, r, s, st, pd)

    # Weights: identical seeded init on every rank (replicated, no broadcast).
    g = torch.Generator().manual_seed(1)
    bound = 1.0 / (c * r * s) ** 0.5
    wr = (torch.rand((k, c, r, s), generator=g) * 2 - 1) * bound
    wi = (torch.rand((k, c, r, s), generator=g) * 2 - 1) * bound
    layer = ComplexConv2d(c, k, (r, s), stride=st, padding=pd, device=dev, precision=args.precision)
    with torch.no_grad():
        layer.weight_real.copy_(wr)
        layer.weight_imag.copy_(wi)
    # This rank's slice of the seeded global batch.  Steps rotate over enough
    # distinct input buffers that their total exceeds twice the 126 MB L2, so
    # no step reads an input left in L2 by an earlier step.
    in_bytes = nb * c * h * w * 8
    nbuf = max(1, -(-256 * 2**20 // in_bytes))
    gx = torch.Generator(device=dev).manual_seed(1000 + rank)
    xs = []
    for _ in range(nbuf):
        xr = torch.randn((nb, c, h, w), generator=gx, device=dev) * std
        xi = torch.randn((nb, c, h, w), generator=gx, device=dev) * std
        xs.append(torch.complex(xr, xi))
    x = xs[0]
    x_planar_r = xr.permute(0, 2, 3, 1).contiguous()
    x_planar_i = xi.permute(0, 2, 3, 1).contiguous()
    del xr, xi
    stream = torch.cuda.current_stream()

    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    phys = visible.split(",")[local] if visible else str(local)
    clocks = ClockSampler(phys)
    with torch.no_grad():
        clocks.start()
        # ---- device-resident timing of the public forward()
        for i in range(args.warmup):
            y = layer(xs[i % nbuf])
        barrier(world)
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(args.steps):
            y = layer(xs[i % nbuf])
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        t_fwd = e0.elapsed_time(e1) / 1e3 / args.steps
        clk = clocks.stop()

        # ---- the dominant kernel alone: forward_planar is one fprop launch
        for _ in range(max(3, args.warmup // 2)):
            yp = layer.forward_planar(x_planar_r, x_planar_i)
        torch.cuda.synchronize()
        e2 = torch.cuda.Event(enable_timing=True)
        e3 = torch.cuda.Event(enable_timing=True)
        e2.record(stream)
        for _ in range(args.steps):
            yp = layer.forward_planar(x_planar_r, x_planar_i)
        e3.record(stream)
        torch.cuda.synchronize()
        t_kernel = e2.elapsed_time(e3) / 1e3 / args.steps
        del yp

        # ---- forward()'s convolution launch alone (planar input, complex64
        # output; forward() adds the complex64 -> planar layout pass)
        from complex_conv2d import _C
        layer._ensure_prepacked()
        prec_code = 1 if args.precision == "3xtf32" else 0
        conv = lambda: _C.forward_planar_to_complex_packed(
            x_planar_r, x_planar_i, layer._w_packed, c, k, r, s, st, st, pd, pd, prec_code)
        for _ in range(max(3, args.warmup // 2)):
            yc = conv()
        torch.cuda.synchronize()
        e6 = torch.cuda.Event(enable_timing=True)
        e7 = torch.cuda.Event(enable_timing=True)
        e6.record(stream)
        for _ in range(args.steps):
            yc = conv()
        e7.record(stream)
        torch.cuda.synchronize()
        t_conv = e6.elapsed_time(e7) / 1e3 / args.steps
        del yc

        # ---- end to end: pinned host input -> device -> forward -> pinned host output
        x_host = x.cpu().pin_memory()
        y_host = torch.empty((nb, k, p, q), dtype=torch.complex64).pin_memory()
        def serial_step():
            xd = x_host.to(dev, non_blocking=True)
            y_host.copy_(layer(xd), non_blocking=True)

        def host_step():
            layer.forward_host(x_host, out=y_host)

        def timed(step):
            for _ in range(max(3, min(args.warmup, 5))):
                step()
            barrier(world)
            torch.cuda.synchronize()
            e4 = torch.cuda.Event(enable_timing=True)
            e5 = torch.cuda.Event(enable_timing=True)
            e4.record(stream)
            for _ in range(args.steps):
                step()
            e5.record(stream)
            torch.cuda.synchronize()
            barrier(world)
            return e4.elapsed_time(e5) / 1e3 / args.steps

        t_e2e_serial = timed(serial_step)
        t_e2e = timed(host_step)

    t_fwd_max = max_over_ranks(t_fwd, world, dev)
    t_e2e_max = max_over_ranks(t_e2e, world, dev)
    t_e2e_serial_max = max_over_ranks(t_e2e_serial, world, dev)
    t_kernel_max = max_over_ranks(t_kernel, world, dev)

    if rank != 0:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return 0

    from complex_conv2d import _C
    prec_code = 1 if args.precision == "3xtf32" else 0
    launches = _C.complex_forward_launches(nb, c, h, w, k, r, s, st, st, pd, pd, prec_code)
    kernel_path = _C.complex_forward_kernel(nb, c, h, w, k, r, s, st, st, pd, pd, prec_code)
    peaks = load_peaks()
    tf32_peak = peaks["bf16_tflops"] / 2.0  # dense TF32 runs at half the bf16 rate
    if args.precision == "3xtf32":
        tf32_peak /= 3.0  # three TF32 products per fp32 product
    # Roofline of the dominant kernel: forward()'s convolution launch, timed
    # alone above (t_conv); the layout pass in front of it is HBM-bound.
    one_launch = launches == 1
    t_dom = t_fwd if one_launch else t_conv
    achieved = flops_rank / t_dom / 1e12
    out_bytes = nb * k * p * q * 8
    line = {
        "metric": METRIC,
        "value": flops_total / t_fwd_max / 1e12,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": t_fwd_max * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": args.precision,
        "data": "synthetic (seeded N(0,1) inputs, U(+-1/sqrt(C*R*S)) weights)",
        "config": {
            "workload": args.workload, "global_batch": n, "per_gpu_batch": nb,
            "c": c, "h": h, "w": w, "k": k, "r": r, "s": s, "stride": st, "pad": pd,
            "parallelism": f"dp{world} batch-sharded, weights replicated, no collective",
            "l2": f"{in_bytes / 1e6:.0f} MB input + {out_bytes / 1e6:.0f} MB output per GPU per "
                  f"step; steps rotate over {nbuf} input buffers ({nbuf * in_bytes / 1e6:.0f} MB "
                  f"> 2x L2), so no step reads an L2-resident input",
            "api": "ComplexConv2d.forward (complex64 NCHW)",
        },
        "forward_planar_ms": t_kernel_max * 1e3,
        "forward_conv_launch_ms": t_conv * 1e3,
        "roofline": {
            "bound": "tensor", "achieved": achieved, "peak": tf32_peak, "unit": UNIT,
            "frac": achieved / tf32_peak,
            # The committed ncu summary covers the single-GPU launch of the
            # workload (whole batch); a per-GPU shard runs a smaller launch.
            "traffic": profiled_traffic("forward_conv", args.workload) if world == 1 else None,
            "kernel": (f"forward() path {kernel_path}: {launches} launch(es); roofline of the "
                       f"convolution launch ({t_dom * 1e3:.4f} ms of {t_fwd * 1e3:.4f} ms per "
                       "forward())"),
            "peak_source": (f"{peaks['source']} bf16 {peaks['bf16_tflops']} TFLOP/s / 2 (dense TF32)"
                            + (" / 3 (3xTF32)" if args.precision == "3xtf32" else "")),
        },
        "e2e": {"value": flops_total / t_e2e_max / 1e12, "unit": UNIT,
                "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": out_bytes,
                "ms_per_step": t_e2e_max * 1e3,
                "api": "ComplexConv2d.forward_host (pinned host in/out, chunked copy pipeline)",
                "serial_ms_per_step": t_e2e_serial_max * 1e3},
        "gpu_launches": args.steps * launches,
        "clocks": clk,
    }
    if world == 1 and not args.no_cpu_baseline:
        cb, _ = cpu_baseline(wl)
        line["cpu_baseline"] = cb
    print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT_WORKLOAD)
    ap.add_argument("--precision", choices=["tf32", "3xtf32"], default="tf32")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        return run_reference(args, wl)
    return run_ours(args, wl)


if __name__ == "__main__":
    sys.exit(main())
