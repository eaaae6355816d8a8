"""Counter sets (stream-K tile counters and layout-warp tickets) are never
shared by two launches in flight.

Each launch that needs counters takes one of the library's sets; a set is
handed out again only after the CUDA event recorded behind its launch has
completed, and a set taken during stream capture stays with the captured
graph.  With every set in flight, a call runs a path without counters (layout
pass instead of layout warps, whole tiles instead of the stream-K split),
which gives the same sums here (whole tiles pinned), so every output must be
bitwise equal to the serial result.
"""

import os

import pytest
import torch

import oracle
from test_parity_gpu import DEV, TF32_TOL, device_status

pytestmark = pytest.mark.gpu

KEYS = ("CCV_FORCE_KERNEL", "CCV_HALO", "CCV_LW", "CCV_STREAMK", "CCV_SUBBOX")
N_SETS = 64


@pytest.fixture
def layout_warps_everywhere():
    from complex_conv2d import _C
    old = {k: os.environ.get(k) for k in KEYS}
    os.environ.update({"CCV_FORCE_KERNEL": "2", "CCV_HALO": "1", "CCV_LW": "1",
                       "CCV_STREAMK": "0"})
    os.environ.pop("CCV_SUBBOX", None)
    _C.reload_config()
    yield
    for k, v in old.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v
    _C.reload_config()
    torch.cuda.synchronize()
    assert device_status() == 0


def _layer(case, wr, wi):
    from complex_conv2d import ComplexConv2d
    layer = ComplexConv2d(case.c, case.k, (case.r, case.s), padding=(case.pad_h, case.pad_w),
                          device=DEV)
    with torch.no_grad():
        layer.weight_real.copy_(wr)
        layer.weight_imag.copy_(wi)
    return layer


def test_more_launches_in_flight_than_sets(layout_warps_everywhere):
    from complex_conv2d import _C
    case = oracle.ConvCase(3, 64, 28, 28, 128, 3, 3, 1, 1, 1, 1)
    assert _C.complex_forward_kernel(case.n, case.c, case.h, case.w, case.k, case.r, case.s,
                                     1, 1, 1, 1, 0) == "halo_pair_layout_warps"
    x, wr, wi = oracle.make_inputs(case, input_seed=71)
    layer = _layer(case, wr, wi)
    xd = x.to(DEV)
    with torch.no_grad():
        want = layer(xd)
    torch.cuda.synchronize()
    assert oracle.rel_frobenius(want.cpu(), oracle.oracle_fp64(case, x, wr, wi)) <= TF32_TOL
    streams = [torch.cuda.Stream() for _ in range(N_SETS + 16)]
    outs = []
    with torch.no_grad():
        for st in streams:
            with torch.cuda.stream(st):
                # Hold the stream so every call below is still in flight when
                # the next one takes its set (a bounded spin of ~10 ms).
                torch.cuda._sleep(20_000_000)
                outs.append(layer(xd))
    torch.cuda.synchronize()
    for i, y in enumerate(outs):
        assert torch.equal(y, want), i


def test_captured_graph_keeps_its_set(layout_warps_everywhere):
    case = oracle.ConvCase(3, 64, 28, 28, 128, 3, 3, 1, 1, 1, 1)
    x, wr, wi = oracle.make_inputs(case, input_seed=72)
    layer = _layer(case, wr, wi)
    xd = x.to(DEV)
    side = torch.cuda.Stream()
    with torch.no_grad():
        want = layer(xd)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            yg = layer(xd)
        for _ in range(3):
            g.replay()
            # Eager calls on another stream while the graph runs.
            with torch.cuda.stream(side):
                ye = layer(xd)
            torch.cuda.synchronize()
            assert torch.equal(yg, want)
            assert torch.equal(ye, want)
    del g
