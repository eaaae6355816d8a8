"""ccv_forward_noalloc: the reference-ABI forward for callers that may not
allocate device memory (for example code running inside another framework's
enqueue/execute callback, where that framework owns the memory pool and a
cudaMalloc could synchronize the device).  Its scratch (the packed weight
image) lives in a fixed 16 MiB device array inside the library instead of a
caller-provided workspace.

The GPU test calls it through the C ABI twice in a row, on two different
problems, and checks each result against ccv_forward (the entry point with a
caller-provided workspace) within the TF32 tolerance of the other parity
tests.  The file is named to be collected last.
"""

import ctypes

import pytest
import torch

import ccv_abi
import oracle

TF32_TOL = 1e-3
MAX_BYTES = 16 * 1024 * 1024


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _inputs(case, seed):
    x, wr, wi = oracle.make_inputs(case, input_seed=seed, weight_seed=seed + 1)
    dev = "cuda:0"
    xr = x.real.permute(0, 2, 3, 1).contiguous().to(dev)
    xi = x.imag.permute(0, 2, 3, 1).contiguous().to(dev)
    wr_k = wr.permute(0, 2, 3, 1).contiguous().to(dev)
    wi_k = wi.permute(0, 2, 3, 1).contiguous().to(dev)
    return xr, xi, wr_k, wi_k


def _outputs(case):
    yr = torch.empty((case.n, case.p, case.q, case.k), device="cuda:0")
    return yr, torch.empty_like(yr)


def _run_with_workspace(lib, case, xr, xi, wr, wi, stream):
    shp = ccv_abi.shape_of(case)
    yr, yi = _outputs(case)
    ws_bytes = lib.ccv_forward_workspace_bytes(ctypes.byref(shp))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda:0")
    ccv_abi.check(lib.ccv_forward(_ptr(xr), _ptr(xi), _ptr(wr), _ptr(wi), _ptr(yr), _ptr(yi),
                                  ctypes.byref(shp), _ptr(ws), ws_bytes, stream), "ccv_forward")
    return yr, yi


def _run_noalloc(lib, case, xr, xi, wr, wi, stream):
    shp = ccv_abi.shape_of(case)
    yr, yi = _outputs(case)
    ccv_abi.check(lib.ccv_forward_noalloc(_ptr(xr), _ptr(xi), _ptr(wr), _ptr(wi), _ptr(yr),
                                          _ptr(yi), ctypes.byref(shp), stream),
                  "ccv_forward_noalloc")
    return yr, yi


def _as_complex(yr, yi):
    return torch.complex(yr, yi).cpu()


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_on_two_calls():
    torch.cuda.set_device(0)
    lib = ccv_abi.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    cases = [
        oracle.ConvCase(2, 64, 20, 24, 96, 3, 3, 1, 1, 1, 1),
        oracle.ConvCase(1, 32, 17, 15, 40, 5, 5, 2, 2, 2, 2),
    ]
    for i, case in enumerate(cases):
        xr, xi, wr, wi = _inputs(case, seed=11 + 2 * i)
        yr_a, yi_a = _run_noalloc(lib, case, xr, xi, wr, wi, stream)
        yr_b, yi_b = _run_with_workspace(lib, case, xr, xi, wr, wi, stream)
        torch.cuda.synchronize()
        got, want = _as_complex(yr_a, yi_a), _as_complex(yr_b, yi_b)
        assert not torch.isnan(got.real).any() and not torch.isnan(got.imag).any()
        assert oracle.rel_frobenius(got, want) <= TF32_TOL, (i, case)
    st = ctypes.c_int(-1)
    ccv_abi.check(lib.ccv_get_device_status(ctypes.byref(st)), "status")
    assert st.value == 0


@pytest.mark.gpu
def test_noalloc_back_to_back_on_one_stream_without_sync():
    """Two calls with different weights enqueued on one stream with no host
    sync between them: the second call's weight prepack rewrites the shared
    array only after the first call's convolution has finished reading it
    (stream order; with programmatic dependent launch the prepack kernel
    waits for the previous kernel to complete before its first global
    access), so each output matches ccv_forward on its own weights."""
    torch.cuda.set_device(0)
    lib = ccv_abi.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    case = oracle.ConvCase(2, 64, 24, 24, 128, 3, 3, 1, 1, 1, 1)
    xr, xi, wr1, wi1 = _inputs(case, seed=21)
    _, _, wr2, wi2 = _inputs(case, seed=23)
    ya = _run_noalloc(lib, case, xr, xi, wr1, wi1, stream)
    yb = _run_noalloc(lib, case, xr, xi, wr2, wi2, stream)
    ra = _run_with_workspace(lib, case, xr, xi, wr1, wi1, stream)
    rb = _run_with_workspace(lib, case, xr, xi, wr2, wi2, stream)
    torch.cuda.synchronize()
    for got, want in ((ya, ra), (yb, rb)):
        g, w = _as_complex(*got), _as_complex(*want)
        assert not torch.isnan(g.real).any() and not torch.isnan(g.imag).any()
        assert oracle.rel_frobenius(g, w) <= TF32_TOL
    # The two weight sets give different outputs (the test can tell them apart).
    assert oracle.rel_frobenius(_as_complex(*ya), _as_complex(*yb)) > 0.1


def test_noalloc_rejects_weights_above_fixed_scratch():
    """Rejected on the host, before any device work: 3x3, K*C above 155,344."""
    lib = ccv_abi.load()
    case = oracle.ConvCase(1, 512, 8, 8, 512, 3, 3, 1, 1, 1, 1)
    assert 3 * 9 * 512 * 512 * 4 > MAX_BYTES
    shp = ccv_abi.shape_of(case)
    dummy = ctypes.c_void_p(16)
    rc = lib.ccv_forward_noalloc(dummy, dummy, dummy, dummy, dummy, dummy, ctypes.byref(shp), None)
    assert rc == ccv_abi.CCV_ERR_WORKSPACE
    assert "fixed scratch" in ccv_abi.last_error()
