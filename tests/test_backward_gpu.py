"""Parity of the backward entry points (data and weight gradients) against
the fp64 gradient oracle, through the C ABI.

The oracle (oracle.backward_autograd_fp64) is pinned to the gradients torch
autograd gives for the reference's own four-conv module
(tests/test_oracle_backward.py); the reference itself has no backward
(README.md:143).  Bars: rel. Frobenius <= 1e-3 for TF32, 1e-5 for the
3xTF32 data gradient (the weight gradient is TF32 only).
"""

import ctypes

import numpy as np
import pytest
import torch

import ccv_abi
import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _dy(case, seed=7):
    g = torch.Generator().manual_seed(seed)
    shape = (case.n, case.k, case.p, case.q)
    return torch.complex(torch.randn(shape, generator=g), torch.randn(shape, generator=g))


def dgrad(case, wr, wi, dy, precision=ccv_abi.CCV_PRECISION_TF32):
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    nb = lib.ccv_packed_weight_bytes(ctypes.byref(shp), precision)
    packed = torch.empty(nb // 4, dtype=torch.float32, device=DEV)
    wr_d, wi_d = wr.to(DEV).contiguous(), wi.to(DEV).contiguous()
    ccv_abi.check(lib.ccv_prepack_weights_dgrad(_ptr(wr_d), _ptr(wi_d), ccv_abi.CCV_WEIGHT_KCRS,
                                                ctypes.byref(shp), precision, _ptr(packed), nb,
                                                _stream()), "dgrad prepack")
    wsb = lib.ccv_dgrad_complex_workspace_bytes(ctypes.byref(shp), precision)
    assert wsb > 0, ccv_abi.last_error()
    ws = torch.empty(wsb, dtype=torch.uint8, device=DEV)
    dy_d = dy.to(DEV).contiguous()
    dx = torch.full((case.n, case.c, case.h, case.w), float("nan"), dtype=torch.complex64,
                    device=DEV)
    ccv_abi.check(lib.ccv_dgrad_complex(_ptr(dy_d), _ptr(packed), _ptr(dx), ctypes.byref(shp),
                                        precision, _ptr(ws), wsb, _stream()), "dgrad")
    torch.cuda.synchronize()
    return dx.cpu()


def wgrad(case, x, dy):
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    wsb = lib.ccv_wgrad_complex_workspace_bytes(ctypes.byref(shp))
    assert wsb > 0, ccv_abi.last_error()
    ws = torch.full((wsb,), 0xFF, dtype=torch.uint8, device=DEV)  # NaN-poisoned scratch
    x_d, dy_d = x.to(DEV).contiguous(), dy.to(DEV).contiguous()
    dwr = torch.full((case.k, case.c, case.r, case.s), float("nan"), device=DEV)
    dwi = torch.full_like(dwr, float("nan"))
    ccv_abi.check(lib.ccv_wgrad_complex(_ptr(x_d), _ptr(dy_d), _ptr(dwr), _ptr(dwi),
                                        ctypes.byref(shp), _ptr(ws), wsb, _stream()), "wgrad")
    torch.cuda.synchronize()
    return dwr.cpu(), dwi.cpu()


CASES = [
    oracle.ConvCase(1, 32, 8, 8, 32, 3, 3, 1, 1, 1, 1),
    oracle.ConvCase(2, 16, 9, 9, 16, 3, 3, 2, 2, 1, 1),
    oracle.ConvCase(1, 8, 10, 10, 16, 3, 3, 1, 1, 0, 0),
    oracle.ConvCase(1, 16, 8, 8, 24, 1, 1, 1, 1, 0, 0),
    oracle.ConvCase(1, 8, 6, 10, 8, 3, 3, 1, 1, 1, 1),
    oracle.ConvCase(1, 4, 11, 13, 8, 7, 7, 2, 2, 3, 3),
    oracle.ConvCase(1, 8, 7, 9, 12, 3, 1, 2, 1, 1, 0),
    oracle.ConvCase(1, 36, 5, 6, 20, 3, 3, 1, 1, 1, 1),
    oracle.ConvCase(2, 64, 20, 20, 128, 3, 3, 1, 1, 1, 1),   # CT = 64
    oracle.ConvCase(1, 160, 12, 12, 144, 3, 3, 1, 1, 1, 1),  # two k tiles, two c tiles
    oracle.ConvCase(2, 32, 40, 40, 64, 3, 3, 2, 2, 1, 1),    # q spans two 32-pixel blocks
]
IDS = [f"n{c.n}c{c.c}h{c.h}w{c.w}k{c.k}r{c.r}s{c.s}st{c.stride_h}{c.stride_w}p{c.pad_h}{c.pad_w}"
       for c in CASES]


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_dgrad_matches_oracle(case):
    x, wr, wi = oracle.make_inputs(case)
    dy = _dy(case)
    ref_dx, _, _ = oracle.backward_autograd_fp64(case, x, wr, wi, dy)
    dx = dgrad(case, wr, wi, dy)
    assert torch.isfinite(torch.view_as_real(dx)).all()
    assert oracle.rel_frobenius(dx, ref_dx) <= 1e-3


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_wgrad_matches_oracle(case):
    x, wr, wi = oracle.make_inputs(case)
    dy = _dy(case)
    _, ref_wr, ref_wi = oracle.backward_autograd_fp64(case, x, wr, wi, dy)
    dwr, dwi = wgrad(case, x, dy)
    assert torch.isfinite(dwr).all() and torch.isfinite(dwi).all()
    got = torch.complex(dwr.double(), dwi.double())
    ref = torch.complex(ref_wr, ref_wi)
    assert oracle.rel_frobenius(got, ref) <= 1e-3


def test_dgrad_3xtf32():
    case = oracle.ConvCase(2, 32, 12, 12, 32, 3, 3, 1, 1, 1, 1)
    x, wr, wi = oracle.make_inputs(case)
    dy = _dy(case)
    ref_dx, _, _ = oracle.backward_autograd_fp64(case, x, wr, wi, dy)
    dx = dgrad(case, wr, wi, dy, ccv_abi.CCV_PRECISION_3XTF32)
    assert oracle.rel_frobenius(dx, ref_dx) <= 1e-5


def test_backward_golden_vectors():
    """The reference module's own autograd gradients (committed fixtures)."""
    import os
    here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    fw = np.load(os.path.join(here, "golden_vectors.npz"))
    bw = np.load(os.path.join(here, "golden_backward.npz"))
    for name in bw["names"]:
        name = str(name)
        case = oracle.ConvCase(*fw[f"{name}/meta"].tolist())
        if case.c % 4 or case.k % 4:
            continue
        x = torch.from_numpy(fw[f"{name}/x"])
        wr, wi = torch.from_numpy(fw[f"{name}/w_real"]), torch.from_numpy(fw[f"{name}/w_imag"])
        dy = torch.from_numpy(bw[f"{name}/dy"])
        dx = dgrad(case, wr, wi, dy)
        assert oracle.rel_frobenius(dx, torch.from_numpy(bw[f"{name}/dx"])) <= 1e-3, name
        dwr, dwi = wgrad(case, x, dy)
        got = torch.complex(dwr.double(), dwi.double())
        ref = torch.complex(torch.from_numpy(bw[f"{name}/dw_real"]),
                            torch.from_numpy(bw[f"{name}/dw_imag"]))
        assert oracle.rel_frobenius(got, ref) <= 1e-3, name


def test_wgrad_deterministic():
    case = oracle.ConvCase(4, 64, 28, 28, 64, 3, 3, 1, 1, 1, 1)
    x, _, _ = oracle.make_inputs(case)
    dy = _dy(case)
    a = wgrad(case, x, dy)
    b = wgrad(case, x, dy)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


@pytest.mark.parametrize("case", [
    oracle.ConvCase(1, 8, 8, 8, 8, 3, 3, 1, 1, 3, 3),      # padding above kernel size - 1
    oracle.ConvCase(2, 8, 12, 10, 16, 3, 3, 3, 2, 2, 1),   # stride 3 x 2 (6 phases)
    oracle.ConvCase(1, 16, 9, 9, 8, 1, 1, 2, 2, 0, 0),     # phases no tap reaches (zero dx)
    oracle.ConvCase(1, 8, 16, 16, 12, 5, 5, 4, 4, 2, 2),   # stride 4
], ids=["pad3_k3", "s3x2", "1x1_s2", "k5_s4"])
def test_dgrad_phases(case):
    """Phase decomposition of the data gradient: strides, big padding, phases
    no filter tap reaches."""
    x, wr, wi = oracle.make_inputs(case)
    dy = _dy(case)
    ref_dx, _, _ = oracle.backward_autograd_fp64(case, x, wr, wi, dy)
    dx = dgrad(case, wr, wi, dy)
    assert torch.isfinite(torch.view_as_real(dx)).all()
    assert oracle.rel_frobenius(dx, ref_dx) <= 1e-3


def _planes(t):
    """complex64 NCHW -> (real, imag) fp32 NHWC planes on the device."""
    t = t.to(DEV)
    return (t.real.permute(0, 2, 3, 1).contiguous(), t.imag.permute(0, 2, 3, 1).contiguous())


@pytest.mark.parametrize("case", CASES[:8] + [oracle.ConvCase(1, 8, 8, 8, 8, 3, 3, 1, 1, 3, 3)],
                         ids=IDS[:8] + ["pad3_k3"])
def test_planar_gradients_match_oracle(case):
    """ccv_dgrad_planar / ccv_wgrad_planar (the forward_planar layouts)."""
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    x, wr, wi = oracle.make_inputs(case)
    dy = _dy(case)
    rx, rwr, rwi = oracle.backward_autograd_fp64(case, x, wr, wi, dy)
    nb = lib.ccv_packed_weight_bytes(ctypes.byref(shp), 0)
    packed = torch.empty(nb // 4, dtype=torch.float32, device=DEV)
    wr_d, wi_d = wr.to(DEV).contiguous(), wi.to(DEV).contiguous()
    ccv_abi.check(lib.ccv_prepack_weights_dgrad(_ptr(wr_d), _ptr(wi_d), ccv_abi.CCV_WEIGHT_KCRS,
                                                ctypes.byref(shp), 0, _ptr(packed), nb,
                                                _stream()), "dgrad prepack")
    dyr, dyi = _planes(dy)
    xr, xi = _planes(x)
    wsb = lib.ccv_dgrad_planar_workspace_bytes(ctypes.byref(shp), 0)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=DEV)
    dxr = torch.full((case.n, case.h, case.w, case.c), float("nan"), device=DEV)
    dxi = torch.full_like(dxr, float("nan"))
    ccv_abi.check(lib.ccv_dgrad_planar(_ptr(dyr), _ptr(dyi), _ptr(packed), _ptr(dxr), _ptr(dxi),
                                       ctypes.byref(shp), 0, _ptr(ws), wsb, _stream()),
                  "dgrad planar")
    wwb = lib.ccv_wgrad_planar_workspace_bytes(ctypes.byref(shp))
    wws = torch.empty(wwb, dtype=torch.uint8, device=DEV)
    dwr = torch.full((case.k, case.c, case.r, case.s), float("nan"), device=DEV)
    dwi = torch.full_like(dwr, float("nan"))
    ccv_abi.check(lib.ccv_wgrad_planar(_ptr(xr), _ptr(xi), _ptr(dyr), _ptr(dyi), _ptr(dwr),
                                       _ptr(dwi), ctypes.byref(shp), _ptr(wws), wwb, _stream()),
                  "wgrad planar")
    torch.cuda.synchronize()
    dx = oracle.planar_nhwc_to_complex_nchw(dxr, dxi).cpu()
    assert oracle.rel_frobenius(dx, rx) <= 1e-3
    got = torch.complex(dwr.cpu().double(), dwi.cpu().double())
    assert oracle.rel_frobenius(got, torch.complex(rwr, rwi)) <= 1e-3
