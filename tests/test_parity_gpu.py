"""GPU parity of the B200 kernels against the fp64 CPU oracle, called through
the C ABI (include/ccv_b200.h via ctypes) with torch-allocated device memory.

Tolerance (north star): relative Frobenius error <= 1e-3 for TF32 against the
fp64 four-conv oracle (benchmarks/baseline.py:5-9 restated in oracle/).
"""

import ctypes

import numpy as np
import pytest
import torch

import ccv_abi
import oracle
from oracle.configs import BASELINE_CASES

from test_oracle import CASES as GOLDEN_CASES

pytestmark = pytest.mark.gpu

TF32_TOL = 1e-3
DEV = "cuda:0"


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def abi_prepack(case, wr, wi, layout=ccv_abi.CCV_WEIGHT_KCRS, precision=ccv_abi.CCV_PRECISION_TF32):
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    nbytes = lib.ccv_packed_weight_bytes(ctypes.byref(shp), precision)
    packed = torch.empty(nbytes // 4, dtype=torch.float32, device=DEV)
    wr = wr.to(DEV).contiguous()
    wi = wi.to(DEV).contiguous()
    if layout == ccv_abi.CCV_WEIGHT_KRSC:
        wr = wr.permute(0, 2, 3, 1).contiguous()
        wi = wi.permute(0, 2, 3, 1).contiguous()
    ccv_abi.check(lib.ccv_prepack_weights(_ptr(wr), _ptr(wi), layout, ctypes.byref(shp), precision,
                                          _ptr(packed), nbytes, _stream()), "prepack")
    return packed


def abi_fprop_planar(case, x, packed, precision=ccv_abi.CCV_PRECISION_TF32, poison=False):
    """x: complex64 NCHW (CPU or GPU). Returns complex128 NCHW on CPU."""
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    xr = x.real.permute(0, 2, 3, 1).contiguous().to(DEV)
    xi = x.imag.permute(0, 2, 3, 1).contiguous().to(DEV)
    fill = float("nan") if poison else 0.0
    yr = torch.full((case.n, case.p, case.q, case.k), fill, dtype=torch.float32, device=DEV)
    yi = torch.full_like(yr, fill)
    ws_bytes = lib.ccv_fprop_planar_workspace_bytes(ctypes.byref(shp), precision)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=DEV)
    ccv_abi.check(lib.ccv_fprop_planar(_ptr(xr), _ptr(xi), _ptr(packed), _ptr(yr), _ptr(yi),
                                       ctypes.byref(shp), precision,
                                       _ptr(ws) if ws_bytes else None, ws_bytes, _stream()),
                  "fprop_planar")
    torch.cuda.synchronize()
    return oracle.planar_nhwc_to_complex_nchw(yr, yi).cpu()


def abi_fprop_complex(case, x, packed, precision=ccv_abi.CCV_PRECISION_TF32, poison=False):
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    xd = x.to(DEV).contiguous()
    y = torch.empty((case.n, case.k, case.p, case.q), dtype=torch.complex64, device=DEV)
    if poison:
        y.real.fill_(float("nan"))
        y.imag.fill_(float("nan"))
    ws_bytes = lib.ccv_fprop_complex_workspace_bytes(ctypes.byref(shp), precision)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=DEV)
    ccv_abi.check(lib.ccv_fprop_complex(_ptr(xd), _ptr(packed), _ptr(y), ctypes.byref(shp),
                                        precision, _ptr(ws), ws_bytes, _stream()), "fprop_complex")
    torch.cuda.synchronize()
    return y.cpu()


def abi_fprop_planar_to_complex(case, x, packed, precision=ccv_abi.CCV_PRECISION_TF32):
    """Planar NHWC in (built from complex64 NCHW x), complex64 NKPQ out."""
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    xr = x.real.permute(0, 2, 3, 1).contiguous().to(DEV)
    xi = x.imag.permute(0, 2, 3, 1).contiguous().to(DEV)
    y = torch.full((case.n, case.k, case.p, case.q), float("nan"), dtype=torch.complex64,
                   device=DEV)
    ws_bytes = lib.ccv_fprop_planar_workspace_bytes(ctypes.byref(shp), precision)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=DEV)
    ccv_abi.check(lib.ccv_fprop_planar_to_complex(_ptr(xr), _ptr(xi), _ptr(packed), _ptr(y),
                                                  ctypes.byref(shp), precision,
                                                  _ptr(ws) if ws_bytes else None, ws_bytes,
                                                  _stream()), "fprop_planar_to_complex")
    torch.cuda.synchronize()
    return y.cpu()


def device_status():
    lib = ccv_abi.load()
    st = ctypes.c_int(-1)
    ccv_abi.check(lib.ccv_get_device_status(ctypes.byref(st)), "status")
    return st.value


@pytest.fixture(autouse=True)
def _clean_status():
    torch.cuda.set_device(0)
    yield
    assert device_status() == 0, "a bounded in-kernel wait ran out"


# ----------------------------------------------------------------- golden set
@pytest.mark.parametrize("name,case,x,wr,wi,y32,y64", GOLDEN_CASES, ids=[c[0] for c in GOLDEN_CASES])
def test_golden_planar(name, case, x, wr, wi, y32, y64):
    packed = abi_prepack(case, torch.from_numpy(wr), torch.from_numpy(wi))
    y = abi_fprop_planar(case, torch.from_numpy(x), packed, poison=True)
    assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any()
    err = oracle.rel_frobenius(y, y64)
    assert err <= TF32_TOL, (name, err)


@pytest.mark.parametrize("name,case,x,wr,wi,y32,y64", GOLDEN_CASES, ids=[c[0] for c in GOLDEN_CASES])
def test_golden_complex_matches_planar_bitwise(name, case, x, wr, wi, y32, y64):
    packed = abi_prepack(case, torch.from_numpy(wr), torch.from_numpy(wi))
    xt = torch.from_numpy(x)
    yc = abi_fprop_complex(case, xt, packed, poison=True)
    yp = abi_fprop_planar(case, xt, packed)
    assert torch.equal(yc, yp.to(torch.complex64))
    assert oracle.rel_frobenius(yc, y64) <= TF32_TOL


@pytest.mark.parametrize("name,case,x,wr,wi,y32,y64", GOLDEN_CASES, ids=[c[0] for c in GOLDEN_CASES])
def test_golden_planar_to_complex_entry(name, case, x, wr, wi, y32, y64):
    """Planar input with complex output runs forward()'s convolution launch:
    bitwise equal to ccv_fprop_complex (which adds the layout pass)."""
    xt = torch.from_numpy(x)
    for prec in (ccv_abi.CCV_PRECISION_TF32, ccv_abi.CCV_PRECISION_3XTF32):
        packed = abi_prepack(case, torch.from_numpy(wr), torch.from_numpy(wi), precision=prec)
        y = abi_fprop_planar_to_complex(case, xt, packed, precision=prec)
        assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any()
        assert torch.equal(y, abi_fprop_complex(case, xt, packed, precision=prec)), (name, prec)


@pytest.mark.parametrize("name,case,x,wr,wi,y32,y64", GOLDEN_CASES[:4], ids=[c[0] for c in GOLDEN_CASES[:4]])
def test_golden_krsc_forward_entry(name, case, x, wr, wi, y32, y64):
    """ccv_forward: the reference `_C.forward` contract with KRSC weights."""
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    xt = torch.from_numpy(x)
    xr = xt.real.permute(0, 2, 3, 1).contiguous().to(DEV)
    xi = xt.imag.permute(0, 2, 3, 1).contiguous().to(DEV)
    wr_k = torch.from_numpy(wr).permute(0, 2, 3, 1).contiguous().to(DEV)
    wi_k = torch.from_numpy(wi).permute(0, 2, 3, 1).contiguous().to(DEV)
    yr = torch.empty((case.n, case.p, case.q, case.k), device=DEV)
    yi = torch.empty_like(yr)
    ws_bytes = lib.ccv_forward_workspace_bytes(ctypes.byref(shp))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
    ccv_abi.check(lib.ccv_forward(_ptr(xr), _ptr(xi), _ptr(wr_k), _ptr(wi_k), _ptr(yr), _ptr(yi),
                                  ctypes.byref(shp), _ptr(ws), ws_bytes, _stream()), "forward")
    torch.cuda.synchronize()
    y = oracle.planar_nhwc_to_complex_nchw(yr, yi).cpu()
    assert oracle.rel_frobenius(y, y64) <= TF32_TOL
    # Same packed image as the KCRS path -> bitwise identical results.
    packed = abi_prepack(case, torch.from_numpy(wr), torch.from_numpy(wi))
    assert torch.equal(y, abi_fprop_planar(case, xt, packed))


# ----------------------------------------------------------------- BASELINE configs
BATCH1 = [c for c in BASELINE_CASES if c[1].n == 1]
BATCHED = [c for c in BASELINE_CASES if c[1].n > 1]


@pytest.mark.parametrize("name,case,std,precs", BATCH1, ids=[c[0] for c in BATCH1])
def test_baseline_batch1_full(name, case, std, precs):
    x, wr, wi = oracle.make_inputs(case, input_std=std)
    packed = abi_prepack(case, wr, wi)
    y = abi_fprop_complex(case, x, packed, poison=True)
    ref = oracle.oracle_fp64(case, x, wr, wi)
    err = oracle.rel_frobenius(y, ref)
    assert err <= TF32_TOL, (name, err)


@pytest.mark.parametrize("name,case,std,precs", BATCHED, ids=[c[0] for c in BATCHED])
def test_baseline_batched_sampled_images(name, case, std, precs):
    """Full-size problem on the GPU; the fp64 oracle checks the first and last
    image (each output image depends only on its own input image)."""
    x, wr, wi = oracle.make_inputs(case, input_std=std)
    packed = abi_prepack(case, wr, wi)
    y = abi_fprop_complex(case, x, packed, poison=True)
    assert not torch.isnan(y.real).any()
    for img in (0, case.n - 1):
        sub = oracle.ConvCase(1, case.c, case.h, case.w, case.k, case.r, case.s,
                              case.stride_h, case.stride_w, case.pad_h, case.pad_w)
        ref = oracle.oracle_fp64(sub, x[img:img + 1], wr, wi)
        err = oracle.rel_frobenius(y[img:img + 1], ref)
        assert err <= TF32_TOL, (name, img, err)


def test_linearity_full_size():
    """conv(a*x1 + x2) == a*conv(x1) + conv(x2) at a BASELINE size (stride-2 layer)."""
    case = [c for c in BASELINE_CASES if c[0].startswith("b32_s2")][0][1]
    case = oracle.ConvCase(8, case.c, case.h, case.w, case.k, case.r, case.s,
                           case.stride_h, case.stride_w, case.pad_h, case.pad_w)
    x1, wr, wi = oracle.make_inputs(case, input_seed=3)
    x2, _, _ = oracle.make_inputs(case, input_seed=4)
    packed = abi_prepack(case, wr, wi)
    a = 0.5  # power of two: exact scaling
    y1 = abi_fprop_complex(case, x1, packed)
    y2 = abi_fprop_complex(case, x2, packed)
    y12 = abi_fprop_complex(case, a * x1 + x2, packed)
    assert oracle.rel_frobenius(y12, a * y1 + y2) <= 2 * TF32_TOL


def test_deterministic_repeat():
    case = BASELINE_CASES[0][1]
    x, wr, wi = oracle.make_inputs(case)
    packed = abi_prepack(case, wr, wi)
    y1 = abi_fprop_complex(case, x, packed)
    y2 = abi_fprop_complex(case, x, packed)
    assert torch.equal(y1, y2)


# ----------------------------------------------------------------- edge shapes
EDGE = [
    oracle.ConvCase(1, 4, 1, 1, 4, 1, 1, 1, 1, 0, 0),        # 1x1 image, tiny channels
    oracle.ConvCase(3, 20, 9, 13, 36, 3, 3, 1, 1, 1, 1),     # C, K not tile multiples
    oracle.ConvCase(2, 16, 17, 19, 132, 3, 3, 1, 1, 1, 1),   # K = 128 + 4: two N tiles
    oracle.ConvCase(1, 8, 30, 30, 8, 7, 7, 1, 1, 3, 3),      # 7x7 taps
    oracle.ConvCase(2, 12, 15, 15, 16, 5, 5, 2, 2, 2, 2),    # 5x5 stride 2
    oracle.ConvCase(1, 8, 40, 9, 12, 3, 3, 3, 1, 0, 2),      # stride 3 x 1, asymmetric pad
    oracle.ConvCase(5, 36, 7, 7, 68, 1, 1, 1, 1, 0, 0),      # flat 1x1, ragged M
    oracle.ConvCase(1, 8, 6, 6, 8, 1, 1, 2, 2, 1, 1),        # 1x1 with stride and pad
    oracle.ConvCase(1, 64, 3, 3, 64, 3, 3, 1, 1, 0, 0),      # output 1x1
]


@pytest.mark.parametrize("case", EDGE, ids=[f"n{c.n}c{c.c}h{c.h}w{c.w}k{c.k}r{c.r}s{c.s}st{c.stride_h}{c.stride_w}p{c.pad_h}{c.pad_w}" for c in EDGE])
def test_edge_shapes(case):
    x, wr, wi = oracle.make_inputs(case, input_seed=7)
    packed = abi_prepack(case, wr, wi)
    y = abi_fprop_planar(case, x, packed, poison=True)
    assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any()
    ref = oracle.oracle_fp64(case, x, wr, wi)
    assert oracle.rel_frobenius(y, ref) <= TF32_TOL


# ----------------------------------------------------------------- failure path
def test_bounded_wait_selftest_reports_timeout():
    """A wait on a barrier nothing arrives on gives up and reports status;
    the context stays usable afterwards."""
    lib = ccv_abi.load()
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    ccv_abi.check(lib.ccv_selftest_bounded_wait(_ptr(st), _stream()), "selftest")
    torch.cuda.synchronize()
    assert st.item() == ccv_abi.CCV_ERR_DEVICE_TIMEOUT
    # The context still works.
    case = EDGE[0]
    x, wr, wi = oracle.make_inputs(case)
    packed = abi_prepack(case, wr, wi)
    y = abi_fprop_planar(case, x, packed)
    assert oracle.rel_frobenius(y, oracle.oracle_fp64(case, x, wr, wi)) <= TF32_TOL
