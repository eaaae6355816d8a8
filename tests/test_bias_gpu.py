"""Complex bias (an extension: the reference rejects bias=True at
modules.py:73-74) on every kernel family and epilogue path, through the C ABI
(ccv_fprop_planar_bias / ccv_fprop_complex_bias) and through
ComplexConv2d(bias=True).  The oracle is the fp64 four-conv of
benchmarks/baseline.py:5-9 plus bias_real[k] + 1j * bias_imag[k] per output
channel (oracle.oracle_fp64).  The bias must be added exactly once: on final
sums, never on split-K / stream-K partials.
"""

import ctypes
import os

import pytest
import torch

import ccv_abi
import oracle
from test_parity_gpu import DEV, TF32_TOL, _ptr, _stream, abi_prepack, device_status

pytestmark = pytest.mark.gpu

C = oracle.ConvCase
X3_TOL = 1e-5

# (id, case, knobs): each pins one kernel family / epilogue path.
PATHS = [
    ("single_cta_splitk", C(1, 64, 14, 14, 128, 3, 3, 1, 1, 1, 1), {}),
    ("single_cta_whole", C(1, 64, 14, 14, 128, 3, 3, 1, 1, 1, 1), {"CCV_SPLITK": "1"}),
    ("single_cta_flat", C(2, 64, 9, 9, 36, 1, 1, 1, 1, 0, 0), {"CCV_FORCE_KERNEL": "1"}),
    ("tap_pair", C(2, 32, 23, 19, 132, 3, 3, 2, 2, 1, 1),
     {"CCV_FORCE_KERNEL": "2", "CCV_HALO": "0", "CCV_STREAMK": "0"}),
    ("tap_pair_flat", C(3, 64, 20, 20, 96, 1, 1, 1, 1, 0, 0),
     {"CCV_FORCE_KERNEL": "2", "CCV_HALO": "0", "CCV_STREAMK": "0"}),
    ("halo_pair", C(2, 64, 30, 26, 132, 3, 3, 1, 1, 1, 1),
     {"CCV_FORCE_KERNEL": "2", "CCV_HALO": "1", "CCV_STREAMK": "0"}),
    ("halo_pair_subbox", C(2, 32, 40, 40, 64, 3, 3, 1, 1, 1, 1),
     {"CCV_FORCE_KERNEL": "2", "CCV_HALO": "1", "CCV_STREAMK": "0"}),
    ("halo_stream_k", C(3, 64, 33, 29, 128, 3, 3, 1, 1, 1, 1),
     {"CCV_FORCE_KERNEL": "2", "CCV_HALO": "1", "CCV_STREAMK": "1", "CCV_MAX_CLUSTERS": "7",
      "CCV_SUBBOX": "0"}),
    ("tap_stream_k", C(3, 64, 33, 33, 128, 3, 3, 2, 2, 1, 1),
     {"CCV_FORCE_KERNEL": "2", "CCV_HALO": "0", "CCV_STREAMK": "1", "CCV_MAX_CLUSTERS": "3"}),
    ("halo_layout_warps", C(3, 64, 28, 28, 128, 3, 3, 1, 1, 1, 1),
     {"CCV_FORCE_KERNEL": "2", "CCV_HALO": "1", "CCV_LW": "1"}),
    ("tap_layout_warps", C(3, 64, 28, 28, 96, 1, 1, 1, 1, 0, 0),
     {"CCV_FORCE_KERNEL": "2", "CCV_HALO": "0", "CCV_LW": "1"}),
    ("planar_no_tma_store", C(2, 64, 30, 26, 132, 3, 3, 1, 1, 1, 1),
     {"CCV_FORCE_KERNEL": "2", "CCV_HALO": "1", "CCV_TMA_STORE": "0", "CCV_STREAMK": "0"}),
]
KEYS = ("CCV_FORCE_KERNEL", "CCV_HALO", "CCV_STREAMK", "CCV_MAX_CLUSTERS", "CCV_SUBBOX",
        "CCV_LW", "CCV_SPLITK", "CCV_TMA_STORE")


@pytest.fixture
def knobs():
    old = {k: os.environ.get(k) for k in KEYS}

    def set_(kv):
        for k in KEYS:
            os.environ.pop(k, None)
        os.environ.update(kv)

    yield set_
    for k, v in old.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v
    torch.cuda.synchronize()
    assert device_status() == 0


def make_bias(k, seed):
    g = torch.Generator().manual_seed(seed)
    br = torch.rand(k, generator=g) * 2 - 1
    bi = torch.rand(k, generator=g) * 2 - 1
    return br, bi


def fprop_planar_bias(case, x, packed, br, bi, precision):
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    xr = x.real.permute(0, 2, 3, 1).contiguous().to(DEV)
    xi = x.imag.permute(0, 2, 3, 1).contiguous().to(DEV)
    yr = torch.full((case.n, case.p, case.q, case.k), float("nan"), device=DEV)
    yi = torch.full_like(yr, float("nan"))
    bdr, bdi = br.to(DEV), bi.to(DEV)
    ws_bytes = lib.ccv_fprop_planar_workspace_bytes(ctypes.byref(shp), precision)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=DEV)
    ccv_abi.check(lib.ccv_fprop_planar_bias(_ptr(xr), _ptr(xi), _ptr(packed), _ptr(bdr), _ptr(bdi),
                                            _ptr(yr), _ptr(yi), ctypes.byref(shp), precision,
                                            _ptr(ws) if ws_bytes else None, ws_bytes, _stream()),
                  "fprop_planar_bias")
    torch.cuda.synchronize()
    return oracle.planar_nhwc_to_complex_nchw(yr, yi).cpu()


def fprop_complex_bias(case, x, packed, br, bi, precision):
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    xd = x.to(DEV).contiguous()
    y = torch.full((case.n, case.k, case.p, case.q), float("nan"), dtype=torch.complex64,
                   device=DEV)
    bdr, bdi = br.to(DEV), bi.to(DEV)
    ws_bytes = lib.ccv_fprop_complex_workspace_bytes(ctypes.byref(shp), precision)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=DEV)
    ccv_abi.check(lib.ccv_fprop_complex_bias(_ptr(xd), _ptr(packed), _ptr(bdr), _ptr(bdi), _ptr(y),
                                             ctypes.byref(shp), precision, _ptr(ws), ws_bytes,
                                             _stream()), "fprop_complex_bias")
    torch.cuda.synchronize()
    return y.cpu()


@pytest.mark.parametrize("name,case,kv", PATHS, ids=[p[0] for p in PATHS])
def test_bias_every_path_tf32(knobs, name, case, kv):
    knobs(kv)
    x, wr, wi = oracle.make_inputs(case, input_seed=31)
    br, bi = make_bias(case.k, 5)
    packed = abi_prepack(case, wr, wi)
    ref = oracle.oracle_fp64(case, x, wr, wi, br, bi)
    yp = fprop_planar_bias(case, x, packed, br, bi, ccv_abi.CCV_PRECISION_TF32)
    yc = fprop_complex_bias(case, x, packed, br, bi, ccv_abi.CCV_PRECISION_TF32)
    for y in (yp, yc):
        assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any(), name
        assert oracle.rel_frobenius(y, ref) <= TF32_TOL, name
    # The bias is added once: against the bias-free result, only the bias
    # (plus one fp32 rounding of the sum) remains.
    zero = torch.zeros(case.k)
    y0 = fprop_planar_bias(case, x, packed, zero, zero, ccv_abi.CCV_PRECISION_TF32)
    diff = (yp - y0).to(torch.complex128)
    b = torch.complex(br.double(), bi.double()).view(1, -1, 1, 1)
    scale = y0.abs().max().item() + b.abs().max().item()
    assert (diff - b).abs().max().item() <= 4 * 2.0 ** -23 * scale, name


@pytest.mark.parametrize("name,case,kv", [PATHS[5], PATHS[7], PATHS[8], PATHS[9]],
                         ids=[PATHS[i][0] for i in (5, 7, 8, 9)])
def test_bias_3xtf32(knobs, name, case, kv):
    knobs(kv)
    p3 = ccv_abi.CCV_PRECISION_3XTF32
    x, wr, wi = oracle.make_inputs(case, input_seed=32)
    br, bi = make_bias(case.k, 6)
    packed = abi_prepack(case, wr, wi, precision=p3)
    ref = oracle.oracle_fp64(case, x, wr, wi, br, bi)
    for y in (fprop_planar_bias(case, x, packed, br, bi, p3),
              fprop_complex_bias(case, x, packed, br, bi, p3)):
        assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any(), name
        assert oracle.rel_frobenius(y, ref) <= X3_TOL, name


def test_bias_rejects_half_pair():
    lib = ccv_abi.load()
    case = C(1, 8, 8, 8, 8, 3, 3, 1, 1, 1, 1)
    shp = ccv_abi.shape_of(case)
    buf = torch.zeros(4096, device=DEV)
    p = _ptr(buf)
    rc = lib.ccv_fprop_planar_bias(p, p, p, p, None, p, p, ctypes.byref(shp), 0, None, 0,
                                   _stream())
    assert rc == ccv_abi.CCV_ERR_INVALID_ARGUMENT
    assert "both" in ccv_abi.last_error()


@pytest.mark.parametrize("precision", ["tf32", "3xtf32"])
@pytest.mark.parametrize("case", [C(2, 32, 20, 20, 64, 3, 3, 1, 1, 1, 1),
                                  C(1, 128, 14, 14, 256, 3, 3, 1, 1, 1, 1),
                                  C(2, 64, 17, 17, 40, 3, 3, 2, 2, 1, 1)],
                         ids=["b2_32_64_20", "b1_128_256_14", "b2_s2_ragged"])
def test_module_bias(precision, case):
    from complex_conv2d import ComplexConv2d
    x, wr, wi = oracle.make_inputs(case, input_seed=41)
    layer = ComplexConv2d(case.c, case.k, (case.r, case.s), stride=(case.stride_h, case.stride_w),
                          padding=(case.pad_h, case.pad_w), bias=True, device=DEV,
                          precision=precision)
    with torch.no_grad():
        layer.weight_real.copy_(wr)
        layer.weight_imag.copy_(wi)
    ref = oracle.oracle_fp64(case, x, wr, wi, layer.bias_real, layer.bias_imag)
    tol = TF32_TOL if precision == "tf32" else X3_TOL
    with torch.no_grad():
        y = layer(x.to(DEV))
        yr, yi = layer.forward_planar(x.real.permute(0, 2, 3, 1).contiguous().to(DEV),
                                      x.imag.permute(0, 2, 3, 1).contiguous().to(DEV))
    torch.cuda.synchronize()
    assert oracle.rel_frobenius(y.cpu(), ref) <= tol
    assert oracle.rel_frobenius(oracle.planar_nhwc_to_complex_nchw(yr, yi).cpu(), ref) <= tol
    # state_dict round trip into a fresh layer gives identical outputs.
    other = ComplexConv2d(case.c, case.k, (case.r, case.s), stride=(case.stride_h, case.stride_w),
                          padding=(case.pad_h, case.pad_w), bias=True, device=DEV,
                          precision=precision)
    other.load_state_dict(layer.state_dict())
    with torch.no_grad():
        assert torch.equal(other(x.to(DEV)), y)
        # A bias edit is seen by the next call (the bias is not cached).
        layer.bias_imag.add_(1.0)
        y2 = layer(x.to(DEV))
    assert oracle.rel_frobenius((y2 - y).cpu(), torch.full_like(ref, 1j)) <= 1e-6
