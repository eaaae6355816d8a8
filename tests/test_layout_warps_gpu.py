"""forward() through layout warps (ccv_layout_role.cuh): two extra warps in
every CTA of the halo or tap pair kernel convert complex64 NCHW into the fp32
NHWC workspace planes while the MMA runs, in one launch.

Checked against the fp64 oracle (TF32 and 3xTF32 bars) and bitwise against
the two-launch path (layout pass + the same kernel), with the workspace
filled with NaN before every call (a plane read before its image was written
would show), repeated calls (the library-owned counters are left zero),
ragged pixel counts (H*W not a multiple of 32), channel counts that are not
multiples of 32, one image, and the two-sub-box tiles.
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
CASES = [
    ("b8_128_56", C(8, 128, 56, 56, 128, 3, 3, 1, 1, 1, 1)),
    ("k64_subbox", C(4, 64, 40, 40, 64, 3, 3, 1, 1, 1, 1)),
    ("ragged_30x41_c36_k20", C(6, 36, 30, 41, 20, 3, 3, 1, 1, 1, 1)),
    ("5x5_p2_k132", C(3, 48, 26, 34, 132, 5, 5, 1, 1, 2, 2)),
    ("one_image_7x9_c8", C(1, 8, 7, 9, 40, 3, 3, 1, 1, 1, 1)),
    ("k32_p0_3x1", C(5, 96, 23, 17, 32, 3, 1, 1, 1, 0, 0)),
]


@pytest.fixture
def knobs():
    keys = ("CCV_FORCE_KERNEL", "CCV_HALO", "CCV_LW", "CCV_STREAMK", "CCV_SUBBOX")
    old = {k: os.environ.get(k) for k in keys}
    os.environ["CCV_FORCE_KERNEL"] = "2"
    os.environ["CCV_HALO"] = "1"
    os.environ.pop("CCV_SUBBOX", None)
    # Layout warps wherever they apply (by default only for grids of two or
    # more waves of tiles).
    os.environ["CCV_LW"] = "1"
    # Whole tiles on the comparison path too (same summation order).
    os.environ["CCV_STREAMK"] = "0"
    yield
    for k, v in old.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v
    torch.cuda.synchronize()
    assert device_status() == 0, "a bounded in-kernel wait ran out"


def kernel_name(case, precision=ccv_abi.CCV_PRECISION_TF32):
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    return lib.ccv_fprop_complex_kernel(ctypes.byref(shp), precision).decode()


def fprop_complex_nan_ws(case, x, packed, precision):
    """ccv_fprop_complex with a NaN-filled workspace and a NaN-filled output."""
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    xd = x.to(DEV).contiguous()
    y = torch.full((case.n, case.k, case.p, case.q), float("nan"), dtype=torch.complex64,
                   device=DEV)
    ws_bytes = lib.ccv_fprop_complex_workspace_bytes(ctypes.byref(shp), precision)
    ws = torch.full((max(ws_bytes, 16),), 0xFF, dtype=torch.uint8, device=DEV)
    ccv_abi.check(lib.ccv_fprop_complex(_ptr(xd), _ptr(packed), _ptr(y), ctypes.byref(shp),
                                        precision, _ptr(ws), ws_bytes, _stream()),
                  "fprop_complex")
    torch.cuda.synchronize()
    return y.cpu()


def launches(case, precision):
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    k = ctypes.c_int(0)
    ccv_abi.check(lib.ccv_fprop_kernel_launches(ctypes.byref(shp), precision, 1, ctypes.byref(k)),
                  "launches")
    return k.value


@pytest.mark.parametrize("name,case", CASES, ids=[c[0] for c in CASES])
def test_layout_warps_tf32(knobs, name, case):
    prec = ccv_abi.CCV_PRECISION_TF32
    assert kernel_name(case) == "halo_pair_layout_warps"
    assert launches(case, prec) == 1
    x, wr, wi = oracle.make_inputs(case, input_seed=61)
    packed = abi_prepack(case, wr, wi)
    y = fprop_complex_nan_ws(case, x, packed, prec)
    assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any()
    sub = C(1, case.c, case.h, case.w, case.k, case.r, case.s, 1, 1, case.pad_h, case.pad_w)
    for img in sorted({0, case.n - 1}):
        ref = oracle.oracle_fp64(sub, x[img:img + 1], wr, wi)
        assert oracle.rel_frobenius(y[img:img + 1], ref) <= TF32_TOL, img
    # Repeated calls give the same bits (counters left zero by each call).
    for _ in range(2):
        assert torch.equal(y, fprop_complex_nan_ws(case, x, packed, prec))
    # The two-launch path: layout pass, then the same kernel.
    os.environ["CCV_LW"] = "0"
    assert kernel_name(case) == "layout_pass+halo_pair"
    assert launches(case, prec) == 2
    assert torch.equal(y, fprop_complex_nan_ws(case, x, packed, prec))


@pytest.mark.parametrize("name,case", [CASES[0], CASES[2]], ids=[CASES[0][0], CASES[2][0]])
def test_layout_warps_3xtf32(knobs, name, case):
    prec = ccv_abi.CCV_PRECISION_3XTF32
    assert kernel_name(case, prec) == "halo_pair_layout_warps"
    x, wr, wi = oracle.make_inputs(case, input_seed=62)
    packed = abi_prepack(case, wr, wi, precision=prec)
    y = fprop_complex_nan_ws(case, x, packed, prec)
    os.environ["CCV_LW"] = "0"
    assert torch.equal(y, fprop_complex_nan_ws(case, x, packed, prec))
    sub = C(1, case.c, case.h, case.w, case.k, case.r, case.s, 1, 1, case.pad_h, case.pad_w)
    for img in (0, case.n - 1):
        ref = oracle.oracle_fp64(sub, x[img:img + 1], wr, wi)
        assert oracle.rel_frobenius(y[img:img + 1], ref) <= 1e-5, img


TAP_CASES = [
    ("s2_c64_k128", C(4, 64, 38, 38, 128, 3, 3, 2, 2, 1, 1)),
    ("s2_ragged_c36_k20", C(3, 36, 21, 27, 20, 3, 3, 2, 2, 1, 1)),
    ("1x1_flat_c96_k160", C(5, 96, 14, 14, 160, 1, 1, 1, 1, 0, 0)),
    # 7x7 images: one 128-row tile spans three images.
    ("1x1_flat_7x7", C(9, 64, 7, 7, 64, 1, 1, 1, 1, 0, 0)),
    ("1x1_s2", C(4, 32, 20, 20, 48, 1, 1, 2, 2, 0, 0)),
]


@pytest.mark.parametrize("name,case", TAP_CASES, ids=[c[0] for c in TAP_CASES])
@pytest.mark.parametrize("prec", [ccv_abi.CCV_PRECISION_TF32, ccv_abi.CCV_PRECISION_3XTF32],
                         ids=["tf32", "3xtf32"])
def test_layout_warps_tap_kernel(knobs, name, case, prec):
    assert kernel_name(case, prec) == "tap_pair_layout_warps"
    assert launches(case, prec) == 1
    x, wr, wi = oracle.make_inputs(case, input_seed=64)
    packed = abi_prepack(case, wr, wi, precision=prec)
    y = fprop_complex_nan_ws(case, x, packed, prec)
    assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any()
    ref = oracle.oracle_fp64(case, x, wr, wi)
    tol = TF32_TOL if prec == ccv_abi.CCV_PRECISION_TF32 else 1e-5
    assert oracle.rel_frobenius(y, ref) <= tol
    assert torch.equal(y, fprop_complex_nan_ws(case, x, packed, prec))
    os.environ["CCV_LW"] = "0"
    assert kernel_name(case, prec) == "layout_pass+tap_pair"
    assert torch.equal(y, fprop_complex_nan_ws(case, x, packed, prec))


def test_layout_warps_not_taken(knobs):
    os.environ.pop("CCV_FORCE_KERNEL")
    os.environ.pop("CCV_HALO")
    # Batch-1 layers run the single-CTA kernel: layout pass first.
    assert kernel_name(C(1, 64, 28, 28, 128, 3, 3, 1, 1, 1, 1)) == "layout_pass+single_cta"
    # Default: inputs of at least 96 MB, at least two waves of tiles and
    # 500 flops per input byte.
    os.environ.pop("CCV_LW")
    assert kernel_name(C(8, 128, 56, 56, 128, 3, 3, 1, 1, 1, 1)) == "layout_pass+halo_pair"
    assert kernel_name(C(16, 128, 56, 56, 128, 3, 3, 1, 1, 1, 1)) == "layout_pass+halo_pair"
    assert kernel_name(C(32, 128, 56, 56, 128, 3, 3, 1, 1, 1, 1)) == "halo_pair_layout_warps"
    assert kernel_name(C(64, 128, 56, 56, 128, 3, 3, 1, 1, 1, 1)) == "halo_pair_layout_warps"
    assert kernel_name(C(8, 64, 320, 320, 64, 3, 3, 1, 1, 1, 1)) == "halo_pair_layout_warps"
    assert kernel_name(C(32, 64, 56, 56, 64, 3, 3, 1, 1, 1, 1)) == "layout_pass+halo_pair"
    assert kernel_name(C(128, 256, 28, 28, 1024, 1, 1, 1, 1, 0, 0)) == "tap_pair_layout_warps"
    assert kernel_name(C(32, 256, 28, 28, 1024, 1, 1, 1, 1, 0, 0)) == "layout_pass+tap_pair"
    # Stride 2 at C = 64: too few flops per input byte (TF32), enough for 3xTF32.
    s2 = C(32, 64, 112, 112, 128, 3, 3, 2, 2, 1, 1)
    assert kernel_name(s2) == "layout_pass+tap_pair"
    assert kernel_name(s2, ccv_abi.CCV_PRECISION_3XTF32) == "tap_pair_layout_warps"


@pytest.mark.parametrize("name,case", [CASES[0], ("b3_c64_ragged", C(3, 64, 45, 29, 96, 3, 3, 1, 1, 1, 1))],
                         ids=[CASES[0][0], "b3_c64_ragged"])
def test_layout_warps_with_stream_k(knobs, name, case):
    # Stream-K forced (CCV_STREAMK=1: a partial last wave is split; layout-warp
    # launches skip the split by default): the split range runs first, so the
    # layout warps convert its images first.  Same plan, same sums as the
    # layout pass + kernel under the same setting.
    os.environ["CCV_STREAMK"] = "1"
    prec = ccv_abi.CCV_PRECISION_TF32
    x, wr, wi = oracle.make_inputs(case, input_seed=63)
    packed = abi_prepack(case, wr, wi)
    y = fprop_complex_nan_ws(case, x, packed, prec)
    assert torch.equal(y, fprop_complex_nan_ws(case, x, packed, prec))
    sub = C(1, case.c, case.h, case.w, case.k, case.r, case.s, 1, 1, case.pad_h, case.pad_w)
    for img in (0, case.n - 1):
        ref = oracle.oracle_fp64(sub, x[img:img + 1], wr, wi)
        assert oracle.rel_frobenius(y[img:img + 1], ref) <= TF32_TOL, img
    os.environ["CCV_LW"] = "0"
    assert torch.equal(y, fprop_complex_nan_ws(case, x, packed, prec))


@pytest.mark.parametrize("name,case", [CASES[0], TAP_CASES[3]], ids=[CASES[0][0], TAP_CASES[3][0]])
def test_layout_warps_without_prefix(knobs, name, case):
    # CCV_LW_PREFIX=0: only the two layout warps convert (no all-warp phase
    # before the roles); same planes, same bits.
    prec = ccv_abi.CCV_PRECISION_TF32
    x, wr, wi = oracle.make_inputs(case, input_seed=65)
    packed = abi_prepack(case, wr, wi)
    y = fprop_complex_nan_ws(case, x, packed, prec)
    os.environ["CCV_LW_PREFIX"] = "0"
    try:
        assert torch.equal(y, fprop_complex_nan_ws(case, x, packed, prec))
    finally:
        os.environ.pop("CCV_LW_PREFIX", None)
    # The warp-run prefix instead of the TMA one (even W, TF32): same bits.
    os.environ["CCV_LW_TMA"] = "0"
    try:
        assert torch.equal(y, fprop_complex_nan_ws(case, x, packed, prec))
    finally:
        os.environ.pop("CCV_LW_TMA", None)
    os.environ["CCV_LW"] = "0"
    assert torch.equal(y, fprop_complex_nan_ws(case, x, packed, prec))


def fprop_planar_nan_ws(case, x, packed, precision):
    """ccv_fprop_planar with a NaN-filled workspace; returns complex64 NCHW."""
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    xr = x.real.permute(0, 2, 3, 1).contiguous().to(DEV)
    xi = x.imag.permute(0, 2, 3, 1).contiguous().to(DEV)
    yr = torch.full((case.n, case.p, case.q, case.k), float("nan"), device=DEV)
    yi = torch.full((case.n, case.p, case.q, case.k), float("nan"), device=DEV)
    ws_bytes = lib.ccv_fprop_planar_workspace_bytes(ctypes.byref(shp), precision)
    ws = torch.full((max(ws_bytes, 16),), 0xFF, dtype=torch.uint8, device=DEV)
    ccv_abi.check(lib.ccv_fprop_planar(_ptr(xr), _ptr(xi), _ptr(packed), _ptr(yr), _ptr(yi),
                                       ctypes.byref(shp), precision, _ptr(ws), ws_bytes,
                                       _stream()), "fprop_planar")
    torch.cuda.synchronize()
    return oracle.planar_nhwc_to_complex_nchw(yr, yi).cpu()


def planar_launches(case, precision):
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    k = ctypes.c_int(0)
    ccv_abi.check(lib.ccv_fprop_kernel_launches(ctypes.byref(shp), precision, 0, ctypes.byref(k)),
                  "launches")
    return k.value


PLANAR_3X_CASES = [CASES[0], CASES[1], CASES[2], TAP_CASES[0], TAP_CASES[3]]


@pytest.mark.parametrize("name,case", PLANAR_3X_CASES, ids=[c[0] for c in PLANAR_3X_CASES])
def test_layout_warps_planar_3xtf32(knobs, name, case):
    # forward_planar() at 3xTF32: the layout warps split the caller's fp32
    # planes into the hi/remainder workspace planes in the convolution
    # launch (one launch); the same bits as the split pass + kernel.
    prec = ccv_abi.CCV_PRECISION_3XTF32
    assert planar_launches(case, prec) == 1
    x, wr, wi = oracle.make_inputs(case, input_seed=66)
    packed = abi_prepack(case, wr, wi, precision=prec)
    y = fprop_planar_nan_ws(case, x, packed, prec)
    assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any()
    ref = oracle.oracle_fp64(case, x, wr, wi)
    assert oracle.rel_frobenius(y, ref) <= 1e-5
    assert torch.equal(y, fprop_planar_nan_ws(case, x, packed, prec))
    os.environ["CCV_LW"] = "0"
    assert planar_launches(case, prec) == 2
    assert torch.equal(y, fprop_planar_nan_ws(case, x, packed, prec))
