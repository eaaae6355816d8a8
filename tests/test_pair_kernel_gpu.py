"""All kernel families on the same problems: the CTA-pair kernels
(ccv_fprop2.cu tap, ccv_fprop2h.cu halo) are pinned with CCV_FORCE_KERNEL=2 / CCV_HALO on the golden and edge
shapes that would normally go to the single-CTA kernel, and against the
fp64 oracle; and the single-CTA kernel (CCV_FORCE_KERNEL=1) on a shape that
would normally go to the pair kernel."""

import ctypes
import os

import pytest
import torch

import ccv_abi
import oracle
from test_oracle import CASES as GOLDEN_CASES
from test_parity_gpu import EDGE, TF32_TOL, abi_fprop_complex, abi_fprop_planar, abi_prepack

pytestmark = pytest.mark.gpu


@pytest.fixture
def force_kernel():
    """Pin the kernel family (1 = single CTA, 2 = CTA pair; 'halo' = CTA pair
    with halo reuse, 'halo_fused' = the same reading complex64 input through
    its converter warps, 'tap' = CTA pair without halo reuse) through the
    library's env knobs."""
    keys = ("CCV_FORCE_KERNEL", "CCV_HALO", "CCV_CD", "CCV_FUSED", "CCV_SUBBOX", "CCV_STREAMK")
    old = {k: os.environ.get(k) for k in keys}
    # These tests pin the planar-operand kernels; the complex-direct kernel
    # has its own tests.  Whole tiles only, so every complex64 path (layout
    # pass, converter clusters, converter warps) sums like the planar one.
    os.environ["CCV_CD"] = "0"
    os.environ["CCV_STREAMK"] = "0"

    def set_(v):
        os.environ.pop("CCV_FUSED", None)
        os.environ.pop("CCV_SUBBOX", None)
        if v == "halo_fused":
            # The converter-warp kernel has one 128-pixel box per CTA; pin the
            # planar reference to the same tiling (same summation order).
            os.environ["CCV_FUSED"] = "1"
            os.environ["CCV_SUBBOX"] = "0"
            v = "halo"
        if v == "halo":
            os.environ["CCV_FORCE_KERNEL"] = "2"
            os.environ["CCV_HALO"] = "1"
        elif v == "tap":
            os.environ["CCV_FORCE_KERNEL"] = "2"
            os.environ["CCV_HALO"] = "0"
        else:
            os.environ["CCV_FORCE_KERNEL"] = str(v)
            os.environ.pop("CCV_HALO", None)

    yield set_
    for k, v in old.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v


@pytest.mark.parametrize("name,case,x,wr,wi,y32,y64", GOLDEN_CASES, ids=[c[0] for c in GOLDEN_CASES])
@pytest.mark.parametrize("family", ["tap", "halo", "halo_fused"])
def test_pair_kernel_golden(force_kernel, family, name, case, x, wr, wi, y32, y64):
    force_kernel(family)
    packed = abi_prepack(case, torch.from_numpy(wr), torch.from_numpy(wi))
    y = abi_fprop_planar(case, torch.from_numpy(x), packed, poison=True)
    assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any()
    assert oracle.rel_frobenius(y, y64) <= TF32_TOL
    yc = abi_fprop_complex(case, torch.from_numpy(x), packed, poison=True)
    assert torch.equal(yc, y.to(torch.complex64))


@pytest.mark.parametrize("case", EDGE, ids=[str(i) for i in range(len(EDGE))])
@pytest.mark.parametrize("family", ["tap", "halo", "halo_fused"])
def test_pair_kernel_edges(force_kernel, family, case):
    force_kernel(family)
    x, wr, wi = oracle.make_inputs(case, input_seed=9)
    packed = abi_prepack(case, wr, wi)
    y = abi_fprop_planar(case, x, packed, poison=True)
    assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any()
    assert oracle.rel_frobenius(y, oracle.oracle_fp64(case, x, wr, wi)) <= TF32_TOL


@pytest.mark.parametrize("family", [1, "tap", "halo", "halo_fused"])
def test_families_agree_on_a_mid_size_problem(force_kernel, family):
    case = oracle.ConvCase(6, 64, 30, 30, 132, 3, 3, 1, 1, 1, 1)
    x, wr, wi = oracle.make_inputs(case, input_seed=21)
    packed = abi_prepack(case, wr, wi)
    force_kernel(family)
    y = abi_fprop_complex(case, x, packed, poison=True)
    sub = oracle.ConvCase(1, 64, 30, 30, 132, 3, 3, 1, 1, 1, 1)
    for img in (0, 5):
        ref = oracle.oracle_fp64(sub, x[img:img + 1], wr, wi)
        assert oracle.rel_frobenius(y[img:img + 1], ref) <= TF32_TOL


@pytest.mark.parametrize("name,case,x,wr,wi,y32,y64", GOLDEN_CASES, ids=[c[0] for c in GOLDEN_CASES])
def test_converter_warps_3xtf32(force_kernel, name, case, x, wr, wi, y32, y64):
    """The converter warps' hi/lo split (3xTF32) against the layout pass's."""
    p3 = ccv_abi.CCV_PRECISION_3XTF32
    packed = abi_prepack(case, torch.from_numpy(wr), torch.from_numpy(wi), precision=p3)
    xt = torch.from_numpy(x)
    force_kernel("halo")
    os.environ["CCV_SUBBOX"] = "0"
    y = abi_fprop_complex(case, xt, packed, precision=p3, poison=True)
    force_kernel("halo_fused")
    yf = abi_fprop_complex(case, xt, packed, precision=p3, poison=True)
    assert torch.equal(yf, y)
    assert oracle.rel_frobenius(yf, y64) <= 1e-5


def test_converter_warps_kernel_name(force_kernel):
    # 16x8 boxes: the 144-row halo slot fits the converter warps' unit budget.
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(oracle.ConvCase(2, 64, 56, 56, 128, 3, 3, 1, 1, 1, 1))
    force_kernel("halo_fused")
    assert lib.ccv_fprop_complex_kernel(ctypes.byref(shp), 0).decode() == "halo_pair_converter_warps"
    force_kernel("halo")
    assert lib.ccv_fprop_complex_kernel(ctypes.byref(shp), 0).decode() == "layout_pass+halo_pair"


@pytest.mark.parametrize("name,case,x,wr,wi,y32,y64", GOLDEN_CASES, ids=[c[0] for c in GOLDEN_CASES])
def test_two_subbox_tiles(force_kernel, name, case, x, wr, wi, y32, y64):
    """Halo kernel with two 128-pixel sub-boxes per CTA (KT <= 64) against the
    one-box kernel without stream-K: identical summation order."""
    force_kernel("halo")
    packed = abi_prepack(case, torch.from_numpy(wr), torch.from_numpy(wi))
    xt = torch.from_numpy(x)
    y2 = abi_fprop_planar(case, xt, packed, poison=True)
    assert oracle.rel_frobenius(y2, y64) <= TF32_TOL
    os.environ["CCV_SUBBOX"] = "0"
    y1 = abi_fprop_planar(case, xt, packed, poison=True)
    assert torch.equal(y1, y2)
