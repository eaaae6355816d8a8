"""All kernel families on the same problems: the CTA-pair kernels
(ccv_fprop2.cu tap, ccv_fprop2h.cu halo) are pinned with CCV_FORCE_KERNEL=2 / CCV_HALO on the golden and edge
shapes that would normally go to the single-CTA kernel, and against the
fp64 oracle; and the single-CTA kernel (CCV_FORCE_KERNEL=1) on a shape that
would normally go to the pair kernel."""

import os

import pytest
import torch

import oracle
from test_oracle import CASES as GOLDEN_CASES
from test_parity_gpu import EDGE, TF32_TOL, abi_fprop_complex, abi_fprop_planar, abi_prepack

pytestmark = pytest.mark.gpu


@pytest.fixture
def force_kernel():
    """Pin the kernel family (1 = single CTA, 2 = CTA pair; 'halo' = CTA pair
    with halo reuse, 'tap' = CTA pair without halo reuse) through the
    library's env knobs."""
    keys = ("CCV_FORCE_KERNEL", "CCV_HALO", "CCV_SUBBOX", "CCV_STREAMK", "CCV_LW")
    old = {k: os.environ.get(k) for k in keys}
    # Whole tiles only and the layout pass for complex input, so every
    # complex64 call sums like the planar one.
    os.environ["CCV_STREAMK"] = "0"
    os.environ["CCV_LW"] = "0"

    def set_(v):
        os.environ.pop("CCV_SUBBOX", None)
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
@pytest.mark.parametrize("family", ["tap", "halo"])
def test_pair_kernel_golden(force_kernel, family, name, case, x, wr, wi, y32, y64):
    force_kernel(family)
    packed = abi_prepack(case, torch.from_numpy(wr), torch.from_numpy(wi))
    y = abi_fprop_planar(case, torch.from_numpy(x), packed, poison=True)
    assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any()
    assert oracle.rel_frobenius(y, y64) <= TF32_TOL
    yc = abi_fprop_complex(case, torch.from_numpy(x), packed, poison=True)
    assert torch.equal(yc, y.to(torch.complex64))


@pytest.mark.parametrize("case", EDGE, ids=[str(i) for i in range(len(EDGE))])
@pytest.mark.parametrize("family", ["tap", "halo"])
def test_pair_kernel_edges(force_kernel, family, case):
    force_kernel(family)
    x, wr, wi = oracle.make_inputs(case, input_seed=9)
    packed = abi_prepack(case, wr, wi)
    y = abi_fprop_planar(case, x, packed, poison=True)
    assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any()
    assert oracle.rel_frobenius(y, oracle.oracle_fp64(case, x, wr, wi)) <= TF32_TOL


@pytest.mark.parametrize("family", [1, "tap", "halo"])
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
