"""Both kernel families on the same problems: the CTA-pair kernel
(ccv_fprop2.cu) is pinned with CCV_FORCE_KERNEL=2 on the golden and edge
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
    old = os.environ.get("CCV_FORCE_KERNEL")

    def set_(v):
        os.environ["CCV_FORCE_KERNEL"] = str(v)

    yield set_
    if old is None:
        os.environ.pop("CCV_FORCE_KERNEL", None)
    else:
        os.environ["CCV_FORCE_KERNEL"] = old


@pytest.mark.parametrize("name,case,x,wr,wi,y32,y64", GOLDEN_CASES, ids=[c[0] for c in GOLDEN_CASES])
def test_pair_kernel_golden(force_kernel, name, case, x, wr, wi, y32, y64):
    force_kernel(2)
    packed = abi_prepack(case, torch.from_numpy(wr), torch.from_numpy(wi))
    y = abi_fprop_planar(case, torch.from_numpy(x), packed, poison=True)
    assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any()
    assert oracle.rel_frobenius(y, y64) <= TF32_TOL
    yc = abi_fprop_complex(case, torch.from_numpy(x), packed, poison=True)
    assert torch.equal(yc, y.to(torch.complex64))


@pytest.mark.parametrize("case", EDGE, ids=[str(i) for i in range(len(EDGE))])
def test_pair_kernel_edges(force_kernel, case):
    force_kernel(2)
    x, wr, wi = oracle.make_inputs(case, input_seed=9)
    packed = abi_prepack(case, wr, wi)
    y = abi_fprop_planar(case, x, packed, poison=True)
    assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any()
    assert oracle.rel_frobenius(y, oracle.oracle_fp64(case, x, wr, wi)) <= TF32_TOL


@pytest.mark.parametrize("family", [1, 2])
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
