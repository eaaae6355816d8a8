"""Complex-direct kernel (ccv_fprop_cd.cu): forward() reading complex64 NCHW
activations by TMA as an MN-major tensor-core operand, with the odd filter
columns assembled in shared memory.

Opted in with CCV_CD=1 (it is not the default: slower than the
converter-warp halo kernel on B200) and pinned to the pair kernels
(CCV_FORCE_KERNEL=2) so that small shapes take it; checked against the fp64
oracle (TF32 bar), against the planar-operand kernels (same products, fp32
summation order only), for determinism and for complete output coverage
(NaN-poisoned outputs).
"""

import ctypes
import os

import pytest
import torch

import ccv_abi
import oracle
from test_parity_gpu import TF32_TOL, abi_fprop_complex, abi_prepack, device_status

pytestmark = pytest.mark.gpu

C = oracle.ConvCase
TF32 = ccv_abi.CCV_PRECISION_TF32

CASES = [
    ("3x3_p1_k128", C(2, 64, 20, 20, 128, 3, 3, 1, 1, 1, 1)),
    ("3x3_ragged_box", C(2, 32, 18, 34, 64, 3, 3, 1, 1, 1, 1)),
    ("c36_k20", C(1, 36, 16, 24, 20, 3, 3, 1, 1, 1, 1)),
    ("p0_k132_two_ntiles", C(2, 64, 24, 24, 132, 3, 3, 1, 1, 0, 0)),
    ("5x5_p2", C(1, 32, 20, 20, 64, 5, 5, 1, 1, 2, 2)),
    ("1x1", C(2, 64, 14, 14, 96, 1, 1, 1, 1, 0, 0)),
    ("3x1", C(1, 32, 12, 16, 48, 3, 1, 1, 1, 1, 0)),
    ("1x3", C(1, 32, 12, 16, 48, 1, 3, 1, 1, 0, 1)),
    ("3x3_p2", C(1, 40, 10, 10, 36, 3, 3, 1, 1, 2, 2)),
    ("kt128_c128", C(3, 128, 28, 28, 256, 3, 3, 1, 1, 1, 1)),
    ("tiny_c4_k4", C(1, 4, 8, 8, 4, 3, 3, 1, 1, 1, 1)),
]


@pytest.fixture
def pair_family():
    keys = ("CCV_FORCE_KERNEL", "CCV_HALO", "CCV_CD")
    old = {k: os.environ.get(k) for k in keys}
    os.environ["CCV_FORCE_KERNEL"] = "2"
    os.environ.pop("CCV_HALO", None)
    os.environ["CCV_CD"] = "1"
    yield
    for k, v in old.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v
    torch.cuda.synchronize()
    assert device_status() == 0, "a bounded in-kernel wait ran out"


def kernel_name(case, precision=TF32):
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    return lib.ccv_fprop_complex_kernel(ctypes.byref(shp), precision).decode()


@pytest.mark.parametrize("name,case", CASES, ids=[c[0] for c in CASES])
def test_complex_direct_parity(pair_family, name, case):
    assert kernel_name(case) == "complex_direct_pair"
    x, wr, wi = oracle.make_inputs(case, input_seed=41)
    packed = abi_prepack(case, wr, wi)
    y = abi_fprop_complex(case, x, packed, poison=True)
    assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any()
    ref = oracle.oracle_fp64(case, x, wr, wi)
    assert oracle.rel_frobenius(y, ref) <= TF32_TOL
    assert torch.equal(y, abi_fprop_complex(case, x, packed, poison=True)), "not deterministic"
    # The planar-operand kernel on the same packed weights: identical TF32
    # products, different fp32 summation order.
    os.environ["CCV_CD"] = "0"
    y_old = abi_fprop_complex(case, x, packed, poison=True)
    os.environ["CCV_CD"] = "1"
    assert oracle.rel_frobenius(y, y_old) <= 1e-5


def test_complex_direct_is_opt_in():
    assert kernel_name(C(64, 128, 56, 56, 128, 3, 3, 1, 1, 1, 1)) != "complex_direct_pair"


def test_complex_direct_not_taken_where_it_does_not_apply(pair_family):
    # Stride 2, an even filter width, an odd image width and a filter too
    # wide for the slot ring each fall back to the other kernels.
    for case in (C(2, 32, 16, 16, 64, 3, 3, 2, 2, 1, 1),
                 C(1, 32, 16, 16, 64, 2, 2, 1, 1, 0, 0),
                 C(1, 32, 15, 15, 64, 3, 3, 1, 1, 1, 1),
                 C(1, 32, 20, 20, 64, 7, 7, 1, 1, 3, 3)):
        assert kernel_name(case) != "complex_direct_pair", case
    assert kernel_name(C(2, 64, 20, 20, 128, 3, 3, 1, 1, 1, 1),
                       ccv_abi.CCV_PRECISION_3XTF32) != "complex_direct_pair"


def test_complex_direct_on_the_batched_layer(pair_family):
    """The BASELINE batched layer (batch 64, 128->128, 56x56): first and last
    image against the oracle."""
    case = C(64, 128, 56, 56, 128, 3, 3, 1, 1, 1, 1)
    name = kernel_name(case)
    assert name == "complex_direct_pair"
    x, wr, wi = oracle.make_inputs(case, input_seed=0)
    packed = abi_prepack(case, wr, wi)
    y = abi_fprop_complex(case, x, packed, poison=True)
    assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any()
    sub = C(1, 128, 56, 56, 128, 3, 3, 1, 1, 1, 1)
    for img in (0, 63):
        ref = oracle.oracle_fp64(sub, x[img:img + 1], wr, wi)
        assert oracle.rel_frobenius(y[img:img + 1], ref) <= TF32_TOL, (name, img)
