"""forward() with in-kernel layout conversion (ccv_cvt_role.cuh): converter
clusters of the halo pair kernel turn complex64 NCHW images into fp32 NHWC
planes that the other clusters read, in one launch (opt-in, CCV_CVT=1).

Checked against the fp64 oracle (TF32 bar) and bitwise against the two-launch
path (layout pass + the same kernel with whole tiles), for several converter
counts, repeated calls (the library-owned counters are left zero), ragged
image sizes and channel counts.
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
CASES = [
    ("b8_128_56", C(8, 128, 56, 56, 128, 3, 3, 1, 1, 1, 1)),
    ("k64_subbox", C(4, 64, 40, 40, 64, 3, 3, 1, 1, 1, 1)),
    ("ragged_30x42_c36_k20", C(6, 36, 30, 42, 20, 3, 3, 1, 1, 1, 1)),
    ("5x5_p2_k132", C(3, 48, 26, 34, 132, 5, 5, 1, 1, 2, 2)),
]


@pytest.fixture
def knobs():
    keys = ("CCV_FORCE_KERNEL", "CCV_HALO", "CCV_CVT", "CCV_CVT_CLUSTERS", "CCV_STREAMK",
            "CCV_CD", "CCV_FUSED", "CCV_LW")
    old = {k: os.environ.get(k) for k in keys}
    os.environ["CCV_FORCE_KERNEL"] = "2"
    os.environ["CCV_HALO"] = "1"
    os.environ["CCV_CVT"] = "1"
    os.environ["CCV_LW"] = "0"  # the comparison path below is the layout pass
    for k in ("CCV_CVT_CLUSTERS", "CCV_CD", "CCV_FUSED"):
        os.environ.pop(k, None)
    yield
    for k, v in old.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v
    torch.cuda.synchronize()
    assert device_status() == 0, "a bounded in-kernel wait ran out"


def kernel_name(case):
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    return lib.ccv_fprop_complex_kernel(ctypes.byref(shp), ccv_abi.CCV_PRECISION_TF32).decode()


@pytest.mark.parametrize("name,case", CASES, ids=[c[0] for c in CASES])
def test_converter_clusters(knobs, name, case):
    assert kernel_name(case) == "halo_pair_converter_clusters"
    x, wr, wi = oracle.make_inputs(case, input_seed=51)
    packed = abi_prepack(case, wr, wi)
    y = abi_fprop_complex(case, x, packed, poison=True)
    assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any()
    sub = C(1, case.c, case.h, case.w, case.k, case.r, case.s, 1, 1, case.pad_h, case.pad_w)
    for img in (0, case.n - 1):
        ref = oracle.oracle_fp64(sub, x[img:img + 1], wr, wi)
        assert oracle.rel_frobenius(y[img:img + 1], ref) <= TF32_TOL, img
    # Repeated calls and other converter counts give the same bits.
    assert torch.equal(y, abi_fprop_complex(case, x, packed, poison=True))
    for n_cvt in ("1", "3"):
        os.environ["CCV_CVT_CLUSTERS"] = n_cvt
        assert torch.equal(y, abi_fprop_complex(case, x, packed, poison=True)), n_cvt
    os.environ.pop("CCV_CVT_CLUSTERS", None)
    # The two-launch path with whole tiles: same kernel, same sums.
    os.environ["CCV_CVT"] = "0"
    os.environ["CCV_STREAMK"] = "0"
    assert kernel_name(case) == "layout_pass+halo_pair"
    assert torch.equal(y, abi_fprop_complex(case, x, packed, poison=True))


def test_converter_clusters_not_taken(knobs):
    # Odd image width (TMA row stride), 3xTF32, stride 2: other paths.
    assert kernel_name(C(2, 32, 20, 21, 64, 3, 3, 1, 1, 1, 1)) != "halo_pair_converter_clusters"
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(C(8, 128, 56, 56, 128, 3, 3, 1, 1, 1, 1))
    assert lib.ccv_fprop_complex_kernel(ctypes.byref(shp), ccv_abi.CCV_PRECISION_3XTF32).decode() \
        != "halo_pair_converter_clusters"
    assert kernel_name(C(2, 32, 20, 20, 64, 3, 3, 2, 2, 1, 1)) != "halo_pair_converter_clusters"
    # Off unless asked for.
    os.environ.pop("CCV_CVT")
    assert kernel_name(C(8, 128, 56, 56, 128, 3, 3, 1, 1, 1, 1)) == "layout_pass+halo_pair"
