"""Stream-K tail split of the CTA-pair kernels (ccv_fprop2.cu tap,
ccv_fprop2h.cu halo).

When the pair tiles do not fill the last wave of the persistent grid, the K
slots of the leftover tiles are spread over all clusters; split tiles are
summed from fp32 partials by whichever piece finishes last, in a fixed
order.  These tests pin a small persistent grid (CCV_MAX_CLUSTERS) so that
small problems get a partial last wave, force the split (CCV_STREAMK=1), and
check: parity with the fp64 oracle, agreement with the unsplit kernel up to
fp32 summation order, bitwise determinism across calls (counters are reset
per call), and the complex entry point matching the planar one bitwise.
"""

import ctypes
import os

import pytest
import torch

import ccv_abi
import oracle
from test_parity_gpu import TF32_TOL, _ptr, _stream, abi_prepack, device_status

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TF32 = ccv_abi.CCV_PRECISION_TF32
X3 = ccv_abi.CCV_PRECISION_3XTF32
TOL = {TF32: TF32_TOL, X3: 1e-5}
C = oracle.ConvCase

CASES = [
    ("halo_kt128", C(3, 64, 20, 20, 128, 3, 3, 1, 1, 1, 1), "halo", TF32),
    ("halo_kt64_ragged", C(2, 48, 17, 23, 64, 3, 3, 1, 1, 1, 1), "halo", TF32),
    ("halo_kt32_5x5", C(2, 32, 16, 16, 24, 5, 5, 1, 1, 2, 2), "halo", TF32),
    ("tap_stride2", C(3, 64, 33, 33, 128, 3, 3, 2, 2, 1, 1), "tap", TF32),
    ("tap_1x1_flat", C(2, 128, 24, 24, 96, 1, 1, 1, 1, 0, 0), "tap", TF32),
    ("halo_3xtf32", C(2, 32, 16, 16, 64, 3, 3, 1, 1, 1, 1), "halo", X3),
    ("tap_3xtf32", C(2, 32, 17, 17, 64, 3, 3, 2, 2, 1, 1), "tap", X3),
]
GRIDS = [3, 7]


@pytest.fixture
def knobs():
    keys = ("CCV_FORCE_KERNEL", "CCV_HALO", "CCV_STREAMK", "CCV_MAX_CLUSTERS", "CCV_SUBBOX",
            "CCV_LW")
    old = {k: os.environ.get(k) for k in keys}
    # The split lives in the pair kernels with one box per CTA.
    os.environ["CCV_SUBBOX"] = "0"
    os.environ["CCV_LW"] = "0"  # complex calls: layout pass + the split kernel

    def set_(family=None, streamk=None, clusters=None):
        if family is not None:
            os.environ["CCV_FORCE_KERNEL"] = "2"
            os.environ["CCV_HALO"] = "1" if family == "halo" else "0"
        for key, val in (("CCV_STREAMK", streamk), ("CCV_MAX_CLUSTERS", clusters)):
            if val is None:
                os.environ.pop(key, None)
            else:
                os.environ[key] = str(val)

    yield set_
    for k, v in old.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v
    torch.cuda.synchronize()
    assert device_status() == 0, "a bounded in-kernel wait ran out"


def planar(case, x, packed, precision, full_workspace=True):
    """ccv_fprop_planar with the recommended workspace (stream-K room) or the
    minimum one (every tile whole).  Returns complex128 NCHW on the CPU."""
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    xr = x.real.permute(0, 2, 3, 1).contiguous().to(DEV)
    xi = x.imag.permute(0, 2, 3, 1).contiguous().to(DEV)
    yr = torch.full((case.n, case.p, case.q, case.k), float("nan"), device=DEV)
    yi = torch.full_like(yr, float("nan"))
    query = (lib.ccv_fprop_planar_workspace_bytes if full_workspace
             else lib.ccv_fprop_planar_min_workspace_bytes)
    nbytes = query(ctypes.byref(shp), precision)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=DEV)
    ccv_abi.check(lib.ccv_fprop_planar(_ptr(xr), _ptr(xi), _ptr(packed), _ptr(yr), _ptr(yi),
                                       ctypes.byref(shp), precision,
                                       _ptr(ws) if nbytes else None, nbytes, _stream()),
                  "fprop_planar")
    torch.cuda.synchronize()
    return oracle.planar_nhwc_to_complex_nchw(yr, yi).cpu()


def complex_(case, x, packed, precision):
    lib = ccv_abi.load()
    shp = ccv_abi.shape_of(case)
    xd = x.to(DEV).contiguous()
    y = torch.full((case.n, case.k, case.p, case.q), float("nan"), dtype=torch.complex64,
                   device=DEV)
    nbytes = lib.ccv_fprop_complex_workspace_bytes(ctypes.byref(shp), precision)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=DEV)
    ccv_abi.check(lib.ccv_fprop_complex(_ptr(xd), _ptr(packed), _ptr(y), ctypes.byref(shp),
                                        precision, _ptr(ws), nbytes, _stream()), "fprop_complex")
    torch.cuda.synchronize()
    return y.cpu()


@pytest.mark.parametrize("name,case,family,precision", CASES, ids=[c[0] for c in CASES])
def test_stream_k_split(knobs, name, case, family, precision):
    x, wr, wi = oracle.make_inputs(case, input_seed=31)
    packed = abi_prepack(case, wr, wi, precision=precision)
    ref = oracle.oracle_fp64(case, x, wr, wi)
    knobs(family=family, streamk=0)
    whole = planar(case, x, packed, precision)
    assert oracle.rel_frobenius(whole, ref) <= TOL[precision]
    reassociated = False
    for grid in GRIDS:
        knobs(family=family, streamk=1, clusters=grid)
        y1 = planar(case, x, packed, precision)
        y2 = planar(case, x, packed, precision)
        assert not torch.isnan(y1.real).any() and not torch.isnan(y1.imag).any(), grid
        assert torch.equal(y1, y2), ("not deterministic", grid)
        assert oracle.rel_frobenius(y1, ref) <= TOL[precision], grid
        # Same products, different fp32 summation order only.
        assert oracle.rel_frobenius(y1, whole) <= 1e-5, grid
        reassociated |= not torch.equal(y1, whole)
        yc = complex_(case, x, packed, precision)
        assert torch.equal(yc, y1.to(torch.complex64)), grid
        # Without stream-K room in the workspace every tile runs whole.
        y0 = planar(case, x, packed, precision, full_workspace=False)
        if precision == TF32:
            knobs(family=family, streamk=0, clusters=grid)
            assert torch.equal(y0, planar(case, x, packed, precision)), grid
    assert reassociated, "no grid produced a stream-K split"


def test_stream_k_many_pieces_per_tile(knobs):
    """One pair tile, 24 K slots, 16 clusters: 12 pieces of 2 slots each."""
    case = C(1, 256, 8, 16, 128, 3, 3, 1, 1, 1, 1)
    x, wr, wi = oracle.make_inputs(case, input_seed=32)
    packed = abi_prepack(case, wr, wi)
    ref = oracle.oracle_fp64(case, x, wr, wi)
    knobs(family="halo", streamk=1, clusters=16)
    y1 = planar(case, x, packed, TF32)
    assert oracle.rel_frobenius(y1, ref) <= TF32_TOL
    assert torch.equal(y1, planar(case, x, packed, TF32))
    assert torch.equal(complex_(case, x, packed, TF32), y1.to(torch.complex64))
    knobs(family="tap", streamk=1, clusters=16)
    y2 = planar(case, x, packed, TF32)
    assert oracle.rel_frobenius(y2, ref) <= TF32_TOL


def test_stream_k_default_policy_batched(knobs):
    """The default policy on the full-size grid: an 8-image 128->128 56x56
    problem (one rank's share of batch 64 on 8 GPUs) leaves a partial last
    wave; results stay within fp32 reassociation of the unsplit kernel."""
    case = C(8, 128, 56, 56, 128, 3, 3, 1, 1, 1, 1)
    x, wr, wi = oracle.make_inputs(case, input_seed=33)
    packed = abi_prepack(case, wr, wi)
    knobs(streamk=0)
    whole = complex_(case, x, packed, TF32)
    knobs()
    split = complex_(case, x, packed, TF32)
    assert oracle.rel_frobenius(split, whole) <= 1e-5
    sub = C(1, 128, 56, 56, 128, 3, 3, 1, 1, 1, 1)
    for img in (0, 7):
        ref = oracle.oracle_fp64(sub, x[img:img + 1], wr, wi)
        assert oracle.rel_frobenius(split[img:img + 1], ref) <= TF32_TOL


@pytest.mark.parametrize("case", [C(1, 32, 56, 56, 64, 3, 3, 1, 1, 1, 1),
                                  C(1, 64, 28, 28, 128, 3, 3, 1, 1, 1, 1),
                                  C(1, 128, 14, 14, 256, 3, 3, 1, 1, 1, 1),
                                  C(1, 256, 7, 7, 512, 3, 3, 1, 1, 1, 1),
                                  C(2, 36, 9, 11, 20, 1, 1, 1, 1, 0, 0)],
                         ids=["b1_32_64_56", "b1_64_128_28", "b1_128_256_14", "b1_256_512_7",
                              "flat_small"])
def test_single_cta_split_through_l2_matches_dsmem(case):
    """The batch-1 kernel's cluster split sums its partials in rank order
    either way: through L2 when the workspace has room (recommended size),
    over distributed shared memory without workspace - bitwise equal, and
    within the TF32 bar of the fp64 oracle."""
    x, wr, wi = oracle.make_inputs(case, input_seed=81)
    packed = abi_prepack(case, wr, wi)
    y_l2 = planar(case, x, packed, TF32, full_workspace=True)
    y_dsmem = planar(case, x, packed, TF32, full_workspace=False)
    assert not torch.isnan(y_l2.real).any() and not torch.isnan(y_l2.imag).any()
    assert torch.equal(y_l2, y_dsmem)
    assert oracle.rel_frobenius(y_l2, oracle.oracle_fp64(case, x, wr, wi)) <= TOL[TF32]


@pytest.mark.parametrize("case,kt,splits",
                         [(C(1, 256, 7, 7, 512, 3, 3, 1, 1, 1, 1), 128, s) for s in (3, 5, 7, 11, 16)]
                         + [(C(1, 64, 28, 28, 128, 3, 3, 1, 1, 1, 1), 64, 9),
                            (C(1, 32, 56, 56, 64, 3, 3, 1, 1, 1, 1), 64, 5),
                            (C(2, 40, 9, 13, 24, 3, 3, 1, 1, 1, 1), 32, 6)],
                         ids=lambda v: str(v) if isinstance(v, int) else f"{v.c}_{v.k}_{v.h}")
def test_single_cta_any_split(case, kt, splits):
    """Cluster splits of any size up to 16 CTAs (not only powers of two): the
    K steps divide unevenly for most sizes, the partials still sum in rank
    order - bitwise equal through L2 and over distributed shared memory - and
    within the TF32 bar of the fp64 oracle.  CCV_SPLITK caps the split and
    the plan takes the largest that shortens the slowest CTA's loop."""
    keys = ("CCV_KT", "CCV_SPLITK", "CCV_FORCE_KERNEL")
    old = {k: os.environ.get(k) for k in keys}
    os.environ.update({"CCV_KT": str(kt), "CCV_SPLITK": str(splits), "CCV_FORCE_KERNEL": "1"})
    try:
        x, wr, wi = oracle.make_inputs(case, input_seed=83)
        packed = abi_prepack(case, wr, wi)
        y_l2 = planar(case, x, packed, TF32, full_workspace=True)
        y_dsmem = planar(case, x, packed, TF32, full_workspace=False)
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    assert not torch.isnan(y_l2.real).any() and not torch.isnan(y_l2.imag).any()
    assert torch.equal(y_l2, y_dsmem)
    assert oracle.rel_frobenius(y_l2, oracle.oracle_fp64(case, x, wr, wi)) <= TOL[TF32]
    assert device_status() == 0, "a bounded in-kernel wait ran out"
