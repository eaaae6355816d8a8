"""A device-side timeout surfaces as an error instead of silent garbage.

When a bounded in-kernel wait runs out, the kernel records the code in the
library's device status word and in a host-mapped copy of it; from then on
every launching entry point returns CCV_ERR_DEVICE (RuntimeError through the
extension, like the reference's TORCH_CHECK failures at
csrc/complex_conv2d.cu:268-306) until ccv_clear_device_status.  The timeout
is made without any fault: the self-test kernel waits on an mbarrier that
nothing arrives on, gives up after its bound and reports through the same
path a real timeout takes.  No GPU is faulted or hung.
"""

import ctypes

import pytest
import torch

import ccv_abi
import oracle
from test_parity_gpu import DEV, TF32_TOL, _ptr, _stream, abi_prepack

pytestmark = pytest.mark.gpu


def _layer(case, wr, wi):
    from complex_conv2d import ComplexConv2d
    layer = ComplexConv2d(case.c, case.k, (case.r, case.s), padding=(case.pad_h, case.pad_w),
                          device=DEV)
    with torch.no_grad():
        layer.weight_real.copy_(wr)
        layer.weight_imag.copy_(wi)
    return layer


def test_timeout_makes_later_calls_raise_until_cleared():
    from complex_conv2d import _C
    torch.cuda.set_device(0)
    case = oracle.ConvCase(2, 32, 20, 20, 64, 3, 3, 1, 1, 1, 1)
    x, wr, wi = oracle.make_inputs(case, input_seed=51)
    layer = _layer(case, wr, wi)
    xd = x.to(DEV)
    ref = oracle.oracle_fp64(case, x, wr, wi)
    with torch.no_grad():
        assert oracle.rel_frobenius(layer(xd).cpu(), ref) <= TF32_TOL
    torch.cuda.synchronize()
    try:
        # A wait on the library's own status word gives up (about 1 s).
        _C.selftest_bounded_wait(0, True)
        torch.cuda.synchronize()
        assert _C.device_status(0) == ccv_abi.CCV_ERR_DEVICE_TIMEOUT
        with torch.no_grad():
            with pytest.raises(RuntimeError, match="bounded wait"):
                layer(xd)
            with pytest.raises(RuntimeError, match="bounded wait"):
                layer.forward_planar(x.real.permute(0, 2, 3, 1).contiguous().to(DEV),
                                     x.imag.permute(0, 2, 3, 1).contiguous().to(DEV))
        # The C ABI reports it too, without launching anything.
        lib = ccv_abi.load()
        packed_ok = layer._w_packed
        shp = ccv_abi.shape_of(case)
        xr = x.real.permute(0, 2, 3, 1).contiguous().to(DEV)
        yr = torch.zeros((case.n, case.p, case.q, case.k), device=DEV)
        yi = torch.zeros_like(yr)
        rc = lib.ccv_fprop_planar(_ptr(xr), _ptr(xr), _ptr(packed_ok), _ptr(yr), _ptr(yi),
                                  ctypes.byref(shp), 0, None, 0, _stream())
        assert rc == 5  # CCV_ERR_DEVICE
        torch.cuda.synchronize()
        assert yr.abs().max().item() == 0.0  # nothing ran
    finally:
        _C.clear_device_status(0)
    assert _C.device_status(0) == 0
    with torch.no_grad():
        y = layer(xd)
    torch.cuda.synchronize()
    assert oracle.rel_frobenius(y.cpu(), ref) <= TF32_TOL


def test_caller_status_selftest_leaves_library_status_clear():
    """The self-test into a caller's int reports there and nowhere else."""
    from complex_conv2d import _C
    torch.cuda.set_device(0)
    assert _C.selftest_bounded_wait(0) == ccv_abi.CCV_ERR_DEVICE_TIMEOUT
    assert _C.device_status(0) == 0
    case = oracle.ConvCase(1, 8, 9, 9, 8, 3, 3, 1, 1, 1, 1)
    x, wr, wi = oracle.make_inputs(case)
    packed = abi_prepack(case, wr, wi)
    assert packed.numel() > 0
