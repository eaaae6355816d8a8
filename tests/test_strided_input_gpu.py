"""forward() on complex64 inputs of any layout, read in place.

The reference makes every input contiguous first (modules.py:198-199); here a
channels-last tensor, a spatial slice, a channel or batch step, a transposed
view and a dense view at an 8-byte (not 16-byte) aligned address go through
ccv_fprop_complex_strided: the layout kernel reads the strides.  Each result
must be bitwise equal to forward() of the same values made contiguous (same
planes, same convolution launch), and within the TF32 / 3xTF32 bar of the
fp64 oracle (benchmarks/baseline.py:5-9 restated in oracle/).
"""

import pytest
import torch

import oracle
from test_parity_gpu import DEV, TF32_TOL, device_status

pytestmark = pytest.mark.gpu

C = oracle.ConvCase


def _layer(case, precision, bias):
    from complex_conv2d import ComplexConv2d
    layer = ComplexConv2d(case.c, case.k, (case.r, case.s), stride=(case.stride_h, case.stride_w),
                          padding=(case.pad_h, case.pad_w), bias=bias, device=DEV,
                          precision=precision)
    _, wr, wi = oracle.make_inputs(case, weight_seed=3)
    with torch.no_grad():
        layer.weight_real.copy_(wr)
        layer.weight_imag.copy_(wi)
    return layer, wr, wi


def _big(shape, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.complex(torch.randn(shape, generator=g, device=DEV),
                         torch.randn(shape, generator=g, device=DEV))


def _views():
    """(name, strided view) pairs; every view has the logical shape (3, 32, 18, 22)."""
    out = []
    base = _big((3, 32, 18, 22), 1)
    out.append(("channels_last", base.contiguous(memory_format=torch.channels_last)))
    out.append(("hw_slice", _big((3, 32, 21, 27), 2)[:, :, 2:20, 3:25]))
    out.append(("channel_step", _big((3, 64, 18, 22), 3)[:, ::2]))
    out.append(("batch_step", _big((6, 32, 18, 22), 4)[::2]))
    out.append(("hw_transposed", _big((3, 32, 22, 18), 5).transpose(2, 3)))
    flat = _big((3 * 32 * 18 * 22 + 1,), 6)
    out.append(("misaligned_dense", flat[1:].view(3, 32, 18, 22)))
    return out


VIEWS = ["channels_last", "hw_slice", "channel_step", "batch_step", "hw_transposed",
         "misaligned_dense"]


@pytest.mark.parametrize("precision", ["tf32", "3xtf32"])
@pytest.mark.parametrize("bias", [False, True], ids=["nobias", "bias"])
@pytest.mark.parametrize("view", VIEWS)
def test_strided_input_matches_contiguous(view, bias, precision):
    torch.cuda.set_device(0)
    x = dict(_views())[view]
    assert x.shape == (3, 32, 18, 22)
    if view == "misaligned_dense":
        assert x.is_contiguous() and x.data_ptr() % 16 == 8
    else:
        assert not x.is_contiguous()
    case = C(3, 32, 18, 22, 40, 3, 3, 1, 1, 1, 1)
    layer, wr, wi = _layer(case, precision, bias)
    with torch.no_grad():
        y = layer(x)
        y_dense = layer(x.contiguous())
    torch.cuda.synchronize()
    assert torch.equal(y, y_dense), view
    br = layer.bias_real if bias else None
    bi = layer.bias_imag if bias else None
    ref = oracle.oracle_fp64(case, x.contiguous().cpu(), wr, wi, br, bi)
    tol = TF32_TOL if precision == "tf32" else 1e-5
    assert oracle.rel_frobenius(y.cpu(), ref) <= tol, view
    assert device_status() == 0


def test_strided_stride2_channels_last():
    """A stride-2 layer (tap kernel) on a channels-last input."""
    torch.cuda.set_device(0)
    case = C(2, 64, 33, 31, 128, 3, 3, 2, 2, 1, 1)
    layer, wr, wi = _layer(case, "tf32", False)
    x = _big((2, 64, 33, 31), 8).contiguous(memory_format=torch.channels_last)
    with torch.no_grad():
        y = layer(x)
        y_dense = layer(x.contiguous())
    torch.cuda.synchronize()
    assert torch.equal(y, y_dense)
    ref = oracle.oracle_fp64(case, x.contiguous().cpu(), wr, wi)
    assert oracle.rel_frobenius(y.cpu(), ref) <= TF32_TOL
