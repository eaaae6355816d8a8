"""ComplexConv2d.forward under autograd: gradients of the input, the weight
planes and the complex bias against the fp64 gradient oracle (pinned to the
reference module's autograd, tests/test_oracle_backward.py).  Bar: rel.
Frobenius <= 1e-3 (TF32), 1e-5 for the 3xTF32 data gradient."""

import pytest
import torch

import oracle
from complex_conv2d import ComplexConv2d

pytestmark = pytest.mark.gpu
DEV = "cuda"

CASES = [
    oracle.ConvCase(2, 32, 14, 14, 64, 3, 3, 1, 1, 1, 1),
    oracle.ConvCase(2, 16, 15, 15, 32, 3, 3, 2, 2, 1, 1),
    oracle.ConvCase(1, 64, 8, 8, 128, 1, 1, 1, 1, 0, 0),
    oracle.ConvCase(1, 128, 7, 7, 256, 3, 3, 1, 1, 1, 1),
]
IDS = [f"c{c.c}k{c.k}h{c.h}r{c.r}st{c.stride_h}" for c in CASES]


def _layer(case, precision="tf32", bias=False):
    x, wr, wi = oracle.make_inputs(case)
    layer = ComplexConv2d(case.c, case.k, (case.r, case.s), stride=(case.stride_h, case.stride_w),
                          padding=(case.pad_h, case.pad_w), bias=bias, device=DEV,
                          precision=precision)
    with torch.no_grad():
        layer.weight_real.copy_(wr)
        layer.weight_imag.copy_(wi)
    return layer, x, wr, wi


def _dy(case):
    g = torch.Generator().manual_seed(11)
    shape = (case.n, case.k, case.p, case.q)
    return torch.complex(torch.randn(shape, generator=g), torch.randn(shape, generator=g))


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_input_and_weight_gradients(case):
    layer, x, wr, wi = _layer(case)
    layer.weight_real.requires_grad_(True)
    layer.weight_imag.requires_grad_(True)
    xd = x.to(DEV).requires_grad_(True)
    y = layer(xd)
    assert y.grad_fn is not None
    dy = _dy(case)
    dx, dwr, dwi = torch.autograd.grad(y, (xd, layer.weight_real, layer.weight_imag),
                                       grad_outputs=dy.to(DEV))
    rx, rwr, rwi = oracle.backward_autograd_fp64(case, x, wr, wi, dy)
    assert oracle.rel_frobenius(dx.cpu(), rx) <= 1e-3
    got = torch.complex(dwr.cpu().double(), dwi.cpu().double())
    assert oracle.rel_frobenius(got, torch.complex(rwr, rwi)) <= 1e-3
    # The forward value is the inference path's.
    with torch.no_grad():
        y0 = layer(x.to(DEV))
    assert torch.equal(y.detach(), y0)


def test_input_gradient_3xtf32():
    case = oracle.ConvCase(2, 32, 12, 12, 32, 3, 3, 1, 1, 1, 1)
    layer, x, wr, wi = _layer(case, precision="3xtf32")
    xd = x.to(DEV).requires_grad_(True)
    dy = _dy(case)
    (dx,) = torch.autograd.grad(layer(xd), xd, grad_outputs=dy.to(DEV))
    rx, _, _ = oracle.backward_autograd_fp64(case, x, wr, wi, dy)
    assert oracle.rel_frobenius(dx.cpu(), rx) <= 1e-5


def test_bias_gradient_and_loss_backward():
    case = oracle.ConvCase(2, 16, 10, 10, 32, 3, 3, 1, 1, 1, 1)
    layer, x, wr, wi = _layer(case, bias=True)
    layer.bias_real.requires_grad_(True)
    layer.bias_imag.requires_grad_(True)
    xd = x.to(DEV).requires_grad_(True)
    dy = _dy(case).to(DEV)
    y = layer(xd)
    # A real loss whose gradient with respect to y is dy: Re <y, dy>.
    loss = (y * dy.conj()).real.sum()
    loss.backward()
    db = dy.sum(dim=(0, 2, 3))
    assert torch.allclose(layer.bias_real.grad, db.real, rtol=1e-5, atol=1e-4)
    assert torch.allclose(layer.bias_imag.grad, db.imag, rtol=1e-5, atol=1e-4)
    rx, _, _ = oracle.backward_autograd_fp64(case, x, wr, wi, dy.cpu())
    assert oracle.rel_frobenius(xd.grad.cpu(), rx) <= 1e-3


def test_no_graph_without_requires_grad():
    case = oracle.ConvCase(1, 8, 8, 8, 8, 3, 3, 1, 1, 1, 1)
    layer, x, _, _ = _layer(case)
    y = layer(x.to(DEV))
    assert y.grad_fn is None and not y.requires_grad


def test_weight_edit_refreshes_data_gradient_filter():
    case = oracle.ConvCase(1, 16, 9, 9, 16, 3, 3, 1, 1, 1, 1)
    layer, x, wr, wi = _layer(case)
    dy = _dy(case)
    for scale in (1.0, -0.5):
        with torch.no_grad():
            layer.weight_real.copy_(wr * scale)
        xd = x.to(DEV).requires_grad_(True)
        (dx,) = torch.autograd.grad(layer(xd), xd, grad_outputs=dy.to(DEV))
        rx, _, _ = oracle.backward_autograd_fp64(case, x, wr * scale, wi, dy)
        assert oracle.rel_frobenius(dx.cpu(), rx) <= 1e-3


@pytest.mark.parametrize("case", CASES[:2], ids=IDS[:2])
def test_forward_planar_gradients(case):
    layer, x, wr, wi = _layer(case)
    layer.weight_real.requires_grad_(True)
    layer.weight_imag.requires_grad_(True)
    xr = x.real.permute(0, 2, 3, 1).contiguous().to(DEV).requires_grad_(True)
    xi = x.imag.permute(0, 2, 3, 1).contiguous().to(DEV).requires_grad_(True)
    yr, yi = layer.forward_planar(xr, xi)
    dy = _dy(case)
    dyr = dy.real.permute(0, 2, 3, 1).contiguous().to(DEV)
    dyi = dy.imag.permute(0, 2, 3, 1).contiguous().to(DEV)
    gxr, gxi, gwr, gwi = torch.autograd.grad(
        (yr, yi), (xr, xi, layer.weight_real, layer.weight_imag), grad_outputs=(dyr, dyi))
    rx, rwr, rwi = oracle.backward_autograd_fp64(case, x, wr, wi, dy)
    dx = oracle.planar_nhwc_to_complex_nchw(gxr, gxi).cpu()
    assert oracle.rel_frobenius(dx, rx) <= 1e-3
    got = torch.complex(gwr.cpu().double(), gwi.cpu().double())
    assert oracle.rel_frobenius(got, torch.complex(rwr, rwi)) <= 1e-3
