"""The reference's own test strategy (tests/test_correctness.py and
tests/test_correctness_extended.py of cutlass-complex-conv), restated for the
B200 module: same shapes, seeds, input generator (torch.randn complex64 on
the GPU), weight hand-over from two nn.Conv2d layers, GPU four-conv oracle
and tolerances (assert_close rtol=atol=1e-3; planar vs public 1e-6).
"""

import pytest
import torch
import torch.nn as nn

from complex_conv2d import ComplexConv2d

import oracle

pytestmark = pytest.mark.gpu


class FourConv(nn.Module):
    """Two bias-free real Conv2d layers combined by the four-conv formula
    (benchmarks/baseline.py:5-45)."""

    def __init__(self, cin, cout, kernel_size, stride=1, padding=0):
        super().__init__()
        self.conv_real = nn.Conv2d(cin, cout, kernel_size, stride=stride, padding=padding, bias=False)
        self.conv_imag = nn.Conv2d(cin, cout, kernel_size, stride=stride, padding=padding, bias=False)

    def forward(self, x):
        re = self.conv_real(x.real) - self.conv_imag(x.imag)
        im = self.conv_real(x.imag) + self.conv_imag(x.real)
        return re.to(torch.complex64) + 1j * im.to(torch.complex64)


REFERENCE_SHAPES = [
    ((1, 32, 32, 32), 32, 3, 1, 1),
    ((1, 32, 56, 56), 64, 3, 1, 1),
    ((1, 64, 28, 28), 128, 3, 1, 1),
    ((1, 128, 14, 14), 256, 3, 1, 1),
    ((1, 256, 7, 7), 512, 3, 1, 1),
    ((1, 32, 32, 32), 64, 1, 1, 0),
    ((1, 32, 32, 32), 64, 3, 2, 1),
    ((1, 32, 32, 32), 64, 3, 1, 0),
    ((2, 32, 32, 32), 64, 3, 1, 1),
    ((1, 32, 32, 48), 64, 3, 1, 1),
]


def _layers(cin, cout, k, stride, padding):
    ref = FourConv(cin, cout, k, stride=stride, padding=padding).cuda().eval()
    mod = ComplexConv2d(cin, cout, k, stride=stride, padding=padding, bias=False, device="cuda").eval()
    with torch.no_grad():
        mod.weight_real.copy_(ref.conv_real.weight)
        mod.weight_imag.copy_(ref.conv_imag.weight)
    return ref, mod


@pytest.mark.parametrize("shape,out_channels,kernel_size,stride,padding", REFERENCE_SHAPES)
def test_matches_four_conv_reference(shape, out_channels, kernel_size, stride, padding):
    torch.manual_seed(0)
    n, cin, h, w = shape
    ref, mod = _layers(cin, out_channels, kernel_size, stride, padding)
    x = torch.randn(n, cin, h, w, device="cuda", dtype=torch.complex64)
    with torch.no_grad():
        y_ref = ref(x)
        y = mod(x)
    assert y.dtype == torch.complex64 and y.is_contiguous()
    torch.testing.assert_close(y, y_ref, rtol=1e-3, atol=1e-3)
    # And the fp64 CPU oracle bar (relative Frobenius).
    y64 = oracle.four_conv(x.cpu(), mod.weight_real.cpu(), mod.weight_imag.cpu(),
                           (stride, stride), (padding, padding))
    assert oracle.rel_frobenius(y.cpu(), y64) <= 1e-3


def test_planar_fast_path_matches_public_forward():
    torch.manual_seed(1)
    layer = ComplexConv2d(32, 64, 3, padding=1, bias=False, device="cuda").eval()
    x = torch.randn(1, 32, 32, 32, device="cuda", dtype=torch.complex64)
    with torch.no_grad():
        y_public = layer(x)
        x_real = x.real.permute(0, 2, 3, 1).contiguous()
        x_imag = x.imag.permute(0, 2, 3, 1).contiguous()
        y_real, y_imag = layer.forward_planar(x_real, x_imag)
        y_planar = torch.complex(y_real.permute(0, 3, 1, 2).contiguous(),
                                 y_imag.permute(0, 3, 1, 2).contiguous())
    torch.testing.assert_close(y_planar, y_public, rtol=1e-6, atol=1e-6)


def test_rejects_wrong_input_channel_count():
    layer = ComplexConv2d(32, 64, 3, padding=1, bias=False, device="cuda").eval()
    x = torch.randn(1, 16, 32, 32, device="cuda", dtype=torch.complex64)
    with pytest.raises(ValueError, match="input channels"):
        layer(x)


def test_rejects_non_complex64_input():
    layer = ComplexConv2d(32, 64, 3, padding=1, bias=False, device="cuda").eval()
    x = torch.randn(1, 32, 32, 32, device="cuda", dtype=torch.float32)
    with pytest.raises(ValueError, match="complex64"):
        layer(x)


def test_planar_rejects_channel_mismatch_and_layout():
    layer = ComplexConv2d(32, 64, 3, padding=1, device="cuda")
    xr = torch.randn(1, 8, 8, 16, device="cuda")
    with pytest.raises(RuntimeError, match="input channel count must match"):
        layer.forward_planar(xr, xr.clone())
    xr = torch.randn(1, 8, 8, 32, device="cuda")
    with pytest.raises(RuntimeError, match="must be contiguous"):
        layer.forward_planar(xr.transpose(1, 2), xr.clone())
    with pytest.raises(RuntimeError, match="float32"):
        layer.forward_planar(xr.double(), xr.double())


def test_extension_forward_krsc_contract():
    """`_C.forward` keeps the reference signature: NHWC planes + KRSC weights."""
    from complex_conv2d._extension import cutlass_complex_conv as ext
    torch.manual_seed(2)
    ref, mod = _layers(16, 24, 3, 2, 1)
    x = torch.randn(2, 16, 15, 15, device="cuda", dtype=torch.complex64)
    wr = mod.weight_real.permute(0, 2, 3, 1).contiguous()
    wi = mod.weight_imag.permute(0, 2, 3, 1).contiguous()
    y_real, y_imag = ext.forward(x.real.permute(0, 2, 3, 1).contiguous(),
                                 x.imag.permute(0, 2, 3, 1).contiguous(), wr, wi, 2, 2, 1, 1)
    assert y_real.shape == (2, 8, 8, 24)
    y = torch.complex(y_real.permute(0, 3, 1, 2), y_imag.permute(0, 3, 1, 2))
    torch.testing.assert_close(y, ref(x), rtol=1e-3, atol=1e-3)
    with pytest.raises(RuntimeError, match="input channel count must match"):
        ext.forward(torch.zeros(1, 4, 4, 8, device="cuda"), torch.zeros(1, 4, 4, 8, device="cuda"),
                    wr, wi, 1, 1, 1, 1)


def test_weight_edit_invalidates_prepack():
    torch.manual_seed(3)
    ref, mod = _layers(8, 8, 3, 1, 1)
    x = torch.randn(1, 8, 10, 10, device="cuda", dtype=torch.complex64)
    y0 = mod(x)
    with torch.no_grad():
        mod.weight_real.mul_(2.0)
        mod.weight_imag.mul_(2.0)
    y1 = mod(x)
    torch.testing.assert_close(y1, 2 * y0, rtol=1e-5, atol=1e-5)


def test_module_to_moves_and_repacks():
    mod = ComplexConv2d(8, 8, 3, padding=1)  # CPU parameters
    x = torch.randn(1, 8, 6, 6, dtype=torch.complex64)
    with pytest.raises(ValueError, match="must be on CUDA"):
        mod(x)
    mod = mod.cuda()
    y = mod(x.cuda())
    y64 = oracle.four_conv(x, mod.weight_real.cpu(), mod.weight_imag.cpu(), (1, 1), (1, 1))
    assert oracle.rel_frobenius(y.cpu(), y64) <= 1e-3


def test_non_contiguous_complex_input():
    torch.manual_seed(4)
    mod = ComplexConv2d(8, 12, 3, padding=1, device="cuda")
    base = torch.randn(1, 10, 8, 8, device="cuda", dtype=torch.complex64)
    x = base[:, 1:9]  # non-contiguous channel slice
    y = mod(x)
    y_ref = mod(x.contiguous())
    assert torch.equal(y, y_ref)


def test_state_dict_round_trip():
    mod = ComplexConv2d(8, 12, 3, padding=1, device="cuda")
    sd = mod.state_dict()
    assert set(sd) == {"weight_real", "weight_imag"}
    assert sd["weight_real"].shape == (12, 8, 3, 3)
    mod2 = ComplexConv2d(8, 12, 3, padding=1, device="cuda")
    mod2.load_state_dict(sd)
    x = torch.randn(1, 8, 9, 9, device="cuda", dtype=torch.complex64)
    assert torch.equal(mod(x), mod2(x))
