"""Host-side behaviour of the drop-in module that needs no GPU: constructor
validation and messages (modules.py:54-80 of the reference), parameter
layout and state_dict keys (modules.py:93-107), input validation order
(modules.py:176-195)."""

import pytest
import torch

from complex_conv2d import ComplexConv2d
from complex_conv2d.modules import _host_chunks, _pair


def test_rejects_unsupported_options():
    with pytest.raises(NotImplementedError, match="groups"):
        ComplexConv2d(32, 64, 3, groups=2)
    with pytest.raises(NotImplementedError, match="dilation"):
        ComplexConv2d(32, 64, 3, dilation=2)
    with pytest.raises(NotImplementedError, match="padding_mode"):
        ComplexConv2d(32, 64, 3, padding_mode="reflect")
    with pytest.raises(NotImplementedError, match="complex64"):
        ComplexConv2d(32, 64, 3, dtype=torch.complex128)


def test_complex_bias_parameters():
    """bias=True (rejected by the reference, modules.py:73-74) adds a complex
    bias per output channel: two fp32 [K] parameters in the state_dict,
    initialised like nn.Conv2d's bias."""
    m = ComplexConv2d(8, 12, (3, 5), bias=True)
    assert m.bias_real.shape == (12,) and m.bias_imag.shape == (12,)
    assert m.bias_real.dtype == torch.float32
    assert not m.bias_real.requires_grad and not m.bias_imag.requires_grad
    assert set(m.state_dict()) == {"weight_real", "weight_imag", "bias_real", "bias_imag"}
    bound = 1.0 / (8 * 15) ** 0.5
    assert m.bias_real.abs().max().item() <= bound and m.bias_imag.abs().max().item() <= bound
    m2 = ComplexConv2d(8, 12, (3, 5), bias=True)
    m2.load_state_dict(m.state_dict())
    assert torch.equal(m2.bias_imag, m.bias_imag)
    assert "bias=True" in repr(m)
    plain = ComplexConv2d(8, 12, 3)
    assert plain.bias_real is None and plain.bias_imag is None


def test_rejects_bad_sizes():
    with pytest.raises(ValueError, match="positive"):
        ComplexConv2d(0, 4, 3)
    with pytest.raises(ValueError, match="kernel_size must be positive"):
        ComplexConv2d(4, 4, 0)
    with pytest.raises(ValueError, match="stride must be positive"):
        ComplexConv2d(4, 4, 3, stride=0)
    with pytest.raises(ValueError, match="padding must be non-negative"):
        ComplexConv2d(4, 4, 3, padding=-1)
    with pytest.raises(TypeError, match="kernel_size must be an int or a pair of ints"):
        ComplexConv2d(4, 4, 3.0)


def test_pair_helper():
    assert _pair(3, "x") == (3, 3)
    assert _pair((2, 5), "x") == (2, 5)
    assert _pair([1, 2], "x") == (1, 2)
    with pytest.raises(TypeError):
        _pair((1, 2, 3), "x")
    with pytest.raises(TypeError):
        _pair((1.0, 2), "x")


def test_parameters_and_state_dict():
    m = ComplexConv2d(8, 12, (3, 5), stride=(2, 1), padding=(1, 2))
    assert m.weight_real.shape == (12, 8, 3, 5)
    assert m.weight_real.dtype == torch.float32
    assert not m.weight_real.requires_grad and not m.weight_imag.requires_grad
    assert set(m.state_dict()) == {"weight_real", "weight_imag"}
    assert m.kernel_size == (3, 5) and m.stride == (2, 1) and m.padding == (1, 2)
    # kaiming_uniform_ default (a=0): U(+-sqrt(6/fan_in))
    bound = (6.0 / (8 * 15)) ** 0.5
    assert m.weight_real.abs().max().item() <= bound


def test_precision_selector():
    assert ComplexConv2d(4, 4, 3).precision == "tf32"
    assert ComplexConv2d(4, 4, 3, precision="3xTF32").precision == "3xtf32"
    with pytest.raises(ValueError, match="precision"):
        ComplexConv2d(4, 4, 3, precision="fp16")


def test_forward_validation_before_any_cuda_use():
    m = ComplexConv2d(4, 4, 3)
    with pytest.raises(ValueError, match="must be on CUDA"):
        m(torch.zeros(1, 4, 5, 5, dtype=torch.complex64))


def test_forward_host_validation_and_output_shape():
    m = ComplexConv2d(4, 8, 3, stride=2, padding=1)
    assert m.output_shape(3, 9, 10) == (3, 8, 5, 5)
    with pytest.raises(ValueError, match="smaller than the kernel"):
        ComplexConv2d(4, 8, 5).output_shape(1, 3, 3)
    with pytest.raises(ValueError, match="complex64"):
        m.forward_host(torch.zeros(1, 4, 5, 5))
    with pytest.raises(ValueError, match="input channels"):
        m.forward_host(torch.zeros(1, 3, 5, 5, dtype=torch.complex64))
    # Pageable (not pinned) host memory is refused before any CUDA use.
    with pytest.raises(ValueError, match="pinned"):
        m.forward_host(torch.zeros(1, 4, 5, 5, dtype=torch.complex64))


def test_prepack_requires_cuda_weights():
    m = ComplexConv2d(4, 4, 3)
    with pytest.raises(RuntimeError, match="weights must be on CUDA"):
        m._ensure_prepacked()


def test_apply_clears_cache():
    m = ComplexConv2d(4, 4, 3)
    m._w_packed = torch.zeros(1)
    m._weight_version = (0, 0)
    m.float()
    assert m._w_packed is None and m._weight_version is None


def test_forward_host_chunk_schedule():
    # Ramp 1, 2, 4 up to the middle size and back down; every image once.
    assert _host_chunks(64, 7) == [1, 2, 4] + [7] * 7 + [1] + [4, 2, 1]
    for n in range(1, 130):
        for middle in (1, 3, 7, 8, 16):
            sizes = _host_chunks(n, middle)
            assert sum(sizes) == n and min(sizes) >= 1 and max(sizes) <= max(middle, 1)
    # Small batches: at least three equal chunks where there are 3 images.
    assert _host_chunks(8, 7) == [3, 3, 2]
    assert _host_chunks(1, 7) == [1]
