"""ComplexConv2d.forward_host: a pinned host batch in, pinned host result out,
chunks of images pipelined over copy-in, convolution and copy-out streams.

Every chunk's output must be bit-identical to ``forward`` of the same chunk on
the device (the kernels are deterministic), and the whole batch must meet the
TF32 bound (relative Frobenius <= 1e-3; 1e-5 at 3xTF32) against the fp64
four-conv oracle.
"""

import pytest
import torch

from complex_conv2d import ComplexConv2d

import oracle

pytestmark = pytest.mark.gpu

TF32_TOL = 1e-3
TOL_3XTF32 = 1e-5


def _layer(cin, cout, k, stride, padding, seed):
    torch.manual_seed(seed)
    return ComplexConv2d(cin, cout, k, stride=stride, padding=padding, device="cuda").eval()


def _host_batch(shape, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.complex(torch.randn(shape, generator=g), torch.randn(shape, generator=g))
    return x.pin_memory()


def _chunk_reference(layer, x, m):
    """forward() of each chunk of m images, brought back to the host."""
    parts = [layer(x[i:i + m].cuda()).cpu() for i in range(0, x.size(0), m)]
    return torch.cat(parts)


@pytest.mark.parametrize("n,cin,hw,cout,k,stride,pad,m", [
    (7, 32, 20, 64, 3, 1, 1, 3),   # ragged last chunk
    (5, 16, 17, 32, 3, 2, 1, 2),   # stride 2, odd spatial size
    (4, 32, 16, 32, 1, 1, 0, 1),   # 1x1, one image per chunk
    (3, 8, 9, 12, 3, 1, 0, 8),     # one chunk larger than the batch
])
def test_chunks_match_forward_and_oracle(n, cin, hw, cout, k, stride, pad, m):
    layer = _layer(cin, cout, k, stride, pad, seed=n + cin)
    x = _host_batch((n, cin, hw, hw), seed=cout)
    y = layer.forward_host(x, images_per_chunk=m)
    torch.cuda.current_stream().synchronize()
    assert y.is_pinned() and tuple(y.shape) == layer.output_shape(n, hw, hw)
    assert torch.equal(y, _chunk_reference(layer, x, m))
    ref = oracle.four_conv(x, layer.weight_real.cpu(), layer.weight_imag.cpu(), (stride, stride),
                           (pad, pad))
    assert oracle.rel_frobenius(y, ref) <= TF32_TOL


def test_3xtf32_chunks():
    torch.manual_seed(11)
    layer = ComplexConv2d(32, 32, 3, padding=1, device="cuda", precision="3xtf32").eval()
    x = _host_batch((5, 32, 18, 18), seed=12)
    y = layer.forward_host(x, images_per_chunk=2)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(y, _chunk_reference(layer, x, 2))
    ref = oracle.four_conv(x, layer.weight_real.cpu(), layer.weight_imag.cpu(), (1, 1), (1, 1))
    assert oracle.rel_frobenius(y, ref) <= TOL_3XTF32


def test_default_chunking_several_chunks():
    # 2 MiB per image: 16 MB gives 8 images, at least 3 chunks gives 4 -> chunks of 4.
    layer = _layer(64, 64, 3, 1, 1, seed=3)
    x = _host_batch((12, 64, 64, 64), seed=4)
    out = torch.empty(layer.output_shape(12, 64, 64), dtype=torch.complex64, pin_memory=True)
    y = layer.forward_host(x, out=out)
    assert y is out
    torch.cuda.current_stream().synchronize()
    assert torch.equal(out, _chunk_reference(layer, x, 4))


def test_default_chunking_small_batch():
    # 3.2 MB per image, batch 8: 16 MB gives 5 images, at least 3 chunks gives 3.
    layer = _layer(128, 128, 3, 1, 1, seed=13)
    x = _host_batch((8, 128, 56, 56), seed=14)
    y = layer.forward_host(x)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(y, _chunk_reference(layer, x, 3))


def test_back_to_back_calls_reuse_out():
    layer = _layer(32, 32, 3, 1, 1, seed=5)
    xa = _host_batch((6, 32, 24, 24), seed=6)
    xb = _host_batch((6, 32, 24, 24), seed=7)
    out_a = torch.full(layer.output_shape(6, 24, 24), float("nan"), dtype=torch.complex64).pin_memory()
    out_b = out_a.clone().pin_memory()
    layer.forward_host(xa, out=out_a, images_per_chunk=2)
    layer.forward_host(xb, out=out_b, images_per_chunk=4)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(out_a, _chunk_reference(layer, xa, 2))
    assert torch.equal(out_b, _chunk_reference(layer, xb, 4))
    # Same output buffer again, other input: no stale chunk survives.
    layer.forward_host(xb, out=out_a, images_per_chunk=3)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(out_a, _chunk_reference(layer, xb, 3))


def test_empty_batch():
    layer = _layer(8, 12, 3, 1, 1, seed=8)
    x = torch.empty((0, 8, 9, 9), dtype=torch.complex64).pin_memory()
    y = layer.forward_host(x)
    assert tuple(y.shape) == (0, 12, 9, 9)


def test_rejects_bad_arguments():
    layer = _layer(8, 12, 3, 1, 1, seed=9)
    x = _host_batch((2, 8, 9, 9), seed=10)
    with pytest.raises(ValueError, match="pinned"):
        layer.forward_host(x.clone())  # pageable copy
    with pytest.raises(ValueError, match="forward for CUDA"):
        layer.forward_host(x.cuda())
    with pytest.raises(ValueError, match="shape"):
        layer.forward_host(x, out=torch.empty((2, 12, 8, 8), dtype=torch.complex64).pin_memory())
    with pytest.raises(ValueError, match="images_per_chunk"):
        layer.forward_host(x, images_per_chunk=0)
