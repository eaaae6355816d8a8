"""Every BASELINE config through ComplexConv2d.forward() and forward_planar(),
checked on EVERY image (the reference's harness checks both entry points on
each case, benchmarks/benchmark_conv2d.py:98-106).

Checker for whole batches: the reference's four-conv formula
(benchmarks/baseline.py:5-9) on the GPU in fp32 (im2col + SGEMM, TF32 off),
itself pinned to the fp64 CPU oracle on the first and last image of each
config (<= 2e-6 relative Frobenius).  Bars (north star): relative Frobenius
<= 1e-3 for TF32 and <= 1e-5 for 3xTF32, here also per image, so one wrong
image in a batch of 64 cannot hide in the batch norm.  The fp32 checker's
own error (<= 2e-6) is subtracted from the 3xTF32 bar.
"""

import pytest
import torch
import torch.nn.functional as F

import oracle
from oracle.configs import BASELINE_CASES

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TF32_TOL = 1e-3
X3_TOL = 1e-5
CHECKER_TOL = 2e-6


def _gpu_inputs(case, std, seed=0):
    """The seeded inputs of oracle.make_inputs, generated on the GPU for the
    large configs (same distributions; CPU copies of two images for the
    fp64 pin)."""
    x, wr, wi = oracle.make_inputs(oracle.ConvCase(1, case.c, 1, 1, case.k, case.r, case.s),
                                   weight_seed=1)
    del x
    g = torch.Generator(device=DEV).manual_seed(seed)
    xr = torch.randn((case.n, case.c, case.h, case.w), generator=g, device=DEV) * std
    xi = torch.randn((case.n, case.c, case.h, case.w), generator=g, device=DEV) * std
    return torch.complex(xr, xi), wr, wi


def fp32_four_conv_gpu(x, wr, wi, case, images_per_chunk=4):
    """benchmarks/baseline.py:5-9 on the GPU in fp32: each real convolution
    as an explicit im2col (F.unfold) and an fp32 matrix product with TF32
    off, so no Winograd/FFT algorithm choice changes the checker's error."""
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        st, pd = (case.stride_h, case.stride_w), (case.pad_h, case.pad_w)
        k = case.k
        wr2 = wr.to(DEV).reshape(k, -1)
        wi2 = wi.to(DEV).reshape(k, -1)
        out = torch.empty((case.n, k, case.p, case.q), dtype=torch.complex64, device=DEV)
        for i0 in range(0, case.n, images_per_chunk):
            i1 = min(case.n, i0 + images_per_chunk)
            cr = F.unfold(x.real[i0:i1], (case.r, case.s), padding=pd, stride=st)
            ci = F.unfold(x.imag[i0:i1], (case.r, case.s), padding=pd, stride=st)
            yr = torch.matmul(wr2, cr) - torch.matmul(wi2, ci)
            yi = torch.matmul(wr2, ci) + torch.matmul(wi2, cr)
            out[i0:i1] = torch.complex(yr, yi).view(i1 - i0, k, case.p, case.q)
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old


def per_image_rel(y, ref):
    """Relative Frobenius error of each image (fp64 on the GPU)."""
    d = (y.to(torch.complex128) - ref.to(torch.complex128)).abs().pow(2).flatten(1).sum(1)
    r = ref.to(torch.complex128).abs().pow(2).flatten(1).sum(1)
    return (d / r).sqrt()


def _module(case, wr, wi, precision):
    from complex_conv2d import ComplexConv2d
    layer = ComplexConv2d(case.c, case.k, (case.r, case.s), stride=(case.stride_h, case.stride_w),
                          padding=(case.pad_h, case.pad_w), device=DEV, precision=precision)
    with torch.no_grad():
        layer.weight_real.copy_(wr)
        layer.weight_imag.copy_(wi)
    return layer


RUNS = [(name, case, std, prec) for name, case, std, precs in BASELINE_CASES for prec in precs]


@pytest.mark.parametrize("name,case,std,precision", RUNS, ids=[f"{r[0]}-{r[3]}" for r in RUNS])
def test_baseline_every_image_forward_and_planar(name, case, std, precision):
    torch.cuda.set_device(0)
    x, wr, wi = _gpu_inputs(case, std)
    ref = fp32_four_conv_gpu(x, wr, wi, case)
    # Pin the checker to the fp64 oracle on the first and last image.
    sub = oracle.ConvCase(1, case.c, case.h, case.w, case.k, case.r, case.s,
                          case.stride_h, case.stride_w, case.pad_h, case.pad_w)
    for img in sorted({0, case.n - 1}):
        ref64 = oracle.oracle_fp64(sub, x[img:img + 1].cpu(), wr, wi)
        assert oracle.rel_frobenius(ref[img:img + 1].cpu(), ref64) <= CHECKER_TOL, (name, img)
    bar = TF32_TOL if precision == "tf32" else X3_TOL - CHECKER_TOL
    layer = _module(case, wr, wi, precision)
    with torch.no_grad():
        y = layer(x)
        torch.cuda.synchronize()
        assert not torch.isnan(y.real).any() and not torch.isnan(y.imag).any(), name
        errs = per_image_rel(y, ref)
        assert errs.max().item() <= bar, (name, "forward", errs.argmax().item(), errs.max().item())
        del y
        xr = x.real.permute(0, 2, 3, 1).contiguous()
        xi = x.imag.permute(0, 2, 3, 1).contiguous()
        yr, yi = layer.forward_planar(xr, xi)
        del xr, xi
        yp = torch.complex(yr.permute(0, 3, 1, 2), yi.permute(0, 3, 1, 2))
        del yr, yi
        torch.cuda.synchronize()
        assert not torch.isnan(yp.real).any() and not torch.isnan(yp.imag).any(), name
        errs = per_image_rel(yp, ref)
        assert errs.max().item() <= bar, (name, "planar", errs.argmax().item(), errs.max().item())


def test_cpu_config_forward_and_planar():
    """configs[0] (the reference's CPU-runnable case) on the GPU against fp64."""
    from oracle.configs import CPU_CASE
    case = CPU_CASE
    x, wr, wi = oracle.make_inputs(case)
    layer = _module(case, wr, wi, "tf32")
    ref = oracle.oracle_fp64(case, x, wr, wi)
    with torch.no_grad():
        y = layer(x.to(DEV))
        yr, yi = layer.forward_planar(x.real.permute(0, 2, 3, 1).contiguous().to(DEV),
                                      x.imag.permute(0, 2, 3, 1).contiguous().to(DEV))
    torch.cuda.synchronize()
    assert oracle.rel_frobenius(y.cpu(), ref) <= TF32_TOL
    assert oracle.rel_frobenius(oracle.planar_nhwc_to_complex_nchw(yr, yi).cpu(), ref) <= TF32_TOL
