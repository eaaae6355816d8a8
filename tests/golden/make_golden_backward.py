"""Generate golden gradient vectors by differentiating the reference's own
four-real-Conv2d module (``benchmarks/baseline.py:12-45``,
``ReferenceComplexConv2d``) with torch autograd in this container.

Run from the repository root, with the reference checkout available:

    python tests/golden/make_golden_backward.py --reference <path-to-reference-checkout>

The reference has no backward of its own CUDA path (its README lists
backward as absent), but its benchmark module is made of ``nn.Conv2d``
layers, so autograd gives the gradients of exactly the reference's
formula.  For each case of ``make_golden.py`` (same inputs and weights) an
upstream gradient ``dy`` (complex64, real/imag iid N(0,1), seeded) is drawn
and

    dx, dw_real, dw_imag = torch.autograd.grad(
        y, (x, conv_real.weight, conv_imag.weight), grad_outputs=dy)

is stored, with the module converted by ``.double()`` and fed a complex128
``x`` (``apply_complex`` casts its result to complex64, so ``dy`` is
complex64 and the gradients are fp64 / complex128).
"""

import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import make_inputs  # noqa: E402


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=os.path.join(HERE, "golden_backward.npz"))
    args = ap.parse_args()
    ref = _load(os.path.join(args.reference, "benchmarks", "baseline.py"), "ref_baseline")
    cases = _load(os.path.join(HERE, "make_golden.py"), "make_golden").CASES
    blobs = {}
    names = []
    for i, (name, c) in enumerate(cases):
        x, wr, wi = make_inputs(c, input_seed=100 + i, weight_seed=200 + i)
        g = torch.Generator().manual_seed(300 + i)
        shape = (c.n, c.k, c.p, c.q)
        dy = torch.complex(torch.randn(shape, generator=g), torch.randn(shape, generator=g))
        m = ref.ReferenceComplexConv2d(c.c, c.k, (c.r, c.s), stride=(c.stride_h, c.stride_w),
                                       padding=(c.pad_h, c.pad_w)).double()
        with torch.no_grad():
            m.conv_real.weight.copy_(wr.double())
            m.conv_imag.weight.copy_(wi.double())
        x64 = x.to(torch.complex128).requires_grad_(True)
        y = m(x64)
        dx, dwr, dwi = torch.autograd.grad(
            y, (x64, m.conv_real.weight, m.conv_imag.weight), grad_outputs=dy)
        names.append(name)
        blobs[f"{name}/dy"] = dy.numpy()
        blobs[f"{name}/dx"] = dx.numpy()
        blobs[f"{name}/dw_real"] = dwr.numpy()
        blobs[f"{name}/dw_imag"] = dwi.numpy()
    blobs["names"] = np.array(names)
    np.savez_compressed(args.out, **blobs)
    print(f"wrote {args.out} ({os.path.getsize(args.out)} bytes, {len(names)} cases)")


if __name__ == "__main__":
    main()
