"""Generate golden input/output vectors by running the reference's own
four-real-Conv2d module (``benchmarks/baseline.py:12-45``,
``ReferenceComplexConv2d``) in this container.

Run from the repository root, with the reference checkout available:

    python tests/golden/make_golden.py --reference <path-to-reference-checkout>

The reference cannot travel to the GPU box, so its outputs are committed as
small fixtures (``golden_vectors.npz``) that the CPU tests use to pin the
oracle.  Inputs are seeded: real/imag input parts iid N(0,1), weight planes
U(+-1/sqrt(C*R*S)), drawn with the oracle's ``make_inputs``.

Two outputs are stored per case:
  * ``y32``: the reference module in fp32 on CPU (its default dtype);
  * ``y64``: the reference module converted with ``.double()`` and fed a
    complex128 input.  ``apply_complex`` casts its result to complex64
    (``baseline.py:7-8``), so this is the fp64 result rounded to complex64.
"""

import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import ConvCase, make_inputs  # noqa: E402

# (name, case, kernel_size as passed to the reference constructor)
CASES = [
    ("k3_s1_p1_c32", ConvCase(1, 32, 8, 8, 32, 3, 3, 1, 1, 1, 1)),
    ("k1_s1_p0", ConvCase(1, 16, 8, 8, 24, 1, 1, 1, 1, 0, 0)),
    ("k3_s2_p1", ConvCase(1, 16, 9, 9, 16, 3, 3, 2, 2, 1, 1)),
    ("k3_s1_p0", ConvCase(1, 8, 10, 10, 16, 3, 3, 1, 1, 0, 0)),
    ("k3_b2", ConvCase(2, 8, 8, 8, 16, 3, 3, 1, 1, 1, 1)),
    ("k3_nonsquare", ConvCase(1, 8, 6, 10, 8, 3, 3, 1, 1, 1, 1)),
    ("k5_s1_p2_c4", ConvCase(1, 4, 7, 7, 4, 5, 5, 1, 1, 2, 2)),
    ("k7_s2_p3", ConvCase(1, 4, 11, 13, 8, 7, 7, 2, 2, 3, 3)),
    ("k3x1_s2x1_p1x0", ConvCase(1, 8, 7, 9, 12, 3, 1, 2, 1, 1, 0)),
    ("k1_1x1_image", ConvCase(1, 4, 1, 1, 4, 1, 1, 1, 1, 0, 0)),
    ("k3_c36_k20", ConvCase(1, 36, 5, 6, 20, 3, 3, 1, 1, 1, 1)),
]


def load_reference(ref_root):
    path = os.path.join(ref_root, "benchmarks", "baseline.py")
    spec = importlib.util.spec_from_file_location("ref_baseline", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                  "golden_vectors.npz"))
    args = ap.parse_args()
    ref = load_reference(args.reference)
    torch.manual_seed(0)
    blobs = {}
    names = []
    for i, (name, c) in enumerate(CASES):
        x, wr, wi = make_inputs(c, input_seed=100 + i, weight_seed=200 + i)
        m = ref.ReferenceComplexConv2d(c.c, c.k, (c.r, c.s), stride=(c.stride_h, c.stride_w),
                                       padding=(c.pad_h, c.pad_w)).eval()
        with torch.no_grad():
            m.conv_real.weight.copy_(wr)
            m.conv_imag.weight.copy_(wi)
            y32 = m(x)
            m64 = m.double()
            y64 = m64(x.to(torch.complex128))
        assert y32.dtype == torch.complex64 and y64.dtype == torch.complex64
        names.append(name)
        blobs[f"{name}/meta"] = np.array([c.n, c.c, c.h, c.w, c.k, c.r, c.s, c.stride_h,
                                          c.stride_w, c.pad_h, c.pad_w], np.int64)
        blobs[f"{name}/x"] = x.numpy()
        blobs[f"{name}/w_real"] = wr.numpy()
        blobs[f"{name}/w_imag"] = wi.numpy()
        blobs[f"{name}/y32"] = y32.numpy()
        blobs[f"{name}/y64"] = y64.numpy()
    blobs["names"] = np.array(names)
    np.savez_compressed(args.out, **blobs)
    print(f"wrote {args.out} ({os.path.getsize(args.out)} bytes, {len(names)} cases)")


if __name__ == "__main__":
    main()
