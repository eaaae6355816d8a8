"""Pin the CPU oracle against the reference's own outputs (golden vectors).

The golden vectors come from running the reference's ReferenceComplexConv2d
(benchmarks/baseline.py:12-45) in fp32 and fp64; see
tests/golden/make_golden.py.  All three oracle restatements must agree with
the fp64 golden output to complex64 rounding, and with the fp32 golden
output to fp32 accumulation error.
"""

import os

import numpy as np
import pytest
import torch

import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_vectors.npz")


def _cases():
    z = np.load(GOLDEN)
    out = []
    for name in z["names"]:
        name = str(name)
        meta = z[f"{name}/meta"].tolist()
        case = oracle.ConvCase(*meta)
        out.append((name, case, z[f"{name}/x"], z[f"{name}/w_real"], z[f"{name}/w_imag"],
                    z[f"{name}/y32"], z[f"{name}/y64"]))
    return out


CASES = _cases()


def test_golden_file_has_all_variants():
    names = {c[0] for c in CASES}
    # 1x1, 3x3 s1 p1, stride 2, pad 0, batch 2, non-square, 5x5, 7x7, rectangular kernel
    assert len(names) >= 10
    kinds = {(c[1].r, c[1].s, c[1].stride_h, c[1].pad_h) for c in CASES}
    assert (1, 1, 1, 0) in kinds and (3, 3, 2, 1) in kinds and (3, 3, 1, 0) in kinds
    assert any(c[1].n > 1 for c in CASES)
    assert any(c[1].h != c[1].w for c in CASES)


@pytest.mark.parametrize("name,case,x,wr,wi,y32,y64", CASES, ids=[c[0] for c in CASES])
def test_four_conv_fp64_matches_reference(name, case, x, wr, wi, y32, y64):
    y = oracle.four_conv(torch.from_numpy(x), torch.from_numpy(wr), torch.from_numpy(wi),
                         (case.stride_h, case.stride_w), (case.pad_h, case.pad_w))
    assert y.shape == (case.n, case.k, case.p, case.q)
    # y64 is the fp64 reference rounded to complex64.
    assert oracle.rel_frobenius(y.numpy(), y64) < 2e-7
    assert oracle.rel_frobenius(y.numpy(), y32) < 2e-6


@pytest.mark.parametrize("name,case,x,wr,wi,y32,y64", CASES, ids=[c[0] for c in CASES])
def test_im2col_numpy_matches_reference(name, case, x, wr, wi, y32, y64):
    y = oracle.im2col_numpy(x, wr, wi, (case.stride_h, case.stride_w), (case.pad_h, case.pad_w))
    assert oracle.rel_frobenius(y, y64) < 2e-7


@pytest.mark.parametrize("name,case,x,wr,wi,y32,y64", CASES, ids=[c[0] for c in CASES])
def test_direct_c_matches_reference(name, case, x, wr, wi, y32, y64):
    y = oracle.direct_c(x, wr, wi, (case.stride_h, case.stride_w), (case.pad_h, case.pad_w))
    assert oracle.rel_frobenius(y, y64) < 2e-7


def test_output_size_rule():
    # complex_conv2d.cu:151-155 (floor division)
    c = oracle.ConvCase(1, 4, 112, 112, 8, 3, 3, 2, 2, 1, 1)
    assert (c.p, c.q) == (56, 56)
    c = oracle.ConvCase(1, 4, 7, 9, 8, 3, 1, 2, 1, 1, 0)
    assert (c.p, c.q) == (4, 9)


def test_flops_and_bytes_convention():
    c = oracle.ConvCase(64, 128, 56, 56, 128, 3, 3, 1, 1, 1, 1)
    assert c.flops == 8 * 64 * 56 * 56 * 128 * 128 * 9
    assert abs(c.flops / 1e9 - 236.8) < 0.1


def test_make_inputs_distribution():
    c = oracle.ConvCase(2, 32, 16, 16, 32, 3, 3, 1, 1, 1, 1)
    x, wr, wi = oracle.make_inputs(c)
    assert x.dtype == torch.complex64
    assert abs(x.real.var().item() - 1.0) < 0.1 and abs(x.imag.var().item() - 1.0) < 0.1
    bound = 1.0 / np.sqrt(32 * 9)
    assert wr.abs().max().item() <= bound and wi.abs().max().item() <= bound
    x2, _, _ = oracle.make_inputs(c)
    assert torch.equal(x, x2)  # seeded


def test_rel_frobenius_detects_planted_error():
    # A mistake planted in the oracle output must be caught at the TF32 bar.
    z = CASES[0]
    y = z[6].astype(np.complex128).copy()
    y.flat[7] += 0.05 * np.abs(y).max()
    assert oracle.rel_frobenius(y, z[6]) > 1e-3
