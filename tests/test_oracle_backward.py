"""Pin the backward oracle against the reference's own gradients.

tests/golden/make_golden_backward.py differentiated the reference's
ReferenceComplexConv2d (benchmarks/baseline.py:12-45) with torch autograd
in fp64 for the golden cases of make_golden.py; both oracle restatements of
the gradients (autograd through the four-conv formula, and the closed forms
dx = conv_transpose(dy, conj W), dW = sum dy conj(x) in numpy loops) must
reproduce them to fp64 rounding.
"""

import os

import numpy as np
import pytest
import torch

import oracle

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _cases():
    fw = np.load(os.path.join(HERE, "golden_vectors.npz"))
    bw = np.load(os.path.join(HERE, "golden_backward.npz"))
    out = []
    for name in bw["names"]:
        name = str(name)
        case = oracle.ConvCase(*fw[f"{name}/meta"].tolist())
        out.append((name, case, fw[f"{name}/x"], fw[f"{name}/w_real"], fw[f"{name}/w_imag"],
                    bw[f"{name}/dy"], bw[f"{name}/dx"], bw[f"{name}/dw_real"],
                    bw[f"{name}/dw_imag"]))
    return out


CASES = _cases()


def test_backward_golden_covers_the_forward_cases():
    assert len(CASES) >= 10
    assert any(c[1].stride_h > 1 for c in CASES) and any(c[1].r == 1 for c in CASES)


@pytest.mark.parametrize("fn", [oracle.backward_autograd_fp64, oracle.backward_formula_fp64],
                         ids=["autograd", "formula"])
@pytest.mark.parametrize("name,case,x,wr,wi,dy,dx,dwr,dwi", CASES, ids=[c[0] for c in CASES])
def test_backward_oracle_matches_reference(fn, name, case, x, wr, wi, dy, dx, dwr, dwi):
    gx, gwr, gwi = fn(case, torch.from_numpy(x), torch.from_numpy(wr), torch.from_numpy(wi),
                      torch.from_numpy(dy))
    assert gx.shape == (case.n, case.c, case.h, case.w)
    assert gwr.shape == (case.k, case.c, case.r, case.s)
    assert oracle.rel_frobenius(gx, torch.from_numpy(dx)) < 1e-12
    assert oracle.rel_frobenius(gwr, torch.from_numpy(dwr)) < 1e-12
    assert oracle.rel_frobenius(gwi, torch.from_numpy(dwi)) < 1e-12
