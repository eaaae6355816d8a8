"""CPU oracle for the complex Conv2d forward path (and its gradients).

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this file:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg use it, and only as the checker or as the timed CPU baseline.

Parity anchor: the reference's own algorithm is the four-real-Conv2d formula
``apply_complex`` in ``benchmarks/baseline.py:5-9`` (duplicated in
``tests/test_correctness.py:8-12``):

    y = (conv_r(x.real) - conv_i(x.imag)) + 1j * (conv_r(x.imag) + conv_i(x.real))

where ``conv_r``/``conv_i`` are bias-free ``nn.Conv2d`` layers holding the real
and imaginary weight planes (KCRS), with the layer's stride and zero padding
(``benchmarks/baseline.py:12-45``).  The result is cast to complex64
(``baseline.py:7-8``).

Three restatements live here:
  * ``four_conv``            - the same four-conv formula on CPU torch, in a
                               chosen precision (fp64 for parity, fp32 for the
                               timed CPU baseline).
  * ``im2col_numpy``         - an independent numpy fp64 restatement (explicit
                               im2col + matmul), used to pin ``four_conv``.
  * ``direct_c`` (ctypes)    - plain C fp64 loops (``complex_conv_direct.c``),
                               a third, loop-level restatement for small cases.

The three are pinned against golden vectors produced by running the
reference's ``ReferenceComplexConv2d`` (``benchmarks/baseline.py:12-45``) in
this container; the generating script is ``tests/golden/make_golden.py``.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np
import torch
import torch.nn.functional as F

_HERE = os.path.dirname(os.path.abspath(__file__))


# --------------------------------------------------------------------------
# Problem description and seeded inputs
# --------------------------------------------------------------------------
@dataclass(frozen=True)
class ConvCase:
    """One complex Conv2d problem: NCHW input, KCRS weight, square stride/pad
    allowed to differ per axis.  Mirrors the arguments of
    ``ReferenceComplexConv2d(in_channels, out_channels, kernel_size, stride,
    padding)`` (``benchmarks/baseline.py:15-22``) plus the batch and image
    size of ``BenchmarkCase`` (``benchmarks/benchmark_conv2d.py:14-25``)."""

    n: int
    c: int
    h: int
    w: int
    k: int
    r: int
    s: int
    stride_h: int = 1
    stride_w: int = 1
    pad_h: int = 0
    pad_w: int = 0

    @property
    def p(self) -> int:
        # Output height, complex_conv2d.cu:151-152 (floor division).
        return (self.h + 2 * self.pad_h - self.r) // self.stride_h + 1

    @property
    def q(self) -> int:
        # Output width, complex_conv2d.cu:154-155.
        return (self.w + 2 * self.pad_w - self.s) // self.stride_w + 1

    @property
    def flops(self) -> int:
        """Effective flops: 8 real flops per complex multiply-accumulate."""
        return 8 * self.n * self.p * self.q * self.k * self.c * self.r * self.s

    @property
    def algorithmic_bytes(self) -> int:
        """Each complex64 tensor (input, weight, output) touched once."""
        return 8 * (self.n * self.h * self.w * self.c
                    + self.k * self.r * self.s * self.c
                    + self.n * self.p * self.q * self.k)


def make_inputs(case: ConvCase, input_seed: int = 0, weight_seed: int = 1,
                input_std: float = 1.0):
    """Seeded synthetic inputs with the distributions BASELINE.json names.

    Real and imaginary input parts are drawn independently as fp32 N(0, std^2)
    (``torch.randn(complex64)`` would give N(0, 1/2) per part instead).
    Weights are U(-1/sqrt(C*R*S), +1/sqrt(C*R*S)) per plane, the default
    ``nn.Conv2d`` initialisation range used by the reference tests
    (``tests/test_correctness.py:72-88``).

    Returns (x complex64 NCHW, w_real fp32 KCRS, w_imag fp32 KCRS), all CPU.
    """
    g = torch.Generator().manual_seed(input_seed)
    xr = torch.randn(case.n, case.c, case.h, case.w, generator=g) * input_std
    xi = torch.randn(case.n, case.c, case.h, case.w, generator=g) * input_std
    x = torch.complex(xr, xi)
    gw = torch.Generator().manual_seed(weight_seed)
    bound = 1.0 / float(np.sqrt(case.c * case.r * case.s))
    shape = (case.k, case.c, case.r, case.s)
    wr = (torch.rand(shape, generator=gw) * 2.0 - 1.0) * bound
    wi = (torch.rand(shape, generator=gw) * 2.0 - 1.0) * bound
    return x, wr.float(), wi.float()


# --------------------------------------------------------------------------
# Restatement 1: the reference's four-real-conv formula on CPU torch
# --------------------------------------------------------------------------
def four_conv(x: torch.Tensor, w_real: torch.Tensor, w_imag: torch.Tensor,
              stride=(1, 1), padding=(0, 0),
              dtype: torch.dtype = torch.float64) -> torch.Tensor:
    """``apply_complex`` (``benchmarks/baseline.py:5-9``) evaluated on CPU.

    ``x`` is complex NCHW; weights are KCRS real planes.  Every conv runs in
    ``dtype``; the result is returned as complex128 for fp64 and complex64
    for fp32 (the reference casts to complex64, ``baseline.py:7-8``).
    """
    xr = x.real.to(dtype)
    xi = x.imag.to(dtype)
    wr = w_real.to(dtype)
    wi = w_imag.to(dtype)

    def conv(inp, w):
        return F.conv2d(inp, w, bias=None, stride=tuple(stride),
                        padding=tuple(padding))

    yr = conv(xr, wr) - conv(xi, wi)
    yi = conv(xi, wr) + conv(xr, wi)
    return torch.complex(yr, yi)


# --------------------------------------------------------------------------
# Restatement 2: explicit im2col + matmul in numpy fp64
# --------------------------------------------------------------------------
def im2col_numpy(x: np.ndarray, w_real: np.ndarray, w_imag: np.ndarray,
                 stride=(1, 1), padding=(0, 0)) -> np.ndarray:
    """Complex cross-correlation (``Mode::kCrossCorrelation``,
    ``complex_conv2d.cu:194``) as an implicit-GEMM restatement:
    M = N*P*Q output pixels, N = K output channels, K = R*S*C reduction, the
    same GEMM view the reference kernel tiles (``kernel/...:286-505``).

    Inputs: x complex NCHW, weights KCRS.  Output complex128 NCHW.
    """
    x = np.asarray(x, dtype=np.complex128)
    w = np.asarray(w_real, np.float64) + 1j * np.asarray(w_imag, np.float64)
    n, c, h, wd = x.shape
    k, c2, r, s = w.shape
    assert c == c2
    sh, sw = stride
    ph, pw = padding
    p = (h + 2 * ph - r) // sh + 1
    q = (wd + 2 * pw - s) // sw + 1
    xp = np.zeros((n, c, h + 2 * ph, wd + 2 * pw), np.complex128)
    xp[:, :, ph:ph + h, pw:pw + wd] = x
    # cols[n, p, q, c, r, s]
    cols = np.empty((n, p, q, c, r, s), np.complex128)
    for rr in range(r):
        for ss in range(s):
            cols[:, :, :, :, rr, ss] = xp[:, :, rr:rr + sh * (p - 1) + 1:sh,
                                          ss:ss + sw * (q - 1) + 1:sw].transpose(0, 2, 3, 1)
    a = cols.reshape(n * p * q, c * r * s)
    b = w.reshape(k, c * r * s).T
    y = a @ b  # complex matmul: (ar*br - ai*bi) + i(ar*bi + ai*br)
    return y.reshape(n, p, q, k).transpose(0, 3, 1, 2)


# --------------------------------------------------------------------------
# Restatement 3: plain C direct loops (fp64), via ctypes
# --------------------------------------------------------------------------
_direct_lib: Optional[ctypes.CDLL] = None


def _lib_path() -> str:
    return os.path.join(_HERE, "_build", "libccv_oracle.so")


def build_c_oracle(verbose: bool = False) -> str:
    """Compile ``complex_conv_direct.c`` with gcc into ``oracle/_build``."""
    import subprocess
    out = _lib_path()
    os.makedirs(os.path.dirname(out), exist_ok=True)
    src = os.path.join(_HERE, "complex_conv_direct.c")
    if (not os.path.exists(out)) or os.path.getmtime(out) < os.path.getmtime(src):
        cmd = ["gcc", "-O2", "-fPIC", "-shared", "-std=c99", src, "-o", out, "-lm"]
        if verbose:
            print(" ".join(cmd))
        subprocess.check_call(cmd)
    return out


def _load_direct() -> ctypes.CDLL:
    global _direct_lib
    if _direct_lib is None:
        path = build_c_oracle()
        lib = ctypes.CDLL(path)
        f = lib.ccv_oracle_direct_fprop
        f.restype = ctypes.c_int
        f.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int64] * 11
        _direct_lib = lib
    return _direct_lib


def direct_c(x: np.ndarray, w_real: np.ndarray, w_imag: np.ndarray,
             stride=(1, 1), padding=(0, 0)) -> np.ndarray:
    """Complex fprop by the C loop restatement.  x complex NCHW, weights KCRS.
    Returns complex128 NCHW."""
    lib = _load_direct()
    x = np.asarray(x)
    n, c, h, wd = x.shape
    k, _, r, s = np.asarray(w_real).shape
    sh, sw = stride
    ph, pw = padding
    p = (h + 2 * ph - r) // sh + 1
    q = (wd + 2 * pw - s) // sw + 1
    xr = np.ascontiguousarray(x.real, np.float64)
    xi = np.ascontiguousarray(x.imag, np.float64)
    wr = np.ascontiguousarray(w_real, np.float64)
    wi = np.ascontiguousarray(w_imag, np.float64)
    yr = np.zeros((n, k, p, q), np.float64)
    yi = np.zeros((n, k, p, q), np.float64)
    rc = lib.ccv_oracle_direct_fprop(
        xr.ctypes.data, xi.ctypes.data, wr.ctypes.data, wi.ctypes.data,
        yr.ctypes.data, yi.ctypes.data, n, h, wd, c, k, r, s, sh, sw, ph, pw)
    if rc != 0:
        raise ValueError(f"ccv_oracle_direct_fprop rejected the problem (rc={rc})")
    return yr + 1j * yi


# --------------------------------------------------------------------------
# Error metrics
# --------------------------------------------------------------------------
def rel_frobenius(y, y_ref) -> float:
    """||y - y_ref||_F / ||y_ref||_F over the complex values, in fp64."""
    a = torch.as_tensor(np.asarray(y.cpu() if torch.is_tensor(y) else y)).to(torch.complex128)
    b = torch.as_tensor(np.asarray(y_ref.cpu() if torch.is_tensor(y_ref) else y_ref)).to(torch.complex128)
    den = torch.linalg.vector_norm(b).item()
    num = torch.linalg.vector_norm(a - b).item()
    return num / den if den > 0 else num


def planar_nhwc_to_complex_nchw(y_real: torch.Tensor, y_imag: torch.Tensor) -> torch.Tensor:
    """The output reconstruction of ``modules.py:204-207``."""
    return torch.complex(y_real.permute(0, 3, 1, 2).contiguous(),
                         y_imag.permute(0, 3, 1, 2).contiguous())


def oracle_fp64(case: ConvCase, x: torch.Tensor, w_real: torch.Tensor,
                w_imag: torch.Tensor, bias_real: Optional[torch.Tensor] = None,
                bias_imag: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The parity oracle used by the GPU tests: fp64 four-conv on CPU.

    With ``bias_real``/``bias_imag`` (K values each), the complex bias
    ``bias_real[k] + 1j * bias_imag[k]`` is added to output channel k - the
    bias of ``torch.nn.Conv2d`` on complex tensors.  The reference has no
    bias (``modules.py:73-74`` rejects it; ``benchmarks/baseline.py:27-42``
    builds its convolutions with ``bias=False``), so this extension is
    restated here from that definition.
    """
    y = four_conv(x.cpu(), w_real.cpu(), w_imag.cpu(),
                  (case.stride_h, case.stride_w), (case.pad_h, case.pad_w),
                  dtype=torch.float64)
    if bias_real is not None:
        b = torch.complex(bias_real.cpu().double(), bias_imag.cpu().double())
        y = y + b.view(1, -1, 1, 1)
    return y


# --------------------------------------------------------------------------
# Backward (data and weight gradients)
# --------------------------------------------------------------------------
def backward_autograd_fp64(case: ConvCase, x: torch.Tensor, w_real: torch.Tensor,
                           w_imag: torch.Tensor, dy: torch.Tensor):
    """Vector-Jacobian product of the four-conv formula, by torch autograd in fp64.

    The reference module is built from ``nn.Conv2d`` layers
    (``benchmarks/baseline.py:12-45``), so autograd differentiates it; with
    the upstream gradient ``dy`` (complex, shape of the output) this returns
    what ``torch.autograd.grad(y, (x, conv_real.weight, conv_imag.weight),
    grad_outputs=dy)`` gives for it: (dx complex128 NCHW, dw_real, dw_imag
    fp64 KCRS).  PyTorch's complex convention (conjugate Wirtinger) makes
    dx = conv_transpose(dy, conj(W)) and dW = sum dy * conj(x).
    """
    xx = x.cpu().to(torch.complex128).requires_grad_(True)
    wr = w_real.cpu().double().requires_grad_(True)
    wi = w_imag.cpu().double().requires_grad_(True)
    y = four_conv(xx, wr, wi, (case.stride_h, case.stride_w), (case.pad_h, case.pad_w),
                  dtype=torch.float64)
    dx, dwr, dwi = torch.autograd.grad(y, (xx, wr, wi),
                                       grad_outputs=dy.cpu().to(torch.complex128))
    return dx.detach(), dwr.detach(), dwi.detach()


def backward_formula_fp64(case: ConvCase, x: torch.Tensor, w_real: torch.Tensor,
                          w_imag: torch.Tensor, dy: torch.Tensor):
    """The same gradients from their closed forms, without autograd:

        dx[n,c,h,w]  = sum_{k,r,s} conj(W[k,c,r,s]) dy[n,k,p,q]
        dW[k,c,r,s]  = sum_{n,p,q} dy[n,k,p,q] conj(x[n,c,h,w])

    over h = p*sh - ph + r, w = q*sw - pw + s (numpy fp64 loops over the
    filter taps; zero padding outside the image).  Returns (dx, dw_real,
    dw_imag) like ``backward_autograd_fp64``.
    """
    xn = x.cpu().to(torch.complex128).numpy()
    g = dy.cpu().to(torch.complex128).numpy()
    W = (w_real.cpu().double() + 1j * w_imag.cpu().double()).numpy()
    n, c, h, w = xn.shape
    k, _, r_, s_ = W.shape
    p, q = case.p, case.q
    sh, sw, ph, pw = case.stride_h, case.stride_w, case.pad_h, case.pad_w
    xp = np.zeros((n, c, h + 2 * ph + sh * p, w + 2 * pw + sw * q), dtype=np.complex128)
    xp[:, :, ph:ph + h, pw:pw + w] = xn
    dxp = np.zeros_like(xp)
    dW = np.zeros_like(W)
    for r in range(r_):
        for s in range(s_):
            # Input pixels read by tap (r, s): rows r + sh*p', cols s + sw*q'.
            patch = xp[:, :, r:r + sh * p:sh, s:s + sw * q:sw]          # n c p q
            dW[:, :, r, s] = np.einsum("nkpq,ncpq->kc", g, np.conj(patch))
            dxp[:, :, r:r + sh * p:sh, s:s + sw * q:sw] += np.einsum(
                "kc,nkpq->ncpq", np.conj(W[:, :, r, s]), g)
    dx = dxp[:, :, ph:ph + h, pw:pw + w]
    return (torch.from_numpy(dx.copy()), torch.from_numpy(dW.real.copy()),
            torch.from_numpy(dW.imag.copy()))


def time_cpu_four_conv(case: ConvCase, iters: int, warmup: int = 1,
                       threads: Optional[int] = None) -> Tuple[float, int]:
    """Time the reference's four-conv path in fp32 on the host CPU.

    Returns (seconds per call, threads used).  This is the reported CPU
    baseline (``benchmarks/baseline.py:5-45`` run on CPU), not a target.
    """
    import time
    if threads is not None:
        torch.set_num_threads(threads)
    x, wr, wi = make_inputs(case)
    st = (case.stride_h, case.stride_w)
    pd = (case.pad_h, case.pad_w)
    with torch.no_grad():
        for _ in range(warmup):
            four_conv(x, wr, wi, st, pd, dtype=torch.float32)
        t0 = time.perf_counter()
        for _ in range(iters):
            four_conv(x, wr, wi, st, pd, dtype=torch.float32)
        dt = (time.perf_counter() - t0) / max(iters, 1)
    return dt, torch.get_num_threads()
