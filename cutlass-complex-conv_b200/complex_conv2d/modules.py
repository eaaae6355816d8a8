"""``ComplexConv2d``: the drop-in module (reference ``complex_conv2d/modules.py``).

Constructor signature, validation, error types and messages, parameters
(``weight_real``/``weight_imag``, fp32 KCRS, ``requires_grad=False``),
initialisation and the cache-invalidation rules follow
``modules.py:21-207`` of the reference.  What changes is what runs:

* the lazy prepack (``modules.py:127-151``) builds the packed weight image of
  the B200 kernels (per tap: -W_im, W_re, W_im planes, TF32-rounded; 3xTF32
  adds the rounding remainders) instead of a KRSC copy;
* ``forward_planar`` calls the tcgen05 kernel on NHWC planes;
* ``forward`` hands the complex64 NCHW tensor to the native entry point,
  which does the NCHW->planar conversion and writes complex64 NCHW output
  itself, instead of the five ATen layout kernels of ``modules.py:198-207``.

One capability is added: ``bias=True`` (rejected by the reference at
``modules.py:73-74``) gives the layer a complex bias per output channel,
``bias_real + 1j * bias_imag``, added in the kernels' epilogue.
"""

import os

import torch
from torch import nn

from ._extension import cutlass_complex_conv

_PRECISIONS = {"tf32": 0, "3xtf32": 1}
# Input bytes per chunk in the middle of forward_host's pipeline.
_HOST_CHUNK_BYTES = 24 << 20


def _host_chunks(n, middle):
    """Chunk sizes (images) of forward_host's default schedule for n images.

    The pipeline's two ends have only one PCIe direction busy: the first
    chunk's copy-in runs before any copy-out and the last chunk's copy-out
    after every copy-in.  So the chunks ramp up 1, 2, 4, ... to `middle`
    images and back down at the end, which keeps both ends short while the
    middle chunks stay large (few calls).  Small batches get >= 3 equal
    chunks.
    """
    head = []
    c = 1
    while c < middle:
        head.append(c)
        c *= 2
    if 2 * sum(head) + middle > n:
        per = max(1, min(middle, -(-n // 3)))
        return [min(per, n - i) for i in range(0, n, per)]
    rest = n - 2 * sum(head)
    mid = [middle] * (rest // middle) + ([rest % middle] if rest % middle else [])
    return head + mid + head[::-1]
_WEIGHT_KCRS = 0


def _pair(value, name):
    """Int or 2-sequence of ints -> tuple (``modules.py:7-18``)."""
    if isinstance(value, int):
        return (value, value)

    if (
        isinstance(value, (tuple, list))
        and len(value) == 2
        and all(isinstance(v, int) for v in value)
    ):
        return (int(value[0]), int(value[1]))

    raise TypeError(f"{name} must be an int or a pair of ints")


def _resolve_precision(precision):
    if precision is None:
        precision = os.environ.get("COMPLEX_CONV2D_PRECISION", "tf32")
    key = str(precision).lower()
    if key not in _PRECISIONS:
        raise ValueError(
            f"precision must be one of {sorted(_PRECISIONS)}, got {precision!r}"
        )
    return key


def _aligned16(t):
    return t.data_ptr() % 16 == 0


class _ComplexConv2dFunction(torch.autograd.Function):
    """``forward()`` as an autograd node: the backward runs the library's data
    gradient (``ccv_dgrad_complex``) and weight gradient
    (``ccv_wgrad_complex``) kernels.  Gradients follow PyTorch's complex
    convention (those torch autograd gives for the reference's four-conv
    module, ``benchmarks/baseline.py:12-45``):
    dx = conv_transpose(dy, conj(W)), dW = sum dy * conj(x),
    d weight_real = Re dW, d weight_imag = Im dW, d bias = sum dy."""

    @staticmethod
    def forward(ctx, x, weight_real, weight_imag, bias_real, bias_imag, module):
        ctx.module = module
        ctx.save_for_backward(x)
        return module._forward_impl(x)

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        m = ctx.module
        dy = dy.contiguous()
        dx = dwr = dwi = dbr = dbi = None
        if ctx.needs_input_grad[0]:
            dx = m._data_grad(dy, x.shape[2], x.shape[3])
        if ctx.needs_input_grad[1] or ctx.needs_input_grad[2]:
            dwr, dwi = cutlass_complex_conv.wgrad_complex(
                x, dy, m.kernel_size[0], m.kernel_size[1], m.stride[0], m.stride[1],
                m.padding[0], m.padding[1])
        if ctx.needs_input_grad[3] or ctx.needs_input_grad[4]:
            db = dy.sum(dim=(0, 2, 3))
            dbr, dbi = db.real.contiguous(), db.imag.contiguous()
        return dx, dwr, dwi, dbr, dbi, None


class _ComplexConv2dPlanarFunction(torch.autograd.Function):
    """``forward_planar()`` as an autograd node (two real outputs): the same
    gradients as ``_ComplexConv2dFunction`` on fp32 planes, from the library's
    planar data- and weight-gradient kernels (``ccv_dgrad_planar``,
    ``ccv_wgrad_planar``)."""

    @staticmethod
    def forward(ctx, x_real, x_imag, weight_real, weight_imag, bias_real, bias_imag, module):
        ctx.module = module
        ctx.save_for_backward(x_real, x_imag)
        y_real, y_imag = module._forward_planar_impl(x_real, x_imag)
        return y_real, y_imag

    @staticmethod
    def backward(ctx, dy_real, dy_imag):
        x_real, x_imag = ctx.saved_tensors
        m = ctx.module
        dy_real = dy_real.contiguous()
        dy_imag = dy_imag.contiguous()
        dxr = dxi = dwr = dwi = dbr = dbi = None
        if ctx.needs_input_grad[0] or ctx.needs_input_grad[1]:
            dxr, dxi = m._data_grad_planar(dy_real, dy_imag, x_real.shape[1], x_real.shape[2])
        if ctx.needs_input_grad[2] or ctx.needs_input_grad[3]:
            dwr, dwi = cutlass_complex_conv.wgrad_planar(
                x_real, x_imag, dy_real, dy_imag, m.kernel_size[0], m.kernel_size[1],
                m.stride[0], m.stride[1], m.padding[0], m.padding[1])
        if ctx.needs_input_grad[4] or ctx.needs_input_grad[5]:
            dbr, dbi = dy_real.sum(dim=(0, 1, 2)), dy_imag.sum(dim=(0, 1, 2))
        return dxr, dxi, dwr, dwi, dbr, dbi, None


class ComplexConv2d(nn.Module):
    """Complex-valued 2D convolution on B200 tensor cores.

    The public ``forward`` method accepts a ``torch.complex64`` tensor in NCHW
    format. ``forward_planar`` exposes the planar path and accepts separate
    real/imaginary float32 tensors in contiguous NHWC format.

    ``precision`` selects the tensor-core arithmetic: ``"tf32"`` (default,
    like the reference) or ``"3xtf32"`` (split-TF32, close to FP32 results).
    ``None`` reads ``COMPLEX_CONV2D_PRECISION`` from the environment.

    ``bias=True`` adds a complex bias per output channel (parameters
    ``bias_real`` and ``bias_imag``, fp32 ``[out_channels]``, initialised like
    ``nn.Conv2d``'s bias: U(+-1/sqrt(in_channels * kernel_h * kernel_w))):
    ``y[:, k] += bias_real[k] + 1j * bias_imag[k]``.

    ``forward`` is differentiable (an extension; the reference is inference
    only): when grad mode is on and the input or a parameter requires grad,
    the backward runs the library's data- and weight-gradient kernels
    (parameters are created with ``requires_grad=False`` as in the
    reference; set it to train them).  The weight gradient computes in TF32;
    the data gradient in the layer's precision.  ``forward_planar`` is
    differentiable the same way (gradients of both planes).

    Current limitations (as in the reference):
      - CUDA only (an sm_100 / B200 device)
      - torch.complex64 only
      - dilation=1
      - groups=1
      - padding_mode="zeros"
      - in/out channel counts multiples of 4 (reference kernel alignment)
    """

    def __init__(
        self,
        in_channels,
        out_channels,
        kernel_size,
        stride=1,
        padding=0,
        dilation=1,
        groups=1,
        bias=False,
        padding_mode="zeros",
        device=None,
        dtype=None,
        precision="tf32",
    ):
        super().__init__()

        if in_channels <= 0 or out_channels <= 0:
            raise ValueError("in_channels and out_channels must be positive")

        kernel_size = _pair(kernel_size, "kernel_size")
        stride = _pair(stride, "stride")
        padding = _pair(padding, "padding")
        dilation = _pair(dilation, "dilation")

        if kernel_size[0] <= 0 or kernel_size[1] <= 0:
            raise ValueError("kernel_size must be positive")
        if stride[0] <= 0 or stride[1] <= 0:
            raise ValueError("stride must be positive")
        if padding[0] < 0 or padding[1] < 0:
            raise ValueError("padding must be non-negative")

        if dilation != (1, 1):
            raise NotImplementedError("dilation != 1 is not supported yet")
        if groups != 1:
            raise NotImplementedError("groups != 1 is not supported yet")
        if padding_mode != "zeros":
            raise NotImplementedError(
                'padding_mode other than "zeros" is not supported yet'
            )
        if dtype not in (None, torch.complex64):
            raise NotImplementedError("only torch.complex64 is supported")

        self.in_channels = int(in_channels)
        self.out_channels = int(out_channels)
        self.kernel_size = kernel_size
        self.stride = stride
        self.padding = padding
        self.dilation = dilation
        self.groups = groups
        self.padding_mode = padding_mode
        self.precision = _resolve_precision(precision)

        # PyTorch-facing weights use KCRS layout. They are packed lazily into
        # the kernel's weight image before the first invocation.
        weight_shape = (
            self.out_channels,
            self.in_channels,
            self.kernel_size[0],
            self.kernel_size[1],
        )

        self.weight_real = nn.Parameter(
            torch.empty(weight_shape, device=device, dtype=torch.float32),
            requires_grad=False,
        )
        self.weight_imag = nn.Parameter(
            torch.empty(weight_shape, device=device, dtype=torch.float32),
            requires_grad=False,
        )

        nn.init.kaiming_uniform_(self.weight_real)
        nn.init.kaiming_uniform_(self.weight_imag)

        if bias:
            fan_in = self.in_channels * self.kernel_size[0] * self.kernel_size[1]
            bound = 1.0 / fan_in ** 0.5
            self.bias_real = nn.Parameter(
                torch.empty(self.out_channels, device=device, dtype=torch.float32)
                .uniform_(-bound, bound),
                requires_grad=False,
            )
            self.bias_imag = nn.Parameter(
                torch.empty(self.out_channels, device=device, dtype=torch.float32)
                .uniform_(-bound, bound),
                requires_grad=False,
            )
        else:
            self.register_parameter("bias_real", None)
            self.register_parameter("bias_imag", None)

        self._clear_prepacked_weights()

    def extra_repr(self):
        return (
            f"{self.in_channels}, {self.out_channels}, kernel_size={self.kernel_size}, "
            f"stride={self.stride}, padding={self.padding}, bias={self.bias_real is not None}, "
            f"precision={self.precision!r}"
        )

    def _bias_args(self):
        """``(bias_real, bias_imag)`` as contiguous tensors, or ``(None, None)``."""
        if self.bias_real is None:
            return None, None
        out = []
        for b in (self.bias_real, self.bias_imag):
            b = b.detach().contiguous()
            out.append(b if _aligned16(b) else b.clone())
        return out[0], out[1]

    def _clear_prepacked_weights(self):
        self._w_packed = None
        self._packed_precision = None
        self._weight_version = None
        self._w_packed_dgrad = None
        self._dgrad_key = None

    def _apply(self, fn, recurse=True):
        # nn.Module.to()/cuda()/cpu() may replace or move Parameter storage.
        # Cached packed weights must never outlive the storage they came from.
        self._clear_prepacked_weights()
        result = super()._apply(fn, recurse=recurse)
        self._clear_prepacked_weights()
        return result

    @torch.no_grad()
    def _prepack_weights(self):
        if not self.weight_real.is_cuda or not self.weight_imag.is_cuda:
            raise RuntimeError("ComplexConv2d weights must be on CUDA")

        self._w_packed = cutlass_complex_conv.prepack(
            self.weight_real.detach().contiguous(),
            self.weight_imag.detach().contiguous(),
            _WEIGHT_KCRS,
            _PRECISIONS[self.precision],
        )
        self._packed_precision = self.precision
        self._weight_version = (
            self.weight_real._version,
            self.weight_imag._version,
        )

    def _ensure_prepacked(self):
        version = (
            self.weight_real._version,
            self.weight_imag._version,
        )

        if (
            self._w_packed is None
            or self._weight_version != version
            or self._packed_precision != self.precision
            or self._w_packed.device != self.weight_real.device
        ):
            self._prepack_weights()

    def forward_planar(self, x_real, x_imag):
        """Run the planar path.

        Args:
            x_real: contiguous CUDA float32 tensor in NHWC layout.
            x_imag: contiguous CUDA float32 tensor in NHWC layout.

        Returns:
            ``[y_real, y_imag]`` as contiguous NHWC float32 tensors.
        """
        if torch.is_grad_enabled() and (
            x_real.requires_grad
            or x_imag.requires_grad
            or self.weight_real.requires_grad
            or self.weight_imag.requires_grad
            or (self.bias_real is not None
                and (self.bias_real.requires_grad or self.bias_imag.requires_grad))
        ):
            return list(_ComplexConv2dPlanarFunction.apply(
                x_real, x_imag, self.weight_real, self.weight_imag, self.bias_real,
                self.bias_imag, self))
        return self._forward_planar_impl(x_real, x_imag)

    def _packed_dgrad(self):
        key = (self.weight_real._version, self.weight_imag._version, self.precision,
               self.weight_real.device)
        if self._w_packed_dgrad is None or self._dgrad_key != key:
            self._w_packed_dgrad = cutlass_complex_conv.prepack_dgrad(
                self.weight_real.detach().contiguous(), self.weight_imag.detach().contiguous(),
                self.stride[0], self.stride[1], self.padding[0], self.padding[1],
                _PRECISIONS[self.precision])
            self._dgrad_key = key
        return self._w_packed_dgrad

    def _data_grad_planar(self, dy_real, dy_imag, in_h, in_w):
        """(dx_real, dx_imag) of ``forward_planar`` for upstream planes dy (NPQK)."""
        return cutlass_complex_conv.dgrad_planar_packed(
            dy_real, dy_imag, self._packed_dgrad(), self.in_channels, in_h, in_w,
            self.kernel_size[0], self.kernel_size[1], self.stride[0], self.stride[1],
            self.padding[0], self.padding[1], _PRECISIONS[self.precision])

    def _forward_planar_impl(self, x_real, x_imag):
        self._ensure_prepacked()

        # TMA needs 16-byte aligned bases; copy the rare misaligned view.
        if x_real.is_cuda and x_real.is_contiguous() and not _aligned16(x_real):
            x_real = x_real.clone()
        if x_imag.is_cuda and x_imag.is_contiguous() and not _aligned16(x_imag):
            x_imag = x_imag.clone()

        bias_real, bias_imag = self._bias_args()
        return cutlass_complex_conv.forward_planar_packed(
            x_real,
            x_imag,
            self._w_packed,
            self.in_channels,
            self.out_channels,
            self.kernel_size[0],
            self.kernel_size[1],
            self.stride[0],
            self.stride[1],
            self.padding[0],
            self.padding[1],
            _PRECISIONS[self.precision],
            bias_real,
            bias_imag,
        )

    def forward(self, x):
        """Run complex Conv2d on a torch.complex64 NCHW tensor."""
        if not x.is_cuda:
            raise ValueError("ComplexConv2d input must be on CUDA")
        if x.dtype != torch.complex64:
            raise ValueError(
                f"ComplexConv2d expects torch.complex64 input, got {x.dtype}"
            )
        if x.dim() != 4:
            raise ValueError(
                f"ComplexConv2d expects a 4D NCHW tensor, got {x.dim()}D"
            )
        if x.size(1) != self.in_channels:
            raise ValueError(
                f"expected {self.in_channels} input channels, got {x.size(1)}"
            )
        if x.device != self.weight_real.device:
            raise ValueError(
                "input and ComplexConv2d weights must be on the same CUDA device"
            )

        if torch.is_grad_enabled() and (
            x.requires_grad
            or self.weight_real.requires_grad
            or self.weight_imag.requires_grad
            or (self.bias_real is not None
                and (self.bias_real.requires_grad or self.bias_imag.requires_grad))
        ):
            return _ComplexConv2dFunction.apply(
                x, self.weight_real, self.weight_imag, self.bias_real, self.bias_imag, self)
        return self._forward_impl(x)

    def _data_grad(self, dy, in_h, in_w):
        """dx of ``forward`` for the upstream gradient dy (complex64 NKPQ)."""
        return cutlass_complex_conv.dgrad_complex_packed(
            dy, self._packed_dgrad(), self.in_channels, in_h, in_w, self.kernel_size[0],
            self.kernel_size[1], self.stride[0], self.stride[1], self.padding[0],
            self.padding[1], _PRECISIONS[self.precision])

    def _forward_impl(self, x):
        self._ensure_prepacked()

        # Any layout is read in place (strided layout pass; the reference
        # makes a contiguous copy first, modules.py:198-199).  A dense input
        # at an address the TMA path cannot use goes through the same
        # strided pass instead of a copy.
        strided = x.is_contiguous() and not _aligned16(x)

        bias_real, bias_imag = self._bias_args()
        return cutlass_complex_conv.forward_complex_packed(
            x,
            self._w_packed,
            self.out_channels,
            self.kernel_size[0],
            self.kernel_size[1],
            self.stride[0],
            self.stride[1],
            self.padding[0],
            self.padding[1],
            _PRECISIONS[self.precision],
            bias_real,
            bias_imag,
            strided,
        )

    def _copy_streams(self, device):
        """Host->device and device->host copy streams of ``device`` (made once)."""
        streams = self.__dict__.setdefault("_host_copy_streams", {})
        if device not in streams:
            streams[device] = (torch.cuda.Stream(device), torch.cuda.Stream(device))
        return streams[device]

    def output_shape(self, n, h, w):
        """``(N, K, P, Q)`` of ``forward`` for an ``(N, C, H, W)`` input."""
        p = (h + 2 * self.padding[0] - self.kernel_size[0]) // self.stride[0] + 1
        q = (w + 2 * self.padding[1] - self.kernel_size[1]) // self.stride[1] + 1
        if p <= 0 or q <= 0:
            raise ValueError(f"input {h}x{w} is smaller than the kernel")
        return (n, self.out_channels, p, q)

    def forward_host(self, x, out=None, images_per_chunk=None):
        """``forward`` for a complex64 NCHW batch in pinned host memory.

        The batch is cut into chunks of whole images.  Chunk i's host->device
        copy, its convolution (``forward`` on the chunk, on the current
        stream) and its device->host copy run on three streams, so copies in
        the two PCIe directions overlap each other and the kernels; a
        serial copy-in, forward, copy-out pays both directions one after the
        other.  Each chunk's output is identical to ``forward`` of that chunk.

        Args:
            x: pinned (``pin_memory()``) CPU complex64 tensor, NCHW, contiguous.
            out: optional pinned CPU complex64 tensor of ``output_shape``;
                allocated (pinned) when None.
            images_per_chunk: images per chunk; None picks chunks of about
                24 MB of input with smaller chunks at both ends (1, 2, 4, ...
                images), so that the start and the end of the pipeline,
                where only one copy direction is busy, stay short.

        Returns:
            ``out``.  Like ``Tensor.copy_(..., non_blocking=True)``, the call
            returns before the copies end: ``out`` holds the result once the
            current CUDA stream has reached this point (e.g. after
            ``torch.cuda.current_stream().synchronize()``).  Until then the
            copy-in stream may still be reading ``x``: a caller that reuses
            a pinned staging buffer must not refill ``x`` before that point
            either.
        """
        if x.is_cuda:
            raise ValueError("forward_host takes a host tensor; use forward for CUDA input")
        if x.dtype != torch.complex64:
            raise ValueError(f"ComplexConv2d expects torch.complex64 input, got {x.dtype}")
        if x.dim() != 4:
            raise ValueError(f"ComplexConv2d expects a 4D NCHW tensor, got {x.dim()}D")
        if x.size(1) != self.in_channels:
            raise ValueError(f"expected {self.in_channels} input channels, got {x.size(1)}")
        # An empty tensor has no storage to pin.
        if not x.is_contiguous() or (x.numel() > 0 and not x.is_pinned()):
            raise ValueError("forward_host input must be contiguous pinned host memory")
        dev = self.weight_real.device
        if not self.weight_real.is_cuda:
            raise RuntimeError("ComplexConv2d weights must be on CUDA")
        n, _, h, w = x.shape
        shape = self.output_shape(n, h, w)
        if out is None:
            out = torch.empty(shape, dtype=torch.complex64, pin_memory=True)
        elif (out.is_cuda or out.dtype != torch.complex64 or tuple(out.shape) != shape
              or not out.is_contiguous() or (out.numel() > 0 and not out.is_pinned())):
            raise ValueError(
                f"out must be a contiguous pinned host complex64 tensor of shape {shape}")
        if n == 0:
            return out
        if images_per_chunk is None:
            middle = max(1, _HOST_CHUNK_BYTES // max(1, x[0].numel() * 8))
            sizes = _host_chunks(n, middle)
        else:
            if images_per_chunk < 1:
                raise ValueError("images_per_chunk must be >= 1")
            sizes = [min(images_per_chunk, n - i) for i in range(0, n, images_per_chunk)]

        cur = torch.cuda.current_stream(dev)
        h2d, d2h = self._copy_streams(dev)
        xd = torch.empty(x.shape, dtype=x.dtype, device=dev)
        # The side streams may touch xd (allocated on cur) only after cur's
        # earlier work on that memory; cur waits for them again at the end.
        h2d.wait_stream(cur)
        d2h.wait_stream(cur)
        i1 = 0
        for size in sizes:
            i0, i1 = i1, i1 + size
            with torch.cuda.stream(h2d):
                xd[i0:i1].copy_(x[i0:i1], non_blocking=True)
            copied = torch.cuda.Event()
            copied.record(h2d)
            cur.wait_event(copied)
            y = self.forward(xd[i0:i1])
            done = torch.cuda.Event()
            done.record(cur)
            d2h.wait_event(done)
            with torch.cuda.stream(d2h):
                out[i0:i1].copy_(y, non_blocking=True)
            # y's memory returns to the allocator at the next iteration; keep
            # it from being reused before d2h has read it.
            y.record_stream(d2h)
        xd.record_stream(h2d)
        cur.wait_stream(h2d)
        cur.wait_stream(d2h)
        return out
