"""ctypes binding of libccv_b200.so for the tests (the C ABI in include/ccv_b200.h).

This is the binding a maintainer of a non-Python caller would write; the GPU
parity tests call the kernels through it with device pointers taken from
torch tensors.
"""

import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ccv_b200.h")
LIB = os.path.join(ROOT, "cutlass-complex-conv_b200", "complex_conv2d", "libccv_b200.so")

CCV_OK = 0
CCV_ERR_INVALID_ARGUMENT = 1
CCV_ERR_UNSUPPORTED = 2
CCV_ERR_WORKSPACE = 3
CCV_ERR_DEVICE_TIMEOUT = 6
CCV_PRECISION_TF32 = 0
CCV_PRECISION_3XTF32 = 1
CCV_WEIGHT_KCRS = 0
CCV_WEIGHT_KRSC = 1


class ConvShape(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in
                ("n", "h", "w", "c", "k", "r", "s", "stride_h", "stride_w", "pad_h", "pad_w")]


def shape_of(case):
    return ConvShape(case.n, case.h, case.w, case.c, case.k, case.r, case.s,
                     case.stride_h, case.stride_w, case.pad_h, case.pad_w)


def declared_functions():
    """Names of the functions declared in include/ccv_b200.h."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(ccv_\w+)\s*\(", text, flags=re.M)))


_lib = None


def load():
    global _lib
    if _lib is not None:
        return _lib
    lib = ctypes.CDLL(LIB)
    vp, sz, i64p = ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int64)
    sp = ctypes.POINTER(ConvShape)
    sig = {
        "ccv_output_size": (ctypes.c_int, [sp, i64p, i64p]),
        "ccv_check_shape": (ctypes.c_int, [sp]),
        "ccv_packed_weight_bytes": (sz, [sp, ctypes.c_int]),
        "ccv_prepack_weights": (ctypes.c_int, [vp, vp, ctypes.c_int, sp, ctypes.c_int, vp, sz, vp]),
        "ccv_fprop_planar_workspace_bytes": (sz, [sp, ctypes.c_int]),
        "ccv_fprop_complex_workspace_bytes": (sz, [sp, ctypes.c_int]),
        "ccv_fprop_planar_min_workspace_bytes": (sz, [sp, ctypes.c_int]),
        "ccv_fprop_complex_min_workspace_bytes": (sz, [sp, ctypes.c_int]),
        "ccv_fprop_kernel_launches": (ctypes.c_int, [sp, ctypes.c_int, ctypes.c_int,
                                                     ctypes.POINTER(ctypes.c_int)]),
        "ccv_fprop_planar": (ctypes.c_int, [vp, vp, vp, vp, vp, sp, ctypes.c_int, vp, sz, vp]),
        "ccv_fprop_complex": (ctypes.c_int, [vp, vp, vp, sp, ctypes.c_int, vp, sz, vp]),
        "ccv_fprop_planar_bias": (ctypes.c_int, [vp, vp, vp, vp, vp, vp, vp, sp, ctypes.c_int, vp,
                                                 sz, vp]),
        "ccv_fprop_complex_bias": (ctypes.c_int, [vp, vp, vp, vp, vp, sp, ctypes.c_int, vp, sz,
                                                  vp]),
        "ccv_fprop_complex_strided": (ctypes.c_int, [vp, i64p, vp, vp, vp, vp, sp, ctypes.c_int,
                                                     vp, sz, vp]),
        "ccv_fprop_planar_to_complex": (ctypes.c_int, [vp, vp, vp, vp, sp, ctypes.c_int, vp, sz,
                                                       vp]),
        "ccv_fprop_complex_kernel": (ctypes.c_char_p, [sp, ctypes.c_int]),
        "ccv_forward_workspace_bytes": (sz, [sp]),
        "ccv_forward": (ctypes.c_int, [vp, vp, vp, vp, vp, vp, sp, vp, sz, vp]),
        "ccv_forward_noalloc": (ctypes.c_int, [vp, vp, vp, vp, vp, vp, sp, vp]),
        "ccv_prepack_weights_dgrad": (ctypes.c_int, [vp, vp, ctypes.c_int, sp, ctypes.c_int, vp,
                                                     sz, vp]),
        "ccv_dgrad_complex_workspace_bytes": (sz, [sp, ctypes.c_int]),
        "ccv_dgrad_complex": (ctypes.c_int, [vp, vp, vp, sp, ctypes.c_int, vp, sz, vp]),
        "ccv_wgrad_complex_workspace_bytes": (sz, [sp]),
        "ccv_wgrad_complex": (ctypes.c_int, [vp, vp, vp, vp, sp, vp, sz, vp]),
        "ccv_dgrad_planar_workspace_bytes": (sz, [sp, ctypes.c_int]),
        "ccv_dgrad_planar": (ctypes.c_int, [vp, vp, vp, vp, vp, sp, ctypes.c_int, vp, sz, vp]),
        "ccv_wgrad_planar_workspace_bytes": (sz, [sp]),
        "ccv_wgrad_planar": (ctypes.c_int, [vp, vp, vp, vp, vp, vp, sp, vp, sz, vp]),
        "ccv_get_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
        "ccv_clear_device_status": (ctypes.c_int, []),
        "ccv_selftest_bounded_wait": (ctypes.c_int, [vp, vp]),
        "ccv_last_error_message": (ctypes.c_char_p, []),
        "ccv_version": (ctypes.c_char_p, []),
        "ccv_reload_config": (ctypes.c_int, []),
    }
    for name, (res, args) in sig.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    _lib = _ConfigTracking(lib)
    return _lib


class _ConfigTracking:
    """The library handle, re-reading the library's CCV_* switches (which it
    reads once) before any call made after the test changed one of them."""

    def __init__(self, lib):
        self._lib = lib
        self._env = None

    def _sync(self):
        snap = tuple(sorted((k, v) for k, v in os.environ.items() if k.startswith("CCV_")))
        if snap != self._env:
            self._lib.ccv_reload_config()
            self._env = snap

    def __getattr__(self, name):
        f = getattr(self._lib, name)
        if not name.startswith("ccv_") or name == "ccv_reload_config":
            return f

        def call(*args):
            self._sync()
            return f(*args)

        return call


def last_error():
    return load().ccv_last_error_message().decode()


def check(rc, what=""):
    if rc != CCV_OK:
        raise RuntimeError(f"{what} failed with status {rc}: {last_error()}")
