"""CPU checks of the C ABI: the library loads, exports every declared entry
point, and its host-side shape logic matches the reference's rules
(csrc/complex_conv2d.cu:94-159 and can_implement in
device/implicit_planar_cgemm_convolution.h:71-187).  No kernel is launched.
"""

import ctypes

import pytest

import ccv_abi
import oracle


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(ccv_abi.LIB)
    names = ccv_abi.declared_functions()
    assert len(names) >= 15, names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    lib = ccv_abi.load()._lib
    for n in ccv_abi.declared_functions():
        assert getattr(lib, n).restype is not None, n


def test_version_string():
    assert b"sm_100a" in ccv_abi.load().ccv_version()


@pytest.mark.parametrize("case", [
    oracle.ConvCase(1, 32, 56, 56, 64, 3, 3, 1, 1, 1, 1),
    oracle.ConvCase(32, 64, 112, 112, 128, 3, 3, 2, 2, 1, 1),
    oracle.ConvCase(32, 256, 28, 28, 1024, 1, 1, 1, 1, 0, 0),
    oracle.ConvCase(1, 4, 11, 13, 8, 7, 7, 2, 2, 3, 3),
    oracle.ConvCase(1, 8, 7, 9, 12, 3, 1, 2, 1, 1, 0),
])
def test_output_size_matches_reference_rule(case):
    lib = ccv_abi.load()
    p = ctypes.c_int64()
    q = ctypes.c_int64()
    shp = ccv_abi.shape_of(case)
    assert lib.ccv_output_size(ctypes.byref(shp), ctypes.byref(p), ctypes.byref(q)) == 0
    assert (p.value, q.value) == (case.p, case.q)


def _rc(**kw):
    base = dict(n=1, h=8, w=8, c=8, k=8, r=3, s=3, stride_h=1, stride_w=1, pad_h=1, pad_w=1)
    base.update(kw)
    shp = ccv_abi.ConvShape(*[base[f] for f, _ in ccv_abi.ConvShape._fields_])
    lib = ccv_abi.load()
    return lib.ccv_check_shape(ctypes.byref(shp)), ccv_abi.last_error()


def test_shape_errors_carry_reference_messages():
    rc, msg = _rc(stride_h=0)
    assert rc == ccv_abi.CCV_ERR_INVALID_ARGUMENT and "stride must be positive" in msg
    rc, msg = _rc(pad_w=-1)
    assert rc == ccv_abi.CCV_ERR_INVALID_ARGUMENT and "padding must be non-negative" in msg
    rc, msg = _rc(r=0)
    assert rc == ccv_abi.CCV_ERR_INVALID_ARGUMENT and "kernel dimensions must be positive" in msg
    rc, msg = _rc(h=2, w=2, pad_h=0, pad_w=0)
    assert rc == ccv_abi.CCV_ERR_INVALID_ARGUMENT and "output spatial size must be positive" in msg


def test_alignment_constraints_like_can_implement():
    # C % 4 and K % 4 (kAlignment of the reference iterators / epilogue).
    rc, msg = _rc(c=6)
    assert rc == ccv_abi.CCV_ERR_UNSUPPORTED and "cannot implement" in msg
    rc, msg = _rc(k=10)
    assert rc == ccv_abi.CCV_ERR_UNSUPPORTED
    rc, _ = _rc(c=4, k=4)
    assert rc == 0


def test_packed_weight_bytes():
    lib = ccv_abi.load()
    case = oracle.ConvCase(1, 64, 28, 28, 128, 3, 3, 1, 1, 1, 1)
    shp = ccv_abi.shape_of(case)
    one = lib.ccv_packed_weight_bytes(ctypes.byref(shp), ccv_abi.CCV_PRECISION_TF32)
    assert one == 9 * 3 * 128 * 64 * 4
    two = lib.ccv_packed_weight_bytes(ctypes.byref(shp), ccv_abi.CCV_PRECISION_3XTF32)
    assert two == 2 * one


def test_null_pointers_rejected_before_any_launch():
    lib = ccv_abi.load()
    case = oracle.ConvCase(1, 8, 8, 8, 8, 3, 3, 1, 1, 1, 1)
    shp = ccv_abi.shape_of(case)
    rc = lib.ccv_fprop_planar(None, None, None, None, None, ctypes.byref(shp), 0, None, 0, None)
    assert rc == ccv_abi.CCV_ERR_INVALID_ARGUMENT
    rc = lib.ccv_fprop_complex(None, None, None, ctypes.byref(shp), 0, None, 0, None)
    assert rc == ccv_abi.CCV_ERR_INVALID_ARGUMENT
