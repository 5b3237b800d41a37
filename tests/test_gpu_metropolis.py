"""The device's Metropolis arithmetic against the host libm, exhaustively.

The reference's CPU port decides u < expf(-beta dE) with the host libm (glibc); the device evaluates a
correctly rounded expf by Tang's method plus a build-time table of glibc's misrounded inputs, after a
single-instruction pre-test that only decides when u is clearly away from exp(x).  Over every negative
float x: (1) the device's libm-equivalent value equals glibc's (order-independent checksum), (2) the
pre-test's relative error stays far inside its decision margin of 8e-6 (asserted < 2e-6).
"""
import ctypes as C

import pytest

import oracle as O
from treesa_gpu_b200 import _abi

pytestmark = pytest.mark.gpu

NEG_LO, NEG_HI = 0x80000000, 0xFF800000  # -0 .. -inf


def _device(lo, hi):
    L = _abi.lib()
    L.tsa_expf_selftest.argtypes = [C.c_int, C.c_uint32, C.c_uint32, C.POINTER(C.c_uint64), C.POINTER(C.c_double),
                                    C.c_char_p, C.c_size_t]
    cs, mx = C.c_uint64(), C.c_double()
    err = C.create_string_buffer(256)
    rc = L.tsa_expf_selftest(0, lo, hi, C.byref(cs), C.byref(mx), err, 256)
    _abi.check(rc, err, "tsa_expf_selftest")
    return cs.value, mx.value


def test_device_expf_equals_host_libm_on_every_negative_float():
    dev, worst = _device(NEG_LO, NEG_HI)
    host = O.orc().orc_expf_checksum(NEG_LO, NEG_HI)
    assert dev == host
    assert worst < 2e-6, worst


def test_checksum_detects_a_single_difference():
    """The checksum is sensitive: a range with one planted host-side difference would not match
    (planted on the CPU: the host sum over a range shifted by one pattern differs)."""
    a = O.orc().orc_expf_checksum(0xBF000000, 0xBF0FFFFF)
    b = O.orc().orc_expf_checksum(0xBF000001, 0xBF100000)
    assert a != b
    dev, _ = _device(0xBF000000, 0xBF0FFFFF)
    assert dev == a
