"""The quantizers divide many values by one scale with div_rn_by (csrc/common.cuh): the reciprocal of the scale
rounded once, then Markstein's correction per value. The reference divides with IEEE division (torch / numpy
float32 `/`), so the codes are bit-exact only if div_rn_by returns the correctly rounded quotient. This test
builds a test-only kernel (tests/native/div_check.cu) and counts differing bits against __fdiv_rn over 2^28
pairs per sweep, including quotients a few ulps from every INT4 / INT8 rounding boundary."""

import ctypes
import os
import subprocess
import tempfile

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "wan-dit-lab_b200", "csrc")


@pytest.fixture(scope="module")
def checker():
    out = os.path.join(tempfile.mkdtemp(prefix="div_check_"), "div_check.so")
    subprocess.run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-shared", "-Xcompiler", "-fPIC",
                    "-I", CSRC, os.path.join(HERE, "native", "div_check.cu"), "-o", out], check=True)
    lib = ctypes.CDLL(out)
    lib.div_check.restype = ctypes.c_int
    lib.div_check.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_uint64,
                              ctypes.POINTER(ctypes.c_ulonglong), ctypes.POINTER(ctypes.c_float)]
    return lib


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_div_rn_by_is_the_ieee_quotient(checker, mode):
    bad = ctypes.c_ulonglong(0)
    example = (ctypes.c_float * 2)()
    assert checker.div_check(12345 + mode, mode, 1 << 28, ctypes.byref(bad), example) == 0
    assert bad.value == 0, f"{bad.value} mismatches, e.g. x={example[0]!r} s={example[1]!r}"
