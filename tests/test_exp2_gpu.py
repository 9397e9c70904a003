"""The attention softmax can evaluate a compile-time share of its exponentials on the FMA pipe (csrc/common.cuh
exp2_fma: round to the nearest integer by the 1.5 * 2^23 shift, a degree-4 polynomial for 2^f on [-0.5, 0.5], the
integer added to the exponent field) instead of the special function unit (sage_attn.cu kAttnPolyShare, 0 as
measured fastest). This checks that function against exact powers of two
(float64) over every argument range the softmax produces (score minus row maximum, times log2(e) and the scales:
<= 0, down to the -100 clamp) and past it, next to CUDA's exp2f on the same arguments."""

import ctypes
import os
import subprocess
import tempfile

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "wan-dit-lab_b200", "csrc")
POLY_BOUND = 3e-6  # the fitted polynomial's float32 error is 2.7e-6; an E4M3 probability step is 6e-2


@pytest.fixture(scope="module")
def checker():
    out = os.path.join(tempfile.mkdtemp(prefix="exp2_check_"), "exp2_check.so")
    subprocess.run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-shared", "-Xcompiler", "-fPIC",
                    "-I", CSRC, os.path.join(HERE, "native", "exp2_check.cu"), "-o", out], check=True)
    lib = ctypes.CDLL(out)
    lib.exp2_check.restype = ctypes.c_int
    lib.exp2_check.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
    return lib


def run(checker, x):
    xd = torch.from_numpy(x).cuda()
    poly, ref = torch.empty_like(xd), torch.empty_like(xd)
    assert checker.exp2_check(xd.data_ptr(), poly.data_ptr(), ref.data_ptr(), xd.numel()) == 0
    return poly.cpu().numpy().astype(np.float64), ref.cpu().numpy().astype(np.float64)


def test_exp2_fma_within_its_bound(checker):
    rng = np.random.default_rng(5)
    x = np.concatenate([
        np.linspace(-1, 1, 1 << 21, dtype=np.float32),           # every fraction, both rounding directions
        np.linspace(-100, 0, 1 << 21, dtype=np.float32),         # the softmax's arguments
        rng.uniform(-100, 30, 1 << 20).astype(np.float32),
        np.arange(-100, 31, dtype=np.float32),                   # exact powers
        np.arange(-100, 30, dtype=np.float32) + np.float32(0.5),  # ties of the rounding
        np.float32([0.0, -0.0, 1e-30, -1e-30]),
    ])
    poly, ref = run(checker, x)
    exact = np.exp2(x.astype(np.float64))
    err_poly = np.abs(poly - exact) / exact
    err_ref = np.abs(ref - exact) / exact
    worst = int(np.argmax(err_poly))
    print(f"exp2_fma max rel err {err_poly.max():.3e} at x={x[worst]!r}; exp2f {err_ref.max():.3e}")
    assert err_poly.max() <= POLY_BOUND
    assert err_ref.max() <= 2.5e-7  # CUDA's exp2f: 2 ulp


def test_exp2_fma_clamps_below(checker):
    x = np.float32([-100.0, -150.0, -1e6, -np.inf])
    poly, _ = run(checker, x)
    assert np.all(np.abs(poly - 2.0 ** -100) <= POLY_BOUND * 2.0 ** -100)  # clamped to 2^-100, never NaN
