"""Every spin-wait of the library's kernels is bounded (csrc/common.cuh mbar_wait): a wait still unsatisfied after
its limit records a code in the device error word, gives up and lets the kernel return, so that a producer that
never arrives ends in an error status instead of a hung GPU. This test makes a wait run out on purpose, in a
test-only kernel (tests/native/wait_check.cu) that waits on an mbarrier nothing ever arrives at, with a limit of
one millisecond passed as a kernel argument: the waits give up after about that long, the kernel returns, the
library's wdl_device_error reports the code (and clears it), and the context stays usable."""

import ctypes
import os
import subprocess
import tempfile

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(os.path.dirname(HERE), "wan-dit-lab_b200")
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "wan_dit_lab_b200")
ERR_WAIT_FULL = 1  # wdl::kErrWaitFull


@pytest.fixture(scope="module")
def checker():
    from wan_dit_lab_b200 import _native
    _native.lib()  # the library first, so that the checker links to the one already loaded
    out = os.path.join(tempfile.mkdtemp(prefix="wait_check_"), "wait_check.so")
    subprocess.run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-shared", "-Xcompiler", "-fPIC",
                    "-I", CSRC, os.path.join(HERE, "native", "wait_check.cu"), "-o", out, f"-L{LIBDIR}", "-lwdl_b200",
                    f"-Xlinker=-rpath,{LIBDIR}"], check=True)
    lib = ctypes.CDLL(out)
    lib.wait_check.restype = ctypes.c_int
    lib.wait_check.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int, ctypes.POINTER(ctypes.c_uint32),
                               ctypes.POINTER(ctypes.c_float)]
    return lib


def test_a_wait_nothing_satisfies_gives_up_and_is_reported(checker):
    from wan_dit_lab_b200 import _native
    torch.cuda.init()
    assert _native.device_error() == 0  # a clean error word
    gave_up, ms = ctypes.c_uint32(0), ctypes.c_float(0)
    assert checker.wait_check(1_000_000, ERR_WAIT_FULL, 64, ctypes.byref(gave_up), ctypes.byref(ms)) == 0
    assert gave_up.value == 64  # every waiting thread returned false
    assert 0.9 <= ms.value < 1000, f"the waits gave up after {ms.value:.3f} ms (limit 1 ms)"
    with pytest.raises(RuntimeError, match="bounded wait"):
        _native.device_error()  # reports the code, then clears it
    assert _native.device_error() == 0
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float(x.sum()) == 1023 * 1024 / 2  # the context is still usable
