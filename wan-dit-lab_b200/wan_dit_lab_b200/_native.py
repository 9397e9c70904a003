"""ctypes binding of libwdl_b200.so (include/wdl_b200.h): the only way this package reaches the GPU kernels.

The library is loaded on first use and must exist: there is no fallback to PyTorch or CPU code. A nonzero
status of an entry point becomes an exception carrying the library's message: ValueError for invalid
arguments (nothing was launched), RuntimeError otherwise.
"""

import ctypes
from pathlib import Path

import torch

LIBRARY = Path(__file__).resolve().parent / "libwdl_b200.so"

OK, ERR_ARGUMENT, ERR_UNSUPPORTED, ERR_CUDA, ERR_DEVICE = 0, 1, 2, 3, 4
BF16, F16, F32 = 0, 1, 2
CODES_INT8, CODES_E4M3, CODES_F16_FOLD, CODES_F16_PRE = 0, 1, 3, 4
DTYPE_CODE = {torch.bfloat16: BF16, torch.float16: F16, torch.float32: F32}

_P, _I, _I64, _SZ, _U32P = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.POINTER(ctypes.c_uint32)



class LowRank(ctypes.Structure):
    """wdl_lowrank (include/wdl_b200.h): an SVDQuant low-rank branch formed in the GEMM epilogue, act [M, ld_act]
    float32 = x proj_down, up [N, rank] float32 = proj_up, rank a multiple of 4. Whoever makes one keeps the
    tensors it points to alive until the GEMM has run (attributes set on the instance do)."""
    _fields_ = [("act", ctypes.c_void_p), ("ld_act", ctypes.c_int64), ("up", ctypes.c_void_p), ("rank", ctypes.c_int)]


_LRP = ctypes.POINTER(LowRank)

# name: (restype, argtypes), in the order of include/wdl_b200.h
SIGNATURES = {
    "wdl_last_error": (ctypes.c_char_p, []),
    "wdl_version": (ctypes.c_char_p, []),
    "wdl_device_error": (_I, [_P, _U32P]),
    "wdl_w4a4_quantize_rows": (_I, [_P, _I, _I64, _P, _I, _I, _I, _I, _P, _P, _P, _P]),
    "wdl_w4a4_unpack_weight": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P]),
    "wdl_w4a4_fold_weight": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P]),
    "wdl_w4a4_gemm": (_I, [_P, _P, _P, _P, _I, _P, _I, _I, _I, _P, _I64, _P]),
    "wdl_w4a4_gemm_residual": (_I, [_P, _P, _P, _P, _I, _P, _P, _P, _I64, _I, _I, _I, _P, _I64, _P]),
    "wdl_w4a4_gemm_group_partials": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _I64, _P]),
    "wdl_w4a4_gemm_add": (_I, [_P, _P, _P, _P, _I, _P, _P, _I64, _I, _I, _I, _P, _I64, _P]),
    "wdl_w4a4_gemm_residual_add": (_I, [_P, _P, _P, _P, _I, _P, _P, _I64, _P, _P, _I64, _I, _I, _I, _P, _I64, _P]),
    "wdl_w4a4_gemm_gelu_u4_add": (_I, [_P, _P, _P, _P, _I, _P, _P, _I64, _P, ctypes.c_float, _I, _I, _I, _I, _P,
                                       _I64, _P, _P, _I64, _P]),
    "wdl_lowrank_down": (_I, [_P, _I, _I64, _I, _I, _P, _I, _P, _I64, _P]),
    "wdl_w4a4_gemm_lowrank": (_I, [_P, _P, _P, _P, _I, _P, _LRP, _I, _I, _I, _P, _I64, _P]),
    "wdl_w4a4_gemm_residual_lowrank": (_I, [_P, _P, _P, _P, _I, _P, _LRP, _P, _P, _I64, _I, _I, _I, _P, _I64, _P]),
    "wdl_w4a4_gemm_gelu_u4_lowrank": (_I, [_P, _P, _P, _P, _I, _P, _LRP, _P, ctypes.c_float, _I, _I, _I, _I, _P,
                                           _I64, _P, _P, _I64, _P]),
    "wdl_w4a4_gemm_f32": (_I, [_P, _P, _P, _P, _I, _P, _P, _I64, _I, _I, _I, _P, _I64, _P]),
    "wdl_w4a4_gemm_f32_lowrank": (_I, [_P, _P, _P, _P, _I, _P, _LRP, _I, _I, _I, _P, _I64, _P]),
    "wdl_w4a4_linear_workspace": (_SZ, [_I, _I]),
    "wdl_w4a4_linear": (_I, [_P, _I64, _I, _I, _P, _I, _P, _P, _I, _P, _I, _P, _I64, _P, _SZ, _P]),
    "wdl_w4a4_linear_noalloc": (_I, [_P, _I64, _I, _I, _P, _I, _P, _P, _I, _P, _I, _P, _I64, _P]),
    "wdl_store_kv_fp8": (_I, [_P, _I, _P, _P, _I, _P, _I, _I, _I, _I, _P, _P, _P, _P, _I, _I, _P]),
    "wdl_rope_apply": (_I, [_P, _I, _P, _I, _I, _I, _I, _P, _P, _I, _P, _I, _I, _P, _I, _P]),
    "wdl_qkv_prep": (_I, [_P, _I64, _I, _I, _P, _P, ctypes.c_float, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P,
                          _I, _I, _P]),
    "wdl_qkv_prep_sharded": (_I, [_P, _I64, _I, _I, _P, _P, ctypes.c_float, _P, _I, _P, _I, _I, _I, _I, _P, _P, _P,
                                  _P, _P, _P, _I, _I, _P]),
    "wdl_w4a4_gemm_gelu_u4": (_I, [_P, _P, _P, _P, _I, _P, _P, ctypes.c_float, _I, _I, _I, _I, _P, _I64, _P, _P]),
    "wdl_ln_quant": (_I, [_P, _I, _I64, _I, _I, ctypes.c_float, _P, _P, _I, _P, _P, _P, _I, _I, _P, _P, _P]),
    "wdl_ln_quant_keep": (_I, [_P, _I, _I64, _I, _I, ctypes.c_float, _P, _P, _I, _P, _P, _P, _I, _I, _P, _P, _P,
                               _I64, _P]),
    "wdl_rms_rows": (_I, [_P, _I64, _I, _I, _P, ctypes.c_float, _P, _I64, _P]),
    "wdl_rms_rows_sharded": (_I, [_P, _I64, _I, _I, _P, ctypes.c_float, _P, _I, _P, _I64, _P]),
    "wdl_rows_sumsq": (_I, [_P, _I64, _I, _I, _I, _I64, _P, _P]),
    "wdl_residual_update": (_I, [_P, _I64, _P, _P, _P, _I64, _I, _I, _P]),
    "wdl_modulation": (_I, [_P, _P, _I, _I, _P, _P]),
    "wdl_sage_prep_kv": (_I, [_P, _P, _P, _P, _I, _P, _I, _I64, _P, _I, _I64, _I, _I, _P, _P, _P, _P, _P, _SZ, _P]),
    "wdl_sage_quant_q": (_I, [_P, _I64, _I, _I, _P, _P, _P]),
    "wdl_sage_prep_workspace": (_SZ, [_I, _I]),
    "wdl_sage_prep": (_I, [_P, _I64, _I, _P, _P, _P, _P, _I, _P, _I, _I64, _P, _I, _I64, _I, _I, _P, _P, _P, _P, _P,
                           _P, _P, _SZ, _P]),
    "wdl_sage_attention": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, ctypes.c_float, _P, _I64, _P]),
    "wdl_sage_attend_workspace": (_SZ, [_I, _I, _I]),
    "wdl_sage_attend": (_I, [_P, _I64, _I, _P, _P, _P, _P, _I, _P, _I, _I64, _P, _I, _I64, _I, _I, ctypes.c_float,
                             _P, _I64, _P, _SZ, _P]),
    "wdl_sage_attend_maps": (_I, [_P, _I64, _I, _P, _P, _P, _P, _I, _I, _P, _P, _I, _P, _I, _I64, _P, _I, _I64, _I,
                                  _I, ctypes.c_float, _P, _I64, _P, _SZ, _P]),
}

_lib = None


def lib():
    """The loaded library, with the argument types of every entry point declared."""
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            raise RuntimeError(f"{LIBRARY} is not built: run `python wan-dit-lab_b200/build.py`")
        handle = ctypes.CDLL(str(LIBRARY))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype, fn.argtypes = restype, argtypes
        _lib = handle
    return _lib


def check(status):
    """Raises for a nonzero status of an entry point."""
    if status == OK:
        return
    message = lib().wdl_last_error().decode()
    raise (ValueError if status == ERR_ARGUMENT else RuntimeError)(message)


def ptr(tensor):
    """Device address of a tensor (None for None)."""
    return None if tensor is None else tensor.data_ptr()


def stream(device=None):
    """The current PyTorch CUDA stream of `device`, as the library takes it."""
    return torch.cuda.current_stream(device).cuda_stream


def device_error(device=None):
    """Synchronises the current stream and reads (and clears) the device error word: 0, or raises RuntimeError
    naming the code a kernel recorded since the last check (a bounded wait given up, or an index map entry out of
    range)."""
    code = ctypes.c_uint32(0)
    check(lib().wdl_device_error(stream(device), ctypes.byref(code)))
    return code.value
