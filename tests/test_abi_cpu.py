"""The C ABI without a GPU: libwdl_b200.so loads, exports every entry point include/wdl_b200.h declares (with the
argument counts the ctypes binding declares), and rejects invalid calls with WDL_ERR_ARGUMENT and a message
before it touches the device, as the reference's operators raise on bad shapes before launching
(kernels/cache_fp8.py:75-100, native/ops/w4a4_ops.cpp:20-35)."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "wdl_b200.h"


def declarations():
    """name -> number of parameters, for every function the header declares."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for m in re.finditer(r"^[A-Za-z_][\w \t\*]*?\b(wdl_\w+)\s*\(([^)]*)\)\s*;", text, flags=re.M):
        params = m.group(2).strip()
        out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


@pytest.fixture(scope="module")
def native():
    from wan_dit_lab_b200 import _native
    return _native


def test_header_declares_the_bound_entry_points(native):
    decl = declarations()
    assert len(decl) >= 25
    assert set(decl) == set(native.SIGNATURES), set(decl) ^ set(native.SIGNATURES)
    for name, count in decl.items():
        assert len(native.SIGNATURES[name][1]) == count, name


def test_library_exports_every_declared_symbol(native):
    raw = ctypes.CDLL(str(native.LIBRARY))
    missing = [name for name in declarations() if not hasattr(raw, name)]
    assert not missing, missing
    lib = native.lib()
    assert lib.wdl_version().startswith(b"wdl_b200")


FAKE = 1 << 20  # a 256-byte aligned address the library only checks, never dereferences, in these calls


def test_gemm_shapes_rejected_before_any_launch(native):
    lib = native.lib()
    st = lib.wdl_w4a4_gemm(FAKE, FAKE, FAKE, FAKE, native.CODES_E4M3, None, 128, 300, 256, FAKE, 512, None)
    assert st == native.ERR_ARGUMENT and b"multiple of 256" in lib.wdl_last_error()
    st = lib.wdl_w4a4_gemm(FAKE, FAKE, FAKE, FAKE, native.CODES_E4M3, None, 128, 256, 200, FAKE, 256, None)
    assert st == native.ERR_ARGUMENT and b"multiple of 128" in lib.wdl_last_error()
    st = lib.wdl_w4a4_gemm(FAKE, FAKE, FAKE + 8, FAKE, native.CODES_E4M3, None, 128, 256, 256, FAKE, 256, None)
    assert st == native.ERR_ARGUMENT and b"16-byte" in lib.wdl_last_error()
    st = lib.wdl_w4a4_gemm(FAKE, FAKE, FAKE, FAKE, native.CODES_F16_PRE, FAKE + 4, 128, 256, 256, FAKE, 256, None)
    assert st == native.ERR_ARGUMENT and b"bias" in lib.wdl_last_error()  # the epilogue loads it 16 bytes at a time
    st = lib.wdl_w4a4_gemm(FAKE, FAKE, FAKE, FAKE, 7, None, 128, 256, 256, FAKE, 256, None)
    assert st == native.ERR_ARGUMENT and b"code format" in lib.wdl_last_error()
    assert lib.wdl_w4a4_gemm(FAKE, FAKE, FAKE, FAKE, native.CODES_E4M3, None, 0, 256, 256, FAKE, 256, None) == 0


def test_epilogue_strides_above_32_bits_rejected(native):
    """The GEMM epilogue carries its row strides as 32-bit ints: a stride of 2^31 elements or more is refused
    before any launch, in each entry point that takes one."""
    lib = native.lib()
    wide = 1 << 31
    lr = native.LowRank(FAKE, wide, FAKE, 8)
    calls = {
        b"ldy": lambda: lib.wdl_w4a4_gemm(FAKE, FAKE, FAKE, FAKE, native.CODES_F16_PRE, None, 128, 256, 256, FAKE,
                                          wide, None),
        b"ldr": lambda: lib.wdl_w4a4_gemm_residual(FAKE, FAKE, FAKE, FAKE, native.CODES_F16_PRE, None, None, FAKE,
                                                   wide, 128, 256, 256, FAKE, 256, None),
        b"ldo": lambda: lib.wdl_w4a4_gemm_f32(FAKE, FAKE, FAKE, FAKE, native.CODES_F16_PRE, None, None, 0, 128, 256,
                                              256, FAKE, wide, None),
        b"addend": lambda: lib.wdl_w4a4_gemm_add(FAKE, FAKE, FAKE, FAKE, native.CODES_F16_PRE, None, FAKE, wide, 128,
                                                 256, 256, FAKE, 256, None),
        b"low-rank": lambda: lib.wdl_w4a4_gemm_lowrank(FAKE, FAKE, FAKE, FAKE, native.CODES_F16_PRE, None, lr, 128,
                                                       256, 256, FAKE, 256, None),
        b"ldc": lambda: lib.wdl_w4a4_gemm_gelu_u4(FAKE, FAKE, FAKE, FAKE, native.CODES_F16_PRE, None, None, 0.171875,
                                                  native.BF16, 128, 256, 256, FAKE, wide, FAKE, None),
        b"gelu_out": lambda: lib.wdl_w4a4_gemm_gelu_u4_add(FAKE, FAKE, FAKE, FAKE, native.CODES_F16_PRE, None, None,
                                                           0, None, 0.171875, native.BF16, 128, 256, 256, FAKE, 256,
                                                           FAKE, FAKE, wide, None),
    }
    for needle, call in calls.items():
        assert call() == native.ERR_ARGUMENT, needle
        assert needle in lib.wdl_last_error() and b"2^31" in lib.wdl_last_error(), (needle, lib.wdl_last_error())


def test_workspace_sizes(native):
    lib = native.lib()
    M, K = 1392, 3072
    # room for float16 codes and float32 group scales, whatever the code format
    assert lib.wdl_w4a4_linear_workspace(M, K) == (M * K * 2 + 255) // 256 * 256 + (K // 64) * M * 4
    assert lib.wdl_w4a4_linear_workspace(0, K) == 0
    L, H = 5568, 24
    assert lib.wdl_sage_prep_workspace(L, H) == (2 * ((L + 63) // 64) + 1) * H * 128 * 4
    np_, lp = 1408, 5632
    up = lambda x: (x + 255) // 256 * 256  # noqa: E731
    want = (up(H * np_ * 128) + up(H * np_ // 32 * 8 * 4) + up(H * lp * 128) + up(H * lp // 64 * 4 * 4) +
            up(lp * H * 128) + up(H * lp * 4) + up(H * 4) + up(lib.wdl_sage_prep_workspace(L, H)))
    assert lib.wdl_sage_attend_workspace(1392, L, H) == want


def test_linear_validation(native):
    lib = native.lib()
    need = lib.wdl_w4a4_linear_workspace(128, 256)
    st = lib.wdl_w4a4_linear(FAKE, 256, 128, 256, None, native.BF16, FAKE, FAKE, native.CODES_E4M3, None, 256, FAKE,
                             256, FAKE, need - 1, None)
    assert st == native.ERR_ARGUMENT and b"workspace" in lib.wdl_last_error()
    st = lib.wdl_w4a4_linear(FAKE, 256, 128, 256, None, native.BF16, FAKE, FAKE, native.CODES_E4M3, None, 256, FAKE,
                             256, FAKE + 16, need, None)
    assert st == native.ERR_ARGUMENT and b"256-byte" in lib.wdl_last_error()
    M = 2 * (16 << 20) // 4096
    st = lib.wdl_w4a4_linear_noalloc(FAKE, 4096, M, 4096, None, native.BF16, FAKE, FAKE, native.CODES_E4M3, None, 256,
                                     FAKE, 256, None)
    assert st == native.ERR_ARGUMENT and b"16 MiB" in lib.wdl_last_error()
    # the quantizer reads smooth 16 bytes at a time: a misaligned smooth is refused before anything runs
    st = lib.wdl_w4a4_linear_noalloc(FAKE, 256, 128, 256, FAKE + 2, native.BF16, FAKE, FAKE, native.CODES_E4M3, None,
                                     256, FAKE, 256, None)
    assert st == native.ERR_ARGUMENT and b"smooth" in lib.wdl_last_error()
    for f in (2, native.CODES_F16_FOLD):  # 2 names no format; the float16 formats are not taken here
        st = lib.wdl_w4a4_linear_noalloc(FAKE, 256, 128, 256, None, native.BF16, FAKE, FAKE, f, None, 256, FAKE, 256,
                                         None)
        assert st == native.ERR_ARGUMENT and b"code format" in lib.wdl_last_error()


def test_norm_and_cache_validation(native):
    lib = native.lib()
    st = lib.wdl_ln_quant(FAKE, native.F32, 1000, 4, 1000, 1e-6, None, None, 0, None, None, None, native.BF16,
                          native.CODES_E4M3, FAKE, FAKE, None)
    assert st == native.ERR_ARGUMENT and b"multiple of 256" in lib.wdl_last_error()
    st = lib.wdl_ln_quant(FAKE, native.F32, 1024, 4, 1024, 1e-6, FAKE, None, 0, None, None, None, native.BF16,
                          native.CODES_E4M3, FAKE, FAKE, None)
    assert st == native.ERR_ARGUMENT and b"pairs" in lib.wdl_last_error()
    st = lib.wdl_ln_quant(FAKE, native.F32, 1024, 4, 1024, 1e-6, FAKE + 4, FAKE, 0, None, None, None, native.BF16,
                          native.CODES_E4M3, FAKE, FAKE, None)
    assert st == native.ERR_ARGUMENT and b"16-byte" in lib.wdl_last_error()
    st = lib.wdl_rms_rows(FAKE, 3072, 4, 3072, FAKE + 4, 1e-6, FAKE, 3072, None)
    assert st == native.ERR_ARGUMENT
    # Sage quantizers: float32 chunk rows must start 16-byte aligned
    work = lib.wdl_sage_prep_workspace(256, 2)
    st = lib.wdl_sage_prep_kv(None, None, None, None, 0, FAKE + 8, native.F32, 256, FAKE, native.BF16, 256, 256, 2,
                              FAKE, FAKE, FAKE, FAKE, FAKE, work, None)
    assert st == native.ERR_ARGUMENT and b"misaligned" in lib.wdl_last_error()
    st = lib.wdl_sage_quant_q(FAKE, 258, 64, 2, FAKE, FAKE, None)
    assert st == native.ERR_ARGUMENT


def test_python_layer_raises_value_error(native):
    lib = native.lib()
    st = lib.wdl_w4a4_gemm(FAKE, FAKE, FAKE, FAKE, native.CODES_E4M3, None, 128, 300, 256, FAKE, 512, None)
    with pytest.raises(ValueError, match="multiple of 256"):
        native.check(st)


def test_new_entry_points_validate_before_any_launch(native):
    """The tensor-parallel, low-rank, prescaled and Forcing-KV entry points reject bad calls up front."""
    lib = native.lib()
    err = lambda: lib.wdl_last_error()  # noqa: E731
    st = lib.wdl_w4a4_gemm_f32(FAKE, FAKE, FAKE, FAKE, native.CODES_F16_PRE, None, None, 0, 128, 256, 256, FAKE, 128,
                               None)
    assert st == native.ERR_ARGUMENT and b"ldo" in err()
    st = lib.wdl_w4a4_gemm_add(FAKE, FAKE, FAKE, FAKE, native.CODES_E4M3, None, FAKE, 255, 128, 256, 256, FAKE, 256,
                               None)
    assert st == native.ERR_ARGUMENT and b"addend" in err()
    st = lib.wdl_w4a4_gemm(FAKE, FAKE, FAKE, FAKE, native.CODES_F16_PRE, None, 128, 200, 256, FAKE, 256, None)
    assert st == native.ERR_ARGUMENT and b"multiple of 128" in err()
    for rank, ld, act in ((6, 8, FAKE), (0, 8, FAKE), (8, 6, FAKE), (8, 8, None), (8, 8, FAKE + 4)):
        lr = native.LowRank(act, ld, FAKE, rank)  # rank in fours, rows that hold it, 16-byte aligned, not null
        st = lib.wdl_w4a4_gemm_lowrank(FAKE, FAKE, FAKE, FAKE, native.CODES_F16_PRE, None, lr, 128, 256, 256, FAKE,
                                       256, None)
        assert st == native.ERR_ARGUMENT and b"low-rank" in err(), (rank, ld, act)
    for args, needle in (((FAKE, native.BF16, 64, 4, 48, FAKE, 8, FAKE, 8), b"multiple of 32"),
                         ((FAKE, native.BF16, 64, 4, 64, FAKE, 6, FAKE, 8), b"multiple of 4"),
                         ((FAKE, native.F16, 64, 4, 64, FAKE, 8, FAKE, 8), b"bf16 or f32"),
                         ((FAKE, native.BF16, 60, 4, 64, FAKE, 8, FAKE, 8), b"ldx"),
                         ((FAKE + 8, native.BF16, 64, 4, 64, FAKE, 8, FAKE, 8), b"misaligned")):
        assert lib.wdl_lowrank_down(*args, None) == native.ERR_ARGUMENT and needle in err(), needle
    lr = native.LowRank(FAKE, 8, FAKE, 6)
    for call in (lambda: lib.wdl_w4a4_gemm_f32_lowrank(FAKE, FAKE, FAKE, FAKE, native.CODES_F16_PRE, None, lr, 128,
                                                       256, 256, FAKE, 256, None),
                 lambda: lib.wdl_w4a4_gemm_gelu_u4_lowrank(FAKE, FAKE, FAKE, FAKE, native.CODES_F16_PRE, None, lr,
                                                           None, 0.171875, native.BF16, 128, 256, 256, FAKE, 256, FAKE,
                                                           None, 0, None)):
        assert call() == native.ERR_ARGUMENT and b"multiple of 4" in err()
    assert lib.wdl_rows_sumsq(FAKE, 256, 4, 0, 1, 0, FAKE, None) == native.ERR_ARGUMENT
    st = lib.wdl_residual_update(FAKE, 8, None, None, FAKE, 8, 4, 6, None)
    assert st == native.ERR_ARGUMENT and b"multiple of 4" in err()
    st = lib.wdl_qkv_prep_sharded(FAKE, 300, 16, 100, FAKE, FAKE, 1e-6, FAKE, 200, FAKE, 64, 4, 4, 0, FAKE, FAKE,
                                  None, None, None, None, 0, 0, None)
    assert st == native.ERR_ARGUMENT and b"multiple of 128" in err()
    st = lib.wdl_rms_rows_sharded(FAKE, 256, 4, 256, FAKE, 1e-6, None, 512, FAKE, 256, None)
    assert st == native.ERR_ARGUMENT and b"norm_dim" in err()
    work = lib.wdl_sage_attend_workspace(64, 128, 2)
    st = lib.wdl_sage_attend_maps(FAKE, 256, 64, FAKE, FAKE, FAKE, FAKE, 128, 4, None, None, 64, FAKE, native.F32, 256,
                                  FAKE, native.BF16, 256, 64, 2, 0.088, FAKE, 256, FAKE, work, None)
    assert st == native.ERR_ARGUMENT and b"head map" in err()
    st = lib.wdl_sage_attend_maps(FAKE, 256, 64, FAKE, FAKE, FAKE, FAKE, 32, 2, None, None, 64, FAKE, native.F32, 256,
                                  FAKE, native.BF16, 256, 64, 2, 0.088, FAKE, 256, FAKE, work, None)
    assert st == native.ERR_ARGUMENT and b"cache_rows" in err()
    st = lib.wdl_ln_quant_keep(FAKE, native.F32, 1024, 4, 1024, 1e-6, None, None, 0, None, None, None, native.F16,
                               native.CODES_F16_PRE, FAKE, FAKE, None, 0, None)
    assert st == native.ERR_ARGUMENT and b"bf16" in err()
    st = lib.wdl_w4a4_quantize_rows(FAKE, native.BF16, 256, None, 4, 256, native.F16, native.CODES_F16_PRE, FAKE, FAKE,
                                    None, None)
    assert st == native.ERR_ARGUMENT and b"bf16" in err()


def test_a_c_program_uses_the_abi(native, tmp_path):
    """include/wdl_b200.h is plain C11 and the library links into a C program (tests/native/abi_consumer.c), which
    gets the version, the workspace sizes and the rejections of invalid calls, with their messages."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    lib = Path(native.LIBRARY)
    exe = tmp_path / "abi_consumer"
    subprocess.run([gcc, "-std=c11", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}",
                    str(ROOT / "tests" / "native" / "abi_consumer.c"), f"-L{lib.parent}", f"-l:{lib.name}",
                    f"-Wl,-rpath,{lib.parent}", "-o", str(exe)], check=True)
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "PASSED" in run.stdout and "version wdl_b200" in run.stdout


def _ctype_of(decl):
    """The ctypes type a C parameter or return declaration maps to: pointers as one kind, scalars by type."""
    decl = decl.strip()
    if "*" in decl:
        return "pointer"
    base = re.sub(r"\b(const|volatile)\b", "", decl).split()
    base = base[0] if len(base) == 1 else base[-2] if len(base) > 1 else ""
    return {"int": ctypes.c_int, "int64_t": ctypes.c_int64, "size_t": ctypes.c_size_t, "float": ctypes.c_float,
            "double": ctypes.c_double, "uint32_t": ctypes.c_uint32}[base]


def test_binding_types_match_the_header_argument_by_argument(native):
    """Every argument of every entry point is bound with the C type the header declares (pointers as pointers,
    int / int64_t / size_t / float as such): a mismatch would pass garbage across the ABI, not fail."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    pointer_types = (ctypes.c_void_p, ctypes.c_char_p)
    for m in re.finditer(r"^([A-Za-z_][\w \t\*]*?)\b(wdl_\w+)\s*\(([^)]*)\)\s*;", text, flags=re.M):
        ret, name, params = m.group(1), m.group(2), m.group(3).strip()
        restype, argtypes = native.SIGNATURES[name]
        want_ret = _ctype_of(ret)
        assert (restype in pointer_types) if want_ret == "pointer" else restype is want_ret, name
        decls = [] if params in ("", "void") else [p for p in params.split(",")]
        for i, (decl, got) in enumerate(zip(decls, argtypes)):
            # a parameter "type name": drop the name to keep the type
            want = _ctype_of(decl.rsplit(None, 1)[0] + (" *" if "*" in decl.rsplit(None, 1)[-1] else ""))
            if want == "pointer":
                assert got in pointer_types or hasattr(got, "_type_"), (name, i, decl)
            else:
                assert got is want, (name, i, decl, got)
