"""Builds libwdl_b200.so, the C-ABI library of the sm_100a kernels, in place next to the Python package.

    python wan-dit-lab_b200/build.py [--jobs N]

Every .cu file under csrc/ is compiled by nvcc for sm_100a only (-gencode arch=compute_100a,code=sm_100a),
with -lineinfo, then linked into one shared library with the CUDA runtime linked statically, so the library
depends on the driver alone and not on the version of libcudart a host process happens to load. Objects go
to _build/ (git-ignored); the library is written only when every file compiled.
"""

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
TARGET = HERE / "wan_dit_lab_b200" / "libwdl_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xptxas", "-v", "--expt-relaxed-constexpr",
         f"-I{HERE.parent / 'include'}"]


def nvcc():
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(cuda) / "bin" / "nvcc"
    return str(path) if path.exists() else (shutil.which("nvcc") or "nvcc")


def compile_one(source):
    obj = BUILD / (source.stem + ".o")
    log = BUILD / (source.stem + ".ptxas.txt")
    deps = [source, *CSRC.glob("*.h"), *CSRC.glob("*.cuh"), HERE.parent / "include" / "wdl_b200.h"]
    if obj.exists() and obj.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return obj, "up to date"
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(source), "-o", str(obj)]
    run = subprocess.run(cmd, capture_output=True, text=True)
    log.write_text(run.stdout + run.stderr)
    if run.returncode != 0:
        raise RuntimeError(f"nvcc failed on {source.name}:\n{run.stderr[-4000:]}")
    return obj, "compiled"


def build(jobs=None, verbose=True):
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs or os.cpu_count()) as pool:
        results = list(pool.map(compile_one, sources))
    objects = [o for o, _ in results]
    temporary = TARGET.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(temporary), *map(str, objects)]
    run = subprocess.run(cmd, capture_output=True, text=True)
    if run.returncode != 0:
        raise RuntimeError(f"link failed:\n{run.stderr[-4000:]}")
    os.replace(temporary, TARGET)
    if verbose:
        for (o, state) in results:
            print(f"{o.name}: {state}")
        print(f"built {TARGET}")
    return TARGET


if __name__ == "__main__":
    parser = argparse.ArgumentParser()
    parser.add_argument("--jobs", type=int, default=None)
    args = parser.parse_args()
    try:
        build(args.jobs)
    except RuntimeError as error:
        print(error, file=sys.stderr)
        sys.exit(1)
