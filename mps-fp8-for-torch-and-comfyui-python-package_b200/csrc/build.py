"""Build libfp8_b200.so (the C-ABI kernel library) in-tree with nvcc.

    python csrc/build.py [--verbose-ptxas]

Compiles every csrc/*.cu for sm_100a only and links them into
fp4_fp8_for_torch_mps/libfp8_b200.so next to the Python package, so the
library travels with the source tree. The CUDA runtime is linked statically;
the driver API (for TMA tensor maps) is reached through
cudaGetDriverEntryPointByVersion, so no libcuda link is needed at build time.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(os.path.dirname(HERE), "fp4_fp8_for_torch_mps")
OUT = os.path.join(PKG, "libfp8_b200.so")
BUILD = os.path.join(HERE, "_build")
HEADER = os.path.join(os.path.dirname(os.path.dirname(HERE)), "include", "fp8_b200.h")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def flags(verbose_ptxas: bool) -> list[str]:
    f = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                "--expt-relaxed-constexpr", "-DNDEBUG"]
    if verbose_ptxas:
        f += ["-Xptxas", "-v"]
    return f


def _deps_newer_than(obj: str) -> bool:
    t = os.path.getmtime(obj)
    deps = glob.glob(os.path.join(HERE, "*.cuh")) + [HEADER, __file__]
    return any(os.path.getmtime(d) > t for d in deps)


def compile_one(src: str, verbose_ptxas: bool) -> tuple[str, str]:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if (os.path.exists(obj) and os.path.getmtime(obj) >= os.path.getmtime(src)
            and not _deps_newer_than(obj) and not verbose_ptxas):
        return obj, ""
    cmd = [nvcc(), *flags(verbose_ptxas), "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stdout + r.stderr


def build(verbose_ptxas: bool = False, quiet: bool = True) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(HERE, "*.cu")))
    with cf.ThreadPoolExecutor(len(srcs)) as ex:
        results = list(ex.map(lambda s: compile_one(s, verbose_ptxas), srcs))
    for _, log in results:
        if log and (verbose_ptxas or not quiet):
            sys.stdout.write(log)
    objs = [o for o, _ in results]
    newest = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(OUT) or os.path.getmtime(OUT) < newest:
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-cudart", "static",
               "-o", OUT, *objs, "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose_ptxas, quiet=False))
