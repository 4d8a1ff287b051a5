"""Builds libafterimage_b200.so in-tree (afterimage_b200/lib/).

nvcc compiles the CUDA translation units for sm_100a only; g++ compiles the
host encoder with OpenMP; the shared library exports only the C ABI declared
in include/afterimage_b200.h (everything else, including the statically
linked CUDA runtime, stays hidden).

Usage: python -m afterimage_b200.csrc.build [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import os
import pathlib
import shutil
import subprocess
import sys
import tempfile

CSRC = pathlib.Path(__file__).resolve().parent
PKG = CSRC.parent
ROOT = PKG.parent
INCLUDE = ROOT / "include"
LIBDIR = PKG / "lib"
LIB = LIBDIR / "libafterimage_b200.so"

CU_SOURCES = ["decode.cu", "tp_ops.cu", "gemv.cu", "gemm_tc.cu", "stripe.cu", "allreduce.cu"]
CPP_SOURCES = ["encode.cpp", "io.cpp"]
HEADERS = ["aib_internal.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the afterimage_b200 CUDA library cannot be built")


def _inputs() -> list[pathlib.Path]:
    return ([CSRC / s for s in CU_SOURCES + CPP_SOURCES + HEADERS]
            + [INCLUDE / "afterimage_b200.h", pathlib.Path(__file__)])


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _inputs())


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    if not force and up_to_date():
        return LIB
    LIBDIR.mkdir(exist_ok=True)
    cc = nvcc()
    with tempfile.TemporaryDirectory(prefix="aib_build_") as td:
        tmp = pathlib.Path(td)
        objs = []
        for s in CU_SOURCES:
            o = tmp / (s + ".o")
            cmd = [cc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                   "-Xcompiler", "-fvisibility=hidden", "-I", str(INCLUDE), "-c", str(CSRC / s),
                   "-o", str(o)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            subprocess.run(cmd, check=True)
            objs.append(o)
        for s in CPP_SOURCES:
            o = tmp / (s + ".o")
            subprocess.run(["g++", "-O3", "-std=c++17", "-fPIC", "-fopenmp", "-fvisibility=hidden",
                            "-I", str(INCLUDE), "-c", str(CSRC / s), "-o", str(o)], check=True)
            objs.append(o)
        out_tmp = LIBDIR / (LIB.name + ".tmp%d" % os.getpid())
        vscript = tmp / "exports.map"
        vscript.write_text("{ global: aib_*; local: *; };\n")  # export only the C ABI
        subprocess.run([cc, *ARCH, "-shared", "-o", str(out_tmp), *map(str, objs),
                        "-Xcompiler", "-fopenmp", "-Xlinker", "--exclude-libs,ALL",
                        "-Xlinker", "--version-script=" + str(vscript)], check=True)
        os.replace(out_tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill report")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
