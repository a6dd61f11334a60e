"""Builds the sampler library in-tree: lib/libq3s_sampler.so for sm_100a.

    python qwen3tts-rs_b200/build.py [--ptxas-verbose]

nvcc compiles the kernels (csrc/*.cu) and the C ABI (csrc/*.cpp) into one
shared library with the CUDA runtime linked statically.  The kernel
translation unit is built with -fmad=false so that no f32 multiply-add is
contracted (the reference rounds every product and sum separately).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libq3s_sampler.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-fmad=false",
          "-ftz=false", "-prec-div=true", "-prec-sqrt=true", f"-I{INCLUDE}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the sampler library needs the CUDA toolkit to build")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    deps = sources() + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + \
        sorted(INCLUDE.glob("*.h")) + [Path(__file__)]
    return all(p.stat().st_mtime <= t for p in deps)


def build(force: bool = False, ptxas_verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, *COMMON, "-shared", "-o", str(tmp), *map(str, sources())]
    if ptxas_verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ptxas-verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force or args.ptxas_verbose, ptxas_verbose=args.ptxas_verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
