"""Build libmiracle_cuda.so in-tree for sm_100a (B200).

    python miraclereasoning-cpu_b200/build.py [--force] [--verbose] [--ptxas-verbose]

nvcc compiles every csrc/*.cu with ``-gencode arch=compute_100a,code=sm_100a``
and links one shared library next to this file.  The build is incremental on
source timestamps.  No GPU is needed to build.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "csrc"
OUT = HERE / "libmiracle_cuda.so"
OBJ = HERE / "_build"
HEADER = HERE.parent / "include" / "miracle_cuda.h"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libmiracle_cuda.so")
    return path


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(d.stat().st_mtime > mtime for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    headers = list(SRC.glob("*.cuh")) + [HEADER]
    OBJ.mkdir(exist_ok=True)
    objects = []
    for src in sorted(SRC.glob("*.cu")):
        obj = OBJ / (src.stem + ".o")
        objects.append(obj)
        if force or ptxas_verbose or _stale(obj, [src, *headers]):
            cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
            if ptxas_verbose:
                cmd += ["-Xptxas", "-v"]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(OUT, objects):
        tmp = OUT.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", *map(str, objects), "-o", str(tmp), "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, OUT)
    return OUT


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--ptxas-verbose", action="store_true")
    args = parser.parse_args(argv)
    print(build(args.force, args.verbose, args.ptxas_verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
