"""Build recipe for the CPU oracle libraries (TEST INFRASTRUCTURE ONLY).

* ``oracle/liboracle_kernels.so`` — the plain-C restatement in ``kernels.c``.
* ``oracle/_ref/libref_kernels.so`` — the reference's own ``kernels.cl``,
  compiled unmodified from the read-only reference checkout through the shim in
  ``ref_host.cpp``.  Built only where that checkout exists; the built file is
  git-ignored but travels with the working tree to machines without it.

Both are compiled with ``-ffp-contract=off`` (the reference kernels declare
``FP_CONTRACT OFF``) and OpenMP for the independent work items.

Usage: ``python oracle/build.py [--reference-root DIR]``; without the
argument the checkout is taken from the ``MIRACLE_REFERENCE_ROOT``
environment variable, and without either only the C restatement is built.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "liboracle_kernels.so"
REF_LIB = HERE / "_ref" / "libref_kernels.so"
_FLAGS = ["-O2", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-shared", "-fPIC"]


def _stale(target: Path, *sources: Path) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(s.stat().st_mtime > mtime for s in sources)


def build_oracle(force: bool = False) -> Path:
    src = HERE / "kernels.c"
    if force or _stale(ORACLE_LIB, src):
        subprocess.run(["gcc", "-std=c11", *_FLAGS, str(src), "-o", str(ORACLE_LIB), "-lm"], check=True)
    return ORACLE_LIB


def build_reference(reference_root: Path | None = None, force: bool = False) -> Path | None:
    root = reference_root or os.environ.get("MIRACLE_REFERENCE_ROOT")
    kernels = Path(root) / "miracle_reasoning" / "kernels.cl" if root else None
    if kernels is None or not kernels.is_file():
        return REF_LIB if REF_LIB.exists() else None
    shim = HERE / "ref_host.cpp"
    if force or _stale(REF_LIB, shim, kernels):
        REF_LIB.parent.mkdir(exist_ok=True)
        subprocess.run(["g++", "-std=c++17", *_FLAGS, "-Wno-unknown-pragmas",
                        f'-DREF_KERNELS_CL="{kernels}"', str(shim), "-o", str(REF_LIB)], check=True)
    return REF_LIB


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference-root", type=Path)
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args(argv)
    print(build_oracle(args.force))
    print(build_reference(args.reference_root, args.force))
    return 0


if __name__ == "__main__":
    sys.exit(main())
