"""Ahead-of-time build of libse12_b200.so (sm_100a) with nvcc.

``python -m se12_b200._build`` (or ``__graft_entry__.build()``) compiles the
single translation unit ``csrc/se12_lib.cu`` into the package directory, so
the shared object travels with the source tree. No JIT, no NVRTC.
"""

from __future__ import annotations

import os
import pathlib
import shutil
import subprocess
import sys

PACKAGE_DIR = pathlib.Path(__file__).resolve().parent
SOURCE = PACKAGE_DIR / "csrc" / "se12_lib.cu"
LIBRARY = PACKAGE_DIR / "libse12_b200.so"
GENCODE = "arch=compute_100a,code=sm_100a"


def nvcc_path() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and pathlib.Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def sources() -> list:
    return sorted((PACKAGE_DIR / "csrc").glob("*.cu*")) + sorted((PACKAGE_DIR / "csrc").glob("*.h")) + [
        PACKAGE_DIR.parent / "include" / "se12.h"
    ]


def up_to_date() -> bool:
    if not LIBRARY.exists():
        return False
    built = LIBRARY.stat().st_mtime
    return all(path.stat().st_mtime <= built for path in sources())


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    if not force and up_to_date():
        return LIBRARY
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [
        nvcc_path(),
        "-gencode",
        GENCODE,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC",
        "-shared",
        "-o",
        str(tmp),
        str(SOURCE),
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stdout}\n{result.stderr}")
    if verbose:
        print(result.stderr, file=sys.stderr)
    tmp.replace(LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
