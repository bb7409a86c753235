"""Builds oracle/_ref/libref_kernels.so: the reference's own CUDA kernels
(gemv_se12.cu, gemv_raw_bf16.cu, se12_common.cuh under
src/lws/adapters/cuda/kernels/ of the reference tree), compiled unchanged
for sm_100a with nvcc from where they lie, plus this directory's launchers
(ref_kernels.cu). Test and comparison infrastructure: the output goes to
oracle/_ref/ only and is never part of the product.

    python oracle/build_ref.py <reference-tree>

Without the reference tree (the GPU box) the prebuilt library is used as
it is; build() in __graft_entry__ calls this when the tree is present.
"""

from __future__ import annotations

import pathlib
import shutil
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "_ref" / "libref_kernels.so"
KERNELS = pathlib.Path("src/lws/adapters/cuda/kernels")


def build(reference_root: str) -> pathlib.Path:
    kernels = pathlib.Path(reference_root) / KERNELS
    for name in ("gemv_se12.cu", "gemv_raw_bf16.cu", "se12_common.cuh"):
        if not (kernels / name).exists():
            raise FileNotFoundError(f"{kernels / name} is missing")
    OUT.parent.mkdir(exist_ok=True)
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           "-I", str(kernels), "-o", str(OUT), str(HERE / "ref_kernels.cu")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python oracle/build_ref.py <reference-tree>")
    print(build(sys.argv[1]))
