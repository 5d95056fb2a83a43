"""Build recipe for kernel-lab's own CUDA kernels, as a test-only comparator.

Compiles kernel-lab's csrc/paged_attention.cu and csrc/rmsnorm.cu where they lie (the reference
tree, read-only) plus this directory's ref_shim.cu (a C ABI over kernel-lab's launchers) with nvcc
for sm_100a, into oracle/_ref/libkernel_lab_ref.so. Nothing is copied from the reference tree and
its own build system (setup.py / torch extension) is not used: the two kernel files and their
header need nothing but the CUDA toolkit (kernel-lab csrc/kernel_lab.h:1-3).

Only tests/ load the result. The reference tree is given by --reference or the environment
variable KL_REFERENCE_DIR; without one (the GPU box has no reference tree), nothing is built and
the prebuilt library, if any, is used as is.

    python oracle/build_ref.py --reference DIR
"""

from __future__ import annotations

import argparse
import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
LIB = OUT_DIR / "libkernel_lab_ref.so"
SOURCES = ("csrc/paged_attention.cu", "csrc/rmsnorm.cu")


def reference_from_env() -> Path | None:
    env = os.environ.get("KL_REFERENCE_DIR")
    return Path(env) if env else None


def build(reference: Path | None = None, force: bool = False) -> Path | None:
    """Compile the comparator library; returns its path, or None without the reference tree."""
    reference = reference if reference is not None else reference_from_env()
    if reference is None:
        return LIB if LIB.exists() else None
    srcs = [reference / s for s in SOURCES]
    if not all(s.exists() for s in srcs):
        return LIB if LIB.exists() else None
    inputs = srcs + [reference / "csrc" / "kernel_lab.h", reference / "csrc" / "common.cuh", HERE / "ref_shim.cu"]
    if LIB.exists() and not force and LIB.stat().st_mtime >= max(p.stat().st_mtime for p in inputs):
        return LIB
    OUT_DIR.mkdir(exist_ok=True)
    nvcc = os.environ.get("NVCC", "nvcc")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo",
           "-Xcompiler", "-fPIC", "-shared", "-cudart", "static", f"-I{reference / 'csrc'}",
           *map(str, srcs), str(HERE / "ref_shim.cu"), "-o", str(LIB)]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", type=Path, default=reference_from_env(),
                    help="kernel-lab's source tree (default: $KL_REFERENCE_DIR)")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.reference, a.force))
