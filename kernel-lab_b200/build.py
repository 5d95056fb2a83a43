"""Build the sm_100a kernels in-tree.

    python kernel-lab_b200/build.py [--force]

Produces, inside ``kernel-lab_b200/kernel_lab/``:

* ``libkernel_lab_b200.so`` -- the kernels and the C ABI declared in
  ``include/kernel_lab_b200.h`` (nvcc, ``-gencode arch=compute_100a,code=sm_100a``,
  CUDA runtime linked statically, no PyTorch);
* ``_C<ext-suffix>.so`` -- the ``torch.ops.kernel_lab`` registrations, a thin C++
  layer over the C ABI, linked against the library above (rpath ``$ORIGIN``).

A target is rebuilt only when one of its sources is newer (or ``--force``).
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = REPO / "include"
OUT_DIR = PKG_ROOT / "kernel_lab"
OBJ_DIR = PKG_ROOT / "_build"
LIB = OUT_DIR / "libkernel_lab_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = ["rmsnorm.cu", "paged_decode.cu", "kv_append.cu"]
HEADERS = [CSRC / "common.cuh", INCLUDE / "kernel_lab_b200.h"]


def cuda_home() -> Path:
    env = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if env:
        return Path(env)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return Path(nvcc).resolve().parent.parent
    return Path("/usr/local/cuda")


def host_cxx() -> str:
    """The C++ compiler for the torch extension. It must link libstdc++ dynamically, like
    torch itself: a toolchain that links it statically gives the extension a second copy of
    the iostream/locale state, and formatting a TORCH_CHECK message then crashes."""
    for cand in (os.environ.get("KL_CXX"), "/usr/bin/g++", os.environ.get("CXX"), "g++"):
        if cand and shutil.which(cand):
            return cand
    raise RuntimeError("no C++ compiler found")


def ext_module_path() -> Path:
    return OUT_DIR / f"_C{sysconfig.get_config_var('EXT_SUFFIX')}"


def stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"build step failed ({proc.returncode}): {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")


def build_library(force: bool = False, verbose: bool = False) -> Path:
    nvcc = str(cuda_home() / "bin" / "nvcc")
    OBJ_DIR.mkdir(exist_ok=True)
    # --split-compile: the device compilation of one file runs in parallel (the decode file's
    # kernel instantiations take minutes on one thread). The count is fixed, not "every core":
    # how the device code is split changes the registers ptxas gives the decode kernels, and with
    # it their spills (bf16 decode kernels, spill loads in total: 13.1 KB split 8 ways, 24.5 KB
    # split over an 8-core machine's "0", 17.5 KB unsplit; the two-n-tile kernel 1,364 against
    # 2,024 bytes, which took ragged MQA from 295 to 409 us). Eight ways is the best measured.
    flags = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", f"-I{INCLUDE}", f"-I{CSRC}",
             "--split-compile=8"]
    objs = []
    jobs = []
    for src in CU_SOURCES:
        obj = OBJ_DIR / (Path(src).stem + ".o")
        objs.append(obj)
        if force or stale(obj, [CSRC / src, *HEADERS]):
            jobs.append([nvcc, *flags, "-c", str(CSRC / src), "-o", str(obj)])
    with ThreadPoolExecutor(max_workers=len(CU_SOURCES)) as pool:
        list(pool.map(lambda c: run(c, verbose), jobs))
    if force or jobs or stale(LIB, objs):
        run([nvcc, *ARCH, "-shared", "-o", str(LIB), *map(str, objs)], verbose)
    return LIB


def build_torch_ext(force: bool = False, verbose: bool = False) -> Path:
    import torch
    from torch.utils.cpp_extension import include_paths, library_paths

    target = ext_module_path()
    src = CSRC / "torch_bindings.cpp"
    if not (force or stale(target, [src, LIB, INCLUDE / "kernel_lab_b200.h"])):
        return target
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [
        host_cxx(),
        "-O2",
        "-std=c++17",
        "-fPIC",
        "-shared",
        str(src),
        "-o",
        str(target),
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        "-DTORCH_EXTENSION_NAME=_C",
        f"-I{INCLUDE}",
        f"-I{sysconfig.get_paths()['include']}",
        f"-I{cuda_home() / 'include'}",
        *[f"-I{p}" for p in include_paths()],
        f"-L{OUT_DIR}",
        "-lkernel_lab_b200",
        "-Wl,-rpath,$ORIGIN",
        *[f"-L{p}" for p in library_paths()],
        "-lc10",
        "-lc10_cuda",
        "-ltorch",
        "-ltorch_cpu",
        "-ltorch_cuda",
        "-ltorch_python",
    ]
    run(cmd, verbose)
    return target


def build(force: bool = False, verbose: bool = False) -> None:
    build_library(force, verbose)
    build_torch_ext(force, verbose)


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    build(args.force, args.verbose)
    print(f"built {LIB.name} and {ext_module_path().name} in {OUT_DIR}", file=sys.stderr)
