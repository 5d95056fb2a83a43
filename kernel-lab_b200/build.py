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
import re
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


def run(cmd: list[str], verbose: bool, cwd: Path | None = None) -> str:
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True, cwd=cwd)
    if proc.returncode != 0:
        raise RuntimeError(f"build step failed ({proc.returncode}): {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    return proc.stderr


def decode_spills(ptxas_log: str) -> dict[str, int]:
    """Spill-load bytes per decode_tc_kernel instantiation, from ptxas's -v report."""
    spills, kernel = {}, None
    for line in ptxas_log.splitlines():
        m = re.search(r"Compiling entry function '(\S+)'", line)
        if m:
            kernel = m.group(1)
        m = re.search(r"(\d+) bytes spill loads", line)
        if m and kernel and "decode_tc_kernel" in kernel:
            spills[kernel] = int(m.group(1))
    return spills


def build_library(force: bool = False, verbose: bool = False) -> Path:
    nvcc = str(cuda_home() / "bin" / "nvcc")
    OBJ_DIR.mkdir(exist_ok=True)
    # The decode kernels run at their register cap (168 a thread), where ptxas's allocation tips on
    # details of its input that have nothing to do with the code: the same source gave the headline
    # kernel 0 or 212 bytes of spill loads and the two-n-tile kernel 1,364 or 2,024 (ragged MQA 295
    # or 409 us) depending on the object file's path, the source path as given to nvcc, -lineinfo
    # and the --split-compile partition count ("0" follows the machine's cores). For one input the
    # result is the same every time. So nvcc runs from the repository root on relative paths,
    # without -lineinfo, with 8 partitions; ptxas's report (-Xptxas -v) is read back, and the decode
    # file is compiled under up to six trial object names, keeping the first whose one-n-tile
    # kernels do not spill (else the fewest spills). The build prints which one it kept.
    rel_include, rel_csrc = INCLUDE.relative_to(REPO), CSRC.relative_to(REPO)
    base = [*ARCH, "-O3", "-std=c++17", "-Xcompiler", "-fPIC", f"-I{rel_include}", f"-I{rel_csrc}", "-Xptxas", "-v"]
    objs = []
    for src in CU_SOURCES:
        obj = OBJ_DIR / (Path(src).stem + ".o")
        objs.append(obj)
        if not (force or stale(obj, [CSRC / src, *HEADERS])):
            continue
        rel_src = str(rel_csrc / src)
        if src != "paged_decode.cu":
            run([nvcc, *base, "--split-compile=8", "-c", rel_src, "-o", str(obj)], verbose, cwd=REPO)
            continue
        best = None
        for k in range(6):
            trial = OBJ_DIR / f"paged_decode.trial{k}.o"
            spills = decode_spills(run([nvcc, *base, "--split-compile=8", "-c", rel_src, "-o", str(trial)],
                                       verbose, cwd=REPO))
            hot = sum(v for name, v in spills.items() if re.search(r"Li(64|128)ELi1E", name))
            key = (hot, sum(spills.values()))
            print(f"decode kernels, trial {k}: {key[1]} bytes of spill loads over {len(spills)} instantiations, "
                  f"{hot} in the one-n-tile kernels", flush=True)
            if best is None or key < best[0]:
                best = (key, trial, k)
            if hot == 0:
                break
        print(f"decode kernels: kept trial {best[2]}", flush=True)
        shutil.copyfile(best[1], obj)
    if force or stale(LIB, objs):
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
