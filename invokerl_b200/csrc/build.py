"""Build the sm_100a shared library `invokerl_b200/libinvokerl_b200.so` with nvcc.

Every `.cu` file in this directory is compiled for sm_100a only and linked into one shared
library that exports the C ABI declared in `include/invokerl_b200.h`.  Objects are rebuilt when
their source, a header, or this file is newer.  Usage: `python -m invokerl_b200.csrc.build`.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
ROOT = PKG.parent
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build" / "invokerl_b200"
LIB = PKG / "libinvokerl_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-v",
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; set NVCC or put CUDA 12.9 on PATH")
    return cand


def _deps() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h")) + [Path(__file__).resolve()]


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    newest = max(p.stat().st_mtime for p in [src, *_deps()])
    if obj.exists() and obj.stat().st_mtime >= newest:
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    log = BUILD / (src.stem + ".ptxas.txt")
    log.write_text(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr[-6000:]}")
    if verbose:
        sys.stderr.write(f"[invokerl_b200] compiled {src.name}\n")
    return obj


def build(verbose: bool = False) -> Path:
    """Compile every kernel source for sm_100a and link `libinvokerl_b200.so` in the package."""
    BUILD.mkdir(parents=True, exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if LIB.exists() and LIB.stat().st_mtime >= newest:
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stderr[-4000:]}")
    os.replace(tmp, LIB)
    if verbose:
        sys.stderr.write(f"[invokerl_b200] linked {LIB}\n")
    return LIB


if __name__ == "__main__":
    print(build(verbose=True))
