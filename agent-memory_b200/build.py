"""Build libamq4.so in-tree with nvcc for sm_100a (B200).

Usage: ``python agent-memory_b200/build.py [--force]``.  The library is written next to
this file so it travels with the source tree; no JIT cache is involved.
"""

from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO / "include"
OUT = PKG_DIR / "libamq4.so"

SOURCES = ["am_abi.cu", "am_quantize.cu", "am_decode.cu", "am_prefill.cu", "am_noalloc.cu",
           "am_blocks.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or Path(cand).exists()):
            return cand
    return "nvcc"


def needs_build() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    deps += list(INCLUDE.glob("*.h"))
    return any(d.stat().st_mtime > t for d in deps)


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile every source to an object file in parallel (one nvcc per file), then link the
    shared library.  Objects go to a build folder next to the sources."""
    if not force and not needs_build():
        return OUT
    objdir = PKG_DIR / "_build"
    objdir.mkdir(exist_ok=True)
    flags = [f for f in NVCC_FLAGS if f != "-shared"]

    def compile_one(src: str) -> Path:
        obj = objdir / (Path(src).stem + ".o")
        cmd = [nvcc(), *flags, f"-I{INCLUDE}", f"-I{CSRC}", "-c", "-o", str(obj), str(CSRC / src)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        return obj

    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(compile_one, SOURCES))
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp),
           *[str(o) for o in objs]]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    build_library(force="--force" in sys.argv, verbose=True)
    print(OUT)
