"""Build libstratum_nf4.so (sm_100a) in-tree with nvcc.

``python -m stratum_b200._build`` compiles every ``csrc/*.cu`` into one shared
library next to this file.  The library is a plain C ABI (include/stratum_nf4.h)
with no torch headers, so it is loaded with ctypes and rebuilt only when a
source is newer than the library.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libstratum_nf4.so"
OBJDIR = PKG / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-Wall",
    f"-I{ROOT / 'include'}",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the NF4 kernels need the CUDA toolkit to build")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in sources() + headers() + [Path(__file__)])


def build(verbose: bool = False, force: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile all kernels; returns the library path."""
    if not force and not needs_build():
        return LIB
    nvcc = nvcc_path()
    OBJDIR.mkdir(exist_ok=True)
    objs = []
    procs = []
    for src in sources():
        obj = OBJDIR / (src.stem + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *(extra_flags or []), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        objs.append(obj)
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            failed.append(f"{src.name}:\n{out}")
        elif verbose and out.strip():
            print(out, flush=True)
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-cudart", "static", "-ldl", "-lrt", "-lpthread"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv, extra_flags=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None)
    print(LIB)
