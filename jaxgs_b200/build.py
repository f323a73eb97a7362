"""Builds libgsb200.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python -m jaxgs_b200.build          # or jaxgs_b200.build.build()

Every .cu file under csrc/ is compiled for sm_100a only
(-gencode arch=compute_100a,code=sm_100a) with -lineinfo, linked with the
static CUDA runtime, and written next to this file.  Rebuilds only when a
source is newer than the library.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
LIB = HERE / "libgsb200.so"
ARCH = "-gencode=arch=compute_100a,code=sm_100a"
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def needs_build() -> bool:
    if not LIB.exists():
        return True
    stamp = LIB.stat().st_mtime
    deps = sources() + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > stamp for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    objdir = HERE / "_build"
    objdir.mkdir(exist_ok=True)
    objs = []
    for src in sources():
        obj = objdir / (src.stem + ".o")
        cmd = [nvcc(), ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *objs]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
