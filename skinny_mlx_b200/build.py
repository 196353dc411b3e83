"""Build the in-tree CUDA library `_skinny_b200.so` for sm_100a with nvcc.

The library is a plain C-ABI shared object (include/skinny_b200.h); Python reaches it through
ctypes (skinny_mlx_b200/_lib.py).  cudart is linked statically so the .so does not depend on
which CUDA runtime the host process loaded.

    python -m skinny_mlx_b200.build            # rebuild if any source is newer than the .so
    python -m skinny_mlx_b200.build --force
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "_skinny_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES = sorted(CSRC.glob("*.cu"))
HEADERS = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted((ROOT / "include").glob("*.h"))


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (Path(cand).exists() or cand == "nvcc"):
            return cand
    raise RuntimeError("nvcc not found")


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    objdir = ROOT / "_build"
    objdir.mkdir(exist_ok=True)
    common = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              "-I", str(ROOT / "include"), "-I", str(CSRC)]
    if verbose:
        common += ["-Xptxas", "-v"]
    objs = []
    for src in SOURCES:
        obj = objdir / (src.stem + ".o")
        cmd = common + ["-c", str(src), "-o", str(obj)]
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    link = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *objs]
    subprocess.run(link, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    out = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(out)
