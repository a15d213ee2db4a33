"""Build the emulator's CUDA library (sm_100a) in-tree.

``python -m tcgen05_b200.build`` compiles every ``csrc/*.cu`` into
``tcgen05_b200/_lib/libt5e.so`` with nvcc, for the B200 architecture only
(``-gencode arch=compute_100a,code=sm_100a``).  The library links the CUDA
runtime statically, so loading it needs no GPU and no CUDA library path.
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
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libt5e.so"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O2"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the emulator needs the CUDA toolkit to build")
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> Path:
    """Compile the library if any source is newer than it; return its path."""
    LIB_DIR.mkdir(exist_ok=True)
    srcs = sources()
    deps = srcs + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "t5e.h"]
    if not force and LIB.exists() and all(LIB.stat().st_mtime >= p.stat().st_mtime for p in deps):
        return LIB
    objs = []
    obj_dir = LIB_DIR / "obj"
    obj_dir.mkdir(exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    for src in srcs:
        obj = obj_dir / (src.stem + ".o")
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    args = set(sys.argv[1:])
    print(build(verbose=True, ptxas_info="--ptxas-info" in args, force="--force" in args))
