"""Build the in-tree C-ABI library ``tricast_b200/_lib/libtricast_b200.so`` for sm_100a.

``python -m tricast_b200.build`` (or ``build()``) compiles each ``csrc/*.cu`` to an object in parallel
(under ``_build/`` at the repository root) and links them; it is skipped when the library is newer
than every source. nvcc cross-compiles on a machine without a GPU.
IEEE semantics matter for bit-exactness, so no fast-math flags are used: fp32 division, square root
and subnormals stay IEEE (``-ftz=false -prec-div=true -prec-sqrt=true``) and ``-fmad=false`` keeps
the compiler from contracting separately rounded multiplies and adds.
"""

from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "_lib" / "libtricast_b200.so"
INCLUDE = PKG.parent / "include"
OBJ = PKG.parent / "_build" / "obj"

NVCC_FLAGS = [
    "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-ftz=false", "-prec-div=true", "-prec-sqrt=true", "-fmad=false",
    "--expt-relaxed-constexpr", "-Xptxas", "-O3",
]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    deps = sources() + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "tricast_b200.h"]
    return any(p.stat().st_mtime > built for p in deps)


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (cand == "nvcc" or Path(cand).exists()):
            return cand
    return "nvcc"


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    LIB.parent.mkdir(parents=True, exist_ok=True)
    OBJ.mkdir(parents=True, exist_ok=True)
    objs = [OBJ / (src.stem + ".o") for src in sources()]

    def compile_one(pair):
        src, obj = pair
        cmd = [nvcc(), *NVCC_FLAGS, "-I", str(INCLUDE), "-c", "-o", str(obj), str(src)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)

    with ThreadPoolExecutor(max_workers=max(1, min(len(objs), os.cpu_count() or 1))) as pool:
        list(pool.map(compile_one, zip(sources(), objs)))
    tmp = LIB.with_suffix(".so.tmp")
    link = [nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(tmp), *map(str, objs)]
    if verbose:
        print(" ".join(link), file=sys.stderr)
    subprocess.run(link, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
