"""Build of the in-tree CUDA library ``libchunkkv_b200.so`` (sm_100a only).

Each ``csrc/*.cu`` compiles to an object under ``_build/`` (rebuilt when it or a
header is newer), then everything links into ``chunkkv_b200/libchunkkv_b200.so``
with the CUDA runtime linked statically, so the library loads on a box that has
only the driver.  nvcc cross-compiles without a GPU.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libchunkkv_b200.so"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden", "-Xptxas", "-O3",
    f"-I{INCLUDE}",
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile changed sources and relink; returns the library path."""
    BUILD.mkdir(exist_ok=True)
    nvcc = _nvcc()
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    objs, relink = [], force or not LIB.exists()
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        stale = force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header)
        if not stale:
            continue
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, *(extra_flags or []), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        relink = True
    manifest = BUILD / "objects.txt"
    names = "\n".join(o.name for o in objs)
    if not manifest.exists() or manifest.read_text() != names:
        relink = True  # an object was added or removed
    if relink or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-cudart", "static",
               "-Xlinker", "--no-undefined", "-lrt", "-ldl", "-lpthread"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB)
        manifest.write_text(names)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
