"""Build recipe for the fusion_b200 C-ABI library (``libfusion_b200.so``).

Compiles every ``csrc/*.cu`` for sm_100a with nvcc, in parallel, and links one shared
library next to this file. The library exports exactly the functions declared in
``include/fusion_b200.h``. Run ``python -m fusion_b200.build`` (or
``__graft_entry__.build()``); nvcc cross-compiles without a GPU.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libfusion_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler", "-fPIC,-ffp-contract=off",
    "-I", str(ROOT / "include"),
]


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src, *CSRC.glob("*.cuh"), *CSRC.glob("*.h"), ROOT / "include" / "fusion_b200.h"]
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def _compile(src: Path, verbose_ptxas: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if not _stale(obj, src):
        return obj
    cmd = [NVCC, *FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose_ptxas:
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> Path:
    """Compile and link; returns the path of the shared library."""
    BUILD.mkdir(exist_ok=True)
    srcs = _sources()
    if force:
        for o in BUILD.glob("*.o"):
            o.unlink()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose_ptxas), srcs))
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv))
