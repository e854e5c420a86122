"""Build libkanb200.so, the sm_100a kernel library, in the source tree.

    python -m kanforge_b200.build [--verbose] [--jobs N]

Every ``csrc/*.cu`` is compiled by nvcc for ``sm_100a`` (``-gencode
arch=compute_100a,code=sm_100a``) into an object, then linked with the static
CUDA runtime into ``kanforge_b200/_lib/libkanb200.so``.  nvcc cross-compiles,
so this works on a machine without a GPU.  Objects are rebuilt only when a
source or header is newer.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
OUT_DIR = PKG / "_lib"
LIB = OUT_DIR / "libkanb200.so"
OBJ_DIR = PKG.parent / "_build" / "obj"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put CUDA's bin on PATH")


def _headers_mtime() -> float:
    files = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((f.stat().st_mtime for f in files), default=0.0)


def _compile(src: Path, verbose: bool, ptxas_info: bool) -> Path:
    obj = OBJ_DIR / (src.stem + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, _headers_mtime()) and not ptxas_info:
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if ptxas_info or verbose:
        print(res.stderr, end="", flush=True)
    return obj


def build(verbose: bool = False, jobs: int | None = None, ptxas_info: bool = False) -> Path:
    """Compile every kernel source for sm_100a and link the shared library."""
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, ptxas_info), sources))
    newest = max(o.stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="rebuild everything with -Xptxas -v")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args(argv)
    print(build(args.verbose, args.jobs, args.ptxas_info))
    return 0


if __name__ == "__main__":
    sys.exit(main())
