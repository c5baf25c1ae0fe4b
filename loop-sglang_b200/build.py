"""Build the sm_100a shared library ``libloopsgl_b200.so`` next to this file.

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` and every host-only
``csrc/*.cpp`` with the host compiler (in parallel, skipping objects newer than
their sources and headers) and links them with the static CUDA runtime. Usable
as a script (``python loop-sglang_b200/build.py``) or via ``__graft_entry__.build()``.
nvcc cross-compiles, so no GPU is needed.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libloopsgl_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         f"-I{ROOT / 'include'}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def cxx() -> str:
    for cand in (os.environ.get("CXX"), shutil.which("g++"), shutil.which("c++")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("no host C++ compiler found")


def _stale(obj: Path, src: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in [src, *deps])


def build(verbose: bool = False, extra: list[str] | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))
    cc = nvcc()
    extra = extra or []

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.name + ".o")
        if _stale(obj, src, headers):
            if src.suffix == ".cpp":
                cmd = [cxx(), "-O3", "-std=c++17", "-fPIC", "-Wall", f"-I{ROOT / 'include'}",
                       "-c", str(src), "-o", str(obj)]
            else:
                cmd = [cc, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"compile failed on {src.name}:\n{r.stdout}\n{r.stderr}")
            if verbose and (r.stdout or r.stderr):
                print(r.stdout + r.stderr, flush=True)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        objs = list(ex.map(compile_one, sources))
    if not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [cc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, extra=["-Xptxas", "-v"] if "--ptxas" in sys.argv else None))
