"""Builds the native library ``carl_b200/libcarlb.so`` for sm_100a.

Device code is compiled with ``--fmad=false`` so every fp32 operation rounds
individually, as in the reference build; host arena code uses
``-ffp-contract=off`` for the same reason.  The CUDA runtime is linked
statically, so the library only needs the NVIDIA driver at run time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
SRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libcarlb.so"
DATA = PKG / "_data"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "--fmad=false", "-lineinfo", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-ffp-contract=off", "--expt-relaxed-constexpr"] + ARCH
CXX_FLAGS = ["-std=c++17", "-O2", "-fPIC", "-ffp-contract=off"]

CUDA_SOURCES = ["tick.cu", "envio.cu", "env.cu"]
CXX_SOURCES = ["arena.cpp", "tables.cpp"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("build failed: " + " ".join(cmd) + "\n" + proc.stdout + proc.stderr)


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compiles changed sources and links libcarlb.so; returns its path."""
    BUILD.mkdir(exist_ok=True)
    headers = sorted(SRC.glob("*.cuh")) + sorted(SRC.glob("*.hpp")) + [PKG.parent / "include" / "carlb.h"]
    nvcc = _nvcc()
    jobs = []
    objects = []
    for name in CUDA_SOURCES:
        src, obj = SRC / name, BUILD / (name + ".o")
        objects.append(obj)
        if _stale(obj, [src] + headers):
            extra = ["-Xptxas", "-v"] if ptxas_info else []
            jobs.append([nvcc, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)])
    cxx = "g++"  # the image's CXX (/opt/gcc) lacks some runtime pieces; the system g++ is complete
    for name in CXX_SOURCES:
        src, obj = SRC / name, BUILD / (name + ".o")
        objects.append(obj)
        if _stale(obj, [src] + headers):
            jobs.append([cxx, *CXX_FLAGS, "-c", str(src), "-o", str(obj)])
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as pool:
        for cmd in jobs:
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
        list(pool.map(_run, jobs))
    if jobs or not LIB.exists():
        _run([nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objects), "-ldl"])
    return LIB


def install_arena(source: str | os.PathLike | None = None) -> Path | None:
    """Copies the arena collision mesh next to the library (``_data/arena.obj``).

    The mesh comes from ``source`` (the reference's ``assets/arena.obj``) or
    from ``$CARL_ARENA_OBJ``.  At run time the library reads ``$CARL_ARENA_OBJ``
    first and falls back to this copy.
    """
    candidates = [source, os.environ.get("CARL_ARENA_OBJ")]
    for cand in candidates:
        if cand and Path(cand).is_file():
            DATA.mkdir(exist_ok=True)
            dst = DATA / "arena.obj"
            if not dst.exists() or Path(cand).stat().st_mtime > dst.stat().st_mtime:
                shutil.copyfile(cand, dst)
            return dst
    dst = DATA / "arena.obj"
    return dst if dst.exists() else None


if __name__ == "__main__":
    print(build(verbose=True, ptxas_info="--ptxas" in sys.argv))
    print(install_arena())
