"""Build the VectorCore CUDA device library for sm_100a (B200).

    python vectorcore_b200/build.py          # -> vectorcore_b200/_lib/libvc_cuda.so

(run by path, not with -m: importing the package loads the library, which
may not exist yet). 
nvcc compiles every ``csrc/*.cu`` for ``sm_100a`` only (no PTX for other
targets), with ``-fmad=false`` (no contraction of a*b+c, so elementwise results
match the reference's CPU arithmetic bit for bit) and IEEE division / square
root. The CUDA runtime is linked statically, so the library does not depend on
which libcudart another component of the process (e.g. torch) loaded. The
build is incremental: objects are rebuilt only when a source or header is
newer. It needs nvcc, not a GPU.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIBDIR = PKG / "_lib"
BUILDDIR = PKG / "_lib" / "obj"
LIBNAME = "libvc_cuda.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH, "-O3", "-lineinfo", "-std=c++17",
    "-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    f"-I{INCLUDE}", f"-I{CSRC}",
]


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build vectorcore_b200")
    return exe


def library_path() -> Path:
    """The built library; VECTORCORE_B200_LIB overrides the location."""
    override = os.environ.get("VECTORCORE_B200_LIB")
    return Path(override) if override else LIBDIR / LIBNAME


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _headers():
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    BUILDDIR.mkdir(parents=True, exist_ok=True)
    exe = nvcc()
    headers = _headers()
    objs = []
    todo = []
    for src in _sources():
        obj = BUILDDIR / (src.stem + ".o")
        objs.append(obj)
        if _stale(obj, [src, *headers, Path(__file__)]):
            todo.append((src, obj))

    def compile_one(item):
        src, obj = item
        cmd = [exe, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
        return src.name

    if todo:
        workers = jobs or min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=workers) as pool:
            for name in pool.map(compile_one, todo):
                if verbose:
                    print(f"  compiled {name}", flush=True)
    lib = library_path()
    if todo or _stale(lib, objs):
        cmd = [exe, *ARCH, "-shared", "-o", str(lib), *map(str, objs), "-ldl", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return lib


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv)
    print(path)
