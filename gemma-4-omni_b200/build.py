"""Builds the listener C-ABI shared library in-tree with nvcc for sm_100a.

``python gemma-4-omni_b200/build.py`` (or ``build_library()``) compiles every
``csrc/*.cu`` into ``_build/*.o`` in parallel and links
``liblistener_b200.so`` next to this file.  Only the CUDA toolkit is needed
(no GPU): nvcc cross-compiles for sm_100a.
"""
from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "liblistener_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", str(HERE.parent / "include")]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the listener library needs the CUDA toolkit to build")


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    deps = [src, *CSRC.glob("*.h"), *CSRC.glob("*.cuh"), *(HERE.parent / "include").glob("*.h")]
    if obj.exists() and obj.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return obj
    cmd = [_nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        print(res.stderr, file=sys.stderr)
    return obj


def build_library(verbose: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    if force:
        for o in BUILD.glob("*.o"):
            o.unlink()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if LIB.exists() and LIB.stat().st_mtime >= max(o.stat().st_mtime for o in objs) and not force:
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build_library(verbose="-v" in sys.argv, force="-f" in sys.argv))
