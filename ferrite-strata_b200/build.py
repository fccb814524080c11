"""Build libstrata_b200.so in-tree for sm_100a.

Every CUDA source is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a -lineinfo``; the plugin's host C++
is compiled by g++.  Objects go to ``_build/`` beside this file and the shared
library to ``libstrata_b200.so`` in this directory, with the CUDA runtime
linked statically so the library does not depend on whichever libcudart the
host process loaded first.  Rebuilds are incremental on file timestamps.

Run directly (``python ferrite-strata_b200/build.py``) or through
``__graft_entry__.build()``.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT_DIR = HERE / "_build"
LIB = HERE / "libstrata_b200.so"
INCLUDE = HERE.parent / "include"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else os.environ.get("CXX", "g++")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
                     "-I" + str(INCLUDE), "--expt-relaxed-constexpr"]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-Wno-unused-function",
             "-I/usr/local/cuda/include", "-I" + str(INCLUDE)]


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted((CSRC / "plugin").glob("*.cpp"))


def _headers() -> list[Path]:
    return (sorted(CSRC.rglob("*.cuh")) + sorted(CSRC.rglob("*.hpp"))
            + sorted(INCLUDE.glob("*.h")))


def _obj(src: Path) -> Path:
    rel = src.relative_to(CSRC)
    return OUT_DIR / (str(rel).replace("/", "_") + ".o")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path) -> tuple[Path, str]:
    obj = _obj(src)
    if src.suffix == ".cu":
        cmd = [NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    else:
        cmd = [CXX, *CXX_FLAGS, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compiling {src.name} failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(verbose: bool = False) -> Path:
    OUT_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    hdrs = _headers()
    todo = [s for s in srcs if _stale(_obj(s), [s, *hdrs])]
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            for obj, err in ex.map(_compile, todo):
                if verbose and err.strip():
                    print(err, file=sys.stderr)
    objs = [_obj(s) for s in srcs]
    if _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs),
               "-ldl", "-lpthread", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"linking failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose=True))
