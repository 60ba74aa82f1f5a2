"""Builds libsvl_b200.so (the sm_100a kernels and the C ABI) in-tree with nvcc.

Run `python semantic-ai_b200/build.py` or call build(). Objects go to semantic-ai_b200/_build/,
the library to semantic-ai_b200/libsvl_b200.so. Only sources newer than their object are
recompiled.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT = PKG / "_build"
LIB = PKG / "libsvl_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

# -fmad=false: no implicit a*b+c contraction, so element-wise arithmetic rounds like the
# reference CPU path; kernels request FMAs with fmaf() where they want them.
NVCC_FLAGS = [
    "-std=c++17", "-O3", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-fmad=false", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden,-O3",
    "-I", str(PKG.parent / "include"),
]


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _deps():
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [PKG.parent / "include" / "svl_cuda.h"]


def _compile(src: Path, extra: list[str]) -> Path:
    obj = OUT / (src.stem + ".o")
    newest_dep = max([src.stat().st_mtime] + [d.stat().st_mtime for d in _deps()])
    if obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj
    cmd = [NVCC, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False, extra: list[str] | None = None) -> Path:
    OUT.mkdir(exist_ok=True)
    extra = extra or []
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), _sources()))
    if LIB.exists() and LIB.stat().st_mtime >= max(o.stat().st_mtime for o in objs):
        return LIB
    cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
           "-Xcompiler", "-fPIC", "-o", str(LIB), *map(str, objs), "-cudart", "static"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    extra = sys.argv[1:]
    build(verbose=True, extra=extra)
