"""Builds libglm5x_moe.so in-tree for sm_100a (nvcc cross-compiles; no GPU needed).

    python -m glm5x_moe.build        (from project-glm5x_b200/)

Object files go to <repo>/_build (git-ignored); the shared library lands next
to this file so it travels with the source tree.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
SRC_ROOT = PKG.parent
CSRC = SRC_ROOT / "csrc"
REPO = SRC_ROOT.parent
BUILD = REPO / "_build"
LIB = PKG / "libglm5x_moe.so"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                  "-Xcompiler", "-fno-fast-math", "--expt-relaxed-constexpr",
                  f"-I{REPO / 'include'}"]
CXXFLAGS = ["-std=c++17", "-O2", "-fPIC", "-ffp-contract=off", f"-I{REPO / 'include'}"]


def _sources():
    return sorted(CSRC.glob("*.cu")), sorted(CSRC.glob("*.cpp"))


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + [REPO / "include" / "glm5x_moe.h"]
    return max(h.stat().st_mtime for h in hs)


def _compile(src: Path) -> Path:
    obj = BUILD / (src.stem + ".o")
    if obj.exists() and obj.stat().st_mtime > max(src.stat().st_mtime, _headers_mtime()):
        return obj
    if src.suffix == ".cu":
        cmd = [NVCC, *NVFLAGS, "-c", str(src), "-o", str(obj)]
    else:
        cmd = ["g++", *CXXFLAGS, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    cu, cpp = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(_compile, cu + cpp))
    newest = max(o.stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose:
        print("built", LIB)
    return LIB


if __name__ == "__main__":
    build(verbose=True)
    sys.exit(0)
