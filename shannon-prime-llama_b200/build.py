"""Build the B200 Shannon-Prime C-ABI library in-tree.

Compiles csrc/*.cu for sm_100a (nvcc -gencode arch=compute_100a,code=sm_100a)
and csrc/*.c / *.cpp with the host compiler, then links
lib/libshannon_prime_b200.so.  Objects go to _build/ beside this file.

    python shannon-prime-llama_b200/build.py [--force] [--jobs N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "lib" / "libshannon_prime_b200.so"
INCLUDE = ROOT / "include"

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = GENCODE + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills",
    f"-I{INCLUDE}", f"-I{CSRC}",
]
HOST_CC = "/usr/bin/gcc" if os.path.exists("/usr/bin/gcc") else "gcc"
HOST_CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"
HOST_FLAGS = ["-O2", "-fPIC", "-Wall", f"-I{INCLUDE}", f"-I{CSRC}",
              f"-I{os.path.join(CUDA_HOME, 'include')}"]


def _headers_mtime() -> float:
    hs = list(INCLUDE.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, force: bool, hdr_mtime: float) -> Path:
    obj = BUILD / (src.name + ".o")
    if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr_mtime):
        return obj
    if src.suffix == ".cu":
        cmd = [NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    elif src.suffix == ".c":
        cmd = [HOST_CC, *HOST_FLAGS, "-std=c11", "-c", str(src), "-o", str(obj)]
    else:
        cmd = [HOST_CXX, *HOST_FLAGS, "-std=c++17", "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    srcs = sorted([*CSRC.glob("*.cu"), *CSRC.glob("*.c"), *CSRC.glob("*.cpp")])
    hdr = _headers_mtime()
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, hdr), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not LIB.exists() or LIB.stat().st_mtime < newest:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [NVCC, *GENCODE, "-shared", "-o", str(tmp), *map(str, objs),
               "-lcudart", "-Xcompiler", "-fPIC"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        shutil.move(str(tmp), str(LIB))
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args()
    print(build(args.force, args.jobs))
