"""Build recipe of libeinsum_ir_b200.so (sm_100a only).

Compiles every CUDA source under csrc/ and every host C++ source under
csrc/host/ with nvcc for `-gencode arch=compute_100a,code=sm_100a`, then links
one shared library in this package directory (in-tree, so it travels with the
repository to the GPU machine). Also builds the C++ drivers (bench_expression,
bench_binary) next to it.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libeinsum_ir_b200.so"
ROOT = PKG.parent

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
          f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{CSRC / 'host'}"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    cu = sorted(CSRC.glob("*.cu"))
    cpp = sorted((CSRC / "host").glob("*.cpp"))
    return cu, cpp


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.relative_to(CSRC).as_posix().replace("/", "__") + ".o")
    deps = [src] + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + \
        sorted((CSRC / "host").glob("*.h")) + sorted((ROOT / "include").glob("*.h"))
    if obj.exists() and all(obj.stat().st_mtime >= d.stat().st_mtime for d in deps if d.exists()):
        return obj
    cmd = [_nvcc(), *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [_nvcc(), *COMMON, "-x", "c++", "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src}\n{r.stdout}\n{r.stderr}")
    return obj


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    cu, cpp = _sources()
    srcs = cu + cpp
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [_nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed\n{r.stdout}\n{r.stderr}")
    _build_drivers(verbose)
    return LIB


def _build_drivers(verbose: bool) -> None:
    drivers = []
    for sub in ("drivers", "tests"):
        if (CSRC / sub).exists():
            drivers += sorted((CSRC / sub).glob("*.cpp"))
    for src in drivers:
        exe = PKG / src.stem
        if exe.exists() and exe.stat().st_mtime >= max(src.stat().st_mtime, LIB.stat().st_mtime):
            continue
        cmd = [_nvcc(), *COMMON, "-x", "c++", str(src), "-o", str(exe), f"-L{PKG}",
               "-leinsum_ir_b200", "-Xlinker", "-rpath=$ORIGIN", "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"driver build failed: {src}\n{r.stdout}\n{r.stderr}")


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
