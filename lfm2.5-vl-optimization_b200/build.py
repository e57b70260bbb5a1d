"""Build recipe for liblfm2q.so: every CUDA source of csrc/ compiled for sm_100a only, linked into one shared library
with a plain C ABI (include/lfm2q.h). No torch headers are involved; the library is loaded with ctypes.

    python lfm2.5-vl-optimization_b200/build.py [--force] [--jobs N]

Objects go to _build/ next to this file; the library to lfm2opt/liblfm2q.so (in-tree, so it travels with the
repository snapshot to the GPU box).
"""

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "lfm2opt" / "liblfm2q.so"
INCLUDE = HERE.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
                     "-diag-suppress", "128", "-I", str(INCLUDE)]


def nvcc():
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found: the CUDA 12.9 toolchain is required to build liblfm2q")
    return exe


def sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def _newer(out: Path, deps) -> bool:
    if not out.exists():
        return False
    t = out.stat().st_mtime
    return all(Path(d).stat().st_mtime <= t for d in deps)


def _compile(src: Path, force: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    deps = [src] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [INCLUDE / "lfm2q.h"]
    if not force and _newer(obj, deps):
        return obj
    cmd = [nvcc()] + NVCC_FLAGS + ["-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, jobs: int = 0, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), srcs))
    if force or not _newer(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", str(LIB)] + [str(o) for o in objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=0)
    a = ap.parse_args()
    try:
        build(a.force, a.jobs, verbose=True)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
