"""Build liblyth_b200.so in-tree with nvcc for sm_100a.

Every CUDA source under lyth_b200/csrc is compiled (in parallel) with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3 -fmad=false`` and linked into
``lyth_b200/liblyth_b200.so``. ``-fmad=false`` keeps every unfused multiply and add of the
reference unfused; the fused steps are written as explicit ``__fmaf_rn``. The library links
the CUDA runtime statically and no libcuda (driver entry points are fetched at run time), so it
loads on a machine without a GPU. Usage: ``python lyth_b200/build.py [-v]`` (by path: importing
the package first would load the previous library).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "liblyth_b200.so")
BUILD = os.path.join(HERE, "_build")

NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + [
    "-lineinfo", "-O3", "-std=c++17", "-fmad=false", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    "-I", os.path.join(ROOT, "include"), "-I", CSRC,
]


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _stale(src: str, obj: str) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    deps = [src, os.path.join(ROOT, "include", "lyth_b200.h")]
    deps += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")]
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if not _stale(src, obj):
        return obj
    cmd = [NVCC, *FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if not os.path.exists(OUT) or any(os.path.getmtime(o) > os.path.getmtime(OUT) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", OUT, *objs, "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
