"""Build libh2cuda.so in-tree with nvcc for sm_100a (B200). No JIT cache: the .so lives next to this file.

Every csrc/*.cu file is one translation unit, compiled to an object in parallel and linked into one shared library.
"""
from __future__ import annotations

import glob
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
OUT = os.path.join(HERE, "libh2cuda.so")
OBJ_DIR = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = [*ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xptxas", "-warn-spills"]


def units():
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")))


def sources():
    return sorted(units() + glob.glob(os.path.join(HERE, "csrc", "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h")))


def _compile(cu: str) -> tuple:
    obj = os.path.join(OBJ_DIR, os.path.basename(cu)[:-3] + ".o")
    r = subprocess.run([NVCC, *CFLAGS, "-c", "-o", obj, cu], capture_output=True, text=True)
    return obj, r


def build(force: bool = False, verbose: bool = False) -> str:
    srcs = sources()
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= max(os.path.getmtime(s) for s in srcs):
        return OUT
    os.makedirs(OBJ_DIR, exist_ok=True)
    with ThreadPoolExecutor(max_workers=max(1, min(len(units()), os.cpu_count() or 1))) as ex:
        results = list(ex.map(_compile, units()))
    log = ""
    for obj, r in results:
        log += r.stdout + r.stderr
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(obj)}:\n" + r.stdout + r.stderr)
    r = subprocess.run([NVCC, *ARCH, "-shared", "-o", OUT + ".tmp", *[o for o, _ in results]], capture_output=True,
                       text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc link failed:\n" + r.stdout + r.stderr)
    if verbose and (log or r.stdout or r.stderr):
        print(log + r.stdout + r.stderr)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force=True, verbose=True))
