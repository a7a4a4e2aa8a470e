"""Build liblonnx_cuda.so in-tree with nvcc for sm_100a (B200).

    python -m onnx_b200.build [--jobs N] [--force]

Compiles every onnx_b200/csrc/*.cu and *.cpp into onnx_b200/_build/*.o and
links onnx_b200/liblonnx_cuda.so (CUDA runtime linked statically, so the
library only needs the driver at run time).  nvcc cross-compiles, so this
runs on a machine without a GPU.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "liblonnx_cuda.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
                     "-Xcompiler", "-fPIC,-fvisibility=hidden,-O3", f"-I{INCLUDE}"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _deps():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _compile(src: str, force: bool, extra) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    newest_dep = max([os.path.getmtime(src)] + [os.path.getmtime(d) for d in _deps()])
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= newest_dep:
        return obj
    cmd = [nvcc()] + NVCC_FLAGS + list(extra) + ["-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [nvcc(), "-x", "cu"] + cmd[1:]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, jobs: int = 8, extra=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, extra), srcs))
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(o) for o in objs):
        return LIB
    cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-cudart", "static", "-lpthread", "-ldl", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def ptxas_report(src_name: str) -> str:
    """Registers / spills / shared memory per kernel (-Xptxas -v) of one source."""
    src = os.path.join(CSRC, src_name)
    cmd = [nvcc()] + NVCC_FLAGS + ["-Xptxas", "-v", "-c", src, "-o", os.devnull]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return r.stdout + r.stderr


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("--ptxas", default=None, help="print -Xptxas -v for one source file")
    a = ap.parse_args()
    if a.ptxas:
        print(ptxas_report(a.ptxas))
    else:
        print(build(a.force, a.jobs))
