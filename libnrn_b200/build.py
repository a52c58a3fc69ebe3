"""Builds the device layer, libnrn_b200/_lib/libnrn_cuda.so, with nvcc for
sm_100a (B200).  The library is built in-tree so it travels with the
repository snapshot.

    python -m libnrn_b200.build [--force]

Kernels are compiled with -fmad=false: the neuron updates, drive samplers and
STDP restate the reference's per-operation fp32 rounding, which a fused
multiply-add would change.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "_lib")
OBJ = os.path.join(OUT, "obj")
LIB = os.path.join(OUT, "libnrn_cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-fmad=false", "-cudart=shared", "-Xcompiler", "-fPIC", "-Xcompiler",
         "-fvisibility=hidden", f"-I{os.path.join(ROOT, 'include')}", f"-I{CSRC}"]
SOURCES = ["neuron.cu", "deliver.cu", "connect.cu", "engine.cu"]


def _headers():
    hs = [os.path.join(ROOT, "include", "nrn_cuda.h")]
    hs += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    return hs


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, extra=()):
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    if _stale(obj, [src] + _headers()):
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr[-6000:]}")
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    if force:
        for f in os.listdir(OBJ):
            os.remove(os.path.join(OBJ, f))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(_compile, srcs))
    if _stale(LIB, objs):
        # one CUDA runtime per process: link the shared runtime (in a torch
        # process the runtime torch loaded is reused)
        cmd = [NVCC, *ARCH, "-shared", "-cudart=shared", "-o", LIB, *objs, "-Xlinker", "--no-undefined",
               "-Xlinker", "-rpath,/usr/local/cuda/lib64"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr[-4000:]}")
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
