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
SOURCES = ["neuron.cu", "deliver.cu", "connect.cu", "engine.cu", "comm.cu", "blockdense.cu", "raster_noalloc.cu", "plastic.cu",
           "exchange.cu", "bsr.cu"]


def _nccl_dir():
    """NCCL of the installed PyTorch wheel (the library torch.distributed
    loads, so one NCCL per process)."""
    import importlib.util
    spec = importlib.util.find_spec("nvidia")
    for base in (spec.submodule_search_locations or []) if spec else []:
        d = os.path.join(base, "nccl")
        if os.path.exists(os.path.join(d, "include", "nccl.h")):
            return d
    raise RuntimeError("NCCL headers not found (nvidia-nccl wheel)")


NCCL = _nccl_dir()
FLAGS.append(f"-I{os.path.join(NCCL, 'include')}")


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


CPP_SOURCES = ["neuron.cpp", "synapse.cpp", "connectivity.cpp", "plasticity.cpp", "monitor.cpp",
               "simulation.cpp", "config.cpp"]
CPP_LIB = os.path.join(OUT, "libnrn.so")


def _torch_dirs():
    import torch  # the LibTorch headers and libraries of the installed wheel
    base = os.path.dirname(torch.__file__)
    return os.path.join(base, "include"), os.path.join(base, "lib")


def _cpp_headers():
    hs = []
    for d, _, fs in os.walk(os.path.join(ROOT, "include")):
        hs += [os.path.join(d, f) for f in fs if f.endswith(".h")]
    cpp = os.path.join(HERE, "cpp")
    hs += [os.path.join(cpp, f) for f in os.listdir(cpp) if f.endswith(".h")]
    return hs


def _compile_cpp(src):
    inc, _ = _torch_dirs()
    obj = os.path.join(OBJ, "cpp_" + os.path.basename(src) + ".o")
    if _stale(obj, [src] + _cpp_headers()):
        cmd = [os.environ.get("CXX", "g++"), "-std=c++20", "-O2", "-fPIC", "-D_GLIBCXX_USE_CXX11_ABI=1",
               f"-I{os.path.join(ROOT, 'include')}", f"-I{inc}", f"-I{os.path.join(inc, 'torch/csrc/api/include')}",
               "-I/usr/local/cuda/include", "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"g++ failed on {src}:\n{r.stderr[-6000:]}")
    return obj


def build_cpp(verbose: bool = False) -> str:
    """Builds libnrn.so, the nrn:: C++ API (links LibTorch and libnrn_cuda.so)."""
    build()
    _, tlib = _torch_dirs()
    srcs = [os.path.join(HERE, "cpp", s) for s in CPP_SOURCES]
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(_compile_cpp, srcs))
    if _stale(CPP_LIB, objs + [LIB]):
        cmd = [os.environ.get("CXX", "g++"), "-shared", "-o", CPP_LIB, *objs, f"-L{OUT}", "-lnrn_cuda",
               f"-L{tlib}", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-lc10", "-lc10_cuda",
               "-L/usr/local/cuda/lib64", "-lcudart", f"-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{tlib}",
               "-Wl,-rpath,/usr/local/cuda/lib64"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link of libnrn.so failed:\n{r.stderr[-4000:]}")
    if verbose:
        print(CPP_LIB)
    return CPP_LIB


CPP_TESTS = ["test_core", "test_gpu_api", "dropin_brunel", "er_dump", "api_bench"]
TEST_DIR = os.path.join(ROOT, "tests", "cpp")
TEST_BIN = os.path.join(TEST_DIR, "_bin")


def build_cpp_tests(verbose: bool = False) -> dict:
    """Builds the C++ API test programs (tests/cpp/*.cpp) against libnrn.so."""
    lib = build_cpp()
    inc, tlib = _torch_dirs()
    os.makedirs(TEST_BIN, exist_ok=True)
    out = {}

    def one(name):
        src = os.path.join(TEST_DIR, name + ".cpp")
        exe = os.path.join(TEST_BIN, name)
        if _stale(exe, [src, os.path.join(TEST_DIR, "nrn_test.h"), lib] + _cpp_headers()):
            cmd = [os.environ.get("CXX", "g++"), "-std=c++20", "-O1", "-D_GLIBCXX_USE_CXX11_ABI=1",
                   f"-I{os.path.join(ROOT, 'include')}", f"-I{inc}", f"-I{os.path.join(inc, 'torch/csrc/api/include')}",
                   "-I/usr/local/cuda/include", src, "-o", exe, f"-L{OUT}", "-lnrn", "-lnrn_cuda", f"-L{tlib}",
                   "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-lc10", "-lc10_cuda", "-L/usr/local/cuda/lib64",
                   "-lcudart", f"-Wl,-rpath,{OUT}", f"-Wl,-rpath,{tlib}", "-Wl,-rpath,/usr/local/cuda/lib64"]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"build of {name} failed:\n{r.stderr[-6000:]}")
        return name, exe

    with cf.ThreadPoolExecutor(max_workers=3) as ex:
        for name, exe in ex.map(one, CPP_TESTS):
            out[name] = exe
    if verbose:
        print(TEST_BIN)
    return out


PROBE = os.path.join(OUT, "l2_probe")


def build_probe(verbose: bool = False) -> str:
    """The random-access throughput probe (csrc/l2_probe.cu), a standalone
    program run by bench.py --probe-l2."""
    os.makedirs(OUT, exist_ok=True)
    src = os.path.join(CSRC, "l2_probe.cu")
    if _stale(PROBE, [src]):
        r = subprocess.run([NVCC, *ARCH, "-O3", "-o", PROBE, src], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr[-4000:]}")
    if verbose:
        print(PROBE)
    return PROBE


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
        nlib = os.path.join(NCCL, "lib")
        cmd = [NVCC, *ARCH, "-shared", "-cudart=shared", "-o", LIB, *objs, f"-L{nlib}", "-l:libnccl.so.2",
               "-Xlinker", "--no-undefined", "-Xlinker", "-rpath,/usr/local/cuda/lib64", "-Xlinker", f"-rpath,{nlib}"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr[-4000:]}")
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    if "--cpp" in sys.argv:
        build_cpp(verbose=True)
    if "--tests" in sys.argv:
        build_cpp_tests(verbose=True)
