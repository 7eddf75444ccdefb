"""Build ``libqlin.so`` (the C-ABI CUDA library) in-tree for sm_100a, and the
torch-tensor Python binding ``_qlin_ext`` on top of it.

    python -m <package>.build          # or __graft_entry__.build()

The library is self-contained (static CUDA runtime, no torch dependency), so
any language can bind ``include/qlin.h`` against it.  ``_qlin_ext`` (host C++
only, linked to ``libqlin.so`` through ``$ORIGIN``) is what the package's
Python entry points call.
"""
import glob
import os
import shutil
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libqlin.so")
EXT = os.path.join(HERE, "_qlin_ext" + sysconfig.get_config_var("EXT_SUFFIX"))
EXT_SRC = os.path.join(CSRC, "pyext.cpp")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def nvcc():
    exe = shutil.which("nvcc")
    if exe is None and os.path.exists("/usr/local/cuda/bin/nvcc"):
        exe = "/usr/local/cuda/bin/nvcc"
    if exe is None:
        raise RuntimeError("nvcc not found")
    return exe


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + [os.path.join(ROOT, "include", "qlin.h")])


def newer_than(target, deps):
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(s) <= t for s in deps)


def up_to_date():
    return newer_than(LIB, sources())


def build(force=False, verbose=False):
    """Compile csrc/*.cu into libqlin.so and csrc/pyext.cpp into the Python
    binding, each unless it is newer than every source."""
    if force or not up_to_date():
        build_lib(verbose)
    if force or not newer_than(EXT, [EXT_SRC, LIB, os.path.join(ROOT, "include", "qlin.h")]):
        build_ext(verbose)
    return LIB


def build_lib(verbose=False):
    cmd = [nvcc(), *NVCC_FLAGS, "-o", LIB + ".tmp", os.path.join(CSRC, "api.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, cwd=HERE, capture_output=not verbose, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    os.replace(LIB + ".tmp", LIB)
    return LIB


def build_ext(verbose=False):
    """g++ the pybind11 module against torch's headers and libqlin.so."""
    import torch
    tdir = os.path.dirname(os.path.abspath(torch.__file__))
    tlib = os.path.join(tdir, "lib")
    cuda_inc = os.path.join(os.path.dirname(os.path.dirname(nvcc())), "include")
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        raise RuntimeError("g++ not found")
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(tdir, "include"),
           "-I", os.path.join(tdir, "include", "torch", "csrc", "api", "include"),
           "-I", cuda_inc, "-I", sysconfig.get_paths()["include"],
           EXT_SRC, "-o", EXT + ".tmp",
           "-L", HERE, "-l:libqlin.so", "-L", tlib, "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
           "-ltorch_python", "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + tlib]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, cwd=HERE, capture_output=not verbose, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"g++ failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    os.replace(EXT + ".tmp", EXT)
    return EXT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
