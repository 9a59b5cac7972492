"""In-tree build of the two native artefacts of consumer_deep_gemm.

* ``consumer_deep_gemm/libcdg_b200.so`` -- the CUDA library behind the C ABI of
  ``include/cdg_b200.h``, compiled by nvcc for sm_100a only;
* ``consumer_deep_gemm/_C<ext-suffix>`` -- the PyTorch binding (pybind11),
  linked against the library with an ``$ORIGIN`` rpath.

Both land next to the Python sources so that they travel with the source tree
and are what ``import consumer_deep_gemm`` loads.  Run ``python build.py`` (or
``build()`` from Python); a target is rebuilt only when a source is newer.
"""

from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
PKG = os.path.join(HERE, "consumer_deep_gemm")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]

LIB = os.path.join(PKG, "libcdg_b200.so")
EXT = os.path.join(PKG, "_C" + sysconfig.get_config_var("EXT_SUFFIX"))

LIB_SOURCES = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".h")))
LIB_SOURCES.append(os.path.join(INCLUDE, "cdg_b200.h"))
EXT_SOURCES = [os.path.join(CSRC, "torch_ext.cpp"), os.path.join(INCLUDE, "cdg_b200.h")]


def _stale(target: str, sources) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _run(cmd):
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_lib(force: bool = False, extra=()) -> str:
    if force or _stale(LIB, LIB_SOURCES):
        _run([NVCC, *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
              "-cudart", "shared", "-Xptxas", "-v", "-I", INCLUDE, "-I", CSRC,
              "-o", LIB, os.path.join(CSRC, "cdg_abi.cu"), os.path.join(CSRC, "cdg_moe.cu"), *extra])
    return LIB


def build_ext(force: bool = False) -> str:
    build_lib(force)
    if not (force or _stale(EXT, EXT_SOURCES + [LIB])):
        return EXT
    import torch
    from torch.utils import cpp_extension

    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    inc = cpp_extension.include_paths() + [sysconfig.get_paths()["include"], os.path.join(CUDA_HOME, "include"),
                                           INCLUDE]
    libdir = cpp_extension.library_paths()[0]
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H", "-w"]
    cmd += [f"-I{p}" for p in inc]
    cmd += [os.path.join(CSRC, "torch_ext.cpp"), "-o", EXT, f"-L{libdir}", f"-L{PKG}",
            "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda", "-lcdg_b200",
            f"-Wl,-rpath,$ORIGIN:{libdir}"]
    _run(cmd)
    return EXT


def build(force: bool = False) -> None:
    build_ext(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
