"""Compile the engine's CUDA sources into the in-tree shared library.

    python per_b200/build.py          # from triton-per_b200/ (the package
                                      # itself cannot be imported before the
                                      # library exists)

Produces per_b200/libper_b200.so for sm_100a (B200) only; the CUDA runtime is
linked statically so the library loads on hosts without a driver (its entry
points then report PER_ERR_CUDA).
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)                      # triton-per_b200/
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB = os.path.join(PKG, "libper_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
    "-shared", "-cudart", "static",
]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _inputs() -> list[str]:
    return (sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
            + glob.glob(os.path.join(INCLUDE, "*.h")))


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in _inputs())


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the engine is CUDA-only and must be compiled for sm_100a")


def build(force: bool = False, verbose: bool = False) -> str:
    if force or needs_build():
        tmp = LIB + ".tmp"
        cmd = [nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-o", tmp, *sources()]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB)
    build_binding(force=force, verbose=verbose)
    return LIB


# ---- the torch-tensor binding (csrc/per_torch.cpp -> per_b200/_per_torch*.so):
# a C++ extension linked against libper_b200.so (found next to it at run time)
BINDING_SRC = os.path.join(CSRC, "per_torch.cpp")


def binding_path() -> str:
    import sysconfig

    return os.path.join(PKG, "_per_torch" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_binding(force: bool = False, verbose: bool = False) -> str:
    import sysconfig

    import torch
    import torch.utils.cpp_extension as ext

    out = binding_path()
    deps = [BINDING_SRC, LIB, os.path.join(INCLUDE, "per_b200.h")]
    if not force and os.path.exists(out) and all(os.path.getmtime(d) <= os.path.getmtime(out)
                                                 for d in deps):
        return out
    cuda_home = ext.CUDA_HOME or "/usr/local/cuda"
    incs = [os.path.join(os.path.dirname(torch.__file__), "include"),
            os.path.join(os.path.dirname(torch.__file__), "include", "torch", "csrc", "api",
                         "include"),
            os.path.join(cuda_home, "include"), sysconfig.get_paths()["include"], INCLUDE]
    libdir = os.path.join(os.path.dirname(torch.__file__), "lib")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-w",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_per_torch",
           "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{i}" for i in incs], BINDING_SRC, "-o", out + ".tmp",
           f"-L{libdir}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
           "-ltorch_python", f"-Wl,-rpath,{libdir}",
           f"-L{PKG}", "-lper_b200", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(out + ".tmp", out)
    return out


if __name__ == "__main__":
    print(build(force=True, verbose=True))
