"""Build the two native libraries of blockfp8_b200, in-tree, for sm_100a.

    python -m blockfp8_b200.build        (or __graft_entry__.build())

  libblockfp8_b200.so  the kernels and the C ABI (include/blockfp8_b200.h):
                       nvcc -gencode arch=compute_100a,code=sm_100a, static
                       CUDA runtime, no torch dependency
  _C.so                the torch.ops.blockfp8 operator library (csrc/ops.cpp),
                       linked against libblockfp8_b200.so through $ORIGIN

Both land next to this file, so they travel with the source tree.  Each is
rebuilt only when a source is newer than it (force=True rebuilds).
"""

import glob
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
CAPI_LIB = os.path.join(HERE, "libblockfp8_b200.so")
OPS_LIB = os.path.join(HERE, "_C.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CUDA_HOME = os.path.dirname(os.path.dirname(NVCC))

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _stale(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _run(cmd: list[str]) -> None:
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_capi(force: bool = False, verbose_ptxas: bool = False) -> str:
    sources = glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(CSRC, "*.inc")) + [os.path.join(INCLUDE, "blockfp8_b200.h")]
    if not force and not _stale(CAPI_LIB, sources):
        return CAPI_LIB
    cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           "-cudart", "static", f"-I{INCLUDE}", f"-I{CSRC}", "-o", CAPI_LIB + ".tmp",
           os.path.join(CSRC, "capi.cu")]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    _run(cmd)
    os.replace(CAPI_LIB + ".tmp", CAPI_LIB)
    return CAPI_LIB


def build_ops(force: bool = False) -> str:
    src = os.path.join(CSRC, "ops.cpp")
    if not force and not _stale(OPS_LIB, [src, CAPI_LIB, os.path.join(INCLUDE, "blockfp8_b200.h")]):
        return OPS_LIB
    import torch
    from torch.utils import cpp_extension

    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = cpp_extension.include_paths() + [os.path.join(CUDA_HOME, "include"), INCLUDE]
    libdirs = cpp_extension.library_paths()
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=_C",
           *[f"-I{i}" for i in incs], f"-I{sysconfig.get_paths()['include']}",
           "-o", OPS_LIB + ".tmp", src,
           *[f"-L{d}" for d in libdirs], f"-L{HERE}", "-lblockfp8_b200",
           "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch",
           "-Wl,-rpath,$ORIGIN", *[f"-Wl,-rpath,{d}" for d in libdirs]]
    _run(cmd)
    os.replace(OPS_LIB + ".tmp", OPS_LIB)
    return OPS_LIB


def build(force: bool = False) -> None:
    build_capi(force)
    build_ops(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
