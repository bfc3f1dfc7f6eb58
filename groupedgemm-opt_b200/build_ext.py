"""In-tree build of the two native libraries of grouped_gemm_opt.

1. ``grouped_gemm_opt/libggo_b200.so``: every CUDA kernel plus the C ABI of ``include/ggo.h``,
   compiled by nvcc for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``), CUDA runtime
   linked statically, no PyTorch dependency.
2. ``grouped_gemm_opt/_C*.so``: the thin PyTorch binding (``csrc/torch_ext.cpp``), compiled by g++
   against torch's headers and linked to ``libggo_b200.so`` through an ``$ORIGIN`` rpath.

Replaces the reference's setup.py CUDAExtension (setup.py:40-74), which targeted sm_90a only.
Usage: ``python build_ext.py [--force]``. Outputs are rebuilt only when a source is newer.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
PKG = HERE / "grouped_gemm_opt"
INCLUDE = HERE.parent / "include"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")

CU_SOURCES = ["ggo_gemm.cu", "ggo_moe.cu"]
CU_HEADERS = ["ggo_gemm.cuh", "ggo_gemm_pair.cuh", "ggo_gemm_wgrad.cuh", "ggo_ptx.cuh", "ggo_internal.h"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
LIB_NAME = "libggo_b200.so"


def _ext_suffix() -> str:
    return sysconfig.get_config_var("EXT_SUFFIX") or ".so"


def lib_path() -> Path:
    return PKG / LIB_NAME


def torch_ext_path() -> Path:
    return PKG / ("_C" + _ext_suffix())


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_cuda_lib(force: bool = False) -> Path:
    out = lib_path()
    deps = [CSRC / s for s in CU_SOURCES + CU_HEADERS] + [INCLUDE / "ggo.h"]
    if not force and not _stale(out, deps):
        return out
    objdir = HERE / "_build"
    objdir.mkdir(exist_ok=True)
    objs = []
    for src in CU_SOURCES:
        obj = objdir / (Path(src).stem + ".o")
        _run([NVCC, "-std=c++17", "-O3", *ARCH_FLAGS, "-lineinfo", "-Xcompiler", "-fPIC",
              "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(CSRC / src), "-o", str(obj)])
        objs.append(str(obj))
    _run([NVCC, "-shared", *ARCH_FLAGS, "-cudart", "static", "-o", str(out), *objs])
    return out


def build_torch_ext(force: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    out = torch_ext_path()
    deps = [CSRC / "torch_ext.cpp", INCLUDE / "ggo.h", lib_path()]
    if not force and not _stale(out, deps):
        return out
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = cpp_extension.include_paths() + [str(CUDA_HOME / "include"), str(INCLUDE),
                                            sysconfig.get_paths()["include"]]
    libdirs = cpp_extension.library_paths() + [str(PKG)]
    cmd = ["g++", "-shared", "-fPIC", "-O2", "-std=c++17", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{i}" for i in incs], str(CSRC / "torch_ext.cpp"), "-o", str(out),
           *[f"-L{d}" for d in libdirs], "-lggo_b200", "-lc10", "-lc10_cuda", "-ltorch",
           "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python", "-Wl,-rpath,$ORIGIN"]
    _run(cmd)
    return out


def build(force: bool = False) -> None:
    build_cuda_lib(force)
    build_torch_ext(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
