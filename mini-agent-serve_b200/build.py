"""Build recipe for the two native libraries of the package, written next to this file (in-tree).

libmas_b200.so        the sm_100a kernels behind the C ABI of include/mas_b200.h: one translation unit
                      (csrc/mas_b200.cu) compiled by nvcc straight to sm_100a SASS, static CUDA runtime,
                      no torch dependency (it loads without a GPU; calls then return MAS_ERR_NO_DEVICE).
libmas_b200_torch.so  the `mas_b200::*` PyTorch operators (csrc/torch_ops.cpp), compiled by the host
                      C++ compiler against torch's headers and linked to libmas_b200.so.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR.parent / "include"
LIB_NAME = "libmas_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME
TORCH_LIB_PATH = PKG_DIR / "libmas_b200_torch.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-shared",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "-Xlinker", f"-soname={LIB_NAME}",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit's bin on PATH")


def _cxx() -> str:
    for cand in (os.environ.get("CXX"), "/usr/bin/g++", shutil.which("g++"), shutil.which("c++")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("no C++ compiler found: set CXX")


def cuda_sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "mas_b200.h"]


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(p.stat().st_mtime > t for p in deps)


def needs_build() -> bool:
    return _stale(LIB_PATH, cuda_sources()) or _stale(TORCH_LIB_PATH, [CSRC / "torch_ops.cpp", INCLUDE / "mas_b200.h", LIB_PATH])


def build_kernels(force: bool = False, verbose: bool = False) -> Path:
    """nvcc csrc/mas_b200.cu -> libmas_b200.so (sm_100a)."""
    if not force and not _stale(LIB_PATH, cuda_sources()):
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", str(tmp), str(CSRC / "mas_b200.cu")]
    if verbose:
        cmd[1:1] = ["-Xptxas", "-v"]
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def build_torch_ops(force: bool = False, verbose: bool = False) -> Path:
    """c++ csrc/torch_ops.cpp -> libmas_b200_torch.so (links libmas_b200.so through $ORIGIN)."""
    if not force and not _stale(TORCH_LIB_PATH, [CSRC / "torch_ops.cpp", INCLUDE / "mas_b200.h", LIB_PATH]):
        return TORCH_LIB_PATH
    import torch
    from torch.utils import cpp_extension as ce

    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = [f"-I{p}" for p in ce.include_paths(device_type="cuda")]
    libdirs = ce.library_paths(device_type="cuda")
    torch_lib = str(Path(torch.__file__).resolve().parent / "lib")
    tmp = TORCH_LIB_PATH.with_suffix(".so.tmp")
    cmd = [_cxx(), "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}", *incs,
           str(CSRC / "torch_ops.cpp"), "-o", str(tmp),
           *[f"-L{d}" for d in libdirs], f"-L{PKG_DIR}",
           "-lmas_b200", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, TORCH_LIB_PATH)
    return TORCH_LIB_PATH


def build(force: bool = False, verbose: bool = False) -> Path:
    """Both libraries, each rebuilt only when its sources changed (or `force`)."""
    build_kernels(force, verbose)
    build_torch_ops(force, verbose)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB_PATH)
    print(TORCH_LIB_PATH)
