"""Build steps for the native parts of pmkl_b200.

* ``libpmkl_b200.so`` -- the CUDA kernels and the C ABI of
  ``include/pmkl_b200.h``, compiled by nvcc for sm_100a only
  (``-gencode arch=compute_100a,code=sm_100a``) into ``pmkl_b200/lib/``.
* ``pmkl_pytorch_ext`` -- the torch binding (``torch_ext/fused_self_attention.cpp``),
  compiled with torch's extension builder into ``pmkl_b200/torch_ext/_build/``
  and linked against ``libpmkl_b200.so`` through an ``$ORIGIN`` rpath.

Both land inside the source tree so that they travel with it; nothing is
installed into site-packages.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
LIB_DIR = PKG / "lib"
LIB_PATH = LIB_DIR / "libpmkl_b200.so"
EXT_SRC_DIR = PKG / "torch_ext"
EXT_BUILD_DIR = EXT_SRC_DIR / "_build"
EXT_NAME = "pmkl_pytorch_ext"

NVCC_ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    return str(cand) if cand.is_file() else "nvcc"


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _newest_input_mtime() -> float:
    files = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max(f.stat().st_mtime for f in files)


def build_lib(force: bool = False, verbose: bool = False) -> Path:
    """Compile every .cu under csrc/ into one shared library for sm_100a."""
    if LIB_PATH.is_file() and not force and LIB_PATH.stat().st_mtime >= _newest_input_mtime():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [
        _nvcc(), *NVCC_ARCH, "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC", "-shared",
        "-I", str(INCLUDE), "-I", str(CSRC),
        *[str(s) for s in _sources()],
        "-o", str(tmp),
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def build_ext(force: bool = False, verbose: bool = False) -> Path:
    """Compile the torch binding in-tree with one g++ command (no shell, so
    the ``$ORIGIN`` rpath reaches the linker verbatim) and return its path."""
    import sysconfig

    import torch
    import torch.utils.cpp_extension as cpp

    build_lib(verbose=verbose)
    EXT_BUILD_DIR.mkdir(parents=True, exist_ok=True)
    so = EXT_BUILD_DIR / f"{EXT_NAME}.so"
    src = EXT_SRC_DIR / "fused_self_attention.cpp"
    newest = max(src.stat().st_mtime, (INCLUDE / "pmkl_b200.h").stat().st_mtime, LIB_PATH.stat().st_mtime)
    if so.is_file() and not force and so.stat().st_mtime >= newest:
        return so
    cuda_home = Path(cpp.CUDA_HOME or "/usr/local/cuda")
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = so.with_suffix(".so.tmp")
    cmd = [
        "g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-w",
        f"-DTORCH_EXTENSION_NAME={EXT_NAME}", "-DTORCH_API_INCLUDE_EXTENSION_H",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        *[f"-I{p}" for p in cpp.include_paths()],
        f"-I{sysconfig.get_paths()['include']}", f"-I{cuda_home / 'include'}", f"-I{INCLUDE}",
        str(src),
        f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_python",
        f"-L{LIB_DIR}", "-lpmkl_b200", "-Wl,-rpath,$ORIGIN/../../lib",
        "-o", str(tmp),
    ]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, so)
    return so


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_lib(force=force, verbose=verbose)
    build_ext(force=force, verbose=verbose)


if __name__ == "__main__":
    build_all(force="-f" in sys.argv, verbose="-v" in sys.argv)
    print("built", LIB_PATH, "and", EXT_NAME)
