"""Recipe that compiles the reference's own CPU code for this path into
``oracle/_ref/`` (git-ignored; it travels to GPU boxes with the rest of the
tree).  TEST INFRASTRUCTURE ONLY: the products are used to pin the oracle and
as the timed CPU baseline, never by the product path.

Two libraries, both built from the reference sources where they lie, unmodified:

* ``pmkl_ref_ext`` -- the reference torch extension
  ``pmkl_pytorch_ext/fused_self_attention.cpp`` (``fused_self_attention_fw`` /
  ``_bw``, CPU implementation ``pmkl_cpu::host_self_attention_forward`` at
  :5-64), compiled with torch's extension builder under another module name so
  that it cannot shadow the product's ``pmkl_pytorch_ext``.  The reference's own
  ``setup.py`` builds it as a ``CppExtension`` with Python's default ``-O2``;
  the same optimisation level is used here.
* ``libpmkl_ref_softmax.so`` -- ``test/test_softmax.cpp``'s
  ``host_softmax_forward`` (:10-28), compiled through ``ref_softmax_shim.cpp``
  with inert launcher stand-ins from ``ref_stubs/``; the test's GPU ``main`` is
  renamed and never runs.

The reference tree is located through ``PMKL_REFERENCE_DIR`` or, by default,
the ``reference`` directory beside this repository.  When it is absent (as on
GPU boxes) nothing is rebuilt and previously built products are used.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
REF_OUT = ORACLE_DIR / "_ref"
REF_EXT_NAME = "pmkl_ref_ext"
REF_SOFTMAX_LIB = REF_OUT / "libpmkl_ref_softmax.so"


def reference_dir() -> Path:
    env = os.environ.get("PMKL_REFERENCE_DIR")
    if env:
        return Path(env)
    return ORACLE_DIR.parent.parent / "reference"


def reference_available() -> bool:
    r = reference_dir()
    return (r / "pmkl_pytorch_ext" / "fused_self_attention.cpp").is_file() and (
        r / "test" / "test_softmax.cpp"
    ).is_file()


def ref_ext_path() -> Path:
    return REF_OUT / f"{REF_EXT_NAME}.so"


def build_ref_softmax(verbose: bool = False) -> Path:
    ref = reference_dir()
    REF_OUT.mkdir(parents=True, exist_ok=True)
    cmd = [
        "g++", "-O2", "-DNDEBUG", "-std=c++17", "-fPIC", "-shared",
        "-I", str(ORACLE_DIR / "ref_stubs"), "-I", str(ref / "test"),
        "-Dmain=pmkl_ref_softmax_test_main",
        str(ORACLE_DIR / "ref_softmax_shim.cpp"), "-o", str(REF_SOFTMAX_LIB),
    ]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return REF_SOFTMAX_LIB


def build_ref_ext(verbose: bool = False):
    import torch.utils.cpp_extension as cpp

    ref = reference_dir()
    REF_OUT.mkdir(parents=True, exist_ok=True)
    return cpp.load(
        name=REF_EXT_NAME,
        sources=[str(ref / "pmkl_pytorch_ext" / "fused_self_attention.cpp")],
        build_directory=str(REF_OUT),
        extra_cflags=["-O2", "-DNDEBUG"],
        with_cuda=False,
        verbose=verbose,
    )


def build(verbose: bool = False) -> bool:
    """Build both reference libraries when the reference tree is present.
    Returns True when they were (re)built, False when the tree is absent."""
    if not reference_available():
        return False
    build_ref_softmax(verbose)
    build_ref_ext(verbose)
    return True


def load_ref_ext():
    """Import the previously built reference extension (no rebuild)."""
    import importlib.machinery
    import importlib.util

    import torch  # noqa: F401  (the extension links against torch's libraries)

    path = ref_ext_path()
    if not path.is_file():
        raise FileNotFoundError(f"reference extension not built: {path}")
    if REF_EXT_NAME in sys.modules:
        return sys.modules[REF_EXT_NAME]
    loader = importlib.machinery.ExtensionFileLoader(REF_EXT_NAME, str(path))
    spec = importlib.util.spec_from_file_location(REF_EXT_NAME, str(path), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[REF_EXT_NAME] = mod
    return mod


def load_ref_softmax():
    import ctypes

    if not REF_SOFTMAX_LIB.is_file():
        raise FileNotFoundError(f"reference softmax not built: {REF_SOFTMAX_LIB}")
    lib = ctypes.CDLL(str(REF_SOFTMAX_LIB))
    fn = lib.pmkl_ref_host_softmax_forward_f32
    fn.restype = None
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    return fn


if __name__ == "__main__":
    ok = build(verbose="-v" in sys.argv)
    print("built oracle/_ref" if ok else "reference tree absent; nothing built")
