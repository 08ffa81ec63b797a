"""CPU-side checks of the drop-in boundary: the C-ABI library loads and
exports every function include/pmkl_b200.h declares, argument errors are
reported before any device work, the C++ shim compiles, and the torch binding
imports and rejects CPU tensors.  No kernel runs here."""
import re
import subprocess
from pathlib import Path

import pytest
import torch

import pmkl_b200

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "pmkl_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(pmkl_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    for n in ("pmkl_causal_attention_fwd", "pmkl_warp_softmax_fwd", "pmkl_status_string"):
        assert n in names


def test_library_exports_every_declared_symbol():
    L = pmkl_b200.capi()
    for name in declared_functions():
        assert hasattr(L, name), f"{name} declared in pmkl_b200.h but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", str(pmkl_b200.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (pmkl_\w+)", out))
    assert set(declared_functions()) <= exported


def test_version_and_status_strings():
    L = pmkl_b200.capi()
    assert L.pmkl_version() == 100
    assert L.pmkl_status_string(0) == b"PMKL_OK"
    for code in range(-1, -10, -1):
        assert L.pmkl_status_string(code).startswith(b"PMKL_ERR_")
    assert L.pmkl_status_string(-99) == b"PMKL_ERR_UNKNOWN"


# Argument errors are detected on the host before the device is touched, so
# these calls are valid without a GPU (pointers are never dereferenced).
FAKE = 0x10000  # non-null, 16-byte aligned, never dereferenced


def attn(L, B=1, H=1, S=8, D=64, dtype=2, out_dtype=2, kernel=0, ptrs=FAKE):
    return L.pmkl_causal_attention_fwd_ex(ptrs, ptrs, ptrs, ptrs, ptrs, ptrs, B, H, S, D, dtype, out_dtype, 1, 0.0,
                                          kernel, None)


def test_attention_argument_errors():
    L = pmkl_b200.capi()
    assert attn(L, B=-1) == -1
    assert attn(L, S=-5) == -1
    assert attn(L, dtype=7) == -2
    assert attn(L, dtype=1, out_dtype=2) == -2  # out dtype must be the input dtype or fp32
    assert attn(L, kernel=9) == -5
    assert attn(L, D=257) == -5
    assert attn(L, ptrs=0) == -3


def test_attention_empty_problem_is_ok_without_device():
    L = pmkl_b200.capi()
    assert attn(L, B=0, ptrs=0) == 0
    assert attn(L, S=0, ptrs=0) == 0
    assert attn(L, H=0, ptrs=0) == 0


def bwd(L, B=1, H=1, S=8, D=64, dtype=2, kernel=0, ptrs=FAKE, ws=0x100000, ws_bytes=1 << 30):
    return L.pmkl_causal_attention_bwd_ex(*([ptrs] * 9), B, H, S, D, dtype, 1, 0.0, ws, ws_bytes, kernel, None)


def test_backward_argument_errors():
    L = pmkl_b200.capi()
    assert bwd(L, B=-1) == -1
    assert bwd(L, dtype=7) == -2
    assert bwd(L, kernel=9) == -5
    assert bwd(L, kernel=4) == -5  # no such backward choice
    assert bwd(L, D=300) == -5
    assert bwd(L, ptrs=0) == -3
    assert bwd(L, ws=0) == -3
    assert bwd(L, ws=0x100010) == -4  # workspace must be 256-byte aligned
    assert bwd(L, B=0, ptrs=0, ws=0) == 0  # empty: nothing to do
    assert bwd(L, S=0, ptrs=0, ws=0) == 0


def test_backward_workspace_size():
    """Tensor-core path: the automatic (fused) route needs the (b, delta) pairs
    only, at a row pitch of seq rounded up to 128; the long route
    (PMKL_ATTN_TCGEN05_SIMPLE) adds the forward's fp32 O, m, l, each region
    256-byte aligned.  The CUDA-core path needs one fp32 delta per row."""
    L = pmkl_b200.capi()
    f = L.pmkl_causal_attention_bwd_workspace_size
    fx = L.pmkl_causal_attention_bwd_workspace_size_ex
    a = lambda x: (x + 255) // 256 * 256  # noqa: E731
    B, H, S, D = 2, 3, 200, 128
    BH = B * H
    fused = a(BH * 256 * 8)
    assert f(B, H, S, D, 2) == fused
    assert fx(B, H, S, D, 2, 0) == fused and fx(B, H, S, D, 2, 2) == fused
    assert fx(B, H, S, D, 2, 3) == fused + a(BH * S * D * 4) + 2 * a(BH * S * 4)
    assert fx(B, H, S, 64, 1, 3) == fused + a(BH * S * 64 * 4) + 2 * a(BH * S * 4)
    assert fx(B, H, S, D, 2, 1) == a(BH * S * 4)  # CUDA-core route
    assert fx(B, H, S, D, 2, 9) == 0  # unknown choice
    assert f(B, H, S, 96, 2) == a(BH * S * 4)  # no tensor-core path for D = 96
    assert f(B, H, S, D, 0) == a(BH * S * 4)  # fp32
    assert f(0, H, S, D, 2) == 0 and f(B, H, 0, D, 2) == 0 and f(B, H, S, D, 9) == 0
    # config 3 (bf16 B16 H32 S4096 D128): 16 MiB, within the static scratch
    assert f(16, 32, 4096, 128, 2) == 16 << 20
    assert f(16, 32, 4096, 128, 2) <= 64 << 20


def test_static_scratch_limit_sizes():
    """The sizes the no-allocation backward's 64 MiB scratch admits on the
    tensor-core route: 2048 slices of 4096 rows fit exactly, 2049 do not (the
    GPU test of that entry point uses both)."""
    L = pmkl_b200.capi()
    f = L.pmkl_causal_attention_bwd_workspace_size
    assert f(1, 2048, 4096, 64, 2) == 64 << 20
    assert f(1, 2049, 4096, 64, 2) > 64 << 20


def test_wait_selftest_argument_errors():
    L = pmkl_b200.capi()
    f = L.pmkl_wait_selftest
    assert f(0, 5_000_000, 0x10000, None) == -1  # no CTA
    assert f(2, 10, 0x10000, None) == -1  # limit below 100 us
    assert f(2, 3_000_000_000, 0x10000, None) == -1  # limit above the 2 s every kernel uses
    assert f(2, 5_000_000, 0, None) == -3
    assert f(2, 5_000_000, 0x10004, None) == -4


def test_strided_argument_errors():
    import ctypes
    L = pmkl_b200.capi()
    s = (ctypes.c_int64 * 3)(64 * 8 * 128, 128, 8 * 128)
    neg = (ctypes.c_int64 * 3)(1, -1, 1)

    def f(heads=8, kv=2, st=s, B=1, S=64):
        return L.pmkl_causal_attention_fwd_strided(*([FAKE] * 6), B, heads, kv, S, 128, st, st, st, st, 2, 2, 1, 0.0,
                                                   0, None)

    assert f(kv=3) == -1  # kv_heads must divide heads
    assert f(kv=0) == -1
    assert f(kv=16) == -1
    assert f(st=neg) == -1
    assert f(B=0) == 0 and f(S=0) == 0  # empty problems: nothing to do


def test_softmax_argument_errors():
    L = pmkl_b200.capi()
    f = L.pmkl_warp_softmax_fwd
    assert f(FAKE, FAKE, 1025, 1025, 4, 0, 0, 0, None) == -1  # warp_softmax.h:162
    assert f(FAKE, FAKE, -1, 8, 4, 0, 0, 0, None) == -1
    assert f(FAKE, FAKE, 16, 8, 4, 0, 0, 0, None) == -1  # stride < elements
    assert f(FAKE, FAKE, 16, 16, -1, 0, 0, 0, None) == -1
    assert f(FAKE, FAKE, 16, 16, 4, 5, 0, 0, None) == -2
    assert f(0, 0, 0, 0, 4, 0, 0, 0, None) == 0  # elements == 0: nothing to do
    assert f(0, 0, 16, 16, 0, 0, 0, 0, None) == 0
    assert f(0, FAKE, 16, 16, 4, 0, 0, 0, None) == -3


def test_cpp_shim_compiles():
    import torch.utils.cpp_extension as cpp

    cuda_inc = Path(cpp.CUDA_HOME or "/usr/local/cuda") / "include"
    subprocess.run(["g++", "-std=c++17", "-fsyntax-only", f"-I{REPO / 'include'}", f"-I{cuda_inc}",
                    str(REPO / "tests" / "cpp" / "shim_test.cpp")], check=True)


def test_torch_binding_imports_and_rejects_cpu():
    import pmkl_pytorch_ext
    from pmkl_function import fused_self_attention

    q = torch.randn(1, 2, 8, 64)
    with pytest.raises(NotImplementedError):
        fused_self_attention(q, q, q, True)
    with pytest.raises(RuntimeError, match="CUDA"):
        pmkl_pytorch_ext.fused_self_attention_fw(q, q, q, True)
    with pytest.raises(RuntimeError, match="shapes must match"):
        pmkl_pytorch_ext.fused_self_attention_fw(q, q[:, :1], q, True)
    with pytest.raises(RuntimeError, match="shapes must match"):
        pmkl_pytorch_ext.fused_self_attention_fw(q[0], q[0], q[0], True)
    assert pmkl_pytorch_ext.KERNEL_TCGEN05 == pmkl_b200.KERNEL_TCGEN05
