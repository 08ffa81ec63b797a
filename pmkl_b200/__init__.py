"""pmkl_b200 -- B200 (sm_100a) implementation of pmkl's fused causal
self-attention and warp-softmax path.

Layers, bottom up:

* ``libpmkl_b200.so`` (``csrc/``): the CUDA kernels behind the C ABI of
  ``include/pmkl_b200.h``;
* ``pmkl_pytorch_ext`` / ``pmkl_function`` (``torch_ext/``): the reference's
  torch extension and autograd wrapper, same names and signatures, calling the
  C ABI on the current CUDA stream;
* this module: locates the built artefacts, puts the torch binding on
  ``sys.path`` so that ``import pmkl_pytorch_ext`` and
  ``from pmkl_function import fused_self_attention`` work as they do with the
  reference installed, and offers a ctypes view of the C ABI (``capi()``).

The library must be built (``python -m pmkl_b200.build``); nothing here falls
back to another implementation when it is missing.
"""
from __future__ import annotations

import ctypes
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "lib" / "libpmkl_b200.so"
EXT_DIR = PKG_DIR / "torch_ext" / "_build"
FUNCTION_DIR = PKG_DIR / "torch_ext"

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
KERNEL_AUTO, KERNEL_SIMT, KERNEL_TCGEN05 = 0, 1, 2
PMKL_OK = 0

for _p in (EXT_DIR, FUNCTION_DIR):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

_capi = None


class PmklError(RuntimeError):
    """A pmkl_status other than PMKL_OK, raised by the ctypes helpers."""

    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what} failed: {capi().pmkl_status_string(status).decode()}")


def capi() -> ctypes.CDLL:
    """The C ABI (include/pmkl_b200.h) through ctypes.  Raises if the library
    has not been built: there is no fallback path."""
    global _capi
    if _capi is None:
        if not LIB_PATH.is_file():
            raise ImportError(f"libpmkl_b200.so is not built ({LIB_PATH}); run python -m pmkl_b200.build")
        L = ctypes.CDLL(str(LIB_PATH))
        vp, i32, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        L.pmkl_causal_attention_fwd.restype = i32
        L.pmkl_causal_attention_fwd.argtypes = [vp] * 6 + [i32] * 7 + [f32, vp]
        L.pmkl_causal_attention_fwd_ex.restype = i32
        L.pmkl_causal_attention_fwd_ex.argtypes = [vp] * 6 + [i32] * 7 + [f32, i32, vp]
        i64p = ctypes.POINTER(ctypes.c_int64)
        L.pmkl_causal_attention_fwd_strided.restype = i32
        L.pmkl_causal_attention_fwd_strided.argtypes = [vp] * 6 + [i32] * 5 + [i64p] * 4 + [i32] * 3 + [f32, i32, vp]
        L.pmkl_causal_attention_bwd.restype = i32
        L.pmkl_causal_attention_bwd.argtypes = [vp] * 9 + [i32] * 6 + [f32, vp, ctypes.c_size_t, vp]
        L.pmkl_causal_attention_bwd_ex.restype = i32
        L.pmkl_causal_attention_bwd_ex.argtypes = [vp] * 9 + [i32] * 6 + [f32, vp, ctypes.c_size_t, i32, vp]
        L.pmkl_causal_attention_bwd_strided.restype = i32
        L.pmkl_causal_attention_bwd_strided.argtypes = [vp] * 9 + [i32] * 5 + [i64p] * 7 + [i32] * 2 + [
            f32, vp, ctypes.c_size_t, i32, vp]
        L.pmkl_causal_attention_bwd_static.restype = i32
        L.pmkl_causal_attention_bwd_static.argtypes = [vp] * 9 + [i32] * 6 + [f32, vp]
        L.pmkl_causal_attention_bwd_workspace_size.restype = ctypes.c_size_t
        L.pmkl_causal_attention_bwd_workspace_size.argtypes = [i32] * 5
        L.pmkl_causal_attention_bwd_workspace_size_ex.restype = ctypes.c_size_t
        L.pmkl_causal_attention_bwd_workspace_size_ex.argtypes = [i32] * 6
        L.pmkl_warp_softmax_fwd.restype = i32
        L.pmkl_warp_softmax_fwd.argtypes = [vp, vp] + [i32] * 6 + [vp]
        L.pmkl_status_string.restype = ctypes.c_char_p
        L.pmkl_status_string.argtypes = [i32]
        L.pmkl_version.restype = i32
        L.pmkl_version.argtypes = []
        L.pmkl_stream_synchronize.restype = i32
        L.pmkl_stream_synchronize.argtypes = [vp]
        L.pmkl_device_error.restype = i32
        L.pmkl_device_error.argtypes = [i32]
        L.pmkl_wait_selftest.restype = i32
        L.pmkl_wait_selftest.argtypes = [i32, ctypes.c_ulonglong, vp, vp]
        L.pmkl_tc_selftest.restype = i32
        L.pmkl_tc_selftest.argtypes = [i32, vp, vp, vp, i32, i32, vp]
        L.pmkl_attention_selected_kernel.restype = i32
        L.pmkl_attention_selected_kernel.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32]
        _capi = L
    return _capi


def torch_dtype_code(dtype) -> int:
    import torch

    return {torch.float32: DTYPE_F32, torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16}[dtype]


def _stream_ptr(stream) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def attention_fwd(q, k, v, o, m, l, is_causal: bool, scale: float = 0.0, kernel: int = KERNEL_AUTO,
                  stream=None) -> None:
    """Calls pmkl_causal_attention_fwd_ex on caller-allocated torch CUDA
    tensors (q, k, v, o: [B, H, S, D]; m, l: [B, H, S]).  Raises PmklError."""
    B, H, S, D = q.shape
    rc = capi().pmkl_causal_attention_fwd_ex(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), m.data_ptr(), l.data_ptr(),
        B, H, S, D, torch_dtype_code(q.dtype), torch_dtype_code(o.dtype), int(bool(is_causal)), float(scale),
        int(kernel), _stream_ptr(stream))
    if rc != PMKL_OK:
        raise PmklError(rc, "pmkl_causal_attention_fwd")


def attention_fwd_strided(q, k, v, o, m, l, is_causal: bool, scale: float = 0.0, kernel: int = KERNEL_AUTO,
                          stream=None) -> None:
    """pmkl_causal_attention_fwd_strided on torch CUDA tensors of logical shape
    [B, H, S, D] (q, o) and [B, H_kv, S, D] (k, v) with any strides whose last
    dimension is contiguous; m, l contiguous [B, H, S]."""
    B, H, S, D = q.shape
    Hkv = k.shape[1]

    def st(t):
        assert t.stride(3) == 1, "the hidden dimension must be contiguous"
        return (ctypes.c_int64 * 3)(t.stride(0), t.stride(1), t.stride(2))

    rc = capi().pmkl_causal_attention_fwd_strided(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), m.data_ptr(), l.data_ptr(), B, H, Hkv, S, D,
        st(q), st(k), st(v), st(o), torch_dtype_code(q.dtype), torch_dtype_code(o.dtype), int(bool(is_causal)),
        float(scale), int(kernel), _stream_ptr(stream))
    if rc != PMKL_OK:
        raise PmklError(rc, "pmkl_causal_attention_fwd_strided")


def attention_bwd_workspace_size(B: int, H: int, S: int, D: int, dtype, kernel: int = KERNEL_AUTO) -> int:
    """Workspace bytes of the backward route that ``kernel`` selects."""
    return int(capi().pmkl_causal_attention_bwd_workspace_size_ex(B, H, S, D, torch_dtype_code(dtype), int(kernel)))


def attention_bwd(dout, q, k, v, m, l, dq, dk, dv, is_causal: bool, scale: float = 0.0, kernel: int = KERNEL_AUTO,
                  workspace=None, stream=None) -> None:
    """Calls pmkl_causal_attention_bwd_ex on caller-allocated torch CUDA tensors
    (dout, q, k, v, dq, dk, dv: [B, H, S, D]; m, l: [B, H, S], all one dtype).
    ``workspace`` is a uint8 CUDA tensor of at least attention_bwd_workspace_size
    bytes; one is allocated when it is None.  Raises PmklError."""
    import torch

    B, H, S, D = q.shape
    if workspace is None:
        workspace = torch.empty(max(attention_bwd_workspace_size(B, H, S, D, q.dtype, kernel), 1), dtype=torch.uint8,
                                device=q.device)
    rc = capi().pmkl_causal_attention_bwd_ex(
        dout.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), m.data_ptr(), l.data_ptr(), dq.data_ptr(),
        dk.data_ptr(), dv.data_ptr(), B, H, S, D, torch_dtype_code(q.dtype), int(bool(is_causal)), float(scale),
        workspace.data_ptr(), workspace.numel(), int(kernel), _stream_ptr(stream))
    if rc != PMKL_OK:
        raise PmklError(rc, "pmkl_causal_attention_bwd")


def attention_bwd_strided(dout, q, k, v, m, l, dq, dk, dv, is_causal: bool, scale: float = 0.0,
                          kernel: int = KERNEL_AUTO, workspace=None, stream=None) -> None:
    """pmkl_causal_attention_bwd_strided on torch CUDA tensors of logical shape
    [B, H, S, D] (dout, q, dq) and [B, H_kv, S, D] (k, v, dk, dv) with any
    strides whose last dimension is contiguous; m, l contiguous [B, H, S]."""
    import torch

    B, H, S, D = q.shape
    Hkv = k.shape[1]

    def st(t):
        assert t.stride(3) == 1 or t.shape[3] <= 1, "the hidden dimension must be contiguous"
        return (ctypes.c_int64 * 3)(t.stride(0), t.stride(1), t.stride(2))

    if workspace is None:
        workspace = torch.empty(max(attention_bwd_workspace_size(B, H, S, D, q.dtype, kernel), 1), dtype=torch.uint8,
                                device=q.device)
    rc = capi().pmkl_causal_attention_bwd_strided(
        dout.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), m.data_ptr(), l.data_ptr(), dq.data_ptr(),
        dk.data_ptr(), dv.data_ptr(), B, H, Hkv, S, D, st(dout), st(q), st(k), st(v), st(dq), st(dk), st(dv),
        torch_dtype_code(q.dtype), int(bool(is_causal)), float(scale), workspace.data_ptr(), workspace.numel(),
        int(kernel), _stream_ptr(stream))
    if rc != PMKL_OK:
        raise PmklError(rc, "pmkl_causal_attention_bwd_strided")


KERNEL_NAMES = {KERNEL_SIMT: "attn_fwd_simt_kernel", KERNEL_TCGEN05: "attn_fwd_pp_kernel",
                3: "attn_fwd_tc_kernel"}


def attention_selected_kernel(q, k, v, o, kernel: int = KERNEL_AUTO) -> int:
    """The PMKL_ATTN_* kernel the library runs for these tensors."""
    rc = capi().pmkl_attention_selected_kernel(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), q.shape[-1],
                                               torch_dtype_code(q.dtype), torch_dtype_code(o.dtype), int(kernel))
    if rc < 0:
        raise PmklError(rc, "pmkl_attention_selected_kernel")
    return rc


def attention_kernel_name(q, k, v, o, kernel: int = KERNEL_AUTO) -> str:
    return KERNEL_NAMES.get(attention_selected_kernel(q, k, v, o, kernel), "unknown")


def warp_softmax_fwd(dst, src, elements: int, stride: int, rows: int, is_log: bool = False, stream=None) -> None:
    """Calls pmkl_warp_softmax_fwd on caller-allocated torch CUDA tensors."""
    rc = capi().pmkl_warp_softmax_fwd(dst.data_ptr(), src.data_ptr(), int(elements), int(stride), int(rows),
                                      torch_dtype_code(src.dtype), torch_dtype_code(dst.dtype), int(bool(is_log)),
                                      _stream_ptr(stream))
    if rc != PMKL_OK:
        raise PmklError(rc, "pmkl_warp_softmax_fwd")


def device_error(clear: bool = True) -> int:
    """pmkl_device_error: synchronises the device, returns the status."""
    return capi().pmkl_device_error(int(bool(clear)))
