"""Python front end of the CPU oracle (``pmkl_oracle.c``) and of the
reference libraries built by ``build_ref.py``.

TEST INFRASTRUCTURE ONLY.  Imported by ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg; the product path never imports it.

All arrays are numpy, C-contiguous.  Attention tensors are ``[B, H, S, D]``
(the reference ext's layout, ``fused_self_attention.cpp:143-150``); the
oracle computes in fp32 on inputs that the caller has already rounded to the
kernel's input dtype and upcast.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
BUILD_DIR = ORACLE_DIR / "_build"
LIB_PATH = BUILD_DIR / "libpmkl_oracle.so"
SRC = ORACLE_DIR / "pmkl_oracle.c"

_lib = None


def build(force: bool = False) -> Path:
    """Compile pmkl_oracle.c with the reference build's optimisation level
    (-O2, no fast-math, no FMA contraction) so fp32 results match it bitwise."""
    if LIB_PATH.is_file() and not force and LIB_PATH.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB_PATH
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    subprocess.run(
        ["gcc", "-O2", "-fPIC", "-shared", "-ffp-contract=off", str(SRC), "-o", str(LIB_PATH), "-lm"],
        check=True,
    )
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB_PATH))
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.pmkl_oracle_attention_fwd_f32.restype = i32
        L.pmkl_oracle_attention_fwd_f32.argtypes = [vp, vp, vp, vp, vp, vp, i64, i32, i32, i32, ctypes.c_float]
        L.pmkl_oracle_attention_rows_f32.restype = i32
        L.pmkl_oracle_attention_rows_f32.argtypes = [vp, vp, vp, i32, i32, i32, ctypes.c_float, vp, vp, i64, vp, vp, vp]
        L.pmkl_oracle_attention_bwd_exact_f32.restype = None
        L.pmkl_oracle_attention_bwd_exact_f32.argtypes = [vp] * 9 + [i64, i32, i32, i32]
        L.pmkl_oracle_attention_bwd_f32.restype = i32
        L.pmkl_oracle_attention_bwd_f32.argtypes = [vp] * 9 + [i64, i32, i32, i32, ctypes.c_float]
        for name in ("pmkl_oracle_softmax_fwd_f32", "pmkl_oracle_log_softmax_fwd_f32"):
            fn = getattr(L, name)
            fn.restype = None
            fn.argtypes = [vp, vp, i32, i32, i32]
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def default_scale(D: int) -> np.float32:
    """1.0f / sqrt((float)D) in fp32, as fused_self_attention.cpp:30 and
    causal_attention.h:192 compute it."""
    return np.float32(1.0) / np.sqrt(np.float32(D))


def attention_fwd(q, k, v, causal: bool, scale=None):
    """Full oracle.  q, k, v: [B, H, S, D] (any float dtype; upcast to fp32).
    Returns (o [B,H,S,D], m [B,H,S], l [B,H,S]) in fp32."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    B, H, S, D = q.shape
    assert k.shape == q.shape and v.shape == q.shape
    scale = default_scale(D) if scale is None else np.float32(scale)
    o = np.empty_like(q)
    m = np.empty((B, H, S), np.float32)
    l = np.empty((B, H, S), np.float32)
    rc = lib().pmkl_oracle_attention_fwd_f32(_ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(m), _ptr(l),
                                              B * H, S, D, int(bool(causal)), float(scale))
    if rc != 0:
        raise MemoryError("oracle scratch allocation failed")
    return o, m, l


def attention_rows(q, k, v, causal: bool, slices, rows, scale=None):
    """Row-sampled oracle: evaluates query row rows[i] of (b*H+h) slice
    slices[i].  Returns packed (o [n, D], m [n], l [n]) in fp32."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    B, H, S, D = q.shape
    scale = default_scale(D) if scale is None else np.float32(scale)
    slices = np.ascontiguousarray(slices, dtype=np.int64)
    rows = np.ascontiguousarray(rows, dtype=np.int32)
    n = len(rows)
    assert len(slices) == n
    assert (slices >= 0).all() and (slices < B * H).all() and (rows >= 0).all() and (rows < S).all()
    o = np.empty((n, D), np.float32)
    m = np.empty(n, np.float32)
    l = np.empty(n, np.float32)
    rc = lib().pmkl_oracle_attention_rows_f32(_ptr(q), _ptr(k), _ptr(v), S, D, int(bool(causal)),
                                               float(scale), _ptr(slices), _ptr(rows), n,
                                               _ptr(o), _ptr(m), _ptr(l))
    if rc != 0:
        raise MemoryError("oracle scratch allocation failed")
    return o, m, l


def attention_bwd(dout, q, k, v, m, l, causal: bool, scale=None, exact: bool = False):
    """Gradients of fused_self_attention (fused_self_attention.cpp:66-135):
    (dq, dk, dv) in fp32 for dout, q, k, v [B, H, S, D] and the forward's m, l
    [B, H, S], all upcast to fp32.  ``exact`` runs the reference's O(S^3 D) loop
    as written (fp32, bit-identical to it; default scale only); otherwise the
    O(S^2 D) double-accumulation form."""
    arrs = [np.ascontiguousarray(a, dtype=np.float32) for a in (dout, q, k, v, m, l)]
    dout, q, k, v, m, l = arrs
    B, H, S, D = q.shape
    assert k.shape == q.shape and v.shape == q.shape and dout.shape == q.shape
    assert m.shape == (B, H, S) and l.shape == (B, H, S)
    dq, dk, dv = np.empty_like(q), np.empty_like(q), np.empty_like(q)
    args = [_ptr(a) for a in (dout, q, k, v, m, l, dq, dk, dv)]
    if exact:
        assert scale is None or np.float32(scale) == default_scale(D)
        lib().pmkl_oracle_attention_bwd_exact_f32(*args, B * H, S, D, int(bool(causal)))
    else:
        scale = default_scale(D) if scale is None else np.float32(scale)
        rc = lib().pmkl_oracle_attention_bwd_f32(*args, B * H, S, D, int(bool(causal)), float(scale))
        if rc != 0:
            raise MemoryError("oracle scratch allocation failed")
    return dq, dk, dv


def softmax_fwd(x, elements: int | None = None, stride: int | None = None, rows: int | None = None,
                is_log: bool = False):
    """Row softmax over the first `elements` entries of each of `rows` rows
    spaced `stride` apart (the reference's argument meaning,
    warp_softmax.h:159-161).  Entries past `elements` in each row are left
    as they are in the returned copy of x."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    flat = x.reshape(-1)
    if elements is None:
        elements = x.shape[-1]
    if stride is None:
        stride = x.shape[-1]
    if rows is None:
        rows = flat.size // stride if stride else 0
    out = flat.copy()
    fn = lib().pmkl_oracle_log_softmax_fwd_f32 if is_log else lib().pmkl_oracle_softmax_fwd_f32
    fn(_ptr(out), _ptr(flat), int(elements), int(stride), int(rows))
    return out.reshape(x.shape)
