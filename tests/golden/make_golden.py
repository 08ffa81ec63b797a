"""Generates the golden fixtures in this directory by running the reference's
own CPU code (built into ``oracle/_ref/`` by ``oracle/build_ref.py``) on seeded
inputs.  Run it where the reference tree is present:

    python tests/golden/make_golden.py

Each ``.npz`` holds the inputs and the reference's outputs; the CPU tests
replay the inputs through the oracle and through the CUDA path.

Attention fixtures call ``fused_self_attention_fw`` of the reference extension
(``pmkl_pytorch_ext/fused_self_attention.cpp:139-173``); backward fixtures
(``attn_bwd_*``) also call ``fused_self_attention_bw`` (``:175-215``).  Softmax fixtures call
``host_softmax_forward<float,float,float>`` (``test/test_softmax.cpp:10-28``).
Half/bfloat16 tensors are stored as their raw 16-bit patterns (numpy has no
bfloat16).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import build_ref  # noqa: E402

# (name, B, H, S, D, causal, torch dtype, seed, std)
ATTN_CASES = [
    # BASELINE config 1 (fp32 B2 H4 S128 D64, causal, N(0,1))
    ("attn_cfg1_f32_causal", 2, 4, 128, 64, True, torch.float32, 1, 1.0),
    # shapes of the reference's Python test (test_fused_self_attention.py:10-14),
    # reduced to B1 H2 to keep the fixtures small
    ("attn_s128_d64_f32_full", 1, 2, 128, 64, False, torch.float32, 2, 1.0),
    ("attn_s128_d128_f32_causal", 1, 2, 128, 128, True, torch.float32, 3, 1.0),
    ("attn_s128_d128_f32_full", 1, 2, 128, 128, False, torch.float32, 4, 1.0),
    # ragged / tiny shapes (S not a multiple of any tile, S = 1)
    ("attn_s77_d128_f32_full", 1, 2, 77, 128, False, torch.float32, 5, 1.0),
    ("attn_s200_d64_f32_causal", 1, 1, 200, 64, True, torch.float32, 6, 1.0),
    ("attn_s1_d64_f32_causal", 1, 3, 1, 64, True, torch.float32, 7, 1.0),
    ("attn_s5_d32_f32_causal", 1, 1, 5, 32, True, torch.float32, 8, 1.0),
    # the reference evaluated in reduced precision (accumulates in the dtype)
    ("attn_s64_d64_bf16_causal", 1, 2, 64, 64, True, torch.bfloat16, 9, 1.0),
    ("attn_s64_d64_f16_causal", 1, 2, 64, 64, True, torch.float16, 10, 1.0),
    ("attn_s64_d128_bf16_causal_std05", 1, 2, 64, 128, True, torch.bfloat16, 11, 0.5),
]

# Backward fixtures: (name, B, H, S, D, causal, torch dtype, seed).  m, l come
# from the reference's forward on the same inputs, dout is N(0, 1).
BWD_CASES = [
    ("attn_bwd_s64_d64_f32_causal", 1, 2, 64, 64, True, torch.float32, 30),
    ("attn_bwd_s77_d128_f32_full", 1, 1, 77, 128, False, torch.float32, 31),
    ("attn_bwd_s130_d64_f32_causal", 1, 1, 130, 64, True, torch.float32, 32),
    ("attn_bwd_s5_d32_f32_causal", 2, 1, 5, 32, True, torch.float32, 33),
    ("attn_bwd_s48_d64_bf16_causal", 1, 2, 48, 64, True, torch.bfloat16, 34),
]

# (name, rows, elements, stride, seed, std)
SOFTMAX_CASES = [
    ("softmax_12x1024", 12, 1024, 1024, 20, 2.0),  # test_softmax.cpp:33-34 shape, N(0,4) values
    ("softmax_ragged_7x1000_s1024", 7, 1000, 1024, 21, 2.0),
    ("softmax_33x37_s40", 33, 37, 40, 22, 2.0),
    ("softmax_5x1", 5, 1, 1, 23, 2.0),
]


def _raw(t: torch.Tensor) -> np.ndarray:
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def make_attention(ext) -> None:
    for name, B, H, S, D, causal, dtype, seed, std in ATTN_CASES:
        g = torch.Generator().manual_seed(seed)
        q, k, v = [(torch.randn(B, H, S, D, generator=g) * std).to(dtype) for _ in range(3)]
        o, m, l = ext.fused_self_attention_fw(q, k, v, causal)
        np.savez_compressed(
            HERE / f"{name}.npz",
            q=_raw(q), k=_raw(k), v=_raw(v), o=_raw(o), m=_raw(m), l=_raw(l),
            causal=np.array(causal), dtype=np.array(str(dtype).replace("torch.", "")),
        )
        print("wrote", name)


def make_attention_bwd(ext) -> None:
    """``fused_self_attention_bw`` (fused_self_attention.cpp:175-215) on the
    forward's own m, l."""
    for name, B, H, S, D, causal, dtype, seed in BWD_CASES:
        g = torch.Generator().manual_seed(seed)
        q, k, v, do = [torch.randn(B, H, S, D, generator=g).to(dtype) for _ in range(4)]
        o, m, l = ext.fused_self_attention_fw(q, k, v, causal)
        dq, dk, dv = ext.fused_self_attention_bw(do, q, k, v, m, l, causal)
        np.savez_compressed(
            HERE / f"{name}.npz",
            q=_raw(q), k=_raw(k), v=_raw(v), do=_raw(do), m=_raw(m), l=_raw(l),
            dq=_raw(dq), dk=_raw(dk), dv=_raw(dv),
            causal=np.array(causal), dtype=np.array(str(dtype).replace("torch.", "")),
        )
        print("wrote", name)


def make_softmax(fn) -> None:
    for name, rows, elements, stride, seed, std in SOFTMAX_CASES:
        g = torch.Generator().manual_seed(seed)
        x = (torch.randn(rows * stride, generator=g) * std).numpy().astype(np.float32)
        y = np.full_like(x, np.nan)
        fn(y.ctypes.data, x.ctypes.data, elements, stride, rows)
        np.savez_compressed(HERE / f"{name}.npz", x=x, y=y, rows=np.array(rows),
                            elements=np.array(elements), stride=np.array(stride))
        print("wrote", name)


def main() -> None:
    if not build_ref.build():
        raise SystemExit("reference tree not found; set PMKL_REFERENCE_DIR")
    torch.set_num_threads(1)
    make_attention(build_ref.load_ref_ext())
    make_attention_bwd(build_ref.load_ref_ext())
    make_softmax(build_ref.load_ref_softmax())


if __name__ == "__main__":
    main()
