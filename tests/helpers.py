"""Shared helpers for the parity tests: golden-fixture loading, seeded input
generation, tolerances, and calls through the C ABI."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"

# Tolerances.
#   fp32: the reference's all_close rule, |a - b| <= 1e-5 + 1e-5 |b|
#         (pmkl/core/utils/measure.h:10-12).
#   fp16/bf16: max |a - b| <= 2e-3 against the fp32 oracle evaluated on the same
#         (already 16-bit) inputs.  When the kernel writes 16-bit outputs, the
#         output rounding itself is up to half an ulp of the dtype at |b|, so
#         the bound is 2e-3 + ulp/2: the kernel's value before its final
#         rounding is within 2e-3 of the oracle.  With fp32 outputs the bound
#         is the plain 2e-3.
F32_ATOL = 1e-5
F32_RTOL = 1e-5
LP_ATOL = 2e-3


def ulp(x: np.ndarray, dtype: torch.dtype) -> np.ndarray:
    """Spacing of `dtype` values around |x| (fp32 numpy in and out)."""
    mant = {torch.bfloat16: 7, torch.float16: 10, torch.float32: 23}[dtype]
    min_exp = {torch.bfloat16: -126, torch.float16: -14, torch.float32: -126}[dtype]
    a = np.abs(x.astype(np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** min_exp)))
    return (2.0 ** (e - mant)).astype(np.float64)


def lp_bound(ref: np.ndarray, out_dtype: torch.dtype) -> np.ndarray:
    if out_dtype == torch.float32:
        return np.full(ref.shape, LP_ATOL)
    return LP_ATOL + 0.5 * ulp(ref, out_dtype)


def assert_lp_close(got: np.ndarray, ref: np.ndarray, out_dtype: torch.dtype, what: str = "") -> float:
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    assert np.isfinite(got).all(), f"{what}: non-finite values"
    err = np.abs(got - ref)
    bound = lp_bound(ref, out_dtype)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(f"{what}: {bad.sum()} values out of tolerance; worst at {i}: got {got[i]}, "
                             f"ref {ref[i]}, err {err[i]:.3e}, bound {bound[i]:.3e}")
    return float(err.max()) if err.size else 0.0


def assert_f32_close(got: np.ndarray, ref: np.ndarray, what: str = "",
                     atol: float = F32_ATOL, rtol: float = F32_RTOL) -> float:
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    err = np.abs(got - ref)
    bound = atol + rtol * np.abs(ref)
    bad = ~(err <= bound)  # NaN counts as a failure, as in measure.h:15
    if bad.any():
        i = np.unravel_index(np.argmax(np.where(np.isnan(err), np.inf, err - bound)), err.shape)
        raise AssertionError(f"{what}: {bad.sum()} values out of tolerance; worst at {i}: got {got[i]}, "
                             f"ref {ref[i]}, err {err[i]:.3e}")
    return float(err.max()) if err.size else 0.0


def load_golden(name: str) -> dict:
    z = np.load(GOLDEN / f"{name}.npz")
    out = {k: z[k] for k in z.files}
    dt = str(out.get("dtype", "float32"))
    if "dtype" in out:
        out["dtype"] = dt
    return out


def golden_tensor(arr: np.ndarray, dtype_name: str) -> torch.Tensor:
    """Rebuild a torch tensor from a golden array (16-bit types are stored raw)."""
    if dtype_name in ("bfloat16", "float16"):
        td = torch.bfloat16 if dtype_name == "bfloat16" else torch.float16
        return torch.from_numpy(arr.view(np.int16).copy()).view(td)
    return torch.from_numpy(arr.copy())


def seeded_qkv(B, H, S, D, dtype, seed, std=1.0):
    """q, k, v ~ N(0, std^2) from torch.Generator().manual_seed(seed), drawn
    on the CPU in the order q, k, v, then cast to dtype (CPU tensors)."""
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(B, H, S, D, generator=g) * std).to(dtype) for _ in range(3)]


def attention_capi(q, k, v, causal, out_fp32=False, kernel=0, scale=0.0):
    """Runs the attention through the C ABI on CUDA copies of q, k, v and
    returns (o, m, l) as CUDA tensors."""
    import pmkl_b200

    qd, kd, vd = (t.cuda().contiguous() for t in (q, k, v))
    B, H, S, D = qd.shape
    odt = torch.float32 if out_fp32 else qd.dtype
    o = torch.empty(B, H, S, D, dtype=odt, device="cuda")
    m = torch.empty(B, H, S, dtype=odt, device="cuda")
    l = torch.empty(B, H, S, dtype=odt, device="cuda")
    pmkl_b200.attention_fwd(qd, kd, vd, o, m, l, causal, scale=scale, kernel=kernel)
    torch.cuda.synchronize()
    return o, m, l


def np32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()
