"""GPU parity tests of the attention kernels, called through the C ABI
(include/pmkl_b200.h) and checked against the CPU oracle (oracle/), which is
itself pinned bit-for-bit to the reference's CPU code (tests/test_oracle.py).

Tolerances are defined in tests/helpers.py: fp32 follows the reference's
all_close (1e-5 abs + 1e-5 rel); fp16/bf16 inputs must land within 2e-3 of the
fp32 oracle on the same 16-bit inputs (plus half an output ulp when the output
itself is 16-bit)."""
import numpy as np
import pytest
import torch

import pmkl_b200
from helpers import (GOLDEN, assert_f32_close, assert_lp_close, attention_capi, golden_tensor, load_golden, np32,
                     seeded_qkv)
from oracle import oracle

pytestmark = pytest.mark.gpu

TC = pmkl_b200.KERNEL_TCGEN05
SIMT = pmkl_b200.KERNEL_SIMT
LP = [torch.bfloat16, torch.float16]
ATTN_F32 = sorted(p.stem for p in GOLDEN.glob("attn_*f32*.npz") if not p.stem.startswith("attn_bwd"))


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    yield
    assert pmkl_b200.device_error(clear=True) == 0, "a kernel abandoned a bounded wait"


def check_lp(q, k, v, causal, o, m, l, what):
    """Full oracle on the (already 16-bit) inputs, compared with kernel outputs."""
    ro, rm, rl = oracle.attention_fwd(np32(q), np32(k), np32(v), causal)
    od = o.dtype
    assert_lp_close(np32(o), ro, od, what + " O")
    assert_lp_close(np32(m), rm, od, what + " m")
    # l grows with the number of keys; compare relative to its size.
    rel = np.abs(np32(l) - rl) / np.maximum(rl, 1.0)
    assert rel.max() <= 2e-3 + (0.5 * 2.0 ** -7 if od == torch.bfloat16 else 0.5 * 2.0 ** -10 if od == torch.float16 else 0), \
        f"{what} l rel err {rel.max()}"


# ------------------------------------------------------------------ tensor-core primitives
@pytest.mark.parametrize("dtype", LP)
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("which", [0, 1])
def test_tc_selftest(which, D, dtype):
    g = torch.Generator().manual_seed(100 + which * 10 + D)
    if which == 0:
        a = torch.randn(128, D, generator=g).to(dtype)
        b = torch.randn(128, D, generator=g).to(dtype)
        ref = a.double() @ b.double().T
    else:
        a = torch.rand(128, 128, generator=g).to(dtype)
        b = torch.randn(128, D, generator=g).to(dtype)
        ref = a.double() @ b.double()
    ad, bd = a.cuda(), b.cuda()
    c = torch.empty(ref.shape, dtype=torch.float32, device="cuda")
    rc = pmkl_b200.capi().pmkl_tc_selftest(which, ad.data_ptr(), bd.data_ptr(), c.data_ptr(), D,
                                          pmkl_b200.torch_dtype_code(dtype), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    err = (c.double().cpu() - ref).abs().max().item()
    assert err < 1e-3, err


# ------------------------------------------------------------------ golden fixtures
@pytest.mark.parametrize("name", ATTN_F32)
def test_golden_fp32(name):
    """fp32 inputs (SIMT path) against the reference's own fp32 outputs."""
    g = load_golden(name)
    q, k, v = (torch.from_numpy(g[x]) for x in ("q", "k", "v"))
    o, m, l = attention_capi(q, k, v, bool(g["causal"]))
    assert_f32_close(np32(m), g["m"], name + " m")
    assert_f32_close(np32(l), g["l"], name + " l")
    assert_f32_close(np32(o), g["o"], name + " O")


@pytest.mark.parametrize("dtype", LP)
@pytest.mark.parametrize("name", [n for n in ATTN_F32 if "d64" in n or "d128" in n])
def test_golden_inputs_lowp_tc(name, dtype):
    """The golden inputs rounded to fp16/bf16 through the tensor-core path."""
    g = load_golden(name)
    q, k, v = (torch.from_numpy(g[x]).to(dtype) for x in ("q", "k", "v"))
    causal = bool(g["causal"])
    o, m, l = attention_capi(q, k, v, causal, kernel=TC)
    check_lp(q, k, v, causal, o, m, l, name)
    o32, m32, l32 = attention_capi(q, k, v, causal, out_fp32=True, kernel=TC)
    check_lp(q, k, v, causal, o32, m32, l32, name + " fp32-out")


@pytest.mark.parametrize("name", [p.stem for p in GOLDEN.glob("attn_*.npz")
                                  if "f32" not in p.stem and not p.stem.startswith("attn_bwd")])
def test_golden_lowp_fixtures(name):
    g = load_golden(name)
    dt = g["dtype"]
    q, k, v = (golden_tensor(g[x], dt) for x in ("q", "k", "v"))
    causal = bool(g["causal"])
    o, m, l = attention_capi(q, k, v, causal)
    check_lp(q, k, v, causal, o, m, l, name)


# ------------------------------------------------------------------ edge shapes
EDGE_S = [1, 2, 5, 64, 127, 128, 129, 200, 255, 256, 257, 384, 515]


@pytest.mark.parametrize("dtype", LP)
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("S", EDGE_S)
def test_edge_shapes_tc(S, causal, D, dtype):
    q, k, v = seeded_qkv(1, 2, S, D, dtype, seed=S * 7 + D + int(causal))
    o, m, l = attention_capi(q, k, v, causal, kernel=TC)
    check_lp(q, k, v, causal, o, m, l, f"S{S} D{D} causal={causal}")


@pytest.mark.parametrize("dtype", [torch.float32] + LP)
@pytest.mark.parametrize("D", [16, 32, 48, 64, 96, 128, 200, 256])
@pytest.mark.parametrize("causal", [True, False])
def test_simt_head_sizes(D, causal, dtype):
    S = 77
    q, k, v = seeded_qkv(1, 3, S, D, dtype, seed=D * 3 + int(causal))
    o, m, l = attention_capi(q, k, v, causal, kernel=SIMT)
    if dtype == torch.float32:
        ro, rm, rl = oracle.attention_fwd(np32(q), np32(k), np32(v), causal)
        assert_f32_close(np32(o), ro, "O")
        assert_f32_close(np32(m), rm, "m")
        assert_f32_close(np32(l), rl, "l")
    else:
        check_lp(q, k, v, causal, o, m, l, f"simt D{D}")


def test_custom_scale():
    q, k, v = seeded_qkv(1, 2, 300, 128, torch.bfloat16, seed=5)
    for sc in (0.05, 0.1):  # score std 0.57 and 1.13
        o, m, l = attention_capi(q, k, v, True, kernel=TC, scale=sc)
        ro, rm, rl = oracle.attention_fwd(np32(q), np32(k), np32(v), True, scale=sc)
        assert_lp_close(np32(o), ro, torch.bfloat16, "O")
        assert_lp_close(np32(m), rm, torch.bfloat16, "m")


def test_peaked_scores_bf16_p_bound():
    """With very peaked scores (scale 0.3: score std 3.4) a row has only a few
    effective keys even far from the start, and the one rounding of P to bf16
    before P.V (2^-9 relative per weight, as in any flash kernel) shows:
    |O - O_ref| <= 2^-8 * max|v| bounds it (plus the output's half ulp)."""
    q, k, v = seeded_qkv(1, 2, 300, 128, torch.bfloat16, seed=5)
    o, m, l = attention_capi(q, k, v, True, kernel=TC, scale=0.3)
    ro, rm, rl = oracle.attention_fwd(np32(q), np32(k), np32(v), True, scale=0.3)
    got = np32(o).astype(np.float64)
    vmax = float(np.abs(np32(v)).max())
    half_ulp = 0.5 * (2.0 ** (np.floor(np.log2(np.maximum(np.abs(ro), 1e-30))) - 7))
    assert (np.abs(got - ro) <= 2.0 ** -8 * vmax + half_ulp).all()
    assert_lp_close(np32(m), rm, torch.bfloat16, "m")


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("dtype", LP)
def test_row_max_jumps_after_first_key_tile(causal, D, dtype):
    """Keys of the later key tiles are scaled up (x6 for keys 128..255, x12
    beyond), so most rows' maxima jump by far more than 2^8 after the first key
    tile: the kernel's exp reference point must move and O be rescaled.
    Same P-rounding bound as the peaked-score test."""
    q, k, v = seeded_qkv(1, 3, 640, D, dtype, seed=17)
    k = k.clone()
    k[:, :, 128:256] *= 6
    k[:, :, 256:] *= 12
    o, m, l = attention_capi(q, k, v, causal, kernel=TC)
    ro, rm, rl = oracle.attention_fwd(np32(q), np32(k), np32(v), causal)
    got = np32(o).astype(np.float64)
    vmax = float(np.abs(np32(v)).max())
    mant = 7 if dtype == torch.bfloat16 else 10
    half_ulp = 0.5 * (2.0 ** (np.floor(np.log2(np.maximum(np.abs(ro), 1e-30))) - mant))
    assert (np.abs(got - ro) <= 2.0 ** -8 * vmax + half_ulp).all()
    assert_lp_close(np32(m), rm, dtype, "m")
    rel = np.abs(np32(l) - rl) / np.maximum(rl, 1.0)
    assert rel.max() <= 2e-3 + 0.5 * 2.0 ** -mant


# ------------------------------------------------------------------ benchmark configurations
def test_config1_fp32():
    """fp32 B2 H4 S128 D64 causal (also a golden fixture)."""
    q, k, v = seeded_qkv(2, 4, 128, 64, torch.float32, seed=11)
    o, m, l = attention_capi(q, k, v, True)
    ro, rm, rl = oracle.attention_fwd(q.numpy(), k.numpy(), v.numpy(), True)
    assert_f32_close(np32(o), ro, "O")
    assert_f32_close(np32(m), rm, "m")
    assert_f32_close(np32(l), rl, "l")


def test_config2_fp16():
    """fp16 B8 H16 S1024 D64 causal.  Every 8th (b, h) slice
    is checked against the full oracle (all rows)."""
    q, k, v = seeded_qkv(8, 16, 1024, 64, torch.float16, seed=12)
    o, m, l = attention_capi(q, k, v, True)
    sl = slice(0, None, 8)
    qs, ks, vs = (t.reshape(128, 1, 1024, 64)[sl] for t in (q, k, v))
    check_lp(qs, ks, vs, True, o.reshape(128, 1, 1024, 64)[sl], m.reshape(128, 1, 1024)[sl],
             l.reshape(128, 1, 1024)[sl], "config2")


def sampled_rows_check(q, k, v, causal, o, m, l, n_slices, rows_per_slice, seed):
    B, H, S, D = q.shape
    rng = np.random.default_rng(seed)
    slices = rng.choice(B * H, size=min(n_slices, B * H), replace=False)
    base_rows = np.array([0, 1, 2, 127, 128, 129, 255, 256, S // 2, S - 129, S - 128, S - 2, S - 1])
    sel_s, sel_r = [], []
    for s in slices:
        rows = np.unique(np.concatenate([base_rows, rng.integers(0, S, rows_per_slice)]))
        sel_s += [s] * len(rows)
        sel_r += list(rows)
    sel_s = np.array(sel_s)
    sel_r = np.array(sel_r)
    qn, kn, vn = np32(q), np32(k), np32(v)
    ro, rm, rl = oracle.attention_rows(qn, kn, vn, causal, sel_s, sel_r)
    od = o.dtype
    idx = torch.from_numpy(sel_s * S + sel_r)
    got_o = np32(o.reshape(B * H * S, D)[idx.to(o.device)])
    got_m = np32(m.reshape(-1)[idx.to(o.device)])
    got_l = np32(l.reshape(-1)[idx.to(o.device)])
    assert_lp_close(got_o, ro, od, "O rows")
    assert_lp_close(got_m, rm, od, "m rows")
    rel = np.abs(got_l - rl) / np.maximum(rl, 1.0)
    assert rel.max() < 2e-3 + 2.0 ** -8


def test_config3_bf16_sampled():
    """bf16 B16 H32 S4096 D128 causal, N(0,1); the oracle
    on sampled rows (tile boundaries included) of sampled slices."""
    q, k, v = seeded_qkv(16, 32, 4096, 128, torch.bfloat16, seed=13)
    o, m, l = attention_capi(q, k, v, True)
    sampled_rows_check(q, k, v, True, o, m, l, n_slices=6, rows_per_slice=20, seed=3)


def test_config4_bf16_sampled():
    """bf16 B1 H32 S32768 D128 causal, N(0, 0.5^2)."""
    q, k, v = seeded_qkv(1, 32, 32768, 128, torch.bfloat16, seed=14, std=0.5)
    o, m, l = attention_capi(q, k, v, True)
    sampled_rows_check(q, k, v, True, o, m, l, n_slices=3, rows_per_slice=8, seed=4)


# ------------------------------------------------------------------ size-independent properties
def test_shard_consistency_bitwise():
    """A (b, h) shard computed on its own equals the same slices of the full
    run bit for bit: the multi-GPU split by (b, h) changes no result."""
    q, k, v = seeded_qkv(4, 8, 1024, 128, torch.bfloat16, seed=15)
    o, m, l = attention_capi(q, k, v, True)
    qs, ks, vs = (t.reshape(32, 1, 1024, 128)[5:13].contiguous() for t in (q, k, v))
    o2, m2, l2 = attention_capi(qs, ks, vs, True)
    assert torch.equal(o.reshape(32, 1, 1024, 128)[5:13], o2)
    assert torch.equal(m.reshape(32, 1, 1024)[5:13], m2)
    assert torch.equal(l.reshape(32, 1, 1024)[5:13], l2)


def test_deterministic_repeat():
    q, k, v = seeded_qkv(2, 4, 2048, 128, torch.bfloat16, seed=16)
    a = attention_capi(q, k, v, True)
    b = attention_capi(q, k, v, True)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_causality_future_keys_do_not_leak():
    """Changing keys/values after row r leaves rows <= r bit-identical."""
    q, k, v = seeded_qkv(1, 4, 1000, 64, torch.bfloat16, seed=17)
    o, m, l = attention_capi(q, k, v, True)
    k2, v2 = k.clone(), v.clone()
    k2[:, :, 600:] = torch.randn_like(k2[:, :, 600:].float()).to(k2.dtype) * 3
    v2[:, :, 600:] = 7.0
    o2, m2, l2 = attention_capi(q, k2, v2, True)
    assert torch.equal(o[:, :, :600], o2[:, :, :600])
    assert torch.equal(m[:, :, :600], m2[:, :, :600])
    assert not torch.equal(o[:, :, 600:], o2[:, :, 600:])


def test_output_bounds_full_size():
    """At config-3 size: every O row is a convex combination of V rows, so each
    element lies within the column range of V; 1 <= l <= number of keys."""
    q, k, v = seeded_qkv(16, 32, 4096, 128, torch.bfloat16, seed=18)
    o, m, l = attention_capi(q, k, v, True)
    vd = v.cuda().float()
    vmin = vd.amin(dim=2, keepdim=True)
    vmax = vd.amax(dim=2, keepdim=True)
    of = o.float()
    tol = 2.0 ** -7 * vd.abs().amax()
    assert bool(((of >= vmin - tol) & (of <= vmax + tol)).all())
    lf = l.float()
    n_keys = torch.arange(1, 4097, device="cuda", dtype=torch.float32).view(1, 1, -1)
    assert bool((lf >= 1 - 1e-2).all()) and bool((lf <= n_keys * (1 + 1e-2)).all())
    assert bool(torch.isfinite(m.float()).all())


def test_simt_and_tc_agree():
    q, k, v = seeded_qkv(2, 4, 700, 128, torch.bfloat16, seed=19)
    a = attention_capi(q, k, v, True, out_fp32=True, kernel=TC)
    b = attention_capi(q, k, v, True, out_fp32=True, kernel=SIMT)
    # each is within 2e-3 of the oracle, so they are within 4e-3 of each other
    assert (a[0] - b[0]).abs().max().item() < 4e-3
    assert (a[1] - b[1]).abs().max().item() < 1e-4


@pytest.mark.parametrize("dtype", LP)
@pytest.mark.parametrize("D", [64, 128])
def test_native_tensor_core_kernel_is_selected(D, dtype):
    """16-bit inputs with head size 64/128 run the persistent tcgen05 kernel
    (not a fallback); fp32 and other head sizes run the CUDA-core kernel."""
    q = torch.zeros(1, 1, 256, D, dtype=dtype, device="cuda")
    assert pmkl_b200.attention_selected_kernel(q, q, q, q) == TC
    q32 = q.float()
    assert pmkl_b200.attention_selected_kernel(q32, q32, q32, q32) == SIMT
    q96 = torch.zeros(1, 1, 256, 96, dtype=dtype, device="cuda")
    assert pmkl_b200.attention_selected_kernel(q96, q96, q96, q96) == SIMT


# ------------------------------------------------------------------ errors on the device path
def test_tc_rejects_unsupported_head_size():
    q = torch.zeros(1, 1, 16, 96, dtype=torch.bfloat16, device="cuda")
    o = torch.empty_like(q)
    m = torch.empty(1, 1, 16, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(pmkl_b200.PmklError, match="UNSUPPORTED"):
        pmkl_b200.attention_fwd(q, q, q, o, m, m.clone(), True, kernel=TC)


def test_unaligned_pointers_take_simt_path():
    q, k, v = seeded_qkv(1, 1, 64, 64, torch.bfloat16, seed=20)
    buf = torch.empty(q.numel() + 1, dtype=torch.bfloat16, device="cuda")
    qv = buf[1:].view(1, 1, 64, 64)  # 2-byte offset: not 16-byte aligned
    qv.copy_(q.cuda())
    o = torch.empty(1, 1, 64, 64, dtype=torch.bfloat16, device="cuda")
    m = torch.empty(1, 1, 64, dtype=torch.bfloat16, device="cuda")
    l = torch.empty_like(m)
    with pytest.raises(pmkl_b200.PmklError):
        pmkl_b200.attention_fwd(qv, k.cuda(), v.cuda(), o, m, l, True, kernel=TC)
    pmkl_b200.attention_fwd(qv, k.cuda(), v.cuda(), o, m, l, True)  # AUTO falls to SIMT on the GPU
    torch.cuda.synchronize()
    check_lp(q, k, v, True, o, m, l, "unaligned")
