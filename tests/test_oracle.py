"""CPU tests of the oracle itself: it must reproduce the reference's own
outputs (golden fixtures made by running the reference's CPU code) before any
kernel is checked against it."""
import numpy as np
import pytest
import torch

from helpers import GOLDEN, golden_tensor, load_golden
from oracle import oracle

ATTN_F32 = sorted(p.stem for p in GOLDEN.glob("attn_*f32*.npz") if not p.stem.startswith("attn_bwd"))
ATTN_LP = sorted(p.stem for p in GOLDEN.glob("attn_*.npz") if "f32" not in p.stem and not p.stem.startswith("attn_bwd"))
BWD_F32 = sorted(p.stem for p in GOLDEN.glob("attn_bwd_*f32*.npz"))
BWD_LP = sorted(p.stem for p in GOLDEN.glob("attn_bwd_*.npz") if "f32" not in p.stem)
SOFTMAX = sorted(p.stem for p in GOLDEN.glob("softmax_*.npz"))


def test_fixture_inventory():
    assert len(ATTN_F32) >= 8 and len(ATTN_LP) >= 3 and len(SOFTMAX) >= 4
    assert len(BWD_F32) >= 4 and len(BWD_LP) >= 1


@pytest.mark.parametrize("name", ATTN_F32)
def test_oracle_matches_reference_fp32_bitwise(name):
    g = load_golden(name)
    o, m, l = oracle.attention_fwd(g["q"], g["k"], g["v"], bool(g["causal"]))
    np.testing.assert_array_equal(o, g["o"])
    np.testing.assert_array_equal(m, g["m"])
    np.testing.assert_array_equal(l, g["l"])


@pytest.mark.parametrize("name", ATTN_F32)
def test_oracle_rows_match_full(name):
    g = load_golden(name)
    B, H, S, D = g["q"].shape
    rng = np.random.default_rng(0)
    n = min(16, B * H * S)
    slices = rng.integers(0, B * H, n)
    rows = rng.integers(0, S, n)
    rows[0] = 0
    rows[-1] = S - 1
    o, m, l = oracle.attention_rows(g["q"], g["k"], g["v"], bool(g["causal"]), slices, rows)
    np.testing.assert_array_equal(o, g["o"].reshape(B * H, S, D)[slices, rows])
    np.testing.assert_array_equal(m, g["m"].reshape(B * H, S)[slices, rows])
    np.testing.assert_array_equal(l, g["l"].reshape(B * H, S)[slices, rows])


@pytest.mark.parametrize("name", ATTN_F32)
def test_oracle_agrees_with_fp64_sdpa(name):
    """The reference's Python test compares against scaled_dot_product_attention
    (pmkl_pytorch_ext/test/test_fused_self_attention.py:6-7)."""
    g = load_golden(name)
    q, k, v = (torch.from_numpy(g[x]).double() for x in ("q", "k", "v"))
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=bool(g["causal"])).numpy()
    o, _, _ = oracle.attention_fwd(g["q"], g["k"], g["v"], bool(g["causal"]))
    assert np.abs(o - ref).max() < 5e-6


@pytest.mark.parametrize("name", ATTN_LP)
def test_reference_lowp_vs_fp32_oracle(name):
    """The reference evaluated in fp16/bf16 accumulates in the 16-bit type; the
    fp32 oracle on the same 16-bit inputs is the parity target instead.  This
    pins how far the reference's own low-precision path is from it."""
    g = load_golden(name)
    dt = g["dtype"]
    q, k, v = (golden_tensor(g[x], dt).float().numpy() for x in ("q", "k", "v"))
    o, m, _ = oracle.attention_fwd(q, k, v, bool(g["causal"]))
    ref_o = golden_tensor(g["o"], dt).float().numpy()
    ref_m = golden_tensor(g["m"], dt).float().numpy()
    err = np.abs(ref_o - o).max()
    assert err < 0.1, err  # bf16 accumulation: a few 1e-2; fp16: a few 1e-3
    assert np.abs(ref_m - m).max() < 0.05


@pytest.mark.parametrize("name", SOFTMAX)
def test_softmax_oracle_matches_reference_bitwise(name):
    g = load_golden(name)
    rows, el, st = int(g["rows"]), int(g["elements"]), int(g["stride"])
    y = oracle.softmax_fwd(g["x"], elements=el, stride=st, rows=rows)
    ref = g["y"]
    for r in range(rows):
        np.testing.assert_array_equal(y[r * st: r * st + el], ref[r * st: r * st + el])


def test_log_softmax_oracle_identity():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((7, 300)) * 2).astype(np.float32)
    y = oracle.softmax_fwd(x)
    ly = oracle.softmax_fwd(x, is_log=True)
    np.testing.assert_allclose(np.exp(ly.astype(np.float64)), y, rtol=2e-6, atol=1e-9)
    np.testing.assert_allclose(y.sum(-1), 1.0, rtol=1e-5)


def test_oracle_causal_prefix_property():
    """Row i of a causal problem depends only on keys [0, i]: truncating the
    sequence after row r leaves rows [0, r] bit-identical."""
    rng = np.random.default_rng(2)
    q, k, v = (rng.standard_normal((1, 2, 50, 16)).astype(np.float32) for _ in range(3))
    o, m, l = oracle.attention_fwd(q, k, v, True)
    o2, m2, l2 = oracle.attention_fwd(q[:, :, :30], k[:, :, :30], v[:, :, :30], True)
    np.testing.assert_array_equal(o[:, :, :30], o2)
    np.testing.assert_array_equal(m[:, :, :30], m2)
    np.testing.assert_array_equal(l[:, :, :30], l2)


# ------------------------------------------------------------------ backward
def _bwd_inputs(g):
    return [golden_tensor(g[x], g["dtype"]).float().numpy() for x in ("do", "q", "k", "v", "m", "l")]


@pytest.mark.parametrize("name", BWD_F32)
def test_bwd_oracle_exact_matches_reference_bitwise(name):
    """The O(S^3 D) restatement reproduces fused_self_attention_bw
    (fused_self_attention.cpp:66-135) bit for bit in fp32."""
    g = load_golden(name)
    dq, dk, dv = oracle.attention_bwd(*_bwd_inputs(g), bool(g["causal"]), exact=True)
    np.testing.assert_array_equal(dq, g["dq"])
    np.testing.assert_array_equal(dk, g["dk"])
    np.testing.assert_array_equal(dv, g["dv"])


@pytest.mark.parametrize("name", BWD_F32)
def test_bwd_oracle_fast_form_matches_reference(name):
    """The O(S^2 D) form used at larger sizes agrees with the reference to
    fp32 rounding (relative to each gradient's largest entry)."""
    g = load_golden(name)
    got = oracle.attention_bwd(*_bwd_inputs(g), bool(g["causal"]))
    for a, key in zip(got, ("dq", "dk", "dv")):
        ref = g[key]
        assert np.abs(a - ref).max() <= 2e-6 * max(np.abs(ref).max(), 1e-30), key


@pytest.mark.parametrize("name", BWD_F32)
def test_bwd_oracle_agrees_with_fp64_autograd(name):
    """The reference's Python test checks the backward against autograd through
    scaled_dot_product_attention (test_fused_self_attention.py:21-38)."""
    g = load_golden(name)
    do, q, k, v, m, l = (torch.from_numpy(a).double() for a in _bwd_inputs(g))
    q, k, v = (t.clone().requires_grad_() for t in (q, k, v))
    out = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=bool(g["causal"]))
    out.backward(do)
    got = oracle.attention_bwd(*_bwd_inputs(g), bool(g["causal"]))
    for a, t in zip(got, (q, k, v)):
        ref = t.grad.numpy()
        assert np.abs(a - ref).max() <= 1e-5 * max(np.abs(ref).max(), 1e-30)


@pytest.mark.parametrize("name", BWD_LP)
def test_bwd_reference_lowp_vs_fp32_oracle(name):
    """In bf16 the reference accumulates every gradient in bf16; the fp32
    oracle on the same 16-bit inputs (and the same 16-bit m, l) is the parity
    target.  This pins how far the reference's own bf16 result is from it."""
    g = load_golden(name)
    got = oracle.attention_bwd(*_bwd_inputs(g), bool(g["causal"]))
    for a, key in zip(got, ("dq", "dk", "dv")):
        ref = golden_tensor(g[key], g["dtype"]).float().numpy()
        rel = np.abs(a - ref).max() / np.abs(a).max()
        assert 1e-4 < rel < 0.5, (key, rel)


def test_bwd_oracle_matches_live_reference():
    """Random case through the reference extension built in oracle/_ref, when
    it is present (it is built wherever the reference tree is)."""
    from oracle import build_ref

    if not build_ref.ref_ext_path().is_file():
        pytest.skip("reference extension not built")
    ext = build_ref.load_ref_ext()
    gen = torch.Generator().manual_seed(99)
    q, k, v, do = (torch.randn(2, 1, 37, 24, generator=gen) for _ in range(4))
    for causal in (True, False):
        _, m, l = ext.fused_self_attention_fw(q, k, v, causal)
        ref = ext.fused_self_attention_bw(do, q, k, v, m, l, causal)
        got = oracle.attention_bwd(do.numpy(), q.numpy(), k.numpy(), v.numpy(), m.numpy(), l.numpy(), causal,
                                   exact=True)
        for a, r in zip(got, ref):
            np.testing.assert_array_equal(a, r.numpy())
