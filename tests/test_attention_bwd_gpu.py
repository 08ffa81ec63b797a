"""GPU parity tests of the attention backward (pmkl_causal_attention_bwd),
called through the C ABI and checked against the CPU oracle's backward
(oracle/pmkl_oracle.c), which is pinned bit-for-bit to the reference's
host_self_attention_backward (fused_self_attention.cpp:66-135) in
tests/test_oracle.py.

Tolerances (max |err| relative to the largest |gradient| of the tensor), set
about 1.3x above the worst errors measured on B200 over this file and the
layout tests (bf16 6.3e-3, fp16 2.3e-3, fp32 8.6e-7):
  fp32 (CUDA-core path)          2e-6   -- fp32 rounding in a different order
  bf16 (tensor-core path)        8e-3   -- P and dS are rounded to 16 bits before
  fp16 (tensor-core path)        3e-3      the gradient products, the outputs once
                                           more; plus half an output ulp per value
The 16-bit reference (the reference's own bf16 run accumulates every gradient in
bf16) is further from the fp32 oracle than this bound; see test_oracle.py."""
import numpy as np
import pytest
import torch

import pmkl_b200
from helpers import GOLDEN, golden_tensor, load_golden, np32, seeded_qkv
from oracle import oracle

pytestmark = pytest.mark.gpu

TC = pmkl_b200.KERNEL_TCGEN05
SIMT = pmkl_b200.KERNEL_SIMT
LP = [torch.bfloat16, torch.float16]
BWD_F32 = sorted(p.stem for p in GOLDEN.glob("attn_bwd_*f32*.npz"))
BWD_LP = sorted(p.stem for p in GOLDEN.glob("attn_bwd_*.npz") if "f32" not in p.stem)
TOL = {torch.float32: 2e-6, torch.bfloat16: 8e-3, torch.float16: 3e-3}


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    yield
    assert pmkl_b200.device_error(clear=True) == 0, "a kernel abandoned a bounded wait"


WORST = {}  # dtype name -> largest error relative to the gradient's max seen in this session


def assert_grad_close(got: np.ndarray, ref: np.ndarray, dtype, what: str) -> float:
    scale = max(float(np.abs(ref).max()), 1e-30)
    err = np.abs(got.astype(np.float64) - ref)
    key = str(dtype).replace("torch.", "")
    WORST[key] = max(WORST.get(key, 0.0), float(np.nanmax(err)) / scale)
    bound = TOL[dtype] * scale
    if dtype != torch.float32:
        mant = 7 if dtype == torch.bfloat16 else 10
        bound = bound + 0.5 * 2.0 ** (np.floor(np.log2(np.maximum(np.abs(ref), 1e-30))) - mant)
    bad = ~(err <= bound)
    if bad.any():
        i = np.unravel_index(np.argmax(np.where(np.isnan(err), np.inf, err / np.maximum(bound, 1e-30))), err.shape)
        raise AssertionError(f"{what}: {bad.sum()} values out of tolerance; worst at {i}: got {got[i]}, ref {ref[i]},"
                             f" rel-to-max err {float(err.max()) / scale:.3e}")
    return float(err.max()) / scale


def run_bwd(dout, q, k, v, m, l, causal, kernel=0, scale=0.0):
    """C ABI on CUDA copies; returns (dq, dk, dv) CUDA tensors."""
    t = [x.cuda().contiguous() for x in (dout, q, k, v, m, l)]
    out = [torch.empty_like(t[1]) for _ in range(3)]
    pmkl_b200.attention_bwd(*t, *out, causal, scale=scale, kernel=kernel)
    torch.cuda.synchronize()
    return out


def fwd_stats(q, k, v, causal, scale=0.0):
    """m, l from this library's forward in the inputs' dtype (what
    fused_self_attention_fw returns and autograd saves)."""
    qd, kd, vd = (x.cuda() for x in (q, k, v))
    B, H, S, D = q.shape
    o = torch.empty_like(qd)
    m = torch.empty(B, H, S, dtype=q.dtype, device="cuda")
    l = torch.empty_like(m)
    pmkl_b200.attention_fwd(qd, kd, vd, o, m, l, causal, scale=scale)
    torch.cuda.synchronize()
    return m.cpu(), l.cpu()


def check(dout, q, k, v, m, l, causal, dtype, what, kernel=0, scale=None):
    got = run_bwd(dout, q, k, v, m, l, causal, kernel=kernel, scale=scale or 0.0)
    ref = oracle.attention_bwd(np32(dout), np32(q), np32(k), np32(v), np32(m), np32(l), causal, scale=scale)
    return [assert_grad_close(np32(a), r, dtype, f"{what} {n}") for a, r, n in zip(got, ref, ("dq", "dk", "dv"))]


# ------------------------------------------------------------------ golden fixtures (reference outputs)
@pytest.mark.parametrize("name", BWD_F32)
def test_golden_fp32_against_reference(name):
    g = load_golden(name)
    t = [torch.from_numpy(g[x]) for x in ("do", "q", "k", "v", "m", "l")]
    got = run_bwd(*t, bool(g["causal"]))
    for a, key in zip(got, ("dq", "dk", "dv")):
        assert_grad_close(np32(a), g[key].astype(np.float64), torch.float32, f"{name} {key}")


@pytest.mark.parametrize("name", BWD_LP)
def test_golden_lowp_inputs(name):
    g = load_golden(name)
    dt = g["dtype"]
    t = [golden_tensor(g[x], dt) for x in ("do", "q", "k", "v", "m", "l")]
    check(*t, bool(g["causal"]), t[1].dtype, name)


@pytest.mark.parametrize("dtype", LP)
@pytest.mark.parametrize("name", BWD_F32)
def test_golden_inputs_rounded_tc(name, dtype):
    """The fp32 fixtures' inputs rounded to 16 bits (with the forward's m, l
    recomputed on them) through the tensor-core path when D allows."""
    g = load_golden(name)
    q, k, v, do = (torch.from_numpy(g[x]).to(dtype) for x in ("q", "k", "v", "do"))
    causal = bool(g["causal"])
    m, l = fwd_stats(q, k, v, causal)
    check(do, q, k, v, m, l, causal, dtype, name)


# ------------------------------------------------------------------ edge shapes, both paths
EDGE_S = [1, 2, 5, 64, 127, 128, 129, 200, 256, 257, 384, 515]


def seeded_bwd_inputs(B, H, S, D, dtype, seed, causal):
    q, k, v = seeded_qkv(B, H, S, D, dtype, seed=seed)
    g = torch.Generator().manual_seed(seed + 1)
    do = torch.randn(B, H, S, D, generator=g).to(dtype)
    m, l = fwd_stats(q, k, v, causal)
    return do, q, k, v, m, l


@pytest.mark.parametrize("dtype", LP)
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("S", EDGE_S)
def test_edge_shapes_tc(S, causal, D, dtype):
    t = seeded_bwd_inputs(1, 2, S, D, dtype, seed=S * 5 + D + int(causal), causal=causal)
    check(*t, causal, dtype, f"S{S} D{D} causal={causal}", kernel=TC)


@pytest.mark.parametrize("dtype", [torch.float32] + LP)
@pytest.mark.parametrize("D", [16, 48, 64, 96, 128, 200, 256])
@pytest.mark.parametrize("causal", [True, False])
def test_simt_head_sizes(D, causal, dtype):
    t = seeded_bwd_inputs(1, 3, 77, D, dtype, seed=D * 3 + int(causal), causal=causal)
    check(*t, causal, dtype, f"simt D{D}", kernel=SIMT)


@pytest.mark.parametrize("S", [33, 300])
def test_fp32_auto_path(S):
    t = seeded_bwd_inputs(2, 2, S, 64, torch.float32, seed=S, causal=True)
    check(*t, True, torch.float32, f"fp32 S{S}")


def test_custom_scale():
    q, k, v = seeded_qkv(1, 2, 300, 128, torch.bfloat16, seed=21)
    m, l = fwd_stats(q, k, v, True, scale=0.05)
    do = torch.randn(q.shape, generator=torch.Generator().manual_seed(22)).to(torch.bfloat16)
    check(do, q, k, v, m, l, True, torch.bfloat16, "scale 0.05", scale=0.05)


def test_stats_used_as_given():
    """p = exp(s - m) / l with the caller's m and l, whatever they are (the
    reference reads them as given, :91): shifted m and scaled l change the
    gradients exactly as the oracle says."""
    do, q, k, v, m, l = seeded_bwd_inputs(1, 2, 200, 128, torch.bfloat16, seed=23, causal=True)
    m2 = (m.float() + 0.75).to(torch.bfloat16)
    l2 = (l.float() * 3.0).to(torch.bfloat16)
    check(do, q, k, v, m2, l2, True, torch.bfloat16, "shifted stats")


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("S", [77, 640])
def test_delta_routes_agree(S, D):
    """delta from the persistent forward's epilogue (default) and from an fp32
    forward plus the row-statistics kernel (PMKL_ATTN_TCGEN05_SIMPLE) feed the
    same gradient kernels; both match the oracle and each other closely."""
    t = seeded_bwd_inputs(1, 2, S, D, torch.bfloat16, seed=40 + S + D, causal=True)
    a = run_bwd(*t, True, kernel=TC)
    b = run_bwd(*t, True, kernel=3)
    check(*t, True, torch.bfloat16, f"simple-delta S{S} D{D}", kernel=3)
    for x, y in zip(a, b):
        scale = y.float().abs().max().item()
        assert (x.float() - y.float()).abs().max().item() <= 1e-2 * scale


def test_tc_and_simt_agree():
    t = seeded_bwd_inputs(1, 2, 333, 128, torch.bfloat16, seed=24, causal=True)
    a = run_bwd(*t, True, kernel=TC)
    b = run_bwd(*t, True, kernel=SIMT)
    for x, y in zip(a, b):
        scale = y.float().abs().max().item()
        assert (x.float() - y.float()).abs().max().item() <= 2e-2 * scale


# ------------------------------------------------------------------ benchmark-sized slices
@pytest.mark.parametrize("D", [64, 128])
def test_long_sequence_one_slice(D):
    """S = 2048: many key/query tiles per CTA, ring stages wrap several times."""
    t = seeded_bwd_inputs(1, 1, 2048, D, torch.bfloat16, seed=25 + D, causal=True)
    check(*t, True, torch.bfloat16, f"S2048 D{D}")


def test_config3_shape_sampled_slice_and_determinism():
    """Config-3 shape (bf16 B16 H32 S4096 D128): the full backward on the GPU,
    one (b, h) slice against the oracle, and a second run bit-identical."""
    B, H, S, D = 16, 32, 4096, 128
    gen = torch.Generator(device="cuda").manual_seed(26)
    q, k, v, do = (torch.randn(B, H, S, D, generator=gen, device="cuda").to(torch.bfloat16) for _ in range(4))
    o = torch.empty_like(q)
    m = torch.empty(B, H, S, dtype=torch.bfloat16, device="cuda")
    l = torch.empty_like(m)
    pmkl_b200.attention_fwd(q, k, v, o, m, l, True)
    outs = []
    for _ in range(2):
        g = [torch.empty_like(q) for _ in range(3)]
        pmkl_b200.attention_bwd(do, q, k, v, m, l, *g, True)
        outs.append(g)
    torch.cuda.synchronize()
    for a, b in zip(*outs):
        assert torch.equal(a, b)
        assert torch.isfinite(a).all()
    b_, h_ = 5, 17
    sl = lambda t: t[b_:b_ + 1, h_:h_ + 1].cpu()  # noqa: E731
    ref = oracle.attention_bwd(*(np32(sl(t)) for t in (do, q, k, v, m, l)), True)
    for a, r, n in zip(outs[0], ref, ("dq", "dk", "dv")):
        assert_grad_close(np32(sl(a)), r, torch.bfloat16, f"config3 slice {n}")


# ------------------------------------------------------------------ argument errors
def test_errors():
    L = pmkl_b200.capi()
    q = torch.zeros(1, 1, 64, 64, dtype=torch.bfloat16, device="cuda")
    m = torch.zeros(1, 1, 64, dtype=torch.bfloat16, device="cuda")
    need = pmkl_b200.attention_bwd_workspace_size(1, 1, 64, 64, torch.bfloat16)
    ws = torch.empty(need + 512, dtype=torch.uint8, device="cuda")
    p = [q.data_ptr()] * 4 + [m.data_ptr()] * 2 + [q.data_ptr()] * 3

    def call(ws_ptr, ws_bytes, kernel=0, dtype=2):
        return L.pmkl_causal_attention_bwd_ex(*p, 1, 1, 64, 64, dtype, 1, 0.0, ws_ptr, ws_bytes, kernel, None)

    assert call(ws.data_ptr(), need - 1) == -9  # PMKL_ERR_WORKSPACE
    assert call(ws.data_ptr() + 16, need) == -4  # workspace not 256-byte aligned
    assert call(0, need) == -3
    assert call(ws.data_ptr(), need, kernel=4) == -5  # no such backward choice
    assert call(ws.data_ptr(), need, kernel=3, dtype=0) == -5  # fp32 has no tensor-core path
    assert call(ws.data_ptr(), need, kernel=TC, dtype=0) == -5  # fp32 has no tensor-core path
    assert call(ws.data_ptr(), need) == 0
    # the long route (PMKL_ATTN_TCGEN05_SIMPLE) needs its own, larger size
    need3 = pmkl_b200.attention_bwd_workspace_size(1, 1, 64, 64, torch.bfloat16, kernel=3)
    assert need3 > need
    ws3 = torch.empty(need3, dtype=torch.uint8, device="cuda")
    assert call(ws3.data_ptr(), need, kernel=3) == -9
    assert call(ws3.data_ptr(), need3, kernel=3) == 0
    torch.cuda.synchronize()
