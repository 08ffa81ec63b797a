"""GPU tests of the reference-facing Python API: pmkl_pytorch_ext and
pmkl_function.fused_self_attention, in the manner of the reference's own test
(pmkl_pytorch_ext/test/test_fused_self_attention.py), which compares against
torch's scaled_dot_product_attention -- with assertions added (the reference
only prints the differences), and the C++ drop-in shim."""
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import pmkl_b200
import pmkl_pytorch_ext
from helpers import assert_f32_close, assert_lp_close, attention_capi, np32, seeded_qkv
from pmkl_function import fused_self_attention

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("is_causal", [False, True])
@pytest.mark.parametrize("hidden_size", [64, 128])
@pytest.mark.parametrize("batch_size", [2, 3])
def test_reference_test_shapes_vs_sdpa(batch_size, hidden_size, is_causal, dtype):
    """Shapes of test_fused_self_attention.py:10-14 (H=16, S=128)."""
    q, k, v = seeded_qkv(batch_size, 16, 128, hidden_size, dtype, seed=batch_size * 1000 + hidden_size + is_causal)
    out, out_m, out_l = fused_self_attention(q.cuda(), k.cuda(), v.cuda(), is_causal)
    assert out.dtype == dtype and out_m.dtype == dtype and out_l.dtype == dtype
    assert out.shape == q.shape and out_m.shape == q.shape[:3] and out_l.shape == q.shape[:3]
    ref = F.scaled_dot_product_attention(q.double(), k.double(), v.double(), is_causal=is_causal).numpy()
    if dtype == torch.float32:
        assert_f32_close(np32(out), ref, "out")
    else:
        assert_lp_close(np32(out), ref, dtype, "out")


def test_matches_capi_bitwise_and_debug_flag_ignored():
    q, k, v = seeded_qkv(2, 4, 300, 128, torch.bfloat16, seed=1)
    a = fused_self_attention(q.cuda(), k.cuda(), v.cuda(), True, True)
    b = attention_capi(q, k, v, True)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_noncontiguous_inputs():
    q, k, v = seeded_qkv(2, 256, 4, 64, torch.bfloat16, seed=2)  # [B, S, H, D]
    qt, kt, vt = (t.cuda().transpose(1, 2) for t in (q, k, v))  # [B, H, S, D] views
    assert not qt.is_contiguous()
    out, m, l = pmkl_pytorch_ext.fused_self_attention_fw(qt, kt, vt, True)
    ref = attention_capi(qt.contiguous(), kt.contiguous(), vt.contiguous(), True)
    assert torch.equal(out, ref[0]) and torch.equal(m, ref[1]) and torch.equal(l, ref[2])


def test_current_stream_is_used():
    q, k, v = seeded_qkv(1, 8, 2048, 128, torch.bfloat16, seed=3)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        out, m, l = pmkl_pytorch_ext.fused_self_attention_fw(qd, kd, vd, True)
    s.synchronize()
    ref = attention_capi(q, k, v, True)
    assert torch.equal(out, ref[0])


def test_fw_ex_fp32_outputs_and_kernels():
    q, k, v = seeded_qkv(1, 2, 200, 64, torch.float16, seed=4)
    o1, m1, l1 = pmkl_pytorch_ext.fused_self_attention_fw_ex(q.cuda(), k.cuda(), v.cuda(), True, out_fp32=True,
                                                             kernel=pmkl_pytorch_ext.KERNEL_TCGEN05)
    o2, m2, l2 = pmkl_pytorch_ext.fused_self_attention_fw_ex(q.cuda(), k.cuda(), v.cuda(), True, out_fp32=True,
                                                             kernel=pmkl_pytorch_ext.KERNEL_SIMT)
    assert o1.dtype == torch.float32
    assert (o1 - o2).abs().max().item() < 2e-3


def test_errors():
    q = torch.randn(1, 2, 8, 64, device="cuda")
    with pytest.raises(RuntimeError, match="shapes must match"):
        pmkl_pytorch_ext.fused_self_attention_fw(q, q[:, :, :4], q, True)
    with pytest.raises(RuntimeError, match="unsupported dtype"):
        pmkl_pytorch_ext.fused_self_attention_fw(q.double(), q.double(), q.double(), True)
    with pytest.raises(RuntimeError, match="same dtype"):
        pmkl_pytorch_ext.fused_self_attention_fw(q, q.half(), q, True)
    with pytest.raises(RuntimeError, match="CUDA"):
        pmkl_pytorch_ext.fused_self_attention_fw(q, q.cpu(), q, True)
    with pytest.raises(RuntimeError, match="UNSUPPORTED"):
        pmkl_pytorch_ext.fused_self_attention_fw(*(torch.zeros(1, 1, 4, 300, device="cuda"),) * 3, True)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("is_causal", [False, True])
@pytest.mark.parametrize("hidden_size", [64, 128])
def test_backward_through_autograd_vs_sdpa(hidden_size, is_causal, dtype):
    """The reference's test also backpropagates through both implementations
    and compares q/k/v gradients (test_fused_self_attention.py:21-38); here the
    reference side is float64 autograd through scaled_dot_product_attention,
    with a bound per dtype."""
    q, k, v = seeded_qkv(2, 16, 128, hidden_size, dtype, seed=hidden_size + 7 * is_causal)
    g = torch.Generator().manual_seed(9)
    dout = torch.randn(q.shape, generator=g).to(dtype)
    qd, kd, vd = (t.cuda().requires_grad_() for t in (q, k, v))
    out, _, _ = fused_self_attention(qd, kd, vd, is_causal)
    out.backward(dout.cuda())
    q64, k64, v64 = (t.double().requires_grad_() for t in (q, k, v))
    F.scaled_dot_product_attention(q64, k64, v64, is_causal=is_causal).backward(dout.double())
    # fp32: the reference's all_close scale.  16-bit: out_m and out_l come back
    # in the 16-bit dtype (as the reference returns them) and the backward uses
    # them as given, so each P entry is off exact math by up to (|m| + 1) 2^-8
    # relative; P, dS and the gradients are also rounded to 16 bits.
    tol = 2e-5 if dtype == torch.float32 else 3e-2
    for got, ref in ((qd.grad, q64.grad), (kd.grad, k64.grad), (vd.grad, v64.grad)):
        assert got.dtype == dtype
        err = (got.double().cpu() - ref).abs().max().item()
        assert err <= tol * ref.abs().max().item(), (err, ref.abs().max().item())


def test_bw_matches_capi_bitwise():
    q, k, v = (t.cuda() for t in seeded_qkv(1, 4, 300, 128, torch.bfloat16, seed=5))
    out, m, l = pmkl_pytorch_ext.fused_self_attention_fw(q, k, v, True)
    dout = torch.randn_like(out)
    dq, dk, dv = pmkl_pytorch_ext.fused_self_attention_bw(dout, q, k, v, m, l, True)
    ref = [torch.empty_like(q) for _ in range(3)]
    pmkl_b200.attention_bwd(dout, q, k, v, m, l, *ref, True)
    torch.cuda.synchronize()
    for a, b in zip((dq, dk, dv), ref):
        assert torch.equal(a, b)


def test_bw_errors():
    q = torch.randn(1, 2, 8, 64, device="cuda")
    m = torch.zeros(1, 2, 8, device="cuda")
    with pytest.raises(RuntimeError, match="shapes must match"):
        pmkl_pytorch_ext.fused_self_attention_bw(q, q, q[:, :1], q[:, :1], m, m, True)  # reference API: equal heads
    with pytest.raises(RuntimeError, match="v's dtype"):
        pmkl_pytorch_ext.fused_self_attention_bw(q, q, q, q, m.half(), m, True)
    with pytest.raises(RuntimeError, match="batch, heads, seq"):
        pmkl_pytorch_ext.fused_self_attention_bw(q, q, q, q, m[:, :1], m, True)
    with pytest.raises(RuntimeError, match="CUDA"):
        pmkl_pytorch_ext.fused_self_attention_bw(q, q.cpu(), q.cpu(), q.cpu(), m, m, True)


def test_bw_strided_hidden_dimension_is_copied():
    """A strided hidden dimension (here a transposed last pair of axes) is
    made contiguous before the call, as the reference makes every input
    contiguous (fused_self_attention.cpp:179); the result matches."""
    q = torch.randn(1, 2, 64, 64, device="cuda")
    qt = q.transpose(2, 3).contiguous().transpose(2, 3)
    assert qt.stride(3) != 1
    m = torch.zeros(1, 2, 64, device="cuda")
    l = torch.ones(1, 2, 64, device="cuda")
    a = pmkl_pytorch_ext.fused_self_attention_bw(q, qt, q, q, m, l, True)
    b = pmkl_pytorch_ext.fused_self_attention_bw(q, q, q, q, m, l, True)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_empty_inputs():
    q = torch.empty(0, 4, 16, 64, device="cuda", dtype=torch.bfloat16)
    out, m, l = pmkl_pytorch_ext.fused_self_attention_fw(q, q, q, True)
    assert out.shape == q.shape and m.shape == (0, 4, 16)
    q = torch.empty(2, 4, 0, 64, device="cuda", dtype=torch.bfloat16)
    out, m, l = pmkl_pytorch_ext.fused_self_attention_fw(q, q, q, True)
    assert out.shape == q.shape


def test_cpp_shim_program(tmp_path):
    """Builds tests/cpp/shim_test.cpp against the shim headers, the library and
    the oracle, then runs it (it prints "ok")."""
    from oracle import oracle

    oracle.build()
    exe = tmp_path / "shim_test"
    cuda = Path("/usr/local/cuda")
    subprocess.run(["g++", "-std=c++17", "-O2", f"-I{REPO / 'include'}", f"-I{cuda / 'include'}",
                    str(REPO / "tests" / "cpp" / "shim_test.cpp"), str(oracle.LIB_PATH),
                    f"-L{pmkl_b200.LIB_PATH.parent}", "-lpmkl_b200", f"-Wl,-rpath,{pmkl_b200.LIB_PATH.parent}",
                    f"-Wl,-rpath,{oracle.LIB_PATH.parent}", f"-L{cuda / 'lib64'}", "-lcudart", "-o", str(exe)],
                   check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip().endswith("ok")
