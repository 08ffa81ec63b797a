"""GPU tests of strided and grouped-query inputs (pmkl_causal_attention_fwd_strided
and the torch binding reading views in place).  Each strided or grouped run
is compared bit for bit with the same kernel on contiguous / repeated-K/V
copies of the same data, which the oracle-based tests already cover; one
grouped case is also checked against the oracle directly."""
import pytest
import torch

import pmkl_b200
import pmkl_pytorch_ext
from helpers import attention_capi, np32
from oracle import oracle
from pmkl_function import fused_self_attention

pytestmark = pytest.mark.gpu

TC = pmkl_b200.KERNEL_TCGEN05
SIMT = pmkl_b200.KERNEL_SIMT


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    yield
    assert pmkl_b200.device_error(clear=True) == 0, "a kernel abandoned a bounded wait"


def randn(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g).to(dtype).cuda()


def outputs(B, H, S, D, dtype, out_dtype=None):
    od = out_dtype or dtype
    return (torch.empty(B, H, S, D, dtype=od, device="cuda"), torch.empty(B, H, S, dtype=od, device="cuda"),
            torch.empty(B, H, S, dtype=od, device="cuda"))


def run_strided(q, k, v, causal, kernel=0, o=None, out_dtype=None):
    B, H, S, D = q.shape
    o_, m, l = outputs(B, H, S, D, q.dtype, out_dtype)
    o = o_ if o is None else o
    pmkl_b200.attention_fwd_strided(q, k, v, o, m, l, causal, kernel=kernel)
    torch.cuda.synchronize()
    return o, m, l


def bshd_view(B, H, S, D, dtype, seed):
    """A [B, S, H, D] tensor seen as [B, H, S, D] (the layout most models keep)."""
    return randn((B, S, H, D), dtype, seed).transpose(1, 2)


@pytest.mark.parametrize("kernel,dtype,D", [(TC, torch.bfloat16, 128), (TC, torch.float16, 64),
                                            (SIMT, torch.float32, 64), (SIMT, torch.bfloat16, 96)])
@pytest.mark.parametrize("causal", [True, False])
def test_bshd_views_match_contiguous(kernel, dtype, D, causal):
    B, H, S = 2, 4, 300
    q, k, v = (bshd_view(B, H, S, D, dtype, s) for s in (1, 2, 3))
    assert not q.is_contiguous()
    got = run_strided(q, k, v, causal, kernel=kernel)
    ref = attention_capi(q.contiguous(), k.contiguous(), v.contiguous(), causal, kernel=kernel)
    for a, b in zip(got, ref):
        assert torch.equal(a, b)


@pytest.mark.parametrize("kernel", [TC, SIMT])
def test_strided_output(kernel):
    B, H, S, D = 2, 3, 257, 128
    q, k, v = (randn((B, H, S, D), torch.bfloat16, s) for s in (4, 5, 6))
    o_bshd = torch.empty(B, S, H, D, dtype=torch.bfloat16, device="cuda")
    o, m, l = run_strided(q, k, v, True, kernel=kernel, o=o_bshd.transpose(1, 2))
    ref = attention_capi(q, k, v, True, kernel=kernel)
    assert torch.equal(o_bshd.transpose(1, 2), ref[0]) and torch.equal(m, ref[1]) and torch.equal(l, ref[2])


@pytest.mark.parametrize("kernel", [TC, SIMT])
def test_strided_fp32_output(kernel):
    B, H, S, D = 1, 2, 200, 64
    q, k, v = (bshd_view(B, H, S, D, torch.float16, s) for s in (7, 8, 9))
    o_bshd = torch.empty(B, S, H, D, dtype=torch.float32, device="cuda")
    o, m, l = run_strided(q, k, v, True, kernel=kernel, o=o_bshd.transpose(1, 2), out_dtype=torch.float32)
    ref = attention_capi(q.contiguous(), k.contiguous(), v.contiguous(), True, out_fp32=True, kernel=kernel)
    assert torch.equal(o_bshd.transpose(1, 2), ref[0]) and torch.equal(m, ref[1])


@pytest.mark.parametrize("kernel", [TC, SIMT])
@pytest.mark.parametrize("kv_heads", [1, 2, 4])
@pytest.mark.parametrize("D", [64, 128])
def test_grouped_query_matches_repeated_kv(kv_heads, D, kernel):
    B, H, S = 2, 8, 384
    q = randn((B, H, S, D), torch.bfloat16, 10)
    k = randn((B, kv_heads, S, D), torch.bfloat16, 11)
    v = randn((B, kv_heads, S, D), torch.bfloat16, 12)
    got = run_strided(q, k, v, True, kernel=kernel)
    g = H // kv_heads
    ref = attention_capi(q, k.repeat_interleave(g, dim=1), v.repeat_interleave(g, dim=1), True, kernel=kernel)
    for a, b in zip(got, ref):
        assert torch.equal(a, b)


def test_grouped_query_against_oracle():
    B, H, Hkv, S, D = 1, 4, 2, 200, 128
    q = randn((B, H, S, D), torch.float16, 13)
    k, v = (bshd_view(B, Hkv, S, D, torch.float16, s) for s in (14, 15))
    o, m, l = run_strided(q, k, v, True)
    ro, rm, _ = oracle.attention_fwd(np32(q), np32(k.repeat_interleave(2, dim=1)), np32(v.repeat_interleave(2, dim=1)),
                                     True)
    assert abs(np32(o) - ro).max() <= 2e-3 + 2.0 ** -11
    assert abs(np32(m) - rm).max() <= 2e-3 + 2.0 ** -11 * abs(rm).max()


def test_unaligned_row_stride_takes_cuda_core_path():
    """Rows padded to D + 1 elements: not a 16-byte multiple, so the CUDA-core
    kernel runs (the tensor-core kernel is refused if asked for)."""
    B, H, S, D = 1, 2, 130, 64
    base = randn((B, H, S, D + 1), torch.bfloat16, 16)
    q = base[..., :D]
    k, v = (randn((B, H, S, D), torch.bfloat16, s) for s in (17, 18))
    got = run_strided(q, k, v, True)
    ref = attention_capi(q.contiguous(), k, v, True, kernel=SIMT)
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    with pytest.raises(pmkl_b200.PmklError, match="UNSUPPORTED"):
        run_strided(q, k, v, True, kernel=TC)


def test_extension_reads_views_without_copies():
    B, H, S, D = 2, 16, 1024, 128
    q, k, v = (bshd_view(B, H, S, D, torch.bfloat16, s) for s in (19, 20, 21))
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    out, m, l = pmkl_pytorch_ext.fused_self_attention_fw(q, k, v, True)
    torch.cuda.synchronize()
    outputs_bytes = out.numel() * out.element_size() + 2 * m.numel() * m.element_size()
    assert torch.cuda.max_memory_allocated() - before <= outputs_bytes + (1 << 20)  # no input copies
    ref = attention_capi(q.contiguous(), k.contiguous(), v.contiguous(), True)
    assert torch.equal(out, ref[0])


def test_extension_grouped_query_entry():
    B, H, S, D = 1, 8, 256, 64
    q = randn((B, H, S, D), torch.float16, 22)
    k, v = (randn((B, 2, S, D), torch.float16, s) for s in (23, 24))
    out, m, l = pmkl_pytorch_ext.fused_self_attention_fw_ex(q, k, v, True)
    ref = attention_capi(q, k.repeat_interleave(4, dim=1), v.repeat_interleave(4, dim=1), True)
    assert torch.equal(out, ref[0])
    with pytest.raises(RuntimeError, match="shapes must match"):
        pmkl_pytorch_ext.fused_self_attention_fw(q, k, v, True)  # the reference API takes equal shapes only
    with pytest.raises(RuntimeError, match="shapes must match"):
        pmkl_pytorch_ext.fused_self_attention_fw_ex(q, k[:, :1].expand(1, 3, S, D), v[:, :1].expand(1, 3, S, D), True)


def test_autograd_through_views():
    B, H, S, D = 1, 4, 256, 64
    q, k, v = (bshd_view(B, H, S, D, torch.bfloat16, s).requires_grad_() for s in (25, 26, 27))
    out, _, _ = fused_self_attention(q, k, v, True)
    dout = randn(out.shape, torch.bfloat16, 28)
    out.backward(dout)
    q2, k2, v2 = (t.detach().contiguous().requires_grad_() for t in (q, k, v))
    out2, _, _ = fused_self_attention(q2, k2, v2, True)
    out2.backward(dout)
    assert torch.equal(out, out2)
    for a, b in ((q.grad, q2.grad), (k.grad, k2.grad), (v.grad, v2.grad)):
        assert torch.equal(a, b)
