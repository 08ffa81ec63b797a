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


# ------------------------------------------------------------------ backward: strided and grouped-query
def stats(q, k, v, causal):
    """m, l of this library's forward in the inputs' dtype (what autograd saves)."""
    _, m, l = run_strided(q, k, v, causal)
    return m, l


def run_bwd_strided(dout, q, k, v, m, l, causal, kernel=0, outs=None):
    dq, dk, dv = outs if outs is not None else (torch.empty(q.shape, dtype=q.dtype, device="cuda"),
                                                torch.empty(k.shape, dtype=k.dtype, device="cuda"),
                                                torch.empty(v.shape, dtype=v.dtype, device="cuda"))
    pmkl_b200.attention_bwd_strided(dout, q, k, v, m, l, dq, dk, dv, causal, kernel=kernel)
    torch.cuda.synchronize()
    return dq, dk, dv


def run_bwd_contiguous(dout, q, k, v, m, l, causal, kernel=0):
    t = [x.contiguous() for x in (dout, q, k, v, m, l)]
    out = [torch.empty_like(t[1]) for _ in range(3)]
    pmkl_b200.attention_bwd(*t, *out, causal, kernel=kernel)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("kernel,dtype,D", [(TC, torch.bfloat16, 128), (TC, torch.float16, 64),
                                            (SIMT, torch.float32, 64), (SIMT, torch.bfloat16, 96)])
@pytest.mark.parametrize("causal", [True, False])
def test_bwd_bshd_views_match_contiguous(kernel, dtype, D, causal):
    """The backward reads [B, S, H, D] views in place: bit for bit the same
    gradients as the same kernel on contiguous copies."""
    B, H, S = 2, 4, 300
    q, k, v, dout = (bshd_view(B, H, S, D, dtype, s) for s in (31, 32, 33, 34))
    m, l = stats(q, k, v, causal)
    got = run_bwd_strided(dout, q, k, v, m, l, causal, kernel=kernel)
    ref = run_bwd_contiguous(dout, q, k, v, m, l, causal, kernel=kernel)
    for a, b in zip(got, ref):
        assert torch.equal(a, b)


@pytest.mark.parametrize("kernel", [TC, SIMT])
def test_bwd_strided_gradients_written_in_place(kernel):
    B, H, S, D = 2, 3, 257, 128
    q, k, v, dout = (randn((B, H, S, D), torch.bfloat16, s) for s in (35, 36, 37, 38))
    m, l = stats(q, k, v, True)
    bufs = [torch.empty(B, S, H, D, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    run_bwd_strided(dout, q, k, v, m, l, True, kernel=kernel, outs=[t.transpose(1, 2) for t in bufs])
    ref = run_bwd_contiguous(dout, q, k, v, m, l, True, kernel=kernel)
    for a, b in zip(bufs, ref):
        assert torch.equal(a.transpose(1, 2), b)


def group_oracle(dout, q, k, v, m, l, causal, g):
    """Oracle gradients of grouped-query attention: the ordinary backward on
    K/V repeated over each group, dk and dv summed over the group's heads."""
    rk, rv = (np32(t).repeat(g, axis=1) for t in (k, v))
    dq, dk, dv = oracle.attention_bwd(np32(dout), np32(q), rk, rv, np32(m), np32(l), causal)
    B, H, S, D = dq.shape
    return dq, dk.reshape(B, H // g, g, S, D).sum(2), dv.reshape(B, H // g, g, S, D).sum(2)


def assert_grads_close(got, ref, dtype, what):
    from test_attention_bwd_gpu import assert_grad_close
    for a, r, n in zip(got, ref, ("dq", "dk", "dv")):
        assert_grad_close(np32(a), r, dtype, f"{what} {n}")


@pytest.mark.parametrize("kernel,dtype,D", [(TC, torch.bfloat16, 128), (TC, torch.float16, 64),
                                            (SIMT, torch.float32, 64), (SIMT, torch.bfloat16, 96)])
@pytest.mark.parametrize("kv_heads", [1, 2])
def test_bwd_grouped_query_against_oracle(kv_heads, kernel, dtype, D):
    """Grouped-query backward: dk, dv of each K/V head are the sums over its
    query heads (formed in fp32 inside the kernel); checked against the
    oracle on repeated K/V with the backward tests' tolerances."""
    B, H, S = 1, 4, 200
    g = H // kv_heads
    q, dout = (randn((B, H, S, D), dtype, s) for s in (40, 41))
    k, v = (bshd_view(B, kv_heads, S, D, dtype, s) for s in (42, 43))
    m, l = stats(q, k, v, True)
    got = run_bwd_strided(dout, q, k, v, m, l, True, kernel=kernel)
    ref = group_oracle(dout, q, k, v, m, l, True, g)
    assert_grads_close(got, ref, dtype, f"gqa kv_heads={kv_heads}")
    # dq reads the shared K/V exactly as the repeated form does: bit for bit.
    rep = run_bwd_contiguous(dout, q, k.repeat_interleave(g, dim=1), v.repeat_interleave(g, dim=1), m, l, True,
                             kernel=kernel)
    assert torch.equal(got[0], rep[0])


@pytest.mark.parametrize("D", [64, 128])
def test_bwd_grouped_query_long_sequence(D):
    """Several query tiles per head and a ring that wraps across the group's
    heads in the dK/dV kernel (S = 1024, 4 query heads per K/V head)."""
    B, H, Hkv, S = 1, 8, 2, 1024
    q, dout = (randn((B, H, S, D), torch.bfloat16, s) for s in (44, 45))
    k, v = (randn((B, Hkv, S, D), torch.bfloat16, s) for s in (46, 47))
    m, l = stats(q, k, v, True)
    got = run_bwd_strided(dout, q, k, v, m, l, True, kernel=TC)
    ref = group_oracle(dout, q, k, v, m, l, True, H // Hkv)
    assert_grads_close(got, ref, torch.bfloat16, f"gqa S1024 D{D}")


def test_bwd_strided_errors():
    import ctypes
    L = pmkl_b200.capi()
    f = 0x10000
    s = (ctypes.c_int64 * 3)(64 * 8 * 128, 128, 8 * 128)
    neg = (ctypes.c_int64 * 3)(1, -1, 1)

    def call(heads=8, kv=2, st=s, kernel=0):
        return L.pmkl_causal_attention_bwd_strided(*([f] * 9), 1, heads, kv, 64, 128, st, st, st, st, st, st, st, 2,
                                                   1, 0.0, f, 1 << 20, kernel, None)

    assert call(kv=3) == -1  # kv_heads must divide heads
    assert call(kv=0) == -1
    assert call(st=neg) == -1
    q, dout = (randn((1, 4, 64, 64), torch.bfloat16, s) for s in (48, 49))
    k, v = (randn((1, 2, 64, 64), torch.bfloat16, s) for s in (50, 51))
    m, l = stats(q, k, v, True)
    with pytest.raises(pmkl_b200.PmklError, match="UNSUPPORTED"):
        run_bwd_strided(dout, q, k, v, m, l, True, kernel=3)  # the long route takes equal heads only


def test_bwd_unaligned_row_stride_takes_cuda_core_path():
    B, H, S, D = 1, 2, 130, 64
    base = randn((B, H, S, D + 1), torch.bfloat16, 52)
    q = base[..., :D]
    k, v, dout = (randn((B, H, S, D), torch.bfloat16, s) for s in (53, 54, 55))
    m, l = stats(q, k, v, True)
    got = run_bwd_strided(dout, q, k, v, m, l, True)
    ref = run_bwd_contiguous(dout, q, k, v, m, l, True, kernel=SIMT)
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    with pytest.raises(pmkl_b200.PmklError, match="UNSUPPORTED"):
        run_bwd_strided(dout, q, k, v, m, l, True, kernel=TC)


def test_extension_backward_reads_views_without_copies():
    B, H, S, D = 2, 16, 1024, 128
    q, k, v, dout = (bshd_view(B, H, S, D, torch.bfloat16, s) for s in (56, 57, 58, 59))
    _, m, l = pmkl_pytorch_ext.fused_self_attention_fw(q, k, v, True)
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    dq, dk, dv = pmkl_pytorch_ext.fused_self_attention_bw(dout, q, k, v, m, l, True)
    torch.cuda.synchronize()
    grads = 3 * q.numel() * q.element_size()
    ws = pmkl_b200.attention_bwd_workspace_size(B, H, S, D, torch.bfloat16)
    assert torch.cuda.max_memory_allocated() - before <= grads + ws + (1 << 20)  # no input copies
    assert dq.stride() == q.stride()  # gradients in their inputs' layout
    ref = run_bwd_contiguous(dout, q, k, v, m, l, True)
    for a, b in zip((dq, dk, dv), ref):
        assert torch.equal(a, b)


def test_autograd_grouped_query():
    """fused_self_attention_ex: autograd through grouped-query K/V views."""
    from pmkl_function import fused_self_attention_ex
    B, H, Hkv, S, D = 1, 8, 2, 256, 128
    q = randn((B, H, S, D), torch.bfloat16, 60).requires_grad_()
    k, v = (bshd_view(B, Hkv, S, D, torch.bfloat16, s).detach().requires_grad_() for s in (61, 62))
    out, m, l = fused_self_attention_ex(q, k, v, True)
    dout = randn(out.shape, torch.bfloat16, 63)
    out.backward(dout)
    assert q.grad.shape == q.shape and k.grad.shape == k.shape and v.grad.shape == v.shape
    ref = group_oracle(dout, q.detach(), k.detach(), v.detach(), m, l, True, H // Hkv)
    assert_grads_close((q.grad, k.grad, v.grad), ref, torch.bfloat16, "autograd gqa")
    fo, _, _ = oracle.attention_fwd(np32(q), np32(k).repeat(H // Hkv, axis=1), np32(v).repeat(H // Hkv, axis=1), True)
    assert abs(np32(out) - fo).max() <= 2e-3 + 2.0 ** -8 * abs(fo).max()


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("S", [1, 77, 300])
def test_bwd_multi_query_ragged(S, causal):
    """Multi-query (one K/V head for 8 query heads), ragged and tiny S, causal
    and not: the dK/dV kernel's group loop over partial tiles."""
    B, H, D = 2, 8, 128
    q, dout = (randn((B, H, S, D), torch.bfloat16, s) for s in (70, 71))
    k, v = (randn((B, 1, S, D), torch.bfloat16, s) for s in (72, 73))
    m, l = stats(q, k, v, causal)
    got = run_bwd_strided(dout, q, k, v, m, l, causal)
    ref = group_oracle(dout, q, k, v, m, l, causal, H)
    assert_grads_close(got, ref, torch.bfloat16, f"mqa S{S} causal={causal}")


def test_extension_grouped_query_backward_entry():
    """fused_self_attention_bw_ex with fewer K/V heads returns dk, dv with k's
    and v's shape (fp16, head size 64, [B, S, H, D] views)."""
    B, H, Hkv, S, D = 2, 6, 3, 333, 64
    q, dout = (bshd_view(B, H, S, D, torch.float16, s) for s in (74, 75))
    k, v = (bshd_view(B, Hkv, S, D, torch.float16, s) for s in (76, 77))
    out, m, l = pmkl_pytorch_ext.fused_self_attention_fw_ex(q, k, v, True)
    dq, dk, dv = pmkl_pytorch_ext.fused_self_attention_bw_ex(dout, q, k, v, m, l, True)
    assert dq.shape == q.shape and dk.shape == k.shape and dv.shape == v.shape
    ref = group_oracle(dout, q, k, v, m, l, True, H // Hkv)
    assert_grads_close((dq, dk, dv), ref, torch.float16, "ext gqa")
    with pytest.raises(RuntimeError, match="shapes must match"):
        pmkl_pytorch_ext.fused_self_attention_bw(dout, q, k, v, m, l, True)  # reference API: equal heads only
