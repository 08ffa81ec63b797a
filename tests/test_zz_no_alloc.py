"""GPU tests of pmkl_causal_attention_bwd_static, the backward entry point that
uses the library's static device scratch instead of a caller workspace.

The file name sorts last, so in a full run these tests execute after every
other test has used the device (and its caching allocator); they also pass on
their own.  Each compares the static entry point with
pmkl_causal_attention_bwd (caller workspace) on the same inputs, bit for bit,
over several calls in a row."""
import gc

import pytest
import torch

import pmkl_b200
from helpers import seeded_qkv

pytestmark = pytest.mark.gpu

STATIC_BYTES = 64 << 20  # PMKL_BWD_STATIC_SCRATCH_BYTES
CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    yield
    assert pmkl_b200.device_error(clear=True) == 0, "a kernel abandoned a bounded wait"


def make_problem(B, H, S, D, dtype, seed, causal):
    q, k, v = (t.cuda() for t in seeded_qkv(B, H, S, D, dtype, seed=seed))
    do = torch.randn(q.shape, generator=torch.Generator().manual_seed(seed + 1)).to(dtype).cuda()
    o = torch.empty_like(q)
    m = torch.empty(B, H, S, dtype=dtype, device="cuda")
    l = torch.empty_like(m)
    pmkl_b200.attention_fwd(q, k, v, o, m, l, causal)
    return do, q, k, v, m, l


def make_problem_on_device(B, H, S, D, dtype, seed, causal):
    """As make_problem, with the inputs drawn on the device (large sizes)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v, do = (torch.randn(B, H, S, D, generator=g, device="cuda").to(dtype) for _ in range(4))
    o = torch.empty_like(q)
    m = torch.empty(B, H, S, dtype=dtype, device="cuda")
    l = torch.empty_like(m)
    pmkl_b200.attention_fwd(q, k, v, o, m, l, causal)
    return do, q, k, v, m, l


def bwd_static(do, q, k, v, m, l, causal):
    grads = [torch.empty_like(q) for _ in range(3)]
    B, H, S, D = q.shape
    rc = pmkl_b200.capi().pmkl_causal_attention_bwd_static(
        *(t.data_ptr() for t in (do, q, k, v, m, l)), *(g.data_ptr() for g in grads), B, H, S, D, CODE[q.dtype],
        int(causal), 0.0, torch.cuda.current_stream().cuda_stream)
    return rc, grads


def bwd_workspace(do, q, k, v, m, l, causal):
    grads = [torch.empty_like(q) for _ in range(3)]
    pmkl_b200.attention_bwd(do, q, k, v, m, l, *grads, causal)
    return grads


CASES = [
    # (B, H, S, D, dtype, seed, causal): tensor-core path, both head sizes, ragged S; CUDA-core path (fp32, D=96)
    (1, 4, 300, 128, torch.bfloat16, 1, True),
    (2, 2, 513, 64, torch.float16, 2, False),
    (1, 2, 1024, 128, torch.bfloat16, 3, True),
    (1, 3, 77, 64, torch.float32, 4, True),
    (1, 2, 130, 96, torch.bfloat16, 5, False),
]


def test_static_matches_workspace_entry_over_consecutive_calls():
    problems = [make_problem(*c) for c in CASES]
    for _ in range(2):  # every case twice, back to back on one stream
        for c, p in zip(CASES, problems):
            rc, got = bwd_static(*p, c[6])
            assert rc == 0, pmkl_b200.capi().pmkl_status_string(rc)
            ref = bwd_workspace(*p, c[6])
            torch.cuda.synchronize()
            for a, b in zip(got, ref):
                assert torch.equal(a, b), c


def test_two_static_calls_in_a_row_before_reading():
    """Two calls enqueued back to back on one stream: the second reuses the
    scratch only after the first's kernels are done, so both results hold."""
    pa = make_problem(*CASES[0])
    pb = make_problem(*CASES[2])
    rca, ga = bwd_static(*pa, True)
    rcb, gb = bwd_static(*pb, True)
    assert rca == 0 and rcb == 0
    ra = bwd_workspace(*pa, True)
    rb = bwd_workspace(*pb, True)
    torch.cuda.synchronize()
    for a, b in zip(ga + gb, ra + rb):
        assert torch.equal(a, b)


def test_no_device_memory_is_allocated():
    p = make_problem(*CASES[1])
    rc, first = bwd_static(*p, False)  # first call: module and scratch address set-up
    assert rc == 0
    torch.cuda.synchronize()
    grads = [torch.empty_like(p[1]) for _ in range(3)]
    # torch's allocator counters of this process (the device-wide free memory
    # would also move with other processes on a shared GPU).  Tensors left
    # unreachable by earlier tests are collected first, and the collector is
    # off during the calls, so that only these calls could move the counters.
    gc.collect()
    gc.disable()
    try:
        alloc0 = torch.cuda.memory_allocated()
        reserved0 = torch.cuda.memory_reserved()
        B, H, S, D = p[1].shape
        for _call in range(3):
            rc = pmkl_b200.capi().pmkl_causal_attention_bwd_static(
                *(t.data_ptr() for t in p), *(g.data_ptr() for g in grads), B, H, S, D, CODE[p[1].dtype], 0, 0.0,
                torch.cuda.current_stream().cuda_stream)
            assert rc == 0
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated() == alloc0 and torch.cuda.memory_reserved() == reserved0
    finally:
        gc.enable()
    for a, b in zip(first, grads):  # the calls also agree with each other
        assert torch.equal(a, b)


def test_oversize_problem_is_rejected_without_launch():
    """The tensor-core route needs 8 bytes per row at a row pitch of seq
    rounded up to 128: 2049 slices of 4096 rows exceed the 64 MiB scratch and
    are refused before any launch; 2048 slices fill it exactly and run."""
    B, S, D = 1, 4096, 64
    assert pmkl_b200.attention_bwd_workspace_size(B, 2049, S, D, torch.bfloat16) > STATIC_BYTES
    x = torch.zeros(1, dtype=torch.bfloat16, device="cuda")
    ptr = x.data_ptr()
    rc = pmkl_b200.capi().pmkl_causal_attention_bwd_static(*([ptr] * 9), B, 2049, S, D, 2, 1, 0.0, None)
    assert rc == -9  # PMKL_ERR_WORKSPACE
    H_fit = 2048
    assert pmkl_b200.attention_bwd_workspace_size(B, H_fit, S, D, torch.bfloat16) == STATIC_BYTES
    p = make_problem_on_device(B, H_fit, S, D, torch.bfloat16, 7, True)
    rc, got = bwd_static(*p, True)
    assert rc == 0, pmkl_b200.capi().pmkl_status_string(rc)
    ref = bwd_workspace(*p, True)
    torch.cuda.synchronize()
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    del p, got, ref
    torch.cuda.empty_cache()


def test_config3_size_runs_from_the_static_scratch():
    """BASELINE config 3's shape (bf16 B16 H32 S4096 D128) needs 16 MiB of
    row statistics and runs from the static scratch, bit for bit like the
    workspace entry point, twice in a row."""
    p = make_problem_on_device(16, 32, 4096, 128, torch.bfloat16, 8, True)
    ref = bwd_workspace(*p, True)
    for _ in range(2):
        rc, got = bwd_static(*p, True)
        assert rc == 0, pmkl_b200.capi().pmkl_status_string(rc)
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert torch.equal(a, b)
    del p, got, ref
    torch.cuda.empty_cache()


def test_argument_errors_match_workspace_entry():
    L = pmkl_b200.capi()
    f = 0x10000
    assert L.pmkl_causal_attention_bwd_static(*([f] * 9), -1, 1, 8, 64, 2, 1, 0.0, None) == -1
    assert L.pmkl_causal_attention_bwd_static(*([f] * 9), 1, 1, 8, 64, 7, 1, 0.0, None) == -2
    assert L.pmkl_causal_attention_bwd_static(*([0] * 9), 0, 1, 8, 64, 2, 1, 0.0, None) == 0
    assert L.pmkl_causal_attention_bwd_static(*([f] * 9), 1, 1, 8, 300, 2, 1, 0.0, None) == -5
    assert L.pmkl_causal_attention_bwd_static(*([0] * 9), 1, 1, 8, 64, 2, 1, 0.0, None) == -3
