"""GPU tests of the failure path behind every bounded wait.

Each tensor-core kernel bounds its mbarrier waits; when one runs out the CTA
raises its abort flag, drains its own copies and tensor-core work, frees
tensor memory and sets the device error word, and CTAs of later launches that
find the word set skip their work.  pmkl_wait_selftest makes one such wait run
out on purpose (an mbarrier nothing arrives on, a limit of a few milliseconds)
through the same mbar_wait and clean-up steps.  No test here faults, traps or
hangs the GPU: every wait ends by its limit, and the context stays usable,
which the last step of each test checks with an ordinary forward."""
import numpy as np
import pytest
import torch

import pmkl_b200
from helpers import seeded_qkv
from oracle import oracle

pytestmark = pytest.mark.gpu

TIMEOUT = -8  # PMKL_ERR_DEVICE_TIMEOUT
LIMIT_NS = 5_000_000  # 5 ms


@pytest.fixture(autouse=True)
def _clean_error_word():
    pmkl_b200.device_error(clear=True)
    yield
    pmkl_b200.device_error(clear=True)


def wait_selftest(ctas, limit_ns=LIMIT_NS):
    out = torch.full((2 * ctas,), -1, dtype=torch.int64, device="cuda")
    rc = pmkl_b200.capi().pmkl_wait_selftest(ctas, limit_ns, out.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0, pmkl_b200.capi().pmkl_status_string(rc)
    torch.cuda.synchronize()
    return out.view(ctas, 2).cpu().tolist()


def forward_matches_oracle(seed=3):
    q, k, v = seeded_qkv(1, 2, 300, 128, torch.bfloat16, seed=seed)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    o = torch.empty_like(qd, dtype=torch.float32)
    m = torch.empty(1, 2, 300, dtype=torch.float32, device="cuda")
    l = torch.empty_like(m)
    pmkl_b200.attention_fwd(qd, kd, vd, o, m, l, True, kernel=pmkl_b200.KERNEL_TCGEN05)
    torch.cuda.synchronize()
    ro, _, _ = oracle.attention_fwd(q.float().numpy(), k.float().numpy(), v.float().numpy(), True)
    return float(np.abs(o.cpu().numpy() - ro).max()) <= 2e-3


def test_wait_runs_out_and_is_reported():
    [(outcome, waited)] = wait_selftest(1)
    assert outcome == 1  # the wait ran out
    assert LIMIT_NS <= waited < LIMIT_NS + 50_000_000  # limit plus at most a few suspend periods
    assert pmkl_b200.device_error(clear=False) == TIMEOUT
    assert pmkl_b200.device_error(clear=True) == TIMEOUT  # reported, then cleared
    assert pmkl_b200.device_error(clear=False) == 0
    assert forward_matches_oracle()


def test_every_cta_of_a_grid_gives_up():
    res = wait_selftest(2)
    assert [r[0] for r in res] == [1, 1]
    assert pmkl_b200.device_error(clear=True) == TIMEOUT
    assert forward_matches_oracle()


def test_later_launches_fast_fail_until_cleared():
    wait_selftest(1)  # sets the error word
    # a two-CTA grid launched afterwards skips its work in both CTAs
    assert [r[0] for r in wait_selftest(2)] == [2, 2]
    # so does the persistent attention kernel: its outputs stay untouched
    q, k, v = (t.cuda() for t in seeded_qkv(1, 4, 512, 128, torch.bfloat16, seed=5))
    o = torch.full_like(q, 7.0)
    m = torch.full((1, 4, 512), 7.0, dtype=torch.bfloat16, device="cuda")
    l = torch.full_like(m, 7.0)
    pmkl_b200.attention_fwd(q, k, v, o, m, l, True, kernel=pmkl_b200.KERNEL_TCGEN05)
    torch.cuda.synchronize()
    assert bool((o == 7.0).all()) and bool((m == 7.0).all()) and bool((l == 7.0).all())
    assert pmkl_b200.device_error(clear=True) == TIMEOUT
    # cleared: the same call now computes
    pmkl_b200.attention_fwd(q, k, v, o, m, l, True, kernel=pmkl_b200.KERNEL_TCGEN05)
    torch.cuda.synchronize()
    assert not bool((o == 7.0).all())
    assert pmkl_b200.device_error(clear=False) == 0
    assert forward_matches_oracle(seed=6)


def test_completed_waits_leave_no_error():
    """The ordinary kernels' waits all complete: a forward, a backward and a
    softmax leave the word clear."""
    assert forward_matches_oracle(seed=7)
    x = torch.randn(256, 1024, device="cuda")
    y = torch.empty_like(x)
    pmkl_b200.warp_softmax_fwd(y, x, 1024, 1024, 256)
    assert pmkl_b200.device_error(clear=False) == 0
