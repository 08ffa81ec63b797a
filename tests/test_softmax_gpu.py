"""GPU parity tests of the warp-softmax kernels through the C ABI, against the
reference's own outputs (golden fixtures) and the CPU oracle, with the
north-star tolerance for fp32 softmax (max abs error <= 1e-5) and the
reference test's all_close rule."""
import numpy as np
import pytest
import torch

import pmkl_b200
from helpers import GOLDEN, assert_f32_close, load_golden
from oracle import oracle

pytestmark = pytest.mark.gpu

SOFTMAX = sorted(p.stem for p in GOLDEN.glob("softmax_*.npz"))


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    yield
    assert pmkl_b200.device_error(clear=True) == 0


def run(x: torch.Tensor, elements, stride, rows, is_log=False, out_dtype=None, dst_offset=0, src_offset=0):
    """x: flat CPU tensor of rows*stride values; returns the flat result."""
    n = x.numel()
    src = torch.empty(n + src_offset, dtype=x.dtype, device="cuda")
    src[src_offset:].copy_(x.cuda())
    od = out_dtype or x.dtype
    dst = torch.full((n + dst_offset,), float("nan"), dtype=od, device="cuda")
    pmkl_b200.warp_softmax_fwd(dst[dst_offset:], src[src_offset:], elements, stride, rows, is_log=is_log)
    torch.cuda.synchronize()
    return dst[dst_offset:].float().cpu().numpy()


def valid(a, elements, stride, rows):
    return np.concatenate([a[r * stride: r * stride + elements] for r in range(rows)]) if rows else a[:0]


@pytest.mark.parametrize("name", SOFTMAX)
def test_golden(name):
    g = load_golden(name)
    rows, el, st = int(g["rows"]), int(g["elements"]), int(g["stride"])
    y = run(torch.from_numpy(g["x"]), el, st, rows)
    assert_f32_close(valid(y, el, st, rows), valid(g["y"], el, st, rows), name)
    assert np.abs(valid(y, el, st, rows) - valid(g["y"], el, st, rows)).max() <= 1e-5
    # entries between rows (stride padding) are not written
    if st > el:
        assert np.isnan(y[el:st]).all()


def test_config5_full():
    """65536 x 1024 fp32, N(0, 4): every row vs the oracle."""
    g = torch.Generator().manual_seed(50)
    x = torch.randn(65536 * 1024, generator=g) * 2
    y = run(x, 1024, 1024, 65536)
    ref = oracle.softmax_fwd(x.numpy(), elements=1024, stride=1024, rows=65536)
    err = np.abs(y - ref).max()
    assert err <= 1e-5, err
    assert_f32_close(y, ref, "config5")


@pytest.mark.parametrize("is_log", [False, True])
@pytest.mark.parametrize("elements", [1, 2, 3, 4, 7, 8, 31, 32, 33, 64, 100, 127, 128, 129, 256, 500, 512, 1000,
                                      1020, 1023, 1024])
def test_element_counts(elements, is_log):
    rows = 37
    stride = elements + (3 if elements % 2 else 4)
    g = torch.Generator().manual_seed(elements)
    x = torch.randn(rows * stride, generator=g) * 2
    y = run(x, elements, stride, rows, is_log=is_log)
    ref = oracle.softmax_fwd(x.numpy(), elements=elements, stride=stride, rows=rows, is_log=is_log)
    assert_f32_close(valid(y, elements, stride, rows), valid(ref, elements, stride, rows), f"el={elements}")


@pytest.mark.parametrize("is_log", [False, True])
def test_vector_path_variants(is_log):
    # aligned, elements % 4 == 0, strided rows
    rows, el, st = 513, 768, 1024
    x = torch.randn(rows * st, generator=torch.Generator().manual_seed(3)) * 2
    y = run(x, el, st, rows, is_log=is_log)
    ref = oracle.softmax_fwd(x.numpy(), elements=el, stride=st, rows=rows, is_log=is_log)
    assert_f32_close(valid(y, el, st, rows), valid(ref, el, st, rows), "vec")
    # misaligned source and destination: the general path
    y2 = run(x, el, st, rows, is_log=is_log, src_offset=1, dst_offset=3)
    assert_f32_close(valid(y2, el, st, rows), valid(ref, el, st, rows), "misaligned")


@pytest.mark.parametrize("in_dt,out_dt", [(torch.float16, torch.float16), (torch.bfloat16, torch.bfloat16),
                                          (torch.bfloat16, torch.float32), (torch.float16, torch.float32),
                                          (torch.float32, torch.bfloat16), (torch.float32, torch.float16)])
@pytest.mark.parametrize("el", [1000, 1024, 256, 1003, 24])
@pytest.mark.parametrize("is_log", [False, True])
def test_dtypes(in_dt, out_dt, el, is_log):
    """16-bit input or output: rows whose length and stride are multiples of 8
    take the 8-element vector kernel, the others the general kernel; both
    match the oracle to the output type's rounding."""
    rows = 65
    x = (torch.randn(rows * el, generator=torch.Generator().manual_seed(4 + el)) * 2).to(in_dt)
    y = run(x, el, el, rows, out_dtype=out_dt, is_log=is_log)
    ref = oracle.softmax_fwd(x.float().numpy(), elements=el, stride=el, rows=rows, is_log=is_log)
    tol = 1e-5 if out_dt == torch.float32 else (2.0 ** -8 if out_dt == torch.bfloat16 else 2.0 ** -11)
    assert (np.abs(y - ref) <= tol * np.maximum(1.0, np.abs(ref)) + 1e-6).all()


def test_16bit_strided_rows_and_misalignment():
    """bf16 rows with a stride of 1032 (a multiple of 8: vector kernel) and the
    same data one element off a 16-byte boundary (general kernel)."""
    rows, el, st = 300, 1024, 1032
    x = (torch.randn(rows * st + 8, generator=torch.Generator().manual_seed(6)) * 2).to(torch.bfloat16)
    ref = oracle.softmax_fwd(x.float().numpy()[:rows * st], elements=el, stride=st, rows=rows)
    y = run(x[:rows * st], el, st, rows, out_dtype=torch.bfloat16)
    assert np.abs(valid(y, el, st, rows) - valid(ref, el, st, rows)).max() <= 2.0 ** -8
    y2 = run(x[:rows * st], el, st, rows, out_dtype=torch.bfloat16, src_offset=1, dst_offset=1)
    assert np.abs(valid(y2, el, st, rows) - valid(ref, el, st, rows)).max() <= 2.0 ** -8


def test_rows_sum_to_one_and_nan_rows():
    rows, el = 8, 1024
    x = torch.randn(rows * el, generator=torch.Generator().manual_seed(5)) * 2
    x[3 * el: 4 * el] = float("-inf")  # all -inf row -> NaN, as the reference
    y = run(x, el, el, rows).reshape(rows, el)
    assert np.isnan(y[3]).all()
    ok = np.delete(y, 3, axis=0)
    np.testing.assert_allclose(ok.sum(-1), 1.0, rtol=1e-5)


def test_argument_errors_on_device():
    x = torch.zeros(8, 1025, device="cuda")
    with pytest.raises(pmkl_b200.PmklError, match="INVALID_SHAPE"):
        pmkl_b200.warp_softmax_fwd(x, x, 1025, 1025, 8)
