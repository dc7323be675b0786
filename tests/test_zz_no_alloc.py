"""The allocation-free GRAIN backward (``ro_grain_backward_noalloc``, exported
with C linkage from the extension library) against the regular entry point.

Collected last on purpose: it must pass both alone in a fresh process and
after every other test has run in the same process.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

from rational_optimizer_b200 import _ext
from rational_optimizer_b200.ops.grain import GRAIN_DENOMINATOR, GRAIN_NUMERATOR


def _entry():
    lib = ctypes.CDLL(_ext.ext().__file__)
    fn = lib.ro_grain_backward_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                           ctypes.c_void_p]
    return fn


def _inputs(rows, hidden, groups, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, hidden, device="cuda", generator=gen) * 2.0
    gy = torch.randn(rows, hidden, device="cuda", generator=gen)
    num = torch.tensor(GRAIN_NUMERATOR, device="cuda").repeat(groups, 1)
    den = torch.tensor(GRAIN_DENOMINATOR, device="cuda").repeat(groups, 1)
    num = num + 0.01 * torch.randn(num.shape, device="cuda", generator=gen)
    den = den + 0.01 * torch.randn(den.shape, device="cuda", generator=gen)
    return x, gy, num, den


def _call(fn, x, gy, num, den, groups, eps):
    rows, hidden = x.shape
    gx = torch.empty_like(x)
    gnum = torch.full_like(num, float("nan"))
    gden = torch.full_like(den, float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(gy.data_ptr(), x.data_ptr(), num.data_ptr(), den.data_ptr(), gx.data_ptr(),
            gnum.data_ptr(), gden.data_ptr(), rows, hidden, groups, eps, stream)
    return rc, gx, gnum, gden


@pytest.mark.parametrize("rows,hidden,groups", [(4096, 4608, 18), (999, 768, 3), (256, 200, 5)])
def test_noalloc_backward_matches_regular_entry_point(rows, hidden, groups):
    fn = _entry()
    C = _ext.ext()
    eps = 1e-6
    x, gy, num, den = _inputs(rows, hidden, groups, rows + groups)
    empty = torch.empty(groups, 0, device="cuda")
    ref_gx, ref_gnum, ref_gden, _ = C.grain_backward(gy, x, num, den, torch.empty(groups, 0, 2, device="cuda"),
                                                     empty, empty, 0.0, eps, hidden, groups, None, None)
    for _ in range(2):  # two calls in a row reuse the same scratch
        rc, gx, gnum, gden = _call(fn, x, gy, num, den, groups, eps)
        torch.cuda.synchronize()
        assert rc == 0
        torch.testing.assert_close(gx, ref_gx, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(gnum, ref_gnum, rtol=1e-5, atol=1e-4)
        torch.testing.assert_close(gden, ref_gden, rtol=1e-5, atol=1e-4)


def test_noalloc_rejects_oversized_problem_without_launching():
    fn = _entry()
    # 7000 groups of width 1: one block row needs 7000 x 10 partials > 65536
    x = torch.zeros(64, 7000, device="cuda")
    gy = torch.zeros_like(x)
    num = torch.zeros(7000, 6, device="cuda")
    den = torch.zeros(7000, 4, device="cuda")
    rc, _, gnum, _ = _call(fn, x, gy, num, den, 7000, 1e-6)
    torch.cuda.synchronize()
    assert rc == -2
    assert torch.isnan(gnum).all()  # nothing was written
    rc, *_ = _call(fn, x, gy, num, den, 7, 1e-6)  # 7000 / 7 = 1000 > 256: unsupported width
    assert rc == -1


def test_noalloc_zero_rows_writes_zero_coefficient_gradients():
    fn = _entry()
    x = torch.zeros(0, 768, device="cuda")
    gy = torch.zeros_like(x)
    num = torch.ones(3, 6, device="cuda")
    den = torch.ones(3, 4, device="cuda")
    for _ in range(2):
        rc, gx, gnum, gden = _call(fn, x, gy, num, den, 3, 1e-6)
        torch.cuda.synchronize()
        assert rc == 0
        assert gx.numel() == 0
        assert torch.equal(gnum, torch.zeros_like(gnum))  # NaN-filled before the call
        assert torch.equal(gden, torch.zeros_like(gden))
