"""ktmoe_linear_noalloc, the accumulate for callers that cannot let a library allocate device memory (for example a
runtime that owns one fixed pool of the GPU and must not see a hidden cudaMalloc/cudaFree): called through the C ABI
twice in a row, each result must equal the regular entry point's (ktmoe_linear) exactly — integer sums, tolerance 0 —
and the second call must leave the device's free memory unchanged. Kept in a file that pytest collects last."""

import ctypes

import numpy as np
import pytest

import tritify_b200 as tb
from tritify_b200 import _native

pytestmark = pytest.mark.gpu
WL = tb.WLEVELS


def _call(x, w, rows, out, k, y, stream=None):
    return tb.lib().ktmoe_linear_noalloc(0, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w.data_ptr()), rows, out,
                                         k, ctypes.c_void_p(y.data_ptr()), stream)


def test_noalloc_linear_equals_the_regular_entry_point_on_two_calls():
    torch = pytest.importorskip("torch")
    ctx = tb.Context(0)
    try:
        rng = np.random.default_rng(2024)
        shapes = [(37, 300, 1023), (64, 1408, 2048)]  # two calls in a row, different shapes and data
        free_before_second = None
        for i, (rows, out, k) in enumerate(shapes):
            xh = rng.integers(-WL, WL + 1, size=rows * k, dtype=np.int32)
            wh = rng.integers(-WL, WL + 1, size=out * k, dtype=np.int32)
            x = torch.from_numpy(xh).cuda()
            w = torch.from_numpy(wh).cuda()
            y = torch.full((rows * out,), -1, dtype=torch.int64, device="cuda")
            torch.cuda.synchronize()
            if i == 1:
                free_before_second = torch.cuda.mem_get_info()[0]
            assert _call(x, w, rows, out, k, y) == _native.OK
            if i == 1:
                assert torch.cuda.mem_get_info()[0] == free_before_second, "the call allocated device memory"
            want = ctx.linear(xh, wh, rows, out, k)
            got = y.cpu().numpy()
            bad = np.nonzero(got != want)[0]
            assert bad.size == 0, f"call {i + 1}: {bad.size} of {got.size} differ"
    finally:
        ctx.close()


def test_noalloc_linear_rejects_sizes_beyond_its_scratch():
    torch = pytest.importorskip("torch")
    x = torch.zeros(16, dtype=torch.int32, device="cuda")
    y = torch.zeros(16, dtype=torch.int64, device="cuda")
    # 3·4096·(4096 rows of x) + 3·4096·4096 bytes of planes is far above 64 MiB
    assert _call(x, x, 4096, 4096, 4096, y) == _native.ERR_UNSUPPORTED
    # and codes outside ±WLEVELS are reported, not computed
    xb = torch.tensor([WL + 1, 2], dtype=torch.int32, device="cuda")
    wb = torch.tensor([3, 4], dtype=torch.int32, device="cuda")
    yb = torch.zeros(1, dtype=torch.int64, device="cuda")
    assert _call(xb, wb, 1, 1, 2, yb) == _native.ERR_RANGE
    ok = torch.tensor([1, 2], dtype=torch.int32, device="cuda")
    assert _call(ok, wb, 1, 1, 2, yb) == _native.OK and int(yb[0]) == 11
