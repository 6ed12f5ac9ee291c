"""ktmoe_linear_noalloc, the accumulate for callers that cannot let a library allocate device memory (for example a
runtime that owns one fixed pool of the GPU and must not see a hidden cudaMalloc/cudaFree): called through the C ABI
several times in a row, each result must equal the exact int64 product x·wᵀ computed on the host and the regular
entry point's (ktmoe_linear) — integer sums, tolerance 0 — and the later calls must leave the device's free memory
unchanged. The object file of the entry point must reference no allocating CUDA routine at all. Kept in a file that
pytest collects last."""

import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest

import tritify_b200 as tb
from tritify_b200 import _native

WL = tb.WLEVELS
OBJ = os.path.join(os.path.dirname(tb.__file__), "_build", "noalloc.cu.o")
ALLOCATORS = ("cudaMalloc", "cudaFree", "cudaHostAlloc", "cudaMemPool", "cudaMallocAsync", "cudaFreeAsync",
              "cuMemAlloc", "cuMemCreate", "cuMemFree", "cuMemMap", "cuMemPool", "cuMemHostAlloc")


def _call(x, w, rows, out, k, y, stream=None):
    return tb.lib().ktmoe_linear_noalloc(0, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w.data_ptr()), rows, out,
                                         k, ctypes.c_void_p(y.data_ptr()), stream)


def _undefined(obj):
    r = subprocess.run(["nm", "-u", obj], capture_output=True, text=True, check=True)
    return {ln.split()[-1] for ln in r.stdout.splitlines() if ln.strip()}


@pytest.mark.skipif(not os.path.exists(OBJ) or not shutil.which("nm"), reason="built object or nm not present")
def test_noalloc_object_references_no_allocator():
    """The entry point's translation unit (with the GEMM templates it instantiates) calls no CUDA allocation routine:
    its undefined symbols contain none, while the regular library's object, which allocates, shows cudaMalloc."""
    syms = _undefined(OBJ)
    assert "cudaGetSymbolAddress" in syms  # the check reads the right object
    bad = sorted(s for s in syms if s.startswith(ALLOCATORS))
    assert not bad, f"noalloc.cu references allocating routines: {bad}"
    other = os.path.join(os.path.dirname(OBJ), "ktmoe.cu.o")
    if os.path.exists(other):
        assert "cudaMalloc" in _undefined(other)


@pytest.mark.gpu
def test_noalloc_linear_equals_the_exact_product_on_consecutive_calls():
    torch = pytest.importorskip("torch")
    ctx = tb.Context(0)
    try:
        rng = np.random.default_rng(2024)
        # consecutive calls with different shapes and data: 16-row tiles (37 rows), 48-row tiles with the last one
        # ragged against the 64-row padding (100 rows: 3 tiles of 48 over 128 padded rows), and a full 64-row shape
        shapes = [(37, 300, 1023), (100, 520, 777), (64, 1408, 2048)]
        free_before = None
        for i, (rows, out, k) in enumerate(shapes):
            xh = rng.integers(-WL, WL + 1, size=rows * k, dtype=np.int32)
            wh = rng.integers(-WL, WL + 1, size=out * k, dtype=np.int32)
            x = torch.from_numpy(xh).cuda()
            w = torch.from_numpy(wh).cuda()
            y = torch.full((rows * out,), -1, dtype=torch.int64, device="cuda")
            torch.cuda.synchronize()
            if i >= 1:
                free_before = torch.cuda.mem_get_info()[0]
            assert _call(x, w, rows, out, k, y) == _native.OK
            if i >= 1:
                assert torch.cuda.mem_get_info()[0] == free_before, "the call allocated device memory"
            got = y.cpu().numpy()
            exact = (xh.reshape(rows, k).astype(np.int64) @ wh.reshape(out, k).astype(np.int64).T).reshape(-1)
            bad = np.nonzero(got != exact)[0]
            assert bad.size == 0, f"call {i + 1}: {bad.size} of {got.size} differ from the exact product"
            assert (got == ctx.linear(xh, wh, rows, out, k)).all(), f"call {i + 1}: differs from ktmoe_linear"
    finally:
        ctx.close()


@pytest.mark.gpu
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


@pytest.mark.gpu
def test_noalloc_first_call_on_a_capturing_stream_is_refused():
    """The first call on a device loads this entry point's kernels there, which a stream capture cannot record: on a
    capturing stream that call returns KTMOE_ERR_ARG and leaves the device set up for nothing, and the next call
    outside the capture sets it up and computes. Run in a fresh process, where no call has set the device up yet."""
    import subprocess
    import sys

    code = r"""
import ctypes, torch
import tritify_b200 as tb
from tritify_b200 import _native
x = torch.tensor([1, 2, 3, 4], dtype=torch.int32, device="cuda")
y = torch.zeros(1, dtype=torch.int64, device="cuda")
def call(stream):
    return tb.lib().ktmoe_linear_noalloc(0, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(x.data_ptr()), 1, 1, 4,
                                         ctypes.c_void_p(y.data_ptr()), stream)
s = torch.cuda.Stream()
g = torch.cuda.CUDAGraph()
with torch.cuda.graph(g, stream=s):
    rc = call(ctypes.c_void_p(s.cuda_stream))
assert rc == _native.ERR_ARG, rc
del g
torch.cuda.synchronize()
assert call(None) == _native.OK and int(y[0]) == 30
print("capture guard ok")
"""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "capture guard ok" in r.stdout, r.stdout + r.stderr
