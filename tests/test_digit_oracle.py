"""The digit decompositions the GPU kernels compute, restated on the CPU as independent GEMMs and pinned to the
reference's Portable linear: the nine-plane balanced base-81 algorithm of kt-cuda (digits.rs, host.rs) reproduces the
equality-gate corpus hash (gate.rs:26-56, tests_cuda.rs:9) and the bound case one flush beyond KT_FLUSH; the
(1, 2)-plane split of the small-code kernels is exact up to its K split and overflows one term beyond it."""

import hashlib
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIT = json.load(open(os.path.join(HERE, "golden", "golden.json")))["reference_literals"]
WL = 265720


def test_digit_gemm_reproduces_the_corpus_hash(oracle):
    h = hashlib.sha256()
    for (label, r, o, k, x, w) in oracle.corpus():
        y = oracle.linear_digits(x, w, r, o, k)
        assert (y == oracle.linear(x, w, r, o, k)).all(), label
        h.update(y.astype("<i8").tobytes())
    assert h.hexdigest() == LIT["corpus_sha256"]["value"]


def test_digit_gemm_needs_its_flush(oracle):
    """gate.rs:61-66: k = (KT_FLUSH + 1)·16, every code +WLEVELS, one weight row +WLEVELS and one -WLEVELS."""
    k = LIT["k_beyond_flush"]["value"]
    x = np.full(k, WL, np.int32)
    w = np.concatenate([np.full(k, WL, np.int32), np.full(k, -WL, np.int32)])
    want = [k * WL * WL, -k * WL * WL]
    assert list(oracle.linear_digits(x, w, 1, 2, k)) == want
    assert list(oracle.linear_digits(x, w, 1, 2, k, flush=k)) != want  # one pass wraps the int32 sums


def test_small_split_is_exact_and_its_bound_is_tight(oracle):
    rng = np.random.default_rng(9)
    for rows, out, k in [(1, 1, 1), (3, 5, 7), (17, 33, 300), (8, 64, 4096)]:
        x = rng.integers(-127, 128, size=rows * k, dtype=np.int32)
        w = rng.integers(-3280, 3281, size=out * k, dtype=np.int32)
        assert (oracle.linear_small(x, w, rows, out, k) == oracle.linear(x, w, rows, out, k)).all()
    bound = oracle.SMALL_FLUSH_TERMS
    assert bound * 127 * 40 <= 2**31 - 1 < (bound + 1) * 127 * 40
    k = bound + 1
    x = np.full(k, 127, np.int32)
    w = np.full(k, 3280, np.int32)  # both digits +40: every term of both sums is 127·40
    assert oracle.linear_small(x, w, 1, 1, k)[0] == k * 127 * 3280
    assert oracle.linear_small(x, w, 1, 1, k, flush=k)[0] != k * 127 * 3280
