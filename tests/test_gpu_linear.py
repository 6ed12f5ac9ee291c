"""LinearBackend on the B200 (ktmoe_linear / ktmoe_linear_weights) against the reference's equality and residency
gates (crates/02-runtime/kt-runtime/src/gate.rs:26-140): the corpus must hash to the reference's own SHA-256."""

import hashlib
import json
import os

import numpy as np
import pytest

import tritify_b200 as tb
from tritify_b200 import _native

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
LIT = json.load(open(os.path.join(HERE, "golden", "golden.json")))["reference_literals"]
WL = tb.WLEVELS


def test_doc_example(ctx):
    ex = LIT["linear_doc_example"]["value"]
    assert list(ctx.linear(ex["x"], ex["w"], ex["rows"], ex["out"], ex["k"])) == ex["y"]


def test_corpus_hash_is_the_references(ctx, oracle):
    h = hashlib.sha256()
    diverged = []
    for (label, r, o, k, x, w) in oracle.corpus():
        y = ctx.linear(x, w, r, o, k)
        if not (y == oracle.linear(x, w, r, o, k)).all():
            diverged.append(label)
        h.update(y.astype("<i8").tobytes())
    assert not diverged, f"cases that differ from the CPU path: {diverged}"
    assert h.hexdigest() == LIT["corpus_sha256"]["value"]


def test_the_bound_case_beyond_one_flush(ctx):
    """gate.rs:61-66: k = (KT_FLUSH + 1)·16, every code +WLEVELS, one weight row +WLEVELS and one -WLEVELS."""
    k = LIT["k_beyond_flush"]["value"]
    x = np.full(k, WL, np.int32)
    w = np.concatenate([np.full(k, WL, np.int32), np.full(k, -WL, np.int32)])
    want = k * WL * WL
    assert list(ctx.linear(x, w, 1, 2, k)) == [want, -want]


def test_long_k_beyond_one_exact_chunk(ctx, oracle):
    """K above the kernel's single-pass bound (447,392) is split and the int64 partials added."""
    k = 600_001
    rng = np.random.default_rng(1)
    x = rng.integers(-WL, WL + 1, size=2 * k, dtype=np.int32)
    w = rng.integers(-WL, WL + 1, size=3 * k, dtype=np.int32)
    assert (ctx.linear(x, w, 2, 3, k) == oracle.linear(x, w, 2, 3, k)).all()
    xe = np.full(k, WL, np.int32)
    assert list(ctx.linear(xe, np.concatenate([xe, -xe]), 1, 2, k)) == [k * WL * WL, -k * WL * WL]


@pytest.mark.parametrize("rows,out,k", [(1, 1, 1), (17, 33, 50), (16, 128, 128), (64, 256, 2048), (65, 129, 129),
                                        (200, 300, 1000), (3, 1408, 2048), (97, 2048, 1408)])
def test_random_shapes_equal_the_cpu_path(ctx, oracle, rows, out, k):
    rng = np.random.default_rng(rows * 1000 + out)
    x = rng.integers(-WL, WL + 1, size=rows * k, dtype=np.int32)
    w = rng.integers(-WL, WL + 1, size=out * k, dtype=np.int32)
    got = ctx.linear(x, w, rows, out, k)
    want = oracle.linear(x, w, rows, out, k)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, f"{bad.size} of {got.size} differ; first at {bad[:5]}: {got[bad[:5]]} vs {want[bad[:5]]}"


@pytest.mark.parametrize("rows,out,k", [(333, 1000, 4096), (64, 256, 128), (1024, 768, 3000)])
def test_pair_and_single_sm_kernels_agree(ctx, oracle, rows, out, k, monkeypatch):
    """Wide calls run on SM pairs (tcgen05 cta_group::2, 256 weight rows x 64 activation rows per tile); KTMOE_PAIR=0
    keeps them on single SMs. Both must equal the CPU path."""
    rng = np.random.default_rng(out + k)
    x = rng.integers(-WL, WL + 1, size=rows * k, dtype=np.int32)
    w = rng.integers(-WL, WL + 1, size=out * k, dtype=np.int32)
    monkeypatch.setenv("KTMOE_PAIR", "1")
    got_pair = ctx.linear(x, w, rows, out, k)
    monkeypatch.setenv("KTMOE_PAIR", "0")
    got_single = ctx.linear(x, w, rows, out, k)
    want = oracle.linear(x, w, rows, out, k)
    for got in (got_pair, got_single):
        bad = np.nonzero(got != want)[0]
        assert bad.size == 0, f"{bad.size} of {got.size} differ; first at {bad[:5]}"


def test_residency_gate(oracle):
    """gate.rs:109-140: the corpus twice, then two weights of one shape interleaved; and with a 1-byte budget."""
    for budget in [None, 1]:
        c = tb.Context(0)
        if budget:
            c.set_weight_budget(budget)
        corpus = oracle.corpus()
        for p in range(2):
            for i, (label, r, o, k, x, w) in enumerate(corpus):
                assert (c.linear(x, w, r, o, k, weight_id=100 + i) == oracle.linear(x, w, r, o, k)).all(), (p, label)
        x = corpus[3][4]
        t0 = tb.lcg_uniform(11, -WL, WL, 64 * 1023)
        t1 = tb.lcg_uniform(12, -WL, WL, 64 * 1023)
        for _ in range(4):
            for wid, w in [(1, t0), (2, t1)]:
                assert (c.linear(x, w, 4, 64, 1023, weight_id=wid) == oracle.linear(x, w, 4, 64, 1023)).all()
        assert (c.resident_bytes() > 0) == (budget is None)
        c.close()


def test_codes_outside_wlevels_fail_loudly(ctx):
    with pytest.raises(tb.KtmoeError) as e:
        ctx.linear(np.array([WL + 1, 2], np.int32), np.array([3, 4], np.int32), 1, 1, 2)
    assert e.value.status == _native.ERR_RANGE
    with pytest.raises(tb.KtmoeError):
        ctx.linear(np.array([1, 2], np.int32), np.array([np.iinfo(np.int32).min, 4], np.int32), 1, 1, 2)
    # the context stays usable
    assert list(ctx.linear(np.array([1, 2], np.int32), np.array([3, 4], np.int32), 1, 1, 2)) == [11]


@pytest.mark.parametrize("rows,out,k", [(1, 128, 4096), (16, 1408, 4096), (5, 300, 1000)])
def test_split_k_equals_one_block_per_tile(ctx, oracle, rows, out, k, monkeypatch):
    """Few rows leave most SMs idle, so blocks share each tile's K range and add their partial sums atomically
    (exact in any order); KTMOE_SPLITK=0 keeps one block per tile. Both must equal the CPU path."""
    rng = np.random.default_rng(rows + out + k)
    x = rng.integers(-WL, WL + 1, size=rows * k, dtype=np.int32)
    w = rng.integers(-WL, WL + 1, size=out * k, dtype=np.int32)
    want = oracle.linear(x, w, rows, out, k)
    for flag in ("1", "0"):
        monkeypatch.setenv("KTMOE_SPLITK", flag)
        got = ctx.linear(x, w, rows, out, k)
        bad = np.nonzero(got != want)[0]
        assert bad.size == 0, f"KTMOE_SPLITK={flag}: {bad.size} of {got.size} differ"


def _small_codes(rng, rows, out, k):
    x = rng.integers(-127, 128, size=rows * k, dtype=np.int32)
    w = rng.integers(-2048, 2048, size=out * k, dtype=np.int32)
    return x, w


@pytest.mark.parametrize("rows,out,k", [(1, 1, 1), (37, 200, 300), (64, 256, 2048), (128, 1024, 4096),
                                        (5, 128, 4096)])
def test_small_codes_equal_the_cpu_path(ctx, oracle, rows, out, k):
    """int8 activations and 12-bit weights (|x| <= 127, |w| <= 3280) run on one raw activation plane and two weight
    digit planes; a single code one past either bound sends the call back to the nine-plane kernel. All equal the
    CPU path, for weights packed per call and resident weights."""
    rng = np.random.default_rng(rows * 7 + out * 3 + k)
    wid = 90_000 + rows * 7 + out * 3 + k
    x, w = _small_codes(rng, rows, out, k)
    x[0] = -127
    w[-1] = 3280
    want = oracle.linear(x, w, rows, out, k)
    assert (ctx.linear(x, w, rows, out, k) == want).all()
    assert ctx.last_gemm()[1] == 1
    assert (ctx.linear(x, w, rows, out, k, weight_id=wid) == want).all()
    assert (ctx.linear(x, w, rows, out, k, weight_id=wid) == want).all()  # resident, small
    assert ctx.last_gemm()[1] == 1
    x2 = x.copy()
    x2[-1] = 128
    want2 = oracle.linear(x2, w, rows, out, k)
    assert (ctx.linear(x2, w, rows, out, k) == want2).all()
    assert ctx.last_gemm()[1] == 3
    assert (ctx.linear(x2, w, rows, out, k, weight_id=wid) == want2).all()  # resident, nine planes
    assert ctx.last_gemm()[1] == 3
    w2 = w.copy()
    w2[0] = -3281
    assert (ctx.linear(x, w2, rows, out, k) == oracle.linear(x, w2, rows, out, k)).all()
    assert ctx.last_gemm()[1] == 3


@pytest.mark.parametrize("pair", ["1", "0"])
def test_small_codes_at_the_standalone_gemm_size(ctx, pair, monkeypatch):
    """The standalone GEMM as the benchmark runs it: M = N = K = 4096, 12-bit weight codes uniform in [-2048, 2047]
    then int8 activations in [-127, 127], one stream of the reference's test LCG seeded 2. The whole exact int64
    result hashes to the CPU oracle's golden (tests/golden/bench_golden.json, the oracle's Portable linear), on SM
    pairs and on single SMs."""
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import bench

    monkeypatch.setenv("KTMOE_PAIR", pair)
    g = json.load(open(os.path.join(root, "tests", "golden", "bench_golden.json")))["workloads"]["gemm4096"]
    w = bench.WORKLOADS["gemm4096"]
    x, wt = bench.gemm_codes(w, tb.lcg_uniform)
    assert hashlib.sha256(np.ascontiguousarray(x, dtype="<i4").tobytes()).hexdigest() == g["x_sha256"]
    assert hashlib.sha256(np.ascontiguousarray(wt, dtype="<i4").tobytes()).hexdigest() == g["w_sha256"]
    n = w["M"]
    y = ctx.linear(x, wt, n, n, n)
    assert ctx.last_gemm()[1] == 1  # the (1, 2)-plane kernels
    assert hashlib.sha256(np.ascontiguousarray(y, dtype="<i8").tobytes()).hexdigest() == g["output"]["data_sha256"]


@pytest.mark.parametrize("rows,out,k", [(300, 1000, 4096), (256, 256, 128), (1000, 384, 3000), (129, 130, 200)])
def test_small_codes_pair_and_single_sm_agree(ctx, oracle, rows, out, k, monkeypatch):
    """From 128 activation rows on, small codes run on SM pairs (256 activation rows x 128 weight rows per tile);
    KTMOE_PAIR=0 keeps them on the one-SM (1, 2) kernel. Both equal the CPU path."""
    rng = np.random.default_rng(rows + 3 * out + k)
    x, w = _small_codes(rng, rows, out, k)
    want = oracle.linear(x, w, rows, out, k)
    for flag in ("1", "0"):
        monkeypatch.setenv("KTMOE_PAIR", flag)
        got = ctx.linear(x, w, rows, out, k)
        assert ctx.last_gemm()[1] == 1
        bad = np.nonzero(got != want)[0]
        assert bad.size == 0, f"KTMOE_PAIR={flag}: {bad.size} of {got.size} differ; first at {bad[:5]}"


@pytest.mark.parametrize("pair", ["1", "0"])
def test_small_codes_beyond_one_exact_chunk(ctx, pair, monkeypatch):
    """K = 450 000 of the largest small codes (x = ±127, w = ±3280, every digit ±40): one int32 diagonal would
    overflow, so K is split at 422 733 and the int64 partials added."""
    monkeypatch.setenv("KTMOE_PAIR", pair)
    rows, out, k = 128, 2, 450_000
    x = np.full(rows * k, 127, np.int32)
    x[k:2 * k] = -127
    w = np.concatenate([np.full(k, 3280, np.int32), np.full(k, -3280, np.int32)])
    y = ctx.linear(x, w, rows, out, k).reshape(rows, out)
    assert ctx.last_gemm()[1] == 1
    e = k * 127 * 3280
    assert y[0].tolist() == [e, -e] and y[1].tolist() == [-e, e] and (y[2:] == y[0]).all()
