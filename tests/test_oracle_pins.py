"""The CPU oracle (test infrastructure) pinned to the reference's own golden vectors and properties."""

import hashlib
import json
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
GOLDEN = json.load(open(os.path.join(HERE, "golden", "golden.json")))
LIT = GOLDEN["reference_literals"]


def test_corpus_hash_is_the_references(oracle):
    """kt-runtime/src/tests_cuda.rs:9: SHA-256 over every i64 accumulator of the equality-gate corpus."""
    h = hashlib.sha256()
    for (_, r, o, k, x, w) in oracle.corpus():
        h.update(oracle.linear(x, w, r, o, k).astype("<i8").tobytes())
    assert h.hexdigest() == LIT["corpus_sha256"]["value"]


def test_kt_int_doc_examples(oracle):
    """kt-int/src/lib.rs:35-39."""
    three_q = oracle.from_ratio(3, 4)
    assert oracle.apply(three_q, 8) == LIT["from_ratio_3_4_apply_8"]["value"]
    assert oracle.apply(oracle.mul(three_q, oracle.from_ratio(4, 3)), 9) == \
        LIT["three_quarters_times_four_thirds_apply_9"]["value"]
    assert oracle.isqrt_u128(144) == LIT["isqrt_144"]["value"]
    # kt-int lib.rs:246-252
    assert oracle.apply(oracle.from_ratio(0, 5), 123) == 0
    assert oracle.apply((0, 0), 999) == 0
    four = oracle.from_ratio(4, 1)
    for v in [-7, 0, 1, 1000, 1_000_000_000]:
        assert oracle.apply(four, v) == 4 * v


def test_backend_doc_example(oracle):
    """kt-core/src/backend.rs:12-15."""
    ex = LIT["linear_doc_example"]["value"]
    y = oracle.linear(np.array(ex["x"]), np.array(ex["w"]), ex["rows"], ex["out"], ex["k"])
    assert list(y) == ex["y"]


def test_digit_bounds_are_the_references():
    """kt-cuda/src/digits.rs:20-23 and tests.rs:68, :88."""
    WL = 265720
    assert 40 * (1 + 81 + 81 * 81) == WL
    kt_flush = (2**31 - 1) // (16 * 40 * 40)
    assert (kt_flush + 1) * 16 == LIT["k_beyond_flush"]["value"]
    assert (2**63 - 1) // (WL * WL) == LIT["k_max"]["value"]


def test_scale_ops_track_f64(oracle):
    """kt-int lib.rs:570-621: from_ratio, mul, apply and recip within their stated f64 bounds."""
    rng = np.random.default_rng(5)
    for _ in range(2000):
        num, den = int(rng.integers(1, 1 << 50)), int(rng.integers(1, 1 << 50))
        m, s = oracle.from_ratio(num, den)
        assert abs(m * 2.0 ** -s - num / den) <= 1e-8 * num / den
        a = oracle.from_f64(1e-6 + rng.random())
        b = oracle.from_f64(1e-3 + rng.random())
        p = oracle.mul(a, b)
        want = a[0] * 2.0 ** -a[1] * b[0] * 2.0 ** -b[1]
        assert abs(p[0] * 2.0 ** -p[1] - want) <= 1e-8 * want
        v = int(rng.integers(-(1 << 39), 1 << 39))
        assert abs(oracle.apply(p, v) - round(v * p[0] * 2.0 ** -p[1])) <= 1
        x = 1e-7 + rng.random() * 100
        r = oracle.recip(oracle.from_f64(x))
        assert abs(r[0] * 2.0 ** -r[1] - 1 / x) <= 1e-8 / x


def test_tables_match_golden_and_end_codes(oracle):
    for kind, name in enumerate(["exp", "silu", "sigmoid"]):
        codes, inv_step, lo_index, code_scale = oracle.table(kind)
        g = GOLDEN["tables"][name]
        assert hashlib.sha256(codes.astype("<i8").tobytes()).hexdigest() == g["codes_sha256"]
        assert list(inv_step) == g["inv_step"] and lo_index == g["lo_index"] and list(code_scale) == g["code_scale"]
    exp_codes = oracle.table(0)[0]
    assert exp_codes[-1] == 1 << 20  # exp(0)·2^20
    sig = oracle.table(2)[0]
    assert [int(sig[0]), int(sig[-1])] == [0, 1 << 20] == LIT["sigmoid_end_codes"]["value"]


@pytest.mark.parametrize("name", ["tiny_softmax", "tiny_softmax_norm_one_row", "tiny_softmax_37rows",
                                  "tiny_router_bias", "tiny_sigmoid_shared", "tiny_sigmoid_raw_shared_one_row",
                                  "small_shared_softmax", "tiny_odd_hidden", "tiny_gated_shared",
                                  "tiny_gated_shared_one_row", "small_gated_shared"])
def test_oracle_reproduces_golden_cases(oracle, name):
    import cases

    c = cases.CASES[name]
    g = GOLDEN["cases"][name]
    x = cases.make_x(c)
    assert cases.sha(x) == g["x_f32_sha256"], "the generator's bytes changed"
    xi, xs = oracle.from_reals_f32(x)
    m = cases.build_oracle(c, oracle)
    y, ys = m.forward(xi, xs)
    assert cases.out_hashes(y, ys) == g["output"]


@pytest.mark.parametrize("rows", [1, 5])
def test_the_seam_is_a_numeric_no_op(oracle, rows):
    """kt-core/src/tests.rs:156-181 and tests_glm.rs:225-237: forward_int_with_experts == forward_int."""
    import cases

    for name in ["tiny_softmax", "tiny_sigmoid_shared"]:
        c = cases.CASES[name]
        m = cases.build_oracle(c, oracle)
        x = np.random.default_rng(rows).standard_normal((rows, c.d)).astype(np.float32)
        xi, xs = oracle.from_reals_f32(x)
        a, sa = m.forward(xi, xs)
        b, sb = m.forward_with_local_experts(xi, xs)
        assert (a == b).all() and sa == sb


def test_topk_ties_go_to_the_lower_index(oracle):
    """layers.rs:800-805: identical router rows give identical logits; the lowest indices win."""
    d, E, f, k = 32, 8, 16, 3
    rng = np.random.default_rng(3)
    row = rng.standard_normal(d).astype(np.float32)
    router_w = np.tile(row, (E, 1))
    experts = rng.standard_normal(E * 3 * f * d).astype(np.float32)
    m = oracle.MoeOracle(d, E, f, k, router_w, experts)
    xi, xs = oracle.from_reals_f32(rng.standard_normal((4, d)).astype(np.float32))
    ex, ec, sumc = m.route(xi, xs)
    assert (ex == np.arange(k)).all()


def test_all_zero_input_gives_zero_output(oracle):
    import cases

    c = cases.CASES["tiny_sigmoid_shared"]
    m = cases.build_oracle(c, oracle)
    y, ys = m.forward(np.zeros((3, c.d), np.int32), (0, 0))
    assert (y == 0).all() and ys == (0, 0)


def test_rsqrt_tracks_f64_like_the_reference(oracle):
    """kt-int lib.rs:620-640 (scale_rsqrt_matches_f64): over log-uniform v in [2^-20, 2^20], Scale::rsqrt is within a
    relative 2e-9 of 1/sqrt(v) (the reference freezes that bound)."""
    rng = np.random.default_rng(0x1557A1)
    worst = 0.0
    for frac in rng.random(20000):
        v = 2.0 ** (-20.0 + 40.0 * frac)
        m, sh = oracle.scale_rsqrt(oracle.from_f64(v))
        got = m * 2.0 ** (-sh)
        worst = max(worst, abs(got - 1.0 / np.sqrt(v)) * np.sqrt(v))
    assert worst < 2e-9


def test_rmsnorm_tracks_float_like_the_reference(oracle):
    """kt-core tests.rs:63-75 (rmsnorm_tracks_float_and_is_deterministic): the integer RmsNorm stays within 1% of the
    float path's peak, and repeats bit for bit."""
    import tritify_b200 as tb

    dim, rows = 128, 3
    w = tb.synth_normal(71, 1.0, dim)
    xf = tb.synth_normal(72, 1.0, rows * dim)
    xi, xs = oracle.from_reals_f32(xf)
    y, ys, _, _, _ = oracle.rmsnorm(w, 1e-6, xi, xs)
    y2, ys2, _, _, _ = oracle.rmsnorm(w, 1e-6, xi, xs)
    assert (y == y2).all() and ys == ys2
    x64 = xi.astype(np.float64).reshape(rows, dim) * xs[0] * 2.0 ** (-xs[1])
    ref = x64 / np.sqrt((x64 ** 2).mean(axis=1, keepdims=True) + 1e-6) * w.astype(np.float64)
    got = y.astype(np.float64).reshape(rows, dim) * ys[0] * 2.0 ** (-ys[1])
    assert np.abs(got - ref).max() <= np.abs(ref).max() * 1e-2


def _gate_case(oracle, gate_w, sigmoid=False):
    """A small layer with a shared expert, optionally behind the sigmoid gate (the extension). Every token's first
    feature is +8, so a gate that weighs only that feature gives every token a logit of the same sign."""
    d, E, f, k, fs, T = 64, 8, 48, 2, 40, 6
    w = oracle.synth_normal(41, 0.02, E * d + E * 3 * f * d + 3 * fs * d)
    router, experts, shared = w[:E * d], w[E * d:E * d + E * 3 * f * d], w[E * d + E * 3 * f * d:]
    sbias = oracle.synth_normal(43, 0.05, E) if sigmoid else None
    m = oracle.MoeOracle(d, E, f, k, router, experts, norm_topk=True, sigmoid_bias=sbias, shared_hidden=fs,
                         shared_w=shared, shared_gate_w=gate_w)
    x = oracle.synth_normal(42, 1.0, T * d).reshape(T, d)
    x[:, 0] = 8.0
    xi, xs = oracle.from_reals_f32(x)
    return m.forward(xi, xs)


@pytest.mark.parametrize("sigmoid", [False, True])
def test_a_saturated_shared_gate_is_the_ungated_layer(oracle, sigmoid):
    """The gated shared expert (extension; the reference refuses it, kt-model-moe/src/lib.rs:152-154) is pinned by an
    exact property of its definition: a gate whose logit is beyond +16 for every token reads the sigmoid table's last
    entry, round(sigmoid(16)·2^20) = 2^20, so the gated tensor is requant_dyn(2^20·y, L, 2^20·L) = y at scale
    ratio(2^48)·y.scale·2^-20 = y.scale — the ungated layer's bits exactly."""
    gw = np.zeros(64, np.float32)
    gw[0] = 50.0  # logit ~ 8·50 = 400 for every token
    gated = _gate_case(oracle, gw, sigmoid=sigmoid)
    plain = _gate_case(oracle, None, sigmoid=sigmoid)
    assert (gated[0] == plain[0]).all() and gated[1] == plain[1]
    # a gate inside the table's range changes the result, deterministically
    g = oracle.synth_normal(44, 0.02, 64)
    a, b = _gate_case(oracle, g, sigmoid=sigmoid), _gate_case(oracle, g, sigmoid=sigmoid)
    assert (a[0] == b[0]).all() and a[1] == b[1]
    assert not ((a[0] == plain[0]).all() and a[1] == plain[1])


def test_oracle_generator_and_lcg_equal_the_products(oracle):
    """The oracle's copy of the build-defined normal generator and of the reference's test LCG give the product
    library's bytes, so the reference arm of the benchmark and the goldens need nothing of the product."""
    import tritify_b200 as tb

    for seed, sigma, n, off in [(1, 0.02, 1 << 21, 0), (0, 1.0, 1000, 17), (3, 1.0, 3 << 20, 123456789)]:
        a = oracle.synth_normal(seed, sigma, n, offset=off)
        b = tb.synth_normal(seed, sigma, n, offset=off)
        assert (a.view(np.uint32) == b.view(np.uint32)).all()
    assert (oracle.lcg_uniform(2, -2048, 2047, 100000) == tb.lcg_uniform(2, -2048, 2047, 100000)).all()


def test_token_parallel_forward_equals_the_serial_forward(oracle):
    """MoeOracle.forward_par (tokens spread over threads, used for the full-size goldens) gives forward's bits."""
    import cases

    for name in ["small_shared_softmax", "tiny_sigmoid_shared", "tiny_gated_shared", "tiny_softmax_norm_one_row"]:
        c = cases.CASES[name]
        xi, xs = oracle.from_reals_f32(cases.make_x(c))
        m = cases.build_oracle(c, oracle)
        a, b = m.forward(xi, xs), m.forward_par(xi, xs, 3)
        assert (a[0] == b[0]).all() and a[1] == b[1], name


def test_the_selection_bias_moves_the_choice_but_not_the_weights(oracle):
    """tests_glm.rs:178-199 (kt-core): with a sigmoid router, a selection bias larger than any sigma difference puts
    an expert the unbiased route left out into the top-k; every chosen expert's weight is still its sigma code
    without the bias (CodeLut::index, clamped read); with norm_topk_prob the weights' sum is sumc, without it sumc is
    2^20 (the raw scores)."""
    d, E, f, k = 32, 16, 8, 4
    rng = np.random.default_rng(0x53)
    router_w = (rng.standard_normal((E, d)) * 0.5).astype(np.float32)
    experts = (rng.standard_normal(E * 3 * f * d) * 0.02).astype(np.float32)
    xi, xs = oracle.from_reals_f32(rng.standard_normal((1, d)).astype(np.float32))

    def moe(bias, norm):
        return oracle.MoeOracle(d, E, f, k, router_w, experts, norm_topk=norm, sigmoid_bias=bias)

    plain = moe(np.zeros(E, np.float32), True)
    ex0, _, _ = plain.route(xi, xs)
    outsider = next(e for e in range(E) if e not in set(ex0[0].tolist()))
    b = np.zeros(E, np.float32)
    b[outsider] = 1.5
    ex1, ec1, sumc1 = moe(b, True).route(xi, xs)
    assert outsider in ex1[0].tolist(), "the bias must move the choice"
    logits, ls = plain.router_logits(xi, xs)
    codes = oracle.table(2)[0]
    for e, c in zip(ex1[0].tolist(), ec1[0].tolist()):
        idx = oracle.table_index(2, int(logits[0, e]), ls[0])
        assert c == int(codes[min(max(idx, 0), len(codes) - 1)]), f"expert {e}: its weight is its sigma code"
    assert sumc1[0] == ec1[0].sum()
    _, _, sumc2 = moe(b, False).route(xi, xs)
    assert sumc2[0] == 1 << 20


def test_sigmoid_codes_track_the_float_sigmoid_and_clamp(oracle):
    """tests_glm.rs:137-154 (kt-core): a logit's sigma code (CodeLut over [-16, 16] with 2^16 entries, clamped read)
    is within one table step of sigma(real)·2^20 (sigma' <= 1/4, so one step moves the code by at most step/4·2^20,
    plus one for the index's rounding), and past the table the codes are 0 and 2^20."""
    import math

    k = float(1 << 20)
    step = 2.0 * 16.0 / ((1 << 16) - 1)
    scale = oracle.from_f64(1.0 / 4096.0)
    codes = oracle.table(2)[0]

    def code(v, s):
        return int(codes[min(max(oracle.table_index(2, v, s), 0), len(codes) - 1)])

    for l in range(-80_000, 80_001, 997):
        for v in (l, -l, 0, int(l / 3)):
            c = code(v, scale)
            real = v / 4096.0
            want = k / (1.0 + math.exp(-real))
            assert abs(c - want) <= step / 4.0 * k + 1.0, (real, c, want)
            assert 0 <= c <= 1 << 20
    one = oracle.from_f64(1.0)
    assert (code(-(1 << 20), one), code(1 << 20, one)) == (0, 1 << 20)


# ── the reference's float-tracking tests (kt-core tests.rs), on their own inputs ──
def _ref_uniforms(seed, n):
    """tests.rs:15-24: the test LCG and unif = ((s >> 40) / 2^24 · 2 - 1) as f32, n draws after `seed`; returns the
    values and the state."""
    s, out = seed, np.empty(n, np.float32)
    for i in range(n):
        s = (s * 6364136223846793005 + 1442695040888963407) & ((1 << 64) - 1)
        out[i] = np.float32((s >> 40) / float(1 << 24) * 2.0 - 1.0)
    return out, s


def _real(scale):
    return scale[0] * 2.0 ** (-scale[1])


def _linear_ref(x, codes, ws):
    """QuantLinear::forward_ref (layers.rs:330-348): f64 sums of x·(code·w_scale), cast to f32."""
    return (x.astype(np.float64) @ (codes.astype(np.float64) * _real(ws)).T).astype(np.float32)


def _swiglu_ref(x, g, u, dn):
    """SwiGluMlp::forward_ref (layers.rs:642-648)."""
    gf, uf = _linear_ref(x, *g).astype(np.float64), _linear_ref(x, *u).astype(np.float64)
    act = (gf / (1.0 + np.exp(-gf)) * uf).astype(np.float32)
    return _linear_ref(act, *dn)


def test_swiglu_tracks_float_like_the_reference(oracle):
    """tests.rs:94-111 (swiglu_tracks_float_and_is_deterministic): dim 64, hidden 128, the test LCG at 0x9999 for the
    gate, up and down weights and the probe; the integer SwiGLU is deterministic and within 2% of the float path's
    peak."""
    dim, hidden = 64, 128
    w, s = _ref_uniforms(0x9999, 3 * hidden * dim)
    p, _ = _ref_uniforms(s, dim)
    m = oracle.MoeOracle(dim, 1, hidden, 1, np.zeros((1, dim), np.float32), w)
    xi, xs = oracle.from_reals_f32(p)
    y, ys = m.expert(0, xi.reshape(-1), xs)
    y2, ys2 = m.expert(0, xi.reshape(-1), xs)
    assert (y == y2).all() and ys == ys2
    x = (xi.reshape(1, dim).astype(np.float64) * _real(xs)).astype(np.float32)
    ref = _swiglu_ref(x, m.weights(1), m.weights(2), m.weights(3)).reshape(-1)
    got = y.astype(np.float64) * _real(ys)
    assert np.abs(got - ref).max() <= np.abs(ref).max() * 2e-2


def test_moe_tracks_float_without_a_routing_flip_like_the_reference(oracle):
    """tests.rs:113-154 (moe_mlp_tracks_float_sparse_and_deterministic): dim 64, hidden 96, 8 experts, top-2, softmax
    router normalised over all experts, weights and probe from the test LCG at 0x30E1; the integer and float routers
    choose the same experts, the integer layer is deterministic and within 3% of MoeMlp::forward_ref's peak."""
    dim, hidden, E, k = 64, 96, 8, 2
    vals, s = _ref_uniforms(0x30E1, E * dim + E * 3 * hidden * dim)
    p, _ = _ref_uniforms(s, dim)
    router_w, experts = vals[:E * dim], vals[E * dim:]
    m = oracle.MoeOracle(dim, E, hidden, k, router_w, experts)
    xi, xs = oracle.from_reals_f32(p)
    y, ys = m.forward(xi, xs)
    y2, ys2 = m.forward(xi, xs)
    assert (y == y2).all() and ys == ys2

    x = (xi.reshape(1, dim).astype(np.float64) * _real(xs)).astype(np.float32)
    logits = _linear_ref(x, *m.weights(0))[0]
    order = sorted(range(E), key=lambda e: (-float(logits[e]), e))[:k]
    li, _ = m.router_logits(xi, xs)
    order_int = sorted(range(E), key=lambda e: (-int(li[0, e]), e))[:k]
    assert order == order_int, "a routing flip between the integer and the float router"
    ex, _, _ = m.route(xi, xs)
    assert ex[0].tolist() == order_int

    exps = np.exp((logits - logits.max()).astype(np.float64))
    out = np.zeros(dim)
    for e in order:
        ye = _swiglu_ref(x, m.weights(1, e), m.weights(2, e), m.weights(3, e))[0]
        out += exps[e] / exps.sum() * ye.astype(np.float64)
    ref = out.astype(np.float32)
    got = y.reshape(-1).astype(np.float64) * _real(ys)
    assert np.abs(got - ref).max() <= np.abs(ref).max() * 3e-2


@pytest.mark.slow
@pytest.mark.parametrize("name", ["config1", "config1_norm_topk"])
def test_oracle_reproduces_the_config1_goldens(oracle, name):
    """BASELINE config 1 (512 tokens, 64 experts of 1408, top-8) through the oracle's token-parallel forward (equal
    to the serial one, test above) over every host core: the committed output and route hashes again."""
    import cases

    c = cases.CASES[name]
    g = GOLDEN["cases"][name]
    x = cases.make_x(c)
    assert cases.sha(x) == g["x_f32_sha256"]
    xi, xs = oracle.from_reals_f32(x)
    m = cases.build_oracle(c, oracle)
    y, ys = m.forward_par(xi, xs)
    assert cases.out_hashes(y, ys) == g["output"]
