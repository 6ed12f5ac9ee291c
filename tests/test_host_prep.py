"""The product's offline host preparation (libktmoe.so, no GPU needed) equals the oracle's restatement bit for bit:
weight/bias quantisers, the coded sigmoid bias, the entry quantiser and the three code tables."""

import hashlib
import json
import os
import sys

import numpy as np

import tritify_b200 as tb

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
GOLDEN = json.load(open(os.path.join(HERE, "golden", "golden.json")))


def test_weight_quantiser_equals_oracle(oracle):
    for seed, n, sigma in [(1, 1, 0.02), (2, 4097, 0.02), (3, 1 << 21, 0.5), (4, 100, 1e-30)]:
        w = tb.synth_normal(seed, sigma, n)
        q = tb.QuantLinear.from_weights("w", w, 1, n)
        codes, s = oracle.quantize_weights(w)
        assert (q.w_codes.reshape(-1) == codes).all() and (q.w_scale.mant, q.w_scale.shift) == s
        assert np.abs(q.w_codes).max() <= tb.WLEVELS
    z = tb.QuantLinear.from_weights("z", np.zeros(8, np.float32), 2, 4)
    assert (z.w_codes == 0).all() and z.w_scale == tb.Scale.ZERO


def test_bias_and_sigmoid_bias_codes_equal_oracle(oracle):
    b = tb.synth_normal(9, 1.0, 64)
    q = tb.QuantLinear.from_weights("r", tb.synth_normal(8, 0.02, 64 * 16), 64, 16).with_bias(b)
    m = oracle.MoeOracle(16, 64, 8, 2, np.zeros((64, 16), np.float32), np.zeros(64 * 3 * 8 * 16, np.float32),
                         router_bias=b, sigmoid_bias=b * 0.05)
    codes, s = m.router_bias()
    assert (q.bias[0] == codes).all() and (q.bias[1].mant, q.bias[1].shift) == s
    layer = tb.MoeMlp("m", q, [None] * 64, 2).with_sigmoid_router(b * 0.05)
    assert (layer.sigmoid_bias_codes == m.sigmoid_bias()).all()
    q0 = tb.QuantLinear.from_weights("r", np.ones(4, np.float32), 4, 1).with_bias(np.zeros(4, np.float32))
    assert q0.bias is None  # an all-zero bias is dropped (layers.rs:250)


def test_entry_quantiser_equals_oracle_and_golden(oracle):
    import cases

    for name in ["tiny_softmax", "config1"]:
        c = cases.CASES[name]
        x = cases.make_x(c)
        t = tb.IntTensor.from_reals(x)
        xi, xs = oracle.from_reals_f32(x)
        assert (t.data == xi.reshape(-1)).all() and (t.scale.mant, t.scale.shift) == xs
        g = GOLDEN["cases"][name]["x_int"]
        assert cases.sha(t.data.astype("<i4")) == g["data_sha256"] and [t.scale.mant, t.scale.shift] == g["scale"]


def test_tables_equal_oracle():
    for kind, name in enumerate(["exp", "silu", "sigmoid"]):
        codes, inv_step, lo_index, code_scale = tb.table(kind)
        g = GOLDEN["tables"][name]
        assert hashlib.sha256(codes.astype("<i8").tobytes()).hexdigest() == g["codes_sha256"]
        assert [inv_step.mant, inv_step.shift] == g["inv_step"] and lo_index == g["lo_index"]
        assert [code_scale.mant, code_scale.shift] == g["code_scale"]


def test_generator_is_offset_consistent_and_thread_independent():
    a = tb.synth_normal(5, 1.0, 3 << 20)
    b = tb.synth_normal(5, 1.0, 1000, offset=(3 << 20) - 1000)
    assert (a[-1000:] == b).all()
    assert abs(float(a.mean())) < 5e-3 and abs(float(a.std()) - 1.0) < 5e-3


def test_lcg_uniform_is_the_reference_lcg():
    """gate.rs:29-36 form: s = s·6364136223846793005 + 1442695040888963407, (s >> 33) mod range + lo."""
    v = tb.lcg_uniform(0x50320B00, -265720, 265720, 5)
    s, want = 0x50320B00, []
    for _ in range(5):
        s = (s * 6364136223846793005 + 1442695040888963407) & ((1 << 64) - 1)
        want.append((s >> 33) % (2 * 265720 + 1) - 265720)
    assert list(v) == want


def test_norm_codes_and_eps_equal_the_references_quantiser(oracle):
    """RmsNorm::new (layers.rs:367-388) quantises its weight like QuantLinear::from_weights, and eps with
    Scale::from_f64: the product's host preparation gives the oracle's codes and scales."""
    import tritify_b200 as tb

    d = 256
    w = tb.synth_normal(63, 1.0, d)
    _, _, wc, ws, es = oracle.rmsnorm(w, 1e-6, np.zeros(d, np.int32), (1, 0))
    q = tb.QuantLinear.from_weights("norm", w, 1, d)
    assert (q.w_codes.reshape(-1) == wc).all() and (q.w_scale.mant, q.w_scale.shift) == ws
    e = tb.scale_from_f64(1e-6)
    assert (e.mant, e.shift) == es


def test_portable_generator_on_the_host_equals_the_oracle(oracle):
    """The portable N(0, sigma) stream that the stack workloads generate on the GPU: the library's host form
    (ktmoe_synth_normal_portable) equals the oracle's restatement bit for bit, at any offset, and a window read at an
    offset equals the same elements of a longer read."""
    for seed, sigma, n, off in [(1, 0.02, 4097, 0), (3, 1.0, 1 << 16, 12345), (7, 0.02, 1000, (1 << 33) + 5)]:
        a = tb.synth_normal_portable(seed, sigma, n, off)
        b = oracle.synth_normal_portable(seed, sigma, n, off)
        assert a.dtype == np.float32 and (a.view("u4") == b.view("u4")).all()
    long = tb.synth_normal_portable(11, 1.0, 5000, 100)
    assert (tb.synth_normal_portable(11, 1.0, 1000, 2100).view("u4") == long[2000:3000].view("u4")).all()
    big = tb.synth_normal_portable(13, 1.0, 1 << 20)
    assert abs(float(big.mean())) < 5e-3 and abs(float(big.std()) - 1.0) < 5e-3


def test_int_tensor_helpers_follow_the_reference(oracle):
    """IntTensor::vector / is_empty / max_abs_data / to_f32 / quantize_probe (tensor.rs:22-49, :119-123) on the
    mirror; quantize_probe is from_reals of the f32 values (the oracle's entry quantiser)."""
    v = tb.IntTensor.vector(np.array([3, -7, 2], np.int32), tb.Scale(3, 2))
    assert v.shape == (3,) and not v.is_empty() and v.max_abs_data() == 7
    assert v.to_f32().tolist() == [2.25, -5.25, 1.5]
    assert tb.IntTensor.vector(np.zeros(0, np.int32), tb.Scale.ZERO).is_empty()
    assert tb.IntTensor.vector(np.array([-(2 ** 31)], np.int32), tb.Scale(1, 0)).max_abs_data() == 2 ** 31
    x = tb.synth_normal(21, 1.0, 257)
    p = tb.IntTensor.quantize_probe(x)
    xi, xs = oracle.from_reals_f32(x)
    assert p.shape == (257,) and (p.data == xi.reshape(-1)).all() and (p.scale.mant, p.scale.shift) == xs


def test_hash_int_and_repro_hash_are_the_reference_hashes():
    """verify::hash_int (verify.rs:35-41) and repro.rs's logits_hash (kt-convert/src/repro.rs:34-42) on the mirror:
    config 1's golden output hashes, and a scale change moves only the repro form."""
    import cases

    g = GOLDEN["cases"]["config1"]["x_int"]
    t = tb.IntTensor.from_reals(cases.make_x(cases.CASES["config1"]))
    assert tb.hash_int(t) == g["data_sha256"]
    want = cases.out_hashes(t.data, t.scale)
    assert tb.repro_hash(t) == want["repro_sha256"]
    u = tb.IntTensor(t.data, t.shape, tb.Scale(t.scale.mant + 1, t.scale.shift))
    assert tb.hash_int(u) == tb.hash_int(t) and tb.repro_hash(u) != tb.repro_hash(t)
    assert tb.hash_int(tb.IntTensor.vector(np.zeros(0, np.int32), tb.Scale.ZERO)) == hashlib.sha256(b"").hexdigest()
