"""The FFN half of a decoder block, y = add(x, moe(rms_norm(x))) (crates/01-engine/kt-core/src/model.rs:175-181), on
the B200 through ktmoe_block_forward, against the oracle's RmsNorm (layers.rs:352-449), MoE layer and add
(layers.rs:121-136): integers, tolerance 0."""

import os
import sys

import numpy as np
import pytest

import tritify_b200 as tb

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import cases  # noqa: E402

EPS = 1e-6


def norm_weight(c):
    return tb.synth_normal(c.wseed + 40, 1.0, c.d)


def expected_block(c, oracle, rows=None):
    o = cases.build_oracle(c, oracle)
    xi, xs = oracle.from_reals_f32(cases.make_x(c))
    xi = xi.reshape(c.T, c.d)
    xn, xns, _, _, _ = oracle.rmsnorm(norm_weight(c), EPS, xi, xs)
    m, ms = o.forward(xn.reshape(c.T, c.d), xns)
    y, ys = oracle.add(xi.reshape(-1), xs, m.reshape(-1), ms)
    return y, ys


def set_norm(dev, c):
    q = tb.QuantLinear.from_weights("norm", norm_weight(c), 1, c.d)
    dev.set_norm(q.w_codes, q.w_scale, tb.scale_from_f64(EPS))


@pytest.mark.parametrize("name", ["tiny_softmax_37rows", "small_shared_softmax", "tiny_sigmoid_shared",
                                  "tiny_sigmoid_raw_shared_one_row"])
@pytest.mark.parametrize("graphs", [False, True])
def test_block_equals_the_oracle(ctx, oracle, name, graphs):
    c = cases.CASES[name]
    m = cases.build_layer(c, ctx)
    dev = m.device_layer()
    set_norm(dev, c)
    dev.set_graphs(graphs)
    try:
        want, ws = expected_block(c, oracle)
        x = tb.IntTensor.from_reals(cases.make_x(c))
        for _ in range(3 if graphs else 1):
            y, ys = dev.block_forward(x.data, c.T, x.scale)
            assert (ys.mant, ys.shift) == ws
            bad = np.nonzero(y != want)[0]
            assert bad.size == 0, f"{bad.size} of {y.size} differ"
    finally:
        dev.set_graphs(False)
