"""A stack of MoE block FFN halves, x ← add(x, moe_l(rms_norm_l(x))) for each layer l (kt-core model.rs:175-181; the
shape of a GLM-4.5-Air-style model's MoE layers with attention excluded), with the residual stream on the device
between layers, against the oracle's layer-by-layer loop; with and without the layers' CUDA graphs."""

import dataclasses
import os
import sys

import pytest

import tritify_b200 as tb

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import cases  # noqa: E402
import test_gpu_block as tgb  # noqa: E402


def _layers(base, n):
    """n layers of the base case's shape, each with its own weights (and norm) stream."""
    return [dataclasses.replace(base, name=f"{base.name}_layer{i}", wseed=base.wseed + 100 * i) for i in range(n)]


@pytest.mark.parametrize("name,n", [("tiny_sigmoid_shared", 3), ("small_shared_softmax", 2),
                                    ("tiny_softmax_norm_one_row", 3)])
@pytest.mark.parametrize("graphs", [False, True])
def test_stack_equals_the_oracle_loop(ctx, oracle, name, n, graphs):
    base = cases.CASES[name]
    layer_cases = _layers(base, n)
    held = []
    for c in layer_cases:
        m = cases.build_layer(c, ctx)
        dev = m.device_layer()
        tgb.set_norm(dev, c)
        dev.set_graphs(graphs)
        held.append((m, dev))
    stack = tb.MoeStack([dev for _, dev in held])
    x = tb.IntTensor.from_reals(cases.make_x(base))
    xi, xs = x.data.reshape(base.T, base.d), (x.scale.mant, x.scale.shift)
    for c in layer_cases:
        o = cases.build_oracle(c, oracle)
        xn, xns, _, _, _ = oracle.rmsnorm(tgb.norm_weight(c), tgb.EPS, xi, xs)
        moe, ms = o.forward(xn.reshape(base.T, base.d), xns)
        y, ys = oracle.add(xi.reshape(-1), xs, moe.reshape(-1), ms)
        xi, xs = y.reshape(base.T, base.d), ys
    try:
        for _ in range(3 if graphs else 1):  # graph replays reuse the stack's buffers
            got = stack.forward(x)
            assert (got.scale.mant, got.scale.shift) == xs
            assert (got.data.reshape(xi.shape) == xi).all()
    finally:
        for _, dev in held:
            dev.set_graphs(False)


def test_stack_rejects_mixed_layers(ctx):
    a = cases.build_layer(cases.CASES["tiny_softmax"], ctx).device_layer()
    b = cases.build_layer(cases.CASES["tiny_softmax_37rows"], ctx).device_layer()
    with pytest.raises(ValueError):
        tb.MoeStack([a, b])
    with pytest.raises(ValueError):
        tb.MoeStack([])
