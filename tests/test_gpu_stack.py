"""A stack of MoE block FFN halves, x ← add(x, moe_l(rms_norm_l(x))) for each layer l (kt-core model.rs:175-181; the
shape of a GLM-4.5-Air-style model's MoE layers with attention excluded), with the residual stream on the device
between layers, against the oracle's layer-by-layer loop; with and without the layers' CUDA graphs."""

import dataclasses
import os
import sys

import numpy as np
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


# ── a stack held as weight slots of one layer, its weights synthesised on the GPU ──
ROOT = os.path.dirname(HERE)
sys.path.insert(0, ROOT)
import bench  # noqa: E402

SMALL_STACK = dict(d=256, E=16, f=192, k=4, T=24, norm=True, sigmoid=True, shared=128, xseed=7, stack=3, lseed=500)


def test_portable_stream_on_the_device_equals_the_host(ctx, oracle):
    """The portable normal stream (own ln and cos from IEEE operations) gives the same f32 bits on the GPU as on the
    host, in the library and in the oracle's restatement."""
    import ctypes

    import torch

    from tritify_b200 import _native

    for seed, sigma, offset, n in [(1000, 0.02, 0, 3_000_017), (7, 1.0, 123_456_789, 65_536)]:
        buf = torch.empty(n, dtype=torch.float32, device=f"cuda:{ctx.device}")
        assert tb.lib().ktmoe_synth_normal_portable_dev(ctx.handle, seed, sigma, offset, n,
                                                        ctypes.c_void_p(buf.data_ptr())) == _native.OK
        got = buf.cpu().numpy().view("u4")
        assert (got == tb.synth_normal_portable(seed, sigma, n, offset).view("u4")).all()
        assert (got == oracle.synth_normal_portable(seed, sigma, n, offset).view("u4")).all()


@pytest.mark.parametrize("gated,sigmoid", [(False, True), (True, False)])
def test_weights_synthesised_on_the_gpu_equal_the_host_quantiser(ctx, oracle, gated, sigmoid):
    """ktmoe_layer_synth_weights (generation, per-tensor quantiser and packing on the GPU) gives the layer the oracle
    builds from the same portable stream with QuantLinear::from_weights on the host: the forwards agree bit for bit."""
    w = dict(SMALL_STACK, gated=gated, sigmoid=sigmoid)
    seed = 4242
    dev = tb.DeviceLayer(ctx, w["d"], w["E"], w["f"], w["k"], w["norm"], w["sigmoid"], w["shared"])
    dev.synth_weights(seed, 0.02, 0.02, gated)
    o = bench.portable_oracle_layer(w, oracle, seed)
    x = tb.IntTensor.from_reals(tb.synth_normal(w["xseed"], 1.0, w["T"] * w["d"]))
    y, ys = dev.forward(x.data, w["T"], x.scale)
    want, ws = o.forward(x.data.reshape(w["T"], w["d"]), (x.scale.mant, x.scale.shift))
    assert (ys.mant, ys.shift) == ws
    assert (y.reshape(want.shape) == want).all()


@pytest.mark.parametrize("graphs", [False, True])
def test_slot_stack_equals_the_oracle_loop(ctx, oracle, graphs):
    """Three blocks held as weight slots of one layer (shared scratch), weights synthesised on the GPU per slot,
    against the oracle's layer loop x <- add(x, moe_l(rms_norm(x))) on the same portable weights."""
    w = dict(SMALL_STACK)
    L = w["stack"]
    dev = tb.DeviceLayer(ctx, w["d"], w["E"], w["f"], w["k"], w["norm"], w["sigmoid"], w["shared"])
    dev.set_depth(L)
    norm = tb.QuantLinear.from_weights("norm", np.ones(w["d"], np.float32), 1, w["d"])
    for i in range(L):
        dev.select(i)
        dev.synth_weights(bench.stack_seed(w, i))
        dev.set_norm(norm.w_codes, norm.w_scale, tb.scale_from_f64(bench.STACK_EPS))
    dev.set_graphs(graphs)
    stack = tb.MoeStack([dev.slot(i) for i in range(L)])
    x = tb.IntTensor.from_reals(tb.synth_normal(w["xseed"], 1.0, w["T"] * w["d"]))
    want, ws = bench.stack_oracle(w, oracle, L)
    try:
        for _ in range(3 if graphs else 1):
            got = stack.forward(x)
            assert (got.scale.mant, got.scale.shift) == ws
            assert (got.data.reshape(want.shape) == want).all()
    finally:
        dev.set_graphs(False)
