"""The MoE layer on the B200 (ktmoe_forward / ktmoe_route) against the oracle and the golden hashes: bit-identical
outputs (data and scale), routing, the edge cases the reference handles, and determinism."""

import json
import os
import sys

import numpy as np
import pytest

import tritify_b200 as tb

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
GOLDEN = json.load(open(os.path.join(HERE, "golden", "golden.json")))

import cases  # noqa: E402

SMALL = ["tiny_softmax", "tiny_softmax_norm_one_row", "tiny_softmax_37rows", "tiny_router_bias",
         "tiny_sigmoid_shared", "tiny_sigmoid_raw_shared_one_row", "small_shared_softmax", "tiny_odd_hidden",
         "tiny_gated_shared", "tiny_gated_shared_one_row", "small_gated_shared"]


def _diff(a, b):
    bad = np.nonzero(a.reshape(-1) != b.reshape(-1))[0]
    return f"{bad.size} of {a.size} differ; first {bad[:5]}: {a.reshape(-1)[bad[:5]]} vs {b.reshape(-1)[bad[:5]]}"


@pytest.mark.parametrize("name", SMALL)
def test_small_cases_equal_the_oracle(ctx, oracle, name):
    c = cases.CASES[name]
    x = tb.IntTensor.from_reals(cases.make_x(c))
    m = cases.build_layer(c, ctx)
    o = cases.build_oracle(c, oracle)
    # stage 1: routing
    ex, ec, sumc = o.route(x.data.reshape(c.T, c.d), (x.scale.mant, x.scale.shift))
    routes = m.route(x)
    got_ex = np.array([r.experts for r in routes])
    got_ec = np.array([r.ec for r in routes])
    got_sumc = np.array([r.sumc for r in routes])
    lg, ls = o.router_logits(x.data.reshape(c.T, c.d), (x.scale.mant, x.scale.shift))
    dl = m.device_layer().debug_fetch(0, c.T)
    dls = m.device_layer().debug_fetch(1, c.T)
    assert (dl == lg).all(), "router logits: " + _diff(dl, lg)
    assert [(s.mant, s.shift) for s in dls] == ls, "router logit scales"
    assert (got_ex == ex).all(), "experts: " + _diff(got_ex, ex)
    assert (got_ec == ec).all(), "ec: " + _diff(got_ec, ec)
    assert (got_sumc == sumc).all(), "sumc: " + _diff(got_sumc, sumc)
    # stage 2: per-token combine outputs
    y = m.forward_int(x)
    ty, tys = o.forward_tokens(x.data.reshape(c.T, c.d), (x.scale.mant, x.scale.shift))
    dty = m.device_layer().debug_fetch(2, c.T)
    dtys = m.device_layer().debug_fetch(3, c.T)
    assert [(s.mant, s.shift) for s in dtys] == tys, "per-token scales"
    assert (dty == ty).all(), "per-token outputs: " + _diff(dty, ty)
    # the layer output, against the oracle and the committed golden hash
    want, ws = o.forward(x.data.reshape(c.T, c.d), (x.scale.mant, x.scale.shift))
    assert (y.scale.mant, y.scale.shift) == ws
    assert (y.data.reshape(want.shape) == want).all(), "output: " + _diff(y.data, want)
    assert cases.out_hashes(y.data, y.scale) == GOLDEN["cases"][name]["output"]


@pytest.mark.parametrize("pair", ["1", "0"])
@pytest.mark.parametrize("name", ["config1", "config1_norm_topk"])
def test_config1_is_bit_identical_to_the_golden_hash(ctx, name, pair, monkeypatch):
    """The CPU-parity layer: d=2048, E=64, f=1408, k=8, T=512 — same SHA-256 as the CPU integer path, with the expert
    GEMMs on SM pairs (64 rows per expert on average) and, with KTMOE_PAIR=0, on single SMs."""
    monkeypatch.setenv("KTMOE_PAIR", pair)
    c = cases.CASES[name]
    g = GOLDEN["cases"][name]
    x = tb.IntTensor.from_reals(cases.make_x(c))
    assert cases.sha(x.data.astype("<i4")) == g["x_int"]["data_sha256"]
    m = cases.build_layer(c, ctx)
    y = m.forward_int(x)
    assert cases.out_hashes(y.data, y.scale) == g["output"]
    y2 = m.forward_int(x)  # determinism: a second run gives the same bytes
    assert (y2.data == y.data).all() and y2.scale == y.scale


def test_zero_input_and_zero_rows(ctx, oracle):
    c = cases.CASES["tiny_sigmoid_shared"]
    m = cases.build_layer(c, ctx)
    o = cases.build_oracle(c, oracle)
    y = m.forward_int(tb.IntTensor(np.zeros(3 * c.d, np.int32), (3, c.d), tb.Scale.ZERO))
    assert (y.data == 0).all() and y.scale == tb.Scale.ZERO
    # a zero row among non-zero rows, and a zero input scale with non-zero data
    x = tb.IntTensor.from_reals(cases.make_x(cases.CASES["tiny_sigmoid_shared"]))
    d = x.data.reshape(c.T, c.d).copy()
    d[2] = 0
    for scale in [x.scale, tb.Scale.ZERO]:
        y = m.forward_int(tb.IntTensor(d, d.shape, scale))
        want, ws = o.forward(d, (scale.mant, scale.shift))
        assert (y.data.reshape(want.shape) == want).all() and (y.scale.mant, y.scale.shift) == ws


def test_router_ties_go_to_the_lower_index(ctx, oracle):
    d, E, f, k = 64, 8, 32, 3
    rng = np.random.default_rng(3)
    router_w = np.tile(rng.standard_normal(d).astype(np.float32), (E, 1))
    experts_w = (rng.standard_normal(E * 3 * f * d) * 0.02).astype(np.float32)
    router = tb.QuantLinear.from_weights("router", router_w, E, d)
    per = 3 * f * d
    experts = [tb.SwiGluMlp(f"e{e}", tb.QuantLinear.from_weights("g", experts_w[e * per:e * per + f * d], f, d),
                            tb.QuantLinear.from_weights("u", experts_w[e * per + f * d:e * per + 2 * f * d], f, d),
                            tb.QuantLinear.from_weights("d", experts_w[e * per + 2 * f * d:(e + 1) * per], d, f))
               for e in range(E)]
    m = tb.MoeMlp("moe", router, experts, k, ctx=ctx)
    x = tb.IntTensor.from_reals(rng.standard_normal((6, d)).astype(np.float32))
    assert all(r.experts == [0, 1, 2] for r in m.route(x))
    o = oracle.MoeOracle(d, E, f, k, router_w, experts_w)
    want, ws = o.forward(x.data.reshape(6, d), (x.scale.mant, x.scale.shift))
    y = m.forward_int(x)
    assert (y.data.reshape(want.shape) == want).all() and (y.scale.mant, y.scale.shift) == ws


@pytest.mark.parametrize("T", [1, 2, 3, 63, 64, 65, 130])
def test_token_counts_around_tile_edges(ctx, oracle, T):
    c = cases.CASES["tiny_softmax_37rows"]
    m = cases.build_layer(c, ctx)
    o = cases.build_oracle(c, oracle)
    x = tb.IntTensor.from_reals(tb.synth_normal(100 + T, 1.0, T * c.d).reshape(T, c.d))
    y = m.forward_int(x)
    want, ws = o.forward(x.data.reshape(T, c.d), (x.scale.mant, x.scale.shift))
    assert (y.scale.mant, y.scale.shift) == ws
    assert (y.data.reshape(want.shape) == want).all(), _diff(y.data, want)


def test_forward_dev_equals_forward(ctx):
    torch = pytest.importorskip("torch")
    c = cases.CASES["small_shared_softmax"]
    m = cases.build_layer(c, ctx)
    x = tb.IntTensor.from_reals(cases.make_x(c))
    y = m.forward_int(x)
    xd = torch.from_numpy(x.data.copy()).cuda()
    xs = torch.tensor([x.scale.mant, x.scale.shift & 0xFFFFFFFF], dtype=torch.int64).cuda()
    yd = torch.empty_like(xd)
    ys = torch.zeros(2, dtype=torch.int64, device="cuda")
    dev = m.device_layer()
    torch.cuda.synchronize()
    dev.forward_dev(xd.data_ptr(), c.T, xs.data_ptr(), yd.data_ptr(), ys.data_ptr(), torch.cuda.current_stream().cuda_stream)
    ctx.sync(torch.cuda.current_stream().cuda_stream)
    assert (yd.cpu().numpy() == y.data).all()
    assert int(ys[0]) == y.scale.mant and (int(ys[1]) & 0xFFFFFFFF) == (y.scale.shift & 0xFFFFFFFF)


@pytest.mark.parametrize("name", ["small_shared_softmax", "tiny_softmax_37rows"])
def test_forward_dev_with_unaligned_device_buffers(ctx, name):
    """Caller buffers that start 4 bytes past a 16-byte boundary take the scalar paths of the vectorised kernels
    and give the same bytes."""
    torch = pytest.importorskip("torch")
    c = cases.CASES[name]
    m = cases.build_layer(c, ctx)
    x = tb.IntTensor.from_reals(cases.make_x(c))
    y = m.forward_int(x)
    n = c.T * c.d
    xbuf = torch.zeros(n + 4, dtype=torch.int32, device="cuda")
    ybuf = torch.full((n + 4,), -7, dtype=torch.int32, device="cuda")
    xbuf[1:n + 1] = torch.from_numpy(x.data.copy()).cuda()
    xs = torch.tensor([x.scale.mant, x.scale.shift & 0xFFFFFFFF], dtype=torch.int64).cuda()
    ys = torch.zeros(2, dtype=torch.int64, device="cuda")
    dev = m.device_layer()
    torch.cuda.synchronize()
    dev.forward_dev(xbuf.data_ptr() + 4, c.T, xs.data_ptr(), ybuf.data_ptr() + 4, ys.data_ptr(),
                    torch.cuda.current_stream().cuda_stream)
    ctx.sync(torch.cuda.current_stream().cuda_stream)
    got = ybuf.cpu().numpy()
    assert (got[1:n + 1] == y.data).all()
    assert got[0] == -7 and (got[n + 1:] == -7).all(), "wrote outside the output"
    assert int(ys[0]) == y.scale.mant


@pytest.mark.parametrize("name", ["small_shared_softmax", "tiny_sigmoid_shared", "config1_norm_topk"])
def test_graph_replays_equal_the_uncaptured_forward(ctx, name):
    """With CUDA graphs on, the first forward of a key runs and is captured, later ones replay the graph: new inputs
    in the same buffers give the same bytes as the forward without graphs."""
    torch = pytest.importorskip("torch")
    c = cases.CASES[name]
    m = cases.build_layer(c, ctx)
    dev = m.device_layer()
    x1 = tb.IntTensor.from_reals(cases.make_x(c))
    x2 = tb.IntTensor.from_reals(cases.make_x(c) * 0.5 + 0.25)
    want = [m.forward_int(x) for x in (x1, x2)]
    dev.set_graphs(True)
    try:
        xd = torch.empty(c.T * c.d, dtype=torch.int32, device="cuda")
        yd = torch.empty_like(xd)
        xs = torch.zeros(2, dtype=torch.int64, device="cuda")
        ys = torch.zeros(2, dtype=torch.int64, device="cuda")
        st = torch.cuda.current_stream().cuda_stream
        for rep in range(3):
            for x, w in zip((x1, x2), want):
                xd.copy_(torch.from_numpy(x.data.copy()))
                xs.copy_(torch.tensor([x.scale.mant, x.scale.shift & 0xFFFFFFFF], dtype=torch.int64))
                torch.cuda.synchronize()
                dev.forward_dev(xd.data_ptr(), c.T, xs.data_ptr(), yd.data_ptr(), ys.data_ptr(), st)
                ctx.sync(st)
                assert (yd.cpu().numpy() == w.data).all(), f"pass {rep}"
                assert int(ys[0]) == w.scale.mant
            # the host-buffer entry point replays its own graph too
            y = m.forward_int(x1)
            assert (y.data == want[0].data).all() and y.scale == want[0].scale
    finally:
        dev.set_graphs(False)


@pytest.mark.parametrize("graphs", [False, True])
def test_async_forwards_equal_the_synchronous_ones(ctx, graphs):
    """ktmoe_forward_async: five back-to-back calls on different inputs (and row counts) from pinned host buffers, two
    in flight at a time, then one wait; every output and scale equals the synchronous ktmoe_forward's."""
    import dataclasses

    import torch

    c = cases.CASES["small_shared_softmax"]
    dev = cases.build_layer(c, ctx).device_layer()
    dev.set_graphs(graphs)
    inputs, want = [], []
    for i, rows in enumerate([c.T, c.T, c.T - 5, c.T, 7]):
        ci = dataclasses.replace(c, T=rows, xseed=c.xseed + 100 + i)
        x = tb.IntTensor.from_reals(cases.make_x(ci))
        inputs.append((x, rows))
        want.append(dev.forward(x.data, rows, x.scale))
    xh = [torch.from_numpy(x.data.copy()).pin_memory() for x, _ in inputs]
    yh = [torch.empty(rows * c.d, dtype=torch.int32).pin_memory() for _, rows in inputs]
    ys = [tb.KtmoeScale() for _ in inputs]
    try:
        for (x, rows), xb, yb, sc in zip(inputs, xh, yh, ys):
            dev.forward_async(xb.data_ptr(), rows, x.scale, yb.data_ptr(), sc)
        dev.forward_async_wait()
        for (y, s), yb, sc in zip(want, yh, ys):
            assert (int(sc.mant), int(sc.shift)) == (s.mant, s.shift)
            assert (yb.numpy() == y).all()
    finally:
        dev.set_graphs(False)
