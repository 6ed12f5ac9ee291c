"""The expert-parallel seam on the B200: MoeMlp::forward_int_with_experts (crates/01-engine/kt-core/src/layers.rs:945-984)
through ktmoe_layer_forward_with_experts, and the worker side (ktmoe_layer_expert_forward). With the layer's own
experts behind the callback the seam is a numeric no-op (kt-core/src/tests.rs:156-181); a router-only coordinator
(MoeMlp::remote) fed by a worker through wire frames equals the local layer (kt-model-moe/src/tests_remote.rs:37-93)."""

import json
import os
import sys

import numpy as np
import pytest

import tritify_b200 as tb
from tritify_b200 import _native

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
GOLDEN = json.load(open(os.path.join(HERE, "golden", "golden.json")))

import cases  # noqa: E402

SEAM = ["tiny_softmax", "tiny_softmax_norm_one_row", "tiny_router_bias", "tiny_sigmoid_shared",
        "tiny_sigmoid_raw_shared_one_row", "small_shared_softmax", "config1"]


def _remote_twin(c, m, ctx):
    """The coordinator of tests_remote.rs: the same router (and shared expert), no routed experts."""
    r = tb.MoeMlp.remote("coordinator", m.router, c.k, ctx=ctx).with_norm_topk_prob(c.norm)
    if m.sigmoid_bias_codes is not None:
        r.sigmoid_bias_codes = m.sigmoid_bias_codes
    if m.shared is not None:
        r = r.with_shared_expert(m.shared)
    return r


@pytest.mark.parametrize("name", SEAM)
def test_seam_with_local_experts_is_a_no_op(ctx, name):
    c = cases.CASES[name]
    x = tb.IntTensor.from_reals(cases.make_x(c))
    m = cases.build_layer(c, ctx)
    want = m.forward_int(x)
    dev = m.device_layer()
    # one batch: the worker entry point on all rows at once
    y, ys = dev.forward_with_experts(x.data, c.T, x.scale, lambda ids, xr, xs: dev.expert_forward(xr, c.T, xs, ids))
    assert ys == want.scale and (y == want.data).all()
    # the reference's per-row callback
    seen = []

    def per_row(ids, row):
        seen.append(ids)
        return m.expert_outputs(row, np.array([ids]))[0]

    got = m.forward_int_with_experts(x, per_row)
    assert got.scale == want.scale and (got.data == want.data).all()
    assert cases.out_hashes(got.data, got.scale) == GOLDEN["cases"][name]["output"]
    assert len(seen) <= c.T and all(len(s) == c.k for s in seen)


@pytest.mark.parametrize("name", ["tiny_sigmoid_shared", "small_shared_softmax"])
def test_remote_coordinator_and_worker_over_wire_frames(ctx, name):
    c = cases.CASES[name]
    x = tb.IntTensor.from_reals(cases.make_x(c))
    local = cases.build_layer(c, ctx)
    want = local.forward_int(x)
    worker_ctx = tb.Context(0)
    worker = cases.build_layer(c, worker_ctx)
    coord = _remote_twin(c, local, ctx)
    wire = {"bytes": 0}

    def remote(ids, row):
        req = row.to_bytes()  # the request crosses the wire; the ids travel beside it
        wire["bytes"] += len(req)
        outs = worker.expert_outputs(tb.IntTensor.from_bytes(req), np.array([ids]))[0]
        blob = b"".join(o.to_bytes() for o in outs)
        wire["bytes"] += len(blob)
        res, off = [], 0
        while off < len(blob):
            t, n = tb.IntTensor.from_bytes(blob[off:], with_length=True)
            res.append(t)
            off += n
        return res

    got = coord.forward_int_with_experts(x, remote)
    assert got.scale == want.scale and (got.data == want.data).all()
    assert wire["bytes"] > 0
    with pytest.raises(RuntimeError):
        coord.forward_int(x)  # a remote layer's own experts fail closed
    del worker
    worker_ctx.close()


def test_expert_forward_equals_the_oracle(ctx, oracle):
    """Requests wider than top_k (run in chunks), repeated experts and empty slots."""
    c = cases.CASES["tiny_softmax_37rows"]
    x = tb.IntTensor.from_reals(cases.make_x(c))
    xs = (x.scale.mant, x.scale.shift)
    X = x.data.reshape(c.T, c.d)
    m = cases.build_layer(c, ctx)
    o = cases.build_oracle(c, oracle)
    rng = np.random.default_rng(3)
    ids = rng.integers(-1, c.E, size=(c.T, 2 * c.k + 1)).astype(np.int32)
    ids[0, :] = 5  # one expert many times
    ids[1, :] = -1  # a row with nothing requested
    y, ys = m.device_layer().expert_forward(x.data, c.T, x.scale, ids)
    for t in range(c.T):
        for j in range(ids.shape[1]):
            e = int(ids[t, j])
            if e < 0:
                assert ys[t][j] == tb.Scale.ZERO and not y[t, j].any()
                continue
            wy, ws = o.expert(e, X[t], xs)
            assert (ys[t][j].mant, ys[t][j].shift) == ws, (t, j, e)
            assert (y[t, j] == wy).all(), (t, j, e)


def test_seam_errors(ctx):
    c = cases.CASES["tiny_softmax"]
    x = tb.IntTensor.from_reals(cases.make_x(c))
    m = cases.build_layer(c, ctx)
    dev = m.device_layer()
    with pytest.raises(tb.KtmoeError) as e:
        dev.expert_forward(x.data, c.T, x.scale, np.full((c.T, 1), c.E, np.int32))
    assert e.value.status == _native.ERR_ARG
    coord = _remote_twin(c, m, ctx)
    with pytest.raises(tb.KtmoeError) as e:
        coord.device_layer().expert_forward(x.data, c.T, x.scale, np.zeros((c.T, 1), np.int32))
    assert e.value.status == _native.ERR_STATE  # the coordinator holds no routed experts

    def broken(ids, row):
        raise ValueError("worker unreachable")

    with pytest.raises(ValueError):
        m.forward_int_with_experts(x, broken)
    with pytest.raises(ValueError):
        m.forward_int_with_experts(x, lambda ids, row: [])  # too few outputs
    want = m.forward_int(x)  # the layer stays usable
    got = m.forward_int_with_experts(x, lambda ids, row: m.expert_outputs(row, np.array([ids]))[0])
    assert got.scale == want.scale and (got.data == want.data).all()


def test_seam_with_zero_input_and_empty_routes(ctx, oracle):
    """A zero input (zero codes, zero scale): the callback sees ids -1 exactly for the rows whose route is empty
    (sumc <= 0), and the result equals the plain forward and the oracle."""
    c = cases.CASES["tiny_sigmoid_shared"]
    m = cases.build_layer(c, ctx)
    x = tb.IntTensor(np.zeros(c.T * c.d, np.int32), (c.T, c.d), tb.Scale.ZERO)
    want = m.forward_int(x)
    o = cases.build_oracle(c, oracle)
    wy, ws = o.forward(x.data.reshape(c.T, c.d), (0, 0))
    assert (want.scale.mant, want.scale.shift) == ws and (want.data.reshape(wy.shape) == wy).all()
    seen = []

    def fn(ids, xr, xs):
        seen.append(ids.copy())
        return m.device_layer().expert_forward(xr, ids.shape[0], xs, ids)

    y, ys = m.device_layer().forward_with_experts(x.data, c.T, x.scale, fn)
    assert ys == want.scale and (y == want.data).all()
    _, _, sumc = o.route(x.data.reshape(c.T, c.d), (0, 0))
    for t in range(c.T):
        assert (seen[0][t] < 0).all() == (sumc[t] <= 0)
