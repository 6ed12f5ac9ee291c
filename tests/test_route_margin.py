"""MoeRoute::margin (layers.rs:816-820, computed at :844-848), the route's read-only boundary diagnostic, on the
host: the library's ktmoe_route_margins equals the reference's formula over the oracle's router logits and routes
(every expert's exp code by CodeLut::index of logit - lmax, 0 below the table; strongest excluded over weakest
selected, 0 when that is 0), and MoeMlp.route attaches it to each softmax route and leaves a sigmoid route's at 0."""

import numpy as np

import tritify_b200 as tb


def _want(oracle, logits, scales, experts):
    """The reference's margin from the oracle's CodeLut index and exp table."""
    codes = oracle.table(0)[0]
    out = []
    for lg, s, ex in zip(logits, scales, experts):
        lmax = int(lg.max())
        ecs = []
        for v in lg.tolist():
            idx = oracle.table_index(0, v - lmax, s)
            ecs.append(0 if idx < 0 else int(codes[min(idx, len(codes) - 1)]))
        chosen = set(int(e) for e in ex)
        weakest = min(ecs[e] for e in chosen)
        strongest = max([ecs[j] for j in range(len(ecs)) if j not in chosen], default=0)
        out.append(strongest / weakest if weakest > 0 else 0.0)
    return np.array(out)


def _layer(oracle, d, E, f, k, seed, router_sigma=0.05):
    rng = np.random.default_rng(seed)
    router = (rng.standard_normal((E, d)) * router_sigma).astype(np.float32)
    experts = (rng.standard_normal(E * 3 * f * d) * 0.02).astype(np.float32)
    return oracle.MoeOracle(d, E, f, k, router, experts), rng


def test_margins_equal_the_references_formula(oracle):
    for d, E, k, seed, sigma in [(32, 8, 2, 1, 0.05), (64, 60, 4, 2, 0.02), (16, 4, 4, 3, 0.3), (32, 16, 8, 4, 2.0)]:
        m, rng = _layer(oracle, d, E, 8, k, seed, sigma)
        xi, xs = oracle.from_reals_f32(rng.standard_normal((40, d)).astype(np.float32))
        ex, _, _ = m.route(xi, xs)
        lg, ls = m.router_logits(xi, xs)
        got = tb.route_margins(lg, [tb.Scale(*s) for s in ls], ex)
        want = _want(oracle, lg, ls, ex)
        assert (got == want).all(), (d, E, k, got[:4], want[:4])
        assert ((got >= 0) & (got <= 1)).all()
        if k == E:
            assert (got == 0).all()  # nothing is excluded
    # identical router rows tie every logit: the cut is a full tie, margin 1
    d, E = 16, 8
    row = np.random.default_rng(5).standard_normal(d).astype(np.float32)
    m = oracle.MoeOracle(d, E, 4, 3, np.tile(row, (E, 1)), np.zeros(E * 3 * 4 * d, np.float32))
    xi, xs = oracle.from_reals_f32(np.random.default_rng(6).standard_normal((3, d)).astype(np.float32))
    ex, _, _ = m.route(xi, xs)
    lg, ls = m.router_logits(xi, xs)
    assert (tb.route_margins(lg, [tb.Scale(*s) for s in ls], ex) == 1.0).all()


class _FakeDevice:
    """Stands in for the device layer: its route and debug buffers are the oracle's."""

    def __init__(self, oracle_layer, xi, xs):
        self.ex, self.ec, self.sumc = oracle_layer.route(xi, xs)
        self.lg, self.ls = oracle_layer.router_logits(xi, xs)
        self.fetched = []

    def route(self, data, rows, scale):
        return self.ex, self.ec, self.sumc

    def debug_fetch(self, which, rows):
        self.fetched.append(which)
        return self.lg if which == 0 else [tb.Scale(*s) for s in self.ls]


def test_route_attaches_the_margin_to_softmax_routes_only(oracle):
    d, E, f, k = 32, 8, 8, 2
    om, rng = _layer(oracle, d, E, f, k, 11)
    x = tb.IntTensor.from_reals(rng.standard_normal(5 * d).astype(np.float32))
    xi, xs = x.data.reshape(5, d), (x.scale.mant, x.scale.shift)
    router = tb.QuantLinear("router", np.zeros((E, d), np.int32), tb.Scale(1, 0), E, d)
    m = tb.MoeMlp.remote("m", router, k)
    fake = _FakeDevice(om, xi, xs)
    m._dev = fake
    routes = m.route(x)
    want = _want(oracle, fake.lg, fake.ls, fake.ex)
    assert [r.margin for r in routes] == want.tolist() and sorted(fake.fetched) == [0, 1]
    assert [r.experts for r in routes] == fake.ex.tolist() and [r.sumc for r in routes] == fake.sumc.tolist()
    m.with_sigmoid_router(np.zeros(E, np.float32))
    fake2 = _FakeDevice(om, xi, xs)
    m._dev = fake2
    assert all(r.margin == 0.0 for r in m.route(x)) and fake2.fetched == []
