"""The Python mirror of the reference's operators refuses what the reference asserts against, with the reference's
messages, before anything reaches a device (so these run on the CPU): layers.rs:226 and :248 (QuantLinear weights and
bias lengths), :591-592 (SwiGluMlp shapes), :680-681 and :699 (MoeMlp top_k and router width), :736 (one selection
bias per expert), :990 (MoE input a multiple of dim). The reference panics; the mirror raises ValueError."""

import numpy as np
import pytest

import tritify_b200 as tb


def _lin(name, out_f, in_f, seed=1):
    return tb.QuantLinear.from_weights(name, tb.synth_normal(seed, 0.02, out_f * in_f), out_f, in_f)


def _expert(d, f, seed):
    return tb.SwiGluMlp(f"e{seed}", _lin("g", f, d, seed), _lin("u", f, d, seed + 1), _lin("d", d, f, seed + 2))


def test_quant_linear_lengths():
    with pytest.raises(ValueError, match="weights are not out·in"):
        tb.QuantLinear.from_weights("w", np.zeros(7, np.float32), 2, 4)
    q = _lin("r", 4, 8)
    with pytest.raises(ValueError, match="r: bias len mismatch"):
        q.with_bias(np.ones(3, np.float32))
    assert q.with_bias(None) is q


def test_swiglu_shapes():
    d, f = 8, 4
    with pytest.raises(ValueError, match="gate/up hidden mismatch"):
        tb.SwiGluMlp("s", _lin("g", f, d), _lin("u", f + 1, d), _lin("d", d, f))
    with pytest.raises(ValueError, match="down input != hidden"):
        tb.SwiGluMlp("s", _lin("g", f, d), _lin("u", f, d), _lin("d", d, f + 1))


def test_moe_top_k_router_width_and_selection_bias():
    d, f, E = 8, 4, 3
    experts = [_expert(d, f, 10 * i) for i in range(E)]
    router = _lin("router", E, d)
    for k in (0, E + 1):
        with pytest.raises(ValueError, match=r"top_k in 1\.\.=E"):
            tb.MoeMlp("m", router, experts, k)
        with pytest.raises(ValueError, match=r"top_k in 1\.\.=E"):
            tb.MoeMlp.remote("m", router, k)
    with pytest.raises(ValueError, match="router out_features != number of experts"):
        tb.MoeMlp("m", _lin("router", E + 1, d), experts, 2)
    m = tb.MoeMlp("m", router, experts, 2)
    with pytest.raises(ValueError, match="m: one selection bias per expert"):
        m.with_sigmoid_router(np.zeros(E + 1, np.float32))
    with pytest.raises(ValueError, match="with_shared_expert_gate needs a shared expert"):
        m.with_shared_expert_gate(_lin("sg", 1, d))
    m.with_shared_expert(_expert(d, f, 99))
    with pytest.raises(ValueError, match=r"the shared-expert gate is a \[1, dim\] linear"):
        m.with_shared_expert_gate(_lin("sg", 2, d))


def test_moe_input_must_be_rows_of_dim():
    d, f, E = 8, 4, 2
    m = tb.MoeMlp("m", _lin("router", E, d), [_expert(d, f, 3), _expert(d, f, 7)], 1)
    x = tb.IntTensor(np.zeros(d + 1, np.int32), (d + 1,), tb.Scale.ZERO)
    with pytest.raises(ValueError, match="m: MoE input length must be a multiple of dim"):
        m.forward_int(x)
    with pytest.raises(ValueError, match="m: MoE input length must be a multiple of dim"):
        m.forward_int_with_experts(x, lambda ids, row: [])
    r = tb.MoeMlp.remote("m", _lin("router", E, d), 1)
    with pytest.raises(RuntimeError, match="the routed experts are remote"):
        r.forward_int(tb.IntTensor(np.zeros(d, np.int32), (d,), tb.Scale.ZERO))


def test_a_remote_layer_takes_one_selection_bias_per_router_output():
    """layers.rs:736 compares the bias with n_experts() (the router's width), so a router-only layer whose experts
    are elsewhere takes a sigmoid router too."""
    d, E = 8, 6
    r = tb.MoeMlp.remote("r", _lin("router", E, d), 2)
    r.with_sigmoid_router(np.zeros(E, np.float32))
    assert r.sigmoid_bias_codes is not None and r.sigmoid_bias_codes.size == E
    with pytest.raises(ValueError, match="r: one selection bias per expert"):
        tb.MoeMlp.remote("r", _lin("router", E, d), 2).with_sigmoid_router(np.zeros(E - 1, np.float32))


def test_router_score_shared_expert_and_router_codes(oracle):
    """MoeMlp::router_score / shared_expert / router_codes (layers.rs:747-755, :784-788) on the mirror: the score
    function and its coded bias, the shared expert as set, and the router's exp code table (the oracle's, read-only)."""
    d, f, E = 8, 4, 3
    m = tb.MoeMlp("m", _lin("router", E, d), [_expert(d, f, 10 * i) for i in range(E)], 2)
    assert m.router_score().kind == "softmax" and m.router_score().bias_codes is None
    assert m.shared_expert() is None
    b = np.array([0.5, -0.25, 0.0], np.float32)
    m.with_sigmoid_router(b)
    sc = m.router_score()
    assert sc.kind == "sigmoid" and sc.bias_codes.tolist() == [1 << 19, -(1 << 18), 0]
    s = _expert(d, f, 77)
    assert m.with_shared_expert(s).shared_expert() is s
    codes = m.router_codes()
    assert (codes == oracle.table(0)[0]).all() and not codes.flags.writeable


def test_a_stack_takes_layers_of_one_context_and_one_width():
    """MoeStack (the block loop of model.rs:175-186 without attention) refuses an empty list and layers that do not
    share one context and one d_model; the check reads only those two attributes, so stand-ins serve here."""
    from types import SimpleNamespace as L

    with pytest.raises(ValueError, match="a stack needs at least one layer"):
        tb.MoeStack([])
    c0, c1 = object(), object()
    with pytest.raises(ValueError, match="share one context and one d_model"):
        tb.MoeStack([L(ctx=c0, d_model=8), L(ctx=c0, d_model=16)])
    with pytest.raises(ValueError, match="share one context and one d_model"):
        tb.MoeStack([L(ctx=c0, d_model=8), L(ctx=c1, d_model=8)])
    s = tb.MoeStack([L(ctx=c0, d_model=8), L(ctx=c0, d_model=8)])
    assert len(s.layers) == 2 and s.d_model == 8 and s.ctx is c0
