"""Seeded MoE-layer cases shared by the parity tests and tests/golden/make_golden.py.

Inputs come from the build-defined generator (tritify_b200.synth_normal: splitmix64 + Box-Muller, f32) because the
reference has no normal RNG. Weights of one case form one stream (seed ``wseed``, sigma 0.02) consumed tensor by
tensor in the order router [E, d], then for each expert gate [f, d], up [f, d], down [d, f], then the shared expert's
gate, up, down, then (gated cases) the shared-expert gate [d]. Hidden states are N(0, 1) from seed ``xseed``. Router bias (QuantLinear::with_bias) and the sigmoid
selection bias come from seeds ``wseed + 1`` and ``wseed + 2``.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass, field

import numpy as np

import tritify_b200 as tb


@dataclass(frozen=True)
class Case:
    name: str
    d: int
    E: int
    f: int
    k: int
    T: int
    norm: bool = False
    sigmoid: bool = False
    shared: int = 0
    router_bias: bool = False
    gated: bool = False  # the shared expert behind a sigmoid gate (extension; Qwen2-MoE shared_expert_gate)
    wseed: int = 1
    xseed: int = 0
    bias_sigma: float = 0.05


CASES = {
    c.name: c
    for c in [
        Case("tiny_softmax", d=64, E=8, f=96, k=2, T=5, wseed=11, xseed=12),
        Case("tiny_softmax_norm_one_row", d=64, E=8, f=96, k=2, T=1, norm=True, wseed=13, xseed=14),
        Case("tiny_softmax_37rows", d=128, E=16, f=64, k=4, T=37, wseed=15, xseed=16),
        Case("tiny_router_bias", d=64, E=12, f=48, k=3, T=9, norm=True, router_bias=True, wseed=17, xseed=18),
        Case("tiny_sigmoid_shared", d=64, E=16, f=48, k=4, T=7, norm=True, sigmoid=True, shared=80, wseed=19,
             xseed=20),
        Case("tiny_sigmoid_raw_shared_one_row", d=64, E=16, f=48, k=4, T=1, norm=False, sigmoid=True, shared=40,
             wseed=21, xseed=22),
        Case("small_shared_softmax", d=256, E=32, f=192, k=6, T=48, norm=True, shared=384, wseed=23, xseed=24),
        # f % 4 != 0: the SwiGLU element pass takes its block-per-row form
        Case("tiny_odd_hidden", d=64, E=6, f=50, k=2, T=11, wseed=25, xseed=26),
        # the gated shared expert (extension), with a softmax and a sigmoid router, one row and several
        Case("tiny_gated_shared", d=64, E=8, f=48, k=2, T=9, norm=True, shared=64, gated=True, wseed=27, xseed=28),
        Case("tiny_gated_shared_one_row", d=64, E=16, f=48, k=4, T=1, norm=True, sigmoid=True, shared=40, gated=True,
             wseed=29, xseed=30),
        Case("small_gated_shared", d=256, E=32, f=192, k=4, T=48, norm=True, shared=512, gated=True, wseed=31,
             xseed=32),
        # The CPU-parity layer: d=2048, E=64, f=1408, k=8, T=512, softmax, norm_topk=false,
        # hidden N(0,1) seed 0, weights N(0,0.02) seed 1.
        Case("config1", d=2048, E=64, f=1408, k=8, T=512, norm=False, wseed=1, xseed=0),
        Case("config1_norm_topk", d=2048, E=64, f=1408, k=8, T=512, norm=True, wseed=1, xseed=0),
    ]
}


def weight_count(c: Case) -> int:
    return c.E * c.d + c.E * 3 * c.f * c.d + 3 * c.shared * c.d + (c.d if c.gated else 0)


def make_weights(c: Case):
    """(router_w [E,d], expert_w flat [E·3·f·d], router_bias or None, sigmoid_bias or None, shared_w or None,
    shared_gate_w [d] or None)."""
    off = 0

    def take(n):
        nonlocal off
        a = tb.synth_normal(c.wseed, 0.02, n, offset=off)
        off += n
        return a

    router = take(c.E * c.d).reshape(c.E, c.d)
    experts = take(c.E * 3 * c.f * c.d)
    shared = take(3 * c.shared * c.d) if c.shared else None
    gate = take(c.d) if c.shared and c.gated else None
    rbias = tb.synth_normal(c.wseed + 1, 1.0, c.E) if c.router_bias else None
    sbias = tb.synth_normal(c.wseed + 2, c.bias_sigma, c.E) if c.sigmoid else None
    return router, experts, rbias, sbias, shared, gate


def make_x(c: Case) -> np.ndarray:
    return tb.synth_normal(c.xseed, 1.0, c.T * c.d).reshape(c.T, c.d)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def out_hashes(y: np.ndarray, scale) -> dict:
    """verify::hash_int (crates/01-engine/kt-core/src/verify.rs:35-41): SHA-256 of the i32 data, little-endian; and the
    repro form that also binds the scale: mant i64 LE ‖ shift i32 LE ‖ data."""
    data = np.ascontiguousarray(y, dtype="<i4")
    mant, shift = (scale.mant, scale.shift) if hasattr(scale, "mant") else scale
    h = hashlib.sha256()
    h.update(np.int64(mant).astype("<i8").tobytes())
    h.update(np.int32(shift).astype("<i4").tobytes())
    h.update(data.tobytes())
    return {"data_sha256": sha(data), "repro_sha256": h.hexdigest(), "scale": [int(mant), int(shift)]}


def build_layer(c: Case, ctx=None) -> "tb.MoeMlp":
    """The reference-shaped layer, built through the product's own host mirror (QuantLinear::from_weights etc.)."""
    router_w, expert_w, rbias, sbias, shared_w, gate_w = make_weights(c)
    router = tb.QuantLinear.from_weights("router", router_w, c.E, c.d).with_bias(rbias)
    per = 3 * c.f * c.d
    experts = []
    for e in range(c.E):
        base = expert_w[e * per:(e + 1) * per]
        experts.append(tb.SwiGluMlp(
            f"expert{e}",
            tb.QuantLinear.from_weights("gate", base[:c.f * c.d], c.f, c.d),
            tb.QuantLinear.from_weights("up", base[c.f * c.d:2 * c.f * c.d], c.f, c.d),
            tb.QuantLinear.from_weights("down", base[2 * c.f * c.d:], c.d, c.f)))
    m = tb.MoeMlp("moe", router, experts, c.k, ctx=ctx).with_norm_topk_prob(c.norm)
    if c.sigmoid:
        m = m.with_sigmoid_router(sbias)
    if c.shared:
        sd = c.shared * c.d
        m = m.with_shared_expert(tb.SwiGluMlp(
            "shared",
            tb.QuantLinear.from_weights("gate", shared_w[:sd], c.shared, c.d),
            tb.QuantLinear.from_weights("up", shared_w[sd:2 * sd], c.shared, c.d),
            tb.QuantLinear.from_weights("down", shared_w[2 * sd:], c.d, c.shared)))
        if c.gated:
            m = m.with_shared_expert_gate(tb.QuantLinear.from_weights("shared_expert_gate", gate_w, 1, c.d))
    return m


def build_oracle(c: Case, O):
    router_w, expert_w, rbias, sbias, shared_w, gate_w = make_weights(c)
    return O.MoeOracle(c.d, c.E, c.f, c.k, router_w, expert_w, router_bias=rbias, norm_topk=c.norm,
                       sigmoid_bias=sbias, shared_hidden=c.shared, shared_w=shared_w, shared_gate_w=gate_w)
