"""bench.py's workloads at their full shapes on the B200 against the CPU oracle's golden hashes
(tests/golden/bench_golden.json, made by tests/golden/make_bench_golden.py): the whole output of the layer, data and
scale, is the reference CPU path's (verify::hash_int, crates/01-engine/kt-core/src/verify.rs:35-41, plus the scale).

These are the shapes the benchmark's numbers are quoted on: K = 14336 in Mixtral's down GEMM with ~2048 rows per
expert, softmax with norm_topk at E = 8, a Zipf-skewed router bias, Qwen's 5632-wide shared expert, GLM's sigmoid
router with selection bias and shared expert at d = 4096, and the decode batches."""

import json
import os
import sys

import numpy as np
import pytest

import tritify_b200 as tb

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, ROOT)

import bench  # noqa: E402

GOLDEN = json.load(open(os.path.join(HERE, "golden", "bench_golden.json")))["workloads"]


def _hashes(y, ys):
    import hashlib

    data = np.ascontiguousarray(y, dtype="<i4").tobytes()
    head = np.int64(ys.mant).astype("<i8").tobytes() + np.int32(ys.shift).astype("<i4").tobytes()
    return {"data_sha256": hashlib.sha256(data).hexdigest(), "repro_sha256": hashlib.sha256(head + data).hexdigest(),
            "scale": [int(ys.mant), int(ys.shift)]}


def _run(ctx, name, monkeypatch, variants):
    w = dict(bench.WORKLOADS[name])
    g = GOLDEN[name]
    dev = bench.build_product_layer(w, ctx)
    x = bench.make_x(w)
    import hashlib

    xh = hashlib.sha256(np.ascontiguousarray(x.data, dtype="<i4").tobytes()).hexdigest()
    assert xh == g["x_int"]["data_sha256"] and [x.scale.mant, x.scale.shift] == g["x_int"]["scale"], \
        "entry quantiser differs from the oracle's"
    for env in variants:
        for k, v in env.items():
            monkeypatch.setenv(k, v)
        y, ys = dev.forward(x.data, w["T"], x.scale)
        assert _hashes(y, ys) == g["output"], f"{name} {env}: output differs from the CPU oracle's golden"
    ex, _, _ = dev.route(x.data, w["T"], x.scale)
    assert np.bincount(ex.reshape(-1), minlength=w["E"]).tolist() == g["rows_per_expert"], "routing load"
    del dev  # frees the layer's device memory before the next workload


@pytest.mark.parametrize("name", ["qwen_decode", "glm_decode", "config1"])
def test_decode_and_config1_workloads_equal_the_golden(ctx, name, monkeypatch):
    # both SwiGLU element kernels: a block per row, and a cluster per row with h in registers (both thread shapes)
    _run(ctx, name, monkeypatch, [{"KTMOE_SWIGLU_CLUSTER": "0"},
                                  {"KTMOE_SWIGLU_CLUSTER": "1", "KTMOE_SWIGLU_SHAPE": "2x256"},
                                  {"KTMOE_SWIGLU_CLUSTER": "1", "KTMOE_SWIGLU_SHAPE": "4x128"},
                                  {"KTMOE_SWIGLU_CLUSTER": "0", "KTMOE_PAIR_ZERO_MMA": "1"},
                                  {"KTMOE_PAIR_ZERO_MMA": "0"},
                                  {"KTMOE_COMBINE": "0"},  # the thread-per-token plan and a CTA per token
                                  {"KTMOE_COMBINE": "1"},  # a warp plan inside each token's cluster of CTAs
                                  {"KTMOE_SWIGLU_INLINE": "0"},  # the SwiGLU row plans and down c as kernels
                                  {"KTMOE_SWIGLU_INLINE": "1"},  # and inside the row kernel
                                  {"KTMOE_PLAN_ONE": "0"},  # the routing plan as count, scan and assign kernels
                                  {"KTMOE_PLAN_ONE": "1"}])  # and as one launch


@pytest.mark.parametrize("name", ["qwen_prefill", "mixtral_prefill", "mixtral_zipf", "glm_prefill"])
def test_prefill_workloads_equal_the_golden(ctx, name, monkeypatch):
    # the pair GEMM with the epilogue zeroing the accumulator, and with the clearing MMA
    variants = [{"KTMOE_SWIGLU_CLUSTER": "0", "KTMOE_PAIR_ZERO_MMA": "0"}, {"KTMOE_PAIR_ZERO_MMA": "1"}]
    # the combine's thread-per-token plan kernel, then back to the warp-per-token one
    variants += [{"KTMOE_COMBINE": "0"}, {"KTMOE_COMBINE": "1"}]
    if name == "mixtral_prefill":
        variants.append({"KTMOE_SWIGLU_CLUSTER": "1"})  # the 14336-wide rows on 8-CTA clusters as well
        variants.append({"KTMOE_SWIGLU_CLUSTER": "0", "KTMOE_SWIGLU_U": "2"})  # and two elements per thread step
        variants.append({"KTMOE_SWIGLU_V": "1", "KTMOE_SWIGLU_U": "4"})  # the first lean element path
        variants.append({"KTMOE_SWIGLU_V": "2"})
        # and split over a 2-CTA cluster with h in shared memory
        variants.append({"KTMOE_SWIGLU_CLUSTER": "0", "KTMOE_SWIGLU_U": "4", "KTMOE_SWIGLU_SLICE": "1"})
    _run(ctx, name, monkeypatch, variants)
