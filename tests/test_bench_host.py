"""Host-side arithmetic of bench.py: the decode roofline's algorithmic bytes, the reference-LCG stream of the
standalone GEMM workload, and the LinearBackend shapes of the reference's cuda_bench example."""

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
import tritify_b200 as tb  # noqa: E402


def test_decode_bytes_count_the_touched_experts():
    w = bench.WORKLOADS["glm_decode"]
    all_touched = np.ones(w["E"], np.int64)
    # 129 experts' planes (128 routed + shared) of 3·4096·1408 codes at 3 B, the router, 128 tokens in and out
    want = 3 * (128 * 3 * 4096 * 1408 + 128 * 4096 + 3 * 4096 * 1408) + 2 * 128 * 4096 * 4
    assert bench.decode_bytes(w, all_touched, 1) == [want]
    per = bench.decode_bytes(w, all_touched, 8)
    assert len(per) == 8 and len(set(per)) == 1 and abs(per[0] / 1e9 - 0.884) < 1e-3
    some = all_touched.copy()
    some[:16] = 0  # GPU 0 of 8 receives nothing: only the replicated router and shared expert
    assert bench.decode_bytes(w, some, 8)[0] == 3 * (128 * 4096 + 3 * 4096 * 1408) + 2 * 16 * 4096 * 4


def test_gemm_codes_are_one_lcg_stream():
    s = 2
    for _ in range(777):
        s = (s * 6364136223846793005 + 1442695040888963407) % (1 << 64)
    assert bench.lcg_state_after(2, 777) == s
    w = dict(M=32, N=16, K=64, seed=2)
    x, wt = bench.gemm_codes(w, tb.lcg_uniform)
    assert (wt == tb.lcg_uniform(2, -2048, 2047, 32 * 64)).all()
    assert x.min() >= -127 and x.max() <= 127 and wt.min() >= -2048 and wt.max() <= 2047
    # the activations continue the same stream: drawing the weights' count first lands on the same state
    assert (x[:8] == tb.lcg_uniform(bench.lcg_state_after(2, 32 * 64), -127, 127, 8)).all()


def test_linear_bench_shapes_are_the_references():
    shapes = [(m, n, k) for m, n, k, _ in bench.linear_bench_shapes()]
    assert shapes[:3] == [(8, 2048, 2048), (1, 4864, 896), (1, 151_936, 896)]
    assert shapes[3:] == [(r, 2048, 2048) for r in (1, 2, 4, 8, 16, 32, 64)]
    x, w = bench.linear_bench_codes(tb.lcg_uniform, 1, 4864, 896)
    assert (x == tb.lcg_uniform(2, -tb.WLEVELS, tb.WLEVELS, 896)).all()
    assert (w[:5] == tb.lcg_uniform(4866, -tb.WLEVELS, tb.WLEVELS, 5)).all()


def test_committed_goldens_describe_the_workloads_bench_runs():
    """Every workload with a committed golden (tests/golden/bench_golden.json) still has the configuration the golden
    was made for, so a bench line's parity verdict compares like with like."""
    import json

    g = json.load(open(os.path.join(ROOT, "tests", "golden", "bench_golden.json")))["workloads"]
    assert {"mixtral_prefill", "glm_decode", "glm_prefill", "qwen_decode", "qwen_prefill", "config1"} <= set(g)
    for name, rec in g.items():
        w = bench.WORKLOADS[name]
        cfg = bench.gemm_config(w, name) if w.get("gemm") else bench.workload_config(w, name)
        assert cfg == rec["config"], name
        if not w.get("gemm"):
            assert (w["T"], w["E"]) == (rec["T"], rec["E"]), name
