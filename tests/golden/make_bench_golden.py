"""Regenerate tests/golden/bench_golden.json: the CPU oracle's output hashes for every workload bench.py measures.

    python tests/golden/make_bench_golden.py [workload ...]     (from the repository root; default: all of them)

Each MoE-layer workload is built in the oracle (oracle/oracle.cpp, the reference's CPU integer path restated) from
the same generator bytes the benchmark feeds the GPU (the oracle's own copy of the build-defined generator, so
nothing of the product library is loaded here), run over all of its tokens, and hashed as verify::hash_int does
(crates/01-engine/kt-core/src/verify.rs:35-41) plus the repro form that binds the output scale. The tokens are spread
over the host's cores (MoeOracle.forward_par: each token's route, experts and combine on one thread, then the
reference's merge and shared expert), which gives the serial forward's bits. The standalone GEMM's golden is the
SHA-256 of its whole exact int64 result from the oracle's Portable linear. bench.py compares every run with these.
Named workloads are (re)computed and merged into the existing file.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
from oracle import oracle as O  # noqa: E402

PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "bench_golden.json")
LAYER_WORKLOADS = ["config1", "qwen_decode", "glm_decode", "qwen_prefill", "mixtral_prefill", "mixtral_zipf",
                   "glm_prefill"]


def sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def out_hashes(y: np.ndarray, scale) -> dict:
    data = np.ascontiguousarray(y, dtype="<i4").tobytes()
    mant, shift = scale
    head = np.int64(mant).astype("<i8").tobytes() + np.int32(shift).astype("<i4").tobytes()
    return {"data_sha256": sha(data), "repro_sha256": sha(head + data), "scale": [int(mant), int(shift)]}


def layer_entry(name: str) -> dict:
    w = dict(bench.WORKLOADS[name])
    t0 = time.time()
    m = bench.build_oracle_layer(w, O)
    t_build = time.time() - t0
    xi, xs = bench.oracle_x(w, O)
    t1 = time.time()
    y, ys = m.forward_par(xi, xs)
    t_fwd = time.time() - t1
    ex, ec, sumc = m.route(xi, xs)
    load = np.bincount(ex.reshape(-1), minlength=w["E"])
    entry = {
        "T": w["T"], "E": w["E"], "config": bench.workload_config(w, name),
        "x_int": {"data_sha256": sha(np.ascontiguousarray(xi, dtype="<i4").tobytes()), "scale": list(xs)},
        "output": out_hashes(y, ys),
        "route_sha256": sha(np.concatenate([ex.reshape(-1).astype("<i8"), ec.reshape(-1).astype("<i8"),
                                            sumc.astype("<i8")]).tobytes()),
        "rows_per_expert": [int(v) for v in load],
        "oracle_seconds": {"build": round(t_build, 1), "forward": round(t_fwd, 1), "threads": os.cpu_count()},
    }
    print(f"{name}: {entry['output']['data_sha256'][:16]} scale {entry['output']['scale']} "
          f"(build {t_build:.0f} s, forward {t_fwd:.0f} s)", flush=True)
    return entry


def stack_entry(name: str) -> dict:
    """The leading bench.STACK_CHECK_LAYERS blocks of a stack workload, their weights from the portable stream the GPU
    synthesises them from."""
    w = dict(bench.WORKLOADS[name])
    t0 = time.time()
    n = min(bench.STACK_CHECK_LAYERS, w["stack"])
    y, ys = bench.stack_oracle(w, O, n)
    print(f"{name}: first {n} layers {out_hashes(y, ys)['data_sha256'][:16]} ({time.time() - t0:.0f} s)", flush=True)
    return {"T": w["T"], "E": w["E"], "layers_checked": n, "config": bench.workload_config(w, name),
            "output": out_hashes(y, ys), "oracle_seconds": round(time.time() - t0, 1)}


def gemm_entry(name: str) -> dict:
    w = dict(bench.WORKLOADS[name])
    t0 = time.time()
    x, wt = bench.gemm_codes(w, O.lcg_uniform)
    O.lib().ko_set_max_threads(0)
    y = O.linear(x, wt, w["N"], w["M"], w["K"])
    h = sha(np.ascontiguousarray(y, dtype="<i8").tobytes())
    print(f"{name}: {h[:16]} ({time.time() - t0:.0f} s)", flush=True)
    return {"T": None, "E": None, "config": bench.gemm_config(w, name), "output": {"data_sha256": h,
                                                                               "repro_sha256": h},
            "x_sha256": sha(np.ascontiguousarray(x, dtype="<i4").tobytes()),
            "w_sha256": sha(np.ascontiguousarray(wt, dtype="<i4").tobytes())}


def main():
    names = sys.argv[1:] or (LAYER_WORKLOADS + ["gemm4096", "glm_stack_decode", "glm_stack_prefill"])
    out = {"about": "CPU-oracle golden hashes of bench.py's workloads (python tests/golden/make_bench_golden.py); "
                    "output.data_sha256 is verify::hash_int of the whole output, repro_sha256 binds the scale.",
           "workloads": {}}
    if os.path.exists(PATH):
        out["workloads"].update(json.load(open(PATH)).get("workloads", {}))
    for n in names:
        kind = bench.WORKLOADS[n]
        out["workloads"][n] = gemm_entry(n) if kind.get("gemm") else stack_entry(n) if kind.get("stack") else \
            layer_entry(n)
        with open(PATH, "w") as fh:
            json.dump(out, fh, indent=1, sort_keys=True)
    print("wrote", PATH)


if __name__ == "__main__":
    main()
