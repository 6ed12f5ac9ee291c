"""Regenerate tests/golden/golden.json (run from the repository root: python tests/golden/make_golden.py).

The reference (Rust) cannot be built or run here, so its only literal golden values for this path are copied in by
hand with their source lines; every other entry is produced by the CPU oracle (oracle/oracle.cpp, a restatement of
the reference's integer path) on the seeded cases of tests/cases.py and committed, so the GPU tests compare against
fixed hashes even where re-running the oracle would be slow.
"""

from __future__ import annotations

import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from oracle import oracle as O  # noqa: E402

import cases  # noqa: E402

REFERENCE_LITERALS = {
    "corpus_sha256": {
        "value": "781285bb99bcd9cb5233f708466676db41e717b6971ce70508b57ed291478352",
        "source": "crates/02-runtime/kt-runtime/src/tests_cuda.rs:9; REPRODUCE.md:16",
    },
    "k_max": {"value": 130629492, "source": "crates/02-runtime/kt-cuda/src/tests.rs:88"},
    "k_beyond_flush": {"value": 1342192, "source": "crates/02-runtime/kt-cuda/src/tests.rs:68"},
    "split_plus_wlevels": {"value": [40, 40, 40], "source": "crates/02-runtime/kt-cuda/src/tests.rs:28"},
    "split_minus_wlevels": {"value": [-40, -40, -40], "source": "crates/02-runtime/kt-cuda/src/tests.rs:29"},
    "from_ratio_3_4_apply_8": {"value": 6, "source": "crates/00-kernels/kt-int/src/lib.rs:35-36"},
    "three_quarters_times_four_thirds_apply_9": {"value": 9, "source": "crates/00-kernels/kt-int/src/lib.rs:38"},
    "isqrt_144": {"value": 12, "source": "crates/00-kernels/kt-int/src/lib.rs:39"},
    "linear_doc_example": {
        "value": {"x": [1, 2, 3, 4, 5, 6], "w": [1, 0, -1, 2, 2, 2], "rows": 2, "out": 2, "k": 3,
                  "y": [-2, 12, -2, 30]},
        "source": "crates/01-engine/kt-core/src/backend.rs:12-15",
    },
    "sigmoid_end_codes": {"value": [0, 1048576], "source": "crates/01-engine/kt-core/src/tests_glm.rs:154-155"},
}

SMALL = ["tiny_softmax", "tiny_softmax_norm_one_row", "tiny_softmax_37rows", "tiny_router_bias",
         "tiny_sigmoid_shared", "tiny_sigmoid_raw_shared_one_row", "small_shared_softmax", "tiny_odd_hidden",
         "tiny_gated_shared", "tiny_gated_shared_one_row", "small_gated_shared"]
LARGE = ["config1", "config1_norm_topk"]


def case_entry(c):
    t0 = time.time()
    router_w, expert_w, rbias, sbias, shared_w, gate_w = cases.make_weights(c)
    x = cases.make_x(c)
    xi, xs = O.from_reals_f32(x)
    m = cases.build_oracle(c, O)
    y, ys = m.forward(xi, xs)
    ex, ec, sumc = m.route(xi, xs)
    entry = {
        "params": {k: getattr(c, k) for k in c.__dataclass_fields__},
        "weights_f32_sha256": cases.sha(np.concatenate([router_w.reshape(-1), expert_w] +
                                                       ([shared_w] if shared_w is not None else []) +
                                                       ([gate_w] if gate_w is not None else []))),
        "x_f32_sha256": cases.sha(x),
        "x_int": {"data_sha256": cases.sha(xi.astype("<i4")), "scale": list(xs)},
        "output": cases.out_hashes(y, ys),
        "route_sha256": cases.sha(np.concatenate([ex.reshape(-1).astype("<i8"), ec.reshape(-1).astype("<i8"),
                                                  sumc.astype("<i8")])),
        "oracle_seconds": round(time.time() - t0, 2),
    }
    print(c.name, entry["output"]["data_sha256"][:16], entry["oracle_seconds"], "s", flush=True)
    return entry


def main():
    names = SMALL + ([] if "--small" in sys.argv else LARGE)
    tables = {}
    for kind, name in enumerate(["exp", "silu", "sigmoid"]):
        codes, inv_step, lo_index, code_scale = O.table(kind)
        tables[name] = {"codes_sha256": cases.sha(codes.astype("<i8")), "inv_step": list(inv_step),
                        "lo_index": int(lo_index), "code_scale": list(code_scale)}
    out = {
        "about": "Golden values for the integer MoE path. reference_literals are copied from the reference with "
                 "their sources; tables and cases are the CPU oracle's outputs on the seeded cases of tests/cases.py "
                 "(regenerate with python tests/golden/make_golden.py).",
        "reference_literals": REFERENCE_LITERALS,
        "tables": tables,
        "cases": {n: case_entry(cases.CASES[n]) for n in names},
    }
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.json")
    if "--small" in sys.argv and os.path.exists(path):
        old = json.load(open(path))
        for n, v in old.get("cases", {}).items():
            out["cases"].setdefault(n, v)
    with open(path, "w") as fh:
        json.dump(out, fh, indent=1, sort_keys=True)
    print("wrote", path)


if __name__ == "__main__":
    main()
