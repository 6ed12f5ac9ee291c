"""The cross-rank steps of expert parallelism, on CPU ranks (gloo, world size 2).

With the layer's tokens split over ranks, the per-token outputs (route + experts + combine) are placement-independent
(crates/01-engine/kt-core/src/layers.rs:888-892), but the merge into one tensor (layers.rs:1001-1019) needs two
values over all ranks' tokens: the common scale, which the reference folds as "the last token whose scale is
largest", and the max |f_t·o_t|. The library exchanges a record (scale, global token index) per rank and reduces it
with the rule larger value first, larger index on ties, then all-reduces the max; this test runs that protocol over
gloo with the oracle's per-token outputs and requires the merged tensor to equal the oracle's single-process forward,
for even splits, uneven splits, and a rank without tokens.
"""

import os
import socket
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)


def _better(O, a, b):
    """(scale, index) a vs b: the larger exact value, the larger index on ties (the library's reduce rule)."""
    ab, ba = O.ge(a[0], b[0]), O.ge(b[0], a[0])
    if ab and not ba:
        return a
    if ba and not ab:
        return b
    return a if a[1] > b[1] else b


def _worker(rank, world, port, name, sizes, outdir):
    import torch
    import torch.distributed as dist

    from oracle import oracle as O

    import cases

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    c = cases.CASES[name]
    m = cases.build_oracle(c, O)
    x = cases.make_x(c)
    xi, xs = O.from_reals_f32(x)
    start = sum(sizes[:rank])
    rows = sizes[rank]
    d = c.d
    # per-token outputs of this rank's tokens (route, experts, combine: independent of where the tokens are)
    if rows:
        outs, scales = m.forward_tokens(xi[start:start + rows], xs)
    else:
        outs, scales = np.zeros((0, d), np.int32), []
    # the record of this rank: its best (scale, global token index), (0, -1) without tokens
    best = ((0, 0), -1)
    for t, s in enumerate(scales):
        best = _better(O, best, (s, start + t))
    rec = torch.tensor([best[0][0], best[0][1], best[1]], dtype=torch.int64)
    recs = [torch.zeros(3, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(recs, rec)
    common = ((0, 0), -1)
    for r in recs:
        common = _better(O, common, ((int(r[0]), int(r[1])), int(r[2])))
    common = common[0]
    gmax = 0
    fs = []
    if common[0]:
        cinv = O.recip(common)
        for t in range(rows):
            f = O.mul(scales[t], cinv)
            fs.append(f)
            gmax = max(gmax, max(abs(O.apply(f, int(v))) for v in outs[t]))
    g = torch.tensor([gmax], dtype=torch.int64)
    dist.all_reduce(g, op=dist.ReduceOp.MAX)
    gmax = int(g.item())
    if common[0] == 0 or gmax == 0:
        y, ys = np.zeros((rows, d), np.int32), (0, 0)
    else:
        y = np.array([[O.requant_dyn(O.apply(fs[t], int(v)), O.ACT_LEVELS, gmax) for v in outs[t]]
                      for t in range(rows)], dtype=np.int32).reshape(rows, d)
        ys = O.mul(O.from_ratio(gmax, O.ACT_LEVELS), common)
    np.savez(os.path.join(outdir, f"rank{rank}.npz"), y=y, mant=ys[0], shift=ys[1], rows=rows)
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("name,sizes", [("tiny_softmax_37rows", [19, 18]), ("tiny_softmax_37rows", [30, 7]),
                                        ("tiny_softmax", [0, 5]), ("tiny_router_bias", [5, 4])])
def test_distributed_merge_equals_one_process(tmp_path, name, sizes):
    import torch.multiprocessing as mp

    from oracle import oracle as O

    import cases

    O.build()
    c = cases.CASES[name]
    assert sum(sizes) == c.T
    mp.spawn(_worker, args=(len(sizes), _free_port(), name, sizes, str(tmp_path)), nprocs=len(sizes), join=True)
    ys, scales = [], set()
    for r in range(len(sizes)):
        z = np.load(tmp_path / f"rank{r}.npz")
        if int(z["rows"]):
            ys.append(z["y"])
            scales.add((int(z["mant"]), int(z["shift"])))
    assert len(scales) == 1
    xi, xs = O.from_reals_f32(cases.make_x(c))
    want, ws = cases.build_oracle(c, O).forward(xi, xs)
    assert scales.pop() == ws
    assert (np.concatenate(ys) == want).all()
