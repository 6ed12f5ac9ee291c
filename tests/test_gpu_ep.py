"""Expert parallelism (ktmoe_layer_create_ep), over NCCL and over peer memory (ktmoe_layer_set_ep_capacity): the rows
of each rank, concatenated in rank order, must be bit-identical to the single-GPU forward (and so to the golden hashes
of the CPU path). Needs two or more GPUs; the ranks run as spawned processes, one per GPU."""

import json
import os
import socket
import sys

import numpy as np
import pytest

import tritify_b200 as tb

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
GOLDEN = json.load(open(os.path.join(HERE, "golden", "golden.json")))

import cases  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _splits(T, world, mode):
    if mode == "even":
        base = [T // world] * world
        for i in range(T % world):
            base[i] += 1
        return base
    if mode == "first_empty":
        return [0] + [T // (world - 1) + (1 if i < T % (world - 1) else 0) for i in range(world - 1)]
    raise ValueError(mode)


def _worker(rank, world, port, name, mode, transport, outdir):
    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    nid = torch.zeros(128, dtype=torch.uint8, device="cuda")
    if rank == 0:
        nid.copy_(torch.frombuffer(bytearray(tb.ep_unique_id()), dtype=torch.uint8))
    dist.broadcast(nid, 0)
    c = cases.CASES[name]
    ctx = tb.Context(rank)
    m = cases.build_layer(c, ctx)  # the host mirror (quantised weights); only this rank's experts go to its device
    dev = tb.DeviceLayer(ctx, c.d, c.E, c.f, c.k, c.norm, c.sigmoid, c.shared,
                         ep=(rank, world, bytes(nid.cpu().numpy().tobytes())))
    dev.set_router(m.router.w_codes, m.router.w_scale, m.router.bias)
    if c.sigmoid:
        dev.set_sigmoid_bias(m.sigmoid_bias_codes)
    for e in dev.experts:
        ex = m.experts[e]
        dev.set_expert(e, (ex.gate.w_codes, ex.gate.w_scale), (ex.up.w_codes, ex.up.w_scale),
                       (ex.down.w_codes, ex.down.w_scale))
    if c.shared:
        s = m.shared
        dev.set_shared((s.gate.w_codes, s.gate.w_scale), (s.up.w_codes, s.up.w_scale), (s.down.w_codes, s.down.w_scale))
        if m.shared_gate is not None:
            dev.set_shared_gate((m.shared_gate.w_codes, m.shared_gate.w_scale))
    block = mode.endswith(":block")
    mode = mode.split(":")[0]
    if block:
        import test_gpu_block as tgb

        tgb.set_norm(dev, c)
    x = tb.IntTensor.from_reals(cases.make_x(c))
    sizes = _splits(c.T, world, mode)
    start = sum(sizes[:rank])
    rows = sizes[rank]
    xr = x.data.reshape(c.T, c.d)[start:start + rows]
    if transport.startswith("peer"):
        dev.set_ep_capacity(max(sizes))  # collective: every rank passes the same capacity
    if transport == "peer_graphs":
        dev.set_graphs(True)
    for rep in range(3):  # the later forwards reuse every buffer (and, over peer memory, the flags)
        y, ys = dev.forward(xr, rows, x.scale, block=block)
    np.savez(os.path.join(outdir, f"rank{rank}.npz"), y=y, mant=ys.mant, shift=ys.shift, rows=rows)
    dev = None
    ctx.sync()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("transport", ["nccl", "peer", "peer_graphs"])
@pytest.mark.parametrize("name,mode", [("tiny_softmax_37rows", "even"), ("small_shared_softmax", "even"),
                                       ("tiny_sigmoid_shared", "first_empty"), ("config1", "even"),
                                       ("tiny_sigmoid_raw_shared_one_row", "first_empty"),
                                       ("small_gated_shared", "even"), ("tiny_gated_shared", "first_empty")])
def test_expert_parallel_equals_one_gpu(tmp_path, name, mode, transport):
    import torch
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("expert parallelism needs two or more GPUs")
    c = cases.CASES[name]
    world = min(world, c.E)
    if mode == "first_empty" and c.T < world - 1:
        world = 2
    mp.spawn(_worker, args=(world, _free_port(), name, mode, transport, str(tmp_path)), nprocs=world, join=True)
    ys, scales = [], set()
    for r in range(world):
        z = np.load(tmp_path / f"rank{r}.npz")
        if int(z["rows"]) > 0:
            ys.append(z["y"])
            scales.add((int(z["mant"]), int(z["shift"])))
    assert len(scales) == 1, f"ranks disagree on the output scale: {scales}"
    y = np.concatenate(ys)
    assert cases.out_hashes(y, scales.pop()) == GOLDEN["cases"][name]["output"]


@pytest.mark.parametrize("transport", ["nccl", "peer", "peer_graphs"])
@pytest.mark.parametrize("name,mode", [("small_shared_softmax", "even"), ("tiny_sigmoid_shared", "first_empty")])
def test_expert_parallel_block_equals_the_oracle(tmp_path, oracle, name, mode, transport):
    """The block x + moe(rms_norm(x)) with the layer's experts spread over the GPUs: the norm's common scale and
    maxima and the residual add's maximum span every rank's rows."""
    import torch
    import torch.multiprocessing as mp

    import test_gpu_block as tgb

    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("expert parallelism needs two or more GPUs")
    c = cases.CASES[name]
    world = min(world, c.E)
    if mode == "first_empty" and c.T < world - 1:
        world = 2
    mp.spawn(_worker, args=(world, _free_port(), name, mode + ":block", transport, str(tmp_path)), nprocs=world,
             join=True)
    want, ws = tgb.expected_block(c, oracle)
    ys, scales = [], set()
    for r in range(world):
        z = np.load(tmp_path / f"rank{r}.npz")
        if int(z["rows"]) > 0:
            ys.append(z["y"])
            scales.add((int(z["mant"]), int(z["shift"])))
    assert scales == {ws}
    assert (np.concatenate(ys) == want).all()


STACK = dict(d=256, E=16, f=192, k=4, T=24, norm=True, sigmoid=True, shared=128, xseed=7, stack=3, lseed=500)


def _stack_worker(rank, world, port, outdir):
    import datetime

    import torch
    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(HERE))
    import bench

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    nid = torch.zeros(128, dtype=torch.uint8, device="cuda")
    if rank == 0:
        nid.copy_(torch.frombuffer(bytearray(tb.ep_unique_id()), dtype=torch.uint8))
    dist.broadcast(nid, 0)
    w = STACK
    ctx = tb.Context(rank)
    dev = tb.DeviceLayer(ctx, w["d"], w["E"], w["f"], w["k"], w["norm"], w["sigmoid"], w["shared"],
                         ep=(rank, world, bytes(nid.cpu().numpy().tobytes())))
    dev.set_depth(w["stack"])
    norm = tb.QuantLinear.from_weights("norm", np.ones(w["d"], np.float32), 1, w["d"])
    for i in range(w["stack"]):
        dev.select(i)
        dev.synth_weights(bench.stack_seed(w, i))  # each rank draws only its own experts
        dev.set_norm(norm.w_codes, norm.w_scale, tb.scale_from_f64(bench.STACK_EPS))
    sizes = _splits(w["T"], world, "even")
    dev.set_ep_capacity(max(sizes))
    dev.set_graphs(True)
    x = tb.IntTensor.from_reals(tb.synth_normal(w["xseed"], 1.0, w["T"] * w["d"]))
    start, rows = sum(sizes[:rank]), sizes[rank]
    xr = tb.IntTensor(x.data.reshape(w["T"], w["d"])[start:start + rows].reshape(-1), (rows, w["d"]), x.scale)
    stack = tb.MoeStack([dev.slot(i) for i in range(w["stack"])])
    for _ in range(3):
        y = stack.forward(xr)
    np.savez(os.path.join(outdir, f"rank{rank}.npz"), y=y.data, mant=y.scale.mant, shift=y.scale.shift, rows=rows)
    stack = dev = None
    ctx.sync()
    dist.barrier()
    dist.destroy_process_group()


def test_expert_parallel_slot_stack_equals_the_oracle(tmp_path, oracle):
    """A stack of three blocks held as weight slots, the experts spread over the GPUs and synthesised there, the
    exchange over peer memory with CUDA graphs: the ranks' rows together equal the oracle's layer loop."""
    import torch
    import torch.multiprocessing as mp

    sys.path.insert(0, os.path.dirname(HERE))
    import bench

    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("expert parallelism needs two or more GPUs")
    mp.spawn(_stack_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    want, ws = bench.stack_oracle(STACK, oracle, STACK["stack"])
    ys, scales = [], set()
    for r in range(world):
        z = np.load(tmp_path / f"rank{r}.npz")
        if int(z["rows"]) > 0:
            ys.append(z["y"].reshape(-1))
            scales.add((int(z["mant"]), int(z["shift"])))
    assert scales == {ws}
    assert (np.concatenate(ys) == want.reshape(-1)).all()
