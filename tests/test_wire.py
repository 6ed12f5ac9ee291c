"""The activation wire format, IntTensor::to_bytes / from_bytes (crates/01-engine/kt-core/src/tensor.rs:51-100), in the
product (ktmoe_wire_encode / ktmoe_wire_decode, host-only) against the oracle's restatement of the layout; and the
expert-parallel seam carried across processes in it (gloo ranks on CPU: a coordinator that routes and combines, a
worker that computes the experts; MoeMlp::forward_int_with_experts, layers.rs:945-984)."""

import os
import socket
import struct
import sys

import numpy as np
import pytest

import tritify_b200 as tb
from tritify_b200 import _native

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)


def _tensors():
    rng = np.random.default_rng(5)
    yield tb.IntTensor(np.zeros(0, np.int32), [0], tb.Scale.ZERO)
    yield tb.IntTensor(np.array([7], np.int32), [], tb.Scale(1, 0))  # ndim 0: one element
    yield tb.IntTensor(np.array([np.iinfo(np.int32).min, -1, 0, 1, np.iinfo(np.int32).max], np.int32), [5],
                       tb.Scale(2**62 + 12345, -17))
    for shape in ([64], [3, 17], [2, 3, 4], [1, 2048]):
        n = int(np.prod(shape))
        yield tb.IntTensor(rng.integers(-(2**28), 2**28, size=n, dtype=np.int32), shape,
                           tb.Scale(int(rng.integers(1, 2**31)), int(rng.integers(-40, 90))))


def test_frames_match_the_reference_layout(oracle):
    for t in _tensors():
        b = t.to_bytes()
        assert b == oracle.to_bytes(t.data, t.shape, t.scale.mant, t.scale.shift)
        assert len(b) == 4 + 8 * len(t.shape) + 8 + 4 + 8 + 4 * t.data.size
        # field by field, little-endian
        assert struct.unpack_from("<I", b, 0)[0] == len(t.shape)
        u = tb.IntTensor.from_bytes(b)
        assert u.shape == t.shape and u.scale == t.scale and (u.data == t.data).all()
        data, shape, scale, used = oracle.from_bytes(b)
        assert shape == list(t.shape) and scale == (t.scale.mant, t.scale.shift) and used == len(b)
        assert (data == t.data).all()


def test_concatenated_frames_read_one_after_another():
    ts = list(_tensors())
    blob = b"".join(t.to_bytes() for t in ts)
    off = 0
    for t in ts:
        u, n = tb.IntTensor.from_bytes(blob[off:], with_length=True)
        assert u.shape == t.shape and u.scale == t.scale and (u.data == t.data).all()
        off += n
    assert off == len(blob)


def test_short_or_malformed_buffers_fail_loudly():
    b = tb.IntTensor(np.arange(6, dtype=np.int32), [2, 3], tb.Scale(3, 4)).to_bytes()
    for cut in range(len(b)):  # every truncation (the reference panics on these)
        with pytest.raises(tb.KtmoeError) as e:
            tb.IntTensor.from_bytes(b[:cut])
        assert e.value.status == _native.ERR_ARG
    huge = struct.pack("<I", 2**31) + bytes(64)  # ndim beyond any buffer
    with pytest.raises(tb.KtmoeError):
        tb.IntTensor.from_bytes(huge)
    lying = bytearray(b)
    struct.pack_into("<Q", lying, 4 + 16 + 12, 10**12)  # ndata larger than the buffer
    with pytest.raises(tb.KtmoeError):
        tb.IntTensor.from_bytes(bytes(lying))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _send(dist, blob: bytes, dst: int):
    import torch

    dist.send(torch.tensor([len(blob)], dtype=torch.int64), dst)
    dist.send(torch.frombuffer(bytearray(blob), dtype=torch.uint8), dst)


def _recv(dist, src: int) -> bytes:
    import torch

    n = torch.zeros(1, dtype=torch.int64)
    dist.recv(n, src)
    buf = torch.zeros(int(n.item()), dtype=torch.uint8)
    dist.recv(buf, src)
    return buf.numpy().tobytes()


def _frames(blob: bytes):
    off, out = 0, []
    while off < len(blob):
        t, n = tb.IntTensor.from_bytes(blob[off:], with_length=True)
        out.append(t)
        off += n
    return out


def _seam_rank(rank, world, port, name, outdir):
    """Rank 0 routes each token and sends (the row, its expert ids) as two frames; rank 1 answers with one frame per
    expert output; rank 0 combines them through the oracle's seam. One request per row, in row order."""
    import torch.distributed as dist

    from oracle import oracle as O

    import cases

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    O.build()
    c = cases.CASES[name]
    o = cases.build_oracle(c, O)
    if rank == 0:
        x = tb.IntTensor.from_reals(cases.make_x(c))
        xs = (x.scale.mant, x.scale.shift)
        X = x.data.reshape(c.T, c.d)
        ex, ec, sumc = o.route(X, xs)
        ye = np.zeros((c.T, c.k, c.d), np.int32)
        yse = [(0, 0)] * (c.T * c.k)
        live = [t for t in range(c.T) if sumc[t] > 0]
        _send(dist, tb.IntTensor(np.array([len(live)], np.int32), [1], tb.Scale.ZERO).to_bytes(), 1)
        for t in live:
            ids = tb.IntTensor(np.asarray(ex[t], np.int32), [c.k], tb.Scale.ZERO)
            _send(dist, tb.IntTensor(X[t], [c.d], x.scale).to_bytes() + ids.to_bytes(), 1)
            outs = _frames(_recv(dist, 1))
            assert len(outs) == c.k
            for j, y in enumerate(outs):
                ye[t, j] = y.data
                yse[t * c.k + j] = (y.scale.mant, y.scale.shift)
        got, gs = o.forward_with_given_experts(X, xs, ye, yse)
        want, ws = o.forward(X, xs)
        np.savez(os.path.join(outdir, "seam.npz"), ok=bool(gs == ws and (got == want).all()))
    else:
        n = int(_frames(_recv(dist, 0))[0].data[0])
        for _ in range(n):
            row, ids = _frames(_recv(dist, 0))
            outs = [o.expert(int(e), row.data, (row.scale.mant, row.scale.shift)) for e in ids.data]
            _send(dist, b"".join(tb.IntTensor(y, [c.d], tb.Scale(*s)).to_bytes() for y, s in outs), 0)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("name", ["tiny_sigmoid_shared", "tiny_softmax_37rows"])
def test_seam_across_processes_in_wire_frames(tmp_path, name):
    import torch.multiprocessing as mp

    mp.spawn(_seam_rank, args=(2, _free_port(), name, str(tmp_path)), nprocs=2, join=True)
    assert bool(np.load(tmp_path / "seam.npz")["ok"])
