"""tritify_b200 — tritify's exact-integer Mixture-of-Experts layer on NVIDIA B200.

The host-side mirror of the reference's operator interfaces, over the C ABI of ``include/ktmoe.h``
(``libktmoe.so``). Names and argument meanings follow tritify (paths relative to the reference project root):

* :class:`Scale`, :class:`IntTensor`             — kt-int ``Scale`` (crates/00-kernels/kt-int/src/lib.rs:175-324),
  kt-core ``IntTensor`` (crates/01-engine/kt-core/src/tensor.rs:10-116)
* :class:`QuantLinear`, :class:`SwiGluMlp`,
  :class:`MoeMlp`, :class:`MoeRoute`               — crates/01-engine/kt-core/src/layers.rs:211-1106
* :class:`B200Linear`                             — a ``LinearBackend`` (crates/01-engine/kt-core/src/backend.rs:46-59)

Every integer a forward produces comes from the sm_100a kernels in libktmoe.so; the only host arithmetic is the
reference's own offline f64 preparation (weight and entry quantisers, code tables), done in C++ in the same library.
"""

from __future__ import annotations

import ctypes
import hashlib
import threading
from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence

import numpy as np

from . import _native
from ._native import KtmoeError, KtmoeLayerConfig, KtmoeScale, check, lib

__all__ = [
    "WLEVELS", "ACT_LEVELS", "ROUTER_CODE_BITS", "Scale", "IntTensor", "QuantLinear", "SwiGluMlp", "MoeMlp", "MoeRoute", "RouterScore",
    "B200Linear", "Context", "DeviceLayer", "LayerSlot", "MoeStack", "device_count", "synth_normal", "synth_normal_portable", "lcg_uniform", "table",
    "route_margins", "hash_int", "repro_hash",
    "KtmoeError",
    "ep_unique_id",
]

WLEVELS = 265720  # (3^12 - 1) / 2, layers.rs:16
ACT_LEVELS = 1 << 28  # layers.rs:18
ROUTER_CODE_BITS = 20  # layers.rs:659


def _p(a: np.ndarray, ct):
    return a.ctypes.data_as(ctypes.POINTER(ct))


@dataclass(frozen=True)
class Scale:
    """A non-negative fixed-point scale ``mant · 2^-shift`` (kt-int ``Scale``)."""

    mant: int
    shift: int

    ZERO = None  # set below

    def to_f64(self) -> float:
        return float(self.mant) * 2.0 ** (-self.shift)

    def _c(self) -> KtmoeScale:
        return KtmoeScale(int(self.mant), int(self.shift))

    @staticmethod
    def _of(s: KtmoeScale) -> "Scale":
        return Scale(int(s.mant), int(s.shift))


Scale.ZERO = Scale(0, 0)


class IntTensor:
    """An activation: int32 data, a shape and one :class:`Scale` (``real = data · scale``)."""

    def __init__(self, data: np.ndarray, shape: Sequence[int], scale: Scale):
        self.data = np.ascontiguousarray(data, dtype=np.int32).reshape(-1)
        self.shape = tuple(int(s) for s in shape)
        self.scale = scale

    def __len__(self) -> int:
        return int(self.data.size)

    @staticmethod
    def vector(data: np.ndarray, scale: Scale) -> "IntTensor":
        """IntTensor::vector (tensor.rs:22-25): a 1-D tensor."""
        d = np.ascontiguousarray(data, dtype=np.int32).reshape(-1)
        return IntTensor(d, (d.size,), scale)

    def is_empty(self) -> bool:
        return self.data.size == 0

    def max_abs_data(self) -> int:
        """IntTensor::max_abs_data (tensor.rs:46-49): the largest |data| (0 when empty)."""
        return int(np.abs(self.data.astype(np.int64)).max()) if self.data.size else 0

    def to_f32(self) -> np.ndarray:
        """IntTensor::to_f32 (tensor.rs:35-38): data · scale in f64, then rounded to f32."""
        return (self.data.astype(np.float64) * self.scale.to_f64()).astype(np.float32)

    @staticmethod
    def quantize_probe(x: np.ndarray, levels: int = ACT_LEVELS) -> "IntTensor":
        """IntTensor::quantize_probe (tensor.rs:119-123): from_reals of an f32 vector, 1-D."""
        return IntTensor.from_reals(np.ascontiguousarray(x, dtype=np.float32).reshape(-1), levels)

    @staticmethod
    def from_reals(values: np.ndarray, levels: int = ACT_LEVELS) -> "IntTensor":
        """IntTensor::from_reals (tensor.rs:106-116) at ACT_LEVELS, on f32 values."""
        if levels != ACT_LEVELS:
            raise ValueError("the entry quantiser here runs at ACT_LEVELS")
        v = np.ascontiguousarray(values, dtype=np.float32)
        data = np.empty(v.size, dtype=np.int32)
        s = KtmoeScale()
        check(lib().ktmoe_from_reals(_p(v, ctypes.c_float), v.size, _p(data, ctypes.c_int32), ctypes.byref(s)))
        return IntTensor(data, v.shape, Scale._of(s))

    def to_f64(self) -> np.ndarray:
        return self.data.astype(np.float64) * self.scale.to_f64()

    def to_bytes(self) -> bytes:
        """IntTensor::to_bytes (tensor.rs:51-67): the reference's interchange frame, byte for byte."""
        shape = np.ascontiguousarray(self.shape, dtype=np.int64)
        n = ctypes.c_uint64()
        check(lib().ktmoe_wire_size(shape.size, self.data.size, ctypes.byref(n)))
        out = np.empty(n.value, dtype=np.uint8)
        check(lib().ktmoe_wire_encode(_p(self.data, ctypes.c_int32), self.data.size, _p(shape, ctypes.c_int64),
                                      shape.size, self.scale._c(), _p(out, ctypes.c_uint8), out.size,
                                      ctypes.byref(n)))
        return out.tobytes()

    @staticmethod
    def from_bytes(b: bytes, with_length: bool = False):
        """IntTensor::from_bytes (tensor.rs:70-100) of the frame at the start of `b`; with_length also returns the
        frame's byte length (frames may be concatenated). A short or malformed buffer raises KtmoeError."""
        buf = np.frombuffer(b, dtype=np.uint8)
        ndim, ndata, used = ctypes.c_int32(), ctypes.c_int64(), ctypes.c_uint64()
        s = KtmoeScale()
        check(lib().ktmoe_wire_decode(_p(buf, ctypes.c_uint8), buf.size, ctypes.byref(ndim), None, 0, ctypes.byref(s),
                                      ctypes.byref(ndata), None, 0, ctypes.byref(used)))
        shape = np.empty(ndim.value, dtype=np.int64)
        data = np.empty(ndata.value, dtype=np.int32)
        check(lib().ktmoe_wire_decode(_p(buf, ctypes.c_uint8), buf.size, ctypes.byref(ndim), _p(shape, ctypes.c_int64),
                                      shape.size, ctypes.byref(s), ctypes.byref(ndata), _p(data, ctypes.c_int32),
                                      data.size, ctypes.byref(used)))
        t = IntTensor(data, shape.tolist(), Scale._of(s))
        return (t, used.value) if with_length else t


def hash_int(t: "IntTensor") -> str:
    """verify::hash_int (verify.rs:35-41): SHA-256 of the tensor's i32 data, little-endian (the scale is not hashed),
    as 64 hex digits: the reference's parity hash."""
    return hashlib.sha256(np.ascontiguousarray(t.data, dtype="<i4").tobytes()).hexdigest()


def repro_hash(t: "IntTensor") -> str:
    """The repro form of the hash (logits_hash, kt-convert/src/repro.rs:34-42), which also binds the scale: SHA-256
    of mant (i64 LE), shift (i32 LE) and the data (i32 LE)."""
    h = hashlib.sha256()
    h.update(np.int64(t.scale.mant).astype("<i8").tobytes())
    h.update(np.int32(t.scale.shift).astype("<i4").tobytes())
    h.update(np.ascontiguousarray(t.data, dtype="<i4").tobytes())
    return h.hexdigest()


def device_count() -> int:
    n = ctypes.c_int(0)
    check(lib().ktmoe_device_count(ctypes.byref(n)))
    return n.value


class Context:
    """One B200 device with its stream and resident-weight cache (kt-cuda's DeviceExec, device.rs:312-327)."""

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        check(lib().ktmoe_open(device, ctypes.byref(h)))
        self._h = h
        self.device = device
        self._lock = threading.Lock()

    @property
    def handle(self):
        return self._h

    def close(self) -> None:
        if self._h:
            lib().ktmoe_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, status: int) -> None:
        check(status, self._h)

    def stream(self) -> int:
        return int(lib().ktmoe_stream(self._h) or 0)

    def launch_count(self) -> int:
        n = ctypes.c_uint64()
        self.check(lib().ktmoe_launch_count(self._h, ctypes.byref(n)))
        return n.value

    def sync(self, stream: int = 0) -> None:
        self.check(lib().ktmoe_sync(self._h, ctypes.c_void_p(stream) if stream else None))

    def linear(self, x: np.ndarray, w: np.ndarray, rows: int, out: int, k: int,
               weight_id: Optional[int] = None) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.int32).reshape(-1)
        w = np.ascontiguousarray(w, dtype=np.int32).reshape(-1)
        if x.size != rows * k or w.size != out * k:
            raise ValueError("linear: x is not rows·k or w is not out·k")
        y = np.empty(rows * out, dtype=np.int64)
        if weight_id is None:
            st = lib().ktmoe_linear(self._h, _p(x, ctypes.c_int32), _p(w, ctypes.c_int32), rows, out, k,
                                    _p(y, ctypes.c_int64))
        else:
            st = lib().ktmoe_linear_weights(self._h, weight_id, _p(x, ctypes.c_int32), _p(w, ctypes.c_int32), rows,
                                            out, k, _p(y, ctypes.c_int64))
        self.check(st)
        return y

    def check_wait_expiry(self) -> int:
        """Failure detection without a fault (ktmoe_check_wait_expiry): the status a forward whose expert-parallel peer
        stopped returns (KTMOE_ERR_KERNEL after the ~2 s bounded wait)."""
        return int(lib().ktmoe_check_wait_expiry(self._h))

    def last_gemm(self) -> tuple:
        """(milliseconds, activation planes) of the last linear call's GEMM, timed with CUDA events on the context's
        stream; planes is 1 for the small-code kernel, 3 for the nine-plane one, 0 before any call."""
        ms, planes = ctypes.c_double(), ctypes.c_int32()
        self.check(lib().ktmoe_linear_last_gemm(self._h, ctypes.byref(ms), ctypes.byref(planes)))
        return ms.value, planes.value

    def set_weight_budget(self, nbytes: int) -> None:
        self.check(lib().ktmoe_set_weight_budget(self._h, nbytes))

    def resident_bytes(self) -> int:
        n = ctypes.c_uint64()
        self.check(lib().ktmoe_resident_bytes(self._h, ctypes.byref(n)))
        return n.value


_default_ctx: Optional[Context] = None
_default_lock = threading.Lock()


def default_context() -> Context:
    global _default_ctx
    with _default_lock:
        if _default_ctx is None:
            _default_ctx = Context(0)
        return _default_ctx


class B200Linear:
    """A tritify ``LinearBackend`` (backend.rs:46-59) on a B200: the exact i32×i32→i64 accumulate as digit-plane
    products on the tensor cores. ``linear_weights`` keeps weights resident by id (``WeightId``)."""

    def __init__(self, ctx: Optional[Context] = None):
        self.ctx = ctx or default_context()

    def name(self) -> str:
        return f"b200:{self.ctx.device}"

    def linear(self, x, w, rows: int, out: int, k: int) -> np.ndarray:
        return self.ctx.linear(x, w, rows, out, k)

    def linear_weights(self, x, weight_id: int, w, rows: int, out: int, k: int) -> np.ndarray:
        return self.ctx.linear(x, w, rows, out, k, weight_id=weight_id)


class QuantLinear:
    """QuantLinear (layers.rs:211-257): per-tensor b=12 weight codes and their scale, optional bias."""

    def __init__(self, name: str, codes: np.ndarray, w_scale: Scale, out_features: int, in_features: int,
                 bias: Optional[tuple] = None):
        self.name = name
        self.out_features, self.in_features = int(out_features), int(in_features)
        self.w_codes = np.ascontiguousarray(codes, dtype=np.int32).reshape(self.out_features, self.in_features)
        self.w_scale = w_scale
        self.bias = bias  # (codes int64 [out], Scale) or None

    @staticmethod
    def from_weights(name: str, w: np.ndarray, out_features: int, in_features: int) -> "QuantLinear":
        w = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
        if w.size != out_features * in_features:
            raise ValueError(f"{name}: weights are not out·in")
        codes = np.empty(w.size, dtype=np.int32)
        s = KtmoeScale()
        check(lib().ktmoe_quantize_weights(_p(w, ctypes.c_float), w.size, _p(codes, ctypes.c_int32), ctypes.byref(s)))
        return QuantLinear(name, codes, Scale._of(s), out_features, in_features)

    def with_bias(self, bias: Optional[np.ndarray]) -> "QuantLinear":
        if bias is None:
            return self
        b = np.ascontiguousarray(bias, dtype=np.float32).reshape(-1)
        if b.size != self.out_features:
            raise ValueError(f"{self.name}: bias len mismatch")
        codes = np.empty(b.size, dtype=np.int64)
        s = KtmoeScale()
        has = ctypes.c_int32()
        check(lib().ktmoe_quantize_bias(_p(b, ctypes.c_float), b.size, _p(codes, ctypes.c_int64), ctypes.byref(s),
                                        ctypes.byref(has)))
        if has.value:
            self.bias = (codes, Scale._of(s))
        return self


class SwiGluMlp:
    """SwiGluMlp (layers.rs:581-640): down(SiLU(gate(x)) ⊙ up(x)) with an integer-code SiLU table."""

    def __init__(self, name: str, gate: QuantLinear, up: QuantLinear, down: QuantLinear):
        if gate.out_features != up.out_features:
            raise ValueError("gate/up hidden mismatch")
        if down.in_features != gate.out_features:
            raise ValueError("down input != hidden")
        self.name, self.gate, self.up, self.down = name, gate, up, down


@dataclass
class MoeRoute:
    """MoeRoute (layers.rs:812-821): the selected experts in top-k order, their codes, the normaliser and the
    boundary margin (the strongest excluded expert's exp code over the weakest selected one's, in (0, 1]; 0 for a
    sigmoid router or a zero weakest code): a read-only diagnostic of how decisive the cut is."""

    experts: List[int]
    ec: List[int]
    sumc: int
    margin: float = 0.0


@dataclass
class RouterScore:
    """RouterScore (router.rs:21-26, the router's score function): ``kind`` "softmax" or "sigmoid"; a sigmoid router
    carries its selection bias coded as round(b·2^20) (SigmoidScore::new, router.rs:37-51)."""

    kind: str
    bias_codes: Optional[np.ndarray]


def route_margins(logits: np.ndarray, scales: Sequence["Scale"], experts: np.ndarray) -> np.ndarray:
    """MoeRoute::margin of softmax routes (ktmoe_route_margins, on the host): router logits [rows][E] with their
    per-row scales and the routes' experts [rows][k] -> margins [rows]."""
    lg = np.ascontiguousarray(logits, dtype=np.int32)
    ex = np.ascontiguousarray(experts, dtype=np.int32)
    rows, n_experts = lg.shape
    if ex.shape[0] != rows or len(scales) != rows:
        raise ValueError("route_margins: one scale and one route per row of logits")
    sc = (KtmoeScale * max(rows, 1))(*[s._c() for s in scales])
    out = np.zeros(rows, dtype=np.float64)
    check(lib().ktmoe_route_margins(_p(lg, ctypes.c_int32), rows, n_experts, sc, _p(ex, ctypes.c_int32),
                                    ex.shape[1], _p(out, ctypes.c_double)))
    return out


class DeviceLayer:
    """One MoE layer resident on a device (ktmoe_layer): weights as digit planes, scratch for the forward."""

    def __init__(self, ctx: Context, d_model: int, n_experts: int, d_ff: int, top_k: int, norm_topk_prob: bool,
                 sigmoid: bool, shared_d_ff: int, ep: Optional[tuple] = None):
        """``ep = (rank, world, nccl_id_bytes)`` makes this rank's part of an expert-parallel layer."""
        self.ctx = ctx
        cfg = KtmoeLayerConfig(d_model, n_experts, d_ff, top_k, 1 if norm_topk_prob else 0, 1 if sigmoid else 0,
                               shared_d_ff)
        h = ctypes.c_void_p()
        if ep is None:
            ctx.check(lib().ktmoe_layer_create(ctx.handle, ctypes.byref(cfg), ctypes.byref(h)))
        else:
            rank, world, nid = ep
            buf = ctypes.create_string_buffer(bytes(nid), len(nid))
            ctx.check(lib().ktmoe_layer_create_ep(ctx.handle, ctypes.byref(cfg), rank, world, buf, ctypes.byref(h)))
        self._h = h
        self.d_model, self.n_experts, self.d_ff, self.top_k, self.shared_d_ff = d_model, n_experts, d_ff, top_k, shared_d_ff
        b, e = ctypes.c_int32(), ctypes.c_int32()
        ctx.check(lib().ktmoe_layer_experts(self._h, ctypes.byref(b), ctypes.byref(e)))
        self.experts = range(b.value, e.value)

    def __del__(self):
        try:
            if self._h:
                lib().ktmoe_layer_destroy(self._h)
                self._h = None
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def set_router(self, codes: np.ndarray, w_scale: Scale, bias: Optional[tuple] = None) -> None:
        codes = np.ascontiguousarray(codes, dtype=np.int32)
        if bias is not None:
            bc = np.ascontiguousarray(bias[0], dtype=np.int64)
            self.ctx.check(lib().ktmoe_layer_set_router(self._h, _p(codes, ctypes.c_int32), w_scale._c(),
                                                        _p(bc, ctypes.c_int64), bias[1]._c()))
        else:
            self.ctx.check(lib().ktmoe_layer_set_router(self._h, _p(codes, ctypes.c_int32), w_scale._c(), None,
                                                        KtmoeScale(0, 0)))

    def set_sigmoid_bias(self, codes: np.ndarray) -> None:
        codes = np.ascontiguousarray(codes, dtype=np.int64)
        self.ctx.check(lib().ktmoe_layer_set_sigmoid_bias(self._h, _p(codes, ctypes.c_int64)))

    def set_expert(self, e: int, gate: tuple, up: tuple, down: tuple) -> None:
        g, u, d = (np.ascontiguousarray(t[0], dtype=np.int32) for t in (gate, up, down))
        self.ctx.check(lib().ktmoe_layer_set_expert(self._h, e, _p(g, ctypes.c_int32), gate[1]._c(),
                                                    _p(u, ctypes.c_int32), up[1]._c(), _p(d, ctypes.c_int32),
                                                    down[1]._c()))

    def set_shared(self, gate: tuple, up: tuple, down: tuple) -> None:
        g, u, d = (np.ascontiguousarray(t[0], dtype=np.int32) for t in (gate, up, down))
        self.ctx.check(lib().ktmoe_layer_set_shared(self._h, _p(g, ctypes.c_int32), gate[1]._c(),
                                                    _p(u, ctypes.c_int32), up[1]._c(), _p(d, ctypes.c_int32),
                                                    down[1]._c()))

    def set_shared_gate(self, gate: Optional[tuple]) -> None:
        """Extension: gate the shared expert with a sigmoid of a [1, d_model] linear's integer logit (Qwen2-MoE's
        shared_expert_gate); ``gate = (codes [d_model], Scale)`` or None to turn it off."""
        if gate is None:
            self.ctx.check(lib().ktmoe_layer_set_shared_gate(self._h, None, KtmoeScale(0, 0)))
            return
        c = np.ascontiguousarray(gate[0], dtype=np.int32).reshape(-1)
        if c.size != self.d_model:
            raise ValueError("the shared-expert gate has d_model codes")
        self.ctx.check(lib().ktmoe_layer_set_shared_gate(self._h, _p(c, ctypes.c_int32), gate[1]._c()))

    def set_depth(self, n_layers: int) -> None:
        """Hold ``n_layers`` weight slots (a stack of layers of this shape sharing one scratch and exchange)."""
        self.ctx.check(lib().ktmoe_layer_set_depth(self._h, int(n_layers)))

    def select(self, slot: int) -> None:
        """Make weight slot ``slot`` the one the setters write and the forwards read."""
        self.ctx.check(lib().ktmoe_layer_select(self._h, int(slot)))

    def slot(self, i: int) -> "LayerSlot":
        """Layer ``i`` of this stack of slots, for :class:`MoeStack`."""
        return LayerSlot(self, i)

    def synth_weights(self, seed: int, sigma: float = 0.02, sigmoid_bias_sigma: float = 0.02,
                      shared_gate: bool = False) -> None:
        """Generate and quantise the selected slot's weights on the GPU from the portable stream ``seed`` (router,
        experts, shared expert, optional shared-expert gate; a sigmoid router's bias from ``seed + 2``)."""
        self.ctx.check(lib().ktmoe_layer_synth_weights(self._h, int(seed), float(sigma), float(sigmoid_bias_sigma),
                                                       1 if shared_gate else 0))

    def set_norm(self, w_codes: np.ndarray, w_scale: Scale, eps_scale: Scale) -> None:
        """The block's FFN input RmsNorm (RmsNorm::new codes and scales) for block_forward."""
        w = np.ascontiguousarray(w_codes, dtype=np.int32)
        self.ctx.check(lib().ktmoe_layer_set_norm(self._h, _p(w, ctypes.c_int32), w_scale._c(), eps_scale._c()))

    def block_forward(self, x: np.ndarray, rows: int, x_scale: Scale):
        """x + moe(rms_norm(x)) (kt-core model.rs:175-181), host buffers: returns (y int32 [rows·d], Scale)."""
        return self.forward(x, rows, x_scale, block=True)

    def forward(self, x: np.ndarray, rows: int, x_scale: Scale, block: bool = False):
        """Host buffers in and out (synchronous): returns (y int32 [rows·d], Scale)."""
        fn = lib().ktmoe_block_forward if block else lib().ktmoe_forward
        x = np.ascontiguousarray(x, dtype=np.int32).reshape(-1)
        if x.size == 0:
            x = np.zeros(1, np.int32)
            y = np.zeros(1, np.int32)
            ys = KtmoeScale()
            self.ctx.check(fn(self._h, _p(x, ctypes.c_int32), 0, x_scale._c(), _p(y, ctypes.c_int32), ctypes.byref(ys)))
            return np.zeros(0, np.int32), Scale._of(ys)
        if x.size != rows * self.d_model:
            raise ValueError("x is not rows·d_model")
        y = np.empty(rows * self.d_model, dtype=np.int32)
        ys = KtmoeScale()
        self.ctx.check(fn(self._h, _p(x, ctypes.c_int32), rows, x_scale._c(), _p(y, ctypes.c_int32),
                                           ctypes.byref(ys)))
        return y, Scale._of(ys)

    def forward_async(self, x_ptr: int, rows: int, x_scale: Scale, y_ptr: int, y_scale: "KtmoeScale") -> None:
        """ktmoe_forward_async on host buffers given as raw pointers (pinned memory for the copies to overlap): returns
        at once; ``y`` and ``y_scale`` hold the result after ``forward_async_wait``."""
        self.ctx.check(lib().ktmoe_forward_async(self._h, ctypes.cast(x_ptr, ctypes.POINTER(ctypes.c_int32)), rows,
                                                 x_scale._c(), ctypes.cast(y_ptr, ctypes.POINTER(ctypes.c_int32)),
                                                 ctypes.byref(y_scale)))

    def forward_async_wait(self) -> None:
        self.ctx.check(lib().ktmoe_forward_async_wait(self._h))

    def set_graphs(self, enable: bool) -> None:
        """Capture the forward in CUDA graphs (per buffers, rows and stream) and replay them."""
        self.ctx.check(lib().ktmoe_layer_set_graphs(self._h, 1 if enable else 0))

    def set_ep_capacity(self, max_tokens_per_rank: int) -> None:
        """Expert-parallel layers: exchange over peer memory (NVLink, CUDA IPC) for forwards of at most this many rows
        per rank; all ranks call it together with the same value (0: back to NCCL)."""
        self.ctx.check(lib().ktmoe_layer_set_ep_capacity(self._h, int(max_tokens_per_rank)))

    def forward_dev(self, x_ptr: int, rows: int, x_scale_ptr: int, y_ptr: int, y_scale_ptr: int, stream: int = 0) -> None:
        """Device buffers (raw pointers), stream-ordered, not synchronised."""
        self.ctx.check(lib().ktmoe_forward_dev(self._h, ctypes.c_void_p(x_ptr), rows, ctypes.c_void_p(x_scale_ptr),
                                               ctypes.c_void_p(y_ptr), ctypes.c_void_p(y_scale_ptr),
                                               ctypes.c_void_p(stream) if stream else None))

    def block_forward_dev(self, x_ptr: int, rows: int, x_scale_ptr: int, y_ptr: int, y_scale_ptr: int,
                          stream: int = 0) -> None:
        """The block x + moe(rms_norm(x)) on device buffers (raw pointers), stream-ordered, not synchronised."""
        self.ctx.check(lib().ktmoe_block_forward_dev(self._h, ctypes.c_void_p(x_ptr), rows,
                                                     ctypes.c_void_p(x_scale_ptr), ctypes.c_void_p(y_ptr),
                                                     ctypes.c_void_p(y_scale_ptr),
                                                     ctypes.c_void_p(stream) if stream else None))

    def route(self, x: np.ndarray, rows: int, x_scale: Scale):
        x = np.ascontiguousarray(x, dtype=np.int32).reshape(-1)
        ex = np.empty(rows * self.top_k, dtype=np.int32)
        ec = np.empty(rows * self.top_k, dtype=np.int64)
        sumc = np.empty(rows, dtype=np.int64)
        self.ctx.check(lib().ktmoe_route(self._h, _p(x, ctypes.c_int32), rows, x_scale._c(), _p(ex, ctypes.c_int32),
                                         _p(ec, ctypes.c_int64), _p(sumc, ctypes.c_int64)))
        return ex.reshape(rows, self.top_k), ec.reshape(rows, self.top_k), sumc

    def expert_forward(self, x: np.ndarray, rows: int, x_scale: Scale, ids: np.ndarray):
        """The seam's worker side (ktmoe_layer_expert_forward): SwiGluMlp::forward_int of expert ids[r][j] on row r
        (ids < 0: empty). Returns (y int32 [rows][n_ids][d], scales [rows][n_ids] as a list of lists of Scale)."""
        x = np.ascontiguousarray(x, dtype=np.int32).reshape(-1)
        ids = np.ascontiguousarray(ids, dtype=np.int32).reshape(rows, -1)
        n_ids = ids.shape[1]
        if x.size != rows * self.d_model:
            raise ValueError("x is not rows·d_model")
        y = np.empty(rows * n_ids * self.d_model, dtype=np.int32)
        ys = (KtmoeScale * max(1, rows * n_ids))()
        self.ctx.check(lib().ktmoe_layer_expert_forward(self._h, _p(x, ctypes.c_int32), rows, x_scale._c(),
                                                        _p(ids, ctypes.c_int32), n_ids, _p(y, ctypes.c_int32), ys))
        sc = [Scale._of(ys[i]) for i in range(rows * n_ids)]
        return y.reshape(rows, n_ids, self.d_model), [sc[r * n_ids:(r + 1) * n_ids] for r in range(rows)]

    def forward_with_experts(self, x: np.ndarray, rows: int, x_scale: Scale, experts_fn: Callable):
        """MoeMlp::forward_int_with_experts (layers.rs:945-984) on the device: route here, call
        ``experts_fn(ids [rows][top_k] int32, x [rows][d] int32, x_scale) -> (y [rows][top_k][d], scales)`` once for
        all rows (rows with an empty route have ids -1; scales: [rows][top_k] of Scale or (mant, shift)), then combine,
        merge and add the shared expert. Returns (y int32 [rows·d], Scale)."""
        x = np.ascontiguousarray(x, dtype=np.int32).reshape(-1)
        if x.size != rows * self.d_model:
            raise ValueError("x is not rows·d_model")
        d = self.d_model
        failure = []

        def tramp(_user, n, k, ids_p, x_p, xs_c, y_p, ys_p):
            try:
                ids = np.ctypeslib.as_array(ids_p, shape=(n, k)).copy()
                xr = np.ctypeslib.as_array(x_p, shape=(n, d)).copy()
                ye, yse = experts_fn(ids, xr, Scale._of(xs_c))
                ye = np.ascontiguousarray(ye, dtype=np.int32).reshape(n, k, d)
                np.ctypeslib.as_array(y_p, shape=(n * k * d,))[:] = ye.reshape(-1)
                for r in range(n):
                    for j in range(k):
                        s = yse[r][j]
                        m, sh = (s.mant, s.shift) if isinstance(s, Scale) else (int(s[0]), int(s[1]))
                        ys_p[r * k + j] = KtmoeScale(m, sh)
                return 0
            except Exception as e:  # reported through KTMOE_ERR_CALLBACK; re-raised below
                failure.append(e)
                return 1

        cb = _native.EXPERTS_FN(tramp)
        y = np.empty(rows * d, dtype=np.int32)
        ys = KtmoeScale()
        status = lib().ktmoe_layer_forward_with_experts(self._h, _p(x, ctypes.c_int32), rows, x_scale._c(), cb, None,
                                                        _p(y, ctypes.c_int32), ctypes.byref(ys))
        if failure:
            raise failure[0]
        self.ctx.check(status)
        return y, Scale._of(ys)

    STAGES = ["route", "dispatch", "exchange_in", "gemm_gate_up", "swiglu", "gemm_down", "exchange_out", "combine",
              "merge", "shared"]

    def set_timing(self, enable: bool) -> None:
        self.ctx.check(lib().ktmoe_layer_set_timing(self._h, 1 if enable else 0))

    def stage_times(self):
        """(per-stage milliseconds summed over the timed forwards, number of timed forwards)."""
        ms = (ctypes.c_double * len(self.STAGES))()
        n = ctypes.c_int32()
        self.ctx.check(lib().ktmoe_layer_stage_times(self._h, ms, len(self.STAGES), ctypes.byref(n)))
        return dict(zip(self.STAGES, list(ms))), n.value

    def debug_fetch(self, which: int, rows: int):
        """Internal buffers of the last forward (router logits / their scales / per-token outputs / their scales)."""
        if which in (0, 2):
            n = rows * (self.n_experts if which == 0 else self.d_model)
            buf = np.empty(n, dtype=np.int32)
            self.ctx.check(lib().ktmoe_layer_debug_fetch(self._h, which, buf.ctypes.data_as(ctypes.c_void_p),
                                                         buf.nbytes))
            return buf.reshape(rows, -1)
        buf = (KtmoeScale * rows)()
        self.ctx.check(lib().ktmoe_layer_debug_fetch(self._h, which, ctypes.cast(buf, ctypes.c_void_p),
                                                     ctypes.sizeof(buf)))
        return [Scale._of(s) for s in buf]


class MoeMlp:
    """MoeMlp (layers.rs:661-1106), its forward on a B200.

    Built like the reference's: ``MoeMlp(name, router, experts, top_k)`` then ``with_norm_topk_prob``,
    ``with_sigmoid_router`` and ``with_shared_expert``. The weights move to the device on the first forward.
    """

    def __init__(self, name: str, router: QuantLinear, experts: List[SwiGluMlp], top_k: int,
                 ctx: Optional[Context] = None):
        if not (1 <= top_k <= len(experts)):
            raise ValueError("top_k in 1..=E")
        if router.out_features != len(experts):
            raise ValueError("router out_features != number of experts")
        self._init(name, router, experts, top_k, ctx)

    @staticmethod
    def remote(name: str, router: QuantLinear, top_k: int, ctx: Optional[Context] = None) -> "MoeMlp":
        """MoeMlp::remote (layers.rs:694-712): the routed experts are elsewhere; route, combine and the shared expert
        run here, and the experts come only through :meth:`forward_int_with_experts`."""
        if not (1 <= top_k <= router.out_features):
            raise ValueError("top_k in 1..=E")
        m = MoeMlp.__new__(MoeMlp)
        m._init(name, router, [], top_k, ctx)
        return m

    def _init(self, name, router, experts, top_k, ctx):
        self.name, self.router, self.experts, self.top_k = name, router, experts, top_k
        self.norm_topk_prob = False
        self.sigmoid_bias_codes: Optional[np.ndarray] = None
        self.shared: Optional[SwiGluMlp] = None
        self.shared_gate: Optional[QuantLinear] = None
        self._ctx = ctx
        self._dev: Optional[DeviceLayer] = None

    def with_norm_topk_prob(self, v: bool) -> "MoeMlp":
        self.norm_topk_prob = bool(v)
        self._dev = None
        return self

    def with_sigmoid_router(self, bias: np.ndarray) -> "MoeMlp":
        b = np.ascontiguousarray(bias, dtype=np.float32).reshape(-1)
        if b.size != self.n_experts():
            raise ValueError(f"{self.name}: one selection bias per expert")
        codes = np.empty(b.size, dtype=np.int64)
        check(lib().ktmoe_code_sigmoid_bias(_p(b, ctypes.c_float), b.size, _p(codes, ctypes.c_int64)))
        self.sigmoid_bias_codes = codes
        self._dev = None
        return self

    def with_shared_expert(self, shared: SwiGluMlp) -> "MoeMlp":
        self.shared = shared
        self._dev = None
        return self

    @property
    def dim(self) -> int:
        return self.router.in_features

    def with_shared_expert_gate(self, gate: "QuantLinear") -> "MoeMlp":
        """Extension (the reference refuses it, kt-model-moe/src/lib.rs:152-154): Qwen2-MoE's sigmoid-gated shared
        expert. ``gate`` is shared_expert_gate as a QuantLinear [1, dim]; each token's shared output is scaled by the
        sigmoid code of the gate's integer logit and requantised before the add."""
        if self.shared is None:
            raise ValueError("with_shared_expert_gate needs a shared expert")
        if gate.out_features != 1 or gate.in_features != self.dim:
            raise ValueError("the shared-expert gate is a [1, dim] linear")
        self.shared_gate = gate
        self._dev = None
        return self

    def n_experts(self) -> int:
        return self.router.out_features

    def is_remote(self) -> bool:
        return not self.experts

    def router_score(self) -> "RouterScore":
        """MoeMlp::router_score (layers.rs:747-750): softmax, or sigmoid with the coded selection bias."""
        if self.sigmoid_bias_codes is None:
            return RouterScore("softmax", None)
        return RouterScore("sigmoid", self.sigmoid_bias_codes.copy())

    def shared_expert(self) -> Optional[SwiGluMlp]:
        """MoeMlp::shared_expert (layers.rs:752-755)."""
        return self.shared

    def router_codes(self) -> np.ndarray:
        """MoeMlp::router_codes (layers.rs:784-788): the router's softmax code table (read-only); every routing code
        is one of its entries or 0."""
        codes = table(0)[0]
        codes.setflags(write=False)
        return codes

    def device_layer(self) -> DeviceLayer:
        if self._dev is None:
            ctx = self._ctx or default_context()
            # a remote layer holds no routed experts: the smallest expert width keeps their (unused) planes small
            d_ff = self.experts[0].gate.out_features if self.experts else 16
            dev = DeviceLayer(ctx, self.dim, self.n_experts(), d_ff, self.top_k, self.norm_topk_prob,
                              self.sigmoid_bias_codes is not None,
                              self.shared.gate.out_features if self.shared else 0)
            dev.set_router(self.router.w_codes, self.router.w_scale, self.router.bias)
            if self.sigmoid_bias_codes is not None:
                dev.set_sigmoid_bias(self.sigmoid_bias_codes)
            for e, m in enumerate(self.experts):
                dev.set_expert(e, (m.gate.w_codes, m.gate.w_scale), (m.up.w_codes, m.up.w_scale),
                               (m.down.w_codes, m.down.w_scale))
            if self.shared is not None:
                s = self.shared
                dev.set_shared((s.gate.w_codes, s.gate.w_scale), (s.up.w_codes, s.up.w_scale),
                               (s.down.w_codes, s.down.w_scale))
                if self.shared_gate is not None:
                    dev.set_shared_gate((self.shared_gate.w_codes, self.shared_gate.w_scale))
            self._dev = dev
        return self._dev

    def forward_int_with_experts(self, x: IntTensor, experts_fn: Callable) -> IntTensor:
        """MoeMlp::forward_int_with_experts (layers.rs:945-951): route and combine here, the experts through
        ``experts_fn(ids: list[int], row: IntTensor) -> list[IntTensor]`` (outputs in ids order), called for each row
        whose route is not empty, in row order, as the reference does."""
        d = self.dim
        if len(x) % d != 0:
            raise ValueError(f"{self.name}: MoE input length must be a multiple of dim")
        rows = len(x) // d

        def batch(ids, xr, xs):
            n, k = ids.shape
            y = np.zeros((n, k, d), dtype=np.int32)
            ys = [[Scale.ZERO] * k for _ in range(n)]
            for r in range(n):
                if ids[r, 0] < 0:
                    continue
                outs = experts_fn([int(e) for e in ids[r]], IntTensor(xr[r], (d,), xs))
                if len(outs) != k:
                    raise ValueError(f"{self.name}: the experts callback returned {len(outs)} outputs for {k} ids")
                for j, o in enumerate(outs):
                    y[r, j] = np.asarray(o.data, dtype=np.int32).reshape(d)
                    ys[r][j] = o.scale
            return y, ys

        y, ys = self.device_layer().forward_with_experts(x.data, rows, x.scale, batch)
        return IntTensor(y, (d,) if rows == 1 else (rows, d), ys)

    def expert_outputs(self, x: IntTensor, ids: np.ndarray) -> List[List[IntTensor]]:
        """The worker side of the seam: ``SwiGluMlp::forward_int`` (layers.rs:609-640) of expert ``ids[r][j]`` on row
        r of ``x`` (ids < 0: empty, a zero output), all rows at ``x.scale``; on the device in one batch."""
        d = self.dim
        rows = len(x) // d
        y, ys = self.device_layer().expert_forward(x.data, rows, x.scale, ids)
        return [[IntTensor(y[r, j], (d,), ys[r][j]) for j in range(y.shape[1])] for r in range(rows)]

    def forward_int(self, x: IntTensor) -> IntTensor:
        """Module::forward_int (layers.rs:1070-1073)."""
        if self.is_remote():
            raise RuntimeError(f"{self.name}: the routed experts are remote (MoeMlp::remote); compute them through "
                               "forward_int_with_experts")
        d = self.dim
        if len(x) % d != 0:
            raise ValueError(f"{self.name}: MoE input length must be a multiple of dim")
        rows = len(x) // d
        y, ys = self.device_layer().forward(x.data, rows, x.scale)
        shape = (d,) if rows == 1 else (rows, d)
        return IntTensor(y, shape, ys)

    def route(self, x: IntTensor) -> List[MoeRoute]:
        """MoeMlp::route (layers.rs:826-862) for each row of ``x``; a softmax route's margin comes from the route's
        router logits (fetched from the device) on the host."""
        rows = len(x) // self.dim
        dev = self.device_layer()
        ex, ec, sumc = dev.route(x.data, rows, x.scale)
        margins = np.zeros(rows)
        if self.sigmoid_bias_codes is None and rows > 0:
            margins = route_margins(dev.debug_fetch(0, rows), dev.debug_fetch(1, rows), ex)
        return [MoeRoute([int(v) for v in ex[t]], [int(v) for v in ec[t]], int(sumc[t]), float(margins[t]))
                for t in range(rows)]

    def route_trace(self, x: IntTensor) -> List[List[int]]:
        """Module::route_trace (layers.rs:1089-1100)."""
        return [r.experts for r in self.route(x)]


class LayerSlot:
    """Layer ``slot`` of a DeviceLayer that holds a stack of weight slots (``DeviceLayer.set_depth``): its forwards
    select the slot, then run on the shared layer (a host-side swap: the launches read the slot's weights)."""

    def __init__(self, dev: "DeviceLayer", slot: int):
        self.dev, self.slot = dev, int(slot)
        self.ctx, self.d_model = dev.ctx, dev.d_model

    def block_forward_dev(self, x_ptr: int, rows: int, x_scale_ptr: int, y_ptr: int, y_scale_ptr: int,
                          stream: int = 0) -> None:
        self.dev.select(self.slot)
        self.dev.block_forward_dev(x_ptr, rows, x_scale_ptr, y_ptr, y_scale_ptr, stream)

    def forward_dev(self, x_ptr: int, rows: int, x_scale_ptr: int, y_ptr: int, y_scale_ptr: int, stream: int = 0) -> None:
        self.dev.select(self.slot)
        self.dev.forward_dev(x_ptr, rows, x_scale_ptr, y_ptr, y_scale_ptr, stream)


class MoeStack:
    """A stack of MoE decoder-block FFN halves with attention excluded (the shape of a GLM-4.5-Air-style model's 45
    MoE layers): for each layer l, x ← add(x, moe_l(rms_norm_l(x))) (kt-core model.rs:175-181), the residual stream
    staying on the device between layers in two ping-pong buffers. Every layer is a :class:`DeviceLayer` with its norm
    set (``set_norm``), all on one context; each layer's block is one ``ktmoe_block_forward_dev`` on that context's
    stream (with the layer's CUDA graphs when enabled: the buffers a layer sees are the same on every call)."""

    def __init__(self, layers: Sequence):
        """``layers``: DeviceLayers, or the LayerSlots of one DeviceLayer with several weight slots."""
        if not layers:
            raise ValueError("a stack needs at least one layer")
        self.layers = list(layers)
        self.ctx = self.layers[0].ctx
        self.d_model = self.layers[0].d_model
        if any(L.ctx is not self.ctx or L.d_model != self.d_model for L in self.layers):
            raise ValueError("the layers of a stack share one context and one d_model")
        self._bufs = None

    def _buffers(self, rows: int):
        """Four int32 [rows·d] buffers and their scales: the input, two ping-pong, the output. Kept across calls, so a
        layer sees the same pointers every time (its CUDA graphs are reused)."""
        import torch  # device memory for the residual stream (plumbing only)

        if self._bufs is None or self._bufs[0] < rows:
            dev = torch.device("cuda", self.ctx.device)
            n = max(1, rows) * self.d_model
            self._bufs = (rows, [torch.empty(n, dtype=torch.int32, device=dev) for _ in range(4)],
                          [torch.zeros(2, dtype=torch.int64, device=dev) for _ in range(4)])
        return self._bufs

    def forward_dev(self, x_ptr: int, rows: int, x_scale_ptr: int, y_ptr: int, y_scale_ptr: int) -> None:
        """Device buffers (raw pointers; a Scale is 16 bytes {i64 mant, i32 shift}); ordered on the context's stream,
        not synchronised."""
        _, xb, sb = self._buffers(rows)
        src, src_s = x_ptr, x_scale_ptr
        for i, L in enumerate(self.layers):
            last = i == len(self.layers) - 1
            dst = y_ptr if last else xb[1 + i % 2].data_ptr()
            dst_s = y_scale_ptr if last else sb[1 + i % 2].data_ptr()
            L.block_forward_dev(src, rows, src_s, dst, dst_s)
            src, src_s = dst, dst_s

    def forward(self, x: IntTensor) -> IntTensor:
        """Host tensors in and out (synchronous)."""
        import torch

        d = self.d_model
        if len(x) % d != 0:
            raise ValueError("stack input length must be a multiple of d_model")
        rows = len(x) // d
        _, xb, sb = self._buffers(rows)
        n = rows * d
        xb[0][:n].copy_(torch.from_numpy(np.ascontiguousarray(x.data, dtype=np.int32)))
        sb[0].copy_(torch.tensor([x.scale.mant, x.scale.shift & 0xFFFFFFFF], dtype=torch.int64))
        torch.cuda.synchronize(xb[0].device)  # the uploads ran on torch's stream; the layers run on the context's
        self.forward_dev(xb[0].data_ptr(), rows, sb[0].data_ptr(), xb[3].data_ptr(), sb[3].data_ptr())
        self.ctx.sync()
        y = xb[3][:n].cpu().numpy().copy()
        s = sb[3].cpu().numpy()
        shift = int(s[1]) & 0xFFFFFFFF
        shift = shift - (1 << 32) if shift >= 1 << 31 else shift
        return IntTensor(y, (d,) if rows == 1 else (rows, d), Scale(int(s[0]), shift))


def scale_from_f64(x: float) -> Scale:
    """Scale::from_f64 (kt-int lib.rs:215-222)."""
    s = KtmoeScale()
    check(lib().ktmoe_scale_from_f64(float(x), ctypes.byref(s)))
    return Scale._of(s)


def ep_unique_id() -> bytes:
    """A new NCCL unique id (128 bytes) for an expert-parallel layer; one rank makes it, all ranks use it."""
    buf = ctypes.create_string_buffer(128)
    check(lib().ktmoe_ep_unique_id(buf, 128))
    return buf.raw


def synth_normal(seed: int, sigma: float, n: int, offset: int = 0) -> np.ndarray:
    """Elements [offset, offset + n) of the build-defined N(0, sigma) stream ``seed`` (splitmix64 + Box-Muller in f64,
    cast to f32)."""
    out = np.empty(n, dtype=np.float32)
    check(lib().ktmoe_synth_normal(seed, sigma, offset, n, _p(out, ctypes.c_float)))
    return out


def synth_normal_portable(seed: int, sigma: float, n: int, offset: int = 0) -> np.ndarray:
    """Elements [offset, offset + n) of the portable N(0, sigma) stream (ktmoe_synth_normal_portable): the stream
    ``DeviceLayer.synth_weights`` draws on the GPU, here on the host with identical bits."""
    out = np.empty(n, dtype=np.float32)
    check(lib().ktmoe_synth_normal_portable(seed, sigma, offset, n, _p(out, ctypes.c_float)))
    return out


def lcg_uniform(seed: int, lo: int, hi: int, n: int) -> np.ndarray:
    """Uniform integers in [lo, hi] from the reference's test LCG."""
    out = np.empty(n, dtype=np.int32)
    check(lib().ktmoe_lcg_uniform(seed, lo, hi, n, _p(out, ctypes.c_int32)))
    return out


def table(kind: int):
    """Code table kind 0 (router exp), 1 (SiLU), 2 (sigmoid): (codes, inv_step, lo_index, code_scale)."""
    codes = np.empty(1 << 16, dtype=np.int64)
    a, b = KtmoeScale(), KtmoeScale()
    lo = ctypes.c_int64()
    check(lib().ktmoe_table(kind, _p(codes, ctypes.c_int64), ctypes.byref(a), ctypes.byref(lo), ctypes.byref(b)))
    return codes, Scale._of(a), lo.value, Scale._of(b)
