"""TEST INFRASTRUCTURE ONLY — ctypes access to the CPU oracle (oracle/oracle.cpp).

The oracle restates tritify's CPU integer path (the reference's Rust crates kt-int, kt-core layers/router/backend)
so the GPU path can be checked against it bit for bit. Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU
legs import this module; the product package ``tritify_b200`` never does.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")


class KoScale(ctypes.Structure):
    _fields_ = [("mant", ctypes.c_int64), ("shift", ctypes.c_int32)]

    def tup(self):
        return (int(self.mant), int(self.shift))


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (g++ only)."""
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
        os.path.join(HERE, "oracle.cpp")
    ):
        subprocess.run(["make", "-s", "-C", HERE] + (["-B"] if force else []), check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        p = ctypes.POINTER
        i32p, i64p, f32p = p(ctypes.c_int32), p(ctypes.c_int64), p(ctypes.c_float)
        sz = ctypes.c_size_t
        sigs = {
            "ko_wlevels": ([], ctypes.c_int64),
            "ko_act_levels": ([], ctypes.c_int64),
            "ko_set_max_threads": ([sz], None),
            "ko_plan_threads": ([sz, sz], sz),
            "ko_frexp": ([ctypes.c_double, p(ctypes.c_double), p(ctypes.c_int32)], None),
            "ko_requant": ([ctypes.c_int64, ctypes.c_int64, ctypes.c_int32], ctypes.c_int64),
            "ko_requant_dyn": ([ctypes.c_int64, ctypes.c_int64, ctypes.c_int64], ctypes.c_int32),
            "ko_from_ratio": ([ctypes.c_uint64] * 4, KoScale),
            "ko_from_f64": ([ctypes.c_double], KoScale),
            "ko_ge": ([KoScale, KoScale], ctypes.c_int),
            "ko_mul": ([KoScale, KoScale], KoScale),
            "ko_apply": ([KoScale, ctypes.c_int64], ctypes.c_int64),
            "ko_recip": ([KoScale], KoScale),
            "ko_isqrt_u128": ([ctypes.c_uint64, ctypes.c_uint64, p(ctypes.c_uint64), p(ctypes.c_uint64)], None),
            "ko_quant_to": ([i32p, sz, ctypes.c_int64, i32p], None),
            "ko_table": ([ctypes.c_int, i64p, sz, p(KoScale), i64p, p(KoScale)], ctypes.c_int),
            "ko_table_index": ([ctypes.c_int, ctypes.c_int64, KoScale], ctypes.c_int64),
            "ko_quantize_weights": ([f32p, sz, i32p, p(KoScale)], None),
            "ko_quantize_bias": ([f32p, sz, i64p, p(KoScale)], ctypes.c_int),
            "ko_from_reals_f32": ([f32p, sz, ctypes.c_int64, i32p, p(KoScale)], None),
            "ko_linear": ([i32p, i32p, sz, sz, sz, i64p], None),
            "ko_linear_digits": ([i32p, i32p, sz, sz, sz, sz, i64p], None),
            "ko_linear_small": ([i32p, i32p, sz, sz, sz, sz, i64p], None),
            "ko_corpus_case": ([ctypes.c_int, p(sz), p(sz), p(sz), i32p, i32p], ctypes.c_int),
            "ko_moe_new": ([sz, sz, sz, sz, f32p, f32p, f32p, ctypes.c_int, f32p, sz, f32p], ctypes.c_void_p),
            "ko_moe_free": ([ctypes.c_void_p], None),
            "ko_moe_set_shared_gate": ([ctypes.c_void_p, f32p], None),
            "ko_moe_weights": ([ctypes.c_void_p, ctypes.c_int, sz, i32p], KoScale),
            "ko_moe_router_bias": ([ctypes.c_void_p, i64p, p(KoScale)], ctypes.c_int),
            "ko_moe_sigmoid_bias": ([ctypes.c_void_p, i64p], ctypes.c_int),
            "ko_moe_forward": ([ctypes.c_void_p, i32p, sz, KoScale, i32p, p(KoScale)], None),
            "ko_moe_forward_tokens": ([ctypes.c_void_p, i32p, sz, KoScale, i32p, p(KoScale)], None),
            "ko_moe_forward_par": ([ctypes.c_void_p, i32p, sz, KoScale, i32p, p(KoScale), sz], None),
            "ko_synth_normal": ([ctypes.c_uint64, ctypes.c_float, ctypes.c_uint64, sz, f32p], None),
            "ko_synth_normal_portable": ([ctypes.c_uint64, ctypes.c_float, ctypes.c_uint64, sz, f32p], None),
            "ko_lcg_uniform": ([ctypes.c_uint64, ctypes.c_int64, ctypes.c_int64, sz, i32p], None),
            "ko_moe_forward_with_local_experts": ([ctypes.c_void_p, i32p, sz, KoScale, i32p, p(KoScale)], None),
            "ko_moe_forward_with_given_experts": ([ctypes.c_void_p, i32p, sz, KoScale, i32p, p(KoScale), i32p,
                                                   p(KoScale)], None),
            "ko_moe_route": ([ctypes.c_void_p, i32p, sz, KoScale, i32p, i64p, i64p], None),
            "ko_moe_router_logits": ([ctypes.c_void_p, i32p, sz, KoScale, i32p, p(KoScale)], None),
            "ko_moe_expert": ([ctypes.c_void_p, sz, i32p, KoScale, i32p, p(KoScale)], None),
            "ko_add": ([i32p, KoScale, i32p, KoScale, sz, i32p, p(KoScale)], None),
            "ko_rmsnorm": ([f32p, sz, ctypes.c_double, i32p, sz, KoScale, i32p, p(KoScale), i32p, p(KoScale),
                            p(KoScale)], None),
            "ko_scale_add": ([KoScale, KoScale], KoScale),
            "ko_scale_rsqrt": ([KoScale], KoScale),
            "ko_scale_from_f64": ([ctypes.c_double], KoScale),
        }
        for name, (args, res) in sigs.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def _p(a: np.ndarray, ct):
    return a.ctypes.data_as(ctypes.POINTER(ct))


def S(t) -> KoScale:
    return KoScale(int(t[0]), int(t[1]))


WLEVELS = 265720
ACT_LEVELS = 1 << 28


# ── kt-int ──
def from_ratio(num: int, den: int):
    m = (1 << 64) - 1
    return lib().ko_from_ratio(num >> 64, num & m, den >> 64, den & m).tup()


def from_f64(x: float):
    return lib().ko_from_f64(x).tup()


def ge(a, b) -> bool:
    return bool(lib().ko_ge(S(a), S(b)))


def mul(a, b):
    return lib().ko_mul(S(a), S(b)).tup()


def apply(s, v: int) -> int:
    return int(lib().ko_apply(S(s), v))


def recip(s):
    return lib().ko_recip(S(s)).tup()


def isqrt_u128(n: int) -> int:
    hi, lo = ctypes.c_uint64(), ctypes.c_uint64()
    lib().ko_isqrt_u128(n >> 64, n & ((1 << 64) - 1), ctypes.byref(hi), ctypes.byref(lo))
    return (hi.value << 64) | lo.value


def requant_dyn(v: int, num_level: int, den: int) -> int:
    return int(lib().ko_requant_dyn(v, num_level, den))


def quant_to(data: np.ndarray, xmax: int) -> np.ndarray:
    data = np.ascontiguousarray(data, dtype=np.int32)
    out = np.empty_like(data)
    lib().ko_quant_to(_p(data, ctypes.c_int32), data.size, xmax, _p(out, ctypes.c_int32))
    return out


def table(kind: int):
    """kind 0 = router exp, 1 = SiLU, 2 = sigmoid → (codes, inv_step_scale, lo_index, code_scale)."""
    codes = np.empty(1 << 16, dtype=np.int64)
    a, b = KoScale(), KoScale()
    lo = ctypes.c_int64()
    n = lib().ko_table(kind, _p(codes, ctypes.c_int64), codes.size, ctypes.byref(a), ctypes.byref(lo), ctypes.byref(b))
    return codes[:n], a.tup(), lo.value, b.tup()


def table_index(kind: int, data: int, s) -> int:
    return int(lib().ko_table_index(kind, data, S(s)))


def quantize_weights(w: np.ndarray):
    w = np.ascontiguousarray(w, dtype=np.float32)
    codes = np.empty(w.shape, dtype=np.int32)
    s = KoScale()
    lib().ko_quantize_weights(_p(w, ctypes.c_float), w.size, _p(codes, ctypes.c_int32), ctypes.byref(s))
    return codes, s.tup()


def from_reals_f32(v: np.ndarray, levels: int = ACT_LEVELS):
    v = np.ascontiguousarray(v, dtype=np.float32)
    data = np.empty(v.shape, dtype=np.int32)
    s = KoScale()
    lib().ko_from_reals_f32(_p(v, ctypes.c_float), v.size, levels, _p(data, ctypes.c_int32), ctypes.byref(s))
    return data, s.tup()


def linear(x: np.ndarray, w: np.ndarray, rows: int, out: int, k: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.int32)
    w = np.ascontiguousarray(w, dtype=np.int32)
    y = np.empty(rows * out, dtype=np.int64)
    lib().ko_linear(_p(x, ctypes.c_int32), _p(w, ctypes.c_int32), rows, out, k, _p(y, ctypes.c_int64))
    return y


KT_FLUSH_TERMS = 83886 * 16  # kt-cuda/src/digits.rs:16-19: KT_FLUSH tiles of 16 terms
SMALL_FLUSH_TERMS = 422733  # the small-code GEMM's split: floor((2^31 - 1) / (127 · 40))


def linear_digits(x: np.ndarray, w: np.ndarray, rows: int, out: int, k: int, flush: int = KT_FLUSH_TERMS):
    """The reference's digit algorithm (kt-cuda host executor): nine wrapping int32 plane sums flushed into i64."""
    x = np.ascontiguousarray(x, dtype=np.int32)
    w = np.ascontiguousarray(w, dtype=np.int32)
    y = np.empty(rows * out, dtype=np.int64)
    lib().ko_linear_digits(_p(x, ctypes.c_int32), _p(w, ctypes.c_int32), rows, out, k, flush, _p(y, ctypes.c_int64))
    return y


def linear_small(x: np.ndarray, w: np.ndarray, rows: int, out: int, k: int, flush: int = SMALL_FLUSH_TERMS):
    """The library's (1, 2)-plane decomposition for |x| <= 127, |w| <= 3280: two wrapping int32 sums flushed into i64."""
    x = np.ascontiguousarray(x, dtype=np.int32)
    w = np.ascontiguousarray(w, dtype=np.int32)
    y = np.empty(rows * out, dtype=np.int64)
    lib().ko_linear_small(_p(x, ctypes.c_int32), _p(w, ctypes.c_int32), rows, out, k, flush, _p(y, ctypes.c_int64))
    return y


def synth_normal(seed: int, sigma: float, n: int, offset: int = 0) -> np.ndarray:
    """Elements [offset, offset + n) of the build-defined N(0, sigma) stream ``seed`` (splitmix64 + Box-Muller in f64,
    rounded to f32), computed by the oracle itself."""
    out = np.empty(n, dtype=np.float32)
    lib().ko_synth_normal(seed, sigma, offset, n, _p(out, ctypes.c_float))
    return out


def synth_normal_portable(seed: int, sigma: float, n: int, offset: int = 0) -> np.ndarray:
    """Elements [offset, offset + n) of the portable N(0, sigma) stream (own ln and cos from IEEE operations), the one
    the GPU library generates weights with on the device."""
    out = np.empty(n, dtype=np.float32)
    lib().ko_synth_normal_portable(seed, sigma, offset, n, _p(out, ctypes.c_float))
    return out


def lcg_uniform(seed: int, lo: int, hi: int, n: int) -> np.ndarray:
    """Uniform integers in [lo, hi] from the reference's test LCG (gate.rs:29-36)."""
    out = np.empty(n, dtype=np.int32)
    lib().ko_lcg_uniform(seed, lo, hi, n, _p(out, ctypes.c_int32))
    return out


def corpus():
    """The reference's equality-gate corpus: a list of (label, rows, out, k, x, w)."""
    labels = ["k=1", "odd tail", "k=33", "k=1023", "k=4099 (long)", "threaded 8×512×2048", "extremes ±WLEVELS",
              "all +WLEVELS"]
    cases = []
    for i in range(8):
        r, o, k = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
        lib().ko_corpus_case(i, ctypes.byref(r), ctypes.byref(o), ctypes.byref(k), None, None)
        x = np.empty(r.value * k.value, dtype=np.int32)
        w = np.empty(o.value * k.value, dtype=np.int32)
        lib().ko_corpus_case(i, ctypes.byref(r), ctypes.byref(o), ctypes.byref(k), _p(x, ctypes.c_int32),
                             _p(w, ctypes.c_int32))
        cases.append((labels[i], r.value, o.value, k.value, x, w))
    return cases


class MoeOracle:
    """The reference MoeMlp (layers.rs:661-1106) restated on the CPU, built from f32 weights."""

    def __init__(self, dim, n_experts, hidden, top_k, router_w, expert_w, *, router_bias=None, norm_topk=False,
                 sigmoid_bias=None, shared_hidden=0, shared_w=None, shared_gate_w=None):
        self.dim, self.n_experts, self.hidden, self.top_k = dim, n_experts, hidden, top_k
        self.shared_hidden = shared_hidden
        keep = []

        def f(a):
            if a is None:
                return None
            a = np.ascontiguousarray(a, dtype=np.float32)
            keep.append(a)
            return _p(a, ctypes.c_float)

        self._h = lib().ko_moe_new(dim, n_experts, hidden, top_k, f(router_w), f(router_bias), f(expert_w),
                                   1 if norm_topk else 0, f(sigmoid_bias), shared_hidden, f(shared_w))
        if shared_gate_w is not None:
            # the extension: Qwen2-MoE's sigmoid-gated shared expert (shared_expert_gate [1, dim])
            lib().ko_moe_set_shared_gate(self._h, f(shared_gate_w))

    def __del__(self):
        if getattr(self, "_h", None):
            lib().ko_moe_free(self._h)
            self._h = None

    def weights(self, which: int, e: int = 0):
        shapes = {0: (self.n_experts, self.dim), 1: (self.hidden, self.dim), 2: (self.hidden, self.dim),
                  3: (self.dim, self.hidden), 4: (self.shared_hidden, self.dim), 5: (self.shared_hidden, self.dim),
                  6: (self.dim, self.shared_hidden), 7: (1, self.dim)}
        codes = np.empty(shapes[which], dtype=np.int32)
        s = lib().ko_moe_weights(self._h, which, e, _p(codes, ctypes.c_int32))
        return codes, s.tup()

    def router_bias(self):
        codes = np.empty(self.n_experts, dtype=np.int64)
        s = KoScale()
        ok = lib().ko_moe_router_bias(self._h, _p(codes, ctypes.c_int64), ctypes.byref(s))
        return (codes, s.tup()) if ok else None

    def sigmoid_bias(self):
        codes = np.empty(self.n_experts, dtype=np.int64)
        ok = lib().ko_moe_sigmoid_bias(self._h, _p(codes, ctypes.c_int64))
        return codes if ok else None

    def _x(self, x):
        x = np.ascontiguousarray(x, dtype=np.int32)
        return x, x.size // self.dim

    def forward(self, x, xs):
        x, rows = self._x(x)
        y = np.empty(rows * self.dim, dtype=np.int32)
        s = KoScale()
        lib().ko_moe_forward(self._h, _p(x, ctypes.c_int32), rows, S(xs), _p(y, ctypes.c_int32), ctypes.byref(s))
        return y.reshape(rows, self.dim), s.tup()

    def forward_par(self, x, xs, threads: int = 0):
        """forward() with the tokens spread over host threads (0 = every core); the same bits as forward()."""
        x, rows = self._x(x)
        y = np.empty(rows * self.dim, dtype=np.int32)
        s = KoScale()
        lib().ko_moe_forward_par(self._h, _p(x, ctypes.c_int32), rows, S(xs), _p(y, ctypes.c_int32), ctypes.byref(s),
                                 threads)
        return y.reshape(rows, self.dim), s.tup()

    def forward_tokens(self, x, xs):
        x, rows = self._x(x)
        y = np.empty(rows * self.dim, dtype=np.int32)
        ss = (KoScale * rows)()
        lib().ko_moe_forward_tokens(self._h, _p(x, ctypes.c_int32), rows, S(xs), _p(y, ctypes.c_int32), ss)
        return y.reshape(rows, self.dim), [s.tup() for s in ss]

    def forward_with_local_experts(self, x, xs):
        x, rows = self._x(x)
        y = np.empty(rows * self.dim, dtype=np.int32)
        s = KoScale()
        lib().ko_moe_forward_with_local_experts(self._h, _p(x, ctypes.c_int32), rows, S(xs), _p(y, ctypes.c_int32),
                                                ctypes.byref(s))
        return y.reshape(rows, self.dim), s.tup()

    def forward_with_given_experts(self, x, xs, ye, yse):
        """The seam with the expert outputs given: ye [rows][top_k][d] int32, yse [rows][top_k] of (mant, shift)."""
        x, rows = self._x(x)
        ye = np.ascontiguousarray(ye, dtype=np.int32)
        ys_arr = (KoScale * max(1, rows * self.top_k))()
        for i, (mt, sh) in enumerate(yse):
            ys_arr[i] = KoScale(int(mt), int(sh))
        y = np.empty(x.size, dtype=np.int32)
        s = KoScale()
        lib().ko_moe_forward_with_given_experts(self._h, _p(x, ctypes.c_int32), rows, S(xs), _p(ye, ctypes.c_int32),
                                                ys_arr, _p(y, ctypes.c_int32), ctypes.byref(s))
        return y.reshape(rows, self.dim), s.tup()

    def route(self, x, xs):
        x, rows = self._x(x)
        ex = np.empty(rows * self.top_k, dtype=np.int32)
        ec = np.empty(rows * self.top_k, dtype=np.int64)
        sumc = np.empty(rows, dtype=np.int64)
        lib().ko_moe_route(self._h, _p(x, ctypes.c_int32), rows, S(xs), _p(ex, ctypes.c_int32),
                           _p(ec, ctypes.c_int64), _p(sumc, ctypes.c_int64))
        return ex.reshape(rows, self.top_k), ec.reshape(rows, self.top_k), sumc

    def router_logits(self, x, xs):
        x, rows = self._x(x)
        lg = np.empty(rows * self.n_experts, dtype=np.int32)
        ss = (KoScale * rows)()
        lib().ko_moe_router_logits(self._h, _p(x, ctypes.c_int32), rows, S(xs), _p(lg, ctypes.c_int32), ss)
        return lg.reshape(rows, self.n_experts), [s.tup() for s in ss]

    def expert(self, e, xrow, xs):
        xrow = np.ascontiguousarray(xrow, dtype=np.int32)
        y = np.empty(self.dim, dtype=np.int32)
        s = KoScale()
        lib().ko_moe_expert(self._h, e, _p(xrow, ctypes.c_int32), S(xs), _p(y, ctypes.c_int32), ctypes.byref(s))
        return y, s.tup()


def add(a, a_s, b, b_s):
    a = np.ascontiguousarray(a, dtype=np.int32)
    b = np.ascontiguousarray(b, dtype=np.int32)
    y = np.empty_like(a)
    s = KoScale()
    lib().ko_add(_p(a, ctypes.c_int32), S(a_s), _p(b, ctypes.c_int32), S(b_s), a.size, _p(y, ctypes.c_int32),
                 ctypes.byref(s))
    return y, s.tup()


def scale_add(a, b):
    """Scale::add (kt-int lib.rs:285-303)."""
    return lib().ko_scale_add(S(a), S(b)).tup()


def scale_rsqrt(a):
    """Scale::rsqrt (kt-int lib.rs:307-318), mant > 0."""
    return lib().ko_scale_rsqrt(S(a)).tup()


def rmsnorm(weight: np.ndarray, eps: float, x: np.ndarray, xs):
    """RmsNorm::new(weight, eps).forward_int (layers.rs:352-449) on rows of x codes: (y, y_scale, wcodes, w_scale,
    eps_scale)."""
    w = np.ascontiguousarray(weight, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.int32)
    dim = w.size
    rows = x.size // dim
    y = np.empty(x.size, np.int32)
    wc = np.empty(dim, np.int32)
    ys, ws, es = KoScale(), KoScale(), KoScale()
    lib().ko_rmsnorm(_p(w, ctypes.c_float), dim, float(eps), _p(x, ctypes.c_int32), rows, S(xs), _p(y, ctypes.c_int32),
                     ctypes.byref(ys), _p(wc, ctypes.c_int32), ctypes.byref(ws), ctypes.byref(es))
    return y.reshape(x.shape), ys.tup(), wc, ws.tup(), es.tup()


def to_bytes(data: np.ndarray, shape, mant: int, shift: int) -> bytes:
    """IntTensor::to_bytes (kt-core/src/tensor.rs:51-67): u32 ndim, ndim x u64 shape, i64 mant, i32 shift, u64 ndata,
    ndata x i32, all little-endian."""
    import struct

    data = np.ascontiguousarray(data, dtype="<i4").reshape(-1)
    head = struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", int(s)) for s in shape)
    return head + struct.pack("<qiQ", int(mant), int(shift), data.size) + data.tobytes()


def from_bytes(b: bytes):
    """IntTensor::from_bytes (kt-core/src/tensor.rs:70-100): (data, shape, (mant, shift), bytes read)."""
    import struct

    (nd,) = struct.unpack_from("<I", b, 0)
    shape = list(struct.unpack_from(f"<{nd}Q", b, 4))
    c = 4 + 8 * nd
    mant, shift, n = struct.unpack_from("<qiQ", b, c)
    c += 20
    data = np.frombuffer(b, dtype="<i4", count=n, offset=c).astype(np.int32)
    return data, shape, (mant, shift), c + 4 * n
