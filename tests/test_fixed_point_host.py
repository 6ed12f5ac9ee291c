"""The product's exact fixed-point source (tritify_b200/csrc/fixed_point.cuh, the same header the kernels include),
compiled for the host and compared with the oracle's restatement of kt-int and kt-core on seeded inputs."""

import ctypes
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class FpScale(ctypes.Structure):
    _fields_ = [("mant", ctypes.c_int64), ("shift", ctypes.c_int32)]


@pytest.fixture(scope="module")
def fp(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("fp") / "libfp.so")
    src = os.path.join(ROOT, "tests", "native", "fixed_point_harness.cpp")
    subprocess.run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-x", "c++", "-I",
                    os.path.join(ROOT, "tritify_b200", "csrc"), src, "-o", out], check=True)
    L = ctypes.CDLL(out)
    P = ctypes.POINTER
    L.fp_from_ratio.argtypes = [ctypes.c_uint64] * 4
    L.fp_from_ratio.restype = FpScale
    L.fp_ge.argtypes = [FpScale, FpScale]
    L.fp_mul.argtypes = [FpScale, FpScale]
    L.fp_mul.restype = FpScale
    L.fp_apply.argtypes = [FpScale, ctypes.c_int64]
    L.fp_apply.restype = ctypes.c_int64
    L.fp_recip.argtypes = [FpScale]
    L.fp_recip.restype = FpScale
    L.fp_requant_act.argtypes = [ctypes.c_int64, ctypes.c_int64]
    L.fp_requant_act.restype = ctypes.c_int32
    L.fp_quant_to.argtypes = [ctypes.c_int32, ctypes.c_int64]
    L.fp_quant_to.restype = ctypes.c_int32
    L.fp_split.argtypes = [ctypes.c_int32, P(ctypes.c_int8)]
    L.fp_requant_act_fast_n.argtypes = [P(ctypes.c_int64), P(ctypes.c_int64), P(ctypes.c_int32), ctypes.c_int64]
    L.fp_apply_small.argtypes = [FpScale, ctypes.c_int64]
    L.fp_apply_small.restype = ctypes.c_int64
    L.fp_quant_to_act.argtypes = [ctypes.c_int32]
    L.fp_quant_to_act.restype = ctypes.c_int32
    L.fp_requant_row_n.argtypes = [P(ctypes.c_int64), P(ctypes.c_int64), P(ctypes.c_int32), ctypes.c_int64]
    L.fp_quant_row_n.argtypes = [P(ctypes.c_int32), P(ctypes.c_int64), P(ctypes.c_int32), ctypes.c_int64]
    L.fp_apply_row.argtypes = [FpScale, ctypes.c_int64]
    L.fp_apply_row.restype = ctypes.c_int64
    L.fp_requant_act_n.argtypes = [P(ctypes.c_int64), P(ctypes.c_int64), P(ctypes.c_int32), ctypes.c_int64]
    L.fp_quant_to_n.argtypes = [P(ctypes.c_int32), P(ctypes.c_int64), P(ctypes.c_int32), ctypes.c_int64]
    L.fp_req_mag_n.argtypes = [P(ctypes.c_int64), P(ctypes.c_int64), ctypes.c_int, P(ctypes.c_uint32),
                               P(ctypes.c_uint8), ctypes.c_int64]
    L.fp_req_exact_n.argtypes = [P(ctypes.c_int64), P(ctypes.c_int64), P(ctypes.c_int64), ctypes.c_int64]
    L.fp_down_code_mismatches.restype = ctypes.c_int64
    return L


def _t(s):
    return (int(s.mant), int(s.shift))


def _lcg(seed):
    s = seed
    while True:
        s = (s * 6364136223846793005 + 1442695040888963407) & ((1 << 64) - 1)
        yield s


def test_from_ratio_mul_recip_ge_apply_equal_the_oracle(fp, oracle):
    g = _lcg(0x5CA1E)
    M = (1 << 64) - 1
    for i in range(6000):
        bits_n = 1 + next(g) % 100
        bits_d = 1 + next(g) % 90
        num = (next(g) | (next(g) << 64)) & ((1 << bits_n) - 1) or 1
        den = (next(g) | (next(g) << 64)) & ((1 << bits_d) - 1) or 1
        a = fp.fp_from_ratio(num >> 64, num & M, den >> 64, den & M)
        assert _t(a) == oracle.from_ratio(num, den), (num, den)
        b = oracle.from_ratio(next(g) % (1 << 50) + 1, next(g) % (1 << 40) + 1)
        bs = FpScale(*b)
        assert _t(fp.fp_mul(a, bs)) == oracle.mul(_t(a), b)
        assert bool(fp.fp_ge(a, bs)) == oracle.ge(_t(a), b)
        assert bool(fp.fp_ge(bs, a)) == oracle.ge(b, _t(a))
        if a.mant:  # the reference asserts a non-zero scale in recip (kt-int lib.rs:276)
            assert _t(fp.fp_recip(a)) == oracle.recip(_t(a))
        v = (next(g) >> 1) - (1 << 62)
        v >>= next(g) % 60
        assert fp.fp_apply(a, v) == oracle.apply(_t(a), v), (a.mant, a.shift, v)
    # equal values with different representations compare equal both ways
    assert fp.fp_ge(FpScale(2, 1), FpScale(1, 0)) and fp.fp_ge(FpScale(1, 0), FpScale(2, 1))
    assert fp.fp_ge(FpScale(0, 0), FpScale(0, 5)) and not fp.fp_ge(FpScale(0, 0), FpScale(1, 0))


def test_requant_act_and_quant_to_equal_the_oracle(fp, oracle):
    rng = np.random.default_rng(7)
    n = 200000
    den = rng.integers(1, 1 << 62, size=n, dtype=np.int64) >> rng.integers(0, 61, size=n)
    den = np.maximum(den, 1)
    v = (rng.integers(-(1 << 62), 1 << 62, size=n, dtype=np.int64) % (den + 1)) * rng.choice([-1, 1], size=n)
    v[:1000] = den[:1000]  # the extremes: |v| == den maps to exactly ±2^28
    v[1000:2000] = -den[1000:2000]
    v[2000:2100] = 0
    out = np.empty(n, dtype=np.int32)
    P = ctypes.POINTER
    fp.fp_requant_act_n(v.ctypes.data_as(P(ctypes.c_int64)), den.ctypes.data_as(P(ctypes.c_int64)),
                        out.ctypes.data_as(P(ctypes.c_int32)), n)
    idx = rng.choice(n, 4000, replace=False)
    want = [oracle.requant_dyn(int(v[i]), 1 << 28, int(den[i])) for i in idx]
    assert list(out[idx]) == want
    assert (out[:1000] == 1 << 28).all() and (out[1000:2000] == -(1 << 28)).all()

    xmax = rng.integers(1, 1 << 31, size=n, dtype=np.int64)
    d = (rng.integers(-(1 << 31), 1 << 31, size=n, dtype=np.int64) % (xmax + 1)).astype(np.int32)
    q = np.empty(n, dtype=np.int32)
    fp.fp_quant_to_n(d.ctypes.data_as(P(ctypes.c_int32)), xmax.ctypes.data_as(P(ctypes.c_int64)),
                     q.ctypes.data_as(P(ctypes.c_int32)), n)
    for i in idx[:2000]:
        assert q[i] == oracle.quant_to(np.array([d[i]]), int(xmax[i]))[0]
    assert np.abs(q).max() <= 265720


def test_digit_split_covers_every_code(fp):
    """kt-cuda/src/tests.rs:21-33: every code in ±WLEVELS is three digits |d| <= 40 and back."""
    d = (ctypes.c_int8 * 3)()
    for v in list(range(-265720, -265000)) + list(range(-3000, 3000)) + list(range(265000, 265721)):
        fp.fp_split(v, d)
        assert all(abs(x) <= 40 for x in d)
        assert d[0] + 81 * d[1] + 6561 * d[2] == v
    fp.fp_split(265720, d)
    assert list(d) == [40, 40, 40]
    fp.fp_split(-265720, d)
    assert list(d) == [-40, -40, -40]


def test_fast_paths_equal_the_exact_ones(fp, oracle):
    """The reciprocal-estimate division, the 64-bit apply and the power-of-two quant_to give the exact results."""
    rng = np.random.default_rng(11)
    n = 300000
    den = np.maximum(rng.integers(1, 1 << 62, size=n, dtype=np.int64) >> rng.integers(0, 62, size=n), 1)
    v = (rng.integers(-(1 << 62), 1 << 62, size=n, dtype=np.int64) % (den + 1)) * rng.choice([-1, 1], size=n)
    v[:500], v[500:1000] = den[:500], -den[500:1000]
    a, b = np.empty(n, np.int32), np.empty(n, np.int32)
    P = ctypes.POINTER
    args = (v.ctypes.data_as(P(ctypes.c_int64)), den.ctypes.data_as(P(ctypes.c_int64)))
    fp.fp_requant_act_n(*args, a.ctypes.data_as(P(ctypes.c_int32)), n)
    fp.fp_requant_act_fast_n(*args, b.ctypes.data_as(P(ctypes.c_int32)), n)
    assert (a == b).all()
    g = _lcg(99)
    for _ in range(20000):
        s = oracle.from_ratio(next(g) % (1 << 60) + 1, next(g) % (1 << 60) + 1)
        s = oracle.mul(s, oracle.from_ratio(next(g) % (1 << 40) + 1, next(g) % (1 << 20) + 1))
        val = int(next(g) % (1 << 31)) - (1 << 30)
        assert fp.fp_apply_small(FpScale(*s), val) == oracle.apply(s, val)
        assert fp.fp_apply_small(FpScale(s[0], s[1] % 70), val) == oracle.apply((s[0], s[1] % 70), val)
    for d in list(range(-(1 << 28), -(1 << 28) + 3000)) + list(range(-5000, 5000)) + list(range((1 << 28) - 3000, (1 << 28) + 1)):
        assert fp.fp_quant_to_act(d) == oracle.quant_to(np.array([d]), 1 << 28)[0]


def test_row_plans_equal_the_exact_ones(fp, oracle):
    """The per-row plans of the hot loops (requant_row, quant_row, apply_row) against the exact i128 forms."""
    rng = np.random.default_rng(12)
    P = ctypes.POINTER
    n = 2_000_000
    for hi in (1 << 52, 1 << 62):  # the 64-bit path and the 128-bit fallback
        den = np.maximum(rng.integers(1, hi, size=n, dtype=np.int64) >> rng.integers(0, 52, size=n), 1)
        v = (rng.integers(0, 1 << 62, size=n, dtype=np.int64) % (den + 1)) * rng.choice([-1, 1], size=n)
        v[::5], v[1::5], v[2::5] = den[::5], -den[1::5], den[2::5] // 2
        v[3::5] = -((den[3::5] + 1) // 2)
        a, b = np.empty(n, np.int32), np.empty(n, np.int32)
        args = (v.ctypes.data_as(P(ctypes.c_int64)), den.ctypes.data_as(P(ctypes.c_int64)))
        fp.fp_requant_act_n(*args, a.ctypes.data_as(P(ctypes.c_int32)), n)
        fp.fp_requant_row_n(*args, b.ctypes.data_as(P(ctypes.c_int32)), n)
        assert (a == b).all()
    xmax = rng.integers(1, 1 << 31, size=n, dtype=np.int64)
    xmax[:1000] = 1
    d = (rng.integers(-(1 << 31), 1 << 31, size=n, dtype=np.int64) % (xmax + 1)).astype(np.int32)
    d[1000:2000] = xmax[1000:2000]
    d[2000:3000] = -xmax[2000:3000]
    a, b = np.empty(n, np.int32), np.empty(n, np.int32)
    fp.fp_quant_to_n(d.ctypes.data_as(P(ctypes.c_int32)), xmax.ctypes.data_as(P(ctypes.c_int64)),
                     a.ctypes.data_as(P(ctypes.c_int32)), n)
    fp.fp_quant_row_n(d.ctypes.data_as(P(ctypes.c_int32)), xmax.ctypes.data_as(P(ctypes.c_int64)),
                      b.ctypes.data_as(P(ctypes.c_int32)), n)
    assert (a == b).all()
    g = _lcg(7)
    for _ in range(40000):
        s = oracle.mul(oracle.from_ratio(next(g) % (1 << 60) + 1, next(g) % (1 << 60) + 1),
                       oracle.from_ratio(next(g) % (1 << 40) + 1, next(g) % (1 << 20) + 1))
        val = int(next(g) % (1 << 32)) - (1 << 31)
        assert fp.fp_apply_row(FpScale(*s), val) == oracle.apply(s, val)
        s2 = (s[0], s[1] % 70 - 3)
        assert fp.fp_apply_row(FpScale(*s2), val) == oracle.apply(s2, val)


def test_certified_paths_near_integer_quotients(fp, oracle):
    """Quotients that sit on or next to an integer, where the double estimate cannot decide and the integer path
    must: requant_row and quant_row against the exact forms."""
    rng = np.random.default_rng(21)
    P = ctypes.POINTER
    n = 600_000
    den = rng.integers(1 << 22, 1 << 52, size=n, dtype=np.int64) >> rng.integers(0, 30, size=n)
    den = np.maximum(den, 1 << 22)
    q = rng.integers(0, 1 << 28, size=n, dtype=np.int64)
    # v with v·2^28 + floor(den/2) at or just around q·den (computed exactly in Python integers)
    v = np.array([min(int(dd), max(0, (int(qq) * int(dd) - int(dd) // 2) // (1 << 28) + int(e)))
                  for qq, dd, e in zip(q, den, rng.integers(-1, 2, size=n))], dtype=np.int64)
    v *= rng.choice([-1, 1], size=n)
    a, b = np.empty(n, np.int32), np.empty(n, np.int32)
    args = (v.ctypes.data_as(P(ctypes.c_int64)), den.ctypes.data_as(P(ctypes.c_int64)))
    fp.fp_requant_act_n(*args, a.ctypes.data_as(P(ctypes.c_int32)), n)
    fp.fp_requant_row_n(*args, b.ctypes.data_as(P(ctypes.c_int32)), n)
    assert (a == b).all()
    xmax = rng.integers(1 << 16, 1 << 31, size=n, dtype=np.int64)
    qd = rng.integers(0, 265721, size=n, dtype=np.int64)
    d = np.array([min(int(xm), max(0, (int(qq) * int(xm) - int(xm) // 2) // 265720 + int(e)))
                  for qq, xm, e in zip(qd, xmax, rng.integers(-1, 2, size=n))], dtype=np.int64)
    d = (d * rng.choice([-1, 1], size=n)).astype(np.int32)
    fp.fp_quant_to_n(d.ctypes.data_as(P(ctypes.c_int32)), xmax.ctypes.data_as(P(ctypes.c_int64)),
                     a.ctypes.data_as(P(ctypes.c_int32)), n)
    fp.fp_quant_row_n(d.ctypes.data_as(P(ctypes.c_int32)), xmax.ctypes.data_as(P(ctypes.c_int64)),
                      b.ctypes.data_as(P(ctypes.c_int32)), n)
    assert (a == b).all()


def test_apply_row_on_int32_values(fp, oracle):
    fp.fp_apply_row32.argtypes = [FpScale, ctypes.c_int32]
    fp.fp_apply_row32.restype = ctypes.c_int64
    g = _lcg(9)
    for _ in range(40000):
        s = oracle.mul(oracle.from_ratio(next(g) % (1 << 60) + 1, next(g) % (1 << 60) + 1),
                       oracle.from_ratio(next(g) % (1 << 40) + 1, next(g) % (1 << 20) + 1))
        for val in (int(next(g) % (1 << 32)) - (1 << 31), -(1 << 31), (1 << 31) - 1, 0, -1, 1):
            assert fp.fp_apply_row32(FpScale(*s), val) == oracle.apply(s, val)


def test_scale_add_rsqrt_isqrt_equal_the_oracle(fp, oracle):
    fp.fp_scale_add.argtypes = [FpScale, FpScale]
    fp.fp_scale_add.restype = FpScale
    fp.fp_scale_rsqrt.argtypes = [FpScale]
    fp.fp_scale_rsqrt.restype = FpScale
    P = ctypes.POINTER
    fp.fp_isqrt.argtypes = [ctypes.c_uint64, ctypes.c_uint64, P(ctypes.c_uint64), P(ctypes.c_uint64)]
    g = _lcg(31)
    for _ in range(20000):
        a = oracle.from_ratio(next(g) % (1 << 62) + 1, next(g) % (1 << 40) + 1)
        b = oracle.from_ratio(next(g) % (1 << 50) + 1, next(g) % (1 << 60) + 1)
        r = fp.fp_scale_add(FpScale(*a), FpScale(*b))
        assert (r.mant, r.shift) == oracle.scale_add(a, b)
        r = fp.fp_scale_rsqrt(FpScale(*a))
        assert (r.mant, r.shift) == oracle.scale_rsqrt(a)
        n = (next(g) << 64) | next(g)
        hi, lo = ctypes.c_uint64(), ctypes.c_uint64()
        fp.fp_isqrt(n >> 64, n & ((1 << 64) - 1), ctypes.byref(hi), ctypes.byref(lo))
        assert (hi.value << 64) | lo.value == oracle.isqrt_u128(n)
    assert oracle.scale_add((0, 0), (5, 3)) == (5, 3)


def test_apply_row_wide_equals_the_oracle(fp, oracle):
    fp.fp_apply_row_wide.argtypes = [FpScale, ctypes.c_int64]
    fp.fp_apply_row_wide.restype = ctypes.c_int64
    g = _lcg(41)
    for _ in range(40000):
        s = oracle.mul(oracle.from_ratio(next(g) % (1 << 60) + 1, next(g) % (1 << 60) + 1),
                       oracle.from_ratio(next(g) % (1 << 40) + 1, next(g) % (1 << 20) + 1))
        val = int(next(g) % (1 << 50)) - (1 << 49)
        assert fp.fp_apply_row_wide(FpScale(*s), val) == oracle.apply(s, val)


def _req_mag(fp, av, den, which):
    P = ctypes.POINTER
    n = len(av)
    q = np.zeros(n, dtype=np.uint32)
    ok = np.zeros(n, dtype=np.uint8)
    fp.fp_req_mag_n(av.ctypes.data_as(P(ctypes.c_int64)), den.ctypes.data_as(P(ctypes.c_int64)), which,
                    q.ctypes.data_as(P(ctypes.c_uint32)), ok.ctypes.data_as(P(ctypes.c_uint8)), n)
    exact = np.zeros(n, dtype=np.int64)
    fp.fp_req_exact_n(av.ctypes.data_as(P(ctypes.c_int64)), den.ctypes.data_as(P(ctypes.c_int64)),
                      exact.ctypes.data_as(P(ctypes.c_int64)), n)
    return q.astype(np.int64), ok.astype(bool), exact


def _near_integer_cases(rng, n):
    """(av, den) whose quotient t = (av·2^28 + floor(den/2)) / den lies within a few 1/den of an integer, from both
    sides: for odd den, av = (delta - floor(den/2)) · 2^-28 mod den puts the numerator at delta mod den."""
    av, den = [], []
    for _ in range(n):
        e = int(rng.integers(22, 52))
        d = int(rng.integers(1 << e, min(1 << (e + 1), 1 << 52))) | 1
        delta = int(rng.choice([0, 1, 2, 3, -1, -2, -3]))
        a = ((delta - d // 2) * pow(1 << 28, -1, d)) % d
        av.append(a)
        den.append(d)
    return np.array(av, dtype=np.int64), np.array(den, dtype=np.int64)


@pytest.mark.parametrize("which", [1, 2])
def test_certified_magnitude_requant_is_exact_or_declines(fp, which):
    """req_mag / req_mag2 (the lean SwiGLU, combine and down-input paths; the same source the kernels compile, with
    the device's fused multiply-add and round-down add taken from the host's IEEE operations) either certify the exact
    floor((|v|·2^28 + floor(den/2)) / den) or decline, for every divisor the lean paths admit (2^22 <= den < 2^52,
    |v| <= den): random magnitudes decline about once in 10^5, quotients placed on and next to integers always
    decline or are exact, and the ends |v| = 0 and |v| = den are exact."""
    rng = np.random.default_rng(28 + which)
    n = 400_000
    e = rng.integers(22, 52, size=n)
    den = np.minimum((rng.random(n) + 1.0) * np.exp2(e), float((1 << 52) - 1)).astype(np.int64)
    av = (rng.random(n) * den).astype(np.int64)
    av = np.minimum(av, den)
    q, ok, exact = _req_mag(fp, av, den, which)
    assert (q[ok] == exact[ok]).all()
    assert (~ok).sum() <= 20  # the near-integer band is 2^-20 wide: about 0.4 expected in 400 000

    av2, den2 = _near_integer_cases(rng, 20_000)
    q2, ok2, exact2 = _req_mag(fp, av2, den2, which)
    assert (q2[ok2] == exact2[ok2]).all()
    assert (~ok2).mean() > 0.9  # t within 3/den of an integer: far inside the band the certificate refuses

    ends_den = np.array([1 << 22, (1 << 22) + 1, 3 << 30, (1 << 52) - 1] * 2, dtype=np.int64)
    ends_av = np.concatenate([np.zeros(4, dtype=np.int64), ends_den[:4]])
    q3, ok3, exact3 = _req_mag(fp, ends_av, ends_den, which)
    assert ok3.all() and (q3 == exact3).all()
    assert (exact3[4:] == 1 << 28).all()


def test_lean_down_code_equals_quant_to_act_for_every_magnitude(fp):
    """The lean paths quantise the down linear's input as (q·WLEVELS + 2^27) >> 28 on |requant| = q, then apply the
    sign; for all 2^28 + 1 magnitudes that equals quant_to_act (layers.rs:23-31 with xmax = 2^28)."""
    assert fp.fp_down_code_mismatches() == 0
