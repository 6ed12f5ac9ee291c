// Exact integer fixed-point arithmetic of tritify's integer path, for host and device.
//
// Every function here is bit-identical to its tritify counterpart (cited file:line, relative to the reference
// project root). The per-element hot operations (requant_dyn at ACT_LEVELS, quant_to, Scale::apply) are written so
// the GPU never runs a 128-bit software division: a double-precision quotient estimate is corrected with exact
// 128-bit integer remainders, which makes the result the exact floor quotient for any input (the correction loop
// runs at most a couple of steps because the estimate is within one unit; a far-off estimate falls back to the
// exact 128-bit division).
#pragma once

#include <stdint.h>

#ifdef __CUDACC__
#define KT_HD __host__ __device__ __forceinline__
#else
#define KT_HD inline
#endif

namespace kt {

#ifdef __CUDACC__
// The first statement of every kernel of this library. Programmatic dependent launch: a kernel launched with the
// programmatic-serialization attribute may be scheduled once the blocks of the kernel before it on its stream have
// exited; griddepcontrol.wait holds it until that kernel has completed and its writes are visible (a no-op for a
// kernel launched without the attribute). Only launch and set-up overlap; as every kernel waits before it can
// complete, completion keeps the stream's order. (No early launch_dependents: blocks of the next kernel parked on
// the SMs measured slower, 0.442 against 0.395 ms on Qwen-shaped decode, taking room from the shared expert's
// kernels on the side stream.)
__device__ __forceinline__ void pdl_enter() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
#endif

typedef __int128 i128;
typedef unsigned __int128 u128;

// crates/01-engine/kt-core/src/layers.rs:16-18
constexpr int64_t WLEVELS = 265720;  // (3^12 - 1) / 2
constexpr int64_t ACT_LEVELS = int64_t(1) << 28;
constexpr int ACT_SHIFT = 28;
// crates/01-engine/kt-core/src/layers.rs:659
constexpr int ROUTER_CODE_BITS = 20;
// Digit planes: a code v, |v| <= WLEVELS, is d0 + 81 d1 + 81^2 d2 with |di| <= 40
// (crates/02-runtime/kt-cuda/src/digits.rs:8-36).
constexpr int DIGIT_BASE = 81;
constexpr int DIGIT_MAX = 40;

struct Scale {
    int64_t mant;
    int32_t shift;
};

KT_HD Scale scale_zero() { return Scale{0, 0}; }

KT_HD int clz64(uint64_t x) {
#ifdef __CUDA_ARCH__
    return __clzll((long long)x);
#else
    return x ? __builtin_clzll(x) : 64;
#endif
}

// crates/00-kernels/kt-int/src/lib.rs:184-186
KT_HD int bits_u128(u128 x) {
    uint64_t hi = (uint64_t)(x >> 64);
    if (hi) return 128 - clz64(hi);
    uint64_t lo = (uint64_t)x;
    return lo ? 64 - clz64(lo) : 0;
}

KT_HD double u128_to_double(u128 x) {
    return (double)(uint64_t)(x >> 64) * 18446744073709551616.0 + (double)(uint64_t)x;
}

// floor(n / d) for d > 0. The double estimate is exact to within one unit whenever the quotient is below 2^52;
// the remainder is then corrected exactly in 128-bit arithmetic.
KT_HD u128 udiv_u128(u128 n, u128 d) {
    if ((d >> 64) == 0 && (n >> 64) == 0) return (u128)((uint64_t)n / (uint64_t)d);
    double qe = u128_to_double(n) / u128_to_double(d);
    if (qe < 4.0e15) {
        int64_t q = (int64_t)qe;
        i128 r = (i128)n - (i128)((u128)q * d);
        int guard = 0;
        while (r < 0 && guard < 4) {
            --q;
            r += (i128)d;
            ++guard;
        }
        while (r >= (i128)d && guard < 8) {
            ++q;
            r -= (i128)d;
            ++guard;
        }
        if (r >= 0 && r < (i128)d) return (u128)q;
    }
    return n / d;
}

// floor(n / d) for n < 2^96-ish, d < 2^63, quotient < 2^52: the hot-path divide (no 128-bit software division).
KT_HD uint64_t udiv_small_q(u128 n, uint64_t d) {
    double qe = u128_to_double(n) / (double)d;
    int64_t q = (int64_t)qe;
    i128 r = (i128)n - (i128)((u128)(uint64_t)q * d);
    int guard = 0;
    while (r < 0 && guard < 4) {
        --q;
        r += (i128)d;
        ++guard;
    }
    while (r >= (i128)d && guard < 8) {
        ++q;
        r -= (i128)d;
        ++guard;
    }
    if (r >= 0 && r < (i128)d) return (uint64_t)q;
    return (uint64_t)(n / (u128)d);
}

// A divisor with its reciprocal, for many divisions by one per-row value: the quotient estimate is one multiply,
// then the same exact 128-bit remainder correction (correct for quotients below 2^52).
struct FastDiv {
    uint64_t d;
    double inv;    // 1 / d
    double inv28;  // 2^28 / d
};

KT_HD FastDiv make_div(uint64_t d) { return FastDiv{d, 1.0 / (double)d, 268435456.0 / (double)d}; }

KT_HD uint64_t fdiv(u128 n, FastDiv f) {
    const double qe = u128_to_double(n) * f.inv;
    int64_t q = (int64_t)qe;
    i128 r = (i128)n - (i128)((u128)(uint64_t)q * f.d);
    int guard = 0;
    while (r < 0 && guard < 4) {
        --q;
        r += (i128)f.d;
        ++guard;
    }
    while (r >= (i128)f.d && guard < 8) {
        ++q;
        r -= (i128)f.d;
        ++guard;
    }
    if (r >= 0 && r < (i128)f.d) return (uint64_t)q;
    return (uint64_t)(n / (u128)f.d);
}

// crates/00-kernels/kt-int/src/lib.rs:191-212 — Scale::from_ratio.
KT_HD Scale from_ratio(u128 num, u128 den) {
    if (num == 0) return scale_zero();
    // den > 0 is asserted by the reference; callers here never pass 0.
    while (bits_u128(num) > 64 || bits_u128(den) > 64) {
        num >>= 1;
        den >>= 1;
    }
    if (den == 0) den = 1;
    int s = 31 - (bits_u128(num) - bits_u128(den));
    u128 mant;
    if (s >= 0) {
        u128 numer = num << s;
        mant = udiv_u128(numer + den / 2, den);
    } else {
        u128 dd = den << (-s);
        mant = udiv_u128(num + dd / 2, dd);
    }
    return Scale{(int64_t)mant, s};
}

// crates/00-kernels/kt-int/src/lib.rs:227-248 — Scale::ge (exact comparison of mant·2^-shift).
KT_HD bool scale_ge(Scale a, Scale o) {
    if (a.mant == 0) return o.mant == 0;
    if (o.mant == 0) return true;
    u128 ma = (u128)(uint64_t)a.mant, mb = (u128)(uint64_t)o.mant;
    int d = o.shift - a.shift;
    if (d >= 0) {
        if ((uint32_t)d + (uint32_t)bits_u128(ma) > 127) return true;
        return (ma << d) >= mb;
    } else {
        uint32_t e = (uint32_t)(-d);
        if (e + (uint32_t)bits_u128(mb) > 127) return false;
        return ma >= (mb << e);
    }
}

// crates/00-kernels/kt-int/src/lib.rs:252-258 — Scale::mul (from_ratio(p, 1) needs no division).
KT_HD Scale scale_mul(Scale a, Scale o) {
    if (a.mant == 0 || o.mant == 0) return scale_zero();
    u128 num = (u128)(uint64_t)a.mant * (u128)(uint64_t)o.mant;
    // from_ratio(num, 1): num < 2^64 here (mantissas are below 2^32), den = 1
    while (bits_u128(num) > 64) num >>= 1;  // den >> 1 == 0 -> 1, as in the reference loop
    int s = 31 - (bits_u128(num) - 1);
    u128 mant;
    if (s >= 0) {
        mant = num << s;
    } else {
        int sh = -s;
        mant = (num + ((u128)1 << (sh - 1))) >> sh;
    }
    return Scale{(int64_t)mant, s + a.shift + o.shift};
}

// crates/00-kernels/kt-int/src/lib.rs:261-272 — Scale::apply: round(value·mant / 2^shift), half away from zero.
KT_HD int64_t scale_apply(Scale s, int64_t value) {
    if (s.mant == 0) return 0;
    i128 prod = (i128)value * (i128)s.mant;
    if (s.shift <= 0) return (int64_t)(prod << (-s.shift));
    if (s.shift >= 127) return 0;  // |prod| < 2^126: rounds to zero (the reference's shift never gets here)
    i128 half = (i128)1 << (s.shift - 1);
    i128 r = prod >= 0 ? (prod + half) >> s.shift : -(((-prod) + half) >> s.shift);
    return (int64_t)r;
}

// Scale::apply for |value| < 2^30 (every activation code here is within ±2^28): the product fits 64 bits, so the
// rounding shift runs in 64-bit arithmetic; other inputs take the general path.
KT_HD int64_t scale_apply_small(Scale s, int64_t value) {
    if (s.mant == 0) return 0;
    if (value >= (int64_t(1) << 30) || value <= -(int64_t(1) << 30) || s.shift <= 0 || s.mant >= (int64_t(1) << 33))
        return scale_apply(s, value);
    if (s.shift >= 64) return 0;  // |prod| < 2^63 <= 2^(shift-1): rounds to zero
    const int64_t prod = value * s.mant;
    const uint64_t ap = prod >= 0 ? (uint64_t)prod : (uint64_t)(-prod);
    const uint64_t r = (ap + (uint64_t(1) << (s.shift - 1))) >> s.shift;
    return prod >= 0 ? (int64_t)r : -(int64_t)r;
}

// crates/00-kernels/kt-int/src/lib.rs:275-280 — Scale::recip (caller guarantees mant != 0).
KT_HD Scale scale_recip(Scale s) {
    Scale r = from_ratio((u128)1 << 40, (u128)(uint64_t)s.mant);
    return Scale{r.mant, r.shift - s.shift + 40};
}

// crates/00-kernels/kt-int/src/lib.rs:285-303 — Scale::add (exact sum of two non-negative scales, renormalised).
KT_HD Scale scale_add(Scale a, Scale o) {
    if (a.mant == 0) return o;
    if (o.mant == 0) return a;
    const int32_t s = a.shift > o.shift ? a.shift : o.shift;
    const uint32_t da = (uint32_t)(s - a.shift), db = (uint32_t)(s - o.shift);
    if (da >= 96) return a;
    if (db >= 96) return o;
    const u128 sum = ((u128)(uint64_t)a.mant << da) + ((u128)(uint64_t)o.mant << db);
    const Scale fr = from_ratio(sum, 1);
    return Scale{fr.mant, fr.shift + s};
}

// crates/00-kernels/kt-int/src/lib.rs:327-340 — floor(sqrt(n)) by Newton's method from above.
KT_HD u128 isqrt_u128(u128 n) {
    if (n == 0) return 0;
    const int bits = bits_u128(n);
    u128 x = (u128)1 << ((bits + 1) / 2);
    for (;;) {
        const u128 y = (x + udiv_u128(n, x)) >> 1;
        if (y >= x) return x;
        x = y;
    }
}

// crates/00-kernels/kt-int/src/lib.rs:307-318 — Scale::rsqrt (mant > 0): an even exponent, an integer square root
// with 31 fractional bits, the reciprocal.
KT_HD Scale scale_rsqrt(Scale a) {
    u128 m = (u128)(uint64_t)a.mant;
    int32_t s = a.shift;
    if (s & 1) {
        m <<= 1;
        s += 1;
    }
    const u128 r = isqrt_u128(m << 62);
    return scale_recip(Scale{(int64_t)r, 31 + s / 2});
}

// from_ratio(v, 2^28) for 0 < v < 2^63: the output-scale factor of every dynamic requant.
KT_HD Scale ratio_act(int64_t v) { return from_ratio((u128)(uint64_t)v, (u128)ACT_LEVELS); }

// requant_dyn(v, ACT_LEVELS, den) with den's reciprocals precomputed (den = the row's max |v|, so |v| <= den).
// For den < 2^52 the quotient estimate is |v|·(2^28/den) in double (|v| converts exactly) and the remainder
// |v|·2^28 + den/2 - q·den is formed in wrapping 64-bit arithmetic: its true value lies in (-2^53, 2^54), so the
// wrapped value is exact, and at most two unit corrections give the exact floor. Larger dens take the 128-bit path.
KT_HD int32_t requant_act_fast(int64_t v, FastDiv den) {
    const uint64_t av = v >= 0 ? (uint64_t)v : (uint64_t)(-(v + 1)) + 1;
    uint64_t q;
    if (den.d < (uint64_t(1) << 52) && av <= den.d) {
        int64_t qi = (int64_t)((double)av * den.inv28);
        int64_t r = (int64_t)((av << ACT_SHIFT) + (den.d >> 1) - (uint64_t)qi * den.d);
        const int64_t d = (int64_t)den.d;
        if (r < 0) {
            --qi;
            r += d;
            if (r < 0) {
                --qi;
                r += d;
            }
        }
        while (r >= d) {
            ++qi;
            r -= d;
        }
        q = (uint64_t)qi;
    } else {
        const u128 n = ((u128)av << ACT_SHIFT) + (u128)(den.d / 2);
        q = fdiv(n, den);
    }
    return (int32_t)(v >= 0 ? (int64_t)q : -(int64_t)q);
}

// quant_to(d, 2^28): the divisor is a power of two, so round-half-away is a shift. Used for the down linear, whose
// input (a dynamic requant to ACT_LEVELS) always has max |.| = 2^28.
KT_HD int32_t quant_to_act(int32_t d) {
    const int64_t num = (int64_t)d * (int64_t)(int32_t)WLEVELS;
    const uint64_t an = num >= 0 ? (uint64_t)num : (uint64_t)(-num);
    const uint64_t q = (an + (uint64_t(1) << (ACT_SHIFT - 1))) >> ACT_SHIFT;
    return (int32_t)(num >= 0 ? (int64_t)q : -(int64_t)q);
}

// crates/01-engine/kt-core/src/layers.rs:34-39 — requant_dyn(v, ACT_LEVELS, den), den > 0.
KT_HD int32_t requant_act(int64_t v, int64_t den) {
    uint64_t av = v >= 0 ? (uint64_t)v : (uint64_t)(-(v + 1)) + 1;
    u128 n = ((u128)av << ACT_SHIFT) + (u128)(uint64_t)(den / 2);
    uint64_t q = udiv_small_q(n, (uint64_t)den);
    int64_t r = v >= 0 ? (int64_t)q : -(int64_t)q;
    return (int32_t)r;
}

// ───── one-rounding double operations ─────
// The device's own IEEE operations (fused multiply-add, an add rounded toward minus infinity, the low word of a
// double); host builds (the tests' harness) get the same results from the C library's fma, a round-to-nearest sum
// stepped down one ulp when its exact error (TwoSum, no multiplications) shows it rounded up, and a bit copy.
KT_HD double fma_rn(double a, double b, double c) {
#ifdef __CUDA_ARCH__
    return __fma_rn(a, b, c);
#else
    return __builtin_fma(a, b, c);
#endif
}

KT_HD double add_rd(double a, double b) {
#ifdef __CUDA_ARCH__
    return __dadd_rd(a, b);
#else
    const double s = a + b, bb = s - a, err = (a - (s - bb)) + (b - bb);
    return err < 0 ? __builtin_nextafter(s, -__builtin_inf()) : s;
#endif
}

KT_HD uint32_t lo_word(double x) {
#ifdef __CUDA_ARCH__
    return (uint32_t)__double2loint(x);
#else
    uint64_t u;
    __builtin_memcpy(&u, &x, sizeof(u));
    return (uint32_t)u;
#endif
}

// ───── certified requant of a magnitude (the lean element paths) ─────
constexpr double RQ_MAGIC = 6755399441055744.0;  // 1.5·2^52: an add rounded down leaves floor(y) in the low bits
constexpr double RQ_EPS = 4.76837158203125e-07;  // 2^-21

// floor(av·inv + 1/2) for 0 <= av <= den < 2^52 with inv = RN(2^28/den) and den >= 2^22: the one-rounding FMA is within
// 2^-25 + 2^-25 + 1/(2·den) < 2^-22 of t = (av·2^28 + floor(den/2))/den (the bound of requant_row's double path,
// tightened by the fused multiply-add), and t is a multiple of 1/den, so y further than 2^-21 from an integer has
// t's floor. Returns false (q unusable) otherwise.
KT_HD bool req_mag(double av, double inv, uint32_t& q) {
    const double y = fma_rn(av, inv, 0.5);
    const double m = add_rd(y, RQ_MAGIC);
    q = lo_word(m);
    const double fr = y - (m - RQ_MAGIC);
    return __builtin_fabs(fr - 0.5) < 0.5 - RQ_EPS;
}

// The same floor as req_mag from two one-rounding estimates 2^-21 below and above: z = av·inv is within 2^-25 of
// av·2^28/den, and t lies in [z + 1/2 - 2^-25 - 1/(2·den), z + 1/2 + 2^-25]; RN(z + 1/2 ∓ 2^-21) err by at most 2^-25,
// so the low estimate is below t and the high one above it, and equal floors (read from the low words after an add
// of 1.5·2^52 rounded down) certify floor(t). One FMA and one add fewer than req_mag's test of the fraction.
KT_HD bool req_mag2(double av, double inv, uint32_t& q) {
    const double lo = add_rd(fma_rn(av, inv, 0.5 - RQ_EPS), RQ_MAGIC);
    const double hi = add_rd(fma_rn(av, inv, 0.5 + RQ_EPS), RQ_MAGIC);
    q = lo_word(lo);
    return lo_word(lo) == lo_word(hi);
}

// ───── per-row plans for the hot loops ─────
// floor(y) for 0 <= y < 2^31 as a double and as an integer. On the device one add rounded toward minus infinity
// of 1.5·2^52 leaves floor(y) in the low mantissa bits (FP64 pipe only, no conversion instruction).
KT_HD double floor_split(double y, int32_t& q) {
#ifdef __CUDA_ARCH__
    const double m = __dadd_rd(y, 6755399441055744.0);  // 2^52 + 2^51: an ulp of 1 from 2^52 on
    q = (int32_t)(uint32_t)__double_as_longlong(m);
    return m - 6755399441055744.0;
#else
    const double f = __builtin_floor(y);
    q = (int32_t)f;
    return f;
#endif
}

// The divisor of a row's requant (den = the row's max |v|, so |v| <= den) with its reciprocal, built once per row.
struct ReqDiv {
    int64_t d;
    int64_t half;  // floor(d / 2)
    double inv28;  // 2^28 / d
    bool tight;    // d < 2^52: the 64-bit path below is exact
    bool dbl;      // 2^22 <= d < 2^52: the certified double path applies
};

KT_HD ReqDiv make_req(int64_t d) {
    ReqDiv r;
    r.d = d > 0 ? d : 1;
    r.half = r.d / 2;
    r.inv28 = 268435456.0 / (double)r.d;
    r.tight = r.d < (int64_t(1) << 52);
    r.dbl = r.tight && r.d >= (int64_t(1) << 22);
    return r;
}

// requant_dyn(v, 2^28, den) for |v| <= den (layers.rs:34-39): q = floor(t), t = (|v|·2^28 + floor(den/2)) / den,
// then the sign of v.
//
// Certified double path (2^22 <= den < 2^52): y = |v|·(2^28/den) + 1/2 in double differs from t by at most
// 2^-24 (the estimate; |v| converts exactly) + 2^-25 (the last rounding) + 1/(2·den) (floor(den/2)/den is 1/2 or
// 1/2 - 1/(2·den)) < 2^-22. t is a multiple of 1/den, so when y lies more than 2^-21 from every integer, t and y
// share their floor and floor(y) is exact. Otherwise (about one value in a million) the integer path decides.
// Integer path (den < 2^52): the same estimate truncated is within one of the floor; the remainder
// |v|·2^28 + half - q·den lies in (-den, 2·den) and is formed exactly in wrapping 64-bit arithmetic, and one signed
// correction gives the floor.
KT_HD int32_t requant_row(int64_t v, const ReqDiv& r) {
    if (!r.tight) return requant_act(v, r.d);
    if (r.dbl) {
        const double y = __builtin_fabs((double)v) * r.inv28 + 0.5;
        int32_t q;
        const double fr = y - floor_split(y, q);
        if (fr > 4.76837158203125e-07 && fr < 1.0 - 4.76837158203125e-07) return v >= 0 ? q : -q;  // 2^-21
    }
    const uint64_t av = v >= 0 ? (uint64_t)v : (uint64_t)(-v);
    int64_t q = (int64_t)((double)(int64_t)av * r.inv28);
    const int64_t rem = (int64_t)((av << ACT_SHIFT) + (uint64_t)r.half - (uint64_t)q * (uint64_t)r.d);
    q += (int64_t)(rem >= r.d) - (int64_t)(rem < 0);
    return (int32_t)(v >= 0 ? q : -q);
}

// Scale::apply for one row's scale over values |v| < 2^31: with 0 < shift < 64 and mant < 2^32 the product is a
// 32x32->64 multiply and the rounding shift is exact in 64 bits; other scales take the general path.
struct ApplyPlan {
    Scale s;
    uint64_t half;
    uint32_t mant;
    uint32_t shift;
    bool tight;
};

KT_HD ApplyPlan make_apply(Scale s) {
    ApplyPlan p;
    p.s = s;
    p.tight = s.mant > 0 && s.mant < (int64_t(1) << 32) && s.shift > 0 && s.shift < 64;
    p.mant = (uint32_t)s.mant;
    p.shift = (uint32_t)(p.tight ? s.shift : 1);
    p.half = uint64_t(1) << (p.shift - 1);
    return p;
}

KT_HD int64_t apply_row(const ApplyPlan& p, int64_t v) {
    if (!p.tight || v >= (int64_t(1) << 31) || v <= -(int64_t(1) << 31)) return scale_apply(p.s, v);
    const uint32_t av = (uint32_t)(v >= 0 ? v : -v);
    const uint64_t r = ((uint64_t)av * p.mant + p.half) >> p.shift;
    return v >= 0 ? (int64_t)r : -(int64_t)r;
}

// The same for an int32 value (no range check: every int32 other than -2^31 has |v| < 2^31).
KT_HD int64_t apply_row(const ApplyPlan& p, int32_t v) {
    if (!p.tight || v == INT32_MIN) return scale_apply(p.s, v);
    const uint32_t av = (uint32_t)(v >= 0 ? v : -v);
    const uint64_t r = ((uint64_t)av * p.mant + p.half) >> p.shift;
    return v >= 0 ? (int64_t)r : -(int64_t)r;
}

// Scale::apply for any int64 value with a tight plan: |v|·mant < 2^95 in 128-bit arithmetic, then the rounding shift.
KT_HD int64_t apply_row_wide(const ApplyPlan& p, int64_t v) {
    if (!p.tight) return scale_apply(p.s, v);
    const uint64_t av = v >= 0 ? (uint64_t)v : (uint64_t)(-(v + 1)) + 1;
    const u128 r = ((u128)av * p.mant + p.half) >> p.shift;
    return v >= 0 ? (int64_t)r : -(int64_t)r;
}

// quant_to(d, xmax) for one row (layers.rs:23-31): x = |d|·WLEVELS/xmax <= WLEVELS is estimated in double, the
// remainder |d|·WLEVELS + xmax/2 - q·xmax (|d|·WLEVELS < 2^50) is exact in 64 bits, and one signed correction gives
// the floor.
struct QuantPlan {
    int64_t xmax;
    int64_t half;
    double inv;  // WLEVELS / xmax
    bool dbl;    // xmax >= 2^16: the certified double path applies
};

KT_HD QuantPlan make_quant(int64_t xmax) {
    QuantPlan p;
    p.xmax = xmax > 0 ? xmax : 1;
    p.half = p.xmax / 2;
    p.inv = (double)WLEVELS / (double)p.xmax;
    p.dbl = p.xmax >= (int64_t(1) << 16);
    return p;
}

// Certified double path as in requant_row: t = (|d|·WLEVELS + floor(xmax/2)) / xmax <= WLEVELS + 1/2, and
// y = |d|·(WLEVELS/xmax) + 1/2 is within 2^-33 + 1/(2·xmax) <= 2^-17 + 2^-33 of it, so y more than 2^-16 from every
// integer has t's floor. |d| <= xmax < 2^31 (int32 codes).
KT_HD int32_t quant_row(int32_t d, const QuantPlan& p) {
    if (p.dbl) {
        const double y = __builtin_fabs((double)d) * p.inv + 0.5;
        int32_t q;
        const double fr = y - floor_split(y, q);
        if (fr > 1.52587890625e-05 && fr < 1.0 - 1.52587890625e-05) return d >= 0 ? q : -q;  // 2^-16
    }
    const int64_t ad = d >= 0 ? (int64_t)d : -(int64_t)d;
    int64_t q = (int64_t)((double)ad * p.inv);
    const int64_t num = ad * WLEVELS;
    const int64_t rem = num + p.half - q * p.xmax;
    q += (int64_t)(rem >= p.xmax) - (int64_t)(rem < 0);
    return (int32_t)(d >= 0 ? q : -q);
}

// crates/01-engine/kt-core/src/layers.rs:34-39 — the general requant_dyn (any level), exact i128.
KT_HD int32_t requant_dyn(int64_t v, int64_t num_level, int64_t den) {
    i128 prod = (i128)v * (i128)num_level;
    i128 half = (i128)den / 2;
    i128 r = prod >= 0 ? (prod + half) / (i128)den : -(((-prod) + half) / (i128)den);
    return (int32_t)r;
}

// crates/01-engine/kt-core/src/layers.rs:23-31 — quant_to: round_half_away(d·WLEVELS / xmax), xmax > 0.
KT_HD int32_t quant_to(int32_t d, int64_t xmax) {
    int64_t num = (int64_t)d * WLEVELS;
    uint64_t an = num >= 0 ? (uint64_t)num : (uint64_t)(-num);
    uint64_t n = an + (uint64_t)(xmax / 2);
    uint64_t q = udiv_small_q((u128)n, (uint64_t)xmax);
    return (int32_t)(num >= 0 ? (int64_t)q : -(int64_t)q);
}

// crates/02-runtime/kt-cuda/src/digits.rs:40-52 — the balanced base-81 digits of a code (|v| <= WLEVELS), low first.
// The balanced representation is unique, so the offset form below gives the reference's digits.
KT_HD void split_digits(int32_t v, int8_t& d0, int8_t& d1, int8_t& d2) {
    uint32_t u = (uint32_t)(v + (int32_t)WLEVELS);
    uint32_t q0 = u / 81u, q1 = q0 / 81u;
    d0 = (int8_t)((int32_t)(u - q0 * 81u) - DIGIT_MAX);
    d1 = (int8_t)((int32_t)(q0 - q1 * 81u) - DIGIT_MAX);
    d2 = (int8_t)((int32_t)q1 - DIGIT_MAX);
}

// The recombination of the five diagonal plane sums: sum_t 81^t S_t (digit_gemm.cu:30-84 of kt-cuda recombines nine
// plane sums with the same weights; products of equal i+j share a diagonal).
KT_HD int64_t recombine(int32_t s0, int32_t s1, int32_t s2, int32_t s3, int32_t s4) {
    return (int64_t)s0 + 81LL * s1 + 6561LL * s2 + 531441LL * s3 + 43046721LL * s4;
}

}  // namespace kt
