// TEST HARNESS: compiles the product's host+device fixed-point header (tritify_b200/csrc/fixed_point.cuh) for the
// host, so its exact arithmetic can be compared with the oracle on the CPU. Exposes a C API for ctypes.
#include "fixed_point.cuh"

extern "C" {
typedef struct {
    int64_t mant;
    int32_t shift;
} fp_scale;

static inline kt::Scale S(fp_scale s) { return kt::Scale{s.mant, s.shift}; }
static inline fp_scale C(kt::Scale s) { return fp_scale{s.mant, s.shift}; }

fp_scale fp_from_ratio(uint64_t nh, uint64_t nl, uint64_t dh, uint64_t dl) {
    return C(kt::from_ratio(((kt::u128)nh << 64) | nl, ((kt::u128)dh << 64) | dl));
}
int fp_ge(fp_scale a, fp_scale b) { return kt::scale_ge(S(a), S(b)) ? 1 : 0; }
fp_scale fp_mul(fp_scale a, fp_scale b) { return C(kt::scale_mul(S(a), S(b))); }
int64_t fp_apply(fp_scale s, int64_t v) { return kt::scale_apply(S(s), v); }
fp_scale fp_recip(fp_scale s) { return C(kt::scale_recip(S(s))); }
int32_t fp_requant_act(int64_t v, int64_t den) { return kt::requant_act(v, den); }
int32_t fp_requant_dyn(int64_t v, int64_t lvl, int64_t den) { return kt::requant_dyn(v, lvl, den); }
int32_t fp_quant_to(int32_t d, int64_t xmax) { return kt::quant_to(d, xmax); }
void fp_split(int32_t v, int8_t* d) { kt::split_digits(v, d[0], d[1], d[2]); }
int64_t fp_recombine(int32_t a, int32_t b, int32_t c, int32_t d, int32_t e) { return kt::recombine(a, b, c, d, e); }

int32_t fp_requant_act_fast(int64_t v, int64_t den) { return kt::requant_act_fast(v, kt::make_div((uint64_t)den)); }
int64_t fp_apply_small(fp_scale s, int64_t v) { return kt::scale_apply_small(S(s), v); }
int32_t fp_quant_to_act(int32_t d) { return kt::quant_to_act(d); }
void fp_requant_act_fast_n(const int64_t* v, const int64_t* den, int32_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = kt::requant_act_fast(v[i], kt::make_div((uint64_t)den[i]));
}

// Batched forms for speed.
void fp_requant_act_n(const int64_t* v, const int64_t* den, int32_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = kt::requant_act(v[i], den[i]);
}
void fp_quant_to_n(const int32_t* d, const int64_t* xmax, int32_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = kt::quant_to(d[i], xmax[i]);
}
void fp_apply_n(const fp_scale* s, const int64_t* v, int64_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = kt::scale_apply(S(s[i]), v[i]);
}
}

extern "C" {
void fp_requant_row_n(const int64_t* v, const int64_t* den, int32_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = kt::requant_row(v[i], kt::make_req(den[i]));
}
void fp_quant_row_n(const int32_t* d, const int64_t* xmax, int32_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = kt::quant_row(d[i], kt::make_quant(xmax[i]));
}
int64_t fp_apply_row(fp_scale s, int64_t v) { return kt::apply_row(kt::make_apply(S(s)), v); }
}

extern "C" {
int64_t fp_apply_row32(fp_scale s, int32_t v) { return kt::apply_row(kt::make_apply(S(s)), v); }
}

extern "C" {
fp_scale fp_scale_add(fp_scale a, fp_scale b) { return C(kt::scale_add(S(a), S(b))); }
fp_scale fp_scale_rsqrt(fp_scale a) { return C(kt::scale_rsqrt(S(a))); }
void fp_isqrt(uint64_t hi, uint64_t lo, uint64_t* out_hi, uint64_t* out_lo) {
    const kt::u128 r = kt::isqrt_u128(((kt::u128)hi << 64) | lo);
    *out_hi = (uint64_t)(r >> 64);
    *out_lo = (uint64_t)r;
}
}

extern "C" {
int64_t fp_apply_row_wide(fp_scale s, int64_t v) { return kt::apply_row_wide(kt::make_apply(S(s)), v); }
}

extern "C" {
// The certified requant of a magnitude as the lean element paths call it: av = |v| converted to double, inv = the
// row divisor's RN(2^28/den) from make_req; which = 1 (req_mag) or 2 (req_mag2). ok[i] = the certificate held.
void fp_req_mag_n(const int64_t* av, const int64_t* den, int which, uint32_t* q, uint8_t* ok, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        const kt::ReqDiv r = kt::make_req(den[i]);
        uint32_t qq = 0;
        const bool k = which == 1 ? kt::req_mag((double)av[i], r.inv28, qq) : kt::req_mag2((double)av[i], r.inv28, qq);
        q[i] = qq;
        ok[i] = k ? 1 : 0;
    }
}

// floor((av·2^28 + floor(den/2)) / den) in 128-bit integers: the value the certificate must give.
void fp_req_exact_n(const int64_t* av, const int64_t* den, int64_t* q, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        const kt::u128 num = ((kt::u128)(uint64_t)av[i] << 28) + (kt::u128)(uint64_t)(den[i] / 2);
        q[i] = (int64_t)(num / (kt::u128)(uint64_t)den[i]);
    }
}

// The down linear's input code on the lean path, (q·WLEVELS + 2^27) >> 28 on a magnitude q, against quant_to_act(q)
// for every q in [0, 2^28]: the count of differences.
int64_t fp_down_code_mismatches() {
    int64_t bad = 0;
    for (uint32_t q = 0; q <= (1u << 28); ++q) {
        const uint32_t t = (uint32_t)(((uint64_t)q * (uint64_t)kt::WLEVELS + (uint64_t(1) << 27)) >> 28);
        bad += (int32_t)t != kt::quant_to_act((int32_t)q);
    }
    return bad;
}
}
