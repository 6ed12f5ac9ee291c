// TEST INFRASTRUCTURE ONLY — the CPU oracle for the integer Mixture-of-Experts path.
//
// This file restates, in plain C++ (with __int128 for the reference's i128/u128 steps), the CPU integer path of
// tritify (the reference, a Rust workspace that cannot be compiled here: no cargo/rustc). Every function cites the
// reference file:line it follows; paths are relative to the reference project root. It is the CHECKER of the GPU
// path, never part of it: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs
// load it. The product library (tritify_b200/libktmoe.so) never links or calls it.
//
// Pinning: the GEMM boundary is pinned by the reference's own golden vector, the SHA-256 of its equality-gate corpus
// (crates/02-runtime/kt-runtime/src/tests_cuda.rs:9), and the fixed-point core by its doc examples and unit-test
// facts (crates/00-kernels/kt-int/src/lib.rs:35-39, :246-252; crates/02-runtime/kt-cuda/src/tests.rs:21-33, :88).
// The MoE layer itself has no literal golden hash in the reference; its semantics follow the restatement below plus
// the reference's property tests (seam no-op, tie rule, sigmoid end codes).
//
// Build: oracle/Makefile (g++ -O3 -ffp-contract=off: the reference's f64 steps are never fused into FMAs).

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <memory>
#include <thread>
#include <vector>

typedef __int128 i128;
typedef unsigned __int128 u128;

extern "C" {
typedef struct {
    int64_t mant;
    int32_t shift;
} ko_scale;
}

namespace ko {

// crates/01-engine/kt-core/src/layers.rs:16-18
static const int64_t WLEVELS = (531441 - 1) / 2;  // (3^12 - 1) / 2 = 265720
static const int64_t ACT_LEVELS = int64_t(1) << 28;
// crates/01-engine/kt-core/src/layers.rs:659
static const uint32_t ROUTER_CODE_BITS = 20;
// crates/01-engine/kt-core/src/router.rs:16-18
static const double SIGMOID_RANGE = 16.0;
static const uint32_t SIGMOID_IDX_BITS = 16;

// ─────────────── kt-int (crates/00-kernels/kt-int/src/lib.rs) ───────────────

// lib.rs:46-60 — frexp by IEEE-754 bit surgery.
static void frexp_bits(double x, double* m_out, int32_t* e_out) {
    if (x == 0.0 || !std::isfinite(x)) {
        *m_out = x;
        *e_out = 0;
        return;
    }
    uint64_t bits;
    std::memcpy(&bits, &x, 8);
    int32_t exp_field = (int32_t)((bits >> 52) & 0x7ff);
    if (exp_field == 0) {
        double m;
        int32_t e;
        frexp_bits(x * 9007199254740992.0, &m, &e);
        *m_out = m;
        *e_out = e - 53;
        return;
    }
    int32_t e = exp_field - 1022;
    uint64_t mantissa = (bits & ~(uint64_t(0x7ff) << 52)) | (uint64_t(1022) << 52);
    double m;
    std::memcpy(&m, &mantissa, 8);
    *m_out = m;
    *e_out = e;
}

// lib.rs:78-86 — requant: round(accum·mant / 2^shift), half away from zero, in i128.
static int64_t requant(int64_t accum, int64_t mant, int32_t shift) {
    i128 prod = (i128)accum * (i128)mant;
    if (shift <= 0) return (int64_t)(prod << (-shift));
    i128 half = (i128)1 << (shift - 1);
    i128 r = prod >= 0 ? (prod + half) >> shift : -(((-prod) + half) >> shift);
    return (int64_t)r;
}

static inline int32_t bits_u128(u128 x) {
    // lib.rs:184-186
    if (x == 0) return 0;
    uint64_t hi = (uint64_t)(x >> 64);
    if (hi) return 128 - __builtin_clzll(hi);
    return 64 - __builtin_clzll((uint64_t)x);
}

struct Scale {
    int64_t mant;
    int32_t shift;
    static Scale zero() { return Scale{0, 0}; }

    // lib.rs:191-212
    static Scale from_ratio(u128 num, u128 den) {
        if (num == 0) return zero();
        if (den == 0) std::abort();  // the reference asserts den > 0
        while (bits_u128(num) > 64 || bits_u128(den) > 64) {
            num >>= 1;
            den >>= 1;
        }
        if (den == 0) den = 1;
        int32_t s = 31 - (bits_u128(num) - bits_u128(den));
        u128 mant;
        if (s >= 0) {
            u128 numer = num << s;
            mant = (numer + den / 2) / den;
        } else {
            u128 dd = den << (-s);
            mant = (num + dd / 2) / dd;
        }
        return Scale{(int64_t)mant, s};
    }

    // lib.rs:215-222
    static Scale from_f64(double x) {
        if (!(x > 0.0 && std::isfinite(x))) return zero();
        double m;
        int32_t e;
        frexp_bits(x, &m, &e);
        return Scale{(int64_t)std::round(m * (double)(uint64_t(1) << 31)), 31 - e};
    }

    // lib.rs:227-248
    bool ge(Scale o) const {
        if (mant == 0) return o.mant == 0;
        if (o.mant == 0) return true;
        u128 ma = (u128)(uint64_t)mant, mb = (u128)(uint64_t)o.mant;
        int32_t d = o.shift - shift;
        if (d >= 0) {
            if ((uint32_t)d + (uint32_t)bits_u128(ma) > 127) return true;
            return (ma << d) >= mb;
        } else {
            uint32_t e = (uint32_t)(-d);
            if (e + (uint32_t)bits_u128(mb) > 127) return false;
            return ma >= (mb << e);
        }
    }

    // lib.rs:252-258
    Scale mul(Scale o) const {
        if (mant == 0 || o.mant == 0) return zero();
        Scale p = from_ratio((u128)(uint64_t)mant * (u128)(uint64_t)o.mant, 1);
        return Scale{p.mant, p.shift + shift + o.shift};
    }

    // lib.rs:261-272
    int64_t apply(int64_t value) const {
        if (mant == 0) return 0;
        i128 prod = (i128)value * (i128)mant;
        if (shift <= 0) return (int64_t)(prod << (-shift));
        i128 half = (i128)1 << (shift - 1);
        i128 r = prod >= 0 ? (prod + half) >> shift : -(((-prod) + half) >> shift);
        return (int64_t)r;
    }

    // lib.rs:275-280
    Scale recip() const {
        if (mant == 0) std::abort();  // the reference asserts
        Scale r = from_ratio((u128)1 << 40, (u128)(uint64_t)mant);
        return Scale{r.mant, r.shift - shift + 40};
    }

    // lib.rs:285-303
    Scale add(Scale o) const {
        if (mant == 0) return o;
        if (o.mant == 0) return *this;
        const int32_t s = std::max(shift, o.shift);
        const uint32_t da = (uint32_t)(s - shift), db = (uint32_t)(s - o.shift);
        if (da >= 96) return *this;
        if (db >= 96) return o;
        const u128 sum = ((u128)(uint64_t)mant << da) + ((u128)(uint64_t)o.mant << db);
        const Scale fr = from_ratio(sum, 1);
        return Scale{fr.mant, fr.shift + s};
    }

    // lib.rs:307-318 (defined after isqrt_u128)
    Scale rsqrt() const;
};

// lib.rs:327-340
static u128 isqrt_u128(u128 n) {
    if (n == 0) return 0;
    uint32_t bits = (uint32_t)bits_u128(n);
    u128 x = (u128)1 << ((bits + 1) / 2);
    for (;;) {
        u128 y = (x + n / x) >> 1;
        if (y >= x) return x;
        x = y;
    }
}

Scale Scale::rsqrt() const {
    if (mant <= 0) std::abort();  // the reference asserts mant > 0
    u128 m = (u128)(uint64_t)mant;
    int32_t s = shift;
    if (s & 1) {
        m <<= 1;
        s += 1;
    }
    const uint32_t k = 31;
    const u128 r = isqrt_u128(m << (2 * k));
    return Scale{(int64_t)r, (int32_t)k + s / 2}.recip();
}

// lib.rs:346-396 — CodeLut: a pointwise nonlinearity tabulated as integer codes.
struct CodeLut {
    std::vector<int64_t> codes;
    Scale inv_step_scale;
    int64_t lo_index;
    size_t n;
    Scale code_scale;
    bool right_identity;

    static CodeLut build(const std::function<double(double)>& f, double lo, double hi, uint32_t idx_bits,
                         uint32_t code_bits, bool right_identity) {
        CodeLut l;
        l.n = size_t(1) << idx_bits;
        double k = (double)(uint64_t(1) << code_bits);
        l.codes.resize(l.n);
        for (size_t i = 0; i < l.n; ++i) {
            double t = (double)i / (double)(l.n - 1);
            double x = lo + (hi - lo) * t;
            l.codes[i] = (int64_t)std::round(f(x) * k);
        }
        double inv_step = (double)(l.n - 1) / (hi - lo);
        l.inv_step_scale = Scale::from_f64(inv_step);
        l.lo_index = (int64_t)std::round(lo * inv_step);
        l.code_scale = Scale::from_f64(1.0 / k);
        l.right_identity = right_identity;
        return l;
    }
    // lib.rs:383-385
    int64_t index(int64_t data, Scale scale) const { return scale.mul(inv_step_scale).apply(data) - lo_index; }
    // lib.rs:393-395
    int64_t code_at(int64_t idx) const {
        int64_t c = std::min<int64_t>(std::max<int64_t>(idx, 0), (int64_t)n - 1);
        return codes[(size_t)c];
    }
};

// The three tables of the MoE path, built exactly as the reference builds them.
// layers.rs:688 (router softmax exp over [-30,0]), layers.rs:599 (SiLU over [-30,30], identity right tail),
// router.rs:40-47 (sigmoid over [-16,16]).
static CodeLut exp_table() {
    return CodeLut::build([](double x) { return std::exp(x); }, -30.0, 0.0, 16, ROUTER_CODE_BITS, false);
}
static CodeLut silu_table() {
    return CodeLut::build([](double x) { return x / (1.0 + std::exp(-x)); }, -30.0, 30.0, 16, 20, true);
}
static CodeLut sigmoid_table() {
    return CodeLut::build([](double x) { return 1.0 / (1.0 + std::exp(-x)); }, -SIGMOID_RANGE, SIGMOID_RANGE,
                          SIGMOID_IDX_BITS, ROUTER_CODE_BITS, false);
}

// ─────────────── kt-core (crates/01-engine/kt-core/src) ───────────────

// tensor.rs:10-14 — an activation: i32 data, shape, one Scale.
struct IntTensor {
    std::vector<int32_t> data;
    std::vector<size_t> shape;
    Scale scale;
    size_t len() const { return data.size(); }
    // tensor.rs:47-49
    int64_t max_abs_data() const {
        int64_t a = 0;
        for (int32_t v : data) a = std::max<int64_t>(a, std::llabs((int64_t)v));
        return a;
    }
};

static IntTensor zeros(size_t n, std::vector<size_t> shape) { return IntTensor{std::vector<int32_t>(n, 0), shape, Scale::zero()}; }

// layers.rs:23-31 — quant_to: round_half_away(d·WLEVELS / xmax), i64.
static std::vector<int32_t> quant_to(const std::vector<int32_t>& data, int64_t xmax) {
    int64_t half = xmax / 2;
    std::vector<int32_t> out(data.size());
    for (size_t i = 0; i < data.size(); ++i) {
        int64_t num = (int64_t)data[i] * WLEVELS;
        out[i] = (int32_t)(num >= 0 ? (num + half) / xmax : -((-num + half) / xmax));
    }
    return out;
}

// layers.rs:34-39 — requant_dyn: round_half_away(v·num_level / den), i128.
static int32_t requant_dyn(int64_t v, int64_t num_level, int64_t den) {
    i128 prod = (i128)v * (i128)num_level;
    i128 half = (i128)den / 2;
    i128 r = prod >= 0 ? (prod + half) / (i128)den : -(((-prod) + half) / (i128)den);
    return (int32_t)r;
}

// tensor.rs:106-116 — the entry quantiser (f64, entry boundary only).
static IntTensor from_reals(const double* real, size_t n, std::vector<size_t> shape, int64_t levels) {
    double mx = 0.0;
    for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, std::fabs(real[i]));
    if (mx == 0.0) return zeros(n, shape);
    double step = mx / (double)levels;
    Scale scale = Scale::from_f64(step);
    double inv = (double)levels / mx;
    IntTensor t{std::vector<int32_t>(n), shape, scale};
    for (size_t i = 0; i < n; ++i) t.data[i] = (int32_t)std::round(real[i] * inv);
    return t;
}

// backend.rs:66-69 — dot_portable: widening i32·i32 → i64.
static int64_t dot_portable(const int32_t* a, const int32_t* b, size_t k) {
    int64_t s = 0;
    for (size_t i = 0; i < k; ++i) s += (int64_t)a[i] * (int64_t)b[i];
    return s;
}

// layers.rs:48-77 — the worker-thread cap (0 = every core).
static size_t g_max_threads = 0;
static size_t resolve_threads(size_t nblocks) {
    size_t want = g_max_threads;
    if (want == 0) {
        want = std::thread::hardware_concurrency();
        if (want == 0) want = 1;
    }
    return std::max<size_t>(1, std::min(want, std::max<size_t>(nblocks, 1)));
}

static size_t isqrt_usize(size_t v) { return (size_t)isqrt_u128((u128)v); }

// Set inside the workers of ko_moe_forward_par, which already spread tokens over the cores: their linears run on the
// calling thread. The partition of a linear never changes its values (each output is one exact i64 dot product).
static thread_local bool tl_serial = false;

// backend.rs:74-94 — plan_threads.
static const size_t WORK_PER_SPAWN = size_t(1) << 17;
static const size_t SERIAL_BELOW = size_t(1) << 20;
static size_t plan_threads(size_t elems, size_t work) {
    if (tl_serial) return 1;
    if (work < SERIAL_BELOW) return 1;
    return std::max<size_t>(1, std::min(resolve_threads(elems), isqrt_usize(work / WORK_PER_SPAWN)));
}

// backend.rs:101-127, :133-140 — linear_cpu: the flat rows×out partition into contiguous runs.
static std::vector<int64_t> linear_cpu(const int32_t* x, const int32_t* w, size_t rows, size_t out, size_t k) {
    std::vector<int64_t> acc(rows * out, 0);
    if (acc.empty()) return acc;
    size_t work = rows * out * k;
    size_t threads = plan_threads(rows * out, work);
    size_t len = acc.size();
    size_t chunk = (len + std::min(std::max<size_t>(threads, 1), len) - 1) / std::min(std::max<size_t>(threads, 1), len);
    auto run = [&](size_t start, size_t n) {
        for (size_t e = 0; e < n; ++e) {
            size_t i = start + e;
            acc[i] = dot_portable(&x[(i / out) * k], &w[(i % out) * k], k);
        }
    };
    if (chunk == len) {
        run(0, len);
        return acc;
    }
    std::vector<std::thread> ts;
    for (size_t start = chunk; start < len; start += chunk) ts.emplace_back(run, start, std::min(chunk, len - start));
    run(0, std::min(chunk, len));
    for (auto& t : ts) t.join();
    return acc;
}

// layers.rs:121-136 — add: two activations at a common scale, i64 sum, global requant.
static IntTensor add(const IntTensor& a, const IntTensor& b) {
    if (a.len() != b.len()) std::abort();
    Scale common = a.scale.ge(b.scale) ? a.scale : b.scale;
    if (common.mant == 0) return zeros(a.len(), a.shape);
    Scale cinv = common.recip();
    Scale fa = a.scale.mul(cinv), fb = b.scale.mul(cinv);
    std::vector<int64_t> sum(a.len());
    for (size_t i = 0; i < a.len(); ++i) sum[i] = fa.apply(a.data[i]) + fb.apply(b.data[i]);
    int64_t gmax = 0;
    for (int64_t z : sum) gmax = std::max<int64_t>(gmax, std::llabs(z));
    if (gmax == 0) return zeros(a.len(), a.shape);
    IntTensor o{std::vector<int32_t>(a.len()), a.shape, Scale::from_ratio((u128)gmax, (u128)ACT_LEVELS).mul(common)};
    for (size_t i = 0; i < a.len(); ++i) o.data[i] = requant_dyn(sum[i], ACT_LEVELS, gmax);
    return o;
}

// layers.rs:211-328 — QuantLinear.
// crates/01-engine/kt-core/src/layers.rs:352-449 — RmsNorm: per row C_r = x.scale·rsqrt(mean(x²)+eps)·w_scale and
// p = x_i·wcode_i (integer); rows to the common (last largest) C, then one dynamic requant of the whole tensor.
struct RmsNorm {
    size_t dim = 0;
    std::vector<int32_t> wcodes;
    Scale w_scale, eps_scale;

    RmsNorm(const float* weight, size_t dim_, double eps) : dim(dim_) {
        double peak = 0.0;
        for (size_t i = 0; i < dim; ++i) peak = std::max(peak, std::fabs((double)weight[i]));
        wcodes.assign(dim, 0);
        if (peak == 0.0) {
            w_scale = Scale::zero();
        } else {
            const double step = peak / (double)WLEVELS;
            w_scale = Scale::from_f64(step);
            for (size_t i = 0; i < dim; ++i) {
                int64_t c = (int64_t)std::round((double)weight[i] / step);
                wcodes[i] = (int32_t)std::max<int64_t>(-WLEVELS, std::min<int64_t>(WLEVELS, c));
            }
        }
        eps_scale = Scale::from_f64(eps);
    }

    IntTensor forward_int(const IntTensor& x) const {
        const size_t rows = x.data.size() / dim;
        std::vector<int64_t> p(x.data.size());
        std::vector<Scale> c(rows);
        for (size_t r = 0; r < rows; ++r) {
            const int32_t* xr = x.data.data() + r * dim;
            i128 ss = 0;
            for (size_t i = 0; i < dim; ++i) ss += (i128)xr[i] * (i128)xr[i];
            const Scale mean_sq = Scale::from_ratio((u128)ss, (u128)dim).mul(x.scale).mul(x.scale);
            const Scale denom = mean_sq.add(eps_scale);
            const Scale inv = denom.mant == 0 ? Scale::zero() : denom.rsqrt();
            c[r] = x.scale.mul(inv).mul(w_scale);
            for (size_t i = 0; i < dim; ++i) p[r * dim + i] = (int64_t)xr[i] * (int64_t)wcodes[i];
        }
        Scale common = Scale::zero();
        for (size_t r = 0; r < rows; ++r)
            if (c[r].ge(common)) common = c[r];
        if (common.mant == 0) return zeros(x.data.size(), x.shape);
        const Scale cinv = common.recip();
        std::vector<int64_t> v(x.data.size());
        int64_t gmax = 0;
        for (size_t r = 0; r < rows; ++r) {
            const Scale f = c[r].mul(cinv);
            for (size_t i = 0; i < dim; ++i) {
                v[r * dim + i] = f.apply(p[r * dim + i]);
                gmax = std::max(gmax, v[r * dim + i] < 0 ? -v[r * dim + i] : v[r * dim + i]);
            }
        }
        if (gmax == 0) return zeros(x.data.size(), x.shape);
        IntTensor out{std::vector<int32_t>(x.data.size()), x.shape,
                      Scale::from_ratio((u128)gmax, (u128)ACT_LEVELS).mul(common)};
        for (size_t i = 0; i < v.size(); ++i) out.data[i] = requant_dyn(v[i], ACT_LEVELS, gmax);
        return out;
    }
};

struct QuantLinear {
    size_t out_features = 0, in_features = 0;
    std::vector<int32_t> w_codes;
    Scale w_scale = Scale::zero();
    bool has_bias = false;
    std::vector<int64_t> bias_codes;
    Scale bias_scale = Scale::zero();

    // layers.rs:225-244 — per-tensor b=12 weight quantiser (f64, offline).
    static QuantLinear from_weights(const float* w, size_t out_features, size_t in_features) {
        QuantLinear q;
        q.out_features = out_features;
        q.in_features = in_features;
        size_t n = out_features * in_features;
        double peak = 0.0;
        for (size_t i = 0; i < n; ++i) peak = std::fmax(peak, std::fabs((double)w[i]));
        q.w_codes.assign(n, 0);
        if (peak == 0.0) {
            q.w_scale = Scale::zero();
        } else {
            double step = peak / (double)WLEVELS;
            for (size_t i = 0; i < n; ++i) {
                int64_t c = (int64_t)std::round((double)w[i] / step);
                c = std::min<int64_t>(std::max<int64_t>(c, -WLEVELS), WLEVELS);
                q.w_codes[i] = (int32_t)c;
            }
            q.w_scale = Scale::from_f64(step);
        }
        return q;
    }

    // layers.rs:246-257 — with_bias: bias coded at ACT_LEVELS against its own peak.
    void with_bias(const float* b) {
        if (!b) return;
        double bmax = 0.0;
        for (size_t i = 0; i < out_features; ++i) bmax = std::fmax(bmax, std::fabs((double)b[i]));
        if (bmax > 0.0) {
            double step = bmax / (double)ACT_LEVELS;
            bias_codes.resize(out_features);
            for (size_t i = 0; i < out_features; ++i) bias_codes[i] = (int64_t)std::round((double)b[i] / step);
            bias_scale = Scale::from_f64(step);
            has_bias = true;
        }
    }

    // layers.rs:275-328 — forward_int.
    IntTensor forward_int(const IntTensor& x) const {
        if (x.len() % in_features != 0) std::abort();
        size_t rows = x.len() / in_features;
        std::vector<size_t> shape = rows == 1 ? std::vector<size_t>{out_features} : std::vector<size_t>{rows, out_features};
        int64_t xmax = x.max_abs_data();
        if (xmax == 0) {
            if (has_bias) {
                IntTensor t{std::vector<int32_t>(), shape, bias_scale};
                t.data.reserve(rows * out_features);
                for (size_t r = 0; r < rows; ++r)
                    for (int64_t c : bias_codes) t.data.push_back((int32_t)c);
                return t;
            }
            return zeros(rows * out_features, shape);
        }
        std::vector<int32_t> qx = quant_to(x.data, xmax);
        Scale s_qx = Scale::from_ratio((u128)xmax, (u128)WLEVELS).mul(x.scale);
        Scale c = s_qx.mul(w_scale);
        if (c.mant == 0) return zeros(rows * out_features, shape);
        std::vector<int64_t> bias_in_c;
        if (has_bias) {
            Scale f = bias_scale.mul(c.recip());
            bias_in_c.resize(out_features);
            for (size_t o = 0; o < out_features; ++o) bias_in_c[o] = f.apply(bias_codes[o]);
        }
        std::vector<int64_t> combined = linear_cpu(qx.data(), w_codes.data(), rows, out_features, in_features);
        if (has_bias)
            for (size_t r = 0; r < rows; ++r)
                for (size_t o = 0; o < out_features; ++o) combined[r * out_features + o] += bias_in_c[o];
        int64_t ymax = 0;
        for (int64_t v : combined) ymax = std::max<int64_t>(ymax, std::llabs(v));
        if (ymax == 0) return zeros(rows * out_features, shape);
        IntTensor o{std::vector<int32_t>(combined.size()), shape,
                    Scale::from_ratio((u128)ymax, (u128)ACT_LEVELS).mul(c)};
        for (size_t i = 0; i < combined.size(); ++i) o.data[i] = requant_dyn(combined[i], ACT_LEVELS, ymax);
        return o;
    }
};

// layers.rs:581-640 — SwiGluMlp.
struct SwiGluMlp {
    QuantLinear gate, up, down;
    CodeLut silu;
    SwiGluMlp(QuantLinear g, QuantLinear u, QuantLinear d)
        : gate(std::move(g)), up(std::move(u)), down(std::move(d)), silu(silu_table()) {}

    IntTensor forward_int(const IntTensor& x) const {
        IntTensor g = gate.forward_int(x);
        IntTensor u = up.forward_int(x);
        size_t hidden = gate.out_features;
        size_t rows = g.len() / hidden;
        Scale id_factor = g.scale.mul(silu.code_scale.recip());
        std::vector<int64_t> h(g.len(), 0);
        for (size_t k = 0; k < g.len(); ++k) {
            int64_t gd = g.data[k];
            int64_t idx = silu.index(gd, g.scale);
            int64_t silu_code;
            if (idx < 0)
                silu_code = 0;
            else if (idx >= (int64_t)silu.n)
                silu_code = id_factor.apply(gd);
            else
                silu_code = silu.code_at(idx);
            h[k] = silu_code * (int64_t)u.data[k];
        }
        Scale h_scale = silu.code_scale.mul(u.scale);
        int64_t hmax = 0;
        for (int64_t z : h) hmax = std::max<int64_t>(hmax, std::llabs(z));
        std::vector<size_t> shape = rows == 1 ? std::vector<size_t>{hidden} : std::vector<size_t>{rows, hidden};
        IntTensor hint;
        if (hmax == 0) {
            hint = zeros(g.len(), shape);
        } else {
            hint = IntTensor{std::vector<int32_t>(h.size()), shape,
                             Scale::from_ratio((u128)hmax, (u128)ACT_LEVELS).mul(h_scale)};
            for (size_t i = 0; i < h.size(); ++i) hint.data[i] = requant_dyn(h[i], ACT_LEVELS, hmax);
        }
        return down.forward_int(hint);
    }
};

// router.rs:29-79 — the sigmoid score with its coded selection bias.
struct SigmoidScore {
    CodeLut table;
    std::vector<int64_t> bias;
    explicit SigmoidScore(const float* b, size_t n) : table(sigmoid_table()) {
        double k = (double)(uint64_t(1) << ROUTER_CODE_BITS);
        bias.resize(n);
        for (size_t i = 0; i < n; ++i) bias[i] = (int64_t)std::round((double)b[i] * k);
    }
    std::vector<int64_t> codes(const IntTensor& logits) const {
        std::vector<int64_t> c(logits.len());
        for (size_t j = 0; j < logits.len(); ++j) c[j] = table.code_at(table.index(logits.data[j], logits.scale));
        return c;
    }
    std::vector<int64_t> choice(const std::vector<int64_t>& codes) const {
        std::vector<int64_t> c(codes.size());
        for (size_t j = 0; j < codes.size(); ++j) c[j] = codes[j] + bias[j];
        return c;
    }
};

// layers.rs:812-821
struct MoeRoute {
    std::vector<size_t> experts;
    std::vector<int64_t> ec;
    int64_t sumc = 0;
};

// layers.rs:800-805 — top-k: descending, ties to the lower index.
template <class T>
static std::vector<size_t> topk(const std::vector<T>& scores, size_t k) {
    std::vector<size_t> idx(scores.size());
    for (size_t i = 0; i < idx.size(); ++i) idx[i] = i;
    std::stable_sort(idx.begin(), idx.end(), [&](size_t a, size_t b) {
        if (scores[b] < scores[a]) return true;
        if (scores[a] < scores[b]) return false;
        return a < b;
    });
    idx.resize(k);
    return idx;
}

// layers.rs:661-1106 — MoeMlp.
struct MoeMlp {
    QuantLinear router;
    std::vector<SwiGluMlp> experts;
    size_t top_k = 1;
    bool norm_topk_prob = false;
    CodeLut exp_code = exp_table();
    std::unique_ptr<SigmoidScore> sigmoid;
    std::unique_ptr<SwiGluMlp> shared;
    // Extension (the reference refuses it, crates/03-models/kt-model-moe/src/lib.rs:152-154, :276-288): Qwen2-MoE's
    // sigmoid-gated shared expert, shared_expert_gate [1, dim]. Off unless set.
    std::unique_ptr<QuantLinear> shared_gate;

    size_t dim() const { return router.in_features; }

    // layers.rs:826-851 (softmax) and :856-862 (sigmoid)
    MoeRoute route(const IntTensor& x) const {
        IntTensor logits = router.forward_int(x);
        MoeRoute r;
        if (sigmoid) {
            std::vector<int64_t> codes = sigmoid->codes(logits);
            r.experts = topk(sigmoid->choice(codes), top_k);
            for (size_t ex : r.experts) r.ec.push_back(codes[ex]);
            if (norm_topk_prob) {
                r.sumc = 0;
                for (int64_t c : r.ec) r.sumc += c;
            } else {
                r.sumc = int64_t(1) << ROUTER_CODE_BITS;
            }
            return r;
        }
        size_t e = logits.len();
        int32_t lmax = INT32_MIN;
        for (int32_t l : logits.data) lmax = std::max(lmax, l);
        std::vector<int64_t> ecs(e, 0);
        int64_t sum_all = 0;
        for (size_t j = 0; j < e; ++j) {
            int64_t idx = exp_code.index((int64_t)(logits.data[j] - lmax), logits.scale);
            ecs[j] = idx < 0 ? 0 : exp_code.code_at(idx);
            sum_all += ecs[j];
        }
        r.experts = topk(logits.data, top_k);
        if (norm_topk_prob) {
            r.sumc = 0;
            for (size_t ex : r.experts) r.sumc += ecs[ex];
        } else {
            r.sumc = sum_all;
        }
        for (size_t ex : r.experts) r.ec.push_back(ecs[ex]);
        return r;
    }

    // layers.rs:893-923 — combine.
    static IntTensor combine(const MoeRoute& route, const std::vector<IntTensor>& ys, size_t dim) {
        if (route.sumc <= 0 || ys.empty()) return zeros(dim, {dim});
        size_t out_dim = ys[0].len();
        Scale common = Scale::zero();
        for (const IntTensor& y : ys) common = y.scale.ge(common) ? y.scale : common;
        if (common.mant == 0) return zeros(out_dim, {out_dim});
        Scale cinv = common.recip();
        std::vector<int64_t> acc(out_dim, 0);
        for (size_t i = 0; i < ys.size(); ++i) {
            Scale f = ys[i].scale.mul(cinv);
            int64_t w = route.ec[i];
            for (size_t d = 0; d < out_dim; ++d) acc[d] += w * f.apply(ys[i].data[d]);
        }
        int64_t gmax = 0;
        for (int64_t z : acc) gmax = std::max<int64_t>(gmax, std::llabs(z));
        if (gmax == 0) return zeros(out_dim, {out_dim});
        Scale out_scale = Scale::from_ratio((u128)gmax, (u128)ACT_LEVELS)
                              .mul(common)
                              .mul(Scale::from_ratio(1, (u128)(uint64_t)route.sumc));
        IntTensor o{std::vector<int32_t>(out_dim), {out_dim}, out_scale};
        for (size_t d = 0; d < out_dim; ++d) o.data[d] = requant_dyn(acc[d], ACT_LEVELS, gmax);
        return o;
    }

    // layers.rs:866-886 — merge_rows (identical to the inline merge of forward_routed, :1001-1019).
    static IntTensor merge_rows(const std::vector<IntTensor>& outs, size_t out_dim) {
        size_t rows = outs.size();
        Scale common = Scale::zero();
        for (const IntTensor& o : outs) common = o.scale.ge(common) ? o.scale : common;
        if (common.mant == 0) return zeros(rows * out_dim, {rows, out_dim});
        Scale cinv = common.recip();
        std::vector<int64_t> a(rows * out_dim);
        for (size_t t = 0; t < rows; ++t) {
            Scale f = outs[t].scale.mul(cinv);
            for (size_t d = 0; d < out_dim; ++d) a[t * out_dim + d] = f.apply(outs[t].data[d]);
        }
        int64_t gmax = 0;
        for (int64_t z : a) gmax = std::max<int64_t>(gmax, std::llabs(z));
        if (gmax == 0) return zeros(rows * out_dim, {rows, out_dim});
        IntTensor o{std::vector<int32_t>(a.size()), {rows, out_dim}, Scale::from_ratio((u128)gmax, (u128)ACT_LEVELS).mul(common)};
        for (size_t i = 0; i < a.size(); ++i) o.data[i] = requant_dyn(a[i], ACT_LEVELS, gmax);
        return o;
    }

    // layers.rs:928-937
    IntTensor forward_one_int(const IntTensor& x) const {
        size_t d = dim();
        MoeRoute r = route(x);
        if (r.sumc <= 0) return zeros(d, {d});
        std::vector<IntTensor> ys;
        for (size_t ex : r.experts) ys.push_back(experts[ex].forward_int(x));
        return combine(r, ys, d);
    }

    static IntTensor row_of(const IntTensor& x, size_t t, size_t d) {
        return IntTensor{std::vector<int32_t>(x.data.begin() + t * d, x.data.begin() + (t + 1) * d), {d}, x.scale};
    }

    // layers.rs:988-1020
    IntTensor forward_routed(const IntTensor& x) const {
        size_t d = dim();
        if (x.len() % d != 0) std::abort();
        size_t rows = x.len() / d;
        if (rows <= 1) return forward_one_int(x);
        std::vector<IntTensor> outs;
        outs.reserve(rows);
        for (size_t t = 0; t < rows; ++t) outs.push_back(forward_one_int(row_of(x, t, d)));
        return merge_rows(outs, outs[0].len());
    }

    // layers.rs:758-780
    IntTensor add_shared(IntTensor routed, const IntTensor& x) const {
        if (!shared) return routed;
        IntTensor y = shared->forward_int(x);
        if (shared_gate) y = gate_shared(y, x);
        return add(routed, y);
    }

    // The gated shared expert (an extension defined by this build in the reference's own terms; parity with the
    // reference is unpinned because the reference has no such path). The gate is a QuantLinear [1, dim] on the whole
    // input (layers.rs:275-328: tensor-global xmax and ymax), its logit per token goes through the sigmoid CodeLut
    // of the GLM router (router.rs:37-51, code_at(index(logit, scale)), codes in units of 2^-20), and each token's
    // shared output row is multiplied by its code and requantised over the whole tensor, as SwiGLU forms and
    // requantises h (layers.rs:618-638): v = code_t·y[t, j] (i64), gmax = max |v|, data = requant_dyn(v, L, gmax),
    // scale = from_ratio(gmax, L)·y.scale·code_scale. The result is then added to the routed output with add.
    IntTensor gate_shared(const IntTensor& y, const IntTensor& x) const {
        const IntTensor logit = shared_gate->forward_int(x);
        const size_t rows = logit.len();
        const size_t d = rows ? y.len() / rows : 0;
        static const CodeLut sig = sigmoid_table();
        std::vector<int64_t> v(y.len(), 0);
        int64_t gmax = 0;
        for (size_t t = 0; t < rows; ++t) {
            const int64_t c = sig.code_at(sig.index(logit.data[t], logit.scale));
            for (size_t j = 0; j < d; ++j) {
                v[t * d + j] = c * (int64_t)y.data[t * d + j];
                gmax = std::max<int64_t>(gmax, std::llabs(v[t * d + j]));
            }
        }
        if (gmax == 0) return zeros(y.len(), y.shape);
        IntTensor o{std::vector<int32_t>(y.len()), y.shape,
                    Scale::from_ratio((u128)gmax, (u128)ACT_LEVELS).mul(y.scale).mul(sig.code_scale)};
        for (size_t i = 0; i < v.size(); ++i) o.data[i] = requant_dyn(v[i], ACT_LEVELS, gmax);
        return o;
    }

    // layers.rs:1070-1073
    IntTensor forward_int(const IntTensor& x) const { return add_shared(forward_routed(x), x); }

    // layers.rs:945-984 — the expert-parallel seam, with the experts supplied by a callback.
    IntTensor forward_int_with_experts(
        const IntTensor& x,
        const std::function<std::vector<IntTensor>(const std::vector<size_t>&, const IntTensor&)>& experts_fn) const {
        size_t d = dim();
        size_t rows = x.len() / d;
        auto row_out = [&](const IntTensor& row) -> IntTensor {
            MoeRoute r = route(row);
            if (r.sumc <= 0) return zeros(d, {d});
            std::vector<IntTensor> ys = experts_fn(r.experts, row);
            return combine(r, ys, d);
        };
        IntTensor routed;
        if (rows <= 1) {
            routed = row_out(x);
        } else {
            std::vector<IntTensor> outs;
            for (size_t t = 0; t < rows; ++t) outs.push_back(row_out(row_of(x, t, d)));
            routed = merge_rows(outs, outs[0].len());
        }
        return add_shared(routed, x);
    }
};

}  // namespace ko

// ─────────────── C API for the test harness (ctypes) ───────────────

using namespace ko;

static inline ko_scale to_c(Scale s) { return ko_scale{s.mant, s.shift}; }
static inline Scale from_c(ko_scale s) { return Scale{s.mant, s.shift}; }
static inline u128 mk128(uint64_t hi, uint64_t lo) { return ((u128)hi << 64) | lo; }

extern "C" {

int64_t ko_wlevels(void) { return WLEVELS; }
int64_t ko_act_levels(void) { return ACT_LEVELS; }
void ko_set_max_threads(size_t n) { g_max_threads = n; }
size_t ko_plan_threads(size_t elems, size_t work) { return plan_threads(elems, work); }

void ko_frexp(double x, double* m, int32_t* e) { frexp_bits(x, m, e); }
int64_t ko_requant(int64_t a, int64_t m, int32_t s) { return requant(a, m, s); }
int32_t ko_requant_dyn(int64_t v, int64_t num_level, int64_t den) { return requant_dyn(v, num_level, den); }
ko_scale ko_from_ratio(uint64_t num_hi, uint64_t num_lo, uint64_t den_hi, uint64_t den_lo) {
    return to_c(Scale::from_ratio(mk128(num_hi, num_lo), mk128(den_hi, den_lo)));
}
ko_scale ko_from_f64(double x) { return to_c(Scale::from_f64(x)); }
int ko_ge(ko_scale a, ko_scale b) { return from_c(a).ge(from_c(b)) ? 1 : 0; }
ko_scale ko_mul(ko_scale a, ko_scale b) { return to_c(from_c(a).mul(from_c(b))); }
int64_t ko_apply(ko_scale s, int64_t v) { return from_c(s).apply(v); }
ko_scale ko_recip(ko_scale s) { return to_c(from_c(s).recip()); }
void ko_isqrt_u128(uint64_t hi, uint64_t lo, uint64_t* out_hi, uint64_t* out_lo) {
    u128 r = isqrt_u128(mk128(hi, lo));
    *out_hi = (uint64_t)(r >> 64);
    *out_lo = (uint64_t)r;
}
void ko_quant_to(const int32_t* data, size_t n, int64_t xmax, int32_t* out) {
    std::vector<int32_t> v(data, data + n);
    std::vector<int32_t> q = quant_to(v, xmax);
    std::memcpy(out, q.data(), n * 4);
}

// Tables: kind 0 = router exp, 1 = SiLU, 2 = sigmoid. Writes the n codes and the index constants.
int ko_table(int kind, int64_t* codes, size_t cap, ko_scale* inv_step_scale, int64_t* lo_index, ko_scale* code_scale) {
    CodeLut l = kind == 0 ? exp_table() : kind == 1 ? silu_table() : sigmoid_table();
    if (cap < l.n) return -1;
    std::memcpy(codes, l.codes.data(), l.n * 8);
    *inv_step_scale = to_c(l.inv_step_scale);
    *lo_index = l.lo_index;
    *code_scale = to_c(l.code_scale);
    return (int)l.n;
}
int64_t ko_table_index(int kind, int64_t data, ko_scale s) {
    static CodeLut t0 = exp_table(), t1 = silu_table(), t2 = sigmoid_table();
    const CodeLut& l = kind == 0 ? t0 : kind == 1 ? t1 : t2;
    return l.index(data, from_c(s));
}

void ko_quantize_weights(const float* w, size_t n, int32_t* codes, ko_scale* scale) {
    QuantLinear q = QuantLinear::from_weights(w, 1, n);
    std::memcpy(codes, q.w_codes.data(), n * 4);
    *scale = to_c(q.w_scale);
}
int ko_quantize_bias(const float* b, size_t n, int64_t* codes, ko_scale* scale) {
    QuantLinear q;
    q.out_features = n;
    q.in_features = 1;
    q.with_bias(b);
    if (!q.has_bias) return 0;
    std::memcpy(codes, q.bias_codes.data(), n * 8);
    *scale = to_c(q.bias_scale);
    return 1;
}
void ko_from_reals_f32(const float* v, size_t n, int64_t levels, int32_t* data, ko_scale* scale) {
    std::vector<double> r(v, v + n);
    IntTensor t = from_reals(r.data(), n, {n}, levels);
    std::memcpy(data, t.data.data(), n * 4);
    *scale = to_c(t.scale);
}

// LinearBackend::linear through the Portable CPU kernel (backend.rs:133-152).
void ko_linear(const int32_t* x, const int32_t* w, size_t rows, size_t out, size_t k, int64_t* y) {
    std::vector<int64_t> r = linear_cpu(x, w, rows, out, k);
    if (!r.empty()) std::memcpy(y, r.data(), r.size() * 8);
}

// ── the digit algorithm as a second, independent GEMM (kt-cuda's host executor) ──
// kt-cuda/src/digits.rs:40-52 (split): a code |v| <= WLEVELS is three balanced base-81 digits, low digit first, each
// the remainder of (r + 40) mod 81 shifted back by 40, the rest carried exactly. Returns false beyond ±WLEVELS.
static bool split_digits(int32_t v, int8_t d[3]) {
    if (v > (int32_t)WLEVELS || v < -(int32_t)WLEVELS) return false;
    int32_t r = v;
    for (int i = 0; i < 3; ++i) {
        int32_t m = (r + 40) % 81;
        if (m < 0) m += 81;  // rem_euclid
        d[i] = (int8_t)(m - 40);
        r = (r - (m - 40)) / 81;
    }
    return r == 0;
}

// kt-cuda/src/host.rs:47-76 (dot_tiles) without the tile layout: nine int32 sums s[i][j] = Σ x_i·w_j that wrap as the
// hardware's accumulators do, added into i64 with weight 81^(i+j) every `flush` terms (digits.rs:16-19: KT_FLUSH tiles
// of 16 terms), so the result equals the plain i64 dot product exactly when the flush bound holds.
void ko_linear_digits(const int32_t* x, const int32_t* w, size_t rows, size_t out, size_t k, size_t flush, int64_t* y) {
    static const int64_t SCALE[5] = {1, 81, 81 * 81, 81 * 81 * 81, 81LL * 81 * 81 * 81};
    std::vector<int8_t> xd(rows * k * 3), wd(out * k * 3);
    for (size_t i = 0; i < rows * k; ++i) split_digits(x[i], &xd[i * 3]);
    for (size_t i = 0; i < out * k; ++i) split_digits(w[i], &wd[i * 3]);
    if (flush == 0) flush = k ? k : 1;
    for (size_t r = 0; r < rows; ++r)
        for (size_t o = 0; o < out; ++o) {
            int64_t acc = 0;
            for (size_t k0 = 0; k0 < k; k0 += flush) {
                const size_t k1 = std::min(k, k0 + flush);
                uint32_t s[3][3] = {};
                for (size_t t = k0; t < k1; ++t) {
                    const int8_t* a = &xd[(r * k + t) * 3];
                    const int8_t* b = &wd[(o * k + t) * 3];
                    for (int i = 0; i < 3; ++i)
                        for (int j = 0; j < 3; ++j) s[i][j] += (uint32_t)(int32_t)(a[i] * b[j]);
                }
                for (int i = 0; i < 3; ++i)
                    for (int j = 0; j < 3; ++j) acc += SCALE[i + j] * (int64_t)(int32_t)s[i][j];
            }
            y[r * out + o] = acc;
        }
}

// The reduced-plane decomposition of the library's small-code GEMM (this build's, not the reference's): x in
// [-127, 127] as one raw int8 plane, w in [-3280, 3280] as its two low balanced digits (the third is zero there);
// two wrapping int32 sums s_j = Σ x·w_j per flush of `flush` terms, recombined as s_0 + 81·s_1.
void ko_linear_small(const int32_t* x, const int32_t* w, size_t rows, size_t out, size_t k, size_t flush, int64_t* y) {
    std::vector<int8_t> wd(out * k * 3);
    for (size_t i = 0; i < out * k; ++i) split_digits(w[i], &wd[i * 3]);
    if (flush == 0) flush = k ? k : 1;
    for (size_t r = 0; r < rows; ++r)
        for (size_t o = 0; o < out; ++o) {
            int64_t acc = 0;
            for (size_t k0 = 0; k0 < k; k0 += flush) {
                const size_t k1 = std::min(k, k0 + flush);
                uint32_t s0 = 0, s1 = 0;
                for (size_t t = k0; t < k1; ++t) {
                    const int32_t a = x[r * k + t];
                    s0 += (uint32_t)(a * wd[(o * k + t) * 3]);
                    s1 += (uint32_t)(a * wd[(o * k + t) * 3 + 1]);
                }
                acc += (int64_t)(int32_t)s0 + 81 * (int64_t)(int32_t)s1;
            }
            y[r * out + o] = acc;
        }
}

// The equality-gate corpus (crates/02-runtime/kt-runtime/src/gate.rs:26-56). ko_corpus_case(i, ...) returns the
// shape of case i (or -1 past the end); with non-null buffers it also writes its operands.
int ko_corpus_case(int i, size_t* rows, size_t* out, size_t* k, int32_t* x, int32_t* w) {
    const int32_t lv = (int32_t)WLEVELS;
    struct Shape {
        size_t r, o, k;
    };
    static const Shape shapes[6] = {{1, 1, 1}, {3, 5, 7}, {2, 17, 33}, {4, 64, 1023}, {1, 9, 4099}, {8, 512, 2048}};
    if (i < 0 || i > 7) return -1;
    if (i < 6) {
        *rows = shapes[i].r;
        *out = shapes[i].o;
        *k = shapes[i].k;
        if (!x) return 0;
        // The LCG stream runs through the cases in order: regenerate from the start.
        uint64_t s = 0x50320b00ULL;
        auto uniform = [&](int32_t* dst, size_t n) {
            for (size_t j = 0; j < n; ++j) {
                s = s * 6364136223846793005ULL + 1442695040888963407ULL;
                int32_t v = (int32_t)((s >> 33) % (uint64_t)(2 * WLEVELS + 1)) - lv;
                if (dst) dst[j] = v;
            }
        };
        for (int c = 0; c <= i; ++c) {
            size_t nx = shapes[c].r * shapes[c].k, nw = shapes[c].o * shapes[c].k;
            if (c < i) {
                uniform(nullptr, nx);
                uniform(nullptr, nw);
            } else {
                uniform(x, nx);
                uniform(w, nw);
            }
        }
        return 0;
    }
    if (i == 6) {  // extremes ±WLEVELS
        *rows = 2;
        *out = 3;
        *k = 1027;
        if (!x) return 0;
        for (size_t j = 0; j < 2 * 1027; ++j) x[j] = (j % 3 == 0) ? -lv : lv;
        for (size_t j = 0; j < 3 * 1027; ++j) w[j] = (j % 2 == 0) ? lv : -lv;
        return 0;
    }
    *rows = 4;  // all +WLEVELS
    *out = 4;
    *k = 2048;
    if (!x) return 0;
    for (size_t j = 0; j < 4 * 2048; ++j) x[j] = lv, w[j] = lv;
    return 0;
}

// ── The MoE layer ──
// Built from f32 weights exactly as the reference builds one (QuantLinear::from_weights on each matrix). The expert
// weights are laid out per expert as gate [hidden×dim], up [hidden×dim], down [dim×hidden], back to back.
void* ko_moe_new(size_t dim, size_t n_experts, size_t hidden, size_t top_k, const float* router_w,
                 const float* router_bias, const float* expert_w, int norm_topk, const float* sigmoid_bias,
                 size_t shared_hidden, const float* shared_w) {
    MoeMlp* m = new MoeMlp();
    m->router = QuantLinear::from_weights(router_w, n_experts, dim);
    m->router.with_bias(router_bias);
    size_t per = 3 * hidden * dim;
    for (size_t e = 0; e < n_experts; ++e) {
        const float* base = expert_w + e * per;
        m->experts.emplace_back(QuantLinear::from_weights(base, hidden, dim),
                                QuantLinear::from_weights(base + hidden * dim, hidden, dim),
                                QuantLinear::from_weights(base + 2 * hidden * dim, dim, hidden));
    }
    m->top_k = top_k;
    m->norm_topk_prob = norm_topk != 0;
    if (sigmoid_bias) m->sigmoid.reset(new SigmoidScore(sigmoid_bias, n_experts));
    if (shared_hidden > 0 && shared_w) {
        m->shared.reset(new SwiGluMlp(QuantLinear::from_weights(shared_w, shared_hidden, dim),
                                      QuantLinear::from_weights(shared_w + shared_hidden * dim, shared_hidden, dim),
                                      QuantLinear::from_weights(shared_w + 2 * shared_hidden * dim, dim, shared_hidden)));
    }
    return m;
}

void ko_moe_free(void* p) { delete (MoeMlp*)p; }

// The extension's shared-expert gate (Qwen2-MoE shared_expert_gate, [1, dim] f32), quantised by QuantLinear::
// from_weights (layers.rs:225-244); a null `w` removes it. Only with a shared expert.
void ko_moe_set_shared_gate(void* p, const float* w) {
    MoeMlp* m = (MoeMlp*)p;
    if (!w) {
        m->shared_gate.reset();
        return;
    }
    m->shared_gate.reset(new QuantLinear(QuantLinear::from_weights(w, 1, m->dim())));
}

// Which = 0 router, 1 gate, 2 up, 3 down (expert e), 4/5/6 shared gate/up/down, 7 the shared-expert gate [1, dim].
// Copies the codes, returns the scale.
ko_scale ko_moe_weights(void* p, int which, size_t e, int32_t* codes) {
    MoeMlp* m = (MoeMlp*)p;
    const QuantLinear* q = which == 0   ? &m->router
                           : which == 1 ? &m->experts[e].gate
                           : which == 2 ? &m->experts[e].up
                           : which == 3 ? &m->experts[e].down
                           : which == 4 ? &m->shared->gate
                           : which == 5 ? &m->shared->up
                           : which == 6 ? &m->shared->down
                                        : m->shared_gate.get();
    if (codes) std::memcpy(codes, q->w_codes.data(), q->w_codes.size() * 4);
    return to_c(q->w_scale);
}
int ko_moe_router_bias(void* p, int64_t* codes, ko_scale* scale) {
    MoeMlp* m = (MoeMlp*)p;
    if (!m->router.has_bias) return 0;
    std::memcpy(codes, m->router.bias_codes.data(), m->router.bias_codes.size() * 8);
    *scale = to_c(m->router.bias_scale);
    return 1;
}
int ko_moe_sigmoid_bias(void* p, int64_t* codes) {
    MoeMlp* m = (MoeMlp*)p;
    if (!m->sigmoid) return 0;
    std::memcpy(codes, m->sigmoid->bias.data(), m->sigmoid->bias.size() * 8);
    return 1;
}

// Module::forward_int of the layer (layers.rs:1070-1073): x is rows×dim.
void ko_moe_forward(void* p, const int32_t* x, size_t rows, ko_scale xs, int32_t* y, ko_scale* ys) {
    MoeMlp* m = (MoeMlp*)p;
    size_t d = m->dim();
    IntTensor t{std::vector<int32_t>(x, x + rows * d), rows == 1 ? std::vector<size_t>{d} : std::vector<size_t>{rows, d},
                from_c(xs)};
    IntTensor o = m->forward_int(t);
    std::memcpy(y, o.data.data(), o.data.size() * 4);
    *ys = to_c(o.scale);
}

// The same Module::forward_int with the per-token work (layers.rs:997-1000: route, experts, combine of one row,
// forward_one_int) spread over `threads` host threads, each token on one thread, then the merge and the shared expert
// exactly as forward_int does them. Every per-token output depends on that token's row alone, so the result is the
// serial one bit for bit (checked against ko_moe_forward in the tests); it exists so that the golden outputs of the
// full-size workloads take minutes rather than an hour.
void ko_moe_forward_par(void* p, const int32_t* x, size_t rows, ko_scale xs, int32_t* y, ko_scale* ys,
                        size_t threads) {
    MoeMlp* m = (MoeMlp*)p;
    size_t d = m->dim();
    IntTensor t{std::vector<int32_t>(x, x + rows * d), rows == 1 ? std::vector<size_t>{d} : std::vector<size_t>{rows, d},
                from_c(xs)};
    IntTensor routed;
    if (rows <= 1) {
        routed = m->forward_one_int(t);
    } else {
        std::vector<IntTensor> outs(rows);
        std::atomic<size_t> next{0};
        auto work = [&]() {
            tl_serial = true;
            for (size_t r; (r = next.fetch_add(1)) < rows;) outs[r] = m->forward_one_int(MoeMlp::row_of(t, r, d));
            tl_serial = false;
        };
        if (threads == 0) threads = std::max<unsigned>(1, std::thread::hardware_concurrency());
        std::vector<std::thread> ts;
        for (size_t i = 1; i < threads; ++i) ts.emplace_back(work);
        work();
        for (auto& th : ts) th.join();
        routed = MoeMlp::merge_rows(outs, outs[0].len());
    }
    IntTensor o = m->add_shared(std::move(routed), t);
    std::memcpy(y, o.data.data(), o.data.size() * 4);
    *ys = to_c(o.scale);
}

// The build-defined synthetic generator (the reference has no normal RNG), restated here so that the checker's inputs
// never come from the product library: element i of stream `seed` takes two uniforms from splitmix64 (Steele, Lea
// and Flood, 2014: state seed + (j+1)·0x9E3779B97F4A7C15, then the xor-shift-multiply finaliser) at positions 2i and
// 2i+1, u = (bits >> 11)·2^-53 with u1 moved into (0, 1], then the Box-Muller transform sqrt(-2 ln u1)·cos(2π u2) in
// f64 (host libm), rounded to f32 and multiplied by sigma in f32.
void ko_synth_normal(uint64_t seed, float sigma, uint64_t offset, size_t n, float* out) {
    auto mix = [](uint64_t s, uint64_t j) {
        uint64_t v = s + (j + 1) * 0x9E3779B97F4A7C15ULL;
        v = (v ^ (v >> 30)) * 0xBF58476D1CE4E5B9ULL;
        v = (v ^ (v >> 27)) * 0x94D049BB133111EBULL;
        return v ^ (v >> 31);
    };
    const double inv53 = 1.0 / 9007199254740992.0;
    auto run = [&](size_t lo, size_t hi) {
        for (size_t j = lo; j < hi; ++j) {
            const uint64_t i = offset + j;
            const double u1 = 1.0 - (double)(mix(seed, 2 * i) >> 11) * inv53;
            const double u2 = (double)(mix(seed, 2 * i + 1) >> 11) * inv53;
            const double r = std::sqrt(-2.0 * std::log(u1));
            out[j] = (float)(r * std::cos(6.283185307179586 * u2)) * sigma;
        }
    };
    const size_t nt = n < (size_t(1) << 20) ? 1 : std::max<unsigned>(1, std::thread::hardware_concurrency());
    std::vector<std::thread> ts;
    const size_t chunk = (n + nt - 1) / nt;
    for (size_t s = chunk; s < n; s += chunk) ts.emplace_back(run, s, std::min(n, s + chunk));
    run(0, std::min(n, chunk));
    for (auto& th : ts) th.join();
}

// The portable normal stream this build defines for weights generated on the GPU (the product's synth.cuh): the same
// splitmix64 uniforms as ko_synth_normal, the Box-Muller deviate with a logarithm and a cosine built from IEEE
// add/mul/div/sqrt only, in a fixed order (this file is compiled with -ffp-contract=off), so the GPU's weights can be
// regenerated here bit for bit. ln(u) = e·ln2 + 2·atanh((m-1)/(m+1)) for u = m·2^e, m in [sqrt(1/2), sqrt(2)), the
// atanh series to s^23; cos(2πu) from the quadrant of 4u and the Taylor series of cos and sin on [0, π/4].
static double portable_ln(double u) {
    static const double inv_odd[11] = {0x1.5555555555555p-2, 0x1.999999999999ap-3, 0x1.2492492492492p-3,
                                       0x1.c71c71c71c71cp-4, 0x1.745d1745d1746p-4, 0x1.3b13b13b13b14p-4,
                                       0x1.1111111111111p-4, 0x1.e1e1e1e1e1e1ep-5, 0x1.af286bca1af28p-5,
                                       0x1.8618618618618p-5, 0x1.642c8590b2164p-5};  // 1/3, 1/5, ..., 1/23
    uint64_t bits;
    std::memcpy(&bits, &u, 8);
    int e = (int)((bits >> 52) & 0x7ff) - 1023;
    const uint64_t mb = (bits & ((uint64_t(1) << 52) - 1)) | (uint64_t(1023) << 52);
    double m;
    std::memcpy(&m, &mb, 8);
    if (m > 0x1.6a09e667f3bcdp+0) {
        m = m * 0.5;
        e = e + 1;
    }
    const double s = (m - 1.0) / (m + 1.0), s2 = s * s;
    double p = inv_odd[10];
    for (int k = 9; k >= 0; --k) p = p * s2 + inv_odd[k];
    return (double)e * 0x1.62e42fefa39efp-1 + 2.0 * (s + s * (s2 * p));
}

static double portable_cos_2pi(double u) {
    static const double cos_c[9] = {-0x1.0000000000000p-1, 0x1.5555555555555p-5,  -0x1.6c16c16c16c17p-10,
                                    0x1.a01a01a01a01ap-16, -0x1.27e4fb7789f5cp-22, 0x1.1eed8eff8d898p-29,
                                    -0x1.93974a8c07c9dp-37, 0x1.ae7f3e733b81fp-45, -0x1.6827863b97d97p-53};
    static const double sin_c[9] = {-0x1.5555555555555p-3, 0x1.1111111111111p-7,  -0x1.a01a01a01a01ap-13,
                                    0x1.71de3a556c734p-19, -0x1.ae64567f544e4p-26, 0x1.6124613a86d09p-33,
                                    -0x1.ae7f3e733b81fp-41, 0x1.952c77030ad4ap-49, -0x1.2f49b46814157p-57};
    const double t = u * 4.0;
    const int quadrant = (int)t;
    const double r = t - (double)quadrant;
    const bool first_half = r <= 0.5;
    const double a = (first_half ? r : 1.0 - r) * 0x1.921fb54442d18p+0;
    const double a2 = a * a;
    double c = cos_c[8], sv = sin_c[8];
    for (int k = 7; k >= 0; --k) {
        c = c * a2 + cos_c[k];
        sv = sv * a2 + sin_c[k];
    }
    const double cos_a = 1.0 + a2 * c, sin_a = a + a * (a2 * sv);
    const double cp = first_half ? cos_a : sin_a, sp = first_half ? sin_a : cos_a;
    switch (quadrant) {
        case 0: return cp;
        case 1: return -sp;
        case 2: return -cp;
        default: return sp;
    }
}

void ko_synth_normal_portable(uint64_t seed, float sigma, uint64_t offset, size_t n, float* out) {
    auto mix = [](uint64_t sd, uint64_t j) {
        uint64_t v = sd + (j + 1) * 0x9E3779B97F4A7C15ULL;
        v = (v ^ (v >> 30)) * 0xBF58476D1CE4E5B9ULL;
        v = (v ^ (v >> 27)) * 0x94D049BB133111EBULL;
        return v ^ (v >> 31);
    };
    auto run = [&](size_t lo, size_t hi) {
        for (size_t j = lo; j < hi; ++j) {
            const uint64_t i = offset + j;
            const double u1 = 1.0 - (double)(mix(seed, 2 * i) >> 11) * 0x1p-53;
            const double u2 = (double)(mix(seed, 2 * i + 1) >> 11) * 0x1p-53;
            const double z = std::sqrt(-2.0 * portable_ln(u1)) * portable_cos_2pi(u2);
            out[j] = (float)z * sigma;
        }
    };
    const size_t nt = n < (size_t(1) << 20) ? 1 : std::max<unsigned>(1, std::thread::hardware_concurrency());
    const size_t chunk = (n + nt - 1) / nt;
    std::vector<std::thread> ts;
    for (size_t s0 = chunk; s0 < n; s0 += chunk) ts.emplace_back(run, s0, std::min(n, s0 + chunk));
    run(0, std::min(n, chunk));
    for (auto& th : ts) th.join();
}

// The reference's test LCG (crates/02-runtime/kt-runtime/src/gate.rs:29-36; kt-core/src/tests.rs:15-24):
// s ← s·6364136223846793005 + 1442695040888963407 (mod 2^64), value = (s >> 33) mod (hi − lo + 1) + lo.
void ko_lcg_uniform(uint64_t seed, int64_t lo, int64_t hi, size_t n, int32_t* out) {
    uint64_t s = seed;
    const uint64_t range = (uint64_t)(hi - lo + 1);
    for (size_t i = 0; i < n; ++i) {
        s = s * 6364136223846793005ULL + 1442695040888963407ULL;
        out[i] = (int32_t)((int64_t)((s >> 33) % range) + lo);
    }
}

// The routed part only, for a subset of tokens (per-token outputs before the merge), for stage-level checks:
// writes each token's combine output and scale.
void ko_moe_forward_tokens(void* p, const int32_t* x, size_t rows, ko_scale xs, int32_t* y, ko_scale* ys) {
    MoeMlp* m = (MoeMlp*)p;
    size_t d = m->dim();
    for (size_t t = 0; t < rows; ++t) {
        IntTensor row{std::vector<int32_t>(x + t * d, x + (t + 1) * d), {d}, from_c(xs)};
        IntTensor o = m->forward_one_int(row);
        std::memcpy(y + t * d, o.data.data(), d * 4);
        ys[t] = to_c(o.scale);
    }
}

// The expert-parallel seam (layers.rs:945-984) with local experts behind the callback: must equal ko_moe_forward.
void ko_moe_forward_with_local_experts(void* p, const int32_t* x, size_t rows, ko_scale xs, int32_t* y, ko_scale* ys) {
    MoeMlp* m = (MoeMlp*)p;
    size_t d = m->dim();
    IntTensor t{std::vector<int32_t>(x, x + rows * d), rows == 1 ? std::vector<size_t>{d} : std::vector<size_t>{rows, d},
                from_c(xs)};
    IntTensor o = m->forward_int_with_experts(t, [&](const std::vector<size_t>& ids, const IntTensor& row) {
        std::vector<IntTensor> v;
        for (size_t e : ids) v.push_back(m->experts[e].forward_int(row));
        return v;
    });
    std::memcpy(y, o.data.data(), o.data.size() * 4);
    *ys = to_c(o.scale);
}

// The seam (layers.rs:945-984) with the expert outputs given: ye [rows][top_k][d] and yse [rows][top_k] in route order,
// as a transport would deliver them. Rows reach the callback in order, skipping those whose route is empty.
void ko_moe_forward_with_given_experts(void* p, const int32_t* x, size_t rows, ko_scale xs, const int32_t* ye,
                                       const ko_scale* yse, int32_t* y, ko_scale* ys) {
    MoeMlp* m = (MoeMlp*)p;
    const size_t d = m->dim(), K = m->top_k;
    IntTensor t{std::vector<int32_t>(x, x + rows * d), rows == 1 ? std::vector<size_t>{d} : std::vector<size_t>{rows, d},
                from_c(xs)};
    std::vector<size_t> live;
    for (size_t r = 0; r < rows; ++r) {
        IntTensor row{std::vector<int32_t>(x + r * d, x + (r + 1) * d), {d}, from_c(xs)};
        if (m->route(row).sumc > 0) live.push_back(r);
    }
    size_t next = 0;
    IntTensor o = m->forward_int_with_experts(t, [&](const std::vector<size_t>& ids, const IntTensor&) {
        const size_t r = live.at(next++);
        std::vector<IntTensor> v;
        for (size_t j = 0; j < ids.size(); ++j) {
            const int32_t* src = ye + (r * K + j) * d;
            v.push_back(IntTensor{std::vector<int32_t>(src, src + d), {d}, from_c(yse[r * K + j])});
        }
        return v;
    });
    std::memcpy(y, o.data.data(), o.data.size() * 4);
    *ys = to_c(o.scale);
}

// MoeMlp::route for each row (layers.rs:826-862).
void ko_moe_route(void* p, const int32_t* x, size_t rows, ko_scale xs, int32_t* experts, int64_t* ec, int64_t* sumc) {
    MoeMlp* m = (MoeMlp*)p;
    size_t d = m->dim();
    for (size_t t = 0; t < rows; ++t) {
        IntTensor row{std::vector<int32_t>(x + t * d, x + (t + 1) * d), {d}, from_c(xs)};
        MoeRoute r = m->route(row);
        for (size_t i = 0; i < m->top_k; ++i) {
            experts[t * m->top_k + i] = (int32_t)r.experts[i];
            ec[t * m->top_k + i] = r.ec[i];
        }
        sumc[t] = r.sumc;
    }
}

// The router logits (QuantLinear::forward_int of the router, rows = 1 per token).
void ko_moe_router_logits(void* p, const int32_t* x, size_t rows, ko_scale xs, int32_t* logits, ko_scale* ls) {
    MoeMlp* m = (MoeMlp*)p;
    size_t d = m->dim(), e = m->router.out_features;
    for (size_t t = 0; t < rows; ++t) {
        IntTensor row{std::vector<int32_t>(x + t * d, x + (t + 1) * d), {d}, from_c(xs)};
        IntTensor l = m->router.forward_int(row);
        std::memcpy(logits + t * e, l.data.data(), e * 4);
        ls[t] = to_c(l.scale);
    }
}

// One expert's SwiGLU on one token (layers.rs:609-640), for stage-level checks.
void ko_moe_expert(void* p, size_t e, const int32_t* x, ko_scale xs, int32_t* y, ko_scale* ys) {
    MoeMlp* m = (MoeMlp*)p;
    size_t d = m->dim();
    IntTensor row{std::vector<int32_t>(x, x + d), {d}, from_c(xs)};
    IntTensor o = m->experts[e].forward_int(row);
    std::memcpy(y, o.data.data(), o.data.size() * 4);
    *ys = to_c(o.scale);
}

// add (layers.rs:121-136) on two equal-length tensors.
// RmsNorm (layers.rs:352-449) built from f32 weights and eps, applied to rows x dim codes.
void ko_rmsnorm(const float* weight, size_t dim, double eps, const int32_t* x, size_t rows, ko_scale xs, int32_t* y,
                ko_scale* ys, int32_t* wcodes, ko_scale* w_scale, ko_scale* eps_scale) {
    RmsNorm nrm(weight, dim, eps);
    IntTensor t{std::vector<int32_t>(x, x + rows * dim), {rows, dim}, from_c(xs)};
    IntTensor o = nrm.forward_int(t);
    std::copy(o.data.begin(), o.data.end(), y);
    *ys = to_c(o.scale);
    if (wcodes) std::copy(nrm.wcodes.begin(), nrm.wcodes.end(), wcodes);
    if (w_scale) *w_scale = to_c(nrm.w_scale);
    if (eps_scale) *eps_scale = to_c(nrm.eps_scale);
}

ko_scale ko_scale_add(ko_scale a, ko_scale b) { return to_c(from_c(a).add(from_c(b))); }
ko_scale ko_scale_rsqrt(ko_scale a) { return to_c(from_c(a).rsqrt()); }
ko_scale ko_scale_from_f64(double x) { return to_c(Scale::from_f64(x)); }

void ko_add(const int32_t* a, ko_scale as, const int32_t* b, ko_scale bs, size_t n, int32_t* y, ko_scale* ys) {
    IntTensor ta{std::vector<int32_t>(a, a + n), {n}, from_c(as)}, tb{std::vector<int32_t>(b, b + n), {n}, from_c(bs)};
    IntTensor o = add(ta, tb);
    std::memcpy(y, o.data.data(), n * 4);
    *ys = to_c(o.scale);
}

}  // extern "C"
