// Host-side, offline preparation of tritify's integer MoE layer: the f64 steps the reference runs once on the host.
//
//   QuantLinear::from_weights   crates/01-engine/kt-core/src/layers.rs:225-244  (per-tensor b=12 weight quantiser)
//   QuantLinear::with_bias      layers.rs:246-257
//   IntTensor::from_reals       crates/01-engine/kt-core/src/tensor.rs:106-116 (the entry quantiser)
//   SigmoidScore::new           crates/01-engine/kt-core/src/router.rs:37-51  (coded selection bias)
//   CodeLut::build              crates/00-kernels/kt-int/src/lib.rs:359-379   (exp, SiLU and sigmoid code tables)
//   Scale::from_f64 / frexp     kt-int lib.rs:46-60, :215-222
// They call the host libm (exp) exactly as the reference does and are compiled with -ffp-contract=off, so no f64
// expression is fused into an FMA. Nothing here runs per token; the GPU path starts from the integer codes.
//
// Also here: the synthetic input generator this build defines (the reference has no normal RNG): splitmix64 streams,
// Box-Muller in f64, cast to f32 and scaled by sigma. Element i of a stream depends only on (seed, i), so threads
// fill disjoint ranges and the bytes never depend on the thread count.

#include "host_prep.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

namespace hp {

static const int64_t WLEVELS = 265720;
static const int64_t ACT_LEVELS = int64_t(1) << 28;

// kt-int lib.rs:46-60
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
    uint64_t mantissa = (bits & ~(uint64_t(0x7ff) << 52)) | (uint64_t(1022) << 52);
    std::memcpy(m_out, &mantissa, 8);
    *e_out = exp_field - 1022;
}

// kt-int lib.rs:215-222
HScale scale_from_f64(double x) {
    if (!(x > 0.0 && std::isfinite(x))) return HScale{0, 0};
    double m;
    int32_t e;
    frexp_bits(x, &m, &e);
    return HScale{(int64_t)std::round(m * (double)(uint64_t(1) << 31)), 31 - e};
}

static size_t worker_count(size_t n) {
    size_t hw = std::thread::hardware_concurrency();
    if (hw == 0) hw = 1;
    size_t by_size = n / (size_t(1) << 20) + 1;
    return std::max<size_t>(1, std::min(hw, by_size));
}

template <class F>
static void parallel_ranges(size_t n, F f) {
    size_t nt = worker_count(n);
    if (nt <= 1) {
        f(0, n);
        return;
    }
    size_t chunk = (n + nt - 1) / nt;
    std::vector<std::thread> ts;
    for (size_t s = 0; s < n; s += chunk) ts.emplace_back(f, s, std::min(n, s + chunk));
    for (auto& t : ts) t.join();
}

// layers.rs:225-244. The peak is a max (order-independent), so the threaded scan gives the serial result.
void quantize_weights(const float* w, size_t n, int32_t* codes, HScale* scale) {
    if (n == 0) {
        *scale = HScale{0, 0};
        return;
    }
    size_t nt = worker_count(n);
    std::vector<double> peaks(nt + 1, 0.0);
    {
        size_t chunk = (n + nt - 1) / std::max<size_t>(nt, 1);
        std::vector<std::thread> ts;
        size_t idx = 0;
        for (size_t s = 0; s < n; s += chunk, ++idx) {
            ts.emplace_back(
                [&, s, idx] {
                    double p = 0.0;
                    for (size_t i = s; i < std::min(n, s + chunk); ++i) p = std::fmax(p, std::fabs((double)w[i]));
                    peaks[idx] = p;
                });
        }
        for (auto& t : ts) t.join();
    }
    double peak = 0.0;
    for (double p : peaks) peak = std::fmax(peak, p);
    if (peak == 0.0) {
        std::memset(codes, 0, n * sizeof(int32_t));
        *scale = HScale{0, 0};
        return;
    }
    const double step = peak / (double)WLEVELS;
    parallel_ranges(n, [&](size_t s, size_t e) {
        for (size_t i = s; i < e; ++i) {
            int64_t c = (int64_t)std::round((double)w[i] / step);
            c = std::min<int64_t>(std::max<int64_t>(c, -WLEVELS), WLEVELS);
            codes[i] = (int32_t)c;
        }
    });
    *scale = scale_from_f64(step);
}

// layers.rs:246-257. Returns false when the bias is all zero (the reference then keeps no bias).
bool quantize_bias(const float* b, size_t n, int64_t* codes, HScale* scale) {
    double bmax = 0.0;
    for (size_t i = 0; i < n; ++i) bmax = std::fmax(bmax, std::fabs((double)b[i]));
    if (!(bmax > 0.0)) return false;
    const double step = bmax / (double)ACT_LEVELS;
    for (size_t i = 0; i < n; ++i) codes[i] = (int64_t)std::round((double)b[i] / step);
    *scale = scale_from_f64(step);
    return true;
}

// router.rs:37-51: round(bias · 2^ROUTER_CODE_BITS).
void code_sigmoid_bias(const float* b, size_t n, int64_t* codes) {
    const double k = (double)(uint64_t(1) << 20);
    for (size_t i = 0; i < n; ++i) codes[i] = (int64_t)std::round((double)b[i] * k);
}

// tensor.rs:106-116 at levels = ACT_LEVELS, from f32 values widened to f64.
void from_reals(const float* v, size_t n, int32_t* data, HScale* scale) {
    double mx = 0.0;
    for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, std::fabs((double)v[i]));
    if (mx == 0.0) {
        std::memset(data, 0, n * sizeof(int32_t));
        *scale = HScale{0, 0};
        return;
    }
    const double step = mx / (double)ACT_LEVELS;
    const double inv = (double)ACT_LEVELS / mx;
    parallel_ranges(n, [&](size_t s, size_t e) {
        for (size_t i = s; i < e; ++i) data[i] = (int32_t)std::round((double)v[i] * inv);
    });
    *scale = scale_from_f64(step);
}

// kt-int lib.rs:359-379, with the three functions of the MoE path:
//   kind 0: exp over [-30, 0], 2^16 entries, 20 code bits (layers.rs:688)
//   kind 1: SiLU x/(1+exp(-x)) over [-30, 30], 2^16 entries, 20 code bits, identity right tail (layers.rs:599)
//   kind 2: sigmoid 1/(1+exp(-x)) over [-16, 16], 2^16 entries, 20 code bits (router.rs:40-47)
void build_table(int kind, HTable* t) {
    double lo, hi;
    if (kind == 0) {
        lo = -30.0;
        hi = 0.0;
    } else if (kind == 1) {
        lo = -30.0;
        hi = 30.0;
    } else {
        lo = -16.0;
        hi = 16.0;
    }
    const size_t n = size_t(1) << 16;
    const double k = (double)(uint64_t(1) << 20);
    t->codes.resize(n);
    for (size_t i = 0; i < n; ++i) {
        const double x = lo + (hi - lo) * ((double)i / (double)(n - 1));
        double fx;
        if (kind == 0)
            fx = std::exp(x);
        else if (kind == 1)
            fx = x / (1.0 + std::exp(-x));
        else
            fx = 1.0 / (1.0 + std::exp(-x));
        t->codes[i] = (int64_t)std::round(fx * k);
    }
    const double inv_step = (double)(n - 1) / (hi - lo);
    t->inv_step = scale_from_f64(inv_step);
    t->lo_index = (int64_t)std::round(lo * inv_step);
    t->code_scale = scale_from_f64(1.0 / k);
}

// The build-defined generator: element i of stream `seed` uses u1, u2 from splitmix64 at positions 2i and 2i+1,
// u = (x >> 11)·2^-53, u1 mapped into (0, 1]; z = sqrt(-2 ln u1)·cos(2π u2) in f64; out[i] = (float)z · sigma
// (the product in f32).
static inline uint64_t splitmix64_at(uint64_t seed, uint64_t pos) {
    uint64_t z = seed + (pos + 1) * 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

void synth_normal(uint64_t seed, float sigma, uint64_t offset, size_t n, float* out) {
    const double two_pi = 6.283185307179586;
    parallel_ranges(n, [&](size_t s, size_t e) {
        for (size_t j = s; j < e; ++j) {
            const uint64_t i = offset + j;
            const double u1 = 1.0 - (double)(splitmix64_at(seed, 2 * i) >> 11) * (1.0 / 9007199254740992.0);
            const double u2 = (double)(splitmix64_at(seed, 2 * i + 1) >> 11) * (1.0 / 9007199254740992.0);
            const double z = std::sqrt(-2.0 * std::log(u1)) * std::cos(two_pi * u2);
            out[j] = (float)z * sigma;
        }
    });
}

// Uniform integers in [lo, hi] from the reference's test LCG (gate.rs:29-36 form): s = s·6364136223846793005 +
// 1442695040888963407, value = (s >> 33) mod (hi - lo + 1) + lo. Serial: each value depends on the previous state.
void lcg_uniform(uint64_t seed, int64_t lo, int64_t hi, size_t n, int32_t* out) {
    uint64_t s = seed;
    const uint64_t range = (uint64_t)(hi - lo + 1);
    for (size_t i = 0; i < n; ++i) {
        s = s * 6364136223846793005ULL + 1442695040888963407ULL;
        out[i] = (int32_t)((int64_t)((s >> 33) % range) + lo);
    }
}

}  // namespace hp
