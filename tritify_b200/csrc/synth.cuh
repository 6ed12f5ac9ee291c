// Synthetic weights made on the device, for layers too large to generate and quantise on the host in reasonable
// time (a GLM-4.5-Air-shaped stack holds about 100 G weights).
//
// The portable normal generator. The reference has no normal RNG; this build defines its inputs. The host generator
// (host_prep.cpp, synth_normal) calls libm's log and cos, whose last bit differs between host and device libraries,
// so a device copy of it would not give the host's bytes. This one computes the same Box-Muller deviate with its own
// logarithm and cosine built only from correctly rounded IEEE-754 additions, multiplications, divisions and square
// roots, evaluated in a fixed order with no fused multiply-add: the host (compiled with -ffp-contract=off) and the
// device (the _rn intrinsics, which the compiler never contracts) produce identical bits, so a weight generated on the
// GPU equals the one the CPU oracle generates for the same (seed, index).
//
//   element i of stream `seed`: two uniforms from splitmix64 at positions 2i and 2i+1 (as the host generator),
//   u1 = 1 - (x >> 11)·2^-53 in (0, 1], u2 = (y >> 11)·2^-53 in [0, 1);
//   z = sqrt(-2·ln(u1))·cos(2π·u2) in f64; out = RN_f32(z)·sigma in f32.
//   ln(u): u = m·2^e with m in [sqrt(1/2), sqrt(2)); ln(m) = 2·atanh(s), s = (m-1)/(m+1), |s| <= 0.1716, as the odd
//   series s + s^3/3 + ... + s^23/23 (Horner in s^2); ln(u) = e·ln2 + ln(m).
//   cos(2π·u): t = 4u = q + r exactly (quadrant q, r in [0, 1)); the angle a = min(r, 1-r)·π/2 <= π/4; cos a and
//   sin a from their Taylor series to the a^18 and a^19 terms; the quadrant and the complement pick the result.
// Measured against libm over 2·10^5 draws: ln within 3.3e-16 relative, cos within 6.4e-16 absolute.
#pragma once

#include <stdint.h>

#include "fixed_point.cuh"

namespace sy {

#ifdef __CUDA_ARCH__
__device__ __forceinline__ double padd(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double pmul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double pdiv(double a, double b) { return __ddiv_rn(a, b); }
__device__ __forceinline__ double psqrt(double a) { return __dsqrt_rn(a); }
__device__ __forceinline__ float pmulf(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float pf32(double a) { return __double2float_rn(a); }
#else
inline double padd(double a, double b) { return a + b; }
inline double pmul(double a, double b) { return a * b; }
inline double pdiv(double a, double b) { return a / b; }
inline double psqrt(double a) { return __builtin_sqrt(a); }
inline float pmulf(float a, float b) { return a * b; }
inline float pf32(double a) { return (float)a; }
#endif

KT_HD uint64_t splitmix64_at(uint64_t seed, uint64_t pos) {
    uint64_t z = seed + (pos + 1) * 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

KT_HD uint64_t dbits(double x) {
#ifdef __CUDA_ARCH__
    return (uint64_t)__double_as_longlong(x);
#else
    uint64_t b;
    __builtin_memcpy(&b, &x, 8);
    return b;
#endif
}
KT_HD double bitsd(uint64_t b) {
#ifdef __CUDA_ARCH__
    return __longlong_as_double((long long)b);
#else
    double x;
    __builtin_memcpy(&x, &b, 8);
    return x;
#endif
}

// ln(u) for a normal u > 0.
KT_HD double plog(double u) {
    const uint64_t b = dbits(u);
    int e = (int)((b >> 52) & 0x7ff) - 1023;
    double m = bitsd((b & ((uint64_t(1) << 52) - 1)) | (uint64_t(1023) << 52));  // [1, 2)
    if (m > 0x1.6a09e667f3bcdp+0) {
        m = pmul(m, 0.5);  // exact
        e += 1;
    }
    const double s = pdiv(padd(m, -1.0), padd(m, 1.0));
    const double s2 = pmul(s, s);
    double p = 0x1.642c8590b2164p-5;  // 1/23
    p = padd(pmul(p, s2), 0x1.8618618618618p-5);
    p = padd(pmul(p, s2), 0x1.af286bca1af28p-5);
    p = padd(pmul(p, s2), 0x1.e1e1e1e1e1e1ep-5);
    p = padd(pmul(p, s2), 0x1.1111111111111p-4);
    p = padd(pmul(p, s2), 0x1.3b13b13b13b14p-4);
    p = padd(pmul(p, s2), 0x1.745d1745d1746p-4);
    p = padd(pmul(p, s2), 0x1.c71c71c71c71cp-4);
    p = padd(pmul(p, s2), 0x1.2492492492492p-3);
    p = padd(pmul(p, s2), 0x1.999999999999ap-3);
    p = padd(pmul(p, s2), 0x1.5555555555555p-2);  // 1/3
    const double atanh = padd(s, pmul(s, pmul(s2, p)));
    return padd(pmul((double)e, 0x1.62e42fefa39efp-1), pmul(2.0, atanh));
}

// cos(2π·u) for u in [0, 1).
KT_HD double pcos2pi(double u) {
    const double t = pmul(u, 4.0);  // exact
    const int q = (int)t;
    const double r = padd(t, -(double)q);  // exact
    const bool lo = r <= 0.5;
    const double a = pmul(lo ? r : padd(1.0, -r), 0x1.921fb54442d18p+0);
    const double a2 = pmul(a, a);
    double c = -0x1.6827863b97d97p-53;  // -1/18!
    c = padd(pmul(c, a2), 0x1.ae7f3e733b81fp-45);
    c = padd(pmul(c, a2), -0x1.93974a8c07c9dp-37);
    c = padd(pmul(c, a2), 0x1.1eed8eff8d898p-29);
    c = padd(pmul(c, a2), -0x1.27e4fb7789f5cp-22);
    c = padd(pmul(c, a2), 0x1.a01a01a01a01ap-16);
    c = padd(pmul(c, a2), -0x1.6c16c16c16c17p-10);
    c = padd(pmul(c, a2), 0x1.5555555555555p-5);
    c = padd(pmul(c, a2), -0x1.0000000000000p-1);
    const double C = padd(1.0, pmul(a2, c));
    double sv = -0x1.2f49b46814157p-57;  // -1/19!
    sv = padd(pmul(sv, a2), 0x1.952c77030ad4ap-49);
    sv = padd(pmul(sv, a2), -0x1.ae7f3e733b81fp-41);
    sv = padd(pmul(sv, a2), 0x1.6124613a86d09p-33);
    sv = padd(pmul(sv, a2), -0x1.ae64567f544e4p-26);
    sv = padd(pmul(sv, a2), 0x1.71de3a556c734p-19);
    sv = padd(pmul(sv, a2), -0x1.a01a01a01a01ap-13);
    sv = padd(pmul(sv, a2), 0x1.1111111111111p-7);
    sv = padd(pmul(sv, a2), -0x1.5555555555555p-3);
    const double S = padd(a, pmul(a, pmul(a2, sv)));
    const double cphi = lo ? C : S, sphi = lo ? S : C;
    return q == 0 ? cphi : q == 1 ? -sphi : q == 2 ? -cphi : sphi;
}

// Element i of the portable N(0, sigma) stream `seed`.
KT_HD float portable_normal(uint64_t seed, float sigma, uint64_t i) {
    const double u1 = padd(1.0, -pmul((double)(splitmix64_at(seed, 2 * i) >> 11), 0x1p-53));
    const double u2 = pmul((double)(splitmix64_at(seed, 2 * i + 1) >> 11), 0x1p-53);
    const double z = pmul(psqrt(pmul(-2.0, plog(u1))), pcos2pi(u2));
    return pmulf(pf32(z), sigma);
}

#ifdef __CUDACC__
__global__ void portable_normal_kernel(uint64_t seed, float sigma, uint64_t offset, long long n, float* __restrict__ out) {
    kt::pdl_enter();
    for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < n; j += (long long)gridDim.x * blockDim.x)
        out[j] = portable_normal(seed, sigma, offset + (uint64_t)j);
}

// max |w| as the bits of a non-negative float (their integer order is their numeric order).
__global__ void absmax_f32_kernel(const float* __restrict__ w, long long n, unsigned* __restrict__ out) {
    kt::pdl_enter();
    unsigned m = 0;
    for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < n; j += (long long)gridDim.x * blockDim.x)
        m = max(m, __float_as_uint(w[j]) & 0x7fffffffu);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0 && m) atomicMax(out, m);
}

// QuantLinear::from_weights' codes (layers.rs:225-244): clamp(round(w / step), ±WLEVELS), the division and the
// rounding (half away from zero) in f64 as on the host.
__global__ void quantize_kernel(const float* __restrict__ w, long long n, double step, int32_t* __restrict__ codes) {
    kt::pdl_enter();
    for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < n; j += (long long)gridDim.x * blockDim.x) {
        double c = round(__ddiv_rn((double)w[j], step));
        c = c > (double)kt::WLEVELS ? (double)kt::WLEVELS : (c < -(double)kt::WLEVELS ? -(double)kt::WLEVELS : c);
        codes[j] = (int32_t)c;
    }
}
#endif

}  // namespace sy
