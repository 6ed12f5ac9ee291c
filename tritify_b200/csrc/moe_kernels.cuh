// The stages of tritify's integer MoE layer around the digit-plane GEMM, as sm_100a kernels.
//
// Reference semantics (paths relative to the reference project root):
//   QuantLinear::forward_int        crates/01-engine/kt-core/src/layers.rs:275-328
//   SwiGluMlp::forward_int          layers.rs:609-640
//   MoeMlp::route / route_sigmoid   layers.rs:826-862, crates/01-engine/kt-core/src/router.rs:64-71
//   MoeMlp::combine                 layers.rs:893-923
//   forward_routed (merge)          layers.rs:988-1020
//   add (routed + shared)           layers.rs:121-136
// The reference runs the routed experts token by token; here every (token, slot) row that chose an expert is one
// row of that expert's grouped GEMM. Every quantity the reference reduces per token (xmax, ymax, hmax, the scales)
// is reduced per row here, and every tensor-global one (merge, shared expert, add) over the whole tensor.
#pragma once

#include <stdint.h>

#include "fixed_point.cuh"

namespace mk {

using kt::Scale;

constexpr int LUT_N = 1 << 16;

// One table of the path (kt-int CodeLut, crates/00-kernels/kt-int/src/lib.rs:346-396): device codes + constants.
struct Lut {
    const int64_t* codes;
    Scale inv_step;
    int64_t lo_index;
    const int32_t* codes32;  // the same codes as int32 when every one fits (half the cache footprint), else nullptr
};

// ───────────── block reductions ─────────────

__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        uint64_t w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w > v ? w : v;
    }
    return v;
}

// Max over the block; every thread gets the result. `red` holds >= 32 entries.
__device__ __forceinline__ uint64_t block_max_u64(uint64_t v, uint64_t* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_max_u64(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    uint64_t r = lane < nw ? red[lane] : 0;
    r = warp_max_u64(r);
    return r;
}

__device__ __forceinline__ uint64_t uabs64(int64_t v) { return v >= 0 ? (uint64_t)v : (uint64_t)(-(v + 1)) + 1; }

__device__ __forceinline__ void store_digits4(int8_t* p0, int8_t* p1, int8_t* p2, const int32_t q[4]) {
    int8_t a[4], b[4], c[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) kt::split_digits(q[j], a[j], b[j], c[j]);
    *(char4*)p0 = make_char4(a[0], a[1], a[2], a[3]);
    *(char4*)p1 = make_char4(b[0], b[1], b[2], b[3]);
    *(char4*)p2 = make_char4(c[0], c[1], c[2], c[3]);
}

// ───────────── per-token quantisation of the layer input (QuantLinear::forward_int, layers.rs:279-298) ─────────────
// For each token row: xmax = max|x|, qx = quant_to(x, xmax) written as three digit planes [3][R_pad][K_pad], and
// s_qx = from_ratio(xmax, WLEVELS)·x.scale. Every linear that reads the row (router, each routed expert's gate and up)
// quantises it identically, so the planes are computed once. `per_token == 0` uses one xmax for the whole tensor
// (the shared expert, whose QuantLinear sees the whole [rows, dim] input): gxmax must hold that max.
__global__ void quant_rows_kernel(const int32_t* __restrict__ x, int rows, int K, int K_pad, long long R_pad,
                                  int8_t* __restrict__ planes, int64_t* __restrict__ row_xmax, Scale* __restrict__ row_sqx,
                                  const Scale* __restrict__ x_scale, const unsigned long long* __restrict__ gxmax) {
    kt::pdl_enter();
    __shared__ uint64_t red[32];
    const int r = blockIdx.x;
    if (r >= rows) return;
    const int32_t* xr = x + (long long)r * K;
    const bool vec = (K & 3) == 0 && ((uintptr_t)x & 15) == 0;  // rows start 16-byte aligned: 4 codes per load
    int64_t xmax;
    if (gxmax) {
        xmax = (int64_t)*gxmax;
    } else {
        uint64_t m = 0;
        if (vec) {
            for (int k4 = threadIdx.x * 4; k4 < K; k4 += blockDim.x * 4) {
                const int4 v = __ldg((const int4*)(xr + k4));
                m = max(max(m, uabs64(v.x)), max(uabs64(v.y), max(uabs64(v.z), uabs64(v.w))));
            }
        } else {
            for (int k = threadIdx.x; k < K; k += blockDim.x) m = max(m, uabs64(xr[k]));
        }
        xmax = (int64_t)block_max_u64(m, red);
    }
    int8_t* p0 = planes + (long long)r * K_pad;
    int8_t* p1 = p0 + R_pad * K_pad;
    int8_t* p2 = p1 + R_pad * K_pad;
    const kt::QuantPlan qp = kt::make_quant(xmax);
    for (int k4 = threadIdx.x * 4; k4 < K_pad; k4 += blockDim.x * 4) {
        int32_t q[4];
        if (vec && k4 < K && xmax > 0) {
            const int4 v = __ldg((const int4*)(xr + k4));
            q[0] = kt::quant_row(v.x, qp);
            q[1] = kt::quant_row(v.y, qp);
            q[2] = kt::quant_row(v.z, qp);
            q[3] = kt::quant_row(v.w, qp);
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int k = k4 + j;
                q[j] = (k < K && xmax > 0) ? kt::quant_row(xr[k], qp) : 0;
            }
        }
        store_digits4(p0 + k4, p1 + k4, p2 + k4, q);
    }
    if (threadIdx.x == 0 && row_xmax) {
        row_xmax[r] = xmax;
        row_sqx[r] = xmax > 0 ? kt::scale_mul(kt::from_ratio((kt::u128)(uint64_t)xmax, (kt::u128)kt::WLEVELS), *x_scale)
                              : kt::scale_zero();
    }
}

// Global max |x| over n values (atomicMax into *out, which the caller zeroes).
__global__ void absmax_i32_kernel(const int32_t* __restrict__ v, long long n, unsigned long long* out) {
    kt::pdl_enter();
    __shared__ uint64_t red[32];
    uint64_t m = 0;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        m = max(m, uabs64(v[i]));
    m = block_max_u64(m, red);
    if (threadIdx.x == 0 && m) atomicMax(out, (unsigned long long)m);
}

// Global max |v| over the columns [c0, c0 + cols) of rows x ld int64 (atomicMax into *out).
__global__ void absmax_i64_cols_kernel(const int64_t* __restrict__ v, int rows, long long ld, int c0, int cols,
                                       unsigned long long* out) {
    kt::pdl_enter();
    __shared__ uint64_t red[32];
    uint64_t m = 0;
    const long long n = (long long)rows * cols;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / cols, c = i % cols;
        m = max(m, uabs64(v[r * ld + c0 + c]));
    }
    m = block_max_u64(m, red);
    if (threadIdx.x == 0 && m) atomicMax(out, (unsigned long long)m);
}

// ───────────── routing: router logits → integer softmax / sigmoid codes → top-k (layers.rs:275-328, :800-862) ──────
struct RouteArgs {
    const int64_t* acc;  // [rows][E] router accumulators
    const int64_t* row_xmax;
    const Scale* row_sqx;
    int rows, E, top_k, norm_topk, sigmoid;
    Scale w_scale;
    const int64_t* bias_codes;  // router QuantLinear bias (with_bias), or nullptr
    Scale bias_scale;
    const int64_t* sig_bias;  // sigmoid selection bias codes, or nullptr
    Lut exp_lut, sig_lut;
    int32_t* top_e;  // [rows][top_k]
    int64_t* top_ec;
    int64_t* sumc;
    int32_t* logits_out;  // optional [rows][E]
    Scale* logit_scale_out;
};

constexpr int ROUTE_MAX_PER_LANE = 16;  // E <= 512

// One warp per token.
__global__ void route_kernel(const RouteArgs a) {
    kt::pdl_enter();
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= a.rows) return;
    const int E = a.E;
    const int per = (E + 31) / 32;
    int64_t acc[ROUTE_MAX_PER_LANE];
    int32_t logit[ROUTE_MAX_PER_LANE];
    const int64_t xmax = a.row_xmax[t];
    Scale lscale = kt::scale_zero();
    bool zero = false;
    if (xmax == 0) {
        // input all zero: the output is the bias codes at the bias scale, or zero (layers.rs:282-295)
        for (int q = 0; q < per; ++q) {
            const int o = lane + 32 * q;
            logit[q] = (o < E && a.bias_codes) ? (int32_t)a.bias_codes[o] : 0;
        }
        lscale = a.bias_codes ? a.bias_scale : kt::scale_zero();
    } else {
        const Scale c = kt::scale_mul(a.row_sqx[t], a.w_scale);
        if (c.mant == 0) {
            zero = true;
        } else {
            Scale fb = kt::scale_zero();
            if (a.bias_codes) fb = kt::scale_mul(a.bias_scale, kt::scale_recip(c));
            uint64_t ymax = 0;
            for (int q = 0; q < per; ++q) {
                const int o = lane + 32 * q;
                int64_t v = 0;
                if (o < E) {
                    v = a.acc[(long long)t * E + o];
                    if (a.bias_codes) v += kt::scale_apply(fb, a.bias_codes[o]);
                }
                acc[q] = v;
                ymax = max(ymax, uabs64(v));
            }
            ymax = warp_max_u64(ymax);
            if (ymax == 0) {
                zero = true;
            } else {
                for (int q = 0; q < per; ++q) logit[q] = kt::requant_act(acc[q], (int64_t)ymax);
                lscale = kt::scale_mul(kt::ratio_act((int64_t)ymax), c);
            }
        }
        if (zero)
            for (int q = 0; q < per; ++q) logit[q] = 0;
    }
    if (a.logits_out) {
        for (int q = 0; q < per; ++q) {
            const int o = lane + 32 * q;
            if (o < E) a.logits_out[(long long)t * E + o] = logit[q];
        }
        if (lane == 0) a.logit_scale_out[t] = lscale;
    }

    // Scores: softmax exp codes (layers.rs:832-840) or sigmoid codes + coded bias (router.rs:64-71).
    int64_t code[ROUTE_MAX_PER_LANE], key[ROUTE_MAX_PER_LANE];
    int64_t sum_all = 0;
    if (!a.sigmoid) {
        int32_t lmax = INT32_MIN;
        for (int q = 0; q < per; ++q)
            if (lane + 32 * q < E) lmax = max(lmax, logit[q]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lmax = max(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
        const Scale is = kt::scale_mul(lscale, a.exp_lut.inv_step);
        for (int q = 0; q < per; ++q) {
            const int o = lane + 32 * q;
            int64_t ec = 0;
            if (o < E) {
                const int64_t idx = kt::scale_apply(is, (int64_t)(logit[q] - lmax)) - a.exp_lut.lo_index;
                ec = idx < 0 ? 0 : a.exp_lut.codes[idx > LUT_N - 1 ? LUT_N - 1 : idx];
            }
            code[q] = ec;
            key[q] = logit[q];
            sum_all += ec;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum_all += __shfl_xor_sync(0xffffffffu, sum_all, o);
    } else {
        const Scale is = kt::scale_mul(lscale, a.sig_lut.inv_step);
        for (int q = 0; q < per; ++q) {
            const int o = lane + 32 * q;
            int64_t c = 0, k = 0;
            if (o < E) {
                int64_t idx = kt::scale_apply(is, (int64_t)logit[q]) - a.sig_lut.lo_index;
                idx = idx < 0 ? 0 : (idx > LUT_N - 1 ? LUT_N - 1 : idx);
                c = a.sig_lut.codes[idx];
                k = c + (a.sig_bias ? a.sig_bias[o] : 0);
            }
            code[q] = c;
            key[q] = k;
        }
    }

    // Top-k: descending key, ties to the lower index (layers.rs:800-805); k rounds of a warp arg-max.
    unsigned taken = 0;  // bit q: this lane's candidate q was chosen
    int64_t sel_sum = 0;
    for (int i = 0; i < a.top_k; ++i) {
        int64_t bk = INT64_MIN;
        int bi = INT32_MAX;
        for (int q = 0; q < per; ++q) {
            const int o = lane + 32 * q;
            if (o < E && !(taken & (1u << q))) {
                if (key[q] > bk || (key[q] == bk && o < bi)) {
                    bk = key[q];
                    bi = o;
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const int64_t ok = __shfl_xor_sync(0xffffffffu, bk, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ok > bk || (ok == bk && oi < bi)) {
                bk = ok;
                bi = oi;
            }
        }
        // the owner lane marks it and publishes its code
        int64_t ec = 0;
        if ((bi & 31) == lane) {
            const int q = bi >> 5;
            taken |= 1u << q;
            ec = code[q];
        }
        ec = __shfl_sync(0xffffffffu, ec, bi & 31);
        sel_sum += ec;
        if (lane == 0) {
            a.top_e[(long long)t * a.top_k + i] = bi;
            a.top_ec[(long long)t * a.top_k + i] = ec;
        }
    }
    if (lane == 0) {
        int64_t s;
        if (a.sigmoid)
            s = a.norm_topk ? sel_sum : (int64_t(1) << kt::ROUTER_CODE_BITS);
        else
            s = a.norm_topk ? sel_sum : sum_all;
        a.sumc[t] = s;
    }
}

// ───────────── dispatch plan: a stable counting sort of (token, slot) by expert ─────────────
constexpr int PLAN_CHUNK = 2048;  // assignments per chunk
constexpr int PLAN_THREADS = 256;

__global__ void plan_count_kernel(const int32_t* __restrict__ top_e, long long n_assign, int E, int* __restrict__ counts) {
    kt::pdl_enter();
    extern __shared__ int hist[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
    __syncthreads();
    const long long base = (long long)blockIdx.x * PLAN_CHUNK;
    for (int j = threadIdx.x; j < PLAN_CHUNK; j += blockDim.x) {
        const long long a = base + j;
        if (a < n_assign) atomicAdd(&hist[top_e[a]], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) counts[(long long)blockIdx.x * E + e] = hist[e];
}

// One block: per-expert offsets, per-chunk offsets within each expert, and the n-tile tables of the grouped GEMMs
// for two tile widths (the gate/up GEMM and the down GEMM may tile the rows differently).
struct TileTable {
    int BN;
    int* tile_group;
    int* tile_row0;
    int* n_tiles;
};

// The exclusive scan over experts of (rows, tiles of width ta.BN, tiles of width tb.BN) from the per-expert totals
// `tot`, by the whole block (blockDim.x a multiple of 32, at most 1024): thread i owns the experts [i·per, (i+1)·per)
// and the threads' sums are scanned with warp shuffles, then over the warps. Writes expert_off, expert_count and
// group_end, the offsets into shared off_s (may be nullptr), toff_a and toff_b, and both tile counts. Ends with a
// barrier.
__device__ __forceinline__ void plan_offsets(const int* __restrict__ tot, int E, const TileTable& ta,
                                             const TileTable& tb, int* __restrict__ expert_off,
                                             int* __restrict__ expert_count, int* __restrict__ group_end,
                                             int* __restrict__ off_s, int* __restrict__ toff_a, int* __restrict__ toff_b) {
    __shared__ int wsum[3][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int per = (E + (int)blockDim.x - 1) / (int)blockDim.x;
    const int e0 = min(E, (int)threadIdx.x * per), e1 = min(E, e0 + per);
    int s0 = 0, s1 = 0, s2 = 0;
    for (int e = e0; e < e1; ++e) {
        s0 += tot[e];
        s1 += (tot[e] + ta.BN - 1) / ta.BN;
        s2 += (tot[e] + tb.BN - 1) / tb.BN;
    }
    int i0 = s0, i1 = s1, i2 = s2;  // inclusive over the warp's lanes
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int a0 = __shfl_up_sync(0xffffffffu, i0, o), a1 = __shfl_up_sync(0xffffffffu, i1, o),
                  a2 = __shfl_up_sync(0xffffffffu, i2, o);
        if (lane >= o) {
            i0 += a0;
            i1 += a1;
            i2 += a2;
        }
    }
    if (lane == 31) {
        wsum[0][warp] = i0;
        wsum[1][warp] = i1;
        wsum[2][warp] = i2;
    }
    __syncthreads();
    if (warp == 0) {  // inclusive over the warps
        int w0 = lane < nw ? wsum[0][lane] : 0, w1 = lane < nw ? wsum[1][lane] : 0, w2 = lane < nw ? wsum[2][lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int a0 = __shfl_up_sync(0xffffffffu, w0, o), a1 = __shfl_up_sync(0xffffffffu, w1, o),
                      a2 = __shfl_up_sync(0xffffffffu, w2, o);
            if (lane >= o) {
                w0 += a0;
                w1 += a1;
                w2 += a2;
            }
        }
        wsum[0][lane] = w0;
        wsum[1][lane] = w1;
        wsum[2][lane] = w2;
    }
    __syncthreads();
    int r = i0 - s0 + (warp ? wsum[0][warp - 1] : 0);
    int qa = i1 - s1 + (warp ? wsum[1][warp - 1] : 0);
    int qb = i2 - s2 + (warp ? wsum[2][warp - 1] : 0);
    for (int e = e0; e < e1; ++e) {
        expert_off[e] = r;
        if (off_s) off_s[e] = r;
        expert_count[e] = tot[e];
        toff_a[e] = qa;
        toff_b[e] = qb;
        r += tot[e];
        group_end[e] = r;
        qa += (tot[e] + ta.BN - 1) / ta.BN;
        qb += (tot[e] + tb.BN - 1) / tb.BN;
    }
    if (threadIdx.x == 0) {
        *ta.n_tiles = wsum[1][nw - 1];
        *tb.n_tiles = wsum[2][nw - 1];
    }
    __syncthreads();
}

// The tile tables of both widths from the scanned offsets: expert e's tiles at toff[e], in row order.
__device__ __forceinline__ void plan_tiles(const int* __restrict__ tot, int E, const int* __restrict__ off,
                                           const int* __restrict__ toff_a, const int* __restrict__ toff_b,
                                           const TileTable& ta, const TileTable& tb) {
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const int na = (tot[e] + ta.BN - 1) / ta.BN, nb = (tot[e] + tb.BN - 1) / tb.BN;
        for (int i = 0; i < na; ++i) {
            ta.tile_group[toff_a[e] + i] = e;
            ta.tile_row0[toff_a[e] + i] = off[e] + i * ta.BN;
        }
        for (int i = 0; i < nb; ++i) {
            tb.tile_group[toff_b[e] + i] = e;
            tb.tile_row0[toff_b[e] + i] = off[e] + i * tb.BN;
        }
    }
}

__global__ void plan_scan_kernel(const int* __restrict__ counts, int n_chunks, int E, int* __restrict__ chunk_off,
                                 int* __restrict__ expert_off, int* __restrict__ group_end,
                                 int* __restrict__ expert_count, TileTable ta, TileTable tb) {
    kt::pdl_enter();
    extern __shared__ int sh[];
    int* tot = sh;             // [E]
    int* toff_a = sh + E;      // [E] tile offsets, table a
    int* toff_b = sh + 2 * E;  // [E] tile offsets, table b
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int run = 0;
        for (int c = 0; c < n_chunks; ++c) {
            chunk_off[(long long)c * E + e] = run;
            run += counts[(long long)c * E + e];
        }
        tot[e] = run;
    }
    __syncthreads();
    plan_offsets(tot, E, ta, tb, expert_off, expert_count, group_end, nullptr, toff_a, toff_b);
    plan_tiles(tot, E, expert_off, toff_a, toff_b, ta, tb);
}

// Stable positions: assignment a = t·k + i goes to expert_off[e] + chunk_off[chunk][e] + (rank among the same expert
// earlier in its chunk). Rounds of blockDim assignments; warp match + per-warp counts give the rank.
__global__ void plan_assign_kernel(const int32_t* __restrict__ top_e, long long n_assign, int E,
                                   const int* __restrict__ chunk_off, const int* __restrict__ expert_off,
                                   int* __restrict__ slot_row, int* __restrict__ row_assign, int* __restrict__ row_expert) {
    kt::pdl_enter();
    extern __shared__ int sm[];
    const int nw = blockDim.x >> 5;
    int* running = sm;           // [E]
    int* wcnt = sm + E;          // [nw][E]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int e = threadIdx.x; e < E; e += blockDim.x) running[e] = 0;
    for (int i = threadIdx.x; i < nw * E; i += blockDim.x) wcnt[i] = 0;
    __syncthreads();
    const long long base = (long long)blockIdx.x * PLAN_CHUNK;
    for (int r0 = 0; r0 < PLAN_CHUNK; r0 += blockDim.x) {
        const long long a = base + r0 + threadIdx.x;
        const bool valid = (r0 + threadIdx.x < PLAN_CHUNK) && a < n_assign;
        const int e = valid ? top_e[a] : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const unsigned lt = (1u << lane) - 1u;
        const int rank_w = __popc(peers & lt);
        const bool leader = (peers & lt) == 0;
        if (valid && leader) wcnt[warp * E + e] = __popc(peers);
        __syncthreads();
        if (valid) {
            int before = running[e];
            for (int w = 0; w < warp; ++w) before += wcnt[w * E + e];
            const int pos = expert_off[e] + chunk_off[(long long)blockIdx.x * E + e] + before + rank_w;
            slot_row[a] = pos;
            row_assign[pos] = (int)a;
            row_expert[pos] = e;
        }
        __syncthreads();
        for (int ee = threadIdx.x; ee < E; ee += blockDim.x) {
            int s = 0;
            for (int w = 0; w < nw; ++w) {
                s += wcnt[w * E + ee];
                wcnt[w * E + ee] = 0;
            }
            running[ee] += s;
        }
        __syncthreads();
    }
}

// The routing plan of one chunk (n_assign <= PLAN_CHUNK, E <= PLAN_ONE_MAX_E) in one launch of one block: the counts
// (plan_count_kernel), the offsets and tile tables (plan_scan_kernel; the chunk offsets are all zero) and the stable
// assignment (plan_assign_kernel, the same per-warp ranks), with the offsets kept in shared memory between them.
constexpr int PLAN_ONE_THREADS = 512;
constexpr int PLAN_ONE_MAX_E = 256;

__global__ void __launch_bounds__(PLAN_ONE_THREADS)
    plan_one_chunk_kernel(const int32_t* __restrict__ top_e, int n_assign, int E, int* __restrict__ chunk_off,
                          int* __restrict__ expert_off, int* __restrict__ group_end, int* __restrict__ expert_count,
                          TileTable ta, TileTable tb, int* __restrict__ slot_row, int* __restrict__ row_assign,
                          int* __restrict__ row_expert) {
    kt::pdl_enter();
    constexpr int NW = PLAN_ONE_THREADS / 32;
    __shared__ int hist[PLAN_ONE_MAX_E], off_s[PLAN_ONE_MAX_E], toff_a[PLAN_ONE_MAX_E], toff_b[PLAN_ONE_MAX_E],
        running[PLAN_ONE_MAX_E];
    __shared__ int wcnt[NW * PLAN_ONE_MAX_E];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        hist[e] = 0;
        running[e] = 0;
        chunk_off[e] = 0;
    }
    for (int i = threadIdx.x; i < NW * E; i += blockDim.x) wcnt[i] = 0;
    __syncthreads();
    for (int j = threadIdx.x; j < n_assign; j += blockDim.x) atomicAdd(&hist[top_e[j]], 1);
    __syncthreads();
    plan_offsets(hist, E, ta, tb, expert_off, expert_count, group_end, off_s, toff_a, toff_b);
    plan_tiles(hist, E, off_s, toff_a, toff_b, ta, tb);
    for (int r0 = 0; r0 < n_assign; r0 += blockDim.x) {
        const int a = r0 + (int)threadIdx.x;
        const bool valid = a < n_assign;
        const int e = valid ? top_e[a] : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const unsigned lt = (1u << lane) - 1u;
        const int rank_w = __popc(peers & lt);
        const bool leader = (peers & lt) == 0;
        if (valid && leader) wcnt[warp * E + e] = __popc(peers);
        __syncthreads();
        if (valid) {
            int before = running[e];
            for (int w = 0; w < warp; ++w) before += wcnt[w * E + e];
            const int pos = off_s[e] + before + rank_w;
            slot_row[a] = pos;
            row_assign[pos] = a;
            row_expert[pos] = e;
        }
        __syncthreads();
        for (int ee = threadIdx.x; ee < E; ee += blockDim.x) {
            int s = 0;
            for (int w = 0; w < NW; ++w) {
                s += wcnt[w * E + ee];
                wcnt[w * E + ee] = 0;
            }
            running[ee] += s;
        }
        __syncthreads();
    }
}

// Gather: row r of the expert-sorted planes is token row_assign[r] / top_k of the token planes.
__global__ void permute_planes_kernel(const int8_t* __restrict__ src, long long src_R_pad, int8_t* __restrict__ dst,
                                      long long dst_R_pad, int K_pad, const int* __restrict__ row_assign, int top_k,
                                      int n_rows) {
    kt::pdl_enter();
    const int r = blockIdx.x;
    if (r >= n_rows) return;
    const int t = row_assign[r] / top_k;
    const int n16 = K_pad / 16;
#pragma unroll
    for (int p = 0; p < 3; ++p) {
        const int4* s = (const int4*)(src + (p * src_R_pad + t) * (long long)K_pad);
        int4* d = (int4*)(dst + (p * dst_R_pad + r) * (long long)K_pad);
        for (int i = threadIdx.x; i < n16; i += blockDim.x) d[i] = s[i];
    }
}

// ───────────── SwiGLU + requant + down-input quantisation for routed rows (layers.rs:609-640, :279-298) ─────────────
// The SwiGLU scales of one row (or of the whole tensor): g and u output scales, SiLU index scale, identity factor,
// as per-row plans for the element loop.
struct SwigluScales {
    Scale gs, us;
    int64_t mg, mu;  // requant divisors (0: that output is all zero)
    kt::ReqDiv rg, ru;
    kt::ApplyPlan is, idf;
    int fast;  // the row meets the conditions of the lean element path (swiglu_fast_ok)
};

// ── the lean element path ──
// A row takes it when both requant divisors admit the certified double path (2^22 <= max < 2^52), the SiLU index
// plan is tight with a shift of at least 32 and keeps every index magnitude below 2^30 for |g| <= 2^28, the identity
// tail keeps every code below 2^31, and the table's codes are held as int32. Every step is the exact arithmetic of
// the general path, written for 32-bit registers where the plan's bounds allow; a certified estimate that lands too
// near an integer falls back to the exact integer path for that element.
using kt::req_mag;   // the certified requant of a magnitude (fixed_point.cuh, where the host tests also reach it)
using kt::req_mag2;

__device__ __forceinline__ bool swiglu_fast_ok(const SwigluScales& q, const Lut& silu) {
    if (!(q.mg > 0 && q.mu > 0 && q.rg.dbl && q.ru.dbl && q.is.tight && q.idf.tight && silu.codes32)) return false;
    if (q.is.shift < 32) return false;
    const uint64_t imax = ((uint64_t(1) << 28) * q.is.mant + q.is.half) >> q.is.shift;
    const uint64_t tmax = ((uint64_t(1) << 28) * q.idf.mant + q.idf.half) >> q.idf.shift;
    const int64_t base = -silu.lo_index;
    return imax < (uint64_t(1) << 30) && tmax < (uint64_t(1) << 31) && base >= 0 && base < (int64_t(1) << 30);
}

// h = silu_code(g)·u of one element on the lean path (the same integers as swiglu_h).
__device__ __forceinline__ int64_t swiglu_h_fast(const SwigluScales& q, const int32_t* __restrict__ lut32, int32_t base,
                                                 int64_t accg, int64_t accu) {
    uint32_t qg, qu;
    const bool okg = req_mag(fabs((double)accg), q.rg.inv28, qg);
    const bool oku = req_mag(fabs((double)accu), q.ru.inv28, qu);
    int32_t g = accg < 0 ? -(int32_t)qg : (int32_t)qg;
    int32_t u = accu < 0 ? -(int32_t)qu : (int32_t)qu;
    if (!okg) g = kt::requant_row(accg, q.rg);
    if (!oku) u = kt::requant_row(accu, q.ru);
    // CodeLut::index = is.apply(g) - lo_index; with shift >= 32 the rounding shift reads the product's high word
    const uint32_t ag = (uint32_t)(g < 0 ? -g : g);
    const uint32_t r = (uint32_t)(((uint64_t)ag * q.is.mant + q.is.half) >> 32) >> (q.is.shift - 32);
    const int32_t idx = g < 0 ? base - (int32_t)r : base + (int32_t)r;
    int32_t c = __ldg(lut32 + min(max(idx, 0), LUT_N - 1));
    if (idx < 0)
        c = 0;
    else if (idx >= LUT_N)
        c = (int32_t)kt::apply_row(q.idf, g);  // identity right tail, in code units (< 2^31 by the plan)
    return (int64_t)c * (int64_t)u;
}

// swiglu_h_fast with magnitudes and signs kept apart: g is never formed as a signed value (the SiLU index needs
// only its magnitude and sign), and |h| = |code|·|u| comes from one 32x32->64 product for the row maximum.
__device__ __forceinline__ int64_t swiglu_h_fast2(const SwigluScales& q, const int32_t* __restrict__ lut32,
                                                  int32_t base, int64_t accg, int64_t accu, uint64_t& habs) {
    uint32_t qg, qu;
    const bool okg = req_mag2(fabs((double)accg), q.rg.inv28, qg);
    const bool oku = req_mag2(fabs((double)accu), q.ru.inv28, qu);
    const bool gneg = accg < 0, uneg = accu < 0;
    if (!okg) {
        const int32_t e = kt::requant_row(accg, q.rg);
        qg = (uint32_t)(e < 0 ? -e : e);
    }
    if (!oku) {
        const int32_t e = kt::requant_row(accu, q.ru);
        qu = (uint32_t)(e < 0 ? -e : e);
    }
    const uint32_t r = (uint32_t)(((uint64_t)qg * q.is.mant + q.is.half) >> 32) >> (q.is.shift - 32);
    const int32_t idx = gneg ? base - (int32_t)r : base + (int32_t)r;
    int32_t c = __ldg(lut32 + min(max(idx, 0), LUT_N - 1));
    if (idx < 0)
        c = 0;
    else if (idx >= LUT_N)
        c = (int32_t)kt::apply_row(q.idf, gneg ? -(int32_t)qg : (int32_t)qg);  // identity right tail
    habs = (uint64_t)(uint32_t)(c < 0 ? -c : c) * (uint64_t)qu;
    return (int64_t)c * (int64_t)(uneg ? -(int32_t)qu : (int32_t)qu);
}

// down_code_fast with the req_mag2 certificate.
__device__ __forceinline__ int32_t down_code_fast2(int64_t h, const kt::ReqDiv& rh) {
    uint32_t q;
    if (!req_mag2(fabs((double)h), rh.inv28, q)) {
        const int32_t e = kt::requant_row(h, rh);
        q = (uint32_t)(e < 0 ? -e : e);
    }
    const uint32_t t = (uint32_t)(((uint64_t)q * (uint64_t)kt::WLEVELS + (uint64_t(1) << 27)) >> 28);
    return h < 0 ? -(int32_t)t : (int32_t)t;
}

// requant_row(v, r) for a divisor with r.dbl, through the req_mag2 certificate (exact integer path on a miss).
__device__ __forceinline__ int32_t requant_fast(int64_t v, const kt::ReqDiv& r) {
    uint32_t q;
    if (!req_mag2(fabs((double)v), r.inv28, q)) return kt::requant_row(v, r);
    return v < 0 ? -(int32_t)q : (int32_t)q;
}

// quant_to_act(requant_row(h, rh)) on the lean path (rh.dbl): both roundings on magnitudes, the sign applied once.
__device__ __forceinline__ int32_t down_code_fast(int64_t h, const kt::ReqDiv& rh) {
    uint32_t q;
    if (!req_mag(fabs((double)h), rh.inv28, q)) {
        const int32_t e = kt::requant_row(h, rh);
        q = (uint32_t)(e < 0 ? -e : e);
    }
    const uint32_t t = (uint32_t)(((uint64_t)q * (uint64_t)kt::WLEVELS + (uint64_t(1) << 27)) >> 28);
    return h < 0 ? -(int32_t)t : (int32_t)t;
}

struct SwigluArgs {
    int64_t* acc;  // [rows][2f]: gate in [0, f), up in [f, 2f); in the tensor-global mode the gate half holds h
    int rows, f, f_pad;
    long long R_pad;  // rows of one plane of `planes`
    const int* row_assign;  // routed: row -> token·top_k + slot (nullptr: row r is token r)
    const int* row_expert;  // routed: row -> expert (nullptr: 0)
    int top_k;
    const Scale* row_sqx;   // per token (routed) ...
    const Scale* g_sqx;     // ... or one scalar for the whole tensor (shared expert)
    const Scale* wscale_g;  // [groups]
    const Scale* wscale_u;
    const Scale* wscale_d;
    Lut silu;
    Scale silu_code_scale, silu_code_scale_recip;
    int8_t* planes;  // down-GEMM input digit planes [3][R_pad][f_pad]
    Scale* row_cd;   // per row: s_qh·w_down (the down linear's c); one word in the tensor-global mode
    // |max| of the gate and up accumulators: per row ([rows][2], from the GEMM epilogue) or global ([2])
    const unsigned long long* ymax;
    int ymax_stride;  // 2 per row, 0 global
    SwigluScales* plans;         // per row ([rows]) or one for the tensor-global mode, from swiglu_plan_kernel
    unsigned long long* row_hmax;  // routed: max |h| per row, for down_c_kernel
    unsigned long long* g_hmax;  // tensor-global mode: phase 1 reduces max |h| here, phase 2 reads it
    int phase;  // 0: per-row (routed, one kernel); 1: global h pass; 2: global quantise pass
    const int* rows_dev;  // routed rows counted on the device (rows is then an upper bound), or nullptr
    // swiglu_rows_kernel only: each row's block computes the row's plan (thread 0, before its loads) and its down
    // linear's c (thread 0, at the end) itself, in place of swiglu_plan_kernel and down_c_kernel
    int inline_plan;
};

__device__ __forceinline__ int swiglu_rows(const SwigluArgs& a) { return a.rows_dev ? *a.rows_dev : a.rows; }

__device__ __forceinline__ SwigluScales swiglu_scales(const SwigluArgs& a, int t, int e, int64_t gmax_g, int64_t gmax_u) {
    SwigluScales q;
    const Scale sqx = a.g_sqx ? *a.g_sqx : a.row_sqx[t];
    const Scale cg = kt::scale_mul(sqx, a.wscale_g[e]);
    const Scale cu = kt::scale_mul(sqx, a.wscale_u[e]);
    // QuantLinear output scale: zero when c or ymax is zero (layers.rs:300-302, :321-326)
    q.gs = (cg.mant == 0 || gmax_g == 0) ? kt::scale_zero() : kt::scale_mul(kt::ratio_act(gmax_g), cg);
    q.us = (cu.mant == 0 || gmax_u == 0) ? kt::scale_zero() : kt::scale_mul(kt::ratio_act(gmax_u), cu);
    q.idf = kt::make_apply(kt::scale_mul(q.gs, a.silu_code_scale_recip));  // id_factor (layers.rs:615)
    q.is = kt::make_apply(kt::scale_mul(q.gs, a.silu.inv_step));          // CodeLut::index (kt-int lib.rs:383-385)
    q.mg = cg.mant == 0 ? 0 : gmax_g;
    q.mu = cu.mant == 0 ? 0 : gmax_u;
    q.rg = kt::make_req(q.mg);
    q.ru = kt::make_req(q.mu);
    q.fast = swiglu_fast_ok(q, a.silu) ? 1 : 0;
    return q;
}

// The per-row scale plans, one thread per row (one thread in the tensor-global mode), so that the element kernels
// start without a serial prologue.
__global__ void swiglu_plan_kernel(const SwigluArgs a) {
    kt::pdl_enter();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (a.ymax_stride == 0) {
        if (r == 0) a.plans[0] = swiglu_scales(a, 0, 0, (int64_t)a.ymax[0], (int64_t)a.ymax[1]);
        return;
    }
    if (r >= swiglu_rows(a)) return;
    const int e = a.row_expert ? a.row_expert[r] : 0;
    const int t = a.row_assign ? a.row_assign[r] / a.top_k : r;
    a.plans[r] = swiglu_scales(a, t, e, (int64_t)a.ymax[(long long)r * a.ymax_stride],
                               (int64_t)a.ymax[(long long)r * a.ymax_stride + 1]);
}

// h = silu_code(g) · u for one element (layers.rs:618-629).
__device__ __forceinline__ int64_t swiglu_h(const SwigluArgs& a, const SwigluScales& q, int64_t accg, int64_t accu) {
    const int32_t g = q.mg ? kt::requant_row(accg, q.rg) : 0;
    const int32_t u = q.mu ? kt::requant_row(accu, q.ru) : 0;
    const int64_t idx = kt::apply_row(q.is, g) - a.silu.lo_index;
    int64_t code;
    if (idx < 0)
        code = 0;
    else if (idx >= LUT_N)
        code = kt::apply_row(q.idf, g);  // identity right tail, in code units
    else
        code = a.silu.codes32 ? (int64_t)__ldg(a.silu.codes32 + idx) : __ldg(a.silu.codes + idx);
    const int32_t c32 = (int32_t)code;
    return c32 == code ? (int64_t)c32 * (int64_t)u : code * (int64_t)u;
}

// The down linear's c for a row whose h has max |h| = hmax (layers.rs:630-638 then :297-299 with xmax = 2^28).
__device__ __forceinline__ Scale down_c(const SwigluArgs& a, Scale us, int64_t hmax, int e) {
    if (hmax <= 0) return kt::scale_zero();
    const Scale h_scale = kt::scale_mul(a.silu_code_scale, us);
    const Scale hint_scale = kt::scale_mul(kt::ratio_act(hmax), h_scale);
    const Scale s_qh = kt::scale_mul(kt::from_ratio((kt::u128)kt::ACT_LEVELS, (kt::u128)kt::WLEVELS), hint_scale);
    return kt::scale_mul(s_qh, a.wscale_d[e]);
}

// Per routed row: the down linear's c from the row's plan and max |h|, one thread per row.
__global__ void down_c_kernel(const SwigluArgs a) {
    kt::pdl_enter();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= swiglu_rows(a)) return;
    const int e = a.row_expert ? a.row_expert[r] : 0;
    a.row_cd[r] = down_c(a, a.plans[r].us, (int64_t)a.row_hmax[r], e);
}

// hint = requant_dyn(h, L, hmax) has max |.| = L exactly, so the down linear's quant_to divides by 2^28.
__device__ __forceinline__ void write_down_planes(const SwigluArgs& a, int r, const int64_t* h, int64_t hmax,
                                                  bool v2 = false) {
    int8_t* p0 = a.planes + (long long)r * a.f_pad;
    int8_t* p1 = p0 + a.R_pad * a.f_pad;
    int8_t* p2 = p1 + a.R_pad * a.f_pad;
    const kt::ReqDiv rh = kt::make_req(hmax);
    if (rh.dbl && v2 && (((uintptr_t)h) & 15) == 0) {  // the lean path, four elements from two 16-byte loads
        for (int k4 = threadIdx.x * 4; k4 < a.f_pad; k4 += blockDim.x * 4) {
            int32_t q[4];
            if (k4 + 3 < a.f) {
                const longlong2 h0 = *(const longlong2*)(h + k4), h1 = *(const longlong2*)(h + k4 + 2);
                q[0] = down_code_fast2(h0.x, rh);
                q[1] = down_code_fast2(h0.y, rh);
                q[2] = down_code_fast2(h1.x, rh);
                q[3] = down_code_fast2(h1.y, rh);
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) q[j] = k4 + j < a.f ? down_code_fast2(h[k4 + j], rh) : 0;
            }
            store_digits4(p0 + k4, p1 + k4, p2 + k4, q);
        }
        return;
    }
    if (rh.dbl) {  // the lean path (2^22 <= hmax < 2^52)
        for (int k4 = threadIdx.x * 4; k4 < a.f_pad; k4 += blockDim.x * 4) {
            int32_t q[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) q[j] = k4 + j < a.f ? down_code_fast(h[k4 + j], rh) : 0;
            store_digits4(p0 + k4, p1 + k4, p2 + k4, q);
        }
        return;
    }
    for (int k4 = threadIdx.x * 4; k4 < a.f_pad; k4 += blockDim.x * 4) {
        int32_t q[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int k = k4 + j;
            q[j] = (k < a.f && hmax > 0) ? kt::quant_to_act(kt::requant_row(h[k], rh)) : 0;
        }
        store_digits4(p0 + k4, p1 + k4, p2 + k4, q);
    }
}

// Bulk prefetch of `bytes` (a multiple of 16, 16-byte aligned) at `p` into L2: a hint, nothing waits on it.
__device__ __forceinline__ void prefetch_l2(const void* p, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Phase 0: blocks walk the routed rows (row r, r + gridDim.x, ...); h stays in shared memory (dynamic, f int64) when
// `h_smem`. U independent elements per thread per step, compiled for MINB resident blocks per SM. The row's scales
// come from swiglu_plan_kernel, or with a.inline_plan from thread 0 of the row's block (then also the down linear's c,
// at the end); its max |h| goes to row_hmax. pf > 0 (element pairs): thread 0 keeps the gate and up accumulators of
// the block's next pf steps on their way into L2, so the other threads' loads meet fewer DRAM latencies.
template <int U, int MINB>
__global__ void __launch_bounds__(256, MINB) swiglu_rows_kernel(const SwigluArgs a, int h_smem, int v2, int pf) {
    kt::pdl_enter();
    extern __shared__ int64_t hs[];
    __shared__ uint64_t red[32];
    __shared__ SwigluScales q_s;
    const int n = swiglu_rows(a);
    const int f = a.f;
    for (int r = blockIdx.x; r < n; r += gridDim.x) {
        int64_t* accg = a.acc + (long long)r * 2 * f;
        const int64_t* accu = accg + f;
        if (a.inline_plan) {
            if (threadIdx.x == 0) {
                const int e = a.row_expert ? a.row_expert[r] : 0;
                const int t = a.row_assign ? a.row_assign[r] / a.top_k : r;
                q_s = swiglu_scales(a, t, e, (int64_t)a.ymax[(long long)r * a.ymax_stride],
                                    (int64_t)a.ymax[(long long)r * a.ymax_stride + 1]);
            }
            __syncthreads();
        }
        const SwigluScales q = a.inline_plan ? q_s : a.plans[r];
        int64_t* h = h_smem ? hs : accg;
        uint64_t hm = 0;
        // the loads of a step are issued before its arithmetic
        int k = threadIdx.x;
        if (q.fast && v2 && (f & 1) == 0 && (((uintptr_t)accg | (uintptr_t)h) & 15) == 0) {
            // element pairs: 16-byte loads of g and u, a 16-byte store of h
            const int32_t base = (int32_t)-a.silu.lo_index;
            const int npairs = f >> 1;
            const int step = U * blockDim.x;  // pairs per step of the block
            // pf > 0: thread 0 keeps the gate and up accumulators of the block's next pf steps on their way to L2
            if (pf > 0 && threadIdx.x == 0) {
                for (int p0 = 0; p0 < min(pf * step, npairs); p0 += step) {
                    const int n = min(step, npairs - p0);
                    prefetch_l2(accg + 2 * p0, (unsigned)n * 16);
                    prefetch_l2(accu + 2 * p0, (unsigned)n * 16);
                }
            }
            int p = threadIdx.x;
            for (; p < npairs; p += step) {
                if (pf > 0 && threadIdx.x == 0 && p + pf * step < npairs) {
                    const int p0 = p + pf * step, n = min(step, npairs - p0);
                    prefetch_l2(accg + 2 * p0, (unsigned)n * 16);
                    prefetch_l2(accu + 2 * p0, (unsigned)n * 16);
                }
                longlong2 gv[U], uv[U];
#pragma unroll
                for (int j = 0; j < U; ++j) {
                    const int pj = p + j * blockDim.x;
                    if (pj < npairs) {
                        gv[j] = __ldcs((const longlong2*)(accg + 2 * pj));
                        uv[j] = __ldcs((const longlong2*)(accu + 2 * pj));
                    }
                }
#pragma unroll
                for (int j = 0; j < U; ++j) {
                    const int pj = p + j * blockDim.x;
                    if (pj < npairs) {
                        uint64_t a0, a1;
                        longlong2 hv;
                        hv.x = swiglu_h_fast2(q, a.silu.codes32, base, gv[j].x, uv[j].x, a0);
                        hv.y = swiglu_h_fast2(q, a.silu.codes32, base, gv[j].y, uv[j].y, a1);
                        *(longlong2*)(h + 2 * pj) = hv;
                        hm = max(hm, max(a0, a1));
                    }
                }
            }
            k = f;
        }
        if (q.fast) {
            const int32_t base = (int32_t)-a.silu.lo_index;
            for (; k + (U - 1) * (int)blockDim.x < f; k += U * blockDim.x) {
                int64_t gv[U], uv[U];
#pragma unroll
                for (int j = 0; j < U; ++j) {
                    gv[j] = accg[k + j * blockDim.x];
                    uv[j] = accu[k + j * blockDim.x];
                }
#pragma unroll
                for (int j = 0; j < U; ++j) {
                    const int64_t v = swiglu_h_fast(q, a.silu.codes32, base, gv[j], uv[j]);
                    h[k + j * blockDim.x] = v;
                    hm = max(hm, uabs64(v));
                }
            }
        }
        for (; k + (U - 1) * (int)blockDim.x < f; k += U * blockDim.x) {
            int64_t gv[U], uv[U];
#pragma unroll
            for (int j = 0; j < U; ++j) {
                gv[j] = accg[k + j * blockDim.x];
                uv[j] = accu[k + j * blockDim.x];
            }
#pragma unroll
            for (int j = 0; j < U; ++j) {
                const int64_t v = swiglu_h(a, q, gv[j], uv[j]);
                h[k + j * blockDim.x] = v;
                hm = max(hm, uabs64(v));
            }
        }
        for (; k < f; k += blockDim.x) {
            const int64_t v = swiglu_h(a, q, accg[k], accu[k]);
            h[k] = v;
            hm = max(hm, uabs64(v));
        }
        const int64_t hmax = (int64_t)block_max_u64(hm, red);  // its barriers also publish h
        write_down_planes(a, r, h, hmax, v2 != 0);
        if (threadIdx.x == 0) {
            a.row_hmax[r] = (unsigned long long)hmax;
            if (a.inline_plan) a.row_cd[r] = down_c(a, q.us, hmax, a.row_expert ? a.row_expert[r] : 0);
        }
        __syncthreads();  // h, red and q_s are reused by the next row
    }
}

// ── Phase 0 on a thread-block cluster: one routed row per cluster, h in registers ──
// The C CTAs of a cluster (C = %cluster_nctarank, at most 8) split the row's f_pad / 4 groups of four elements;
// thread t of CTA c owns groups gt, gt + C·NT, ... (gt = c·NT + t), at most G of them. Each thread loads all of its
// gate and up accumulators first (16-byte loads, coalesced across the warp), turns them into h = silu_code(g)·u in
// registers (the LUT reads of a thread issued together), and reduces max |h|: over the CTA with warp shuffles, then
// over the cluster by writing each CTA's partial into slot c of every CTA's shared memory (distributed shared
// memory) between two cluster barriers. The down linear's digit planes are then written from the registers. Per
// element 16 bytes are read and 3 written, and h never leaves the SM, so a wide expert needs no row buffer: a row
// of 14336 elements is spread over 7 CTAs of 128 threads. Requires f % 4 == 0 (so the accumulator rows are 16-byte
// aligned) and f_pad <= 4·G·NT·8.
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Store v into the shared-memory word `local` (this CTA's address) of CTA `rank` of the cluster.
__device__ __forceinline__ void st_cluster_u64(uint64_t* local, uint32_t rank, uint64_t v) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(local);
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
    asm volatile("st.shared::cluster.u64 [%0], %1;" ::"r"(ra), "l"(v) : "memory");
}

template <int G, int NT>
__global__ void __launch_bounds__(NT, 2048 / (NT * G)) swiglu_cluster_kernel(const SwigluArgs a) {
    kt::pdl_enter();
    __shared__ uint64_t red[32];
    __shared__ uint64_t part[8];
    const int r = (int)cluster_id_x();
    if (r >= swiglu_rows(a)) return;  // the same for every CTA of the cluster: no barrier is left waiting
    const uint32_t C = cluster_size(), rank = cluster_rank();
    cluster_arrive_relaxed();  // every CTA of the cluster has started before any writes into another's memory
    const int f = a.f, ngroups = a.f_pad >> 2;
    const int gt = (int)rank * NT + (int)threadIdx.x, stride = (int)C * NT;
    const int64_t* accg = a.acc + (long long)r * 2 * f;
    const int64_t* accu = accg + f;

    // the accumulators' loads go out first; the row's plan is read while they are in flight
    longlong2 gv[G][2], uv[G][2];
#pragma unroll
    for (int i = 0; i < G; ++i) {
        const int k = (gt + i * stride) << 2;
        if (k < f) {
            gv[i][0] = __ldcs((const longlong2*)(accg + k));
            gv[i][1] = __ldcs((const longlong2*)(accg + k + 2));
            uv[i][0] = __ldcs((const longlong2*)(accu + k));
            uv[i][1] = __ldcs((const longlong2*)(accu + k + 2));
        } else {
            gv[i][0] = gv[i][1] = uv[i][0] = uv[i][1] = make_longlong2(0, 0);
        }
    }
    const SwigluScales q = a.plans[r];
    int64_t h[G][4];
    uint64_t hm = 0;
    if (q.fast) {
        const int32_t base = (int32_t)-a.silu.lo_index;
#pragma unroll
        for (int i = 0; i < G; ++i) {
            const int64_t gg[4] = {gv[i][0].x, gv[i][0].y, gv[i][1].x, gv[i][1].y};
            const int64_t uu[4] = {uv[i][0].x, uv[i][0].y, uv[i][1].x, uv[i][1].y};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                h[i][j] = swiglu_h_fast(q, a.silu.codes32, base, gg[j], uu[j]);
                hm = max(hm, uabs64(h[i][j]));
            }
        }
    } else {
#pragma unroll
    for (int i = 0; i < G; ++i) {
        const int64_t gg[4] = {gv[i][0].x, gv[i][0].y, gv[i][1].x, gv[i][1].y};
        const int64_t uu[4] = {uv[i][0].x, uv[i][0].y, uv[i][1].x, uv[i][1].y};
        int32_t g32[4], u32[4];
        int64_t idx[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            g32[j] = q.mg ? kt::requant_row(gg[j], q.rg) : 0;
            u32[j] = q.mu ? kt::requant_row(uu[j], q.ru) : 0;
            idx[j] = kt::apply_row(q.is, g32[j]) - a.silu.lo_index;
        }
        int64_t code[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t ix = idx[j] < 0 ? 0 : (idx[j] >= LUT_N ? LUT_N - 1 : idx[j]);
            code[j] = a.silu.codes32 ? (int64_t)__ldg(a.silu.codes32 + ix) : __ldg(a.silu.codes + ix);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int64_t c = code[j];
            if (idx[j] < 0)
                c = 0;
            else if (idx[j] >= LUT_N)
                c = kt::apply_row(q.idf, g32[j]);  // identity right tail, in code units
            const int32_t c32 = (int32_t)c;
            const int64_t v = c32 == c ? (int64_t)c32 * (int64_t)u32[j] : c * (int64_t)u32[j];
            h[i][j] = v;
            hm = max(hm, uabs64(v));
        }
    }
    }
    // max |h| over the row: the CTA, then the cluster through distributed shared memory
    const uint64_t bm = block_max_u64(hm, red);
    cluster_wait_acquire();  // (the relaxed arrive above) every CTA is running
    if (threadIdx.x == 0)
        for (uint32_t c = 0; c < C; ++c) st_cluster_u64(&part[rank], c, bm);
    cluster_arrive_release();
    cluster_wait_acquire();
    uint64_t hmu = 0;
    for (uint32_t c = 0; c < C; ++c) hmu = max(hmu, part[c]);
    const int64_t hmax = (int64_t)hmu;
    const kt::ReqDiv rh = kt::make_req(hmax);
    int8_t* p0 = a.planes + (long long)r * a.f_pad;
    int8_t* p1 = p0 + a.R_pad * a.f_pad;
    int8_t* p2 = p1 + a.R_pad * a.f_pad;
#pragma unroll
    for (int i = 0; i < G; ++i) {
        const int gi = gt + i * stride;
        if (gi >= ngroups) continue;
        const int k = gi << 2;
        int32_t qv[4];
        if (rh.dbl) {
#pragma unroll
            for (int j = 0; j < 4; ++j) qv[j] = k + j < f ? down_code_fast(h[i][j], rh) : 0;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                qv[j] = (k + j < f && hmax > 0) ? kt::quant_to_act(kt::requant_row(h[i][j], rh)) : 0;
        }
        store_digits4(p0 + k, p1 + k, p2 + k, qv);
    }
    if (rank == 0 && threadIdx.x == 0) a.row_hmax[r] = hmu;
}

// ── Phase 0 for wide rows on a cluster, h in shared memory ──
// Row r = %clusterid.x is split into C = %cluster_nctarank contiguous slices of f_pad / C elements (f_pad is a multiple
// of 128, so every slice is a multiple of 4 long); CTA c keeps its slice's h in dynamic shared memory (f_pad / C · 8
// bytes: 57 KB for Mixtral's 14336 on 2 CTAs, which leaves room for 3 CTAs per SM), so phase 2 reads h from shared
// memory instead of back from L2. The row's max |h| is reduced over the CTA, then over the cluster through distributed
// shared memory between two cluster barriers. U elements per thread per step as in swiglu_rows_kernel.
template <int U>
__global__ void __launch_bounds__(256, 3) swiglu_slice_kernel(const SwigluArgs a) {
    kt::pdl_enter();
    extern __shared__ int64_t hs[];
    __shared__ uint64_t red[32];
    __shared__ uint64_t part[8];
    const int r = (int)cluster_id_x();
    if (r >= swiglu_rows(a)) return;  // the same for every CTA of the cluster
    const uint32_t C = cluster_size(), rank = cluster_rank();
    cluster_arrive_relaxed();
    const int f = a.f, slice = a.f_pad / (int)C, k0 = (int)rank * slice;
    const int k_end = min(f, k0 + slice);  // the slice's data elements [k0, k_end); the rest is padding
    const int64_t* accg = a.acc + (long long)r * 2 * f;
    const int64_t* accu = accg + f;
    const SwigluScales q = a.plans[r];
    uint64_t hm = 0;
    int k = k0 + threadIdx.x;
    if (q.fast) {
        const int32_t base = (int32_t)-a.silu.lo_index;
        for (; k + (U - 1) * (int)blockDim.x < k_end; k += U * blockDim.x) {
            int64_t gv[U], uv[U];
#pragma unroll
            for (int j = 0; j < U; ++j) {
                gv[j] = __ldcs(accg + k + j * blockDim.x);
                uv[j] = __ldcs(accu + k + j * blockDim.x);
            }
#pragma unroll
            for (int j = 0; j < U; ++j) {
                const int64_t v = swiglu_h_fast(q, a.silu.codes32, base, gv[j], uv[j]);
                hs[k - k0 + j * blockDim.x] = v;
                hm = max(hm, uabs64(v));
            }
        }
    }
    for (; k < k_end; k += blockDim.x) {
        const int64_t v = swiglu_h(a, q, accg[k], accu[k]);
        hs[k - k0] = v;
        hm = max(hm, uabs64(v));
    }
    const uint64_t bm = block_max_u64(hm, red);  // its barriers also publish hs
    cluster_wait_acquire();
    if (threadIdx.x == 0)
        for (uint32_t c = 0; c < C; ++c) st_cluster_u64(&part[rank], c, bm);
    cluster_arrive_release();
    cluster_wait_acquire();
    uint64_t hmu = 0;
    for (uint32_t c = 0; c < C; ++c) hmu = max(hmu, part[c]);
    const int64_t hmax = (int64_t)hmu;
    const kt::ReqDiv rh = kt::make_req(hmax);
    int8_t* p0 = a.planes + (long long)r * a.f_pad;
    int8_t* p1 = p0 + a.R_pad * a.f_pad;
    int8_t* p2 = p1 + a.R_pad * a.f_pad;
    for (int k4 = k0 + threadIdx.x * 4; k4 < k0 + slice; k4 += blockDim.x * 4) {
        int32_t qv[4];
        if (rh.dbl) {
#pragma unroll
            for (int j = 0; j < 4; ++j) qv[j] = k4 + j < f ? down_code_fast(hs[k4 + j - k0], rh) : 0;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                qv[j] = (k4 + j < f && hmax > 0) ? kt::quant_to_act(kt::requant_row(hs[k4 + j - k0], rh)) : 0;
        }
        store_digits4(p0 + k4, p1 + k4, p2 + k4, qv);
    }
    if (rank == 0 && threadIdx.x == 0) a.row_hmax[r] = hmu;
}

// Phases 1 and 2: the shared expert, whose maxima are over the whole tensor (one block per row each phase; one plan).
__global__ void swiglu_global_kernel(const SwigluArgs a) {
    kt::pdl_enter();
    __shared__ uint64_t red[32];
    const int r = blockIdx.x;
    if (r >= a.rows) return;
    const int f = a.f;
    int64_t* accg = a.acc + (long long)r * 2 * f;
    const int64_t* accu = accg + f;
    if (a.phase == 1) {
        const SwigluScales q = a.plans[0];
        uint64_t hm = 0;
        if (q.fast) {
            const int32_t base = (int32_t)-a.silu.lo_index;
            for (int k = threadIdx.x; k < f; k += blockDim.x) {
                uint64_t av;
                accg[k] = swiglu_h_fast2(q, a.silu.codes32, base, accg[k], accu[k], av);
                hm = max(hm, av);
            }
        } else {
            for (int k = threadIdx.x; k < f; k += blockDim.x) {
                const int64_t v = swiglu_h(a, q, accg[k], accu[k]);
                accg[k] = v;
                hm = max(hm, uabs64(v));
            }
        }
        hm = block_max_u64(hm, red);
        if (threadIdx.x == 0 && hm) atomicMax(a.g_hmax, (unsigned long long)hm);
        return;
    }
    const int64_t hmax = (int64_t)*a.g_hmax;
    write_down_planes(a, r, accg, hmax, true);
    if (r == 0 && threadIdx.x == 0) a.row_cd[0] = down_c(a, a.plans[0].us, hmax, 0);
}

// A common scale is the LAST item whose scale value is maximal (fold `if b.ge(a) {b} else {a}`, over a token's slots
// in combine and over the tokens in merge): a reduction over (exact value, index), the larger index winning ties,
// gives the same item for any partition.
struct ScaleIdx {
    Scale s;
    int idx;
};

__device__ __forceinline__ ScaleIdx better(ScaleIdx x, ScaleIdx y) {
    const bool xy = kt::scale_ge(x.s, y.s), yx = kt::scale_ge(y.s, x.s);
    if (xy && !yx) return x;
    if (yx && !xy) return y;
    return x.idx > y.idx ? x : y;
}

// ───────────── combine: one token's selected experts → its output (layers.rs:893-923) ─────────────
struct CombineArgs {
    const int64_t* acc_d;  // [rows][dim] down accumulators (expert-sorted rows)
    const unsigned long long* ymax_d;  // [rows]: max |acc_d| of the row, from the GEMM epilogue
    const Scale* row_cd;
    const int* slot_row;   // [T][top_k] → row
    const int64_t* top_ec;
    const int64_t* sumc;
    int T, top_k, dim;
    int32_t* out;   // [T][dim]
    Scale* out_scale;  // [T]
};

constexpr int COMBINE_MAX_K = 16;

// The per-token combine plan: live slot count (-1: the token's output is zero), the common scale, and per live slot
// (packed to the front in slot order) its row, routing code, requant divisor and rescale to the common scale.
struct CombinePlan {
    int* n;             // [T]
    Scale* common;      // [T]
    int* row;           // [T][K]
    int64_t* ec;        // [T][K]
    kt::ReqDiv* ry;     // [T][K]
    kt::ApplyPlan* f;   // [T][K]
};

// One thread per token: ys_i = ratio_act(ymax_i)·c_i (zero when c_i or ymax_i is zero, layers.rs:300-302,
// :321-326), common = the last of the largest (fold with ge, layers.rs:898), and the live slots' plans.
__global__ void combine_plan_kernel(const CombineArgs a, const CombinePlan p) {
    kt::pdl_enter();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= a.T) return;
    const int K = a.top_k;
    if (a.sumc[t] <= 0) {
        p.n[t] = -1;
        return;
    }
    Scale ys[COMBINE_MAX_K];
    Scale common = kt::scale_zero();
    for (int i = 0; i < K; ++i) {
        const int row = a.slot_row[(long long)t * K + i];
        const int64_t ym = (int64_t)a.ymax_d[row];
        const Scale cd = a.row_cd[row];
        ys[i] = (cd.mant == 0 || ym == 0) ? kt::scale_zero() : kt::scale_mul(kt::ratio_act(ym), cd);
        if (kt::scale_ge(ys[i], common)) common = ys[i];
    }
    if (common.mant == 0) {
        p.n[t] = -1;
        return;
    }
    const Scale cinv = kt::scale_recip(common);
    int n = 0;
    for (int i = 0; i < K; ++i) {
        if (ys[i].mant == 0) continue;
        const long long o = (long long)t * K + n;
        const int row = a.slot_row[(long long)t * K + i];
        p.row[o] = row;
        p.ec[o] = a.top_ec[(long long)t * K + i];
        p.ry[o] = kt::make_req((int64_t)a.ymax_d[row]);
        p.f[o] = kt::make_apply(kt::scale_mul(ys[i], cinv));
        ++n;
    }
    p.n[t] = n;
    p.common[t] = common;
}

// One block per token, from its plan. A thread owns CE elements per chunk and walks the live slots: a slot's plan
// is read from shared memory once per chunk and its CE loads are in flight together.
constexpr int CE = 8;

__global__ void __launch_bounds__(256, 3) combine_kernel(const CombineArgs a, const CombinePlan p) {
    kt::pdl_enter();
    extern __shared__ int64_t acc_s[];  // [dim]
    __shared__ uint64_t red[32];
    __shared__ kt::ReqDiv ry_s[COMBINE_MAX_K];
    __shared__ kt::ApplyPlan f_s[COMBINE_MAX_K];
    __shared__ int64_t ec_s[COMBINE_MAX_K];
    __shared__ int row_s[COMBINE_MAX_K];
    const int t = blockIdx.x;
    if (t >= a.T) return;
    const int D = a.dim;
    int32_t* o = a.out + (long long)t * D;
    const int n = p.n[t];
    if (n < 0) {
        for (int d = threadIdx.x; d < D; d += blockDim.x) o[d] = 0;
        if (threadIdx.x == 0) a.out_scale[t] = kt::scale_zero();
        return;
    }
    const int K = a.top_k;
    if ((int)threadIdx.x < n) {
        const long long q = (long long)t * K + threadIdx.x;
        row_s[threadIdx.x] = p.row[q];
        ec_s[threadIdx.x] = p.ec[q];
        ry_s[threadIdx.x] = p.ry[q];
        f_s[threadIdx.x] = p.f[q];
    }
    __syncthreads();
    // the lean path when every live slot's divisor admits the certified double path, its rescale is tight and its code
    // fits 31 bits: the rescaled value (|requant| <= 2^28 times a factor of about 1 at most, the common scale being
    // the largest) then fits 32 bits and the weighting is one widening multiply
    bool lean = true;
    for (int j = 0; j < n; ++j)
        lean = lean && ry_s[j].dbl && f_s[j].tight && ec_s[j] >= 0 && ec_s[j] < (int64_t(1) << 31);
    uint64_t gm = 0;
    for (int d0 = threadIdx.x; d0 < D; d0 += CE * blockDim.x) {
        int64_t acc[CE];
#pragma unroll
        for (int u = 0; u < CE; ++u) acc[u] = 0;
        for (int j = 0; j < n; ++j) {
            const kt::ReqDiv ry = ry_s[j];
            const kt::ApplyPlan f = f_s[j];
            const int64_t ec = ec_s[j];
            const int64_t* b = a.acc_d + (long long)row_s[j] * D;
            int64_t v[CE];
#pragma unroll
            for (int u = 0; u < CE; ++u) {
                const int d = d0 + u * blockDim.x;
                v[u] = d < D ? __ldg(b + d) : 0;
            }
            if (lean) {
#pragma unroll
                for (int u = 0; u < CE; ++u)
                    acc[u] += (int64_t)(int32_t)ec * (int64_t)(int32_t)kt::apply_row(f, requant_fast(v[u], ry));
            } else {
#pragma unroll
                for (int u = 0; u < CE; ++u) acc[u] += ec * kt::apply_row(f, kt::requant_row(v[u], ry));
            }
        }
#pragma unroll
        for (int u = 0; u < CE; ++u) {
            const int d = d0 + u * blockDim.x;
            if (d < D) {
                acc_s[d] = acc[u];
                gm = max(gm, uabs64(acc[u]));
            }
        }
    }
    gm = block_max_u64(gm, red);
    const int64_t gmax = (int64_t)gm;
    const kt::ReqDiv rg = kt::make_req(gmax);
    if (rg.dbl) {
        for (int d = threadIdx.x; d < D; d += blockDim.x) o[d] = requant_fast(acc_s[d], rg);
    } else {
        for (int d = threadIdx.x; d < D; d += blockDim.x) o[d] = gmax ? kt::requant_row(acc_s[d], rg) : 0;
    }
    if (threadIdx.x == 0) {
        const int64_t sumc = a.sumc[t];
        a.out_scale[t] = gmax == 0 ? kt::scale_zero()
                                   : kt::scale_mul(kt::scale_mul(kt::ratio_act(gmax), p.common[t]),
                                                   kt::from_ratio(1, (kt::u128)(uint64_t)sumc));
    }
}

// ───────────── merge: per-token outputs → one tensor at one scale (layers.rs:1001-1019 / :866-886) ─────────────

// One block: common scale over `n` scales (index offset idx0), result + its reciprocal into out[0..1].
__global__ void common_scale_kernel(const Scale* __restrict__ scales, int n, int idx0, Scale* __restrict__ out,
                                    int* __restrict__ out_idx, const int* __restrict__ idx0_dev = nullptr) {
    kt::pdl_enter();
    __shared__ ScaleIdx sm[1024];
    if (idx0_dev) idx0 = *idx0_dev;
    ScaleIdx b{kt::scale_zero(), -1};
    for (int i = threadIdx.x; i < n; i += blockDim.x) b = better(b, ScaleIdx{scales[i], idx0 + i});
    sm[threadIdx.x] = b;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) sm[threadIdx.x] = better(sm[threadIdx.x], sm[threadIdx.x + s]);
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const Scale c = sm[0].s;
        out[0] = c;
        out[1] = c.mant ? kt::scale_recip(c) : kt::scale_zero();
        if (out_idx) *out_idx = sm[0].idx;
    }
}

// Pass 1 of the merge: max over all tokens of |f_t.apply(o_t[d])| (atomicMax into *gmax).
__global__ void merge_max_kernel(const int32_t* __restrict__ o, const Scale* __restrict__ o_scale, int T, int D,
                                 const Scale* __restrict__ common, unsigned long long* __restrict__ gmax) {
    kt::pdl_enter();
    __shared__ uint64_t red[32];
    const int t = blockIdx.x;
    if (t >= T) return;
    const Scale cinv = common[1];
    if (common[0].mant == 0) return;
    const kt::ApplyPlan f = kt::make_apply(kt::scale_mul(o_scale[t], cinv));
    const int32_t* ot = o + (long long)t * D;
    uint64_t m = 0;
    if ((D & 3) == 0 && ((uintptr_t)o & 15) == 0) {
        for (int d = threadIdx.x * 4; d < D; d += blockDim.x * 4) {
            const int4 v = __ldg((const int4*)(ot + d));
            m = max(max(m, uabs64(kt::apply_row(f, v.x))), uabs64(kt::apply_row(f, v.y)));
            m = max(max(m, uabs64(kt::apply_row(f, v.z))), uabs64(kt::apply_row(f, v.w)));
        }
    } else {
        for (int d = threadIdx.x; d < D; d += blockDim.x) m = max(m, uabs64(kt::apply_row(f, ot[d])));
    }
    m = block_max_u64(m, red);
    if (threadIdx.x == 0 && m) atomicMax(gmax, (unsigned long long)m);
}

// Pass 2: y = requant_dyn(f_t.apply(o_t), L, gmax); scale = from_ratio(gmax, L)·common.
__global__ void merge_final_kernel(const int32_t* __restrict__ o, const Scale* __restrict__ o_scale, int T, int D,
                                   const Scale* __restrict__ common, const unsigned long long* __restrict__ gmax_p,
                                   int32_t* __restrict__ y, Scale* __restrict__ y_scale,
                                   const int* __restrict__ t_total = nullptr) {
    kt::pdl_enter();
    const int t = blockIdx.x;
    if (t >= T) return;
    if (t_total && *t_total == 1) {
        // one token in the whole layer: the routed output is its combine output (layers.rs:992-994)
        for (int d = threadIdx.x; d < D; d += blockDim.x) y[(long long)t * D + d] = o[(long long)t * D + d];
        if (threadIdx.x == 0) *y_scale = o_scale[t];
        return;
    }
    const int64_t gmax = (int64_t)*gmax_p;
    const bool zero = common[0].mant == 0 || gmax == 0;
    const kt::ApplyPlan f = kt::make_apply(zero ? kt::scale_zero() : kt::scale_mul(o_scale[t], common[1]));
    const kt::ReqDiv rg = kt::make_req(gmax);
    const int32_t* ot = o + (long long)t * D;
    int32_t* yt = y + (long long)t * D;
    if ((D & 3) == 0 && (((uintptr_t)o | (uintptr_t)y) & 15) == 0) {
        for (int d = threadIdx.x * 4; d < D; d += blockDim.x * 4) {
            int4 r = make_int4(0, 0, 0, 0);
            if (!zero) {
                const int4 v = __ldg((const int4*)(ot + d));
                if (rg.dbl) {  // the certified double path through the two-estimate test
                    r.x = requant_fast(kt::apply_row(f, v.x), rg);
                    r.y = requant_fast(kt::apply_row(f, v.y), rg);
                    r.z = requant_fast(kt::apply_row(f, v.z), rg);
                    r.w = requant_fast(kt::apply_row(f, v.w), rg);
                } else {
                    r.x = kt::requant_row(kt::apply_row(f, v.x), rg);
                    r.y = kt::requant_row(kt::apply_row(f, v.y), rg);
                    r.z = kt::requant_row(kt::apply_row(f, v.z), rg);
                    r.w = kt::requant_row(kt::apply_row(f, v.w), rg);
                }
            }
            *(int4*)(yt + d) = r;
        }
    } else {
        for (int d = threadIdx.x; d < D; d += blockDim.x) yt[d] = zero ? 0 : kt::requant_row(kt::apply_row(f, ot[d]), rg);
    }
    if (t == 0 && threadIdx.x == 0) *y_scale = zero ? kt::scale_zero() : kt::scale_mul(kt::ratio_act(gmax), common[0]);
}

// One token (rows == 1): the routed output is the combine output itself (layers.rs:992-994).
__global__ void copy_row_kernel(const int32_t* __restrict__ o, const Scale* __restrict__ os, int D, int32_t* __restrict__ y,
                                Scale* __restrict__ ys) {
    kt::pdl_enter();
    for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < D; d += gridDim.x * blockDim.x) y[d] = o[d];
    if (blockIdx.x == 0 && threadIdx.x == 0) *ys = os[0];
}

// ───────────── shared expert output and the final add (layers.rs:758-780, :121-136) ─────────────
// Shared output: y_s = requant_dyn(acc, L, ymax) at scale from_ratio(ymax, L)·c_d, with ymax over the whole tensor.
// add(routed, shared): common = routed.scale.ge(shared.scale) ? routed : shared.
struct AddArgs {
    const int32_t* a;  // routed [n]
    const Scale* a_scale;
    const int64_t* s_acc;  // shared down accumulators [n]
    const unsigned long long* s_ymax;
    const Scale* s_cd;  // shared down c (row_cd[0])
    long long n;
    unsigned long long* gmax;  // pass 1 out / pass 2 in
    Scale* scratch;            // [0] shared scale, [1] common, [2] fa, [3] fb
    int32_t* y;
    Scale* y_scale;
};

__global__ void add_prepare_kernel(const AddArgs p) {
    kt::pdl_enter();
    const int64_t ymax = (int64_t)*p.s_ymax;
    const Scale cd = *p.s_cd;
    const Scale ss = (cd.mant == 0 || ymax == 0) ? kt::scale_zero() : kt::scale_mul(kt::ratio_act(ymax), cd);
    const Scale as = *p.a_scale;
    const Scale common = kt::scale_ge(as, ss) ? as : ss;
    p.scratch[0] = ss;
    p.scratch[1] = common;
    if (common.mant) {
        const Scale cinv = kt::scale_recip(common);
        p.scratch[2] = kt::scale_mul(as, cinv);
        p.scratch[3] = kt::scale_mul(ss, cinv);
    } else {
        p.scratch[2] = p.scratch[3] = kt::scale_zero();
    }
}

__device__ __forceinline__ int64_t add_sum(const AddArgs& p, long long i, const kt::ApplyPlan& fa,
                                           const kt::ApplyPlan& fb, const kt::ReqDiv& ry, int64_t ymax) {
    const int32_t sv = ymax ? kt::requant_row(p.s_acc[i], ry) : 0;
    return kt::apply_row(fa, p.a[i]) + kt::apply_row(fb, sv);
}

// Four consecutive elements from i (i a multiple of 4; the buffers are 16-byte aligned): a as one int4, the shared
// accumulators as two 16-byte loads.
__device__ __forceinline__ void add_sum4(const AddArgs& p, long long i, const kt::ApplyPlan& fa,
                                         const kt::ApplyPlan& fb, const kt::ReqDiv& ry, int64_t ymax, int64_t (&out)[4]) {
    const int4 av = __ldg((const int4*)(p.a + i));
    const longlong2 s0 = __ldg((const longlong2*)(p.s_acc + i));
    const longlong2 s1 = __ldg((const longlong2*)(p.s_acc + i + 2));
    const int64_t sv[4] = {s0.x, s0.y, s1.x, s1.y};
    const int32_t a4[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
        out[j] = kt::apply_row(fa, a4[j]) + kt::apply_row(fb, ymax ? kt::requant_row(sv[j], ry) : 0);
}

__global__ void add_max_kernel(const AddArgs p) {
    kt::pdl_enter();
    __shared__ uint64_t red[32];
    const kt::ApplyPlan fa = kt::make_apply(p.scratch[2]), fb = kt::make_apply(p.scratch[3]);
    const int64_t ymax = (int64_t)*p.s_ymax;
    const kt::ReqDiv ry = kt::make_req(ymax);
    uint64_t m = 0;
    if (p.scratch[1].mant) {
        const bool vec = (((uintptr_t)p.a | (uintptr_t)p.s_acc) & 15) == 0;
        const long long n4 = vec ? p.n & ~3LL : 0, stride = (long long)gridDim.x * blockDim.x;
        for (long long i = (blockIdx.x * (long long)blockDim.x + threadIdx.x) * 4; i < n4; i += stride * 4) {
            int64_t v[4];
            add_sum4(p, i, fa, fb, ry, ymax, v);
            m = max(max(m, max(uabs64(v[0]), uabs64(v[1]))), max(uabs64(v[2]), uabs64(v[3])));
        }
        for (long long i = n4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < p.n; i += stride)
            m = max(m, uabs64(add_sum(p, i, fa, fb, ry, ymax)));
    }
    m = block_max_u64(m, red);
    if (threadIdx.x == 0 && m) atomicMax(p.gmax, (unsigned long long)m);
}

__global__ void add_final_kernel(const AddArgs p) {
    kt::pdl_enter();
    const kt::ApplyPlan fa = kt::make_apply(p.scratch[2]), fb = kt::make_apply(p.scratch[3]);
    const Scale common = p.scratch[1];
    const int64_t ymax = (int64_t)*p.s_ymax;
    const int64_t gmax = (int64_t)*p.gmax;
    const kt::ReqDiv ry = kt::make_req(ymax), rg = kt::make_req(gmax);
    const bool zero = common.mant == 0 || gmax == 0;
    const bool vec = (((uintptr_t)p.a | (uintptr_t)p.s_acc | (uintptr_t)p.y) & 15) == 0;
    const long long n4 = vec ? p.n & ~3LL : 0, stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (blockIdx.x * (long long)blockDim.x + threadIdx.x) * 4; i < n4; i += stride * 4) {
        int4 r = make_int4(0, 0, 0, 0);
        if (!zero) {
            int64_t v[4];
            add_sum4(p, i, fa, fb, ry, ymax, v);
            r.x = kt::requant_row(v[0], rg);
            r.y = kt::requant_row(v[1], rg);
            r.z = kt::requant_row(v[2], rg);
            r.w = kt::requant_row(v[3], rg);
        }
        *(int4*)(p.y + i) = r;
    }
    for (long long i = n4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < p.n; i += stride)
        p.y[i] = zero ? 0 : kt::requant_row(add_sum(p, i, fa, fb, ry, ymax), rg);
    if (blockIdx.x == 0 && threadIdx.x == 0) *p.y_scale = zero ? kt::scale_zero() : kt::scale_mul(kt::ratio_act(gmax), common);
}

// ───────────── the FFN half of a decoder block: x + moe(rms_norm(x)) (kt-core model.rs:175-181) ─────────────
// RmsNorm (layers.rs:352-449): per row C_r = x.scale·rsqrt(mean(x²)·x.scale² + eps)·w_scale, p = x_i·wcode_i; all
// rows to the common (last largest) C, one dynamic requant over the whole tensor.

// One block per row: the row's C (the sum of squares in 128 bits, as the reference's i128).
__global__ void rms_rows_kernel(const int32_t* __restrict__ x, int rows, int dim, const Scale* __restrict__ x_scale,
                                Scale w_scale, Scale eps_scale, Scale* __restrict__ c) {
    kt::pdl_enter();
    __shared__ unsigned long long part[2][256];
    const int r = blockIdx.x;
    if (r >= rows) return;
    const int32_t* xr = x + (long long)r * dim;
    kt::u128 ss = 0;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ss += (kt::u128)((int64_t)xr[i] * (int64_t)xr[i]);
    part[0][threadIdx.x] = (unsigned long long)ss;
    part[1][threadIdx.x] = (unsigned long long)(ss >> 64);
    __syncthreads();
    if (threadIdx.x == 0) {
        kt::u128 t = 0;
        for (int i = 0; i < (int)blockDim.x; ++i) t += ((kt::u128)part[1][i] << 64) | part[0][i];
        const Scale xs = *x_scale;
        const Scale mean_sq = kt::scale_mul(kt::scale_mul(kt::from_ratio(t, (kt::u128)dim), xs), xs);
        const Scale denom = kt::scale_add(mean_sq, eps_scale);
        const Scale inv = denom.mant == 0 ? kt::scale_zero() : kt::scale_rsqrt(denom);
        c[r] = kt::scale_mul(kt::scale_mul(xs, inv), w_scale);
    }
}

// Pass 1: max over the tensor of |f_r.apply(x_i·wcode_i)|, f_r = C_r·common⁻¹ (atomicMax into *gmax).
__global__ void rms_max_kernel(const int32_t* __restrict__ x, const int32_t* __restrict__ wcodes, int rows, int dim,
                               const Scale* __restrict__ c, const Scale* __restrict__ common,
                               unsigned long long* __restrict__ gmax) {
    kt::pdl_enter();
    __shared__ uint64_t red[32];
    const int r = blockIdx.x;
    if (r >= rows || common[0].mant == 0) return;
    const kt::ApplyPlan f = kt::make_apply(kt::scale_mul(c[r], common[1]));
    const int32_t* xr = x + (long long)r * dim;
    uint64_t m = 0;
    for (int i = threadIdx.x; i < dim; i += blockDim.x)
        m = max(m, uabs64(kt::apply_row_wide(f, (int64_t)xr[i] * (int64_t)wcodes[i])));
    m = block_max_u64(m, red);
    if (threadIdx.x == 0 && m) atomicMax(gmax, (unsigned long long)m);
}

// Pass 2: y = requant_dyn(f_r.apply(x_i·wcode_i), L, gmax); scale = from_ratio(gmax, L)·common.
__global__ void rms_final_kernel(const int32_t* __restrict__ x, const int32_t* __restrict__ wcodes, int rows, int dim,
                                 const Scale* __restrict__ c, const Scale* __restrict__ common,
                                 const unsigned long long* __restrict__ gmax_p, int32_t* __restrict__ y) {
    kt::pdl_enter();
    const int r = blockIdx.x;
    if (r >= rows) return;
    const int64_t gmax = (int64_t)*gmax_p;
    const bool zero = common[0].mant == 0 || gmax == 0;
    int32_t* yr = y + (long long)r * dim;
    if (zero) {
        for (int i = threadIdx.x; i < dim; i += blockDim.x) yr[i] = 0;
    } else {
        const kt::ApplyPlan f = kt::make_apply(kt::scale_mul(c[r], common[1]));
        const kt::ReqDiv rg = kt::make_req(gmax);
        const int32_t* xr = x + (long long)r * dim;
        for (int i = threadIdx.x; i < dim; i += blockDim.x)
            yr[i] = kt::requant_row(kt::apply_row_wide(f, (int64_t)xr[i] * (int64_t)wcodes[i]), rg);
    }
}

// The scale of a dynamic requant over a whole tensor: from_ratio(gmax, L)·common (zero when either is).
__global__ void gmax_scale_kernel(const Scale* __restrict__ common, const unsigned long long* __restrict__ gmax_p,
                                  Scale* __restrict__ out) {
    kt::pdl_enter();
    const int64_t gmax = (int64_t)*gmax_p;
    *out = (common[0].mant == 0 || gmax == 0) ? kt::scale_zero() : kt::scale_mul(kt::ratio_act(gmax), common[0]);
}

// add(a, b) of two activations (layers.rs:121-136): common = a.scale.ge(b.scale) ? a : b; sum = fa.apply(a) +
// fb.apply(b); one dynamic requant over the tensor. `plan` holds {common, fa, fb}.
__global__ void add2_prepare_kernel(const Scale* __restrict__ a_scale, const Scale* __restrict__ b_scale,
                                    Scale* __restrict__ plan) {
    kt::pdl_enter();
    const Scale as = *a_scale, bs = *b_scale;
    const Scale common = kt::scale_ge(as, bs) ? as : bs;
    plan[0] = common;
    if (common.mant) {
        const Scale cinv = kt::scale_recip(common);
        plan[1] = kt::scale_mul(as, cinv);
        plan[2] = kt::scale_mul(bs, cinv);
    } else {
        plan[1] = plan[2] = kt::scale_zero();
    }
}

__global__ void add2_max_kernel(const int32_t* __restrict__ a, const int32_t* __restrict__ b, long long n,
                                const Scale* __restrict__ plan, unsigned long long* __restrict__ gmax) {
    kt::pdl_enter();
    __shared__ uint64_t red[32];
    const kt::ApplyPlan fa = kt::make_apply(plan[1]), fb = kt::make_apply(plan[2]);
    uint64_t m = 0;
    if (plan[0].mant)
        for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
            m = max(m, uabs64(kt::apply_row(fa, a[i]) + kt::apply_row(fb, b[i])));
    m = block_max_u64(m, red);
    if (threadIdx.x == 0 && m) atomicMax(gmax, (unsigned long long)m);
}

__global__ void add2_final_kernel(const int32_t* __restrict__ a, const int32_t* __restrict__ b, long long n,
                                  const Scale* __restrict__ plan, const unsigned long long* __restrict__ gmax_p,
                                  int32_t* __restrict__ y) {
    kt::pdl_enter();
    const kt::ApplyPlan fa = kt::make_apply(plan[1]), fb = kt::make_apply(plan[2]);
    const int64_t gmax = (int64_t)*gmax_p;
    const bool zero = plan[0].mant == 0 || gmax == 0;
    const kt::ReqDiv rg = kt::make_req(gmax);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        y[i] = zero ? 0 : kt::requant_row(kt::apply_row(fa, a[i]) + kt::apply_row(fb, b[i]), rg);
}

// ───────────── extension: the sigmoid-gated shared expert (Qwen2-MoE's shared_expert_gate) ─────────────
// The reference refuses this path (crates/03-models/kt-model-moe/src/lib.rs:152-154); it is defined here in the
// reference's own terms and restated in the CPU oracle: gate = QuantLinear [1, d] on the whole input (tensor-global
// xmax and ymax, layers.rs:275-328), code_t = sigmoid CodeLut at the token's logit (router.rs:37-51), and the shared
// output y becomes requant_dyn(code_t·y[t, j], L, max |.|) at scale ratio(gmax)·y.scale·code_scale before add.

// Gate logit accumulators acc[t] = sum_k qx[t, k]·w[k] from the shared expert's input planes, which hold the
// tensor-global quant_to of x — the gate linear's own input quantisation (layers.rs:297-298). One warp per token,
// 16 elements per lane step (w is zero-padded to d_pad like the planes); max |acc| into *ymax.
__global__ void gate_logit_kernel(const int8_t* __restrict__ planes, int T, int d_pad, long long R_pad,
                                  const int32_t* __restrict__ w, int64_t* __restrict__ acc,
                                  unsigned long long* __restrict__ ymax) {
    kt::pdl_enter();
    const int t = (int)((blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (t >= T) return;
    const int8_t* p0 = planes + (long long)t * d_pad;
    const int8_t* p1 = p0 + R_pad * d_pad;
    const int8_t* p2 = p1 + R_pad * d_pad;
    int64_t s = 0;
    for (int k = lane * 16; k < d_pad; k += 32 * 16) {
        const int4 a0 = __ldg((const int4*)(p0 + k)), a1 = __ldg((const int4*)(p1 + k)), a2 = __ldg((const int4*)(p2 + k));
        const int8_t* b0 = (const int8_t*)&a0;
        const int8_t* b1 = (const int8_t*)&a1;
        const int8_t* b2 = (const int8_t*)&a2;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int32_t q = (int32_t)b0[j] + 81 * (int32_t)b1[j] + 6561 * (int32_t)b2[j];
            s += (int64_t)q * (int64_t)__ldg(w + k + j);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) {
        acc[t] = s;
        if (s) atomicMax(ymax, (unsigned long long)uabs64(s));
    }
}

// One thread per token: the gate linear's output (logit = requant_dyn(acc, L, ymax) at ratio(ymax)·s_qx·w_scale, or
// zeros when that scale or ymax is zero, layers.rs:300-326) and its sigmoid code code_at(index(logit, scale)).
__global__ void gate_code_kernel(const int64_t* __restrict__ acc, int T, const unsigned long long* __restrict__ ymax_p,
                                 const Scale* __restrict__ sqx, Scale w_scale, Lut sig, int64_t* __restrict__ code) {
    kt::pdl_enter();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    const int64_t ymax = (int64_t)*ymax_p;
    const Scale c = kt::scale_mul(*sqx, w_scale);
    const bool zero = c.mant == 0 || ymax == 0;
    const Scale ls = zero ? kt::scale_zero() : kt::scale_mul(kt::ratio_act(ymax), c);
    const int32_t logit = zero ? 0 : kt::requant_act(acc[t], ymax);
    int64_t idx = kt::scale_apply(kt::scale_mul(ls, sig.inv_step), (int64_t)logit) - sig.lo_index;
    idx = idx < 0 ? 0 : (idx > LUT_N - 1 ? LUT_N - 1 : idx);
    code[t] = sig.codes[idx];
}

struct GateArgs {
    const int64_t* s_acc;  // shared down accumulators [T][d]
    const unsigned long long* s_ymax;
    const Scale* s_cd;       // shared down c
    const int64_t* code;     // [T] sigmoid codes
    int T, d;
    unsigned long long* gmax;  // pass 1 out / pass 2 in
    Scale code_scale;          // the sigmoid table's code scale (2^-20)
    int32_t* y;                // [T][d] the gated shared output
    Scale* y_scale;
};

// The shared expert's output element i (SwiGluMlp's down QuantLinear: requant_dyn(acc, L, ymax), zero when its
// scale is zero) times the token's code.
__device__ __forceinline__ int64_t gated_value(const GateArgs& p, bool live, const kt::ReqDiv& ry, int64_t c,
                                               int64_t acc) {
    return live ? c * (int64_t)kt::requant_row(acc, ry) : 0;
}

// Pass 1 (one block per token): max |code_t·y[t, j]| into *gmax.
__global__ void gated_max_kernel(const GateArgs p) {
    kt::pdl_enter();
    __shared__ uint64_t red[32];
    const int t = blockIdx.x;
    if (t >= p.T) return;
    const int64_t ymax = (int64_t)*p.s_ymax;
    const bool live = ymax != 0 && p.s_cd->mant != 0;
    const kt::ReqDiv ry = kt::make_req(ymax);
    const int64_t c = p.code[t];
    const int64_t* a = p.s_acc + (long long)t * p.d;
    uint64_t m = 0;
    for (int j = threadIdx.x; j < p.d; j += blockDim.x) m = max(m, uabs64(gated_value(p, live, ry, c, a[j])));
    m = block_max_u64(m, red);
    if (threadIdx.x == 0 && m) atomicMax(p.gmax, (unsigned long long)m);
}

// Pass 2: y[t, j] = requant_dyn(code_t·y_s[t, j], L, gmax); scale = ratio(gmax)·y_s.scale·code_scale.
__global__ void gated_final_kernel(const GateArgs p) {
    kt::pdl_enter();
    const int t = blockIdx.x;
    if (t >= p.T) return;
    const int64_t ymax = (int64_t)*p.s_ymax, gmax = (int64_t)*p.gmax;
    const Scale cd = *p.s_cd;
    const bool live = ymax != 0 && cd.mant != 0;
    const kt::ReqDiv ry = kt::make_req(ymax), rg = kt::make_req(gmax);
    const int64_t c = p.code[t];
    const int64_t* a = p.s_acc + (long long)t * p.d;
    int32_t* y = p.y + (long long)t * p.d;
    for (int j = threadIdx.x; j < p.d; j += blockDim.x)
        y[j] = gmax ? kt::requant_row(gated_value(p, live, ry, c, a[j]), rg) : 0;
    if (t == 0 && threadIdx.x == 0) {
        const Scale ys = live ? kt::scale_mul(kt::ratio_act(ymax), cd) : kt::scale_zero();
        *p.y_scale = gmax == 0 ? kt::scale_zero() : kt::scale_mul(kt::scale_mul(kt::ratio_act(gmax), ys), p.code_scale);
    }
}

// The first global row of this rank from every rank's row count ([world] u64, rank order).
__global__ void row_offset_kernel(const unsigned long long* __restrict__ counts, int rank, int* __restrict__ offset) {
    kt::pdl_enter();
    int o = 0;
    for (int q = 0; q < rank; ++q) o += (int)counts[q];
    *offset = o;
}

// ───────────── expert parallelism: the exchange around the routed experts ─────────────
// A home rank sends, for every (token, slot) row in expert order, the row's digit planes and its s_qx; the owner of
// the expert returns the expert's output as the reference's seam returns it (an IntTensor: i32 data + Scale,
// crates/01-engine/kt-core/src/layers.rs:945-984), and the home combines. combine depends only on (ec, ys, scales), so
// the placement of the experts cannot change a bit (layers.rs:888-892).

// meta[pos] = s_qx of the token of expert-sorted row pos (as {mant, shift} int64 pairs).
__global__ void pack_meta_kernel(const int* __restrict__ row_assign, int top_k, const Scale* __restrict__ tok_sqx,
                                 int n_rows, int64_t* __restrict__ meta) {
    kt::pdl_enter();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n_rows) return;
    const Scale s = tok_sqx[row_assign[r] / top_k];
    meta[2 * (long long)r] = s.mant;
    meta[2 * (long long)r + 1] = s.shift;
}

__global__ void meta_to_scale_kernel(const int64_t* __restrict__ meta, int n_rows, Scale* __restrict__ out) {
    kt::pdl_enter();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n_rows) return;
    out[r] = Scale{meta[2 * (long long)r], (int32_t)meta[2 * (long long)r + 1]};
}

// row_expert for received rows: run i covers rows [start[i], start[i] + count[i]) of local expert group[i].
__global__ void runs_to_rows_kernel(const int* __restrict__ start, const int* __restrict__ count,
                                    const int* __restrict__ group, int n_runs, int* __restrict__ row_expert) {
    kt::pdl_enter();
    const int i = blockIdx.x;
    if (i >= n_runs) return;
    for (int j = threadIdx.x; j < count[i]; j += blockDim.x) row_expert[start[i] + j] = group[i];
}

// The expert's output as an IntTensor: y = requant_dyn(acc, L, ymax), scale = from_ratio(ymax, L)·c (layers.rs:321-327).
__global__ void expert_out_kernel(const int64_t* __restrict__ acc, const unsigned long long* __restrict__ ymax_d,
                                  const Scale* __restrict__ row_cd, int n_rows, int D, int32_t* __restrict__ y,
                                  Scale* __restrict__ ys) {
    kt::pdl_enter();
    const int r = blockIdx.x;
    if (r >= n_rows) return;
    const int64_t ymax = (int64_t)ymax_d[r];
    const Scale cd = row_cd[r];
    const bool zero = ymax == 0 || cd.mant == 0;
    const kt::ReqDiv rq = kt::make_req(ymax);
    for (int d = threadIdx.x; d < D; d += blockDim.x)
        y[(long long)r * D + d] = zero ? 0 : kt::requant_row(acc[(long long)r * D + d], rq);
    if (threadIdx.x == 0) ys[r] = zero ? kt::scale_zero() : kt::scale_mul(kt::ratio_act(ymax), cd);
}

// The seam's worker side: the expert outputs of one chunk of at most K requested experts per row. Expert-sorted row
// r is assignment a = row_assign[r] = t·K + slot; slot < Kc is request (t, j0 + slot) of the n_ids per row, written to
// y[(t·n_ids + j0 + slot)·D ..] and ys[..] as expert_out_kernel does; a request with id < 0 (an empty slot that ran on
// a stand-in expert) gets zeros and a zero scale.
__global__ void seam_out_kernel(const int64_t* __restrict__ acc, const unsigned long long* __restrict__ ymax_d,
                                const Scale* __restrict__ row_cd, const int* __restrict__ row_assign, int n_rows, int D,
                                int K, int Kc, int n_ids, int j0, const int32_t* __restrict__ ids,
                                int32_t* __restrict__ y, Scale* __restrict__ ys) {
    kt::pdl_enter();
    const int r = blockIdx.x;
    if (r >= n_rows) return;
    const int a = row_assign[r], t = a / K, slot = a % K;
    if (slot >= Kc) return;
    const long long o = (long long)t * n_ids + j0 + slot;
    const int64_t ymax = (int64_t)ymax_d[r];
    const Scale cd = row_cd[r];
    const bool zero = ids[o] < 0 || ymax == 0 || cd.mant == 0;
    const kt::ReqDiv rq = kt::make_req(zero ? 1 : ymax);
    for (int d = threadIdx.x; d < D; d += blockDim.x)
        y[o * D + d] = zero ? 0 : kt::requant_row(acc[(long long)r * D + d], rq);
    if (threadIdx.x == 0) ys[o] = zero ? kt::scale_zero() : kt::scale_mul(kt::ratio_act(ymax), cd);
}

__global__ void iota_kernel(int* __restrict__ p, long long n) {
    kt::pdl_enter();
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        p[i] = (int)i;
}

// combine (layers.rs:893-923) from expert outputs given as IntTensors (y rows + scales), row = slot_row[t·K + i].
struct CombineYArgs {
    const int32_t* y;
    const Scale* ys;
    const int* slot_row;
    const int64_t* top_ec;
    const int64_t* sumc;
    int T, top_k, dim;
    int32_t* out;
    Scale* out_scale;
};

// One thread per token: the plan of combine from expert outputs given as IntTensors (their scales are final, so each
// live slot needs only its rescale to the common scale); the same CombinePlan layout (ry unused).
__global__ void combine_y_plan_kernel(const CombineYArgs a, const CombinePlan p) {
    kt::pdl_enter();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= a.T) return;
    const int K = a.top_k;
    if (a.sumc[t] <= 0) {
        p.n[t] = -1;
        return;
    }
    Scale common = kt::scale_zero();
    for (int i = 0; i < K; ++i) {
        const Scale ys = a.ys[a.slot_row[(long long)t * K + i]];
        if (kt::scale_ge(ys, common)) common = ys;
    }
    if (common.mant == 0) {
        p.n[t] = -1;
        return;
    }
    const Scale cinv = kt::scale_recip(common);
    int n = 0;
    for (int i = 0; i < K; ++i) {
        const int row = a.slot_row[(long long)t * K + i];
        const Scale ys = a.ys[row];
        if (ys.mant == 0) continue;
        const long long o = (long long)t * K + n;
        p.row[o] = row;
        p.ec[o] = a.top_ec[(long long)t * K + i];
        p.f[o] = kt::make_apply(kt::scale_mul(ys, cinv));
        ++n;
    }
    p.n[t] = n;
    p.common[t] = common;
}

// combine (layers.rs:893-923) from expert outputs given as IntTensors (y rows + scales), row = slot_row[t·K + i]: one
// block per token from its plan, each thread CE elements per chunk, one slot's plan at a time.
__global__ void __launch_bounds__(256, 3) combine_y_kernel(const CombineYArgs a, const CombinePlan p) {
    kt::pdl_enter();
    extern __shared__ int64_t acc_s[];  // [dim]
    __shared__ uint64_t red[32];
    __shared__ kt::ApplyPlan f_s[COMBINE_MAX_K];
    __shared__ int64_t ec_s[COMBINE_MAX_K];
    __shared__ int row_s[COMBINE_MAX_K];
    const int t = blockIdx.x;
    if (t >= a.T) return;
    const int D = a.dim;
    int32_t* o = a.out + (long long)t * D;
    const int n = p.n[t];
    if (n < 0) {
        for (int d = threadIdx.x; d < D; d += blockDim.x) o[d] = 0;
        if (threadIdx.x == 0) a.out_scale[t] = kt::scale_zero();
        return;
    }
    const int K = a.top_k;
    if ((int)threadIdx.x < n) {
        const long long q = (long long)t * K + threadIdx.x;
        row_s[threadIdx.x] = p.row[q];
        ec_s[threadIdx.x] = p.ec[q];
        f_s[threadIdx.x] = p.f[q];
    }
    __syncthreads();
    uint64_t gm = 0;
    for (int d0 = threadIdx.x; d0 < D; d0 += CE * blockDim.x) {
        int64_t acc[CE];
#pragma unroll
        for (int u = 0; u < CE; ++u) acc[u] = 0;
        for (int j = 0; j < n; ++j) {
            const kt::ApplyPlan f = f_s[j];
            const int64_t ec = ec_s[j];
            const int32_t* b = a.y + (long long)row_s[j] * D;
            int32_t v[CE];
#pragma unroll
            for (int u = 0; u < CE; ++u) {
                const int d = d0 + u * blockDim.x;
                v[u] = d < D ? __ldg(b + d) : 0;
            }
#pragma unroll
            for (int u = 0; u < CE; ++u) acc[u] += ec * kt::apply_row(f, v[u]);
        }
#pragma unroll
        for (int u = 0; u < CE; ++u) {
            const int d = d0 + u * blockDim.x;
            if (d < D) {
                acc_s[d] = acc[u];
                gm = max(gm, uabs64(acc[u]));
            }
        }
    }
    gm = block_max_u64(gm, red);
    const int64_t gmax = (int64_t)gm;
    const kt::ReqDiv rg = kt::make_req(gmax);
    for (int d = threadIdx.x; d < D; d += blockDim.x) o[d] = gmax ? kt::requant_row(acc_s[d], rg) : 0;
    if (threadIdx.x == 0) {
        const int64_t sumc = a.sumc[t];
        a.out_scale[t] = gmax == 0 ? kt::scale_zero()
                                   : kt::scale_mul(kt::scale_mul(kt::ratio_act(gmax), p.common[t]),
                                                   kt::from_ratio(1, (kt::u128)(uint64_t)sumc));
    }
}

// ───────────── combine with a warp per token's plan, one token over a cluster ─────────────
// The same arithmetic as combine_plan_kernel / combine_kernel (Y = false: the down accumulators) and
// combine_y_plan_kernel / combine_y_kernel (Y = true: expert outputs given as IntTensors), arranged for latency:
// the plan is one warp per token with lane i on slot i (top_k <= 32), and a token's output row is split over a
// cluster of C CTAs whose row maximum is reduced through distributed shared memory.

// One token's plan by one warp, written at p's pointers (offset by the caller): the slot scales (the expert outputs'
// own for Y, else ratio_act(ymax)·c, zero when either is zero: layers.rs:300-302, :321-326), common = the last of the
// largest as a warp reduction over (value, slot) (the fold of layers.rs:898), and the live slots packed to the front
// in slot order by their rank in the ballot. *p.n = -1 when the token's output is zero (sumc <= 0 or every slot zero).
template <bool Y, class A>
__device__ __forceinline__ void combine_plan_warp(const A& a, int t, const CombinePlan& p) {
    const int lane = threadIdx.x & 31, K = a.top_k;
    if (a.sumc[t] <= 0) {
        if (lane == 0) *p.n = -1;
        return;
    }
    const bool in = lane < K;
    const int row = in ? a.slot_row[(long long)t * K + lane] : 0;
    Scale ys = kt::scale_zero();
    int64_t ym = 0;
    if (in) {
        if constexpr (Y) {
            ys = a.ys[row];
        } else {
            ym = (int64_t)a.ymax_d[row];
            const Scale cd = a.row_cd[row];
            if (cd.mant != 0 && ym != 0) ys = kt::scale_mul(kt::ratio_act(ym), cd);
        }
    }
    ScaleIdx b{ys, in ? lane : -1};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ScaleIdx w;
        w.s.mant = __shfl_xor_sync(0xffffffffu, b.s.mant, o);
        w.s.shift = __shfl_xor_sync(0xffffffffu, b.s.shift, o);
        w.idx = __shfl_xor_sync(0xffffffffu, b.idx, o);
        b = better(b, w);
    }
    const Scale common = b.s;
    if (common.mant == 0) {
        if (lane == 0) *p.n = -1;
        return;
    }
    const bool live = in && ys.mant != 0;
    const unsigned m = __ballot_sync(0xffffffffu, live);
    if (live) {
        const int o = __popc(m & ((1u << lane) - 1u));
        p.row[o] = row;
        p.ec[o] = a.top_ec[(long long)t * K + lane];
        if constexpr (!Y) p.ry[o] = kt::make_req(ym);
        p.f[o] = kt::make_apply(kt::scale_mul(ys, kt::scale_recip(common)));
    }
    if (lane == 0) {
        *p.n = __popc(m);
        *p.common = common;
    }
}

// The plan of every token into global memory, a warp per token, for combine_kernel / combine_y_kernel (where tokens
// are many and a plan inside every token's CTA would hold up its loads).
template <bool Y, class A>
__global__ void combine_plan_warp_kernel(const A a, const CombinePlan p) {
    kt::pdl_enter();
    const int t = (int)((blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5);
    if (t >= a.T) return;  // the same for the whole warp
    const long long q = (long long)t * a.top_k;
    combine_plan_warp<Y>(a, t, CombinePlan{p.n + t, p.common + t, p.row + q, p.ec + q, Y ? nullptr : p.ry + q, p.f + q});
}

// Token t = %clusterid.x over the C = %cluster_nctarank CTAs of its cluster (C <= 8; a plain launch is a cluster of
// one): CTA c owns the output elements [c·S, min(D, (c+1)·S)), S = ceil(D / C), and the slice's accumulators in
// shared memory (S int64). Warp 0 of every CTA computes the token's plan (the same one). The row maximum: the CTA's,
// then each CTA stores it into slot c of every CTA's `part` between two cluster barriers (the first, relaxed, arrive
// is made before the loads so that every CTA has started by the time it is waited on), and each takes the max of
// its C slots. Every CTA of a cluster takes the same branch at the zero-token test, so no cluster barrier is left
// waiting. For few tokens (decode); with many, combine_plan_warp_kernel and combine_kernel / combine_y_kernel.
template <bool Y, class A>
__global__ void __launch_bounds__(256, 3) combine_tok_kernel(const A a) {
    kt::pdl_enter();
    extern __shared__ int64_t acc_s[];  // [S]
    __shared__ uint64_t red[32];
    __shared__ uint64_t part[8];
    __shared__ kt::ReqDiv ry_s[COMBINE_MAX_K];
    __shared__ kt::ApplyPlan f_s[COMBINE_MAX_K];
    __shared__ int64_t ec_s[COMBINE_MAX_K];
    __shared__ int row_s[COMBINE_MAX_K];
    __shared__ int n_s;
    __shared__ Scale common_s;
    const uint32_t C = cluster_size(), c = cluster_rank();
    const int t = (int)cluster_id_x();
    if (t >= a.T) return;  // the same for every CTA of the cluster
    const int D = a.dim;
    const int S = (D + (int)C - 1) / (int)C;
    const int d_lo = min(D, (int)c * S), d_hi = min(D, d_lo + S);
    if (threadIdx.x < 32) combine_plan_warp<Y>(a, t, CombinePlan{&n_s, &common_s, row_s, ec_s, ry_s, f_s});
    __syncthreads();
    const int n = n_s;
    int32_t* o = a.out + (long long)t * D;
    if (n < 0) {
        for (int d = d_lo + threadIdx.x; d < d_hi; d += blockDim.x) o[d] = 0;
        if (c == 0 && threadIdx.x == 0) a.out_scale[t] = kt::scale_zero();
        return;
    }
    if (C > 1) cluster_arrive_relaxed();
    bool lean = !Y;
    if constexpr (!Y) {
        for (int j = 0; j < n; ++j)
            lean = lean && ry_s[j].dbl && f_s[j].tight && ec_s[j] >= 0 && ec_s[j] < (int64_t(1) << 31);
    }
    uint64_t gm = 0;
    for (int d0 = d_lo + threadIdx.x; d0 < d_hi; d0 += CE * blockDim.x) {
        int64_t acc[CE];
#pragma unroll
        for (int u = 0; u < CE; ++u) acc[u] = 0;
        for (int j = 0; j < n; ++j) {
            const kt::ApplyPlan f = f_s[j];
            const int64_t ec = ec_s[j];
            if constexpr (Y) {
                const int32_t* b = a.y + (long long)row_s[j] * D;
                int32_t v[CE];
#pragma unroll
                for (int u = 0; u < CE; ++u) {
                    const int d = d0 + u * blockDim.x;
                    v[u] = d < d_hi ? __ldg(b + d) : 0;
                }
#pragma unroll
                for (int u = 0; u < CE; ++u) acc[u] += ec * kt::apply_row(f, v[u]);
            } else {
                const kt::ReqDiv ry = ry_s[j];
                const int64_t* b = a.acc_d + (long long)row_s[j] * D;
                int64_t v[CE];
#pragma unroll
                for (int u = 0; u < CE; ++u) {
                    const int d = d0 + u * blockDim.x;
                    v[u] = d < d_hi ? __ldg(b + d) : 0;
                }
                if (lean) {
#pragma unroll
                    for (int u = 0; u < CE; ++u)
                        acc[u] += (int64_t)(int32_t)ec * (int64_t)(int32_t)kt::apply_row(f, requant_fast(v[u], ry));
                } else {
#pragma unroll
                    for (int u = 0; u < CE; ++u) acc[u] += ec * kt::apply_row(f, kt::requant_row(v[u], ry));
                }
            }
        }
#pragma unroll
        for (int u = 0; u < CE; ++u) {
            const int d = d0 + u * blockDim.x;
            if (d < d_hi) {
                acc_s[d - d_lo] = acc[u];
                gm = max(gm, uabs64(acc[u]));
            }
        }
    }
    gm = block_max_u64(gm, red);
    if (C > 1) {
        cluster_wait_acquire();  // (the relaxed arrive above) every CTA of the cluster is running
        if (threadIdx.x < C) st_cluster_u64(&part[c], threadIdx.x, gm);
        cluster_arrive_release();
        cluster_wait_acquire();
        gm = 0;
        for (uint32_t k = 0; k < C; ++k) gm = max(gm, part[k]);
    }
    const int64_t gmax = (int64_t)gm;
    const kt::ReqDiv rg = kt::make_req(gmax);
    if (rg.dbl) {
        for (int d = d_lo + threadIdx.x; d < d_hi; d += blockDim.x) o[d] = requant_fast(acc_s[d - d_lo], rg);
    } else {
        for (int d = d_lo + threadIdx.x; d < d_hi; d += blockDim.x)
            o[d] = gmax ? kt::requant_row(acc_s[d - d_lo], rg) : 0;
    }
    if (c == 0 && threadIdx.x == 0) {
        const int64_t sumc = a.sumc[t];
        a.out_scale[t] = gmax == 0 ? kt::scale_zero()
                                   : kt::scale_mul(kt::scale_mul(kt::ratio_act(gmax), common_s),
                                                   kt::from_ratio(1, (kt::u128)(uint64_t)sumc));
    }
}

// This rank's best (common-scale candidate, global token index) as an int64 record {mant, shift, index}.
__global__ void scale_record_kernel(const Scale* __restrict__ best, const int* __restrict__ best_idx,
                                    int64_t* __restrict__ rec) {
    kt::pdl_enter();
    rec[0] = best[0].mant;
    rec[1] = best[0].shift;
    rec[2] = *best_idx;
}

// The record of a rank without tokens: no candidate ({0, 0, -1}).
__global__ void empty_record_kernel(int64_t* __restrict__ rec) {
    kt::pdl_enter();
    rec[0] = 0;
    rec[1] = 0;
    rec[2] = -1;
}

// The common scale over the ranks' records (in rank order; the index decides ties, so the order does not matter).
__global__ void reduce_records_kernel(const int64_t* __restrict__ recs, int n, Scale* __restrict__ out) {
    kt::pdl_enter();
    ScaleIdx b{kt::scale_zero(), -1};
    for (int i = 0; i < n; ++i)
        b = better(b, ScaleIdx{Scale{recs[3 * i], (int32_t)recs[3 * i + 1]}, (int)recs[3 * i + 2]});
    out[0] = b.s;
    out[1] = b.s.mant ? kt::scale_recip(b.s) : kt::scale_zero();
}

// ───────────── LinearBackend helpers ─────────────
// Pack int32 codes [rows][K] into three digit planes [3][R_pad][K_pad]; counts codes beyond ±WLEVELS into *bad.
// Optionally counts the codes beyond ±big_lim into *big, and writes the codes as one raw int8 plane [R_pad][K_pad]
// into `raw` (0 where |v| > 127), for the reduced-plane GEMM.
__global__ void pack_codes_kernel(const int32_t* __restrict__ codes, long long rows, int K, int K_pad, long long R_pad,
                                  int8_t* __restrict__ planes, unsigned long long* __restrict__ bad,
                                  unsigned long long* __restrict__ big = nullptr, int32_t big_lim = 0,
                                  int8_t* __restrict__ raw = nullptr) {
    kt::pdl_enter();
    const long long r = blockIdx.x;
    if (r >= rows) return;
    const int32_t* c = codes + r * K;
    int8_t* p0 = planes + r * K_pad;
    int8_t* p1 = p0 + R_pad * K_pad;
    int8_t* p2 = p1 + R_pad * K_pad;
    int8_t* pr = raw ? raw + r * K_pad : nullptr;
    unsigned nbad = 0, nbig = 0;
    for (int k4 = threadIdx.x * 4; k4 < K_pad; k4 += blockDim.x * 4) {
        int32_t q[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int k = k4 + j;
            int32_t v = k < K ? c[k] : 0;
            if (v > (int32_t)kt::WLEVELS || v < -(int32_t)kt::WLEVELS) {
                ++nbad;
                v = 0;
            }
            nbig += (v > big_lim || v < -big_lim) ? 1u : 0u;
            q[j] = v;
        }
        store_digits4(p0 + k4, p1 + k4, p2 + k4, q);
        if (pr) {
            uint32_t packed = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int32_t v = (q[j] > 127 || q[j] < -127) ? 0 : q[j];
                packed |= (uint32_t)(uint8_t)(int8_t)v << (8 * j);
            }
            *reinterpret_cast<uint32_t*>(pr + k4) = packed;  // K_pad is a multiple of 64: 4-byte aligned
        }
    }
    if (nbad && bad) atomicAdd(bad, (unsigned long long)nbad);
    if (nbig && big) atomicAdd(big, (unsigned long long)nbig);
}

}  // namespace mk
