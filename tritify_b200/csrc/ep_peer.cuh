// Expert parallelism over peer memory: the exchange steps of an expert-parallel layer as kernels that write into the
// other GPUs' memory over NVLink (CUDA IPC mappings of one region per rank), with no host synchronisation.
//
// Every rank owns one region, laid out identically on all ranks (byte offsets in `Peers`):
//   box      flags[point][source] (u64 sequence numbers) and vals[point][source][4] (u64 payloads);
//   counts   [world][E + 1] int32: each source's rows per expert and its token count;
//   planes   [3][cap_rows][d_pad] int8: the digit planes of the rows this rank's experts receive, expert-major
//            (expert e's rows from source 0, then source 1, ...), so each local expert is one GEMM group;
//   meta     [cap_rows][4] int64: per received row {s_qx mant, s_qx shift, expert, home rank << 32 | home row};
//   ret_y    [cap_home][d] int32 and ret_ys [cap_home] Scale: the expert outputs of this rank's rows, written by
//            their owners at the row's position in this rank's expert-sorted order (the reference seam's IntTensors,
//            crates/01-engine/kt-core/src/layers.rs:945-984).
// A step writes its data, then stores its flag with release semantics at system scope; a reader waits (bounded)
// until every source's flag for the step holds the forward's sequence number, with acquire semantics. Ranks run
// their forwards in the same order, so a flag value identifies the forward; a rank cannot reach the next forward's
// first step in a peer's memory before that peer has finished reading the current one (every forward ends with an
// exchange that all ranks must pass).
#pragma once

#include <stdint.h>

#include "fixed_point.cuh"
#include "moe_kernels.cuh"

namespace ep {

using kt::Scale;

constexpr int MAXW = 8;
enum Point : int {
    P_COUNTS = 0, P_DISPATCH, P_RETURN, P_REC, P_MERGE, P_SX, P_SYG, P_SHMAX, P_SYD, P_ADD,
    P_TOK, P_NREC, P_NMAX, P_RADD,  // the block around the layer: row counts, the norm's record and max, the residual add
    P_GYMAX, P_GATED,               // the gated shared expert: the gate logits' max, the gated output's max
    NPOINT
};
enum : int { ERR_WAIT = 21, ERR_BOUNDS = 22 };

struct Box {
    unsigned long long flags[NPOINT][MAXW];
    unsigned long long vals[NPOINT][MAXW][4];
};

struct Peers {
    unsigned char* base[MAXW];  // every rank's region, this rank's included
    int world, rank, E, e_begin, e_end;
    int d, d_pad;
    long long off_counts, off_planes, off_meta, off_rety, off_retys;
    long long cap_rows, cap_home;
    unsigned long long* seq;  // this rank's forward counter (device memory, so a captured graph advances it too)

    __device__ __forceinline__ Box* box(int r) const { return (Box*)base[r]; }
    __device__ __forceinline__ int* counts(int r) const { return (int*)(base[r] + off_counts); }
    __device__ __forceinline__ int8_t* planes(int r) const { return (int8_t*)(base[r] + off_planes); }
    __device__ __forceinline__ long long* meta(int r) const { return (long long*)(base[r] + off_meta); }
    __device__ __forceinline__ int32_t* ret_y(int r) const { return (int32_t*)(base[r] + off_rety); }
    __device__ __forceinline__ Scale* ret_ys(int r) const { return (Scale*)(base[r] + off_retys); }
};

// The owner of expert e: the rank r with r·E/world <= e < (r+1)·E/world.
__device__ __forceinline__ int owner_of(const Peers& P, int e) {
    int r = (int)((long long)e * P.world / P.E);
    while (r + 1 < P.world && (long long)(r + 1) * P.E / P.world <= e) ++r;
    while (r > 0 && (long long)r * P.E / P.world > e) --r;
    return r;
}

__device__ __forceinline__ void st_release(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Wait (bounded, ~2 s) until this rank's flag of `point` from `src` reaches `seq`. On expiry, or once another wait of
// this forward failed (the error word is set), record the error and give up.
__device__ __forceinline__ bool wait_flag(const Peers& P, int point, int src, unsigned long long seq, int* err) {
    const unsigned long long* f = &P.box(P.rank)->flags[point][src];
    if (ld_acquire(f) >= seq) return true;
    const uint64_t t0 = now_ns();
    for (uint32_t it = 1;; ++it) {
        if (ld_acquire(f) >= seq) return true;
        if ((it & 63u) == 0) {
            if (*(volatile int*)err != 0) return false;
            if (now_ns() - t0 > 2000000000ull) {
                atomicCAS(err, 0, ERR_WAIT);
                return false;
            }
        }
    }
}

// Exchange up to four u64 words with every rank (one block, >= world threads): writes `src` into every rank's
// vals[point][rank], raises the flags, waits for all ranks, then gives all ranks' words ([world][n], rank order) in
// `all` and/or their maxima in `mx` (in place allowed: mx may equal src).
__global__ void exchange_kernel(const Peers P, int point, const unsigned long long* src, int n, unsigned long long* all,
                                unsigned long long* mx, int* err) {
    kt::pdl_enter();
    const unsigned long long seq = *P.seq;
    __shared__ unsigned long long v[4];
    __shared__ int ok;
    const int i = threadIdx.x;
    if (i < n) v[i] = src[i];
    if (i == 0) ok = 1;
    __syncthreads();
    if (i < P.world) {
        Box* b = P.box(i);
        for (int j = 0; j < n; ++j) b->vals[point][P.rank][j] = v[j];
        st_release(&b->flags[point][P.rank], seq);
        if (!wait_flag(P, point, i, seq, err)) ok = 0;
    }
    __syncthreads();
    if (!ok) return;
    if (i < n) {
        const Box* b = P.box(P.rank);
        unsigned long long m = 0;
        for (int s = 0; s < P.world; ++s) {
            const unsigned long long w = b->vals[point][s][i];
            if (all) all[s * n + i] = w;
            m = w > m ? w : m;
        }
        if (mx) mx[i] = m;
    }
}

// Publish this rank's counts (E experts + its token count) into counts[rank] of every rank, raise P_COUNTS, wait for
// all ranks. One block.
__global__ void counts_exchange_kernel(const Peers P, const int* __restrict__ expert_count, int T, int* err) {
    kt::pdl_enter();
    const unsigned long long seq = *P.seq;
    const int E1 = P.E + 1;
    for (int q = 0; q < P.world; ++q) {
        int* c = P.counts(q) + (long long)P.rank * E1;
        for (int e = threadIdx.x; e < E1; e += blockDim.x) c[e] = e < P.E ? expert_count[e] : T;
    }
    __threadfence_system();
    __syncthreads();
    if ((int)threadIdx.x < P.world) {
        st_release(&P.box(threadIdx.x)->flags[P_COUNTS][P.rank], seq);
        wait_flag(P, P_COUNTS, threadIdx.x, seq, err);
    }
}

// After the counts exchange (one block): where this rank's rows of each expert go in the owner's expert-major buffer
// (dst_base[e] + r for expert-sorted row r), and the owner side of this rank: per local expert its received rows,
// group ends, the two tile tables and the number of received rows.
__global__ void ep_plan_kernel(const Peers P, const int* __restrict__ expert_off, int* __restrict__ dst_base,
                               int* __restrict__ group_end, int* __restrict__ rows_recv, mk::TileTable ta,
                               mk::TileTable tb, int* __restrict__ tok_offset, int* __restrict__ tok_total,
                               int* err) {
    kt::pdl_enter();
    extern __shared__ int sh[];  // [E] total rows per expert over all sources, [E] rows of lower sources
    int* tot = sh;
    int* below = sh + P.E;
    const int E1 = P.E + 1;
    const int* cnt = P.counts(P.rank);
    for (int e = threadIdx.x; e < P.E; e += blockDim.x) {
        int t = 0, b = 0;
        for (int s = 0; s < P.world; ++s) {
            const int c = cnt[(long long)s * E1 + e];
            if (s < P.rank) b += c;
            t += c;
        }
        tot[e] = t;
        below[e] = b;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        // this rank's rows of expert e start at owner_base(e) + below[e] in the owner's buffer
        int q_prev = -1, run = 0;
        for (int e = 0; e < P.E; ++e) {
            const int q = owner_of(P, e);
            if (q != q_prev) {
                run = 0;
                q_prev = q;
            }
            dst_base[e] = run + below[e] - expert_off[e];
            run += tot[e];
        }
        // the owner side: local experts [e_begin, e_end) are the groups 0.. of the received rows
        int off = 0, na = 0, nb = 0;
        for (int e = P.e_begin; e < P.e_end; ++e) {
            const int g = e - P.e_begin;
            int c = tot[e];
            if (c < 0 || off + (long long)c > P.cap_rows) {  // only if a rank passed more rows than the capacity
                atomicCAS(err, 0, ERR_BOUNDS);
                c = c < 0 ? 0 : (int)(P.cap_rows - off);
            }
            for (int r0 = 0; r0 < c; r0 += ta.BN) {
                ta.tile_group[na] = g;
                ta.tile_row0[na++] = off + r0;
            }
            for (int r0 = 0; r0 < c; r0 += tb.BN) {
                tb.tile_group[nb] = g;
                tb.tile_row0[nb++] = off + r0;
            }
            off += c;
            group_end[g] = off;
        }
        *ta.n_tiles = na;
        *tb.n_tiles = nb;
        *rows_recv = off;
        // this rank's first token in the layer's token order, and the layer's token count
        int before = 0, all = 0;
        for (int s = 0; s < P.world; ++s) {
            const int ts = cnt[(long long)s * E1 + P.E];
            if (s < P.rank) before += ts;
            all += ts;
        }
        *tok_offset = before;
        *tok_total = all;
    }
}

// Signal `point` to every rank once every block of this grid has finished its writes (the last block to finish
// raises the flags). `ctr` is a zeroed counter of this rank, left zeroed.
__device__ __forceinline__ void last_block_signal(const Peers& P, int point, unsigned long long seq, int* ctr) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int prev = atomicAdd(ctr, 1);
        if (prev == (int)gridDim.x - 1) {
            __threadfence_system();
            for (int q = 0; q < P.world; ++q) st_release(&P.box(q)->flags[point][P.rank], seq);
            *ctr = 0;
        }
    }
}

// Dispatch (the permute and the send in one pass): expert-sorted row r of this rank (token row_assign[r] / K, expert
// row_expert[r]) is copied from the token's digit planes straight into its owner's receive buffer at
// dst_base[e] + r, with its meta. One warp per row (16-byte loads and stores, many rows in flight per SM); then
// P_DISPATCH to every rank.
__global__ void dispatch_kernel(const Peers P, int R, const int* __restrict__ row_assign,
                                const int* __restrict__ row_expert, int K, const int8_t* __restrict__ tok_planes,
                                long long T_pad, const Scale* __restrict__ tok_sqx, const int* __restrict__ dst_base,
                                int* ctr, int* err) {
    kt::pdl_enter();
    const unsigned long long seq = *P.seq;
    const int n16 = P.d_pad / 16;
    const int lane = threadIdx.x & 31;
    const int warps = (int)(gridDim.x * blockDim.x) >> 5;
    for (int r = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5); r < R; r += warps) {
        const int e = row_expert[r];
        const int t = row_assign[r] / K;
        const int q = owner_of(P, e);
        const long long dst = (long long)dst_base[e] + r;
        if (dst < 0 || dst >= P.cap_rows) {
            if (lane == 0) atomicCAS(err, 0, ERR_BOUNDS);
            continue;
        }
        int8_t* pq = P.planes(q);
#pragma unroll
        for (int p = 0; p < 3; ++p) {
            const int4* src = (const int4*)(tok_planes + ((long long)p * T_pad + t) * P.d_pad);
            int4* dp = (int4*)(pq + ((long long)p * P.cap_rows + dst) * P.d_pad);
            for (int i = lane; i < n16; i += 32) dp[i] = __ldg(src + i);
        }
        if (lane == 0) {
            long long* m = P.meta(q) + dst * 4;
            const Scale sq = tok_sqx[t];
            m[0] = sq.mant;
            m[1] = sq.shift;
            m[2] = e;
            m[3] = ((long long)P.rank << 32) | (unsigned)r;
        }
    }
    last_block_signal(P, P_DISPATCH, seq, ctr);
}

// A new forward: the next sequence number (one thread).
__global__ void seq_bump_kernel(const Peers P) { kt::pdl_enter(); *P.seq += 1; }

// Wait for `point` from every rank (one block, >= world threads).
__global__ void wait_all_kernel(const Peers P, int point, int* err) {
    kt::pdl_enter();
    if ((int)threadIdx.x < P.world) wait_flag(P, point, threadIdx.x, *P.seq, err);
}

// The owner's per-row s_qx and local expert from the meta of its received rows.
__global__ void meta_unpack_kernel(const Peers P, const int* __restrict__ rows_recv, Scale* __restrict__ row_sqx,
                                   int* __restrict__ row_expert_local) {
    kt::pdl_enter();
    const int n = *rows_recv;
    const long long* m = P.meta(P.rank);
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < n; r += gridDim.x * blockDim.x) {
        row_sqx[r] = Scale{m[4 * (long long)r], (int32_t)m[4 * (long long)r + 1]};
        row_expert_local[r] = (int)m[4 * (long long)r + 2] - P.e_begin;
    }
}

// Return (the expert output and the send in one pass): received row r's output, requant_dyn(acc, L, ymax) as i32 with
// scale from_ratio(ymax, L)·c (the QuantLinear output the seam returns), written into its home rank's ret_y / ret_ys
// at the home row. Grid-stride over rows; then P_RETURN to every rank.
__global__ void return_kernel(const Peers P, const int* __restrict__ rows_recv,
                              const int64_t* __restrict__ acc, const unsigned long long* __restrict__ ymax_row,
                              const Scale* __restrict__ row_cd, int* ctr, int* err) {
    kt::pdl_enter();
    const unsigned long long seq = *P.seq;
    const int n = *rows_recv;
    const int D = P.d;
    const long long* m = P.meta(P.rank);
    for (int r = blockIdx.x; r < n; r += gridDim.x) {
        const long long hw = m[4 * (long long)r + 3];
        const int h = (int)(hw >> 32), hr = (int)(hw & 0xffffffffLL);
        if (h < 0 || h >= P.world || hr < 0 || hr >= P.cap_home) {
            if (threadIdx.x == 0) atomicCAS(err, 0, ERR_BOUNDS);
            continue;
        }
        const int64_t ymax = (int64_t)ymax_row[r];
        const Scale cd = row_cd[r];
        const bool zero = ymax == 0 || cd.mant == 0;
        const kt::ReqDiv rq = kt::make_req(ymax);
        const int64_t* a = acc + (long long)r * D;
        int32_t* y = P.ret_y(h) + (long long)hr * D;
        if ((D & 3) == 0) {
            for (int i = threadIdx.x * 4; i < D; i += blockDim.x * 4) {
                int4 o = make_int4(0, 0, 0, 0);
                if (!zero) {
                    const longlong2 a0 = __ldg((const longlong2*)(a + i)), a1 = __ldg((const longlong2*)(a + i + 2));
                    o.x = kt::requant_row(a0.x, rq);
                    o.y = kt::requant_row(a0.y, rq);
                    o.z = kt::requant_row(a1.x, rq);
                    o.w = kt::requant_row(a1.y, rq);
                }
                *(int4*)(y + i) = o;
            }
        } else {
            for (int i = threadIdx.x; i < D; i += blockDim.x) y[i] = zero ? 0 : kt::requant_row(a[i], rq);
        }
        if (threadIdx.x == 0) P.ret_ys(h)[hr] = zero ? kt::scale_zero() : kt::scale_mul(kt::ratio_act(ymax), cd);
    }
    last_block_signal(P, P_RETURN, seq, ctr);
}

}  // namespace ep
