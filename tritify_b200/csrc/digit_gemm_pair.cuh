// The digit-plane GEMM on an SM pair: tcgen05.mma.cta_group::2 over a 256-row weight tile.
//
// Same product as dg::digit_gemm_kernel (three weight planes x three stacked activation planes, five int32 diagonal
// accumulators in TMEM, int64 recombination in the epilogue), but each MMA spans two SMs of a cluster: M = 256 weight
// rows (128 in each SM's shared memory and TMEM) and N = 3·64 stacked activation rows, of which each SM holds half
// (SM 0 the rows 0-95: plane 0 and the first 32 rows of plane 1; SM 1 the rows 96-191). Each SM then reads from its
// shared memory all of its A tile but only half of the B tile per MMA, which is what bounds the one-SM kernel: per
// K step (32 bytes) an SM moves 24576 + 192·BN bytes through shared memory for 4.5·BN tensor cycles, against
// 24576 + 384·BN on one SM, so at BN = 64 the pair needs 128 B/clk where one SM needs 171.
//
// Roles (320 threads per CTA): warps 0-7 epilogue (warp w reads TMEM lanes 32·(w%4).. and columns 32·(w/4)..),
// warp 8 TMA producer (both CTAs load their own halves; every copy completes on CTA 0's barrier), warp 9 MMA issuer
// (CTA 0 only). One accumulator buffer (5·64 = 320 of 512 columns): the epilogue loads its whole share of the
// accumulator into registers, zeroes diagonals 3 and 4 (the next tile's first K step overwrites 0-2 and accumulates
// into 3-4), and releases TMEM before it recombines and stores, so the MMAs of the next tile wait only for the
// TMEM reads. With args.zero_mma the MMA issuer clears diagonals 2-4 itself at a tile's first K step (one MMA whose
// B operand is an all-zero tile in shared memory, 1/384 of the tile's tensor work) and the epilogue skips its TMEM
// stores, which shortens the time the accumulator is held. No load uses cluster multicast; every wait is bounded as in the one-SM kernel.
#pragma once

#include "digit_gemm.cuh"

namespace dg {

namespace pair {

constexpr int BN = 64;
constexpr int BM2 = 256;          // weight rows per pair tile
constexpr int HALF_ROWS = 96;     // stacked activation rows held by one CTA (3·BN / 2)
constexpr int BOX_ROWS = 32;      // activation rows per TMA box (three boxes per CTA per stage)
constexpr int THREADS = 320;
constexpr int EPI_WARPS = 8;
constexpr int STAGES = 3;
constexpr int A_PLANE = BM * BK;                       // 16 KB: one weight plane of this CTA's 128 rows
constexpr int B_STAGE = HALF_ROWS * BK;                // 12 KB
constexpr int CTA_STAGE_BYTES = 3 * A_PLANE + B_STAGE;  // what one CTA's copies of a stage bring
constexpr int ACC_COLS = NDIAG * BN;                   // 320
constexpr int TMEM_COLS = 512;
constexpr int ZERO_B = B_STAGE;                        // an all-zero B tile: the operand of the clearing MMA
constexpr int SMEM_BYTES = 1024 + STAGES * CTA_STAGE_BYTES + ZERO_B + 256;
static_assert(SMEM_BYTES <= 232448, "shared memory per block");
static_assert(B_STAGE % 1024 == 0 && A_PLANE % 1024 == 0, "swizzle atoms stay 1024-byte aligned");

// kind::i8 instruction descriptor for the pair MMA: D = s32, A = B = s8, K-major, M = 256, N = 3·BN.
__host__ __device__ constexpr uint32_t idesc() {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)((3 * BN) >> 3) << 17) | ((uint32_t)(BM2 >> 4) << 24);
}

__device__ __forceinline__ uint32_t cta_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t cluster_index() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t cluster_count() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}

// The shared::cluster address of the same shared-memory word in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// Arrive on an mbarrier given by its shared::cluster address (this CTA's or the peer's), release at cluster scope.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded waits with cluster-scope acquire (the pair's barriers are signalled from both CTAs). `drain` waits for
// work already issued and ignores the error word; the others give up as soon as another wait of the launch failed.
__device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity, int* err, int code, bool drain = false) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (!drain && err && *(volatile int*)err != 0) return false;
            if (globaltimer() - t0 > 2000000000ull) {
                if (err) atomicCAS(err, 0, code);
                return false;
            }
        }
    }
}

// A TMA tile load into this CTA's shared memory whose completion is counted on the barrier at `bar_cluster`
// (CTA 0's), the pair form of cp.async.bulk.tensor; no multicast.
__device__ __forceinline__ void tma_load_2d_to(void* smem_dst, const CUtensorMap* map, int x, int y,
                                               uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}

__device__ __forceinline__ void umma_i8_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t id,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(id), "r"(accumulate));
}

// Arrive once on the barrier at this shared-memory offset in both CTAs of the pair when the MMAs issued so far
// complete.
__device__ __forceinline__ void umma_commit_both(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"((uint16_t)3)
        : "memory");
}

__device__ __forceinline__ void tmem_st16_zero(uint32_t taddr) {
    const uint32_t z = 0;
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
        "r"(z)
        : "memory");
}

// Max over the 32 lanes of each of 32 values, transposed: afterwards lane l holds the maximum of value l over all
// lanes (31 shuffles instead of 5 per value).
__device__ __forceinline__ unsigned long long lane_max_transpose(unsigned long long (&v)[32], int lane) {
#pragma unroll
    for (int half = 16; half >= 1; half >>= 1) {
        const bool upper = (lane & half) != 0;
#pragma unroll
        for (int k = 0; k < half; ++k) {
            const unsigned long long send = upper ? v[k] : v[k + half];
            const unsigned long long keep = upper ? v[k + half] : v[k];
            const unsigned long long got = __shfl_xor_sync(0xffffffffu, send, half);
            v[k] = got > keep ? got : keep;
        }
    }
    return v[0];
}

struct TileIter2 {
    int per_group, limit;
    __device__ __forceinline__ bool get(const GemmArgs& a, int L, int& tile, int& m0) const {
        if (L >= limit) return false;
        const int grp = L / per_group, rem = L % per_group;
        tile = grp * a.group_n + rem % a.group_n;
        m0 = (rem / a.group_n) * BM2;
        return true;
    }
};

}  // namespace pair

// args.m_tiles counts 256-row pair tiles here; args.M_pad is a multiple of 256. Launched with clusters of 2 CTAs.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair::THREADS, 1)
    digit_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const GemmArgs args) {
    kt::pdl_enter();
    using namespace pair;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem;                                  // [STAGES][3][128 rows][BK]
    uint8_t* sB = smem + STAGES * 3 * A_PLANE;           // [STAGES][96 rows][BK]
    uint8_t* sZ = smem + STAGES * CTA_STAGE_BYTES;       // [96 rows][BK] of zeros
    uint64_t* full = (uint64_t*)(sZ + ZERO_B);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;   // this CTA's accumulator half is complete (commit from CTA 0)
    uint64_t* acc_empty = acc_full + 1;    // CTA 0: both CTAs' epilogues have read the accumulator (16 warp arrivals)
    uint64_t* mma_done = acc_empty + 1;    // every MMA of the pair has completed (waited before TMEM is freed)
    uint32_t* tmem_slot = (uint32_t*)(mma_done + 1);

    const uint32_t rank = cta_rank();
    const int cid = (int)cluster_index(), ncl = (int)cluster_count();
    const int n_tiles = args.n_tiles ? *args.n_tiles : args.n_tiles_max;
    const int n_groups = (n_tiles + args.group_n - 1) / args.group_n;
    const TileIter2 it{args.m_tiles * args.group_n, args.m_tiles * args.group_n * n_groups};
    // Both CTAs of a cluster see the same cid and n_tiles, so they leave together, before any barrier or allocation.
    if (cid >= it.limit) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkb = args.num_k_blocks;

    const bool zero_mma = args.zero_mma != 0;
    if (zero_mma) {
        // the clearing MMA reads this tile through the async proxy: write it, then make it visible there
        for (int i = threadIdx.x; i < ZERO_B / 16; i += blockDim.x) ((uint4*)sZ)[i] = make_uint4(0, 0, 0, 0);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 2 * EPI_WARPS);
        mbar_init(mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
        asm volatile("tcgen05.fence::before_thread_sync;");
    }
    __syncthreads();
    cluster_sync_all();  // the peer's barriers are initialised before anyone signals them
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tmem_slot;
    const uint32_t acc_empty_leader = peer_addr(acc_empty, 0);

    if (warp == 8) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
            int q = 0;
            bool alive = true;
            int tile, m0;
            for (int L = cid; alive && it.get(args, L, tile, m0); L += ncl) {
                if (tile >= n_tiles) continue;
                const TileInfo ti = tile_info(args, tile, BN);
                if (ti.n_valid <= 0) continue;
                for (int kb = 0; kb < nkb; ++kb, ++q) {
                    const int s = q % STAGES;
                    const uint32_t ph = (uint32_t)(q / STAGES) & 1u;
                    if (!wait(&empty[s], ph ^ 1u, args.err, ERR_TIMEOUT_EMPTY)) {
                        alive = false;
                        break;
                    }
                    if (rank == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(2 * CTA_STAGE_BYTES));
                    const uint32_t bar = peer_addr(&full[s], 0);
                    const int kx = (args.k_block0 + kb) * BK;
#pragma unroll
                    for (int p = 0; p < 3; ++p)
                        tma_load_2d_to(sA + (s * 3 + p) * A_PLANE, &tmA, kx,
                                       (ti.group * 3 + p) * args.M_pad + m0 + (int)rank * BM, bar);
                    // stacked row block i = 3·rank + j (32 rows): plane i / 2, rows 32·(i % 2) of the tile
#pragma unroll
                    for (int j = 0; j < 3; ++j) {
                        const int i = 3 * (int)rank + j;
                        tma_load_2d_to(sB + s * B_STAGE + j * BOX_ROWS * BK, &tmB, kx,
                                       (i >> 1) * args.R_pad + ti.row0 + (i & 1) * BOX_ROWS, bar);
                    }
                }
            }
            // CTA 0 lets every copy still in flight (its own and the peer's) land before the pair can leave.
            if (rank == 0)
                for (int j = max(0, q - STAGES); j < q; ++j)
                    wait(&full[j % STAGES], (uint32_t)(j / STAGES) & 1u, args.err, ERR_TIMEOUT_FULL, true);
        }
    } else if (warp == 9) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t id = idesc();
            int q = 0, tc = 0;
            bool alive = true;
            int tile, m0;
            for (int L = cid; alive && it.get(args, L, tile, m0); L += ncl) {
                if (tile >= n_tiles) continue;
                const TileInfo ti = tile_info(args, tile, BN);
                if (ti.n_valid <= 0) continue;
                // phase tc completes when both epilogues have released the accumulator (phase 0: the initial zeroing)
                if (!wait(acc_empty, (uint32_t)tc & 1u, args.err, ERR_TIMEOUT_ACCUM)) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                for (int kb = 0; kb < nkb; ++kb, ++q) {
                    const int s = q % STAGES;
                    const uint32_t ph = (uint32_t)(q / STAGES) & 1u;
                    if (!wait(&full[s], ph, args.err, ERR_TIMEOUT_FULL)) {
                        alive = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    const uint32_t a_base = smem_u32(sA + s * 3 * A_PLANE);
                    const uint32_t b_base = smem_u32(sB + s * B_STAGE);
                    if (zero_mma && kb == 0)  // diagonals 2-4 := A·0; plane 0 then overwrites 0-2, planes 1-2 add
                        umma_i8_pair(tmem + 2 * BN, smem_desc_sw128(a_base), smem_desc_sw128(smem_u32(sZ)), id, 0u);
#pragma unroll
                    for (int kk = 0; kk < BK / UMMA_K; ++kk) {
                        const uint64_t bd = smem_desc_sw128(b_base + kk * UMMA_K);
                        // weight plane j times the three stacked activation planes lands on diagonals j..j+2;
                        // diagonals 3 and 4 were zeroed by the epilogue, so only plane 0's first MMA overwrites
                        const uint32_t first = (kb == 0 && kk == 0) ? 0u : 1u;
                        umma_i8_pair(tmem + 0 * BN, smem_desc_sw128(a_base + 0 * A_PLANE + kk * UMMA_K), bd, id, first);
                        umma_i8_pair(tmem + 1 * BN, smem_desc_sw128(a_base + 1 * A_PLANE + kk * UMMA_K), bd, id, 1u);
                        umma_i8_pair(tmem + 2 * BN, smem_desc_sw128(a_base + 2 * A_PLANE + kk * UMMA_K), bd, id, 1u);
                    }
                    umma_commit_both(&empty[s]);
                }
                umma_commit_both(acc_full);
                ++tc;
            }
            umma_commit_both(mma_done);
            wait(mma_done, 0u, args.err, ERR_TIMEOUT_ACCUM, true);
        }
    } else {
        // Epilogue: warp w reads TMEM lanes 32·(w%4).. (weight rows) and columns 32·(w/4).. (activation rows).
        const int quad = warp & 3, chalf = warp >> 2;
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
        // Before the first tile: zero diagonals 3 and 4 (unless the MMAs clear them) and release the accumulator.
        if (!zero_mma) {
            tmem_st16_zero(lane_base + 3 * BN + chalf * 32);
            tmem_st16_zero(lane_base + 3 * BN + chalf * 32 + 16);
            tmem_st16_zero(lane_base + 4 * BN + chalf * 32);
            tmem_st16_zero(lane_base + 4 * BN + chalf * 32 + 16);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        asm volatile("tcgen05.fence::before_thread_sync;");
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(acc_empty_leader);

        const bool do_max = args.rowmax != nullptr;
        int tc = 0;
        int tile, m0;
        for (int L = cid; it.get(args, L, tile, m0); L += ncl) {
            if (tile >= n_tiles) continue;
            const TileInfo ti = tile_info(args, tile, BN);
            if (ti.n_valid <= 0) continue;
            bool ok = wait(acc_full, (uint32_t)tc & 1u, args.err, ERR_TIMEOUT_ACCUM);
            ok = __all_sync(0xffffffffu, ok);
            asm volatile("tcgen05.fence::after_thread_sync;");
            int64_t v[32];  // this lane's row, the warp's 32 columns, recombined
            if (ok) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    int32_t s0[16], s1[16], s2[16], s3[16], s4[16];
                    const uint32_t col = lane_base + chalf * 32 + c * 16;
                    tmem_ld16(col + 0 * BN, s0);
                    tmem_ld16(col + 1 * BN, s1);
                    tmem_ld16(col + 2 * BN, s2);
                    tmem_ld16(col + 3 * BN, s3);
                    tmem_ld16(col + 4 * BN, s4);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[c * 16 + j] = kt::recombine(s0[j], s1[j], s2[j], s3[j], s4[j]);
                }
                if (!zero_mma) {
                    tmem_st16_zero(lane_base + 3 * BN + chalf * 32);
                    tmem_st16_zero(lane_base + 3 * BN + chalf * 32 + 16);
                    tmem_st16_zero(lane_base + 4 * BN + chalf * 32);
                    tmem_st16_zero(lane_base + 4 * BN + chalf * 32 + 16);
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                }
            }
            // the accumulator is in registers: the next tile's MMAs may start
            asm volatile("tcgen05.fence::before_thread_sync;");
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(acc_empty_leader);
            ++tc;
            if (!ok) continue;  // later waits give up at once: the error word is set
            const int m = m0 + (int)rank * BM + quad * 32 + lane;
            const bool m_ok = m < args.M_valid;
            const int my_slot = m >= args.rowmax_split ? 1 : 0;
            unsigned long long av[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int n = chalf * 32 + j;
                int64_t x = v[j];
                const bool live = m_ok && n < ti.n_valid;
                if (live) {
                    int64_t* p = args.out + (long long)(ti.row0 + n) * args.ld_out + m;
                    if (args.accumulate) x += *p;
                    *p = x;
                }
                av[j] = live ? (unsigned long long)(x >= 0 ? x : -x) : 0ull;
            }
            if (do_max) {
                const int n = chalf * 32 + lane;  // the column whose maximum this lane ends up holding
                const bool one_slot = __all_sync(0xffffffffu, my_slot == __shfl_sync(0xffffffffu, my_slot, 0));
                auto publish = [&](unsigned long long mx, int sl) {
                    if (n >= ti.n_valid) mx = 0;
                    if (args.rowmax_stride == 0) {
                        // one word for the whole output: reduce the warp's columns first (one atomic per warp)
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) {
                            const unsigned long long w = __shfl_xor_sync(0xffffffffu, mx, o);
                            mx = w > mx ? w : mx;
                        }
                        if (lane == 0 && mx) atomicMax(args.rowmax + sl, mx);
                    } else if (mx) {
                        atomicMax(args.rowmax + (long long)(ti.row0 + n) * args.rowmax_stride + sl, mx);
                    }
                };
                if (one_slot) {
                    // the warp's 32 weight rows lie on one side of rowmax_split (the usual case): reduce in place
                    publish(lane_max_transpose(av, lane), my_slot);
                } else {
#pragma unroll 1
                    for (int sl = 0; sl < 2; ++sl) {
                        unsigned long long bv[32];
#pragma unroll
                        for (int j = 0; j < 32; ++j) bv[j] = my_slot == sl ? av[j] : 0ull;
                        publish(lane_max_transpose(bv, lane), sl);
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    cluster_sync_all();  // neither CTA frees TMEM or leaves while the pair's MMAs, copies or arrivals may touch it
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    }
}


// ───────────── small codes on an SM pair ─────────────
// The (1, 2) product (one raw activation plane, |x| <= 127; two weight digit planes, |w| <= 3280) with the roles of
// the kernel above swapped: the MMA's M side is 256 activation rows (128 in each SM's shared memory and TMEM), its N
// side the two digit planes of 128 weight rows stacked (N = 256; SM 0 holds plane 0, SM 1 plane 1). One
// tcgen05.mma.cta_group::2 per 32-byte K step puts x·w0 into columns 0-127 and x·w1 into columns 128-255 of each SM's
// accumulator: the two diagonals. Per K step an SM takes 8 KB from TMA and its MMA reads 8 KB of shared memory for
// 128 tensor cycles (128 B/clk), against 224 B/clk for the one-SM (1, 2) kernel at BN = 128. Two accumulator buffers
// of 256 columns let the epilogue of one tile overlap the MMAs of the next. A TMEM lane is an activation row, so an
// epilogue thread writes 16 consecutive int64 outputs (128 bytes) of its row per step. No fused row maxima and no
// split K: the LinearBackend path is its only user. No load uses cluster multicast; every wait is bounded.
namespace pair_small {

constexpr int BM_ACT = 256;                         // activation rows per pair tile (128 per SM)
constexpr int BN_W = 128;                           // weight rows per tile
constexpr int N = 2 * BN_W;                         // the two weight planes, stacked
constexpr int THREADS = 192;                        // warps 0-3 epilogue, 4 TMA producer, 5 MMA issuer (CTA 0)
constexpr int EPI_WARPS = 4;
constexpr int STAGES = 6;
constexpr int ACC = 2;
constexpr int X_TILE = 128 * BK;                    // 16 KB: this SM's activation rows
constexpr int W_TILE = BN_W * BK;                   // 16 KB: this SM's weight plane
constexpr int CTA_STAGE_BYTES = X_TILE + W_TILE;
constexpr int ACC_COLS = N;
constexpr int TMEM_COLS = 512;
constexpr int SMEM_BYTES = 1024 + STAGES * CTA_STAGE_BYTES + 256;
static_assert(SMEM_BYTES <= 232448, "shared memory per block");
static_assert(ACC * ACC_COLS <= TMEM_COLS, "the accumulator buffers must fit TMEM");
static_assert(X_TILE % 1024 == 0 && W_TILE % 1024 == 0, "swizzle atoms stay 1024-byte aligned");

// kind::i8 instruction descriptor: D = s32, A = B = s8, K-major, M = 256, N = 256.
__host__ __device__ constexpr uint32_t idesc() {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(BM_ACT >> 4) << 24);
}

// Slot L of the raster: activation tile `at` (256 rows) and weight rows w0.. (128). group_n consecutive activation
// tiles share each weight tile, as in the other kernels (args.m_tiles counts 128-row weight tiles here,
// args.n_tiles_max activation tiles).
__device__ __forceinline__ bool tile_of(const GemmArgs& a, int per_group, int limit, int L, int& at, int& w0) {
    if (L >= limit) return false;
    const int grp = L / per_group, rem = L % per_group;
    at = grp * a.group_n + rem % a.group_n;
    w0 = (rem / a.group_n) * BN_W;
    return true;
}

}  // namespace pair_small

// tmX: the activations' raw plane [R_pad][k_pad]; tmW: the weight planes [3][M_pad][k_pad] (planes 0 and 1 used).
// out[r][m] (+= with args.accumulate) for r < single_rows, m < M_valid. Launched with clusters of 2 CTAs.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair_small::THREADS, 1)
    digit_gemm_pair_small_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                                 const GemmArgs args) {
    kt::pdl_enter();
    using namespace pair;
    namespace ps = pair_small;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sX = smem;                                  // [STAGES][128 rows][BK]
    uint8_t* sW = smem + ps::STAGES * ps::X_TILE;        // [STAGES][128 rows][BK]
    uint64_t* full = (uint64_t*)(smem + ps::STAGES * ps::CTA_STAGE_BYTES);
    uint64_t* empty = full + ps::STAGES;
    uint64_t* acc_full = empty + ps::STAGES;  // [ACC]: this CTA's accumulator half is complete (commit from CTA 0)
    uint64_t* acc_empty = acc_full + ps::ACC;  // [ACC], CTA 0: both CTAs' epilogues have read buffer b (8 arrivals)
    uint64_t* mma_done = acc_empty + ps::ACC;  // every MMA of the pair has completed (waited before TMEM is freed)
    uint32_t* tmem_slot = (uint32_t*)(mma_done + 1);

    const uint32_t rank = cta_rank();
    const int cid = (int)cluster_index(), ncl = (int)cluster_count();
    const int n_at = args.n_tiles_max;
    const int n_groups = (n_at + args.group_n - 1) / args.group_n;
    const int per_group = args.m_tiles * args.group_n, limit = per_group * n_groups;
    // Both CTAs of a cluster see the same cid, so they leave together, before any barrier or allocation.
    if (cid >= limit) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkb = args.num_k_blocks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ps::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < ps::ACC; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 2 * ps::EPI_WARPS);
        }
        mbar_init(mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(ps::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
        asm volatile("tcgen05.fence::before_thread_sync;");
    }
    __syncthreads();
    cluster_sync_all();  // the peer's barriers are initialised before anyone signals them
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
            int q = 0;
            bool alive = true;
            int at, w0;
            for (int L = cid; alive && ps::tile_of(args, per_group, limit, L, at, w0); L += ncl) {
                if (at >= n_at) continue;
                const int x0 = at * ps::BM_ACT + (int)rank * 128;
                for (int kb = 0; kb < nkb; ++kb, ++q) {
                    const int s = q % ps::STAGES;
                    const uint32_t ph = (uint32_t)(q / ps::STAGES) & 1u;
                    if (!wait(&empty[s], ph ^ 1u, args.err, ERR_TIMEOUT_EMPTY)) {
                        alive = false;
                        break;
                    }
                    if (rank == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(2 * ps::CTA_STAGE_BYTES));
                    const uint32_t bar = peer_addr(&full[s], 0);
                    const int kx = (args.k_block0 + kb) * BK;
                    tma_load_2d_to(sX + s * ps::X_TILE, &tmX, kx, x0, bar);
                    tma_load_2d_to(sW + s * ps::W_TILE, &tmW, kx, (int)rank * args.M_pad + w0, bar);
                }
            }
            // CTA 0 lets every copy still in flight (its own and the peer's) land before the pair can leave.
            if (rank == 0)
                for (int j = max(0, q - ps::STAGES); j < q; ++j)
                    wait(&full[j % ps::STAGES], (uint32_t)(j / ps::STAGES) & 1u, args.err, ERR_TIMEOUT_FULL, true);
        }
    } else if (warp == 5) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t id = ps::idesc();
            int q = 0, tc = 0;
            bool alive = true;
            int at, w0;
            for (int L = cid; alive && ps::tile_of(args, per_group, limit, L, at, w0); L += ncl) {
                if (at >= n_at) continue;
                const int b = tc % ps::ACC;
                const uint32_t acc = tmem + (uint32_t)(b * ps::ACC_COLS);
                // buffer b is free once both epilogues have read its previous tile (the first use passes at once)
                if (!wait(&acc_empty[b], ((uint32_t)(tc / ps::ACC) & 1u) ^ 1u, args.err, ERR_TIMEOUT_ACCUM)) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                for (int kb = 0; kb < nkb; ++kb, ++q) {
                    const int s = q % ps::STAGES;
                    const uint32_t ph = (uint32_t)(q / ps::STAGES) & 1u;
                    if (!wait(&full[s], ph, args.err, ERR_TIMEOUT_FULL)) {
                        alive = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    const uint32_t x_base = smem_u32(sX + s * ps::X_TILE);
                    const uint32_t w_base = smem_u32(sW + s * ps::W_TILE);
#pragma unroll
                    for (int kk = 0; kk < BK / UMMA_K; ++kk)
                        umma_i8_pair(acc, smem_desc_sw128(x_base + kk * UMMA_K), smem_desc_sw128(w_base + kk * UMMA_K),
                                     id, (kb == 0 && kk == 0) ? 0u : 1u);
                    umma_commit_both(&empty[s]);
                }
                umma_commit_both(&acc_full[b]);
                ++tc;
            }
            umma_commit_both(mma_done);
            wait(mma_done, 0u, args.err, ERR_TIMEOUT_ACCUM, true);
        }
    } else {
        // Epilogue: warp w reads TMEM lanes 32w..32w+31; lane l holds activation row x0 + 32w + l.
        int tc = 0;
        int at, w0;
        for (int L = cid; ps::tile_of(args, per_group, limit, L, at, w0); L += ncl) {
            if (at >= n_at) continue;
            const int b = tc % ps::ACC;
            bool ok = wait(&acc_full[b], (uint32_t)(tc / ps::ACC) & 1u, args.err, ERR_TIMEOUT_ACCUM);
            ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective: keep the branch warp-uniform
            asm volatile("tcgen05.fence::after_thread_sync;");
            const uint32_t lane_base = tmem + (uint32_t)(b * ps::ACC_COLS) + ((uint32_t)(warp * 32) << 16);
            const int r = at * ps::BM_ACT + (int)rank * 128 + warp * 32 + lane;
            const bool r_ok = r < args.single_rows;
            int64_t* orow = args.out + (long long)(r_ok ? r : 0) * args.ld_out;
#pragma unroll 1
            for (int c = 0; c < ps::BN_W / 16; ++c) {
                int32_t s0[16], s1[16];
                if (ok) {
                    tmem_ld16(lane_base + c * 16, s0);
                    tmem_ld16(lane_base + ps::BN_W + c * 16, s1);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                }
                if (c == ps::BN_W / 16 - 1) {
                    // this warp has read all of buffer b: the MMAs of a later tile may overwrite it
                    asm volatile("tcgen05.fence::before_thread_sync;");
                    __syncwarp();
                    if (lane == 0) mbar_arrive_remote(peer_addr(&acc_empty[b], 0));
                }
                if (!ok || !r_ok) continue;
                const int m = w0 + c * 16;
                int64_t v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = (int64_t)s0[j] + 81LL * s1[j];
                int64_t* p = orow + m;
                if (m + 16 <= args.M_valid && !args.accumulate && ((reinterpret_cast<uintptr_t>(p) & 15u) == 0)) {
#pragma unroll
                    for (int j = 0; j < 16; j += 2)
                        *reinterpret_cast<longlong2*>(p + j) = make_longlong2(v[j], v[j + 1]);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        if (m + j >= args.M_valid) break;
                        int64_t x = v[j];
                        if (args.accumulate) x += p[j];
                        p[j] = x;
                    }
                }
            }
            ++tc;
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    cluster_sync_all();  // neither CTA frees TMEM or leaves while the pair's MMAs, copies or arrivals may touch it
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ps::TMEM_COLS));
    }
}

}  // namespace dg
