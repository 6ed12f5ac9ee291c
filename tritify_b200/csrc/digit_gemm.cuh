// The exact integer linear accumulate Y[r,m] = sum_k X[r,k]·W[m,k] on sm_100a tensor cores.
//
// tritify's codes are 12-trit integers (|v| <= 265720). Each code is three balanced base-81 digits (|d| <= 40, an
// int8), so one code product is sum_{i,j} 81^(i+j) x_i w_j: nine int8 x int8 products
// (crates/02-runtime/kt-cuda/src/digits.rs:1-36 states the split; digit_gemm.cu there computes the nine products
// with WMMA). Here the nine products are tcgen05.mma kind::i8 instructions issued by one thread, operands staged in
// shared memory by TMA (128-byte swizzle, no multicast), and the products that share a diagonal t = i+j accumulate
// into the same int32 TMEM accumulator: five accumulators of BN columns. A diagonal sums at most three plane
// products, each |.| <= K·40², so K <= 447,392 keeps every int32 sum exact (the host splits longer K and adds the
// int64 partial results in the epilogue, the analogue of kt-cuda's KT_FLUSH). The epilogue recombines
// sum_t 81^t S_t in int64.
//
// Layout ("swap AB", so that a handful of tokens still fills the 128-row MMA):
//   A (MMA M side) = weight digit planes, K-major: global [groups][3 planes][M_pad rows][K_pad] int8.
//   B (MMA N side) = activation digit planes, K-major: global [3 planes][R_pad rows][K_pad] int8.
//   D (TMEM)      = 128 lanes (weight rows) x 5·BN columns (5 diagonals x BN activation rows).
//   out           = int64 [rows][ld_out]; element (r, m) at out[r*ld_out + m] (coalesced across lanes).
//
// Roles (192 threads): warps 0-3 epilogue (TMEM lanes 32w..32w+31), warp 4 TMA producer, warp 5 MMA issuer.
// Every mbarrier wait is bounded by a global-timer limit; on expiry the kernel records an error code, stops issuing,
// lets its in-flight copies and MMAs land, frees its TMEM and returns.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "fixed_point.cuh"

namespace dg {

constexpr int BM = 128;     // weight rows per tile = TMEM lanes
constexpr int BK = 128;     // K bytes per pipeline stage = one 128-byte swizzle atom row
constexpr int UMMA_K = 32;  // K of one kind::i8 MMA
constexpr int NDIAG = 5;
constexpr int THREADS = 192;
constexpr int64_t K_EXACT_MAX = 447392;  // floor((2^31 - 1) / (3 · 1600)): one pass without int32 overflow
constexpr int64_t K_EXACT_MAX_SMALL = 422733;  // floor((2^31 - 1) / (127 · 40)): the same for the (1, 2) planes

enum : int { ERR_NONE = 0, ERR_TIMEOUT_FULL = 1, ERR_TIMEOUT_EMPTY = 2, ERR_TIMEOUT_ACCUM = 3 };

struct GemmArgs {
    int64_t* out;
    long long ld_out;
    int M_valid;        // valid weight rows of one group
    int M_pad;          // rows of one (group, plane) block in A: multiple of 128
    int k_block0;       // first K block of this launch (K is split into chunks of at most K_EXACT_MAX)
    int num_k_blocks;   // K blocks in this launch
    int R_pad;          // rows of one plane in B
    const int* tile_group;     // per n-tile: group (nullptr: single group 0)
    const int* tile_row0;      // per n-tile: first activation row (nullptr: tile * BN)
    const int* group_row_end;  // per group: end row, exclusive (nullptr: single_rows)
    const int* tile_row_end;   // per n-tile: end row, exclusive (overrides group_row_end; a group may have several runs)
    const int* n_tiles;        // device count of valid n-tiles (nullptr: n_tiles_max)
    int n_tiles_max;           // upper bound of n-tiles (the launch covers m_tiles x n_tiles_max, rounded up)
    int m_tiles;               // weight tiles of one group (M_pad / BM)
    int group_n;               // raster: GROUP_N consecutive n-tiles share each weight tile while it is in L2
    int single_rows;
    int accumulate;  // 1: out += result (the second and later K chunks)
    int* err;        // device error word (first error wins)
    // Optional fused reduction: atomicMax of |out[r][m]| into rowmax[r * rowmax_stride + (m >= rowmax_split)]
    // (rowmax_stride 0 reduces the whole output into one or two words). Only valid without K chunking.
    unsigned long long* rowmax;
    int rowmax_stride;
    int rowmax_split;
    // Split K: k_splits > 1 blocks share a tile, each over its own K range, and add their partial results into `out`
    // with 64-bit atomics (integer sums: exact in any order; `out` starts at zero; no fused row maxima).
    int k_splits;
    // Pair kernel only: 1 clears diagonals 2-4 of a tile's accumulator with one MMA of a zero B operand at its first
    // K step, so the epilogue releases TMEM without zeroing it (0: the epilogue zeroes diagonals 3-4).
    int zero_mma;
};

// PX, PW: digit planes of the activations and the weights per stage (3, 3 for any code; 1, 2 for small codes).
template <int BN, int STAGES, int ACC, int PX = 3, int PW = 3>
struct Cfg {
    static constexpr int A_PLANE = BM * BK;
    static constexpr int B_PLANE = BN * BK;
    static constexpr int STAGE_BYTES = PW * A_PLANE + PX * B_PLANE;
    static constexpr int DIAGS = PX + PW - 1;
    static constexpr int ACC_COLS = DIAGS * BN;  // one accumulator buffer: a diagonal of BN columns per plane sum
    static constexpr int TMEM_COLS = ACC * ACC_COLS <= 32    ? 32
                                     : ACC * ACC_COLS <= 64  ? 64
                                     : ACC * ACC_COLS <= 128 ? 128
                                     : ACC * ACC_COLS <= 256 ? 256
                                                             : 512;
    static constexpr int RED_BYTES = 2 * 4 * BN * 8;  // row-max staging: [slot][epilogue warp][column]
    static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256 + RED_BYTES;
    static_assert((PX == 3 && PW == 3) || (PX == 1 && PW == 2), "plane counts");
    static_assert(BN % 16 == 0 && BN >= 16 && PX * BN <= 256, "BN: a multiple of 16, PX·BN <= 256 (one MMA's N)");
    static_assert(ACC * ACC_COLS <= 512, "the accumulator buffers must fit TMEM");
    static_assert(B_PLANE % 1024 == 0, "swizzle atoms stay 1024-byte aligned");
    static_assert(SMEM_BYTES <= 232448, "shared memory per block");
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait of the pipeline: false (and the error word set) after ~2 s, or as soon as another wait of the launch
// has failed (the error word is set), so that a failed launch ends in about one limit rather than one per tile.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (err && *(volatile int*)err != 0) return false;
            if (globaltimer() - t0 > 2000000000ull) {
                if (err) atomicCAS(err, 0, code);
                return false;
            }
        }
    }
}

// Bounded wait for work already issued (copies or MMAs in flight) before the block frees what they touch: ~2 s,
// whatever the error word says.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity, int* err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0 && globaltimer() - t0 > 2000000000ull) {
            if (err) atomicCAS(err, 0, code);
            return false;
        }
    }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;              // leading byte offset (unused for swizzled K-major), 16 B
    d |= (uint64_t)(1024 >> 4) << 32;    // stride byte offset: 1024 B between 8-row groups
    d |= (uint64_t)1 << 46;              // descriptor version (sm100)
    d |= (uint64_t)2 << 61;              // SWIZZLE_128B
    return d;
}

// Instruction descriptor: kind::i8, D = s32, A = s8, B = s8, both K-major, M = 128, N = bn.
__host__ __device__ constexpr uint32_t idesc_i8(int bn) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, int32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
        "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// The tiles of one launch, in raster order. Slot L (0 <= L < m_tiles · group_n · n_groups) is weight tile
// m = (L mod per_group) / group_n of n-tile (L / per_group) · group_n + L mod group_n: the blocks resident at one time
// walk group_n activation tiles for each weight tile, so both stay in L2 while they are reused.
struct TileIter {
    int per_group, limit, n_tiles;  // limit: slots of one K split
    int splits;
    __device__ __forceinline__ bool get(const GemmArgs& a, int L, int& tile, int& m0, int& split) const {
        if (L >= limit * splits) return false;
        split = L / limit;
        L -= split * limit;
        const int grp = L / per_group, rem = L % per_group;
        tile = grp * a.group_n + rem % a.group_n;
        m0 = (rem / a.group_n) * BM;
        return true;
    }
};

struct TileInfo {
    int group, row0, n_valid;
};

__device__ __forceinline__ TileInfo tile_info(const GemmArgs& a, int tile, int bn) {
    TileInfo t;
    t.group = a.tile_group ? a.tile_group[tile] : 0;
    t.row0 = a.tile_row0 ? a.tile_row0[tile] : tile * bn;
    const int row_end = a.tile_row_end ? a.tile_row_end[tile] : a.group_row_end ? a.group_row_end[t.group] : a.single_rows;
    t.n_valid = min(bn, row_end - t.row0);
    return t;
}

// Persistent: gridDim.x blocks (at most one per SM) walk the raster with stride gridDim.x. The TMA producer and the
// MMA issuer run ahead across tile boundaries; ACC accumulator buffers in TMEM let the epilogue of one tile overlap
// the MMAs of the next.
//
// PX, PW: digit planes of the activations and the weights. (3, 3) is every 12-trit code. (1, 2) serves small codes
// (|x| <= 127 stored as one raw int8 plane, |w| <= 3280 as two base-81 digits): two MMAs of N = BN per K step, product
// x·w_j on diagonal j, two diagonals recombined.
template <int BN, int STAGES, int ACC, int PX = 3, int PW = 3>
__global__ void __launch_bounds__(THREADS, 1)
    digit_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const GemmArgs args) {
    kt::pdl_enter();
    using C = Cfg<BN, STAGES, ACC, PX, PW>;
    constexpr int NDIAG_USED = C::DIAGS;
    constexpr uint32_t TX_BYTES = (uint32_t)C::STAGE_BYTES;  // what one stage's copies bring
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem;                              // [STAGES][PW] weight planes
    uint8_t* sB = smem + STAGES * PW * C::A_PLANE;   // [STAGES][PX] activation planes
    uint64_t* full = (uint64_t*)(smem + STAGES * C::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;     // [ACC]: the MMAs of a tile completed into buffer b
    uint64_t* acc_empty = acc_full + ACC;    // [ACC]: the epilogue has read buffer b (128 arrivals)
    uint64_t* mma_done = acc_empty + ACC;    // every MMA of the block has completed (waited before TMEM is freed)
    uint32_t* tmem_slot = (uint32_t*)(mma_done + 1);
    unsigned long long* sred = (unsigned long long*)(smem + STAGES * C::STAGE_BYTES + 256);

    const int n_tiles = args.n_tiles ? *args.n_tiles : args.n_tiles_max;
    const int n_groups = (n_tiles + args.group_n - 1) / args.group_n;
    const int ks = args.k_splits > 1 ? args.k_splits : 1;
    const TileIter it{args.m_tiles * args.group_n, args.m_tiles * args.group_n * n_groups, n_tiles, ks};
    if ((int)blockIdx.x >= it.limit * ks) return;  // no tile for this block: leave before any barrier or allocation
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkb = args.num_k_blocks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < ACC; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 128);
        }
        mbar_init(mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(C::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        asm volatile("tcgen05.fence::before_thread_sync;");
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
            int q = 0;  // k-blocks issued by this block so far (its position in the stage ring)
            bool alive = true;
            int tile, m0, split;
            for (int L = blockIdx.x; alive && it.get(args, L, tile, m0, split); L += gridDim.x) {
                if (tile >= n_tiles) continue;
                const TileInfo ti = tile_info(args, tile, BN);
                if (ti.n_valid <= 0) continue;
                const int kb1 = (int)((long long)(split + 1) * nkb / ks);
                for (int kb = (int)((long long)split * nkb / ks); kb < kb1; ++kb, ++q) {
                    const int s = q % STAGES;
                    const uint32_t ph = (uint32_t)(q / STAGES) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, args.err, ERR_TIMEOUT_EMPTY)) {
                        alive = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], TX_BYTES);
                    const int kx = (args.k_block0 + kb) * BK;
#pragma unroll
                    for (int p = 0; p < PW; ++p)
                        tma_load_2d(sA + (s * PW + p) * C::A_PLANE, &tmA, kx, (ti.group * 3 + p) * args.M_pad + m0,
                                    &full[s]);
#pragma unroll
                    for (int p = 0; p < PX; ++p)
                        tma_load_2d(sB + (s * PX + p) * C::B_PLANE, &tmB, kx, p * args.R_pad + ti.row0, &full[s]);
                }
            }
            // Let the copies still in flight land before the block can leave (bounded).
            for (int j = max(0, q - STAGES); j < q; ++j)
                mbar_wait_drain(&full[j % STAGES], (uint32_t)(j / STAGES) & 1u, args.err, ERR_TIMEOUT_FULL);
        }
    } else if (warp == 5) {
        if (lane == 0) {
            // The three activation planes sit back to back in shared memory, so one MMA of N = 3·BN multiplies a
            // weight plane i by all three: its D starts at column i·BN and product (i, j) lands on diagonal i+j.
            constexpr uint32_t id1 = idesc_i8(BN), id2 = idesc_i8(PX * BN >= 2 * BN ? 2 * BN : BN),
                               id3 = idesc_i8(PX * BN >= 3 * BN ? 3 * BN : BN);
            int q = 0, tc = 0;
            bool alive = true;
            int tile, m0, split;
            for (int L = blockIdx.x; alive && it.get(args, L, tile, m0, split); L += gridDim.x) {
                if (tile >= n_tiles) continue;
                const TileInfo ti = tile_info(args, tile, BN);
                if (ti.n_valid <= 0) continue;
                const int b = tc % ACC;
                const uint32_t acc = tmem + (uint32_t)(b * C::ACC_COLS);
                if (!mbar_wait(&acc_empty[b], ((uint32_t)(tc / ACC) & 1u) ^ 1u, args.err, ERR_TIMEOUT_ACCUM)) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const int kb0 = (int)((long long)split * nkb / ks), kb1 = (int)((long long)(split + 1) * nkb / ks);
                for (int kb = kb0; kb < kb1; ++kb, ++q) {
                    const int s = q % STAGES;
                    const uint32_t ph = (uint32_t)(q / STAGES) & 1u;
                    if (!mbar_wait(&full[s], ph, args.err, ERR_TIMEOUT_FULL)) {
                        alive = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    const uint32_t a_base = smem_u32(sA + s * PW * C::A_PLANE);
                    const uint32_t b_base = smem_u32(sB + s * PX * C::B_PLANE);
                    if constexpr (PX == 3) {
#pragma unroll
                        for (int kk = 0; kk < BK / UMMA_K; ++kk) {
                            const uint64_t a0 = smem_desc_sw128(a_base + 0 * C::A_PLANE + kk * UMMA_K);
                            const uint64_t a1 = smem_desc_sw128(a_base + 1 * C::A_PLANE + kk * UMMA_K);
                            const uint64_t a2 = smem_desc_sw128(a_base + 2 * C::A_PLANE + kk * UMMA_K);
                            const uint64_t b0 = smem_desc_sw128(b_base + 0 * C::B_PLANE + kk * UMMA_K);
                            const uint64_t b2 = smem_desc_sw128(b_base + 2 * C::B_PLANE + kk * UMMA_K);
                            if (kb == kb0 && kk == 0) {
                                // first K step: every diagonal's first product overwrites, the others accumulate
                                umma_i8(acc + 0 * BN, a0, b0, id3, 0u);  // (0,0) (0,1) (0,2) -> diagonals 0, 1, 2
                                umma_i8(acc + 1 * BN, a1, b0, id2, 1u);  // (1,0) (1,1)       -> diagonals 1, 2
                                umma_i8(acc + 3 * BN, a1, b2, id1, 0u);  // (1,2)             -> diagonal 3
                                umma_i8(acc + 2 * BN, a2, b0, id2, 1u);  // (2,0) (2,1)       -> diagonals 2, 3
                                umma_i8(acc + 4 * BN, a2, b2, id1, 0u);  // (2,2)             -> diagonal 4
                            } else {
                                umma_i8(acc + 0 * BN, a0, b0, id3, 1u);
                                umma_i8(acc + 1 * BN, a1, b0, id3, 1u);
                                umma_i8(acc + 2 * BN, a2, b0, id3, 1u);
                            }
                        }
                    } else {
#pragma unroll
                        for (int kk = 0; kk < BK / UMMA_K; ++kk) {
                            const uint64_t bd = smem_desc_sw128(b_base + kk * UMMA_K);
                            const uint32_t first = (kb == kb0 && kk == 0) ? 0u : 1u;  // each MMA owns its diagonal
#pragma unroll
                            for (int j = 0; j < PW; ++j)
                                umma_i8(acc + j * BN, smem_desc_sw128(a_base + j * C::A_PLANE + kk * UMMA_K), bd,
                                        id1, first);
                        }
                    }
                    umma_commit(&empty[s]);  // frees the stage once these MMAs have read it
                }
                umma_commit(&acc_full[b]);  // fires when every MMA issued so far has completed
                ++tc;
            }
            umma_commit(mma_done);
            mbar_wait_drain(mma_done, 0u, args.err, ERR_TIMEOUT_ACCUM);
        }
    } else {
        // Epilogue: warp w reads TMEM lanes 32w..32w+31 (its lane quadrant); lane l holds weight row m0+32w+l.
        const bool do_max = args.rowmax != nullptr;
        int tc = 0;
        int tile, m0, split;
        for (int L = blockIdx.x; it.get(args, L, tile, m0, split); L += gridDim.x) {
            if (tile >= n_tiles) continue;
            const TileInfo ti = tile_info(args, tile, BN);
            if (ti.n_valid <= 0) continue;
            const int b = tc % ACC;
            bool ok = mbar_wait(&acc_full[b], (uint32_t)(tc / ACC) & 1u, args.err, ERR_TIMEOUT_ACCUM);
            ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective: keep the branch warp-uniform
            asm volatile("tcgen05.fence::after_thread_sync;");
            const int m = m0 + warp * 32 + lane;
            const bool m_ok = m < args.M_valid;
            const int my_slot = m >= args.rowmax_split ? 1 : 0;
            const bool one_slot = __all_sync(0xffffffffu, my_slot == __shfl_sync(0xffffffffu, my_slot, 0));
            if (do_max) {
                for (int i = threadIdx.x; i < 2 * 4 * BN; i += 128) sred[i] = 0;
                asm volatile("bar.sync 1, 128;" ::: "memory");
            }
            const uint32_t lane_addr = tmem + (uint32_t)(b * C::ACC_COLS) + ((uint32_t)(warp * 32) << 16);
            const int n_chunks = (ti.n_valid + 15) / 16;
#pragma unroll 1
            for (int c = 0; c < n_chunks; ++c) {
                int32_t s0[16], s1[16], s2[16], s3[16], s4[16];
                if (ok) {
                    tmem_ld16(lane_addr + 0 * BN + c * 16, s0);
                    tmem_ld16(lane_addr + 1 * BN + c * 16, s1);
                    if constexpr (NDIAG_USED == 5) {
                        tmem_ld16(lane_addr + 2 * BN + c * 16, s2);
                        tmem_ld16(lane_addr + 3 * BN + c * 16, s3);
                        tmem_ld16(lane_addr + 4 * BN + c * 16, s4);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) s2[j] = s3[j] = s4[j] = 0;
                    }
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                }
                if (c == n_chunks - 1) {
                    // this thread has read all of buffer b: the MMAs of a later tile may overwrite it
                    asm volatile("tcgen05.fence::before_thread_sync;");
                    mbar_arrive(&acc_empty[b]);
                }
                if (!ok) continue;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int n = c * 16 + j;
                    int64_t v = kt::recombine(s0[j], s1[j], s2[j], s3[j], s4[j]);
                    const bool live = m_ok && n < ti.n_valid;
                    if (live) {
                        int64_t* p = args.out + (long long)(ti.row0 + n) * args.ld_out + m;
                        if (ks > 1) {
                            atomicAdd((unsigned long long*)p, (unsigned long long)v);
                        } else {
                            if (args.accumulate) v += *p;
                            *p = v;
                        }
                    }
                    if (do_max) {
                        unsigned long long av = live ? (unsigned long long)(v >= 0 ? v : -v) : 0ull;
                        if (one_slot) {
#pragma unroll
                            for (int o = 16; o > 0; o >>= 1) {
                                const unsigned long long w = __shfl_xor_sync(0xffffffffu, av, o);
                                av = w > av ? w : av;
                            }
                            if (lane == 0) sred[(my_slot * 4 + warp) * BN + n] = av;
                        } else {
#pragma unroll
                            for (int sl = 0; sl < 2; ++sl) {
                                unsigned long long bv = my_slot == sl ? av : 0ull;
#pragma unroll
                                for (int o = 16; o > 0; o >>= 1) {
                                    const unsigned long long w = __shfl_xor_sync(0xffffffffu, bv, o);
                                    bv = w > bv ? w : bv;
                                }
                                if (lane == 0) sred[(sl * 4 + warp) * BN + n] = bv;
                            }
                        }
                    }
                }
            }
            if (do_max) {
                asm volatile("bar.sync 1, 128;" ::: "memory");
                if (args.rowmax_stride == 0) {
                    // one word per slot for the whole output: reduce the tile's columns first (one atomic per warp)
                    unsigned long long v[2] = {0ull, 0ull};
                    for (int i = threadIdx.x; i < 2 * BN; i += 128) {
                        const int sl = i / BN, n = i % BN;
                        if (n >= ti.n_valid) continue;
#pragma unroll
                        for (int w = 0; w < 4; ++w) v[sl] = max(v[sl], sred[(sl * 4 + w) * BN + n]);
                    }
#pragma unroll
                    for (int sl = 0; sl < 2; ++sl) {
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) {
                            const unsigned long long w = __shfl_xor_sync(0xffffffffu, v[sl], o);
                            v[sl] = w > v[sl] ? w : v[sl];
                        }
                        if (lane == 0 && v[sl]) atomicMax(args.rowmax + sl, v[sl]);
                    }
                } else {
                    for (int i = threadIdx.x; i < 2 * BN; i += 128) {
                        const int sl = i / BN, n = i % BN;
                        unsigned long long v = 0;
#pragma unroll
                        for (int w = 0; w < 4; ++w) v = max(v, sred[(sl * 4 + w) * BN + n]);
                        if (v && n < ti.n_valid)
                            atomicMax(args.rowmax + (long long)(ti.row0 + n) * args.rowmax_stride + sl, v);
                    }
                }
                asm volatile("bar.sync 1, 128;" ::: "memory");  // sred is reused by the next tile
            }
            ++tc;
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
    }
}

// Row maxima of an output written by a K-split launch (the fused epilogue reduction needs final values):
// rowmax[r * stride + (m >= split)] = max |out[r][m]| over m < M_valid (stride 0: one or two words for the whole
// output). One block per row (grid-stride); the words start at zero.
static __global__ void rowmax_kernel(const int64_t* __restrict__ out, long long ld, int rows, int M_valid, int split,
                              unsigned long long* __restrict__ rowmax, int stride) {
    kt::pdl_enter();
    __shared__ unsigned long long red[2][32];
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
        unsigned long long v[2] = {0ull, 0ull};
        for (int m = threadIdx.x; m < M_valid; m += blockDim.x) {
            const int64_t x = out[(long long)r * ld + m];
            const unsigned long long a = (unsigned long long)(x >= 0 ? x : -x);
            const int sl = m >= split ? 1 : 0;
            v[sl] = a > v[sl] ? a : v[sl];
        }
#pragma unroll
        for (int sl = 0; sl < 2; ++sl) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long w = __shfl_xor_sync(0xffffffffu, v[sl], o);
                v[sl] = w > v[sl] ? w : v[sl];
            }
            if ((threadIdx.x & 31) == 0) red[sl][threadIdx.x >> 5] = v[sl];
        }
        __syncthreads();
        if (threadIdx.x < 2) {
            unsigned long long m = 0;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = red[threadIdx.x][w] > m ? red[threadIdx.x][w] : m;
            if (m) atomicMax(rowmax + (long long)r * stride + threadIdx.x, m);
        }
        __syncthreads();
    }
}

}  // namespace dg
