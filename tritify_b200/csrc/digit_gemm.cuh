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
    const int* n_tiles;        // device count of valid n-tiles (nullptr: gridDim.y)
    int single_rows;
    int accumulate;  // 1: out += result (the second and later K chunks)
    int* err;        // device error word (first error wins)
};

__host__ __device__ constexpr int tmem_cols_for(int bn) {
    return (NDIAG * bn <= 32) ? 32 : (NDIAG * bn <= 64) ? 64 : (NDIAG * bn <= 128) ? 128 : (NDIAG * bn <= 256) ? 256 : 512;
}

template <int BN, int STAGES>
struct Cfg {
    static constexpr int A_PLANE = BM * BK;
    static constexpr int B_PLANE = BN * BK;
    static constexpr int STAGE_BYTES = 3 * (A_PLANE + B_PLANE);
    static constexpr int TMEM_COLS = tmem_cols_for(BN);
    static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256;
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 96, "BN: a multiple of 16 in [16, 96]");
    static_assert(NDIAG * BN <= 512, "five accumulators must fit TMEM");
    static_assert(B_PLANE % 1024 == 0, "swizzle atoms stay 1024-byte aligned");
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

// Bounded wait: false (and the error word set) after ~2 s.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
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

template <int BN, int STAGES>
__global__ void __launch_bounds__(THREADS, 1)
    digit_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const GemmArgs args) {
    using C = Cfg<BN, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * 3 * C::A_PLANE;
    uint64_t* full = (uint64_t*)(smem + STAGES * C::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* accum = empty + STAGES;
    uint32_t* tmem_slot = (uint32_t*)(accum + 1);

    const int tile = blockIdx.y;
    const int n_tiles = args.n_tiles ? *args.n_tiles : (int)gridDim.y;
    if (tile >= n_tiles) return;  // the whole CTA leaves before any barrier or allocation
    const int group = args.tile_group ? args.tile_group[tile] : 0;
    const int row0 = args.tile_row0 ? args.tile_row0[tile] : tile * BN;
    const int row_end = args.group_row_end ? args.group_row_end[group] : args.single_rows;
    const int n_valid = min(BN, row_end - row0);
    const int m0 = blockIdx.x * BM;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkb = args.num_k_blocks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
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
        if (lane == 0 && n_valid > 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
            int issued = 0;
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % STAGES;
                const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
                if (!mbar_wait(&empty[s], ph ^ 1u, args.err, ERR_TIMEOUT_EMPTY)) break;
                mbar_arrive_expect_tx(&full[s], (uint32_t)C::STAGE_BYTES);
                const int kx = (args.k_block0 + kb) * BK;
#pragma unroll
                for (int p = 0; p < 3; ++p) {
                    tma_load_2d(sA + (s * 3 + p) * C::A_PLANE, &tmA, kx, (group * 3 + p) * args.M_pad + m0, &full[s]);
                    tma_load_2d(sB + (s * 3 + p) * C::B_PLANE, &tmB, kx, p * args.R_pad + row0, &full[s]);
                }
                issued = kb + 1;
            }
            // Let the copies still in flight land before the CTA can leave (bounded).
            for (int kb = max(0, issued - STAGES); kb < issued; ++kb)
                mbar_wait(&full[kb % STAGES], (uint32_t)(kb / STAGES) & 1u, args.err, ERR_TIMEOUT_FULL);
        }
    } else if (warp == 5) {
        if (lane == 0 && n_valid > 0) {
            constexpr uint32_t idesc = idesc_i8(BN);
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % STAGES;
                const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
                if (!mbar_wait(&full[s], ph, args.err, ERR_TIMEOUT_FULL)) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t a_base = smem_u32(sA + s * 3 * C::A_PLANE);
                const uint32_t b_base = smem_u32(sB + s * 3 * C::B_PLANE);
#pragma unroll
                for (int kk = 0; kk < BK / UMMA_K; ++kk) {
#pragma unroll
                    for (int i = 0; i < 3; ++i) {
#pragma unroll
                        for (int j = 0; j < 3; ++j) {
                            const uint64_t ad = smem_desc_sw128(a_base + i * C::A_PLANE + kk * UMMA_K);
                            const uint64_t bd = smem_desc_sw128(b_base + j * C::B_PLANE + kk * UMMA_K);
                            // The first product of each diagonal in the first K step overwrites its accumulator.
                            const uint32_t acc = (kb > 0 || kk > 0 || !(i == 0 || j == 2)) ? 1u : 0u;
                            umma_i8(tmem + (uint32_t)((i + j) * BN), ad, bd, idesc, acc);
                        }
                    }
                }
                umma_commit(&empty[s]);  // frees the stage once these MMAs have read it
            }
            umma_commit(accum);  // fires when every MMA issued above has completed
        }
    } else {
        // Epilogue: warp w reads TMEM lanes 32w..32w+31 (its lane quadrant); lane l holds weight row m0+32w+l.
        bool ok = true;
        if (n_valid > 0) ok = mbar_wait(accum, 0, args.err, ERR_TIMEOUT_ACCUM);
        ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective: keep the branch warp-uniform
        asm volatile("tcgen05.fence::after_thread_sync;");
        const int m = m0 + warp * 32 + lane;
        const bool m_ok = m < args.M_valid;
        if (ok && n_valid > 0) {
            const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
            for (int c = 0; c < BN / 16; ++c) {
                if (c * 16 >= n_valid) break;
                int32_t s0[16], s1[16], s2[16], s3[16], s4[16];
                tmem_ld16(lane_addr + 0 * BN + c * 16, s0);
                tmem_ld16(lane_addr + 1 * BN + c * 16, s1);
                tmem_ld16(lane_addr + 2 * BN + c * 16, s2);
                tmem_ld16(lane_addr + 3 * BN + c * 16, s3);
                tmem_ld16(lane_addr + 4 * BN + c * 16, s4);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (m_ok) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = c * 16 + j;
                        if (n < n_valid) {
                            const int64_t v = kt::recombine(s0[j], s1[j], s2[j], s3[j], s4[j]);
                            int64_t* p = args.out + (long long)(row0 + n) * args.ld_out + m;
                            *p = args.accumulate ? *p + v : v;
                        }
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
    }
}

}  // namespace dg
