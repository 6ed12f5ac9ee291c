// ktmoe: tritify's integer MoE layer and its exact linear accumulate on B200, behind the C ABI of include/ktmoe.h.
//
// Host side: contexts (device + stream + resident weights), TMA tensor maps, the launch sequence of one layer forward
// and of the decoder block around it, the expert-parallel exchange (NCCL, or peer memory through ep_peer.cuh), the
// seam entry points for experts on other hosts, and the offline f64 preparation entry points. Device side:
// digit_gemm.cuh and digit_gemm_pair.cuh (the tcgen05 digit-plane GEMMs, nine-plane and small-code), moe_kernels.cuh
// (routing, dispatch, SwiGLU/requant, combine, merge, shared expert, RmsNorm, add). The activation wire format is in
// wire.cpp. There is no CPU compute path: every result comes from the kernels in this library (only the routes'
// read-only margin diagnostic is worked out on the host, from logits the kernels produced), and a context on a device
// that is not sm_100 fails to open.

#include <cuda.h>
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <list>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "digit_gemm.cuh"
#include "digit_gemm_pair.cuh"
#include "ep_peer.cuh"
#include "fixed_point.cuh"
#include "host_prep.h"
#include "ktmoe.h"
#include "moe_kernels.cuh"
#include "synth.cuh"

using kt::Scale;

namespace {

inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }
inline Scale S(ktmoe_scale s) { return Scale{s.mant, s.shift}; }
inline ktmoe_scale C(Scale s) { return ktmoe_scale{s.mant, s.shift}; }
inline Scale S(hp::HScale s) { return Scale{s.mant, s.shift}; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    });
    return fn;
}

// A device buffer that only grows.
struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    cudaError_t ensure(size_t want) {
        if (want <= bytes) return cudaSuccess;
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
        cudaError_t e = cudaMalloc(&p, want);
        if (e == cudaSuccess) bytes = want;
        return e;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    template <class T>
    T* as() const {
        return (T*)p;
    }
};

// Pinned host memory, grown on demand (the staging of small LinearBackend transfers).
struct HostBuf {
    void* p = nullptr;
    size_t bytes = 0;
    cudaError_t ensure(size_t want) {
        if (want <= bytes) return cudaSuccess;
        if (p) cudaFreeHost(p);
        p = nullptr;
        bytes = 0;
        cudaError_t e = cudaHostAlloc(&p, want, cudaHostAllocDefault);
        if (e == cudaSuccess) bytes = want;
        return e;
    }
    void release() {
        if (p) cudaFreeHost(p);
        p = nullptr;
        bytes = 0;
    }
};

// Digit planes: [groups][3][rows_pad][k_pad] int8.
struct Planes {
    int8_t* ptr = nullptr;
    int64_t groups = 1, rows_pad = 0, k = 0, k_pad = 0;
};

struct Resident {
    DevBuf buf;
    int64_t out = 0, k = 0, out_pad = 0, k_pad = 0;
    bool small = false;  // every code within ±3280: planes 0 and 1 hold it, plane 2 is zero
    uint64_t last_use = 0;
};

}  // namespace

struct ktmoe_ctx {
    int device = 0;
    int num_sms = 148;
    int pair_clusters = 0;  // co-resident clusters of the pair GEMM on this device (0: not yet queried)
    cudaStream_t stream = nullptr;
    cudaStream_t side = nullptr;  // the shared expert runs here, beside the routed experts
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    cudaEvent_t ev_g0 = nullptr, ev_g1 = nullptr;  // around the last linear call's GEMM (ktmoe_linear_last_gemm)
    int last_gemm_planes = 0;                      // 0: no GEMM timed yet; 3: nine-plane kernel; 1: (1, 2) kernel
    int* d_err = nullptr;
    // pinned host words for the status a linear call reads back with its result: [0..2] the packing counters, [3]
    // the error word (one synchronisation for both, instead of a blocking copy each)
    unsigned long long* h_status = nullptr;
    std::string last_error = "";
    uint64_t launches = 0;
    std::mutex mu;
    // LinearBackend scratch
    DevBuf lin_xi, lin_wi, lin_xp, lin_xr, lin_wp, lin_y, lin_bad;
    // pinned staging of a call's activations and result up to LIN_STAGE_MAX bytes each: a copy through pageable
    // memory costs the driver's own staging and a blocking wait per transfer, which dominate decode-sized calls
    HostBuf lin_hx, lin_hy;
    // resident weights (linear_weights)
    std::unordered_map<uint64_t, Resident*> cache;
    uint64_t budget = 0, resident = 0, tick = 0;
};

namespace {

int fail(ktmoe_ctx* ctx, int status, const std::string& what) {
    if (ctx) ctx->last_error = what;
    return status;
}

int fail_cuda(ktmoe_ctx* ctx, cudaError_t e, const char* what) {
    return fail(ctx, KTMOE_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define CK(expr)                                                        \
    do {                                                                \
        cudaError_t e__ = (expr);                                       \
        if (e__ != cudaSuccess) return fail_cuda(ctx, e__, #expr);      \
    } while (0)

#define CKL(ctx)                                                        \
    do {                                                                \
        ++(ctx)->launches;                                              \
        cudaError_t e__ = cudaGetLastError();                           \
        if (e__ != cudaSuccess) return fail_cuda(ctx, e__, "kernel launch"); \
    } while (0)

// Programmatic dependent launch of this library's kernels (every one begins with kt::pdl_enter(), which waits for
// the kernel before it on the stream): a kernel is scheduled while its predecessor finishes, which hides most of the
// gap between two dependent launches. KTMOE_PDL=0, read once, launches them plainly.
bool pdl_on() {
    static const bool on = [] {
        const char* e = getenv("KTMOE_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

// One launch of `kernel` on clusters of `cluster` CTAs along x (1: no cluster attribute).
template <typename... KArgs, typename... Args>
int launch_kc(ktmoe_ctx* ctx, cudaStream_t st, dim3 grid, dim3 block, size_t smem, unsigned cluster,
              void (*kernel)(KArgs...), Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    int na = 0;
    if (pdl_on()) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (cluster > 1) {
        at[na].id = cudaLaunchAttributeClusterDimension;
        at[na].val.clusterDim.x = cluster;
        at[na].val.clusterDim.y = 1;
        at[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = at;
    cfg.numAttrs = na;
    CK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
    CKL(ctx);
    return KTMOE_OK;
}

template <typename... KArgs, typename... Args>
int launch_k(ktmoe_ctx* ctx, cudaStream_t st, dim3 grid, dim3 block, size_t smem, void (*kernel)(KArgs...),
             Args&&... args) {
    return launch_kc(ctx, st, grid, block, smem, 1u, kernel, std::forward<Args>(args)...);
}

// KLAUNCH(stream, grid, block, shared bytes, (kernel), args...): launch_k, returning its status on failure; one
// statement (safe under an unbraced if / else).
#define KLAUNCH(...)                                                   \
    do {                                                               \
        if (int r_kl__ = launch_k(ctx, __VA_ARGS__)) return r_kl__;    \
    } while (0)
// KLAUNCHC(stream, grid, block, shared bytes, cluster size, (kernel), args...): the same through launch_kc.
#define KLAUNCHC(...)                                                  \
    do {                                                               \
        if (int r_kl__ = launch_kc(ctx, __VA_ARGS__)) return r_kl__;   \
    } while (0)

int make_map(ktmoe_ctx* ctx, CUtensorMap* map, const void* base, int64_t k_pad, int64_t rows_total, int box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(ctx, KTMOE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t gdim[2] = {(cuuint64_t)k_pad, (cuuint64_t)rows_total};
    cuuint64_t gstride[1] = {(cuuint64_t)k_pad};
    cuuint32_t box[2] = {(cuuint32_t)dg::BK, (cuuint32_t)box_rows};
    cuuint32_t estride[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), gdim, gstride, box, estride,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(ctx, KTMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return KTMOE_OK;
}

template <int BN, int ST, int ACC, int PX = 3, int PW = 3>
int launch_gemm_t(ktmoe_ctx* ctx, cudaStream_t st, const CUtensorMap& ma, const CUtensorMap& mb, dim3 grid,
                  const dg::GemmArgs& args) {
    using Cf = dg::Cfg<BN, ST, ACC, PX, PW>;
    static bool attr_set[64] = {};
    if (!attr_set[ctx->device & 63]) {
        CK(cudaFuncSetAttribute(dg::digit_gemm_kernel<BN, ST, ACC, PX, PW>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM_BYTES));
        attr_set[ctx->device & 63] = true;
    }
    KLAUNCH(st, grid, dg::THREADS, Cf::SMEM_BYTES, (dg::digit_gemm_kernel<BN, ST, ACC, PX, PW>), ma, mb, args);
    return KTMOE_OK;
}

// The pair GEMM (tcgen05 cta_group::2) is used for 64-row tiles of weights padded to 256 rows unless KTMOE_PAIR=0.
bool pair_enabled() {
    const char* e = getenv("KTMOE_PAIR");
    return !(e && e[0] == '0');
}

int launch_gemm_pair(ktmoe_ctx* ctx, cudaStream_t st, const CUtensorMap& ma, const CUtensorMap& mb, int64_t slots,
                     const dg::GemmArgs& args) {
    static bool attr_set[64] = {};
    if (!attr_set[ctx->device & 63]) {
        CK(cudaFuncSetAttribute(dg::digit_gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                dg::pair::SMEM_BYTES));
        attr_set[ctx->device & 63] = true;
    }
    if (ctx->pair_clusters == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(2 * (ctx->num_sms / 2)));
        cfg.blockDim = dim3(dg::pair::THREADS);
        cfg.dynamicSmemBytes = dg::pair::SMEM_BYTES;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 2;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, dg::digit_gemm_pair_kernel, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = ctx->num_sms / 2;
        }
        ctx->pair_clusters = std::min(n, ctx->num_sms / 2);
    }
    const int64_t clusters = std::min<int64_t>(slots, ctx->pair_clusters);
    KLAUNCH(st, dim3((unsigned)(2 * clusters)), dg::pair::THREADS, dg::pair::SMEM_BYTES, (dg::digit_gemm_pair_kernel),
            ma, mb, args);
    return KTMOE_OK;
}

struct GemmCall {
    Planes A;        // weights: groups x 3 x M_pad x k_pad
    int64_t M_valid;
    Planes B;        // activations: 3 x R_pad x k_pad (one raw plane R_pad x k_pad when `small`)
    bool small = false;  // |x| <= 127 and |w| <= 3280: the (1, 2) plane GEMM on weight planes 0 and 1
    cudaEvent_t ev0 = nullptr;  // when set, recorded on the stream just before the first launch (after the maps)
    int64_t* out;
    int64_t ld_out;
    int BN;
    int64_t grid_y;
    const int* tile_group = nullptr;
    const int* tile_row0 = nullptr;
    const int* group_end = nullptr;
    const int* tile_row_end = nullptr;
    const int* n_tiles = nullptr;
    int64_t single_rows = 0;
    unsigned long long* rowmax = nullptr;  // fused |max| per (row, slot); see dg::GemmArgs
    int rowmax_stride = 0;
    int64_t rowmax_split = 0;
};

// The small-code GEMM on SM pairs (dg::digit_gemm_pair_small_kernel): 256 activation rows x 128 weight rows per
// tile, clusters of 2, one launch per K chunk.
int launch_gemm_pair_small(ktmoe_ctx* ctx, cudaStream_t st, const CUtensorMap& mx, const CUtensorMap& mw,
                           int64_t slots, const dg::GemmArgs& args) {
    namespace ps = dg::pair_small;
    static bool attr_set[64] = {};
    static int clusters_of[64] = {};
    const int dev = ctx->device & 63;
    if (!attr_set[dev]) {
        CK(cudaFuncSetAttribute(dg::digit_gemm_pair_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                ps::SMEM_BYTES));
        attr_set[dev] = true;
    }
    if (clusters_of[dev] == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(2 * (ctx->num_sms / 2)));
        cfg.blockDim = dim3(ps::THREADS);
        cfg.dynamicSmemBytes = ps::SMEM_BYTES;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 2;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, dg::digit_gemm_pair_small_kernel, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = ctx->num_sms / 2;
        }
        clusters_of[dev] = std::min(n, ctx->num_sms / 2);
    }
    const int64_t clusters = std::min<int64_t>(slots, clusters_of[dev]);
    KLAUNCH(st, dim3((unsigned)(2 * clusters)), ps::THREADS, ps::SMEM_BYTES, (dg::digit_gemm_pair_small_kernel), mx, mw,
            args);
    return KTMOE_OK;
}

// Small codes with at least 128 activation rows, one weight matrix and no fused row maxima go to the SM pairs
// (KTMOE_PAIR=0 keeps them on the one-SM (1, 2) kernel).
bool small_pair_ok(const GemmCall& g) {
    return g.small && pair_enabled() && g.single_rows >= 128 && !g.rowmax && !g.tile_group && !g.tile_row0 &&
           !g.group_end && !g.tile_row_end && !g.n_tiles && g.A.groups == 1 &&
           g.A.rows_pad % dg::pair_small::BN_W == 0;
}

int run_gemm_small_pair(ktmoe_ctx* ctx, cudaStream_t st, const GemmCall& g) {
    namespace ps = dg::pair_small;
    const int64_t rows = g.single_rows;
    const int64_t w_tiles = g.A.rows_pad / ps::BN_W;
    const int64_t a_tiles = (rows + ps::BM_ACT - 1) / ps::BM_ACT;
    const int64_t group_n = std::min<int64_t>(16, a_tiles);
    const int64_t n_groups = (a_tiles + group_n - 1) / group_n;
    const int64_t slots = w_tiles * group_n * n_groups;
    if (slots > INT32_MAX) return fail(ctx, KTMOE_ERR_UNSUPPORTED, "too many tiles for one launch");
    CUtensorMap mx, mw;
    int r = make_map(ctx, &mx, g.B.ptr, g.B.k_pad, g.B.rows_pad, 128);
    if (r) return r;
    r = make_map(ctx, &mw, g.A.ptr, g.A.k_pad, g.A.groups * 3 * g.A.rows_pad, ps::BN_W);
    if (r) return r;
    if (g.ev0) CK(cudaEventRecord(g.ev0, st));
    const int64_t total_kb = (g.A.k + dg::BK - 1) / dg::BK;
    const int64_t chunk_kb = dg::K_EXACT_MAX_SMALL / dg::BK;
    for (int64_t kb0 = 0; kb0 < total_kb; kb0 += chunk_kb) {
        dg::GemmArgs a{};
        a.out = g.out;
        a.ld_out = g.ld_out;
        a.M_valid = (int)g.M_valid;
        a.M_pad = (int)g.A.rows_pad;
        a.k_block0 = (int)kb0;
        a.num_k_blocks = (int)std::min(chunk_kb, total_kb - kb0);
        a.R_pad = (int)g.B.rows_pad;
        a.n_tiles_max = (int)a_tiles;
        a.m_tiles = (int)w_tiles;
        a.group_n = (int)group_n;
        a.single_rows = (int)rows;
        a.accumulate = kb0 > 0 ? 1 : 0;
        a.err = ctx->d_err;
        a.k_splits = 1;
        r = launch_gemm_pair_small(ctx, st, mx, mw, slots, a);
        if (r) return r;
    }
    return KTMOE_OK;
}

// Launch the digit GEMM, splitting K into chunks whose int32 diagonal sums cannot overflow.
int run_gemm(ktmoe_ctx* ctx, cudaStream_t st, const GemmCall& g) {
    if (g.grid_y <= 0 || g.M_valid <= 0) return KTMOE_OK;
    if (small_pair_ok(g)) return run_gemm_small_pair(ctx, st, g);
    const bool pair = !g.small && g.BN == dg::pair::BN && g.A.rows_pad % dg::pair::BM2 == 0 && pair_enabled();
    const int64_t group_n = std::min<int64_t>(16, g.grid_y);
    const int64_t m_tiles = g.A.rows_pad / (pair ? dg::pair::BM2 : dg::BM);
    const int64_t n_groups = (g.grid_y + group_n - 1) / group_n;
    if (m_tiles * group_n * n_groups > INT32_MAX) return fail(ctx, KTMOE_ERR_UNSUPPORTED, "too many tiles for one launch");
    CUtensorMap ma, mb;
    int r = make_map(ctx, &ma, g.A.ptr, g.A.k_pad, g.A.groups * 3 * g.A.rows_pad, dg::BM);
    if (r) return r;
    r = make_map(ctx, &mb, g.B.ptr, g.B.k_pad, (g.small ? 1 : 3) * g.B.rows_pad, pair ? dg::pair::BOX_ROWS : g.BN);
    if (r) return r;
    const int64_t total_kb = (g.A.k + dg::BK - 1) / dg::BK;
    const int64_t chunk_kb = (g.small ? dg::K_EXACT_MAX_SMALL : dg::K_EXACT_MAX) / dg::BK;
    if (g.rowmax && total_kb > chunk_kb) return fail(ctx, KTMOE_ERR_UNSUPPORTED, "fused row max with a chunked K");
    // Split K when the tiles cannot fill the SMs (small row counts): one output matrix (no groups), one K chunk, the
    // one-SM kernel; the row maxima then come from a pass over the finished output. KTMOE_SPLITK=0 turns it off.
    const int64_t slots = m_tiles * group_n * n_groups;
    int ks = 1;
    {
        const char* e = getenv("KTMOE_SPLITK");
        const bool single = !g.tile_group && !g.group_end && !g.tile_row_end && !g.n_tiles;
        if (!(e && e[0] == '0') && !pair && single && total_kb <= chunk_kb && 2 * slots <= ctx->num_sms) {
            ks = (int)std::min<int64_t>({ctx->num_sms / slots, total_kb / 2, 16});
            if (ks < 2) ks = 1;
        }
    }
    if (g.ev0) CK(cudaEventRecord(g.ev0, st));
    if (ks > 1) CK(cudaMemsetAsync(g.out, 0, (size_t)g.single_rows * g.ld_out * 8, st));
    // persistent: at most one block per SM walks the tile raster
    dim3 grid((unsigned)std::min<int64_t>(slots * ks, ctx->num_sms));
    for (int64_t kb0 = 0; kb0 < total_kb; kb0 += chunk_kb) {
        dg::GemmArgs a{};
        a.out = g.out;
        a.ld_out = g.ld_out;
        a.M_valid = (int)g.M_valid;
        a.M_pad = (int)g.A.rows_pad;
        a.k_block0 = (int)kb0;
        a.num_k_blocks = (int)std::min(chunk_kb, total_kb - kb0);
        a.R_pad = (int)g.B.rows_pad;
        a.tile_group = g.tile_group;
        a.tile_row0 = g.tile_row0;
        a.group_row_end = g.group_end;
        a.tile_row_end = g.tile_row_end;
        a.n_tiles = g.n_tiles;
        a.n_tiles_max = (int)g.grid_y;
        a.m_tiles = (int)m_tiles;
        a.group_n = (int)group_n;
        a.single_rows = (int)g.single_rows;
        a.accumulate = kb0 > 0 ? 1 : 0;
        a.err = ctx->d_err;
        a.rowmax = ks > 1 ? nullptr : g.rowmax;
        a.rowmax_stride = g.rowmax_stride;
        a.rowmax_split = (int)std::min<int64_t>(g.rowmax_split, INT32_MAX);
        a.k_splits = ks;
        {
            const char* ze = getenv("KTMOE_PAIR_ZERO_MMA");
            a.zero_mma = (ze && ze[0] == '1') ? 1 : 0;
        }
        if (pair) {
            r = launch_gemm_pair(ctx, st, ma, mb, m_tiles * group_n * n_groups, a);
            if (r) return r;
            continue;
        }
        if (g.small) {
            switch (g.BN) {
                case 16: r = launch_gemm_t<16, 4, 2, 1, 2>(ctx, st, ma, mb, grid, a); break;
                case 32: r = launch_gemm_t<32, 3, 2, 1, 2>(ctx, st, ma, mb, grid, a); break;
                case 48: r = launch_gemm_t<48, 3, 2, 1, 2>(ctx, st, ma, mb, grid, a); break;
                case 64: r = launch_gemm_t<64, 3, 1, 1, 2>(ctx, st, ma, mb, grid, a); break;
                case 128: r = launch_gemm_t<128, 4, 2, 1, 2>(ctx, st, ma, mb, grid, a); break;
                default: return fail(ctx, KTMOE_ERR_ARG, "unsupported BN");
            }
            if (r) return r;
            continue;
        }
        switch (g.BN) {
            case 16: r = launch_gemm_t<16, 4, 2>(ctx, st, ma, mb, grid, a); break;
            case 32: r = launch_gemm_t<32, 3, 2>(ctx, st, ma, mb, grid, a); break;
            case 48: r = launch_gemm_t<48, 3, 2>(ctx, st, ma, mb, grid, a); break;
            case 64: r = launch_gemm_t<64, 3, 1>(ctx, st, ma, mb, grid, a); break;
            default: return fail(ctx, KTMOE_ERR_ARG, "unsupported BN");
        }
        if (r) return r;
    }
    if (ks > 1 && g.rowmax) {
        KLAUNCH(st, (unsigned)std::max<int64_t>(1, std::min<int64_t>(g.single_rows, ctx->num_sms * 4)), 256, 0,
                (dg::rowmax_kernel), g.out, g.ld_out, (int)g.single_rows, (int)g.M_valid,
                (int)std::min<int64_t>(g.rowmax_split, INT32_MAX), g.rowmax, g.rowmax_stride);
    }
    return KTMOE_OK;
}

// Activation rows per tile. With weights padded to 256 rows and at least 64 rows per group, 64-row tiles on the SM
// pair (each SM reads half of the stacked activation tile). Otherwise, on one SM, 48 keeps two accumulator buffers
// in TMEM (the epilogue overlaps the next tile's MMAs) while three stacked planes still give one 144-wide MMA per
// weight plane. KTMOE_BN overrides it (16/32/48/64).
int pick_bn(double rows_per_group, bool pair_ok = false) {
    static int forced = [] {
        const char* e = getenv("KTMOE_BN");
        int v = e ? atoi(e) : 0;
        return (v == 16 || v == 32 || v == 48 || v == 64) ? v : 0;
    }();
    if (forced) return forced;
    if (pair_ok && rows_per_group >= 64.0 && pair_enabled()) return 64;
    if (rows_per_group >= 40.0) return 48;
    if (rows_per_group >= 20.0) return 32;
    return 16;
}

// Activation rows per tile of the small-code (1, 2) kernel: 128 once there are enough rows — two MMAs of N = 128
// per K step against 48 KB of operands per 128-byte K block, with two accumulator buffers of 2·128 TMEM columns —
// else the one-SM choice of the nine-plane kernel. KTMOE_BN_SMALL overrides it (16/32/48/64/128).
int pick_bn_small(double rows) {
    static int forced = [] {
        const char* e = getenv("KTMOE_BN_SMALL");
        int v = e ? atoi(e) : 0;
        return (v == 16 || v == 32 || v == 48 || v == 64 || v == 128) ? v : 0;
    }();
    if (forced) return forced;
    if (rows >= 96.0) return 128;
    return pick_bn(rows, false);
}

__global__ void sqx_kernel(const unsigned long long* gxmax, const Scale* x_scale, Scale* out) {
    kt::pdl_enter();
    const int64_t xm = (int64_t)*gxmax;
    *out = xm > 0 ? kt::scale_mul(kt::from_ratio((kt::u128)(uint64_t)xm, (kt::u128)kt::WLEVELS), *x_scale)
                  : kt::scale_zero();
}

// The down GEMM's width: a long K (d_ff >= 4096) amortises a single-buffered accumulator, and a 64-row tile reads
// the least shared memory per MMA; otherwise the same choice as the gate/up GEMM. KTMOE_BN_DOWN overrides it.
int pick_bn_long_k(double rows_per_group, int64_t k, bool pair_ok = false) {
    static int forced = [] {
        const char* e = getenv("KTMOE_BN_DOWN");
        int v = e ? atoi(e) : 0;
        return (v == 16 || v == 32 || v == 48 || v == 64) ? v : 0;
    }();
    if (forced) return forced;
    if (k >= 4096 && rows_per_group >= 48.0) return 64;
    return pick_bn(rows_per_group, pair_ok);
}

int set_device(ktmoe_ctx* ctx) {
    CK(cudaSetDevice(ctx->device));
    return KTMOE_OK;
}

int check_err_word(ktmoe_ctx* ctx) {
    int h = 0;
    CK(cudaMemcpy(&h, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (h != 0) {
        CK(cudaMemset(ctx->d_err, 0, sizeof(int)));
        return fail(ctx, KTMOE_ERR_KERNEL, "a kernel's bounded wait expired (code " + std::to_string(h) + ")");
    }
    return KTMOE_OK;
}

}  // namespace

// ───────────────────────────── the layer ─────────────────────────────

// The weights of one layer of a stack (ktmoe_layer_set_depth): every buffer and scale the forward reads that differs
// from one layer to the next. The selected slot's weights live in the layer's own fields (ktmoe_layer_select swaps
// them in and out); scratch, tables and the expert-parallel exchange are shared by all slots.
struct WeightSet {
    Planes w_router, w_gu, w_dn, w_sgu, w_sdn;
    DevBuf b_router, b_gu, b_dn, b_sgu, b_sdn, b_rbias, b_sigbias, b_wsc, b_norm, b_sgate;
    std::vector<Scale> h_wsc;
    std::vector<char> expert_set;
    Scale router_ws{0, 0}, router_bscale{0, 0}, norm_ws{0, 0}, norm_eps{0, 0}, sgate_ws{0, 0};
    bool has_rbias = false, router_set = false, shared_set = false, sigbias_set = false, norm_set = false,
         sgate_set = false;
};

static void release_weights(WeightSet& w) {
    DevBuf* bufs[] = {&w.b_router, &w.b_gu, &w.b_dn, &w.b_sgu, &w.b_sdn, &w.b_rbias, &w.b_sigbias, &w.b_wsc,
                      &w.b_norm, &w.b_sgate};
    for (DevBuf* b : bufs) b->release();
}

struct ktmoe_layer {
    ktmoe_ctx* ctx = nullptr;
    ktmoe_layer_config cfg{};
    int64_t d = 0, E = 0, f = 0, K = 0, fs = 0;
    // expert parallelism: this rank owns experts [e_begin, e_end) of E (E_local = e_end - e_begin)
    int rank = 0, world = 1;
    int64_t e_begin = 0, e_end = 0, E_local = 0;
    ncclComm_t comm = nullptr;
    DevBuf ep_counts, ep_counts_all, ep_meta_send, ep_meta_recv, ep_recv_planes, ep_recv_sqx, ep_recv_row_expert,
        ep_y_send, ep_ys_send, ep_y_back, ep_ys_back, ep_tiles, ep_runs, ep_rec, ep_recs, ep_best_idx;
    std::vector<int> h_counts;
    int64_t ep_tok_offset = 0, ep_tok_total = 0;
    // the peer-memory transport (ktmoe_layer_set_ep_capacity): one IPC-shared region per rank
    struct Peer {
        bool on = false;
        int64_t cap_T = 0, cap_rows = 0, cap_home = 0, bytes = 0;
        DevBuf region;
        void* opened[ep::MAXW] = {};
        ep::Peers P{};
        DevBuf seq_dev, ctr, dst_base, rows_recv, group_end, tiles, tok_info, recv_sqx, recv_expert;
    } peer;
    int64_t d_pad = 0, f_pad = 0, fs_pad = 0;
    Planes w_router, w_gu, w_dn, w_sgu, w_sdn;
    DevBuf b_router, b_gu, b_dn, b_sgu, b_sdn;
    bool router_set = false, shared_set = false, sigbias_set = false;
    std::vector<char> expert_set;
    Scale router_ws{0, 0}, router_bscale{0, 0};
    bool has_rbias = false;
    DevBuf b_rbias, b_sigbias;
    // extension: the sigmoid-gated shared expert (ktmoe_layer_set_shared_gate); the gate's codes zero-padded to d_pad
    bool sgate_set = false;
    DevBuf b_sgate, sg_acc, sg_code, y_gated;
    Scale sgate_ws{0, 0};
    // device scales: [0,E) gate, [E,2E) up, [2E,3E) down, then shared gate, up, down
    DevBuf b_wsc;
    std::vector<Scale> h_wsc;
    DevBuf b_luts;  // 3 x 65536 int64: exp, SiLU, sigmoid
    DevBuf b_silu32;  // the SiLU codes as int32 (they all fit: |silu(x)|·2^20 < 2^25 on [-30, 30])
    bool silu32 = false;
    hp::HTable tabs[3];
    Scale silu_code_scale_recip{0, 0};
    int64_t swiglu_smem = 0;  // dynamic shared bytes holding one row's h (0: h stays in global memory)
    // scratch for `cap` tokens
    int64_t cap = 0;
    DevBuf x_in, y_out, scal;  // scal: Scales and u64 scalars
    DevBuf tok_planes, tok_xmax, tok_sqx, router_acc, logits, logit_scale, top_e, top_ec, sumc;
    DevBuf counts, chunk_off, expert_off, group_end, expert_count, tile_group, tile_row0, tile_group2, tile_row02,
        slot_row, row_assign, row_expert;
    DevBuf xg_planes, acc_gu, hq_planes, row_cd, acc_d, tok_out, tok_scale, y_routed, rowmax_gu, rowmax_d;
    DevBuf swiglu_plans, row_hmax, shared_plan;  // per-row SwiGLU scale plans and max |h|; the shared expert's plan
    DevBuf cp_n, cp_common, cp_row, cp_ec, cp_ry, cp_f;  // per-token combine plans
    DevBuf xs_planes, acc_sgu, hs_planes, acc_sd;
    DevBuf seam_y, seam_ys, seam_ids;  // the expert-output seam (ktmoe_layer_expert_forward / _forward_with_experts)
    // optional per-stage CUDA-event timing: one event per stage boundary per timed forward
    bool timing = false;
    // the block around the layer (ktmoe_layer_set_norm): the FFN input RmsNorm and the residual add
    bool norm_set = false;
    DevBuf b_norm;  // int32 [d]: the norm's weight codes
    Scale norm_ws{0, 0}, norm_eps{0, 0};
    DevBuf blk_c, blk_xn, blk_m, blk_sc, blk_u64, blk_off;
    int64_t blk_cap = 0;
    // CUDA graphs of the forward (ktmoe_layer_set_graphs), keyed by the call's pointers, rows and stream
    struct Graph {
        const void *x, *xs, *y, *ys;
        int64_t T;
        cudaStream_t st;
        cudaGraphExec_t exec;
        uint64_t launches;  // this library's kernels in the graph
        bool block;         // the block forward (norm, layer, residual add) rather than the layer alone
        int slot;           // the weight slot it ran with
    };
    bool graphs = false;
    std::vector<Graph> graph_cache;
    std::vector<cudaEvent_t> events;
    // a stack of layers in one object (ktmoe_layer_set_depth): slots[active] is empty while its weights are in the
    // fields above
    std::vector<WeightSet> slots;
    int active = 0;
    // asynchronous host-buffer forwards (ktmoe_forward_async): two slots of device buffers, an upload and a download
    // stream ordered against the context stream by events, so one call's copies overlap another's forward
    struct Async {
        bool init = false;
        cudaStream_t up = nullptr, down = nullptr;
        DevBuf x[2], y[2], sc;  // sc: per slot {x scale, y scale}
        HostBuf hsc;            // pinned: per slot {x scale, y scale}
        cudaEvent_t ev_up[2] = {}, ev_fwd[2] = {}, ev_down[2] = {};
        bool pending[2] = {false, false};
        ktmoe_scale* ys_out[2] = {nullptr, nullptr};
        uint64_t calls = 0;
    } as;
};

namespace {

// Scalar slots inside layer->scal.
enum ScalarSlot {
    SL_XSCALE = 0,   // Scale
    SL_YSCALE = 1,   // Scale (routed result scale when a shared expert follows)
    SL_COMMON = 2,   // Scale[2]: common, its reciprocal
    SL_GSQX = 4,     // Scale: the shared expert's s_qx
    SL_ADD = 5,      // Scale[4]: add scratch
    SL_SCD = 9,      // Scale: shared down c
    SL_YROUTED = 10, // Scale: routed scale (with shared)
    SL_GATED = 12,   // Scale: the gated shared output's scale
    SL_ADD2 = 13,    // Scale[3]: add(routed, gated) plan {common, fa, fb}
    SL_NSCALES = 16
};
enum U64Slot { U_MERGE_GMAX = 0, U_GXMAX, U_SYG, U_SYU, U_SHMAX, U_SYD, U_ADDGMAX, U_GYMAX, U_GATEDMAX, U_NTILES_PAD,
               U_N };
// the two n-tile counts live in the two 32-bit halves of U_NTILES_PAD

Scale* scal_scale(ktmoe_layer* L, int slot) { return L->scal.as<Scale>() + slot; }
unsigned long long* scal_u64(ktmoe_layer* L, int slot) {
    return (unsigned long long*)(L->scal.as<uint8_t>() + SL_NSCALES * sizeof(Scale)) + slot;
}
int* n_tiles_ptr(ktmoe_layer* L) { return (int*)(scal_u64(L, U_NTILES_PAD)); }
int* n_tiles2_ptr(ktmoe_layer* L) { return (int*)(scal_u64(L, U_NTILES_PAD)) + 1; }

// Buffers of the routed experts for `rows` expert rows (the home's rows on one rank, the received rows with EP).
int ensure_rows(ktmoe_layer* L, int64_t rows) {
    ktmoe_ctx* ctx = L->ctx;
    const int64_t n = std::max<int64_t>(rows, 1), n_pad = round_up(n, 64);
    CK(L->acc_gu.ensure(n * 2 * L->f * 8));
    CK(L->hq_planes.ensure(3 * n_pad * L->f_pad));
    CK(L->row_cd.ensure(n * sizeof(Scale)));
    CK(L->acc_d.ensure(n * L->d * 8));
    CK(L->rowmax_gu.ensure(n * 2 * 8));
    CK(L->rowmax_d.ensure(n * 8));
    CK(L->swiglu_plans.ensure(n * sizeof(mk::SwigluScales)));
    CK(L->row_hmax.ensure(n * 8));
    return KTMOE_OK;
}

void graphs_clear(ktmoe_layer* L) {
    if (L->graph_cache.empty()) return;
    for (auto& g : L->graph_cache) cudaStreamSynchronize(g.st);  // no launch of these graphs is still in flight
    for (auto& g : L->graph_cache) cudaGraphExecDestroy(g.exec);
    L->graph_cache.clear();
}

int ensure_scratch(ktmoe_layer* L, int64_t T) {
    ktmoe_ctx* ctx = L->ctx;
    if (T <= L->cap && L->cap > 0 && (!L->sgate_set || L->y_gated.bytes >= (size_t)(T * L->d * 4))) return KTMOE_OK;
    graphs_clear(L);  // the scratch moves: graphs that name it are stale
    const int64_t d = L->d, E = L->E, K = L->K, fs = L->fs;
    T = std::max<int64_t>(T, 1);
    const int64_t R = T * K;
    const int64_t T_pad = round_up(std::max<int64_t>(T, 1), 64), R_pad = round_up(std::max<int64_t>(R, 1), 64);
    const int64_t nchunks = (R + mk::PLAN_CHUNK - 1) / mk::PLAN_CHUNK;
    const int64_t max_tiles = (R + 15) / 16 + E;
    CK(L->x_in.ensure(T * d * 4));
    CK(L->y_out.ensure(T * d * 4));
    CK(L->scal.ensure(SL_NSCALES * sizeof(Scale) + U_N * 8));
    CK(L->tok_planes.ensure(3 * T_pad * L->d_pad));
    CK(L->tok_xmax.ensure(T * 8));
    CK(L->tok_sqx.ensure(T * sizeof(Scale)));
    CK(L->router_acc.ensure(T * E * 8));
    CK(L->logits.ensure(T * E * 4));
    CK(L->logit_scale.ensure(T * sizeof(Scale)));
    CK(L->top_e.ensure(R * 4));
    CK(L->top_ec.ensure(R * 8));
    CK(L->cp_n.ensure(T * 4));
    CK(L->cp_common.ensure(T * sizeof(Scale)));
    CK(L->cp_row.ensure(R * 4));
    CK(L->cp_ec.ensure(R * 8));
    CK(L->cp_ry.ensure(R * sizeof(kt::ReqDiv)));
    CK(L->cp_f.ensure(R * sizeof(kt::ApplyPlan)));
    CK(L->sumc.ensure(T * 8));
    CK(L->counts.ensure(std::max<int64_t>(nchunks, 1) * E * 4));
    CK(L->chunk_off.ensure(std::max<int64_t>(nchunks, 1) * E * 4));
    CK(L->expert_off.ensure(E * 4));
    CK(L->group_end.ensure(E * 4));
    CK(L->expert_count.ensure(E * 4));
    CK(L->tile_group.ensure(max_tiles * 4));
    CK(L->tile_row0.ensure(max_tiles * 4));
    CK(L->tile_group2.ensure(max_tiles * 4));
    CK(L->tile_row02.ensure(max_tiles * 4));
    CK(L->slot_row.ensure(R * 4));
    CK(L->row_assign.ensure(R * 4));
    CK(L->row_expert.ensure(R * 4));
    CK(L->xg_planes.ensure(3 * R_pad * L->d_pad));
    if (int r = ensure_rows(L, R)) return r;
    CK(L->tok_out.ensure(T * d * 4));
    CK(L->tok_scale.ensure(T * sizeof(Scale)));
    if (fs > 0) {
        CK(L->y_routed.ensure(T * d * 4));
        CK(L->xs_planes.ensure(3 * T_pad * L->d_pad));
        CK(L->acc_sgu.ensure(T * 2 * fs * 8));
        CK(L->hs_planes.ensure(3 * T_pad * L->fs_pad));
        CK(L->acc_sd.ensure(T * d * 8));
        if (L->sgate_set) {
            CK(L->sg_acc.ensure(T * 8));
            CK(L->sg_code.ensure(T * 8));
            CK(L->y_gated.ensure(T * d * 4));
        }
    }
    L->cap = T;
    return KTMOE_OK;
}

bool layer_complete(const ktmoe_layer* L) {
    if (!L->router_set) return false;
    for (char c : L->expert_set)
        if (!c) return false;
    if (L->fs > 0 && !L->shared_set) return false;
    if (L->cfg.router_score == 1 && !L->sigbias_set) return false;
    return true;
}

// Stage boundaries recorded when timing is on (see ktmoe_layer_stage_times).
// ST_XIN (the wait for the rows other ranks send) and ST_XOUT (the return of expert outputs to their home ranks) are
// empty on one GPU: every path records the same boundaries.
enum Stage {
    ST_ROUTE = 0, ST_DISPATCH, ST_XIN, ST_GEMM_GU, ST_SWIGLU, ST_GEMM_DOWN, ST_XOUT, ST_COMBINE, ST_MERGE, ST_SHARED,
    ST_N
};

int mark(ktmoe_layer* L, cudaStream_t st) {
    if (!L->timing) return KTMOE_OK;
    ktmoe_ctx* ctx = L->ctx;
    cudaEvent_t e;
    CK(cudaEventCreate(&e));
    L->events.push_back(e);
    CK(cudaEventRecord(e, st));
    return KTMOE_OK;
}

#define MARK(L, st)                              \
    do {                                         \
        if (int m__ = mark((L), (st))) return m__; \
    } while (0)

mk::Lut lut(const ktmoe_layer* L, int kind) {
    mk::Lut l;
    l.codes = L->b_luts.as<int64_t>() + (int64_t)kind * mk::LUT_N;
    l.codes32 = (kind == 1 && L->silu32) ? L->b_silu32.as<int32_t>() : nullptr;
    l.inv_step = S(L->tabs[kind].inv_step);
    l.lo_index = L->tabs[kind].lo_index;
    return l;
}

// Each token row's quantiser (xmax, quant_to, the digit planes, s_qx): tok_planes, tok_xmax, tok_sqx.
int stage_quant(ktmoe_layer* L, int64_t T, const int32_t* x_dev, const Scale* xs_dev, cudaStream_t st) {
    ktmoe_ctx* ctx = L->ctx;
    KLAUNCH(st, (unsigned)T, 256, 0, (mk::quant_rows_kernel), x_dev, (int)T, (int)L->d, (int)L->d_pad, round_up(T, 64),
            L->tok_planes.as<int8_t>(), L->tok_xmax.as<int64_t>(), L->tok_sqx.as<Scale>(), xs_dev, nullptr);
    return KTMOE_OK;
}

// Quantise, route (router GEMM + top-k) for T tokens already in x_in / SL_XSCALE.
int stage_route(ktmoe_layer* L, int64_t T, const int32_t* x_dev, const Scale* xs_dev, cudaStream_t st) {
    ktmoe_ctx* ctx = L->ctx;
    const int64_t d = L->d, E = L->E;
    const int64_t T_pad = round_up(T, 64);
    if (int r = stage_quant(L, T, x_dev, xs_dev, st)) return r;
    GemmCall g;
    g.A = L->w_router;
    g.M_valid = E;
    g.B = Planes{L->tok_planes.as<int8_t>(), 1, T_pad, d, L->d_pad};
    g.out = L->router_acc.as<int64_t>();
    g.ld_out = E;
    g.BN = pick_bn((double)T);
    g.grid_y = (T + g.BN - 1) / g.BN;
    g.single_rows = T;
    int r = run_gemm(ctx, st, g);
    if (r) return r;
    mk::RouteArgs ra;
    ra.acc = L->router_acc.as<int64_t>();
    ra.row_xmax = L->tok_xmax.as<int64_t>();
    ra.row_sqx = L->tok_sqx.as<Scale>();
    ra.rows = (int)T;
    ra.E = (int)E;
    ra.top_k = (int)L->K;
    ra.norm_topk = L->cfg.norm_topk_prob;
    ra.sigmoid = L->cfg.router_score == 1;
    ra.w_scale = L->router_ws;
    ra.bias_codes = L->has_rbias ? L->b_rbias.as<int64_t>() : nullptr;
    ra.bias_scale = L->router_bscale;
    ra.sig_bias = L->cfg.router_score == 1 ? L->b_sigbias.as<int64_t>() : nullptr;
    ra.exp_lut = lut(L, 0);
    ra.sig_lut = lut(L, 2);
    ra.top_e = L->top_e.as<int32_t>();
    ra.top_ec = L->top_ec.as<int64_t>();
    ra.sumc = L->sumc.as<int64_t>();
    ra.logits_out = L->logits.as<int32_t>();
    ra.logit_scale_out = L->logit_scale.as<Scale>();
    KLAUNCH(st, (unsigned)((T + 3) / 4), 128, 0, (mk::route_kernel), ra);
    return KTMOE_OK;
}

// ── collectives of an expert-parallel layer (no-ops on one rank) ──
int nccl_check(ktmoe_ctx* ctx, ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return KTMOE_OK;
    return fail(ctx, KTMOE_ERR_CUDA, std::string(what) + ": " + ncclGetErrorString(r));
}

#define NK(expr)                                                          \
    do {                                                                  \
        if (int r__ = nccl_check(ctx, (expr), #expr)) return r__;         \
    } while (0)

// max over the ranks of n u64 words, in place
// max over the ranks of n u64 words, in place; `point` names the step for the peer transport
int allreduce_max(ktmoe_layer* L, unsigned long long* p, size_t n, cudaStream_t st, int point) {
    if (L->world == 1) return KTMOE_OK;
    ktmoe_ctx* ctx = L->ctx;
    if (L->peer.on) {
        KLAUNCH(st, 1, 32, 0, (ep::exchange_kernel), L->peer.P, point, p, (int)n, nullptr, p, ctx->d_err);
        return KTMOE_OK;
    }
    NK(ncclAllReduce(p, p, n, ncclUint64, ncclMax, L->comm, st));
    return KTMOE_OK;
}

// KTMOE_PLAN_ONE=0: the three-kernel routing plan (count, scan, assign) also for one chunk; the same result. Read per
// call.
bool plan_one_enabled() {
    const char* e = getenv("KTMOE_PLAN_ONE");
    return !(e && e[0] == '0');
}

int plan_chunks(ktmoe_layer* L, int64_t R, int64_t nchunks, const mk::TileTable& ta, const mk::TileTable& tb,
                cudaStream_t st);

// Dispatch plan of the home rank: a stable counting sort of the T·K (token, slot) rows by expert, the tile tables of
// the grouped GEMMs (widths BN and BN2) and the rows' digit planes gathered in that order (xg_planes).
int plan_and_permute(ktmoe_layer* L, int64_t T, int BN, int BN2, cudaStream_t st, bool permute = true) {
    ktmoe_ctx* ctx = L->ctx;
    const int64_t E = L->E, K = L->K, R = T * K;
    const int64_t T_pad = round_up(std::max<int64_t>(T, 1), 64), R_pad = round_up(std::max<int64_t>(R, 1), 64);
    if (R == 0) {
        CK(cudaMemsetAsync(L->expert_count.p, 0, E * 4, st));
        return KTMOE_OK;
    }
    const int64_t nchunks = (R + mk::PLAN_CHUNK - 1) / mk::PLAN_CHUNK;
    const mk::TileTable ta{BN, L->tile_group.as<int>(), L->tile_row0.as<int>(), n_tiles_ptr(L)};
    const mk::TileTable tb{BN2, L->tile_group2.as<int>(), L->tile_row02.as<int>(), n_tiles2_ptr(L)};
    if (nchunks == 1 && E <= mk::PLAN_ONE_MAX_E && plan_one_enabled()) {
        // one chunk (every decode batch): count, scan, tile tables and assignment in one launch
        KLAUNCH(st, 1, mk::PLAN_ONE_THREADS, 0, (mk::plan_one_chunk_kernel), L->top_e.as<int32_t>(), (int)R, (int)E,
                L->chunk_off.as<int>(), L->expert_off.as<int>(), L->group_end.as<int>(), L->expert_count.as<int>(),
                ta, tb, L->slot_row.as<int>(), L->row_assign.as<int>(), L->row_expert.as<int>());
    } else {
        if (int r = plan_chunks(L, R, nchunks, ta, tb, st)) return r;
    }
    if (!permute) return KTMOE_OK;
    KLAUNCH(st, (unsigned)R, 128, 0, (mk::permute_planes_kernel), L->tok_planes.as<int8_t>(), T_pad,
            L->xg_planes.as<int8_t>(), R_pad, (int)L->d_pad, L->row_assign.as<int>(), (int)K, (int)R);
    return KTMOE_OK;
}

// The routing plan over several chunks of PLAN_CHUNK rows: per-chunk counts, the scan, the assignment.
int plan_chunks(ktmoe_layer* L, int64_t R, int64_t nchunks, const mk::TileTable& ta, const mk::TileTable& tb,
                cudaStream_t st) {
    ktmoe_ctx* ctx = L->ctx;
    const int64_t E = L->E;
    KLAUNCH(st, (unsigned)nchunks, mk::PLAN_THREADS, E * 4, (mk::plan_count_kernel), L->top_e.as<int32_t>(), R, (int)E,
            L->counts.as<int>());
    const int scan_threads = (int)std::min<int64_t>(1024, round_up(E, 32));
    KLAUNCH(st, 1, scan_threads, 3 * E * 4, (mk::plan_scan_kernel), L->counts.as<int>(), (int)nchunks, (int)E,
            L->chunk_off.as<int>(), L->expert_off.as<int>(), L->group_end.as<int>(), L->expert_count.as<int>(), ta, tb);
    KLAUNCH(st, (unsigned)nchunks, mk::PLAN_THREADS, (E + (mk::PLAN_THREADS / 32) * E) * 4, (mk::plan_assign_kernel),
            L->top_e.as<int32_t>(), R, (int)E, L->chunk_off.as<int>(), L->expert_off.as<int>(), L->slot_row.as<int>(),
            L->row_assign.as<int>(), L->row_expert.as<int>());
    return KTMOE_OK;
}

// The routed experts over n_rows rows of digit planes `B` (R_pad rows per plane): gate/up GEMM with fused row maxima,
// SwiGLU + requant + the down input planes, down GEMM with fused row maxima (acc_d, rowmax_d, row_cd).
struct ExpertRows {
    Planes B;
    int64_t n_rows;
    int BN, BN2;
    int64_t grid_a, grid_b;  // n-tile bounds of the two tables
    const int *tg_a, *tr_a, *te_a, *nt_a;  // table a: group, row0, row end (or nullptr + group_end), count
    const int *tg_b, *tr_b, *te_b, *nt_b;
    const int* group_end;
    const int* row_assign;  // nullptr: row_sqx is per row
    const int* row_expert;
    const Scale* row_sqx;
    const int* n_rows_dev = nullptr;  // rows counted on the device (n_rows is then an upper bound)
};

// The SwiGLU element pass for wide rows (h beyond one block's shared-memory budget): KTMOE_SWIGLU_SLICE=1 splits a row
// over a cluster of swiglu_slices(L) CTAs with h in shared memory (mk::swiglu_slice_kernel).
bool swiglu_slice_enabled() {
    const char* e = getenv("KTMOE_SWIGLU_SLICE");
    return e && e[0] == '1';
}

// The fewest CTAs (a power of two, at most 8) whose slices of f_pad elements hold h in 60 KB each; 0 if none does.
int swiglu_slices(const ktmoe_layer* L) {
    for (int c = 1; c <= 8; c *= 2)
        if (L->f_pad % (4 * c) == 0 && (L->f_pad / c) * 8 <= 60 * 1024) return c;
    return 0;
}

// Routed rows up to which swiglu_rows_kernel computes each row's plan itself (KTMOE_SWIGLU_INLINE=0: never): one wave
// of its blocks (four per SM). Every wave waits on its rows' plans, so beyond one the plan kernel wins (ms per
// forward, inline against not, measured at three blocks per SM: 256 rows 0.389 against 0.399, 1024 rows 1.233
// against 1.234, 4096 rows 0.620 against 0.600).
int64_t swiglu_inline_rows(const ktmoe_ctx* ctx) {
    const char* e = getenv("KTMOE_SWIGLU_INLINE");
    return (e && e[0] == '0') ? 0 : 4 * (int64_t)ctx->num_sms;
}

int run_experts(ktmoe_layer* L, const ExpertRows& x, cudaStream_t st) {
    ktmoe_ctx* ctx = L->ctx;
    const int64_t d = L->d, f = L->f, R = x.n_rows;
    if (R == 0) {
        MARK(L, st);
        MARK(L, st);
        return KTMOE_OK;
    }
    GemmCall g;
    g.A = L->w_gu;
    g.M_valid = 2 * f;
    g.B = x.B;
    g.out = L->acc_gu.as<int64_t>();
    g.ld_out = 2 * f;
    g.BN = x.BN;
    g.grid_y = x.grid_a;
    g.tile_group = x.tg_a;
    g.tile_row0 = x.tr_a;
    g.tile_row_end = x.te_a;
    g.group_end = x.group_end;
    g.n_tiles = x.nt_a;
    g.rowmax = L->rowmax_gu.as<unsigned long long>();
    g.rowmax_stride = 2;
    g.rowmax_split = f;
    CK(cudaMemsetAsync(L->rowmax_gu.p, 0, R * 2 * 8, st));
    CK(cudaMemsetAsync(L->rowmax_d.p, 0, R * 8, st));
    if (int r = run_gemm(ctx, st, g)) return r;
    MARK(L, st);

    mk::SwigluArgs sa;
    std::memset(&sa, 0, sizeof(sa));
    sa.acc = L->acc_gu.as<int64_t>();
    sa.rows = (int)R;
    sa.f = (int)f;
    sa.f_pad = (int)L->f_pad;
    sa.R_pad = x.B.rows_pad;
    sa.row_assign = x.row_assign;
    sa.row_expert = x.row_expert;
    sa.top_k = (int)L->K;
    sa.row_sqx = x.row_sqx;
    sa.wscale_g = L->b_wsc.as<Scale>();
    sa.wscale_u = L->b_wsc.as<Scale>() + L->E_local;
    sa.wscale_d = L->b_wsc.as<Scale>() + 2 * L->E_local;
    sa.silu = lut(L, 1);
    sa.silu_code_scale = S(L->tabs[1].code_scale);
    sa.silu_code_scale_recip = L->silu_code_scale_recip;
    sa.planes = L->hq_planes.as<int8_t>();
    sa.row_cd = L->row_cd.as<Scale>();
    sa.ymax = L->rowmax_gu.as<unsigned long long>();
    sa.ymax_stride = 2;
    sa.plans = L->swiglu_plans.as<mk::SwigluScales>();
    sa.row_hmax = L->row_hmax.as<unsigned long long>();
    sa.rows_dev = x.n_rows_dev;
    sa.phase = 0;
    // KTMOE_SWIGLU_CLUSTER=1: a cluster per row with h in registers (mk::swiglu_cluster_kernel). The block-per-row
    // kernel below is the default: it spreads a row's per-row work over more elements per thread, and measured faster
    // on the Mixtral rows (2.37 against 2.54 ms); it also takes rows the cluster form cannot (f % 4 != 0, wider than
    // 8 CTAs hold).
    const char* ce = getenv("KTMOE_SWIGLU_CLUSTER");
    const bool use_cluster = ce && ce[0] == '1';
    // groups of four elements per thread x threads per CTA: 4 x 128 (KTMOE_SWIGLU_SHAPE=4x128) or 2 x 256
    const char* se = getenv("KTMOE_SWIGLU_SHAPE");
    const bool wide = !(se && se[0] == '4');
    const int SG = wide ? 2 : 4, SNT = wide ? 256 : 128;
    int csize = 1;
    while (csize < 8 && (int64_t)csize * SG * SNT * 4 < L->f_pad) csize *= 2;
    const bool cluster_path = use_cluster && f % 4 == 0 && (int64_t)csize * SG * SNT * 4 >= L->f_pad;
    const bool slice_path = !cluster_path && swiglu_slice_enabled() && L->swiglu_smem == 0 && swiglu_slices(L) > 0;
    // with few rows the row kernel computes each row's plan and down c itself (two launches fewer); with many the
    // plan kernel runs first, so that no row's loads wait on its plan
    sa.inline_plan = (!cluster_path && !slice_path && R <= swiglu_inline_rows(ctx)) ? 1 : 0;
    if (!sa.inline_plan) {
        KLAUNCH(st, (unsigned)((R + 127) / 128), 128, 0, (mk::swiglu_plan_kernel), sa);
    }
    if (cluster_path) {
        const dim3 grid((unsigned)(R * csize));
        if (wide)
            KLAUNCHC(st, grid, SNT, 0, (unsigned)csize, (mk::swiglu_cluster_kernel<2, 256>), sa);
        else
            KLAUNCHC(st, grid, SNT, 0, (unsigned)csize, (mk::swiglu_cluster_kernel<4, 128>), sa);
    } else if (slice_path) {
        // a wide row (h does not fit one block's budget) split over a cluster, h in shared memory
        const int C = swiglu_slices(L);
        const size_t smem = (size_t)(L->f_pad / C) * 8;
        static bool attr_set[64] = {};
        if (!attr_set[ctx->device & 63]) {
            CK(cudaFuncSetAttribute(mk::swiglu_slice_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)(60 * 1024)));
            attr_set[ctx->device & 63] = true;
        }
        KLAUNCHC(st, (unsigned)(R * C), 256, smem, (unsigned)C, (mk::swiglu_slice_kernel<4>), sa);
    } else {
        const int h_smem = L->swiglu_smem > 0 ? 1 : 0;
        const size_t sm = h_smem ? (size_t)L->swiglu_smem : 0;
        // steps per thread (KTMOE_SWIGLU_U = 1, 2 or 4) of one element (the first lean path) or one pair (v2): v2 at 2
        // measured 1.82-1.86 ms on the Mixtral rows with the fewest instructions (113 M against 120 M at 4 on a
        // 2048-row capture); the first lean path wanted 4 (2.07-2.28 ms)
        const char* ue = getenv("KTMOE_SWIGLU_U");
        const int uv = ue ? atoi(ue) : 2;
        const int unroll = (uv == 1 || uv == 2 || uv == 4) ? uv : 2;
        // a block per row (rows beyond a device-side count leave at once): blocks that wait at a row's barrier
        // are replaced by new ones, which keeps the SMs busier than blocks walking several rows (ncu: 617 vs 696 us)
        const unsigned grid = (unsigned)R;
        // KTMOE_SWIGLU_V=1: the first lean element path; 2 (default): magnitudes and signs apart, a cheaper
        // certificate, element pairs through 16-byte loads and stores
        const char* ve = getenv("KTMOE_SWIGLU_V");
        const int v2 = (ve && ve[0] == '1') ? 0 : 1;
        // KTMOE_SWIGLU_PF=n: thread 0 prefetches the row's accumulators n block steps ahead into L2 (default 2; 0:
        // none): on the Mixtral rows 1-2% faster than none
        const char* pe = getenv("KTMOE_SWIGLU_PF");
        const int pf = pe ? std::max(0, std::min(16, atoi(pe))) : 2;
        // two pairs per thread step compiled for four resident blocks per SM (64 registers, a few spills): the pass
        // is latency bound, and against three blocks of 80 registers it measured 11-17% faster on those rows
        // (Mixtral 1.94 -> 1.73 ms, GLM 2.29 -> 1.91, Qwen 0.262 -> 0.220)
        if (unroll == 1)
            KLAUNCH(st, grid, 256, sm, (mk::swiglu_rows_kernel<1, 3>), sa, h_smem, v2, pf);
        else if (unroll == 4)
            KLAUNCH(st, grid, 256, sm, (mk::swiglu_rows_kernel<4, 3>), sa, h_smem, v2, pf);
        else
            KLAUNCH(st, grid, 256, sm, (mk::swiglu_rows_kernel<2, 4>), sa, h_smem, v2, pf);
    }
    if (!sa.inline_plan) {
        KLAUNCH(st, (unsigned)((R + 127) / 128), 128, 0, (mk::down_c_kernel), sa);
    }
    MARK(L, st);

    g.A = L->w_dn;
    g.M_valid = d;
    g.B = Planes{L->hq_planes.as<int8_t>(), 1, x.B.rows_pad, f, L->f_pad};
    g.out = L->acc_d.as<int64_t>();
    g.ld_out = d;
    g.BN = x.BN2;
    g.grid_y = x.grid_b;
    g.tile_group = x.tg_b;
    g.tile_row0 = x.tr_b;
    g.tile_row_end = x.te_b;
    g.n_tiles = x.nt_b;
    g.rowmax = L->rowmax_d.as<unsigned long long>();
    g.rowmax_stride = 1;
    g.rowmax_split = INT32_MAX;
    if (int r = run_gemm(ctx, st, g)) return r;
    return KTMOE_OK;
}

// KTMOE_COMBINE=0: the thread-per-token plan kernel (combine_plan_kernel / combine_y_plan_kernel) at every size, in
// place of the warp-per-token plans; for comparison only, the results are the same. Read per call.
bool combine_tok_enabled() {
    const char* e = getenv("KTMOE_COMBINE");
    return !(e && e[0] == '0');
}

// Below this many tokens each token's CTAs compute its plan themselves (combine_tok_kernel, one launch); from it on
// a warp-per-token plan kernel runs first and a CTA per token reads it (combine_kernel / combine_y_kernel), so that
// the plan does not hold up the loads of every token's CTA.
constexpr int64_t COMBINE_FUSED_T = 1024;

// The CTAs per token of combine_tok_kernel: the largest power of two up to 8 that keeps the launch to one wave (three
// CTAs per SM, the kernel's launch bound), as every CTA spends the plan's latency before its loads.
int combine_cluster(const ktmoe_ctx* ctx, int64_t T) {
    int C = 1;
    while (C < 8 && T * C * 2 <= 3 * (int64_t)ctx->num_sms) C *= 2;
    return C;
}

// The combine of T > 0 tokens (layers.rs:893-923) into tok_out / tok_scale: Y = false from the down accumulators
// (mk::CombineArgs), Y = true from expert outputs given as IntTensors (mk::CombineYArgs). The plan goes through `cp`
// unless the token's CTAs compute it.
template <bool Y, class A>
int launch_combine(ktmoe_layer* L, const A& a, const mk::CombinePlan& cp, int64_t T, cudaStream_t st) {
    ktmoe_ctx* ctx = L->ctx;
    const int64_t d = L->d;
    const bool tok = combine_tok_enabled();
    if (tok && T < COMBINE_FUSED_T) {
        const int C = combine_cluster(ctx, T);
        const size_t smem = (size_t)((d + C - 1) / C) * 8;
        KLAUNCHC(st, (unsigned)(T * C), 256, smem, (unsigned)C, (mk::combine_tok_kernel<Y, A>), a);
        return KTMOE_OK;
    }
    if (tok) {
        KLAUNCH(st, (unsigned)((T + 7) / 8), 256, 0, (mk::combine_plan_warp_kernel<Y, A>), a, cp);
    } else if constexpr (Y) {
        KLAUNCH(st, (unsigned)((T + 127) / 128), 128, 0, (mk::combine_y_plan_kernel), a, cp);
    } else {
        KLAUNCH(st, (unsigned)((T + 127) / 128), 128, 0, (mk::combine_plan_kernel), a, cp);
    }
    if constexpr (Y) {
        KLAUNCH(st, (unsigned)T, 256, d * 8, (mk::combine_y_kernel), a, cp);
    } else {
        KLAUNCH(st, (unsigned)T, 256, d * 8, (mk::combine_kernel), a, cp);
    }
    return KTMOE_OK;
}

// Expert parallelism: exchange the home rank's expert-sorted rows with the experts' owners, run the local experts on
// what arrives, return their outputs (i32 + Scale per row) and combine at home. Grouped ncclSend/ncclRecv over the
// world; every rank takes the same collective steps.
int ep_routed(ktmoe_layer* L, int64_t T, cudaStream_t st) {
    ktmoe_ctx* ctx = L->ctx;
    const int64_t d = L->d, E = L->E, K = L->K, R = T * K, G = L->world, rk = L->rank;
    const int64_t R_pad = round_up(std::max<int64_t>(R, 1), 64);
    const int BN = pick_bn((double)R * G / (double)E, true), BN2 = pick_bn_long_k((double)R * G / (double)E, L->f, true);
    if (int r = plan_and_permute(L, T, BN, BN2, st)) return r;
    // per-row s_qx for the owners, and this rank's per-expert counts (+ its token count) for everyone
    CK(L->ep_meta_send.ensure(std::max<int64_t>(R, 1) * 16));
    if (R > 0) {
        KLAUNCH(st, (unsigned)((R + 255) / 256), 256, 0, (mk::pack_meta_kernel), L->row_assign.as<int>(), (int)K,
                L->tok_sqx.as<Scale>(), (int)R, L->ep_meta_send.as<int64_t>());
    }
    CK(L->ep_counts.ensure((E + 1) * 4));
    CK(L->ep_counts_all.ensure(G * (E + 1) * 4));
    CK(cudaMemcpyAsync(L->ep_counts.p, L->expert_count.p, E * 4, cudaMemcpyDeviceToDevice, st));
    const int32_t t32 = (int32_t)T;
    CK(cudaMemcpyAsync(L->ep_counts.as<int32_t>() + E, &t32, 4, cudaMemcpyHostToDevice, st));
    NK(ncclAllGather(L->ep_counts.p, L->ep_counts_all.p, E + 1, ncclInt32, L->comm, st));
    L->h_counts.resize(G * (E + 1));
    CK(cudaMemcpyAsync(L->h_counts.data(), L->ep_counts_all.p, G * (E + 1) * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    const std::vector<int>& hc = L->h_counts;
    auto cnt = [&](int64_t src, int64_t e) { return (int64_t)hc[src * (E + 1) + e]; };
    auto begin_of = [&](int64_t q) { return q * E / G; };
    std::vector<int64_t> send_rows(G), send_off(G), recv_rows(G), recv_off(G);
    int64_t so = 0, ro = 0;
    L->ep_tok_offset = 0;
    L->ep_tok_total = 0;
    for (int64_t q = 0; q < G; ++q) {
        int64_t sr = 0, rr = 0;
        for (int64_t e = begin_of(q); e < begin_of(q + 1); ++e) sr += cnt(rk, e);
        for (int64_t e = L->e_begin; e < L->e_end; ++e) rr += cnt(q, e);
        send_rows[q] = sr;
        send_off[q] = so;
        recv_rows[q] = rr;
        recv_off[q] = ro;
        so += sr;
        ro += rr;
        if (q < rk) L->ep_tok_offset += cnt(q, E);
        L->ep_tok_total += cnt(q, E);
    }
    const int64_t Rr = ro, Rr_pad = round_up(std::max<int64_t>(Rr, 1), 64);
    // received rows come in source order, each source's rows sorted by expert: runs (source, local expert) with
    // their tiles for the two GEMM widths
    std::vector<int> runs_start, runs_count, runs_group, ta_g, ta_r, ta_e, tb_g, tb_r, tb_e;
    for (int64_t q = 0; q < G; ++q) {
        int64_t at = recv_off[q];
        for (int64_t e = L->e_begin; e < L->e_end; ++e) {
            const int64_t c = cnt(q, e);
            if (c == 0) continue;
            runs_start.push_back((int)at);
            runs_count.push_back((int)c);
            runs_group.push_back((int)(e - L->e_begin));
            for (int64_t r0 = 0; r0 < c; r0 += BN) {
                ta_g.push_back((int)(e - L->e_begin));
                ta_r.push_back((int)(at + r0));
                ta_e.push_back((int)(at + c));
            }
            for (int64_t r0 = 0; r0 < c; r0 += BN2) {
                tb_g.push_back((int)(e - L->e_begin));
                tb_r.push_back((int)(at + r0));
                tb_e.push_back((int)(at + c));
            }
            at += c;
        }
    }
    const int64_t n_runs = (int64_t)runs_start.size(), na = (int64_t)ta_g.size(), nb = (int64_t)tb_g.size();
    std::vector<int> tiles;  // [na | na | na | nb | nb | nb | na | nb] then runs [3][n_runs]
    tiles.insert(tiles.end(), ta_g.begin(), ta_g.end());
    tiles.insert(tiles.end(), ta_r.begin(), ta_r.end());
    tiles.insert(tiles.end(), ta_e.begin(), ta_e.end());
    tiles.insert(tiles.end(), tb_g.begin(), tb_g.end());
    tiles.insert(tiles.end(), tb_r.begin(), tb_r.end());
    tiles.insert(tiles.end(), tb_e.begin(), tb_e.end());
    tiles.push_back((int)na);
    tiles.push_back((int)nb);
    tiles.insert(tiles.end(), runs_start.begin(), runs_start.end());
    tiles.insert(tiles.end(), runs_count.begin(), runs_count.end());
    tiles.insert(tiles.end(), runs_group.begin(), runs_group.end());
    CK(L->ep_tiles.ensure(tiles.size() * 4));
    CK(cudaMemcpyAsync(L->ep_tiles.p, tiles.data(), tiles.size() * 4, cudaMemcpyHostToDevice, st));
    const int* td = L->ep_tiles.as<int>();

    // the exchange of rows: three digit planes and the s_qx words
    CK(L->ep_recv_planes.ensure(3 * Rr_pad * L->d_pad));
    CK(L->ep_meta_recv.ensure(std::max<int64_t>(Rr, 1) * 16));
    MARK(L, st);
    NK(ncclGroupStart());
    for (int64_t q = 0; q < G; ++q) {
        for (int p = 0; p < 3; ++p) {
            if (send_rows[q])
                NK(ncclSend(L->xg_planes.as<int8_t>() + (p * R_pad + send_off[q]) * L->d_pad, send_rows[q] * L->d_pad,
                            ncclInt8, (int)q, L->comm, st));
            if (recv_rows[q])
                NK(ncclRecv(L->ep_recv_planes.as<int8_t>() + (p * Rr_pad + recv_off[q]) * L->d_pad,
                            recv_rows[q] * L->d_pad, ncclInt8, (int)q, L->comm, st));
        }
        if (send_rows[q])
            NK(ncclSend(L->ep_meta_send.as<int64_t>() + 2 * send_off[q], 2 * send_rows[q], ncclInt64, (int)q, L->comm,
                        st));
        if (recv_rows[q])
            NK(ncclRecv(L->ep_meta_recv.as<int64_t>() + 2 * recv_off[q], 2 * recv_rows[q], ncclInt64, (int)q, L->comm,
                        st));
    }
    NK(ncclGroupEnd());
    MARK(L, st);

    // the owner side: this rank's experts on the rows it received
    if (int r = ensure_rows(L, Rr)) return r;
    CK(L->ep_recv_sqx.ensure(std::max<int64_t>(Rr, 1) * sizeof(Scale)));
    CK(L->ep_recv_row_expert.ensure(std::max<int64_t>(Rr, 1) * 4));
    if (Rr > 0) {
        KLAUNCH(st, (unsigned)((Rr + 255) / 256), 256, 0, (mk::meta_to_scale_kernel), L->ep_meta_recv.as<int64_t>(),
                (int)Rr, L->ep_recv_sqx.as<Scale>());
        const int* runs = td + 3 * na + 3 * nb + 2;
        KLAUNCH(st, (unsigned)n_runs, 128, 0, (mk::runs_to_rows_kernel), runs, runs + n_runs, runs + 2 * n_runs,
                (int)n_runs, L->ep_recv_row_expert.as<int>());
    }
    ExpertRows xr;
    xr.B = Planes{L->ep_recv_planes.as<int8_t>(), 1, Rr_pad, d, L->d_pad};
    xr.n_rows = Rr;
    xr.BN = BN;
    xr.BN2 = BN2;
    xr.grid_a = std::max<int64_t>(na, 1);
    xr.grid_b = std::max<int64_t>(nb, 1);
    xr.tg_a = td;
    xr.tr_a = td + na;
    xr.te_a = td + 2 * na;
    xr.tg_b = td + 3 * na;
    xr.tr_b = td + 3 * na + nb;
    xr.te_b = td + 3 * na + 2 * nb;
    xr.nt_a = td + 3 * na + 3 * nb;
    xr.nt_b = td + 3 * na + 3 * nb + 1;
    xr.group_end = nullptr;
    xr.row_assign = nullptr;
    xr.row_expert = L->ep_recv_row_expert.as<int>();
    xr.row_sqx = L->ep_recv_sqx.as<Scale>();
    if (int r = run_experts(L, xr, st)) return r;
    CK(L->ep_y_send.ensure(std::max<int64_t>(Rr, 1) * d * 4));
    CK(L->ep_ys_send.ensure(std::max<int64_t>(Rr, 1) * sizeof(Scale)));
    if (Rr > 0) {
        KLAUNCH(st, (unsigned)Rr, 256, 0, (mk::expert_out_kernel), L->acc_d.as<int64_t>(),
                L->rowmax_d.as<unsigned long long>(), L->row_cd.as<Scale>(), (int)Rr, (int)d,
                L->ep_y_send.as<int32_t>(), L->ep_ys_send.as<Scale>());
    }
    MARK(L, st);

    // the outputs go home, in the order the rows came
    CK(L->ep_y_back.ensure(std::max<int64_t>(R, 1) * d * 4));
    CK(L->ep_ys_back.ensure(std::max<int64_t>(R, 1) * sizeof(Scale)));
    NK(ncclGroupStart());
    for (int64_t q = 0; q < G; ++q) {
        if (recv_rows[q]) {
            NK(ncclSend(L->ep_y_send.as<int32_t>() + recv_off[q] * d, recv_rows[q] * d, ncclInt32, (int)q, L->comm, st));
            NK(ncclSend(L->ep_ys_send.as<Scale>() + recv_off[q], recv_rows[q] * sizeof(Scale), ncclInt8, (int)q,
                        L->comm, st));
        }
        if (send_rows[q]) {
            NK(ncclRecv(L->ep_y_back.as<int32_t>() + send_off[q] * d, send_rows[q] * d, ncclInt32, (int)q, L->comm, st));
            NK(ncclRecv(L->ep_ys_back.as<Scale>() + send_off[q], send_rows[q] * sizeof(Scale), ncclInt8, (int)q,
                        L->comm, st));
        }
    }
    NK(ncclGroupEnd());
    MARK(L, st);
    if (T > 0) {
        mk::CombineYArgs ca;
        ca.y = L->ep_y_back.as<int32_t>();
        ca.ys = L->ep_ys_back.as<Scale>();
        ca.slot_row = L->slot_row.as<int>();
        ca.top_ec = L->top_ec.as<int64_t>();
        ca.sumc = L->sumc.as<int64_t>();
        ca.T = (int)T;
        ca.top_k = (int)K;
        ca.dim = (int)d;
        ca.out = L->tok_out.as<int32_t>();
        ca.out_scale = L->tok_scale.as<Scale>();
        const mk::CombinePlan cp{L->cp_n.as<int>(), L->cp_common.as<Scale>(), L->cp_row.as<int>(),
                                 L->cp_ec.as<int64_t>(), L->cp_ry.as<kt::ReqDiv>(), L->cp_f.as<kt::ApplyPlan>()};
        if (int r = launch_combine<true>(L, ca, cp, T, st)) return r;
    }
    MARK(L, st);
    return KTMOE_OK;
}

// Expert parallelism over peer memory (ktmoe_layer_set_ep_capacity): the counts go to every rank, each rank writes
// its rows straight into the owners' expert-major buffers, the owners run their experts on what arrived and write the
// outputs straight back into the home ranks' buffers; no host synchronisation and no copies through NCCL.
int ep_routed_peer(ktmoe_layer* L, int64_t T, cudaStream_t st) {
    ktmoe_ctx* ctx = L->ctx;
    auto& pr = L->peer;
    const int64_t d = L->d, E = L->E, K = L->K, R = T * K, G = L->world;
    const int64_t T_pad = round_up(std::max<int64_t>(T, 1), 64);
    // tile widths from the balanced estimate of the rows an owner receives
    const int BN = pick_bn((double)R * G / (double)E, true), BN2 = pick_bn_long_k((double)R * G / (double)E, L->f, true);
    if (R > 0) {
        if (int r = plan_and_permute(L, T, BN, BN2, st, false)) return r;
    } else {
        CK(cudaMemsetAsync(L->expert_count.p, 0, E * 4, st));
        CK(cudaMemsetAsync(L->expert_off.p, 0, E * 4, st));
    }
    KLAUNCH(st, 1, 256, 0, (ep::counts_exchange_kernel), pr.P, L->expert_count.as<int>(), (int)T, ctx->d_err);
    int* tiles = pr.tiles.as<int>();
    const int64_t tmax = pr.cap_rows / 16 + L->E_local + 1;
    const mk::TileTable ta{BN, tiles, tiles + tmax, tiles + 4 * tmax};
    const mk::TileTable tb{BN2, tiles + 2 * tmax, tiles + 3 * tmax, tiles + 4 * tmax + 1};
    int* tok_info = pr.tok_info.as<int>();  // [0] this rank's first token, [1] the layer's tokens
    KLAUNCH(st, 1, 256, 2 * E * 4, (ep::ep_plan_kernel), pr.P, L->expert_off.as<int>(), pr.dst_base.as<int>(),
            pr.group_end.as<int>(), pr.rows_recv.as<int>(), ta, tb, tok_info, tok_info + 1, ctx->d_err);
    KLAUNCH(st, (unsigned)std::max<int64_t>(1, std::min<int64_t>((R + 7) / 8, ctx->num_sms * 8)), 256, 0,
            (ep::dispatch_kernel), pr.P, (int)R, L->row_assign.as<int>(), L->row_expert.as<int>(), (int)K,
            L->tok_planes.as<int8_t>(), T_pad, L->tok_sqx.as<Scale>(), pr.dst_base.as<int>(), pr.ctr.as<int>(),
            ctx->d_err);
    MARK(L, st);
    KLAUNCH(st, 1, 32, 0, (ep::wait_all_kernel), pr.P, ep::P_DISPATCH, ctx->d_err);
    MARK(L, st);

    // the owner side: this rank's experts on the rows that arrived (their count is on the device)
    KLAUNCH(st, (unsigned)std::min<int64_t>((pr.cap_rows + 255) / 256, ctx->num_sms * 4), 256, 0,
            (ep::meta_unpack_kernel), pr.P, pr.rows_recv.as<int>(), pr.recv_sqx.as<Scale>(), pr.recv_expert.as<int>());
    ExpertRows xr;
    xr.B = Planes{(int8_t*)((unsigned char*)pr.region.p + pr.P.off_planes), 1, pr.cap_rows, d, L->d_pad};
    xr.n_rows = pr.cap_rows;
    xr.n_rows_dev = pr.rows_recv.as<int>();
    xr.BN = BN;
    xr.BN2 = BN2;
    xr.grid_a = pr.cap_rows / BN + L->E_local;
    xr.grid_b = pr.cap_rows / BN2 + L->E_local;
    xr.tg_a = ta.tile_group;
    xr.tr_a = ta.tile_row0;
    xr.te_a = nullptr;
    xr.nt_a = ta.n_tiles;
    xr.tg_b = tb.tile_group;
    xr.tr_b = tb.tile_row0;
    xr.te_b = nullptr;
    xr.nt_b = tb.n_tiles;
    xr.group_end = pr.group_end.as<int>();
    xr.row_assign = nullptr;
    xr.row_expert = pr.recv_expert.as<int>();
    xr.row_sqx = pr.recv_sqx.as<Scale>();
    if (int r = run_experts(L, xr, st)) return r;
    MARK(L, st);
    KLAUNCH(st, (unsigned)(ctx->num_sms * 8), 256, 0, (ep::return_kernel), pr.P, pr.rows_recv.as<int>(),
            L->acc_d.as<int64_t>(), L->rowmax_d.as<unsigned long long>(), L->row_cd.as<Scale>(), pr.ctr.as<int>(),
            ctx->d_err);
    KLAUNCH(st, 1, 32, 0, (ep::wait_all_kernel), pr.P, ep::P_RETURN, ctx->d_err);
    MARK(L, st);
    if (T > 0) {
        mk::CombineYArgs ca;
        ca.y = (const int32_t*)((unsigned char*)pr.region.p + pr.P.off_rety);
        ca.ys = (const Scale*)((unsigned char*)pr.region.p + pr.P.off_retys);
        ca.slot_row = L->slot_row.as<int>();
        ca.top_ec = L->top_ec.as<int64_t>();
        ca.sumc = L->sumc.as<int64_t>();
        ca.T = (int)T;
        ca.top_k = (int)K;
        ca.dim = (int)d;
        ca.out = L->tok_out.as<int32_t>();
        ca.out_scale = L->tok_scale.as<Scale>();
        const mk::CombinePlan cp{L->cp_n.as<int>(), L->cp_common.as<Scale>(), L->cp_row.as<int>(),
                                 L->cp_ec.as<int64_t>(), L->cp_ry.as<kt::ReqDiv>(), L->cp_f.as<kt::ApplyPlan>()};
        if (int r = launch_combine<true>(L, ca, cp, T, st)) return r;
    }
    MARK(L, st);
    return KTMOE_OK;
}

// The shared expert on the whole tensor (layers.rs:758-780; its QuantLinears see the whole [rows, dim] input, so its
// maxima are global): everything up to the down accumulators and their max, on stream `st`.
// The token tile of one of the shared expert's GEMMs (one matrix of M weight rows over all T tokens). Routing the
// decode-sized ones to the one-SM kernel with split K when the pair's tiles fill few SMs measured no faster (Qwen
// decode: shared stage 0.170 against 0.159 ms; the split adds a memset, atomics and a row-max pass), so the pair
// keeps every launch of 64 tokens and more.
int shared_bn(const ktmoe_ctx* ctx, int64_t M, int64_t T) {
    (void)ctx;
    (void)M;
    return pick_bn((double)T, true);
}

int shared_expert(ktmoe_layer* L, int64_t T, const int32_t* x_dev, const Scale* xs_dev, cudaStream_t st) {
    ktmoe_ctx* ctx = L->ctx;
    const int64_t d = L->d, fs = L->fs;
    const int64_t T_pad = round_up(std::max<int64_t>(T, 1), 64);
    const int64_t n = T * d;
    const unsigned red_blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>(1184, (n + 255) / 256));
    if (T > 0) {
        KLAUNCH(st, red_blocks, 256, 0, (mk::absmax_i32_kernel), x_dev, n, scal_u64(L, U_GXMAX));
    }
    if (int r = allreduce_max(L, scal_u64(L, U_GXMAX), 1, st, ep::P_SX)) return r;
    KLAUNCH(st, 1, 1, 0, (sqx_kernel), scal_u64(L, U_GXMAX), xs_dev, scal_scale(L, SL_GSQX));
    GemmCall s;
    if (T > 0) {
        KLAUNCH(st, (unsigned)T, 256, 0, (mk::quant_rows_kernel), x_dev, (int)T, (int)d, (int)L->d_pad, T_pad,
                L->xs_planes.as<int8_t>(), nullptr, nullptr, xs_dev, scal_u64(L, U_GXMAX));
        s.A = L->w_sgu;
        s.M_valid = 2 * fs;
        s.B = Planes{L->xs_planes.as<int8_t>(), 1, T_pad, d, L->d_pad};
        s.out = L->acc_sgu.as<int64_t>();
        s.ld_out = 2 * fs;
        s.BN = shared_bn(ctx, 2 * fs, T);
        s.grid_y = (T + s.BN - 1) / s.BN;
        s.single_rows = T;
        s.rowmax = scal_u64(L, U_SYG);  // [U_SYG] gate, [U_SYU] up: maxima over the whole tensor
        s.rowmax_stride = 0;
        s.rowmax_split = fs;
        if (int r = run_gemm(ctx, st, s)) return r;
    }
    if (int r = allreduce_max(L, scal_u64(L, U_SYG), 2, st, ep::P_SYG)) return r;
    mk::SwigluArgs sh;
    std::memset(&sh, 0, sizeof(sh));
    sh.acc = L->acc_sgu.as<int64_t>();
    sh.rows = (int)T;
    sh.f = (int)fs;
    sh.f_pad = (int)L->fs_pad;
    sh.R_pad = T_pad;
    sh.top_k = 1;
    sh.g_sqx = scal_scale(L, SL_GSQX);
    sh.wscale_g = L->b_wsc.as<Scale>() + 3 * L->E_local;
    sh.wscale_u = L->b_wsc.as<Scale>() + 3 * L->E_local + 1;
    sh.wscale_d = L->b_wsc.as<Scale>() + 3 * L->E_local + 2;
    sh.silu = lut(L, 1);
    sh.silu_code_scale = S(L->tabs[1].code_scale);
    sh.silu_code_scale_recip = L->silu_code_scale_recip;
    sh.planes = L->hs_planes.as<int8_t>();
    sh.row_cd = scal_scale(L, SL_SCD);
    sh.ymax = scal_u64(L, U_SYG);
    sh.ymax_stride = 0;
    sh.g_hmax = scal_u64(L, U_SHMAX);
    CK(L->shared_plan.ensure(sizeof(mk::SwigluScales)));
    sh.plans = L->shared_plan.as<mk::SwigluScales>();
    sh.phase = 1;
    KLAUNCH(st, 1, 32, 0, (mk::swiglu_plan_kernel), sh);
    if (T > 0) {
        KLAUNCH(st, (unsigned)T, 256, 0, (mk::swiglu_global_kernel), sh);
    }
    if (int r = allreduce_max(L, scal_u64(L, U_SHMAX), 1, st, ep::P_SHMAX)) return r;
    sh.phase = 2;
    if (T > 0) {
        KLAUNCH(st, (unsigned)T, 256, 0, (mk::swiglu_global_kernel), sh);
        s.A = L->w_sdn;
        s.M_valid = d;
        s.B = Planes{L->hs_planes.as<int8_t>(), 1, T_pad, fs, L->fs_pad};
        s.BN = shared_bn(ctx, d, T);
        s.grid_y = (T + s.BN - 1) / s.BN;
        s.out = L->acc_sd.as<int64_t>();
        s.ld_out = d;
        s.rowmax = scal_u64(L, U_SYD);
        s.rowmax_stride = 0;
        s.rowmax_split = INT32_MAX;
        if (int r = run_gemm(ctx, st, s)) return r;
    }
    if (int r = allreduce_max(L, scal_u64(L, U_SYD), 1, st, ep::P_SYD)) return r;
    if (!L->sgate_set) return KTMOE_OK;

    // the sigmoid gate of the shared expert (extension): gate logits from the same input planes, their sigmoid
    // codes, then the shared output scaled per token and requantised over the whole tensor (all ranks)
    if (T > 0) {
        KLAUNCH(st, (unsigned)((T + 7) / 8), 256, 0, (mk::gate_logit_kernel), L->xs_planes.as<int8_t>(), (int)T,
                (int)L->d_pad, T_pad, L->b_sgate.as<int32_t>(), L->sg_acc.as<int64_t>(), scal_u64(L, U_GYMAX));
    }
    if (int r = allreduce_max(L, scal_u64(L, U_GYMAX), 1, st, ep::P_GYMAX)) return r;
    mk::GateArgs ga;
    ga.s_acc = L->acc_sd.as<int64_t>();
    ga.s_ymax = scal_u64(L, U_SYD);
    ga.s_cd = scal_scale(L, SL_SCD);
    ga.code = L->sg_code.as<int64_t>();
    ga.T = (int)T;
    ga.d = (int)d;
    ga.gmax = scal_u64(L, U_GATEDMAX);
    ga.code_scale = S(L->tabs[2].code_scale);
    ga.y = L->y_gated.as<int32_t>();
    ga.y_scale = scal_scale(L, SL_GATED);
    if (T > 0) {
        KLAUNCH(st, (unsigned)((T + 127) / 128), 128, 0, (mk::gate_code_kernel), L->sg_acc.as<int64_t>(), (int)T,
                scal_u64(L, U_GYMAX), scal_scale(L, SL_GSQX), L->sgate_ws, lut(L, 2), L->sg_code.as<int64_t>());
        KLAUNCH(st, (unsigned)T, 256, 0, (mk::gated_max_kernel), ga);
    }
    if (int r = allreduce_max(L, scal_u64(L, U_GATEDMAX), 1, st, ep::P_GATED)) return r;
    if (T > 0) {
        KLAUNCH(st, (unsigned)T, 256, 0, (mk::gated_final_kernel), ga);
    }
    return KTMOE_OK;
}

int merge_and_add(ktmoe_layer* L, int64_t T, int64_t T_total, int64_t tok_offset, const int32_t* x_dev,
                  const Scale* xs_dev, int32_t* y_dev, Scale* ys_dev, cudaStream_t st, bool side_shared);

int stage_forward(ktmoe_layer* L, int64_t T, const int32_t* x_dev, const Scale* xs_dev, int32_t* y_dev, Scale* ys_dev,
                  cudaStream_t st, bool bump = true) {
    ktmoe_ctx* ctx = L->ctx;
    const int64_t d = L->d, E = L->E, f = L->f, K = L->K, fs = L->fs;
    const int64_t R = T * K;
    const int64_t T_pad = round_up(std::max<int64_t>(T, 1), 64), R_pad = round_up(std::max<int64_t>(R, 1), 64);
    CK(cudaMemsetAsync(scal_u64(L, 0), 0, U_N * 8, st));
    if (L->peer.on && bump) {
        KLAUNCH(st, 1, 1, 0, (ep::seq_bump_kernel), L->peer.P);  // a new forward for every exchange below
        CKL(ctx);
    }
    // the shared expert depends only on x: it runs on the side stream while the routed experts run on st (not with
    // per-stage timing, and not with the NCCL exchange, whose collectives must keep one order on every rank)
    const bool side_shared = fs > 0 && !L->timing && (L->world == 1 || L->peer.on);
    if (side_shared) {
        CK(cudaEventRecord(ctx->ev_fork, st));
        CK(cudaStreamWaitEvent(ctx->side, ctx->ev_fork, 0));
        if (int r = shared_expert(L, T, x_dev, xs_dev, ctx->side)) return r;
        CK(cudaEventRecord(ctx->ev_join, ctx->side));
    }
    MARK(L, st);
    if (T > 0) {
        if (int r = stage_route(L, T, x_dev, xs_dev, st)) return r;
    }
    MARK(L, st);

    int64_t T_total = T, tok_offset = 0;
    if (L->world == 1) {
        const int BN = pick_bn((double)R / (double)E, true);
        const int BN2 = pick_bn_long_k((double)R / (double)E, f, true);
        if (int r = plan_and_permute(L, T, BN, BN2, st)) return r;
        MARK(L, st);
        MARK(L, st);  // no exchange on one GPU
        ExpertRows xr;
        xr.B = Planes{L->xg_planes.as<int8_t>(), 1, R_pad, d, L->d_pad};
        xr.n_rows = R;
        xr.BN = BN;
        xr.BN2 = BN2;
        xr.grid_a = (R + BN - 1) / BN + E;
        xr.grid_b = (R + BN2 - 1) / BN2 + E;
        xr.tg_a = L->tile_group.as<int>();
        xr.tr_a = L->tile_row0.as<int>();
        xr.te_a = nullptr;
        xr.nt_a = n_tiles_ptr(L);
        xr.tg_b = L->tile_group2.as<int>();
        xr.tr_b = L->tile_row02.as<int>();
        xr.te_b = nullptr;
        xr.nt_b = n_tiles2_ptr(L);
        xr.group_end = L->group_end.as<int>();
        xr.row_assign = L->row_assign.as<int>();
        xr.row_expert = L->row_expert.as<int>();
        xr.row_sqx = L->tok_sqx.as<Scale>();
        if (int r = run_experts(L, xr, st)) return r;
        MARK(L, st);
        MARK(L, st);  // no exchange on one GPU
        mk::CombineArgs ca;
        ca.acc_d = L->acc_d.as<int64_t>();
        ca.ymax_d = L->rowmax_d.as<unsigned long long>();
        ca.row_cd = L->row_cd.as<Scale>();
        ca.slot_row = L->slot_row.as<int>();
        ca.top_ec = L->top_ec.as<int64_t>();
        ca.sumc = L->sumc.as<int64_t>();
        ca.T = (int)T;
        ca.top_k = (int)K;
        ca.dim = (int)d;
        ca.out = L->tok_out.as<int32_t>();
        ca.out_scale = L->tok_scale.as<Scale>();
        const mk::CombinePlan cp{L->cp_n.as<int>(), L->cp_common.as<Scale>(), L->cp_row.as<int>(),
                                 L->cp_ec.as<int64_t>(), L->cp_ry.as<kt::ReqDiv>(), L->cp_f.as<kt::ApplyPlan>()};
        if (int r = launch_combine<false>(L, ca, cp, T, st)) return r;
        MARK(L, st);
    } else if (L->peer.on) {
        if (int r = ep_routed_peer(L, T, st)) return r;
        T_total = -1;  // on the device (peer.tok_info): the merge kernels read it there
    } else {
        if (int r = ep_routed(L, T, st)) return r;
        T_total = L->ep_tok_total;
        tok_offset = L->ep_tok_offset;
    }
    return merge_and_add(L, T, T_total, tok_offset, x_dev, xs_dev, y_dev, ys_dev, st, side_shared);
}

// The end of the forward, after each token's combine (tok_out, tok_scale): merge the rows at one scale over all the
// layer's tokens (T_total of them, this rank's from tok_offset; -1: counted on the device by the peer transport),
// then add the shared expert (run here unless side_shared, when it ran on the side stream).
int merge_and_add(ktmoe_layer* L, int64_t T, int64_t T_total, int64_t tok_offset, const int32_t* x_dev,
                  const Scale* xs_dev, int32_t* y_dev, Scale* ys_dev, cudaStream_t st, bool side_shared) {
    ktmoe_ctx* ctx = L->ctx;
    const int64_t d = L->d, fs = L->fs;
    const int* tok_info = L->peer.on ? L->peer.tok_info.as<int>() : nullptr;  // [0] first token, [1] tokens

    // merge (layers.rs:1001-1019): one common scale and one gmax over all the layer's tokens, on every rank
    int32_t* routed = fs > 0 ? L->y_routed.as<int32_t>() : y_dev;
    Scale* routed_scale = fs > 0 ? scal_scale(L, SL_YROUTED) : ys_dev;
    if (T_total == 1) {
        if (T == 1) {
            KLAUNCH(st, (unsigned)((d + 255) / 256), 256, 0, (mk::copy_row_kernel), L->tok_out.as<int32_t>(),
                    L->tok_scale.as<Scale>(), (int)d, routed, routed_scale);
        }
    } else {
        if (L->world == 1) {
            KLAUNCH(st, 1, 1024, 0, (mk::common_scale_kernel), L->tok_scale.as<Scale>(), (int)T, 0,
                    scal_scale(L, SL_COMMON), nullptr, nullptr);
        } else {
            CK(L->ep_rec.ensure(3 * 8));
            CK(L->ep_recs.ensure(L->world * 3 * 8));
            CK(L->ep_best_idx.ensure(4));
            if (T > 0) {
                KLAUNCH(st, 1, 1024, 0, (mk::common_scale_kernel), L->tok_scale.as<Scale>(), (int)T, (int)tok_offset,
                        scal_scale(L, SL_COMMON), L->ep_best_idx.as<int>(), tok_info);
                KLAUNCH(st, 1, 1, 0, (mk::scale_record_kernel), scal_scale(L, SL_COMMON), L->ep_best_idx.as<int>(),
                        L->ep_rec.as<int64_t>());
            } else {
                KLAUNCH(st, 1, 1, 0, (mk::empty_record_kernel), L->ep_rec.as<int64_t>());
            }
            if (L->peer.on) {
                KLAUNCH(st, 1, 32, 0, (ep::exchange_kernel), L->peer.P, ep::P_REC, L->ep_rec.as<unsigned long long>(),
                        3, L->ep_recs.as<unsigned long long>(), nullptr, ctx->d_err);
            } else {
                NK(ncclAllGather(L->ep_rec.p, L->ep_recs.p, 3, ncclInt64, L->comm, st));
            }
            KLAUNCH(st, 1, 1, 0, (mk::reduce_records_kernel), L->ep_recs.as<int64_t>(), L->world,
                    scal_scale(L, SL_COMMON));
        }
        if (T > 0) {
            KLAUNCH(st, (unsigned)T, 256, 0, (mk::merge_max_kernel), L->tok_out.as<int32_t>(), L->tok_scale.as<Scale>(),
                    (int)T, (int)d, scal_scale(L, SL_COMMON), scal_u64(L, U_MERGE_GMAX));
        }
        if (int r = allreduce_max(L, scal_u64(L, U_MERGE_GMAX), 1, st, ep::P_MERGE)) return r;
        if (T > 0) {
            KLAUNCH(st, (unsigned)T, 256, 0, (mk::merge_final_kernel), L->tok_out.as<int32_t>(),
                    L->tok_scale.as<Scale>(), (int)T, (int)d, scal_scale(L, SL_COMMON), scal_u64(L, U_MERGE_GMAX),
                    routed, routed_scale, tok_info ? tok_info + 1 : nullptr);
        }
    }
    MARK(L, st);
    if (fs == 0) return KTMOE_OK;

    // add(routed, shared) (layers.rs:121-136), after the shared expert (run here, or beside the routed experts)
    if (side_shared) {
        CK(cudaStreamWaitEvent(st, ctx->ev_join, 0));
    } else if (int r = shared_expert(L, T, x_dev, xs_dev, st)) {
        return r;
    }
    const int64_t n = T * d;
    const unsigned red_blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>(1184, (n + 255) / 256));
    if (L->sgate_set) {  // add(routed, gated shared output) of two int32 tensors
        Scale* plan = scal_scale(L, SL_ADD2);
        if (T > 0) {
            KLAUNCH(st, 1, 1, 0, (mk::add2_prepare_kernel), routed_scale, scal_scale(L, SL_GATED), plan);
            KLAUNCH(st, red_blocks, 256, 0, (mk::add2_max_kernel), routed, L->y_gated.as<int32_t>(), n, plan,
                    scal_u64(L, U_ADDGMAX));
        }
        if (int r = allreduce_max(L, scal_u64(L, U_ADDGMAX), 1, st, ep::P_ADD)) return r;
        if (T > 0) {
            KLAUNCH(st, red_blocks, 256, 0, (mk::add2_final_kernel), routed, L->y_gated.as<int32_t>(), n, plan,
                    scal_u64(L, U_ADDGMAX), y_dev);
            KLAUNCH(st, 1, 1, 0, (mk::gmax_scale_kernel), plan, scal_u64(L, U_ADDGMAX), ys_dev);
        }
        MARK(L, st);
        return KTMOE_OK;
    }
    // a rank without tokens still needs the shared down c for nothing: only ranks with rows produce output
    mk::AddArgs aa;
    aa.a = routed;
    aa.a_scale = routed_scale;
    aa.s_acc = L->acc_sd.as<int64_t>();
    aa.s_ymax = scal_u64(L, U_SYD);
    aa.s_cd = scal_scale(L, SL_SCD);
    aa.n = n;
    aa.gmax = scal_u64(L, U_ADDGMAX);
    aa.scratch = scal_scale(L, SL_ADD);
    aa.y = y_dev;
    aa.y_scale = ys_dev;
    if (T > 0) {
        KLAUNCH(st, 1, 1, 0, (mk::add_prepare_kernel), aa);
        KLAUNCH(st, red_blocks, 256, 0, (mk::add_max_kernel), aa);
    }
    if (int r = allreduce_max(L, scal_u64(L, U_ADDGMAX), 1, st, ep::P_ADD)) return r;
    if (T > 0) {
        KLAUNCH(st, red_blocks, 256, 0, (mk::add_final_kernel), aa);
    }
    MARK(L, st);
    return KTMOE_OK;
}

__global__ void set_u64_kernel(unsigned long long* p, unsigned long long v) { kt::pdl_enter(); *p = v; }

int ensure_block(ktmoe_layer* L, int64_t T) {
    ktmoe_ctx* ctx = L->ctx;
    CK(L->blk_sc.ensure(8 * sizeof(Scale)));
    CK(L->blk_u64.ensure((3 + ep::MAXW) * 8));
    CK(L->blk_off.ensure(4));
    CK(L->ep_rec.ensure(3 * 8));
    CK(L->ep_recs.ensure(L->world * 3 * 8));
    CK(L->ep_best_idx.ensure(4));
    if (T <= L->blk_cap && L->blk_cap > 0) return KTMOE_OK;
    graphs_clear(L);
    const int64_t n = std::max<int64_t>(T, 1);
    CK(L->blk_c.ensure(n * sizeof(Scale)));
    CK(L->blk_xn.ensure(n * L->d * 4));
    CK(L->blk_m.ensure(n * L->d * 4));
    L->blk_cap = n;
    return KTMOE_OK;
}

// The FFN half of a decoder block with this layer as its FFN (kt-core model.rs:175-181): y = add(x, moe(norm(x))),
// norm the RmsNorm of ktmoe_layer_set_norm (layers.rs:352-449), add the residual add (layers.rs:121-136). Every
// reduction over the tensor (the norm's common scale and max, the add's max) spans all ranks.
int stage_block(ktmoe_layer* L, int64_t T, const int32_t* x_dev, const Scale* xs_dev, int32_t* y_dev, Scale* ys_dev,
                cudaStream_t st) {
    ktmoe_ctx* ctx = L->ctx;
    const int64_t d = L->d;
    Scale* sc = L->blk_sc.as<Scale>();  // [0..1] the norm's common and its reciprocal, [2] x_norm, [3] moe, [4..6] add
    unsigned long long* u = L->blk_u64.as<unsigned long long>();  // [0] norm gmax, [1] add gmax, [2] T, [3..] counts
    Scale* c = L->blk_c.as<Scale>();
    int32_t* xn = L->blk_xn.as<int32_t>();
    int32_t* m = L->blk_m.as<int32_t>();
    CK(cudaMemsetAsync(u, 0, 2 * 8, st));
    if (L->peer.on) {
        KLAUNCH(st, 1, 1, 0, (ep::seq_bump_kernel), L->peer.P);
    }
    const int* off = nullptr;
    if (L->world > 1) {
        // every rank's row count, for this rank's first global row (the tie rule of the common scale)
        KLAUNCH(st, 1, 1, 0, (set_u64_kernel), u + 2, (unsigned long long)T);
        if (L->peer.on) {
            KLAUNCH(st, 1, 32, 0, (ep::exchange_kernel), L->peer.P, ep::P_TOK, u + 2, 1, u + 3, nullptr, ctx->d_err);
        } else {
            NK(ncclAllGather(u + 2, u + 3, 1, ncclUint64, L->comm, st));
        }
        KLAUNCH(st, 1, 1, 0, (mk::row_offset_kernel), u + 3, L->rank, L->blk_off.as<int>());
        off = L->blk_off.as<int>();
    }
    if (T > 0) {
        KLAUNCH(st, (unsigned)T, 256, 0, (mk::rms_rows_kernel), x_dev, (int)T, (int)d, xs_dev, L->norm_ws, L->norm_eps,
                c);
    }
    if (L->world == 1) {
        KLAUNCH(st, 1, 1024, 0, (mk::common_scale_kernel), c, (int)T, 0, sc, nullptr, nullptr);
    } else {
        if (T > 0) {
            KLAUNCH(st, 1, 1024, 0, (mk::common_scale_kernel), c, (int)T, 0, sc, L->ep_best_idx.as<int>(), off);
            KLAUNCH(st, 1, 1, 0, (mk::scale_record_kernel), sc, L->ep_best_idx.as<int>(), L->ep_rec.as<int64_t>());
        } else {
            KLAUNCH(st, 1, 1, 0, (mk::empty_record_kernel), L->ep_rec.as<int64_t>());
        }
        if (L->peer.on) {
            KLAUNCH(st, 1, 32, 0, (ep::exchange_kernel), L->peer.P, ep::P_NREC, L->ep_rec.as<unsigned long long>(), 3,
                    L->ep_recs.as<unsigned long long>(), nullptr, ctx->d_err);
        } else {
            NK(ncclAllGather(L->ep_rec.p, L->ep_recs.p, 3, ncclInt64, L->comm, st));
        }
        KLAUNCH(st, 1, 1, 0, (mk::reduce_records_kernel), L->ep_recs.as<int64_t>(), L->world, sc);
    }
    if (T > 0) {
        KLAUNCH(st, (unsigned)T, 256, 0, (mk::rms_max_kernel), x_dev, L->b_norm.as<int32_t>(), (int)T, (int)d, c, sc,
                u);
    }
    if (int r = allreduce_max(L, u, 1, st, ep::P_NMAX)) return r;
    if (T > 0) {
        KLAUNCH(st, (unsigned)T, 256, 0, (mk::rms_final_kernel), x_dev, L->b_norm.as<int32_t>(), (int)T, (int)d, c, sc,
                u, xn);
    }
    KLAUNCH(st, 1, 1, 0, (mk::gmax_scale_kernel), sc, u, sc + 2);
    if (int r = stage_forward(L, T, xn, sc + 2, m, sc + 3, st, false)) return r;
    const int64_t n = T * d;
    const unsigned rb = (unsigned)std::max<int64_t>(1, std::min<int64_t>(1184, (n + 255) / 256));
    KLAUNCH(st, 1, 1, 0, (mk::add2_prepare_kernel), xs_dev, sc + 3, sc + 4);
    if (T > 0) {
        KLAUNCH(st, rb, 256, 0, (mk::add2_max_kernel), x_dev, m, n, sc + 4, u + 1);
    }
    if (int r = allreduce_max(L, u + 1, 1, st, ep::P_RADD)) return r;
    if (T > 0) {
        KLAUNCH(st, rb, 256, 0, (mk::add2_final_kernel), x_dev, m, n, sc + 4, u + 1, y_dev);
    }
    KLAUNCH(st, 1, 1, 0, (mk::gmax_scale_kernel), sc + 4, u + 1, ys_dev);
    return KTMOE_OK;
}

// The forward through a CUDA graph when graphs are on and the forward has no host synchronisation (one rank, or the
// peer transport): the first call with a key runs the forward, then captures the same launch sequence; later calls
// with that key launch the graph. Timing (per-stage events) and the NCCL exchange always run uncaptured.
int run_forward(ktmoe_layer* L, int64_t T, const int32_t* x, const Scale* xs, int32_t* y, Scale* ys, cudaStream_t st,
                bool block = false) {
    ktmoe_ctx* ctx = L->ctx;
    auto once = [&]() { return block ? stage_block(L, T, x, xs, y, ys, st) : stage_forward(L, T, x, xs, y, ys, st); };
    if (!L->graphs || L->timing || (L->world > 1 && !L->peer.on)) return once();
    for (auto& g : L->graph_cache)
        if (g.x == x && g.xs == xs && g.y == y && g.ys == ys && g.T == T && g.st == st && g.block == block &&
            g.slot == L->active) {
            CK(cudaGraphLaunch(g.exec, st));
            ctx->launches += g.launches;
            return KTMOE_OK;
        }
    if (int r = once()) return r;
    const uint64_t l0 = ctx->launches;
    cudaGraph_t graph = nullptr;
    CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    const int r = once();
    const cudaError_t e = cudaStreamEndCapture(st, &graph);
    ctx->launches = l0;  // nothing ran during the capture
    if (r != KTMOE_OK || e != cudaSuccess || !graph) {
        if (graph) cudaGraphDestroy(graph);
        cudaGetLastError();
        L->graphs = false;  // this forward cannot be captured here: stay uncaptured (its result is already computed)
        return KTMOE_OK;
    }
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    uint64_t n = 0;
    size_t nodes = 0;
    if (cudaGraphGetNodes(graph, nullptr, &nodes) == cudaSuccess) {
        std::vector<cudaGraphNode_t> v(nodes);
        if (nodes && cudaGraphGetNodes(graph, v.data(), &nodes) == cudaSuccess)
            for (auto nd : v) {
                cudaGraphNodeType t;
                if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++n;
            }
    }
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) {
        cudaGetLastError();
        L->graphs = false;
        return KTMOE_OK;
    }
    if (L->graph_cache.size() >= std::max<size_t>(16, 2 * L->slots.size() + 4)) {
        cudaStreamSynchronize(L->graph_cache.front().st);  // no launch of the evicted graph is still in flight
        cudaGraphExecDestroy(L->graph_cache.front().exec);
        L->graph_cache.erase(L->graph_cache.begin());
    }
    L->graph_cache.push_back({x, xs, y, ys, T, st, exec, n, block, L->active});
    return KTMOE_OK;
}

// Upload codes [groups? one matrix] rows x k (int32, row-major) into planes at (group g) of P, packed on the device.
int upload_matrix(ktmoe_ctx* ctx, const Planes& P, int64_t g, const int32_t* codes, int64_t rows, int64_t k,
                  int64_t row0) {
    DevBuf tmp;
    CK(tmp.ensure((size_t)rows * k * 4));
    DevBuf bad;
    CK(bad.ensure(8));
    CK(cudaMemsetAsync(bad.p, 0, 8, ctx->stream));
    CK(cudaMemcpyAsync(tmp.p, codes, (size_t)rows * k * 4, cudaMemcpyHostToDevice, ctx->stream));
    int8_t* base = P.ptr + (g * 3) * P.rows_pad * P.k_pad + row0 * P.k_pad;
    KLAUNCH(ctx->stream, (unsigned)rows, 128, 0, (mk::pack_codes_kernel), tmp.as<int32_t>(), rows, (int)k, (int)P.k_pad,
            P.rows_pad, base, bad.as<unsigned long long>(), nullptr, 0, nullptr);
    unsigned long long hbad = 0;
    CK(cudaMemcpyAsync(&hbad, bad.p, 8, cudaMemcpyDeviceToHost, ctx->stream));
    CK(cudaStreamSynchronize(ctx->stream));
    tmp.release();
    bad.release();
    if (hbad) return fail(ctx, KTMOE_ERR_RANGE, "a weight code lies outside +-WLEVELS");
    return KTMOE_OK;
}

int alloc_planes(ktmoe_ctx* ctx, DevBuf& buf, Planes& P, int64_t groups, int64_t rows_valid, int64_t k) {
    P.groups = groups;
    P.rows_pad = rows_valid > dg::BM ? round_up(rows_valid, dg::pair::BM2) : dg::BM;  // 256-row pair tiles
    P.k = k;
    P.k_pad = round_up(k, dg::BK);
    CK(buf.ensure((size_t)(groups * 3 * P.rows_pad * P.k_pad)));
    CK(cudaMemset(buf.p, 0, buf.bytes));
    P.ptr = buf.as<int8_t>();
    return KTMOE_OK;
}

}  // namespace

extern "C" {

const char* ktmoe_error_string(int status) {
    switch (status) {
        case KTMOE_OK: return "ok";
        case KTMOE_ERR_CUDA: return "CUDA error";
        case KTMOE_ERR_ARG: return "invalid argument";
        case KTMOE_ERR_RANGE: return "code outside +-WLEVELS";
        case KTMOE_ERR_KERNEL: return "kernel bounded wait expired";
        case KTMOE_ERR_UNSUPPORTED: return "unsupported configuration";
        case KTMOE_ERR_NO_DEVICE: return "no sm_100 device";
        case KTMOE_ERR_STATE: return "layer incomplete";
        case KTMOE_ERR_CALLBACK: return "the experts callback failed";
        default: return "unknown status";
    }
}

int ktmoe_device_count(int* n) {
    if (!n) return KTMOE_ERR_ARG;
    *n = 0;
    cudaError_t e = cudaGetDeviceCount(n);
    if (e != cudaSuccess) {
        *n = 0;
        return e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver ? KTMOE_OK : KTMOE_ERR_CUDA;
    }
    return KTMOE_OK;
}

int ktmoe_open(int device, ktmoe_ctx** out) {
    if (!out) return KTMOE_ERR_ARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return KTMOE_ERR_NO_DEVICE;
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, device) != cudaSuccess) return KTMOE_ERR_NO_DEVICE;
    if (p.major != 10) return KTMOE_ERR_NO_DEVICE;  // the kernels are built for sm_100a only
    ktmoe_ctx* ctx = new ktmoe_ctx();
    ctx->device = device;
    if (cudaSetDevice(device) != cudaSuccess || cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&ctx->d_err, sizeof(int)) != cudaSuccess || cudaMemset(ctx->d_err, 0, sizeof(int)) != cudaSuccess) {
        delete ctx;
        return KTMOE_ERR_CUDA;
    }
    if (cudaStreamCreateWithFlags(&ctx->side, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->ev_fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->ev_join, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreate(&ctx->ev_g0) != cudaSuccess || cudaEventCreate(&ctx->ev_g1) != cudaSuccess ||
        cudaHostAlloc((void**)&ctx->h_status, 4 * sizeof(unsigned long long), cudaHostAllocDefault) != cudaSuccess) {
        delete ctx;
        return KTMOE_ERR_CUDA;
    }
    cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device);
    size_t free_b = 0, total_b = 0;
    cudaMemGetInfo(&free_b, &total_b);
    ctx->budget = free_b / 5 * 4;
    *out = ctx;
    return KTMOE_OK;
}

int ktmoe_close(ktmoe_ctx* ctx) {
    if (!ctx) return KTMOE_ERR_ARG;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    for (auto& kv : ctx->cache) {
        kv.second->buf.release();
        delete kv.second;
    }
    ctx->lin_xi.release();
    ctx->lin_wi.release();
    ctx->lin_xp.release();
    ctx->lin_xr.release();
    ctx->lin_wp.release();
    ctx->lin_y.release();
    ctx->lin_bad.release();
    ctx->lin_hx.release();
    ctx->lin_hy.release();
    cudaFree(ctx->d_err);
    cudaStreamDestroy(ctx->stream);
    if (ctx->side) cudaStreamDestroy(ctx->side);
    if (ctx->ev_fork) cudaEventDestroy(ctx->ev_fork);
    if (ctx->ev_join) cudaEventDestroy(ctx->ev_join);
    if (ctx->h_status) cudaFreeHost(ctx->h_status);
    if (ctx->ev_g0) cudaEventDestroy(ctx->ev_g0);
    if (ctx->ev_g1) cudaEventDestroy(ctx->ev_g1);
    delete ctx;
    return KTMOE_OK;
}

const char* ktmoe_last_error(const ktmoe_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "no context"; }
void* ktmoe_stream(ktmoe_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

int ktmoe_launch_count(ktmoe_ctx* ctx, uint64_t* n) {
    if (!ctx || !n) return KTMOE_ERR_ARG;
    *n = ctx->launches;
    return KTMOE_OK;
}

int ktmoe_sync(ktmoe_ctx* ctx, void* stream) {
    if (!ctx) return KTMOE_ERR_ARG;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    if (stream) CK(cudaStreamSynchronize((cudaStream_t)stream));
    CK(cudaStreamSynchronize(ctx->stream));
    return check_err_word(ctx);
}

int ktmoe_set_weight_budget(ktmoe_ctx* ctx, uint64_t bytes) {
    if (!ctx) return KTMOE_ERR_ARG;
    std::lock_guard<std::mutex> lk(ctx->mu);
    ctx->budget = bytes;
    return KTMOE_OK;
}

int ktmoe_resident_bytes(ktmoe_ctx* ctx, uint64_t* bytes) {
    if (!ctx || !bytes) return KTMOE_ERR_ARG;
    std::lock_guard<std::mutex> lk(ctx->mu);
    *bytes = ctx->resident;
    return KTMOE_OK;
}

constexpr size_t LIN_STAGE_MAX = 256u << 10;

static int linear_impl(ktmoe_ctx* ctx, const uint64_t* weight_id, const int32_t* x, const int32_t* w, int64_t rows,
                       int64_t out, int64_t k, int64_t* y) {
    if (!ctx || rows < 0 || out < 0 || k < 0) return KTMOE_ERR_ARG;
    if (rows == 0 || out == 0) return KTMOE_OK;
    if (!x || !w || !y) return KTMOE_ERR_ARG;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    cudaStream_t st = ctx->stream;
    if (k == 0) {
        std::memset(y, 0, (size_t)(rows * out) * 8);
        return KTMOE_OK;
    }
    const int64_t k_pad = round_up(k, dg::BK);
    // weights of more than one 128-row tile are padded to 256 rows, so that wide calls can use the pair GEMM
    const int64_t out_pad = out > dg::BM ? round_up(out, dg::pair::BM2) : dg::BM;
    const int64_t rows_pad = round_up(rows, 64);
    // counters: [0] codes beyond +-WLEVELS, [1] weight codes beyond +-3280, [2] activation codes beyond +-127
    CK(ctx->lin_bad.ensure(24));
    CK(cudaMemsetAsync(ctx->lin_bad.p, 0, 24, st));
    unsigned long long* counters = ctx->lin_bad.as<unsigned long long>();
    // Small codes (|x| <= 127, |w| <= 3280) take the (1, 2) plane GEMM unless KTMOE_SMALL=0.
    static const bool small_enabled = [] {
        const char* e = getenv("KTMOE_SMALL");
        return !(e && e[0] == '0');
    }();
    bool small_w = false;
    // weights: resident by id, else packed for this call
    Planes W{nullptr, 1, out_pad, k, k_pad};
    Resident* res = nullptr;
    if (weight_id) {
        auto it = ctx->cache.find(*weight_id);
        if (it != ctx->cache.end() && it->second->out == out && it->second->k == k) {
            res = it->second;
            res->last_use = ++ctx->tick;
        } else if (it != ctx->cache.end()) {
            // the id now names weights of another shape: drop the old planes before packing the new ones
            CK(cudaStreamSynchronize(st));
            ctx->resident -= it->second->buf.bytes;
            it->second->buf.release();
            delete it->second;
            ctx->cache.erase(it);
        }
    }
    unsigned long long hbad_w[2] = {0, 0};
    if (res) {
        W.ptr = res->buf.as<int8_t>();
        small_w = res->small;
    } else {
        const size_t wbytes = (size_t)(3 * out_pad * k_pad);
        DevBuf* target = &ctx->lin_wp;
        Resident* fresh = nullptr;
        if (weight_id && wbytes <= ctx->budget) {
            // evict least recently used until the new weights fit
            while (ctx->resident + wbytes > ctx->budget && !ctx->cache.empty()) {
                auto lru = ctx->cache.begin();
                for (auto it = ctx->cache.begin(); it != ctx->cache.end(); ++it)
                    if (it->second->last_use < lru->second->last_use) lru = it;
                ctx->resident -= lru->second->buf.bytes;
                lru->second->buf.release();
                delete lru->second;
                ctx->cache.erase(lru);
            }
            fresh = new Resident();
            target = &fresh->buf;
        }
        cudaError_t e = target->ensure(wbytes);
        if (e != cudaSuccess) {
            delete fresh;
            return fail_cuda(ctx, e, "weight planes");
        }
        CK(cudaMemsetAsync(target->p, 0, wbytes, st));
        CK(ctx->lin_wi.ensure((size_t)(out * k) * 4));
        CK(cudaMemcpyAsync(ctx->lin_wi.p, w, (size_t)(out * k) * 4, cudaMemcpyHostToDevice, st));
        KLAUNCH(st, (unsigned)out, 128, 0, (mk::pack_codes_kernel), ctx->lin_wi.as<int32_t>(), out, (int)k, (int)k_pad,
                out_pad, target->as<int8_t>(), counters, counters + 1, 3280, nullptr);
        CK(cudaMemcpyAsync(hbad_w, ctx->lin_bad.p, 16, cudaMemcpyDeviceToHost, st));
        CK(cudaStreamSynchronize(st));
        small_w = hbad_w[1] == 0;
        if (hbad_w[0]) {
            delete fresh;
            return fail(ctx, KTMOE_ERR_RANGE, "a weight code lies outside +-WLEVELS");
        }
        if (fresh) {
            fresh->out = out;
            fresh->k = k;
            fresh->out_pad = out_pad;
            fresh->k_pad = k_pad;
            fresh->small = small_w;
            fresh->last_use = ++ctx->tick;
            ctx->cache[*weight_id] = fresh;
            ctx->resident += fresh->buf.bytes;
        }
        W.ptr = target->as<int8_t>();
    }
    CK(ctx->lin_xi.ensure((size_t)(rows * k) * 4));
    CK(ctx->lin_xp.ensure((size_t)(3 * rows_pad * k_pad)));
    CK(ctx->lin_y.ensure((size_t)(rows * out) * 8));
    const size_t x_bytes = (size_t)(rows * k) * 4, y_bytes = (size_t)(rows * out) * 8;
    const bool stage_x = x_bytes <= LIN_STAGE_MAX && ctx->lin_hx.ensure(x_bytes) == cudaSuccess;
    const bool stage_y = y_bytes <= LIN_STAGE_MAX && ctx->lin_hy.ensure(y_bytes) == cudaSuccess;
    cudaGetLastError();  // a failed pinned allocation only means the pageable path
    if (stage_x) {
        CK(cudaStreamSynchronize(st));  // an earlier call that failed may have left its copy from the staging in flight
        std::memcpy(ctx->lin_hx.p, x, x_bytes);
        CK(cudaMemcpyAsync(ctx->lin_xi.p, ctx->lin_hx.p, x_bytes, cudaMemcpyHostToDevice, st));
    } else {
        CK(cudaMemcpyAsync(ctx->lin_xi.p, x, x_bytes, cudaMemcpyHostToDevice, st));
    }
    // with small weights, the activations are also written as one raw plane and their range decides the kernel
    const bool try_small = small_enabled && small_w;
    if (try_small) CK(ctx->lin_xr.ensure((size_t)(rows_pad * k_pad)));
    KLAUNCH(st, (unsigned)rows, 128, 0, (mk::pack_codes_kernel), ctx->lin_xi.as<int32_t>(), rows, (int)k, (int)k_pad,
            rows_pad, ctx->lin_xp.as<int8_t>(), counters, try_small ? counters + 2 : nullptr, 127,
            try_small ? ctx->lin_xr.as<int8_t>() : nullptr);
    bool small = false;
    if (try_small) {
        CK(cudaMemcpyAsync(ctx->h_status + 2, counters + 2, 8, cudaMemcpyDeviceToHost, st));
        CK(cudaStreamSynchronize(st));
        small = ctx->h_status[2] == 0;
    }
    const int BN = small ? pick_bn_small((double)rows) : pick_bn((double)rows, out_pad % dg::pair::BM2 == 0);
    GemmCall g;
    g.A = W;
    g.M_valid = out;
    g.B = small ? Planes{ctx->lin_xr.as<int8_t>(), 1, rows_pad, k, k_pad}
                : Planes{ctx->lin_xp.as<int8_t>(), 1, rows_pad, k, k_pad};
    g.small = small;
    ctx->last_gemm_planes = 0;
    g.ev0 = ctx->ev_g0;
    g.out = ctx->lin_y.as<int64_t>();
    g.ld_out = out;
    g.BN = BN;
    g.grid_y = (rows + BN - 1) / BN;
    g.single_rows = rows;
    if (int r = run_gemm(ctx, st, g)) return r;
    CK(cudaEventRecord(ctx->ev_g1, st));
    CK(cudaMemcpyAsync(ctx->h_status, ctx->lin_bad.p, 8, cudaMemcpyDeviceToHost, st));
    ctx->h_status[3] = 0;
    CK(cudaMemcpyAsync(ctx->h_status + 3, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(stage_y ? ctx->lin_hy.p : (void*)y, ctx->lin_y.p, y_bytes, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (stage_y) std::memcpy(y, ctx->lin_hy.p, y_bytes);
    if (ctx->h_status[3] != 0) {
        const int code = (int)(uint32_t)ctx->h_status[3];
        CK(cudaMemset(ctx->d_err, 0, sizeof(int)));
        return fail(ctx, KTMOE_ERR_KERNEL, "a kernel's bounded wait expired (code " + std::to_string(code) + ")");
    }
    if (ctx->h_status[0]) return fail(ctx, KTMOE_ERR_RANGE, "an activation code lies outside +-WLEVELS");
    ctx->last_gemm_planes = small ? 1 : 3;
    return KTMOE_OK;
}

int ktmoe_linear_last_gemm(ktmoe_ctx* ctx, double* ms, int32_t* act_planes) {
    if (!ctx || !ms || !act_planes) return KTMOE_ERR_ARG;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    *ms = 0.0;
    *act_planes = ctx->last_gemm_planes;
    if (ctx->last_gemm_planes == 0) return KTMOE_OK;
    CK(cudaEventSynchronize(ctx->ev_g1));
    float t = 0.f;
    CK(cudaEventElapsedTime(&t, ctx->ev_g0, ctx->ev_g1));
    *ms = t;
    return KTMOE_OK;
}

int ktmoe_linear(ktmoe_ctx* ctx, const int32_t* x, const int32_t* w, int64_t rows, int64_t out, int64_t k, int64_t* y) {
    return linear_impl(ctx, nullptr, x, w, rows, out, k, y);
}

int ktmoe_linear_weights(ktmoe_ctx* ctx, uint64_t weight_id, const int32_t* x, const int32_t* w, int64_t rows,
                         int64_t out, int64_t k, int64_t* y) {
    return linear_impl(ctx, &weight_id, x, w, rows, out, k, y);
}

static int layer_create(ktmoe_ctx* ctx, const ktmoe_layer_config* cfg, int rank, int world, const void* nccl_id,
                        ktmoe_layer** out) {
    if (!ctx || !cfg || !out) return KTMOE_ERR_ARG;
    *out = nullptr;
    if (world < 1 || rank < 0 || rank >= world || (world > 1 && !nccl_id)) return fail(ctx, KTMOE_ERR_ARG, "rank/world");
    if (cfg->n_experts < world) return fail(ctx, KTMOE_ERR_ARG, "fewer experts than ranks");
    const ktmoe_layer_config c = *cfg;
    if (c.d_model <= 0 || c.n_experts <= 0 || c.d_ff <= 0 || c.top_k <= 0 || c.shared_d_ff < 0)
        return fail(ctx, KTMOE_ERR_ARG, "layer dimensions must be positive");
    if (c.top_k > c.n_experts) return fail(ctx, KTMOE_ERR_ARG, "top_k exceeds the number of experts");
    if (c.n_experts > 512 || c.top_k > mk::COMBINE_MAX_K)
        return fail(ctx, KTMOE_ERR_UNSUPPORTED, "at most 512 experts and top_k <= 16");
    if (c.router_score != 0 && c.router_score != 1) return fail(ctx, KTMOE_ERR_ARG, "router_score is 0 or 1");
    if ((int64_t)c.d_model * 8 > 200 * 1024) return fail(ctx, KTMOE_ERR_UNSUPPORTED, "d_model above 25600");
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    ktmoe_layer* L = new ktmoe_layer();
    L->ctx = ctx;
    L->cfg = c;
    L->d = c.d_model;
    L->E = c.n_experts;
    L->f = c.d_ff;
    L->K = c.top_k;
    L->fs = c.shared_d_ff;
    L->d_pad = round_up(L->d, dg::BK);
    L->f_pad = round_up(L->f, dg::BK);
    L->fs_pad = round_up(std::max<int64_t>(L->fs, 1), dg::BK);
    L->rank = rank;
    L->world = world;
    L->e_begin = (int64_t)rank * L->E / world;
    L->e_end = (int64_t)(rank + 1) * L->E / world;
    L->E_local = L->e_end - L->e_begin;
    L->expert_set.assign(L->E_local, 0);
    int r = KTMOE_OK;
    auto bail = [&](int code) {
        delete L;
        return code;
    };
    if ((r = alloc_planes(ctx, L->b_router, L->w_router, 1, L->E, L->d))) return bail(r);
    if ((r = alloc_planes(ctx, L->b_gu, L->w_gu, L->E_local, 2 * L->f, L->d))) return bail(r);
    if ((r = alloc_planes(ctx, L->b_dn, L->w_dn, L->E_local, L->d, L->f))) return bail(r);
    if (L->fs > 0) {
        if ((r = alloc_planes(ctx, L->b_sgu, L->w_sgu, 1, 2 * L->fs, L->d))) return bail(r);
        if ((r = alloc_planes(ctx, L->b_sdn, L->w_sdn, 1, L->d, L->fs))) return bail(r);
    }
    L->h_wsc.assign(3 * L->E_local + 3, Scale{0, 0});
    if (L->b_wsc.ensure(L->h_wsc.size() * sizeof(Scale)) != cudaSuccess) return bail(fail(ctx, KTMOE_ERR_CUDA, "scales"));
    for (int kind = 0; kind < 3; ++kind) hp::build_table(kind, &L->tabs[kind]);
    L->silu_code_scale_recip = kt::scale_recip(S(L->tabs[1].code_scale));
    if (L->b_luts.ensure(3 * mk::LUT_N * 8) != cudaSuccess) return bail(fail(ctx, KTMOE_ERR_CUDA, "tables"));
    for (int kind = 0; kind < 3; ++kind)
        if (cudaMemcpy(L->b_luts.as<int64_t>() + kind * mk::LUT_N, L->tabs[kind].codes.data(), mk::LUT_N * 8,
                       cudaMemcpyHostToDevice) != cudaSuccess)
            return bail(fail(ctx, KTMOE_ERR_CUDA, "tables"));
    {
        std::vector<int32_t> c32(mk::LUT_N);
        L->silu32 = true;
        for (int i = 0; i < mk::LUT_N; ++i) {
            const int64_t c = L->tabs[1].codes[i];
            L->silu32 = L->silu32 && c == (int64_t)(int32_t)c;
            c32[i] = (int32_t)c;
        }
        if (L->silu32 && (L->b_silu32.ensure(mk::LUT_N * 4) != cudaSuccess ||
                          cudaMemcpy(L->b_silu32.p, c32.data(), mk::LUT_N * 4, cudaMemcpyHostToDevice) != cudaSuccess))
            return bail(fail(ctx, KTMOE_ERR_CUDA, "tables"));
    }
    if (L->b_rbias.ensure(L->E * 8) != cudaSuccess || L->b_sigbias.ensure(L->E * 8) != cudaSuccess)
        return bail(fail(ctx, KTMOE_ERR_CUDA, "bias"));
    // h of one row stays in shared memory only while that still leaves room for several resident blocks per SM;
    // a wide expert (Mixtral's 14336) keeps h in place of its gate accumulators, which the block just read.
    if (L->f * 8 <= 24 * 1024) {
        L->swiglu_smem = L->f * 8;
        if (L->swiglu_smem > 48 * 1024 &&
            (cudaFuncSetAttribute(mk::swiglu_rows_kernel<1, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)L->swiglu_smem) != cudaSuccess ||
             cudaFuncSetAttribute(mk::swiglu_rows_kernel<2, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)L->swiglu_smem) != cudaSuccess ||
             cudaFuncSetAttribute(mk::swiglu_rows_kernel<4, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)L->swiglu_smem) != cudaSuccess))
            return bail(fail(ctx, KTMOE_ERR_CUDA, "SwiGLU shared memory"));
    }
    if ((size_t)L->d * 8 > 48 * 1024) {
        const int cs = (int)(L->d * 8);
        if (cudaFuncSetAttribute(mk::combine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, cs) != cudaSuccess)
            return bail(fail(ctx, KTMOE_ERR_CUDA, "combine shared memory"));
        if (cudaFuncSetAttribute(mk::combine_y_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(L->d * 8)) !=
            cudaSuccess)
            return bail(fail(ctx, KTMOE_ERR_CUDA, "combine shared memory"));
        if (cudaFuncSetAttribute(mk::combine_tok_kernel<false, mk::CombineArgs>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, cs) != cudaSuccess ||
            cudaFuncSetAttribute(mk::combine_tok_kernel<true, mk::CombineYArgs>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, cs) != cudaSuccess)
            return bail(fail(ctx, KTMOE_ERR_CUDA, "combine shared memory"));
    }
    if (world > 1) {
        ncclUniqueId id;
        std::memcpy(&id, nccl_id, sizeof(id));
        ncclResult_t nr = ncclCommInitRank(&L->comm, world, id, rank);
        if (nr != ncclSuccess) {
            L->comm = nullptr;
            return bail(fail(ctx, KTMOE_ERR_CUDA, std::string("ncclCommInitRank: ") + ncclGetErrorString(nr)));
        }
    }
    *out = L;
    return KTMOE_OK;
}

int ktmoe_layer_create(ktmoe_ctx* ctx, const ktmoe_layer_config* cfg, ktmoe_layer** out) {
    return layer_create(ctx, cfg, 0, 1, nullptr, out);
}

int ktmoe_ep_unique_id(void* id, int64_t bytes) {
    if (!id || bytes < (int64_t)sizeof(ncclUniqueId)) return KTMOE_ERR_ARG;
    ncclUniqueId u;
    if (ncclGetUniqueId(&u) != ncclSuccess) return KTMOE_ERR_CUDA;
    std::memcpy(id, &u, sizeof(u));
    return KTMOE_OK;
}

int ktmoe_layer_create_ep(ktmoe_ctx* ctx, const ktmoe_layer_config* cfg, int32_t rank, int32_t world,
                          const void* nccl_id, ktmoe_layer** out) {
    return layer_create(ctx, cfg, rank, world, nccl_id, out);
}

int ktmoe_layer_experts(const ktmoe_layer* L, int32_t* begin, int32_t* end) {
    if (!L || !begin || !end) return KTMOE_ERR_ARG;
    *begin = (int32_t)L->e_begin;
    *end = (int32_t)L->e_end;
    return KTMOE_OK;
}

// Min over the ranks of one int (host value; NCCL on the context stream, synchronous). Also a barrier.
static int allreduce_min_host(ktmoe_layer* L, int v, int* out) {
    ktmoe_ctx* ctx = L->ctx;
    DevBuf b;
    CK(b.ensure(4));
    CK(cudaMemcpy(b.p, &v, 4, cudaMemcpyHostToDevice));
    NK(ncclAllReduce(b.p, b.p, 1, ncclInt32, ncclMin, L->comm, ctx->stream));
    CK(cudaMemcpyAsync(out, b.p, 4, cudaMemcpyDeviceToHost, ctx->stream));
    CK(cudaStreamSynchronize(ctx->stream));
    b.release();
    return KTMOE_OK;
}

// Unmap the peers' regions and free this rank's. `collective`: every rank does the same now, so a barrier makes sure
// no rank frees its region while another still has it mapped.
static void peer_close(ktmoe_layer* L, bool collective) {
    auto& pr = L->peer;
    for (int q = 0; q < ep::MAXW; ++q)
        if (pr.opened[q]) {
            cudaIpcCloseMemHandle(pr.opened[q]);
            pr.opened[q] = nullptr;
        }
    if (collective && pr.region.p) {
        int all = 0;
        allreduce_min_host(L, 1, &all);
    }
    DevBuf* bufs[] = {&pr.region, &pr.seq_dev, &pr.ctr, &pr.dst_base, &pr.rows_recv, &pr.group_end, &pr.tiles, &pr.tok_info,
                      &pr.recv_sqx, &pr.recv_expert};
    for (DevBuf* b : bufs) b->release();
    pr.on = false;
    pr.cap_T = pr.cap_rows = pr.cap_home = pr.bytes = 0;
}

int ktmoe_layer_set_ep_capacity(ktmoe_layer* L, int64_t max_tokens_per_rank) {
    if (!L || max_tokens_per_rank < 0 || max_tokens_per_rank > (int64_t(1) << 24)) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    if (L->world == 1) return KTMOE_OK;
    if (L->world > ep::MAXW) return fail(ctx, KTMOE_ERR_UNSUPPORTED, "the peer transport serves at most 8 ranks");
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    CK(cudaStreamSynchronize(ctx->stream));
    graphs_clear(L);
    peer_close(L, L->peer.on);
    if (max_tokens_per_rank == 0) return KTMOE_OK;
    auto& pr = L->peer;
    const int64_t G = L->world, E = L->E, K = L->K, d = L->d, dp = L->d_pad;
    auto a256 = [](int64_t x) { return (x + 255) / 256 * 256; };
    pr.cap_T = max_tokens_per_rank;
    pr.cap_home = pr.cap_T * K;
    pr.cap_rows = round_up(G * pr.cap_T * K, 64);  // every rank's rows could go to one owner
    ep::Peers& P = pr.P;
    std::memset(&P, 0, sizeof(P));
    P.world = (int)G;
    P.rank = L->rank;
    P.E = (int)E;
    P.e_begin = (int)L->e_begin;
    P.e_end = (int)L->e_end;
    P.d = (int)d;
    P.d_pad = (int)dp;
    int64_t off = a256(sizeof(ep::Box));
    P.off_counts = off;
    off += a256(G * (E + 1) * 4);
    P.off_planes = off;
    off += a256(3 * pr.cap_rows * dp);
    P.off_meta = off;
    off += a256(pr.cap_rows * 32);
    P.off_rety = off;
    off += a256(pr.cap_home * d * 4);
    P.off_retys = off;
    off += a256(pr.cap_home * (int64_t)sizeof(Scale));
    P.cap_rows = pr.cap_rows;
    P.cap_home = pr.cap_home;
    pr.bytes = off;
    // every step below is taken by every rank (the collectives stay matched when one rank fails locally)
    int ok = 1;
    cudaIpcMemHandle_t h;
    std::memset(&h, 0, sizeof(h));
    if (pr.region.ensure((size_t)off) != cudaSuccess || cudaMemset(pr.region.p, 0, (size_t)off) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess || cudaIpcGetMemHandle(&h, pr.region.p) != cudaSuccess)
        ok = 0;
    const int64_t tmax = pr.cap_rows / 16 + L->E_local + 1;
    if (ok && (pr.seq_dev.ensure(8) != cudaSuccess || cudaMemset(pr.seq_dev.p, 0, 8) != cudaSuccess ||
               pr.ctr.ensure(4) != cudaSuccess || cudaMemset(pr.ctr.p, 0, 4) != cudaSuccess ||
               pr.dst_base.ensure(E * 4) != cudaSuccess || pr.rows_recv.ensure(4) != cudaSuccess ||
               pr.group_end.ensure(L->E_local * 4) != cudaSuccess || pr.tiles.ensure((4 * tmax + 2) * 4) != cudaSuccess ||
               pr.tok_info.ensure(2 * 4) != cudaSuccess || pr.recv_sqx.ensure(pr.cap_rows * sizeof(Scale)) != cudaSuccess ||
               pr.recv_expert.ensure(pr.cap_rows * 4) != cudaSuccess || ensure_rows(L, pr.cap_rows) != KTMOE_OK))
        ok = 0;
    // every rank's region handle to every rank (NCCL, host-synchronous: this is set-up, not the forward)
    DevBuf hs;
    CK(hs.ensure((size_t)(G + 1) * sizeof(h)));
    CK(cudaMemcpy(hs.p, &h, sizeof(h), cudaMemcpyHostToDevice));
    NK(ncclAllGather(hs.p, (unsigned char*)hs.p + sizeof(h), sizeof(h), ncclInt8, L->comm, ctx->stream));
    std::vector<cudaIpcMemHandle_t> all(G);
    CK(cudaMemcpyAsync(all.data(), (unsigned char*)hs.p + sizeof(h), G * sizeof(h), cudaMemcpyDeviceToHost,
                       ctx->stream));
    CK(cudaStreamSynchronize(ctx->stream));
    hs.release();
    cudaError_t open_err = cudaSuccess;
    for (int64_t q = 0; q < G && ok; ++q) {
        if (q == L->rank) {
            P.base[q] = (unsigned char*)pr.region.p;
            continue;
        }
        void* ptr = nullptr;
        open_err = cudaIpcOpenMemHandle(&ptr, all[q], cudaIpcMemLazyEnablePeerAccess);
        if (open_err != cudaSuccess) {
            ok = 0;
            break;
        }
        pr.opened[q] = ptr;
        P.base[q] = (unsigned char*)ptr;
    }
    // all ranks learn whether all succeeded; this is also the barrier before anyone writes into a peer
    int all_ok = 0;
    if (int r = allreduce_min_host(L, ok, &all_ok)) return r;
    if (!all_ok) {
        peer_close(L, true);
        if (open_err != cudaSuccess) return fail_cuda(ctx, open_err, "cudaIpcOpenMemHandle");
        return fail(ctx, KTMOE_ERR_CUDA, ok ? "the peer transport could not be set up on another rank"
                                            : "the peer transport could not be set up");
    }
    P.seq = pr.seq_dev.as<unsigned long long>();
    pr.on = true;
    return KTMOE_OK;
}

int ktmoe_check_wait_expiry(ktmoe_ctx* ctx) {
    if (!ctx) return KTMOE_ERR_ARG;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    cudaStream_t st = ctx->stream;
    // two "ranks" whose regions are both this GPU's memory: rank 0 runs the exchange, rank 1 never does, so the wait
    // for rank 1's flag expires; every access stays inside these two allocations
    DevBuf a, b, words;
    struct Release {
        DevBuf* bufs[3];
        ~Release() {
            for (DevBuf* d : bufs) d->release();
        }
    } release{{&a, &b, &words}};
    CK(a.ensure(sizeof(ep::Box)));
    CK(b.ensure(sizeof(ep::Box)));
    CK(words.ensure(3 * sizeof(unsigned long long)));  // [0] seq, [1] the word sent, [2] the maximum received
    CK(cudaMemsetAsync(a.p, 0, sizeof(ep::Box), st));
    CK(cudaMemsetAsync(b.p, 0, sizeof(ep::Box), st));
    const unsigned long long init[3] = {1, 7, 0};
    CK(cudaMemcpyAsync(words.p, init, sizeof(init), cudaMemcpyHostToDevice, st));
    ep::Peers P{};
    P.base[0] = a.as<unsigned char>();
    P.base[1] = b.as<unsigned char>();
    P.world = 2;
    P.rank = 0;
    P.seq = words.as<unsigned long long>();
    KLAUNCH(st, 1, 32, 0, (ep::exchange_kernel), P, ep::P_MERGE, words.as<unsigned long long>() + 1, 1, nullptr,
            words.as<unsigned long long>() + 2, ctx->d_err);
    CK(cudaStreamSynchronize(st));
    return check_err_word(ctx);  // KTMOE_ERR_KERNEL with the wait's code; the error word is cleared
}

namespace {
void async_release(ktmoe_layer* L);  // the asynchronous forwards' streams, events and buffers (defined below)
}

int ktmoe_layer_destroy(ktmoe_layer* L) {
    if (!L) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    std::lock_guard<std::mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    DevBuf* bufs[] = {&L->b_router, &L->b_gu, &L->b_dn, &L->b_sgu, &L->b_sdn, &L->b_rbias, &L->b_sigbias, &L->b_wsc,
                      &L->b_luts, &L->b_silu32, &L->x_in, &L->y_out, &L->scal, &L->tok_planes, &L->tok_xmax, &L->tok_sqx,
                      &L->router_acc, &L->logits, &L->logit_scale, &L->top_e, &L->top_ec, &L->sumc, &L->counts,
                      &L->chunk_off, &L->expert_off, &L->group_end, &L->expert_count, &L->tile_group, &L->tile_row0, &L->tile_group2, &L->tile_row02,
                      &L->slot_row, &L->row_assign, &L->row_expert, &L->xg_planes, &L->acc_gu, &L->hq_planes,
                      &L->row_cd, &L->acc_d, &L->rowmax_gu, &L->rowmax_d, &L->tok_out, &L->tok_scale, &L->y_routed, &L->xs_planes, &L->acc_sgu,
                      &L->hs_planes, &L->acc_sd, &L->swiglu_plans, &L->row_hmax, &L->shared_plan,
                      &L->cp_n, &L->cp_common, &L->cp_row, &L->cp_ec, &L->cp_ry, &L->cp_f};
    for (DevBuf* b : bufs) b->release();
    DevBuf* blk_bufs[] = {&L->b_norm, &L->blk_c, &L->blk_xn, &L->blk_m, &L->blk_sc, &L->blk_u64, &L->blk_off,
                          &L->b_sgate, &L->sg_acc, &L->sg_code, &L->y_gated};
    for (DevBuf* b : blk_bufs) b->release();
    DevBuf* ep_bufs[] = {&L->ep_counts, &L->ep_counts_all, &L->ep_meta_send, &L->ep_meta_recv, &L->ep_recv_planes,
                         &L->ep_recv_sqx, &L->ep_recv_row_expert, &L->ep_y_send, &L->ep_ys_send, &L->ep_y_back,
                         &L->ep_ys_back, &L->ep_tiles, &L->ep_runs, &L->ep_rec, &L->ep_recs, &L->ep_best_idx};
    for (DevBuf* b : ep_bufs) b->release();
    for (WeightSet& w : L->slots) release_weights(w);
    async_release(L);
    graphs_clear(L);
    peer_close(L, L->peer.on);  // an expert-parallel layer is destroyed on every rank
    if (L->comm) ncclCommDestroy(L->comm);
    delete L;
    return KTMOE_OK;
}

static int push_scales(ktmoe_layer* L) {
    ktmoe_ctx* ctx = L->ctx;
    CK(cudaMemcpy(L->b_wsc.p, L->h_wsc.data(), L->h_wsc.size() * sizeof(Scale), cudaMemcpyHostToDevice));
    return KTMOE_OK;
}

int ktmoe_layer_set_router(ktmoe_layer* L, const int32_t* codes, ktmoe_scale w_scale, const int64_t* bias_codes,
                           ktmoe_scale bias_scale) {
    if (!L || !codes) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    std::lock_guard<std::mutex> lk(ctx->mu);
    graphs_clear(L);  // captured launches hold some of the layer's scales by value
    if (int r = set_device(ctx)) return r;
    if (int r = upload_matrix(ctx, L->w_router, 0, codes, L->E, L->d, 0)) return r;
    L->router_ws = S(w_scale);
    L->has_rbias = bias_codes != nullptr;
    if (bias_codes) {
        for (int64_t o = 0; o < L->E; ++o)
            if (bias_codes[o] > (int64_t)INT32_MAX || bias_codes[o] < (int64_t)INT32_MIN)
                return fail(ctx, KTMOE_ERR_RANGE, "a router bias code does not fit int32");
        CK(cudaMemcpy(L->b_rbias.p, bias_codes, L->E * 8, cudaMemcpyHostToDevice));
        L->router_bscale = S(bias_scale);
    }
    L->router_set = true;
    return KTMOE_OK;
}

int ktmoe_layer_set_sigmoid_bias(ktmoe_layer* L, const int64_t* bias_codes) {
    if (!L || !bias_codes) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    if (L->cfg.router_score != 1) return fail(ctx, KTMOE_ERR_ARG, "the layer's router is not sigmoid");
    std::lock_guard<std::mutex> lk(ctx->mu);
    graphs_clear(L);  // captured launches hold some of the layer's scales by value
    if (int r = set_device(ctx)) return r;
    CK(cudaMemcpy(L->b_sigbias.p, bias_codes, L->E * 8, cudaMemcpyHostToDevice));
    L->sigbias_set = true;
    return KTMOE_OK;
}

int ktmoe_layer_set_expert(ktmoe_layer* L, int32_t e, const int32_t* gate, ktmoe_scale gate_scale, const int32_t* up,
                           ktmoe_scale up_scale, const int32_t* down, ktmoe_scale down_scale) {
    if (!L || !gate || !up || !down || e < L->e_begin || e >= L->e_end) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    std::lock_guard<std::mutex> lk(ctx->mu);
    graphs_clear(L);  // captured launches hold some of the layer's scales by value
    if (int r = set_device(ctx)) return r;
    const int64_t le = e - L->e_begin;  // this rank's experts are stored from 0
    if (int r = upload_matrix(ctx, L->w_gu, le, gate, L->f, L->d, 0)) return r;
    if (int r = upload_matrix(ctx, L->w_gu, le, up, L->f, L->d, L->f)) return r;
    if (int r = upload_matrix(ctx, L->w_dn, le, down, L->d, L->f, 0)) return r;
    L->h_wsc[le] = S(gate_scale);
    L->h_wsc[L->E_local + le] = S(up_scale);
    L->h_wsc[2 * L->E_local + le] = S(down_scale);
    if (int r = push_scales(L)) return r;
    L->expert_set[le] = 1;
    return KTMOE_OK;
}

int ktmoe_layer_set_shared(ktmoe_layer* L, const int32_t* gate, ktmoe_scale gate_scale, const int32_t* up,
                           ktmoe_scale up_scale, const int32_t* down, ktmoe_scale down_scale) {
    if (!L || !gate || !up || !down) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    if (L->fs <= 0) return fail(ctx, KTMOE_ERR_ARG, "the layer has no shared expert");
    std::lock_guard<std::mutex> lk(ctx->mu);
    graphs_clear(L);  // captured launches hold some of the layer's scales by value
    if (int r = set_device(ctx)) return r;
    if (int r = upload_matrix(ctx, L->w_sgu, 0, gate, L->fs, L->d, 0)) return r;
    if (int r = upload_matrix(ctx, L->w_sgu, 0, up, L->fs, L->d, L->fs)) return r;
    if (int r = upload_matrix(ctx, L->w_sdn, 0, down, L->d, L->fs, 0)) return r;
    L->h_wsc[3 * L->E_local] = S(gate_scale);
    L->h_wsc[3 * L->E_local + 1] = S(up_scale);
    L->h_wsc[3 * L->E_local + 2] = S(down_scale);
    if (int r = push_scales(L)) return r;
    L->shared_set = true;
    return KTMOE_OK;
}

// ── a stack of layers in one object: weight slots that share the scratch and the exchange ──
namespace {

void swap_weights(ktmoe_layer* L, WeightSet& w) {
    using std::swap;
    swap(L->w_router, w.w_router);
    swap(L->w_gu, w.w_gu);
    swap(L->w_dn, w.w_dn);
    swap(L->w_sgu, w.w_sgu);
    swap(L->w_sdn, w.w_sdn);
    swap(L->b_router, w.b_router);
    swap(L->b_gu, w.b_gu);
    swap(L->b_dn, w.b_dn);
    swap(L->b_sgu, w.b_sgu);
    swap(L->b_sdn, w.b_sdn);
    swap(L->b_rbias, w.b_rbias);
    swap(L->b_sigbias, w.b_sigbias);
    swap(L->b_wsc, w.b_wsc);
    swap(L->b_norm, w.b_norm);
    swap(L->b_sgate, w.b_sgate);
    swap(L->h_wsc, w.h_wsc);
    swap(L->expert_set, w.expert_set);
    swap(L->router_ws, w.router_ws);
    swap(L->router_bscale, w.router_bscale);
    swap(L->norm_ws, w.norm_ws);
    swap(L->norm_eps, w.norm_eps);
    swap(L->sgate_ws, w.sgate_ws);
    swap(L->has_rbias, w.has_rbias);
    swap(L->router_set, w.router_set);
    swap(L->shared_set, w.shared_set);
    swap(L->sigbias_set, w.sigbias_set);
    swap(L->norm_set, w.norm_set);
    swap(L->sgate_set, w.sgate_set);
}

// One matrix [rows][k] of the portable normal stream `seed` from element `offset`, quantised per tensor as
// QuantLinear::from_weights does it (layers.rs:225-244) and packed into group g of P from row row0; its Scale out.
int synth_matrix(ktmoe_ctx* ctx, uint64_t seed, float sigma, uint64_t offset, const Planes& P, int64_t g, int64_t rows,
                 int64_t k, int64_t row0, DevBuf& fbuf, DevBuf& cbuf, DevBuf& wbuf, Scale* scale) {
    cudaStream_t st = ctx->stream;
    const int64_t n = rows * k;
    CK(fbuf.ensure((size_t)n * 4));
    CK(cbuf.ensure((size_t)n * 4));
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, ctx->num_sms * 8));
    KLAUNCH(st, grid, 256, 0, (sy::portable_normal_kernel), seed, sigma, offset, n, fbuf.as<float>());
    CK(cudaMemsetAsync(wbuf.p, 0, 4, st));  // the peak; word 1 counts codes out of range over the whole layer
    KLAUNCH(st, grid, 256, 0, (sy::absmax_f32_kernel), fbuf.as<float>(), n, wbuf.as<unsigned>());
    unsigned pbits = 0;
    CK(cudaMemcpyAsync(&pbits, wbuf.p, 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    float peak;
    std::memcpy(&peak, &pbits, 4);
    if (peak == 0.0f) {
        CK(cudaMemsetAsync(cbuf.p, 0, (size_t)n * 4, st));
        *scale = Scale{0, 0};
    } else {
        const double step = (double)peak / (double)kt::WLEVELS;
        KLAUNCH(st, grid, 256, 0, (sy::quantize_kernel), fbuf.as<float>(), n, step, cbuf.as<int32_t>());
        *scale = S(hp::scale_from_f64(step));
    }
    int8_t* base = P.ptr + (g * 3) * P.rows_pad * P.k_pad + row0 * P.k_pad;
    KLAUNCH(st, (unsigned)rows, 128, 0, (mk::pack_codes_kernel), cbuf.as<int32_t>(), rows, (int)k, (int)P.k_pad,
            P.rows_pad, base, wbuf.as<unsigned long long>() + 1, nullptr, 0, nullptr);
    return KTMOE_OK;
}

}  // namespace

int ktmoe_layer_set_depth(ktmoe_layer* L, int32_t n_layers) {
    if (!L || n_layers < 1) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!L->slots.empty()) return fail(ctx, KTMOE_ERR_ARG, "the layer's depth is already set");
    if (int r = set_device(ctx)) return r;
    graphs_clear(L);
    L->slots.resize((size_t)n_layers);  // slot 0 is the weights already in the layer
    for (int32_t i = 1; i < n_layers; ++i) {
        WeightSet& w = L->slots[(size_t)i];
        if (int r = alloc_planes(ctx, w.b_router, w.w_router, 1, L->E, L->d)) return r;
        if (int r = alloc_planes(ctx, w.b_gu, w.w_gu, L->E_local, 2 * L->f, L->d)) return r;
        if (int r = alloc_planes(ctx, w.b_dn, w.w_dn, L->E_local, L->d, L->f)) return r;
        if (L->fs > 0) {
            if (int r = alloc_planes(ctx, w.b_sgu, w.w_sgu, 1, 2 * L->fs, L->d)) return r;
            if (int r = alloc_planes(ctx, w.b_sdn, w.w_sdn, 1, L->d, L->fs)) return r;
        }
        w.h_wsc.assign(3 * L->E_local + 3, Scale{0, 0});
        w.expert_set.assign(L->E_local, 0);
        CK(w.b_wsc.ensure(w.h_wsc.size() * sizeof(Scale)));
        CK(w.b_rbias.ensure(L->E * 8));
        CK(w.b_sigbias.ensure(L->E * 8));
    }
    L->active = 0;
    return KTMOE_OK;
}

int ktmoe_layer_select(ktmoe_layer* L, int32_t slot) {
    if (!L) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    const int32_t n = std::max<int32_t>(1, (int32_t)L->slots.size());
    if (slot < 0 || slot >= n) return fail(ctx, KTMOE_ERR_ARG, "no such weight slot");
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (slot == L->active) return KTMOE_OK;
    swap_weights(L, L->slots[(size_t)L->active]);  // the current weights back into their slot
    swap_weights(L, L->slots[(size_t)slot]);
    L->active = slot;
    return KTMOE_OK;
}

int ktmoe_layer_synth_weights(ktmoe_layer* L, uint64_t seed, float sigma, float sigmoid_bias_sigma,
                              int32_t shared_gate) {
    if (!L || !(sigma > 0.0f)) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    if (shared_gate && L->fs <= 0) return fail(ctx, KTMOE_ERR_ARG, "the layer has no shared expert to gate");
    std::lock_guard<std::mutex> lk(ctx->mu);
    graphs_clear(L);
    if (int r = set_device(ctx)) return r;
    const int64_t d = L->d, E = L->E, f = L->f, fs = L->fs;
    DevBuf fbuf, cbuf, wbuf;
    auto done = [&](int r) {
        fbuf.release();
        cbuf.release();
        wbuf.release();
        return r;
    };
    CK(wbuf.ensure(16));
    CK(cudaMemsetAsync(wbuf.p, 0, 16, ctx->stream));
    Scale sc{0, 0};
    // one stream: router [E][d], expert e's gate [f][d], up [f][d], down [d][f], then the shared expert's gate, up,
    // down, then the shared expert's gate [1][d]; this rank draws only its own experts' ranges
    if (int r = synth_matrix(ctx, seed, sigma, 0, L->w_router, 0, E, d, 0, fbuf, cbuf, wbuf, &sc)) return done(r);
    L->router_ws = sc;
    L->has_rbias = false;
    const uint64_t base = (uint64_t)(E * d), per = (uint64_t)(3 * f * d);
    for (int64_t le = 0; le < L->E_local; ++le) {
        const uint64_t o = base + (uint64_t)(L->e_begin + le) * per;
        if (int r = synth_matrix(ctx, seed, sigma, o, L->w_gu, le, f, d, 0, fbuf, cbuf, wbuf, &sc)) return done(r);
        L->h_wsc[le] = sc;
        if (int r = synth_matrix(ctx, seed, sigma, o + f * d, L->w_gu, le, f, d, f, fbuf, cbuf, wbuf, &sc))
            return done(r);
        L->h_wsc[L->E_local + le] = sc;
        if (int r = synth_matrix(ctx, seed, sigma, o + 2 * f * d, L->w_dn, le, d, f, 0, fbuf, cbuf, wbuf, &sc))
            return done(r);
        L->h_wsc[2 * L->E_local + le] = sc;
        L->expert_set[le] = 1;
    }
    if (fs > 0) {
        const uint64_t o = base + (uint64_t)E * per;
        if (int r = synth_matrix(ctx, seed, sigma, o, L->w_sgu, 0, fs, d, 0, fbuf, cbuf, wbuf, &sc)) return done(r);
        L->h_wsc[3 * L->E_local] = sc;
        if (int r = synth_matrix(ctx, seed, sigma, o + fs * d, L->w_sgu, 0, fs, d, fs, fbuf, cbuf, wbuf, &sc))
            return done(r);
        L->h_wsc[3 * L->E_local + 1] = sc;
        if (int r = synth_matrix(ctx, seed, sigma, o + 2 * fs * d, L->w_sdn, 0, d, fs, 0, fbuf, cbuf, wbuf, &sc))
            return done(r);
        L->h_wsc[3 * L->E_local + 2] = sc;
        L->shared_set = true;
        L->sgate_set = false;
        if (shared_gate) {
            // the gate's d codes through the same device quantiser, then into the gate buffer (zero-padded to d_pad)
            CK(fbuf.ensure((size_t)d * 4));
            CK(cbuf.ensure((size_t)L->d_pad * 4));
            KLAUNCH(ctx->stream, (unsigned)((d + 255) / 256), 256, 0, (sy::portable_normal_kernel), seed, sigma,
                    o + 3 * fs * d, d, fbuf.as<float>());
            CK(cudaMemsetAsync(wbuf.p, 0, 4, ctx->stream));
            KLAUNCH(ctx->stream, (unsigned)((d + 255) / 256), 256, 0, (sy::absmax_f32_kernel), fbuf.as<float>(), d,
                    wbuf.as<unsigned>());
            unsigned pbits = 0;
            CK(cudaMemcpyAsync(&pbits, wbuf.p, 4, cudaMemcpyDeviceToHost, ctx->stream));
            CK(cudaStreamSynchronize(ctx->stream));
            float peak;
            std::memcpy(&peak, &pbits, 4);
            CK(cudaMemsetAsync(cbuf.p, 0, (size_t)L->d_pad * 4, ctx->stream));
            L->sgate_ws = Scale{0, 0};
            if (peak > 0.0f) {
                const double step = (double)peak / (double)kt::WLEVELS;
                KLAUNCH(ctx->stream, (unsigned)((d + 255) / 256), 256, 0, (sy::quantize_kernel), fbuf.as<float>(), d,
                        step, cbuf.as<int32_t>());
                L->sgate_ws = S(hp::scale_from_f64(step));
            }
            CK(L->b_sgate.ensure(L->d_pad * 4));
            CK(cudaMemcpyAsync(L->b_sgate.p, cbuf.p, L->d_pad * 4, cudaMemcpyDeviceToDevice, ctx->stream));
            L->sgate_set = true;
        }
    }
    L->router_set = true;
    if (L->cfg.router_score == 1) {
        // the sigmoid selection bias: E values of the portable stream seed + 2, coded round(b·2^20) (router.rs:35-51)
        std::vector<float> b((size_t)E);
        for (int64_t e = 0; e < E; ++e) b[(size_t)e] = sy::portable_normal(seed + 2, sigmoid_bias_sigma, (uint64_t)e);
        std::vector<int64_t> codes((size_t)E);
        hp::code_sigmoid_bias(b.data(), (size_t)E, codes.data());
        CK(cudaMemcpyAsync(L->b_sigbias.p, codes.data(), E * 8, cudaMemcpyHostToDevice, ctx->stream));
        L->sigbias_set = true;
    }
    CK(cudaMemcpyAsync(L->b_wsc.p, L->h_wsc.data(), L->h_wsc.size() * sizeof(Scale), cudaMemcpyHostToDevice,
                       ctx->stream));
    CK(cudaStreamSynchronize(ctx->stream));
    unsigned long long nbad = 0;
    CK(cudaMemcpy(&nbad, wbuf.as<unsigned long long>() + 1, 8, cudaMemcpyDeviceToHost));
    if (nbad) return done(fail(ctx, KTMOE_ERR_RANGE, "a synthesised code lies outside +-WLEVELS"));
    if (L->sgate_set) L->cap = 0;  // the next forward allocates the gate's scratch
    return done(KTMOE_OK);
}

int ktmoe_synth_normal_portable(uint64_t seed, float sigma, uint64_t offset, int64_t n, float* out) {
    if (n < 0 || (n > 0 && !out)) return KTMOE_ERR_ARG;
    for (int64_t j = 0; j < n; ++j) out[j] = sy::portable_normal(seed, sigma, offset + (uint64_t)j);
    return KTMOE_OK;
}

int ktmoe_synth_normal_portable_dev(ktmoe_ctx* ctx, uint64_t seed, float sigma, uint64_t offset, int64_t n,
                                    float* out_dev) {
    if (!ctx || n < 0 || (n > 0 && !out_dev)) return KTMOE_ERR_ARG;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    if (n == 0) return KTMOE_OK;
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, ctx->num_sms * 8));
    KLAUNCH(ctx->stream, grid, 256, 0, (sy::portable_normal_kernel), seed, sigma, offset, n, out_dev);
    CK(cudaStreamSynchronize(ctx->stream));
    return KTMOE_OK;
}

int ktmoe_layer_set_shared_gate(ktmoe_layer* L, const int32_t* codes, ktmoe_scale w_scale) {
    if (!L) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    if (L->fs <= 0) return fail(ctx, KTMOE_ERR_ARG, "the layer has no shared expert to gate");
    std::lock_guard<std::mutex> lk(ctx->mu);
    graphs_clear(L);
    if (int r = set_device(ctx)) return r;
    if (!codes) {
        L->sgate_set = false;
        return KTMOE_OK;
    }
    for (int64_t k = 0; k < L->d; ++k)
        if (codes[k] > (int32_t)kt::WLEVELS || codes[k] < -(int32_t)kt::WLEVELS)
            return fail(ctx, KTMOE_ERR_RANGE, "shared-expert gate codes beyond +-WLEVELS");
    std::vector<int32_t> padded((size_t)L->d_pad, 0);
    std::copy(codes, codes + L->d, padded.begin());
    CK(L->b_sgate.ensure(L->d_pad * 4));
    CK(cudaMemcpy(L->b_sgate.p, padded.data(), L->d_pad * 4, cudaMemcpyHostToDevice));
    L->sgate_ws = S(w_scale);
    L->sgate_set = true;
    L->cap = 0;  // the next forward allocates the gate's scratch
    return KTMOE_OK;
}

int ktmoe_forward_dev(ktmoe_layer* L, const int32_t* x_dev, int64_t rows, const ktmoe_scale* x_scale_dev,
                      int32_t* y_dev, ktmoe_scale* y_scale_dev, void* stream) {
    if (!L || !x_scale_dev || rows < 0 || (rows == 0 && L->world == 1)) return KTMOE_ERR_ARG;
    if (L->peer.on && rows > L->peer.cap_T) return fail(L->ctx, KTMOE_ERR_ARG, "more rows than the EP capacity");
    if (rows > 0 && (!x_dev || !y_dev || !y_scale_dev)) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    if (!layer_complete(L)) return fail(ctx, KTMOE_ERR_STATE, "a weight of the layer is not set");
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    if (int r = ensure_scratch(L, rows)) return r;
    cudaStream_t st = stream ? (cudaStream_t)stream : ctx->stream;
    return run_forward(L, rows, x_dev, (const Scale*)x_scale_dev, y_dev, (Scale*)y_scale_dev, st);
}

int ktmoe_forward(ktmoe_layer* L, const int32_t* x, int64_t rows, ktmoe_scale x_scale, int32_t* y,
                  ktmoe_scale* y_scale) {
    if (!L || !y_scale || rows < 0 || (rows == 0 && L->world == 1)) return KTMOE_ERR_ARG;
    if (L->peer.on && rows > L->peer.cap_T) return fail(L->ctx, KTMOE_ERR_ARG, "more rows than the EP capacity");
    if (rows > 0 && (!x || !y)) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    if (!layer_complete(L)) return fail(ctx, KTMOE_ERR_STATE, "a weight of the layer is not set");
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    if (int r = ensure_scratch(L, rows)) return r;
    cudaStream_t st = ctx->stream;
    const size_t n = (size_t)(rows * L->d);
    Scale xs = S(x_scale);
    if (n) CK(cudaMemcpyAsync(L->x_in.p, x, n * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(scal_scale(L, SL_XSCALE), &xs, sizeof(Scale), cudaMemcpyHostToDevice, st));
    if (int r = run_forward(L, rows, L->x_in.as<int32_t>(), scal_scale(L, SL_XSCALE), L->y_out.as<int32_t>(),
                              scal_scale(L, SL_YSCALE), st))
        return r;
    Scale ys{0, 0};
    if (n) CK(cudaMemcpyAsync(y, L->y_out.p, n * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(&ys, scal_scale(L, SL_YSCALE), sizeof(Scale), cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (int r = check_err_word(ctx)) return r;
    *y_scale = C(ys);
    return KTMOE_OK;
}

// ── asynchronous host-buffer forwards ──
namespace {

int async_init(ktmoe_layer* L) {
    ktmoe_ctx* ctx = L->ctx;
    auto& a = L->as;
    if (a.init) return KTMOE_OK;
    CK(cudaStreamCreateWithFlags(&a.up, cudaStreamNonBlocking));
    CK(cudaStreamCreateWithFlags(&a.down, cudaStreamNonBlocking));
    for (int s = 0; s < 2; ++s) {
        CK(cudaEventCreateWithFlags(&a.ev_up[s], cudaEventDisableTiming));
        CK(cudaEventCreateWithFlags(&a.ev_fwd[s], cudaEventDisableTiming));
        CK(cudaEventCreateWithFlags(&a.ev_down[s], cudaEventDisableTiming));
    }
    CK(a.sc.ensure(4 * sizeof(Scale)));
    CK(a.hsc.ensure(4 * sizeof(Scale)));
    a.init = true;
    return KTMOE_OK;
}

// Complete slot s's call: wait for its download, hand its output scale to the caller.
int async_finish(ktmoe_layer* L, int s) {
    ktmoe_ctx* ctx = L->ctx;
    auto& a = L->as;
    if (!a.pending[s]) return KTMOE_OK;
    a.pending[s] = false;
    CK(cudaEventSynchronize(a.ev_down[s]));
    const Scale ys = ((const Scale*)a.hsc.p)[2 * s + 1];
    if (a.ys_out[s]) *a.ys_out[s] = C(ys);
    return KTMOE_OK;
}

void async_release(ktmoe_layer* L) {
    auto& a = L->as;
    if (!a.init) return;
    if (a.up) cudaStreamSynchronize(a.up);
    if (a.down) cudaStreamSynchronize(a.down);
    for (int s = 0; s < 2; ++s) {
        cudaEventDestroy(a.ev_up[s]);
        cudaEventDestroy(a.ev_fwd[s]);
        cudaEventDestroy(a.ev_down[s]);
        a.x[s].release();
        a.y[s].release();
    }
    a.sc.release();
    a.hsc.release();
    cudaStreamDestroy(a.up);
    cudaStreamDestroy(a.down);
    a.init = false;
}

}  // namespace

int ktmoe_forward_async(ktmoe_layer* L, const int32_t* x, int64_t rows, ktmoe_scale x_scale, int32_t* y,
                        ktmoe_scale* y_scale) {
    if (!L || !y_scale || rows < 0 || (rows == 0 && L->world == 1)) return KTMOE_ERR_ARG;
    if (L->peer.on && rows > L->peer.cap_T) return fail(L->ctx, KTMOE_ERR_ARG, "more rows than the EP capacity");
    if (rows > 0 && (!x || !y)) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    if (!layer_complete(L)) return fail(ctx, KTMOE_ERR_STATE, "a weight of the layer is not set");
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    if (int r = async_init(L)) return r;
    auto& a = L->as;
    const int s = (int)(a.calls++ & 1);
    if (int r = async_finish(L, s)) return r;  // the call two back used this slot
    if (int r = ensure_scratch(L, rows)) return r;
    const size_t n = (size_t)(rows * L->d);
    CK(a.x[s].ensure(std::max<size_t>(n, 1) * 4));
    CK(a.y[s].ensure(std::max<size_t>(n, 1) * 4));
    Scale* hsc = (Scale*)a.hsc.p + 2 * s;
    Scale* dsc = a.sc.as<Scale>() + 2 * s;
    hsc[0] = S(x_scale);
    // upload: tokens and scale into slot s
    if (n) CK(cudaMemcpyAsync(a.x[s].p, x, n * 4, cudaMemcpyHostToDevice, a.up));
    CK(cudaMemcpyAsync(dsc, hsc, sizeof(Scale), cudaMemcpyHostToDevice, a.up));
    CK(cudaEventRecord(a.ev_up[s], a.up));
    // the forward, after the upload, on the context stream (after every earlier forward)
    CK(cudaStreamWaitEvent(ctx->stream, a.ev_up[s], 0));
    if (int r = run_forward(L, rows, a.x[s].as<int32_t>(), dsc, a.y[s].as<int32_t>(), dsc + 1, ctx->stream)) return r;
    CK(cudaEventRecord(a.ev_fwd[s], ctx->stream));
    // download: result and scale, after the forward
    CK(cudaStreamWaitEvent(a.down, a.ev_fwd[s], 0));
    if (n) CK(cudaMemcpyAsync(y, a.y[s].p, n * 4, cudaMemcpyDeviceToHost, a.down));
    CK(cudaMemcpyAsync(hsc + 1, dsc + 1, sizeof(Scale), cudaMemcpyDeviceToHost, a.down));
    CK(cudaEventRecord(a.ev_down[s], a.down));
    a.pending[s] = true;
    a.ys_out[s] = y_scale;
    return KTMOE_OK;
}

int ktmoe_forward_async_wait(ktmoe_layer* L) {
    if (!L) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    if (!L->as.init) return KTMOE_OK;
    int status = KTMOE_OK;
    for (int k = 0; k < 2; ++k) {
        const int s = (int)((L->as.calls + k) & 1);  // the older call first
        if (int r = async_finish(L, s)) status = status ? status : r;
    }
    if (int r = check_err_word(ctx)) status = status ? status : r;
    return status;
}

int ktmoe_layer_set_norm(ktmoe_layer* L, const int32_t* w_codes, ktmoe_scale w_scale, ktmoe_scale eps_scale) {
    if (!L || !w_codes) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    for (int64_t i = 0; i < L->d; ++i)
        if (w_codes[i] > kt::WLEVELS || w_codes[i] < -kt::WLEVELS) return fail(ctx, KTMOE_ERR_RANGE, "norm code");
    CK(cudaStreamSynchronize(ctx->stream));
    CK(L->b_norm.ensure(L->d * 4));
    CK(cudaMemcpy(L->b_norm.p, w_codes, L->d * 4, cudaMemcpyHostToDevice));
    L->norm_ws = S(w_scale);
    L->norm_eps = S(eps_scale);
    L->norm_set = true;
    graphs_clear(L);  // graphs captured the old scales as kernel arguments
    return KTMOE_OK;
}

int ktmoe_block_forward_dev(ktmoe_layer* L, const int32_t* x_dev, int64_t rows, const ktmoe_scale* x_scale_dev,
                            int32_t* y_dev, ktmoe_scale* y_scale_dev, void* stream) {
    if (!L || !x_scale_dev || rows < 0 || (rows == 0 && L->world == 1)) return KTMOE_ERR_ARG;
    if (L->peer.on && rows > L->peer.cap_T) return fail(L->ctx, KTMOE_ERR_ARG, "more rows than the EP capacity");
    if (rows > 0 && (!x_dev || !y_dev || !y_scale_dev)) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    if (!layer_complete(L) || !L->norm_set) return fail(ctx, KTMOE_ERR_STATE, "a weight of the block is not set");
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    if (int r = ensure_scratch(L, rows)) return r;
    if (int r = ensure_block(L, rows)) return r;
    cudaStream_t st = stream ? (cudaStream_t)stream : ctx->stream;
    return run_forward(L, rows, x_dev, (const Scale*)x_scale_dev, y_dev, (Scale*)y_scale_dev, st, true);
}

int ktmoe_block_forward(ktmoe_layer* L, const int32_t* x, int64_t rows, ktmoe_scale x_scale, int32_t* y,
                        ktmoe_scale* y_scale) {
    if (!L || !y_scale || rows < 0 || (rows == 0 && L->world == 1)) return KTMOE_ERR_ARG;
    if (L->peer.on && rows > L->peer.cap_T) return fail(L->ctx, KTMOE_ERR_ARG, "more rows than the EP capacity");
    if (rows > 0 && (!x || !y)) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    if (!layer_complete(L) || !L->norm_set) return fail(ctx, KTMOE_ERR_STATE, "a weight of the block is not set");
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    if (int r = ensure_scratch(L, rows)) return r;
    if (int r = ensure_block(L, rows)) return r;
    cudaStream_t st = ctx->stream;
    const size_t n = (size_t)(rows * L->d);
    Scale xs = S(x_scale);
    if (n) CK(cudaMemcpyAsync(L->x_in.p, x, n * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(scal_scale(L, SL_XSCALE), &xs, sizeof(Scale), cudaMemcpyHostToDevice, st));
    if (int r = run_forward(L, rows, L->x_in.as<int32_t>(), scal_scale(L, SL_XSCALE), L->y_out.as<int32_t>(),
                            scal_scale(L, SL_YSCALE), st, true))
        return r;
    Scale ys{0, 0};
    if (n) CK(cudaMemcpyAsync(y, L->y_out.p, n * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(&ys, scal_scale(L, SL_YSCALE), sizeof(Scale), cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (int r = check_err_word(ctx)) return r;
    *y_scale = C(ys);
    return KTMOE_OK;
}

int ktmoe_scale_from_f64(double x, ktmoe_scale* out) {
    if (!out) return KTMOE_ERR_ARG;
    const hp::HScale h = hp::scale_from_f64(x);
    *out = ktmoe_scale{h.mant, h.shift};
    return KTMOE_OK;
}

int ktmoe_route(ktmoe_layer* L, const int32_t* x, int64_t rows, ktmoe_scale x_scale, int32_t* experts, int64_t* ec,
                int64_t* sumc) {
    if (!L || !x || !experts || !ec || !sumc || rows <= 0) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    if (!L->router_set || (L->cfg.router_score == 1 && !L->sigbias_set))
        return fail(ctx, KTMOE_ERR_STATE, "the router is not set");
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    if (int r = ensure_scratch(L, rows)) return r;
    cudaStream_t st = ctx->stream;
    Scale xs = S(x_scale);
    CK(cudaMemcpyAsync(L->x_in.p, x, (size_t)(rows * L->d) * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(scal_scale(L, SL_XSCALE), &xs, sizeof(Scale), cudaMemcpyHostToDevice, st));
    if (int r = stage_route(L, rows, L->x_in.as<int32_t>(), scal_scale(L, SL_XSCALE), st)) return r;
    CK(cudaMemcpyAsync(experts, L->top_e.p, (size_t)(rows * L->K) * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(ec, L->top_ec.p, (size_t)(rows * L->K) * 8, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(sumc, L->sumc.p, (size_t)rows * 8, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    return check_err_word(ctx);
}

// ── the expert-parallel seam: MoeMlp::forward_int_with_experts (layers.rs:945-984) with the experts elsewhere ──

int ktmoe_layer_expert_forward(ktmoe_layer* L, const int32_t* x, int64_t rows, ktmoe_scale x_scale,
                               const int32_t* ids, int32_t n_ids, int32_t* y, ktmoe_scale* y_scale) {
    if (!L || rows < 0 || n_ids < 0) return KTMOE_ERR_ARG;
    if (rows == 0 || n_ids == 0) return KTMOE_OK;
    if (!x || !ids || !y || !y_scale) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    if (L->world != 1) return fail(ctx, KTMOE_ERR_UNSUPPORTED, "the seam runs on a single-rank layer");
    const int64_t n_req = rows * (int64_t)n_ids;
    int32_t fill = -1;  // a set expert that stands in for empty slots (its outputs there are discarded)
    for (int64_t i = 0; i < n_req; ++i) {
        const int32_t e = ids[i];
        if (e >= L->E) return fail(ctx, KTMOE_ERR_ARG, "an expert id is out of range");
        if (e < 0) continue;
        if (!L->expert_set[e]) return fail(ctx, KTMOE_ERR_STATE, "a requested expert is not set");
        if (fill < 0) fill = e;
    }
    if (fill < 0) {  // nothing requested: every output is zero with a zero scale
        std::memset(y, 0, (size_t)(n_req * L->d) * 4);
        for (int64_t i = 0; i < n_req; ++i) y_scale[i] = ktmoe_scale{0, 0};
        return KTMOE_OK;
    }
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    if (int r = ensure_scratch(L, rows)) return r;
    cudaStream_t st = ctx->stream;
    const int64_t d = L->d, E = L->E, f = L->f, K = L->K, T = rows, R = T * K;
    const int64_t R_pad = round_up(R, 64);
    CK(L->seam_y.ensure((size_t)(n_req * d) * 4));
    CK(L->seam_ys.ensure((size_t)n_req * sizeof(Scale)));
    CK(L->seam_ids.ensure((size_t)n_req * 4));
    Scale xs = S(x_scale);
    CK(cudaMemcpyAsync(L->x_in.p, x, (size_t)(T * d) * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(scal_scale(L, SL_XSCALE), &xs, sizeof(Scale), cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(L->seam_ids.p, ids, (size_t)n_req * 4, cudaMemcpyHostToDevice, st));
    if (int r = stage_quant(L, T, L->x_in.as<int32_t>(), scal_scale(L, SL_XSCALE), st)) return r;
    // the requests in chunks of K per row, each through the layer's routed pipeline with the ids as its top-k
    std::vector<int32_t> te((size_t)R);
    const int BN = pick_bn((double)R / (double)E, true), BN2 = pick_bn_long_k((double)R / (double)E, f, true);
    for (int32_t j0 = 0; j0 < n_ids; j0 += (int32_t)K) {
        const int32_t Kc = (int32_t)std::min<int64_t>(K, n_ids - j0);
        for (int64_t t = 0; t < T; ++t)
            for (int64_t s = 0; s < K; ++s) {
                const int32_t e = s < Kc ? ids[t * n_ids + j0 + s] : -1;
                te[(size_t)(t * K + s)] = e >= 0 ? e : fill;
            }
        CK(cudaMemcpyAsync(L->top_e.p, te.data(), (size_t)R * 4, cudaMemcpyHostToDevice, st));
        if (int r = plan_and_permute(L, T, BN, BN2, st)) return r;
        ExpertRows xr;
        xr.B = Planes{L->xg_planes.as<int8_t>(), 1, R_pad, d, L->d_pad};
        xr.n_rows = R;
        xr.BN = BN;
        xr.BN2 = BN2;
        xr.grid_a = (R + BN - 1) / BN + E;
        xr.grid_b = (R + BN2 - 1) / BN2 + E;
        xr.tg_a = L->tile_group.as<int>();
        xr.tr_a = L->tile_row0.as<int>();
        xr.te_a = nullptr;
        xr.nt_a = n_tiles_ptr(L);
        xr.tg_b = L->tile_group2.as<int>();
        xr.tr_b = L->tile_row02.as<int>();
        xr.te_b = nullptr;
        xr.nt_b = n_tiles2_ptr(L);
        xr.group_end = L->group_end.as<int>();
        xr.row_assign = L->row_assign.as<int>();
        xr.row_expert = L->row_expert.as<int>();
        xr.row_sqx = L->tok_sqx.as<Scale>();
        if (int r = run_experts(L, xr, st)) return r;
        KLAUNCH(st, (unsigned)R, 256, 0, (mk::seam_out_kernel), L->acc_d.as<int64_t>(),
                L->rowmax_d.as<unsigned long long>(), L->row_cd.as<Scale>(), L->row_assign.as<int>(), (int)R, (int)d,
                (int)K, Kc, n_ids, j0, L->seam_ids.as<int32_t>(), L->seam_y.as<int32_t>(), L->seam_ys.as<Scale>());
        // te is reused by the next chunk: its copy must have left the host buffer first
        CK(cudaStreamSynchronize(st));
    }
    std::vector<Scale> hs((size_t)n_req);
    CK(cudaMemcpyAsync(y, L->seam_y.p, (size_t)(n_req * d) * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(hs.data(), L->seam_ys.p, (size_t)n_req * sizeof(Scale), cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (int r = check_err_word(ctx)) return r;
    for (int64_t i = 0; i < n_req; ++i) y_scale[i] = C(hs[(size_t)i]);
    return KTMOE_OK;
}

int ktmoe_layer_forward_with_experts(ktmoe_layer* L, const int32_t* x, int64_t rows, ktmoe_scale x_scale,
                                     ktmoe_experts_fn experts_fn, void* user, int32_t* y, ktmoe_scale* y_scale) {
    if (!L || !experts_fn || !y_scale || rows <= 0 || !x || !y) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    if (L->world != 1) return fail(ctx, KTMOE_ERR_UNSUPPORTED, "the seam runs on a single-rank layer");
    if (!L->router_set || (L->cfg.router_score == 1 && !L->sigbias_set) || (L->fs > 0 && !L->shared_set))
        return fail(ctx, KTMOE_ERR_STATE, "the router or the shared expert is not set");
    const int64_t d = L->d, K = L->K, T = rows, R = T * K;
    const Scale xs = S(x_scale);
    cudaStream_t st = ctx->stream;
    std::vector<int32_t> ids((size_t)R);
    std::vector<int64_t> ec((size_t)R), sumc((size_t)T);
    {
        // route; the callback runs without the context's lock (it may call into this library, even this layer),
        // so what the combine needs from the route is kept on the host across it
        std::lock_guard<std::mutex> lk(ctx->mu);
        if (int r = set_device(ctx)) return r;
        if (int r = ensure_scratch(L, T)) return r;
        CK(cudaMemcpyAsync(L->x_in.p, x, (size_t)(T * d) * 4, cudaMemcpyHostToDevice, st));
        CK(cudaMemcpyAsync(scal_scale(L, SL_XSCALE), &xs, sizeof(Scale), cudaMemcpyHostToDevice, st));
        if (int r = stage_route(L, T, L->x_in.as<int32_t>(), scal_scale(L, SL_XSCALE), st)) return r;
        CK(cudaMemcpyAsync(ids.data(), L->top_e.p, (size_t)R * 4, cudaMemcpyDeviceToHost, st));
        CK(cudaMemcpyAsync(ec.data(), L->top_ec.p, (size_t)R * 8, cudaMemcpyDeviceToHost, st));
        CK(cudaMemcpyAsync(sumc.data(), L->sumc.p, (size_t)T * 8, cudaMemcpyDeviceToHost, st));
        CK(cudaStreamSynchronize(st));
        if (int r = check_err_word(ctx)) return r;
    }
    // a row whose route is empty never reaches the callback in the reference: its ids are -1 here
    for (int64_t t = 0; t < T; ++t)
        if (sumc[(size_t)t] <= 0)
            for (int64_t i = 0; i < K; ++i) ids[(size_t)(t * K + i)] = -1;
    std::vector<int32_t> ye((size_t)(R * d), 0);
    std::vector<ktmoe_scale> yse((size_t)R, ktmoe_scale{0, 0});
    const int cb = experts_fn(user, T, (int32_t)K, ids.data(), x, x_scale, ye.data(), yse.data());
    if (cb != 0) return fail(ctx, KTMOE_ERR_CALLBACK, "the experts callback returned " + std::to_string(cb));
    std::vector<Scale> ys_h((size_t)R);
    for (int64_t i = 0; i < R; ++i) ys_h[(size_t)i] = S(yse[(size_t)i]);

    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    if (int r = ensure_scratch(L, T)) return r;
    CK(L->seam_y.ensure((size_t)(R * d) * 4));
    CK(L->seam_ys.ensure((size_t)R * sizeof(Scale)));
    CK(cudaMemsetAsync(scal_u64(L, 0), 0, U_N * 8, st));
    CK(cudaMemcpyAsync(L->x_in.p, x, (size_t)(T * d) * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(scal_scale(L, SL_XSCALE), &xs, sizeof(Scale), cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(L->top_ec.p, ec.data(), (size_t)R * 8, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(L->sumc.p, sumc.data(), (size_t)T * 8, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(L->seam_y.p, ye.data(), (size_t)(R * d) * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(L->seam_ys.p, ys_h.data(), (size_t)R * sizeof(Scale), cudaMemcpyHostToDevice, st));
    KLAUNCH(st, (unsigned)std::min<int64_t>((R + 255) / 256, 1024), 256, 0, (mk::iota_kernel), L->slot_row.as<int>(),
            R);
    mk::CombineYArgs ca;
    ca.y = L->seam_y.as<int32_t>();
    ca.ys = L->seam_ys.as<Scale>();
    ca.slot_row = L->slot_row.as<int>();
    ca.top_ec = L->top_ec.as<int64_t>();
    ca.sumc = L->sumc.as<int64_t>();
    ca.T = (int)T;
    ca.top_k = (int)K;
    ca.dim = (int)d;
    ca.out = L->tok_out.as<int32_t>();
    ca.out_scale = L->tok_scale.as<Scale>();
    const mk::CombinePlan cp{L->cp_n.as<int>(), L->cp_common.as<Scale>(), L->cp_row.as<int>(),
                             L->cp_ec.as<int64_t>(), L->cp_ry.as<kt::ReqDiv>(), L->cp_f.as<kt::ApplyPlan>()};
    if (int r = launch_combine<true>(L, ca, cp, T, st)) return r;
    if (int r = merge_and_add(L, T, T, 0, L->x_in.as<int32_t>(), scal_scale(L, SL_XSCALE), L->y_out.as<int32_t>(),
                              scal_scale(L, SL_YSCALE), st, false))
        return r;
    Scale ys{0, 0};
    CK(cudaMemcpyAsync(y, L->y_out.p, (size_t)(T * d) * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(&ys, scal_scale(L, SL_YSCALE), sizeof(Scale), cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (int r = check_err_word(ctx)) return r;
    *y_scale = C(ys);
    return KTMOE_OK;
}

int ktmoe_layer_set_graphs(ktmoe_layer* L, int32_t enable) {
    if (!L) return KTMOE_ERR_ARG;
    std::lock_guard<std::mutex> lk(L->ctx->mu);
    if (int r = set_device(L->ctx)) return r;
    cudaStreamSynchronize(L->ctx->stream);
    graphs_clear(L);
    L->graphs = enable != 0;
    return KTMOE_OK;
}

int ktmoe_layer_set_timing(ktmoe_layer* L, int32_t enable) {
    if (!L) return KTMOE_ERR_ARG;
    std::lock_guard<std::mutex> lk(L->ctx->mu);
    L->timing = enable != 0;
    return KTMOE_OK;
}

int ktmoe_layer_stage_times(ktmoe_layer* L, double* ms, int32_t n_stages, int32_t* n_forwards) {
    if (!L || !ms || !n_forwards || n_stages < ST_N) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    for (int i = 0; i < n_stages; ++i) ms[i] = 0.0;
    *n_forwards = 0;
    // Each timed forward recorded 1 + (stages it ran) events; stages run in order, so split the sequence at
    // every first event (the one recorded before routing) by counting: a forward records ST_MERGE + 2 events
    // without a shared expert and ST_SHARED + 2 with one.
    const size_t per = (size_t)((L->fs > 0 ? ST_SHARED : ST_MERGE) + 2);
    const size_t nf = L->events.size() / per;
    for (size_t f = 0; f < nf; ++f) {
        for (size_t i = 0; i + 1 < per; ++i) {
            cudaEvent_t a = L->events[f * per + i], b = L->events[f * per + i + 1];
            CK(cudaEventSynchronize(b));
            float t = 0.f;
            CK(cudaEventElapsedTime(&t, a, b));
            ms[i] += t;
        }
    }
    for (cudaEvent_t e : L->events) cudaEventDestroy(e);
    L->events.clear();
    *n_forwards = (int32_t)nf;
    return KTMOE_OK;
}

// Internal buffers of the last forward, for stage-level checks: which = 0 router logits [rows][E] int32,
// 1 logit scales [rows], 2 per-token combine outputs [rows][d] int32, 3 their scales [rows].
int ktmoe_layer_debug_fetch(ktmoe_layer* L, int32_t which, void* host, int64_t bytes) {
    if (!L || !host || bytes < 0) return KTMOE_ERR_ARG;
    ktmoe_ctx* ctx = L->ctx;
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (int r = set_device(ctx)) return r;
    const DevBuf* b = which == 0 ? &L->logits : which == 1 ? &L->logit_scale : which == 2 ? &L->tok_out : &L->tok_scale;
    if ((size_t)bytes > b->bytes) return fail(ctx, KTMOE_ERR_ARG, "debug fetch beyond the buffer");
    CK(cudaStreamSynchronize(ctx->stream));
    CK(cudaMemcpy(host, b->p, (size_t)bytes, cudaMemcpyDeviceToHost));
    return KTMOE_OK;
}

// ── offline host preparation ──
int ktmoe_quantize_weights(const float* w, int64_t n, int32_t* codes, ktmoe_scale* scale) {
    if (n < 0 || (n > 0 && (!w || !codes)) || !scale) return KTMOE_ERR_ARG;
    hp::HScale s;
    hp::quantize_weights(w, (size_t)n, codes, &s);
    *scale = ktmoe_scale{s.mant, s.shift};
    return KTMOE_OK;
}

int ktmoe_quantize_bias(const float* b, int64_t n, int64_t* codes, ktmoe_scale* scale, int32_t* has_bias) {
    if (!b || !codes || !scale || !has_bias || n < 0) return KTMOE_ERR_ARG;
    hp::HScale s{0, 0};
    *has_bias = hp::quantize_bias(b, (size_t)n, codes, &s) ? 1 : 0;
    *scale = ktmoe_scale{s.mant, s.shift};
    return KTMOE_OK;
}

int ktmoe_code_sigmoid_bias(const float* b, int64_t n, int64_t* codes) {
    if (!b || !codes || n < 0) return KTMOE_ERR_ARG;
    hp::code_sigmoid_bias(b, (size_t)n, codes);
    return KTMOE_OK;
}

int ktmoe_from_reals(const float* v, int64_t n, int32_t* data, ktmoe_scale* scale) {
    if (!v || !data || !scale || n < 0) return KTMOE_ERR_ARG;
    hp::HScale s;
    hp::from_reals(v, (size_t)n, data, &s);
    *scale = ktmoe_scale{s.mant, s.shift};
    return KTMOE_OK;
}

int ktmoe_table(int32_t kind, int64_t* codes, ktmoe_scale* inv_step, int64_t* lo_index, ktmoe_scale* code_scale) {
    if (kind < 0 || kind > 2 || !codes || !inv_step || !lo_index || !code_scale) return KTMOE_ERR_ARG;
    hp::HTable t;
    hp::build_table(kind, &t);
    std::memcpy(codes, t.codes.data(), t.codes.size() * 8);
    *inv_step = ktmoe_scale{t.inv_step.mant, t.inv_step.shift};
    *lo_index = t.lo_index;
    *code_scale = ktmoe_scale{t.code_scale.mant, t.code_scale.shift};
    return KTMOE_OK;
}

// MoeRoute::margin of softmax routes (layers.rs:831-849): per row, every expert's exp code (CodeLut::index of
// logit - lmax at the row's logit scale, layers.rs:837-838: 0 below the table, the clamped code above it), then the
// strongest code left out of the route over the weakest chosen one, 0 when that is 0. Host only, exact integers up
// to the final division.
int ktmoe_route_margins(const int32_t* logits, int64_t rows, int32_t n_experts, const ktmoe_scale* scales,
                        const int32_t* experts, int32_t top_k, double* margins) {
    if (rows < 0 || n_experts <= 0 || top_k <= 0 || top_k > n_experts) return KTMOE_ERR_ARG;
    if (rows > 0 && (!logits || !scales || !experts || !margins)) return KTMOE_ERR_ARG;
    static const hp::HTable t = [] {
        hp::HTable x;
        hp::build_table(0, &x);
        return x;
    }();
    const int64_t n = (int64_t)t.codes.size();
    std::vector<int64_t> ecs(n_experts);
    std::vector<char> chosen(n_experts);
    for (int64_t r = 0; r < rows; ++r) {
        const int32_t* lg = logits + r * n_experts;
        int32_t lmax = INT32_MIN;
        for (int32_t j = 0; j < n_experts; ++j) lmax = std::max(lmax, lg[j]);
        const Scale s = kt::scale_mul(S(scales[r]), S(t.inv_step));
        for (int32_t j = 0; j < n_experts; ++j) {
            const int64_t idx = kt::scale_apply(s, (int64_t)lg[j] - lmax) - t.lo_index;
            ecs[j] = idx < 0 ? 0 : t.codes[(size_t)std::min(idx, n - 1)];
        }
        std::fill(chosen.begin(), chosen.end(), 0);
        int64_t weakest = INT64_MAX, strongest = 0;
        for (int32_t i = 0; i < top_k; ++i) {
            const int32_t e = experts[r * top_k + i];
            if (e < 0 || e >= n_experts) return KTMOE_ERR_ARG;
            chosen[e] = 1;
            weakest = std::min(weakest, ecs[e]);
        }
        for (int32_t j = 0; j < n_experts; ++j)
            if (!chosen[j]) strongest = std::max(strongest, ecs[j]);
        margins[r] = weakest > 0 ? (double)strongest / (double)weakest : 0.0;
    }
    return KTMOE_OK;
}

int ktmoe_synth_normal(uint64_t seed, float sigma, uint64_t offset, int64_t n, float* out) {
    if (n < 0 || (n > 0 && !out)) return KTMOE_ERR_ARG;
    hp::synth_normal(seed, sigma, offset, (size_t)n, out);
    return KTMOE_OK;
}

int ktmoe_lcg_uniform(uint64_t seed, int64_t lo, int64_t hi, int64_t n, int32_t* out) {
    if (n < 0 || (n > 0 && !out) || hi < lo) return KTMOE_ERR_ARG;
    hp::lcg_uniform(seed, lo, hi, (size_t)n, out);
    return KTMOE_OK;
}

}  // extern "C"
