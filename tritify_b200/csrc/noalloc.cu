// ktmoe_linear_noalloc: the exact linear accumulate (Y = X·Wᵀ, int32 codes -> int64) for callers that cannot let a
// library allocate device memory.
//
// Who needs it: a host that owns every byte of device memory itself — a serving runtime that carves one pool out of
// the GPU at start-up and forbids later allocations, or a caller that runs under a memory budget where a
// cudaMalloc/cudaFree from inside a library call would break its accounting or stall its other streams. Such a
// caller hands in device buffers for the inputs and the output; this entry point keeps its own scratch (the digit
// planes of X and W, and two control words) in the file-scope device array below, so it calls no cudaMalloc,
// cudaFree or allocating library routine.
//
// The array is part of this file's device code: every GPU on which this entry point runs holds it (64 MiB) until the
// process exits. Its address is looked up once per device with cudaGetSymbolAddress, by the first call on that device,
// which also loads this entry point's kernels there (so that first call should come before any CUDA stream capture; a
// first call on a stream that is being captured returns KTMOE_ERR_ARG). All calls on one device share that device's
// array and it keeps the last call's contents, so two calls whose GPU work overlaps on one device (two streams, or two
// host threads) race and must be serialised by the caller; calls on different devices use different copies. The call
// is synchronous: it returns after its work on `stream` has finished. The control words are cleared at the start of
// every call; the planes need no clearing, because every byte a product reads is written first (rows past the data
// are only read into output columns the epilogue discards).
//
// Shares the digit-plane GEMM of digit_gemm.cuh with ktmoe_linear; the existing entry points are unchanged.

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "digit_gemm.cuh"
#include "fixed_point.cuh"
#include "ktmoe.h"

namespace {

// The scratch: [0, 256) control words (bad-code counter, kernel error word), then the planes of X, then of W.
constexpr size_t kScratchBytes = size_t(64) << 20;
constexpr size_t kControlBytes = 256;
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

// Every accepted shape has 3·k_pad·(rows_pad + out_pad) <= kScratchBytes with rows_pad >= 64 and out_pad >= 128, so
// k_pad stays below the longest K whose int32 diagonal sums cannot overflow (dg::K_EXACT_MAX): the K-chunk loop in
// ktmoe_linear_noalloc makes exactly one pass at this array size and would split K only if the array grew.
static_assert(kScratchBytes / (3 * (64 + 128)) < (size_t)dg::K_EXACT_MAX, "the scratch cap keeps K within one chunk");

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char* g_scratch_dev[kMaxDevices] = {};  // the array's device address, per device (null until set up)

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
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

inline int64_t up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// int32 codes [rows][K] -> three digit planes [3][R_pad][K_pad]; codes beyond ±WLEVELS are counted in *bad and
// stored as 0.
__global__ void pack_planes(const int32_t* __restrict__ codes, long long rows, int K, int K_pad, long long R_pad,
                            int8_t* __restrict__ planes, unsigned long long* __restrict__ bad) {
    const long long r = blockIdx.x;
    if (r >= rows) return;
    const int32_t* c = codes + r * K;
    int8_t* p0 = planes + r * K_pad;
    int8_t* p1 = p0 + R_pad * K_pad;
    int8_t* p2 = p1 + R_pad * K_pad;
    unsigned nbad = 0;
    for (int k = threadIdx.x; k < K_pad; k += blockDim.x) {
        int32_t v = k < K ? c[k] : 0;
        if (v > (int32_t)kt::WLEVELS || v < -(int32_t)kt::WLEVELS) {
            ++nbad;
            v = 0;
        }
        int8_t d0, d1, d2;
        kt::split_digits(v, d0, d1, d2);
        p0[k] = d0;
        p1[k] = d1;
        p2[k] = d2;
    }
    if (nbad) atomicAdd(bad, (unsigned long long)nbad);
}

int make_map(CUtensorMap* map, const void* base, int64_t k_pad, int64_t rows_total, int box_rows) {
    EncodeTiledFn enc = encoder();
    if (!enc) return KTMOE_ERR_CUDA;
    cuuint64_t gdim[2] = {(cuuint64_t)k_pad, (cuuint64_t)rows_total};
    cuuint64_t gstride[1] = {(cuuint64_t)k_pad};
    cuuint32_t box[2] = {(cuuint32_t)dg::BK, (cuuint32_t)box_rows};
    cuuint32_t estride[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), gdim, gstride, box, estride,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
               ? KTMOE_OK
               : KTMOE_ERR_CUDA;
}

template <int BN, int ST, int ACC>
cudaError_t launch(const CUtensorMap& ma, const CUtensorMap& mb, unsigned grid, const dg::GemmArgs& a, cudaStream_t st) {
    using C = dg::Cfg<BN, ST, ACC>;
    dg::digit_gemm_kernel<BN, ST, ACC><<<grid, dg::THREADS, C::SMEM_BYTES, st>>>(ma, mb, a);
    return cudaGetLastError();
}

template <int BN, int ST, int ACC>
cudaError_t prepare_gemm() {
    using C = dg::Cfg<BN, ST, ACC>;
    cudaFuncAttributes at;
    cudaError_t e = cudaFuncGetAttributes(&at, dg::digit_gemm_kernel<BN, ST, ACC>);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(dg::digit_gemm_kernel<BN, ST, ACC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                C::SMEM_BYTES);
}

// Set-up of one device (the current one), done by the first call there: the array's device address, and every kernel
// of this entry point loaded and configured now, so that no later call makes the driver load code (which takes device
// memory) or change a function attribute.
int setup_device(unsigned char** base) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || !p) return KTMOE_ERR_CUDA;
    cudaFuncAttributes at;
    if (cudaFuncGetAttributes(&at, pack_planes) != cudaSuccess) return KTMOE_ERR_CUDA;
    if (prepare_gemm<16, 4, 2>() != cudaSuccess || prepare_gemm<48, 3, 2>() != cudaSuccess) return KTMOE_ERR_CUDA;
    *base = (unsigned char*)p;
    return KTMOE_OK;
}

}  // namespace

extern "C" int ktmoe_linear_noalloc(int32_t device, const int32_t* x, const int32_t* w, int64_t rows, int64_t out,
                                    int64_t k, int64_t* y, void* stream) {
    if (device < 0 || device >= kMaxDevices || rows < 0 || out < 0 || k < 0) return KTMOE_ERR_ARG;
    if (rows == 0 || out == 0) return KTMOE_OK;
    if (!y || (k > 0 && (!x || !w))) return KTMOE_ERR_ARG;
    const int64_t k_pad = up(k, dg::BK), rows_pad = up(rows, 64), out_pad = up(out, dg::BM);
    const int64_t x_bytes = 3 * rows_pad * k_pad, w_bytes = 3 * out_pad * k_pad;
    if ((size_t)(kControlBytes + up(x_bytes, 256) + w_bytes) > kScratchBytes) return KTMOE_ERR_UNSUPPORTED;

    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) return KTMOE_ERR_CUDA;
    if (cudaSetDevice(device) != cudaSuccess) return KTMOE_ERR_NO_DEVICE;
    int status = KTMOE_OK;
    unsigned char* base = nullptr;
    cudaStream_t st = (cudaStream_t)stream;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_scratch_dev[device]) {
            // the set-up loads code onto the device, which a stream being captured would not record: a first call
            // under capture is refused (KTMOE_ERR_ARG) instead of failing part-way through
            cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
            unsigned char* p = nullptr;
            if (cudaStreamIsCapturing(st, &cs) != cudaSuccess)
                status = KTMOE_ERR_CUDA;
            else if (cs != cudaStreamCaptureStatusNone)
                status = KTMOE_ERR_ARG;
            else
                status = setup_device(&p);
            if (status == KTMOE_OK) g_scratch_dev[device] = p;
        }
        base = g_scratch_dev[device];
    }
    if (k == 0) {  // empty sums
        const bool ok = status == KTMOE_OK && cudaMemsetAsync(y, 0, (size_t)(rows * out) * 8, st) == cudaSuccess &&
                        cudaStreamSynchronize(st) == cudaSuccess;
        cudaSetDevice(prev);
        return status != KTMOE_OK ? status : ok ? KTMOE_OK : KTMOE_ERR_CUDA;
    }
    unsigned long long* bad = (unsigned long long*)base;
    int* err = (int*)(base + 64);
    int8_t* xp = (int8_t*)(base + kControlBytes);
    int8_t* wp = xp + up(x_bytes, 256);
    if (status == KTMOE_OK && cudaMemsetAsync(base, 0, kControlBytes, st) != cudaSuccess) status = KTMOE_ERR_CUDA;
    if (status == KTMOE_OK) {
        pack_planes<<<(unsigned)rows, 128, 0, st>>>(x, rows, (int)k, (int)k_pad, rows_pad, xp, bad);
        pack_planes<<<(unsigned)out, 128, 0, st>>>(w, out, (int)k, (int)k_pad, out_pad, wp, bad);
        if (cudaGetLastError() != cudaSuccess) status = KTMOE_ERR_CUDA;
    }
    // one weight group, one activation group; K is split into chunks whose int32 plane sums cannot overflow (one
    // chunk at this array size, see the static_assert above)
    const int BN = rows >= 40 ? 48 : 16;
    CUtensorMap ma, mb;
    if (status == KTMOE_OK) status = make_map(&ma, wp, k_pad, 3 * out_pad, dg::BM);
    if (status == KTMOE_OK) status = make_map(&mb, xp, k_pad, 3 * rows_pad, BN);
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    const int64_t n_tiles = (rows + BN - 1) / BN, group_n = std::min<int64_t>(16, n_tiles);
    const int64_t m_tiles = out_pad / dg::BM, n_groups = (n_tiles + group_n - 1) / group_n;
    const unsigned grid = (unsigned)std::min<int64_t>(m_tiles * group_n * n_groups, sms);
    const int64_t total_kb = (k + dg::BK - 1) / dg::BK, chunk_kb = dg::K_EXACT_MAX / dg::BK;
    for (int64_t kb0 = 0; status == KTMOE_OK && kb0 < total_kb; kb0 += chunk_kb) {
        dg::GemmArgs a{};
        a.out = y;
        a.ld_out = out;
        a.M_valid = (int)out;
        a.M_pad = (int)out_pad;
        a.k_block0 = (int)kb0;
        a.num_k_blocks = (int)std::min(chunk_kb, total_kb - kb0);
        a.R_pad = (int)rows_pad;
        a.n_tiles_max = (int)n_tiles;
        a.m_tiles = (int)m_tiles;
        a.group_n = (int)group_n;
        a.single_rows = (int)rows;
        a.accumulate = kb0 > 0 ? 1 : 0;
        a.err = err;
        a.rowmax_split = INT32_MAX;
        const cudaError_t e = BN == 48 ? launch<48, 3, 2>(ma, mb, grid, a, st) : launch<16, 4, 2>(ma, mb, grid, a, st);
        if (e != cudaSuccess) status = KTMOE_ERR_CUDA;
    }
    unsigned long long n_bad = 0;
    int kernel_err = 0;
    if (status == KTMOE_OK &&
        (cudaMemcpyAsync(&n_bad, bad, sizeof(n_bad), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
         cudaMemcpyAsync(&kernel_err, err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
         cudaStreamSynchronize(st) != cudaSuccess))
        status = KTMOE_ERR_CUDA;
    if (status == KTMOE_OK && kernel_err != 0) status = KTMOE_ERR_KERNEL;
    if (status == KTMOE_OK && n_bad != 0) status = KTMOE_ERR_RANGE;
    cudaSetDevice(prev);
    return status;
}
