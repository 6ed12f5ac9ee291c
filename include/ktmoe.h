/*
 * ktmoe — tritify's exact-integer Mixture-of-Experts FFN layer on NVIDIA B200 (sm_100a), behind a plain C ABI.
 *
 * Every entry point returns an int status (KTMOE_OK = 0) and never aborts; results come back through out-parameters.
 * Pointers are plain host pointers unless the name says "dev". No CUDA or torch type appears in a signature: streams
 * are passed as `void*` (a cudaStream_t, or NULL for the context's own stream).
 *
 * Reference interfaces replaced (paths within the tritify project):
 *   LinearBackend::linear / linear_weights   crates/01-engine/kt-core/src/backend.rs:46-59
 *   kt-cuda's C ABI (kt_cuda_*)              crates/02-runtime/kt-cuda/src/digit_gemm.cu:86-147, device.rs:9-38
 *   Module::forward_int of MoeMlp            crates/01-engine/kt-core/src/layers.rs:1061-1073
 *   MoeMlp::route                            layers.rs:826-862
 *   QuantLinear::from_weights / with_bias    layers.rs:225-257
 *   IntTensor::from_reals                    crates/01-engine/kt-core/src/tensor.rs:106-116
 *   SigmoidScore::new (coded bias)           crates/01-engine/kt-core/src/router.rs:37-51
 *   Scale {mant, shift}                      crates/00-kernels/kt-int/src/lib.rs:175-178
 */
#ifndef KTMOE_H
#define KTMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define KTMOE_OK 0
#define KTMOE_ERR_CUDA 1          /* a CUDA runtime/driver call failed (ktmoe_last_error has the message) */
#define KTMOE_ERR_ARG 2           /* an argument is invalid (null, negative, inconsistent shape) */
#define KTMOE_ERR_RANGE 3         /* a code lies outside +-WLEVELS (265720): the digit planes cannot hold it */
#define KTMOE_ERR_KERNEL 4        /* a kernel reported a bounded wait that expired (no result was produced) */
#define KTMOE_ERR_UNSUPPORTED 5   /* a configuration outside what this build implements */
#define KTMOE_ERR_NO_DEVICE 6     /* no sm_100 device, or the device index does not exist */
#define KTMOE_ERR_STATE 7         /* the layer is incomplete (a weight not set) */
#define KTMOE_ERR_CALLBACK 8      /* the caller's experts callback returned non-zero */

/* A non-negative fixed-point scale mant * 2^-shift (kt-int Scale; mant == 0 means exactly zero). */
typedef struct ktmoe_scale {
    int64_t mant;
    int32_t shift;
} ktmoe_scale;

typedef struct ktmoe_ctx ktmoe_ctx;     /* one device, its stream and resident-weight cache */
typedef struct ktmoe_layer ktmoe_layer; /* one MoE layer's resident weights and scratch */

/* Layer shape and knobs (MoeMlp: layers.rs:661-674; MoeArch wiring: crates/03-models/kt-model-moe/src/lib.rs:456-501). */
typedef struct ktmoe_layer_config {
    int32_t d_model;        /* dim: router in_features */
    int32_t n_experts;      /* E: router out_features (1..512) */
    int32_t d_ff;           /* routed expert hidden size */
    int32_t top_k;          /* 1..min(E, 16) */
    int32_t norm_topk_prob; /* 1: normalise over the top-k codes; 0: over all E (softmax) or 2^20 (sigmoid) */
    int32_t router_score;   /* 0: softmax (OLMoE, Mixtral, Qwen-MoE); 1: sigmoid with selection bias (GLM-4.5) */
    int32_t shared_d_ff;    /* hidden size of the unweighted shared expert, 0 for none */
} ktmoe_layer_config;

/* ── devices and contexts (kt_cuda_device_count / kt_cuda_device_info) ── */
int ktmoe_device_count(int* n);
int ktmoe_open(int device, ktmoe_ctx** out);
int ktmoe_close(ktmoe_ctx* ctx);
const char* ktmoe_error_string(int status);
/* The last error message recorded on this context (never NULL). */
const char* ktmoe_last_error(const ktmoe_ctx* ctx);
/* The context's CUDA stream (a cudaStream_t), for callers that order their own work with it. */
void* ktmoe_stream(ktmoe_ctx* ctx);

/* ── LinearBackend (backend.rs:46-59): Y[r,o] = sum_k x[r*k+i]*w[o*k+i], i64, x rows x k, w out x k ──
 * Host pointers; synchronous. Codes beyond +-WLEVELS return KTMOE_ERR_RANGE (the reference hands such calls to its
 * Portable CPU kernel, counted; this library has no CPU path). Any k >= 1 is exact: long k is split into chunks whose
 * int32 plane sums cannot overflow, added in int64. */
int ktmoe_linear(ktmoe_ctx* ctx, const int32_t* x, const int32_t* w, int64_t rows, int64_t out, int64_t k, int64_t* y);
/* The same, with the weights kept resident on the device under `weight_id` (WeightId, backend.rs:22-35). The codes
 * behind an id must never change. */
int ktmoe_linear_weights(ktmoe_ctx* ctx, uint64_t weight_id, const int32_t* x, const int32_t* w, int64_t rows,
                         int64_t out, int64_t k, int64_t* y);
/* Small codes: when every weight code lies within +-3280 and every activation code within +-127 (int8 activations,
 * 12-bit weights), the call runs on one raw activation plane and two weight digit planes (two int8 products per
 * code product instead of nine); otherwise on three planes each. Same result either way. KTMOE_SMALL=0 forces the
 * nine-plane kernel. */
/* Tracing: the device time in milliseconds of the last successful linear call's GEMM (CUDA events on the context's
 * stream around the GEMM launches, after the codes are packed) and the activation planes it used (1 or 3; 0 and
 * *ms = 0 when no call has completed). No counterpart in the reference. */
int ktmoe_linear_last_gemm(ktmoe_ctx* ctx, double* ms, int32_t* act_planes);
/* The same accumulate for callers that cannot let a library allocate device memory (a runtime that owns one fixed
 * pool, or runs under a budget where a hidden cudaMalloc/cudaFree would break its accounting). No counterpart in the
 * reference. x [rows][k], w [out][k] (int32 codes) and y [rows][out] (int64) are DEVICE buffers on `device`; the
 * call allocates nothing: its scratch is a 64 MiB file-scope device array that every GPU running this entry point
 * holds until exit; the first call on a device looks up its address and loads this entry point's kernels there
 * (make that first call before any stream capture; a first call on a capturing stream returns KTMOE_ERR_ARG).
 * Limit: 256 + 3*ceil64(rows)*ceil128(k) (rounded up to 256) + 3*ceil128(out)*ceil128(k) <= 64 MiB, else
 * KTMOE_ERR_UNSUPPORTED. Calls on one device share the array and keep the last call's contents; calls whose GPU work
 * overlaps on one device race, so serialise them. Synchronous: returns when the work on `stream` (NULL: the legacy
 * default stream) is done. */
int ktmoe_linear_noalloc(int32_t device, const int32_t* x, const int32_t* w, int64_t rows, int64_t out, int64_t k,
                         int64_t* y, void* stream);
/* Resident-weight budget in bytes (LRU eviction; a weight larger than the budget is used once and dropped). */
int ktmoe_set_weight_budget(ktmoe_ctx* ctx, uint64_t bytes);
int ktmoe_resident_bytes(ktmoe_ctx* ctx, uint64_t* bytes);

/* ── the MoE layer (MoeMlp) ── */
int ktmoe_layer_create(ktmoe_ctx* ctx, const ktmoe_layer_config* cfg, ktmoe_layer** out);
int ktmoe_layer_destroy(ktmoe_layer* layer);
/* ── expert parallelism over NCCL (NVLink / NVSwitch) ──
 * One process (or one context) per GPU. Rank r of `world` owns experts [r*E/world, (r+1)*E/world) and passes its own
 * token rows to ktmoe_forward / ktmoe_forward_dev (any count, 0 included); the result is bit-identical to one
 * ktmoe_forward over all ranks' rows concatenated in rank order. All ranks must call every forward together.
 * The unique id (128 bytes) is made by one rank with ktmoe_ep_unique_id and handed to the others out of band. */
int ktmoe_ep_unique_id(void* id, int64_t bytes);
int ktmoe_layer_create_ep(ktmoe_ctx* ctx, const ktmoe_layer_config* cfg, int32_t rank, int32_t world,
                          const void* nccl_id, ktmoe_layer** out);
/* The experts this layer holds: [*begin, *end). ktmoe_layer_set_expert takes global expert ids in that range. */
int ktmoe_layer_experts(const ktmoe_layer* layer, int32_t* begin, int32_t* end);
/* Peer-memory transport (all ranks call it together, with the same value; at most 8 ranks): afterwards every forward
 * passes at most max_tokens_per_rank rows on each rank, and the exchanges run as kernels that write into the other
 * GPUs' memory over NVLink (CUDA IPC mappings) instead of NCCL calls, with no host synchronisation in the forward.
 * Results are the same bytes. 0 returns to the NCCL exchange. Device memory per rank: the receive planes
 * (3 * world * max * top_k * d_model bytes) and the experts' scratch for that many rows. Replaces the reference's
 * forward_int_with_experts transport (crates/01-engine/kt-core/src/layers.rs:945-984) inside one node. */
int ktmoe_layer_set_ep_capacity(ktmoe_layer* layer, int64_t max_tokens_per_rank);

/* Router codes [E][d_model] (QuantLinear w_codes, row-major) and w_scale; bias_codes [E] + bias_scale from
 * QuantLinear::with_bias, or NULL for no bias. */
int ktmoe_layer_set_router(ktmoe_layer* layer, const int32_t* codes, ktmoe_scale w_scale, const int64_t* bias_codes,
                           ktmoe_scale bias_scale);
/* Sigmoid router only: the coded selection bias [E], round(bias * 2^20) (SigmoidScore::new). */
int ktmoe_layer_set_sigmoid_bias(ktmoe_layer* layer, const int64_t* bias_codes);
/* Expert e's SwiGLU: gate [d_ff][d_model], up [d_ff][d_model], down [d_model][d_ff] codes and scales. */
int ktmoe_layer_set_expert(ktmoe_layer* layer, int32_t e, const int32_t* gate, ktmoe_scale gate_scale,
                           const int32_t* up, ktmoe_scale up_scale, const int32_t* down, ktmoe_scale down_scale);
/* The shared expert (layers.rs:741-745): gate/up [shared_d_ff][d_model], down [d_model][shared_d_ff]. */
int ktmoe_layer_set_shared(ktmoe_layer* layer, const int32_t* gate, ktmoe_scale gate_scale, const int32_t* up,
                           ktmoe_scale up_scale, const int32_t* down, ktmoe_scale down_scale);
/* Extension, off by default: Qwen2-MoE's sigmoid-gated shared expert. The reference refuses this configuration
 * (crates/03-models/kt-model-moe/src/lib.rs:152-154, :276-288); this library defines it in the reference's terms:
 * `codes` [d_model] are shared_expert_gate's QuantLinear::from_weights codes (a [1][d_model] linear, layers.rs:225-244)
 * at `w_scale`; per token the gate's integer logit (QuantLinear::forward_int over the whole input) picks a code of
 * the sigmoid CodeLut (router.rs:37-51), the shared output row is multiplied by it and the tensor requantised
 * (requant_dyn at the tensor's max) before add. NULL codes turn the gate off. Needs a shared expert. */
int ktmoe_layer_set_shared_gate(ktmoe_layer* layer, const int32_t* codes, ktmoe_scale w_scale);
/* A stack of layers of one shape in one object (a decoder's MoE blocks, model.rs:175-186, attention excluded): the
 * layer holds n_layers weight slots that share its scratch, tables and expert-parallel exchange. Slot 0 keeps the
 * weights set so far; ktmoe_layer_select(layer, i) makes slot i the one that the setters write and the forwards read
 * (a host-side swap, no device work). Set the depth once, before the first forward. */
int ktmoe_layer_set_depth(ktmoe_layer* layer, int32_t n_layers);
int ktmoe_layer_select(ktmoe_layer* layer, int32_t slot);
/* Fill the selected slot on the device, for layers too large to quantise on the host: weights N(0, sigma) from the
 * portable stream `seed` (ktmoe_synth_normal_portable), in the order router [E][d], expert e's gate [f][d], up [f][d],
 * down [d][f] for every e, then the shared expert's gate, up, down and, with shared_gate, its gate [1][d]; this rank
 * draws only its own experts' ranges. Each matrix is quantised per tensor as QuantLinear::from_weights does it
 * (layers.rs:225-244): the same codes and scales as the host quantiser on the same f32 values. A sigmoid router also
 * gets its selection bias: E values of the stream seed + 2 at sigmoid_bias_sigma, coded round(b * 2^20). Synchronous. */
int ktmoe_layer_synth_weights(ktmoe_layer* layer, uint64_t seed, float sigma, float sigmoid_bias_sigma,
                              int32_t shared_gate);
/* Module::forward_int: x [rows][d_model] at x_scale -> y [rows][d_model] at *y_scale. Host buffers; synchronous. */
int ktmoe_forward(ktmoe_layer* layer, const int32_t* x, int64_t rows, ktmoe_scale x_scale, int32_t* y,
                  ktmoe_scale* y_scale);
/* The same, asynchronous: enqueues the upload of x (and x_scale), the forward and the download of y (and the scale
 * into *y_scale) and returns at once. Two calls can be in flight: the layer keeps two slots of device buffers, an
 * upload and a download stream, so one call's copies overlap the forward of the one before or after it (PCIe runs both
 * ways at once). A call waits only for the call two back, which used the same slot. x must stay unchanged and y and
 * *y_scale unread until ktmoe_forward_async_wait returns; give pinned host memory, or the copies stage through the
 * driver and overlap nothing. No counterpart in the reference (its CPU path has no copies). */
int ktmoe_forward_async(ktmoe_layer* layer, const int32_t* x, int64_t rows, ktmoe_scale x_scale, int32_t* y,
                        ktmoe_scale* y_scale);
/* Wait for every ktmoe_forward_async of the layer; the first error of any of them. */
int ktmoe_forward_async_wait(ktmoe_layer* layer);
/* The same on device buffers, ordered on `stream` (NULL: the context stream) and not synchronised: x_dev and y_dev
 * hold rows x d_model int32, x_scale_dev and y_scale_dev one ktmoe_scale each. Kernel errors surface on the next
 * ktmoe_sync. */
int ktmoe_forward_dev(ktmoe_layer* layer, const int32_t* x_dev, int64_t rows, const ktmoe_scale* x_scale_dev,
                      int32_t* y_dev, ktmoe_scale* y_scale_dev, void* stream);
/* Wait for the context's stream (and `stream` if not NULL); reports a kernel error word if one was raised. */
int ktmoe_sync(ktmoe_ctx* ctx, void* stream);
/* The FFN half of a decoder block with this layer as its FFN (crates/01-engine/kt-core/src/model.rs:175-181):
 * y = add(x, moe(rms_norm(x))), the RmsNorm of layers.rs:352-449 and the residual add of layers.rs:121-136, each
 * reduction over the whole tensor (over every rank's rows with expert parallelism). The norm's weight codes and
 * scale come from ktmoe_quantize_weights (RmsNorm::new quantises like QuantLinear::from_weights), eps as
 * ktmoe_scale_from_f64(eps). Host and device entry points as for the layer. */
int ktmoe_layer_set_norm(ktmoe_layer* layer, const int32_t* w_codes, ktmoe_scale w_scale, ktmoe_scale eps_scale);
int ktmoe_block_forward(ktmoe_layer* layer, const int32_t* x, int64_t rows, ktmoe_scale x_scale, int32_t* y,
                        ktmoe_scale* y_scale);
int ktmoe_block_forward_dev(ktmoe_layer* layer, const int32_t* x_dev, int64_t rows, const ktmoe_scale* x_scale_dev,
                            int32_t* y_dev, ktmoe_scale* y_scale_dev, void* stream);
/* Scale::from_f64 (crates/00-kernels/kt-int/src/lib.rs:215-222), for offline constants such as a norm's eps. */
int ktmoe_scale_from_f64(double x, ktmoe_scale* out);
/* MoeMlp::route for each row: experts [rows][top_k] (top-k order), ec [rows][top_k] codes, sumc [rows]. */
int ktmoe_route(ktmoe_layer* layer, const int32_t* x, int64_t rows, ktmoe_scale x_scale, int32_t* experts,
                int64_t* ec, int64_t* sumc);
/* MoeRoute::margin (layers.rs:816-820, computed at :844-848) of softmax routes, on the host: from each row's router
 * logits [rows][n_experts] (ktmoe_layer_debug_fetch 0 after ktmoe_route), their scales [rows] (fetch 1) and the
 * route's experts [rows][top_k], margins[r] = the strongest excluded expert's exp code over the weakest selected
 * one's, 0 when that is 0. A read-only diagnostic of how decisive each cut is; a sigmoid route's margin is 0. */
int ktmoe_route_margins(const int32_t* logits, int64_t rows, int32_t n_experts, const ktmoe_scale* scales,
                        const int32_t* experts, int32_t top_k, double* margins);
/* ── the expert-parallel seam: MoeMlp::forward_int_with_experts (layers.rs:945-984) with the experts elsewhere ──
 * A layer whose routed experts live on other hosts (MoeMlp::remote, layers.rs:694-712) routes, combines, merges and
 * adds its shared expert here, and gets the expert outputs through a callback; a worker holding experts computes
 * those outputs with ktmoe_layer_expert_forward. Both take host pointers, are synchronous and run on a single-rank
 * layer (world 1). The outputs cross hosts in the IntTensor wire format below (ktmoe_wire_encode/decode).
 *
 * The worker side: SwiGluMlp::forward_int (layers.rs:609-640) of expert ids[r·n_ids + j] on row r of x (rows x d,
 * every row at x_scale, as the reference hands each row over with the input's scale) into y [rows][n_ids][d] and
 * y_scale [rows][n_ids]. An id < 0 is an empty slot (zeros, zero scale); an id >= n_experts is KTMOE_ERR_ARG and an
 * expert never set KTMOE_ERR_STATE. The router and the shared expert are not needed. */
int ktmoe_layer_expert_forward(ktmoe_layer* layer, const int32_t* x, int64_t rows, ktmoe_scale x_scale,
                               const int32_t* ids, int32_t n_ids, int32_t* y, ktmoe_scale* y_scale);
/* The coordinator side's callback: for each row r, the outputs of experts ids[r·top_k + j] (the route's order) on
 * row r of x into y [rows][top_k][d] and y_scale [rows][top_k] (both zero-filled on entry). A row whose route is empty
 * (sumc <= 0, which the reference never hands to its callback) has ids -1 and its outputs are ignored. Return 0; any
 * other value ends the forward with KTMOE_ERR_CALLBACK. */
typedef int (*ktmoe_experts_fn)(void* user, int64_t rows, int32_t top_k, const int32_t* ids, const int32_t* x,
                                ktmoe_scale x_scale, int32_t* y, ktmoe_scale* y_scale);
/* The coordinator side: route x, call experts_fn once for all rows, then combine, merge the rows and add the shared
 * expert exactly as ktmoe_forward does: with experts_fn returning what the layer's own experts compute, y and y_scale
 * equal ktmoe_forward's (the reference's seam property, kt-core/src/tests.rs:156-181). The routed experts of this
 * layer need not be set. */
int ktmoe_layer_forward_with_experts(ktmoe_layer* layer, const int32_t* x, int64_t rows, ktmoe_scale x_scale,
                                     ktmoe_experts_fn experts_fn, void* user, int32_t* y, ktmoe_scale* y_scale);
/* Failure detection, checked without a fault: runs the expert-parallel peer-exchange kernel against two regions of
 * this GPU's own memory standing for two ranks, the second of which never takes part, so the kernel's bounded wait for
 * it expires (about 2 s) and the call returns KTMOE_ERR_KERNEL, as a forward whose peer stopped does. The context
 * stays usable afterwards. No counterpart in the reference (its CPU path has no waits). */
int ktmoe_check_wait_expiry(ktmoe_ctx* ctx);
/* Kernel launches of this library on the context since open (the device work is all this library's own kernels). */
int ktmoe_launch_count(ktmoe_ctx* ctx, uint64_t* n);

/* Per-stage timing with CUDA events on the forward's stream (tracing; off by default). With it on, every forward
 * records one event per stage boundary; ktmoe_layer_stage_times waits for them, returns the summed milliseconds per
 * stage over the timed forwards (stages: 0 quantise+route, 1 dispatch (permute; with expert parallelism also the
 * counts exchange and the sends), 2 exchange in (the wait for the rows other ranks send; empty on one GPU), 3 gate/up
 * GEMM, 4 SwiGLU, 5 down GEMM, 6 exchange out (expert outputs back to their home ranks; empty on one GPU),
 * 7 combine, 8 merge, 9 shared expert + add; n_stages >= 10) and forgets them. */
int ktmoe_layer_set_timing(ktmoe_layer* layer, int32_t enable);
/* CUDA graphs for the forward (off by default): with it on, the first forward with given buffers, row count and
 * stream runs normally and is then captured; later forwards with the same ones launch the graph (fewer launch
 * gaps at decode sizes). Applies on one rank and with the peer transport; the NCCL exchange and per-stage timing run
 * uncaptured. The layer's weights may change between calls (they are read in place); growing the scratch (more rows
 * than ever before) drops the graphs. No counterpart in the reference (its CPU path launches nothing). */
int ktmoe_layer_set_graphs(ktmoe_layer* layer, int32_t enable);
int ktmoe_layer_stage_times(ktmoe_layer* layer, double* ms, int32_t n_stages, int32_t* n_forwards);

/* Diagnostics: copy an internal buffer of the last forward or route (which = 0: router logits [rows][E] int32,
 * 1: their scales [rows], 2: per-token combine outputs [rows][d_model] int32, 3: their scales [rows]). */
int ktmoe_layer_debug_fetch(ktmoe_layer* layer, int32_t which, void* host, int64_t bytes);

/* ── host-side, offline preparation (f64, as the reference does it once on the host) ── */
int ktmoe_quantize_weights(const float* w, int64_t n, int32_t* codes, ktmoe_scale* scale);
/* Returns KTMOE_OK; *has_bias = 0 when the bias is all zero (the reference then keeps none). */
int ktmoe_quantize_bias(const float* b, int64_t n, int64_t* codes, ktmoe_scale* scale, int32_t* has_bias);
int ktmoe_code_sigmoid_bias(const float* b, int64_t n, int64_t* codes);
int ktmoe_from_reals(const float* v, int64_t n, int32_t* data, ktmoe_scale* scale);
/* The three code tables: kind 0 router exp, 1 SiLU, 2 sigmoid; codes has 65536 entries. */
int ktmoe_table(int32_t kind, int64_t* codes, ktmoe_scale* inv_step, int64_t* lo_index, ktmoe_scale* code_scale);
/* Synthetic inputs defined by this build: elements [offset, offset + n) of the N(0, sigma) stream `seed` (splitmix64
 * + Box-Muller in f64, cast to f32), and the reference's LCG uniform integers in [lo, hi]. */
int ktmoe_synth_normal(uint64_t seed, float sigma, uint64_t offset, int64_t n, float* out);
/* The portable normal stream (tritify_b200/csrc/synth.cuh): the same splitmix64 uniforms as ktmoe_synth_normal, the
 * Box-Muller deviate with this library's own logarithm and cosine from correctly rounded IEEE operations only, so the
 * host and the device give identical bits (libm's log and cos differ between them in the last place). The _dev form
 * writes device memory on the context's stream and returns when it is done. */
int ktmoe_synth_normal_portable(uint64_t seed, float sigma, uint64_t offset, int64_t n, float* out);
int ktmoe_synth_normal_portable_dev(ktmoe_ctx* ctx, uint64_t seed, float sigma, uint64_t offset, int64_t n,
                                    float* out_dev);
int ktmoe_lcg_uniform(uint64_t seed, int64_t lo, int64_t hi, int64_t n, int32_t* out);

/* ── wire format: IntTensor::to_bytes / IntTensor::from_bytes (kt-core/src/tensor.rs:51-100) ──
 * The reference's interchange form of an activation between workers, byte for byte, little-endian:
 *   u32 ndim | ndim x u64 shape | i64 scale.mant | i32 scale.shift | u64 ndata | ndata x i32 codes
 * Host-only (no device needed). ktmoe_wire_size gives the frame's bytes. ktmoe_wire_encode writes one frame into
 * out (cap bytes) and its length into *written. ktmoe_wire_decode reads the frame at the start of b (len bytes):
 * ndim, the shape (when shape is not NULL; shape_cap >= ndim), the scale, ndata and, when data is not NULL, the codes
 * (data_cap >= ndata); *consumed is the frame's length, so concatenated frames are read one after another. A buffer
 * shorter than its header declares, or a cap too small, is KTMOE_ERR_ARG (the reference panics on a short buffer). */
int ktmoe_wire_size(int32_t ndim, int64_t ndata, uint64_t* bytes);
int ktmoe_wire_encode(const int32_t* data, int64_t ndata, const int64_t* shape, int32_t ndim, ktmoe_scale scale,
                      uint8_t* out, uint64_t cap, uint64_t* written);
int ktmoe_wire_decode(const uint8_t* b, uint64_t len, int32_t* ndim, int64_t* shape, int32_t shape_cap,
                      ktmoe_scale* scale, int64_t* ndata, int32_t* data, int64_t data_cap, uint64_t* consumed);

#ifdef __cplusplus
}
#endif

#endif /* KTMOE_H */
