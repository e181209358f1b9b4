/*
 * inzg.h -- C ABI of the B200 (sm_100a) implementation of inferenZ's mixture-of-experts layer.
 *
 * Drop-in for the routed part of the reference's `moe_block` (src/model_fwd.c:992-1140): the F16 router with softmax
 * and top-k, the dispatch of tokens to experts, the gate|up -> SiLU*up -> down products over Q4L / Q8G expert blobs,
 * and the routing-weighted rank-order combine. The expert cache's blob pointers (ec_try_acquire / ec_acquire /
 * ec_release, src/expert_cache.h:55-71) are replaced by an HBM-resident pool filled once per layer from the
 * `blk.%d.experts` tensor (src/engine.c:336-400). Plain C types only; no CUDA or torch types in the signatures.
 *
 * Threading: one context per engine, called from the engine thread (the reference's control flow is
 * single-threaded, src/threadpool.c:221-247); not re-entrant. Host pointers are borrowed for the duration of a call;
 * weights are copied into the context. Errors are status codes (the reference exits through inz_die,
 * src/util.c:22-30; a host shim maps a non-OK status onto it).
 */
#ifndef INZG_H
#define INZG_H

#if defined(__GNUC__)
#define INZG_EXPORT __attribute__((visibility("default")))
#else
#define INZG_EXPORT
#endif

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* tensor type ids, as in the reference's GGUF (src/quant.h:25-37) */
#define INZG_T_F16 1
#define INZG_T_Q4L 102
#define INZG_T_Q8G 103

typedef enum {
    INZG_OK = 0,
    INZG_BAD_ARG = 1,        /* a size, pointer or layer index out of range */
    INZG_CORRUPT_BLOB = 2,   /* bad INZQ magic or rows/cols mismatch, as src/model_fwd.c:854-855 / 958-960 */
    INZG_OOM = 3,            /* device allocation failed */
    INZG_CUDA = 4,           /* a CUDA call failed; inzg_last_error has the text */
    INZG_NCCL = 5,           /* a collective failed (expert-parallel mode) */
    INZG_TIMEOUT = 6,        /* a bounded device-side wait ran out */
    INZG_DEVICE_CHECK = 7,   /* a kernel's own bounds check fired (expert id, slot, capacity) */
    INZG_UNSUPPORTED = 8,    /* a shape or format this build does not implement */
    INZG_NOT_READY = 9       /* layer has no router or no experts yet */
} inzg_status;

typedef struct inzg_ctx inzg_ctx;

typedef struct {
    int hidden;       /* H: 2048 (benchmark configurations) or 2560 (the reference model, src/model.h:11) */
    int ff;           /* expert FFN width, 640 (src/model.h:53) */
    int n_expert;     /* 512 (src/model.h:51) */
    int topk;         /* 10 (src/model.h:52) */
    int max_tokens;   /* largest n of one forward call (the reference's Q_MAX_T is 512, src/engine_internal.h:82) */
    int n_layers;     /* layer slots: 49 = 48 layers + the MTP layer (src/model_fwd.c:1435) */
    int device;       /* CUDA device ordinal */
} inzg_config;

#define INZG_IO_DEVICE 1u   /* xin, y, logit_bias and logits_override are device pointers (xin, y, logits_override
                             * 16-byte aligned, else INZG_BAD_ARG); the call is stream-ordered */
#define INZG_DUMP_ROUTE 2u  /* keep the routing products of this call for inzg_moe_route_dump */
#define INZG_PROFILE 4u     /* time every stage with CUDA events on the call's stream; the call then synchronises */
#define INZG_NO_GRAPH 8u    /* launch the kernels one by one instead of replaying the cached CUDA graph */
#define INZG_GEMM_SIMT 16u  /* prefill-path experts on the CUDA-core int8 GEMM instead of tcgen05 (cross-check) */
#define INZG_NO_FUSED 32u   /* calls of 1-2 tokens through the separate kernels instead of the single fused decode
                             * launch (cross-check; both give the same bits) */

/* stages timed under INZG_PROFILE (the reference's diag stages are coarser: DG_ROUTER, DG_EXPERT_*, DG_SHARED) */
#define INZG_N_STAGES 12

typedef struct {
    unsigned flags;
    const float *logit_bias;       /* optional [n_expert], added to the router logits before the softmax (test hook,
                                      no counterpart in the reference) */
    const float *logits_override;  /* optional [n][n_expert], replaces the router logits (test hook) */
    void *stream;                  /* cudaStream_t to run on; NULL = the context's own (non-blocking) stream, so
                                      pass cudaStreamLegacy to order a call on CUDA's legacy default stream */
} inzg_moe_opts;

typedef struct {
    uint64_t calls, tokens;
    uint64_t units, dec_units, gemm_units;   /* of the last call with INZG_DUMP_ROUTE */
    uint64_t pool_bytes;
    int last_launches;                       /* kernels launched by the last forward call */
} inzg_stats;

/* Context on one device; replaces the engine's expert-cache set-up (src/engine.c:336-400 -> ec_open). */
INZG_EXPORT inzg_ctx *inzg_create(const inzg_config *cfg, inzg_status *status);
INZG_EXPORT void inzg_destroy(inzg_ctx *ctx);
INZG_EXPORT const char *inzg_last_error(const inzg_ctx *ctx);
INZG_EXPORT const char *inzg_status_str(inzg_status st);

/* Router of one layer: F16 [rows = n_expert][cols = hidden], as bound by q_bind_lin (src/model_fwd.c:87-96) and
 * multiplied by inz_matvec_f16_rows / inz_matmul_f16_rows (src/quant.c:1290-1366). Copied and re-laid out. */
INZG_EXPORT inzg_status inzg_set_router(inzg_ctx *ctx, int layer, const uint16_t *w_f16, int rows, int cols);

/* Experts of one layer: the GGUF tensor `blk.%d.experts` (n_expert blobs of blob_bytes, gate|up then down,
 * src/convert.c:565-584), replacing ec_preload of the layer (src/engine.c:389-397) and the per-expert
 * q_bind_lin views (src/model_fwd.c:853-855, 958-960). Blobs are validated (magic, type, rows, cols), copied to HBM
 * and re-laid out for the kernels. */
INZG_EXPORT inzg_status inzg_pool_add_layer(inzg_ctx *ctx, int layer, int expert_type, const void *blobs, uint64_t blob_bytes,
                                int n_expert);

/* ---- Experts straight from the engine's GGUF model file: the lookups of setup_experts (src/engine.c:336-351) over
 * the file as the reference's gguf_open reads it (src/gguf.c:80-160: GGUF v2/v3, data at the header's end rounded
 * up to "general.alignment", a tensor's size = distance to the next tensor's offset). Host code; the file stays
 * mapped read-only until inzg_gguf_close. */
typedef struct inzg_gguf inzg_gguf;
typedef struct {
    int expert_type;       /* "inz.expert_type"; absent: INZG_T_Q8G, the engine's default (src/engine.c:338) */
    uint64_t blob_bytes;   /* "inz.expert_blob_bytes" (0 when absent) */
    int n_layers;          /* "blk.%d.experts" present for layers 0 .. n_layers-1 */
    int has_mtp;           /* "mtp.experts" present: the engine numbers it layer n_layers (src/engine.c:343-348) */
    uint64_t alignment;    /* "general.alignment" (32 when absent) */
    uint64_t data_offset;  /* file offset of the tensor data section */
} inzg_gguf_info;

/* Opens and parses `path`; NULL on failure with the reason in err (err_len bytes, may be NULL). info: optional. */
INZG_EXPORT inzg_gguf *inzg_gguf_open(const char *path, inzg_gguf_info *info, char *err, size_t err_len);
INZG_EXPORT inzg_status inzg_gguf_get_info(const inzg_gguf *g, inzg_gguf_info *info);
/* Layer `layer`'s expert tensor (layer == n_layers: "mtp.experts"): *data points into the mapping, *nbytes is its size
 * (padding to the next tensor included), *file_offset its absolute offset; each output optional. INZG_BAD_ARG when
 * the file has no such tensor. */
INZG_EXPORT inzg_status inzg_gguf_experts(const inzg_gguf *g, int layer, const void **data, uint64_t *nbytes,
                                          uint64_t *file_offset);
/* Pool slot `layer` of ctx from the file's layer `gguf_layer`, with setup_experts' checks (blob size a positive
 * multiple of 4096 and the tensor at least n_expert blobs long, src/engine.c:340-350; INZG_CORRUPT_BLOB otherwise),
 * then inzg_pool_add_layer on the mapped blobs of the file's expert type. */
INZG_EXPORT inzg_status inzg_pool_add_layer_gguf(inzg_ctx *ctx, int layer, const inzg_gguf *g, int gguf_layer);
INZG_EXPORT void inzg_gguf_close(inzg_gguf *g);

/* The layer's shared expert (src/model_fwd.c:1041-1069, 1141-1148; the engine's `sh.gate_up`, `sh.down` and
 * `sh.gate` tensors, src/engine.c:175-177): blob holds the gate|up matrix (2*ff x hidden) followed by the down matrix
 * (hidden x ff) at inzg_qmat_bytes(type, 2*ff, hidden) -- the layout of one expert blob; gate [hidden] fp32. Once
 * set, inzg_moe_forward adds y += sigmoid(gate . x) * down(silu(gate_up x) * up x) per token after the routed sum,
 * with the reference's numerics (lin_mm's path rule: decode numerics below 12 tokens, GEMM numerics otherwise). */
INZG_EXPORT inzg_status inzg_set_shared(inzg_ctx *ctx, int layer, int expert_type, const void *blob, uint64_t blob_bytes,
                                        const float *gate);

/* The MoE layer: y[n][hidden] = sum over the top-k experts of w_k * down(silu(gate x) * up x), in rank order,
 * OVERWRITING y (src/model_fwd.c:1033, 1134-1140), plus the shared expert when one is set (inzg_set_shared). xin [n][hidden] fp32. Same per-expert numeric path as the
 * reference: experts with fewer than 12 tokens (or every expert when n <= 8) use the decode numerics
 * (src/quant.c:611-671, 767-953), the others the prefill GEMM numerics (src/quant.c:1407-1668). */
INZG_EXPORT inzg_status inzg_moe_forward(inzg_ctx *ctx, int layer, int n, const float *xin, float *y, const inzg_moe_opts *opt);

/* Routing products of the last forward call made with INZG_DUMP_ROUTE (host pointers, each optional):
 * sel [n][topk], w [n][topk] (renormalised), logits [n][n_expert] (after the test hook), probs [n][n_expert],
 * unit_expert [n_units] in the reference's first-touch order (src/model_fwd.c:1020-1022), *n_units. */
INZG_EXPORT inzg_status inzg_moe_route_dump(inzg_ctx *ctx, int n, int32_t *sel, float *w, float *logits, float *probs,
                                int32_t *unit_expert, int *n_units);

INZG_EXPORT inzg_status inzg_get_stats(const inzg_ctx *ctx, inzg_stats *out);

/* Per-stage device time (ms, summed over the calls made with INZG_PROFILE) and the number of such calls; reset != 0
 * clears them after reading. Stage i is named by inzg_stage_name(i), i < INZG_N_STAGES. The per-stage counterpart of
 * the reference's diag_add accounting (src/diag.c:67-83). */
INZG_EXPORT inzg_status inzg_stage_times(inzg_ctx *ctx, double *ms, uint64_t *calls, int reset);
INZG_EXPORT const char *inzg_stage_name(int stage);

/* Allocation-free routing: no counterpart in the reference. For callers that cannot allocate device memory on the
 * call path -- an engine whose device-memory plan is fixed at start-up, or a latency-critical decode loop in which a
 * cudaMalloc/cudaFree would synchronise the device -- this runs the router, softmax and top-k of one layer (the
 * routing stage of inzg_moe_forward, same results bit for bit) with its intermediate logits in a static device array
 * of the library instead of allocated scratch. x_dev [n][hidden] (16-byte aligned), logit_bias_dev [n_expert]
 * (optional), sel_dev [n][topk] and w_dev [n][topk] are device pointers; the call is ordered on `stream` (NULL = the
 * context's stream, as for inzg_route) and returns without synchronising; the caller's current device is left as it
 * was. Limits: n <= 64 and n_expert <= 512 (the array is 64 x 512 fp32 = 128 KiB, held by every GPU that loads the
 * library until exit); larger calls return INZG_BAD_ARG. The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) and should come before any stream capture. All calls share the array: calls that
 * overlap on the GPU race. A device-side wait that runs out leaves sel = -1 and w = NaN in every output slot and
 * makes inzg_device_status report INZG_TIMEOUT. */
INZG_EXPORT inzg_status inzg_route_topk_noalloc(inzg_ctx *ctx, int layer, int n, const float *x_dev,
                                                const float *logit_bias_dev, int32_t *sel_dev, float *w_dev,
                                                void *stream);

/* ---- Expert parallelism (no counterpart in the reference, which runs on one host). A rank owns experts
 * [e_first, e_first + n_local) of a layer and its share of the batch's tokens. Per layer: inzg_route on the rank's
 * tokens; ship every token row to the ranks owning its selected experts (NCCL all-to-all in the caller);
 * inzg_moe_experts on the rows received; ship the per-slot outputs back; inzg_combine. Each expert sees the same
 * tokens as in a single-GPU call, so its numeric path and outputs are the single-GPU ones bit for bit. All pointers
 * are device pointers (16-byte aligned where rows are copied); calls are ordered on `stream` (NULL = the context's
 * stream) and return without synchronising; inzg_device_status synchronises and reports device-side checks. */

/* Experts [e_first, e_first + n_local) of the layer: blobs holds those n_local blobs in order. inzg_pool_add_layer
 * is the whole range (0, n_expert); inzg_moe_forward needs the whole range. */
INZG_EXPORT inzg_status inzg_pool_add_layer_range(inzg_ctx *ctx, int layer, int expert_type, const void *blobs,
                                                  uint64_t blob_bytes, int e_first, int n_local);

/* The same from blobs already in this context's device memory (e.g. encoded there by inzg_synth_layer_blobs_device):
 * the headers are checked after a small copy to the host, the blobs re-laid out on the device without a host trip. */
INZG_EXPORT inzg_status inzg_pool_add_layer_device(inzg_ctx *ctx, int layer, int expert_type, const void *blobs_dev,
                                                   uint64_t blob_bytes, int e_first, int n_local);

/* Router, softmax and top-k of n tokens (the routing stage of inzg_moe_forward): sel_dev [n][topk] (expert ids),
 * w_dev [n][topk] (renormalised weights). logit_bias_dev: the test hook, optional. */
INZG_EXPORT inzg_status inzg_route(inzg_ctx *ctx, int layer, int n, const float *x_dev, const float *logit_bias_dev,
                                   int32_t *sel_dev, float *w_dev, void *stream);

/* The experts this rank owns, on m received token rows x_dev [m][hidden]: sel_dev [m][topk] holds, per row and rank
 * k, the LOCAL expert index (global id - e_first) or -1 when that expert lives on another rank; w_dev [m][topk] the
 * routing weights. n_batch is the whole batch's token count across ranks (the reference decodes every expert when
 * it is <= 8). Writes out_dev[r][k][hidden] = w * expert(x_r) for the entries present; other slots are untouched. */
INZG_EXPORT inzg_status inzg_moe_experts(inzg_ctx *ctx, int layer, int m, const float *x_dev, const int32_t *sel_dev,
                                         const float *w_dev, int n_batch, float *out_dev, void *stream);

/* y_dev[t] = ((0 + s[t][0]) + s[t][1]) + ... + s[t][topk-1] for slots_dev [n][topk][hidden] (src/model_fwd.c:1134-1140). */
INZG_EXPORT inzg_status inzg_combine(inzg_ctx *ctx, int n, const float *slots_dev, float *y_dev, void *stream);

/* The shared expert of `layer` on this rank's n tokens: y_dev[t] += sigmoid(gate . x_t) * shared(x_t), after the
 * rank's inzg_combine (the reference adds it after the routed sum). n_batch: the whole batch's token count, which picks
 * the numeric path as in a single-GPU call. */
INZG_EXPORT inzg_status inzg_shared_expert(inzg_ctx *ctx, int layer, int n, const float *x_dev, float *y_dev,
                                           int n_batch, void *stream);

/* ---- Hyper-connections around the layer: the steps either side of moe_block in q_forward (src/model_fwd.c:1264-1267).
 * The residual X [n][4*hidden] holds four streams of `hidden` floats per token. */
#define INZG_HC_RANK 320  /* Q_HC_RANK, src/model.h:14 */

/* The hyper-connection weights of `layer` (the reference's hcw L->mhc, src/engine_internal.h:27-32, bound by
 * src/engine.c:152-153): norm [4*hidden] fp32 (1 + w, folded), down [320][4*hidden] and up [4*hidden][320] as fp16
 * bits (the converter's hc type, src/convert.c:148, 251-252), inject [4][4*hidden] fp32 or NULL (the final mixer has
 * none). Host pointers, copied to the device. */
INZG_EXPORT inzg_status inzg_set_hc(inzg_ctx *ctx, int layer, const float *norm, const uint16_t *down_f16,
                                    const uint16_t *up_f16, const float *inject);

/* hc_in (src/model_fwd.c:432-439), which makes the layer's input: X_dev [n][4*hidden] -> xin_dev [n][hidden] and
 * inj_dev [n][4] (NULL: not computed; INZG_BAD_ARG when the layer was set without inject vectors). Device pointers, 16-byte aligned; stream NULL = the context's stream. The
 * first call with more tokens than before allocates the step's scratch (call it once at full size before any stream
 * capture). Bit-exact with the reference except the SiLU of the 320-wide bottleneck and the inject sigmoid, whose
 * glibc expf is evaluated in double and rounded once (one ulp apart on ~1e-4 of inputs). */
INZG_EXPORT inzg_status inzg_hc_in(inzg_ctx *ctx, int layer, int n, const float *X_dev, float *xin_dev, float *inj_dev,
                                   void *stream);

/* hc_out (src/model_fwd.c:442-450), which consumes the layer's output: X[t][s][:] += inj[t][s] * y[t][:] for the four
 * streams s, one fma per element as in the reference build. Device pointers (X_dev and y_dev 16-byte aligned). */
INZG_EXPORT inzg_status inzg_hc_out(inzg_ctx *ctx, int n, float *X_dev, const float *inj_dev, const float *y_dev,
                                    void *stream);

/* q_forward's MoE step for one layer (src/model_fwd.c:1264-1267) on the device: hc_in with the layer's weights,
 * inzg_moe_forward (INZG_IO_DEVICE implied; INZG_DUMP_ROUTE and INZG_PROFILE refused), hc_out; X_dev [n][4*hidden]
 * is updated in place. */
INZG_EXPORT inzg_status inzg_moe_block_hc(inzg_ctx *ctx, int layer, int n, float *X_dev, const inzg_moe_opts *opt);

/* Waits for `stream` and reports the device-side checks of the calls since the last routing step
 * (INZG_TIMEOUT / INZG_DEVICE_CHECK), including a timed-out expert-parallel exchange. */
INZG_EXPORT inzg_status inzg_device_status(inzg_ctx *ctx, void *stream);

/* ---- Expert parallelism with the exchange in the library: peer memory over NVLink / NVSwitch, no collective library.
 * One context per GPU (one rank per GPU: a connect that finds two ranks on one device fails), rank r of `world`
 * (<= 8) holding experts [r * n_expert / world, (r + 1) * n_expert / world) of every layer it runs
 * (inzg_pool_add_layer_range) and the router. Each rank exposes one device buffer to the others; a step ships every
 * (token, owning rank) row once and every owned output slot once, directly into the peer's memory, with device-side
 * epoch flags instead of host synchronisation, and ends with the rank-order combine -- the single-GPU bits.
 *
 * Between processes: inzg_ep_attach on every rank, exchange the INZG_EP_HANDLE_BYTES handles (any host channel),
 * inzg_ep_connect with all of them in rank order. In one process: inzg_ep_attach on every context, then
 * inzg_ep_connect_local with the contexts in rank order (peer access is enabled between their devices).
 * `capacity`: the most tokens a rank passes to one inzg_ep_forward; the context's max_tokens must be at least
 * world * capacity (the rows a rank can receive). */
#define INZG_EP_HANDLE_BYTES 128
INZG_EXPORT inzg_status inzg_ep_attach(inzg_ctx *ctx, int rank, int world, int capacity, void *handle_out);
INZG_EXPORT inzg_status inzg_ep_connect(inzg_ctx *ctx, const void *handles);
INZG_EXPORT inzg_status inzg_ep_connect_local(inzg_ctx *const *ctxs, int world);

/* One expert-parallel MoE layer on this rank's n <= capacity tokens x_dev [n][hidden] -> y_dev [n][hidden] (device
 * pointers, 16-byte aligned): route, dispatch, the owned experts, return, combine, and the layer's shared expert if
 * set. Every rank calls it for the same layers in the same order (n may differ per rank, n_batch is the sum). Ordered
 * on `stream` (NULL = the context's stream), captured in a CUDA graph per (layer, n, pointers); returns without
 * synchronising. A peer that never arrives makes the step's waits run out after about a second: the outputs are then
 * incomplete and inzg_device_status reports INZG_TIMEOUT. */
INZG_EXPORT inzg_status inzg_ep_forward(inzg_ctx *ctx, int layer, int n, const float *x_dev, const float *logit_bias_dev,
                                        float *y_dev, int n_batch, void *stream);

/* Device-side rendezvous of all ranks on `stream`, outside any step (every rank calls it the same number of times):
 * the stream continues once every rank's stream has reached its own call. For timing steps from a common start; a peer
 * that never arrives makes it give up after about a second (INZG_TIMEOUT at inzg_device_status). */
INZG_EXPORT inzg_status inzg_ep_barrier(inzg_ctx *ctx, void *stream);

/* Leaves the exchange (after every rank's last inzg_ep_forward has completed): closes the peers' mappings and frees
 * this rank's buffer. inzg_destroy does it too. */
INZG_EXPORT inzg_status inzg_ep_detach(inzg_ctx *ctx);

#ifdef __cplusplus
}
#endif
#endif
