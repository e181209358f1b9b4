/*
 * ref_harness.c -- TEST INFRASTRUCTURE ONLY (the "_ref" leg of the oracle).
 *
 * This file is compiled together with the reference engine's own MoE sources, read where they lie in the
 * reference tree (src/model_fwd.c, src/quant.c, src/sampler.c, src/threadpool.c, src/util.c, src/diag.c,
 * src/json.c), by oracle/Makefile into oracle/_ref/libinzref_*.so. Nothing of the reference is copied here: the
 * reference's model_fwd.c is #included from the reference tree with the hidden size and the per-call token cap
 * overridden through its include guards (model.h:4-5 guards Q_H, engine_internal.h guards Q_MAX_T).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm load the resulting library,
 * and only as the checker or as the timed reference CPU path -- never as part of the product.
 *
 * What it exposes:
 *   ref_quantize / ref_encode_expert  -- the reference quantizer (src/quant.c:422-556) with the converter's
 *                                        recipe for expert matrices (src/convert.c:190-200)
 *   ref_moe_routed                    -- the routed part of moe_block (src/model_fwd.c:992-1140) restated as a
 *                                        driver around the reference's own static functions (lin_mm,
 *                                        softmax_inplace, topk_f32, experts_batch, expert_compute), with all
 *                                        experts resident in RAM and a test-only router bias / logit override
 *                                        between the router and the softmax (no such hook exists in the
 *                                        reference; it is needed for the skewed-routing configurations).
 *   ref_shared                        -- the shared expert of moe_block (src/model_fwd.c:1041-1069 without the
 *                                        lookahead, and :1141-1148) around the reference's lin_mm, siluf,
 *                                        sigmoidf and dot_f32.
 *   ref_hc_in / ref_hc_out            -- the hyper-connection steps either side of the layer (src/model_fwd.c:
 *                                        404-450), the reference's own functions.
 */
#include "model.h"
#undef Q_H
#define Q_H REF_Q_H
#include "engine_internal.h"
#undef Q_MAX_T
#define Q_MAX_T REF_MAX_T
#include "model_fwd.c"

#include <pthread.h>
#include <sched.h>

#define API __attribute__((visibility("default")))

/* ---- expert cache stubs: every expert resident (the engine's all-resident mode, src/engine.c:370-399) ---- */
uint64_t ec_read_bytes(const ec_cache *c) { (void)c; return 0; }
int ec_resident_level(const ec_cache *c, int layer, int expert) { (void)c; (void)layer; (void)expert; return 1; }
void ec_request(ec_cache *c, int layer, int expert, float weight, int level) { (void)c; (void)layer; (void)expert; (void)weight; (void)level; }
bool ec_prefetch(ec_cache *c, int layer, int expert, float weight, int level) { (void)c; (void)layer; (void)expert; (void)weight; (void)level; return true; }
const uint8_t *ec_try_acquire(ec_cache *c, int layer, int expert, float weight, int min_level, int *level_out) {
    (void)c; (void)layer; (void)expert; (void)weight; (void)min_level; *level_out = 1; return NULL;
}
const uint8_t *ec_acquire(ec_cache *c, int layer, int expert, float weight, int level, int *level_out) {
    (void)c; (void)layer; (void)expert; (void)weight; (void)level; *level_out = 1; return NULL;
}
void ec_release(ec_cache *c, int layer, int expert) { (void)c; (void)layer; (void)expert; }
bool ec_wait_any(ec_cache *c) { (void)c; return false; }

/* ---- context: the scratch the MoE path of the engine uses (subset of q_scratch_alloc, model_fwd.c:1157-1200) ---- */
typedef struct {
    inz_engine *e;
    float *logits;
    int max_tokens;
    cpu_set_t caller_cpus;   /* tp_create pins the calling thread to its first CPU (src/threadpool.c:200); the
                                caller's mask is restored by ref_ctx_destroy */
    int have_cpus;
} ref_ctx;

API int ref_hidden(void) { return Q_H; }
API int ref_max_tokens(void) { return Q_MAX_T; }
API int ref_ff(void) { return Q_FF; }
API int ref_n_expert(void) { return Q_N_EXPERT; }
API int ref_topk_k(void) { return Q_TOPK; }
API int ref_gemm_min_t(void) { return GEMM_MIN_T; }
API const char *ref_isa(void) { return inz_kernel_isa(); }

API void *ref_ctx_create(int threads, int expert_type) {
    ref_ctx *c = calloc(1, sizeof(*c));
    inz_engine *e = calloc(1, sizeof(*e));
    c->e = e;
    c->max_tokens = Q_MAX_T;
    c->have_cpus = pthread_getaffinity_np(pthread_self(), sizeof(c->caller_cpus), &c->caller_cpus) == 0;
    e->tp = tp_create(threads, NULL);
    const size_t T = Q_MAX_T;
    const int nthr = tp_size(e->tp);
    e->expert_type = expert_type;
    e->gu_bytes = inz_mat_bytes(expert_type, 2 * Q_FF, Q_H);
    e->ex_x = inz_aligned(64, sizeof(float) * T * Q_H);
    e->ex_gu = inz_aligned(64, sizeof(float) * T * 2 * Q_FF);
    e->ex_d = inz_aligned(64, sizeof(float) * T * Q_H);
    e->moe_out = inz_aligned(64, sizeof(float) * T * Q_TOPK * Q_H);
    e->eb_items = inz_calloc(EB_MAX, sizeof(ebatch_item));
    e->eb_gu = inz_aligned(64, sizeof(float) * EB_MAX * 2 * Q_FF);
    e->eb_d = inz_aligned(64, sizeof(float) * EB_MAX * Q_H);
    e->eb_acts = inz_calloc(EB_MAX, sizeof(inz_act));
    for (int i = 0; i < EB_MAX; i++) inz_act_alloc(&e->eb_acts[i], Q_FF);
    e->eb_xa = inz_calloc(8, sizeof(inz_act));
    for (int i = 0; i < 8; i++) inz_act_alloc(&e->eb_xa[i], Q_H);
    e->units = inz_calloc(Q_N_EXPERT, sizeof(unit));
    e->acts = inz_calloc(GEMM_MIN_T, sizeof(inz_act));     /* decode numerics: at most GEMM_MIN_T-1 tokens */
    for (int i = 0; i < GEMM_MIN_T; i++) inz_act_alloc(&e->acts[i], Q_H);
    e->gemm_tb = inz_calloc((size_t)nthr, sizeof(uint8_t *));
    e->gemm_tmp = inz_calloc((size_t)nthr, sizeof(float *));
    for (int i = 0; i < nthr; i++) {
        e->gemm_tb[i] = inz_aligned(64, inz_gemm_tilebuf_bytes(Q_H));
        e->gemm_tmp[i] = inz_aligned(64, sizeof(float) * Q_H + 64);
    }
    inz_xq_alloc(&e->gemm_x, Q_MAX_T, Q_H);
    c->logits = inz_aligned(64, sizeof(float) * T * Q_N_EXPERT);
    return c;
}

API int ref_tp_size(void *ctx) { return tp_size(((ref_ctx *)ctx)->e->tp); }

API void ref_ctx_destroy(void *ctx) {
    ref_ctx *c = ctx;
    if (!c) return;
    inz_engine *e = c->e;
    const int nthr = tp_size(e->tp);
    free(e->ex_x); free(e->ex_gu); free(e->ex_d); free(e->moe_out);
    for (int i = 0; i < EB_MAX; i++) inz_act_free(&e->eb_acts[i]);
    for (int i = 0; i < 8; i++) inz_act_free(&e->eb_xa[i]);
    free(e->eb_items); free(e->eb_gu); free(e->eb_d); free(e->eb_acts); free(e->eb_xa);
    free(e->units);
    for (int i = 0; i < GEMM_MIN_T; i++) inz_act_free(&e->acts[i]);
    free(e->acts);
    for (int i = 0; i < nthr; i++) { free(e->gemm_tb[i]); free(e->gemm_tmp[i]); }
    free(e->gemm_tb); free(e->gemm_tmp);
    inz_xq_free(&e->gemm_x);
    tp_destroy(e->tp);
    free(e);
    free(c->logits);
    if (c->have_cpus) pthread_setaffinity_np(pthread_self(), sizeof(c->caller_cpus), &c->caller_cpus);
    free(c);
}

/* ---- quantizer ---- */
API size_t ref_qmat_bytes(int type, int rows, int cols) { return inz_qmat_bytes(type, rows, cols); }

API double ref_quantize(const float *W, int rows, int cols, int type, int rot_block, uint32_t seed, int threads, void *out) {
    inz_quant_params p = {.type = type, .rot_block = rot_block, .rot_seed = seed, .threads = threads};
    return inz_quantize(W, rows, cols, &p, out);
}

/* One expert blob as the converter writes it (src/convert.c:179-200, 565-584): gate|up rows (2*FF x H) then down
 * (H x FF) at offset mat_bytes(type, 2FF, H), the blob padded to 4 KiB. No importance matrix (all-ones == NULL,
 * src/quant.c:449-456). rot8: Q8G rotated with the automatic block, as the converter's default. */
API uint64_t ref_blob_bytes(int type) {
    uint64_t b = inz_mat_bytes(type, 2 * Q_FF, Q_H) + inz_mat_bytes(type, Q_H, Q_FF);
    return INZ_ALIGN_UP(b, 4096);
}

API void ref_encode_expert(const float *GU, const float *D, int type, int rot8, void *blob) {
    memset(blob, 0, ref_blob_bytes(type));
    inz_quant_params p = {.type = type, .threads = 1};
    p.rot_block = type == INZ_T_Q8G ? (rot8 ? inz_auto_rot_block(Q_H) : -1) : 0;
    inz_quantize(GU, 2 * Q_FF, Q_H, &p, blob);
    p.rot_block = type == INZ_T_Q8G ? (rot8 ? inz_auto_rot_block(Q_FF) : -1) : 0;
    inz_quantize(D, Q_H, Q_FF, &p, (uint8_t *)blob + inz_mat_bytes(type, 2 * Q_FF, Q_H));
}

/* ---- single kernels, for unit-level parity ---- */
API void ref_router_logits(const uint16_t *W, int n, const float *X, float *Y) {
    for (int t = 0; t < n; t++) inz_matvec_f16_rows(W, Q_H, X + (size_t)t * Q_H, Y + (size_t)t * Q_N_EXPERT, 0, Q_N_EXPERT);
}

API void ref_softmax(float *s, int n) { softmax_inplace(s, n); }

API int ref_topk(const float *x, int n, int k, int32_t *idx) { return topk_f32(x, n, k, idx); }

API void ref_act_quantize(const float *x, int n, int rot_block, uint32_t seed, int8_t *q, float *s, float *bsum) {
    inz_act a;
    inz_act_alloc(&a, n);
    inz_act_quantize(&a, x, n, rot_block, seed);
    memcpy(q, a.q, (size_t)n);
    memcpy(s, a.s, sizeof(float) * (size_t)(n / INZ_GROUP));
    memcpy(bsum, a.bsum, sizeof(float) * (size_t)(n / INZ_GROUP));
    inz_act_free(&a);
}

/* Y[t][r] = W[r] . x_t through the decode kernels (n < GEMM_MIN_T numerics): inz_matvec_rows for n == 1,
 * inz_matmul_rows otherwise; the activations quantized per token with the matrix's rotation. */
API void ref_matmul_decode(const void *payload, int n, const float *X, float *Y) {
    inz_qmat m;
    if (!inz_qmat_view(&m, payload)) return;
    inz_act *acts = calloc((size_t)n, sizeof(inz_act));
    for (int t = 0; t < n; t++) {
        inz_act_alloc(&acts[t], m.cols);
        inz_act_quantize(&acts[t], X + (size_t)t * m.cols, m.cols, m.rot_block, m.rot_seed);
    }
    if (n == 1) inz_matvec_rows(&m, acts, Y, 0, m.rows);
    else inz_matmul_rows(&m, acts, n, Y, m.rows, 0, m.rows);
    for (int t = 0; t < n; t++) inz_act_free(&acts[t]);
    free(acts);
}

/* Y[t][r] through the prefill GEMM (n >= GEMM_MIN_T numerics): 256-block activations, weight-tile requant. */
API void ref_matmul_gemm(const void *payload, int n, const float *X, float *Y) {
    inz_qmat m;
    if (!inz_qmat_view(&m, payload)) return;
    inz_xq x;
    inz_xq_alloc(&x, n, m.cols);
    inz_xq_quantize(&x, X, m.cols, n, m.cols, m.rot_block, m.rot_seed);
    uint8_t *tb = inz_aligned(64, inz_gemm_tilebuf_bytes(m.cols));
    inz_gemm_rows(&m, &x, Y, m.rows, 0, m.rows, tb);
    free(tb);
    inz_xq_free(&x);
}

API void ref_xq(const float *X, int n, int K, int rot_block, uint32_t seed, int8_t *q, float *s, int32_t *sum) {
    inz_xq x;
    inz_xq_alloc(&x, n, K);
    inz_xq_quantize(&x, X, K, n, K, rot_block, seed);
    memcpy(q, x.q, (size_t)n * K);
    memcpy(s, x.s, sizeof(float) * (size_t)n * x.nkb);
    memcpy(sum, x.sum, sizeof(int32_t) * (size_t)n * x.nkb);
    inz_xq_free(&x);
}

/* ---- the routed MoE layer ----
 * Follows moe_block (src/model_fwd.c:992-1140) step by step for an all-resident expert set, minus the shared
 * expert (:1041-1069, :1141-1148), the lookahead (off when all experts are resident, :1044) and diagnostics:
 *   router lin_mm (:997) -> [test hook: logits += bias, or logits = override] -> per token softmax_inplace,
 *   topk_f32, renormalised weights and first-touch units (:1001-1031) -> y = 0 (:1033) -> experts: one
 *   experts_batch when n <= 8 (:1070-1089), else expert_compute per unit (:1080) -> rank-order combine (:1134-1140).
 * Dumps (all optional): logits [n][512] after the hook, probs [n][512], sel [n][10], w [n][10] (renormalised),
 * unit_expert [nu] (first-touch order), moe_out [n][10][H].
 * Returns the number of units, or -1 on a corrupt blob. */
API int ref_moe_routed(void *ctx, const uint16_t *router, const uint8_t *blobs, uint64_t blob_bytes, int n,
                       const float *xin, const float *bias, const float *logits_override, float *y, float *logits_out,
                       float *probs_out, int32_t *sel_out, float *w_out, int32_t *unit_expert_out, float *moe_out_out) {
    ref_ctx *c = ctx;
    inz_engine *e = c->e;
    if (n <= 0 || n > Q_MAX_T) return -1;
    lin rl;
    q_bind_lin(&rl, INZ_T_F16, Q_N_EXPERT, Q_H, (const uint8_t *)router);
    float *logits = c->logits;
    lin_mm(e, &rl, xin, Q_H, n, logits, Q_N_EXPERT);
    if (logits_override) memcpy(logits, logits_override, sizeof(float) * (size_t)n * Q_N_EXPERT);
    else if (bias)
        for (int t = 0; t < n; t++)
            for (int x = 0; x < Q_N_EXPERT; x++) logits[(size_t)t * Q_N_EXPERT + x] += bias[x];
    if (logits_out) memcpy(logits_out, logits, sizeof(float) * (size_t)n * Q_N_EXPERT);
    unit *units = e->units;
    int uid[Q_N_EXPERT];
    for (int x = 0; x < Q_N_EXPERT; x++) uid[x] = -1;
    int nu = 0;
    for (int t = 0; t < n; t++) {
        float *pr = logits + (size_t)t * Q_N_EXPERT;
        softmax_inplace(pr, Q_N_EXPERT);
        if (probs_out) memcpy(probs_out + (size_t)t * Q_N_EXPERT, pr, sizeof(float) * Q_N_EXPERT);
        int32_t sel[Q_TOPK];
        float w[Q_TOPK], sum = 0;
        topk_f32(pr, Q_N_EXPERT, Q_TOPK, sel);
        for (int k = 0; k < Q_TOPK; k++) {
            w[k] = pr[sel[k]];
            sum += w[k];
        }
        for (int k = 0; k < Q_TOPK; k++) {
            const int x = sel[k];
            if (uid[x] < 0) { uid[x] = nu; units[nu].expert = x; units[nu].ntok = 0; nu++; }
            unit *u = &units[uid[x]];
            u->tok[u->ntok] = t;
            u->slot[u->ntok] = t * Q_TOPK + k;
            u->w[u->ntok] = w[k] / sum;
            u->ntok++;
            if (sel_out) sel_out[(size_t)t * Q_TOPK + k] = x;
            if (w_out) w_out[(size_t)t * Q_TOPK + k] = w[k] / sum;
        }
    }
    memset(y, 0, sizeof(float) * (size_t)n * Q_H);
    for (int i = 0; i < nu; i++) {
        inz_qmat g;
        if (!inz_qmat_view(&g, blobs + (size_t)units[i].expert * blob_bytes)) return -1;
    }
    const bool batch = n <= 8 && nu <= EB_MAX && e->expert_type != INZ_T_F16 && e->expert_type != INZ_T_F32;
    if (batch) {
        const unit *bu[EB_MAX];
        const uint8_t *bb[EB_MAX];
        for (int i = 0; i < nu; i++) { bu[i] = &units[i]; bb[i] = blobs + (size_t)units[i].expert * blob_bytes; }
        experts_batch(e, bu, bb, nu, n, xin);
    } else {
        for (int i = 0; i < nu; i++) expert_compute(e, blobs + (size_t)units[i].expert * blob_bytes, &units[i], xin, e->moe_out);
    }
    for (int t = 0; t < n; t++) {
        float *yt = y + (size_t)t * Q_H;
        for (int k = 0; k < Q_TOPK; k++) {
            const float *o = e->moe_out + ((size_t)t * Q_TOPK + k) * Q_H;
            for (int cc = 0; cc < Q_H; cc++) yt[cc] += o[cc];
        }
    }
    if (unit_expert_out) for (int i = 0; i < nu; i++) unit_expert_out[i] = units[i].expert;
    if (moe_out_out) memcpy(moe_out_out, e->moe_out, sizeof(float) * (size_t)n * Q_TOPK * Q_H);
    return nu;
}

/* ---- the shared expert ----
 * gate|up (lin_mm, :1047-1050), SiLU * up in place (:1064-1067), down (lin_mm, :1068), then per token
 * y += sigmoid(sh_gate . x) * D (:1141-1148). blob: the gate|up matrix followed by the down matrix at gu_bytes (the
 * expert-blob layout); gate [H] fp32; y [n][H] is updated in place; D_out [n][H] optional.
 * Returns 0, or -1 on a matrix that does not match the shared expert's shape. */
_Static_assert(Q_SHARED_FF == Q_FF, "the harness reuses the expert scratch for the shared expert");
API int ref_shared(void *ctx, const uint8_t *blob, uint64_t gu_bytes, int type, const float *gate, int n,
                   const float *xin, float *y, float *D_out) {
    ref_ctx *c = ctx;
    inz_engine *e = c->e;
    if (n <= 0 || n > Q_MAX_T) return -1;
    lin gu, dn;
    if (!q_bind_lin(&gu, type, 2 * Q_SHARED_FF, Q_H, blob) || !q_bind_lin(&dn, type, Q_H, Q_SHARED_FF, blob + gu_bytes))
        return -1;
    float *GU = e->ex_gu, *D = e->ex_d;
    lin_mm(e, &gu, xin, Q_H, n, GU, 2 * Q_SHARED_FF);
    for (int t = 0; t < n; t++) {
        float *r = GU + (size_t)t * 2 * Q_SHARED_FF;
        for (int k = 0; k < Q_SHARED_FF; k++) r[k] = siluf(r[k]) * r[Q_SHARED_FF + k];
    }
    lin_mm(e, &dn, GU, 2 * Q_SHARED_FF, n, D, Q_H);
    for (int t = 0; t < n; t++) {
        const float sg = sigmoidf(dot_f32(gate, xin + (size_t)t * Q_H, Q_H));
        float *yt = y + (size_t)t * Q_H;
        const float *dt = D + (size_t)t * Q_H;
        for (int k = 0; k < Q_H; k++) yt[k] += sg * dt[k];
    }
    if (D_out) memcpy(D_out, D, sizeof(float) * (size_t)n * Q_H);
    return 0;
}

/* ---- hyper-connections around the MoE layer ----
 * hc_in (src/model_fwd.c:432-439) and hc_out (:442-450) themselves, with F16 down/up matrices (the converter's
 * default hc type, src/convert.c:148) bound by q_bind_lin. norm [4H], down [320][4H] f16 bits, up [4H][320] f16 bits,
 * inject [4][4H] (NULL: no inj, as the final mixer); X [n][4H] -> xin [n][H], inj [n][4]. hc_in's scratch (e->Xn,
 * e->tmp, e->big) is allocated for this call's n only. Returns 0, or -1 on a bad n. */
API int ref_hc_rank(void) { return Q_HC_RANK; }

API int ref_hc_in(void *ctx, const float *norm, const uint16_t *down, const uint16_t *up, const float *inject, int n,
                  const float *X, float *xin, float *inj) {
    ref_ctx *c = ctx;
    inz_engine *e = c->e;
    if (n <= 0 || n > Q_MAX_T) return -1;
    hcw w;
    memset(&w, 0, sizeof(w));
    w.norm = norm;
    w.inject = inject;
    if (!q_bind_lin(&w.down, INZ_T_F16, Q_HC_RANK, Q_HCW, (const uint8_t *)down) ||
        !q_bind_lin(&w.up, INZ_T_F16, Q_HCW, Q_HC_RANK, (const uint8_t *)up))
        return -1;
    float *sXn = e->Xn, *stmp = e->tmp, *sbig = e->big;
    e->Xn = inz_aligned(64, sizeof(float) * (size_t)n * Q_HCW);
    e->tmp = inz_aligned(64, sizeof(float) * (size_t)n * Q_HC_RANK);
    e->big = inz_aligned(64, sizeof(float) * (size_t)n * Q_HCW);
    hc_in(e, &w, n, X, xin, inject ? inj : NULL);
    free(e->Xn); free(e->tmp); free(e->big);
    e->Xn = sXn; e->tmp = stmp; e->big = sbig;
    return 0;
}

API void ref_hc_out(int n, float *X, const float *inj, const float *y) { hc_out(n, X, inj, y); }
