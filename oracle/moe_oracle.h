/*
 * moe_oracle.h -- TEST INFRASTRUCTURE ONLY: a plain-C restatement of inferenZ's MoE layer arithmetic, used by
 * tests/ (and by bench.py's CPU-baseline leg when the compiled reference is not available) as the checker of the
 * CUDA path. Not part of the product; the product never links it.
 *
 * Every function follows the reference file:line given beside it. Floating-point operations are written out one by
 * one (explicit fmaf where the reference uses an FMA, -ffp-contract=off everywhere else) so the results are
 * bit-identical to the reference's AVX2/VNNI kernels, including their 8-lane accumulation orders.
 * Parity of this restatement with the compiled reference (oracle/_ref) is asserted by tests/test_oracle.py.
 */
#ifndef INZ_MOE_ORACLE_H
#define INZ_MOE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#define ORC_GROUP 64          /* src/quant.h:21 INZ_GROUP */
#define ORC_LUT_BIAS 64       /* src/quant.h:22 INZ_LUT_BIAS */
#define ORC_KB 256            /* src/quant.h:152 INZ_KB */
#define ORC_GEMM_MIN_T 12     /* src/model_fwd.c:126 GEMM_MIN_T */
#define ORC_T_F16 1
#define ORC_T_Q4L 102
#define ORC_T_Q8G 103
#define ORC_T_Q4N 107         /* src/quant.h:34 INZ_T_Q4N (NVFP4 repacked: e2m1 codes, e4m3 scale per 16, global) */

#ifdef __cplusplus
extern "C" {
#endif

/* view over one serialized quantized matrix: 64-byte header, indices [rows][ng][gb], fp16 scales [rows][ng]
 * (src/quant.h:40-67, src/quant.c:69-91) */
typedef struct {
    int type, bits, rows, cols, ng, rot_block;
    uint32_t rot_seed;
    const uint8_t *lut;
    const uint8_t *q;
    const uint16_t *d;
    size_t gb;
    const uint8_t *s8;  /* Q4N: e4m3 scales [rows][ng][4], one per 16 weights (d is NULL) */
    float gscale;       /* Q4N: weight = (lut[code] - 64) * e4m3 * gscale */
} orc_qmat;

int orc_qmat_view(orc_qmat *m, const void *payload);
size_t orc_qmat_bytes(int type, int rows, int cols);
float orc_f16_to_f32(uint16_t h);

/* router: Y[t][e] = sum_k f16(W[e][k]) * X[t][k] in the 8-lane FMA order + hsum8 tree */
void orc_router_logits(const uint16_t *W, int E, int H, const float *X, int n, float *Y);
/* softmax in place over n values (n % 8 == 0), Cephes exp, 8-lane sum */
void orc_softmax(float *s, int n);
/* top-k indices by (value desc, index asc); returns k */
int orc_topk(const float *x, int n, int k, int32_t *idx);
/* randomized Hadamard rotation in place */
void orc_rotate(float *x, int n, int block, uint32_t seed);
/* decode-path activation: rotate, int8 per 64-group; q [n], s [n/64], bsum [n/64] */
void orc_act_quantize(const float *x, int n, int rot_block, uint32_t seed, int8_t *q, float *s, float *bsum);
/* decode-path product of one token: y[r] = W[r] . x for all rows (mv_q4l / mv_q8g numerics). q8_vnni selects the
 * VNNI Q8G variant (bias removed after the float sum) over the AVX2 split path. */
void orc_matvec_decode(const orc_qmat *m, const int8_t *q, const float *s, const float *bsum, float *y, int q8_vnni);
/* prefill-path activation: rotate, int8 per 256-block (last block partial); q [K], s [nkb], sum [nkb] */
void orc_xq(const float *x, int K, int rot_block, uint32_t seed, int8_t *q, float *s, int32_t *sum);
/* prefill-path weight requantization of one row: w8 [K] signed (the reference's u8 minus 128), ws [nkb] */
void orc_gemm_requant_row(const orc_qmat *m, int row, int8_t *w8, float *ws);
/* prefill-path product: Y[t][r] for n tokens (inz_gemm_rows numerics) */
void orc_matmul_gemm(const orc_qmat *m, int n, const int8_t *q, const float *s, const int32_t *sum, float *Y);

/* whole routed layer (moe_block's routed part). Blobs: n_expert blobs of blob_bytes, gate|up matrix first, down at
 * gu_bytes. bias / logits_override: optional test hook between router and softmax. Dumps optional.
 * Returns the number of units (distinct experts), or -1 on a corrupt blob. */
int orc_moe_routed(int H, int FF, int E, int topk, const uint16_t *router, const uint8_t *blobs, uint64_t blob_bytes,
                   uint64_t gu_bytes, int n, const float *xin, const float *bias, const float *logits_override, float *y,
                   float *logits_out, float *probs_out, int32_t *sel_out, float *w_out, int32_t *unit_expert_out,
                   float *moe_out, int q8_vnni);

/* hyper-connections (src/model_fwd.c:404-450): hc_in X [n][4H] -> xin [n][H], inj [n][4] (inj NULL: not computed);
 * norm [4H], down [rank][4H] f16, up [4H][rank] f16, inject [4][4H]. hc_out: X [n][4H] += inj * y in place. */
void orc_hc_in(int H, int rank, const float *norm, const uint16_t *down, const uint16_t *up, const float *inject,
               int n, const float *X, float *xin, float *inj);
void orc_hc_out(int H, int n, float *X, const float *inj, const float *y);

/* one matrix payload times n tokens, activations quantized here as the reference's lin_mm does: decode numerics
 * (gemm = 0: one activation per token, mv for n == 1, mm otherwise) or prefill GEMM numerics (gemm = 1).
 * Y [n][rows]. Returns 0, or -1 on a payload or shape this restatement does not cover. */
int orc_matmul_payload(const void *payload, int n, const float *X, float *Y, int gemm, int q8_vnni);

/* ---- seeded synthetic inputs (test infrastructure): the LCG + Box-Muller normal of the reference's tests
 * (tests/test_quant.c:10-17), so that the CPU side of a test or of the benchmark's reference arm draws its inputs
 * without the product library ---- */
uint64_t orc_synth_jump(uint64_t state, uint64_t n_normals);
uint64_t orc_synth_randn(uint64_t state, int64_t n, float scale, float *out);
/* expert e of a layer seeded `seed`: gu [2FF][H] (gate rows, then up rows), dn [H][FF], each randn * sqrt(1/H) */
void orc_synth_expert(uint64_t seed, int H, int FF, int e, float *gu, float *dn);
/* router [E][H] fp16 bits from randn * 0.02, rounded to nearest even (the reference's inz_f32_to_f16) */
void orc_synth_router(uint64_t seed, int E, int H, uint16_t *w);
/* hidden states [n][H] from randn, each row divided by sqrt(mean(x^2) + 1e-6) */
void orc_synth_hidden(uint64_t seed, int n, int H, float *x);

#ifdef __cplusplus
}
#endif
#endif
