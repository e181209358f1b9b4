/*
 * moe_oracle.c -- TEST INFRASTRUCTURE ONLY. Plain-C restatement of the reference's MoE layer arithmetic (the
 * checker of the CUDA path; see moe_oracle.h). Each function names the reference lines it restates. Built with
 * -ffp-contract=off: every multiply, add and FMA below is one IEEE operation, in the reference's order.
 */
#include "moe_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#define QMAGIC 0x515A4E49u /* "INZQ", src/quant.c:12 */

/* ---------------- formats ---------------- */

/* index bytes per 64-weight group: bits * 64 / 8 (src/quant.c:25) */
static size_t group_bytes(int type) {
    return type == ORC_T_Q4L || type == ORC_T_Q4N ? 32 : type == ORC_T_Q8G ? 64 : 0;
}

/* src/quant.c:30-36 (Q4L / Q8G / Q4N: four e4m3 scales per group in place of one fp16) */
size_t orc_qmat_bytes(int type, int rows, int cols) {
    size_t ng = (size_t)cols / ORC_GROUP;
    size_t n = 64 + (size_t)rows * ng * group_bytes(type) + (size_t)rows * ng * 2;
    if (type == ORC_T_Q4N) n += (size_t)rows * ng * 2;
    return (n + 63) / 64 * 64;
}

/* src/quant.c:69-91 (header layout src/quant.h:40-50) */
int orc_qmat_view(orc_qmat *m, const void *payload) {
    const uint8_t *h = payload;
    uint32_t magic, rows, cols, seed;
    uint16_t type, rot;
    memcpy(&magic, h, 4);
    if (magic != QMAGIC) return 0;
    memcpy(&type, h + 4, 2);
    memcpy(&rot, h + 6, 2);
    memcpy(&rows, h + 8, 4);
    memcpy(&cols, h + 12, 4);
    memcpy(&seed, h + 16, 4);
    memset(m, 0, sizeof(*m));
    m->type = type;
    m->bits = h[20];
    m->rows = (int)rows;
    m->cols = (int)cols;
    m->ng = m->cols / ORC_GROUP;
    m->rot_block = rot;
    m->rot_seed = seed;
    m->lut = h + 24;
    m->gb = group_bytes(type);
    m->q = h + 64;
    m->d = (const uint16_t *)(m->q + (size_t)m->rows * m->ng * m->gb);
    if (type == ORC_T_Q4N) {  /* src/quant.c:85-89: scales where the fp16 ones would be, gscale in pad2 */
        m->s8 = (const uint8_t *)m->d;
        m->d = NULL;
        memcpy(&m->gscale, h + 56, 4);
    }
    return m->gb != 0;
}

/* inz_e4m3_to_f32, src/util.c:119-126 */
static float e4m3_to_f32(uint8_t x) {
    const uint32_t sg = x >> 7, e = (x >> 3) & 0xF, mt = x & 7;
    float v;
    if (e == 0) v = (float)mt / 8.0f / 64.0f;
    else if (e == 15 && mt == 7) v = NAN;
    else v = (1.0f + (float)mt / 8.0f) * ldexpf(1.0f, (int)e - 7);
    return sg ? -v : v;
}

/* IEEE half -> float, exact (src/util.c:116 _cvtsh_ss) */
float orc_f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023, bits;
    if (e == 0) {
        if (m == 0) bits = s;
        else {                                    /* subnormal: normalise */
            int sh = 0;
            while (!(m & 1024)) { m <<= 1; sh++; }
            m &= 1023;
            bits = s | ((uint32_t)(127 - 15 + 1 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) bits = s | 0x7F800000u | (m << 13);
    else bits = s | ((e + 127 - 15) << 23) | (m << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* hsum8 / hsum256_ps / hsum8f: src/quant.c:705-711, src/vmath.h:27-32, src/quant.c:224-230 */
static float hsum8(const float a[8]) {
    float b0 = a[0] + a[4], b1 = a[1] + a[5], b2 = a[2] + a[6], b3 = a[3] + a[7];
    return (b0 + b2) + (b1 + b3);
}

/* ---------------- router ---------------- */

/* inz_matvec_f16_rows, src/quant.c:1290-1304 (inz_matmul_f16_rows 1330-1366 is bit-identical per (row, token),
 * tests/test_kernels.c:40-46). H % 8 == 0 in every configuration, so the scalar tail is never used. */
void orc_router_logits(const uint16_t *W, int E, int H, const float *X, int n, float *Y) {
    for (int t = 0; t < n; t++) {
        const float *x = X + (size_t)t * H;
        for (int e = 0; e < E; e++) {
            const uint16_t *w = W + (size_t)e * H;
            float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int j = 0; j + 8 <= H; j += 8)
                for (int l = 0; l < 8; l++) a[l] = fmaf(orc_f16_to_f32(w[j + l]), x[j + l], a[l]);
            Y[(size_t)t * E + e] = hsum8(a);
        }
    }
}

/* exp256_ps (Cephes), src/vmath.h:9-25, one lane */
static float cephes_exp(float x) {
    x = fminf(fmaxf(x, -87.3f), 88.3f);
    const float fx = rintf(x * 1.44269504088896341f);
    x = fmaf(-fx, 0.693359375f, x);
    x = fmaf(-fx, -2.12194440e-4f, x);
    const float z = x * x;
    float y = 1.9875691500e-4f;
    y = fmaf(y, x, 1.3981999507e-3f);
    y = fmaf(y, x, 8.3334519073e-3f);
    y = fmaf(y, x, 4.1665795894e-2f);
    y = fmaf(y, x, 1.6666665459e-1f);
    y = fmaf(y, x, 5.0000001201e-1f);
    y = fmaf(y, z, x) + 1.0f;
    const uint32_t eb = (uint32_t)((int)fx + 127) << 23;
    float p;
    memcpy(&p, &eb, 4);
    return y * p;
}

/* softmax_inplace, src/vmath.h:42-60 (n % 8 == 0) */
void orc_softmax(float *s, int n) {
    float mx = -INFINITY;
    for (int i = 0; i < n; i++) mx = s[i] > mx ? s[i] : mx;
    float vs[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = 0; i < n; i++) {
        s[i] = cephes_exp(s[i] - mx);
        vs[i & 7] = vs[i & 7] + s[i];
    }
    const float inv = 1.0f / hsum8(vs);
    for (int i = 0; i < n; i++) s[i] = s[i] * inv;
}

/* topk_f32, src/sampler.c:95-127: the k best by (value desc, index asc), in that order */
int orc_topk(const float *x, int n, int k, int32_t *idx) {
    if (k <= 0 || k > n) k = n;
    for (int i = 0; i < k; i++) {
        int best = -1;
        for (int j = 0; j < n; j++) {
            int used = 0;
            for (int q = 0; q < i; q++) used |= idx[q] == j;
            if (used) continue;
            if (best < 0 || x[j] > x[best]) best = j;   /* equal values keep the lower index */
        }
        idx[i] = best;
    }
    return k;
}

/* ---------------- activations ---------------- */

/* rot_sign, src/quant.c:118-122 */
static float rot_sign(uint32_t seed, uint32_t i) {
    uint32_t h = (i + 1) * 0x9E3779B1u ^ seed;
    h ^= h >> 15; h *= 0x2C1B3C6Du; h ^= h >> 12; h *= 0x297A2D39u; h ^= h >> 15;
    return (h & 1) ? -1.0f : 1.0f;
}

/* inz_rotate + fwht, src/quant.c:124-154 */
void orc_rotate(float *x, int n, int block, uint32_t seed) {
    if (block <= 1) return;
    const float norm = 1.0f / sqrtf((float)block);
    for (int i = 0; i < n; i++) x[i] = x[i] * rot_sign(seed, (uint32_t)i);
    for (int b = 0; b < n; b += block) {
        float *v = x + b;
        for (int len = 1; len < block; len <<= 1)
            for (int i = 0; i < block; i += len << 1)
                for (int j = i; j < i + len; j++) {
                    const float a = v[j], c = v[j + len];
                    v[j] = a + c;
                    v[j + len] = a - c;
                }
        for (int i = 0; i < block; i++) v[i] = v[i] * norm;
    }
}

/* inz_act_quantize + act_quantize_groups, src/quant.c:611-655 */
void orc_act_quantize(const float *x, int n, int rot_block, uint32_t seed, int8_t *q, float *s, float *bsum) {
    float *r = malloc(sizeof(float) * (size_t)n);
    memcpy(r, x, sizeof(float) * (size_t)n);
    if (rot_block > 1) orc_rotate(r, n, rot_block, seed);
    for (int g = 0; g < n / ORC_GROUP; g++) {
        const float *xg = r + (size_t)g * ORC_GROUP;
        float amax = 0;
        for (int j = 0; j < ORC_GROUP; j++) amax = fmaxf(amax, fabsf(xg[j]));
        const float sc = amax / 127.0f;
        const float inv = sc > 0 ? 1.0f / sc : 0;
        int sum = 0;
        for (int j = 0; j < ORC_GROUP; j++) {
            const int v = (int)rintf(xg[j] * inv);     /* _mm256_cvtps_epi32 under the default MXCSR: RNE */
            q[g * ORC_GROUP + j] = (int8_t)v;
            sum += v;
        }
        s[g] = sc;
        bsum[g] = sc * (float)sum;
    }
    free(r);
}

/* inz_xq_rows, src/quant.c:1407-1429 (one token) */
void orc_xq(const float *x, int K, int rot_block, uint32_t seed, int8_t *q, float *s, int32_t *sum) {
    float *r = malloc(sizeof(float) * (size_t)K);
    memcpy(r, x, sizeof(float) * (size_t)K);
    if (rot_block > 1) orc_rotate(r, K, rot_block, seed);
    const int nkb = (K + ORC_KB - 1) / ORC_KB;
    for (int b = 0; b < nkb; b++) {
        const int k0 = b * ORC_KB, k1 = k0 + ORC_KB < K ? k0 + ORC_KB : K;
        float amax = 0;
        for (int k = k0; k < k1; k++) amax = fmaxf(amax, fabsf(r[k]));
        const float sc = amax / 127.0f, inv = sc > 0 ? 1.0f / sc : 0;
        int32_t acc = 0;
        for (int k = k0; k < k1; k++) {
            const int v = (int)lrintf(r[k] * inv);
            q[k] = (int8_t)v;
            acc += v;
        }
        s[b] = sc;
        sum[b] = acc;
    }
    free(r);
}

/* ---------------- decode-path products ---------------- */

/* mv_q4l (DEFINE_MV_LUT, src/quant.c:767-875) and mm_q4l (1179-1225, identical per token); mv_q8g (881-917) and
 * mm_q8g (922-953). Lane l of the 8-wide accumulators holds, per group, the integer dot of weights
 * {4l..4l+3} and {32+4l..32+4l+3} (two VPDPBUSD over the two 32-byte halves of the group). */
void orc_matvec_decode(const orc_qmat *m, const int8_t *q, const float *s, const float *bsum, float *y, int q8_vnni) {
    const int ng = m->ng, ng8 = ng & ~7;
    const int q8 = m->type == ORC_T_Q8G;
    for (int r = 0; r < m->rows; r++) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0}, bl[8] = {0, 0, 0, 0, 0, 0, 0, 0}, b = 0;
        for (int g = 0; g < ng; g++) {
            const uint8_t *w = m->q + ((size_t)r * ng + g) * m->gb;
            const int8_t *x = q + (size_t)g * ORC_GROUP;
            const float dd = orc_f16_to_f32(m->d[(size_t)r * ng + g]);
            const float ds = dd * s[g];
            for (int l = 0; l < 8; l++) {
                int32_t I = 0;
                for (int i = 0; i < 4; i++) {
                    const int j = 4 * l + i;
                    int u0, u1;
                    if (q8) {
                        u0 = w[j];
                        u1 = w[32 + j];
                        if (!q8_vnni) { u0 -= 128; u1 -= 128; }
                    } else {
                        u0 = m->lut[w[j] & 15];
                        u1 = m->lut[w[j] >> 4];
                    }
                    I += u0 * x[j] + u1 * x[32 + j];
                }
                acc[l] = fmaf((float)I, ds, acc[l]);
            }
            if (q8) {
                if (q8_vnni) b = fmaf(dd, bsum[g], b);
            } else if (g < ng8) bl[g & 7] = fmaf(dd, bsum[g], bl[g & 7]);
        }
        if (q8) y[r] = hsum8(acc) - 128.0f * b;
        else {
            float bb = hsum8(bl);
            for (int g = ng8; g < ng; g++) bb = fmaf(orc_f16_to_f32(m->d[(size_t)r * ng + g]), bsum[g], bb);
            y[r] = hsum8(acc) - (float)ORC_LUT_BIAS * bb;
        }
    }
}

/* Q4N lane partials of one group (src/quant.c:1089-1104, 1150-1157): VPDPBUSD from the activation's LUT bias
 * -64 * sum4 (nb4) over the biased codes, i.e. lane k of the low half = sum over weights 4k..4k+3 of (lut - 64) * x,
 * lane k of the high half = the same over weights 32+4k..32+4k+3 (code = high nibble of byte 4k+i). Exact. */
static void q4n_partials(const orc_qmat *m, const uint8_t *w, const int8_t *x, int32_t i0[8], int32_t i1[8]) {
    for (int k = 0; k < 8; k++) {
        int32_t a = 0, b = 0;
        for (int i = 0; i < 4; i++) {
            const int j = 4 * k + i;
            a += ((int)m->lut[w[j] & 15] - ORC_LUT_BIAS) * x[j];
            b += ((int)m->lut[w[j] >> 4] - ORC_LUT_BIAS) * x[32 + j];
        }
        i0[k] = a;
        i1[k] = b;
    }
}

/* mv_q4n, src/quant.c:1065-1105 (row pairs, even group count: the expert shapes): per group and lane,
 * acc = fma(i0, scale_block * xs, acc) then fma(i1, scale_block' * xs, acc), block = k / 4 (low half) or 2 + k / 4;
 * y = hsum8(acc) * gscale. */
static void q4n_mv(const orc_qmat *m, const int8_t *q, const float *s, float *y) {
    const int ng = m->ng;
    for (int r = 0; r < m->rows; r++) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int g = 0; g < ng; g++) {
            int32_t i0[8], i1[8];
            q4n_partials(m, m->q + ((size_t)r * ng + g) * 32, q + (size_t)g * ORC_GROUP, i0, i1);
            const uint8_t *sc = m->s8 + ((size_t)r * ng + g) * 4;
            for (int k = 0; k < 8; k++) acc[k] = fmaf((float)i0[k], e4m3_to_f32(sc[k / 4]) * s[g], acc[k]);
            for (int k = 0; k < 8; k++) acc[k] = fmaf((float)i1[k], e4m3_to_f32(sc[2 + k / 4]) * s[g], acc[k]);
        }
        y[r] = hsum8(acc) * m->gscale;
    }
}

/* mm_q4n, src/quant.c:1139-1163: per group and lane part = fma(i1, S1, i0 * S0), acc = fma(part, xs, acc);
 * y = hsum8(acc) * gscale (a different rounding order from mv_q4n: one token through mm differs from mv). */
static void q4n_mm_token(const orc_qmat *m, const int8_t *q, const float *s, float *y) {
    const int ng = m->ng;
    for (int r = 0; r < m->rows; r++) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int g = 0; g < ng; g++) {
            int32_t i0[8], i1[8];
            q4n_partials(m, m->q + ((size_t)r * ng + g) * 32, q + (size_t)g * ORC_GROUP, i0, i1);
            const uint8_t *sc = m->s8 + ((size_t)r * ng + g) * 4;
            for (int k = 0; k < 8; k++) {
                const float part = fmaf((float)i1[k], e4m3_to_f32(sc[2 + k / 4]), (float)i0[k] * e4m3_to_f32(sc[k / 4]));
                acc[k] = fmaf(part, s[g], acc[k]);
            }
        }
        y[r] = hsum8(acc) * m->gscale;
    }
}

/* ---------------- prefill-path (GEMM) products ---------------- */

/* _mm256_mulhrs_epi16 on one lane: bits 16..1 of ((a*b >> 14) + 1) */
static int16_t mulhrs(int16_t a, int16_t b) {
    const int32_t t = (((int32_t)a * (int32_t)b) >> 14) + 1;
    return (int16_t)(uint16_t)((uint32_t)t >> 1);
}

static int sat_u8(int v) { return v < 0 ? 0 : v > 255 ? 255 : v; }

/* gemm_decode_tile, src/quant.c:1532-1613, for one row: per 256-block scale ws = dmax * maxlev / 127 and
 * per-group factor F = lrint(512 * d / ws), int8 weight = sat_u8(mulhrs(level * 64, F) + 128) - 128. */
/* gemm_decode_tile_q4n, src/quant.c:1479-1530, for one row: per 256-block sc = max e4m3 scale * maxlev / 127,
 * ws = sc * gscale; per 16-weight block F = lrint(e4m3 * 512 / sc); int8 weight = sat_u8(mulhrs(level * 64, F) + 128)
 * - 128 with the block's F (weights 0-15, 16-31 of a group from the low nibbles, 32-47, 48-63 from the high ones). */
static void q4n_requant_row(const orc_qmat *m, int row, int8_t *w8, float *ws) {
    const int K = m->cols, ng = m->ng, nkb = (K + ORC_KB - 1) / ORC_KB, nsb = ng * 4, spb = ORC_KB / 16;
    int maxlev = 1;
    int16_t lv[16];
    for (int c = 0; c < 16; c++) {
        lv[c] = (int16_t)(((int)m->lut[c] - ORC_LUT_BIAS) * 64);
        if (abs((int)m->lut[c] - ORC_LUT_BIAS) > maxlev) maxlev = abs((int)m->lut[c] - ORC_LUT_BIAS);
    }
    int16_t *F = malloc(sizeof(int16_t) * (size_t)nsb);
    const uint8_t *sr = m->s8 + (size_t)row * nsb;
    for (int b = 0; b < nkb; b++) {
        const int k0 = b * spb, k1 = k0 + spb < nsb ? k0 + spb : nsb;
        float smax = 0;
        for (int k = k0; k < k1; k++) smax = fmaxf(smax, e4m3_to_f32(sr[k]));
        const float sc = smax * (float)maxlev / 127.0f;
        ws[b] = sc * m->gscale;
        const float inv = sc > 0 ? 512.0f / sc : 0;
        for (int k = k0; k < k1; k++) F[k] = (int16_t)lrintf(e4m3_to_f32(sr[k]) * inv);
    }
    for (int g = 0; g < ng; g++) {
        const uint8_t *qg = m->q + ((size_t)row * ng + g) * 32;
        int8_t *o = w8 + (size_t)g * ORC_GROUP;
        for (int j = 0; j < 32; j++) {
            const int16_t f0 = F[g * 4 + j / 16], f1 = F[g * 4 + 2 + j / 16];
            o[j] = (int8_t)(sat_u8((int16_t)(mulhrs(lv[qg[j] & 15], f0) + 128)) - 128);
            o[32 + j] = (int8_t)(sat_u8((int16_t)(mulhrs(lv[qg[j] >> 4], f1) + 128)) - 128);
        }
    }
    free(F);
}

void orc_gemm_requant_row(const orc_qmat *m, int row, int8_t *w8, float *ws) {
    if (m->type == ORC_T_Q4N) {
        q4n_requant_row(m, row, w8, ws);
        return;
    }
    const int K = m->cols, ng = m->ng, nkb = (K + ORC_KB - 1) / ORC_KB, gpb = ORC_KB / ORC_GROUP;
    const int q8 = m->type == ORC_T_Q8G;
    const int bias = q8 ? 128 : ORC_LUT_BIAS;
    int maxlev = 127;
    int16_t lv[16] = {0};
    if (!q8) {
        maxlev = 1;
        for (int i = 0; i < 16; i++) {
            lv[i] = (int16_t)((int)m->lut[i] - bias);
            if (abs(lv[i]) > maxlev) maxlev = abs(lv[i]);
        }
    }
    int16_t *F = malloc(sizeof(int16_t) * (size_t)ng);
    const uint16_t *d = m->d + (size_t)row * ng;
    for (int b = 0; b < nkb; b++) {
        const int g0 = b * gpb, g1 = g0 + gpb < ng ? g0 + gpb : ng;
        float dmax = 0;
        for (int g = g0; g < g1; g++) dmax = fmaxf(dmax, fabsf(orc_f16_to_f32(d[g])));
        const float sc = dmax * (float)maxlev / 127.0f;
        ws[b] = sc;
        const float inv = sc > 0 ? 512.0f / sc : 0;
        for (int g = g0; g < g1; g++) F[g] = (int16_t)lrintf(orc_f16_to_f32(d[g]) * inv);
    }
    for (int g = 0; g < ng; g++) {
        const uint8_t *qg = m->q + ((size_t)row * ng + g) * m->gb;
        int8_t *o = w8 + (size_t)g * ORC_GROUP;
        if (q8) {
            for (int j = 0; j < 64; j++) {
                const int16_t w = (int16_t)(((int)qg[j] - 128) << 6);
                o[j] = (int8_t)(sat_u8((int16_t)(mulhrs(w, F[g]) + 128)) - 128);
            }
        } else {
            int tab[16];
            for (int i = 0; i < 16; i++) tab[i] = sat_u8((int16_t)(mulhrs((int16_t)(lv[i] * 64), F[g]) + 128)) - 128;
            for (int j = 0; j < 32; j++) {
                o[j] = (int8_t)tab[qg[j] & 15];
                o[32 + j] = (int8_t)tab[qg[j] >> 4];
            }
        }
    }
    free(F);
}

/* inz_gemm_rows, src/quant.c:1615-1668: per 256-block an exact integer dot, then f = fma(dot, ws * xs, f) in block
 * order (the reference's float(acc) - 128 * sum equals the signed dot exactly: every term is below 2^24). */
void orc_matmul_gemm(const orc_qmat *m, int n, const int8_t *q, const float *s, const int32_t *sum, float *Y) {
    (void)sum;
    const int K = m->cols, nkb = (K + ORC_KB - 1) / ORC_KB;
    int8_t *w8 = malloc((size_t)K);
    float *ws = malloc(sizeof(float) * (size_t)nkb);
    for (int r = 0; r < m->rows; r++) {
        orc_gemm_requant_row(m, r, w8, ws);
        for (int t = 0; t < n; t++) {
            const int8_t *x = q + (size_t)t * K;
            float f = 0;
            for (int b = 0; b < nkb; b++) {
                const int k0 = b * ORC_KB, k1 = k0 + ORC_KB < K ? k0 + ORC_KB : K;
                int32_t D = 0;
                for (int k = k0; k < k1; k++) D += (int32_t)w8[k] * x[k];
                f = fmaf((float)D, ws[b] * s[(size_t)t * nkb + b], f);
            }
            Y[(size_t)t * m->rows + r] = f;
        }
    }
    free(w8);
    free(ws);
}

int orc_matmul_payload(const void *payload, int n, const float *X, float *Y, int gemm, int q8_vnni) {
    orc_qmat m;
    if (n <= 0 || !orc_qmat_view(&m, payload)) return -1;
    if (m.type == ORC_T_Q4N && ((m.rows & 1) || (m.ng & 1))) return -1;  /* the scalar tails are not restated */
    const int K = m.cols, nkb = (K + ORC_KB - 1) / ORC_KB;
    int8_t *q = malloc((size_t)n * K);
    float *s = malloc(sizeof(float) * (size_t)n * (K / ORC_GROUP + nkb)), *b = malloc(sizeof(float) * (size_t)K);
    int32_t *sum = malloc(sizeof(int32_t) * (size_t)n * nkb);
    if (gemm) {
        for (int t = 0; t < n; t++)
            orc_xq(X + (size_t)t * K, K, m.rot_block, m.rot_seed, q + (size_t)t * K, s + (size_t)t * nkb, sum + (size_t)t * nkb);
        orc_matmul_gemm(&m, n, q, s, sum, Y);
    } else {
        for (int t = 0; t < n; t++) {
            int8_t *qt = q + (size_t)t * K;
            float *st = s + (size_t)t * (K / ORC_GROUP);
            orc_act_quantize(X + (size_t)t * K, K, m.rot_block, m.rot_seed, qt, st, b);
            float *yt = Y + (size_t)t * m.rows;
            if (m.type != ORC_T_Q4N) orc_matvec_decode(&m, qt, st, b, yt, q8_vnni);
            else if (n == 1) q4n_mv(&m, qt, st, yt);
            else q4n_mm_token(&m, qt, st, yt);
        }
    }
    free(q); free(s); free(b); free(sum);
    return 0;
}

/* ---------------- the routed layer ---------------- */

/* siluf, src/model_fwd.c:43 */
static float siluf(float x) { return x / (1.0f + expf(-x)); }

/* moe_block's routed part, src/model_fwd.c:992-1140; per unit expert_compute (852-876) / experts_batch (952-989).
 * Path per unit: decode numerics when the whole call has n <= 8 tokens (batch) or the unit has fewer than
 * GEMM_MIN_T tokens (lin_mm_after, 223-257), GEMM numerics otherwise. */
int orc_moe_routed(int H, int FF, int E, int topk, const uint16_t *router, const uint8_t *blobs, uint64_t blob_bytes,
                   uint64_t gu_bytes, int n, const float *xin, const float *bias, const float *logits_override, float *y,
                   float *logits_out, float *probs_out, int32_t *sel_out, float *w_out, int32_t *unit_expert_out,
                   float *moe_out, int q8_vnni) {
    float *lg = malloc(sizeof(float) * (size_t)n * E);
    if (logits_override) memcpy(lg, logits_override, sizeof(float) * (size_t)n * E);
    else {
        orc_router_logits(router, E, H, xin, n, lg);
        if (bias)
            for (int t = 0; t < n; t++)
                for (int e = 0; e < E; e++) lg[(size_t)t * E + e] = lg[(size_t)t * E + e] + bias[e];
    }
    if (logits_out) memcpy(logits_out, lg, sizeof(float) * (size_t)n * E);
    int32_t *sel = malloc(sizeof(int32_t) * (size_t)n * topk);
    float *wt = malloc(sizeof(float) * (size_t)n * topk);
    int *uid = malloc(sizeof(int) * (size_t)E), *order = malloc(sizeof(int) * (size_t)E), *cnt = calloc((size_t)E, sizeof(int));
    for (int e = 0; e < E; e++) uid[e] = -1;
    int nu = 0;
    for (int t = 0; t < n; t++) {
        float *pr = lg + (size_t)t * E;
        orc_softmax(pr, E);
        if (probs_out) memcpy(probs_out + (size_t)t * E, pr, sizeof(float) * (size_t)E);
        int32_t *st = sel + (size_t)t * topk;
        orc_topk(pr, E, topk, st);
        float sum = 0;
        for (int k = 0; k < topk; k++) sum = sum + pr[st[k]];
        for (int k = 0; k < topk; k++) {
            wt[(size_t)t * topk + k] = pr[st[k]] / sum;
            if (uid[st[k]] < 0) { uid[st[k]] = nu; order[nu++] = st[k]; }
            cnt[st[k]]++;
        }
    }
    if (sel_out) memcpy(sel_out, sel, sizeof(int32_t) * (size_t)n * topk);
    if (w_out) memcpy(w_out, wt, sizeof(float) * (size_t)n * topk);
    if (unit_expert_out) memcpy(unit_expert_out, order, sizeof(int32_t) * (size_t)nu);

    float *mo = moe_out ? moe_out : malloc(sizeof(float) * (size_t)n * topk * H);
    const int nkbH = (H + ORC_KB - 1) / ORC_KB, nkbF = (FF + ORC_KB - 1) / ORC_KB;
    int8_t *qx = malloc((size_t)n * H), *qd = malloc((size_t)n * FF);
    float *sx = malloc(sizeof(float) * (size_t)n * (H / ORC_GROUP + nkbH)), *bx = malloc(sizeof(float) * (size_t)n * H / ORC_GROUP);
    float *sd = malloc(sizeof(float) * (size_t)n * (FF / ORC_GROUP + nkbF)), *bd = malloc(sizeof(float) * (size_t)n * FF / ORC_GROUP);
    int32_t *sumx = malloc(sizeof(int32_t) * (size_t)n * nkbH), *sumd = malloc(sizeof(int32_t) * (size_t)n * nkbF);
    float *GU = malloc(sizeof(float) * (size_t)n * 2 * FF), *D = malloc(sizeof(float) * (size_t)n * H);
    int *tok = malloc(sizeof(int) * (size_t)n), *slot = malloc(sizeof(int) * (size_t)n);
    float *tw = malloc(sizeof(float) * (size_t)n);
    int rc = nu;
    for (int u = 0; u < nu && rc >= 0; u++) {
        const int e = order[u];
        int nt = 0;
        for (int t = 0; t < n; t++)
            for (int k = 0; k < topk; k++)
                if (sel[(size_t)t * topk + k] == e) { tok[nt] = t; slot[nt] = t * topk + k; tw[nt] = wt[(size_t)t * topk + k]; nt++; }
        orc_qmat gu, dn;
        const uint8_t *blob = blobs + (size_t)e * blob_bytes;
        if (!orc_qmat_view(&gu, blob) || !orc_qmat_view(&dn, blob + gu_bytes) || gu.rows != 2 * FF || gu.cols != H ||
            dn.rows != H || dn.cols != FF) { rc = -1; break; }
        const int decode = n <= 8 || nt < ORC_GEMM_MIN_T;
        for (int i = 0; i < nt; i++) {
            const float *x = xin + (size_t)tok[i] * H;
            if (decode) {
                orc_act_quantize(x, H, gu.rot_block, gu.rot_seed, qx, sx, bx);
                orc_matvec_decode(&gu, qx, sx, bx, GU + (size_t)i * 2 * FF, q8_vnni);
            } else orc_xq(x, H, gu.rot_block, gu.rot_seed, qx + (size_t)i * H, sx + (size_t)i * nkbH, sumx + (size_t)i * nkbH);
        }
        if (!decode) orc_matmul_gemm(&gu, nt, qx, sx, sumx, GU);
        for (int i = 0; i < nt; i++) {
            float *g = GU + (size_t)i * 2 * FF;
            for (int c = 0; c < FF; c++) g[c] = siluf(g[c]) * g[FF + c];
            if (decode) {
                orc_act_quantize(g, FF, dn.rot_block, dn.rot_seed, qd, sd, bd);
                orc_matvec_decode(&dn, qd, sd, bd, D + (size_t)i * H, q8_vnni);
            } else orc_xq(g, FF, dn.rot_block, dn.rot_seed, qd + (size_t)i * FF, sd + (size_t)i * nkbF, sumd + (size_t)i * nkbF);
        }
        if (!decode) orc_matmul_gemm(&dn, nt, qd, sd, sumd, D);
        for (int i = 0; i < nt; i++) {
            float *o = mo + (size_t)slot[i] * H;
            for (int c = 0; c < H; c++) o[c] = tw[i] * D[(size_t)i * H + c];
        }
    }
    if (rc >= 0)
        for (int t = 0; t < n; t++) {                 /* rank-order combine, src/model_fwd.c:1134-1140 */
            float *yt = y + (size_t)t * H;
            for (int c = 0; c < H; c++) yt[c] = 0;
            for (int k = 0; k < topk; k++) {
                const float *o = mo + ((size_t)t * topk + k) * H;
                for (int c = 0; c < H; c++) yt[c] = yt[c] + o[c];
            }
        }
    if (!moe_out) free(mo);
    free(lg); free(sel); free(wt); free(uid); free(order); free(cnt);
    free(qx); free(qd); free(sx); free(bx); free(sd); free(bd); free(sumx); free(sumd); free(GU); free(D);
    free(tok); free(slot); free(tw);
    return rc;
}

/* ---------------- hyper-connections around the layer ---------------- */

/* dot_f32, src/model_fwd.c:24-34: two 8-lane fma accumulators over 16-element blocks (s0: elements 16i + l, s1:
 * 16i + 8 + l), added lane-wise, then hsum256_ps. n % 16 == 0 here (4H and H), so the scalar tail never runs. */
static float dot_f32(const float *a, const float *b, int n) {
    float s0[8] = {0, 0, 0, 0, 0, 0, 0, 0}, s1[8] = {0, 0, 0, 0, 0, 0, 0, 0}, v[8];
    for (int i = 0; i + 16 <= n; i += 16)
        for (int l = 0; l < 8; l++) {
            s0[l] = fmaf(a[i + l], b[i + l], s0[l]);
            s1[l] = fmaf(a[i + 8 + l], b[i + 8 + l], s1[l]);
        }
    for (int l = 0; l < 8; l++) v[l] = s0[l] + s1[l];
    return hsum8(v);
}

/* sigmoidf, src/model_fwd.c:42 (glibc expf) */
static float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

/* sigmoid256, src/model_fwd.c:397-400, one lane: 1 / (1 + exp256_ps(0 - x)) */
static float sigmoid_cephes(float x) { return 1.0f / (1.0f + cephes_exp(0.0f - x)); }

/* hc_in, src/model_fwd.c:404-439 with rmsnorm 37-40 (eps 1e-6f, src/model.h:18) and lin_mm's F16 path (the
 * router's numerics, inz_matvec_f16_rows / inz_matmul_f16_rows). W = 4H; rank = 320 (Q_HC_RANK). */
void orc_hc_in(int H, int rank, const float *norm, const uint16_t *down, const uint16_t *up, const float *inject,
               int n, const float *X, float *xin, float *inj) {
    const int W = 4 * H;
    float *Xn = calloc((size_t)n * W, sizeof(float)), *d = malloc(sizeof(float) * (size_t)n * rank);
    float *m = malloc(sizeof(float) * (size_t)n * W);
    for (int t = 0; t < n; t++)
        for (int s = 0; s < 4; s++) {
            const float *x = X + (size_t)t * W + (size_t)s * H;
            float *o = Xn + (size_t)t * W + (size_t)s * H;
            const float r = 1.0f / sqrtf(dot_f32(x, x, H) / (float)H + 1e-6f);
            for (int i = 0; i < H; i++) o[i] = x[i] * r * norm[s * H + i];
        }
    orc_router_logits(down, rank, W, Xn, n, d);
    for (size_t i = 0; i < (size_t)n * rank; i++) d[i] = siluf(d[i] / 4.0f);
    orc_router_logits(up, W, rank, d, n, m);
    for (int t = 0; t < n; t++) {
        const float *mt = m + (size_t)t * W, *xt = Xn + (size_t)t * W;
        for (int i = 0; i < H; i++) {
            float acc = 0.0f;
            for (int s = 0; s < 4; s++) acc = fmaf(sigmoid_cephes(mt[s * H + i]), xt[s * H + i], acc);
            xin[(size_t)t * H + i] = acc * 0.25f;
        }
        if (inj)
            for (int s = 0; s < 4; s++) inj[t * 4 + s] = 2.0f * sigmoidf_(dot_f32(inject + (size_t)s * W, xt, W) / 4.0f);
    }
    free(Xn); free(d); free(m);
}

/* hc_out, src/model_fwd.c:442-450: X_s += inj_s * y, one fma per element (the reference build contracts it) */
void orc_hc_out(int H, int n, float *X, const float *inj, const float *y) {
    for (int t = 0; t < n; t++)
        for (int s = 0; s < 4; s++) {
            float *x = X + (size_t)t * 4 * H + (size_t)s * H;
            const float w = inj[t * 4 + s];
            for (int i = 0; i < H; i++) x[i] = fmaf(w, y[(size_t)t * H + i], x[i]);
        }
}

/* ---------------- seeded synthetic inputs (tests/test_quant.c:10-17) ---------------- */

#define LCG_A 6364136223846793005ull
#define LCG_C 1442695040888963407ull

static float synth_randn(uint64_t *s) {
    double u1, u2;
    *s = *s * LCG_A + LCG_C;
    u1 = ((*s >> 11) + 1.0) / 9007199254740993.0;
    *s = *s * LCG_A + LCG_C;
    u2 = (*s >> 11) / 9007199254740992.0;
    return (float)(sqrt(-2 * log(u1)) * cos(2 * M_PI * u2));
}

/* the state after n steps of s -> s * A + C, composing the affine map by repeated squaring */
uint64_t orc_synth_jump(uint64_t s, uint64_t n_normals) {
    uint64_t n = 2 * n_normals, ma = 1, mc = 0, a = LCG_A, c = LCG_C;
    for (; n; n >>= 1) {
        if (n & 1) {
            ma *= a;
            mc = mc * a + c;
        }
        c = c * a + c;
        a *= a;
    }
    return s * ma + mc;
}

uint64_t orc_synth_randn(uint64_t state, int64_t n, float scale, float *out) {
    for (int64_t i = 0; i < n; i++) out[i] = synth_randn(&state) * scale;
    return state;
}

void orc_synth_expert(uint64_t seed, int H, int FF, int e, float *gu, float *dn) {
    const uint64_t per = (uint64_t)3 * FF * H;
    const float sd = (float)sqrt(1.0 / H);
    uint64_t s = orc_synth_jump(seed, per * (uint64_t)e);
    for (size_t i = 0; i < (size_t)2 * FF * H; i++) gu[i] = synth_randn(&s) * sd;
    for (size_t i = 0; i < (size_t)H * FF; i++) dn[i] = synth_randn(&s) * sd;
}

void orc_synth_router(uint64_t seed, int E, int H, uint16_t *w) {
    uint64_t s = seed;
    for (size_t i = 0; i < (size_t)E * H; i++) w[i] = _cvtss_sh(synth_randn(&s) * 0.02f, 0);
}

void orc_synth_hidden(uint64_t seed, int n, int H, float *x) {
    uint64_t s = seed;
    for (int t = 0; t < n; t++) {
        float *r = x + (size_t)t * H;
        double ss = 0;
        for (int i = 0; i < H; i++) {
            r[i] = synth_randn(&s);
            ss += (double)r[i] * r[i];
        }
        const float k = (float)(1.0 / sqrt(ss / H + 1e-6));
        for (int i = 0; i < H; i++) r[i] = r[i] * k;
    }
}
