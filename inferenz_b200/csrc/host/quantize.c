/*
 * quantize.c -- the engine's offline quantizer for expert matrices (Q4L, Q8G), host side of libinzg.
 *
 * Produces byte-identical output to the reference quantizer inz_quantize (src/quant.c:422-556) with the converter's
 * recipe (src/convert.c:190-200), so that expert blobs built here on a GPU host equal the ones the reference
 * converter writes. Scalar C; the reference's 8-lane AVX accumulations are kept lane by lane where their order
 * changes a float result (fit_group's num/den/err sums and their hsum8 tree). Threads: OpenMP over rows.
 */
#include "inzg_host.h"

#include <float.h>
#include <omp.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#define QMAGIC 0x515A4E49u
#define GROUP 64
#define LUT_BIAS 64

static size_t group_bytes(int type) { return type == INZG_T_Q4L ? 32 : type == INZG_T_Q8G ? 64 : 0; }

INZG_API size_t inzg_qmat_bytes(int type, int rows, int cols) {
    size_t ng = (size_t)cols / GROUP;
    size_t n = 64 + (size_t)rows * ng * group_bytes(type) + (size_t)rows * ng * 2;
    return (n + 63) / 64 * 64;
}

/* largest power of two <= 256 dividing cols, at least 64 (src/quant.c:166-170) */
INZG_API int inzg_auto_rot_block(int cols) {
    for (int b = 256; b >= GROUP; b >>= 1)
        if (cols % b == 0) return b;
    return 0;
}

static float rot_sign(uint32_t seed, uint32_t i) {
    uint32_t h = (i + 1) * 0x9E3779B1u ^ seed;
    h ^= h >> 15; h *= 0x2C1B3C6Du; h ^= h >> 12; h *= 0x297A2D39u; h ^= h >> 15;
    return (h & 1) ? -1.0f : 1.0f;
}

/* the randomized Hadamard rotation of src/quant.c:118-154 */
static void rotate(float *x, int n, int block, uint32_t seed) {
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

static float hsum8(const float a[8]) {
    float b0 = a[0] + a[4], b1 = a[1] + a[5], b2 = a[2] + a[6], b3 = a[3] + a[7];
    return (b0 + b2) + (b1 + b3);
}

/* sorted levels and the midpoints between neighbours; assignment = number of midpoints strictly below v
 * (src/quant.c:189-211; the midpoints of sorted levels are sorted, so a binary search counts them) */
typedef struct {
    int nl;
    float lmax;
    float L[16], T[15];
} lvlset;

static void lvlset_init(lvlset *ls, const float *L, int nl) {
    ls->nl = nl;
    ls->lmax = 0;
    for (int k = 0; k < nl; k++) {
        ls->lmax = fmaxf(ls->lmax, fabsf(L[k]));
        ls->L[k] = L[k];
    }
    for (int k = 0; k + 1 < nl; k++) ls->T[k] = 0.5f * (L[k] + L[k + 1]);
}

static inline int lvl_assign(const lvlset *ls, float v) {
    int c = 0;                            /* number of midpoints strictly below v (NaN: none) */
    for (int k = 0; k + 1 < ls->nl; k++) c += v > ls->T[k];
    return c;
}

/* levels of the 64 elements of x * inv: idx[j] and lv[j] = L[idx[j]] (vectorisable form of lvl_assign) */
static inline void assign64(const lvlset *ls, const float *x, float inv, uint8_t *idx, float *lv) {
    int c[GROUP];
    for (int j = 0; j < GROUP; j++) c[j] = 0;
    for (int k = 0; k + 1 < ls->nl; k++) {
        const float t = ls->T[k];
        for (int j = 0; j < GROUP; j++) c[j] += x[j] * inv > t;
    }
    for (int j = 0; j < GROUP; j++) {
        idx[j] = (uint8_t)c[j];
        lv[j] = ls->L[c[j]];
    }
}

/* scale and indices of one 64-weight group (src/quant.c:232-296); the eight vector registers of the reference hold
 * elements 8j + lane, so lane = element % 8 and the per-lane sums run over j in order */
static float fit_group(const float *x, const float *w, const lvlset *ls, float *d_out, uint8_t *idx) {
    float amax = 0;
    for (int j = 0; j < GROUP; j++) amax = fmaxf(amax, fabsf(x[j]));
    if (amax == 0 || ls->lmax == 0) {
        *d_out = 0;
        memset(idx, lvl_assign(ls, 0.0f), GROUP);
        return 0;
    }
    static const float cand[] = {0.82f, 0.88f, 0.94f, 1.0f, 1.06f};
    float best_err = FLT_MAX, best_d = amax / ls->lmax;
    uint8_t best_i[GROUP], I[GROUP];
    float lv[GROUP];
    for (size_t c = 0; c < sizeof(cand) / sizeof(cand[0]); c++) {
        float d = amax / ls->lmax * cand[c];
        float inv = 1.0f / d;
        float num[8] = {0, 0, 0, 0, 0, 0, 0, 0}, den[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        assign64(ls, x, inv, I, lv);
        for (int jj = 0; jj < GROUP; jj += 8)
            for (int l = 0; l < 8; l++) {
                const float wl = w[jj + l] * lv[jj + l];
                num[l] = fmaf(wl, x[jj + l], num[l]);
                den[l] = fmaf(wl, lv[jj + l], den[l]);
            }
        const float dn = hsum8(den);
        if (dn > 0) d = hsum8(num) / dn;
        if (!(d > 0)) continue;
        inv = 1.0f / d;
        float err[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        assign64(ls, x, inv, I, lv);
        for (int jj = 0; jj < GROUP; jj += 8)
            for (int l = 0; l < 8; l++) {
                const float e = fmaf(-d, lv[jj + l], x[jj + l]);
                err[l] = fmaf(e * e, w[jj + l], err[l]);
            }
        const float er = hsum8(err);
        if (er < best_err) {
            best_err = er;
            best_d = d;
            memcpy(best_i, I, GROUP);
        }
    }
    if (best_err == FLT_MAX) {
        const float inv = 1.0f / best_d;
        best_err = 0;
        assign64(ls, x, inv, best_i, lv);
    }
    memcpy(idx, best_i, GROUP);
    *d_out = best_d;
    return best_err;
}

/* Lloyd-Max normalised Gaussian levels (src/quant.c:177-185), 4 bits */
static void gaussian_levels4(float *L) {
    static const float g4[] = {-2.7326f, -2.0690f, -1.6181f, -1.2562f, -0.9423f, -0.6568f, -0.3880f, -0.1284f,
                               0.1284f,  0.3880f,  0.6568f,  0.9423f,  1.2562f,  1.6181f,  2.0690f,  2.7326f};
    for (int i = 0; i < 16; i++) L[i] = g4[i] / g4[15];
}

/* weighted Lloyd-Max on a deterministic subsample of groups (src/quant.c:369-418); levels -63..63 */
static void learn_lut(const float *Wr, int rows, int cols, const float *imp, float *Lout) {
    const int nl = 16, ng = cols / GROUP, iters = 5;
    const int64_t total = (int64_t)rows * ng;
    int64_t ns = 8192;
    if (ns > total) ns = total;
    float L[16];
    gaussian_levels4(L);
    float *dsc = malloc(sizeof(float) * (size_t)ns);
    uint8_t *ix = malloc((size_t)ns * GROUP);
    const int64_t stride = total / ns;
    for (int it = 0; it < iters; it++) {
        lvlset ls;
        lvlset_init(&ls, L, nl);
        double num[16] = {0}, den[16] = {0};
        for (int64_t s = 0; s < ns; s++) {
            const int64_t gi = s * stride;
            const int r = (int)(gi / ng), g = (int)(gi % ng);
            const float *x = Wr + (size_t)r * cols + (size_t)g * GROUP;
            const float *w = imp + g * GROUP;
            fit_group(x, w, &ls, &dsc[s], ix + s * GROUP);
            const float d = dsc[s];
            if (d == 0) continue;
            for (int j = 0; j < GROUP; j++) {
                const int k = ix[s * GROUP + j];
                num[k] += (double)w[j] * d * x[j];
                den[k] += (double)w[j] * d * d;
            }
        }
        for (int k = 0; k < nl; k++)
            if (den[k] > 0) L[k] = (float)(num[k] / den[k]);
        for (int a = 1; a < nl; a++) {
            const float v = L[a];
            int b = a - 1;
            while (b >= 0 && L[b] > v) { L[b + 1] = L[b]; b--; }
            L[b + 1] = v;
        }
    }
    float lmax = 0;
    for (int k = 0; k < nl; k++) lmax = fmaxf(lmax, fabsf(L[k]));
    for (int k = 0; k < nl; k++) {
        int v = (int)lrintf(L[k] / lmax * 63.0f);
        v = v < -63 ? -63 : v > 63 ? 63 : v;
        Lout[k] = (float)v;
    }
    for (int k = 1; k < nl; k++)
        if (Lout[k] <= Lout[k - 1]) Lout[k] = Lout[k - 1] + 1;
    free(dsc);
    free(ix);
}

/* rot_block: 0 = automatic, < 0 = none, else the block. Q8G is rotated only for an explicit block
 * (src/quant.c:433-436). threads: OpenMP threads for the row loops (1 = single thread). Returns 0, or -1 for an
 * unsupported type / shape. */
INZG_API int inzg_quantize(const float *W, int rows, int cols, int type, int rot_block, uint32_t rot_seed, int threads,
                           void *out) {
    if ((type != INZG_T_Q4L && type != INZG_T_Q8G) || cols % GROUP || rows <= 0) return -1;
    const int ng = cols / GROUP;
    int rot = rot_block == 0 ? inzg_auto_rot_block(cols) : rot_block < 0 ? 0 : rot_block;
    if (rot && cols % rot) return -1;
    if (type == INZG_T_Q8G && rot_block <= 0) rot = 0;
    const uint32_t seed = rot_seed ? rot_seed : 0x5EEDu;
    const size_t bytes = inzg_qmat_bytes(type, rows, cols);
    memset(out, 0, bytes);
    uint8_t *h = out;
    const uint32_t magic = QMAGIC, urows = (uint32_t)rows, ucols = (uint32_t)cols;
    const uint16_t utype = (uint16_t)type, urot = (uint16_t)rot;
    memcpy(h, &magic, 4);
    memcpy(h + 4, &utype, 2);
    memcpy(h + 6, &urot, 2);
    memcpy(h + 8, &urows, 4);
    memcpy(h + 12, &ucols, 4);
    memcpy(h + 16, &seed, 4);
    h[20] = type == INZG_T_Q4L ? 4 : 8;
    uint8_t *qout = h + 64;
    uint16_t *dout = (uint16_t *)(qout + (size_t)rows * ng * group_bytes(type));
    float *imp = malloc(sizeof(float) * (size_t)cols);
    for (int j = 0; j < cols; j++) imp[j] = 1.0f;     /* no importance matrix */
    float *Wr = malloc(sizeof(float) * (size_t)rows * cols);
    const int nthr = threads > 0 ? threads : 0;
    #pragma omp parallel for schedule(static) if (nthr != 1) num_threads(nthr > 0 ? nthr : omp_get_max_threads())
    for (int r = 0; r < rows; r++) {
        memcpy(Wr + (size_t)r * cols, W + (size_t)r * cols, sizeof(float) * (size_t)cols);
        if (rot) rotate(Wr + (size_t)r * cols, cols, rot, seed);
    }
    if (type == INZG_T_Q8G) {
        #pragma omp parallel for schedule(static) if (nthr != 1) num_threads(nthr > 0 ? nthr : omp_get_max_threads())
        for (int r = 0; r < rows; r++)
            for (int g = 0; g < ng; g++) {
                const float *x = Wr + (size_t)r * cols + (size_t)g * GROUP;
                float amax = 0;
                for (int j = 0; j < GROUP; j++) amax = fmaxf(amax, fabsf(x[j]));
                const float d = amax / 127.0f, inv = d > 0 ? 1.0f / d : 0;
                uint8_t *o = qout + ((size_t)r * ng + g) * 64;
                for (int j = 0; j < GROUP; j++) {
                    int q = (int)lrintf(x[j] * inv);
                    q = q < -127 ? -127 : q > 127 ? 127 : q;
                    o[j] = (uint8_t)(q + 128);
                }
                dout[(size_t)r * ng + g] = inzg_f32_to_f16(d);
            }
    } else {
        float Lq[16];
        learn_lut(Wr, rows, cols, imp, Lq);
        for (int k = 0; k < 16; k++) h[24 + k] = (uint8_t)((int)Lq[k] + LUT_BIAS);
        lvlset ls;
        lvlset_init(&ls, Lq, 16);
        #pragma omp parallel for schedule(static) if (nthr != 1) num_threads(nthr > 0 ? nthr : omp_get_max_threads())
        for (int r = 0; r < rows; r++) {
            uint8_t idx[GROUP];
            for (int g = 0; g < ng; g++) {
                float d;
                fit_group(Wr + (size_t)r * cols + (size_t)g * GROUP, imp + g * GROUP, &ls, &d, idx);
                uint8_t *o = qout + ((size_t)r * ng + g) * 32;
                for (int i = 0; i < 32; i++) o[i] = (uint8_t)(idx[i] | (idx[i + 32] << 4));
                dout[(size_t)r * ng + g] = inzg_f32_to_f16(d);
            }
        }
    }
    free(Wr);
    free(imp);
    return 0;
}

/* One expert blob (src/convert.c:179-200, 565-584): gate|up [2FF][H] at 0, down [H][FF] at qmat_bytes(2FF, H),
 * zero padding to a 4 KiB multiple. Q8G rotated with the automatic block (the converter's rot8 default). */
INZG_API uint64_t inzg_blob_bytes(int type, int H, int FF) {
    const uint64_t b = inzg_qmat_bytes(type, 2 * FF, H) + inzg_qmat_bytes(type, H, FF);
    return (b + 4095) / 4096 * 4096;
}

INZG_API int inzg_encode_expert(const float *GU, const float *D, int type, int H, int FF, void *blob) {
    memset(blob, 0, inzg_blob_bytes(type, H, FF));
    const int rg = type == INZG_T_Q8G ? inzg_auto_rot_block(H) : 0;
    const int rd = type == INZG_T_Q8G ? inzg_auto_rot_block(FF) : 0;
    if (inzg_quantize(GU, 2 * FF, H, type, rg, 0, 1, blob)) return -1;
    return inzg_quantize(D, H, FF, type, rd, 0, 1, (uint8_t *)blob + inzg_qmat_bytes(type, 2 * FF, H));
}

/* Experts [e0, e1) of one synthetic layer, generated and encoded in parallel over experts:
 * blobs [e1-e0][blob_bytes]. */
INZG_API int inzg_synth_layer_blobs(uint64_t seed, int type, int H, int FF, int e0, int e1, void *blobs) {
    const uint64_t bb = inzg_blob_bytes(type, H, FF);
    int bad = 0;
    #pragma omp parallel for schedule(dynamic, 1) reduction(| : bad)
    for (int e = e0; e < e1; e++) {
        float *gu = malloc(sizeof(float) * (size_t)2 * FF * H), *dn = malloc(sizeof(float) * (size_t)H * FF);
        inzg_synth_expert(seed, H, FF, e, gu, dn);
        bad |= inzg_encode_expert(gu, dn, type, H, FF, (uint8_t *)blobs + (size_t)(e - e0) * bb) != 0;
        free(gu);
        free(dn);
    }
    return bad ? -1 : 0;
}

/* Only the listed experts of a synthetic layer are generated and encoded (in parallel); every other expert gets the
 * two matrix headers of the first listed one and a zero payload -- a valid blob that must not be routed to.
 * blobs: [E][blob_bytes], zero-filled here. Returns 0, or -1 on an encoding failure or a bad expert id. */
INZG_API int inzg_synth_layer_blobs_subset(uint64_t seed, int type, int H, int FF, int E, const int32_t *experts,
                                           int n_experts, void *blobs) {
    const uint64_t bb = inzg_blob_bytes(type, H, FF), gu_bytes = inzg_qmat_bytes(type, 2 * FF, H);
    uint8_t *out = blobs;
    memset(out, 0, bb * (size_t)E);
    if (n_experts <= 0) return -1;
    for (int i = 0; i < n_experts; i++)
        if (experts[i] < 0 || experts[i] >= E) return -1;
    int bad = 0;
    #pragma omp parallel for schedule(dynamic, 1) reduction(| : bad)
    for (int i = 0; i < n_experts; i++) {
        const int e = experts[i];
        float *gu = malloc(sizeof(float) * (size_t)2 * FF * H), *dn = malloc(sizeof(float) * (size_t)H * FF);
        inzg_synth_expert(seed, H, FF, e, gu, dn);
        bad |= inzg_encode_expert(gu, dn, type, H, FF, out + (size_t)e * bb) != 0;
        free(gu);
        free(dn);
    }
    if (bad) return -1;
    const uint8_t *src = out + (size_t)experts[0] * bb;
    for (int e = 0; e < E; e++) {
        uint8_t *dst = out + (size_t)e * bb;
        uint32_t magic;
        memcpy(&magic, dst, 4);
        if (magic == QMAGIC) continue;
        memcpy(dst, src, 64);
        memcpy(dst + gu_bytes, src + gu_bytes, 64);
    }
    return 0;
}
