/*
 * synth.c -- seeded synthetic inputs for the MoE layer (host side of libinzg).
 *
 * Generator: the LCG + Box-Muller normal of the reference's own tests (tests/test_quant.c:10-17), with a jump-ahead
 * so that the draws of one expert can start on any thread at the state the sequential generator would have there.
 * Draw order for one layer (seed = layer index): per expert e = 0..E-1, gate [FF][H], up [FF][H], down [H][FF],
 * row-major, each value randn * sqrt(1/H) in fp32 -- the configuration's "N(0, 1/d) fp32 from seed 0".
 */
#include "inzg_host.h"

#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define LCG_A 6364136223846793005ull
#define LCG_C 1442695040888963407ull

/* state after n steps of s -> s * A + C (mod 2^64), by squaring the affine map */
static uint64_t lcg_jump(uint64_t s, uint64_t n) {
    uint64_t acc_a = 1, acc_c = 0, a = LCG_A, c = LCG_C;
    while (n) {
        if (n & 1) { acc_a *= a; acc_c = acc_c * a + c; }
        c = c * a + c;
        a *= a;
        n >>= 1;
    }
    return s * acc_a + acc_c;
}

static float randn(uint64_t *s) {
    double u1, u2;
    *s = *s * LCG_A + LCG_C;
    u1 = ((*s >> 11) + 1.0) / 9007199254740993.0;
    *s = *s * LCG_A + LCG_C;
    u2 = (*s >> 11) / 9007199254740992.0;
    return (float)(sqrt(-2 * log(u1)) * cos(2 * M_PI * u2));
}

INZG_API uint64_t inzg_synth_jump(uint64_t state, uint64_t n_normals) { return lcg_jump(state, 2 * n_normals); }

INZG_API uint64_t inzg_synth_randn(uint64_t state, int64_t n, float scale, float *out) {
    for (int64_t i = 0; i < n; i++) out[i] = randn(&state) * scale;
    return state;
}

/* fp32 -> IEEE half, round to nearest even (the reference's _cvtss_sh(x, 0), src/util.c:117) */
INZG_API uint16_t inzg_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u | ((ax >> 13) & 0x3FFu) : 0));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);          /* rounds to >= 65520: infinity */
    if (ax < 0x38800000u) {                                             /* half subnormal: q * 2^-24 */
        if (ax < 0x33000000u) return (uint16_t)sign;                    /* below 2^-25: rounds to zero */
        const uint32_t e = ax >> 23, m = (ax & 0x7FFFFFu) | 0x800000u;
        const uint32_t sh = 126 - e;                                    /* q = m * 2^(e-126), shift 14..24 */
        uint32_t q = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1), mid = 1u << (sh - 1);
        if (rem > mid || (rem == mid && (q & 1))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t h = ((ax >> 13) - (112u << 10));                           /* rebias exponent 127 -> 15 */
    const uint32_t rem = ax & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) h++;
    return (uint16_t)(sign | h);
}

/* One expert of one layer: gate|up [2FF][H] (gate rows, then up rows) and down [H][FF], drawn from the stream of
 * the layer's seed at the offset where the sequential generator reaches expert e. */
INZG_API void inzg_synth_expert(uint64_t seed, int H, int FF, int e, float *gu, float *dn) {
    const uint64_t per = (uint64_t)3 * FF * H;                         /* normals per expert */
    const float sd = (float)sqrt(1.0 / H);
    uint64_t s = lcg_jump(seed, 2 * per * (uint64_t)e);
    for (size_t i = 0; i < (size_t)2 * FF * H; i++) gu[i] = randn(&s) * sd;
    for (size_t i = 0; i < (size_t)H * FF; i++) dn[i] = randn(&s) * sd;
}

/* Router [E][H] f16 from N(0, 0.02^2) (fp32 draw, then round to half). */
INZG_API void inzg_synth_router(uint64_t seed, int E, int H, uint16_t *w) {
    uint64_t s = seed;
    for (size_t i = 0; i < (size_t)E * H; i++) w[i] = inzg_f32_to_f16(randn(&s) * 0.02f);
}

/* Hidden states [n][H] from N(0, 1), each row RMS-normalised without weight (x / sqrt(mean(x^2) + 1e-6)). */
INZG_API void inzg_synth_hidden(uint64_t seed, int n, int H, float *x) {
    uint64_t s = seed;
    for (int t = 0; t < n; t++) {
        float *r = x + (size_t)t * H;
        double ss = 0;
        for (int i = 0; i < H; i++) { r[i] = randn(&s); ss += (double)r[i] * r[i]; }
        const float k = (float)(1.0 / sqrt(ss / H + 1e-6));
        for (int i = 0; i < H; i++) r[i] = r[i] * k;
    }
}

void inzg__synth_experts_host(uint64_t seed, int H, int FF, const int32_t *experts, int n, float *gu, float *dn) {
    #pragma omp parallel for schedule(dynamic, 1)
    for (int i = 0; i < n; i++)
        inzg_synth_expert(seed, H, FF, experts[i], gu + (size_t)i * 2 * FF * H, dn + (size_t)i * H * FF);
}
