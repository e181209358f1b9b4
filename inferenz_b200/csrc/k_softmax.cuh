// k_softmax.cuh -- per-token softmax (Cephes exp, 8-lane sum), top-k and renormalised weights, one warp per token.
// softmax_inplace (src/vmath.h:9-60), topk_f32 (src/sampler.c:95-127: value desc, index asc), weights
// (src/model_fwd.c:1006-1011, 1028: sum left to right, w_k = p_k / sum). Shared by k_router.cu and k_route.cu.
#pragma once

#include "inzg_internal.h"

namespace inzg {

// exp256_ps (Cephes), src/vmath.h:9-25, one lane
__device__ __forceinline__ float cephes_exp(float x) {
    x = fminf(fmaxf(x, -87.3f), 88.3f);
    const float fx = rintf(__fmul_rn(x, 1.44269504088896341f));
    x = __fmaf_rn(-fx, 0.693359375f, x);
    x = __fmaf_rn(-fx, -2.12194440e-4f, x);
    const float z = __fmul_rn(x, x);
    float y = 1.9875691500e-4f;
    y = __fmaf_rn(y, x, 1.3981999507e-3f);
    y = __fmaf_rn(y, x, 8.3334519073e-3f);
    y = __fmaf_rn(y, x, 4.1665795894e-2f);
    y = __fmaf_rn(y, x, 1.6666665459e-1f);
    y = __fmaf_rn(y, x, 5.0000001201e-1f);
    y = __fadd_rn(__fmaf_rn(y, z, x), 1.0f);
    return __fmul_rn(y, __int_as_float(((int)fx + 127) << 23));
}

constexpr int kMaxPerLane = 32;  // E <= 1024, E % 32 == 0

// order-preserving map of a float to an unsigned key (for warp max reductions on redux.sync)
__device__ __forceinline__ uint32_t f2ord(float x) {
    const uint32_t b = __float_as_uint(x);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float ord2f(uint32_t k) { return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k); }

// One warp, one token: lg [E] logits -> sel [topk], w [topk]; ex: E floats of shared scratch for this warp;
// probs (optional) [E]. Lane j holds elements j + 32 m.
// Top-k: k rounds; each lane keeps its best untaken probability (ties: smaller m, i.e. smaller index), the warp
// takes the largest value (redux max over the probability bits + 1; probabilities are >= 0, so the bits are
// ordered) and, among the lanes holding it, the smallest index (redux min) -- the reference's (value desc, index asc).
__device__ __forceinline__ void softmax_topk_warp(const float *__restrict__ lg, int E, int topk, float *ex,
                                                  float *__restrict__ probs, int32_t *sel, float *w) {
    const int lane = threadIdx.x & 31, per = E / 32;
    float v[kMaxPerLane];
    uint32_t mk = 0;
#pragma unroll
    for (int m = 0; m < kMaxPerLane; m++)
        if (m < per) {
            v[m] = lg[lane + 32 * m];
            mk = max(mk, f2ord(v[m]));
        }
    const float mx = ord2f(__reduce_max_sync(0xffffffffu, mk));
#pragma unroll
    for (int m = 0; m < kMaxPerLane; m++)
        if (m < per) {
            v[m] = cephes_exp(__fsub_rn(v[m], mx));
            ex[lane + 32 * m] = v[m];
        }
    __syncwarp();
    // 8 lane sums: accumulator l adds elements l, l+8, l+16, ... in order (the reference's 8-wide running sum)
    float part = 0.0f;
    if (lane < 8) {
#pragma unroll 8
        for (int i = lane; i < E; i += 8) part = __fadd_rn(part, ex[i]);
    }
    const float sum = __shfl_sync(0xffffffffu, hsum8_lanes(part), 0);
    const float inv = __fdiv_rn(1.0f, sum);
#pragma unroll
    for (int m = 0; m < kMaxPerLane; m++)
        if (m < per) {
            v[m] = __fmul_rn(v[m], inv);
            if (probs) probs[lane + 32 * m] = v[m];
        }
    unsigned taken = 0;  // bit m: element lane + 32 m already selected
    float wsum = 0.0f, wk = 0.0f;
    int ik = 0;
    for (int k = 0; k < topk; k++) {
        uint32_t bk = 0;
        int bm = 0;
#pragma unroll
        for (int m = 0; m < kMaxPerLane; m++)
            if (m < per && !((taken >> m) & 1u)) {
                const uint32_t key = __float_as_uint(v[m]) + 1u;
                if (key > bk) { bk = key; bm = m; }
            }
        const uint32_t wmax = __reduce_max_sync(0xffffffffu, bk);
        const uint32_t widx = __reduce_min_sync(0xffffffffu, bk == wmax ? (uint32_t)(lane + 32 * bm) : 0xFFFFFFFFu);
        if ((int)(widx & 31) == lane) taken |= 1u << (widx >> 5);
        const float pv = __uint_as_float(wmax - 1u);
        wsum = __fadd_rn(wsum, pv);            // identical in every lane: (((0 + p0) + p1) + ...)
        if (lane == k) { wk = pv; ik = (int)widx; }  // lane k keeps rank k (topk <= 16)
    }
    if (lane < topk) {
        sel[lane] = ik;
        w[lane] = __fdiv_rn(wk, wsum);
    }
}

}  // namespace inzg
