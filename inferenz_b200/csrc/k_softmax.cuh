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

// One warp, one token: lg [E] logits -> sel [topk], w [topk]; ex: E floats of shared scratch for this warp;
// probs (optional) [E]. Lane j holds elements j + 32 m.
__device__ __forceinline__ void softmax_topk_warp(const float *__restrict__ lg, int E, int topk, float *ex,
                                                  float *__restrict__ probs, int32_t *sel, float *w) {
    const int lane = threadIdx.x & 31, per = E / 32;
    float v[kMaxPerLane];
    float mx = -INFINITY;
#pragma unroll
    for (int m = 0; m < kMaxPerLane; m++)
        if (m < per) {
            v[m] = lg[lane + 32 * m];
            mx = v[m] > mx ? v[m] : mx;
        }
    for (int o = 16; o; o >>= 1) {
        const float q = __shfl_xor_sync(0xffffffffu, mx, o);
        mx = q > mx ? q : mx;
    }
#pragma unroll
    for (int m = 0; m < kMaxPerLane; m++)
        if (m < per) {
            v[m] = cephes_exp(__fsub_rn(v[m], mx));
            ex[lane + 32 * m] = v[m];
        }
    __syncwarp();
    // 8 lane sums: accumulator l adds elements l, l+8, l+16, ... in order (the reference's 8-wide running sum)
    float part = 0.0f;
    if (lane < 8)
        for (int i = lane; i < E; i += 8) part = __fadd_rn(part, ex[i]);
    const float sum = __shfl_sync(0xffffffffu, hsum8_lanes(part), 0);
    const float inv = __fdiv_rn(1.0f, sum);
#pragma unroll
    for (int m = 0; m < kMaxPerLane; m++)
        if (m < per) {
            v[m] = __fmul_rn(v[m], inv);
            if (probs) probs[lane + 32 * m] = v[m];
        }
    // top-k: k rounds of a warp arg-max under (value desc, index asc); the winner is removed by its owner
    unsigned taken = 0;  // bit m: element lane + 32 m already selected
    float wsum = 0.0f;
    float wk = 0.0f;
    int ik = 0;
    for (int k = 0; k < topk; k++) {
        float bv = -INFINITY;
        int bi = 0x7FFFFFFF;
#pragma unroll
        for (int m = 0; m < kMaxPerLane; m++)
            if (m < per && !((taken >> m) & 1u)) {
                const int i = lane + 32 * m;
                if (v[m] > bv || (v[m] == bv && i < bi)) { bv = v[m]; bi = i; }
            }
        for (int o = 16; o; o >>= 1) {
            const float qv = __shfl_xor_sync(0xffffffffu, bv, o);
            const int qi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (qv > bv || (qv == bv && qi < bi)) { bv = qv; bi = qi; }
        }
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
        wsum = __fadd_rn(wsum, bv);          // identical in every lane: (((0 + p0) + p1) + ...)
        if (lane == k) { wk = bv; ik = bi; }  // lane k keeps rank k (topk <= 16)
    }
    if (lane < topk) {
        sel[lane] = ik;
        w[lane] = __fdiv_rn(wk, wsum);
    }
}

}  // namespace inzg
