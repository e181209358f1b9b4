// k_warpq.cuh -- warp-level activation rotation and int8 quantization (no block barriers), shared by k_act.cu and
// the fused decode kernel. Numerics: the reference's rotation (src/quant.c:118-154) and its decode / prefill
// activation quantizers (src/quant.c:611-637, 1407-1429).
#pragma once

#include "inzg_internal.h"

namespace inzg {

// Warp-level versions (no block barriers): one warp per row of NB rotation blocks of B = 32 * VPL elements; lane L
// holds elements b*B + L*VPL + r. Butterfly stage len pairs (i, i+len): inside a lane when len < VPL, else with lane
// L ^ (len / VPL) through a shuffle; the lower element gets a + b, the upper a - b, exactly as the reference.
template <int NB, int VPL>
__device__ __forceinline__ void warp_rotate(float (&v)[NB][VPL], uint32_t seed, float norm, int lane, int base = 0) {
    constexpr int B = 32 * VPL;
#pragma unroll
    for (int b = 0; b < NB; b++)
#pragma unroll
        for (int r = 0; r < VPL; r++)
            if (rot_sign_bit(seed, (uint32_t)(base + b * B + lane * VPL + r))) v[b][r] = -v[b][r];
#pragma unroll
    for (int len = 1; len < B; len <<= 1) {
        if (len < VPL) {
#pragma unroll
            for (int b = 0; b < NB; b++)
#pragma unroll
                for (int r = 0; r < VPL; r++)
                    if (!(r & len)) {
                        const float a = v[b][r], c = v[b][r + len];
                        v[b][r] = __fadd_rn(a, c);
                        v[b][r + len] = __fsub_rn(a, c);
                    }
        } else {
            const int lm = len / VPL;
            const bool upper = lane & lm;
#pragma unroll
            for (int b = 0; b < NB; b++)
#pragma unroll
                for (int r = 0; r < VPL; r++) {
                    const float o = __shfl_xor_sync(0xffffffffu, v[b][r], lm);
                    v[b][r] = upper ? __fsub_rn(o, v[b][r]) : __fadd_rn(v[b][r], o);
                }
        }
    }
#pragma unroll
    for (int b = 0; b < NB; b++)
#pragma unroll
        for (int r = 0; r < VPL; r++) v[b][r] = __fmul_rn(v[b][r], norm);
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    return (uint32_t)(a & 255) | ((uint32_t)(b & 255) << 8) | ((uint32_t)(c & 255) << 16) | ((uint32_t)(d & 255) << 24);
}

// decode numerics of a row held as v[NB][VPL] (64-groups span 64/VPL lanes): q64, sb = (s, bsum); prefill numerics
// (256-blocks, the last one partial): q256, s256
template <int NB, int VPL>
__device__ __forceinline__ void warp_quantize(const float (&v)[NB][VPL], int n, int lane, int8_t *q64, float2 *sb64,
                                              int8_t *q256, float *s256) {
    constexpr int B = 32 * VPL, LPG = kGroup / VPL;  // lanes per 64-group
    if (q64) {
#pragma unroll
        for (int b = 0; b < NB; b++) {
            float amax = 0.0f;
#pragma unroll
            for (int r = 0; r < VPL; r++) amax = fmaxf(amax, fabsf(v[b][r]));
#pragma unroll
            for (int o = 1; o < LPG; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const float s = __fdiv_rn(amax, 127.0f);
            const float inv = s > 0 ? __fdiv_rn(1.0f, s) : 0.0f;
            int q[VPL], sum = 0;
#pragma unroll
            for (int r = 0; r < VPL; r++) {
                q[r] = __float2int_rn(__fmul_rn(v[b][r], inv));
                sum += q[r];
            }
#pragma unroll
            for (int o = 1; o < LPG; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            const int j0 = b * B + lane * VPL, g = j0 / kGroup;
#pragma unroll
            for (int r = 0; r < VPL; r += 4)
                *reinterpret_cast<uint32_t *>(q64 + j0 + r) = pack4(q[r], q[r + 1], q[r + 2], q[r + 3]);
            if ((lane % LPG) == 0) sb64[g] = make_float2(s, __fmul_rn(s, (float)sum));
        }
    }
    if (q256) {
        constexpr int BPK = kKB / B;  // rotation blocks per 256-block
#pragma unroll
        for (int kb = 0; kb < (NB + BPK - 1) / BPK; kb++) {
            float amax = 0.0f;
#pragma unroll
            for (int b = kb * BPK; b < kb * BPK + BPK && b < NB; b++)
#pragma unroll
                for (int r = 0; r < VPL; r++) amax = fmaxf(amax, fabsf(v[b][r]));
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const float s = __fdiv_rn(amax, 127.0f);
            const float inv = s > 0 ? __fdiv_rn(1.0f, s) : 0.0f;
#pragma unroll
            for (int b = kb * BPK; b < kb * BPK + BPK && b < NB; b++)
#pragma unroll
                for (int r = 0; r < VPL; r += 4) {
                    int q[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) q[i] = __float2int_rn(__fmul_rn(v[b][r + i], inv));
                    *reinterpret_cast<uint32_t *>(q256 + b * B + lane * VPL + r) = pack4(q[0], q[1], q[2], q[3]);
                }
            if (lane == 0) s256[kb] = s;
        }
    }
    (void)n;
}

}  // namespace inzg
