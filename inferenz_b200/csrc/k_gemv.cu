// k_gemv.cu -- decode-path grouped GEMV over the routed experts (Q4L / Q8G), sm_100a.
//
// Experts with fewer than 12 tokens (every expert when n <= 8) take the reference's decode numerics
// (src/quant.c:611-671, 767-953): int8 activations per 64-group (scale s_g), weights = LUT level (Q4L, biased by 64)
// or byte (Q8G, biased by 128) with an fp16 scale d_g per 64-group, and per row and token
//     y = sum_g d_g * s_g * (sum_j u_j q_j - bias * sum_j q_j).
// The integer group dots are exact; they run on the int8 tensor pipe (mma.m16n8k32, u8 weights x s8 activations,
// s32 accumulate -- one 16-row x 8-token tile per warp and 64-column group), the bias is removed with the group's
// exact integer sum of q, and each group is folded into fp32 with one fma per element. The reference keeps 8
// accumulation lanes per row and adds the bias in float; the values are the same integers and the same scales,
// summed in another order, so results agree to about 1e-7 relative (tests/test_gpu_parity.py).
//
// Work: items = (decode expert, 16-row tile); one warp per item, warps run free and load the next 4 groups' weights
// while the current 4 compute. Activations of the (<= 11) tokens come from L1.
#include "inzg_internal.h"
#include "k_launch.h"

#include <cuda_fp16.h>

namespace inzg {


__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// 4 nibble selectors (bits 0..15 of w) -> 4 LUT bytes. Levels are <= 127, so a selector with bit 3 set makes PRMT
// replicate a zero sign bit: each half-table lookup yields 0 where the other half applies.
__device__ __forceinline__ uint32_t lut16(uint32_t w, uint4 T) {
    return prmt(T.x, T.y, w) | prmt(T.z, T.w, w ^ 0x88888888u);
}

__device__ __forceinline__ float h2f16(uint32_t bits) { return __half2float(__ushort_as_half((unsigned short)bits)); }


__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// KIND 0: gate|up, activation row = token, output GU[entry][row]. KIND 1: down, activation row = entry, output
// moe_out[slot][row] = w * y. NT: token tiles of 8 (1, or 2 when an expert can hold up to 11 tokens).
template <bool Q8, int NG, int KIND, int NT>
__global__ void __launch_bounds__(128) gemv_mma_kernel(const uint8_t *__restrict__ pool, uint64_t slab_bytes,
                                                       MatLayout M, const uint8_t *__restrict__ luts, int lut_off,
                                                       RouteDev R, const int8_t *__restrict__ aq,
                                                       const int2 *__restrict__ asq, float *__restrict__ out,
                                                       int out_ld, int meta_items) {
    constexpr int K = NG * kGroup, GD = (NG + 3) / 4, WV = Q8 ? 2 : 1;  // uint4 per lane per group
    constexpr int BIAS = Q8 ? 128 : kLutBias;
    const int nitems = R.meta[meta_items];
    const int per = M.rows / 16;
    const int lane = threadIdx.x & 31, gr = lane >> 2, t = lane & 3;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), nw = gridDim.x * (blockDim.x >> 5);
    for (int item = gw; item < nitems; item += nw) {
        const int u = item / per, rt = item % per;
        const int e = R.dec_units[u];
        const int base = R.off[e], ntok = min(R.cnt[e], 8 * NT);
        const uint8_t *slab = pool + (size_t)e * slab_bytes;
        const uint4 *aw = reinterpret_cast<const uint4 *>(slab + M.q_off) + (size_t)rt * NG * 32 * WV + lane * WV;
        const uint4 *ad = reinterpret_cast<const uint4 *>(slab + M.d_off) + (size_t)rt * GD * 8 + gr;
        uint4 T = make_uint4(0, 0, 0, 0);
        if (!Q8) T = __ldg(reinterpret_cast<const uint4 *>(luts + (size_t)e * 32 + lut_off));
        // B operand: token gr (+8 per tile); C columns: tokens 2t, 2t+1 (+8 per tile)
        int brow[NT], crow[NT][2];
        bool bok[NT], cok[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const int bt = nt * 8 + gr, c0 = nt * 8 + 2 * t;
            bok[nt] = bt < ntok;
            brow[nt] = bok[nt] ? (KIND == 0 ? R.etok[base + bt] : base + bt) : 0;
#pragma unroll
            for (int j = 0; j < 2; j++) {
                cok[nt][j] = c0 + j < ntok;
                crow[nt][j] = cok[nt][j] ? (KIND == 0 ? R.etok[base + c0 + j] : base + c0 + j) : 0;
            }
        }
        const bool tile2 = NT == 2 && ntok > 8;
        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) acc[nt][i] = 0.0f;
        uint4 wcur[4][WV], wnxt[4][WV];
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int v = 0; v < WV; v++) wcur[j][v] = j < NG ? __ldg(aw + (size_t)j * 32 * WV + v) : make_uint4(0, 0, 0, 0);
        for (int g4 = 0; g4 < GD; g4++) {
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int v = 0; v < WV; v++) {
                    const int g = (g4 + 1) * 4 + j;
                    wnxt[j][v] = g < NG ? __ldg(aw + (size_t)g * 32 * WV + v) : make_uint4(0, 0, 0, 0);
                }
            const uint4 dq = __ldg(ad + (size_t)g4 * 8);  // (d[r][g], d[r+8][g]) for the 4 groups
            const uint32_t dw[4] = {dq.x, dq.y, dq.z, dq.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int g = g4 * 4 + j;
                if (g < NG) {
                    uint32_t A1[4], A2[4];
                    if (Q8) {
                        const uint4 w0 = wcur[j][0], w1 = wcur[j][1];
                        A1[0] = w0.x; A1[1] = w1.x; A1[2] = w0.y; A1[3] = w1.y;
                        A2[0] = w0.z; A2[1] = w1.z; A2[2] = w0.w; A2[3] = w1.w;
                    } else {
                        const uint4 w = wcur[j][0];
                        A1[0] = lut16(w.x, T); A1[1] = lut16(w.z, T); A1[2] = lut16(w.y, T); A1[3] = lut16(w.w, T);
                        A2[0] = lut16(w.x >> 16, T); A2[1] = lut16(w.z >> 16, T);
                        A2[2] = lut16(w.y >> 16, T); A2[3] = lut16(w.w >> 16, T);
                    }
                    const float d0 = h2f16(dw[j] & 0xFFFFu), d8 = h2f16(dw[j] >> 16);
#pragma unroll
                    for (int nt = 0; nt < NT; nt++) {
                        if (nt == 1 && !tile2) continue;
                        const uint4 b = bok[nt] ? __ldg(reinterpret_cast<const uint4 *>(aq + (size_t)brow[nt] * K + g * kGroup) + t)
                                                : make_uint4(0, 0, 0, 0);
                        int D[4] = {0, 0, 0, 0};
                        mma_u8s8(D, A1[0], A1[1], A1[2], A1[3], b.x, b.y);
                        mma_u8s8(D, A2[0], A2[1], A2[2], A2[3], b.z, b.w);
                        const int2 q0 = __ldg(asq + (size_t)crow[nt][0] * NG + g);
                        const int2 q1 = __ldg(asq + (size_t)crow[nt][1] * NG + g);
                        const float sc0 = __int_as_float(q0.x), sc1 = __int_as_float(q1.x);
                        const int s0 = q0.y * BIAS, s1 = q1.y * BIAS;
                        acc[nt][0] = __fmaf_rn((float)(D[0] - s0), __fmul_rn(d0, sc0), acc[nt][0]);
                        acc[nt][1] = __fmaf_rn((float)(D[1] - s1), __fmul_rn(d0, sc1), acc[nt][1]);
                        acc[nt][2] = __fmaf_rn((float)(D[2] - s0), __fmul_rn(d8, sc0), acc[nt][2]);
                        acc[nt][3] = __fmaf_rn((float)(D[3] - s1), __fmul_rn(d8, sc1), acc[nt][3]);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int v = 0; v < WV; v++) wcur[j][v] = wnxt[j][v];
        }
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int tok = nt * 8 + 2 * t + (i & 1);
                const int row = rt * 16 + gr + (i >> 1) * 8;
                if (tok < ntok) {
                    const int pos = base + tok;
                    if (KIND == 0) out[(size_t)pos * out_ld + row] = acc[nt][i];
                    else out[(size_t)R.eslot[pos] * out_ld + row] = __fmul_rn(R.ew[pos], acc[nt][i]);
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------
template <bool Q8, int NG, int KIND>
static void launch_one(const LayerDev &L, const MatLayout &M, const RouteDev &R, const int8_t *aq, const int2 *asq,
                       float *out, int out_ld, int meta_items, int maxt, int grid, cudaStream_t st) {
    const int lo = KIND == 0 ? 0 : 16;
    if (maxt <= 8)
        gemv_mma_kernel<Q8, NG, KIND, 1><<<grid, 128, 0, st>>>(L.pool, L.slab_bytes, M, L.luts, lo, R, aq, asq, out,
                                                               out_ld, meta_items);
    else
        gemv_mma_kernel<Q8, NG, KIND, 2><<<grid, 128, 0, st>>>(L.pool, L.slab_bytes, M, L.luts, lo, R, aq, asq, out,
                                                               out_ld, meta_items);
}

// Returns the number of kernels launched, 0 for a geometry probe (kind 2/3), or -1 if the geometry has no
// instantiation. asq: per activation row and group, (scale as int bits, sum of q). maxt: most tokens an expert on
// this path can have in the call (8 when n <= 8, else 11).
int launch_gemv_decode(const LayerDev &L, int kind, const RouteDev &R, const int8_t *aq, const int2 *asq, float *out,
                       int out_ld, int maxt, int grid, cudaStream_t st) {
    if (kind < 0)  // geometry probe: both matrices must have an instantiation
        return launch_gemv_decode(L, 2, R, aq, asq, out, out_ld, maxt, grid, st) < 0 ||
                       launch_gemv_decode(L, 3, R, aq, asq, out, out_ld, maxt, grid, st) < 0 ? -1 : 0;
    const bool probe = kind >= 2;
    if (probe) kind -= 2;
    const MatLayout &M = kind == 0 ? L.gu : L.dn;
    const int mi = kind == 0 ? kMetaDecItemsGU : kMetaDecItemsDN;
    const bool q8 = L.type == INZG_T_Q8G;
    if (M.rows % 16) return -1;
#define INZG_GEMV_CASE(Q, N)                                                                                     \
    if (q8 == Q && M.ng == N) {                                                                                  \
        if (probe) return 0;                                                                                     \
        if (kind == 0) launch_one<Q, N, 0>(L, M, R, aq, asq, out, out_ld, mi, maxt, grid, st);                  \
        else launch_one<Q, N, 1>(L, M, R, aq, asq, out, out_ld, mi, maxt, grid, st);                            \
        return 1;                                                                                                \
    }
    INZG_GEMV_CASE(false, 32)   // Q4L K = 2048
    INZG_GEMV_CASE(false, 40)   // Q4L K = 2560
    INZG_GEMV_CASE(false, 10)   // Q4L K = 640
    INZG_GEMV_CASE(true, 32)    // Q8G K = 2048
    INZG_GEMV_CASE(true, 40)    // Q8G K = 2560
    INZG_GEMV_CASE(true, 10)    // Q8G K = 640
#undef INZG_GEMV_CASE
    return -1;
}

void gemv_set_attributes() {}

}  // namespace inzg
