// k_gemv.cu -- decode-path grouped GEMV over the routed experts (Q4L / Q8G), sm_100a.
//
// Numerics of the reference's mv_q4l / mm_q4l (DEFINE_MV_LUT / DEFINE_MM_LUT, src/quant.c:767-875, 1179-1225) and
// mv_q8g / mm_q8g (881-953): per row and token, 8 fp32 accumulators; accumulator l receives, for every 64-group g
// in order, fma(I_gl, d_g * s_g) where I_gl is the exact integer dot of weights {4l..4l+3, 32+4l..32+4l+3} with the
// int8 activation. Q4L: the LUT bias is removed with fma chains over d_g * bsum_g kept in 8 lanes (g % 8) for the
// first ng&~7 groups, then a scalar tail; y = hsum8(acc) - 64 * b. Q8G (VNNI form): y = hsum8(acc) - 128 * b with b a
// sequential fma chain. Thread (row, l) of a warp runs lane l's accumulator, so the result is the reference's bits.
//
// Work: items = (decode expert, block of 32 rows); a persistent grid walks the device-built item list. The tokens'
// activations (<= 11 per expert on this path) are staged in shared memory; weights stream once from HBM with one
// vector load per thread per chunk of groups (layout in inzg_internal.h).
#include "inzg_internal.h"
#include "k_launch.h"

#include <cuda_fp16.h>

namespace inzg {

constexpr int kMaxDecTok = kGemmMinT - 1;  // 11: an expert with more tokens takes the prefill path (or n <= 8)

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

template <int VB>
struct VecT;
template <>
struct VecT<16> { using T = uint4; };
template <>
struct VecT<8> { using T = uint2; };

__device__ __forceinline__ uint32_t vword(const uint4 &v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
__device__ __forceinline__ uint32_t vword(const uint2 &v, int i) { return i == 0 ? v.x : v.y; }

// KIND 0: gate|up, activation row = token, output GU[entry][row]. KIND 1: down, activation row = entry,
// output moe_out[slot][row] = w * y. MAXT: largest token count of an expert in this call (1, 8 or 11).
// Work item = (decode expert, quad of rows), one per warp; warps run free (no block barrier): a warp loads the
// weights of its next item before it computes the current one. Activations (<= 11 tokens x K bytes) and their
// (scale, bias-sum) pairs stay in L1.
template <bool Q8, int NCH, int GC, int KIND, int MAXT>
__global__ void __launch_bounds__(128) gemv_decode_kernel(const uint8_t *__restrict__ pool, uint64_t slab_bytes,
                                                          MatLayout M, const uint8_t *__restrict__ luts, int lut_off,
                                                          RouteDev R, const int8_t *__restrict__ aq,
                                                          const float2 *__restrict__ asb, float *__restrict__ out,
                                                          int out_ld, int meta_items) {
    constexpr int WB = Q8 ? 8 : 4;
    constexpr int VB = GC * WB;
    constexpr int ng = NCH * GC, ng8 = ng & ~7, K = ng * kGroup;
    using V = typename VecT<VB>::T;
    const int nitems = R.meta[meta_items];
    const int per = M.rows / 4;  // row quads per expert
    const int lane = threadIdx.x & 31, r4 = lane >> 3, l = lane & 7;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), nw = gridDim.x * (blockDim.x >> 5);
    int item = gw;
    if (item >= nitems) return;
    auto load = [&](int it, V *wv, uint4 &T, int &e, int &rq) {
        const int u = it / per;
        rq = it % per;
        e = R.dec_units[u];
        const uint8_t *slab = pool + (size_t)e * slab_bytes;
        const V *wq = reinterpret_cast<const V *>(slab + M.q_off) + ((size_t)rq * NCH) * 32 + lane;
#pragma unroll
        for (int c = 0; c < NCH; c++) wv[c] = __ldg(wq + (size_t)c * 32);
        if (!Q8) T = __ldg(reinterpret_cast<const uint4 *>(luts + (size_t)e * 32 + lut_off));
    };
    V cur[NCH], nxt[NCH];
    uint4 Tc = make_uint4(0, 0, 0, 0), Tn = make_uint4(0, 0, 0, 0);
    int ec, rqc, en = 0, rqn = 0;
    load(item, cur, Tc, ec, rqc);
    while (true) {
        const int next = item + nw;
        const bool more = next < nitems;
        if (more) load(next, nxt, Tn, en, rqn);
        // ---- compute item (ec, rqc) ----
        const int base = R.off[ec], ntok = min(R.cnt[ec], MAXT);
        const int row = rqc * 4 + r4;
        const __half *wd = reinterpret_cast<const __half *>(pool + (size_t)ec * slab_bytes + M.d_off) +
                           ((size_t)rqc * NCH * 4 + r4) * GC;
        int arow[MAXT];  // activation row of each token (32-bit: rows * K < 2^31 for every supported size)
#pragma unroll
        for (int t = 0; t < MAXT; t++) arow[t] = t < ntok ? (KIND == 0 ? R.etok[base + t] : base + t) : 0;
        float acc[MAXT], bl[MAXT];
#pragma unroll
        for (int t = 0; t < MAXT; t++) { acc[t] = 0.0f; bl[t] = 0.0f; }
        float dtail[ng - ng8 > 0 ? ng - ng8 : 1];
#pragma unroll
        for (int c = 0; c < NCH; c++) {
            // the chunk's scales: gc halves, one load
            __half dh[GC];
            if (GC == 4) *reinterpret_cast<uint2 *>(dh) = __ldg(reinterpret_cast<const uint2 *>(wd + (size_t)c * 4 * GC));
            else if (GC == 2) *reinterpret_cast<uint32_t *>(dh) = __ldg(reinterpret_cast<const unsigned int *>(wd + (size_t)c * 4 * GC));
            else dh[0] = wd[(size_t)c * 4 * GC];
#pragma unroll
            for (int gq = 0; gq < GC; gq++) {
                const int g = c * GC + gq;
                const float d = __half2float(dh[gq]);
                uint32_t lo4, hi4;
                if (Q8) {
                    lo4 = vword(cur[c], 2 * gq);
                    hi4 = vword(cur[c], 2 * gq + 1);
                } else {
                    const uint32_t w = vword(cur[c], gq);
                    lo4 = lut16(w, Tc);
                    hi4 = lut16(w >> 16, Tc);
                }
                if (!Q8 && g >= ng8) dtail[g - ng8] = d;
#pragma unroll
                for (int t = 0; t < MAXT; t++) {
                    if (t < ntok) {
                        const int2 x = __ldg(reinterpret_cast<const int2 *>(aq + arow[t] * K + g * kGroup + l * 8));
                        const float2 sb = __ldg(asb + arow[t] * ng + g);
                        int I;
                        if (Q8) I = dp4a_us(hi4, x.y, dp4a_us(lo4, x.x, 0));
                        else I = dp4a_ss((int)hi4, x.y, dp4a_ss((int)lo4, x.x, 0));
                        acc[t] = __fmaf_rn((float)I, __fmul_rn(d, sb.x), acc[t]);
                        if (Q8) bl[t] = __fmaf_rn(d, sb.y, bl[t]);
                        else if (g < ng8 && (g & 7) == l) bl[t] = __fmaf_rn(d, sb.y, bl[t]);
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < MAXT; t++) {
            if (t < ntok) {  // ntok is uniform over the warp: the shuffles below are converged
                const float a = hsum8_lanes(acc[t]);
                float y;
                if (Q8) y = __fsub_rn(a, __fmul_rn(128.0f, bl[t]));
                else {
                    float b = hsum8_lanes(bl[t]);
#pragma unroll
                    for (int g = ng8; g < ng; g++) b = __fmaf_rn(dtail[g - ng8], __ldg(asb + arow[t] * ng + g).y, b);
                    y = __fsub_rn(a, __fmul_rn((float)kLutBias, b));
                }
                if (l == 0) {
                    const int pos = base + t;
                    if (KIND == 0) out[(size_t)pos * out_ld + row] = y;
                    else out[(size_t)R.eslot[pos] * out_ld + row] = __fmul_rn(R.ew[pos], y);
                }
            }
        }
        if (!more) break;
        item = next;
#pragma unroll
        for (int c = 0; c < NCH; c++) cur[c] = nxt[c];
        Tc = Tn;
        ec = en;
        rqc = rqn;
    }
}

// ---------------------------------------------------------------------------------------------------------------
template <bool Q8, int NCH, int GC, int KIND>
static void launch_one(const LayerDev &L, const MatLayout &M, const RouteDev &R, const int8_t *aq, const float2 *asb,
                       float *out, int out_ld, int meta_items, int maxt, int grid, cudaStream_t st) {
    const int lo = KIND == 0 ? 0 : 16;
    if (maxt <= 1)
        gemv_decode_kernel<Q8, NCH, GC, KIND, 1><<<grid, 128, 0, st>>>(L.pool, L.slab_bytes, M, L.luts, lo, R, aq, asb,
                                                                       out, out_ld, meta_items);
    else if (maxt <= 8)
        gemv_decode_kernel<Q8, NCH, GC, KIND, 8><<<grid, 128, 0, st>>>(L.pool, L.slab_bytes, M, L.luts, lo, R, aq, asb,
                                                                       out, out_ld, meta_items);
    else
        gemv_decode_kernel<Q8, NCH, GC, KIND, kMaxDecTok><<<grid, 128, 0, st>>>(L.pool, L.slab_bytes, M, L.luts, lo, R,
                                                                                aq, asb, out, out_ld, meta_items);
}

// Returns the number of kernels launched, 0 for a geometry probe (kind 2/3), or -1 if the geometry has no
// instantiation. asb: per activation row and group, (scale, bias sum). maxt: tokens of the call, capped at 11.
int launch_gemv_decode(const LayerDev &L, int kind, const RouteDev &R, const int8_t *aq, const float2 *asb, float *out,
                       int out_ld, int maxt, int grid, cudaStream_t st) {
    if (kind < 0)  // geometry probe: both matrices must have an instantiation
        return launch_gemv_decode(L, 2, R, aq, asb, out, out_ld, maxt, grid, st) < 0 ||
                       launch_gemv_decode(L, 3, R, aq, asb, out, out_ld, maxt, grid, st) < 0 ? -1 : 0;
    const bool probe = kind >= 2;
    if (probe) kind -= 2;
    const MatLayout &M = kind == 0 ? L.gu : L.dn;
    const int mi = kind == 0 ? kMetaDecItemsGU : kMetaDecItemsDN;
    const bool q8 = L.type == INZG_T_Q8G;
#define INZG_GEMV_CASE(Q, N, G)                                                                                  \
    if (q8 == Q && M.nch == N && M.gc == G) {                                                                    \
        if (probe) return 0;                                                                                     \
        if (kind == 0) launch_one<Q, N, G, 0>(L, M, R, aq, asb, out, out_ld, mi, maxt, grid, st);               \
        else launch_one<Q, N, G, 1>(L, M, R, aq, asb, out, out_ld, mi, maxt, grid, st);                         \
        return 1;                                                                                                \
    }
    INZG_GEMV_CASE(false, 8, 4)    // Q4L K = 2048
    INZG_GEMV_CASE(false, 10, 4)   // Q4L K = 2560
    INZG_GEMV_CASE(false, 5, 2)    // Q4L K = 640
    INZG_GEMV_CASE(true, 16, 2)    // Q8G K = 2048
    INZG_GEMV_CASE(true, 20, 2)    // Q8G K = 2560
    INZG_GEMV_CASE(true, 5, 2)     // Q8G K = 640
#undef INZG_GEMV_CASE
    return -1;
}

void gemv_set_attributes() {}

}  // namespace inzg
