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
// output moe_out[slot][row] = w * y.
template <bool Q8, int NCH, int GC, int KIND>
__global__ void __launch_bounds__(256) gemv_decode_kernel(const uint8_t *__restrict__ pool, uint64_t slab_bytes,
                                                          MatLayout M, const uint8_t *__restrict__ luts, int lut_off,
                                                          RouteDev R, const int8_t *__restrict__ aq,
                                                          const float *__restrict__ as, const float *__restrict__ ab,
                                                          float *__restrict__ out, int out_ld, int meta_items) {
    constexpr int WB = Q8 ? 8 : 4;
    constexpr int VB = GC * WB;
    constexpr int ng = NCH * GC, ng8 = ng & ~7, K = ng * kGroup;
    using V = typename VecT<VB>::T;
    extern __shared__ __align__(16) uint8_t smem[];
    // shared: activations [kMaxDecTok][K] bytes, scales [kMaxDecTok][ng], bias sums [kMaxDecTok][ng]
    int8_t *sq = reinterpret_cast<int8_t *>(smem);
    float *ss = reinterpret_cast<float *>(smem + (size_t)kMaxDecTok * K);
    float *sb = ss + (size_t)kMaxDecTok * ng;
    const int nitems = R.meta[meta_items];
    const int per = M.rows / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r4 = lane >> 3, l = lane & 7;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
        const int u = item / per, rb = item % per;
        const int e = R.dec_units[u];
        const int base = R.off[e], ntok = min(R.cnt[e], kMaxDecTok);
        __syncthreads();  // previous item's readers are done with the staged activations
        for (int i = threadIdx.x; i < ntok * (K / 16); i += blockDim.x) {
            const int t = i / (K / 16), c = i % (K / 16);
            const int row = KIND == 0 ? R.etok[base + t] : base + t;
            reinterpret_cast<uint4 *>(sq + (size_t)t * K)[c] = reinterpret_cast<const uint4 *>(aq + (size_t)row * K)[c];
        }
        for (int i = threadIdx.x; i < ntok * ng; i += blockDim.x) {
            const int t = i / ng, g = i % ng;
            const int row = KIND == 0 ? R.etok[base + t] : base + t;
            ss[t * ng + g] = as[(size_t)row * ng + g];
            sb[t * ng + g] = ab[(size_t)row * ng + g];
        }
        __syncthreads();
        const int rq = rb * 8 + warp;
        const int row = rq * 4 + r4;
        const uint8_t *slab = pool + (size_t)e * slab_bytes;
        const V *wq = reinterpret_cast<const V *>(slab + M.q_off) + ((size_t)rq * NCH) * 32 + lane;
        const __half *wd = reinterpret_cast<const __half *>(slab + M.d_off) + ((size_t)rq * NCH * 4 + r4) * GC;
        V wv[NCH];
#pragma unroll
        for (int c = 0; c < NCH; c++) wv[c] = __ldg(wq + (size_t)c * 32);
        uint4 T = make_uint4(0, 0, 0, 0);
        if (!Q8) T = *reinterpret_cast<const uint4 *>(luts + (size_t)e * 32 + lut_off);
        float acc[kMaxDecTok], bl[kMaxDecTok];
#pragma unroll
        for (int t = 0; t < kMaxDecTok; t++) { acc[t] = 0.0f; bl[t] = 0.0f; }
        float dtail[ng - ng8 > 0 ? ng - ng8 : 1];
#pragma unroll
        for (int c = 0; c < NCH; c++) {
#pragma unroll
            for (int gq = 0; gq < GC; gq++) {
                const int g = c * GC + gq;
                const float d = __half2float(wd[(size_t)c * 4 * GC + gq]);
                uint32_t lo4, hi4;
                if (Q8) {
                    lo4 = vword(wv[c], 2 * gq);
                    hi4 = vword(wv[c], 2 * gq + 1);
                } else {
                    const uint32_t w = vword(wv[c], gq);
                    lo4 = lut16(w, T);
                    hi4 = lut16(w >> 16, T);
                }
                if (!Q8 && g >= ng8) dtail[g - ng8] = d;
#pragma unroll
                for (int t = 0; t < kMaxDecTok; t++) {
                    if (t < ntok) {
                        const int2 x = *reinterpret_cast<const int2 *>(sq + (size_t)t * K + g * kGroup + l * 8);
                        int I;
                        if (Q8) I = dp4a_us(hi4, x.y, dp4a_us(lo4, x.x, 0));
                        else I = dp4a_ss((int)hi4, x.y, dp4a_ss((int)lo4, x.x, 0));
                        acc[t] = __fmaf_rn((float)I, __fmul_rn(d, ss[t * ng + g]), acc[t]);
                        if (Q8) bl[t] = __fmaf_rn(d, sb[t * ng + g], bl[t]);
                        else if (g < ng8 && (g & 7) == l) bl[t] = __fmaf_rn(d, sb[t * ng + g], bl[t]);
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < kMaxDecTok; t++) {
            if (t < ntok) {  // ntok is uniform over the block: the shuffles below are warp-converged
                const float a = hsum8_lanes(acc[t]);
                float y;
                if (Q8) y = __fsub_rn(a, __fmul_rn(128.0f, bl[t]));
                else {
                    float b = hsum8_lanes(bl[t]);
#pragma unroll
                    for (int g = ng8; g < ng; g++) b = __fmaf_rn(dtail[g - ng8], sb[t * ng + g], b);
                    y = __fsub_rn(a, __fmul_rn((float)kLutBias, b));
                }
                if (l == 0) {
                    const int pos = base + t;
                    if (KIND == 0) out[(size_t)pos * out_ld + row] = y;
                    else out[(size_t)R.eslot[pos] * out_ld + row] = __fmul_rn(R.ew[pos], y);
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------
template <bool Q8, int NCH, int GC, int KIND>
static void launch_one(const LayerDev &L, const MatLayout &M, const RouteDev &R, const int8_t *aq, const float *as,
                       const float *ab, float *out, int out_ld, int meta_items, int grid, cudaStream_t st) {
    const size_t smem = (size_t)kMaxDecTok * M.cols + (size_t)2 * kMaxDecTok * M.ng * sizeof(float);
    auto k = gemv_decode_kernel<Q8, NCH, GC, KIND>;
    k<<<grid, 256, smem, st>>>(L.pool, L.slab_bytes, M, L.luts, KIND == 0 ? 0 : 16, R, aq, as, ab, out, out_ld, meta_items);
}

// Returns the number of kernels launched, or -1 if the geometry has no instantiation.
int launch_gemv_decode(const LayerDev &L, int kind, const RouteDev &R, const int8_t *aq, const float *as,
                       const float *ab, float *out, int out_ld, int grid, cudaStream_t st) {
    if (kind < 0)  // geometry probe: both matrices must have an instantiation
        return launch_gemv_decode(L, 2, R, aq, as, ab, out, out_ld, grid, st) < 0 ||
                       launch_gemv_decode(L, 3, R, aq, as, ab, out, out_ld, grid, st) < 0 ? -1 : 0;
    const bool probe = kind >= 2;
    if (probe) kind -= 2;
    const MatLayout &M = kind == 0 ? L.gu : L.dn;
    const int mi = kind == 0 ? kMetaDecItemsGU : kMetaDecItemsDN;
    const bool q8 = L.type == INZG_T_Q8G;
#define INZG_GEMV_CASE(Q, N, G)                                                                                  \
    if (q8 == Q && M.nch == N && M.gc == G) {                                                                    \
        if (probe) return 0;                                                                                     \
        if (kind == 0) launch_one<Q, N, G, 0>(L, M, R, aq, as, ab, out, out_ld, mi, grid, st);                  \
        else launch_one<Q, N, G, 1>(L, M, R, aq, as, ab, out, out_ld, mi, grid, st);                            \
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

// The dynamic shared memory of every instantiation stays below 48 KB except at H = 4096+; set the opt-in anyway.
void gemv_set_attributes() {
#define INZG_GEMV_ATTR(Q, N, G)                                                                                  \
    cudaFuncSetAttribute(gemv_decode_kernel<Q, N, G, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024); \
    cudaFuncSetAttribute(gemv_decode_kernel<Q, N, G, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
    INZG_GEMV_ATTR(false, 8, 4)
    INZG_GEMV_ATTR(false, 10, 4)
    INZG_GEMV_ATTR(false, 5, 2)
    INZG_GEMV_ATTR(true, 16, 2)
    INZG_GEMV_ATTR(true, 20, 2)
    INZG_GEMV_ATTR(true, 5, 2)
#undef INZG_GEMV_ATTR
}

}  // namespace inzg
