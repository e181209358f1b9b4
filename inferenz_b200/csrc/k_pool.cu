// k_pool.cu -- re-layout of uploaded expert blobs into the HBM pool (tile layout, inzg_internal.h).
//
// Source: one blob per expert as the converter writes it (src/convert.c:565-584): gate|up matrix, down matrix at
// gu_bytes; each matrix = 64-byte header (src/quant.h:40-50), indices [rows][ng][gb], fp16 scales [rows][ng].
// Only the order of bytes changes (values are untouched), so the pool holds exactly the blob's information.
#include "inzg_internal.h"
#include "k_launch.h"

#include <cuda_fp16.h>

namespace inzg {

__global__ void pool_repack_kernel(const uint8_t *__restrict__ blobs, uint64_t blob_bytes, uint64_t gu_bytes, int e0,
                                   int ne, LayerDev L, uint8_t *__restrict__ pool, uint8_t *__restrict__ luts) {
    const bool q8 = L.type == INZG_T_Q8G;
    const int gb = q8 ? 64 : 32;
    const int64_t pairs_gu = (int64_t)L.gu.rows * L.gu.ng, pairs_dn = (int64_t)L.dn.rows * L.dn.ng;
    const int64_t per_e = pairs_gu + pairs_dn;
    const int64_t total = per_e * ne;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int el = (int)(i / per_e);
        int64_t p = i % per_e;
        const bool dn = p >= pairs_gu;
        if (dn) p -= pairs_gu;
        const MatLayout &M = dn ? L.dn : L.gu;
        const uint8_t *src = blobs + (size_t)el * blob_bytes + (dn ? gu_bytes : 0);
        const int r = (int)(p / M.ng), g = (int)(p % M.ng);
        const uint8_t *sq = src + 64 + ((size_t)r * M.ng + g) * gb;
        const uint16_t *sd = reinterpret_cast<const uint16_t *>(src + 64 + (size_t)M.rows * M.ng * gb);
        uint8_t *slab = pool + (size_t)(e0 + el) * L.slab_bytes;
        const int rt = r >> 4, rr = r & 7, hi = (r >> 3) & 1;  // row tile, row within the 8-row half, half
        uint8_t *tile = slab + M.q_off + ((size_t)rt * M.ng + g) * 32 * M.wb;
        // lane (rr, t) of MMA h: fragment registers a0/a1 carry lane l = 4h + t/2, a2/a3 lane l + 2, of part t % 2
        // (part 0: weights 4l..4l+3, part 1: weights 32+4l..32+4l+3); hi selects a0/a2 (row rr) or a1/a3 (row rr + 8)
        for (int t = 0; t < 4; t++) {
            const int lane = rr * 4 + t, p = t & 1;
            for (int h = 0; h < 2; h++) {
                const int l0 = 4 * h + (t >> 1), l1 = l0 + 2;
                if (q8) {
                    uint8_t *dst = tile + (size_t)h * 512 + (size_t)lane * 16;
                    for (int j = 0; j < 4; j++) {
                        dst[hi * 4 + j] = sq[32 * p + 4 * l0 + j];      // a0 (row rr) / a1 (row rr + 8)
                        dst[8 + hi * 4 + j] = sq[32 * p + 4 * l1 + j];  // a2 / a3
                    }
                } else {
                    uint32_t w = 0;
                    for (int j = 0; j < 4; j++) {
                        w |= (uint32_t)((sq[4 * l0 + j] >> (4 * p)) & 15) << (4 * j);
                        w |= (uint32_t)((sq[4 * l1 + j] >> (4 * p)) & 15) << (16 + 4 * j);
                    }
                    *reinterpret_cast<uint32_t *>(tile + (size_t)lane * 16 + (2 * h + hi) * 4) = w;
                }
            }
        }
        uint16_t *dd = reinterpret_cast<uint16_t *>(slab + M.d_off);
        dd[((((size_t)rt * M.gd + (g >> 2)) * 8 + rr) * 4 + (g & 3)) * 2 + hi] = sd[(size_t)r * M.ng + g];
        if (p == 0) {  // the matrix's LUT (header bytes 24..39)
            for (int k = 0; k < 16; k++) luts[(size_t)(e0 + el) * 32 + (dn ? 16 : 0) + k] = src[24 + k];
        }
    }
}

// Prefill-path weights, materialised once per layer: the reference's per-(row, 256-block) requantization
// (gemm_decode_tile, src/quant.c:1532-1613) is a fixed function of the blob, so its int8 weights and block scales are
// computed here once instead of in every GEMM tile: sc = dmax * maxlev / 127, F_g = (int16)lrint(d_g * (512 / sc)),
// w = sat_u8(mulhrs(level * 64, F_g) + 128) - 128. Output: w8 [rows][K] (K-major rows for TMA) and ws [rows][nkb].
__device__ __forceinline__ int mulhrs16(int a, int b) {
    const int t = ((a * b) >> 14) + 1;
    return (int)(int16_t)(uint16_t)((uint32_t)t >> 1);
}
__device__ __forceinline__ int requant_w(int lv, int F) {
    const int v = (int)(int16_t)(mulhrs16((int)(int16_t)(lv * 64), F) + 128);
    return (v < 0 ? 0 : v > 255 ? 255 : v) - 128;
}

__global__ void pool_requant_kernel(const uint8_t *__restrict__ blobs, uint64_t blob_bytes, uint64_t gu_bytes, int e0,
                                    int ne, int type, int H, int FF, int8_t *__restrict__ w8_gu,
                                    float *__restrict__ ws_gu, int8_t *__restrict__ w8_dn, float *__restrict__ ws_dn) {
    const bool q8 = type == INZG_T_Q8G;
    const int gb = q8 ? 64 : 32;
    // one work unit = (expert, matrix, row); a warp per unit, lanes over the row's 256-blocks and groups
    const int rows_gu = 2 * FF, rows_dn = H;
    const int64_t per_e = rows_gu + rows_dn;
    const int64_t total = per_e * ne;
    const int lane = threadIdx.x & 31;
    for (int64_t u = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / 32; u < total;
         u += (int64_t)gridDim.x * blockDim.x / 32) {
        const int el = (int)(u / per_e);
        int r = (int)(u % per_e);
        const bool dn = r >= rows_gu;
        if (dn) r -= rows_gu;
        const int K = dn ? FF : H, ng = K / kGroup, nkb = (K + kKB - 1) / kKB;
        const uint8_t *src = blobs + (size_t)el * blob_bytes + (dn ? gu_bytes : 0);
        const uint8_t *q = src + 64 + (size_t)r * ng * gb;
        const uint16_t *d = reinterpret_cast<const uint16_t *>(src + 64 + (size_t)(dn ? rows_dn : rows_gu) * ng * gb) + (size_t)r * ng;
        int maxlev = 127;
        if (!q8) {
            maxlev = 1;
            for (int i = 0; i < 16; i++) maxlev = max(maxlev, abs((int)src[24 + i] - kLutBias));
        }
        int8_t *w8 = (dn ? w8_dn : w8_gu) + ((size_t)(e0 + el) * (dn ? rows_dn : rows_gu) + r) * K;
        float *ws = (dn ? ws_dn : ws_gu) + ((size_t)(e0 + el) * (dn ? rows_dn : rows_gu) + r) * nkb;
        for (int g = lane; g < ng; g += 32) {
            const int b = g / 4, g0 = b * 4, g1 = min(g0 + 4, ng);
            float dmax = 0.0f;
            for (int h = g0; h < g1; h++) dmax = fmaxf(dmax, fabsf(__half2float(__ushort_as_half(d[h]))));
            const float sc = __fdiv_rn(__fmul_rn(dmax, (float)maxlev), 127.0f);
            if (g == g0) ws[b] = sc;
            const float inv = sc > 0 ? __fdiv_rn(512.0f, sc) : 0.0f;
            const int F = (int)(int16_t)__float2int_rn(__fmul_rn(__half2float(__ushort_as_half(d[g])), inv));
            const uint8_t *qg = q + (size_t)g * gb;
            int8_t *o = w8 + (size_t)g * kGroup;
            if (q8) {
                for (int j = 0; j < 64; j++) o[j] = (int8_t)requant_w((int)qg[j] - 128, F);
            } else {
                for (int j = 0; j < 32; j++) {
                    o[j] = (int8_t)requant_w((int)src[24 + (qg[j] & 15)] - kLutBias, F);
                    o[32 + j] = (int8_t)requant_w((int)src[24 + (qg[j] >> 4)] - kLutBias, F);
                }
            }
        }
    }
}

void launch_pool_requant(const uint8_t *blobs, uint64_t blob_bytes, uint64_t gu_bytes, int e0, int ne, const LayerDev &L,
                         cudaStream_t st) {
    pool_requant_kernel<<<1024, 256, 0, st>>>(blobs, blob_bytes, gu_bytes, e0, ne, L.type, L.H, L.FF, L.w8_gu, L.ws_gu,
                                              L.w8_dn, L.ws_dn);
}

void launch_pool_repack(const uint8_t *blobs, uint64_t blob_bytes, uint64_t gu_bytes, int e0, int ne, const LayerDev &L,
                        uint8_t *pool, uint8_t *luts, cudaStream_t st) {
    pool_repack_kernel<<<1024, 256, 0, st>>>(blobs, blob_bytes, gu_bytes, e0, ne, L, pool, luts);
}

}  // namespace inzg
