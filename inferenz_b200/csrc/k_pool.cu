// k_pool.cu -- re-layout of uploaded expert blobs into the HBM pool (decode layout, inzg_internal.h).
//
// Source: one blob per expert as the converter writes it (src/convert.c:565-584): gate|up matrix, down matrix at
// gu_bytes; each matrix = 64-byte header (src/quant.h:40-50), indices [rows][ng][gb], fp16 scales [rows][ng].
// Only the order of bytes changes (values are untouched), so the pool holds exactly the blob's information.
#include "inzg_internal.h"
#include "k_launch.h"

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
        const int rq = r >> 2, r4 = r & 3, c = g / M.gc, gq = g % M.gc;
        const int VB = M.gc * M.wb;
        for (int l = 0; l < 8; l++) {
            uint8_t *dst = slab + M.q_off + ((size_t)(rq * M.nch + c) * 32 + r4 * 8 + l) * VB + gq * M.wb;
            if (q8) {
                for (int j = 0; j < 4; j++) {
                    dst[j] = sq[4 * l + j];
                    dst[4 + j] = sq[32 + 4 * l + j];
                }
            } else {
                uint32_t w = 0;
                for (int j = 0; j < 4; j++) {
                    const uint32_t b = sq[4 * l + j];
                    w |= (b & 15u) << (4 * j);          // weight 4l+j      -> selector nibble j of the low half
                    w |= (b >> 4) << (16 + 4 * j);      // weight 32+4l+j   -> selector nibble j of the high half
                }
                *reinterpret_cast<uint32_t *>(dst) = w;
            }
        }
        uint16_t *dd = reinterpret_cast<uint16_t *>(slab + M.d_off);
        dd[((size_t)(rq * M.nch + c) * 4 + r4) * M.gc + gq] = sd[(size_t)r * M.ng + g];
        if (p == 0) {  // the matrix's LUT (header bytes 24..39)
            for (int k = 0; k < 16; k++) luts[(size_t)(e0 + el) * 32 + (dn ? 16 : 0) + k] = src[24 + k];
        }
    }
}

void launch_pool_repack(const uint8_t *blobs, uint64_t blob_bytes, uint64_t gu_bytes, int e0, int ne, const LayerDev &L,
                        uint8_t *pool, uint8_t *luts, cudaStream_t st) {
    pool_repack_kernel<<<1024, 256, 0, st>>>(blobs, blob_bytes, gu_bytes, e0, ne, L, pool, luts);
}

}  // namespace inzg
