// k_gemm.cu -- prefill-path grouped GEMM (experts with >= 12 tokens), CUDA-core int8 version.
//
// Numerics of the reference's prefill GEMM (gemm_decode_tile + inz_gemm_rows, src/quant.c:1532-1668):
//   per (row, 256-block): sc = dmax * maxlev / 127, F_g = (int16)lrint(d_g * (512 / sc)) for the block's groups,
//   int8 weight w = sat_u8(mulhrs(level * 64, F_g) + 128) - 128 (Q8G: level = u - 128);
//   per (row, token): f = fma((float)dot_b, sc_b * xs_b, f) over blocks b in order, dot_b the exact integer dot of the
//   block's int8 weights and the token's 256-block int8 activation (the reference's float(acc) - 128 * sum equals it:
//   every term is an integer below 2^24).
// Tile: 64 rows x 64 tokens per block of 256 threads, K in 256-blocks; weights decoded into shared memory per block.
#include "inzg_internal.h"
#include "k_launch.h"

#include <cuda_fp16.h>

namespace inzg {

constexpr int kTM = 64, kTN = 64, kLd = kKB + 16;  // shared row pitch (bytes): 16-byte aligned, banks spread

template <int KIND>
__global__ void __launch_bounds__(256) gemm_v1_kernel(const int8_t *__restrict__ w8, const float *__restrict__ wsc,
                                                      MatLayout M, RouteDev R, const int8_t *__restrict__ aq,
                                                      const float *__restrict__ as, float *__restrict__ out, int out_ld,
                                                      int meta_tiles) {
    __shared__ __align__(16) int8_t W8[kTM][kLd];
    __shared__ __align__(16) int8_t X8[kTN][kLd];
    __shared__ float ws[kTM], xs[kTN];
    const int K = M.cols, nkb = (K + kKB - 1) / kKB;
    const int nrb = M.rows / kTM;
    const int nitems = R.meta[meta_tiles] * nrb * 2;  // a 128-token tile = two halves of kTN tokens
    const int tid = threadIdx.x;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
        const int half = item & 1, tile = R.gemm_tiles[(item >> 1) / nrb], rb = (item >> 1) % nrb;
        const int e = R.gemm_units[tile >> 16], tt = tile & 0xFFFF;
        const int base = R.off[e], ntok = R.cnt[e];
        const int t0 = tt * 2 * kTN + half * kTN, nt = min(kTN, ntok - t0);
        if (nt <= 0) continue;
        __syncthreads();
        float f[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) f[i][j] = 0.0f;
        for (int kb = 0; kb < nkb; kb++) {
            const int k0 = kb * kKB, klen = min(kKB, K - k0);
            // ---- weights: the materialised int8 rows (thread = row, 64-byte quarter) ----
            {
                const int rr = tid >> 2, part = tid & 3;
                const int r = rb * kTM + rr;
                if (part * kGroup < klen) {
                    const uint4 *src = reinterpret_cast<const uint4 *>(w8 + ((size_t)e * M.rows + r) * K + k0 + part * kGroup);
                    uint4 *dst = reinterpret_cast<uint4 *>(&W8[rr][part * kGroup]);
                    for (int i = 0; i < 4; i++) dst[i] = src[i];
                }
                if (part == 0) ws[rr] = wsc[((size_t)e * M.rows + r) * nkb + kb];
            }
            // ---- activations: thread = (token, 64-byte quarter) ----
            {
                const int t = tid >> 2, part = tid & 3;
                const bool ok = t < nt && part * kGroup < klen;
                uint4 *dst = reinterpret_cast<uint4 *>(&X8[t][part * kGroup]);
                if (ok) {
                    const int row = KIND == 0 ? R.etok[base + t0 + t] : base + t0 + t;
                    const uint4 *src = reinterpret_cast<const uint4 *>(aq + (size_t)row * K + k0 + part * kGroup);
                    for (int i = 0; i < 4; i++) dst[i] = src[i];
                    if (part == 0) xs[t] = as[(size_t)row * nkb + kb];
                } else {
                    for (int i = 0; i < 4; i++) dst[i] = make_uint4(0, 0, 0, 0);
                    if (part == 0) xs[t] = 0.0f;
                }
            }
            __syncthreads();
            // ---- 4 rows x 4 tokens per thread: rows (tid>>4) + 16 i, tokens (tid&15) + 16 j ----
            int D[4][4];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) D[i][j] = 0;
            const int ry = tid >> 4, tx = tid & 15;
            for (int kw = 0; kw < klen / 4; kw += 4) {
                int4 wv[4], xv[4];
#pragma unroll
                for (int i = 0; i < 4; i++) wv[i] = *reinterpret_cast<const int4 *>(&W8[ry + 16 * i][kw * 4]);
#pragma unroll
                for (int j = 0; j < 4; j++) xv[j] = *reinterpret_cast<const int4 *>(&X8[tx + 16 * j][kw * 4]);
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        int a = D[i][j];
                        a = __dp4a(wv[i].x, xv[j].x, a);
                        a = __dp4a(wv[i].y, xv[j].y, a);
                        a = __dp4a(wv[i].z, xv[j].z, a);
                        a = __dp4a(wv[i].w, xv[j].w, a);
                        D[i][j] = a;
                    }
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++)
                    f[i][j] = __fmaf_rn((float)D[i][j], __fmul_rn(ws[ry + 16 * i], xs[tx + 16 * j]), f[i][j]);
            __syncthreads();
        }
        const int ry = tid >> 4, tx = tid & 15;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int t = tx + 16 * j;
            if (t >= nt) continue;
            const int pos = base + t0 + t;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int r = rb * kTM + ry + 16 * i;
                if (KIND == 0) out[(size_t)pos * out_ld + r] = f[i][j];
                else out[(size_t)R.eslot[pos] * out_ld + r] = __fmul_rn(R.ew[pos], f[i][j]);
            }
        }
    }
}

int launch_gemm_v1(const LayerDev &L, int kind, const RouteDev &R, const int8_t *aq, const float *as, float *out,
                   int out_ld, int grid, cudaStream_t st) {
    const MatLayout &M = kind == 0 ? L.gu : L.dn;
    const int mt = kind == 0 ? kMetaGemmTilesGU : kMetaGemmTilesDN;
    if (M.rows % kTM) return -1;
    if (kind == 0) gemm_v1_kernel<0><<<grid, 256, 0, st>>>(L.w8_gu, L.ws_gu, M, R, aq, as, out, out_ld, mt);
    else gemm_v1_kernel<1><<<grid, 256, 0, st>>>(L.w8_dn, L.ws_dn, M, R, aq, as, out, out_ld, mt);
    return 1;
}

int gemm_token_tile() { return 2 * kTN; }

}  // namespace inzg
