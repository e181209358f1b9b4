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

__device__ __forceinline__ int mulhrs16(int a, int b) {
    const int t = ((a * b) >> 14) + 1;
    return (int)(int16_t)(uint16_t)((uint32_t)t >> 1);
}
__device__ __forceinline__ int sat_u8(int v) { return v < 0 ? 0 : v > 255 ? 255 : v; }

// int8 weight of level value lv (LUT level - 64, or Q8G byte - 128) under factor F
__device__ __forceinline__ int requant_w(int lv, int F) {
    return sat_u8((int)(int16_t)(mulhrs16((int)(int16_t)(lv * 64), F) + 128)) - 128;
}

template <bool Q8, int KIND>
__global__ void __launch_bounds__(256) gemm_v1_kernel(const uint8_t *__restrict__ pool, uint64_t slab_bytes, MatLayout M,
                                                      const uint8_t *__restrict__ luts, int lut_off, RouteDev R,
                                                      const int8_t *__restrict__ aq, const float *__restrict__ as,
                                                      float *__restrict__ out, int out_ld, int meta_tiles) {
    __shared__ __align__(16) int8_t W8[kTM][kLd];
    __shared__ __align__(16) int8_t X8[kTN][kLd];
    __shared__ float ws[kTM], xs[kTN];
    __shared__ int lv[16];
    __shared__ int maxlev_s;
    constexpr int WB = Q8 ? 8 : 4;
    const int K = M.cols, nkb = (K + kKB - 1) / kKB, GC = M.gc, VB = GC * WB, nch = M.nch;
    const int nrb = M.rows / kTM;
    const int nitems = R.meta[meta_tiles] * nrb;
    const int tid = threadIdx.x;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
        const int tile = R.gemm_tiles[item / nrb], rb = item % nrb;
        const int e = R.gemm_units[tile >> 16], tt = tile & 0xFFFF;
        const int base = R.off[e], ntok = R.cnt[e];
        const int t0 = tt * kTN, nt = min(kTN, ntok - t0);
        const uint8_t *slab = pool + (size_t)e * slab_bytes;
        __syncthreads();
        if (tid < 16) lv[tid] = Q8 ? 0 : (int)luts[(size_t)e * 32 + lut_off + tid] - kLutBias;
        __syncthreads();
        if (tid == 0) {
            int m = 127;
            if (!Q8) {
                m = 1;
                for (int i = 0; i < 16; i++) m = max(m, abs(lv[i]));
            }
            maxlev_s = m;
        }
        __syncthreads();
        const float maxlev = (float)maxlev_s;
        float f[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) f[i][j] = 0.0f;
        for (int kb = 0; kb < nkb; kb++) {
            const int k0 = kb * kKB, klen = min(kKB, K - k0), gpb = klen / kGroup;
            // ---- weights: thread = (row rr, group gq of the block) ----
            {
                const int rr = tid >> 2, gq = tid & 3;
                const int r = rb * kTM + rr, rq = r >> 2, r4 = r & 3;
                const __half *dbase = reinterpret_cast<const __half *>(slab + M.d_off);
                float dmax = 0.0f;
                for (int q = 0; q < gpb; q++) {
                    const int g = kb * 4 + q;
                    dmax = fmaxf(dmax, fabsf(__half2float(dbase[((size_t)(rq * nch + g / GC) * 4 + r4) * GC + g % GC])));
                }
                const float sc = __fdiv_rn(__fmul_rn(dmax, maxlev), 127.0f);
                if (gq == 0) ws[rr] = sc;
                if (gq < gpb) {
                    const int g = kb * 4 + gq;
                    const float inv = sc > 0 ? __fdiv_rn(512.0f, sc) : 0.0f;
                    const float d = __half2float(dbase[((size_t)(rq * nch + g / GC) * 4 + r4) * GC + g % GC]);
                    const int F = (int)(int16_t)__float2int_rn(__fmul_rn(d, inv));
                    const uint8_t *qb = slab + M.q_off + ((size_t)(rq * nch + g / GC) * 32 + r4 * 8) * VB + (g % GC) * WB;
                    int8_t *dst = &W8[rr][gq * kGroup];
                    for (int l = 0; l < 8; l++) {
                        if (Q8) {
                            const uint32_t lo = *reinterpret_cast<const uint32_t *>(qb + (size_t)l * VB);
                            const uint32_t hi = *reinterpret_cast<const uint32_t *>(qb + (size_t)l * VB + 4);
                            for (int i = 0; i < 4; i++) {
                                dst[4 * l + i] = (int8_t)requant_w((int)((lo >> (8 * i)) & 255) - 128, F);
                                dst[32 + 4 * l + i] = (int8_t)requant_w((int)((hi >> (8 * i)) & 255) - 128, F);
                            }
                        } else {
                            const uint32_t w = *reinterpret_cast<const uint32_t *>(qb + (size_t)l * VB);
                            for (int i = 0; i < 4; i++) {
                                dst[4 * l + i] = (int8_t)requant_w(lv[(w >> (4 * i)) & 15], F);
                                dst[32 + 4 * l + i] = (int8_t)requant_w(lv[(w >> (16 + 4 * i)) & 15], F);
                            }
                        }
                    }
                }
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
    const bool q8 = L.type == INZG_T_Q8G;
    if (q8) {
        if (kind == 0) gemm_v1_kernel<true, 0><<<grid, 256, 0, st>>>(L.pool, L.slab_bytes, M, L.luts, 0, R, aq, as, out, out_ld, mt);
        else gemm_v1_kernel<true, 1><<<grid, 256, 0, st>>>(L.pool, L.slab_bytes, M, L.luts, 16, R, aq, as, out, out_ld, mt);
    } else {
        if (kind == 0) gemm_v1_kernel<false, 0><<<grid, 256, 0, st>>>(L.pool, L.slab_bytes, M, L.luts, 0, R, aq, as, out, out_ld, mt);
        else gemm_v1_kernel<false, 1><<<grid, 256, 0, st>>>(L.pool, L.slab_bytes, M, L.luts, 16, R, aq, as, out, out_ld, mt);
    }
    return 1;
}

int gemm_token_tile() { return kTN; }

}  // namespace inzg
