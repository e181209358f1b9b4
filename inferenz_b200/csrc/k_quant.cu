// k_quant.cu -- the expert encoder on the GPU: the engine's Q4L / Q8G quantizer for expert matrices, and seeded
// synthetic experts generated on the device.
//
// Output: byte for byte what the reference quantizer writes (inz_quantize, src/quant.c:422-556) under the
// converter's expert recipe (encode, src/convert.c:190-200): the 64-byte INZQ header, the packed indices
// [rows][ng][group bytes] and the fp16 scales [rows][ng]. No importance matrix is taken: the converter writes the
// synthetic experts without one, which the reference treats as all ones (src/quant.c:449-456).
//
// One batch is a set of matrices of one shape (the gate|up matrices of a range of experts, or their down matrices):
//  1. Rotation (rot_block > 1): one warp per (row, rotation block); lane l holds elements l + 32 i. Butterflies of
//     len < 32 pair lanes through shuffles, the wider ones pair registers of one lane. The stages run in the
//     reference's order (len = 1, 2, 4, ...), so every element sees the same IEEE adds (src/quant.c:118-154).
//  2. Level learning (Q4L): one CTA per matrix runs the weighted Lloyd-Max iterations (src/quant.c:369-418) on the
//     matrix's sample groups. Group fits are parallel: 8 lanes per 64-group, lane k holding elements 8m + k as the
//     reference's AVX accumulator lane k does, and the 8 lane partials meet in the reference's hsum8 tree. The
//     per-level sums are sequential double sums in the reference: each stays one chain here. Warp w owns levels 2w
//     and 2w + 1 and walks the chunk's groups in order; inside a group, a ballot mask of the entries on its level
//     gives them in ascending element order.
//  3. Final fit and packing: 8 lanes per 64-group, one CTA per slice of one matrix. Q8G: amax/127 scale, lrintf
//     to [-127, 127], +128 (src/quant.c:494-520).
// Every float operation is an explicitly rounded intrinsic (no contraction), matching the reference's SSE/AVX
// arithmetic, which has no flush-to-zero.
#include "inzg_internal.h"
#include "k_launch.h"
#include "host/inzg_host.h"

#include <cuda_fp16.h>
#include <float.h>
#include <math.h>
#include <string.h>

#include <algorithm>
#include <vector>

namespace inzg {

namespace {

constexpr uint32_t kQMagic = 0x515A4E49u;   // "INZQ"
constexpr int kSampleGroups = 8192;         // Lloyd-Max sample (lut_sample_groups default, src/quant.c:372)
constexpr int kLutIters = 5;                // Lloyd-Max iterations (lut_iters default, src/quant.c:374)
constexpr int kLearnCH = 128;               // sample groups fitted per chunk of the learning kernel
constexpr int kFitPasses = 4;               // passes of 32 groups per CTA of the final fit

// Lloyd-Max levels of a unit Gaussian, 4 bits (the reference's starting point, src/quant.c:177-185)
__constant__ float kGauss4[16] = {-2.7326f, -2.0690f, -1.6181f, -1.2562f, -0.9423f, -0.6568f, -0.3880f, -0.1284f,
                                  0.1284f,  0.3880f,  0.6568f,  0.9423f,  1.2562f,  1.6181f,  2.0690f,  2.7326f};
// candidate scale factors of one group fit (src/quant.c:254)
__constant__ float kCand[5] = {0.82f, 0.88f, 0.94f, 1.0f, 1.06f};

struct LevelSet {
    float L[16];  // sorted levels
    float T[16];  // midpoints T[k] = (L[k] + L[k+1]) / 2, k < 15
    float lmax;   // max |L|
};

// levels -> midpoints and largest magnitude (lvlset_init, src/quant.c:197-207); one thread
__device__ void levels_init(LevelSet &S) {
    float lmax = 0.0f;
    for (int k = 0; k < 16; k++) lmax = fmaxf(lmax, fabsf(S.L[k]));
    S.lmax = lmax;
    for (int k = 0; k < 15; k++) S.T[k] = __fmul_rn(0.5f, __fadd_rn(S.L[k], S.L[k + 1]));
    S.T[15] = 0.0f;
}

// index of the nearest level = number of midpoints strictly below v (lvl_assign, src/quant.c:209-213): a binary
// search over the sorted midpoints counts the same prefix; NaN compares false everywhere and gives 0, as there
__device__ __forceinline__ int assign16(const float *T, float v) {
    int i = T[7] < v ? 8 : 0;
    i += T[i + 3] < v ? 4 : 0;
    i += T[i + 1] < v ? 2 : 0;
    i += T[i] < v ? 1 : 0;
    return i;
}

// One 64-group fit (fit_group, src/quant.c:232-296) by the 8 lanes of an aligned lane octet: lane k holds
// x[m] = element 8m + k. Every lane of the warp must call it (the sums are shuffles). Returns the scale in d and
// this lane's 8 level indices.
__device__ void fit_group8(const float (&x)[8], const LevelSet &S, float &d_out, int (&idx)[8]) {
    float amax = 0.0f;
#pragma unroll
    for (int m = 0; m < 8; m++) amax = fmaxf(amax, fabsf(x[m]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    const float lmax = S.lmax;
    const bool zero = amax == 0.0f || lmax == 0.0f;
    const float base = __fdiv_rn(amax, lmax);
    float best_err = FLT_MAX, best_d = base;
#pragma unroll
    for (int m = 0; m < 8; m++) idx[m] = 0;
#pragma unroll 1
    for (int c = 0; c < 5; c++) {
        float d = __fmul_rn(base, kCand[c]);
        float inv = __fdiv_rn(1.0f, d);
        float num = 0.0f, den = 0.0f;
#pragma unroll
        for (int m = 0; m < 8; m++) {
            const float lv = S.L[assign16(S.T, __fmul_rn(x[m], inv))];
            num = __fmaf_rn(lv, x[m], num);  // weight 1: w * lv == lv
            den = __fmaf_rn(lv, lv, den);
        }
        const float dn = hsum8_lanes(den), nm = hsum8_lanes(num);
        if (dn > 0.0f) d = __fdiv_rn(nm, dn);
        const bool ok = d > 0.0f;  // the reference skips the candidate otherwise
        inv = __fdiv_rn(1.0f, d);
        float err = 0.0f;
        int I[8];
#pragma unroll
        for (int m = 0; m < 8; m++) {
            I[m] = assign16(S.T, __fmul_rn(x[m], inv));
            const float e = __fmaf_rn(-d, S.L[I[m]], x[m]);
            err = __fmaf_rn(__fmul_rn(e, e), 1.0f, err);
        }
        const float er = hsum8_lanes(err);
        if (ok && er < best_err) {
            best_err = er;
            best_d = d;
#pragma unroll
            for (int m = 0; m < 8; m++) idx[m] = I[m];
        }
    }
    if (best_err == FLT_MAX) {  // degenerate group: the amax scale
        const float inv = __fdiv_rn(1.0f, best_d);
#pragma unroll
        for (int m = 0; m < 8; m++) idx[m] = assign16(S.T, __fmul_rn(x[m], inv));
    }
    if (zero) {
        const int z = assign16(S.T, 0.0f);
#pragma unroll
        for (int m = 0; m < 8; m++) idx[m] = z;
        best_d = 0.0f;
    }
    d_out = best_d;
}

// ---------------------------------------------------------------------------------------------------------------
// 1. rotation: Wr[row] = rotate(W[row]), one warp per (row, block); block in {64, 128, 256}
template <int BLK>
__global__ void __launch_bounds__(256) rotate_rows_kernel(const float *__restrict__ W, float *__restrict__ Wr,
                                                          int64_t total_rows, int cols, uint32_t seed, float norm) {
    constexpr int R = BLK / 32;
    const int lane = threadIdx.x & 31;
    const int nb = cols / BLK;
    const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= total_rows * nb) return;
    const int64_t row = item / nb;
    const int b = (int)(item % nb);
    const float *src = W + row * cols + (int64_t)b * BLK;
    float *dst = Wr + row * cols + (int64_t)b * BLK;
    float v[R];
#pragma unroll
    for (int i = 0; i < R; i++) {
        v[i] = src[lane + 32 * i];
        if (rot_sign_bit(seed, (uint32_t)(b * BLK + lane + 32 * i))) v[i] = -v[i];
    }
#pragma unroll
    for (int len = 1; len < 32; len <<= 1)
#pragma unroll
        for (int i = 0; i < R; i++) {
            const float o = __shfl_xor_sync(0xffffffffu, v[i], len);
            v[i] = (lane & len) ? __fsub_rn(o, v[i]) : __fadd_rn(v[i], o);
        }
#pragma unroll
    for (int h = 1; h < R; h <<= 1)
#pragma unroll
        for (int i = 0; i < R; i++)
            if (!(i & h)) {
                const float a = v[i], c = v[i + h];
                v[i] = __fadd_rn(a, c);
                v[i + h] = __fsub_rn(a, c);
            }
#pragma unroll
    for (int i = 0; i < R; i++) dst[lane + 32 * i] = __fmul_rn(v[i], norm);
}

// ---------------------------------------------------------------------------------------------------------------
// 2. Q4L levels of each matrix (inz_learn_lut_rotated, src/quant.c:369-418): one CTA of 8 warps per matrix.
// Output: lut_out[matrix][16] in integer units (-63..63, sorted, distinct).
__global__ void __launch_bounds__(256) lut_learn_kernel(const float *__restrict__ Wr, int rows, int cols,
                                                        int64_t mat_stride, int ns, int64_t stride,
                                                        float *__restrict__ lut_out) {
    __shared__ LevelSet S;
    __shared__ float xs[kLearnCH][64];
    __shared__ uint8_t ix[kLearnCH][64];
    __shared__ float ds[kLearnCH];
    __shared__ double sums[16][2];
    const float *W = Wr + (int64_t)blockIdx.x * mat_stride;
    const int ng = cols / kGroup;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, k8 = lane & 7;
    if (tid < 16) S.L[tid] = __fdiv_rn(kGauss4[tid], kGauss4[15]);
    for (int it = 0; it < kLutIters; it++) {
        __syncthreads();
        if (tid == 0) levels_init(S);
        __syncthreads();
        // lane b < 2 of warp w: the sums of level 2w + b (numerator and denominator chains)
        const int lvl = 2 * warp + (lane & 1);
        double num = 0.0, den = 0.0;
        for (int c0 = 0; c0 < ns; c0 += kLearnCH) {
            const int nc = min(kLearnCH, ns - c0);
            for (int p0 = 0; p0 < kLearnCH; p0 += 32) {  // uniform trip count: every lane takes the shuffles
                const int p = p0 + warp * 4 + (lane >> 3);
                const bool valid = p < nc;
                float x[8];
                if (valid) {
                    const int64_t gi = (int64_t)(c0 + p) * stride;
                    const float *g = W + (gi / ng) * cols + (gi % ng) * kGroup + k8;
#pragma unroll
                    for (int m = 0; m < 8; m++) x[m] = g[8 * m];
                } else {
#pragma unroll
                    for (int m = 0; m < 8; m++) x[m] = 0.0f;
                }
                float d;
                int idx[8];
                fit_group8(x, S, d, idx);
                if (valid) {
#pragma unroll
                    for (int m = 0; m < 8; m++) {
                        xs[p][8 * m + k8] = x[m];
                        ix[p][8 * m + k8] = (uint8_t)idx[m];
                    }
                    if (k8 == 0) ds[p] = d;
                }
            }
            __syncthreads();
            for (int p = 0; p < nc; p++) {
                const float d = ds[p];
                if (d == 0.0f) continue;  // the reference skips all-zero groups (src/quant.c:390)
                const int ilo = ix[p][lane], ihi = ix[p][lane + 32];
                const float xlo = xs[p][lane], xhi = xs[p][lane + 32];
                const uint32_t a0 = __ballot_sync(0xffffffffu, ilo == 2 * warp);
                const uint32_t a1 = __ballot_sync(0xffffffffu, ilo == 2 * warp + 1);
                const uint32_t b0 = __ballot_sync(0xffffffffu, ihi == 2 * warp);
                const uint32_t b1 = __ballot_sync(0xffffffffu, ihi == 2 * warp + 1);
                uint32_t mlo = lane >= 2 ? 0u : (lane ? a1 : a0), mhi = lane >= 2 ? 0u : (lane ? b1 : b0);
                const double dd = (double)d, d2 = __dmul_rn(dd, dd);
                // entries of this lane's level in ascending element order: first j < 32, then j >= 32
                const int nlo = max(__popc(a0), __popc(a1)), nhi = max(__popc(b0), __popc(b1));
                for (int t = 0; t < nlo; t++) {
                    const int j = __ffs(mlo) - 1;
                    const float xj = __shfl_sync(0xffffffffu, xlo, j & 31);
                    if (mlo) {
                        num = __dadd_rn(num, __dmul_rn(dd, (double)xj));
                        den = __dadd_rn(den, d2);
                        mlo &= mlo - 1;
                    }
                }
                for (int t = 0; t < nhi; t++) {
                    const int j = __ffs(mhi) - 1;
                    const float xj = __shfl_sync(0xffffffffu, xhi, j & 31);
                    if (mhi) {
                        num = __dadd_rn(num, __dmul_rn(dd, (double)xj));
                        den = __dadd_rn(den, d2);
                        mhi &= mhi - 1;
                    }
                }
            }
            __syncthreads();
        }
        if (lane < 2) {
            sums[lvl][0] = num;
            sums[lvl][1] = den;
        }
        __syncthreads();
        if (tid < 16 && sums[tid][1] > 0.0) S.L[tid] = __double2float_rn(__ddiv_rn(sums[tid][0], sums[tid][1]));
        __syncthreads();
        if (tid == 0) {  // ascending order (insertion sort, src/quant.c:400-405: any sort yields the same array)
            for (int a = 1; a < 16; a++) {
                const float v = S.L[a];
                int b = a - 1;
                while (b >= 0 && S.L[b] > v) {
                    S.L[b + 1] = S.L[b];
                    b--;
                }
                S.L[b + 1] = v;
            }
        }
    }
    __syncthreads();
    if (tid == 0) {  // integer units, clamped, duplicates nudged apart (src/quant.c:407-415)
        float lmax = 0.0f;
        for (int k = 0; k < 16; k++) lmax = fmaxf(lmax, fabsf(S.L[k]));
        float out[16];
        for (int k = 0; k < 16; k++) {
            int v = __float2int_rn(__fmul_rn(__fdiv_rn(S.L[k], lmax), 63.0f));
            v = v < -63 ? -63 : v > 63 ? 63 : v;
            out[k] = (float)v;
        }
        for (int k = 1; k < 16; k++)
            if (out[k] <= out[k - 1]) out[k] = out[k - 1] + 1.0f;
        for (int k = 0; k < 16; k++) lut_out[(size_t)blockIdx.x * 16 + k] = out[k];
    }
}

// ---------------------------------------------------------------------------------------------------------------
// 3. final fit and packing: grid (slices, matrices); 8 warps x 4 groups x kFitPasses groups per CTA
template <bool Q8>
__global__ void __launch_bounds__(256) fit_pack_kernel(const float *__restrict__ Wr, int rows, int cols,
                                                       int64_t mat_stride, const float *__restrict__ luts, int rot,
                                                       uint32_t seed, uint8_t *__restrict__ out, uint64_t out_stride) {
    __shared__ LevelSet S;
    const int mi = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, k8 = lane & 7;
    if (!Q8) {
        if (tid < 16) S.L[tid] = luts[(size_t)mi * 16 + tid];
        __syncthreads();
        if (tid == 0) levels_init(S);
        __syncthreads();
    }
    const int ng = cols / kGroup;
    const int64_t total = (int64_t)rows * ng;
    const int gb = Q8 ? 64 : 32;
    uint8_t *o = out + (uint64_t)mi * out_stride;
    uint8_t *qout = o + 64;
    uint16_t *dout = reinterpret_cast<uint16_t *>(qout + total * gb);
    const float *W = Wr + (int64_t)mi * mat_stride;
    if (blockIdx.x == 0 && tid < 64) {  // header (src/quant.c:440-448); the rest of it stays zero
        uint8_t hb = 0;
        const uint32_t w32[6] = {kQMagic, (uint32_t)(Q8 ? INZG_T_Q8G : INZG_T_Q4L) | ((uint32_t)rot << 16),
                                 (uint32_t)rows, (uint32_t)cols, seed, Q8 ? 8u : 4u};
        if (tid < 24) hb = (uint8_t)(w32[tid / 4] >> (8 * (tid % 4)));
        else if (!Q8 && tid >= 24 && tid < 40) hb = (uint8_t)((int)S.L[tid - 24] + kLutBias);
        o[tid] = hb;
    }
    for (int pass = 0; pass < kFitPasses; pass++) {
        const int64_t gi = ((int64_t)blockIdx.x * kFitPasses + pass) * 32 + warp * 4 + (lane >> 3);
        const bool valid = gi < total;
        float x[8];
        if (valid) {
            const float *g = W + (gi / ng) * cols + (gi % ng) * kGroup + k8;
#pragma unroll
            for (int m = 0; m < 8; m++) x[m] = g[8 * m];
        } else {
#pragma unroll
            for (int m = 0; m < 8; m++) x[m] = 0.0f;
        }
        if (Q8) {
            float amax = 0.0f;
#pragma unroll
            for (int m = 0; m < 8; m++) amax = fmaxf(amax, fabsf(x[m]));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            const float d = __fdiv_rn(amax, 127.0f);
            const float inv = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            if (valid) {
#pragma unroll
                for (int m = 0; m < 8; m++) {
                    int q = __float2int_rn(__fmul_rn(x[m], inv));
                    q = q < -127 ? -127 : q > 127 ? 127 : q;
                    qout[gi * 64 + 8 * m + k8] = (uint8_t)(q + 128);
                }
                if (k8 == 0) dout[gi] = __half_as_ushort(__float2half_rn(d));
            }
        } else {
            float d;
            int idx[8];
            fit_group8(x, S, d, idx);
            if (valid) {
#pragma unroll
                for (int m = 0; m < 4; m++) qout[gi * 32 + 8 * m + k8] = (uint8_t)(idx[m] | (idx[m + 4] << 4));
                if (k8 == 0) dout[gi] = __half_as_ushort(__float2half_rn(d));
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------
// Seeded synthetic experts on the device: the LCG + Box-Muller normal of the reference's tests
// (tests/test_quant.c:10-17) in its draw order (per expert: gate [FF][H], up [FF][H], down [H][FF], row-major).
// The LCG is exact integer arithmetic; the transform uses CUDA's double log, cos and sqrt, which agree with glibc's
// to within an ulp or two of double, so a float draw can differ from the host generator's only when the double
// result lies within that distance of a float rounding boundary.
constexpr uint64_t kLcgA = 6364136223846793005ull, kLcgC = 1442695040888963407ull;
constexpr int kSynthSeg = 512;  // draws per thread

__device__ __forceinline__ uint64_t lcg_jump_dev(uint64_t s, uint64_t n) {
    uint64_t acc_a = 1, acc_c = 0, a = kLcgA, c = kLcgC;
    while (n) {
        if (n & 1) {
            acc_a *= a;
            acc_c = acc_c * a + c;
        }
        c = c * a + c;
        a *= a;
        n >>= 1;
    }
    return s * acc_a + acc_c;
}

__device__ __forceinline__ float randn_dev(uint64_t &s) {
    s = s * kLcgA + kLcgC;
    const double u1 = __ddiv_rn(__dadd_rn((double)(s >> 11), 1.0), 9007199254740992.0);
    s = s * kLcgA + kLcgC;
    const double u2 = __ddiv_rn((double)(s >> 11), 9007199254740992.0);
    const double r = sqrt(__dmul_rn(-2.0, log(u1)));
    return __double2float_rn(__dmul_rn(r, cos(__dmul_rn(6.283185307179586, u2))));
}

// experts [e0, e0 + ne): gu [ne][2FF][H], dn [ne][H][FF]
__global__ void synth_experts_kernel(uint64_t seed, int H, int FF, int e0, int ne, float sd, float *__restrict__ gu,
                                     float *__restrict__ dn) {
    const uint64_t per = (uint64_t)3 * FF * H, ngu = (uint64_t)2 * FF * H;
    const uint64_t total = per * ne;
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t first = t * kSynthSeg;
    if (first >= total) return;
    const uint64_t last = min(first + kSynthSeg, total);
    uint64_t s = lcg_jump_dev(seed, 2 * (per * (uint64_t)e0 + first));
    for (uint64_t i = first; i < last; i++) {
        const float v = __fmul_rn(randn_dev(s), sd);
        const uint64_t e = i / per, r = i % per;
        if (r < ngu) gu[e * ngu + r] = v;
        else dn[e * (per - ngu) + (r - ngu)] = v;
    }
}

}  // namespace

// ---------------------------------------------------------------------------------------------------------------
// host side

int auto_rot_block(int cols) {
    for (int b = 256; b >= kGroup; b >>= 1)
        if (cols % b == 0) return b;
    return 0;
}

// Quantize `count` matrices W[i] = W + i * rows * cols (device fp32) into out + i * out_stride (device; the caller
// zero-fills the output first). scratch: count * rows * cols floats when the matrices are rotated, plus count * 16
// floats. Returns 0, or -1 for an unsupported type or shape.
static int encode_batch(const float *W, int count, int rows, int cols, int type, int rot_block, uint32_t rot_seed,
                        uint8_t *out, uint64_t out_stride, float *scratch, cudaStream_t st) {
    if ((type != INZG_T_Q4L && type != INZG_T_Q8G) || rows <= 0 || cols <= 0 || cols % kGroup || count <= 0) return -1;
    int hdr_rot = rot_block == 0 ? auto_rot_block(cols) : rot_block < 0 ? 0 : rot_block;
    if (type == INZG_T_Q8G && rot_block <= 0) hdr_rot = 0;  // Q8G is rotated only on request (src/quant.c:432-434)
    if (hdr_rot && cols % hdr_rot) return -1;
    const int rot = hdr_rot > 1 ? hdr_rot : 0;  // a block of 1 is stored but rotates nothing (src/quant.c:147)
    if (rot && rot != 64 && rot != 128 && rot != 256) return -1;
    const uint32_t seed = rot_seed ? rot_seed : 0x5EEDu;
    const int64_t mat = (int64_t)rows * cols;
    const float *Wr = W;
    float *luts = scratch + (rot ? (size_t)count * mat : 0);
    if (rot) {
        float *R = scratch;
        const float norm = 1.0f / sqrtf((float)rot);
        const int64_t items = (int64_t)count * rows * (cols / rot);
        const int blocks = (int)((items + 7) / 8);
        if (rot == 256) rotate_rows_kernel<256><<<blocks, 256, 0, st>>>(W, R, (int64_t)count * rows, cols, seed, norm);
        else if (rot == 128) rotate_rows_kernel<128><<<blocks, 256, 0, st>>>(W, R, (int64_t)count * rows, cols, seed, norm);
        else rotate_rows_kernel<64><<<blocks, 256, 0, st>>>(W, R, (int64_t)count * rows, cols, seed, norm);
        Wr = R;
    }
    const int64_t total = (int64_t)rows * (cols / kGroup);
    const dim3 grid((unsigned)((total + 32 * kFitPasses - 1) / (32 * kFitPasses)), (unsigned)count);
    if (type == INZG_T_Q4L) {
        const int ns = (int)std::min<int64_t>(kSampleGroups, total);
        lut_learn_kernel<<<count, 256, 0, st>>>(Wr, rows, cols, mat, ns, total / ns, luts);
        fit_pack_kernel<false><<<grid, 256, 0, st>>>(Wr, rows, cols, mat, luts, hdr_rot, seed, out, out_stride);
    } else {
        fit_pack_kernel<true><<<grid, 256, 0, st>>>(Wr, rows, cols, mat, luts, hdr_rot, seed, out, out_stride);
    }
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace inzg

using namespace inzg;

namespace {

size_t qmat_bytes(int type, int rows, int cols) {
    const size_t gb = type == INZG_T_Q4L ? 32 : type == INZG_T_Q8G ? 64 : 0;
    const size_t ng = (size_t)cols / kGroup;
    const size_t n = 64 + (size_t)rows * ng * gb + (size_t)rows * ng * 2;
    return (n + 63) / 64 * 64;
}

uint64_t blob_bytes(int type, int H, int FF) {
    const uint64_t b = qmat_bytes(type, 2 * FF, H) + qmat_bytes(type, H, FF);
    return (b + 4095) / 4096 * 4096;
}

// Encode ne experts from device fp32 (gu [ne][2FF][H], dn [ne][H][FF]) into device blobs [ne][blob_bytes] with the
// converter's recipe: Q4L with the automatic rotation, Q8G rotated with the automatic block (rot8 default,
// src/convert.c:157, 195-198). scratch: ne * 3 * FF * H + ne * 32 floats.
int encode_experts(const float *gu, const float *dn, int ne, int type, int H, int FF, uint8_t *blobs, float *scratch,
                   cudaStream_t st) {
    const uint64_t bb = blob_bytes(type, H, FF), gub = qmat_bytes(type, 2 * FF, H);
    if (cudaMemsetAsync(blobs, 0, bb * ne, st) != cudaSuccess) return -1;
    const int rg = type == INZG_T_Q8G ? auto_rot_block(H) : 0, rd = type == INZG_T_Q8G ? auto_rot_block(FF) : 0;
    float *s_gu = scratch, *s_dn = scratch + (size_t)ne * 2 * FF * H + (size_t)ne * 16;
    if (encode_batch(gu, ne, 2 * FF, H, type, rg, 0, blobs, bb, s_gu, st)) return -1;
    return encode_batch(dn, ne, H, FF, type, rd, 0, blobs + gub, bb, s_dn, st);
}

size_t encode_scratch_floats(int ne, int H, int FF) { return (size_t)ne * 3 * FF * H + (size_t)ne * 32; }

struct DevBuf {
    void *p = nullptr;
    bool alloc(size_t bytes) {
        if (cudaMalloc(&p, bytes ? bytes : 1) != cudaSuccess) {
            cudaGetLastError();
            p = nullptr;
            return false;
        }
        return true;
    }
    ~DevBuf() {
        if (p) cudaFree(p);
    }
};

constexpr int kExpertBatch = 16;   // experts per device batch of the host-drawn layer generators
constexpr int kDeviceBatch = 128;  // experts per batch when drawn on the device too (one level-learning CTA each)

}  // namespace

extern "C" {

INZG_API size_t inzg_qmat_bytes(int type, int rows, int cols) { return qmat_bytes(type, rows, cols); }
INZG_API int inzg_auto_rot_block(int cols) { return auto_rot_block(cols); }
INZG_API uint64_t inzg_blob_bytes(int type, int H, int FF) { return blob_bytes(type, H, FF); }

INZG_API int inzg_quantize_device(const float *W_dev, int rows, int cols, int type, int rot_block, uint32_t rot_seed,
                                  void *out_dev, void *stream) {
    if (!W_dev || !out_dev || (type != INZG_T_Q4L && type != INZG_T_Q8G) || rows <= 0 || cols <= 0 || cols % kGroup)
        return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    DevBuf scratch;
    if (!scratch.alloc(sizeof(float) * ((size_t)rows * cols + 16))) return -1;
    if (cudaMemsetAsync(out_dev, 0, qmat_bytes(type, rows, cols), st) != cudaSuccess) return -1;
    if (encode_batch(W_dev, 1, rows, cols, type, rot_block, rot_seed, static_cast<uint8_t *>(out_dev), 0,
                     static_cast<float *>(scratch.p), st))
        return -1;
    return cudaStreamSynchronize(st) == cudaSuccess ? 0 : -1;
}

INZG_API int inzg_quantize(const float *W, int rows, int cols, int type, int rot_block, uint32_t rot_seed, void *out) {
    if (!W || !out || (type != INZG_T_Q4L && type != INZG_T_Q8G) || rows <= 0 || cols <= 0 || cols % kGroup) return -1;
    const size_t nb = qmat_bytes(type, rows, cols), nw = (size_t)rows * cols;
    DevBuf w, o;
    if (!w.alloc(sizeof(float) * nw) || !o.alloc(nb)) return -1;
    if (cudaMemcpy(w.p, W, sizeof(float) * nw, cudaMemcpyHostToDevice) != cudaSuccess) return -1;
    if (inzg_quantize_device(static_cast<float *>(w.p), rows, cols, type, rot_block, rot_seed, o.p, nullptr)) return -1;
    return cudaMemcpy(out, o.p, nb, cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -1;
}

INZG_API int inzg_encode_experts_device(const float *gu_dev, const float *dn_dev, int n, int type, int H, int FF,
                                        void *blobs_dev, void *stream) {
    if (!gu_dev || !dn_dev || !blobs_dev || n <= 0 || (type != INZG_T_Q4L && type != INZG_T_Q8G) || H % kGroup ||
        FF % kGroup)
        return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    DevBuf scratch;
    if (!scratch.alloc(sizeof(float) * encode_scratch_floats(n, H, FF))) return -1;
    if (encode_experts(gu_dev, dn_dev, n, type, H, FF, static_cast<uint8_t *>(blobs_dev),
                       static_cast<float *>(scratch.p), st))
        return -1;
    return cudaStreamSynchronize(st) == cudaSuccess ? 0 : -1;
}

INZG_API int inzg_encode_expert(const float *GU, const float *D, int type, int H, int FF, void *blob) {
    if (!GU || !D || !blob) return -1;
    const size_t ngu = (size_t)2 * FF * H, ndn = (size_t)H * FF;
    const uint64_t bb = blob_bytes(type, H, FF);
    DevBuf g, d, o;
    if (!g.alloc(sizeof(float) * ngu) || !d.alloc(sizeof(float) * ndn) || !o.alloc(bb)) return -1;
    if (cudaMemcpy(g.p, GU, sizeof(float) * ngu, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(d.p, D, sizeof(float) * ndn, cudaMemcpyHostToDevice) != cudaSuccess)
        return -1;
    if (inzg_encode_experts_device(static_cast<float *>(g.p), static_cast<float *>(d.p), 1, type, H, FF, o.p, nullptr))
        return -1;
    return cudaMemcpy(blob, o.p, bb, cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -1;
}

INZG_API int inzg_synth_experts_device(uint64_t seed, int H, int FF, int e0, int n, float *gu_dev, float *dn_dev,
                                       void *stream) {
    if (n <= 0 || e0 < 0 || !gu_dev || !dn_dev || H <= 0 || FF <= 0) return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const uint64_t threads = ((uint64_t)3 * FF * H * n + kSynthSeg - 1) / kSynthSeg;
    synth_experts_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(seed, H, FF, e0, n, (float)sqrt(1.0 / H),
                                                                          gu_dev, dn_dev);
    if (cudaGetLastError() != cudaSuccess) return -1;
    return cudaStreamSynchronize(st) == cudaSuccess ? 0 : -1;
}

// Experts [e0, e1) of a synthetic layer, generated on the device and encoded there: blobs_dev [(e1-e0)][blob_bytes].
INZG_API int inzg_synth_layer_blobs_device(uint64_t seed, int type, int H, int FF, int e0, int e1, void *blobs_dev,
                                           void *stream) {
    if (e1 <= e0 || e0 < 0 || !blobs_dev || (type != INZG_T_Q4L && type != INZG_T_Q8G) || H % kGroup || FF % kGroup)
        return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int nb = std::min(kDeviceBatch, e1 - e0);
    const size_t per = (size_t)3 * FF * H;
    DevBuf wbuf, scratch;
    if (!wbuf.alloc(sizeof(float) * per * nb) || !scratch.alloc(sizeof(float) * encode_scratch_floats(nb, H, FF)))
        return -1;
    float *gu = static_cast<float *>(wbuf.p), *dn = gu + (size_t)nb * 2 * FF * H;
    const float sd = (float)sqrt(1.0 / H);
    const uint64_t bb = blob_bytes(type, H, FF);
    for (int e = e0; e < e1; e += nb) {
        const int ne = std::min(nb, e1 - e);
        const uint64_t threads = (per * ne + kSynthSeg - 1) / kSynthSeg;
        synth_experts_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(seed, H, FF, e, ne, sd, gu, dn);
        if (encode_experts(gu, dn, ne, type, H, FF, static_cast<uint8_t *>(blobs_dev) + (size_t)(e - e0) * bb,
                           static_cast<float *>(scratch.p), st))
            return -1;
    }
    return cudaStreamSynchronize(st) == cudaSuccess ? 0 : -1;
}

// Host-generated experts (the host generator draws the reference's exact stream), encoded on the device.
// expert experts[i] lands at out + (experts[i] - base) * blob_bytes
static int host_experts_to_blobs(uint64_t seed, int type, int H, int FF, const int32_t *experts, int n, uint8_t *out,
                                 int base) {
    const int nb = std::min(kExpertBatch, n);
    const size_t ngu = (size_t)2 * FF * H, ndn = (size_t)H * FF;
    const uint64_t bb = blob_bytes(type, H, FF);
    std::vector<float> hgu(ngu * nb), hdn(ndn * nb);
    DevBuf wbuf, obuf, scratch;
    if (!wbuf.alloc(sizeof(float) * (ngu + ndn) * nb) || !obuf.alloc(bb * nb) ||
        !scratch.alloc(sizeof(float) * encode_scratch_floats(nb, H, FF)))
        return -1;
    float *gu = static_cast<float *>(wbuf.p), *dn = gu + ngu * nb;
    for (int i0 = 0; i0 < n; i0 += nb) {
        const int ne = std::min(nb, n - i0);
        inzg__synth_experts_host(seed, H, FF, experts + i0, ne, hgu.data(), hdn.data());
        if (cudaMemcpy(gu, hgu.data(), sizeof(float) * ngu * ne, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(dn, hdn.data(), sizeof(float) * ndn * ne, cudaMemcpyHostToDevice) != cudaSuccess)
            return -1;
        if (encode_experts(gu, dn, ne, type, H, FF, static_cast<uint8_t *>(obuf.p), static_cast<float *>(scratch.p),
                           nullptr))
            return -1;
        for (int i = 0; i < ne; i++)
            if (cudaMemcpy(out + (size_t)(experts[i0 + i] - base) * bb, static_cast<uint8_t *>(obuf.p) + (size_t)i * bb, bb,
                           cudaMemcpyDeviceToHost) != cudaSuccess)
                return -1;
    }
    return 0;
}

INZG_API int inzg_synth_layer_blobs(uint64_t seed, int type, int H, int FF, int e0, int e1, void *blobs) {
    if (e1 <= e0 || e0 < 0 || !blobs || (type != INZG_T_Q4L && type != INZG_T_Q8G) || H % kGroup || FF % kGroup)
        return -1;
    std::vector<int32_t> ex(e1 - e0);
    for (int e = e0; e < e1; e++) ex[e - e0] = e;
    return host_experts_to_blobs(seed, type, H, FF, ex.data(), e1 - e0, static_cast<uint8_t *>(blobs), e0);
}

INZG_API int inzg_synth_layer_blobs_subset(uint64_t seed, int type, int H, int FF, int E, const int32_t *experts,
                                           int n_experts, void *blobs) {
    if (!blobs || !experts || n_experts <= 0 || (type != INZG_T_Q4L && type != INZG_T_Q8G)) return -1;
    const uint64_t bb = blob_bytes(type, H, FF), gub = qmat_bytes(type, 2 * FF, H);
    uint8_t *out = static_cast<uint8_t *>(blobs);
    memset(out, 0, bb * (size_t)E);
    for (int i = 0; i < n_experts; i++)
        if (experts[i] < 0 || experts[i] >= E) return -1;
    if (host_experts_to_blobs(seed, type, H, FF, experts, n_experts, out, 0)) return -1;
    // every other expert: the first listed expert's two headers and a zero payload (valid, never routed to)
    const uint8_t *src = out + (size_t)experts[0] * bb;
    for (int e = 0; e < E; e++) {
        uint8_t *dst = out + (size_t)e * bb;
        uint32_t magic;
        memcpy(&magic, dst, 4);
        if (magic == kQMagic) continue;
        memcpy(dst, src, 64);
        memcpy(dst + gub, src + gub, 64);
    }
    return 0;
}

}  // extern "C"
