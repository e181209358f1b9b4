// k_gemv.cu -- decode-path grouped GEMV over the routed experts (Q4L / Q8G), sm_100a.
//
// Numerics: the reference's decode matvec, bit for bit (mv_q4l / mm_q4l: src/quant.c:767-875, 1179-1225; mv_q8g /
// mm_q8g: src/quant.c:881-953, VNNI form). Per row and token the reference keeps 8 fp32 accumulators; accumulator l
// takes, for every 64-group g in order,
//     acc_l = fma((float)I_lg, d_g * s_g, acc_l),   I_lg = sum_{i<4} u[4l+i] x[4l+i] + u[32+4l+i] x[32+4l+i]
// (I_lg is the 32-bit lane l of two VPDPBUSD over the group's two 32-byte halves; u = biased LUT level or raw byte),
// then y = hsum8(acc) - bias * b, where b is the fma chain of d_g * bsum_g: Q4L keeps 8 chains (g % 8) over the
// first ng & ~7 groups, reduces them with hsum8 and continues with the remaining groups in order; Q8G keeps one chain.
//
// Tensor pipe: the lane partials I_lg come straight out of the int8 MMA (mma.m16n8k32, u8 x s8 -> s32). The K = 32 of
// one MMA holds 4 lanes x 8 elements (element i < 4: x[4l+i], else x[32+4l+i-4]); the activation operand is
// block-diagonal -- column n carries lane n's 8 activations in lane n's rows and zeros elsewhere -- so D[row][n] is
// exactly I_n. Two tokens share the 8 columns (token A lanes in columns 0-3, token B in 4-7), so two MMAs (lanes 0-3,
// lanes 4-7) give all 8 partials of a 16-row tile for two tokens. Thread (r, t) of the MMA holds, for token t >> 1,
// lanes 2(t&1), 2(t&1)+1 of both MMAs for rows r and r+8, folds them into its accumulators with the reference's fma
// (packed f32x2 instructions, each lane rounded as its own fma), and hsum8 becomes one add per lane pair and one quad
// shuffle that pair the lanes as the reference does: ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)).
//
// Pipeline (one CTA per SM, persistent): an item is up to W row tiles of 16 rows of one decode expert's matrix (W = 15
// for calls of 4 tokens or more, 8 below; the last item of a matrix holds the remaining tiles). A producer warp takes
// items from the call's work queue (experts with the most tokens first), brings the item's token activations, their
// (s, bsum) and the item's row-tile scales into a double-buffered item buffer, and streams the weights in stages of
// 2-8 64-groups through a 3- or 4-deep ring -- all with bulk copies (cp.async.bulk on the TMA engine, completion
// counted on mbarriers). W consumer warps each own one 16-row tile of the item: per group, the LUT decode of the
// weight fragment, then two MMAs and the reference's fma per token. The bias chains need only the
// scales and bsum, so they run once per item in the epilogue. Every wait is bounded; a CTA that gives up records
// INZG_TIMEOUT and drains its copies before it leaves.
//
// GEMM items (calls of 9-32 tokens): the experts such a call sends down the reference's prefill numerics (>= 12 tokens)
// run in the same launch instead of a separate gather + GEMM. Their items -- up to 15 row tiles of one expert with all
// its tokens -- lead the work queue; a stage then carries 128 bytes of K of the requantized int8 row tiles (tensor
// copies) and of the token rows (bulk copies), and each warp runs ldmatrix + s8 x s8 MMAs with the per-256-block fp32
// fold (gemm_item). The kernel instantiation with GEMM items takes them in a loop of their own before the decode loop;
// calls without them run the decode-only instantiation.
#include "inzg_internal.h"
#include "k_async.cuh"
#include "k_launch.h"
#include "k_gemv_core.cuh"

#include <cuda_fp16.h>
#include <string.h>

namespace inzg {

template <bool Q8, int NG, int KIND, int W = 8, bool HG = false>
struct DecGeo {
    // Consumer warps, one 16-row tile each: an item is up to W row tiles of one expert matrix (the last item of a
    // matrix holds the remaining tiles). W = 8: 9 warps per CTA, items of 128 rows, for calls of a few tokens whose
    // items are fewer than the SMs. W = 15: 16 warps per CTA -- 4 per SM sub-partition, whose 16 K registers then
    // allow 128 per thread -- so twice the warps hide the latency of the decode -> MMA -> fold chains.
    static constexpr int WARPS = W;
    static constexpr int STAGES = (W > 8 && NG >= 40) ? 3 : 4;
    static constexpr int KC = W > 8 ? (Q8 ? 2 : 4) : (Q8 ? 4 : 8);  // 64-groups per stage
    static constexpr int NCH = (NG + KC - 1) / KC;   // stages per item
    static constexpr int NG8 = NG & ~7;
    static constexpr int WB = Q8 ? 32 : 16;          // weight bytes per lane per group
    static constexpr int GD = (NG + 3) / 4;
    static constexpr int WQ = KC * 32 * WB;          // weight bytes of one row tile in one stage
    // GEMM items (wide geometry only) also bring, per stage, the 128-byte K chunk of each of their <= 32 token rows,
    // after the weights at a padded stride (the 8 rows an ldmatrix reads fall in 8 different bank quads)
    static constexpr int TSTR = 144, TOK = HG ? 32 * TSTR : 0;
    static constexpr int STAGE = (WARPS * WQ + TOK + 1023) / 1024 * 1024;
    static constexpr int K = NG * kGroup;
    static constexpr int MT = 12;                    // most tokens of a decode expert: 11 (8 when n <= 8)
    // item buffer: token activations [MT][K], their (s, bsum) [MT][NG], the row tiles' scales [WARPS][GD][8][4][2]
    static constexpr int IB_SB = MT * K, IB_D = IB_SB + MT * NG * 8;
    static constexpr int IBUF = ((IB_D + WARPS * GD * 128) + 127) / 128 * 128;
    static constexpr int HDR = 1024;
    static constexpr int SMEM = HDR + STAGES * STAGE + 2 * IBUF;
    static constexpr int THREADS = (WARPS + 1) * 32;
};

// Item descriptor written by the producer warp, read by the consumers after the item's buffer has landed
// (e == kDecEnd: the work queue is empty).
constexpr int kDecEnd = -3;
constexpr int kGemmEnd = -4;  // the CTA's GEMM items are over: decode items follow
struct DecItem {
    int e, base, ntok, rb, ntiles;
    uint4 lut;
    int oslot[32];  // down matrix: each token's output slot and routing weight (decode items <= 12 tokens, GEMM
    float ow[32];   // items <= 32)
    int trow[32];   // GEMM items: activation row of each token (gate|up: the token, down: the entry)
};

struct DecShared {
    uint64_t full[4], empty[4], afull[2], aempty[2];
    int abort, never;  // never: drains ignore the abort flag
    DecItem item[2];
};

// Consumer: the item's TC >= ntok tokens on this warp's 16-row tile. q: running stage counter (advanced by NCH).
template <bool Q8, int NG, int KIND, int W, bool HG, int TC>
__device__ __forceinline__ bool dec_item(DecShared &S, const uint8_t *stages, const uint8_t *ib, const DecItem &it,
                                         int &q, float *__restrict__ out, int out_ld, uint32_t one) {
    using G = DecGeo<Q8, NG, KIND, W, HG>;
    volatile int *abort = &S.abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gr = lane >> 2, t = lane & 3;
    // Tokens go through the MMAs in pairs (A = 2p, B = 2p + 1). Column n = gr of the activation operand carries token
    // 2p + (n >> 2), chain lane 4h + (n & 3) in MMA h, block-diagonally: its 8 activations sit in the K rows of lane
    // n & 3 and the rest of the column is zero. Thread (gr, t) holds K rows 4t..4t+3 (register 0) and 16+4t.. (register
    // 1), i.e. the first or second half (t & 1) of lane t >> 1 (register 0) or lane 2 + (t >> 1) (register 1).
    // (0/1 factors: the operand is selected with an integer multiply, which issues on the FMA pipe)
    const int lc = gr & 3;
    const uint32_t s0 = lc == (t >> 1) ? one : 0u, s1 = lc == 2 + (t >> 1) ? one : 0u;
    const uint32_t k16 = one << 16;
    const uint8_t *xq = ib + (size_t)(gr >> 2) * G::K + 32 * (t & 1) + 4 * lc;
    const float2 *xsb = reinterpret_cast<const float2 *>(ib + G::IB_SB);
    // scale pairs (d[r][g], d[r+8][g]) of this warp's row tile: word (g / 4) * 32 + gr * 4 + g % 4
    const uint32_t *wd = reinterpret_cast<const uint32_t *>(ib + G::IB_D + (size_t)warp * G::GD * 128) + gr * 4;
    const uint4 T = it.lut;
    const bool valid = it.e >= 0 && warp < it.ntiles;  // the last item of a matrix may hold fewer tiles than warps
    const int ntok = it.ntok;
    constexpr int NP = (TC + 1) / 2;
    const int jcol = gr >> 2, jd = t >> 1;  // token of this thread's operand column / of its accumulator columns

    // acc[p][h][r]: token 2p + jd, row gr + 8r, chain lanes 4h + 2(t & 1) and 4h + 2(t & 1) + 1
    float2 acc[NP][2][2];
#pragma unroll
    for (int p = 0; p < NP; p++)
#pragma unroll
        for (int h = 0; h < 2; h++) acc[p][h][0] = acc[p][h][1] = make_float2(0.0f, 0.0f);
    const float2 neg_magic = make_float2(-12582912.0f, -12582912.0f);

    // one 64-group: g global index, i index inside the stage
    auto group = [&](const uint8_t *wq, int g, int i) {
        uint32_t A0[4], A1[4];  // MMA h = 0 (lanes 0-3) and h = 1 (lanes 4-7)
        if (Q8) {
            const uint4 w0 = *reinterpret_cast<const uint4 *>(wq + (size_t)i * 1024);
            const uint4 w1 = *reinterpret_cast<const uint4 *>(wq + (size_t)i * 1024 + 512);
            A0[0] = w0.x; A0[1] = w0.y; A0[2] = w0.z; A0[3] = w0.w;
            A1[0] = w1.x; A1[1] = w1.y; A1[2] = w1.z; A1[3] = w1.w;
        } else {
            const uint4 w = *reinterpret_cast<const uint4 *>(wq + (size_t)i * 512);
            const uint4 x = make_uint4(w.x ^ 0x88888888u, w.y ^ 0x88888888u, w.z ^ 0x88888888u, w.w ^ 0x88888888u);
            A0[0] = lut16(w.x, x.x, T, one); A0[1] = lut16(w.y, x.y, T, one);
            A0[2] = lut16(hi16(w.x, k16), hi16(x.x, k16), T, one); A0[3] = lut16(hi16(w.y, k16), hi16(x.y, k16), T, one);
            A1[0] = lut16(w.z, x.z, T, one); A1[1] = lut16(w.w, x.w, T, one);
            A1[2] = lut16(hi16(w.z, k16), hi16(x.z, k16), T, one); A1[3] = lut16(hi16(w.w, k16), hi16(x.w, k16), T, one);
        }
        const float2 dd = h2f16x2(wd[(g >> 2) * 32 + (g & 3)]);
#pragma unroll
        for (int p = 0; p < NP; p++) {
            if (2 * p >= ntok) continue;
            const bool col_live = 2 * p + jcol < ntok;
            const uint8_t *xp = xq + (size_t)(2 * p) * G::K + g * kGroup;
            const uint32_t x0 = col_live ? *reinterpret_cast<const uint32_t *>(xp) : 0u;
            const uint32_t x1 = col_live ? *reinterpret_cast<const uint32_t *>(xp + 16) : 0u;
            const float sx = 2 * p + jd < ntok ? xsb[(2 * p + jd) * NG + g].x : 0.0f;
            // the accumulators start at the bits of 1.5 * 2^23: D then holds 12582912 + I as a float (|I| < 2^22)
            int D0[4], D1[4];
            mma_u8s8_c(D0, A0[0], A0[1], A0[2], A0[3], x0 * s0, x0 * s1, 0x4B400000);
            mma_u8s8_c(D1, A1[0], A1[1], A1[2], A1[3], x1 * s0, x1 * s1, 0x4B400000);
            const float ds0 = __fmul_rn(dd.x, sx), ds8 = __fmul_rn(dd.y, sx);
            const float2 m0 = make_float2(ds0, ds0), m8 = make_float2(ds8, ds8);
            acc[p][0][0] = __ffma2_rn(__fadd2_rn(make_float2(__int_as_float(D0[0]), __int_as_float(D0[1])), neg_magic),
                                      m0, acc[p][0][0]);
            acc[p][0][1] = __ffma2_rn(__fadd2_rn(make_float2(__int_as_float(D0[2]), __int_as_float(D0[3])), neg_magic),
                                      m8, acc[p][0][1]);
            acc[p][1][0] = __ffma2_rn(__fadd2_rn(make_float2(__int_as_float(D1[0]), __int_as_float(D1[1])), neg_magic),
                                      m0, acc[p][1][0]);
            acc[p][1][1] = __ffma2_rn(__fadd2_rn(make_float2(__int_as_float(D1[2]), __int_as_float(D1[3])), neg_magic),
                                      m8, acc[p][1][1]);
        }
    };

#pragma unroll 1
    for (int c = 0; c < G::NCH; c++, q++) {
        const int s = q % G::STAGES;
        if (!mbar_wait(&S.full[s], (q / G::STAGES) & 1, abort)) return false;
        if (valid) {
            const uint8_t *wq = stages + (size_t)s * G::STAGE + (size_t)warp * G::WQ + lane * 16;
            const int g0 = c * G::KC;
            if (g0 + G::KC <= NG) {
#pragma unroll 4
                for (int i = 0; i < G::KC; i++) group(wq, g0 + i, i);
            } else {
                for (int i = 0; i < NG - g0; i++) group(wq, g0 + i, i);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.empty[s]);
    }
    if (!valid) return true;

    // bias chains of token j for rows gr, gr + 8: b = fma chain of d_g * bsum_g (Q8G: one per row, in order; Q4L: 8
    // chains g % 8 over the first ng & ~7 groups, hsum8, then the remaining groups in order). Thread t keeps Q4L chains
    // 2t, 2t+1 of both rows; every thread of the quad ends with both rows' values.
    auto bias_rows = [&](int j, float (&b)[2]) {
        const float2 *sb = xsb + j * NG;
        if (Q8) {
#pragma unroll 4
            for (int h = 0; h < 2; h++) {
                float c = 0.0f;
                for (int g = 0; g < NG; g++) {
                    const uint32_t dv = wd[(g >> 2) * 32 + (g & 3)];
                    c = __fmaf_rn(h2f16(h ? dv >> 16 : dv & 0xFFFFu), sb[g].y, c);
                }
                b[h] = c;
            }
        } else {
            float ch[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // row r chain 2t, 2t+1, row r+8 chain 2t, 2t+1
#pragma unroll 2
            for (int g8 = 0; g8 < G::NG8; g8 += 8) {
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int g = g8 + 2 * t + e;
                    const uint32_t dv = wd[(g >> 2) * 32 + (g & 3)];
                    const float bs = sb[g].y;
                    ch[e] = __fmaf_rn(h2f16(dv & 0xFFFFu), bs, ch[e]);
                    ch[2 + e] = __fmaf_rn(h2f16(dv >> 16), bs, ch[2 + e]);
                }
            }
#pragma unroll
            for (int i = 0; i < 4; i++) ch[i] = __fadd_rn(ch[i], __shfl_xor_sync(0xffffffffu, ch[i], 2));
#pragma unroll
            for (int i = 0; i < 4; i++) ch[i] = __fadd_rn(ch[i], __shfl_xor_sync(0xffffffffu, ch[i], 1));
            b[0] = __fadd_rn(ch[0], ch[1]);
            b[1] = __fadd_rn(ch[2], ch[3]);
#pragma unroll
            for (int g = G::NG8; g < NG; g++) {
                const uint32_t dv = wd[(g >> 2) * 32 + (g & 3)];
                b[0] = __fmaf_rn(h2f16(dv & 0xFFFFu), sb[g].y, b[0]);
                b[1] = __fmaf_rn(h2f16(dv >> 16), sb[g].y, b[1]);
            }
        }
    };

#pragma unroll
    for (int p = 0; p < NP; p++) {
        if (2 * p >= ntok) continue;
        // hsum8 of token 2p + jd, rows gr and gr + 8: this thread holds lanes {2u, 2u+1, 4+2u, 5+2u} (u = t & 1), its
        // partner t ^ 1 the others: ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7))
        float sr[2];
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const float u0 = __fadd_rn(acc[p][0][r].x, acc[p][1][r].x), u1 = __fadd_rn(acc[p][0][r].y, acc[p][1][r].y);
            const float v0 = __fadd_rn(u0, __shfl_xor_sync(0xffffffffu, u0, 1));
            const float v1 = __fadd_rn(u1, __shfl_xor_sync(0xffffffffu, u1, 1));
            sr[r] = __fadd_rn(v0, v1);
        }
        float bA[2], bB[2] = {0.0f, 0.0f};
        bias_rows(2 * p, bA);
        if (2 * p + 1 < ntok) bias_rows(2 * p + 1, bB);  // uniform over the warp
        const int j = 2 * p + jd, r = t & 1;
        if (j < ntok) {
            const float b = jd ? (r ? bB[1] : bB[0]) : (r ? bA[1] : bA[0]);
            const float y = __fsub_rn(r ? sr[1] : sr[0], __fmul_rn(Q8 ? 128.0f : (float)kLutBias, b));
            const int row = (it.rb * G::WARPS + warp) * 16 + gr + 8 * r;
            if (KIND == 0) out[(size_t)(it.base + j) * out_ld + row] = y;
            else out[(size_t)it.oslot[j] * out_ld + row] = __fmul_rn(it.ow[j], y);
        }
    }
    return true;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t &r0, uint32_t &r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void mma_s8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Consumer of a GEMM item: up to 8 * NTG tokens of a prefill-numerics expert on this warp's 16-row tile, with the
// reference's prefill arithmetic (inz_gemm_rows, src/quant.c:1615-1668) -- per 256-block the exact int32 dot of the
// requantized int8 weights and the token's int8 block, then f = fma((float)dot_b, ws_b * xs_b, f) over the blocks in
// order (the tcgen05 GEMM's float sequence, k_gemm_tc.cu). A stage holds 128 bytes of K of the tile's 16 rows as the
// tensor copy left them (128-byte swizzle: 16-byte chunk c of row r at chunk c ^ (r & 7)) and the same 128 bytes of
// every token row; ldmatrix gives the MMA's A fragments from the first, its B fragments from the second. The accumulators start at the bits of 1.5 * 2^23, so
// one add of -12582912 gives (float)dot exactly (|dot| <= 256 * 127 * 127 < 2^22).
template <bool Q8, int NG, int KIND, int W, int NTG>
__device__ __forceinline__ bool gemm_item(DecShared &S, const uint8_t *stages, const DecItem &it,
                                          int &q, float *__restrict__ out, int out_ld, const float *__restrict__ as,
                                          const float *__restrict__ wsc, int mrows) {
    using G = DecGeo<Q8, NG, KIND, W, true>;
    constexpr int K = G::K, NCHG = K / 128, NKB = (K + 255) / 256;
    volatile int *abort = &S.abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gr = lane >> 2, t = lane & 3;
    const bool valid = it.e >= 0 && warp < it.ntiles;
    const int ntok = it.ntok;
    const int row0 = (it.rb * G::WARPS + warp) * 16 + gr;  // this thread's rows row0 and row0 + 8
    const float *ws0 = wsc + ((size_t)(it.e < 0 ? 0 : it.e) * mrows + row0) * NKB, *ws1 = ws0 + 8 * NKB;
    // the block-scale rows of this thread's accumulator columns (tokens 8 tg + 2t, 8 tg + 2t + 1); a column past the
    // item's tokens reads token 0's (its outputs are not written)
    int xsr[NTG][2];
#pragma unroll
    for (int tg = 0; tg < NTG; tg++)
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int j = tg * 8 + 2 * t + h;
            xsr[tg][h] = it.trow[j < ntok ? j : 0] * NKB;
        }
    // ldmatrix lane addresses: A matrix lane >> 3 = (rows 0-7 | 8-15) x (first | second 16 bytes of a 32-byte K step);
    // B matrix (lane >> 3) & 1 = first | second 16 bytes of the step for token rows lane & 7
    const int ar = lane & 15;
    const uint32_t a_row = (uint32_t)ar * 128, a_sw = (uint32_t)(ar & 7), a_hi = (uint32_t)(lane >> 4);
    const uint32_t b_lane = (uint32_t)(G::WARPS * G::WQ + (lane & 7) * G::TSTR + 16 * ((lane >> 3) & 1));
    int D[NTG][4];
    float2 f[NTG][2];
#pragma unroll
    for (int tg = 0; tg < NTG; tg++) f[tg][0] = f[tg][1] = make_float2(0.0f, 0.0f);
    const float2 neg_magic = make_float2(-12582912.0f, -12582912.0f);
    float w0 = 0.0f, w1 = 0.0f, xv[NTG][2];
#pragma unroll 1
    for (int c = 0; c < NCHG; c++, q++) {
        const int s = q % G::STAGES;
        if (!(c & 1) && valid) {  // a block begins: its scales load while its MMAs run
            const int b = c >> 1;
            w0 = __ldg(ws0 + b);
            w1 = __ldg(ws1 + b);
#pragma unroll
            for (int tg = 0; tg < NTG; tg++) {
                xv[tg][0] = __ldg(as + xsr[tg][0] + b);
                xv[tg][1] = __ldg(as + xsr[tg][1] + b);
#pragma unroll
                for (int i = 0; i < 4; i++) D[tg][i] = 0x4B400000;
            }
        }
        if (!mbar_wait(&S.full[s], (q / G::STAGES) & 1, abort)) return false;
        if (valid) {
            const uint32_t sb = smem_u32(stages + (size_t)s * G::STAGE), wt = sb + (uint32_t)(warp * G::WQ) + a_row;
#pragma unroll
            for (int ks = 0; ks < 4; ks++) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(wt + ((((uint32_t)(2 * ks) + a_hi) ^ a_sw) << 4), a0, a1, a2, a3);
#pragma unroll
                for (int tg = 0; tg < NTG; tg++) {
                    uint32_t b0, b1;
                    ldsm_x2(sb + b_lane + (uint32_t)(tg * 8 * G::TSTR + 32 * ks), b0, b1);
                    mma_s8s8(D[tg], a0, a1, a2, a3, b0, b1);
                }
            }
            if ((c & 1) || c == NCHG - 1) {  // the block's dot is complete: fold it
                const float2 wp0 = make_float2(w0, w0), wp1 = make_float2(w1, w1);
#pragma unroll
                for (int tg = 0; tg < NTG; tg++) {
                    const float2 xp = make_float2(xv[tg][0], xv[tg][1]);
                    const float2 p0 = __fmul2_rn(wp0, xp), p1 = __fmul2_rn(wp1, xp);
                    const float2 d01 = __fadd2_rn(make_float2(__int_as_float(D[tg][0]), __int_as_float(D[tg][1])),
                                                  neg_magic);
                    const float2 d23 = __fadd2_rn(make_float2(__int_as_float(D[tg][2]), __int_as_float(D[tg][3])),
                                                  neg_magic);
                    f[tg][0] = __ffma2_rn(d01, p0, f[tg][0]);
                    f[tg][1] = __ffma2_rn(d23, p1, f[tg][1]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.empty[s]);
    }
    if (!valid) return true;
#pragma unroll
    for (int tg = 0; tg < NTG; tg++)
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int j = tg * 8 + 2 * t + h;
            if (j >= ntok) continue;
#pragma unroll
            for (int r = 0; r < 2; r++) {
                const float v = h ? f[tg][r].y : f[tg][r].x;
                const int row = row0 + 8 * r;
                if (KIND == 0) out[(size_t)(it.base + j) * out_ld + row] = v;
                else out[(size_t)it.oslot[j] * out_ld + row] = __fmul_rn(it.ow[j], v);
            }
        }
    return true;
}

// GEMM phase of the producer warp (kernels with GEMM items): takes items from the queue while they are GEMM items
// (they precede every decode item) and issues, per item, its stages of 128 bytes of K: the row tiles by tensor copies
// (16 rows, 128-byte swizzle) and the token rows' chunks by bulk copies; then publishes the kGemmEnd marker and hands
// the first non-GEMM item back in `pending`. A loop of its own ahead of the decode loop (and the GEMM items a kernel
// instantiation of their own), so the decode loop compiles as in the decode-only kernel. Returns false when a wait ran
// out.
template <bool Q8, int NG, int KIND, int W>
__device__ __forceinline__ bool gemm_produce(DecShared &S, uint8_t *stages, const MatLayout &M, int E, const RouteDev &R,
                                          const CUtensorMap *wmap, const int8_t *__restrict__ gaq, int meta_work,
                                          int ngi, int per, int &q, int &li, int &na, int &pending) {
    using G = DecGeo<Q8, NG, KIND, W, true>;
    volatile int *abort = &S.abort;
    const int lane = threadIdx.x & 31, tiles = M.rows / 16;
    for (;; li++) {
        const int ab = li & 1;
        if (li >= 2 && !mbar_wait(&S.aempty[ab], ((li >> 1) + 1) & 1, abort)) return false;
        DecItem &D = S.item[ab];
        int item = 0;
        if (lane == 0) item = atomicAdd(R.meta + meta_work, 1);
        item = __shfl_sync(0xffffffffu, item, 0);
        if (item >= ngi) {
            if (lane == 0) {
                D.e = kGemmEnd;
                mbar_arrive(&S.afull[ab]);
            }
            pending = item;
            na++;
            li++;
            return true;
        }
        int e = 0, base = 0, ntok = 0;
        if (lane == 0) {  // (unit << 16 | token tile) of a prefill-numerics expert
            const int tl = __ldg(R.gemm_tiles + item / per), u = tl >> 16, tt = tl & 0xFFFF;
            e = u < E ? __ldg(R.gemm_units + u) : -1;
            if (e < 0 || e >= E) { set_error(R.meta, kErrBadExpert); e = -1; }
            else {
                base = __ldg(R.off + e) + tt * kGemvGemmTile;
                ntok = __ldg(R.cnt + e) - tt * kGemvGemmTile;
                ntok = ntok < kGemvGemmTile ? ntok : kGemvGemmTile;  // the ring's token rows hold 32
                if (ntok <= 0) { set_error(R.meta, kErrOverflow); e = -1; ntok = 0; }
            }
        }
        e = __shfl_sync(0xffffffffu, e, 0);
        base = __shfl_sync(0xffffffffu, base, 0);
        ntok = __shfl_sync(0xffffffffu, ntok, 0);
        int row = 0;
        if (lane < ntok) {
            row = KIND == 0 ? __ldg(R.etok + base + lane) : base + lane;
            if (KIND == 1) { D.oslot[lane] = __ldg(R.eslot + base + lane); D.ow[lane] = __ldg(R.ew + base + lane); }
            D.trow[lane] = row;
        }
        const int rb = item % per, rt0 = rb * G::WARPS, nt = tiles - rt0 < G::WARPS ? tiles - rt0 : G::WARPS;
        if (lane == 0) {
            D.e = e; D.base = base; D.ntok = ntok; D.rb = rb; D.ntiles = nt;
            D.lut = make_uint4(0, 0, 0, 0);
        }
        __syncwarp();  // every lane's trow / oslot / ow before the release
        if (lane == 0) mbar_arrive(&S.afull[ab]);  // nothing in the item buffer: every operand comes with the stages
        na++;
        for (int c = 0; c < G::K / 128; c++, q++) {
            const int s = q % G::STAGES;
            if (q >= G::STAGES && !mbar_wait(&S.empty[s], ((q / G::STAGES) + 1) & 1, abort)) return false;
            uint8_t *sp = stages + (size_t)s * G::STAGE;
            if (lane == 0) {
                if (e >= 0) mbar_expect_tx(&S.full[s], (uint32_t)(nt * 2048 + ntok * 128));
                else mbar_arrive(&S.full[s]);
            }
            __syncwarp();
            if (e >= 0 && lane < nt)
                tma_load_2d(sp + (size_t)lane * G::WQ, wmap, c * 128, e * M.rows + (rt0 + lane) * 16, &S.full[s]);
            if (e >= 0 && lane < ntok)
                bulk_g2s(sp + G::WARPS * G::WQ + lane * G::TSTR, gaq + (size_t)row * G::K + c * 128, 128, &S.full[s]);
        }
    }
}

// GEMM phase of a consumer warp: GEMM items up to the kGemmEnd marker. Returns 0 (decode items follow), 1 (the queue
// is over) or -1 (a wait ran out).
template <bool Q8, int NG, int KIND, int W>
__device__ __forceinline__ int gemm_consume(DecShared &S, const uint8_t *stages, int &q, int &li, float *__restrict__ out,
                                         int out_ld, const float *__restrict__ gas, const float *__restrict__ gws,
                                         int mrows) {
    volatile int *abort = &S.abort;
    const int lane = threadIdx.x & 31;
    for (;; li++) {
        const int ab = li & 1;
        if (!mbar_wait(&S.afull[ab], (li >> 1) & 1, abort)) return -1;
        const DecItem &it = S.item[ab];
        if (it.e == kDecEnd) return 1;
        const bool end = it.e == kGemmEnd;
        if (!end) {
            // prefill-numerics experts have at least 12 tokens: 2-4 groups of 8 MMA columns
            const int nt = it.ntok;
            bool ok;
            if (nt <= 16) ok = gemm_item<Q8, NG, KIND, W, 2>(S, stages, it, q, out, out_ld, gas, gws, mrows);
            else if (nt <= 24) ok = gemm_item<Q8, NG, KIND, W, 3>(S, stages, it, q, out, out_ld, gas, gws, mrows);
            else ok = gemm_item<Q8, NG, KIND, W, 4>(S, stages, it, q, out, out_ld, gas, gws, mrows);
            if (!ok) return -1;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.aempty[ab]);
        if (end) {
            li++;
            return 0;
        }
    }
}

template <bool Q8, int NG, int KIND, int W, bool HG>
__global__ void __launch_bounds__(DecGeo<Q8, NG, KIND, W, HG>::THREADS, 1)
    gemv_decode_kernel(const uint8_t *__restrict__ pool, uint64_t slab_bytes, MatLayout M, const uint8_t *__restrict__ luts,
                       int lut_off, int E, RouteDev R, const int8_t *__restrict__ aq, const float2 *__restrict__ asb,
                       float *__restrict__ out, int out_ld, int meta_items, int meta_work, uint32_t one,
                       const __grid_constant__ CUtensorMap wmap, const int8_t *__restrict__ gaq,
                       const float *__restrict__ gas, const float *__restrict__ gws, int meta_gtiles) {
    using G = DecGeo<Q8, NG, KIND, W, HG>;
    extern __shared__ __align__(1024) uint8_t smem[];
    DecShared &S = *reinterpret_cast<DecShared *>(smem);
    // the stage ring starts on a 1024-byte boundary (the 128-byte swizzle of the GEMM items' tensor copies): HDR and
    // STAGE are multiples of 1024 and the dynamic shared memory starts on one (checked: a CTA that finds otherwise
    // fails the call)
    uint8_t *stages = smem + G::HDR;
    uint8_t *ibufs = stages + (size_t)G::STAGES * G::STAGE;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles = M.rows / 16, per = (tiles + G::WARPS - 1) / G::WARPS;  // items per matrix
    // HG: the call's GEMM items (prefill-numerics experts, the heaviest work) come first in the queue, then the decode
    // items
    const int ngi = HG ? R.meta[meta_gtiles] * per : 0;
    const int nitems = R.meta[meta_items] + ngi;
    if ((int)blockIdx.x >= nitems) return;
    if (HG && (smem_u32(smem) & 1023u)) {
        if (threadIdx.x == 0) set_error(R.meta, kErrBadSlot);
        return;
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < G::STAGES; i++) { mbar_init(&S.full[i], 1); mbar_init(&S.empty[i], G::WARPS); }
        for (int i = 0; i < 2; i++) { mbar_init(&S.afull[i], 1); mbar_init(&S.aempty[i], G::WARPS); }
        S.abort = 0;
        S.never = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    volatile int *abort = &S.abort;

    if (warp == G::WARPS) {
        // ---------------- producer warp ----------------
        // items come from the call's work queue (the route kernel lists experts heaviest first and clears the counter)
        int q = 0, li = 0, na = 0;  // stages issued, items begun, items whose buffers were issued
        bool ok = true;
        // HG: the GEMM phase first; its kGemmEnd marker tells the consumers that decode items follow
        int pending = -1;
        if constexpr (HG)
            ok = gemm_produce<Q8, NG, KIND, W>(S, stages, M, E, R, &wmap, gaq, meta_work, ngi, per, q, li, na, pending);
        for (; ok; li++) {
            const int ab = li & 1;
            if (li >= 2 && !mbar_wait(&S.aempty[ab], ((li >> 1) + 1) & 1, abort)) { ok = false; break; }
            DecItem &D = S.item[ab];
            int item = pending;
            if (!HG || item < 0) {
                if (lane == 0) item = atomicAdd(R.meta + meta_work, 1);
                item = __shfl_sync(0xffffffffu, item, 0);
            }
            pending = -1;
            if (item >= nitems) {
                if (lane == 0) {
                    D.e = kDecEnd;
                    mbar_arrive(&S.afull[ab]);
                }
                break;
            }
            const int unit_item = item - ngi, rb = unit_item % per;
            int e = 0, base = 0, ntok = 0;
            if (lane == 0) {
                e = __ldg(R.dec_units + unit_item / per);
                if (e < 0 || e >= E) { set_error(R.meta, kErrBadExpert); e = -1; }
                else {
                    base = __ldg(R.off + e);
                    ntok = __ldg(R.cnt + e);
                    if (ntok > G::MT) { set_error(R.meta, kErrOverflow); ntok = G::MT; }
                }
            }
            e = __shfl_sync(0xffffffffu, e, 0);
            base = __shfl_sync(0xffffffffu, base, 0);
            ntok = __shfl_sync(0xffffffffu, ntok, 0);
            int row = 0;
            if (lane < ntok) {
                row = KIND == 0 ? __ldg(R.etok + base + lane) : base + lane;
                if (KIND == 1) { D.oslot[lane] = __ldg(R.eslot + base + lane); D.ow[lane] = __ldg(R.ew + base + lane); }
            }
            const int rt0 = rb * G::WARPS, nt = tiles - rt0 < G::WARPS ? tiles - rt0 : G::WARPS;
            const uint8_t *slab = pool + (size_t)(e < 0 ? 0 : e) * slab_bytes;
            if (lane == 0) {
                D.e = e; D.base = base; D.ntok = ntok; D.rb = rb; D.ntiles = nt;
                D.lut = (!Q8 && e >= 0) ? __ldg(reinterpret_cast<const uint4 *>(luts + (size_t)e * 32 + lut_off))
                                        : make_uint4(0, 0, 0, 0);
            }
            __syncwarp();
            uint8_t *ib = ibufs + (size_t)ab * G::IBUF;
            const uint32_t dbytes = e >= 0 ? (uint32_t)(nt * G::GD * 128) : 0u;
            if (lane == 0) mbar_expect_tx(&S.afull[ab], (uint32_t)(ntok * (G::K + NG * 8)) + dbytes);
            __syncwarp();
            if (KIND == 0) {
                if (lane < ntok) {
                    bulk_g2s(ib + (size_t)lane * G::K, aq + (size_t)row * G::K, G::K, &S.afull[ab]);
                    bulk_g2s(ib + G::IB_SB + (size_t)lane * NG * 8, asb + (size_t)row * NG, NG * 8, &S.afull[ab]);
                }
            } else if (lane == 0 && ntok > 0) {
                bulk_g2s(ib, aq + (size_t)base * G::K, ntok * G::K, &S.afull[ab]);
                bulk_g2s(ib + G::IB_SB, asb + (size_t)base * NG, ntok * NG * 8, &S.afull[ab]);
            }
            if (lane == 31 && e >= 0)
                bulk_g2s(ib + G::IB_D, slab + M.d_off + (size_t)rt0 * G::GD * 128, dbytes, &S.afull[ab]);
            na++;
            // weights of the item's nt row tiles, one stage per KC groups
            for (int c = 0; c < G::NCH; c++, q++) {
                const int s = q % G::STAGES;
                if (q >= G::STAGES && !mbar_wait(&S.empty[s], ((q / G::STAGES) + 1) & 1, abort)) { ok = false; break; }
                const int g0 = c * G::KC, kc = NG - g0 < G::KC ? NG - g0 : G::KC;
                const uint32_t wbytes = (uint32_t)(kc * 32 * G::WB);
                if (lane == 0) {
                    if (e >= 0) mbar_expect_tx(&S.full[s], nt * wbytes);
                    else mbar_arrive(&S.full[s]);
                }
                __syncwarp();
                if (e >= 0 && lane < nt)
                    bulk_g2s(stages + (size_t)s * G::STAGE + (size_t)lane * G::WQ,
                             slab + M.q_off + ((size_t)(rt0 + lane) * NG + g0) * 32 * G::WB, wbytes, &S.full[s]);
            }
            if (!ok) break;
        }
        // Normal end: the consumers wait for every issued copy before they see the end marker, so nothing is in
        // flight when the CTA leaves. After an abort the producer drains what it issued (bounded): the last use of
        // each stage slot and of each item buffer (no end marker was published, so each is the barrier's latest phase).
        if (!ok) {
            if (lane == 0) set_error(R.meta, kErrTimeout);
            *abort = 1;
            volatile int *never = &S.never;
            for (int k = (q > G::STAGES ? q - G::STAGES : 0); k < q; k++)
                mbar_wait(&S.full[k % G::STAGES], (k / G::STAGES) & 1, never);
            for (int k = (na > 2 ? na - 2 : 0); k < na; k++) mbar_wait(&S.afull[k & 1], (k >> 1) & 1, never);
        }
        return;
    }

    // ---------------- consumer warps ----------------
    int q = 0, li = 0;
    bool fail = false;
    if constexpr (HG) {
        const int r = gemm_consume<Q8, NG, KIND, W>(S, stages, q, li, out, out_ld, gas, gws, M.rows);
        if (r == 1) return;
        fail = r < 0;
    }
    for (; !fail; li++) {
        const int ab = li & 1;
        if (!mbar_wait(&S.afull[ab], (li >> 1) & 1, abort)) break;
        const DecItem &it = S.item[ab];
        if (it.e == kDecEnd) return;
        const uint8_t *ib = ibufs + (size_t)ab * G::IBUF;
        const int nt = it.ntok;
        bool ok;
        if (nt <= 1) ok = dec_item<Q8, NG, KIND, W, HG, 1>(S, stages, ib, it, q, out, out_ld, one);
        else if (nt <= 2) ok = dec_item<Q8, NG, KIND, W, HG, 2>(S, stages, ib, it, q, out, out_ld, one);
        else if (nt <= 3) ok = dec_item<Q8, NG, KIND, W, HG, 3>(S, stages, ib, it, q, out, out_ld, one);
        else if (nt <= 4) ok = dec_item<Q8, NG, KIND, W, HG, 4>(S, stages, ib, it, q, out, out_ld, one);
        else if (nt <= 6) ok = dec_item<Q8, NG, KIND, W, HG, 6>(S, stages, ib, it, q, out, out_ld, one);
        else if (nt <= 8) ok = dec_item<Q8, NG, KIND, W, HG, 8>(S, stages, ib, it, q, out, out_ld, one);
        else ok = dec_item<Q8, NG, KIND, W, HG, 12>(S, stages, ib, it, q, out, out_ld, one);
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.aempty[ab]);
    }
    if (lane == 0) set_error(R.meta, kErrTimeout);
    *abort = 1;
}

// ---------------------------------------------------------------------------------------------------------------
template <bool Q8, int NG, int KIND, int W, bool HG>
static void launch_one(const LayerDev &L, const MatLayout &M, const RouteDev &R, const int8_t *aq, const float2 *asb,
                       float *out, int out_ld, int meta_items, int num_sms, cudaStream_t st, const DecGemm *gm) {
    using G = DecGeo<Q8, NG, KIND, W, HG>;
    static_assert(G::SMEM <= 227 * 1024, "decode GEMV shared memory");
    static_assert(sizeof(DecShared) <= G::HDR, "decode GEMV header");
    static_assert(G::WARPS < 32, "one producer lane per row tile");
    // GEMM items: a stage holds 128 bytes of K of every row tile (16 rows), the item buffer 16 token rows
    static_assert(!HG || (G::WARPS == 15 && G::WQ == 2048), "GEMM item stage geometry");
    static_assert(!HG || kGemvGemmTile <= 32, "GEMM item token rows");
    static_assert(G::HDR % 1024 == 0 && G::STAGE % 1024 == 0, "stage ring alignment");
    static_assert(G::K % 128 == 0, "GEMM item K chunks");
    cudaFuncSetAttribute(gemv_decode_kernel<Q8, NG, KIND, W, HG>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM);
    CUtensorMap none;
    memset(&none, 0, sizeof(none));
    const bool g = HG && gm != nullptr;
    gemv_decode_kernel<Q8, NG, KIND, W, HG><<<num_sms, G::THREADS, G::SMEM, st>>>(
        L.pool, L.slab_bytes, M, L.luts, KIND == 0 ? 0 : 16, L.E, R, aq, asb, out, out_ld, meta_items,
        KIND == 0 ? kMetaWorkGU : kMetaWorkDN, 1u, g ? *reinterpret_cast<const CUtensorMap *>(gm->wmap) : none,
        g ? gm->aq : nullptr, g ? gm->as : nullptr, g ? gm->ws : nullptr,
        g ? (KIND == 0 ? kMetaGemmTilesGU : kMetaGemmTilesDN) : -1);
}

// Row tiles per item for a call of n token rows: wide items (15 tiles, 16 warps per CTA) once the call has enough
// work to occupy every SM (4 tokens give about 40 experts: 200 gate|up and 360 down items); 8 tiles below that, so a
// few experts still spread over many SMs. The route kernels size the work queue with the same rule.
static int tiles_per_item(int n) { return n >= 4 ? 15 : 8; }

int gemv_items_per_unit(const LayerDev &L, int kind, int n) {
    const MatLayout &M = kind == 0 ? L.gu : L.dn;
    const int W = tiles_per_item(n);
    return (M.rows / 16 + W - 1) / W;
}

// Returns the number of kernels launched, 0 for a geometry probe (kind 2/3), or -1 if the geometry has no
// instantiation. asb: per activation row and 64-group, (scale, scale * sum of q) as the reference keeps them.
int launch_gemv_decode(const LayerDev &L, int kind, const RouteDev &R, const int8_t *aq, const float2 *asb, float *out,
                       int out_ld, int num_sms, cudaStream_t st, const DecGemm *gm) {
    if (kind < 0)  // geometry probe: both matrices must have an instantiation
        return launch_gemv_decode(L, 2, R, aq, asb, out, out_ld, num_sms, st) < 0 ||
                       launch_gemv_decode(L, 3, R, aq, asb, out, out_ld, num_sms, st) < 0 ? -1 : 0;
    const bool probe = kind >= 2;
    if (probe) kind -= 2;
    const MatLayout &M = kind == 0 ? L.gu : L.dn;
    const int mi = kind == 0 ? kMetaDecItemsGU : kMetaDecItemsDN;
    const bool q8 = L.type == INZG_T_Q8G;
    if (M.rows % 16) return -1;
    const bool wide = tiles_per_item(R.n) == 15;
    if (gm && !probe && (!wide || !gm->wmap || !gm->aq || !gm->as || !gm->ws)) return -1;  // GEMM items: wide only
#define INZG_GEMV_CASE(Q, N)                                                                                     \
    if (q8 == Q && M.ng == N) {                                                                                  \
        if (probe) return 0;                                                                                     \
        if (kind == 0) {                                                                                         \
            if (gm) launch_one<Q, N, 0, 15, true>(L, M, R, aq, asb, out, out_ld, mi, num_sms, st, gm);          \
            else if (wide) launch_one<Q, N, 0, 15, false>(L, M, R, aq, asb, out, out_ld, mi, num_sms, st, gm);  \
            else launch_one<Q, N, 0, 8, false>(L, M, R, aq, asb, out, out_ld, mi, num_sms, st, nullptr);        \
        } else {                                                                                                 \
            if (gm) launch_one<Q, N, 1, 15, true>(L, M, R, aq, asb, out, out_ld, mi, num_sms, st, gm);          \
            else if (wide) launch_one<Q, N, 1, 15, false>(L, M, R, aq, asb, out, out_ld, mi, num_sms, st, gm);  \
            else launch_one<Q, N, 1, 8, false>(L, M, R, aq, asb, out, out_ld, mi, num_sms, st, nullptr);        \
        }                                                                                                        \
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
