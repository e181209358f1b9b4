// k_fused.cu -- the whole routed MoE layer in one persistent launch, for decode calls of 1 or 2 tokens (kernel code
// for up to 8; every expert then takes the decode numerics, src/model_fwd.c:1071): router -> softmax / top-k -> dispatch -> gate|up -> SiLU*up
// + quantization -> down -> rank-order combine. This is the path the reference engine runs per generated token
// (moe_block -> experts_batch, src/model_fwd.c:992-1140, 878-989); one launch replaces the chain of seven kernels
// whose launch and ramp gaps dominate a one-token call.
//
// One CTA per SM (cooperative launch, so every CTA is resident), 12 warps each:
//  A. Router logits (the reference's 8-lane F16 FMA chains, src/quant.c:1290-1304) as warp tasks (4 experts x 8
//     lanes, one token), the decode-numerics quantization of the inputs (one warp per token and 256-block), and the
//     zeroing of this call's hand-off counters. Then the one grid barrier of the call (bounded).
//  B. Every CTA computes the routing of all n tokens itself (softmax, top-k, weights: k_softmax.cuh, bit-exact) and
//     the dispatch lists in shared memory, so the experts' work needs no second barrier; CTA 0 writes the routing
//     products for the caller.
//  C. Gate|up row tiles (16 rows of one expert) are warp items spread over all SMs. A warp streams its items' weight
//     fragments through a 3-stage bulk-copy ring (cp.async.bulk, mbarrier completion) and runs the decode GEMV's
//     exact lane-partial MMAs (k_gemv_core.cuh). The warp that completes an expert's last gate|up tile (a per-expert
//     counter) computes SiLU*up, the rotation and the 64-group quantization of the expert's entries and releases the
//     expert's ready flag.
//  D. Down row tiles: a warp waits for the expert's flag (acquire, bounded), copies the entries' quantized inputs,
//     writes w * y into each entry's slot, and counts (token, row tile) completions; the K-th slot of a token's row
//     tile sums the token's K slots in rank order into y (src/model_fwd.c:1134-1140).
// Each warp takes every gate|up item of its share before any down item, and gate|up items never wait on another
// warp, so the flag waits always end. Every wait is bounded; one that runs out records INZG_TIMEOUT, skips the rest
// of the warp's items and drains the warp's copies before the CTA leaves.
#include <type_traits>

#include "inzg_internal.h"
#include "k_async.cuh"
#include "k_gemv_core.cuh"
#include "k_launch.h"
#include "k_softmax.cuh"
#include "k_warpq.cuh"

namespace inzg {

namespace {

constexpr int kFW = 12;                        // warps per CTA
constexpr int kFThreads = kFW * 32;
constexpr int kFMaxTok = 8;                    // tokens of a fused call
constexpr int kFMaxEnt = kFMaxTok * kMaxTopK;  // entries (token, rank)
constexpr int kFMaxStages = 8;                 // weight ring stages per warp (as many as shared memory allows)
constexpr int kFChunk = 4096;                  // bytes per stage: 8 Q4L or 4 Q8G 64-groups of a 16-row tile
constexpr int kFNB = 8;                        // most 128-column blocks of a down input (FF <= 1024)
constexpr uint32_t kFSpin = 1u << 22;          // polls of a flag or the barrier before the wait is declared stuck

struct FusedArgs {
    const uint8_t *pool;
    uint64_t slab_bytes;
    MatLayout gu, dn;
    const uint8_t *luts;
    const uint4 *router;
    int gu_rot, dn_rot;
    uint32_t gu_seed, dn_seed;
    float gu_norm, dn_norm;
    int H, FF, E, K, n;
    const float *x, *bias, *ovr;
    float *logits, *probs;
    int32_t *sel;
    float *w;
    int32_t *units, *meta;
    int8_t *xq64;
    float2 *xsb64;
    float *GU;
    int8_t *dq64;
    float2 *dsb64;
    float *mo, *y;
    int32_t *sync;     // [2]: barrier arrivals, barrier generation (self-resetting across calls)
    int32_t *gu_done;  // [E][kFNB] gate|up tiles finished per (expert, 128-column block of the down input)
    int32_t *ready;    // [E] 128-column blocks of the expert's down inputs written
    int32_t *ycnt;     // [n][H/16] slots finished per (token, down row tile)
};

struct FShared {
    uint64_t pa;  // phase A: the CTA's router quad and the call's inputs have landed
    uint64_t full[kFW][kFMaxStages];
    uint64_t sfull[kFW][2];
    uint64_t afull[kFW];
    int32_t sel[kFMaxEnt];
    float w[kFMaxEnt];
    int32_t nunits;
    int32_t unit_e[kFMaxEnt];
    int32_t unit_off[kFMaxEnt + 1];
    int32_t etok[kFMaxEnt], eslot[kFMaxEnt], esort[kFMaxEnt];
    float ew[kFMaxEnt];
    int32_t scan[32];
    int32_t bar_ok;
};

// dynamic shared memory: FShared | quantized inputs [n][H] | their (s, bsum) [n][H/64] | per warp: weight ring,
// 2 scale blocks, the down item's inputs [n][FF] and their (s, bsum) [n][FF/64]
struct FLayout {
    int xq, xsb, warp0, stages, sblk, dact, dsb, per_warp, total;
};

constexpr int kFSmemMax = 227 * 1024;

// stages: the deepest ring (<= kFMaxStages) whose layout fits kFSmemMax (at least 2)
__host__ __device__ inline FLayout fused_layout(int n, int H, int FF) {
    FLayout L;
    const int ngu = H / kGroup, ndn = FF / kGroup;
    const int gd = ((ngu > ndn ? ngu : ndn) + 3) / 4;
    L.xq = (int)((sizeof(FShared) + 127) / 128 * 128);
    L.xsb = L.xq + (n * H + 127) / 128 * 128;
    L.warp0 = L.xsb + (n * ngu * 8 + 127) / 128 * 128;
    const int rest = 2 * gd * 128 + (n * FF + 127) / 128 * 128 + (n * ndn * 8 + 127) / 128 * 128;
    int st = (kFSmemMax - L.warp0 - kFW * rest) / (kFW * kFChunk);
    st = st > kFMaxStages ? kFMaxStages : st < 2 ? 2 : st;
    L.stages = st;
    L.sblk = st * kFChunk;
    L.dact = L.sblk + 2 * gd * 128;
    L.dsb = L.dact + (n * FF + 127) / 128 * 128;
    L.per_warp = L.dsb + (n * ndn * 8 + 127) / 128 * 128;
    L.total = L.warp0 + kFW * L.per_warp;
    return L;
}

__device__ __forceinline__ int ld_acquire(const int32_t *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release(int32_t *p, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int atom_add_acq_rel(int32_t *p, int v) {
    int o;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(o) : "l"(p), "r"(v) : "memory");
    return o;
}

// bounded grid barrier over all CTAs (generation counter: needs no reset between calls); false if it timed out
__device__ bool grid_barrier(FShared &S, int32_t *sync, int32_t *meta) {
    __syncthreads();
    if (threadIdx.x == 0) {
        S.bar_ok = 1;
        const int gen = ld_acquire(sync + 1);
        __threadfence();
        if (atom_add_acq_rel(sync, 1) == (int)gridDim.x - 1) {
            sync[0] = 0;  // the last CTA resets the arrivals, then opens the next generation
            st_release(sync + 1, gen + 1);
        } else {
            uint32_t i = 0;
            while (ld_acquire(sync + 1) == gen && ++i < kFSpin) __nanosleep(64);
            if (i >= kFSpin) {
                S.bar_ok = 0;
                set_error(meta, kErrTimeout);
            }
        }
    }
    __syncthreads();
    return S.bar_ok != 0;
}

// bounded wait of one lane for *flag >= target (acquire)
__device__ bool wait_flag(const int32_t *flag, int target) {
    for (uint32_t i = 0; i < kFSpin; i++) {
        if (ld_acquire(flag) >= target) return true;
        if (i > 64) __nanosleep(32);
    }
    return false;
}

// ---------------------------------------------------------------------------------------------------------------
// Phase A: the logits of experts 4q..4q+3 for all n tokens (lane = expert 4q + lane / 8, chain lane l = lane % 8) from
// shared memory: wq = the quad's block of the router's repacked layout Wr[q][H/64][4 experts][8 lanes][8 halves]
// (k_router.cu); xs = the inputs re-laid out as [n][H/64][8 lanes][8 steps], so chunk jc's 8 chain steps of lane l
// are two 16-byte loads. Each thread runs n independent chains of the reference's FMAs (k = 64 jc + 8 s + l).
__device__ void router_quad(const FusedArgs &A, int q, const uint4 *wq, const float *xs) {
    const int lane = threadIdx.x & 31, l = lane & 7, n = A.n, H = A.H;
    const int SC = H / 64;
    float a[kFMaxTok];
#pragma unroll
    for (int t = 0; t < kFMaxTok; t++) a[t] = 0.0f;
#pragma unroll 4
    for (int jc = 0; jc < SC; jc++) {
        const uint4 v = wq[(size_t)jc * 32 + lane];
        const uint32_t hw[4] = {v.x, v.y, v.z, v.w};
        float wv[8];
#pragma unroll
        for (int s = 0; s < 8; s++) wv[s] = __half2float(__ushort_as_half((unsigned short)(hw[s >> 1] >> (16 * (s & 1)))));
#pragma unroll
        for (int t = 0; t < kFMaxTok; t++) {
            if (t >= n) break;
            const float4 *xc = reinterpret_cast<const float4 *>(xs + (size_t)t * H + jc * 64 + l * 8);
            const float4 x0 = xc[0], x1 = xc[1];
            a[t] = __fmaf_rn(wv[0], x0.x, a[t]); a[t] = __fmaf_rn(wv[1], x0.y, a[t]);
            a[t] = __fmaf_rn(wv[2], x0.z, a[t]); a[t] = __fmaf_rn(wv[3], x0.w, a[t]);
            a[t] = __fmaf_rn(wv[4], x1.x, a[t]); a[t] = __fmaf_rn(wv[5], x1.y, a[t]);
            a[t] = __fmaf_rn(wv[6], x1.z, a[t]); a[t] = __fmaf_rn(wv[7], x1.w, a[t]);
        }
    }
    const int e = q * 4 + (lane >> 3);
#pragma unroll
    for (int t = 0; t < kFMaxTok; t++) {
        if (t >= n) break;
        float sum = hsum8_lanes(a[t]);
        if (A.bias) sum = __fadd_rn(sum, A.bias[e]);  // test hook: logits += bias before the softmax
        if (l == 0) A.logits[(size_t)t * A.E + e] = sum;
    }
}

// Phase A task: decode-numerics quantization of token t's 256-block b (gate|up rotation), as act_quant_x_warp_kernel
template <int NGU>
__device__ void actq_task(const FusedArgs &A, int t, int b) {
    const int lane = threadIdx.x & 31;
    constexpr int H = NGU * kGroup;
    float v[1][8];
    const float *xb = A.x + (size_t)t * H + b * 256 + lane * 8;
    const float4 p = reinterpret_cast<const float4 *>(xb)[0], r = reinterpret_cast<const float4 *>(xb)[1];
    v[0][0] = p.x; v[0][1] = p.y; v[0][2] = p.z; v[0][3] = p.w;
    v[0][4] = r.x; v[0][5] = r.y; v[0][6] = r.z; v[0][7] = r.w;
    if (A.gu_rot > 1) warp_rotate<1, 8>(v, A.gu_seed, A.gu_norm, lane, b * 256);
    const size_t o = (size_t)t * H + b * 256;
    warp_quantize<1, 8>(v, 256, lane, A.xq64 + o, A.xsb64 + o / kGroup, nullptr, nullptr);
}

// ---------------------------------------------------------------------------------------------------------------
// One 16-row tile of one expert matrix for ntok <= TC tokens: the decode GEMV's numerics (k_gemv.cu explains the
// lane-partial MMA, the fma fold, the hsum8 pairing and the bias chains).
template <bool Q8, int NG, int TC>
struct TileArgs {
    const uint8_t *ring;
    uint64_t *full;
    int q0;      // stages consumed before the tile's first chunk
    int stages;  // ring depth
    const uint32_t *sblk;
    uint4 lut;
    // token j's activations: xbase + row(j) * xstride bytes; its (s, bsum): sbase + row(j) * sstride, where
    // row(j) = tok[j] (gate|up: the entry's token) or j (down: the warp's staged entries)
    const int8_t *xbase;
    const float2 *sbase;
    const int32_t *tok;
    int xstride, sstride;
    int ntok;
    __device__ __forceinline__ int row(int j) const { return tok ? tok[j] : j; }
    __device__ __forceinline__ const int8_t *x(int j) const { return xbase + (size_t)row(j) * xstride; }
    __device__ __forceinline__ const float2 *sb(int j) const { return sbase + (size_t)row(j) * sstride; }
};

// Returns false if a ring wait ran out. yout[p]: this thread's output of pair p -- token 2p + (lane & 3) / 2, row
// (lane >> 2) + 8 * (lane & 1) of the tile (the quad's two threads split the two rows). issue(c) is called once the
// warp is done with the tile's chunk c (its stage may be refilled).
template <bool Q8, int NG, int TC, class Issue>
__device__ __forceinline__ bool fused_tile(const TileArgs<Q8, NG, TC> &T, float (&yout)[(TC + 1) / 2], Issue &&issue) {
    constexpr int KC = Q8 ? 4 : 8, NCH = (NG + KC - 1) / KC, GB = Q8 ? 1024 : 512, NG8 = NG & ~7;
    constexpr int NP = (TC + 1) / 2;
    const int lane = threadIdx.x & 31, gr = lane >> 2, t = lane & 3;
    const int lc = gr & 3, jcol = gr >> 2, jd = t >> 1;
    const uint32_t s0 = lc == (t >> 1) ? 1u : 0u, s1 = lc == 2 + (t >> 1) ? 1u : 0u;
    const uint32_t *wd = T.sblk + gr * 4;
    const int ntok = T.ntok;
    float2 acc[NP][2][2];
#pragma unroll
    for (int p = 0; p < NP; p++)
#pragma unroll
        for (int h = 0; h < 2; h++) acc[p][h][0] = acc[p][h][1] = make_float2(0.0f, 0.0f);
    const float2 neg_magic = make_float2(-12582912.0f, -12582912.0f);
    const int xo = 32 * (t & 1) + 4 * lc;
    // per pair p: this thread's operand-column token (2p + jcol) and accumulator token (2p + jd), resolved once
    const int8_t *xr[NP];
    const float2 *sr_[NP];
    bool live[NP], alive[NP];
#pragma unroll
    for (int p = 0; p < NP; p++) {
        const int jc_ = 2 * p + jcol, ja = 2 * p + jd;
        live[p] = jc_ < ntok;
        alive[p] = ja < ntok;
        xr[p] = T.x(live[p] ? jc_ : 0) + xo;
        sr_[p] = T.sb(alive[p] ? ja : 0);
    }
    bool ok = true;
    for (int c = 0; c < NCH; c++) {
        const int q = T.q0 + c, s = q % T.stages;
        ok = __all_sync(0xffffffffu, ok && mbar_wait_bounded(&T.full[s], (q / T.stages) & 1));  // warp-uniform
        const uint8_t *wq = T.ring + (size_t)s * kFChunk + lane * 16;
        const int g0 = c * KC, gn = NG - g0 < KC ? NG - g0 : KC;
        // one 64-group (i: index inside the chunk); a full chunk is unrolled so its groups' loads, LUT decodes and
        // MMAs overlap -- only the fp32 fold is ordered
        auto group = [&](int i) {
            const int g = g0 + i;
            uint32_t A0[4], A1[4];
            if (Q8) {
                const uint4 w0 = *reinterpret_cast<const uint4 *>(wq + (size_t)i * GB);
                const uint4 w1 = *reinterpret_cast<const uint4 *>(wq + (size_t)i * GB + 512);
                A0[0] = w0.x; A0[1] = w0.y; A0[2] = w0.z; A0[3] = w0.w;
                A1[0] = w1.x; A1[1] = w1.y; A1[2] = w1.z; A1[3] = w1.w;
            } else {
                const uint4 w = *reinterpret_cast<const uint4 *>(wq + (size_t)i * GB);
                const uint4 x = make_uint4(w.x ^ 0x88888888u, w.y ^ 0x88888888u, w.z ^ 0x88888888u,
                                           w.w ^ 0x88888888u);
                const uint32_t k16 = 1u << 16;
                A0[0] = lut16(w.x, x.x, T.lut, 1u); A0[1] = lut16(w.y, x.y, T.lut, 1u);
                A0[2] = lut16(hi16(w.x, k16), hi16(x.x, k16), T.lut, 1u);
                A0[3] = lut16(hi16(w.y, k16), hi16(x.y, k16), T.lut, 1u);
                A1[0] = lut16(w.z, x.z, T.lut, 1u); A1[1] = lut16(w.w, x.w, T.lut, 1u);
                A1[2] = lut16(hi16(w.z, k16), hi16(x.z, k16), T.lut, 1u);
                A1[3] = lut16(hi16(w.w, k16), hi16(x.w, k16), T.lut, 1u);
            }
            const float2 dd = h2f16x2(wd[(g >> 2) * 32 + (g & 3)]);
#pragma unroll
            for (int p = 0; p < NP; p++) {
                if (2 * p >= ntok) continue;
                const int8_t *xp = xr[p] + g * kGroup;
                const uint32_t x0 = live[p] ? *reinterpret_cast<const uint32_t *>(xp) : 0u;
                const uint32_t x1 = live[p] ? *reinterpret_cast<const uint32_t *>(xp + 16) : 0u;
                const float sx = alive[p] ? sr_[p][g].x : 0.0f;
                int D0[4], D1[4];
                mma_u8s8_c(D0, A0[0], A0[1], A0[2], A0[3], x0 * s0, x0 * s1, 0x4B400000);
                mma_u8s8_c(D1, A1[0], A1[1], A1[2], A1[3], x1 * s0, x1 * s1, 0x4B400000);
                const float ds0 = __fmul_rn(dd.x, sx), ds8 = __fmul_rn(dd.y, sx);
                const float2 m0 = make_float2(ds0, ds0), m8 = make_float2(ds8, ds8);
                acc[p][0][0] = __ffma2_rn(
                    __fadd2_rn(make_float2(__int_as_float(D0[0]), __int_as_float(D0[1])), neg_magic), m0,
                    acc[p][0][0]);
                acc[p][0][1] = __ffma2_rn(
                    __fadd2_rn(make_float2(__int_as_float(D0[2]), __int_as_float(D0[3])), neg_magic), m8,
                    acc[p][0][1]);
                acc[p][1][0] = __ffma2_rn(
                    __fadd2_rn(make_float2(__int_as_float(D1[0]), __int_as_float(D1[1])), neg_magic), m0,
                    acc[p][1][0]);
                acc[p][1][1] = __ffma2_rn(
                    __fadd2_rn(make_float2(__int_as_float(D1[2]), __int_as_float(D1[3])), neg_magic), m8,
                    acc[p][1][1]);
            }
        };
        if (ok) {
            if (gn == KC) {
#pragma unroll
                for (int i = 0; i < KC; i++) group(i);
            } else {
                for (int i = 0; i < gn; i++) group(i);
            }
        }
        __syncwarp();
        issue(c);
    }
    // bias chains of token j for rows gr, gr + 8 (Q8G: one chain per row; Q4L: 8 chains g % 8, hsum8, the tail)
    auto bias_rows = [&](int j, float (&b)[2]) {
        const float2 *sb = T.sb(j);
        if (Q8) {
            for (int h = 0; h < 2; h++) {
                float c = 0.0f;
                for (int g = 0; g < NG; g++) {
                    const uint32_t dv = wd[(g >> 2) * 32 + (g & 3)];
                    c = __fmaf_rn(h2f16(h ? dv >> 16 : dv & 0xFFFFu), sb[g].y, c);
                }
                b[h] = c;
            }
        } else {
            float ch[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int g8 = 0; g8 < NG8; g8 += 8) {
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
            for (int g = NG8; g < NG; g++) {
                const uint32_t dv = wd[(g >> 2) * 32 + (g & 3)];
                b[0] = __fmaf_rn(h2f16(dv & 0xFFFFu), sb[g].y, b[0]);
                b[1] = __fmaf_rn(h2f16(dv >> 16), sb[g].y, b[1]);
            }
        }
    };
    const int r = t & 1;
#pragma unroll
    for (int p = 0; p < NP; p++) {
        yout[p] = 0.0f;
        if (2 * p >= ntok) continue;
        float sr[2];
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            const float u0 = __fadd_rn(acc[p][0][rr].x, acc[p][1][rr].x);
            const float u1 = __fadd_rn(acc[p][0][rr].y, acc[p][1][rr].y);
            const float v0 = __fadd_rn(u0, __shfl_xor_sync(0xffffffffu, u0, 1));
            const float v1 = __fadd_rn(u1, __shfl_xor_sync(0xffffffffu, u1, 1));
            sr[rr] = __fadd_rn(v0, v1);
        }
        float bA[2], bB[2] = {0.0f, 0.0f};
        bias_rows(2 * p, bA);
        if (2 * p + 1 < ntok) bias_rows(2 * p + 1, bB);  // uniform over the warp
        const float b = jd ? bB[r] : bA[r];
        yout[p] = __fsub_rn(sr[r], __fmul_rn(Q8 ? 128.0f : (float)kLutBias, b));
    }
    return ok;
}

// ---------------------------------------------------------------------------------------------------------------
// SiLU*up of 128-column block b of one expert's entries, rotated and quantized for the down matrix (decode
// numerics), by one warp: h = g / (1 + exp(-g)) * u (siluf, src/model_fwd.c:43; exp in double, rounded once, as
// swiglu_quant_warp_kernel), the down matrix's 128-block rotation, then s = amax / 127 per 64-group
// (src/quant.c:611-637). A block needs gate rows [128b, 128b + 128) and the matching up rows: 16 gate|up tiles.
template <int FF>
__device__ void swiglu_block(const FusedArgs &A, int ent0, int n_ent, int b) {
    const int lane = threadIdx.x & 31;
    for (int j = 0; j < n_ent; j++) {
        const int ent = ent0 + j;
        const float *g = A.GU + (size_t)ent * 2 * FF + b * 128 + lane * 4;
        const float4 a = __ldcg(reinterpret_cast<const float4 *>(g));
        const float4 u = __ldcg(reinterpret_cast<const float4 *>(g + FF));
        const float av[4] = {a.x, a.y, a.z, a.w}, uv[4] = {u.x, u.y, u.z, u.w};
        float v[1][4];
#pragma unroll
        for (int r = 0; r < 4; r++)
            v[0][r] = __fmul_rn(__fdiv_rn(av[r], __fadd_rn(1.0f, (float)exp(-(double)av[r]))), uv[r]);
        if (A.dn_rot > 1) warp_rotate<1, 4>(v, A.dn_seed, A.dn_norm, lane, b * 128);
        const size_t o = (size_t)ent * FF + b * 128;
        warp_quantize<1, 4>(v, 128, lane, A.dq64 + o, A.dsb64 + o / kGroup, nullptr, nullptr);
    }
}

// ---------------------------------------------------------------------------------------------------------------
template <bool Q8, int NGU, int NDN>
__global__ void __launch_bounds__(kFThreads, 1) fused_decode_kernel(const FusedArgs A) {
    constexpr int H = NGU * kGroup, FF = NDN * kGroup;
    constexpr int TGU = 2 * FF / 16, TDN = H / 16;  // row tiles per expert matrix
    constexpr int KC = Q8 ? 4 : 8, GB = Q8 ? 1024 : 512;
    constexpr int NCH_GU = (NGU + KC - 1) / KC, NCH_DN = (NDN + KC - 1) / KC;
    constexpr int GD_GU = (NGU + 3) / 4, GD_DN = (NDN + 3) / 4, GD = GD_GU > GD_DN ? GD_GU : GD_DN;
    extern __shared__ __align__(1024) uint8_t fsm[];
    FShared &S = *reinterpret_cast<FShared *>(fsm);
    const FLayout Lo = fused_layout(A.n, H, FF);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, n = A.n, E = A.E, K = A.K;
    int8_t *xq_s = reinterpret_cast<int8_t *>(fsm + Lo.xq);
    float2 *xsb_s = reinterpret_cast<float2 *>(fsm + Lo.xsb);
    uint8_t *wbase = fsm + Lo.warp0 + (size_t)warp * Lo.per_warp;
    uint8_t *ring = wbase;
    uint32_t *sblk = reinterpret_cast<uint32_t *>(wbase + Lo.sblk);  // [2][GD * 32] words
    int8_t *dact = reinterpret_cast<int8_t *>(wbase + Lo.dact);
    float2 *dsb = reinterpret_cast<float2 *>(wbase + Lo.dsb);

    if (threadIdx.x == 0) {
        mbar_init(&S.pa, 1);
        for (int w = 0; w < kFW; w++) {
            for (int s = 0; s < kFMaxStages; s++) mbar_init(&S.full[w][s], 1);
            mbar_init(&S.sfull[w][0], 1);
            mbar_init(&S.sfull[w][1], 1);
            mbar_init(&S.afull[w], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (blockIdx.x == 0) {  // this call's error words start clear (before any CTA can pass the barrier)
            A.meta[kMetaError] = kErrNone;
            A.meta[kMetaRouterError] = kErrNone;
        }
    }
    // ---------------- phase A ----------------
    __syncthreads();  // the barriers are initialised
    {
        // router: quad q = blockIdx.x, blockIdx.x + G, ... on warp 0; its weights by bulk copy, the inputs re-laid out
        // by the whole CTA, both into the (still unused) warp buffers
        const int nq = E / 4, SC = H / 64;
        float *xs = reinterpret_cast<float *>(fsm + Lo.warp0);
        uint4 *wq = reinterpret_cast<uint4 *>(fsm + Lo.warp0 + (size_t)n * H * 4);
        if (!A.ovr && (int)blockIdx.x < nq) {
            if (threadIdx.x == 0) {
                mbar_expect_tx(&S.pa, (uint32_t)(SC * 512));
                bulk_g2s(wq, A.router + (size_t)blockIdx.x * SC * 32, (uint32_t)(SC * 512), &S.pa);
            }
            for (int i = threadIdx.x; i < n * H; i += kFThreads) {
                const int t = i / H, k = i % H;  // k = 64 jc + 8 s + l  ->  [t][jc][l][s]
                xs[(size_t)t * H + (k / 64) * 64 + (k % 8) * 8 + (k / 8) % 8] = __ldg(A.x + i);
            }
            __syncthreads();
            int ph = 0;
            bool rok = true;
            for (int qd = blockIdx.x; warp == 0 && qd < nq; qd += G, ph ^= 1) {
                if (qd != (int)blockIdx.x && lane == 0) {  // a further quad (more quads than SMs)
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mbar_expect_tx(&S.pa, (uint32_t)(SC * 512));
                    bulk_g2s(wq, A.router + (size_t)qd * SC * 32, (uint32_t)(SC * 512), &S.pa);
                }
                if (!__all_sync(0xffffffffu, mbar_wait_bounded(&S.pa, ph))) {
                    rok = false;
                    break;
                }
                router_quad(A, qd, wq, xs);
                __syncwarp();
            }
            if (!rok && lane == 0) {
                set_error(A.meta, kErrTimeout);
                for (int r = 0; r < 64 && !mbar_wait_bounded(&S.pa, ph); r++) {
                }
            }
        }
        // decode-numerics quantization of the inputs: (token, 256-block) tasks on warps 1.. of every CTA
        const int na = n * (H / 256);
        if (warp >= 1)
            for (int a = blockIdx.x + G * (warp - 1); a < na; a += G * (kFW - 1))
                actq_task<NGU>(A, a / (H / 256), a % (H / 256));
        // this call's hand-off counters (ordered before any use by the grid barrier)
        const int nt = n * TDN;
        for (int i = blockIdx.x * kFThreads + threadIdx.x; i < (kFNB + 1) * E + nt; i += G * kFThreads) {
            if (i < kFNB * E) A.gu_done[i] = 0;
            else if (i < (kFNB + 1) * E) A.ready[i - kFNB * E] = 0;
            else A.ycnt[i - (kFNB + 1) * E] = 0;
        }
    }
    if (!grid_barrier(S, A.sync, A.meta)) return;

    // ---------------- phase B: routing of all n tokens, in every CTA ----------------
    {
        float *ex = reinterpret_cast<float *>(fsm + Lo.warp0);  // n x E floats over the warps' rings (unused yet)
        if (warp < n) {
            float *lg = ex + (size_t)warp * E;
            const float *src = A.ovr ? A.ovr + (size_t)warp * E : A.logits + (size_t)warp * E;
            for (int i = lane; i < E; i += 32) lg[i] = __ldcg(src + i);
            __syncwarp();
            if (blockIdx.x == 0 && A.ovr && A.ovr != A.logits)
                for (int i = lane; i < E; i += 32) A.logits[(size_t)warp * E + i] = lg[i];
            __syncwarp();
            softmax_topk_warp(lg, E, K, lg, (blockIdx.x == 0 && A.probs) ? A.probs + (size_t)warp * E : nullptr,
                              S.sel + warp * K, S.w + warp * K);
        }
        __syncthreads();
        // dispatch: the entries sorted by expert and, inside an expert, by (token, rank) -- entry i lands at
        // #{j : e_j < e_i} + #{j < i : e_j == e_i}; a unit starts where the expert changes
        const int nk = n * K;
        if ((int)threadIdx.x < nk) {
            const int i = threadIdx.x, ei = S.sel[i];
            int pos = 0;
            for (int j = 0; j < nk; j++) {
                const int ej = S.sel[j];
                pos += (ej < ei) | ((ej == ei) & (j < i));
            }
            S.etok[pos] = i / K;
            S.eslot[pos] = i;
            S.ew[pos] = S.w[i];
            S.esort[pos] = ei;
        }
        __syncthreads();
        int start = 0;
        if (warp < kFMaxEnt / 32) {
            const int p = threadIdx.x;
            start = p < nk && (p == 0 || S.esort[p - 1] != S.esort[p]);
            const uint32_t m = __ballot_sync(0xffffffffu, start);
            if (lane == 0) S.scan[warp] = __popc(m);
            start = start ? 1 + __popc(m & ((1u << lane) - 1u)) : 0;  // 1 + rank inside the warp
        }
        __syncthreads();
        if (start) {
            int u = start - 1;
            for (int w = 0; w < warp; w++) u += S.scan[w];
            S.unit_e[u] = S.esort[threadIdx.x];
            S.unit_off[u] = threadIdx.x;
        }
        if (threadIdx.x == 0) {
            int nu = 0;
            for (int w = 0; w < kFMaxEnt / 32; w++) nu += S.scan[w];
            S.nunits = nu;
            S.unit_off[nu] = nk;
        }
        __syncthreads();
        if (blockIdx.x == 0) {
            for (int i = threadIdx.x; i < nk; i += kFThreads) {
                A.sel[i] = S.sel[i];
                A.w[i] = S.w[i];
            }
            for (int i = threadIdx.x; i < S.nunits; i += kFThreads) A.units[i] = S.unit_e[i];
            if (threadIdx.x == 0) {
                A.meta[kMetaNUnits] = S.nunits;
                A.meta[kMetaNDec] = S.nunits;
                A.meta[kMetaNGemm] = 0;

            }
        }
        // the call's quantized inputs (written by phase-A tasks of other CTAs: read through L2)
        for (int i = threadIdx.x; i < n * H / 16; i += kFThreads)
            reinterpret_cast<uint4 *>(xq_s)[i] = __ldcg(reinterpret_cast<const uint4 *>(A.xq64) + i);
        for (int i = threadIdx.x; i < n * NGU; i += kFThreads) xsb_s[i] = __ldcg(A.xsb64 + i);
        __syncthreads();  // the rings may now be written (the softmax scratch is dead)
    }

    // ---------------- phases C and D: this warp's items ----------------
    const int U = S.nunits;
    const int ngu = U * TGU, nitems = ngu + U * TDN;
    const int NST = Lo.stages;
    const int NW = G * kFW, wid = warp * G + blockIdx.x;  // consecutive items go to different SMs
    auto item_of = [&](int k) { return wid + k * NW; };
    auto decode_item = [&](int i, int &kind, int &u, int &rt) {
        if (i < ngu) {
            kind = 0;
            u = i / TGU;
            rt = i % TGU;
        } else {
            kind = 1;
            u = (i - ngu) / TDN;
            rt = (i - ngu) % TDN;
        }
    };
    // lane 0's issue cursor: this warp's item ik (k-th item), chunk ic; `issued` stages in total
    int ik = 0, ic = 0, issued = 0;
    auto issue_upto = [&](int target, int kmax) {
        if (lane != 0) return;
        while (issued < target) {
            const int i = item_of(ik);
            if (i >= nitems || ik > kmax) break;
            int kind, u, rt;
            decode_item(i, kind, u, rt);
            const int e = S.unit_e[u];
            const MatLayout &M = kind ? A.dn : A.gu;
            const int ng = kind ? NDN : NGU, nch = kind ? NCH_DN : NCH_GU;
            const uint8_t *slab = A.pool + (size_t)e * A.slab_bytes;
            if (ic == 0) {  // the tile's scale block, with its first chunk, into the item's scale buffer
                const uint32_t sb = (uint32_t)((kind ? GD_DN : GD_GU) * 128);
                uint64_t *bar = &S.sfull[warp][ik & 1];
                mbar_expect_tx(bar, sb);
                bulk_g2s(sblk + (ik & 1) * GD * 32, slab + M.d_off + (size_t)rt * sb, sb, bar);
            }
            const int g0 = ic * KC, gn = ng - g0 < KC ? ng - g0 : KC;
            const int s = issued % NST;
            uint64_t *bar = &S.full[warp][s];
            mbar_expect_tx(bar, (uint32_t)(gn * GB));
            bulk_g2s(ring + (size_t)s * kFChunk, slab + M.q_off + ((size_t)rt * ng + g0) * GB, (uint32_t)(gn * GB), bar);
            issued++;
            if (++ic == nch) {
                ic = 0;
                ik++;
            }
        }
    };
    bool ok = true;
    int q = 0;     // stages consumed
    int ndn = 0;   // down items begun (phase of the activation barrier)
    int nsb = 0;   // items begun (scale blocks consumed)
    int act_out = 0;  // an activation copy is in flight
    if (lane == 0) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // after phases A/B's reads
    issue_upto(NST, 1);
    for (int k = 0; ok; k++) {
        const int i = item_of(k);
        if (i >= nitems) break;
        int kind, u, rt;
        decode_item(i, kind, u, rt);
        const int e = S.unit_e[u], ent0 = S.unit_off[u], nt = S.unit_off[u + 1] - ent0;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&S.sfull[warp][k & 1], (k >> 1) & 1))) {
            ok = false;
            break;
        }
        nsb = k + 1;
        const uint4 lut = Q8 ? make_uint4(0, 0, 0, 0)
                             : __ldg(reinterpret_cast<const uint4 *>(A.luts + (size_t)e * 32 + (kind ? 16 : 0)));
        if (kind == 1) {  // the expert's down inputs: wait for its SiLU warp's flag, then copy them in
            int got = 0;
            if (lane == 0) {
                got = wait_flag(A.ready + e, FF / 128) ? 1 : 0;
                if (got) {
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mbar_expect_tx(&S.afull[warp], (uint32_t)(nt * (FF + NDN * 8)));
                    bulk_g2s(dact, A.dq64 + (size_t)ent0 * FF, (uint32_t)(nt * FF), &S.afull[warp]);
                    bulk_g2s(dsb, A.dsb64 + (size_t)ent0 * NDN, (uint32_t)(nt * NDN * 8), &S.afull[warp]);
                }
            }
            got = __shfl_sync(0xffffffffu, got, 0);
            if (!got) {
                ok = false;
                break;
            }
            act_out = 1;
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&S.afull[warp], ndn & 1))) {
                ok = false;
                break;
            }
            act_out = 0;
            ndn++;
        }
        const uint32_t *sb = sblk + (k & 1) * GD * 32;
        const int q0 = q;
        // a consumed stage is refilled once every lane has used its values (the MMAs and folds that read them have
        // executed, so no read of the stage is still in flight)
        auto issue = [&](int c) { issue_upto(q0 + c + 1 + NST, k + 1); };
        float yv[kFMaxTok / 2];
        bool tok = false;
        auto run = [&](auto tc) {
            constexpr int TC = decltype(tc)::value;
            float yo[(TC + 1) / 2];
            if (kind == 0) {
                TileArgs<Q8, NGU, TC> T;
                T.ring = ring; T.full = S.full[warp]; T.q0 = q0; T.stages = NST; T.sblk = sb; T.lut = lut; T.ntok = nt;
                T.xbase = xq_s; T.sbase = xsb_s; T.tok = S.etok + ent0; T.xstride = H; T.sstride = NGU;
                tok = fused_tile<Q8, NGU, TC>(T, yo, issue);
            } else {
                TileArgs<Q8, NDN, TC> T;
                T.ring = ring; T.full = S.full[warp]; T.q0 = q0; T.stages = NST; T.sblk = sb; T.lut = lut; T.ntok = nt;
                T.xbase = dact; T.sbase = dsb; T.tok = nullptr; T.xstride = FF; T.sstride = NDN;
                tok = fused_tile<Q8, NDN, TC>(T, yo, issue);
            }
#pragma unroll
            for (int p = 0; p < (TC + 1) / 2; p++) yv[p] = yo[p];
        };
        if (nt <= 1) run(std::integral_constant<int, 1>());
        else if (nt <= 2) run(std::integral_constant<int, 2>());
        else if (nt <= 4) run(std::integral_constant<int, 4>());
        else if (nt <= 6) run(std::integral_constant<int, 6>());
        else run(std::integral_constant<int, 8>());
        q += kind ? NCH_DN : NCH_GU;
        if (!tok) {
            ok = false;
            break;
        }
        // this thread's outputs: token j = 2p + (lane & 3) / 2, row (lane >> 2) + 8 (lane & 1)
        const int gr = lane >> 2, jd = (lane & 3) >> 1, row = rt * 16 + gr + 8 * (lane & 1);
#pragma unroll
        for (int p = 0; p < kFMaxTok / 2; p++) {
            const int j = 2 * p + jd;
            if (j >= nt) continue;
            if (kind == 0) A.GU[(size_t)(ent0 + j) * 2 * FF + row] = yv[p];
            else A.mo[(size_t)S.eslot[ent0 + j] * H + row] = __fmul_rn(S.ew[ent0 + j], yv[p]);
        }
        __threadfence();
        __syncwarp();
        if (kind == 0) {
            // the last of the 16 gate|up tiles feeding 128-column block b of the down input: SiLU*up and quantization
            // of the block for all the expert's entries; the expert's flag counts finished blocks
            const int b = (rt % (TGU / 2)) / 8;
            int last = 0;
            if (lane == 0) last = atom_add_acq_rel(A.gu_done + e * kFNB + b, 1) == 15;
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
                __threadfence();
                swiglu_block<FF>(A, ent0, nt, b);
                __threadfence();
                __syncwarp();
                if (lane == 0) atom_add_acq_rel(A.ready + e, 1);
            }
        } else {
            // (token, row tile) completions: the K-th slot sums the token's K slots in rank order
            int done = 0, tk = 0;
            if (lane < nt) {
                tk = S.etok[ent0 + lane];
                done = atom_add_acq_rel(A.ycnt + (size_t)tk * TDN + rt, 1) == K - 1;
            }
            uint32_t m = __ballot_sync(0xffffffffu, done);
            if (m) __threadfence();
            while (m) {
                const int j = __ffs(m) - 1;
                m &= m - 1;
                const int tt = __shfl_sync(0xffffffffu, tk, j);
                if (lane < 16) {
                    const int rr = rt * 16 + lane;
                    float acc = 0.0f;
                    for (int kk = 0; kk < K; kk++) acc = __fadd_rn(acc, __ldcg(A.mo + ((size_t)tt * K + kk) * H + rr));
                    A.y[(size_t)tt * H + rr] = acc;
                }
            }
        }
        __syncwarp();
    }
    if (!ok && lane == 0) {
        set_error(A.meta, kErrTimeout);
        // drain, bounded: every bulk copy this warp issued lands before the CTA can leave
        for (int qq = issued - NST > q ? issued - NST : q; qq < issued; qq++)
            mbar_wait_bounded(&S.full[warp][qq % NST], (qq / NST) & 1);
        for (int kk = nsb; kk < ik + (ic > 0 ? 1 : 0); kk++) mbar_wait_bounded(&S.sfull[warp][kk & 1], (kk >> 1) & 1);
        if (act_out) mbar_wait_bounded(&S.afull[warp], ndn & 1);
    }
}

template <bool Q8, int NGU, int NDN>
void launch_one(const FusedArgs &A, int grid, size_t smem, cudaStream_t st) {
    cudaFuncSetAttribute(fused_decode_kernel<Q8, NGU, NDN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kFThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, fused_decode_kernel<Q8, NGU, NDN>, A);
}

}  // namespace

size_t fused_counter_ints(int E, int n_max, int H) {
    return (size_t)2 + (size_t)(kFNB + 1) * E + (size_t)n_max * (H / 16);
}

// The fused launch is taken for calls of at most kFUseMaxTok tokens: measured on B200 (decode layer, d = 2048), it
// beats the separate kernels at 1 and 2 tokens (43 vs 49 us, 55 vs 62 us) and loses from 3 tokens on, where the
// separate GEMV's wider items keep more warps busy per SM than the fused kernel's one warp per 16-row tile.
constexpr int kFUseMaxTok = 2;

bool fused_decode_fits(const LayerDev &L, int n, int K, bool have_router_or_ovr) {
    const int ngu = L.H / kGroup, ndn = L.FF / kGroup;
    if (n < 1 || n > kFUseMaxTok || K < 1 || K > kMaxTopK || L.E % 32 || L.E > 32 * kMaxPerLane) return false;
    if (ndn != 10 || (ngu != 32 && ngu != 40) || (L.gu_rot > 1 && L.gu_rot != 256) || (L.dn_rot > 1 && L.dn_rot != 128))
        return false;  // (FF = 640: five 128-column blocks, each fed by 8 gate and 8 up tiles)
    if (!have_router_or_ovr || (L.type != INZG_T_Q4L && L.type != INZG_T_Q8G)) return false;
    const FLayout Lo = fused_layout(n, L.H, L.FF);
    // the softmax scratch (n x E floats) lives over the warps' buffers
    // phase A stages the inputs and a router quad, phase B the softmax scratch (n x E floats), over the warps' buffers
    const size_t scratch = (size_t)kFW * Lo.per_warp;
    return Lo.total <= kFSmemMax && (size_t)n * L.E * 4 <= scratch &&
           (size_t)n * L.H * 4 + (size_t)(L.H / 64) * 512 <= scratch;
}

int launch_fused_decode(const LayerDev &L, int n, int K, const float *x, const float *bias, const float *ovr,
                        float *logits, float *probs, int32_t *sel, float *w, int32_t *units, int32_t *meta,
                        int8_t *xq64, float2 *xsb64, float *GU, int8_t *dq64, float2 *dsb64, float *mo, float *y,
                        int32_t *counters, int num_sms, cudaStream_t st) {
    if (!fused_decode_fits(L, n, K, L.router || ovr)) return -1;
    const int H = L.H, FF = L.FF, E = L.E;
    const bool q8 = L.type == INZG_T_Q8G;
    const FLayout Lo = fused_layout(n, H, FF);
    FusedArgs A{};
    A.pool = L.pool; A.slab_bytes = L.slab_bytes; A.gu = L.gu; A.dn = L.dn; A.luts = L.luts; A.router = L.router;
    A.gu_rot = L.gu_rot; A.dn_rot = L.dn_rot; A.gu_seed = L.gu_seed; A.dn_seed = L.dn_seed;
    A.gu_norm = L.gu_rot > 1 ? 1.0f / sqrtf((float)L.gu_rot) : 1.0f;
    A.dn_norm = L.dn_rot > 1 ? 1.0f / sqrtf((float)L.dn_rot) : 1.0f;
    A.H = H; A.FF = FF; A.E = E; A.K = K; A.n = n;
    A.x = x; A.bias = bias; A.ovr = ovr; A.logits = logits; A.probs = probs; A.sel = sel; A.w = w; A.units = units;
    A.meta = meta; A.xq64 = xq64; A.xsb64 = xsb64; A.GU = GU; A.dq64 = dq64; A.dsb64 = dsb64; A.mo = mo; A.y = y;
    A.sync = counters; A.gu_done = counters + 2; A.ready = counters + 2 + kFNB * E;
    A.ycnt = counters + 2 + (kFNB + 1) * E;
    const size_t smem = (size_t)Lo.total;
    if (q8) {
        if (H == 2048) launch_one<true, 32, 10>(A, num_sms, smem, st);
        else launch_one<true, 40, 10>(A, num_sms, smem, st);
    } else {
        if (H == 2048) launch_one<false, 32, 10>(A, num_sms, smem, st);
        else launch_one<false, 40, 10>(A, num_sms, smem, st);
    }
    return 1;
}

}  // namespace inzg
