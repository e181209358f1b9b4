// k_router.cu -- F16 router, softmax and top-k on sm_100a, bit-exact with the reference CPU path.
//
// Logits: the reference's inz_matvec_f16_rows (src/quant.c:1290-1304) keeps 8 fp32 accumulators per (row, token):
// lane l accumulates f16(W[e][8j+l]) * x[8j+l] over j = 0, 1, ... with one FMA each, then hsum8
// ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)) (src/quant.c:705-711). Here one thread owns one (expert, lane) chain and
// runs the same FMAs in the same order; the 8 threads of an expert finish with the same add tree over shuffles.
// The router is re-laid out at upload so that a warp (4 experts x 8 lanes) reads one contiguous 512-byte segment per
// 8 chain steps: Wr[eq][jc][e%4][l][8 halves], eq = e/4, jc = j/8.
#include "inzg_internal.h"
#include "k_launch.h"
#include "k_softmax.cuh"
#include "k_async.cuh"

#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>

namespace inzg {

// W [E][H] f16 -> Wr (see above). One thread per output uint4.
__global__ void router_repack_kernel(const uint16_t *__restrict__ W, uint4 *__restrict__ Wr, int E, int H) {
    const int S = H / 8, SC = S / 8;  // chain steps per lane, 8-step chunks
    const int64_t total = (int64_t)(E / 4) * SC * 32;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int l = (int)(i % 8), e4 = (int)((i / 8) % 4), jc = (int)((i / 32) % SC), eq = (int)(i / (32 * SC));
        const int e = eq * 4 + e4;
        uint16_t h[8];
        for (int s = 0; s < 8; s++) h[s] = W[(size_t)e * H + 8 * (jc * 8 + s) + l];
        uint4 v;
        v.x = h[0] | ((uint32_t)h[1] << 16);
        v.y = h[2] | ((uint32_t)h[3] << 16);
        v.z = h[4] | ((uint32_t)h[5] << 16);
        v.w = h[6] | ((uint32_t)h[7] << 16);
        Wr[i] = v;
    }
}

__device__ __forceinline__ float h2f(uint32_t bits16) { return __half2float(__ushort_as_half((unsigned short)bits16)); }

// x tile of TT tokens -> shared [tt][l][S + 4] (lane-major: a thread reads its chain steps contiguously; the pad of 4
// floats puts the 8 lanes of an expert on distinct banks). float4 global loads, all in flight together.
template <int TT>
__device__ __forceinline__ void stage_x(float *xs, const float *__restrict__ X, int t0, int nt, int H) {
    const int S = H / 8, SP = S + 4, H4 = H / 4;
    for (int i = threadIdx.x; i < TT * H4; i += blockDim.x) {
        const int tt = i / H4, k4 = i % H4;
        const float4 v = tt < nt ? reinterpret_cast<const float4 *>(X + (size_t)(t0 + tt) * H)[k4]
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        const int k = 4 * k4;  // k, k+1, k+2, k+3: lanes (k&7)..(k&7)+3 of step k>>3
        float *d = xs + (size_t)tt * 8 * SP + (k & 7) * SP + (k >> 3);
        d[0] = v.x; d[SP] = v.y; d[2 * SP] = v.z; d[3 * SP] = v.w;
    }
}

__device__ __forceinline__ void h8(const uint4 &v, float w[8]) {
    w[0] = h2f(v.x & 0xFFFF); w[1] = h2f(v.x >> 16); w[2] = h2f(v.y & 0xFFFF); w[3] = h2f(v.y >> 16);
    w[4] = h2f(v.z & 0xFFFF); w[5] = h2f(v.z >> 16); w[6] = h2f(v.w & 0xFFFF); w[7] = h2f(v.w >> 16);
}

// 8 chain steps of one (expert, lane) for one token: r = fma(w[s], x[s], r), s = 0..7 in order
__device__ __forceinline__ float chain8(float r, const float w[8], const float *xp) {
    const float4 a = reinterpret_cast<const float4 *>(xp)[0], b = reinterpret_cast<const float4 *>(xp)[1];
    r = __fmaf_rn(w[0], a.x, r); r = __fmaf_rn(w[1], a.y, r); r = __fmaf_rn(w[2], a.z, r); r = __fmaf_rn(w[3], a.w, r);
    r = __fmaf_rn(w[4], b.x, r); r = __fmaf_rn(w[5], b.y, r); r = __fmaf_rn(w[6], b.z, r); r = __fmaf_rn(w[7], b.w, r);
    return r;
}

__device__ __forceinline__ void write_logit(float acc, int l, int tt, int nt, int t0, int e, int E,
                                            const float *__restrict__ bias, float *__restrict__ logits) {
    float s = hsum8_lanes(acc);
    if (l == 0 && tt < nt && e < E) {
        if (bias) s = __fadd_rn(s, bias[e]);  // test hook: logits[x] += bias[x] before the softmax
        logits[(size_t)(t0 + tt) * E + e] = s;
    }
}

// Few tokens: thread (q, l) of a warp owns lane l of two experts, 8b + q and 8b + 4 + q (one from each of two
// consecutive quads of the re-laid-out router), for TT tokens. The block requests everything at once with bulk
// copies -- its 2 x WPB quads of weights (contiguous in Wr) and the TT token rows in natural layout -- then runs the
// chains from shared memory: per 8 chain steps one 16-byte load of weights per expert and one 4-byte load of x per
// step and token (the warp's 8 lanes read 8 consecutive floats; the 4 q's share them), each x feeding two FMAs.
template <int TT, int WPB>
__global__ void __launch_bounds__(WPB * 32) router_small_kernel(const uint4 *__restrict__ Wr, const float *__restrict__ X,
                                                                 int n, int H, int E, const float *__restrict__ bias,
                                                                 float *__restrict__ logits, int32_t *__restrict__ meta) {
    extern __shared__ __align__(128) uint8_t rsm[];
    const int S = H / 8, SC = S / 8;
    uint64_t *bar = reinterpret_cast<uint64_t *>(rsm);
    uint4 *ws = reinterpret_cast<uint4 *>(rsm + 128);                            // [2 * WPB quads][SC][32]
    float *xs = reinterpret_cast<float *>(rsm + 128 + (size_t)2 * WPB * SC * 512);  // [TT][H]
    const int t0 = blockIdx.y * TT, nt = min(TT, n - t0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int eq0 = blockIdx.x * 2 * WPB, nq = min(2 * WPB, E / 4 - eq0);  // expert quads of this block
    if (nq <= 0) return;
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        mbar_expect_tx(bar, (uint32_t)(nq * SC * 512 + nt * H * 4));
        bulk_g2s(ws, Wr + (size_t)eq0 * SC * 32, (uint32_t)(nq * SC * 512), bar);
        for (int tt = 0; tt < nt; tt++) bulk_g2s(xs + (size_t)tt * H, X + (size_t)(t0 + tt) * H, (uint32_t)(H * 4), bar);
    }
    __syncthreads();
    if (!mbar_wait_bounded(bar, 0)) {
        // the copies did not land in time: record it, then let thread 0 keep polling (up to 64 more bounded rounds)
        // -- the CTA's shared memory stays allocated while any of its threads runs, so a late copy cannot land in
        // the next CTA's (no barrier here: other threads may have seen the phase complete)
        if (lane == 0 && meta) atomicCAS(&meta[kMetaRouterError], 0, kErrTimeout);
        if (threadIdx.x == 0)
            for (int r = 0; r < 64 && !mbar_wait_bounded(bar, 0); r++) {
            }
        return;
    }
    const int qa = 2 * warp, l = lane & 7;
    if (qa >= nq) return;
    const bool hb = qa + 1 < nq;
    const uint4 *wa = ws + (size_t)qa * SC * 32 + lane, *wb = wa + (size_t)SC * 32;
    const float *xl = xs + l;
    float A[TT], B[TT];
#pragma unroll
    for (int tt = 0; tt < TT; tt++) A[tt] = B[tt] = 0.0f;
#pragma unroll 1
    for (int jc = 0; jc < SC; jc++) {
        float w1[8], w2[8];
        h8(wa[(size_t)jc * 32], w1);
        h8(hb ? wb[(size_t)jc * 32] : make_uint4(0, 0, 0, 0), w2);
#pragma unroll
        for (int s = 0; s < 8; s++) {
#pragma unroll
            for (int tt = 0; tt < TT; tt++) {
                const float x = xl[(size_t)tt * H + (jc * 8 + s) * 8];
                A[tt] = __fmaf_rn(w1[s], x, A[tt]);
                B[tt] = __fmaf_rn(w2[s], x, B[tt]);
            }
        }
    }
    const int ea = (eq0 + qa) * 4 + (lane >> 3), eb = ea + 4;
#pragma unroll
    for (int tt = 0; tt < TT; tt++) {
        write_logit(A[tt], l, tt, nt, t0, ea, E, bias, logits);
        if (hb) write_logit(B[tt], l, tt, nt, t0, eb, E, bias, logits);
    }
}

// Many tokens: FMA-bound (4.3 G FMA at 4096 tokens). Thread = (lane l, 2 experts from two quads, 8 tokens): each
// 16-byte shared load of x (4 chain steps of one token) feeds 8 FMAs; the next chunk's weights load during the FMAs.
// Block = 8 warps = 16 expert quads = 64 experts; grid = (E / 64, n / 8).
// LT tokens per block: 8 for many tokens (8 FMAs per x load); 2 or 4 for decode-sized calls, where the grid needs
// more blocks than tokens / 8 to put several warps of chains on every SM (the weights then come from L2 once per
// token block).
constexpr int kLT = 8;
template <int LT, int EPT = 2>
__global__ void __launch_bounds__(256) router_large_kernel(const uint4 *__restrict__ Wr, const float *__restrict__ X,
                                                           int n, int H, int E, const float *__restrict__ bias,
                                                           float *__restrict__ logits) {
    extern __shared__ __align__(16) float xs[];
    const int S = H / 8, SC = S / 8, SP = S + 4;
    const int t0 = blockIdx.y * LT, nt = min(LT, n - t0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, l = lane & 7;
    // the warp's expert quads: qa, and qb = qa + 1 when a thread runs two experts
    const int qa = blockIdx.x * 8 * EPT + warp * EPT, qb = qa + 1;
    const int ea = qa * 4 + (lane >> 3), eb = qb * 4 + (lane >> 3);
    const bool live = qa * 4 < E;
    const uint4 *wa = Wr + (size_t)qa * SC * 32 + lane, *wb = Wr + (size_t)qb * SC * 32 + lane;
    const bool hasb = EPT == 2 && qb * 4 < E;
    // the weights stream from L2 through an 8-chunk register ring
    constexpr int PF = 8;
    uint4 ra[PF], rb[PF];
#pragma unroll
    for (int u = 0; u < PF; u++) {  // u < SC: a matrix narrower than 8 chunks (K < 512) has fewer to fetch
        ra[u] = live && u < SC ? __ldg(wa + (size_t)u * 32) : make_uint4(0, 0, 0, 0);
        rb[u] = hasb && u < SC ? __ldg(wb + (size_t)u * 32) : make_uint4(0, 0, 0, 0);
    }
    stage_x<LT>(xs, X, t0, nt, H);
    __syncthreads();
    if (!live) return;
    float A[LT], B[LT];
#pragma unroll
    for (int tt = 0; tt < LT; tt++) { A[tt] = 0.0f; B[tt] = 0.0f; }
    for (int jc0 = 0; jc0 < SC; jc0 += PF) {
#pragma unroll
        for (int u = 0; u < PF; u++) {
            const int jc = jc0 + u;
            if (jc >= SC) break;  // H % 512 != 0: the last pass is partial
            float w1[8], w2[8];
            h8(ra[u], w1);
            if (EPT == 2) h8(rb[u], w2);
            if (jc + PF < SC) {
                ra[u] = __ldg(wa + (size_t)(jc + PF) * 32);
                if (hasb) rb[u] = __ldg(wb + (size_t)(jc + PF) * 32);
            }
#pragma unroll
            for (int tt = 0; tt < LT; tt++) {
                const float *xp = xs + (size_t)tt * 8 * SP + l * SP + jc * 8;
                const float4 a = reinterpret_cast<const float4 *>(xp)[0], b = reinterpret_cast<const float4 *>(xp)[1];
                float r = A[tt];
                r = __fmaf_rn(w1[0], a.x, r); r = __fmaf_rn(w1[1], a.y, r); r = __fmaf_rn(w1[2], a.z, r);
                r = __fmaf_rn(w1[3], a.w, r); r = __fmaf_rn(w1[4], b.x, r); r = __fmaf_rn(w1[5], b.y, r);
                r = __fmaf_rn(w1[6], b.z, r); r = __fmaf_rn(w1[7], b.w, r);
                A[tt] = r;
                if (EPT == 2) {
                    float q = B[tt];
                    q = __fmaf_rn(w2[0], a.x, q); q = __fmaf_rn(w2[1], a.y, q); q = __fmaf_rn(w2[2], a.z, q);
                    q = __fmaf_rn(w2[3], a.w, q); q = __fmaf_rn(w2[4], b.x, q); q = __fmaf_rn(w2[5], b.y, q);
                    q = __fmaf_rn(w2[6], b.z, q); q = __fmaf_rn(w2[7], b.w, q);
                    B[tt] = q;
                }
            }
        }
    }
#pragma unroll
    for (int tt = 0; tt < LT; tt++) {
        write_logit(A[tt], l, tt, nt, t0, ea, E, bias, logits);
        if (hasb) write_logit(B[tt], l, tt, nt, t0, eb, E, bias, logits);
    }
}

// Many tokens, fp32 router copy: eight SIMT sub-GEMMs, one per chain lane l (warp l of the block):
// C_l[t][e] = sum_j f16(W[e][8j+l]) * x[t][8j+l], j in order, one FMA each -- the reference's accumulator l of (e, t);
// the block then adds the eight in the reference's tree. Block = 64 tokens x 32 experts; thread (warp l, token group
// tg = lane & 7, expert group eg = lane >> 3) holds tokens tg + 8i (i < 8) x experts 8 eg + m (m < 8): per chain step
// 8 scalar loads of x, 2 vector loads of weights and 64 FMAs (32 packed f32x2 FMAs, each lane rounded as its own FMA).
// Per 16-step chunk the block's fp32 weights arrive in one 16 KB bulk copy (layout [l][j][e], made at upload) and the
// 64 token rows' 128 floats in four 64 x 32-float tensor copies with 128-byte swizzle: the 16-byte column group g of
// row t lands at group g ^ (t % 8), so the 8 token groups of a load (t % 8 = tg) sit on distinct banks; rows past
// the call's tokens read as zeros. Two chunks in flight, one block barrier per chunk; two blocks per SM.
constexpr int kRT = 64, kRE = 32, kRJ = 16, kRStages = 2;
constexpr int kRWBytes = 8 * kRJ * kRE * 4, kRBoxBytes = kRT * 32 * 4, kRXBytes = (kRJ * 8 / 32) * kRBoxBytes;
constexpr int kRStageBytes = kRWBytes + kRXBytes;  // a multiple of 1024: every box starts 1024-byte aligned
constexpr int kRRedStride = kRE + 1;  // reduction rows [l][t][e], padded: a warp's 32 lanes hit 32 banks
constexpr int kRouterGemmMinTokens = 320;  // below: the f16 kernel, whose 8-token tiles spread over every SM

size_t router_gemm_smem() {
    const size_t red = (size_t)8 * kRT * kRRedStride * 4, stages = (size_t)kRStages * kRStageBytes;
    return 1024 + (red > stages ? red : stages);
}

// 128-column chunks of an H-wide matrix; a last partial chunk is padded with zero weights, and the tensor copies of x
// read zeros past column H, so each padded step is fma(0, 0, acc) = acc: the chains stay exact (acc is never -0, as
// every chain starts at +0)
__host__ __device__ __forceinline__ int router_chunks(int H) { return (H + 8 * kRJ - 1) / (8 * kRJ); }

size_t router32_floats(int E, int H) { return (size_t)E * router_chunks(H) * 8 * kRJ; }

// W [E][H] f16 -> Wf [E/32][chunks][8][16][32] fp32 (see above). One thread per output float.
__global__ void router_repack32_kernel(const uint16_t *__restrict__ W, float *__restrict__ Wf, int E, int H) {
    const int nch = router_chunks(H);
    const int64_t total = (int64_t)E * nch * 8 * kRJ;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int e_ = (int)(i % kRE), j_ = (int)((i / kRE) % kRJ), l = (int)((i / (kRE * kRJ)) % 8);
        const int c = (int)((i / (kRE * kRJ * 8)) % nch), eb = (int)(i / ((int64_t)kRE * kRJ * 8 * nch));
        const int k = 8 * (c * kRJ + j_) + l;
        Wf[i] = k < H ? h2f(W[(size_t)(eb * kRE + e_) * H + k]) : 0.0f;
    }
}

__global__ void __launch_bounds__(256, 2) router_gemm_kernel(const __grid_constant__ CUtensorMap mapX,
                                                            const float *__restrict__ Wf, int n, int H, int E,
                                                            const float *__restrict__ bias,
                                                            float *__restrict__ logits, int32_t *__restrict__ meta) {
    extern __shared__ uint8_t rgs_raw[];
    __shared__ uint64_t bar[kRStages];
    uint8_t *stage0 = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(rgs_raw) + 1023) & ~uintptr_t(1023));
    const int eb = blockIdx.x, t0 = blockIdx.y * kRT, nt = min(kRT, n - t0);
    const int nch = router_chunks(H);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tg = lane & 7, eg = lane >> 3;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kRStages; s++) mbar_init(&bar[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // one thread requests chunk c into stage c % kRStages
    auto issue = [&](int c) {
        const int s = c % kRStages;
        uint8_t *st = stage0 + (size_t)s * kRStageBytes;
        mbar_expect_tx(&bar[s], (uint32_t)kRStageBytes);
        bulk_g2s(st, Wf + ((size_t)eb * nch + c) * (8 * kRJ * kRE), kRWBytes, &bar[s]);
#pragma unroll
        for (int b = 0; b < kRJ * 8 / 32; b++)
            tma_load_2d(st + kRWBytes + b * kRBoxBytes, &mapX, c * kRJ * 8 + b * 32, t0, &bar[s]);
    };
    if (threadIdx.x == 0)
        for (int c = 0; c < kRStages && c < nch; c++) issue(c);
    // x[t][8j + l] of chunk-local step j: box j / 4, column 8 (j % 4) + l, i.e. 16-byte group 2 (j % 4) + l / 4
    // (swizzled with t % 8 = tg) and word l % 4; token t = tg + 8i adds 8i rows of 32 floats
    int xoff[4];
#pragma unroll
    for (int q = 0; q < 4; q++) xoff[q] = tg * 32 + (((2 * q + (warp >> 2)) ^ tg) * 4) + (warp & 3);
    float2 acc[8][4];  // [token i][expert pair]: experts 8 eg + 2p, 8 eg + 2p + 1
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int p = 0; p < 4; p++) acc[i][p] = make_float2(0.0f, 0.0f);
    int failed = -1;  // the chunk whose copies did not land (the same for every thread)
    for (int c = 0; c < nch; c++) {
        const int s = c % kRStages;
        const bool got = mbar_wait_bounded(&bar[s], (c / kRStages) & 1);
        if (got) {
            const uint8_t *st = stage0 + (size_t)s * kRStageBytes;
            const float *wl = reinterpret_cast<const float *>(st) + warp * (kRJ * kRE) + eg * 8;
            const float *xb = reinterpret_cast<const float *>(st + kRWBytes);
#pragma unroll 4
            for (int j = 0; j < kRJ; j++) {
                const float4 wa = *reinterpret_cast<const float4 *>(wl + j * kRE);
                const float4 wb = *reinterpret_cast<const float4 *>(wl + j * kRE + 4);
                const float2 w2[4] = {make_float2(wa.x, wa.y), make_float2(wa.z, wa.w), make_float2(wb.x, wb.y),
                                      make_float2(wb.z, wb.w)};
                const float *xl = xb + (j >> 2) * (kRBoxBytes / 4) + xoff[j & 3];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float xv = xl[i * 8 * 32];
                    const float2 x2 = make_float2(xv, xv);
#pragma unroll
                    for (int p = 0; p < 4; p++) acc[i][p] = __ffma2_rn(w2[p], x2, acc[i][p]);
                }
            }
        }
        if (__syncthreads_or(!got)) {  // every warp is done with stage s (or the copies did not land)
            failed = c;
            break;
        }
        if (threadIdx.x == 0 && c + kRStages < nch) {
            fence_proxy_async_smem();
            issue(c + kRStages);
        }
    }
    if (failed >= 0) {  // record it, wait (bounded) for what is in flight, leave
        if (threadIdx.x == 0) {
            if (meta) atomicCAS(&meta[kMetaRouterError], 0, kErrTimeout);
            for (int c = failed; c < nch && c < failed + kRStages; c++)
                mbar_wait_bounded(&bar[c % kRStages], (c / kRStages) & 1);
        }
        __syncthreads();
        return;
    }
    // the eight chain lanes of every (token, expert) meet in shared memory: red[l][t][e]
    float *red = reinterpret_cast<float *>(stage0);
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int p = 0; p < 4; p++) {
            float *r = red + ((size_t)warp * kRT + tg + 8 * i) * kRRedStride + eg * 8 + 2 * p;
            r[0] = acc[i][p].x;
            r[1] = acc[i][p].y;
        }
    __syncthreads();
    for (int idx = threadIdx.x; idx < kRT * kRE; idx += blockDim.x) {
        const int t = idx / kRE, e_ = idx % kRE;
        float a[8];
#pragma unroll
        for (int l = 0; l < 8; l++) a[l] = red[((size_t)l * kRT + t) * kRRedStride + e_];
        float v = __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[4]), __fadd_rn(a[2], a[6])),
                            __fadd_rn(__fadd_rn(a[1], a[5]), __fadd_rn(a[3], a[7])));
        const int e = eb * kRE + e_;
        if (t < nt) {
            if (bias) v = __fadd_rn(v, bias[e]);  // test hook: logits[x] += bias[x] before the softmax
            logits[(size_t)(t0 + t) * E + e] = v;
        }
    }
}

// One warp per token: the routing weights of every token (see k_softmax.cuh).
__global__ void __launch_bounds__(256) softmax_topk_kernel(const float *__restrict__ logits, int n, int E, int topk,
                                                            int32_t *__restrict__ sel, float *__restrict__ wsel,
                                                            float *__restrict__ probs_out) {
    __shared__ float ex[8][1024];
    const int warp = threadIdx.x >> 5;
    const int t = blockIdx.x * (blockDim.x >> 5) + warp;
    if (t >= n) return;
    softmax_topk_warp(logits + (size_t)t * E, E, topk, ex[warp], probs_out ? probs_out + (size_t)t * E : nullptr,
                      sel + (size_t)t * topk, wsel + (size_t)t * topk);
}

// ---------------------------------------------------------------------------------------------------------------
void launch_router_repack(const uint16_t *W, uint4 *Wr, int E, int H, cudaStream_t st) {
    const int64_t total = (int64_t)(E / 4) * (H / 64) * 32;
    const int blocks = (int)((total + 255) / 256);
    router_repack_kernel<<<blocks, 256, 0, st>>>(W, Wr, E, H);
}

void launch_router_repack32(const uint16_t *W, float *Wf, int E, int H, cudaStream_t st) {
    const int64_t total = (int64_t)router32_floats(E, H);
    router_repack32_kernel<<<(int)std::min<int64_t>((total + 255) / 256, 65535), 256, 0, st>>>(W, Wf, E, H);
}

bool router_gemm_fits(int E, int H) { return E % kRE == 0 && H % 64 == 0; }

static size_t router_smem(int TT, int H) { return (size_t)TT * 8 * (H / 8 + 4) * sizeof(float); }
static size_t router_small_smem(int TT, int WPB, int H) { return 128 + (size_t)2 * WPB * H * 8 + (size_t)TT * H * 4; }

// the opt-in shared memory per block of the current device
static size_t smem_optin() {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    return (size_t)v;
}

// Raises a kernel's dynamic shared memory limit on the current device to `bytes` (never lowers it: contexts of
// different widths share the kernels); sizes above the device's limit are skipped -- launch_f16_rows does not pick
// those kernels. The current limit is read back from the device, so each device (and a re-created context) is set
// on its own.
template <class F>
static void raise_smem(F *fn, size_t bytes, size_t cap) {
    cudaFuncAttributes fa{};
    if (bytes > cap) return;
    if (cudaFuncGetAttributes(&fa, fn) == cudaSuccess && (size_t)fa.maxDynamicSharedSizeBytes >= bytes) return;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
        cudaGetLastError();
}

void router_set_attributes(int H) {
    const size_t cap = smem_optin();
    raise_smem(router_large_kernel<kLT>, router_smem(kLT, H), cap);
    raise_smem(router_large_kernel<4, 2>, router_smem(4, H), cap);
    raise_smem(router_large_kernel<2, 2>, router_smem(2, H), cap);
    raise_smem(router_gemm_kernel, router_gemm_smem(), cap);
    raise_smem(router_small_kernel<1, 1>, router_small_smem(1, 1, H), cap);
    raise_smem(router_small_kernel<2, 1>, router_small_smem(2, 1, H), cap);
}

int launch_router_logits(const uint4 *Wr, const float *Wf, const float *X, int n, int H, int E, const float *bias,
                         float *logits, int32_t *meta, cudaStream_t st) {
    CUtensorMap mapX;
    // 1-2 tokens: every block pulls its experts' weights and the token tile in one go, one warp (8 experts) per block so
    // the 2 MB router spreads over every SM. 3-64 tokens: 64 experts x 2-4 tokens per block of 8 warps, weights
    // streamed from L2. Many tokens: 64 experts x 8 tokens per block (or the TMA-tiled kernel), FMA-bound.
    if (n <= 1) {
        router_small_kernel<1, 1><<<dim3((E / 4 + 1) / 2, n), 32, router_small_smem(1, 1, H), st>>>(Wr, X, n, H, E, bias, logits, meta);
    } else if (n <= 2) {
        router_small_kernel<2, 1><<<dim3((E / 4 + 1) / 2, 1), 32, router_small_smem(2, 1, H), st>>>(Wr, X, n, H, E, bias, logits, meta);
    } else if (n <= 32) {  // ROUTER_SMALL_CALL
        router_large_kernel<2, 2><<<dim3((E + 63) / 64, (n + 1) / 2), 256, router_smem(2, H), st>>>(Wr, X, n, H, E, bias, logits);
    } else if (n <= 64) {
        router_large_kernel<4, 2><<<dim3((E + 63) / 64, (n + 3) / 4), 256, router_smem(4, H), st>>>(Wr, X, n, H, E, bias, logits);
    } else if (Wf && n >= kRouterGemmMinTokens && router_gemm_fits(E, H) && make_tma_map_f32(&mapX, X, n, H, kRT)) {
        router_gemm_kernel<<<dim3(E / kRE, (n + kRT - 1) / kRT), 256, router_gemm_smem(), st>>>(mapX, Wf, n, H, E, bias,
                                                                                              logits, meta);
    } else {
        dim3 grid((E + 63) / 64, (n + kLT - 1) / kLT);
        router_large_kernel<kLT><<<grid, 256, router_smem(kLT, H), st>>>(Wr, X, n, H, E, bias, logits);
    }
    return 1;
}

// Y[t][r] = sum_k f16(W[r][k]) x[t][k] in the router's chain order for any rows % 4 == 0 and K % 64 == 0 -- lin_mm's
// F16 path (src/model_fwd.c:104-121), used for the hyper-connection matrices (320 x 4H and 4H x 320): the router's
// kernels, each picked only when its shared memory at this K fits the device (router_set_attributes(K) first).
// Returns the number of kernels launched, -1 when no kernel fits.
int launch_f16_rows(const uint4 *Wr, const float *Wf, const float *X, int n, int K, int rows, float *Y, int32_t *meta,
                    cudaStream_t st) {
    if (n <= 0 || rows % 4 || K % 64) return -1;
    const size_t cap = smem_optin();
    CUtensorMap mapX;
    if (n == 1 && router_small_smem(1, 1, K) <= cap) {
        router_small_kernel<1, 1><<<dim3((rows / 4 + 1) / 2, 1), 32, router_small_smem(1, 1, K), st>>>(Wr, X, n, K, rows, nullptr, Y, meta);
    } else if (n == 2 && router_small_smem(2, 1, K) <= cap) {
        router_small_kernel<2, 1><<<dim3((rows / 4 + 1) / 2, 1), 32, router_small_smem(2, 1, K), st>>>(Wr, X, n, K, rows, nullptr, Y, meta);
    } else if (n <= 32 && router_smem(2, K) <= cap) {
        router_large_kernel<2, 2><<<dim3((rows + 63) / 64, (n + 1) / 2), 256, router_smem(2, K), st>>>(Wr, X, n, K, rows, nullptr, Y);
    } else if (n <= 64 && router_smem(4, K) <= cap) {
        router_large_kernel<4, 2><<<dim3((rows + 63) / 64, (n + 3) / 4), 256, router_smem(4, K), st>>>(Wr, X, n, K, rows, nullptr, Y);
    } else if (Wf && n >= kRouterGemmMinTokens && router_gemm_fits(rows, K) && make_tma_map_f32(&mapX, X, n, K, kRT)) {
        router_gemm_kernel<<<dim3(rows / kRE, (n + kRT - 1) / kRT), 256, router_gemm_smem(), st>>>(mapX, Wf, n, K, rows,
                                                                                                 nullptr, Y, meta);
    } else if (router_smem(kLT, K) <= cap) {
        router_large_kernel<kLT><<<dim3((rows + 63) / 64, (n + kLT - 1) / kLT), 256, router_smem(kLT, K), st>>>(Wr, X, n, K, rows, nullptr, Y);
    } else if (router_smem(4, K) <= cap) {
        router_large_kernel<4, 2><<<dim3((rows + 63) / 64, (n + 3) / 4), 256, router_smem(4, K), st>>>(Wr, X, n, K, rows, nullptr, Y);
    } else {
        return -1;
    }
    return 1;
}

int launch_softmax_topk(const float *logits, int n, int E, int topk, int32_t *sel, float *w, float *probs,
                        cudaStream_t st) {
    softmax_topk_kernel<<<(n + 7) / 8, 256, 0, st>>>(logits, n, E, topk, sel, w, probs);
    return 1;
}

}  // namespace inzg
