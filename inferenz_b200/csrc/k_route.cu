// k_route.cu -- token -> expert dispatch lists on the device.
//
// The reference builds, per token in order, "units" = per-expert lists of (token, slot = t*topk + k, weight)
// (src/model_fwd.c:1001-1031). The lists here hold the same entries, sorted by expert and, within an expert, by
// token -- the order the reference appends them -- without atomics on positions, so the result is deterministic:
//   route_mask    per 64-token chunk (one block): a 64-bit token mask per expert (shared-memory atomicOr), the
//                 chunk's count per expert = the mask's popcount
//   route_scan    one block: per-expert prefix over chunks, counts, offsets, expert lists and the
//                 per-expert numeric path (decode numerics when n <= 8 or the expert has < GEMM_MIN_T tokens,
//                 src/model_fwd.c:229-249, 1070), work counts for the expert kernels
//   route_scatter per chunk: entry position = off[e] + chunk prefix + popcount of the expert's mask below the token
// The decode-path expert list is the one list in scheduling order: heaviest experts (most tokens) first, so the
// decode GEMV's work queue ends on light items. Every output position is fixed by the entry lists, so that order
// (which is not deterministic within one token count) never changes a result.
#include "inzg_internal.h"
#include "k_launch.h"
#include "k_softmax.cuh"

#include <cooperative_groups.h>

namespace cg = cooperative_groups;

namespace inzg {

constexpr int kChunk = 64;  // tokens per route chunk: one 64-bit mask word per expert

// Decode experts in descending token count (bins by count, positions inside a bin by shared atomics); every thread
// of the block calls it. bins: 32 ints of shared scratch. Also clears the decode GEMV work-queue counters.
__device__ void order_dec_units(int is_dec, int c, int e, int32_t *__restrict__ dec_units, int32_t *__restrict__ meta,
                                int32_t *bins) {
    if (threadIdx.x < 32) bins[threadIdx.x] = 0;
    __syncthreads();
    const int b = c < 15 ? c : 15;
    if (is_dec) atomicAdd(&bins[b], 1);
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        for (int k = 15; k >= 0; k--) {
            const int v = bins[k];
            bins[16 + k] = run;
            run += v;
        }
        meta[kMetaWorkGU] = 0;
        meta[kMetaWorkDN] = 0;
    }
    __syncthreads();
    if (is_dec) dec_units[atomicAdd(&bins[16 + b], 1)] = e;
}

// Chunk masks: bit (t % 64) of cmask[chunk][e] is set when token t chose expert e. A token that names one expert
// twice is an error (a top-k row holds distinct experts).
__global__ void __launch_bounds__(256) route_mask_kernel(const int32_t *__restrict__ sel, int n, int topk, int E,
                                                         int absent_ok, int32_t *__restrict__ ccnt,
                                                         uint64_t *__restrict__ cmask, int32_t *__restrict__ meta) {
    __shared__ unsigned long long m[1024];
    const int chunk = blockIdx.x, t0 = chunk * kChunk;
    for (int e = threadIdx.x; e < E; e += blockDim.x) m[e] = 0ull;
    __syncthreads();
    const int nt = min(kChunk, n - t0);
    for (int i = threadIdx.x; i < nt * topk; i += blockDim.x) {
        const int e = sel[(size_t)t0 * topk + i];
        if (e < 0 && absent_ok) continue;
        if (e < 0 || e >= E) { set_error(meta, kErrBadExpert); continue; }
        const unsigned long long bit = 1ull << (i / topk);
        if (atomicOr(&m[e], bit) & bit) set_error(meta, kErrBadExpert);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        cmask[(size_t)chunk * E + e] = m[e];
        ccnt[(size_t)chunk * E + e] = __popcll(m[e]);
    }
}

// inclusive block-wide scan of (a, p) over the threads of the block (blockDim.x <= 1024): shuffles inside each warp,
// the warp totals through shared memory (two block barriers). p carries four 16-bit counters side by side.
__device__ __forceinline__ void block_scan2(int &a, uint64_t &p, int *wa, uint64_t *wp) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int ta = __shfl_up_sync(0xffffffffu, a, o);
        const uint64_t tp = __shfl_up_sync(0xffffffffu, p, o);
        if (lane >= o) { a += ta; p += tp; }
    }
    if (lane == 31) { wa[w] = a; wp[w] = p; }
    __syncthreads();
    if (w == 0) {
        int x = lane < nw ? wa[lane] : 0;
        uint64_t y = lane < nw ? wp[lane] : 0ull;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int tx = __shfl_up_sync(0xffffffffu, x, o);
            const uint64_t ty = __shfl_up_sync(0xffffffffu, y, o);
            if (lane >= o) { x += tx; y += ty; }
        }
        if (lane < nw) { wa[lane] = x; wp[lane] = y; }  // inclusive prefix of the warp totals
    }
    __syncthreads();
    if (w > 0) { a += wa[w - 1]; p += wp[w - 1]; }
}

// one block of E threads (E <= 1024)
__global__ void __launch_bounds__(1024) route_scan_kernel(int n, int n_rule, int absent_ok, int topk, int E, int nchunk,
                                                          int gu_items_per_unit,
                                                          int dn_items_per_unit, int gemm_tn,
                                                          int32_t *__restrict__ ccnt, int32_t *__restrict__ cnt,
                                                          int32_t *__restrict__ off, int32_t *__restrict__ units,
                                                          int32_t *__restrict__ dec_units, int32_t *__restrict__ gemm_units,
                                                          int32_t *__restrict__ gemm_tiles, int32_t *__restrict__ upath,
                                                          int32_t *__restrict__ meta) {
    __shared__ int32_t wa[32], bins[32];
    __shared__ uint64_t wp[32];
    const int e = threadIdx.x;
    int run = 0;
    if (e < E)
        for (int c0 = 0; c0 < nchunk; c0 += 32) {  // 32 independent loads in flight, then the running prefix
            int v[32];
#pragma unroll
            for (int j = 0; j < 32; j++) v[j] = c0 + j < nchunk ? ccnt[(size_t)(c0 + j) * E + e] : 0;
#pragma unroll
            for (int j = 0; j < 32; j++) {
                if (c0 + j < nchunk) ccnt[(size_t)(c0 + j) * E + e] = run;
                run += v[j];
            }
        }
    const int c = e < E ? run : 0;
    const int is_unit = c > 0;
    const int is_dec = is_unit && (n_rule <= 8 || c < kGemmMinT);
    const int is_gemm = is_unit && !is_dec;
    const int tiles = is_gemm ? (c + gemm_tn - 1) / gemm_tn : 0;
    // inclusive scans: entries; units | decode units | GEMM units | GEMM tiles (16 bits each: <= 1024 experts,
    // tiles <= n * topk / gemm_tn + E, checked on the host)
    int sc = c;
    uint64_t sp = (uint64_t)is_unit | ((uint64_t)is_dec << 16) | ((uint64_t)is_gemm << 32) | ((uint64_t)tiles << 48);
    block_scan2(sc, sp, wa, wp);
    const int su = (int)(sp & 0xFFFF), sd = (int)((sp >> 16) & 0xFFFF), sg = (int)((sp >> 32) & 0xFFFF),
              stl = (int)(sp >> 48);
    if (e < E) {
        cnt[e] = c;
        off[e] = sc - c;
        if (e == E - 1) off[E] = sc;
        upath[e] = is_gemm;
        if (is_unit) units[su - 1] = e;
        if (is_gemm) {
            gemm_units[sg - 1] = e;
            const int base = stl - tiles;
            for (int i = 0; i < tiles; i++) gemm_tiles[base + i] = ((sg - 1) << 16) | i;
        }
    }
    order_dec_units(is_dec, c, e, dec_units, meta, bins);
    if (e == blockDim.x - 1) {
        const int rerr = meta[kMetaRouterError];  // the router ran before this call's counters were cleared
        if (rerr) set_error(meta, rerr);
        meta[kMetaRouterError] = kErrNone;
        meta[kMetaNUnits] = su;
        meta[kMetaNDec] = sd;
        meta[kMetaNGemm] = sg;
        meta[kMetaDecItemsGU] = sd * gu_items_per_unit;
        meta[kMetaDecItemsDN] = sd * dn_items_per_unit;
        meta[kMetaGemmTilesGU] = stl;
        meta[kMetaGemmTilesDN] = stl;
        if (absent_ok ? sc > n * topk : sc != n * topk) set_error(meta, kErrOverflow);
    }
}

__global__ void __launch_bounds__(256) route_scatter_kernel(const int32_t *__restrict__ sel, const float *__restrict__ w,
                                                            int n, int topk, int E, const int32_t *__restrict__ ccnt,
                                                            const uint64_t *__restrict__ cmask,
                                                            const int32_t *__restrict__ off, int32_t *__restrict__ etok,
                                                            int32_t *__restrict__ eslot, float *__restrict__ ew,
                                                            int32_t *__restrict__ eexp) {
    const int chunk = blockIdx.x, t0 = chunk * kChunk;
    const int nt = min(kChunk, n - t0);
    for (int i = threadIdx.x; i < nt * topk; i += blockDim.x) {
        const int slot = t0 * topk + i, e = sel[slot];
        if (e < 0 || e >= E) continue;
        const int tl = i / topk;
        const uint64_t below = cmask[(size_t)chunk * E + e] & ((1ull << tl) - 1ull);
        const int pos = off[e] + ccnt[(size_t)chunk * E + e] + __popcll(below);
        etok[pos] = t0 + tl;
        eslot[pos] = slot;
        ew[pos] = w[slot];
        eexp[pos] = e;
    }
}

// inclusive scan of v over the block (blockDim.x <= 1024); ws: 32 ints of shared scratch
__device__ __forceinline__ int block_scan_incl(int v, int *ws) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
    }
    if (lane == 31) ws[w] = v;
    __syncthreads();
    if (w == 0) {
        int s = lane < nw ? ws[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += t;
        }
        ws[lane] = s;
    }
    __syncthreads();
    if (w > 0) v += ws[w - 1];
    __syncthreads();
    return v;
}

// Calls of up to 256 token rows: the whole dispatch in one block of E threads (thread e = expert e). Every selection
// sets bit t of its expert's 256-bit token mask, so an expert's count is a popcount, its first-touch key the first
// token's slot, and an entry's place in the expert's token-ordered list the popcount of the lower tokens -- the
// reference's order without any scan over the selections.
constexpr int kSmallRouteMax = 256, kSmallRouteWords = kSmallRouteMax / 64;
__global__ void __launch_bounds__(1024) route_small_kernel(const int32_t *__restrict__ sel, const float *__restrict__ w,
                                                           int n, int topk, int E, int gu_items_per_unit,
                                                           int dn_items_per_unit, int gemm_tn, RouteDev R,
                                                           int32_t *__restrict__ upath, int32_t *__restrict__ eexp) {
    __shared__ unsigned long long em[kSmallRouteWords][1024];
    __shared__ int32_t soff[1024], ws[32], bins[32];
    const int e = threadIdx.x, nk = n * topk, nw = (n + 63) / 64;
    for (int j = 0; j < nw; j++)
        if (e < E) em[j][e] = 0ull;
    if (e == 0) begin_call_errors(R.meta);  // this call's sticky error code starts with the router's
    __syncthreads();
    for (int i = e; i < nk; i += blockDim.x) {
        const int x = sel[i], t = i / topk;
        if (x >= 0 && x < E) {
            const unsigned long long bit = 1ull << (t & 63);
            if (atomicOr(&em[t >> 6][x], bit) & bit) set_error(R.meta, kErrBadExpert);  // one expert named twice
        } else if (x >= E || !R.absent_ok) {
            set_error(R.meta, kErrBadExpert);
        }
    }
    __syncthreads();
    int c = 0, first = 0x7F7F7F7F;
    if (e < E) {
        int t0 = -1;
        for (int j = nw - 1; j >= 0; j--) {
            const unsigned long long m = em[j][e];
            c += __popcll(m);
            if (m) t0 = j * 64 + __ffsll((long long)m) - 1;
        }
        if (t0 >= 0)
            for (int k = 0; k < topk; k++)
                if (sel[t0 * topk + k] == e) first = t0 * topk + k;
    }
    const int is_unit = c > 0, is_dec = is_unit && (R.n_rule <= 8 || c < kGemmMinT), is_gemm = is_unit && !is_dec;
    const int tiles = is_gemm ? (c + gemm_tn - 1) / gemm_tn : 0;
    // two scans: counts (12 bits: at most 256 x 16 entries) | tiles, units | decode | prefill counts (10 bits each)
    const int sa = block_scan_incl(c | (tiles << 12), ws);
    const int sb = block_scan_incl(is_unit | (is_dec << 10) | (is_gemm << 20), ws);
    const int c_incl = sa & 4095, t_incl = sa >> 12;
    const int u_incl = sb & 1023, d_incl = (sb >> 10) & 1023, g_incl = sb >> 20;
    if (e < E) {
        const int off = c_incl - c;
        soff[e] = off;
        R.cnt[e] = c;
        R.off[e] = off;
        R.first[e] = first;
        if (e == E - 1) R.off[E] = c_incl;
        upath[e] = is_gemm;
        if (is_unit) R.units[u_incl - 1] = e;
        if (is_gemm) {
            R.gemm_units[g_incl - 1] = e;
            for (int i = 0; i < tiles; i++) R.gemm_tiles[t_incl - tiles + i] = ((g_incl - 1) << 16) | i;
        }
    }
    order_dec_units(is_dec, c, e, R.dec_units, R.meta, bins);
    if (e == blockDim.x - 1) {
        R.meta[kMetaNUnits] = u_incl;
        R.meta[kMetaNDec] = d_incl;
        R.meta[kMetaNGemm] = g_incl;
        R.meta[kMetaDecItemsGU] = d_incl * gu_items_per_unit;
        R.meta[kMetaDecItemsDN] = d_incl * dn_items_per_unit;
        R.meta[kMetaGemmTilesGU] = t_incl;
        R.meta[kMetaGemmTilesDN] = t_incl;
        if (R.absent_ok ? c_incl > nk : c_incl != nk) set_error(R.meta, kErrOverflow);
    }
    __syncthreads();
    for (int i = e; i < nk; i += blockDim.x) {
        const int x = sel[i], t = i / topk;
        if (x < 0 || x >= E) continue;
        int pos = soff[x] + __popcll(em[t >> 6][x] & ((1ull << (t & 63)) - 1ull));
        for (int j = 0; j < (t >> 6); j++) pos += __popcll(em[j][x]);
        R.etok[pos] = t;
        R.eslot[pos] = i;
        R.ew[pos] = w[i];
        eexp[pos] = x;
    }
}

// Small calls (n <= 64) in one cluster of kRouteCluster blocks of 1024 threads. Softmax + top-k run one warp per
// token, the tokens spread over the cluster's SMs (token t on block t % kRouteCluster), each warp writing its token's
// selections straight into block 0's shared memory (distributed shared memory). After the cluster barrier block 0
// alone builds the dispatch lists. Each expert keeps a 64-bit mask of the tokens that chose it, so its count is a
// popcount, its first-touch key is the first token's slot, and an entry's rank in the expert's token-ordered list is
// the popcount of the lower tokens -- the reference's order, without a scan over earlier entries.
constexpr int kFusedMax = 64, kRouteCluster = 8;
__global__ void __cluster_dims__(kRouteCluster, 1, 1) __launch_bounds__(1024)
    route_fused_kernel(const float *__restrict__ logits, int n, int E, int topk, float *__restrict__ probs_out,
                       int gu_items_per_unit, int dn_items_per_unit, int gemm_tn, RouteDev R,
                       int32_t *__restrict__ upath, int32_t *__restrict__ eexp) {
    extern __shared__ __align__(16) float ex[];  // [32][E] softmax scratch
    __shared__ unsigned long long emask[1024];
    __shared__ int32_t ss[kFusedMax * kMaxTopK], soff[1024], ws[32], bins[32];
    __shared__ float sw[kFusedMax * kMaxTopK];
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int tid = threadIdx.x, warp = tid >> 5, nk = n * topk;
    int32_t *ss0 = cluster.map_shared_rank(ss, 0);
    float *sw0 = cluster.map_shared_rank(sw, 0);
    for (int t = rank + kRouteCluster * warp; t < n; t += kRouteCluster * (blockDim.x >> 5))
        softmax_topk_warp(logits + (size_t)t * E, E, topk, ex + (size_t)warp * E,
                          probs_out ? probs_out + (size_t)t * E : nullptr, ss0 + t * topk, sw0 + t * topk);
    if (rank == 0) {
        if (tid == 0) begin_call_errors(R.meta);
        for (int e = tid; e < E; e += blockDim.x) emask[e] = 0ull;
    }
    cluster.sync();  // every token's selections are in block 0 (release / acquire at cluster scope)
    if (rank != 0) return;
    int e_i = -1;
    if (tid < nk) {
        e_i = ss[tid];
        R.sel[tid] = e_i;
        R.w[tid] = sw[tid];
        if (e_i < 0 || e_i >= E) { set_error(R.meta, kErrBadExpert); e_i = -1; }
        else atomicOr(&emask[e_i], 1ull << (tid / topk));
    }
    __syncthreads();
    const int e = tid;
    const unsigned long long mask = e < E ? emask[e] : 0ull;
    const int c = __popcll(mask);
    int first = 0x7F7F7F7F;
    if (c) {
        const int t0 = __ffsll((long long)mask) - 1;
        for (int k = 0; k < topk; k++)
            if (ss[t0 * topk + k] == e) first = t0 * topk + k;
    }
    const int is_unit = c > 0, is_dec = is_unit && (n <= 8 || c < kGemmMinT), is_gemm = is_unit && !is_dec;
    const int tiles = is_gemm ? (c + gemm_tn - 1) / gemm_tn : 0;
    // two scans: counts | tiles (11 bits each), units | decode | prefill counts (10 bits each)
    const int sa = block_scan_incl(c | (tiles << 11), ws);
    const int sb = block_scan_incl(is_unit | (is_dec << 10) | (is_gemm << 20), ws);
    const int c_incl = sa & 2047, t_incl = sa >> 11;
    const int u_incl = sb & 1023, d_incl = (sb >> 10) & 1023, g_incl = sb >> 20;
    if (e < E) {
        const int off = c_incl - c;
        soff[e] = off;
        R.cnt[e] = c;
        R.off[e] = off;
        R.first[e] = first;
        if (e == E - 1) R.off[E] = c_incl;
        upath[e] = is_gemm;
        if (is_unit) R.units[u_incl - 1] = e;
        if (is_gemm) {
            R.gemm_units[g_incl - 1] = e;
            for (int i = 0; i < tiles; i++) R.gemm_tiles[t_incl - tiles + i] = ((g_incl - 1) << 16) | i;
        }
    }
    order_dec_units(is_dec, c, e, R.dec_units, R.meta, bins);
    if (tid == blockDim.x - 1) {
        R.meta[kMetaNUnits] = u_incl;
        R.meta[kMetaNDec] = d_incl;
        R.meta[kMetaNGemm] = g_incl;
        R.meta[kMetaDecItemsGU] = d_incl * gu_items_per_unit;
        R.meta[kMetaDecItemsDN] = d_incl * dn_items_per_unit;
        R.meta[kMetaGemmTilesGU] = t_incl;
        R.meta[kMetaGemmTilesDN] = t_incl;
        if (c_incl != nk) set_error(R.meta, kErrOverflow);
    }
    __syncthreads();
    if (tid < nk && e_i >= 0) {
        const int t = tid / topk;
        const int pos = soff[e_i] + __popcll(emask[e_i] & ((1ull << t) - 1ull));
        R.etok[pos] = t;
        R.eslot[pos] = tid;
        R.ew[pos] = sw[tid];
        eexp[pos] = e_i;
    }
}

// The shared expert as a one-unit dispatch list (src/model_fwd.c:1047-1068): expert 0 of its own pool takes every
// token t of the call at entry t (output slot t, weight 1: the gate is applied by shared_add_kernel); its numeric path
// is the lin_mm rule on the whole batch, decode below GEMM_MIN_T tokens (src/model_fwd.c:234).
__global__ void shared_route_kernel(int n, int gemm, int gu_items_per_unit, int dn_items_per_unit, int gemm_tn,
                                   RouteDev R, int32_t *__restrict__ upath, int32_t *__restrict__ eexp) {
    const int tiles = gemm ? (n + gemm_tn - 1) / gemm_tn : 0;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        R.cnt[0] = n;
        R.off[0] = 0;
        R.off[1] = n;
        R.first[0] = 0;
        upath[0] = gemm;
        R.units[0] = 0;
        if (gemm) R.gemm_units[0] = 0;
        else R.dec_units[0] = 0;
        R.meta[kMetaNUnits] = 1;
        R.meta[kMetaNDec] = !gemm;
        R.meta[kMetaNGemm] = gemm;
        R.meta[kMetaDecItemsGU] = gemm ? 0 : gu_items_per_unit;
        R.meta[kMetaDecItemsDN] = gemm ? 0 : dn_items_per_unit;
        R.meta[kMetaGemmTilesGU] = tiles;
        R.meta[kMetaGemmTilesDN] = tiles;
        R.meta[kMetaError] = kErrNone;
        R.meta[kMetaWorkGU] = 0;
        R.meta[kMetaWorkDN] = 0;
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        R.etok[i] = i;
        R.eslot[i] = i;
        R.ew[i] = 1.0f;
        eexp[i] = 0;
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < tiles; i += gridDim.x * blockDim.x) R.gemm_tiles[i] = i;
}

int launch_shared_route(const RouteDev &R, int n, int gemm, int gu_items_per_unit, int dn_items_per_unit, int gemm_tn,
                        int32_t *upath, int32_t *eexp, cudaStream_t st) {
    shared_route_kernel<<<(n + 255) / 256, 256, 0, st>>>(n, gemm, gu_items_per_unit, dn_items_per_unit, gemm_tn, R, upath,
                                                         eexp);
    return 1;
}

int launch_route_fused(const RouteDev &R, const float *logits, float *probs, int gu_items_per_unit,
                       int dn_items_per_unit, int gemm_tn, int32_t *upath, int32_t *eexp, cudaStream_t st) {
    if (R.n > kFusedMax || R.E > 1024 || R.n * R.topk > kFusedMax * kMaxTopK) return -1;
    const size_t smem = (size_t)32 * R.E * sizeof(float);
    route_fused_kernel<<<kRouteCluster, 1024, smem, st>>>(logits, R.n, R.E, R.topk, probs, gu_items_per_unit,
                                                          dn_items_per_unit, gemm_tn, R, upath, eexp);
    return 1;
}

void route_set_attributes(int E) {
    cudaFuncSetAttribute(route_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 32 * E * (int)sizeof(float));
}

int launch_route(const RouteDev &R, int gu_items_per_unit, int dn_items_per_unit, int gemm_tn,
                 int32_t *upath, int32_t *eexp, cudaStream_t st) {
    const int n = R.n, topk = R.topk, E = R.E;
    if (n <= kSmallRouteMax && n * topk < 4096 && E < 1024) {  // the packed scans' field widths
        const int threads = (E + 31) / 32 * 32;
        route_small_kernel<<<1, threads, 0, st>>>(R.sel, R.w, n, topk, E, gu_items_per_unit, dn_items_per_unit, gemm_tn,
                                                  R, upath, eexp);
        return 1;
    }
    const int nchunk = route_chunks(n);
    cudaMemsetAsync(R.meta, 0, sizeof(int32_t) * kMetaRouterError, st);  // the router's word is folded in by route_scan
    route_mask_kernel<<<nchunk, 256, 0, st>>>(R.sel, n, topk, E, R.absent_ok, R.ccnt, R.cmask, R.meta);
    const int threads = (E + 31) / 32 * 32;
    route_scan_kernel<<<1, threads, 0, st>>>(n, R.n_rule, R.absent_ok, topk, E, nchunk, gu_items_per_unit, dn_items_per_unit,
                                             gemm_tn, R.ccnt, R.cnt, R.off, R.units, R.dec_units, R.gemm_units,
                                             R.gemm_tiles, upath, R.meta);
    route_scatter_kernel<<<nchunk, 256, 0, st>>>(R.sel, R.w, n, topk, E, R.ccnt, R.cmask, R.off, R.etok, R.eslot, R.ew,
                                                 eexp);
    return 3;
}

int route_chunks(int n) { return (n + kChunk - 1) / kChunk; }

}  // namespace inzg
