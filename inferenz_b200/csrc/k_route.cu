// k_route.cu -- token -> expert dispatch lists on the device.
//
// The reference builds, per token in order, "units" = per-expert lists of (token, slot = t*topk + k, weight)
// (src/model_fwd.c:1001-1031). The lists here hold the same entries, sorted by expert and, within an expert, by
// token -- the order the reference appends them -- without atomics on positions, so the result is deterministic:
//   route_count   per 32-token chunk (one warp): chunk-local rank of every (t, k) among the chunk's tokens that chose
//                 the same expert, per-chunk counts, first-touch key per expert
//   route_scan    one block: per-expert prefix over chunks, counts, offsets, expert lists and the per-expert numeric
//                 path (decode numerics when n <= 8 or the expert has < GEMM_MIN_T tokens, src/model_fwd.c:229-249,
//                 1070), work counts for the expert kernels
//   route_scatter per chunk: entry position = off[e] + chunk prefix + rank
#include "inzg_internal.h"
#include "k_launch.h"

namespace inzg {

constexpr int kChunk = 32;

// rank of (lane's token, k) among the earlier tokens of the chunk that selected the same expert
__device__ __forceinline__ int chunk_rank(const int32_t (*s)[kMaxTopK], int topk, int t, int e) {
    int r = 0;
    for (int u = 0; u < t; u++)
        for (int k = 0; k < topk; k++) r += s[u][k] == e;
    return r;
}

__global__ void __launch_bounds__(128) route_count_kernel(const int32_t *__restrict__ sel, int n, int topk, int E,
                                                          int32_t *__restrict__ ccnt, int32_t *__restrict__ first,
                                                          int32_t *__restrict__ meta) {
    __shared__ int32_t s[4][kChunk][kMaxTopK];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int chunk = blockIdx.x * 4 + warp;
    const int t = chunk * kChunk + lane;
    const bool valid = t < n;
    for (int k = 0; k < topk; k++) s[warp][lane][k] = valid ? sel[(size_t)t * topk + k] : -1;
    __syncwarp();
    if (chunk * kChunk >= n) return;
    if (!valid) return;
    for (int k = 0; k < topk; k++) {
        const int e = s[warp][lane][k];
        if (e < 0 || e >= E) { set_error(meta, kErrBadExpert); continue; }
        atomicAdd(&ccnt[(size_t)chunk * E + e], 1);
        atomicMin(&first[e], t * topk + k);
    }
}

// one block of E threads (E <= 1024)
__global__ void __launch_bounds__(1024) route_scan_kernel(int n, int topk, int E, int nchunk, int gu_items_per_unit,
                                                          int dn_items_per_unit, int gemm_tn,
                                                          int32_t *__restrict__ ccnt, int32_t *__restrict__ cnt,
                                                          int32_t *__restrict__ off, int32_t *__restrict__ units,
                                                          int32_t *__restrict__ dec_units, int32_t *__restrict__ gemm_units,
                                                          int32_t *__restrict__ gemm_tiles, int32_t *__restrict__ upath,
                                                          int32_t *__restrict__ meta) {
    __shared__ int32_t sc[1024], su[1024], sd[1024], sg[1024], st[1024];
    const int e = threadIdx.x;
    int run = 0;
    if (e < E)
        for (int c = 0; c < nchunk; c++) {
            const int v = ccnt[(size_t)c * E + e];
            ccnt[(size_t)c * E + e] = run;
            run += v;
        }
    const int c = e < E ? run : 0;
    const int is_unit = c > 0;
    const int is_dec = is_unit && (n <= 8 || c < kGemmMinT);
    const int is_gemm = is_unit && !is_dec;
    const int tiles = is_gemm ? (c + gemm_tn - 1) / gemm_tn : 0;
    sc[e] = c; su[e] = is_unit; sd[e] = is_dec; sg[e] = is_gemm; st[e] = tiles;
    __syncthreads();
    // inclusive Hillis-Steele scans over the five arrays
    for (int o = 1; o < blockDim.x; o <<= 1) {
        int a = 0, b = 0, d = 0, g = 0, h = 0;
        if (e >= o) { a = sc[e - o]; b = su[e - o]; d = sd[e - o]; g = sg[e - o]; h = st[e - o]; }
        __syncthreads();
        if (e >= o) { sc[e] += a; su[e] += b; sd[e] += d; sg[e] += g; st[e] += h; }
        __syncthreads();
    }
    if (e < E) {
        cnt[e] = c;
        off[e] = sc[e] - c;
        if (e == E - 1) off[E] = sc[e];
        upath[e] = is_gemm;
        if (is_unit) units[su[e] - 1] = e;
        if (is_dec) dec_units[sd[e] - 1] = e;
        if (is_gemm) {
            gemm_units[sg[e] - 1] = e;
            const int base = st[e] - tiles;
            for (int i = 0; i < tiles; i++) gemm_tiles[base + i] = ((sg[e] - 1) << 16) | i;
        }
    }
    if (e == blockDim.x - 1) {
        meta[kMetaNUnits] = su[e];
        meta[kMetaNDec] = sd[e];
        meta[kMetaNGemm] = sg[e];
        meta[kMetaDecItemsGU] = sd[e] * gu_items_per_unit;
        meta[kMetaDecItemsDN] = sd[e] * dn_items_per_unit;
        meta[kMetaGemmTilesGU] = st[e];
        meta[kMetaGemmTilesDN] = st[e];
        if (sc[e] != n * topk) set_error(meta, kErrOverflow);
    }
}

__global__ void __launch_bounds__(128) route_scatter_kernel(const int32_t *__restrict__ sel, const float *__restrict__ w,
                                                            int n, int topk, int E, const int32_t *__restrict__ ccnt,
                                                            const int32_t *__restrict__ off, int32_t *__restrict__ etok,
                                                            int32_t *__restrict__ eslot, float *__restrict__ ew,
                                                            int32_t *__restrict__ eexp) {
    __shared__ int32_t s[4][kChunk][kMaxTopK];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int chunk = blockIdx.x * 4 + warp;
    const int t = chunk * kChunk + lane;
    const bool valid = t < n;
    for (int k = 0; k < topk; k++) s[warp][lane][k] = valid ? sel[(size_t)t * topk + k] : -1;
    __syncwarp();
    if (!valid) return;
    for (int k = 0; k < topk; k++) {
        const int e = s[warp][lane][k];
        if (e < 0 || e >= E) continue;
        const int pos = off[e] + ccnt[(size_t)chunk * E + e] + chunk_rank(s[warp], topk, lane, e);
        etok[pos] = t;
        eslot[pos] = t * topk + k;
        ew[pos] = w[(size_t)t * topk + k];
        eexp[pos] = e;
    }
}

// Small calls (n <= 64): the whole dispatch in one block of E threads, thread e = expert e. Counting, the
// first-touch key and the token-ordered scatter read the call's n * topk selections from shared memory.
constexpr int kSmallRouteMax = 64;
__global__ void __launch_bounds__(1024) route_small_kernel(const int32_t *__restrict__ sel, const float *__restrict__ w,
                                                           int n, int topk, int E, int gu_items_per_unit,
                                                           int dn_items_per_unit, int gemm_tn, RouteDev R,
                                                           int32_t *__restrict__ upath, int32_t *__restrict__ eexp) {
    __shared__ int32_t ss[kSmallRouteMax * kMaxTopK];
    __shared__ int32_t sc[1024], su[1024], sd[1024], sg[1024], st[1024];
    const int e = threadIdx.x, nk = n * topk;
    for (int i = e; i < nk; i += blockDim.x) ss[i] = sel[i];
    if (e == 0) R.meta[kMetaError] = kErrNone;  // this call's sticky error code starts clear
    __syncthreads();
    int c = 0, first = 0x7F7F7F7F;
    if (e < E)
        for (int i = 0; i < nk; i++)
            if (ss[i] == e) { c++; first = min(first, i); }
    if (e == 0)
        for (int i = 0; i < nk; i++)
            if (ss[i] < 0 || ss[i] >= E) set_error(R.meta, kErrBadExpert);
    const int is_unit = c > 0;
    const int is_dec = is_unit && (n <= 8 || c < kGemmMinT);
    const int is_gemm = is_unit && !is_dec;
    const int tiles = is_gemm ? (c + gemm_tn - 1) / gemm_tn : 0;
    sc[e] = c; su[e] = is_unit; sd[e] = is_dec; sg[e] = is_gemm; st[e] = tiles;
    __syncthreads();
    for (int o = 1; o < blockDim.x; o <<= 1) {
        int a = 0, b = 0, d = 0, g = 0, h = 0;
        if (e >= o) { a = sc[e - o]; b = su[e - o]; d = sd[e - o]; g = sg[e - o]; h = st[e - o]; }
        __syncthreads();
        if (e >= o) { sc[e] += a; su[e] += b; sd[e] += d; sg[e] += g; st[e] += h; }
        __syncthreads();
    }
    if (e < E) {
        const int off = sc[e] - c;
        R.cnt[e] = c;
        R.off[e] = off;
        R.first[e] = first;
        if (e == E - 1) R.off[E] = sc[e];
        upath[e] = is_gemm;
        if (is_unit) R.units[su[e] - 1] = e;
        if (is_dec) R.dec_units[sd[e] - 1] = e;
        if (is_gemm) {
            R.gemm_units[sg[e] - 1] = e;
            const int base = st[e] - tiles;
            for (int i = 0; i < tiles; i++) R.gemm_tiles[base + i] = ((sg[e] - 1) << 16) | i;
        }
        int pos = off;  // scan in (token, k) order: tokens ascending inside the expert's list
        for (int i = 0; i < nk && pos < off + c; i++)
            if (ss[i] == e) {
                R.etok[pos] = i / topk;
                R.eslot[pos] = i;
                R.ew[pos] = w[i];
                eexp[pos] = e;
                pos++;
            }
    }
    if (e == blockDim.x - 1) {
        R.meta[kMetaNUnits] = su[e];
        R.meta[kMetaNDec] = sd[e];
        R.meta[kMetaNGemm] = sg[e];
        R.meta[kMetaDecItemsGU] = sd[e] * gu_items_per_unit;
        R.meta[kMetaDecItemsDN] = sd[e] * dn_items_per_unit;
        R.meta[kMetaGemmTilesGU] = st[e];
        R.meta[kMetaGemmTilesDN] = st[e];
        if (sc[e] != nk) set_error(R.meta, kErrOverflow);
    }
}

int launch_route(const RouteDev &R, int nchunk, int gu_items_per_unit, int dn_items_per_unit, int gemm_tn,
                 int32_t *upath, int32_t *eexp, cudaStream_t st) {
    const int n = R.n, topk = R.topk, E = R.E;
    if (n <= kSmallRouteMax) {
        const int threads = (E + 31) / 32 * 32;
        route_small_kernel<<<1, threads, 0, st>>>(R.sel, R.w, n, topk, E, gu_items_per_unit, dn_items_per_unit, gemm_tn,
                                                  R, upath, eexp);
        return 1;
    }
    cudaMemsetAsync(R.ccnt, 0, sizeof(int32_t) * (size_t)nchunk * E, st);
    cudaMemsetAsync(R.first, 0x7F, sizeof(int32_t) * (size_t)E, st);
    cudaMemsetAsync(R.meta, 0, sizeof(int32_t) * 16, st);
    const int blocks = (nchunk + 3) / 4;
    route_count_kernel<<<blocks, 128, 0, st>>>(R.sel, n, topk, E, R.ccnt, R.first, R.meta);
    const int threads = (E + 31) / 32 * 32;
    route_scan_kernel<<<1, threads, 0, st>>>(n, topk, E, nchunk, gu_items_per_unit, dn_items_per_unit, gemm_tn, R.ccnt,
                                             R.cnt, R.off, R.units, R.dec_units, R.gemm_units, R.gemm_tiles, upath, R.meta);
    route_scatter_kernel<<<blocks, 128, 0, st>>>(R.sel, R.w, n, topk, E, R.ccnt, R.off, R.etok, R.eslot, R.ew, eexp);
    return 3;
}

}  // namespace inzg
