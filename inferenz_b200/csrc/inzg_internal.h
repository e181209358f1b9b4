// inzg_internal.h -- shared definitions of the libinzg CUDA implementation (device layouts, work lists, helpers).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/inzg.h"

namespace inzg {

constexpr int kGroup = 64;     // weights per quantization group (src/quant.h:21)
constexpr int kLutBias = 64;   // LUT levels are stored biased by 64 (src/quant.h:22)
constexpr int kKB = 256;       // prefill activation block (src/quant.h:152)
constexpr int kGemmMinT = 12;  // experts with >= 12 tokens use the prefill numerics (src/model_fwd.c:126)
constexpr int kMaxTopK = 16;

// ---------------------------------------------------------------------------------------------------------------
// Tile layout of one expert matrix (M rows x K cols, ng = K/64 groups), matched to the fragments of the int8 MMA
// (mma.m16n8k32: thread (r = lane/4, t = lane%4) holds A[r][4t..4t+3], A[r+8][4t..], A[r][16+4t..], A[r+8][16+4t..]).
// The decode GEMV runs two MMAs per group whose K = 32 holds 4 of the reference's 8 VNNI lanes each (lane l covers
// weights 4l..4l+3 and 32+4l..32+4l+3), so thread (r, t) of MMA h needs lane 4h + t/2 (registers a0, a1) and lane
// 4h + 2 + t/2 (a2, a3), part t%2 of each (part 0: weights 4l.., part 1: weights 32+4l..).
// Weights: [M/16 row tiles][ng][32 lanes][wb bytes].
//   Q4L (wb = 16): 4 words per lane, word 2h + s (s = 0: row r, 1: row r+8): bits 0-15 the 4 nibble selectors of
//   registers a0/a1 of MMA h, bits 16-31 those of a2/a3.
//   Q8G (wb = 32): [h][32 lanes][4 words a0 a1 a2 a3], each word 4 raw bytes.
// Scales: [M/16][gd = ceil(ng/4)][8 rows r][4 groups][2] fp16 -- (d[r][g], d[r+8][g]) pairs, zero past ng.
// A warp reads one 16-row x 64-column tile with one 512-byte (Q4L) or two (Q8G) conflict-free shared-memory loads.
// ---------------------------------------------------------------------------------------------------------------
struct MatLayout {
    int rows, cols, ng, gd, wb;
    uint64_t q_off, d_off;  // byte offsets of the weight and scale regions inside the expert's slab
};

// Per-layer, per-matrix metadata shared by all experts of the layer (rotation) plus per-expert LUTs.
struct LayerDev {
    int type;                 // INZG_T_Q4L / INZG_T_Q8G
    int H, FF, E;
    MatLayout gu, dn;         // identical geometry for every expert
    uint64_t slab_bytes;      // bytes per expert in the pool (gu region + dn region)
    int gu_rot, dn_rot;
    uint32_t gu_seed, dn_seed;
    const uint8_t *pool;      // [E][slab_bytes]
    const uint8_t *luts;      // [E][2][16]: biased levels of gate|up, down
    const uint4 *router;      // repacked F16 router, see router layout in k_router.cu
    // prefill path: requantized int8 weights (K-major rows) and per-(row, 256-block) scales
    int8_t *w8_gu, *w8_dn;    // [E][2FF][H], [E][H][FF]
    float *ws_gu, *ws_dn;     // [E][2FF][H/256], [E][H][ceil(FF/256)]
};

// The expert-parallel exchange (k_ep.cu): every rank's exposed buffer, as seen from this rank (peer pointers).
constexpr int kEpMaxRanks = 8;
struct EpPeers {
    int rank, world, cap, topk, hidden, e_per;
    int32_t *rsel[kEpMaxRanks];  // [world][cap][topk] local expert of each received slot, -1 if not owned there
    float *rw[kEpMaxRanks];      // [world][cap][topk] routing weights
    float *rx[kEpMaxRanks];      // [world][cap][hidden] received rows
    float *out[kEpMaxRanks];     // [world * cap][topk][hidden] the rank's expert outputs for every row it received
    uint32_t *flags[kEpMaxRanks];  // [3][world] dispatch / outputs-ready / rendezvous epochs written by each peer
};

// Routing products of one forward call (device).
struct RouteDev {
    int n, topk, E;
    int n_rule;          // batch size of the decode-numerics rule (n <= 8: every expert decodes): n, or the whole
                         // batch across ranks when this call holds one rank's share of an expert-parallel batch
    int absent_ok;       // entries with a negative expert id are not on this rank (expert parallel), not errors
    int32_t *sel;        // [n][topk]
    float *w;            // [n][topk]  renormalised
    int32_t *cnt;        // [E] tokens per expert
    int32_t *off;        // [E+1] exclusive prefix of cnt (entries sorted by expert, then token)
    int32_t *first;      // [E] first slot t*topk+k that chose the expert (first-touch order key)
    int32_t *etok;       // [n*topk] token of each entry
    int32_t *eslot;      // [n*topk] slot t*topk+k of each entry
    float *ew;           // [n*topk] weight of each entry
    int32_t *ccnt;       // [nchunk][E] per-64-token-chunk counts, then their exclusive prefix per expert
    uint64_t *cmask;     // [nchunk][E] per-chunk token masks: bit t % 64 set when token t chose the expert
    int32_t *units;      // [E] experts with cnt > 0, ascending
    int32_t *meta;       // [16] counters: 0 nunits, 1 n_dec_units, 2 n_gemm_units, 3 n_dec_items_gu, 4 n_dec_items_dn,
                         //      5 n_gemm_tiles_gu, 6 n_gemm_tiles_dn, 7 device error code, 8/9 decode GEMV work
                         //      queues (gate|up, down), 10 router error code
    int32_t *dec_units;  // [E] decode-path experts, most tokens first
    int32_t *gemm_units; // [E] prefill-path experts
    int32_t *gemm_tiles; // [E * tiles] (unit index << 16 | token tile) for the GEMM path
};

constexpr int kMetaNUnits = 0, kMetaNDec = 1, kMetaNGemm = 2, kMetaDecItemsGU = 3, kMetaDecItemsDN = 4,
              kMetaGemmTilesGU = 5, kMetaGemmTilesDN = 6, kMetaError = 7, kMetaWorkGU = 8, kMetaWorkDN = 9,
              kMetaRouterError = 10;  // the router's own error word, folded into kMetaError by the route kernel

// device error codes (sticky, first one wins)
constexpr int kErrNone = 0, kErrBadExpert = 1, kErrBadSlot = 2, kErrOverflow = 3, kErrTimeout = 4;

// ---------------------------------------------------------------------------------------------------------------
// IEEE helpers with explicit rounding (no contraction, no fast math)
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ float hsum8_tree(const float a[8]) {
    float b0 = __fadd_rn(a[0], a[4]), b1 = __fadd_rn(a[1], a[5]), b2 = __fadd_rn(a[2], a[6]), b3 = __fadd_rn(a[3], a[7]);
    return __fadd_rn(__fadd_rn(b0, b2), __fadd_rn(b1, b3));
}

// The reference's hsum8 over 8 consecutive lanes of a warp (lane & 7 = accumulator lane): result valid in all 8.
__device__ __forceinline__ float hsum8_lanes(float v) {
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));  // (a0+a4) (a1+a5) (a2+a6) (a3+a7)
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));  // ((a0+a4)+(a2+a6)) ((a1+a5)+(a3+a7))
    return __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
}

__device__ __forceinline__ uint32_t rot_sign_bit(uint32_t seed, uint32_t i) {
    uint32_t h = (i + 1) * 0x9E3779B1u ^ seed;
    h ^= h >> 15; h *= 0x2C1B3C6Du; h ^= h >> 12; h *= 0x297A2D39u; h ^= h >> 15;
    return h & 1u;
}

__device__ __forceinline__ int dp4a_ss(int a, int b, int c) { return __dp4a(a, b, c); }
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ void set_error(int32_t *meta, int code) { atomicCAS(&meta[kMetaError], 0, code); }

// first device error of this call: what the router recorded (it runs before the route kernel clears the word)
__device__ __forceinline__ void begin_call_errors(int32_t *meta) {
    meta[kMetaError] = meta[kMetaRouterError];
    meta[kMetaRouterError] = kErrNone;
}

}  // namespace inzg
