// k_gemm_tc.cu -- prefill-path grouped GEMM on the 5th-generation tensor cores (tcgen05.mma kind::i8), sm_100a.
//
// Numerics: the reference's prefill GEMM (inz_gemm_rows, src/quant.c:1615-1668). Per (row, 256-block) the weights are
// the reference's requantized int8 (materialised once per layer at upload, k_pool.cu) with block scale ws; the token
// is int8 per 256-block with scale xs (src/quant.c:1407-1429). The integer dot of one block is exact in int32 (the
// tensor core accumulates s8 x s8 in s32), and the output is f = fma((float)dot_b, ws_b * xs_b, f) over the blocks
// in order -- the reference's own float sequence, so a GEMM-path expert output is the reference's bits.
//
// Work item: 128 weight rows x 128 tokens of one expert; K in 128-byte halves (two per 256-block). Persistent: one CTA
// per SM walks the items blockIdx.x, blockIdx.x + gridDim.x, ... (row blocks of one token tile are consecutive, so
// neighbouring SMs share the tile's activations in L2); every role counts stages and accumulators across items, so
// the next item's loads and MMAs overlap the previous item's epilogue.
//   warp 0      TMA producer: A (weights, [E*rows][K] int8) and B (tokens, [entries][K] int8) boxes of 128 x 128 bytes,
//               128-byte swizzle, into a 4-stage ring (no multicast)
//   warp 1      allocates all 512 TMEM columns once (four 128-column int32 accumulators, so the MMAs can run up to
//               three 256-blocks ahead of the epilogue's per-block fold), one lane issues 4 MMAs (K = 32) per half;
//               tcgen05.commit frees the smem stage and, after a block's 8 MMAs, hands the accumulator over
//   warps 2-9   epilogue: thread = (weight row = TMEM lane, half of the tile's tokens); per block tcgen05.ld of its 64
//               int32 dots, the per-block FMA into 64 fp32 registers (packed f32x2 add / mul / fma, two tokens per
//               instruction), then the accumulator is refilled and released; at the item's end its outputs are
//               written. Each accumulator starts at the bits of 1.5 * 2^23 (tcgen05.st after every read), so a block's
//               int32 dot reads as the float 12582912 + dot and one add of -12582912 gives (float)dot exactly
//               (|dot| <= 256*128*127 < 2^22), in place of a quarter-rate conversion.
// Every mbarrier wait is bounded; on expiry the CTA records an error (INZG_TIMEOUT to the host), drains what it
// issued, frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "inzg_internal.h"
#include "k_launch.h"
#include "k_async.cuh"

namespace inzg {

constexpr int TBM = 128, TBN = 128, TBK = 128, TSTAGES = 4;
constexpr int kEpiWarps = 8, kEpiThreads = kEpiWarps * 32, kHalfN = TBN / 2;  // two epilogue warps per TMEM quadrant
constexpr int kThreads = 64 + kEpiThreads;
constexpr int kMagicI = 0x4B400000;  // 1.5 * 2^23 as a float: kMagicI + x reads as 12582912 + x for |x| < 2^22
constexpr int kStageBytes = (TBM + TBN) * TBK;  // 32 KiB
// more than half of an SM's shared memory per CTA, so a CTA is alone on its SM with all 512 TMEM columns
static_assert(TSTAGES * kStageBytes > 116 * 1024, "one gemm_tc CTA per SM");
constexpr int kMaxKB = 10;                      // 256-blocks of K: up to 2560, the reference model's width

struct TcShared {
    uint64_t full[TSTAGES], empty[TSTAGES], acc_full[4], acc_empty[4], drain;
    uint64_t xs_full[2];               // every epilogue thread has written the item's xs / oslot / ow [parity]
    uint64_t xs_empty[2];              // every epilogue thread has finished the item that used buffer [parity]
    uint32_t tmem_base;
    int abort, never;                  // never: drains ignore the abort flag
    alignas(16) float xs[2][kMaxKB][TBN];  // token block scales per item parity, [block][token] (K <= 2560)
    int oslot[2][TBN];                 // down matrix: each token's output slot and routing weight, per item parity
    float ow[2][TBN];
};



// K-major operand in shared memory, 128-byte swizzle: 8-row atoms of 1024 bytes, SBO = 1024 B, LBO unused (1)
__device__ __forceinline__ uint64_t umma_desc(const void *smem) {
    const uint64_t a = smem_u32(smem);
    return ((a & 0x3FFFFull) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, int (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 consecutive columns of this warp's 32 TMEM lanes set to `c`
__device__ __forceinline__ void tmem_fill32(uint32_t taddr, int c) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
        "%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr), "r"(c)
        : "memory");
}

// instruction descriptor: s32 accumulate, s8 x s8, both K-major, N = TBN, M = TBM
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TBN >> 3) << 17) | ((uint32_t)(TBM >> 4) << 24);

// KIND 0: gate|up, out = GU[entry][row]; KIND 1: down, out = moe_out[slot][row] = w * f.
template <int KIND>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap mapA,
                                                         const __grid_constant__ CUtensorMap mapB,
                                                         const float *__restrict__ wsc, int rows, int K,
                                                         RouteDev R, const float *__restrict__ xs_e,
                                                         float *__restrict__ out, int out_ld, int meta_tiles) {
    extern __shared__ __align__(1024) uint8_t dyn[];
    const int nrb = rows / TBM;
    const int nitems = R.meta[meta_tiles] * nrb;
    if ((int)blockIdx.x >= nitems) return;  // uniform over the CTA: nothing allocated yet
    const int nkh = K / TBK, nkb = (K + kKB - 1) / kKB;
    uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dyn) + 1023) & ~uintptr_t(1023));
    TcShared &S = *reinterpret_cast<TcShared *>(ring + TSTAGES * kStageBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    volatile int *abort = &S.abort;
    volatile int *never = &S.never;

    if (threadIdx.x == 0) {
        for (int s = 0; s < TSTAGES; s++) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        for (int b = 0; b < 4; b++) {
            mbar_init(&S.acc_full[b], 1);
            mbar_init(&S.acc_empty[b], kEpiThreads);
        }
        mbar_init(&S.drain, 1);
        mbar_init(&S.xs_full[0], kEpiThreads);
        mbar_init(&S.xs_full[1], kEpiThreads);
        mbar_init(&S.xs_empty[0], kEpiThreads);
        mbar_init(&S.xs_empty[1], kEpiThreads);
        S.abort = 0;
        S.never = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&S.tmem_base)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = S.tmem_base;
    if (warp >= 2) {  // both accumulators start at the bits of 1.5 * 2^23 (the epilogue's int -> float step)
        const uint32_t q = tmem + ((uint32_t)((warp & 3) * 32) << 16) + ((warp - 2) >> 2) * kHalfN;
        for (int b = 0; b < 4; b++)
            for (int c = 0; c < kHalfN; c += 32) tmem_fill32(q + b * TBN + c, kMagicI);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int kg = 0;  // stages issued by this CTA
            bool ok = true;
            for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
                const int tile = item / nrb, rb = item % nrb;
                const int tv = R.gemm_tiles[tile];
                const int e = R.gemm_units[tv >> 16];
                const int arow = e * rows + rb * TBM, brow = R.off[e] + (tv & 0xFFFF) * TBN;
                for (int kh = 0; kh < nkh; kh++, kg++) {
                    const int s = kg % TSTAGES;
                    if (kg >= TSTAGES && !mbar_wait(&S.empty[s], ((kg / TSTAGES) - 1) & 1, abort)) {
                        S.abort = 1;
                        ok = false;
                        break;
                    }
                    uint8_t *stage = ring + s * kStageBytes;
                    mbar_expect_tx(&S.full[s], kStageBytes);
                    tma_load_2d(stage, &mapA, kh * TBK, arow, &S.full[s]);
                    tma_load_2d(stage + TBM * TBK, &mapB, kh * TBK, brow, &S.full[s]);
                }
            }
            // drain: every issued copy has landed before the CTA may leave (bounded; each slot's latest phase)
            for (int k = max(0, kg - TSTAGES); k < kg; k++) mbar_wait(&S.full[k % TSTAGES], (k / TSTAGES) & 1, never);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            bool ok = true;
            int kg = 0, bg = 0;  // stages consumed, blocks accumulated by this CTA
            for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
                for (int kh = 0; kh < nkh; kh++, kg++) {
                    const int s = kg % TSTAGES, buf = bg & 3;
                    const bool first_half = (kh & 1) == 0;
                    if (first_half && bg >= 4 && !mbar_wait(&S.acc_empty[buf], ((bg / 4) - 1) & 1, abort)) { ok = false; break; }
                    if (!mbar_wait(&S.full[s], (kg / TSTAGES) & 1, abort)) { ok = false; break; }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint8_t *stage = ring + s * kStageBytes;
                    const uint64_t da = umma_desc(stage), db = umma_desc(stage + TBM * TBK);
                    const uint32_t d = tmem + buf * TBN;
#pragma unroll
                    for (int k = 0; k < TBK / 32; k++)  // 4 MMAs of K = 32 bytes; the descriptor start moves 32 B
                        mma_i8(d, da + (uint64_t)(k * 2), db + (uint64_t)(k * 2), kIdesc, 1u);  // onto 1.5 * 2^23
                    mma_commit(&S.empty[s]);  // stage reusable once these MMAs finish
                    if (!first_half || kh == nkh - 1) {  // block's dot products are done
                        mma_commit(&S.acc_full[buf]);
                        bg++;
                    }
                }
            }
            if (!ok) S.abort = 1;
            // every MMA issued by this CTA has completed before TMEM and shared memory are released (bounded)
            mma_commit(&S.drain);
            mbar_wait(&S.drain, 0, never);
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: thread = (weight row, half of the tile's tokens) ----------------
        // TMEM lane quadrant = warp % 4 (the lanes a warp may access); warps 2-5 take tokens 0-63, warps 6-9 64-127
        const int sub = warp & 3, half = (warp - 2) >> 2;
        const int r = sub * 32 + lane, c0 = half * kHalfN;
        const int et = threadIdx.x - 64;  // 0..255 among the epilogue threads
        bool ok = true;
        int bg = 0, it = 0;
        // the next item's metadata is loaded one item ahead
        auto item_meta = [&](int item, int &e, int &base, int &t0, int &nt, int &rb) {
            const int tile = item / nrb;
            rb = item % nrb;
            const int tv = R.gemm_tiles[tile];
            e = R.gemm_units[tv >> 16];
            base = R.off[e];
            t0 = (tv & 0xFFFF) * TBN;
            nt = min(TBN, R.cnt[e] - t0);
        };
        // An item's token scales (zero past the expert's tokens) and, for the down matrix, each token's output slot
        // and weight are staged in shared memory one item ahead: loaded into registers when the item before it
        // starts, stored after that item's first block, so the loads overlap its MMAs.
        constexpr int kPre = (kMaxKB * TBN + kEpiThreads - 1) / kEpiThreads;  // scales per thread (nkb <= kMaxKB)
        float pre[kPre];
        int pslot = 0;
        float pw = 0.0f;
        auto load_next = [&](int base_, int t0_, int nt_) {
#pragma unroll
            for (int k = 0; k < kPre; k++) {
                const int i = et + k * kEpiThreads, n = i % TBN, b = i / TBN;
                pre[k] = (b < nkb && n < nt_) ? __ldg(xs_e + (size_t)(base_ + t0_ + n) * nkb + b) : 0.0f;
            }
            if (KIND == 1 && et < TBN) {
                pslot = et < nt_ ? R.eslot[base_ + t0_ + et] : 0;
                pw = et < nt_ ? R.ew[base_ + t0_ + et] : 0.0f;
            }
        };
        // item j's data into buffer j&1, once every epilogue thread has finished item j-2 (its last reader)
        auto store_next = [&](int j) -> bool {
            const int pb = j & 1;
            if (j >= 2 && !mbar_wait(&S.xs_empty[pb], ((j - 2) >> 1) & 1, abort)) return false;
#pragma unroll
            for (int k = 0; k < kPre; k++) {
                const int i = et + k * kEpiThreads;
                if (i / TBN < nkb) S.xs[pb][i / TBN][i % TBN] = pre[k];
            }
            if (KIND == 1 && et < TBN) {
                S.oslot[pb][et] = pslot;
                S.ow[pb][et] = pw;
            }
            mbar_arrive(&S.xs_full[pb]);
            return true;
        };
        int e, base, t0, nt, rb;
        item_meta(blockIdx.x, e, base, t0, nt, rb);
        load_next(base, t0, nt);
        store_next(0);
        for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x, it++) {
            const bool has_next = item + (int)gridDim.x < nitems;
            int ne = 0, nbase = 0, nt0 = 0, nnt = 0, nrb_ = 0;
            if (has_next) item_meta(item + gridDim.x, ne, nbase, nt0, nnt, nrb_);
            const int row = rb * TBM + r;
            float(*xs)[TBN] = S.xs[it & 1];
            if (!mbar_wait(&S.xs_full[it & 1], (it >> 1) & 1, abort)) {
                ok = false;
                S.abort = 1;
                break;
            }
            if (has_next) load_next(nbase, nt0, nnt);
            const float *wsr = wsc + ((size_t)e * rows + row) * nkb;
            // f[j] holds tokens c0 + 2j, c0 + 2j + 1: the packed f32x2 instructions round each lane like their scalar
            // forms, so f is the scalar sequence's bits. 32-token chunks past the tile's last token are not read.
            float2 f[kHalfN / 2];
#pragma unroll
            for (int j = 0; j < kHalfN / 2; j++) f[j] = make_float2(0.0f, 0.0f);
            const float2 neg_magic = make_float2(-12582912.0f, -12582912.0f);
            for (int b = 0; b < nkb; b++, bg++) {
                const int buf = bg & 3;
                const float wsb = __ldg(wsr + b);  // in flight while the block's MMAs finish
                if (!mbar_wait(&S.acc_full[buf], (bg / 4) & 1, abort)) {
                    ok = false;
                    S.abort = 1;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const float2 ws2 = make_float2(wsb, wsb);
#pragma unroll
                for (int c = 0; c < kHalfN / 32; c++) {
                    const uint32_t ta = tmem + ((uint32_t)(sub * 32) << 16) + buf * TBN + c0 + c * 32;
                    if (c0 + c * 32 < nt) {
                        int v[32];
                        tmem_ld32(ta, v);
#pragma unroll
                        for (int j4 = 0; j4 < 8; j4++) {
                            const float4 x4 = *reinterpret_cast<const float4 *>(&xs[b][c0 + c * 32 + j4 * 4]);
                            const float2 p01 = __fmul2_rn(ws2, make_float2(x4.x, x4.y));
                            const float2 p23 = __fmul2_rn(ws2, make_float2(x4.z, x4.w));
                            const float2 d01 = __fadd2_rn(
                                make_float2(__int_as_float(v[j4 * 4]), __int_as_float(v[j4 * 4 + 1])), neg_magic);
                            const float2 d23 = __fadd2_rn(
                                make_float2(__int_as_float(v[j4 * 4 + 2]), __int_as_float(v[j4 * 4 + 3])), neg_magic);
                            const int j = c * 16 + j4 * 2;
                            f[j] = __ffma2_rn(d01, p01, f[j]);
                            f[j + 1] = __ffma2_rn(d23, p23, f[j + 1]);
                        }
                    }
                    tmem_fill32(ta, kMagicI);  // the next block in this buffer accumulates onto 1.5 * 2^23 again
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                mbar_arrive(&S.acc_empty[buf]);
                if (b == 0 && has_next && !store_next(it + 1)) {
                    ok = false;
                    S.abort = 1;
                    break;
                }
            }
            if (!ok) break;
#pragma unroll
            for (int j = 0; j < kHalfN; j++) {
                const int tn = c0 + j;
                const float fj = (j & 1) ? f[j >> 1].y : f[j >> 1].x;
                if (tn < nt) {
                    if (KIND == 0) out[(size_t)(base + t0 + tn) * out_ld + row] = fj;
                    else out[(size_t)S.oslot[it & 1][tn] * out_ld + row] = __fmul_rn(S.ow[it & 1][tn], fj);
                }
            }
            mbar_arrive(&S.xs_empty[it & 1]);  // this thread has finished reading buffer it&1
            e = ne; base = nbase; t0 = nt0; nt = nnt; rb = nrb_;
        }
        if (!ok) S.abort = 1;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (S.abort && threadIdx.x == 0) atomicCAS(&R.meta[kMetaError], 0, kErrTimeout);
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
}

// ---------------------------------------------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D int8 map over [rows][cols] (row pitch = cols bytes) with 128 x 128-byte boxes and 128-byte swizzle
bool make_tma_map_i8(void *map_out, const void *base, uint64_t rows, uint64_t cols, int box_rows) {
    auto fn = encode_fn();
    if (!fn || cols % 16 || reinterpret_cast<uintptr_t>(base) % 16) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols};
    const cuuint32_t box[2] = {(cuuint32_t)TBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(reinterpret_cast<CUtensorMap *>(map_out), CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims,
              strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D fp32 map over [rows][cols] (row pitch = cols floats) with box_rows x 32-float boxes and 128-byte swizzle; rows
// past `rows` read as zeros
bool make_tma_map_f32(void *map_out, const float *base, uint64_t rows, uint64_t cols, int box_rows) {
    auto fn = encode_fn();
    if (!fn || (cols * 4) % 16 || reinterpret_cast<uintptr_t>(base) % 16) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 4};
    const cuuint32_t box[2] = {32u, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(reinterpret_cast<CUtensorMap *>(map_out), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base),
              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t gemm_tc_smem() { return (size_t)TSTAGES * kStageBytes + sizeof(TcShared) + 1024; }

void gemm_tc_set_attributes() {
    cudaFuncSetAttribute(gemm_tc_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_tc_smem());
    cudaFuncSetAttribute(gemm_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_tc_smem());
}

// grid: an upper bound on (token tiles x row tiles); CTAs past the device-built tile count return at once
int launch_gemm_tc(int kind, const void *mapA, const void *mapB, const float *wsc, int rows, int K, const RouteDev &R,
                   const float *xs_e, float *out, int out_ld, int max_tiles, cudaStream_t st) {
    if (rows % TBM || K % TBK || K > kMaxKB * kKB) return -1;
    const int mt = kind == 0 ? kMetaGemmTilesGU : kMetaGemmTilesDN;
    static int sms[64] = {0};  // persistent grid: one CTA per SM (at most the items the call can have)
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    const int nsm = dev >= 0 && dev < 64 && sms[dev] > 0 ? sms[dev] : 148;
    const int grid = std::min(nsm, max_tiles * (rows / TBM));
    const CUtensorMap &a = *reinterpret_cast<const CUtensorMap *>(mapA);
    const CUtensorMap &b = *reinterpret_cast<const CUtensorMap *>(mapB);
    if (kind == 0) gemm_tc_kernel<0><<<grid, kThreads, gemm_tc_smem(), st>>>(a, b, wsc, rows, K, R, xs_e, out, out_ld, mt);
    else gemm_tc_kernel<1><<<grid, kThreads, gemm_tc_smem(), st>>>(a, b, wsc, rows, K, R, xs_e, out, out_ld, mt);
    return 1;
}

int gemm_tc_token_tile() { return TBN; }

}  // namespace inzg
