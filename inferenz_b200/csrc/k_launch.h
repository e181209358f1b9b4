// k_launch.h -- host launchers of the libinzg kernels (each returns the number of kernels it launched, -1 = no
// instantiation for the geometry).
#pragma once

#include "inzg_internal.h"

namespace inzg {

void router_set_attributes(int H);
void launch_router_repack(const uint16_t *W, uint4 *Wr, int E, int H, cudaStream_t st);
void launch_router_repack32(const uint16_t *W, float *Wf, int E, int H, cudaStream_t st);
bool router_gemm_fits(int E, int H);
size_t router32_floats(int E, int H);  // floats of the fp32 copy (launch_router_repack32), whole 128-column chunks
// Wf: the fp32 copy (nullptr: the f16 kernels only)
int launch_router_logits(const uint4 *Wr, const float *Wf, const float *X, int n, int H, int E, const float *bias,
                         float *logits, int32_t *meta, cudaStream_t st);
// lin_mm's F16 path for any rows % 4 == 0, K % 64 == 0 (W in the router layout, Wf its fp32 copy or nullptr)
int launch_f16_rows(const uint4 *Wr, const float *Wf, const float *X, int n, int K, int rows, float *Y, int32_t *meta,
                    cudaStream_t st);
int launch_softmax_topk(const float *logits, int n, int E, int topk, int32_t *sel, float *w, float *probs,
                        cudaStream_t st);

int launch_route_fused(const RouteDev &R, const float *logits, float *probs, int gu_items_per_unit,
                       int dn_items_per_unit, int gemm_tn, int32_t *upath, int32_t *eexp, cudaStream_t st);
void route_set_attributes(int E);
int launch_route(const RouteDev &R, int gu_items_per_unit, int dn_items_per_unit, int gemm_tn,
                 int32_t *upath, int32_t *eexp, cudaStream_t st);
int route_chunks(int n);  // chunks of the large-n route (64 tokens each): rows of RouteDev::ccnt / cmask

int launch_act_quant_x(const float *X, int n, int H, int rot, uint32_t seed, int8_t *q64, float2 *sb64, int8_t *q256,
                       float *s256, cudaStream_t st);
int launch_swiglu_quant(const float *GU, int FF, int n_entries, const int32_t *eexp, const int32_t *upath, int rot,
                        uint32_t seed, int8_t *q64, float2 *sb64, int8_t *q256, float *s256, cudaStream_t st);
int launch_combine(const float *mo, int n, int H, int topk, float *y, int num_sms, cudaStream_t st);
int launch_shared_add(const float *X, const float *gate, const float *D, float *y, int n, int H, const int32_t *sh_meta,
                      int32_t *meta, cudaStream_t st);
int launch_shared_route(const RouteDev &R, int n, int gemm, int gu_items_per_unit, int dn_items_per_unit, int gemm_tn,
                        int32_t *upath, int32_t *eexp, cudaStream_t st);

void gemv_set_attributes();
// Prefill-numerics experts of a decode-sized call (at most kGemvGemmMaxTokens token rows), run by the decode GEMV
// kernel itself as GEMM items (the call's R.gemm_tiles, built with a token tile of kGemvGemmTile: an expert with more
// tokens takes one item per tile and row block): int8 activations per 256-block by token (gate|up) or by entry
// (down), their block scales, the layer's per-(row, 256-block) weight scales and a TMA map over the requantized int8
// weights with 16-row boxes (make_tma_map_i8(..., 16)).
constexpr int kGemvGemmTile = 32, kGemvGemmMaxTokens = 256;
struct DecGemm {
    const int8_t *aq;
    const float *as;
    const float *ws;
    const void *wmap;
};
int launch_gemv_decode(const LayerDev &L, int kind, const RouteDev &R, const int8_t *aq, const float2 *asb, float *out,
                       int out_ld, int num_sms, cudaStream_t st, const DecGemm *gm = nullptr);
int gemv_items_per_unit(const LayerDev &L, int kind, int n);  // n: token rows of the call (R.n)
int launch_gemm_v1(const LayerDev &L, int kind, const RouteDev &R, const int8_t *aq, const float *as, float *out,
                   int out_ld, int grid, cudaStream_t st);
int gemm_token_tile();
bool make_tma_map_i8(void *map_out, const void *base, uint64_t rows, uint64_t cols, int box_rows);
bool make_tma_map_f32(void *map_out, const float *base, uint64_t rows, uint64_t cols, int box_rows);
size_t gemm_tc_smem();
void gemm_tc_set_attributes();
int launch_gemm_tc(int kind, const void *mapA, const void *mapB, const float *wsc, int rows, int K, const RouteDev &R,
                   const float *xs_e, float *out, int out_ld, int max_tiles, cudaStream_t st);
int gemm_tc_token_tile();
int launch_gather_gemm_rows(const int8_t *q, const float *s, int K, int nkb, const int32_t *etok, const int32_t *eexp,
                            const int32_t *upath, int n_entries, int8_t *qe, float *se, cudaStream_t st);

void launch_pool_requant(const uint8_t *blobs, uint64_t blob_bytes, uint64_t gu_bytes, int e0, int ne, const LayerDev &L,
                         cudaStream_t st);
void launch_pool_repack(const uint8_t *blobs, uint64_t blob_bytes, uint64_t gu_bytes, int e0, int ne,
                        const LayerDev &L, uint8_t *pool, uint8_t *luts, cudaStream_t st);

// Hyper-connections around the layer (k_hc.cu, src/model_fwd.c:404-450). Weights of one block on the device.
struct HcDev {
    const float *norm = nullptr;    // [4H], the folded 1 + w
    const uint4 *down = nullptr;    // [rank][4H] f16 in the router layout
    const float *down32 = nullptr;  // its fp32 copy for the many-token kernel (nullptr: not used)
    const uint4 *up = nullptr;      // [4H][rank] f16 in the router layout
    const float *up32 = nullptr;    // its fp32 copy (nullptr: not used)
    const float *inject = nullptr;  // [4][4H] (nullptr: no inject, as the final mixer)
    int rank = 0;
};
void hc_set_attributes(int H);
// X [n][4H] -> xin [n][H], inj [n][4] (skipped when w.inject or inj is null); scratch Xn [n][4H], d [n][rank],
// m [n][4H]. Returns the number of kernels launched, -1 when a matrix shape has no kernel.
int launch_hc_in(const HcDev &w, int n, int H, const float *X, float *Xn, float *d, float *m, float *xin, float *inj,
                 int32_t *meta, int num_sms, cudaStream_t st);
int launch_hc_out(float *X, const float *inj, const float *y, int n, int H, int num_sms, cudaStream_t st);

// Expert-parallel exchange over peer memory (k_ep.cu). epoch_dev: the rank's step counter; tickets: one int per kernel.
// route + dispatch from the router logits [n][E] (softmax and top-k per token inside; sel_out [n][topk] kept for the
// combine)
int launch_ep_dispatch(const float *logits, const float *x, int n, int E, const EpPeers &P, int32_t *sel_out,
                       const uint32_t *epoch_dev, int32_t *ticket, cudaStream_t st);
int launch_ep_signal(const EpPeers &P, const uint32_t *epoch_dev, cudaStream_t st);
int launch_ep_barrier(const EpPeers &P, uint32_t *bar_epoch, int32_t *err, cudaStream_t st);
int launch_ep_combine(const int32_t *sel, int n, const EpPeers &P, float *y, int num_sms, cudaStream_t st);
int launch_ep_wait(const uint32_t *flags, int world, int which, uint32_t *epoch_dev, bool advance, int32_t *err,
                   cudaStream_t st);

// The whole routed layer in one cooperative launch for calls of 1-2 tokens (k_fused.cu); -1 when the shape has no
// instantiation. counters: fused_counter_ints(E, 8, H) ints, all zero before the first call.
size_t fused_counter_ints(int E, int n_max, int H);
bool fused_decode_fits(const LayerDev &L, int n, int K, bool have_router_or_ovr);
int launch_fused_decode(const LayerDev &L, int n, int K, const float *x, const float *bias, const float *ovr,
                        float *logits, float *probs, int32_t *sel, float *w, int32_t *units, int32_t *meta,
                        int8_t *xq64, float2 *xsb64, float *GU, int8_t *dq64, float2 *dsb64, float *mo, float *y,
                        int32_t *counters, int num_sms, cudaStream_t st);

}  // namespace inzg
