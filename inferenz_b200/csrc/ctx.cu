// ctx.cu -- the C ABI of libinzg (include/inzg.h): context, HBM expert pool, and the routed MoE forward.
//
// One forward call (all on one stream, no host synchronisation until the result is copied back):
//   router logits (bit-exact F16 GEMV)  ->  softmax + top-k + renormalised weights  ->  activation quantization of
//   the inputs (both numeric paths)  ->  dispatch lists  ->  gate|up (decode GEMV / prefill GEMM)  ->  SiLU*up +
//   quantization  ->  down (GEMV / GEMM) writing w * y into the token's slot  ->  rank-order combine.
// Reference: moe_block, src/model_fwd.c:992-1140; the expert cache (src/expert_cache.c) is replaced by the pool.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/inzg.h"
#include "host/inzg_host.h"
#include "inzg_internal.h"
#include "k_launch.h"

using namespace inzg;

namespace {

constexpr uint32_t kMagic = 0x515A4E49u;  // "INZQ"

struct QHeader {  // src/quant.h:40-50
    uint32_t magic;
    uint16_t type, rot_block;
    uint32_t rows, cols, rot_seed;
    uint8_t bits, pad[3];
    uint8_t lut[32];
    uint8_t pad2[8];
};
static_assert(sizeof(QHeader) == 64, "header is 64 bytes");

struct TmaMap {
    alignas(64) unsigned char bytes[128];  // a CUtensorMap, opaque here
};

struct LayerSlot {
    bool has_router = false, has_experts = false;
    int e_first = 0;            // the pool holds experts [e_first, e_first + dev.E) of the layer's n_expert
    bool has_maps = false;
    TmaMap map_gu, map_dn;      // TMA maps over the prefill-path int8 weights
    TmaMap map16_gu, map16_dn;  // the same weights in 16-row boxes (GEMM items of the decode GEMV)
    uint4 *router = nullptr;
    float *router32 = nullptr;  // the same router in fp32, laid out for the many-token kernel (nullptr: not used)
    uint8_t *pool = nullptr;
    uint8_t *luts = nullptr;
    uint8_t *gemm_w = nullptr;  // one allocation: w8_gu | w8_dn | ws_gu | ws_dn
    LayerDev dev{};
};

// hyper-connection weights of one layer (inzg_set_hc): one allocation, norm | inject | down32 | up32 | down | up
struct HcSlot {
    uint8_t *mem = nullptr;
    HcDev dev{};
};

template <class T>
T *dalloc(size_t count, bool &ok) {
    void *p = nullptr;
    if (count == 0) count = 1;
    if (cudaMalloc(&p, sizeof(T) * count) != cudaSuccess) {
        ok = false;
        cudaGetLastError();
        return nullptr;
    }
    return static_cast<T *>(p);
}

MatLayout make_layout(int type, int rows, int cols) {
    MatLayout m{};
    m.rows = rows;
    m.cols = cols;
    m.ng = cols / kGroup;
    m.gd = (m.ng + 3) / 4;
    m.wb = type == INZG_T_Q8G ? 32 : 16;
    return m;
}

uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

}  // namespace

// This rank's part of the expert-parallel exchange (k_ep.cu): its exposed buffer, the peers' mappings, the step
// counter and the local scratch of a step.
struct EpState {
    int rank = 0, world = 0, cap = 0;
    uint8_t *base = nullptr;            // exposed: rsel | rw | rx | out | flags
    size_t bytes = 0;
    size_t o_rsel = 0, o_rw = 0, o_rx = 0, o_out = 0, o_flags = 0;
    std::vector<void *> opened;          // peers' buffers opened through IPC (closed at detach)
    EpPeers P{};
    bool connected = false;
    uint8_t *local = nullptr;            // epoch | tickets[2] | err | rendezvous epoch | sel [cap][K] (own selections)
    uint32_t *epoch = nullptr, *bar_epoch = nullptr;
    int32_t *tickets = nullptr, *err = nullptr, *sel = nullptr;
};

struct inzg_ctx {
    inzg_config cfg{};
    EpState *ep = nullptr;
    int num_sms = 0;
    cudaStream_t stream = nullptr;
    std::vector<LayerSlot> layers;
    std::vector<LayerSlot> shared;           // per layer: the shared expert as a one-expert pool (inzg_set_shared)
    std::vector<float *> sh_gate;            // per layer: the shared expert's gate vector [hidden]
    std::vector<HcSlot> hc;                  // per layer: the hyper-connection weights around the MoE (inzg_set_hc)
    float *hc_Xn = nullptr, *hc_d = nullptr, *hc_m = nullptr, *hc_inj = nullptr;  // hc_in scratch, hc_cap tokens
    int hc_cap = 0;
    std::string err;
    inzg_stats stats{};
    // scratch
    float *xin = nullptr, *y = nullptr, *logits = nullptr, *probs = nullptr, *bias = nullptr;
    int32_t *sel = nullptr;
    float *w = nullptr;
    int8_t *xq64 = nullptr, *xq256 = nullptr;
    float2 *xsb64 = nullptr;
    float *xs256 = nullptr;
    int32_t *cnt = nullptr, *off = nullptr, *first = nullptr, *etok = nullptr, *eslot = nullptr, *ccnt = nullptr;
    int32_t *units = nullptr, *meta = nullptr, *dec_units = nullptr, *gemm_units = nullptr, *gemm_tiles = nullptr;
    int32_t *upath = nullptr, *eexp = nullptr;
    int32_t *fused_cnt = nullptr;  // the fused decode kernel's barrier and hand-off counters
    uint64_t *cmask = nullptr;
    float *ew = nullptr, *GU = nullptr, *mo = nullptr;
    int8_t *dq64 = nullptr, *dq256 = nullptr;
    float2 *dsb64 = nullptr;
    float *ds256 = nullptr;
    // the shared expert's one-unit dispatch list
    int32_t *sh_cnt = nullptr, *sh_off = nullptr, *sh_first = nullptr, *sh_etok = nullptr, *sh_eslot = nullptr;
    int32_t *sh_eexp = nullptr, *sh_upath = nullptr, *sh_units = nullptr, *sh_dec = nullptr, *sh_gemm = nullptr;
    int32_t *sh_tiles = nullptr, *sh_meta = nullptr;
    float *sh_ew = nullptr;
    int8_t *xqe = nullptr;      // prefill-path token activations in entry order [n*topk][H]
    float *xse = nullptr;       // their block scales [n*topk][H/256]
    TmaMap map_xqe, map_dq;     // TMA maps over xqe and dq256
    bool have_tc = false;
    int last_n = 0;
    bool last_dump = false;
    // per-stage profile
    double stage_ms[INZG_N_STAGES] = {0};
    uint64_t profiled_calls = 0;
    cudaEvent_t ev[INZG_N_STAGES + 1] = {};
    // CUDA graphs of the forward, keyed by everything a replay bakes in
    struct GraphKey {
        int layer, n;
        const void *x, *y, *bias, *ovr;
        unsigned flags;
        int aux;  // expert-parallel steps: the batch size of the numeric-path rule (forward calls: 0)
        bool operator==(const GraphKey &o) const {
            return layer == o.layer && n == o.n && x == o.x && y == o.y && bias == o.bias && ovr == o.ovr &&
                   flags == o.flags && aux == o.aux;
        }
    };
    struct GraphEntry {
        GraphKey key;
        cudaGraphExec_t exec;
        int launches;
        uint64_t last_use;
    };
    std::vector<GraphEntry> graphs;
    uint64_t use_clock = 0;
    cudaStream_t capture_stream = nullptr;
    cudaStream_t side = nullptr;            // branch for the input quantization, joined before the experts
    cudaEvent_t fork = nullptr, join = nullptr;
};

static const char *kStageNames[INZG_N_STAGES] = {"router_logits", "softmax_topk_route", "act_quant", "route",
                                                 "gate_up_gemv", "gate_up_gemm", "swiglu_quant", "down_gemv",
                                                 "down_gemm", "combine", "fused_decode", "shared_expert"};

static void drop_graphs(inzg_ctx *c) {
    for (auto &g : c->graphs) cudaGraphExecDestroy(g.exec);
    c->graphs.clear();
}

static inzg_status fail(inzg_ctx *c, inzg_status st, const std::string &msg) {
    if (c) c->err = msg;
    return st;
}

static inzg_status cuda_fail(inzg_ctx *c, cudaError_t e, const char *what) {
    return fail(c, INZG_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

extern "C" {

const char *inzg_status_str(inzg_status st) {
    switch (st) {
    case INZG_OK: return "ok";
    case INZG_BAD_ARG: return "bad argument";
    case INZG_CORRUPT_BLOB: return "corrupt expert blob";
    case INZG_OOM: return "out of device memory";
    case INZG_CUDA: return "CUDA error";
    case INZG_NCCL: return "NCCL error";
    case INZG_TIMEOUT: return "device wait timed out";
    case INZG_DEVICE_CHECK: return "device-side check failed";
    case INZG_UNSUPPORTED: return "unsupported shape or format";
    case INZG_NOT_READY: return "layer not loaded";
    }
    return "unknown status";
}

const char *inzg_last_error(const inzg_ctx *c) { return c ? c->err.c_str() : "no context"; }

static void free_scratch(inzg_ctx *c) {
    void *ptrs[] = {c->xin, c->y, c->logits, c->probs, c->bias, c->sel, c->w, c->xq64, c->xq256, c->xsb64,
                    c->xs256, c->cnt, c->off, c->first, c->etok, c->eslot, c->ccnt, c->units, c->meta, c->dec_units,
                    c->gemm_units, c->gemm_tiles, c->upath, c->eexp, c->ew, c->GU, c->mo, c->dq64, c->dq256, c->dsb64,
                    c->ds256, c->xqe, c->xse, c->sh_cnt, c->sh_off, c->sh_first, c->sh_etok, c->sh_eslot,
                    c->sh_eexp, c->sh_upath, c->sh_units, c->sh_dec, c->sh_gemm, c->sh_tiles, c->sh_meta, c->sh_ew,
                    c->cmask, c->fused_cnt};
    for (void *p : ptrs)
        if (p) cudaFree(p);
}

inzg_ctx *inzg_create(const inzg_config *cfg, inzg_status *status) {
    inzg_status dummy;
    inzg_status &st = status ? *status : dummy;
    if (!cfg || cfg->hidden <= 0 || cfg->hidden % 256 || cfg->ff <= 0 || cfg->ff % kGroup || cfg->n_expert <= 0 ||
        cfg->n_expert % 32 || cfg->n_expert > 1024 || cfg->topk <= 0 || cfg->topk > kMaxTopK ||
        cfg->topk > cfg->n_expert || cfg->max_tokens <= 0 || cfg->n_layers <= 0) {
        st = INZG_BAD_ARG;
        return nullptr;
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || cfg->device < 0 || cfg->device >= ndev) {
        cudaGetLastError();
        st = INZG_CUDA;
        return nullptr;
    }
    if (cudaSetDevice(cfg->device) != cudaSuccess) {
        st = INZG_CUDA;
        return nullptr;
    }
    inzg_ctx *c = new inzg_ctx();
    c->cfg = *cfg;
    c->layers.resize(cfg->n_layers);
    c->shared.resize(cfg->n_layers);
    c->hc.resize(cfg->n_layers);
    c->sh_gate.assign(cfg->n_layers, nullptr);
    cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, cfg->device);
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete c;
        st = INZG_CUDA;
        return nullptr;
    }
    const size_t T = cfg->max_tokens, H = cfg->hidden, E = cfg->n_expert, K = cfg->topk, FF = cfg->ff;
    const size_t NE = T * K, nkbH = (H + kKB - 1) / kKB, nkbF = (FF + kKB - 1) / kKB;
    const size_t nchunk = (size_t)route_chunks((int)T);
    if (NE / (size_t)gemm_token_tile() + E >= 65536) {  // the dispatch scan counts GEMM tiles in 16 bits
        cudaStreamDestroy(c->stream);
        delete c;
        st = INZG_BAD_ARG;
        return nullptr;
    }
    bool ok = true;
    c->xin = dalloc<float>(T * H, ok);
    c->y = dalloc<float>(T * H, ok);
    c->logits = dalloc<float>(T * E, ok);
    c->probs = dalloc<float>(T * E, ok);
    c->bias = dalloc<float>(E, ok);
    c->sel = dalloc<int32_t>(NE, ok);
    c->w = dalloc<float>(NE, ok);
    c->xq64 = dalloc<int8_t>(T * H, ok);
    c->xq256 = dalloc<int8_t>(T * H, ok);
    c->xsb64 = dalloc<float2>(T * H / kGroup, ok);
    c->xs256 = dalloc<float>(T * nkbH, ok);
    c->cnt = dalloc<int32_t>(E, ok);
    c->off = dalloc<int32_t>(E + 1, ok);
    c->first = dalloc<int32_t>(E, ok);
    c->etok = dalloc<int32_t>(NE, ok);
    c->eslot = dalloc<int32_t>(NE, ok);
    c->eexp = dalloc<int32_t>(NE, ok);
    c->ew = dalloc<float>(NE, ok);
    c->ccnt = dalloc<int32_t>(nchunk * E, ok);
    c->cmask = dalloc<uint64_t>(nchunk * E, ok);
    c->units = dalloc<int32_t>(E, ok);
    c->meta = dalloc<int32_t>(16, ok);
    c->dec_units = dalloc<int32_t>(E, ok);
    c->gemm_units = dalloc<int32_t>(E, ok);
    c->gemm_tiles = dalloc<int32_t>(NE / 16 + E, ok);
    c->upath = dalloc<int32_t>(E, ok);
    c->GU = dalloc<float>(NE * 2 * FF, ok);
    c->mo = dalloc<float>(NE * H, ok);
    c->dq64 = dalloc<int8_t>(NE * FF, ok);
    c->dq256 = dalloc<int8_t>(NE * FF, ok);
    c->dsb64 = dalloc<float2>(NE * FF / kGroup, ok);
    c->ds256 = dalloc<float>(NE * nkbF, ok);
    c->xqe = dalloc<int8_t>(NE * H, ok);
    c->xse = dalloc<float>(NE * nkbH, ok);
    c->sh_cnt = dalloc<int32_t>(1, ok);
    c->sh_off = dalloc<int32_t>(2, ok);
    c->sh_first = dalloc<int32_t>(1, ok);
    c->sh_etok = dalloc<int32_t>(T, ok);
    c->sh_eslot = dalloc<int32_t>(T, ok);
    c->sh_eexp = dalloc<int32_t>(T, ok);
    c->sh_ew = dalloc<float>(T, ok);
    c->sh_upath = dalloc<int32_t>(1, ok);
    c->sh_units = dalloc<int32_t>(1, ok);
    c->sh_dec = dalloc<int32_t>(1, ok);
    c->sh_gemm = dalloc<int32_t>(1, ok);
    c->sh_tiles = dalloc<int32_t>(T / 16 + 2, ok);
    c->sh_meta = dalloc<int32_t>(16, ok);
    c->fused_cnt = dalloc<int32_t>(fused_counter_ints((int)E, 8, (int)H), ok);
    if (ok && cudaMemset(c->fused_cnt, 0, sizeof(int32_t) * fused_counter_ints((int)E, 8, (int)H)) != cudaSuccess)
        ok = false;
    if (!ok) {
        free_scratch(c);
        cudaStreamDestroy(c->stream);
        delete c;
        st = INZG_OOM;
        return nullptr;
    }
    router_set_attributes(cfg->hidden);
    gemv_set_attributes();
    gemm_tc_set_attributes();
    c->have_tc = make_tma_map_i8(c->map_xqe.bytes, c->xqe, NE, H, 128) && make_tma_map_i8(c->map_dq.bytes, c->dq256, NE, FF, 128);
    for (int i = 0; i <= INZG_N_STAGES; i++) cudaEventCreate(&c->ev[i]);
    cudaStreamCreateWithFlags(&c->capture_stream, cudaStreamNonBlocking);
    cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking);
    cudaEventCreateWithFlags(&c->fork, cudaEventDisableTiming);
    cudaEventCreateWithFlags(&c->join, cudaEventDisableTiming);
    route_set_attributes(cfg->n_expert);
    st = INZG_OK;
    return c;
}

void inzg_destroy(inzg_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->cfg.device);
    cudaStreamSynchronize(c->stream);
    inzg_ep_detach(c);
    for (auto *v : {&c->layers, &c->shared})
        for (auto &L : *v) {
            if (L.router) cudaFree(L.router);
            if (L.router32) cudaFree(L.router32);
            if (L.pool) cudaFree(L.pool);
            if (L.luts) cudaFree(L.luts);
            if (L.gemm_w) cudaFree(L.gemm_w);
        }
    for (float *g : c->sh_gate)
        if (g) cudaFree(g);
    for (auto &h : c->hc)
        if (h.mem) cudaFree(h.mem);
    for (float *p : {c->hc_Xn, c->hc_d, c->hc_m, c->hc_inj})
        if (p) cudaFree(p);
    drop_graphs(c);
    for (int i = 0; i <= INZG_N_STAGES; i++)
        if (c->ev[i]) cudaEventDestroy(c->ev[i]);
    if (c->capture_stream) cudaStreamDestroy(c->capture_stream);
    if (c->side) cudaStreamDestroy(c->side);
    if (c->fork) cudaEventDestroy(c->fork);
    if (c->join) cudaEventDestroy(c->join);
    free_scratch(c);
    cudaStreamDestroy(c->stream);
    delete c;
}

inzg_status inzg_set_router(inzg_ctx *c, int layer, const uint16_t *w, int rows, int cols) {
    if (!c) return INZG_BAD_ARG;
    if (layer < 0 || layer >= c->cfg.n_layers || !w) return fail(c, INZG_BAD_ARG, "set_router: bad layer or pointer");
    if (rows != c->cfg.n_expert || cols != c->cfg.hidden)
        return fail(c, INZG_BAD_ARG, "set_router: router must be n_expert x hidden");
    cudaSetDevice(c->cfg.device);
    drop_graphs(c);
    LayerSlot &L = c->layers[layer];
    const size_t bytes = (size_t)rows * cols * 2;
    uint16_t *tmp = nullptr;
    cudaError_t e = cudaMalloc(&tmp, bytes);
    if (e != cudaSuccess) return fail(c, INZG_OOM, "set_router: staging buffer");
    if (!L.router && cudaMalloc(&L.router, bytes) != cudaSuccess) {
        cudaFree(tmp);
        return fail(c, INZG_OOM, "set_router: router buffer");
    }
    if (router_gemm_fits(rows, cols) && !L.router32 &&
        cudaMalloc(&L.router32, sizeof(float) * router32_floats(rows, cols)) != cudaSuccess) {
        cudaFree(tmp);
        return fail(c, INZG_OOM, "set_router: router buffer");
    }
    e = cudaMemcpyAsync(tmp, w, bytes, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) {
        launch_router_repack(tmp, L.router, rows, cols, c->stream);
        if (L.router32) launch_router_repack32(tmp, L.router32, rows, cols, c->stream);
        e = cudaStreamSynchronize(c->stream);
    }
    cudaFree(tmp);
    if (e != cudaSuccess) return cuda_fail(c, e, "set_router");
    L.has_router = true;
    L.dev.router = L.router;
    return INZG_OK;
}

// setup_experts' checks on the file (src/engine.c:339-350), then the pool upload from the mapping
inzg_status inzg_pool_add_layer_gguf(inzg_ctx *c, int layer, const inzg_gguf *g, int gguf_layer) {
    if (!c) return INZG_BAD_ARG;
    inzg_gguf_info info;
    if (inzg_gguf_get_info(g, &info) != INZG_OK) return fail(c, INZG_BAD_ARG, "pool_add_layer_gguf: no GGUF file");
    char name[64];
    if (gguf_layer < info.n_layers) snprintf(name, sizeof(name), "blk.%d.experts", gguf_layer);
    else snprintf(name, sizeof(name), "mtp.experts");
    const void *data = nullptr;
    uint64_t nbytes = 0;
    if (inzg_gguf_experts(g, gguf_layer, &data, &nbytes, nullptr) != INZG_OK)
        return fail(c, INZG_BAD_ARG, std::string("pool_add_layer_gguf: the file has no ") + name);
    if (!info.blob_bytes || info.blob_bytes % 4096)
        return fail(c, INZG_CORRUPT_BLOB, "pool_add_layer_gguf: expert blob size " + std::to_string(info.blob_bytes) +
                                              " is not a positive multiple of 4096");
    if (nbytes / info.blob_bytes < (uint64_t)c->cfg.n_expert)
        return fail(c, INZG_CORRUPT_BLOB, std::string("pool_add_layer_gguf: missing or short ") + name);
    return inzg_pool_add_layer(c, layer, info.expert_type, data, info.blob_bytes, c->cfg.n_expert);
}

inzg_status inzg_pool_add_layer(inzg_ctx *c, int layer, int type, const void *blobs, uint64_t blob_bytes, int n_expert) {
    if (!c) return INZG_BAD_ARG;
    if (n_expert != c->cfg.n_expert) return fail(c, INZG_BAD_ARG, "pool_add_layer: n_expert differs from the context");
    return inzg_pool_add_layer_range(c, layer, type, blobs, blob_bytes, 0, n_expert);
}

// Validate, upload and re-lay out experts [e_first, e_first + n_local) into slot L (a layer's routed pool, or a
// layer's shared expert as a one-expert pool).
static inzg_status load_pool(inzg_ctx *c, LayerSlot &L, int type, const void *blobs, uint64_t blob_bytes, int e_first,
                             int n_local, bool dev_src = false) {
    const inzg_config &cf = c->cfg;
    if (e_first < 0 || n_local < 1 || e_first + n_local > cf.n_expert)
        return fail(c, INZG_BAD_ARG, "pool_add_layer: expert range outside the layer's experts");
    if (type != INZG_T_Q4L && type != INZG_T_Q8G)
        return fail(c, INZG_UNSUPPORTED, "pool_add_layer: expert type must be Q4L or Q8G");
    const int H = cf.hidden, FF = cf.ff, E = n_local;
    const uint64_t gu_bytes = inzg_qmat_bytes(type, 2 * FF, H), dn_bytes = inzg_qmat_bytes(type, H, FF);
    if (blob_bytes < gu_bytes + dn_bytes) return fail(c, INZG_BAD_ARG, "pool_add_layer: blob smaller than its matrices");
    // validate every blob the way q_bind_lin does (src/model_fwd.c:87-96, 853-855): magic, type, rows, cols
    const uint8_t *b = static_cast<const uint8_t *>(blobs);
    std::vector<QHeader> dev_hdr;  // device blobs: their two headers copied to the host first
    if (dev_src) {
        cudaSetDevice(cf.device);
        dev_hdr.resize((size_t)2 * E);
        if (cudaMemcpy2D(dev_hdr.data(), 2 * sizeof(QHeader), b, blob_bytes, 64, E, cudaMemcpyDeviceToHost) !=
                cudaSuccess ||
            cudaMemcpy2D(dev_hdr.data() + 1, 2 * sizeof(QHeader), b + gu_bytes, blob_bytes, 64, E,
                         cudaMemcpyDeviceToHost) != cudaSuccess) {
            cudaGetLastError();
            return fail(c, INZG_BAD_ARG, "pool_add_layer_device: blobs are not readable device memory");
        }
    }
    auto header = [&](int e, bool down, QHeader &h) {
        if (dev_src) h = dev_hdr[(size_t)2 * e + (down ? 1 : 0)];
        else memcpy(&h, b + (size_t)e * blob_bytes + (down ? gu_bytes : 0), 64);
    };
    QHeader h0g, h0d;
    header(0, false, h0g);
    header(0, true, h0d);
    for (int e = 0; e < E; e++) {
        QHeader hg, hd;
        header(e, false, hg);
        header(e, true, hd);
        if (hg.magic != kMagic || hd.magic != kMagic || hg.type != type || hd.type != type || hg.rows != (uint32_t)(2 * FF) ||
            hg.cols != (uint32_t)H || hd.rows != (uint32_t)H || hd.cols != (uint32_t)FF) {
            char msg[128];
            snprintf(msg, sizeof(msg), "expert blob is corrupt (expert %d)", e_first + e);
            return fail(c, INZG_CORRUPT_BLOB, msg);
        }
        // one activation quantization per layer input needs one rotation for all experts' gate|up (and down)
        if (hg.rot_block != h0g.rot_block || hg.rot_seed != h0g.rot_seed || hd.rot_block != h0d.rot_block ||
            hd.rot_seed != h0d.rot_seed)
            return fail(c, INZG_UNSUPPORTED, "pool_add_layer: experts of one layer must share their rotations");
    }
    if ((h0g.rot_block > 1 && H % h0g.rot_block) || (h0d.rot_block > 1 && FF % h0d.rot_block))
        return fail(c, INZG_CORRUPT_BLOB, "pool_add_layer: rotation block does not divide the matrix width");
    cudaSetDevice(cf.device);
    drop_graphs(c);
    LayerDev &D = L.dev;
    L.e_first = e_first;
    D.type = type;
    D.H = H;
    D.FF = FF;
    D.E = E;
    D.gu = make_layout(type, 2 * FF, H);
    D.dn = make_layout(type, H, FF);
    if (D.gu.rows % 16 || D.dn.rows % 16)
        return fail(c, INZG_UNSUPPORTED, "pool_add_layer: matrix rows must be a multiple of 16");
    const uint64_t gb = type == INZG_T_Q8G ? 64 : 32;
    D.gu.q_off = 0;
    D.gu.d_off = align_up(D.gu.q_off + (uint64_t)D.gu.rows * D.gu.ng * gb, 256);
    D.dn.q_off = align_up(D.gu.d_off + (uint64_t)D.gu.rows * D.gu.gd * 4 * 2, 256);
    D.dn.d_off = align_up(D.dn.q_off + (uint64_t)D.dn.rows * D.dn.ng * gb, 256);
    D.slab_bytes = align_up(D.dn.d_off + (uint64_t)D.dn.rows * D.dn.gd * 4 * 2, 256);
    D.gu_rot = h0g.rot_block;
    D.gu_seed = h0g.rot_seed;
    D.dn_rot = h0d.rot_block;
    D.dn_seed = h0d.rot_seed;
    if (L.pool) { cudaFree(L.pool); L.pool = nullptr; }
    if (L.luts) { cudaFree(L.luts); L.luts = nullptr; }
    if (L.gemm_w) { cudaFree(L.gemm_w); L.gemm_w = nullptr; }
    L.has_experts = false;
    if (cudaMalloc(&L.pool, D.slab_bytes * E) != cudaSuccess || cudaMalloc(&L.luts, (size_t)E * 32) != cudaSuccess) {
        cudaGetLastError();
        return fail(c, INZG_OOM, "pool_add_layer: pool allocation");
    }
    D.pool = L.pool;
    D.luts = L.luts;
    {   // prefill-path copy: int8 weights + block scales
        const uint64_t ngu = (uint64_t)E * 2 * FF * H, ndn = (uint64_t)E * H * FF;
        const uint64_t sgu = (uint64_t)E * 2 * FF * ((H + kKB - 1) / kKB), sdn = (uint64_t)E * H * ((FF + kKB - 1) / kKB);
        const uint64_t o_dn = align_up(ngu, 256), o_sgu = align_up(o_dn + ndn, 256), o_sdn = align_up(o_sgu + 4 * sgu, 256);
        if (cudaMalloc(&L.gemm_w, o_sdn + 4 * sdn) != cudaSuccess) {
            cudaGetLastError();
            return fail(c, INZG_OOM, "pool_add_layer: prefill weight allocation");
        }
        D.w8_gu = reinterpret_cast<int8_t *>(L.gemm_w);
        D.w8_dn = reinterpret_cast<int8_t *>(L.gemm_w + o_dn);
        D.ws_gu = reinterpret_cast<float *>(L.gemm_w + o_sgu);
        D.ws_dn = reinterpret_cast<float *>(L.gemm_w + o_sdn);
    }
    cudaMemsetAsync(L.pool, 0, D.slab_bytes * E, c->stream);  // scale padding past ng stays zero
    // stage blobs through a device buffer in chunks of experts and re-lay them out on the device
    // device blobs: re-laid out in place of the source; host blobs: staged through a device buffer in chunks
    const int chunk = std::min(E, 32);
    uint8_t *stage = nullptr;
    if (!dev_src && cudaMalloc(&stage, blob_bytes * chunk) != cudaSuccess) {
        cudaGetLastError();
        return fail(c, INZG_OOM, "pool_add_layer: staging buffer");
    }
    cudaError_t err = cudaSuccess;
    for (int e0 = 0; e0 < E && err == cudaSuccess; e0 += chunk) {
        const int ne = std::min(chunk, E - e0);
        const uint8_t *src = dev_src ? b + (size_t)e0 * blob_bytes : stage;
        if (!dev_src)
            err = cudaMemcpyAsync(stage, b + (size_t)e0 * blob_bytes, blob_bytes * ne, cudaMemcpyHostToDevice, c->stream);
        if (err == cudaSuccess) {
            launch_pool_repack(src, blob_bytes, gu_bytes, e0, ne, D, L.pool, L.luts, c->stream);
            launch_pool_requant(src, blob_bytes, gu_bytes, e0, ne, D, c->stream);
        }
        if (err == cudaSuccess) err = cudaStreamSynchronize(c->stream);
    }
    if (stage) cudaFree(stage);
    if (err != cudaSuccess) return cuda_fail(c, err, "pool_add_layer");
    L.has_maps = make_tma_map_i8(L.map_gu.bytes, D.w8_gu, (uint64_t)E * 2 * FF, H, 128) &&
                 make_tma_map_i8(L.map_dn.bytes, D.w8_dn, (uint64_t)E * H, FF, 128) &&
                 make_tma_map_i8(L.map16_gu.bytes, D.w8_gu, (uint64_t)E * 2 * FF, H, 16) &&
                 make_tma_map_i8(L.map16_dn.bytes, D.w8_dn, (uint64_t)E * H, FF, 16);
    err = cudaGetLastError();
    if (err != cudaSuccess) return cuda_fail(c, err, "pool_add_layer repack");
    L.has_experts = true;
    c->stats.pool_bytes = 0;
    for (auto *v : {&c->layers, &c->shared})
        for (auto &S : *v)
            if (S.has_experts) c->stats.pool_bytes += S.dev.slab_bytes * S.dev.E;
    return INZG_OK;
}

inzg_status inzg_pool_add_layer_range(inzg_ctx *c, int layer, int type, const void *blobs, uint64_t blob_bytes,
                                      int e_first, int n_local) {
    if (!c) return INZG_BAD_ARG;
    if (layer < 0 || layer >= c->cfg.n_layers || !blobs) return fail(c, INZG_BAD_ARG, "pool_add_layer: bad layer or pointer");
    return load_pool(c, c->layers[layer], type, blobs, blob_bytes, e_first, n_local);
}

inzg_status inzg_pool_add_layer_device(inzg_ctx *c, int layer, int type, const void *blobs_dev, uint64_t blob_bytes,
                                       int e_first, int n_local) {
    if (!c) return INZG_BAD_ARG;
    if (layer < 0 || layer >= c->cfg.n_layers || !blobs_dev)
        return fail(c, INZG_BAD_ARG, "pool_add_layer_device: bad layer or pointer");
    return load_pool(c, c->layers[layer], type, blobs_dev, blob_bytes, e_first, n_local, true);
}

inzg_status inzg_set_shared(inzg_ctx *c, int layer, int type, const void *blob, uint64_t blob_bytes, const float *gate) {
    if (!c) return INZG_BAD_ARG;
    const inzg_config &cf = c->cfg;
    if (layer < 0 || layer >= cf.n_layers || !blob || !gate)
        return fail(c, INZG_BAD_ARG, "set_shared: bad layer or pointer");
    const inzg_status st = load_pool(c, c->shared[layer], type, blob, blob_bytes, 0, 1);
    if (st != INZG_OK) return st;
    if (!c->sh_gate[layer] && cudaMalloc(&c->sh_gate[layer], sizeof(float) * cf.hidden) != cudaSuccess) {
        cudaGetLastError();
        c->shared[layer].has_experts = false;
        return fail(c, INZG_OOM, "set_shared: gate vector");
    }
    const cudaError_t e = cudaMemcpy(c->sh_gate[layer], gate, sizeof(float) * cf.hidden, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(c, e, "set_shared");
    return INZG_OK;
}

// The shared expert of layer `layer` on X [n][H], adding sigmoid(gate . x) * D into y (src/model_fwd.c:1041-1069,
// 1141-1148). n_rule: the batch size of the lin_mm path rule (decode below GEMM_MIN_T tokens). quantized: X's
// gate|up quantization for both numeric paths is already in the scratch with this rotation (the routed part's).
static int enqueue_shared(inzg_ctx *c, int layer, int n, const float *X, float *y, int n_rule, bool quantized,
                          cudaStream_t st) {
    const inzg_config &cf = c->cfg;
    const LayerSlot &S = c->shared[layer];
    const LayerDev &D = S.dev;
    const int H = cf.hidden, FF = cf.ff;
    const int gemm = n_rule >= kGemmMinT;
    int launches = 0;
    bool bad = false;
    auto add = [&](int r) {  // a launcher that has no kernel for the shape fails the call (no silent skip)
        if (r < 0) bad = true;
        else launches += r;
    };
    if (!quantized)
        add(launch_act_quant_x(X, n, H, D.gu_rot, D.gu_seed, c->xq64, c->xsb64, gemm ? c->xq256 : nullptr,
                                       c->xs256, st));
    RouteDev R{};
    R.n = n; R.topk = 1; R.E = 1; R.n_rule = n_rule; R.absent_ok = 0;
    R.cnt = c->sh_cnt; R.off = c->sh_off; R.first = c->sh_first; R.etok = c->sh_etok; R.eslot = c->sh_eslot;
    R.ew = c->sh_ew; R.units = c->sh_units; R.meta = c->sh_meta; R.dec_units = c->sh_dec; R.gemm_units = c->sh_gemm;
    R.gemm_tiles = c->sh_tiles;
    add(launch_shared_route(R, n, gemm, gemv_items_per_unit(D, 0, R.n), gemv_items_per_unit(D, 1, R.n), gemm_token_tile(),
                                    c->sh_upath, c->sh_eexp, st));
    const bool tc = c->have_tc && S.has_maps;
    if (gemm && !tc) return -2;  // the prefill GEMM needs its tensor maps: no silent CUDA-core fallback
    const int max_tiles = (n + gemm_token_tile() - 1) / gemm_token_tile() + 1;
    const int grid = c->num_sms * 4;
    if (!gemm) {
        add(launch_gemv_decode(D, 0, R, c->xq64, c->xsb64, c->GU, 2 * FF, c->num_sms, st));
    } else if (tc) {
        add(launch_gather_gemm_rows(c->xq256, c->xs256, H, (H + kKB - 1) / kKB, c->sh_etok, c->sh_eexp,
                                            c->sh_upath, n, c->xqe, c->xse, st));
        add(launch_gemm_tc(0, S.map_gu.bytes, c->map_xqe.bytes, D.ws_gu, 2 * FF, H, R, c->xse, c->GU, 2 * FF,
                                   max_tiles, st));
    } else {
        add(launch_gemm_v1(D, 0, R, c->xq256, c->xs256, c->GU, 2 * FF, grid, st));
    }
    add(launch_swiglu_quant(c->GU, FF, n, c->sh_eexp, c->sh_upath, D.dn_rot, D.dn_seed, c->dq64, c->dsb64,
                                    c->dq256, c->ds256, st));
    if (!gemm) add(launch_gemv_decode(D, 1, R, c->dq64, c->dsb64, c->mo, H, c->num_sms, st));
    else if (tc) add(launch_gemm_tc(1, S.map_dn.bytes, c->map_dq.bytes, D.ws_dn, H, FF, R, c->ds256, c->mo, H,
                                           max_tiles, st));
    else add(launch_gemm_v1(D, 1, R, c->dq256, c->ds256, c->mo, H, grid, st));
    add(launch_shared_add(X, c->sh_gate[layer], c->mo, y, n, H, c->sh_meta, c->meta, st));
    return bad ? -1 : launches;
}

// Enqueue the whole layer on `st`. ev != nullptr: record ev[i] before stage i and ev[N] at the end.
static int enqueue_forward(inzg_ctx *c, int layer, const LayerSlot &L, int n, const float *X, float *yd, const float *bias,
                           const float *ovr, bool ovr_on_device, bool dump, bool simt_gemm, bool no_fused,
                           cudaEvent_t *ev, cudaStream_t st) {
    const inzg_config &cf = c->cfg;
    const int H = cf.hidden, E = cf.n_expert, K = cf.topk, FF = cf.ff;
    const int NE = n * K;
    const LayerDev &D = L.dev;
    int launches = 0;
    bool bad = false;
    auto add = [&](int r) {  // a launcher that has no kernel for the shape fails the call (no silent skip)
        if (r < 0) bad = true;
        else launches += r;
    };
    auto mark = [&](int i) {
        if (ev) cudaEventRecord(ev[i], st);
    };
    auto shared_stage = [&]() -> int {  // y += sigmoid(gate . x) * shared(x), after the routed sum (:1141-1148)
        if (!c->shared[layer].has_experts) return 0;
        const LayerDev &S = c->shared[layer].dev;
        const bool same_rot = S.gu_rot == D.gu_rot && S.gu_seed == D.gu_seed;
        return enqueue_shared(c, layer, n, X, yd, n, same_rot, st);
    };
    // Decode calls of up to 8 tokens: the whole routed layer as one persistent launch (k_fused.cu). The logits
    // override of a host call was copied into c->logits by the caller.
    if (!no_fused && fused_decode_fits(D, n, K, L.has_router || ovr)) {
        for (int i = 0; i <= 10; i++) mark(i);
        const float *ov = ovr ? (ovr_on_device ? ovr : c->logits) : nullptr;
        add(launch_fused_decode(D, n, K, X, ov ? nullptr : bias, ov, c->logits, dump ? c->probs : nullptr, c->sel, c->w,
                                c->units, c->meta, c->xq64, c->xsb64, c->GU, c->dq64, c->dsb64, c->mo, yd,
                                c->fused_cnt, c->num_sms, st));
        mark(11);
        const int r = shared_stage();
        if (r == -2) return -2;
        add(r);
        mark(12);
        return bad ? -1 : launches;
    }
    const bool any_gemm = n > 8 && (int64_t)n * K >= kGemmMinT;
    // the inputs' quantization (both numeric paths) depends on x only: a side branch when not profiling
    const bool branch = ev == nullptr;
    if (branch) {
        cudaEventRecord(c->fork, st);
        cudaStreamWaitEvent(c->side, c->fork, 0);
        add(launch_act_quant_x(X, n, H, D.gu_rot, D.gu_seed, c->xq64, c->xsb64, any_gemm ? c->xq256 : nullptr,
                                       c->xs256, c->side));
        cudaEventRecord(c->join, c->side);
    }
    mark(0);
    if (ovr) {
        if (ovr_on_device)
            cudaMemcpyAsync(c->logits, ovr, sizeof(float) * (size_t)n * E, cudaMemcpyDeviceToDevice, st);
    } else {
        add(launch_router_logits(L.router, L.router32, X, n, H, E, bias, c->logits, c->meta, st));
    }
    mark(1);
    RouteDev R{};
    R.n = n; R.topk = K; R.E = E; R.n_rule = n; R.absent_ok = 0;
    R.sel = c->sel; R.w = c->w; R.cnt = c->cnt; R.off = c->off; R.first = c->first; R.etok = c->etok; R.eslot = c->eslot;
    R.ew = c->ew; R.ccnt = c->ccnt; R.cmask = c->cmask; R.units = c->units; R.meta = c->meta; R.dec_units = c->dec_units;
    R.gemm_units = c->gemm_units; R.gemm_tiles = c->gemm_tiles;
    const bool tc = !simt_gemm && c->have_tc && L.has_maps;
    // the prefill GEMM runs on tcgen05 unless the caller asked for the CUDA-core cross-check (INZG_GEMM_SIMT); a
    // context without tensor maps fails the call instead of falling back silently
    if (any_gemm && !simt_gemm && !tc) return -2;
    // decode-sized calls: the prefill-numerics experts run inside the decode GEMV launches as 16-token GEMM items
    const bool in_gemv = any_gemm && tc && n <= kGemvGemmMaxTokens;
    const int gtile = in_gemv ? kGemvGemmTile : gemm_token_tile();
    const DecGemm gm_gu{c->xq256, c->xs256, D.ws_gu, L.map16_gu.bytes}, gm_dn{c->dq256, c->ds256, D.ws_dn,
                                                                               L.map16_dn.bytes};
    const int fused = launch_route_fused(R, c->logits, dump ? c->probs : nullptr, gemv_items_per_unit(D, 0, R.n), gemv_items_per_unit(D, 1, R.n),
                                         gtile, c->upath, c->eexp, st);
    if (fused > 0) {
        add(fused);
        mark(2);
    } else {
        add(launch_softmax_topk(c->logits, n, E, K, c->sel, c->w, dump ? c->probs : nullptr, st));
        mark(2);
    }
    if (!branch)
        add(launch_act_quant_x(X, n, H, D.gu_rot, D.gu_seed, c->xq64, c->xsb64, any_gemm ? c->xq256 : nullptr,
                                       c->xs256, st));
    mark(3);
    if (fused <= 0) add(launch_route(R, gemv_items_per_unit(D, 0, R.n), gemv_items_per_unit(D, 1, R.n), gtile, c->upath, c->eexp, st));
    const int nkbH = (H + kKB - 1) / kKB;
    const int max_tiles = (NE + gemm_token_tile() - 1) / gemm_token_tile() + std::min(E, NE / kGemmMinT) + 1;
    if (branch) cudaStreamWaitEvent(st, c->join, 0);
    mark(4);
    const int grid = c->num_sms * 4;
    add(launch_gemv_decode(D, 0, R, c->xq64, c->xsb64, c->GU, 2 * FF, c->num_sms, st, in_gemv ? &gm_gu : nullptr));
    mark(5);
    if (any_gemm && !in_gemv) {
        if (tc) {
            add(launch_gather_gemm_rows(c->xq256, c->xs256, H, nkbH, c->etok, c->eexp, c->upath, NE, c->xqe,
                                                c->xse, st));
            add(launch_gemm_tc(0, L.map_gu.bytes, c->map_xqe.bytes, D.ws_gu, 2 * FF, H, R, c->xse, c->GU,
                                       2 * FF, max_tiles, st));
        } else {
            add(launch_gemm_v1(D, 0, R, c->xq256, c->xs256, c->GU, 2 * FF, grid, st));
        }
    }
    mark(6);
    add(launch_swiglu_quant(c->GU, FF, NE, c->eexp, c->upath, D.dn_rot, D.dn_seed, c->dq64, c->dsb64, c->dq256,
                                    c->ds256, st));
    mark(7);
    add(launch_gemv_decode(D, 1, R, c->dq64, c->dsb64, c->mo, H, c->num_sms, st, in_gemv ? &gm_dn : nullptr));
    mark(8);
    if (any_gemm && !in_gemv) {
        if (tc) add(launch_gemm_tc(1, L.map_dn.bytes, c->map_dq.bytes, D.ws_dn, H, FF, R, c->ds256, c->mo, H,
                                           max_tiles, st));
        else add(launch_gemm_v1(D, 1, R, c->dq256, c->ds256, c->mo, H, grid, st));
    }
    mark(9);
    add(launch_combine(c->mo, n, H, K, yd, c->num_sms, st));
    mark(10);
    mark(11);
    const int r = shared_stage();
    if (r == -2) return -2;
    add(r);
    mark(12);
    return bad ? -1 : launches;
}

inzg_status inzg_moe_forward(inzg_ctx *c, int layer, int n, const float *xin, float *y, const inzg_moe_opts *opt) {
    if (!c) return INZG_BAD_ARG;
    const inzg_config &cf = c->cfg;
    if (layer < 0 || layer >= cf.n_layers) return fail(c, INZG_BAD_ARG, "moe_forward: bad layer");
    if (n <= 0 || n > cf.max_tokens || !xin || !y) return fail(c, INZG_BAD_ARG, "moe_forward: bad n or pointer");
    LayerSlot &L = c->layers[layer];
    const unsigned flags = opt ? opt->flags : 0;
    const bool dev_io = flags & INZG_IO_DEVICE, dump = flags & INZG_DUMP_ROUTE, profile = flags & INZG_PROFILE;
    const float *ovr = opt ? opt->logits_override : nullptr;
    const float *bias = opt ? opt->logit_bias : nullptr;
    if (!L.has_experts || (!L.has_router && !ovr)) return fail(c, INZG_NOT_READY, "moe_forward: layer not loaded");
    if (L.e_first != 0 || L.dev.E != cf.n_expert)
        return fail(c, INZG_NOT_READY, "moe_forward: the pool holds a subset of the experts (use inzg_moe_experts)");
    // the kernels move token rows with 16-byte vector loads and bulk copies
    if (dev_io && ((reinterpret_cast<uintptr_t>(xin) | reinterpret_cast<uintptr_t>(y) |
                    reinterpret_cast<uintptr_t>(ovr)) & 15))
        return fail(c, INZG_BAD_ARG, "moe_forward: device xin, y and logits_override must be 16-byte aligned");
    cudaSetDevice(cf.device);
    cudaStream_t st = opt && opt->stream ? static_cast<cudaStream_t>(opt->stream) : c->stream;
    const int H = cf.hidden, E = cf.n_expert;
    const LayerDev &D = L.dev;
    if (launch_gemv_decode(D, -1, RouteDev{}, nullptr, nullptr, nullptr, 0, 0, st) < 0)
        return fail(c, INZG_UNSUPPORTED, "moe_forward: no decode kernel for this geometry");
    cudaError_t e = cudaSuccess;
    const float *X = xin;
    if (!dev_io) {  // host buffers: stage into the context's device buffers (outside any graph)
        e = cudaMemcpyAsync(c->xin, xin, sizeof(float) * (size_t)n * H, cudaMemcpyHostToDevice, st);
        X = c->xin;
        if (e == cudaSuccess && bias) {
            e = cudaMemcpyAsync(c->bias, bias, sizeof(float) * E, cudaMemcpyHostToDevice, st);
            bias = c->bias;
        }
        if (e == cudaSuccess && ovr)
            e = cudaMemcpyAsync(c->logits, ovr, sizeof(float) * (size_t)n * E, cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) return cuda_fail(c, e, "moe_forward: input copy");
    }
    float *yd = dev_io ? y : c->y;
    int launches = 0;
    if (profile || (flags & INZG_NO_GRAPH)) {
        launches = enqueue_forward(c, layer, L, n, X, yd, bias, ovr, dev_io, dump, flags & INZG_GEMM_SIMT,
                                   flags & INZG_NO_FUSED,
                                   profile ? c->ev : nullptr, st);
    } else {
        inzg_ctx::GraphKey key{layer, n, X, yd, bias, ovr,
                               flags & (INZG_IO_DEVICE | INZG_DUMP_ROUTE | INZG_GEMM_SIMT | INZG_NO_FUSED), 0};
        inzg_ctx::GraphEntry *g = nullptr;
        for (auto &ge : c->graphs)
            if (ge.key == key) g = &ge;
        if (!g) {
            cudaStream_t cs = c->capture_stream;
            e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
            if (e != cudaSuccess) return cuda_fail(c, e, "moe_forward: begin capture");
            const int nl = enqueue_forward(c, layer, L, n, X, yd, bias, ovr, dev_io, dump, flags & INZG_GEMM_SIMT,
                                           flags & INZG_NO_FUSED, nullptr, cs);
            cudaGraph_t graph = nullptr;
            e = cudaStreamEndCapture(cs, &graph);
            if (e != cudaSuccess || nl < 0) {
                if (graph) cudaGraphDestroy(graph);
                return e != cudaSuccess ? cuda_fail(c, e, "moe_forward: capture")
                       : nl == -2       ? fail(c, INZG_UNSUPPORTED, "moe_forward: no tensor maps for the prefill GEMM")
                                        : fail(c, INZG_UNSUPPORTED, "moe_forward: no kernel for this shape");
            }
            cudaGraphExec_t exec = nullptr;
            e = cudaGraphInstantiate(&exec, graph, 0);
            cudaGraphDestroy(graph);
            if (e != cudaSuccess) return cuda_fail(c, e, "moe_forward: graph instantiate");
            if (c->graphs.size() >= 64) {  // evict the least recently used
                auto it = std::min_element(c->graphs.begin(), c->graphs.end(),
                                           [](const inzg_ctx::GraphEntry &a, const inzg_ctx::GraphEntry &b) {
                                               return a.last_use < b.last_use;
                                           });
                cudaGraphExecDestroy(it->exec);
                c->graphs.erase(it);
            }
            c->graphs.push_back({key, exec, nl, 0});
            g = &c->graphs.back();
        }
        g->last_use = ++c->use_clock;
        launches = g->launches;
        e = cudaGraphLaunch(g->exec, st);
        if (e != cudaSuccess) return cuda_fail(c, e, "moe_forward: graph launch");
    }
    if (launches == -2) return fail(c, INZG_UNSUPPORTED, "moe_forward: no tensor maps for the prefill GEMM");
    if (launches < 0) return fail(c, INZG_UNSUPPORTED, "moe_forward: no kernel for this geometry");
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, "moe_forward: kernel launch");
    c->stats.calls++;
    c->stats.tokens += n;
    c->stats.last_launches = launches;
    c->last_n = n;
    c->last_dump = dump;
    if (profile) {
        e = cudaEventSynchronize(c->ev[INZG_N_STAGES]);
        if (e != cudaSuccess) return cuda_fail(c, e, "moe_forward: profile");
        for (int i = 0; i < INZG_N_STAGES; i++) {
            float ms = 0;
            cudaEventElapsedTime(&ms, c->ev[i], c->ev[i + 1]);
            c->stage_ms[i] += ms;
        }
        c->profiled_calls++;
    }
    if (!dev_io) {
        e = cudaMemcpyAsync(y, c->y, sizeof(float) * (size_t)n * H, cudaMemcpyDeviceToHost, st);
        int32_t meta[16];
        if (e == cudaSuccess) e = cudaMemcpyAsync(meta, c->meta, sizeof(meta), cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) return cuda_fail(c, e, "moe_forward");
        if (meta[kMetaError] != kErrNone) {
            char msg[96];
            snprintf(msg, sizeof(msg), "moe_forward: device check failed (code %d)", meta[kMetaError]);
            return fail(c, meta[kMetaError] == kErrTimeout ? INZG_TIMEOUT : INZG_DEVICE_CHECK, msg);
        }
    }
    return INZG_OK;
}

// ---------------------------------------------------------------------------------------------------------------
// Expert-parallel building blocks. A rank routes its own tokens (inzg_route), ships each token's row to the ranks
// owning its experts, runs the experts it owns on the rows it received (inzg_moe_experts: the same kernels as the
// whole-layer forward, entries of other ranks marked absent), ships the per-slot outputs home and combines them in
// rank order (inzg_combine). Every expert sees exactly the tokens it would see on one GPU, so its numeric path and
// its outputs are the single-GPU ones bit for bit.

inzg_status inzg_route(inzg_ctx *c, int layer, int n, const float *x_dev, const float *logit_bias_dev, int32_t *sel_dev,
                       float *w_dev, void *stream) {
    if (!c) return INZG_BAD_ARG;
    const inzg_config &cf = c->cfg;
    if (layer < 0 || layer >= cf.n_layers) return fail(c, INZG_BAD_ARG, "route: bad layer");
    if (n <= 0 || n > cf.max_tokens || !x_dev || !sel_dev || !w_dev) return fail(c, INZG_BAD_ARG, "route: bad n or pointer");
    if (reinterpret_cast<uintptr_t>(x_dev) & 15) return fail(c, INZG_BAD_ARG, "route: x must be 16-byte aligned");
    LayerSlot &L = c->layers[layer];
    if (!L.has_router) return fail(c, INZG_NOT_READY, "route: layer has no router");
    cudaSetDevice(cf.device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    launch_router_logits(L.router, L.router32, x_dev, n, cf.hidden, cf.n_expert, logit_bias_dev, c->logits, c->meta,
                         st);
    launch_softmax_topk(c->logits, n, cf.n_expert, cf.topk, sel_dev, w_dev, nullptr, st);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? INZG_OK : cuda_fail(c, e, "route: kernel launch");
}

// The experts of the context's pool on m token rows (the body of inzg_moe_experts and of an expert-parallel step):
// launches, or -1 (a launcher has no kernel for the shape) / -2 (the prefill GEMM has no tensor maps).
static int enqueue_experts(inzg_ctx *c, LayerSlot &L, int m, const float *x_dev, const int32_t *sel_dev,
                           const float *w_dev, int n_batch, float *out_dev, cudaStream_t st) {
    const inzg_config &cf = c->cfg;
    const LayerDev &D = L.dev;
    const int H = cf.hidden, K = cf.topk, FF = cf.ff, E = D.E;
    const int NE = m * K;
    const bool any_gemm = n_batch > 8 && NE >= kGemmMinT;
    const bool tc = c->have_tc && L.has_maps;
    if (any_gemm && !tc) return -2;
    int launches = 0;
    bool bad = false;
    auto add = [&](int r) {
        if (r < 0) bad = true;
        else launches += r;
    };
    add(launch_act_quant_x(x_dev, m, H, D.gu_rot, D.gu_seed, c->xq64, c->xsb64, any_gemm ? c->xq256 : nullptr,
                           c->xs256, st));
    RouteDev R{};
    R.n = m; R.topk = K; R.E = E; R.n_rule = n_batch; R.absent_ok = 1;
    R.sel = const_cast<int32_t *>(sel_dev); R.w = const_cast<float *>(w_dev);
    R.cnt = c->cnt; R.off = c->off; R.first = c->first; R.etok = c->etok; R.eslot = c->eslot;
    R.ew = c->ew; R.ccnt = c->ccnt; R.cmask = c->cmask; R.units = c->units; R.meta = c->meta; R.dec_units = c->dec_units;
    R.gemm_units = c->gemm_units; R.gemm_tiles = c->gemm_tiles;
    const bool in_gemv = any_gemm && m <= kGemvGemmMaxTokens;  // GEMM items inside the decode GEMV launches
    add(launch_route(R, gemv_items_per_unit(D, 0, R.n), gemv_items_per_unit(D, 1, R.n),
                     in_gemv ? kGemvGemmTile : gemm_token_tile(), c->upath, c->eexp, st));
    const DecGemm gm_gu{c->xq256, c->xs256, D.ws_gu, L.map16_gu.bytes}, gm_dn{c->dq256, c->ds256, D.ws_dn,
                                                                               L.map16_dn.bytes};
    const int nkbH = (H + kKB - 1) / kKB;
    const int max_tiles = (NE + gemm_token_tile() - 1) / gemm_token_tile() + std::min(E, NE / kGemmMinT) + 1;
    add(launch_gemv_decode(D, 0, R, c->xq64, c->xsb64, c->GU, 2 * FF, c->num_sms, st, in_gemv ? &gm_gu : nullptr));
    if (any_gemm && !in_gemv) {
        add(launch_gather_gemm_rows(c->xq256, c->xs256, H, nkbH, c->etok, c->eexp, c->upath, NE, c->xqe, c->xse, st));
        add(launch_gemm_tc(0, L.map_gu.bytes, c->map_xqe.bytes, D.ws_gu, 2 * FF, H, R, c->xse, c->GU, 2 * FF,
                           max_tiles, st));
    }
    add(launch_swiglu_quant(c->GU, FF, NE, c->eexp, c->upath, D.dn_rot, D.dn_seed, c->dq64, c->dsb64, c->dq256,
                            c->ds256, st));
    add(launch_gemv_decode(D, 1, R, c->dq64, c->dsb64, out_dev, H, c->num_sms, st, in_gemv ? &gm_dn : nullptr));
    if (any_gemm && !in_gemv)
        add(launch_gemm_tc(1, L.map_dn.bytes, c->map_dq.bytes, D.ws_dn, H, FF, R, c->ds256, out_dev, H, max_tiles, st));
    return bad ? -1 : launches;
}

inzg_status inzg_moe_experts(inzg_ctx *c, int layer, int m, const float *x_dev, const int32_t *sel_dev,
                             const float *w_dev, int n_batch, float *out_dev, void *stream) {
    if (!c) return INZG_BAD_ARG;
    const inzg_config &cf = c->cfg;
    if (layer < 0 || layer >= cf.n_layers) return fail(c, INZG_BAD_ARG, "moe_experts: bad layer");
    if (m <= 0 || m > cf.max_tokens || n_batch < 1 || !x_dev || !sel_dev || !w_dev || !out_dev)
        return fail(c, INZG_BAD_ARG, "moe_experts: bad m, n_batch or pointer");
    if ((reinterpret_cast<uintptr_t>(x_dev) | reinterpret_cast<uintptr_t>(out_dev)) & 15)
        return fail(c, INZG_BAD_ARG, "moe_experts: x and out must be 16-byte aligned");
    LayerSlot &L = c->layers[layer];
    if (!L.has_experts) return fail(c, INZG_NOT_READY, "moe_experts: layer has no experts");
    cudaSetDevice(cf.device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    if (launch_gemv_decode(L.dev, -1, RouteDev{}, nullptr, nullptr, nullptr, 0, 0, st) < 0)
        return fail(c, INZG_UNSUPPORTED, "moe_experts: no decode kernel for this geometry");
    const int r = enqueue_experts(c, L, m, x_dev, sel_dev, w_dev, n_batch, out_dev, st);
    if (r == -2) return fail(c, INZG_UNSUPPORTED, "moe_experts: no tensor maps for the prefill GEMM");
    if (r < 0) return fail(c, INZG_UNSUPPORTED, "moe_experts: no kernel for this shape");
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? INZG_OK : cuda_fail(c, e, "moe_experts: kernel launch");
}

inzg_status inzg_combine(inzg_ctx *c, int n, const float *slots_dev, float *y_dev, void *stream) {
    if (!c) return INZG_BAD_ARG;
    const inzg_config &cf = c->cfg;
    if (n <= 0 || !slots_dev || !y_dev) return fail(c, INZG_BAD_ARG, "combine: bad n or pointer");
    if ((reinterpret_cast<uintptr_t>(slots_dev) | reinterpret_cast<uintptr_t>(y_dev)) & 15)
        return fail(c, INZG_BAD_ARG, "combine: pointers must be 16-byte aligned");
    cudaSetDevice(cf.device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    launch_combine(slots_dev, n, cf.hidden, cf.topk, y_dev, c->num_sms, st);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? INZG_OK : cuda_fail(c, e, "combine: kernel launch");
}

inzg_status inzg_shared_expert(inzg_ctx *c, int layer, int n, const float *x_dev, float *y_dev, int n_batch,
                               void *stream) {
    if (!c) return INZG_BAD_ARG;
    const inzg_config &cf = c->cfg;
    if (layer < 0 || layer >= cf.n_layers) return fail(c, INZG_BAD_ARG, "shared_expert: bad layer");
    if (n <= 0 || n > cf.max_tokens || n_batch < n || !x_dev || !y_dev)
        return fail(c, INZG_BAD_ARG, "shared_expert: bad n, n_batch or pointer");
    if ((reinterpret_cast<uintptr_t>(x_dev) | reinterpret_cast<uintptr_t>(y_dev)) & 15)
        return fail(c, INZG_BAD_ARG, "shared_expert: pointers must be 16-byte aligned");
    if (!c->shared[layer].has_experts) return fail(c, INZG_NOT_READY, "shared_expert: layer has no shared expert");
    cudaSetDevice(cf.device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    const int r = enqueue_shared(c, layer, n, x_dev, y_dev, n_batch, false, st);
    if (r < 0) return fail(c, INZG_UNSUPPORTED, r == -2 ? "shared_expert: no tensor maps for the prefill GEMM"
                                                        : "shared_expert: no kernel for this shape");
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? INZG_OK : cuda_fail(c, e, "shared_expert: kernel launch");
}

inzg_status inzg_device_status(inzg_ctx *c, void *stream) {
    if (!c) return INZG_BAD_ARG;
    cudaSetDevice(c->cfg.device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    int32_t meta[16];
    cudaError_t e = cudaMemcpyAsync(meta, c->meta, sizeof(meta), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(c, e, "device_status");
    const int code = meta[kMetaError] != kErrNone ? meta[kMetaError] : meta[kMetaRouterError];
    if (code != kErrNone) {
        char msg[96];
        snprintf(msg, sizeof(msg), "device check failed (code %d)", code);
        return fail(c, code == kErrTimeout ? INZG_TIMEOUT : INZG_DEVICE_CHECK, msg);
    }
    if (c->ep && c->ep->err) {  // the exchange's own error word (sticky until read here)
        int32_t ep_err = 0;
        e = cudaMemcpy(&ep_err, c->ep->err, sizeof(ep_err), cudaMemcpyDeviceToHost);
        if (e == cudaSuccess && ep_err != kErrNone) e = cudaMemset(c->ep->err, 0, sizeof(int32_t));
        if (e != cudaSuccess) return cuda_fail(c, e, "device_status");
        if (ep_err != kErrNone) return fail(c, INZG_TIMEOUT, "expert-parallel exchange: a peer did not arrive in time");
    }
    return INZG_OK;
}

// ---------------------------------------------------------------------------------------------------------------
// Expert parallelism over peer memory (k_ep.cu)
// ---------------------------------------------------------------------------------------------------------------
namespace {

// the exported handle: the IPC handle of the rank's buffer, the device's UUID and the exchange's shape
struct EpHandle {
    cudaIpcMemHandle_t ipc;
    unsigned char uuid[16];
    int32_t rank, world, cap, hidden, topk, n_expert;
    unsigned char pad[INZG_EP_HANDLE_BYTES - sizeof(cudaIpcMemHandle_t) - 16 - 6 * sizeof(int32_t)];
};
static_assert(sizeof(EpHandle) == INZG_EP_HANDLE_BYTES, "EP handle size");

void ep_free(EpState *ep) {
    for (void *p : ep->opened)
        if (p) cudaIpcCloseMemHandle(p);
    ep->opened.clear();
    if (ep->base) cudaFree(ep->base);
    if (ep->local) cudaFree(ep->local);
    delete ep;
}

// every peer's regions from its base (all ranks share the layout)
void ep_bind(EpState *ep, int d, uint8_t *b) {
    ep->P.rsel[d] = reinterpret_cast<int32_t *>(b + ep->o_rsel);
    ep->P.rw[d] = reinterpret_cast<float *>(b + ep->o_rw);
    ep->P.rx[d] = reinterpret_cast<float *>(b + ep->o_rx);
    ep->P.out[d] = reinterpret_cast<float *>(b + ep->o_out);
    ep->P.flags[d] = reinterpret_cast<uint32_t *>(b + ep->o_flags);
}

}  // namespace

inzg_status inzg_ep_attach(inzg_ctx *c, int rank, int world, int capacity, void *handle_out) {
    if (!c) return INZG_BAD_ARG;
    const inzg_config &cf = c->cfg;
    if (world < 1 || world > kEpMaxRanks || rank < 0 || rank >= world || capacity < 1 || !handle_out)
        return fail(c, INZG_BAD_ARG, "ep_attach: bad rank, world (1..8), capacity or handle");
    if (cf.n_expert % world) return fail(c, INZG_BAD_ARG, "ep_attach: n_expert must be a multiple of world");
    if ((int64_t)world * capacity > cf.max_tokens)
        return fail(c, INZG_BAD_ARG, "ep_attach: max_tokens must be at least world * capacity");
    if (c->ep) return fail(c, INZG_BAD_ARG, "ep_attach: already attached");
    cudaSetDevice(cf.device);
    const size_t G = world, C = capacity, K = cf.topk, H = cf.hidden;
    EpState *ep = new EpState();
    ep->rank = rank;
    ep->world = world;
    ep->cap = capacity;
    size_t o = 0;
    ep->o_rsel = o; o = align_up(o + G * C * K * 4, 256);
    ep->o_rw = o; o = align_up(o + G * C * K * 4, 256);
    ep->o_rx = o; o = align_up(o + G * C * H * 4, 256);
    ep->o_out = o; o = align_up(o + G * C * K * H * 4, 256);
    ep->o_flags = o; o = align_up(o + 3 * G * 4, 256);
    ep->bytes = o;
    const size_t lb = 256 + align_up(C * K * 4, 256);
    cudaError_t e = cudaMalloc(&ep->base, ep->bytes);
    if (e == cudaSuccess) e = cudaMemset(ep->base, 0, ep->bytes);
    if (e == cudaSuccess) e = cudaMemset(ep->base + ep->o_rsel, 0xFF, G * C * K * 4);  // no slot owned yet
    if (e == cudaSuccess) e = cudaMalloc(&ep->local, lb);
    if (e == cudaSuccess) e = cudaMemset(ep->local, 0, 256);
    EpHandle h{};
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h.ipc, ep->base);
    cudaDeviceProp prop{};
    if (e == cudaSuccess) e = cudaGetDeviceProperties(&prop, cf.device);
    if (e != cudaSuccess) {
        ep_free(ep);
        return cuda_fail(c, e, "ep_attach");
    }
    ep->epoch = reinterpret_cast<uint32_t *>(ep->local);
    ep->tickets = reinterpret_cast<int32_t *>(ep->local + 16);
    ep->err = reinterpret_cast<int32_t *>(ep->local + 32);
    ep->bar_epoch = reinterpret_cast<uint32_t *>(ep->local + 48);
    ep->sel = reinterpret_cast<int32_t *>(ep->local + 256);
    ep->P.rank = rank;
    ep->P.world = world;
    ep->P.cap = capacity;
    ep->P.topk = cf.topk;
    ep->P.hidden = cf.hidden;
    ep->P.e_per = cf.n_expert / world;
    ep_bind(ep, rank, ep->base);
    memcpy(h.uuid, &prop.uuid, 16);
    h.rank = rank; h.world = world; h.cap = capacity; h.hidden = cf.hidden; h.topk = cf.topk; h.n_expert = cf.n_expert;
    memcpy(handle_out, &h, sizeof(h));
    c->ep = ep;
    return INZG_OK;
}

inzg_status inzg_ep_connect(inzg_ctx *c, const void *handles) {
    if (!c) return INZG_BAD_ARG;
    EpState *ep = c->ep;
    if (!ep || !handles) return fail(c, INZG_BAD_ARG, "ep_connect: attach first; handles missing");
    if (ep->connected) return fail(c, INZG_BAD_ARG, "ep_connect: already connected");
    cudaSetDevice(c->cfg.device);
    const EpHandle *hs = static_cast<const EpHandle *>(handles);
    for (int d = 0; d < ep->world; d++) {
        const EpHandle &h = hs[d];
        if (h.rank != d || h.world != ep->world || h.cap != ep->cap || h.hidden != c->cfg.hidden ||
            h.topk != c->cfg.topk || h.n_expert != c->cfg.n_expert)
            return fail(c, INZG_BAD_ARG, "ep_connect: handles disagree on rank order or the exchange's shape");
        for (int j = 0; j < d; j++)
            if (!memcmp(hs[j].uuid, h.uuid, 16))
                return fail(c, INZG_BAD_ARG, "ep_connect: two ranks on one GPU (one rank per device)");
    }
    ep->opened.assign(ep->world, nullptr);
    for (int d = 0; d < ep->world; d++) {
        if (d == ep->rank) continue;
        void *p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, hs[d].ipc, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (void *q : ep->opened)
                if (q) cudaIpcCloseMemHandle(q);
            ep->opened.clear();
            return cuda_fail(c, e, "ep_connect: open a peer's buffer");
        }
        ep->opened[d] = p;
        ep_bind(ep, d, static_cast<uint8_t *>(p));
    }
    ep->connected = true;
    return INZG_OK;
}

inzg_status inzg_ep_connect_local(inzg_ctx *const *ctxs, int world) {
    if (!ctxs || world < 1 || world > kEpMaxRanks) return INZG_BAD_ARG;
    for (int d = 0; d < world; d++) {
        inzg_ctx *c = ctxs[d];
        if (!c || !c->ep || c->ep->connected || c->ep->world != world || c->ep->rank != d) {
            if (c) fail(c, INZG_BAD_ARG, "ep_connect_local: every context attached once, in rank order");
            return INZG_BAD_ARG;
        }
        for (int j = 0; j < d; j++)
            if (ctxs[j]->cfg.device == c->cfg.device)
                return fail(c, INZG_BAD_ARG, "ep_connect_local: two ranks on one GPU (one rank per device)");
    }
    for (int d = 0; d < world; d++) {
        inzg_ctx *c = ctxs[d];
        cudaSetDevice(c->cfg.device);
        for (int j = 0; j < world; j++) {
            if (j == d) continue;
            cudaError_t e = cudaDeviceEnablePeerAccess(ctxs[j]->cfg.device, 0);
            if (e == cudaErrorPeerAccessAlreadyEnabled) {
                cudaGetLastError();
                e = cudaSuccess;
            }
            if (e != cudaSuccess) return cuda_fail(c, e, "ep_connect_local: peer access");
            ep_bind(c->ep, j, ctxs[j]->ep->base);
        }
    }
    for (int d = 0; d < world; d++) ctxs[d]->ep->connected = true;
    return INZG_OK;
}

inzg_status inzg_ep_barrier(inzg_ctx *c, void *stream) {
    if (!c) return INZG_BAD_ARG;
    EpState *ep = c->ep;
    if (!ep || !ep->connected) return fail(c, INZG_NOT_READY, "ep_barrier: attach and connect first");
    cudaSetDevice(c->cfg.device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    launch_ep_barrier(ep->P, ep->bar_epoch, ep->err, st);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? INZG_OK : cuda_fail(c, e, "ep_barrier: kernel launch");
}

inzg_status inzg_ep_detach(inzg_ctx *c) {
    if (!c) return INZG_BAD_ARG;
    if (!c->ep) return INZG_OK;
    cudaSetDevice(c->cfg.device);
    cudaDeviceSynchronize();
    drop_graphs(c);  // graphs of expert-parallel steps hold the peers' pointers
    ep_free(c->ep);
    c->ep = nullptr;
    return INZG_OK;
}

// One expert-parallel step of this rank (k_ep.cu): launches, or -1 / -2 as enqueue_experts.
static int enqueue_ep(inzg_ctx *c, int layer, int n, const float *x, const float *bias, float *y, int n_batch,
                      cudaStream_t st) {
    const inzg_config &cf = c->cfg;
    EpState *ep = c->ep;
    LayerSlot &L = c->layers[layer];
    const int H = cf.hidden, E = cf.n_expert;
    int launches = 0;
    bool bad = false;
    auto add = [&](int r) {
        if (r < 0) bad = true;
        else launches += r;
    };
    add(launch_router_logits(L.router, L.router32, x, n, H, E, bias, c->logits, c->meta, st));
    add(launch_ep_dispatch(c->logits, x, n, E, ep->P, ep->sel, ep->epoch, ep->tickets, st));
    add(launch_ep_wait(ep->P.flags[ep->rank], ep->world, 0, ep->epoch, false, ep->err, st));
    const int r = enqueue_experts(c, L, ep->world * ep->cap, ep->P.rx[ep->rank], ep->P.rsel[ep->rank],
                                  ep->P.rw[ep->rank], n_batch, ep->P.out[ep->rank], st);
    if (r == -2) return -2;
    add(r);
    add(launch_ep_signal(ep->P, ep->epoch, st));
    add(launch_ep_wait(ep->P.flags[ep->rank], ep->world, 1, ep->epoch, true, ep->err, st));
    add(launch_ep_combine(ep->sel, n, ep->P, y, c->num_sms, st));
    if (c->shared[layer].has_experts) {
        const int rs = enqueue_shared(c, layer, n, x, y, n_batch, false, st);
        if (rs == -2) return -2;
        add(rs);
    }
    return bad ? -1 : launches;
}

inzg_status inzg_ep_forward(inzg_ctx *c, int layer, int n, const float *x_dev, const float *logit_bias_dev,
                            float *y_dev, int n_batch, void *stream) {
    if (!c) return INZG_BAD_ARG;
    const inzg_config &cf = c->cfg;
    EpState *ep = c->ep;
    if (!ep || !ep->connected) return fail(c, INZG_NOT_READY, "ep_forward: attach and connect first");
    if (layer < 0 || layer >= cf.n_layers) return fail(c, INZG_BAD_ARG, "ep_forward: bad layer");
    if (n < 1 || n > ep->cap || n_batch < n || !x_dev || !y_dev)
        return fail(c, INZG_BAD_ARG, "ep_forward: bad n (1..capacity), n_batch or pointer");
    if ((reinterpret_cast<uintptr_t>(x_dev) | reinterpret_cast<uintptr_t>(y_dev)) & 15)
        return fail(c, INZG_BAD_ARG, "ep_forward: x and y must be 16-byte aligned");
    LayerSlot &L = c->layers[layer];
    if (!L.has_router || !L.has_experts) return fail(c, INZG_NOT_READY, "ep_forward: layer not loaded");
    if (L.e_first != ep->rank * ep->P.e_per || L.dev.E != ep->P.e_per)
        return fail(c, INZG_NOT_READY, "ep_forward: the pool must hold exactly this rank's experts");
    cudaSetDevice(cf.device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    if (launch_gemv_decode(L.dev, -1, RouteDev{}, nullptr, nullptr, nullptr, 0, 0, st) < 0)
        return fail(c, INZG_UNSUPPORTED, "ep_forward: no decode kernel for this geometry");
    inzg_ctx::GraphKey key{layer, n, x_dev, y_dev, logit_bias_dev, nullptr, 0x80000000u, n_batch};
    inzg_ctx::GraphEntry *g = nullptr;
    for (auto &ge : c->graphs)
        if (ge.key == key) g = &ge;
    cudaError_t e = cudaSuccess;
    if (!g) {
        cudaStream_t cs = c->capture_stream;
        e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) return cuda_fail(c, e, "ep_forward: begin capture");
        const int nl = enqueue_ep(c, layer, n, x_dev, logit_bias_dev, y_dev, n_batch, cs);
        cudaGraph_t graph = nullptr;
        e = cudaStreamEndCapture(cs, &graph);
        if (e != cudaSuccess || nl < 0) {
            if (graph) cudaGraphDestroy(graph);
            return e != cudaSuccess ? cuda_fail(c, e, "ep_forward: capture")
                   : nl == -2       ? fail(c, INZG_UNSUPPORTED, "ep_forward: no tensor maps for the prefill GEMM")
                                    : fail(c, INZG_UNSUPPORTED, "ep_forward: no kernel for this shape");
        }
        cudaGraphExec_t exec = nullptr;
        e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) return cuda_fail(c, e, "ep_forward: graph instantiate");
        if (c->graphs.size() >= 64) {
            auto it = std::min_element(c->graphs.begin(), c->graphs.end(),
                                       [](const inzg_ctx::GraphEntry &a, const inzg_ctx::GraphEntry &b) {
                                           return a.last_use < b.last_use;
                                       });
            cudaGraphExecDestroy(it->exec);
            c->graphs.erase(it);
        }
        c->graphs.push_back({key, exec, nl, 0});
        g = &c->graphs.back();
    }
    g->last_use = ++c->use_clock;
    e = cudaGraphLaunch(g->exec, st);
    if (e != cudaSuccess) return cuda_fail(c, e, "ep_forward: graph launch");
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, "ep_forward: kernel launch");
    c->stats.calls++;
    c->stats.tokens += n;
    c->stats.last_launches = g->launches;
    return INZG_OK;
}

inzg_status inzg_stage_times(inzg_ctx *c, double *ms, uint64_t *calls, int reset) {
    if (!c) return INZG_BAD_ARG;
    if (ms)
        for (int i = 0; i < INZG_N_STAGES; i++) ms[i] = c->stage_ms[i];
    if (calls) *calls = c->profiled_calls;
    if (reset) {
        for (int i = 0; i < INZG_N_STAGES; i++) c->stage_ms[i] = 0;
        c->profiled_calls = 0;
    }
    return INZG_OK;
}

// internal helpers for noalloc.cu (hidden: not part of the exported ABI)
int inzg__router_view(const inzg_ctx *c, int layer, const void **router, int *device, int *hidden, int *n_expert,
                      int *topk, void **stream, int32_t **meta) {
    if (!c || layer < 0 || layer >= c->cfg.n_layers || !c->layers[layer].has_router) return 0;
    *router = c->layers[layer].router;
    *device = c->cfg.device;
    *hidden = c->cfg.hidden;
    *n_expert = c->cfg.n_expert;
    *topk = c->cfg.topk;
    *stream = c->stream;
    *meta = c->meta;
    return 1;
}

void inzg__set_error(inzg_ctx *c, const char *msg) {
    if (c) c->err = msg;
}

const char *inzg_stage_name(int stage) { return stage >= 0 && stage < INZG_N_STAGES ? kStageNames[stage] : nullptr; }

inzg_status inzg_moe_route_dump(inzg_ctx *c, int n, int32_t *sel, float *w, float *logits, float *probs,
                                int32_t *unit_expert, int *n_units) {
    if (!c) return INZG_BAD_ARG;
    if (!c->last_dump || n != c->last_n) return fail(c, INZG_BAD_ARG, "route_dump: no dumped call with this n");
    cudaSetDevice(c->cfg.device);
    const int E = c->cfg.n_expert, K = c->cfg.topk;
    cudaError_t e = cudaStreamSynchronize(c->stream);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess && sel) e = cudaMemcpy(sel, c->sel, sizeof(int32_t) * (size_t)n * K, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && w) e = cudaMemcpy(w, c->w, sizeof(float) * (size_t)n * K, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && logits) e = cudaMemcpy(logits, c->logits, sizeof(float) * (size_t)n * E, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && probs) e = cudaMemcpy(probs, c->probs, sizeof(float) * (size_t)n * E, cudaMemcpyDeviceToHost);
    int32_t meta[16] = {0};
    if (e == cudaSuccess) e = cudaMemcpy(meta, c->meta, sizeof(meta), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(c, e, "route_dump");
    const int nu = meta[kMetaNUnits];
    std::vector<int32_t> units(nu), ssel((size_t)n * K), first(E, 0x7F7F7F7F);
    if (nu > 0) e = cudaMemcpy(units.data(), c->units, sizeof(int32_t) * nu, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(ssel.data(), c->sel, sizeof(int32_t) * (size_t)n * K, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(c, e, "route_dump");
    // first-touch order of the reference's units: ascending first slot t*topk+k
    for (size_t i = ssel.size(); i-- > 0;)
        if (ssel[i] >= 0 && ssel[i] < E) first[ssel[i]] = (int32_t)i;
    std::sort(units.begin(), units.end(), [&](int a, int b) { return first[a] < first[b]; });
    if (unit_expert) std::copy(units.begin(), units.end(), unit_expert);
    if (n_units) *n_units = nu;
    c->stats.units = nu;
    c->stats.dec_units = meta[kMetaNDec];
    c->stats.gemm_units = meta[kMetaNGemm];
    return INZG_OK;
}

inzg_status inzg_get_stats(const inzg_ctx *c, inzg_stats *out) {
    if (!c || !out) return INZG_BAD_ARG;
    *out = c->stats;
    return INZG_OK;
}

// ---- hyper-connections around the layer (src/model_fwd.c:404-450, 1264-1267) ----

inzg_status inzg_set_hc(inzg_ctx *c, int layer, const float *norm, const uint16_t *down, const uint16_t *up,
                        const float *inject) {
    if (!c) return INZG_BAD_ARG;
    const inzg_config &cf = c->cfg;
    if (layer < 0 || layer >= cf.n_layers || !norm || !down || !up) return fail(c, INZG_BAD_ARG, "set_hc: bad layer or pointer");
    cudaSetDevice(cf.device);
    drop_graphs(c);
    const int W = 4 * cf.hidden, R = INZG_HC_RANK;
    const size_t f16 = (size_t)R * W * 2;
    const size_t o_inj = (size_t)W * 4, o_d32 = o_inj + (size_t)4 * W * 4, o_u32 = o_d32 + router32_floats(R, W) * 4,
                 o_dn = o_u32 + router32_floats(W, R) * 4, o_up = o_dn + f16, total = o_up + f16;
    HcSlot &h = c->hc[layer];
    if (!h.mem && cudaMalloc(&h.mem, total) != cudaSuccess) {
        cudaGetLastError();
        h.mem = nullptr;
        return fail(c, INZG_OOM, "set_hc: weight buffer");
    }
    uint16_t *tmp = nullptr;
    if (cudaMalloc(&tmp, 2 * f16) != cudaSuccess) {
        cudaGetLastError();
        return fail(c, INZG_OOM, "set_hc: staging buffer");
    }
    cudaStream_t st = c->stream;
    cudaError_t e = cudaMemcpyAsync(h.mem, norm, (size_t)W * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess && inject) e = cudaMemcpyAsync(h.mem + o_inj, inject, (size_t)4 * W * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(tmp, down, f16, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(tmp + (size_t)R * W, up, f16, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) {
        launch_router_repack(tmp, reinterpret_cast<uint4 *>(h.mem + o_dn), R, W, st);
        launch_router_repack32(tmp, reinterpret_cast<float *>(h.mem + o_d32), R, W, st);
        launch_router_repack(tmp + (size_t)R * W, reinterpret_cast<uint4 *>(h.mem + o_up), W, R, st);
        launch_router_repack32(tmp + (size_t)R * W, reinterpret_cast<float *>(h.mem + o_u32), W, R, st);
        e = cudaStreamSynchronize(st);
    }
    cudaFree(tmp);
    if (e != cudaSuccess) return cuda_fail(c, e, "set_hc");
    hc_set_attributes(cf.hidden);
    HcDev &d = h.dev;
    d.norm = reinterpret_cast<const float *>(h.mem);
    d.inject = inject ? reinterpret_cast<const float *>(h.mem + o_inj) : nullptr;
    d.down32 = router_gemm_fits(R, W) ? reinterpret_cast<const float *>(h.mem + o_d32) : nullptr;
    d.down = reinterpret_cast<const uint4 *>(h.mem + o_dn);
    d.up = reinterpret_cast<const uint4 *>(h.mem + o_up);
    d.up32 = router_gemm_fits(W, R) ? reinterpret_cast<const float *>(h.mem + o_u32) : nullptr;
    d.rank = R;
    return INZG_OK;
}

// hc_in's scratch for n tokens (grown, never shrunk; allocated outside any stream capture by the first call that
// needs it)
static inzg_status hc_scratch(inzg_ctx *c, int n) {
    if (n <= c->hc_cap) return INZG_OK;
    drop_graphs(c);  // captured hc_in steps name the old scratch
    for (float **p : {&c->hc_Xn, &c->hc_d, &c->hc_m, &c->hc_inj})
        if (*p) {
            cudaFree(*p);
            *p = nullptr;
        }
    c->hc_cap = 0;
    const size_t W = 4 * (size_t)c->cfg.hidden;
    bool ok = true;
    c->hc_Xn = dalloc<float>((size_t)n * W, ok);
    c->hc_m = dalloc<float>((size_t)n * W, ok);
    c->hc_d = dalloc<float>((size_t)n * INZG_HC_RANK, ok);
    c->hc_inj = dalloc<float>((size_t)n * 4, ok);
    if (!ok) return fail(c, INZG_OOM, "hc_in: scratch");
    c->hc_cap = n;
    return INZG_OK;
}

// validates and enqueues hc_in; inj_dev nullptr: the inject weights are not computed
static inzg_status hc_in_enqueue(inzg_ctx *c, int layer, int n, const float *X_dev, float *xin_dev, float *inj_dev,
                                 cudaStream_t st) {
    const inzg_config &cf = c->cfg;
    if ((reinterpret_cast<uintptr_t>(X_dev) | reinterpret_cast<uintptr_t>(xin_dev) | reinterpret_cast<uintptr_t>(inj_dev)) & 15)
        return fail(c, INZG_BAD_ARG, "hc_in: pointers must be 16-byte aligned");
    const HcSlot &h = c->hc[layer];
    if (!h.mem) return fail(c, INZG_NOT_READY, "hc_in: layer has no hyper-connection weights (inzg_set_hc)");
    if (inj_dev && !h.dev.inject) return fail(c, INZG_BAD_ARG, "hc_in: the layer's hyper-connection has no inject vectors");
    // the step's kernels are captured once per (layer, n, buffers) into a CUDA graph and replayed, as the layer's
    const inzg_ctx::GraphKey key{layer, n, X_dev, xin_dev, inj_dev, nullptr, 0x40000000u, 0};
    inzg_ctx::GraphEntry *g = nullptr;
    for (auto &ge : c->graphs)
        if (ge.key == key) g = &ge;
    cudaError_t e = cudaSuccess;
    if (!g) {
        cudaStream_t cs = c->capture_stream;
        e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) return cuda_fail(c, e, "hc_in: begin capture");
        const int nl = launch_hc_in(h.dev, n, cf.hidden, X_dev, c->hc_Xn, c->hc_d, c->hc_m, xin_dev, inj_dev, c->meta,
                                    c->num_sms, cs);
        cudaGraph_t graph = nullptr;
        e = cudaStreamEndCapture(cs, &graph);
        if (e != cudaSuccess || nl < 0) {
            if (graph) cudaGraphDestroy(graph);
            return e != cudaSuccess ? cuda_fail(c, e, "hc_in: capture") : fail(c, INZG_UNSUPPORTED, "hc_in: no kernel for this width");
        }
        cudaGraphExec_t exec = nullptr;
        e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) return cuda_fail(c, e, "hc_in: graph instantiate");
        if (c->graphs.size() >= 64) {  // evict the least recently used
            auto it = std::min_element(c->graphs.begin(), c->graphs.end(),
                                       [](const inzg_ctx::GraphEntry &a, const inzg_ctx::GraphEntry &b) {
                                           return a.last_use < b.last_use;
                                       });
            cudaGraphExecDestroy(it->exec);
            c->graphs.erase(it);
        }
        c->graphs.push_back({key, exec, nl, 0});
        g = &c->graphs.back();
    }
    g->last_use = ++c->use_clock;
    e = cudaGraphLaunch(g->exec, st);
    if (e != cudaSuccess) return cuda_fail(c, e, "hc_in: graph launch");
    e = cudaGetLastError();
    return e == cudaSuccess ? INZG_OK : cuda_fail(c, e, "hc_in: kernel launch");
}

inzg_status inzg_hc_in(inzg_ctx *c, int layer, int n, const float *X_dev, float *xin_dev, float *inj_dev, void *stream) {
    if (!c) return INZG_BAD_ARG;
    const inzg_config &cf = c->cfg;
    if (layer < 0 || layer >= cf.n_layers || n <= 0 || n > cf.max_tokens || !X_dev || !xin_dev)
        return fail(c, INZG_BAD_ARG, "hc_in: bad layer, n or pointer");
    cudaSetDevice(cf.device);
    const inzg_status s = hc_scratch(c, n);
    if (s != INZG_OK) return s;
    return hc_in_enqueue(c, layer, n, X_dev, xin_dev, inj_dev, stream ? static_cast<cudaStream_t>(stream) : c->stream);
}

inzg_status inzg_hc_out(inzg_ctx *c, int n, float *X_dev, const float *inj_dev, const float *y_dev, void *stream) {
    if (!c) return INZG_BAD_ARG;
    const inzg_config &cf = c->cfg;
    if (n <= 0 || n > cf.max_tokens || !X_dev || !inj_dev || !y_dev) return fail(c, INZG_BAD_ARG, "hc_out: bad n or pointer");
    if ((reinterpret_cast<uintptr_t>(X_dev) | reinterpret_cast<uintptr_t>(y_dev)) & 15)
        return fail(c, INZG_BAD_ARG, "hc_out: X and y must be 16-byte aligned");
    cudaSetDevice(cf.device);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    launch_hc_out(X_dev, inj_dev, y_dev, n, cf.hidden, c->num_sms, st);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? INZG_OK : cuda_fail(c, e, "hc_out: kernel launch");
}

inzg_status inzg_moe_block_hc(inzg_ctx *c, int layer, int n, float *X_dev, const inzg_moe_opts *opt) {
    if (!c) return INZG_BAD_ARG;
    const inzg_config &cf = c->cfg;
    if (layer < 0 || layer >= cf.n_layers || n <= 0 || n > cf.max_tokens || !X_dev)
        return fail(c, INZG_BAD_ARG, "moe_block_hc: bad layer, n or pointer");
    if (opt && (opt->flags & (INZG_DUMP_ROUTE | INZG_PROFILE)))
        return fail(c, INZG_BAD_ARG, "moe_block_hc: route dumps and profiling are for inzg_moe_forward");
    inzg_moe_opts o = opt ? *opt : inzg_moe_opts{};
    o.flags |= INZG_IO_DEVICE;
    cudaSetDevice(cf.device);
    inzg_status s = hc_scratch(c, n);
    if (s != INZG_OK) return s;
    cudaStream_t st = o.stream ? static_cast<cudaStream_t>(o.stream) : c->stream;
    // X -> (xin, inj) -> the layer (y) -> X += inj * y, with the context's own device buffers in between
    s = hc_in_enqueue(c, layer, n, X_dev, c->xin, c->hc_inj, st);
    if (s != INZG_OK) return s;
    s = inzg_moe_forward(c, layer, n, c->xin, c->y, &o);
    if (s != INZG_OK) return s;
    return inzg_hc_out(c, n, X_dev, c->hc_inj, c->y, o.stream);
}

}  // extern "C"
