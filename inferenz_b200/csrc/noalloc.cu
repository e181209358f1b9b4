// noalloc.cu -- inzg_route_topk_noalloc: router logits -> softmax -> top-k with no device allocation.
//
// Some callers cannot allocate device memory on the call path: engines that fix their whole device-memory plan at
// start-up (the reference engine sizes its memory once and refuses to start when it does not fit), and
// latency-critical decode loops in which a cudaMalloc / cudaFree would synchronise the device. This entry point runs
// the same two kernels as inzg_moe_forward's routing stage, but their intermediate logits live in the file-scope
// array below instead of the context's scratch, so a call allocates nothing. The caller passes the inputs and the
// outputs (device pointers); the router weights are the ones inzg_set_router already placed on the device.
//
// The array: g_noalloc_logits, kNoAllocMaxTokens x kNoAllocMaxExperts fp32 (64 x 512 x 4 B = 128 KiB), held by every
// GPU that loads this library until the process exits. Host code cannot use the array's name as a device address
// (it names a host-side stand-in); the device address is looked up once per device, with that device current, by
// cudaGetSymbolAddress, and passed to the kernels. That set-up happens in the first call on each device, so the
// first call on a device should come before any stream capture. Every call shares the array and finds the previous
// call's logits in it; nothing in it must start at zero (the router kernel writes every logit it later reads). Calls
// whose executions overlap on the GPU race on the array.
//
// Failure reporting allocates nothing either: the router records a bounded wait that ran out in the context's own
// status words (allocated once by inzg_create), which the call clears first; a short kernel after the top-k then
// overwrites the call's outputs with sel = -1 and w = NaN, so logits left by an earlier call never pass for this
// call's routing, and inzg_device_status reports INZG_TIMEOUT.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/inzg.h"
#include "inzg_internal.h"
#include "k_launch.h"

namespace {

constexpr int kNoAllocMaxTokens = 64;
constexpr int kNoAllocMaxExperts = 512;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_logits[kNoAllocMaxTokens * kNoAllocMaxExperts];

std::mutex g_setup_mutex;
float *g_dev_ptr[kMaxDevices] = {};

// device address of g_noalloc_logits on `device` (current), looked up once per device; nullptr on failure
float *scratch_for(int device, cudaError_t *err) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (device < 0 || device >= kMaxDevices) {
        *err = cudaErrorInvalidDevice;
        return nullptr;
    }
    if (!g_dev_ptr[device]) {
        void *p = nullptr;
        *err = cudaGetSymbolAddress(&p, g_noalloc_logits);
        if (*err != cudaSuccess) return nullptr;
        g_dev_ptr[device] = static_cast<float *>(p);
    }
    *err = cudaSuccess;
    return g_dev_ptr[device];
}

// a router wait that ran out (the context's router status word is set): poison the call's outputs
__global__ void noalloc_poison_kernel(const int32_t *__restrict__ meta, int32_t *__restrict__ sel,
                                      float *__restrict__ w, int count) {
    if (meta[inzg::kMetaRouterError] == inzg::kErrNone) return;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
        sel[i] = -1;
        w[i] = __int_as_float(0x7FC00000);
    }
}

// restores the caller's current device when the call returns
struct DeviceGuard {
    int saved = -1;
    DeviceGuard() {
        if (cudaGetDevice(&saved) != cudaSuccess) {
            cudaGetLastError();
            saved = -1;
        }
    }
    ~DeviceGuard() {
        if (saved >= 0) cudaSetDevice(saved);
    }
};

}  // namespace

// Defined in ctx.cu: the layer's device router, the context's device, shapes, stream and status words (no allocation).
extern "C" int inzg__router_view(const inzg_ctx *ctx, int layer, const void **router, int *device, int *hidden,
                                 int *n_expert, int *topk, void **stream, int32_t **meta);
extern "C" void inzg__set_error(inzg_ctx *ctx, const char *msg);

extern "C" INZG_EXPORT inzg_status inzg_route_topk_noalloc(inzg_ctx *ctx, int layer, int n, const float *x_dev,
                                                           const float *logit_bias_dev, int32_t *sel_dev,
                                                           float *w_dev, void *stream) {
    if (!ctx) return INZG_BAD_ARG;
    const void *router = nullptr;
    int device = 0, H = 0, E = 0, K = 0;
    void *ctx_stream = nullptr;
    int32_t *meta = nullptr;
    if (!inzg__router_view(ctx, layer, &router, &device, &H, &E, &K, &ctx_stream, &meta)) {
        inzg__set_error(ctx, "route_topk_noalloc: layer has no router");
        return INZG_NOT_READY;
    }
    if (n <= 0 || n > kNoAllocMaxTokens) {
        inzg__set_error(ctx, "route_topk_noalloc: n must be 1..64 (the size of the entry point's static scratch)");
        return INZG_BAD_ARG;
    }
    if (E > kNoAllocMaxExperts) {
        inzg__set_error(ctx, "route_topk_noalloc: more than 512 experts exceed the entry point's static scratch");
        return INZG_BAD_ARG;
    }
    if (!x_dev || !sel_dev || !w_dev) {
        inzg__set_error(ctx, "route_topk_noalloc: null device pointer");
        return INZG_BAD_ARG;
    }
    if (reinterpret_cast<uintptr_t>(x_dev) & 15) {  // token rows are moved by bulk copies
        inzg__set_error(ctx, "route_topk_noalloc: x_dev must be 16-byte aligned");
        return INZG_BAD_ARG;
    }
    DeviceGuard guard;
    cudaError_t e = cudaSetDevice(device);
    float *logits = e == cudaSuccess ? scratch_for(device, &e) : nullptr;
    if (!logits) {
        inzg__set_error(ctx, "route_topk_noalloc: cudaGetSymbolAddress of the static scratch failed");
        return INZG_CUDA;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream ? stream : ctx_stream);
    e = cudaMemsetAsync(meta + inzg::kMetaRouterError, 0, sizeof(int32_t), st);
    if (e != cudaSuccess) {
        inzg__set_error(ctx, "route_topk_noalloc: clearing the status word failed");
        return INZG_CUDA;
    }
    inzg::launch_router_logits(static_cast<const uint4 *>(router), nullptr, x_dev, n, H, E, logit_bias_dev, logits, meta,
                               st);
    inzg::launch_softmax_topk(logits, n, E, K, sel_dev, w_dev, nullptr, st);
    noalloc_poison_kernel<<<1, 256, 0, st>>>(meta, sel_dev, w_dev, n * K);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        inzg__set_error(ctx, "route_topk_noalloc: kernel launch failed");
        return INZG_CUDA;
    }
    return INZG_OK;
}
