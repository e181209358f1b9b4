// k_ep.cu -- expert-parallel exchange over peer memory (NVLink / NVSwitch), sm_100a.
//
// The reference runs every expert in one process (src/model_fwd.c:1071-1140); here rank g of G owns experts
// [g*E/G, (g+1)*E/G) and routes its own share of the batch. Every rank exposes one device buffer to its peers (CUDA IPC
// between processes, plain peer pointers inside one process):
//   rsel [G][C][K] int32  local expert of each (source rank, row, rank-k slot) owned here, -1 otherwise
//   rw   [G][C][K] f32    the routing weight of that slot
//   rx   [G][C][H] f32    the rows sources sent here (a row only when the token has an expert here)
//   slot [C][K][H] f32    this rank's tokens' expert outputs, written by the owner of each slot
//   flags [2][G] u32      dispatch / return epochs written by each peer
// One step on every rank: route -> ep_dispatch (each (token, owner) row and its slot metadata straight into the
// owner's buffer, then a release of the owner's dispatch flag) -> ep_wait (acquire every peer's dispatch flag) ->
// the owned experts on all received rows (the single-GPU experts path; its numeric-path rule uses the whole batch) ->
// ep_return (each owned slot straight into its home's slot buffer, then a release of the home's return flag) ->
// ep_wait (every peer's return flag) -> the rank-order combine of the K slots (src/model_fwd.c:1134-1140). Slots are
// returned individually, so the combine adds them in the reference's order and the output is the single-GPU bits.
//
// Synchronisation is by epochs: every rank keeps its step number in device memory (read by every kernel of the step,
// advanced by the last wait), so a step can be captured in a CUDA graph. A buffer written at step e is read only after
// the peer's flag for e, and rewritten at e + 1 only after the writer has seen the reader's return flag for e, so one
// copy of each buffer is enough. Every wait is bounded: a wait that runs out records INZG_TIMEOUT in the call's error
// word and lets the step finish with whatever landed (the call then fails at inzg_device_status). Kernels write peer
// memory with ordinary stores; there is no tensor-copy multicast and no library kernel touches peer memory.
#include <cuda_runtime.h>

#include <algorithm>

#include "inzg_internal.h"
#include "k_launch.h"

namespace inzg {

namespace {

constexpr uint64_t kEpWaitNs = 1000000000ull;  // a wait gives up after a second without its peer
constexpr uint32_t kEpSpin = 1u << 26;          // and after this many polls in any case

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// the last block of a grid to finish releases `epoch` into flag[me] of every peer's flag array `which`
__device__ void release_peers(const EpPeers &P, int which, uint32_t epoch, int32_t *ticket) {
    __threadfence_system();  // this block's peer stores before its ticket
    __syncthreads();
    if (threadIdx.x == 0) {
        const int t = atomicAdd(ticket, 1);
        if (t == (int)gridDim.x - 1) {
            __threadfence_system();  // every block's stores (their fences preceded their tickets) before the flags
            for (int d = 0; d < P.world; d++) st_release_sys(P.flags[d] + which * P.world + P.rank, epoch);
            *ticket = 0;  // the next step's kernels start after this one ends
        }
    }
}

// dispatch: pair (row t, destination d) per warp; t < n carries a token (its K selections), t >= n only clears
// its metadata. A row is sent once to every rank owning at least one of its experts.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const float *__restrict__ x, int n, const int32_t *__restrict__ sel,
                                                          const float *__restrict__ w, EpPeers P, const uint32_t *epoch_dev,
                                                          int32_t *ticket) {
    const uint32_t epoch = *epoch_dev + 1;
    const int K = P.topk, H = P.hidden, C = P.cap, G = P.world;
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), nw = gridDim.x * (blockDim.x >> 5);
    for (int p = gw; p < C * G; p += nw) {
        const int t = p / G, d = p % G;
        int loc = -1;
        float wk = 0.0f;
        if (lane < K && t < n) {
            const int e = sel[(size_t)t * K + lane];
            if (e >= d * P.e_per && e < (d + 1) * P.e_per) {
                loc = e - d * P.e_per;
                wk = w[(size_t)t * K + lane];
            }
        }
        const size_t row = (size_t)P.rank * C + t;
        if (lane < K) {
            P.rsel[d][row * K + lane] = loc;
            P.rw[d][row * K + lane] = wk;
        }
        if (__any_sync(0xffffffffu, loc >= 0)) {
            const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)t * H);
            float4 *dst = reinterpret_cast<float4 *>(P.rx[d] + row * H);
            for (int i = lane; i < H / 4; i += 32) dst[i] = __ldg(src + i);
        }
    }
    release_peers(P, 0, epoch, ticket);
}

// return: one warp per (received row, rank-k slot) owned here; the slot's H outputs go to the home's slot buffer
__global__ void __launch_bounds__(256) ep_return_kernel(const float *__restrict__ out, EpPeers P,
                                                        const uint32_t *epoch_dev, int32_t *ticket) {
    const uint32_t epoch = *epoch_dev + 1;
    const int K = P.topk, H = P.hidden, C = P.cap, G = P.world;
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), nw = gridDim.x * (blockDim.x >> 5);
    const int32_t *mine = P.rsel[P.rank];
    for (int p = gw; p < G * C * K; p += nw) {
        if (mine[p] < 0) continue;  // uniform over the warp
        const int r = p / K, k = p % K, s = r / C, t = r % C;
        const float4 *src = reinterpret_cast<const float4 *>(out + (size_t)p * H);
        float4 *dst = reinterpret_cast<float4 *>(P.slot[s] + ((size_t)t * K + k) * H);
        for (int i = lane; i < H / 4; i += 32) dst[i] = src[i];
    }
    release_peers(P, 1, epoch, ticket);
}

// wait until every peer has released this step into flags[which][*]; `advance`: the step's last wait, which then
// moves the step number on. A wait that runs out records the timeout and returns.
__global__ void ep_wait_kernel(const uint32_t *flags, int world, int which, uint32_t *epoch_dev, int advance,
                               int32_t *err) {
    const uint32_t epoch = *epoch_dev + 1;
    const int lane = threadIdx.x;
    bool ok = true;
    if (lane < world) {
        const uint32_t *f = flags + which * world + lane;
        const uint64_t t0 = globaltimer_ns();
        uint32_t i = 0;
        while ((int32_t)(ld_acquire_sys(f) - epoch) < 0) {
            if (++i >= kEpSpin || ((i & 255) == 0 && globaltimer_ns() - t0 > kEpWaitNs)) {
                ok = false;
                break;
            }
            if ((i & 63) == 0) __nanosleep(128);
        }
    }
    if (!ok) atomicCAS(err, 0, kErrTimeout);
    __syncwarp();
    if (advance && lane == 0) *epoch_dev = epoch;
}

}  // namespace

int launch_ep_dispatch(const float *x, int n, const int32_t *sel, const float *w, const EpPeers &P,
                       const uint32_t *epoch_dev, int32_t *ticket, int num_sms, cudaStream_t st) {
    const int pairs = P.cap * P.world, blocks = std::min((pairs + 7) / 8, num_sms * 4);
    ep_dispatch_kernel<<<blocks, 256, 0, st>>>(x, n, sel, w, P, epoch_dev, ticket);
    return 1;
}

int launch_ep_return(const float *out, const EpPeers &P, const uint32_t *epoch_dev, int32_t *ticket, int num_sms,
                     cudaStream_t st) {
    const int slots = P.world * P.cap * P.topk, blocks = std::min((slots + 7) / 8, num_sms * 4);
    ep_return_kernel<<<blocks, 256, 0, st>>>(out, P, epoch_dev, ticket);
    return 1;
}

int launch_ep_wait(const uint32_t *flags, int world, int which, uint32_t *epoch_dev, bool advance, int32_t *err,
                   cudaStream_t st) {
    ep_wait_kernel<<<1, 32, 0, st>>>(flags, world, which, epoch_dev, advance ? 1 : 0, err);
    return 1;
}

}  // namespace inzg
