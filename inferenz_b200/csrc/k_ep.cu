// k_ep.cu -- expert-parallel exchange over peer memory (NVLink / NVSwitch), sm_100a.
//
// The reference runs every expert in one process (src/model_fwd.c:1071-1140); here rank g of G owns experts
// [g*E/G, (g+1)*E/G) and routes its own share of the batch. Every rank exposes one device buffer to its peers (CUDA IPC
// between processes, plain peer pointers inside one process):
//   rsel [G][C][K] int32  local expert of each (source rank, row, rank-k slot) owned here, -1 otherwise
//   rw   [G][C][K] f32    the routing weight of that slot
//   rx   [G][C][H] f32    the rows sources sent here (a row only when the token has an expert here)
//   out  [G*C][K][H] f32  this rank's expert outputs, per received row and rank-k slot (owned slots only)
//   flags [3][G] u32      dispatch / outputs-ready / rendezvous epochs written by each peer
// One step on every rank: router logits -> ep_dispatch (per token the reference's softmax and top-k, then its row and
// slot metadata straight into each owner's buffer, then a release of the owners' dispatch flags) -> ep_wait (acquire
// every peer's dispatch flag) -> the owned experts on all received rows (the single-GPU experts path; its
// numeric-path rule uses the whole batch) into `out` -> ep_signal (release of every peer's outputs-ready flag) ->
// ep_wait (every peer's outputs ready) -> ep_combine: each token adds its K slots, read straight from their owners'
// `out` over NVLink, in rank order (src/model_fwd.c:1134-1140) -- the single-GPU bits.
//
// Synchronisation is by epochs: every rank keeps its step number in device memory (read by every kernel of the step,
// advanced by the last wait), so a step can be captured in a CUDA graph. A buffer written at step e is read only after
// the peer's flag for e, and rewritten at e + 1 only after every reader has moved on to e + 1 (a rank dispatches e + 1
// only after its combine of e has read its slots), so one copy of each buffer is enough. Every wait is bounded: a wait that runs out records INZG_TIMEOUT in the call's error
// word and lets the step finish with whatever landed (the call then fails at inzg_device_status). Kernels write peer
// memory with ordinary stores; there is no tensor-copy multicast and no library kernel touches peer memory.
#include <cuda_runtime.h>

#include <algorithm>

#include "inzg_internal.h"
#include "k_launch.h"
#include "k_softmax.cuh"

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
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// the last block of a grid to finish releases `epoch` into flag[me] of every peer's flag array `which`: the block's
// stores are ordered before thread 0's system-scope release fence by the barrier, the fence before the ticket (the
// grid-wide barrier pattern), and the last block's acquire-release fence before its release stores of the flags
__device__ void release_peers(const EpPeers &P, int which, uint32_t epoch, int32_t *ticket) {
    __syncthreads();
    if (threadIdx.x == 0) {
        fence_acq_rel_sys();
        const int t = atomicAdd(ticket, 1);
        if (t == (int)gridDim.x - 1) {
            fence_acq_rel_sys();
            for (int d = 0; d < P.world; d++) st_release_sys(P.flags[d] + which * P.world + P.rank, epoch);
            *ticket = 0;  // the next step's kernels start after this one ends
        }
    }
}

// copy of one row of H floats by the calling group of `nthr` threads (index `tid`): all loads of a pass are in flight
// before its stores
__device__ __forceinline__ void copy_row(float4 *__restrict__ dst, const float4 *__restrict__ src, int n4, int tid,
                                         int nthr) {
    constexpr int U = 8;
    for (int i0 = tid; i0 < n4; i0 += U * nthr) {
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; u++)
            if (i0 + u * nthr < n4) v[u] = __ldg(src + i0 + u * nthr);
#pragma unroll
        for (int u = 0; u < U; u++)
            if (i0 + u * nthr < n4) dst[i0 + u * nthr] = v[u];
    }
}

// route + dispatch, one block per row t of the rank's capacity: warp 0 runs the reference's softmax and top-k of token
// t on its router logits (t < n), then the block writes the row's slot metadata into every rank (-1 where that rank
// owns none of the token's experts; rows t >= n only clear theirs) and the token's fp32 row once into every rank owning
// at least one of its experts.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const float *__restrict__ logits, const float *__restrict__ x,
                                                          int n, int E, EpPeers P, int32_t *__restrict__ sel_out,
                                                          const uint32_t *epoch_dev, int32_t *ticket) {
    extern __shared__ float ex[];  // [E] softmax scratch of warp 0
    __shared__ int32_t ssel[kMaxTopK];
    __shared__ float sw[kMaxTopK];
    const uint32_t epoch = *epoch_dev + 1;
    const int K = P.topk, H = P.hidden, C = P.cap, G = P.world, t = blockIdx.x, tid = threadIdx.x;
    if (t < n) {
        if (tid < 32) softmax_topk_warp(logits + (size_t)t * E, E, K, ex, nullptr, ssel, sw);
    } else if (tid < K) {
        ssel[tid] = -1;
        sw[tid] = 0.0f;
    }
    __syncthreads();
    if (t < n && tid < K) sel_out[(size_t)t * K + tid] = ssel[tid];  // the combine finds each slot's owner from it
    const size_t row = (size_t)P.rank * C + t;
    for (int d = 0; d < G; d++) {
        const int lo = d * P.e_per;
        bool here = false;
        for (int k = 0; k < K; k++) here |= ssel[k] >= lo && ssel[k] < lo + P.e_per;
        if (tid < K) {
            const int e = ssel[tid];
            const bool own = e >= lo && e < lo + P.e_per;
            P.rsel[d][row * K + tid] = own ? e - lo : -1;
            P.rw[d][row * K + tid] = own ? sw[tid] : 0.0f;
        }
        if (here)
            copy_row(reinterpret_cast<float4 *>(P.rx[d] + row * H), reinterpret_cast<const float4 *>(x + (size_t)t * H),
                     H / 4, tid, blockDim.x);
    }
    release_peers(P, 0, epoch, ticket);
}

// the rank's expert outputs of this step are complete (stream order): release every peer's outputs-ready flag
__global__ void ep_signal_kernel(EpPeers P, const uint32_t *epoch_dev) {
    const uint32_t epoch = *epoch_dev + 1;
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int d = 0; d < P.world; d++) st_release_sys(P.flags[d] + P.world + P.rank, epoch);
    }
}

// combine: y[t] = ((0 + o_0) + o_1) + ... + o_{K-1}, slot k read from its owner's outputs (row rank * C + t). The
// slot's owner comes from the token's selections (this rank's top-k); all K loads are in flight before the adds.
__global__ void __launch_bounds__(256) ep_combine_kernel(const int32_t *__restrict__ sel, int n, EpPeers P,
                                                         float *__restrict__ y) {
    const int K = P.topk, H4 = P.hidden / 4;
    const int64_t total = (int64_t)n * H4;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / H4), c4 = (int)(i % H4);
        float4 v[kMaxTopK];
#pragma unroll
        for (int k = 0; k < kMaxTopK; k++)
            if (k < K) {
                const int e = __ldg(sel + (size_t)t * K + k);
                const int d = e / P.e_per;
                const float4 *o = reinterpret_cast<const float4 *>(P.out[d] + (((size_t)P.rank * P.cap + t) * K + k) *
                                                                                  P.hidden);
                v[k] = __ldcg(o + c4);  // the owner's memory (over NVLink for a peer), not cached in L1
            }
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < kMaxTopK; k++)
            if (k < K) {
                acc.x = __fadd_rn(acc.x, v[k].x); acc.y = __fadd_rn(acc.y, v[k].y);
                acc.z = __fadd_rn(acc.z, v[k].z); acc.w = __fadd_rn(acc.w, v[k].w);
            }
        reinterpret_cast<float4 *>(y + (size_t)t * P.hidden)[c4] = acc;
    }
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

// device-side rendezvous of all ranks (outside any step): advance the rank's rendezvous epoch, release it into every
// peer's rendezvous flag and wait (bounded) until every peer has released the same epoch
__global__ void ep_barrier_kernel(EpPeers P, uint32_t *bar_epoch, int32_t *err) {
    const uint32_t epoch = *bar_epoch + 1;
    const int lane = threadIdx.x;
    if (lane == 0) {
        __threadfence_system();
        for (int d = 0; d < P.world; d++) st_release_sys(P.flags[d] + 2 * P.world + P.rank, epoch);
    }
    __syncwarp();
    bool ok = true;
    if (lane < P.world) {
        const uint32_t *f = P.flags[P.rank] + 2 * P.world + lane;
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
    if (lane == 0) *bar_epoch = epoch;
}

}  // namespace

int launch_ep_barrier(const EpPeers &P, uint32_t *bar_epoch, int32_t *err, cudaStream_t st) {
    ep_barrier_kernel<<<1, 32, 0, st>>>(P, bar_epoch, err);
    return 1;
}

int launch_ep_dispatch(const float *logits, const float *x, int n, int E, const EpPeers &P, int32_t *sel_out,
                       const uint32_t *epoch_dev, int32_t *ticket, cudaStream_t st) {
    if (E % 32 || E > 32 * kMaxPerLane || P.topk > kMaxTopK) return -1;
    ep_dispatch_kernel<<<P.cap, 256, (size_t)E * sizeof(float), st>>>(logits, x, n, E, P, sel_out, epoch_dev, ticket);
    return 1;
}

int launch_ep_signal(const EpPeers &P, const uint32_t *epoch_dev, cudaStream_t st) {
    ep_signal_kernel<<<1, 32, 0, st>>>(P, epoch_dev);
    return 1;
}

int launch_ep_combine(const int32_t *sel, int n, const EpPeers &P, float *y, int num_sms, cudaStream_t st) {
    const int64_t total = (int64_t)n * P.hidden / 4;
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms * 8);
    ep_combine_kernel<<<blocks, 256, 0, st>>>(sel, n, P, y);
    return 1;
}

int launch_ep_wait(const uint32_t *flags, int world, int which, uint32_t *epoch_dev, bool advance, int32_t *err,
                   cudaStream_t st) {
    ep_wait_kernel<<<1, 32, 0, st>>>(flags, world, which, epoch_dev, advance ? 1 : 0, err);
    return 1;
}

}  // namespace inzg
