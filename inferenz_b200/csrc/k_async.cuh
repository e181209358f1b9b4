// k_async.cuh -- mbarrier and bulk-copy (TMA engine) primitives shared by the pipelined kernels, sm_100a.
// Every wait is bounded: a wait that runs out returns false and the caller records kErrTimeout.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace inzg {

constexpr uint32_t kWaitLimit = 1u << 20;  // try_wait rounds before a wait is declared stuck

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t *b, uint32_t par) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(par)
        : "memory");
    return ok != 0;
}
// bounded wait for the phase with parity `par` to complete
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *b, uint32_t par) {
    for (uint32_t i = 0; i < kWaitLimit; i++)
        if (mbar_try(b, par)) return true;
    return false;
}

// bounded wait that also gives up once another warp of the CTA has raised `abort`
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t par, volatile int *abort) {
    for (uint32_t i = 0; i < kWaitLimit; i++) {
        if (mbar_try(b, par)) return true;
        if ((i & 255) == 255 && *abort) return false;
    }
    return false;
}

// one bulk copy global -> shared (this CTA), completion counted on `bar` as transaction bytes.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// one tiled tensor copy global -> shared (this CTA, no multicast) of the box at (x, y); x * element size must be a
// multiple of 16 bytes
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// order this thread's earlier generic-proxy shared-memory accesses before later async-proxy (bulk copy) writes
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

}  // namespace inzg
