// k_probe.cu -- roofline probe of the int8 tensor pipe (tcgen05.mma kind::i8), the denominator of the prefill GEMM's
// tensor-pipe fraction. The B200 counterpart of the reference's own roofline probe (the RAM bandwidth probe of its
// diagnostics, src/diag.c:363-394): one CTA per SM issues back-to-back 128 x 256 x 32 int8 MMAs from shared memory
// into two TMEM accumulators -- no global traffic -- and the host divides the MMAs' integer operations by the kernel's
// CUDA-event time. Every wait is bounded; a CTA whose commit never arrives records it and still frees its TMEM.
#include <cuda_runtime.h>

#include "inzg_internal.h"
#include "k_async.cuh"
#include "host/inzg_host.h"

namespace inzg {
namespace {

constexpr int kPM = 128, kPN = 256, kPK = 128;  // one 128-byte K chunk: 4 MMAs of K = 32
constexpr int kPAbytes = kPM * kPK, kPBbytes = kPN * kPK;

__device__ __forceinline__ uint64_t probe_desc(const void *smem) {  // K-major, 128-byte swizzle, SBO 1024 B
    const uint64_t a = smem_u32(smem);
    return ((a & 0x3FFFFull) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// s32 accumulate, s8 x s8, K-major A and B, N = 256, M = 128
constexpr uint32_t kProbeIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kPN >> 3) << 17) |
                                 ((uint32_t)(kPM >> 4) << 24);

__global__ void __launch_bounds__(64, 1) tensor_i8_probe_kernel(int iters, int32_t *status) {
    extern __shared__ __align__(1024) uint8_t dyn[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dyn) + 1023) & ~uintptr_t(1023));
    uint8_t *A = base, *B = base + kPAbytes;
    __shared__ uint64_t done;
    __shared__ uint32_t tmem_base;
    const int warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < (kPAbytes + kPBbytes) / 4; i += blockDim.x)
        reinterpret_cast<uint32_t *>(A)[i] = 0x01010101u * (uint32_t)(i & 7);
    fence_proxy_async_smem();
    if (threadIdx.x == 0) {
        mbar_init(&done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&tmem_base)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base;
    if (threadIdx.x == 32) {
        for (int it = 0; it < iters; it++) {
            const uint32_t d = tmem + (uint32_t)((it & 1) * kPN);
#pragma unroll
            for (int k = 0; k < kPK / 32; k++) {
                const uint64_t a = probe_desc(A + 32 * k), b = probe_desc(B + 32 * k);
                asm volatile(
                    "{\n\t.reg .pred p;\n\t"
                    "setp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d),
                    "l"(a), "l"(b), "r"(kProbeIdesc), "r"(k | (it >> 1)), "r"(0), "r"(0), "r"(0), "r"(0));
            }
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&done))
                     : "memory");
    }
    __syncwarp();
    if (threadIdx.x == 32 || threadIdx.x == 0) {
        if (!mbar_wait_bounded(&done, 0)) {
            if (threadIdx.x == 0) atomicExch(status, kErrTimeout);
            // the MMAs may still write TMEM: keep waiting (bounded) before the columns are released
            for (int r = 0; r < 64 && !mbar_wait_bounded(&done, 0); r++) {
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

}  // namespace
}  // namespace inzg

extern "C" INZG_API int inzg_probe_tensor_i8(int device, int iters, double *tops, double *ms) {
    using namespace inzg;
    if (!tops || iters < 2) return -1;
    int saved = -1;
    cudaGetDevice(&saved);
    if (cudaSetDevice(device) != cudaSuccess) return -1;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    // more shared memory than two CTAs can hold on one SM: one probe CTA per SM, each with all 512 TMEM columns
    const int smem = 120 * 1024;
    int32_t *status = nullptr;
    cudaEvent_t a = nullptr, b = nullptr;
    int rc = -1;
    float t = 0.0f;
    if (cudaMalloc(&status, sizeof(int32_t)) == cudaSuccess && cudaMemset(status, 0, sizeof(int32_t)) == cudaSuccess &&
        cudaFuncSetAttribute(tensor_i8_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess &&
        cudaEventCreate(&a) == cudaSuccess && cudaEventCreate(&b) == cudaSuccess) {
        tensor_i8_probe_kernel<<<sms, 64, smem>>>(iters / 8, status);  // warm-up
        cudaEventRecord(a);
        tensor_i8_probe_kernel<<<sms, 64, smem>>>(iters, status);
        cudaEventRecord(b);
        int32_t st = 0;
        if (cudaEventSynchronize(b) == cudaSuccess && cudaEventElapsedTime(&t, a, b) == cudaSuccess &&
            cudaMemcpy(&st, status, sizeof(st), cudaMemcpyDeviceToHost) == cudaSuccess && st == 0 && t > 0.0f) {
            const double ops = (double)sms * iters * (kPK / 32) * 2.0 * kPM * kPN * 32;
            *tops = ops / (t * 1e-3) / 1e12;
            if (ms) *ms = t;
            rc = 0;
        }
    }
    cudaGetLastError();
    if (a) cudaEventDestroy(a);
    if (b) cudaEventDestroy(b);
    if (status) cudaFree(status);
    if (saved >= 0) cudaSetDevice(saved);
    return rc;
}

// The architecture the library's kernels were built for and run as on `device`: cudaFuncGetAttributes of one of them
// (binaryVersion 100 = sm_100 SASS, loaded without a PTX recompilation).
extern "C" INZG_API int inzg_kernel_arch(int device, int *binary_version, int *ptx_version) {
    int saved = -1;
    cudaGetDevice(&saved);
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    cudaFuncAttributes fa{};
    const cudaError_t e = cudaFuncGetAttributes(&fa, inzg::tensor_i8_probe_kernel);
    if (saved >= 0) cudaSetDevice(saved);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    if (binary_version) *binary_version = fa.binaryVersion;
    if (ptx_version) *ptx_version = fa.ptxVersion;
    return 0;
}
