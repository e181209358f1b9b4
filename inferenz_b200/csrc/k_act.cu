// k_act.cu -- activation rotation + int8 quantization, SiLU*up, and the rank-order combine.
//
// Rotation: signs x_i * rot_sign(seed, i), then the unnormalised Walsh-Hadamard butterflies a+b / a-b with
// len = 1, 2, 4, ... inside each block, then * 1/sqrt(block) (src/quant.c:118-154). The butterfly network is the
// reference's, stage by stage, so every element sees the same sequence of IEEE adds.
// Decode numerics (src/quant.c:611-637): per 64-group s = amax/127, q = rne(x * (1/s)), and the group's sum of q
// (the reference keeps bsum = s * sum(q); the GEMV removes the LUT bias with the exact integer sum instead). The
// quantized bytes are stored in MMA B-fragment order: inside a group, thread t of a quad reads 16 bytes,
// q[4t..4t+3], q[16+4t..], q[32+4t..], q[48+4t..].
// Prefill numerics (src/quant.c:1407-1429): per 256-block (the last one partial) s = amax/127, q = lrint(x * (1/s)).
#include "inzg_internal.h"
#include "k_launch.h"

namespace inzg {

__device__ __forceinline__ int bfrag_pos(int j) { return ((j >> 2) & 3) * 16 + (j >> 4) * 4 + (j & 3); }

// in-place rotation of v[0..n) in shared memory by the whole block; n % block == 0
__device__ void rotate_smem(float *v, int n, int block, uint32_t seed, float norm) {
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        if (rot_sign_bit(seed, (uint32_t)i)) v[i] = -v[i];
    __syncthreads();
    const int half = n / 2;
    for (int len = 1; len < block; len <<= 1) {
        for (int p = threadIdx.x; p < half; p += blockDim.x) {
            const int b = p / (block / 2), q = p % (block / 2);
            const int i = b * block + (q / len) * 2 * len + (q % len), j = i + len;
            const float a = v[i], c = v[j];
            v[i] = __fadd_rn(a, c);
            v[j] = __fsub_rn(a, c);
        }
        __syncthreads();
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) v[i] = __fmul_rn(v[i], norm);
    __syncthreads();
}

// quantize v[0..n) (shared) by warps: 64-groups into q64 (B-fragment order) and sb64 = (scale bits, sum of q);
// and/or 256-blocks into q256, s256
__device__ void quantize_smem(const float *v, int n, int8_t *q64, int2 *sb64, int8_t *q256, float *s256) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (q64)
        for (int g = warp; g < n / kGroup; g += nw) {
            const float x0 = v[g * kGroup + lane], x1 = v[g * kGroup + 32 + lane];
            float amax = fmaxf(fabsf(x0), fabsf(x1));
            for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const float s = __fdiv_rn(amax, 127.0f);
            const float inv = s > 0 ? __fdiv_rn(1.0f, s) : 0.0f;
            const int a = __float2int_rn(__fmul_rn(x0, inv)), b = __float2int_rn(__fmul_rn(x1, inv));
            int sum = a + b;
            for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            q64[g * kGroup + bfrag_pos(lane)] = (int8_t)a;
            q64[g * kGroup + bfrag_pos(32 + lane)] = (int8_t)b;
            if (lane == 0) sb64[g] = make_int2(__float_as_int(s), sum);
        }
    if (q256) {
        const int nkb = (n + kKB - 1) / kKB;
        for (int b = warp; b < nkb; b += nw) {
            const int k0 = b * kKB, len = min(kKB, n - k0);
            float amax = 0.0f;
            for (int k = lane; k < len; k += 32) amax = fmaxf(amax, fabsf(v[k0 + k]));
            for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const float s = __fdiv_rn(amax, 127.0f);
            const float inv = s > 0 ? __fdiv_rn(1.0f, s) : 0.0f;
            for (int k = lane; k < len; k += 32) q256[k0 + k] = (int8_t)__float2int_rn(__fmul_rn(v[k0 + k], inv));
            if (lane == 0) s256[b] = s;
        }
    }
}

// one block per token: x [n][H] -> decode activations (q64, s64, b64) and prefill activations (q256, s256)
__global__ void __launch_bounds__(256) act_quant_x_kernel(const float *__restrict__ X, int n, int H, int rot, uint32_t seed,
                                                          float norm, int8_t *__restrict__ q64, int2 *__restrict__ sb64,
                                                          int8_t *__restrict__ q256, float *__restrict__ s256) {
    extern __shared__ float v[];
    const int t = blockIdx.x;
    for (int i = threadIdx.x; i < H; i += blockDim.x) v[i] = X[(size_t)t * H + i];
    __syncthreads();
    if (rot > 1) rotate_smem(v, H, rot, seed, norm);
    const int ng = H / kGroup, nkb = (H + kKB - 1) / kKB;
    quantize_smem(v, H, q64 + (size_t)t * H, sb64 + (size_t)t * ng, q256 ? q256 + (size_t)t * H : nullptr,
                  q256 ? s256 + (size_t)t * nkb : nullptr);
}

// The expert's input to its down matrix, one block per entry: h = silu(g) * u (src/model_fwd.c:43, 859-862, 925,
// siluf = x / (1 + expf(-x))), rotated with the down matrix's rotation, then quantized with the numerics of the
// expert's path. exp is evaluated in double and rounded once (glibc's expf agrees with that on all but ~1e-4 of
// inputs, by at most one ulp).
__global__ void __launch_bounds__(128) swiglu_quant_kernel(const float *__restrict__ GU, int FF, int n_entries,
                                                           const int32_t *__restrict__ eexp, const int32_t *__restrict__ upath,
                                                           int rot, uint32_t seed, float norm, int8_t *__restrict__ q64,
                                                           int2 *__restrict__ sb64, int8_t *__restrict__ q256,
                                                           float *__restrict__ s256) {
    extern __shared__ float v[];
    const int pos = blockIdx.x;
    if (pos >= n_entries) return;
    const float *g = GU + (size_t)pos * 2 * FF;
    for (int c = threadIdx.x; c < FF; c += blockDim.x) {
        const float x = g[c];
        const float ex = (float)exp(-(double)x);
        v[c] = __fmul_rn(__fdiv_rn(x, __fadd_rn(1.0f, ex)), g[FF + c]);
    }
    __syncthreads();
    if (rot > 1) rotate_smem(v, FF, rot, seed, norm);
    const int ng = FF / kGroup, nkb = (FF + kKB - 1) / kKB;
    const bool gemm = upath[eexp[pos]] != 0;
    if (gemm) quantize_smem(v, FF, nullptr, nullptr, q256 + (size_t)pos * FF, s256 + (size_t)pos * nkb);
    else quantize_smem(v, FF, q64 + (size_t)pos * FF, sb64 + (size_t)pos * ng, nullptr, nullptr);
}

// y[t][c] = (((0 + o[t,0][c]) + o[t,1][c]) + ...) in rank order (src/model_fwd.c:1033, 1134-1140)
__global__ void combine_kernel(const float *__restrict__ mo, int n, int H, int topk, float *__restrict__ y) {
    const int64_t total = (int64_t)n * H / 4;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / (H / 4), c4 = i % (H / 4);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k = 0; k < topk; k++) {
            const float4 o = reinterpret_cast<const float4 *>(mo + ((size_t)t * topk + k) * H)[c4];
            acc.x = __fadd_rn(acc.x, o.x); acc.y = __fadd_rn(acc.y, o.y);
            acc.z = __fadd_rn(acc.z, o.z); acc.w = __fadd_rn(acc.w, o.w);
        }
        reinterpret_cast<float4 *>(y + (size_t)t * H)[c4] = acc;
    }
}

// Prefill-path token activations in entry order (entries sorted by expert, then token), so a GEMM tile's tokens are
// consecutive rows for TMA: qe[pos] = q[etok[pos]], se[pos] = s[etok[pos]] for entries of prefill-path experts.
__global__ void gather_gemm_rows_kernel(const int8_t *__restrict__ q, const float *__restrict__ s, int K, int nkb,
                                        const int32_t *__restrict__ etok, const int32_t *__restrict__ eexp,
                                        const int32_t *__restrict__ upath, int n_entries, int8_t *__restrict__ qe,
                                        float *__restrict__ se) {
    const int K16 = K / 16;
    for (int pos = blockIdx.x; pos < n_entries; pos += gridDim.x) {
        if (!upath[eexp[pos]]) continue;  // uniform over the block
        const int t = etok[pos];
        const uint4 *src = reinterpret_cast<const uint4 *>(q + (size_t)t * K);
        uint4 *dst = reinterpret_cast<uint4 *>(qe + (size_t)pos * K);
        for (int i = threadIdx.x; i < K16; i += blockDim.x) dst[i] = src[i];
        if (threadIdx.x < nkb) se[(size_t)pos * nkb + threadIdx.x] = s[(size_t)t * nkb + threadIdx.x];
    }
}

int launch_gather_gemm_rows(const int8_t *q, const float *s, int K, int nkb, const int32_t *etok, const int32_t *eexp,
                            const int32_t *upath, int n_entries, int8_t *qe, float *se, cudaStream_t st) {
    const int blocks = n_entries < 4096 ? n_entries : 4096;
    gather_gemm_rows_kernel<<<blocks, 128, 0, st>>>(q, s, K, nkb, etok, eexp, upath, n_entries, qe, se);
    return 1;
}

int launch_act_quant_x(const float *X, int n, int H, int rot, uint32_t seed, int8_t *q64, int2 *sb64, int8_t *q256,
                       float *s256, cudaStream_t st) {
    const float norm = rot > 1 ? 1.0f / sqrtf((float)rot) : 1.0f;
    act_quant_x_kernel<<<n, 256, H * sizeof(float), st>>>(X, n, H, rot, seed, norm, q64, sb64, q256, s256);
    return 1;
}

int launch_swiglu_quant(const float *GU, int FF, int n_entries, const int32_t *eexp, const int32_t *upath, int rot,
                        uint32_t seed, int8_t *q64, int2 *sb64, int8_t *q256, float *s256, cudaStream_t st) {
    const float norm = rot > 1 ? 1.0f / sqrtf((float)rot) : 1.0f;
    swiglu_quant_kernel<<<n_entries, 128, FF * sizeof(float), st>>>(GU, FF, n_entries, eexp, upath, rot, seed, norm, q64,
                                                                     sb64, q256, s256);
    return 1;
}

int launch_combine(const float *mo, int n, int H, int topk, float *y, int num_sms, cudaStream_t st) {
    const int64_t total = (int64_t)n * H / 4;
    int blocks = (int)((total + 255) / 256);
    if (blocks > num_sms * 8) blocks = num_sms * 8;
    combine_kernel<<<blocks, 256, 0, st>>>(mo, n, H, topk, y);
    return 1;
}

}  // namespace inzg
