// k_act.cu -- activation rotation + int8 quantization, SiLU*up, and the rank-order combine.
//
// Rotation: signs x_i * rot_sign(seed, i), then the unnormalised Walsh-Hadamard butterflies a+b / a-b with
// len = 1, 2, 4, ... inside each block, then * 1/sqrt(block) (src/quant.c:118-154). The butterfly network is the
// reference's, stage by stage, so every element sees the same sequence of IEEE adds.
// Decode numerics (src/quant.c:611-637): per 64-group s = amax/127, q = rne(x * (1/s)), bsum = s * sum(q); the
// bytes stay in natural order and each group's (s, bsum) is one float2.
// Prefill numerics (src/quant.c:1407-1429): per 256-block (the last one partial) s = amax/127, q = lrint(x * (1/s)).
#include "inzg_internal.h"
#include "k_launch.h"
#include "k_warpq.cuh"

namespace inzg {

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

// quantize v[0..n) (shared) by warps: 64-groups into q64 and sb64 = (s, bsum); and/or 256-blocks into q256, s256
__device__ void quantize_smem(const float *v, int n, int8_t *q64, float2 *sb64, int8_t *q256, float *s256) {
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
            q64[g * kGroup + lane] = (int8_t)a;
            q64[g * kGroup + 32 + lane] = (int8_t)b;
            if (lane == 0) sb64[g] = make_float2(s, __fmul_rn(s, (float)sum));
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
                                                          float norm, int8_t *__restrict__ q64, float2 *__restrict__ sb64,
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
// expert's path. exp is evaluated in double and rounded once: glibc's expf gives the same float on all but ~1e-4 of
// inputs (by one ulp), where CUDA's expf (2 ulp) differs far more often -- every SiLU ulp can flip an int8 rounding
// of the down projection's input.
__global__ void __launch_bounds__(128) swiglu_quant_kernel(const float *__restrict__ GU, int FF, int n_entries,
                                                           const int32_t *__restrict__ eexp, const int32_t *__restrict__ upath,
                                                           int rot, uint32_t seed, float norm, int8_t *__restrict__ q64,
                                                           float2 *__restrict__ sb64, int8_t *__restrict__ q256,
                                                           float *__restrict__ s256) {
    extern __shared__ float v[];
    const int pos = blockIdx.x;
    if (pos >= n_entries) return;
    const float *g = GU + (size_t)pos * 2 * FF;
    for (int c = threadIdx.x; c < FF; c += blockDim.x) {
        const float x = g[c];
        v[c] = __fmul_rn(__fdiv_rn(x, __fadd_rn(1.0f, (float)exp(-(double)x))), g[FF + c]);
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

// one warp per (token, 256-element rotation block): x [n][H] (H = NB * 256); the block is also a 256-block of the
// prefill numerics and holds four 64-groups of the decode numerics, so every warp works alone
template <int NB>
__global__ void __launch_bounds__(256) act_quant_x_warp_kernel(const float *__restrict__ X, int n, uint32_t seed,
                                                               float norm, int8_t *__restrict__ q64,
                                                               float2 *__restrict__ sb64, int8_t *__restrict__ q256,
                                                               float *__restrict__ s256) {
    constexpr int VPL = 8, H = NB * 256;
    const int lane = threadIdx.x & 31;
    const int wi = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int t = wi / NB, b = wi % NB;
    if (t >= n) return;
    float v[1][VPL];
    const float *x = X + (size_t)t * H + b * 256;
    const float4 a = reinterpret_cast<const float4 *>(x + lane * 8)[0];
    const float4 c = reinterpret_cast<const float4 *>(x + lane * 8)[1];
    v[0][0] = a.x; v[0][1] = a.y; v[0][2] = a.z; v[0][3] = a.w;
    v[0][4] = c.x; v[0][5] = c.y; v[0][6] = c.z; v[0][7] = c.w;
    warp_rotate<1, VPL>(v, seed, norm, lane, b * 256);
    const size_t o = (size_t)t * H + b * 256;
    warp_quantize<1, VPL>(v, 256, lane, q64 + o, sb64 + o / kGroup, q256 ? q256 + o : nullptr,
                          q256 ? s256 + (size_t)t * (H / kKB) + b : nullptr);
}

// One block of NB warps per entry: h = silu(g) * u over FF = NB * 128 values (siluf, src/model_fwd.c:43), warp w
// rotates block w (rotation block 128). Decode-path entries quantize per 64-group inside each warp; prefill-path
// entries quantize per 256-block (blocks 2w, 2w+1 -- the last one partial), the two warps of a block meeting in
// shared memory for its amax.
template <int NB>
__global__ void __launch_bounds__(NB * 32) swiglu_quant_warp_kernel(const float *__restrict__ GU, int n_entries,
                                                                    const int32_t *__restrict__ eexp,
                                                                    const int32_t *__restrict__ upath, uint32_t seed,
                                                                    float norm, int8_t *__restrict__ q64,
                                                                    float2 *__restrict__ sb64, int8_t *__restrict__ q256,
                                                                    float *__restrict__ s256) {
    constexpr int VPL = 4, FF = NB * 128, NKB = (FF + kKB - 1) / kKB;
    __shared__ float amax_w[NB];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int pos = blockIdx.x;
    if (pos >= n_entries) return;
    const float *g = GU + (size_t)pos * 2 * FF;
    float v[1][VPL];
    {
        const float4 a = reinterpret_cast<const float4 *>(g + w * 128 + lane * 4)[0];
        const float4 u = reinterpret_cast<const float4 *>(g + FF + w * 128 + lane * 4)[0];
        const float av[4] = {a.x, a.y, a.z, a.w}, uv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int r = 0; r < 4; r++)
            v[0][r] = __fmul_rn(__fdiv_rn(av[r], __fadd_rn(1.0f, (float)exp(-(double)av[r]))), uv[r]);
    }
    warp_rotate<1, VPL>(v, seed, norm, lane, w * 128);
    const bool gemm = upath[eexp[pos]] != 0;
    if (!gemm) {
        const size_t o = (size_t)pos * FF + w * 128;
        warp_quantize<1, VPL>(v, 128, lane, q64 + o, sb64 + o / kGroup, nullptr, nullptr);
        return;
    }
    float am = 0.0f;
#pragma unroll
    for (int r = 0; r < VPL; r++) am = fmaxf(am, fabsf(v[0][r]));
#pragma unroll
    for (int o = 16; o; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    if (lane == 0) amax_w[w] = am;
    __syncthreads();
    const int kb = w >> 1;
    const float amax = (2 * kb + 1 < NB) ? fmaxf(amax_w[2 * kb], amax_w[2 * kb + 1]) : amax_w[2 * kb];
    const float sc = __fdiv_rn(amax, 127.0f);
    const float inv = sc > 0 ? __fdiv_rn(1.0f, sc) : 0.0f;
    int q[4];
#pragma unroll
    for (int r = 0; r < 4; r++) q[r] = __float2int_rn(__fmul_rn(v[0][r], inv));
    *reinterpret_cast<uint32_t *>(q256 + (size_t)pos * FF + w * 128 + lane * 4) = pack4(q[0], q[1], q[2], q[3]);
    if (lane == 0 && (w & 1) == 0) s256[(size_t)pos * NKB + kb] = sc;
}

// Shared-expert gate and add (src/model_fwd.c:1141-1148), one block per token:
//   sg = sigmoidf(dot_f32(sh_gate, x)) -- dot_f32 (src/model_fwd.c:24-34) keeps two 8-lane fma accumulators over
//   16-element blocks (s0: elements 16i + l, s1: 16i + 8 + l), adds them lane-wise and reduces with hsum8;
//   sigmoidf = 1 / (1 + expf(-x)), exp in double rounded once (as SiLU's) --
// then y = fma(sg, D, y) per element (the reference build contracts `y += sg * D` into one fma).
// Also carries the shared unit's device error word into the call's.
__global__ void __launch_bounds__(256) shared_add_kernel(const float *__restrict__ X, const float *__restrict__ gate,
                                                         const float *__restrict__ D, float *__restrict__ y, int H,
                                                         const int32_t *__restrict__ sh_meta, int32_t *__restrict__ meta) {
    __shared__ float sg_s;
    const int t = blockIdx.x, tid = threadIdx.x;
    const float *x = X + (size_t)t * H;
    if (tid < 32) {
        // lanes 0-7: s0 lane l; lanes 8-15: s1 lane l (element 16i + 8 + l); each a chain over the 16-blocks in order
        float a = 0.0f;
        if (tid < 16)
            for (int i = 0; i + 16 <= H; i += 16) a = __fmaf_rn(gate[i + tid], x[i + tid], a);
        const float v = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 8));  // s0 + s1, lane-wise (lanes 0-7)
        const float s = hsum8_lanes(v);                                     // valid in lanes 0-7
        if (tid == 0) sg_s = __fdiv_rn(1.0f, __fadd_rn(1.0f, (float)exp(-(double)s)));  // H % 16 == 0: no tail
    }
    __syncthreads();
    const float sg = sg_s;
    float *yt = y + (size_t)t * H;
    const float *dt = D + (size_t)t * H;
    for (int c = tid; c < H; c += blockDim.x) yt[c] = __fmaf_rn(sg, dt[c], yt[c]);
    if (t == 0 && tid == 0 && sh_meta[kMetaError] != kErrNone) set_error(meta, sh_meta[kMetaError]);
}

int launch_shared_add(const float *X, const float *gate, const float *D, float *y, int n, int H, const int32_t *sh_meta,
                      int32_t *meta, cudaStream_t st) {
    shared_add_kernel<<<n, 256, 0, st>>>(X, gate, D, y, H, sh_meta, meta);
    return 1;
}

int launch_act_quant_x(const float *X, int n, int H, int rot, uint32_t seed, int8_t *q64, float2 *sb64, int8_t *q256,
                       float *s256, cudaStream_t st) {
    const float norm = rot > 1 ? 1.0f / sqrtf((float)rot) : 1.0f;
    if (rot == 256 && H == 2048) {
        act_quant_x_warp_kernel<8><<<n, 256, 0, st>>>(X, n, seed, norm, q64, sb64, q256, s256);
    } else if (rot == 256 && H == 2560) {
        act_quant_x_warp_kernel<10><<<(n * 10 + 7) / 8, 256, 0, st>>>(X, n, seed, norm, q64, sb64, q256, s256);
    } else {
        act_quant_x_kernel<<<n, 256, H * sizeof(float), st>>>(X, n, H, rot, seed, norm, q64, sb64, q256, s256);
    }
    return 1;
}

int launch_swiglu_quant(const float *GU, int FF, int n_entries, const int32_t *eexp, const int32_t *upath, int rot,
                        uint32_t seed, int8_t *q64, float2 *sb64, int8_t *q256, float *s256, cudaStream_t st) {
    const float norm = rot > 1 ? 1.0f / sqrtf((float)rot) : 1.0f;
    if (rot == 128 && FF == 640) {
        swiglu_quant_warp_kernel<5><<<n_entries, 160, 0, st>>>(GU, n_entries, eexp, upath, seed, norm, q64, sb64, q256,
                                                               s256);
        return 1;
    }
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
