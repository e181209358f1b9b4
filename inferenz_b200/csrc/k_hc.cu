// k_hc.cu -- the hyper-connection steps either side of the MoE layer on sm_100a (src/model_fwd.c:404-450):
//   hc_in:  Xn = per-stream rmsnorm(X) * norm; d = silu((down . Xn) / 4); m = up . d;
//           xin = (sum_s fma(sigmoid(m_s), Xn_s)) * 0.25; inj_s = 2 sigmoid((inject_s . Xn) / 4)
//   hc_out: X_s = fma(inj_s, y, X_s)
// The down/up products are lin_mm's F16 path (the router's kernels, launch_f16_rows). Everything is bit-exact with
// the reference build except the two places glibc's expf enters (the SiLU of the rank-320 bottleneck and the inject
// sigmoid): there exp is evaluated in double and rounded once, as for the experts' SiLU.
#include "inzg_internal.h"
#include "k_launch.h"
#include "k_softmax.cuh"

namespace inzg {

// dot_f32 (src/model_fwd.c:24-34) by one warp: lane l < 8 runs accumulator s0's lane l (elements 16i + l), lane 8 + l
// runs s1's lane l (16i + 8 + l), each over the 16-element blocks in order; then s0 + s1 lane-wise and hsum8. n % 16
// == 0. The result is valid in lanes 0-7.
__device__ __forceinline__ float warp_dot_f32(const float *a, const float *b, int n) {
    const int lane = threadIdx.x & 31;
    float acc = 0.0f;
    if (lane < 16) {
#pragma unroll 8
        for (int i = 0; i < n; i += 16) acc = __fmaf_rn(a[i + lane], b[i + lane], acc);
    }
    return hsum8_lanes(__fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 8)));
}

// rmsnorm (src/model_fwd.c:37-40) of one stream of one token per block: r = 1 / sqrtf(dot_f32(x, x, H) / H + 1e-6f),
// out = (x * r) * norm
__global__ void __launch_bounds__(256) hc_norm_kernel(const float *__restrict__ X, const float *__restrict__ norm,
                                                      int H, float *__restrict__ Xn) {
    extern __shared__ __align__(16) float xs[];
    __shared__ float r_s;
    const int t = blockIdx.x >> 2, s = blockIdx.x & 3, tid = threadIdx.x;
    const size_t off = (size_t)t * 4 * H + (size_t)s * H;
    for (int i = tid; i < H / 4; i += blockDim.x)
        reinterpret_cast<float4 *>(xs)[i] = reinterpret_cast<const float4 *>(X + off)[i];
    __syncthreads();
    if (tid < 32) {
        const float d = warp_dot_f32(xs, xs, H);
        if (tid == 0) r_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(d, (float)H), 1e-6f)));
    }
    __syncthreads();
    const float r = r_s;
    const float *w = norm + (size_t)s * H;
    float *o = Xn + off;
    for (int i = tid; i < H; i += blockDim.x) o[i] = __fmul_rn(__fmul_rn(xs[i], r), w[i]);
}

// d = siluf(d / 4) (src/model_fwd.c:436), exp in double rounded once
__global__ void hc_silu_kernel(float *__restrict__ d, int count) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
        const float x = __fdiv_rn(d[i], 4.0f);
        d[i] = __fdiv_rn(x, __fadd_rn(1.0f, (float)exp(-(double)x)));
    }
}

// xin[t][i] = (sum over s of fma(sigmoid256(m[t][sH + i]), Xn[t][sH + i], acc)) * 0.25 (src/model_fwd.c:413-424);
// sigmoid256 = 1 / (1 + exp256_ps(0 - x)), the Cephes exp (src/model_fwd.c:397-400)
__global__ void hc_mix_kernel(const float *__restrict__ m, const float *__restrict__ Xn, int n, int H,
                              float *__restrict__ xin) {
    const int64_t total = (int64_t)n * H;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = idx / H, i = idx % H;
        const float *mt = m + t * 4 * H + i, *xt = Xn + t * 4 * H + i;
        float acc = 0.0f;
#pragma unroll
        for (int s = 0; s < 4; s++) {
            const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, cephes_exp(__fsub_rn(0.0f, mt[(size_t)s * H]))));
            acc = __fmaf_rn(sg, xt[(size_t)s * H], acc);
        }
        xin[idx] = __fmul_rn(acc, 0.25f);
    }
}

// inj[t][s] = 2 sigmoidf(dot_f32(inject_s, Xn_t, 4H) / 4) (src/model_fwd.c:425-427), one block per (token, stream):
// both vectors staged in shared memory, then one warp runs the 16 accumulator chains
__global__ void __launch_bounds__(256) hc_inj_kernel(const float *__restrict__ Xn, const float *__restrict__ inject,
                                                     int H, float *__restrict__ inj) {
    extern __shared__ __align__(16) float sv[];  // [2][4H]
    const int t = blockIdx.x >> 2, s = blockIdx.x & 3, W = 4 * H, tid = threadIdx.x;
    const float4 *a = reinterpret_cast<const float4 *>(inject + (size_t)s * W);
    const float4 *b = reinterpret_cast<const float4 *>(Xn + (size_t)t * W);
    for (int i = tid; i < W / 4; i += blockDim.x) {
        reinterpret_cast<float4 *>(sv)[i] = a[i];
        reinterpret_cast<float4 *>(sv + W)[i] = b[i];
    }
    __syncthreads();
    if (tid < 32) {
        const float d = warp_dot_f32(sv, sv + W, W);
        if (tid == 0) {
            const float x = __fdiv_rn(d, 4.0f);
            inj[(size_t)t * 4 + s] = __fmul_rn(2.0f, __fdiv_rn(1.0f, __fadd_rn(1.0f, (float)exp(-(double)x))));
        }
    }
}

// X[t][sH + i] = fma(inj[t][s], y[t][i], X[t][sH + i]) (src/model_fwd.c:442-450; the reference build contracts
// `x += w * y` into one fma), four elements per thread
__global__ void hc_out_kernel(float *__restrict__ X, const float *__restrict__ inj, const float *__restrict__ y, int n,
                              int H) {
    const int H4 = H / 4;
    const int64_t total = (int64_t)n * 4 * H4;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = idx / (4 * H4);
        const int s = (int)((idx / H4) % 4), i4 = (int)(idx % H4);
        const float w = inj[t * 4 + s];
        const float4 yv = reinterpret_cast<const float4 *>(y + t * H)[i4];
        float4 &xv = reinterpret_cast<float4 *>(X)[idx];
        float4 v = xv;
        v.x = __fmaf_rn(w, yv.x, v.x); v.y = __fmaf_rn(w, yv.y, v.y);
        v.z = __fmaf_rn(w, yv.z, v.z); v.w = __fmaf_rn(w, yv.w, v.w);
        xv = v;
    }
}

static int grid_for(int64_t items, int threads, int num_sms) {
    const int64_t b = (items + threads - 1) / threads, cap = (int64_t)num_sms * 8;
    return (int)(b < 1 ? 1 : b > cap ? cap : b);
}

void hc_set_attributes(int H) {
    cudaFuncSetAttribute(hc_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, H * 4);
    cudaFuncSetAttribute(hc_inj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 4 * H * 4);
    router_set_attributes(4 * H);  // the down matrix is 4H wide
}

int launch_hc_in(const HcDev &w, int n, int H, const float *X, float *Xn, float *d, float *m, float *xin, float *inj,
                 int32_t *meta, int num_sms, cudaStream_t st) {
    const int W = 4 * H;
    int launches = 0;
    hc_norm_kernel<<<n * 4, 256, H * 4, st>>>(X, w.norm, H, Xn);
    launches++;
    int k = launch_f16_rows(w.down, w.down32, Xn, n, W, w.rank, d, meta, st);
    if (k < 0) return -1;
    launches += k;
    hc_silu_kernel<<<grid_for((int64_t)n * w.rank, 256, num_sms), 256, 0, st>>>(d, n * w.rank);
    launches++;
    k = launch_f16_rows(w.up, w.up32, d, n, w.rank, W, m, meta, st);
    if (k < 0) return -1;
    launches += k;
    hc_mix_kernel<<<grid_for((int64_t)n * H, 256, num_sms), 256, 0, st>>>(m, Xn, n, H, xin);
    launches++;
    if (w.inject && inj) {
        hc_inj_kernel<<<n * 4, 256, 2 * W * 4, st>>>(Xn, w.inject, H, inj);
        launches++;
    }
    return launches;
}

int launch_hc_out(float *X, const float *inj, const float *y, int n, int H, int num_sms, cudaStream_t st) {
    hc_out_kernel<<<grid_for((int64_t)n * H, 256, num_sms), 256, 0, st>>>(X, inj, y, n, H);
    return 1;
}

}  // namespace inzg
