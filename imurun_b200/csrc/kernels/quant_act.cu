// quant_act.cu — activation quantisation and the kernels that produce it.
//
// The int8 activation records must be byte-identical to the reference's
// (src/quant.cpp:400-434, src/quant_x86.cpp:499-570): per block
//   amax = max |x|, d = amax / 127 (IEEE division), id = d > 0 ? 1/d : 0,
//   q = clamp(round_half_even(x * id), -127, 127), sums of q.
// Every float step uses an explicitly rounded intrinsic so no contraction or
// approximate reciprocal can change a byte.
//
// Work split: a row of K values is cut into 256-value chunks; one warp owns a
// chunk (lane = 8 consecutive values) and a CTA of 4 warps owns 4 chunks, so a
// single decode token still spreads over K/1024 CTAs.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace fb {

constexpr int kQWarps = 4;

__device__ __forceinline__ uint2 pack8(const int (&q)[8]) {
    uint2 p;
    p.x = (q[0] & 0xFF) | ((q[1] & 0xFF) << 8) | ((q[2] & 0xFF) << 16) | ((uint32_t)(q[3] & 0xFF) << 24);
    p.y = (q[4] & 0xFF) | ((q[5] & 0xFF) << 8) | ((q[6] & 0xFF) << 16) | ((uint32_t)(q[7] & 0xFF) << 24);
    return p;
}

__device__ __forceinline__ int quant8(const float (&v)[8], float id, int (&q)[8]) {
    int s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        int r = __float2int_rn(__fmul_rn(v[i], id));
        r = max(-127, min(127, r));
        q[i] = r;
        s += r;
    }
    return s;
}

// Quantise chunk c (values 256c .. 256c+255, lane holds 8 of them) of row t.
// A partial last chunk (K % 256 != 0) only gets the 32-value layout, which
// matches the reference: the 256 layout exists only when K % 256 == 0
// (src/ops.cpp:166-174).
__device__ __forceinline__ void quant_chunk(const float (&v)[8], int lane, int K, int t, int c, const ActQ& a,
                                            int want32, int wantk) {
    const int base = c * 256;
    const bool full = base + 256 <= K;
    float am = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(v[i]));
    if (wantk && full) {
        const float amax = warp_max(am);
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        int q[8];
        int s = quant8(v, id, q);
        *reinterpret_cast<uint2*>(a.qk + (size_t)t * a.ld + base + 8 * lane) = pack8(q);
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if ((lane & 3) == 0) a.bsk[(size_t)t * (a.K / 32) + base / 32 + (lane >> 2)] = (int16_t)s;
        if (lane == 0) a.dk[(size_t)t * (a.K / 256) + c] = d;
    }
    if (want32) {
        // 32-value blocks: lanes 4g .. 4g+3 hold block g of the chunk
        float b = am;
        b = fmaxf(b, __shfl_xor_sync(0xffffffffu, b, 1));
        b = fmaxf(b, __shfl_xor_sync(0xffffffffu, b, 2));
        const float d = __fdiv_rn(b, 127.0f);
        const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        int q[8];
        int s = quant8(v, id, q);
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if (base + 8 * lane < K) {
            *reinterpret_cast<uint2*>(a.q32 + (size_t)t * a.ld + base + 8 * lane) = pack8(q);
            if ((lane & 3) == 0) {
                a.d32[(size_t)t * (a.K / 32) + base / 32 + (lane >> 2)] = d;
                if (a.s32) a.s32[(size_t)t * (a.K / 32) + base / 32 + (lane >> 2)] = s;
            }
        }
    }
}

__device__ __forceinline__ void load8(const float* src, int base, int lane, int K, float (&v)[8]) {
    const int i0 = base + 8 * lane;
    if (i0 + 8 <= K) {
        const float4 a = *reinterpret_cast<const float4*>(src + i0);
        const float4 b = *reinterpret_cast<const float4*>(src + i0 + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    }
}

__global__ void __launch_bounds__(128) k_quantize_rows(const float* __restrict__ x, int ldx, int K, ActQ a, int want32,
                                                       int wantk) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.y, lane = threadIdx.x & 31;
    const int c = blockIdx.x * kQWarps + (threadIdx.x >> 5);
    if (c * 256 >= K) return;
    float v[8];
    load8(x + (size_t)t * ldx, c * 256, lane, K, v);
    quant_chunk(v, lane, K, t, c, a, want32, wantk);
}

// RMSNorm (src/ops.cpp:18-23: sum of squares in double; out = x*scale*w with
// scale = 1/sqrt(float(sum/n) + eps)) then quantisation. A CTA has the
// kNormWarps warps of the shared summation order (common.cuh) and quantises
// chunks 8*blockIdx.x + warp; every CTA of a row reduces the whole row in that
// order, so all of them, and the fused GEMV prologue, get the same scale.
__global__ void __launch_bounds__(32 * kNormWarps) k_rmsnorm_quant(const float* __restrict__ x, int ldx,
                                                                  const float* __restrict__ w, float eps, int K,
                                                                  float* __restrict__ xb, int ldxb, ActQ a, int want32,
                                                                  int wantk) {
    pdl_trigger();
    pdl_wait();
    __shared__ double part[kNormWarps];
    const int t = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n_chunks = (K + 255) / 256;
    const float* xr = x + (size_t)t * ldx;
    double s = 0.0;
    for (int c = warp; c < n_chunks; c += kNormWarps) {
        float v[8];
        load8(xr, c * 256, lane, K, v);
        s = __dadd_rn(s, sumsq8(v));
    }
    s = warp_sum_d(s);
    if (lane == 0) part[warp] = s;
    __syncthreads();
    const float sc = norm_total(part, K, eps);
    const int c = blockIdx.x * kNormWarps + warp;
    if (c >= n_chunks) return;
    float v[8];
    load8(xr, c * 256, lane, K, v);
    const int i0 = c * 256 + 8 * lane;
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = i0 + i < K ? __fmul_rn(__fmul_rn(v[i], sc), w[i0 + i]) : 0.0f;
    if (xb && i0 < K) {
        float* o = xb + (size_t)t * ldxb + i0;
#pragma unroll
        for (int i = 0; i < 8; ++i) if (i0 + i < K) o[i] = v[i];
    }
    if (want32 || wantk) quant_chunk(v, lane, K, t, c, a, want32, wantk);
}

// h = act(g) * u, then quantised: act = silu (src/ops.cpp:25-31,
// src/model.cpp:1501-1506), or with gelu set the tanh form of GELU
// (src/ops.cpp:32-38, gemma2), 0.5 v (1 + tanh(sqrt(2/pi) (v + 0.044715 v^3))).
__device__ __forceinline__ float gelu_tanh(float v) {
    const float c = 0.7978845608028654f;
    const float v3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v);
    return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(__fmul_rn(c, __fadd_rn(v, v3)))));
}

__global__ void __launch_bounds__(128) k_silu_mul_quant(const float* __restrict__ g, int ldg, const float* __restrict__ u,
                                                        int ldu, int F, float* __restrict__ h, int ldh, ActQ a,
                                                        int want32, int wantk, int gelu) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.y, lane = threadIdx.x & 31;
    const int c = blockIdx.x * kQWarps + (threadIdx.x >> 5);
    if (c * 256 >= F) return;
    float gv[8], uv[8], v[8];
    load8(g + (size_t)t * ldg, c * 256, lane, F, gv);
    load8(u + (size_t)t * ldu, c * 256, lane, F, uv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float sv = gelu ? gelu_tanh(gv[i]) : __fdiv_rn(gv[i], __fadd_rn(1.0f, expf(-gv[i])));
        v[i] = __fmul_rn(sv, uv[i]);
    }
    const int i0 = c * 256 + 8 * lane;
    if (h && i0 < F) {
        float* o = h + (size_t)t * ldh + i0;
#pragma unroll
        for (int i = 0; i < 8; ++i) if (i0 + i < F) o[i] = v[i];
    }
    if (want32 || wantk) quant_chunk(v, lane, F, t, c, a, want32, wantk);
}

// Gemma-2's post norms (src/model.cpp post_attention_norm / post_ffw_norm):
// x[t] += rmsnorm(y[t]) * w, the norm's squares summed in the order of every
// other RMSNorm here (sumsq8 per 256-value chunk, chunks by warp, warps in
// order).
__global__ void __launch_bounds__(32 * kNormWarps) k_rmsnorm_add(float* __restrict__ x, int ldx,
                                                                const float* __restrict__ y, int ldy,
                                                                const float* __restrict__ w, float eps, int K) {
    pdl_trigger();
    pdl_wait();
    __shared__ double part[kNormWarps];
    const int t = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n_chunks = (K + 255) / 256;
    const float* yr = y + (size_t)t * ldy;
    double s = 0.0;
    for (int c = warp; c < n_chunks; c += kNormWarps) {
        float v[8];
        load8(yr, c * 256, lane, K, v);
        s = __dadd_rn(s, sumsq8(v));
    }
    s = warp_sum_d(s);
    if (lane == 0) part[warp] = s;
    __syncthreads();
    const float sc = norm_total(part, K, eps);
    const int c = blockIdx.x * kNormWarps + warp;
    if (c >= n_chunks) return;
    float v[8];
    load8(yr, c * 256, lane, K, v);
    const int i0 = c * 256 + 8 * lane;
    float* xr = x + (size_t)t * ldx;
#pragma unroll
    for (int i = 0; i < 8; ++i)
        if (i0 + i < K) xr[i0 + i] = __fadd_rn(xr[i0 + i], __fmul_rn(__fmul_rn(v[i], sc), w[i0 + i]));
}

// x[i] *= s (gemma2's embedding scale, src/model.cpp:1624-1627)
__global__ void k_scale(float* __restrict__ x, size_t n, float s) {
    pdl_trigger();
    pdl_wait();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        x[i] = __fmul_rn(x[i], s);
}

// y = 1 / (1 + exp(-x)), or 1 where x is null (the shared expert's gate,
// src/model.cpp:1588-1592)
__global__ void k_sigmoid(const float* __restrict__ x, float* __restrict__ y, int n) {
    pdl_trigger();
    pdl_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        y[i] = x ? __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x[i]))) : 1.0f;
}

// cap * tanh(x / cap) (gemma2's final logit soft cap, src/model.cpp:1802-1805)
__global__ void k_softcap(float* __restrict__ x, int n, int ldx, float cap) {
    pdl_trigger();
    pdl_wait();
    float* r = x + (size_t)blockIdx.y * ldx;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        r[i] = __fmul_rn(cap, tanhf(__fdiv_rn(r[i], cap)));
}

}  // namespace fb

using namespace fb;

static dim3 qgrid(int K, int T) {
    const int chunks = (K + 255) / 256;
    return dim3((chunks + kQWarps - 1) / kQWarps, T);
}

extern "C" int fbk_quantize_rows(const float* x, int ldx, int T, int K, const ActQ* a, int want32, int wantk,
                                 cudaStream_t st) {
    if (T <= 0) return 0;
    if (K % 8 || ldx % 4) return (int)cudaErrorInvalidValue;
    return (int)fbk_launch(k_quantize_rows, qgrid(K, T), dim3(32 * kQWarps), 0, st, x, ldx, K, *a, want32, wantk);
}

extern "C" int fbk_rmsnorm_quant(const float* x, int ldx, const float* w, float eps, int T, int K, float* xb,
                                 int ldxb, const ActQ* a, int want32, int wantk, cudaStream_t st) {
    if (T <= 0) return 0;
    if (K % 8 || ldx % 4) return (int)cudaErrorInvalidValue;
    const dim3 grid(((K + 255) / 256 + kNormWarps - 1) / kNormWarps, T);
    return (int)fbk_launch(k_rmsnorm_quant, grid, dim3(32 * kNormWarps), 0, st, x, ldx, w, eps, K, xb, ldxb, *a, want32,
                           wantk);
}

extern "C" int fbk_silu_mul_quant(const float* g, int ldg, const float* u, int ldu, int T, int F, float* h, int ldh,
                                  const ActQ* a, int want32, int wantk, cudaStream_t st) {
    return fbk_act_mul_quant(g, ldg, u, ldu, T, F, h, ldh, a, want32, wantk, 0, st);
}

extern "C" int fbk_act_mul_quant(const float* g, int ldg, const float* u, int ldu, int T, int F, float* h, int ldh,
                                 const ActQ* a, int want32, int wantk, int gelu, cudaStream_t st) {
    if (T <= 0) return 0;
    if (F % 8 || ldg % 4 || ldu % 4) return (int)cudaErrorInvalidValue;
    return (int)fbk_launch(k_silu_mul_quant, qgrid(F, T), dim3(32 * kQWarps), 0, st, g, ldg, u, ldu, F, h, ldh, *a, want32,
                           wantk, gelu);
}

extern "C" int fbk_rmsnorm_add(float* x, int ldx, const float* y, int ldy, const float* w, float eps, int T, int K,
                               cudaStream_t st) {
    if (T <= 0) return 0;
    if (K % 8 || ldy % 4) return (int)cudaErrorInvalidValue;
    const dim3 grid(((K + 255) / 256 + kNormWarps - 1) / kNormWarps, T);
    return (int)fbk_launch(k_rmsnorm_add, grid, dim3(32 * kNormWarps), 0, st, x, ldx, y, ldy, w, eps, K);
}

extern "C" int fbk_scale(float* x, size_t n, float s, cudaStream_t st) {
    if (n == 0) return 0;
    const int ctas = (int)std::min<size_t>(1184, (n + 255) / 256);
    return (int)fbk_launch(k_scale, dim3(ctas), dim3(256), 0, st, x, n, s);
}

extern "C" int fbk_sigmoid(const float* x, float* y, int n, cudaStream_t st) {
    if (n <= 0) return 0;
    return (int)fbk_launch(k_sigmoid, dim3((n + 255) / 256), dim3(256), 0, st, x, y, n);
}

extern "C" int fbk_softcap(float* x, int n, int rows, int ldx, float cap, cudaStream_t st) {
    if (rows <= 0 || n <= 0) return 0;
    if (!(cap > 0.0f)) return (int)cudaErrorInvalidValue;
    return (int)fbk_launch(k_softcap, dim3((n + 1023) / 1024, rows), dim3(256), 0, st, x, n, ldx, cap);
}
