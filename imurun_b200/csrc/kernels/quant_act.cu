// quant_act.cu — activation quantisation and the kernels that produce it.
//
// The int8 activation records must be byte-identical to the reference's
// (src/quant.cpp:400-434, src/quant_x86.cpp:499-570): per block
//   amax = max |x|, d = amax / 127 (IEEE division), id = d > 0 ? 1/d : 0,
//   q = clamp(round_half_even(x * id), -127, 127), sums of q.
// Every float step uses an explicitly rounded intrinsic so no contraction or
// approximate reciprocal can change a byte.
#include "common.cuh"
#include "kernels.h"

namespace fb {

// One warp quantises 256 consecutive values v[0..255] (lane holds 8, values
// 8*lane .. 8*lane+7) into both layouts.
__device__ __forceinline__ void warp_quantize256(const float (&v)[8], int lane, int want32, int wantk,
                                                 int8_t* q32, float* d32, int32_t* s32,
                                                 int8_t* qk, float* dk, int16_t* bsk) {
    float a = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) a = fmaxf(a, fabsf(v[i]));
    if (wantk) {
        const float amax = warp_max(a);
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        int qv[8];
        int s = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            int r = __float2int_rn(__fmul_rn(v[i], id));
            r = max(-127, min(127, r));
            qv[i] = r;
            s += r;
        }
        uint2 packed;
        packed.x = (qv[0] & 0xFF) | ((qv[1] & 0xFF) << 8) | ((qv[2] & 0xFF) << 16) | ((uint32_t)(qv[3] & 0xFF) << 24);
        packed.y = (qv[4] & 0xFF) | ((qv[5] & 0xFF) << 8) | ((qv[6] & 0xFF) << 16) | ((uint32_t)(qv[7] & 0xFF) << 24);
        *reinterpret_cast<uint2*>(qk + 8 * lane) = packed;
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if ((lane & 3) == 0) bsk[lane >> 2] = static_cast<int16_t>(s);
        if (lane == 0) *dk = d;
    }
    if (want32) {
        // 32-value blocks: lanes 4g .. 4g+3 hold block g.
        float am = a;
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
        const float d = __fdiv_rn(am, 127.0f);
        const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        int qv[8];
        int s = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            int r = __float2int_rn(__fmul_rn(v[i], id));
            r = max(-127, min(127, r));
            qv[i] = r;
            s += r;
        }
        uint2 packed;
        packed.x = (qv[0] & 0xFF) | ((qv[1] & 0xFF) << 8) | ((qv[2] & 0xFF) << 16) | ((uint32_t)(qv[3] & 0xFF) << 24);
        packed.y = (qv[4] & 0xFF) | ((qv[5] & 0xFF) << 8) | ((qv[6] & 0xFF) << 16) | ((uint32_t)(qv[7] & 0xFF) << 24);
        *reinterpret_cast<uint2*>(q32 + 8 * lane) = packed;
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if ((lane & 3) == 0) {
            d32[lane >> 2] = d;
            if (s32) s32[lane >> 2] = s;
        }
    }
}

// Quantise a row held in `src` (global or shared) of length K (multiple of 32).
// A trailing partial 256-chunk (K % 256 != 0) only gets the 32-layout, which
// matches the reference: the 256 layout exists only when K % 256 == 0
// (src/ops.cpp:166-174).
__device__ void block_quantize_row(const float* src, int K, int t, const ActQ& a, int want32, int wantk) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int n256 = (K + 255) / 256;
    for (int c = warp; c < n256; c += nw) {
        const int base = c * 256;
        const bool full = base + 256 <= K;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int idx = base + 8 * lane + i;
            v[i] = idx < K ? src[idx] : 0.0f;
        }
        const int wk = wantk && full;
        if (full) {
            warp_quantize256(v, lane, want32, wk,
                             a.q32 ? a.q32 + (size_t)t * a.ld + base : nullptr,
                             a.d32 ? a.d32 + (size_t)t * (a.K / 32) + base / 32 : nullptr,
                             a.s32 ? a.s32 + (size_t)t * (a.K / 32) + base / 32 : nullptr,
                             wk ? a.qk + (size_t)t * a.ld + base : nullptr,
                             wk ? a.dk + (size_t)t * (a.K / 256) + c : nullptr,
                             wk ? a.bsk + (size_t)t * (a.K / 32) + base / 32 : nullptr);
        } else if (want32) {
            // partial chunk: K - base is a multiple of 32; lanes beyond it idle.
            float am = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(v[i]));
            am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
            am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
            const float d = __fdiv_rn(am, 127.0f);
            const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            int s = 0;
            int qv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                int r = __float2int_rn(__fmul_rn(v[i], id));
                r = max(-127, min(127, r));
                qv[i] = r;
                s += r;
            }
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            if (base + 8 * lane < K) {
                int8_t* q = a.q32 + (size_t)t * a.ld + base + 8 * lane;
#pragma unroll
                for (int i = 0; i < 8; ++i) q[i] = static_cast<int8_t>(qv[i]);
                if ((lane & 3) == 0) {
                    a.d32[(size_t)t * (a.K / 32) + base / 32 + (lane >> 2)] = d;
                    if (a.s32) a.s32[(size_t)t * (a.K / 32) + base / 32 + (lane >> 2)] = s;
                }
            }
        }
    }
}

__global__ void k_quantize_rows(const float* __restrict__ x, int ldx, int K, ActQ a, int want32, int wantk) {
    const int t = blockIdx.x;
    block_quantize_row(x + (size_t)t * ldx, K, t, a, want32, wantk);
}

// RMSNorm (src/ops.cpp:18-23: sum of squares in double; out = x*scale*w with
// scale = 1/sqrt(float(sum/n) + eps)) followed by quantisation of the result.
// One CTA per token row; the normalised row is staged in shared memory.
__global__ void k_rmsnorm_quant(const float* __restrict__ x, int ldx, const float* __restrict__ w, float eps,
                                int K, float* __restrict__ xb, int ldxb, ActQ a, int want32, int wantk) {
    extern __shared__ float srow[];
    __shared__ double part[32];
    __shared__ float s_scale;
    const int t = blockIdx.x;
    const float* xr = x + (size_t)t * ldx;
    double s = 0.0;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        const float v = xr[i];
        srow[i] = v;
        s += (double)v * (double)v;
    }
    s = warp_sum_d(s);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double tot = 0.0;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += part[i];
        const float ms = (float)(tot / K);
        s_scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
    }
    __syncthreads();
    const float sc = s_scale;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        const float v = __fmul_rn(__fmul_rn(srow[i], sc), w[i]);
        srow[i] = v;
        if (xb) xb[(size_t)t * ldxb + i] = v;
    }
    __syncthreads();
    if (want32 || wantk) block_quantize_row(srow, K, t, a, want32, wantk);
}

// h = silu(g) * u (src/ops.cpp:25-31, src/model.cpp:1501-1506), then quantised.
// g and u are [T][F] with row strides ldg / ldu.
__global__ void k_silu_mul_quant(const float* __restrict__ g, int ldg, const float* __restrict__ u, int ldu,
                                 int F, float* __restrict__ h, int ldh, ActQ a, int want32, int wantk) {
    extern __shared__ float srow[];
    const int t = blockIdx.x;
    for (int i = threadIdx.x; i < F; i += blockDim.x) {
        const float gv = g[(size_t)t * ldg + i];
        const float sv = __fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv)));
        const float v = __fmul_rn(sv, u[(size_t)t * ldu + i]);
        srow[i] = v;
        if (h) h[(size_t)t * ldh + i] = v;
    }
    __syncthreads();
    if (want32 || wantk) block_quantize_row(srow, F, t, a, want32, wantk);
}

}  // namespace fb

// ---------------------------------------------------------------- launchers

using namespace fb;

extern "C" int fbk_quantize_rows(const float* x, int ldx, int T, int K, const ActQ* a, int want32, int wantk,
                                 cudaStream_t st) {
    if (T <= 0) return 0;
    k_quantize_rows<<<T, 256, 0, st>>>(x, ldx, K, *a, want32, wantk);
    return (int)cudaGetLastError();
}

extern "C" int fbk_rmsnorm_quant(const float* x, int ldx, const float* w, float eps, int T, int K, float* xb,
                                 int ldxb, const ActQ* a, int want32, int wantk, cudaStream_t st) {
    if (T <= 0) return 0;
    const size_t smem = (size_t)K * sizeof(float);
    if (smem > 48 * 1024) {
        static bool attr_set = false;
        if (!attr_set) {
            cudaFuncSetAttribute(k_rmsnorm_quant, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
            attr_set = true;
        }
    }
    k_rmsnorm_quant<<<T, 256, smem, st>>>(x, ldx, w, eps, K, xb, ldxb, *a, want32, wantk);
    return (int)cudaGetLastError();
}

extern "C" int fbk_silu_mul_quant(const float* g, int ldg, const float* u, int ldu, int T, int F, float* h, int ldh,
                                  const ActQ* a, int want32, int wantk, cudaStream_t st) {
    if (T <= 0) return 0;
    const size_t smem = (size_t)F * sizeof(float);
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(k_silu_mul_quant, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr_set = true;
    }
    k_silu_mul_quant<<<T, 256, smem, st>>>(g, ldg, u, ldu, F, h, ldh, *a, want32, wantk);
    return (int)cudaGetLastError();
}
