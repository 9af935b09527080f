// common.cuh — shared device helpers for the FISH B200 kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fb {

// ggml type ids (GGUF specification; reference include/fish/gguf.h:25-33).
enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_BF16 = 30 };

constexpr int kWarp = 32;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// RMSNorm sum of squares (src/ops.cpp:18-23 sums x*x in double). Every kernel
// that normalises a row sums in this one order, so fused and unfused paths
// give the same scale bit for bit: 8 warps, warp w takes the 256-value chunks
// w, w+8, ... in ascending order, lane l values 8l .. 8l+7 of a chunk
// (sumsq8, left to right); each lane adds its chunk sums in order, the warp
// reduces with warp_sum_d, and the 8 warp sums are added in warp order
// (norm_total). Products of two floats are exact in double, so no
// contraction choice can change a partial.
constexpr int kNormWarps = 8;
__device__ __forceinline__ double sumsq8(const float (&v)[8]) {
    double s = __dmul_rn((double)v[0], (double)v[0]);
#pragma unroll
    for (int i = 1; i < 8; ++i) s = __dadd_rn(s, __dmul_rn((double)v[i], (double)v[i]));
    return s;
}
__device__ __forceinline__ float norm_total(const double* part, int K, float eps) {
    double tot = 0.0;
#pragma unroll
    for (int i = 0; i < kNormWarps; ++i) tot = __dadd_rn(tot, part[i]);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)__ddiv_rn(tot, (double)K), eps)));
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// Argmax key of logit v at index i: ordered float bits above, inverted index
// below, so an unsigned max picks the largest value and, among equal values,
// the first index — the reference's strict '>' scan from -inf
// (src/model.cpp:1939-1946). NaN and -inf never win (key 0 decodes to 0).
__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
    if (!(v > -INFINITY)) return 0ull;
    uint32_t b = v == 0.0f ? 0u : __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)i);
}
__device__ __forceinline__ int argmax_index(unsigned long long key) {
    return key ? (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull)) : 0;
}

// Programmatic dependent launch (no-ops for launches without the attribute):
// wait until the previous kernel on the stream has completed and its writes
// are visible / let the next kernel be scheduled.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Streaming 128-bit load that bypasses L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
__device__ __forceinline__ uint2 ldg_stream2(const void* p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}

// Device activation batch, structure-of-arrays form of the reference's
// Q8Act / Q8ActK records (include/fish/quant.h:58-70): same values, aligned
// planes so they can be read with 128-bit loads.
//   q32[t][K], d32[t][K/32], s32[t][K/32]        (32-value blocks)
//   qk [t][K], dk [t][K/256], bsk[t][K/32]       (256-value blocks, bsums)
struct ActQ {
    int8_t* q32;
    float* d32;
    int32_t* s32;
    int8_t* qk;
    float* dk;
    int16_t* bsk;
    int K;       // row length
    int ld;      // row stride of q planes (>= K, multiple of 16)
};

}  // namespace fb
