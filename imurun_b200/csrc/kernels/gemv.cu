// gemv.cu — decode/small-batch quantised matrix-vector products.
//
// y[t][r] = W_r . x_t for T <= 8 tokens, W in Q8_0 / Q4_K / Q6_K (int8 path,
// src/quant_x86.cpp:299-309, 346-382, 431-495) or F32 / F16 (f32 path,
// src/ops.cpp:219-250).
//
// The work unit is 32 weight values of one row (unit_math.cuh); the lanes that
// hold the units of one super-block add their integer partials with shuffles,
// so every super-block's integer sums
//     Q4_K  sumi = sum_g sc_g sum_l q x,   mins = sum_g m_g bsums_g
//     Q6_K  sumi = sum_j sc_j sum (q6-32) x
//     Q8_0  s    = sum w x
// are formed exactly as the reference forms them, then combined in float once
// per block. Decode is HBM-bound; two kernels stream the weights:
//   k_gemv_stream  quantised rows, T <= 4: a producer warp streams 8-row x
//                  2048-value pieces into a ring of shared-memory stages with
//                  cp.async.bulk (TMA) and mbarriers; 8 consumer warps compute
//                  from shared memory with the activations held in registers.
//   k_gemv         F32/F16 rows (router, small tensors) and T = 5..8, with
//                  direct 128-bit loads.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"
#include "layout.cuh"
#include "unit_math.cuh"

namespace fb {

size_t dev_row_bytes(int type, int n) {
    size_t b = 0;
    switch (type) {
        case T_Q4_K: case T_Q6_K: case T_Q8_0: return row_bytes_dev(type, n);
        case T_F32: b = (size_t)n * 4; break;
        case T_F16: b = (size_t)n * 2; break;
        default: return 0;
    }
    return (b + 15) / 16 * 16;
}

void repack_row(int type, const uint8_t* src, uint8_t* dst, int n) {
    const size_t db = dev_row_bytes(type, n);
    for (size_t i = 0; i < db; ++i) dst[i] = 0;
    switch (type) {
        case T_Q4_K:
            for (size_t i = 0; i < (size_t)(n / 256) * 144; ++i) dst[i] = src[i];
            break;
        case T_Q6_K: {
            const int nb = n / 256;
            for (int b = 0; b < nb; ++b) {
                const size_t qo = block_offset(T_Q6_K, b), dof = dscale_offset(T_Q6_K, nb, b);
                for (int i = 0; i < 208; ++i) dst[qo + i] = src[(size_t)b * 210 + i];
                dst[dof] = src[(size_t)b * 210 + 208];
                dst[dof + 1] = src[(size_t)b * 210 + 209];
            }
            break;
        }
        case T_Q8_0: {
            const int nb = n / 32;
            for (int b = 0; b < nb; ++b) {
                const size_t qo = block_offset(T_Q8_0, b), dof = dscale_offset(T_Q8_0, nb, b);
                for (int i = 0; i < 32; ++i) dst[qo + i] = src[(size_t)b * 34 + 2 + i];
                dst[dof] = src[(size_t)b * 34];
                dst[dof + 1] = src[(size_t)b * 34 + 1];
            }
            break;
        }
        case T_F32:
            for (size_t i = 0; i < (size_t)n * 4; ++i) dst[i] = src[i];
            break;
        case T_F16:
            for (size_t i = 0; i < (size_t)n * 2; ++i) dst[i] = src[i];
            break;
        default: break;
    }
}

// ============================================================ activation access
// Activations are read through L1 (every row of a launch reads the same x).

__device__ __forceinline__ void x_q4k(const ActQ& a, int t, int b, int p, uint4& x0, uint4& x1, uint4& x2, uint4& x3,
                                      uint32_t& bs) {
    const int8_t* xq = a.qk + (size_t)t * a.ld + (size_t)b * 256 + 64 * p;
    x0 = __ldg(reinterpret_cast<const uint4*>(xq));
    x1 = __ldg(reinterpret_cast<const uint4*>(xq + 16));
    x2 = __ldg(reinterpret_cast<const uint4*>(xq + 32));
    x3 = __ldg(reinterpret_cast<const uint4*>(xq + 48));
    bs = __ldg(reinterpret_cast<const uint32_t*>(a.bsk + (size_t)t * (a.K / 32) + (size_t)b * 8 + 2 * p));
}

__device__ __forceinline__ void x_q6k(const ActQ& a, int t, int b, int j, uint2 (&x)[4]) {
    const int8_t* xq = a.qk + (size_t)t * a.ld + (size_t)b * 256 + 128 * (j >> 2) + 8 * (j & 3);
#pragma unroll
    for (int q = 0; q < 4; ++q) x[q] = __ldg(reinterpret_cast<const uint2*>(xq + 32 * q));
}

// ============================================================ direct kernel rows

template <int NT, bool SUMS>
__device__ __forceinline__ void row_q4k(const uint8_t* __restrict__ row, int nb, const ActQ& a, int lane,
                                        float (&acc)[NT], int32_t* sumi_out, int32_t* mins_out) {
    const int nunits = nb * 4;
    for (int u = lane; u - lane < nunits; u += 32) {
        const bool ok = u < nunits;
        const int b = u >> 2, p = u & 3;
        Q4kUnit un;
        uint4 h = make_uint4(0, 0, 0, 0);
        if (ok) {
            const uint8_t* blk = row + (size_t)b * 144;
            h = ldg_stream(blk);
            un.load(h, ldg_stream(blk + 16 + 32 * p), ldg_stream(blk + 32 + 32 * p), p);
        }
        const float dw = h2f((uint16_t)(h.x & 0xFFFFu)), dmw = h2f((uint16_t)(h.x >> 16));
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            int si = 0, mi = 0;
            if (ok) {
                uint4 x0, x1, x2, x3;
                uint32_t bs;
                x_q4k(a, t, b, p, x0, x1, x2, x3, bs);
                un.dot(x0, x1, x2, x3, bs, si, mi);
            }
            si += __shfl_xor_sync(0xffffffffu, si, 1);
            si += __shfl_xor_sync(0xffffffffu, si, 2);
            mi += __shfl_xor_sync(0xffffffffu, mi, 1);
            mi += __shfl_xor_sync(0xffffffffu, mi, 2);
            if (ok && p == 0) {
                if (SUMS) { sumi_out[b] = si; mins_out[b] = mi; }
                else {
                    const float dx = __ldg(a.dk + (size_t)t * (a.K / 256) + b);
                    acc[t] += __fmul_rn(dw, dx) * (float)si - __fmul_rn(dmw, dx) * (float)mi;
                }
            }
        }
    }
}

template <int NT, bool SUMS>
__device__ __forceinline__ void row_q6k(const uint8_t* __restrict__ row, int nb, const ActQ& a, int lane,
                                        float (&acc)[NT], int32_t* sumi_out) {
    const int nunits = nb * 8;
    for (int u = lane; u - lane < nunits; u += 32) {
        const bool ok = u < nunits;
        const int b = u >> 3, j = u & 7, hh = j >> 2, jj = j & 3;
        Q6kUnit un;
        float dw = 0.0f;
        if (ok) {
            const uint8_t* blk = row + block_offset(T_Q6_K, b);
            un.load(ldg_stream2(blk + 64 * hh + 8 * jj), ldg_stream2(blk + 64 * hh + 32 + 8 * jj),
                    ldg_stream2(blk + 128 + 32 * hh + 8 * jj), ldg_stream2(blk + 192 + 8 * hh), jj);
            dw = h2f(*reinterpret_cast<const uint16_t*>(row + dscale_offset(T_Q6_K, nb, b)));
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            int si = 0;
            if (ok) {
                uint2 x[4];
                x_q6k(a, t, b, j, x);
                const int xs[4] = {sum8(x[0]), sum8(x[1]), sum8(x[2]), sum8(x[3])};
                si = un.dot(x, xs);
            }
            si += __shfl_xor_sync(0xffffffffu, si, 1);
            si += __shfl_xor_sync(0xffffffffu, si, 2);
            si += __shfl_xor_sync(0xffffffffu, si, 4);
            if (ok && j == 0) {
                if (SUMS) sumi_out[b] = si;
                else acc[t] += __fmul_rn(dw, __ldg(a.dk + (size_t)t * (a.K / 256) + b)) * (float)si;
            }
        }
    }
}

template <int NT, bool SUMS>
__device__ __forceinline__ void row_q80(const uint8_t* __restrict__ row, int nb, const ActQ& a, int lane,
                                        float (&acc)[NT], int32_t* sumi_out) {
    for (int b = lane; b < nb; b += 32) {
        const uint8_t* q = row + block_offset(T_Q8_0, b);
        const uint4 w0 = ldg_stream(q), w1 = ldg_stream(q + 16);
        const float dw = h2f(*reinterpret_cast<const uint16_t*>(row + dscale_offset(T_Q8_0, nb, b)));
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const int8_t* xq = a.q32 + (size_t)t * a.ld + (size_t)b * 32;
            const int s = q80_dot(w0, w1, __ldg(reinterpret_cast<const uint4*>(xq)),
                                  __ldg(reinterpret_cast<const uint4*>(xq + 16)));
            if (SUMS) sumi_out[b] = s;
            else acc[t] += __fmul_rn(dw, __ldg(a.d32 + (size_t)t * (a.K / 32) + b)) * (float)s;
        }
    }
}

template <int NT>
__device__ __forceinline__ void row_float(int type, const uint8_t* __restrict__ row, int K, const float* xf, int ldxf,
                                          int lane, float (&acc)[NT]) {
    for (int k = lane; k < K; k += 32) {
        const float w = type == T_F32 ? reinterpret_cast<const float*>(row)[k]
                                      : h2f(reinterpret_cast<const uint16_t*>(row)[k]);
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] += w * xf[(size_t)t * ldxf + k];
    }
}

__device__ __forceinline__ void store_out(const GemvSeg& g, int rr, int t, float v) {
    if (g.bias) v += g.bias[rr];
    float* yp = g.y + (size_t)t * g.ldy + rr;
    if (g.epi == EPI_ADD) *yp += v;
    else *yp = v;
}

template <int NT>
__global__ void __launch_bounds__(256) k_gemv(GemvArgs args) {
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    int total = 0;
#pragma unroll
    for (int s = 0; s < kMaxSeg; ++s) if (s < args.nseg) total += args.seg[s].rows;
    for (int r = gw; r < total; r += nw) {
        int s = 0, rr = r;
        while (s < args.nseg - 1 && rr >= args.seg[s].rows) { rr -= args.seg[s].rows; ++s; }
        const GemvSeg& g = args.seg[s];
        const uint8_t* base = g.expert ? g.w + (size_t)__ldg(g.expert) * g.expert_bytes : g.w;
        const uint8_t* row = base + (size_t)rr * g.row_stride;
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
        switch (g.type) {
            case T_Q4_K: row_q4k<NT, false>(row, args.K / 256, args.act, lane, acc, nullptr, nullptr); break;
            case T_Q6_K: row_q6k<NT, false>(row, args.K / 256, args.act, lane, acc, nullptr); break;
            case T_Q8_0: row_q80<NT, false>(row, args.K / 32, args.act, lane, acc, nullptr); break;
            default: row_float<NT>(g.type, row, args.K, args.xf, args.ldxf, lane, acc); break;
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const float v = warp_sum(acc[t]);
            if (lane == 0 && t < args.T) store_out(g, rr, t, v);
        }
    }
}

__global__ void k_block_sums(int type, const uint8_t* __restrict__ w, size_t stride, int rows, int K, ActQ a,
                             int32_t* sumi, int32_t* mins) {
    const int lane = threadIdx.x & 31;
    const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (r >= rows) return;
    float acc[1] = {0.0f};
    const int nb = type == T_Q8_0 ? K / 32 : K / 256;
    const uint8_t* row = w + (size_t)r * stride;
    switch (type) {
        case T_Q4_K: row_q4k<1, true>(row, nb, a, lane, acc, sumi + (size_t)r * nb, mins + (size_t)r * nb); break;
        case T_Q6_K: row_q6k<1, true>(row, nb, a, lane, acc, sumi + (size_t)r * nb); break;
        case T_Q8_0: row_q80<1, true>(row, nb, a, lane, acc, sumi + (size_t)r * nb); break;
        default: break;
    }
}

// ============================================================ TMA-streamed kernel

constexpr int kBulkConsumers = 8;                 // consumer warps; tile = 8 rows
constexpr int kBulkRows = kBulkConsumers;
constexpr int kMaxStages = 32;
constexpr int kBulkHeader = 2 * kMaxStages * 8;   // mbarriers
constexpr long long kSpinLimit = 1LL << 26;       // bounded mbarrier waits

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: false after kSpinLimit polls (the caller records an error).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    for (long long i = 0; i < kSpinLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Activation chunk of one lane for one 2048-value group, held in registers
// while every row of the CTA's tiles passes through (the same x serves all
// rows): Q4_K unit (block lane/4, pair lane%4): 64 int8 + bsums + d;
// Q6_K units u = lane, lane+32: 2 x 32 int8 + 2 d; Q8_0 blocks lane, lane+32:
// 2 x 32 int8 + 2 d.
struct XRegs {
    uint4 q[4];
    uint32_t a0, a1;   // Q4_K: bsums pair, d bits | Q6_K/Q8_0: d bits of the two units
    int xs[8];         // Q6_K: sums of the 8-value pieces (unit k, quad q at 4k + q)
};

__device__ __forceinline__ void load_x(int type, const ActQ& a, int t, int gi, int lane, int nb, XRegs& x) {
    const int8_t* base = (type == T_Q8_0 ? a.q32 : a.qk) + (size_t)t * a.ld;
    x.q[0] = x.q[1] = x.q[2] = x.q[3] = make_uint4(0, 0, 0, 0);
    x.a0 = x.a1 = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) x.xs[i] = 0;
    if (type == T_Q4_K) {
        const int b = gi * 8 + (lane >> 2), p = lane & 3;
        if (b < nb) {
            const int8_t* xq = base + (size_t)b * 256 + 64 * p;
#pragma unroll
            for (int i = 0; i < 4; ++i) x.q[i] = __ldg(reinterpret_cast<const uint4*>(xq + 16 * i));
            x.a0 = __ldg(reinterpret_cast<const uint32_t*>(a.bsk + (size_t)t * (a.K / 32) + (size_t)b * 8 + 2 * p));
            x.a1 = __float_as_uint(__ldg(a.dk + (size_t)t * (a.K / 256) + b));
        }
    } else if (type == T_Q6_K) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int u = lane + 32 * k, b = gi * 8 + (u >> 3), j = u & 7;
            if (b < nb) {
                const int8_t* xq = base + (size_t)b * 256 + 128 * (j >> 2) + 8 * (j & 3);
                const uint2 v0 = __ldg(reinterpret_cast<const uint2*>(xq));
                const uint2 v1 = __ldg(reinterpret_cast<const uint2*>(xq + 32));
                const uint2 v2 = __ldg(reinterpret_cast<const uint2*>(xq + 64));
                const uint2 v3 = __ldg(reinterpret_cast<const uint2*>(xq + 96));
                x.q[2 * k] = make_uint4(v0.x, v0.y, v1.x, v1.y);
                x.q[2 * k + 1] = make_uint4(v2.x, v2.y, v3.x, v3.y);
                x.xs[4 * k + 0] = sum8(v0);
                x.xs[4 * k + 1] = sum8(v1);
                x.xs[4 * k + 2] = sum8(v2);
                x.xs[4 * k + 3] = sum8(v3);
                const uint32_t d = __float_as_uint(__ldg(a.dk + (size_t)t * (a.K / 256) + b));
                if (k == 0) x.a0 = d; else x.a1 = d;
            }
        }
    } else {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int b = gi * 64 + lane + 32 * k;
            if (b < nb) {
                const int8_t* xq = base + (size_t)b * 32;
                x.q[2 * k] = __ldg(reinterpret_cast<const uint4*>(xq));
                x.q[2 * k + 1] = __ldg(reinterpret_cast<const uint4*>(xq + 16));
                const uint32_t d = __float_as_uint(__ldg(a.d32 + (size_t)t * (a.K / 32) + b));
                if (k == 0) x.a0 = d; else x.a1 = d;
            }
        }
    }
}

// Float contribution of one lane for one (row, group) piece in shared memory.
// Integer sums per super-block are reduced across the lanes that share it
// (Q4_K: 4 lanes, Q6_K: 8 lanes) before the one float combine per block.
template <int NT>
__device__ __forceinline__ void piece_dot(int type, const uint8_t* pc, int gbk, int lane, const XRegs (&x)[NT],
                                          float (&c)[NT]) {
#pragma unroll
    for (int t = 0; t < NT; ++t) c[t] = 0.0f;
    if (type == T_Q4_K) {
        const int bl = lane >> 2, p = lane & 3;
        const bool ok = bl < gbk;
        Q4kUnit un;
        uint4 h = make_uint4(0, 0, 0, 0);
        if (ok) {
            const uint8_t* blk = pc + bl * 144;
            h = *reinterpret_cast<const uint4*>(blk);
            un.load(h, *reinterpret_cast<const uint4*>(blk + 16 + 32 * p), *reinterpret_cast<const uint4*>(blk + 32 + 32 * p), p);
        }
        const float dw = h2f((uint16_t)(h.x & 0xFFFFu)), dmw = h2f((uint16_t)(h.x >> 16));
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            int si = 0, mi = 0;
            if (ok) un.dot(x[t].q[0], x[t].q[1], x[t].q[2], x[t].q[3], x[t].a0, si, mi);
            si += __shfl_xor_sync(0xffffffffu, si, 1);
            si += __shfl_xor_sync(0xffffffffu, si, 2);
            mi += __shfl_xor_sync(0xffffffffu, mi, 1);
            mi += __shfl_xor_sync(0xffffffffu, mi, 2);
            if (ok && p == 0) {
                const float dx = __uint_as_float(x[t].a1);
                c[t] = __fmul_rn(dw, dx) * (float)si - __fmul_rn(dmw, dx) * (float)mi;
            }
        }
    } else if (type == T_Q6_K) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int u = lane + 32 * k, bl = u >> 3, j = u & 7, hh = j >> 2, jj = j & 3;
            const bool ok = bl < gbk;
            Q6kUnit un;
            float dw = 0.0f;
            if (ok) {
                const uint8_t* blk = pc + bl * 208;
                un.load(*reinterpret_cast<const uint2*>(blk + 64 * hh + 8 * jj),
                        *reinterpret_cast<const uint2*>(blk + 64 * hh + 32 + 8 * jj),
                        *reinterpret_cast<const uint2*>(blk + 128 + 32 * hh + 8 * jj),
                        *reinterpret_cast<const uint2*>(blk + 192 + 8 * hh), jj);
                dw = h2f(*reinterpret_cast<const uint16_t*>(pc + gbk * 208 + 2 * bl));
            }
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                int si = 0;
                if (ok) {
                    const uint4 qa = x[t].q[2 * k], qb = x[t].q[2 * k + 1];
                    const uint2 xv[4] = {make_uint2(qa.x, qa.y), make_uint2(qa.z, qa.w), make_uint2(qb.x, qb.y),
                                         make_uint2(qb.z, qb.w)};
                    const int xs[4] = {x[t].xs[4 * k], x[t].xs[4 * k + 1], x[t].xs[4 * k + 2], x[t].xs[4 * k + 3]};
                    si = un.dot(xv, xs);
                }
                si += __shfl_xor_sync(0xffffffffu, si, 1);
                si += __shfl_xor_sync(0xffffffffu, si, 2);
                si += __shfl_xor_sync(0xffffffffu, si, 4);
                if (ok && j == 0) c[t] += __fmul_rn(dw, __uint_as_float(k ? x[t].a1 : x[t].a0)) * (float)si;
            }
        }
    } else {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int bl = lane + 32 * k;
            if (bl < gbk) {
                const uint4 w0 = *reinterpret_cast<const uint4*>(pc + bl * 32);
                const uint4 w1 = *reinterpret_cast<const uint4*>(pc + bl * 32 + 16);
                const float dw = h2f(*reinterpret_cast<const uint16_t*>(pc + gbk * 32 + 2 * bl));
#pragma unroll
                for (int t = 0; t < NT; ++t)
                    c[t] += __fmul_rn(dw, __uint_as_float(k ? x[t].a1 : x[t].a0)) *
                            (float)q80_dot(w0, w1, x[t].q[2 * k], x[t].q[2 * k + 1]);
            }
        }
    }
}

struct BulkJobs {
    // tiles of 8 rows; segment s owns tiles [tile0[s], tile0[s+1])
    int tile0[kMaxSeg + 1];
    int n_groups;       // 2048-value groups per row
    int stages;         // ring slots (<= kMaxStages)
    int piece;          // bytes per row piece in a slot (largest group of the launch's types)
    int tiles_per_cta;  // <= kMaxTiles
    int* err;           // device error flag (nullable)
};

constexpr int kMaxTiles = 16;   // tiles one CTA accumulates in shared memory (x NT <= 16)

__device__ __forceinline__ int seg_of(const GemvArgs& args, const BulkJobs& jobs, int tile) {
    int s = 0;
    while (s < args.nseg - 1 && tile >= jobs.tile0[s + 1]) ++s;
    return s;
}

// CTA c owns tiles [c*tpc, (c+1)*tpc) and walks them group-major: for every
// 2048-value group gi, all its tiles' 8-row pieces stream through the ring
// (stage = one tile x one group), so each lane's activation chunk for gi is
// loaded once into registers. Per-lane float partials accumulate in shared
// memory across groups; a warp reduction per row happens once at the end.
template <int NT>
__global__ void __launch_bounds__(32 * (kBulkConsumers + 1)) k_gemv_stream(GemvArgs args, BulkJobs jobs) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ volatile int s_abort;
    const int S = jobs.stages, piece = jobs.piece, stage_bytes = jobs.piece * kBulkRows;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    float* accs = reinterpret_cast<float*>(smem + kBulkHeader);   // [consumer warp][tile][lane][NT]
    uint8_t* stage_mem = smem + kBulkHeader + (size_t)kBulkConsumers * kMaxTiles * 32 * sizeof(float);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tiles = jobs.tile0[args.nseg];
    const int t_begin = blockIdx.x * jobs.tiles_per_cta;
    const int t_end = min(n_tiles, t_begin + jobs.tiles_per_cta);
    const int G = jobs.n_groups;
    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kBulkConsumers);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == kBulkConsumers) {
        if (lane == 0) {
            int it = 0, slot = 0, round = 0;
            bool failed = false;
            for (int gi = 0; gi < G && !failed; ++gi) {
                for (int tile = t_begin; tile < t_end; ++tile) {
                    const int s = seg_of(args, jobs, tile);
                    const GemvSeg& g = args.seg[s];
                    const int r0 = (tile - jobs.tile0[s]) * kBulkRows;
                    const int nr = min(kBulkRows, g.rows - r0);
                    const uint8_t* base = g.expert ? g.w + (size_t)__ldg(g.expert) * g.expert_bytes : g.w;
                    const int nb = row_blocks(g.type, args.K);
                    if (s_abort || (round > 0 && !mbar_wait(&empty[slot], (round - 1) & 1))) {
                        if (jobs.err) atomicExch(jobs.err, 1);
                        s_abort = 1;
                        failed = true;
                        break;
                    }
                    const uint32_t gb = (uint32_t)group_bytes(g.type, group_blocks(g.type, nb, gi));
                    mbar_expect_tx(&full[slot], gb * nr);
                    uint8_t* dst = stage_mem + (size_t)slot * stage_bytes;
                    const uint8_t* src = base + (size_t)r0 * g.row_stride + group_offset(g.type, gi);
                    for (int r = 0; r < nr; ++r) bulk_g2s(dst + (size_t)r * piece, src + (size_t)r * g.row_stride, gb, &full[slot]);
                    ++it;
                    if (++slot == S) { slot = 0; ++round; }
                }
            }
            if (failed)
                for (int k = max(0, it - S); k < it; ++k) mbar_wait(&full[k % S], (k / S) & 1);
        }
        return;
    }

    float* myacc = accs + (size_t)warp * kMaxTiles * 32;
    for (int i = lane; i < kMaxTiles * 32; i += 32) myacc[i] = 0.0f;
    int slot = 0, round = 0;
    int cur_type = -1, cur_gi = -1;
    XRegs x[NT];
    for (int gi = 0; gi < G; ++gi) {
        for (int tile = t_begin; tile < t_end; ++tile) {
            const int s = seg_of(args, jobs, tile);
            const GemvSeg& g = args.seg[s];
            const int nb = row_blocks(g.type, args.K);
            if (g.type != cur_type || gi != cur_gi) {
#pragma unroll
                for (int t = 0; t < NT; ++t) load_x(g.type, args.act, t, gi, lane, nb, x[t]);
                cur_type = g.type;
                cur_gi = gi;
            }
            if (s_abort || !mbar_wait(&full[slot], round & 1)) {
                if (jobs.err && lane == 0) atomicExch(jobs.err, 2);
                s_abort = 1;
                return;
            }
            const int row = (tile - jobs.tile0[s]) * kBulkRows + warp;
            if (row < g.rows) {
                float c[NT];
                piece_dot<NT>(g.type, stage_mem + (size_t)slot * stage_bytes + (size_t)warp * piece,
                              group_blocks(g.type, nb, gi), lane, x, c);
                // per-lane partial of (local tile, token): slot (tile - t_begin) * NT + t
                float* a = myacc + (size_t)(tile - t_begin) * NT * 32 + lane;
#pragma unroll
                for (int t = 0; t < NT; ++t) a[t * 32] += c[t];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == S) { slot = 0; ++round; }
        }
    }
    for (int tile = t_begin; tile < t_end; ++tile) {
        const int s = seg_of(args, jobs, tile);
        const GemvSeg& g = args.seg[s];
        const int row = (tile - jobs.tile0[s]) * kBulkRows + warp;
        const float* a = myacc + (size_t)(tile - t_begin) * NT * 32 + lane;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const float v = warp_sum(a[t * 32]);
            if (row < g.rows && lane == 0 && t < args.T) store_out(g, row, t, v);
        }
    }
}
}  // namespace fb

using namespace fb;

static int g_num_sms = 0;

static int num_sms() {
    if (!g_num_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    return g_num_sms;
}

static int* g_err = nullptr;

extern "C" int* fbk_gemv_error_flag() {
    if (!g_err) {
        if (cudaMalloc(&g_err, sizeof(int)) != cudaSuccess) return nullptr;
        cudaMemset(g_err, 0, sizeof(int));
    }
    return g_err;
}

static int env_or(const char* name, int def) {
    const char* v = getenv(name);
    return v && *v ? atoi(v) : def;
}

// Pipeline geometry: the shared-memory budget per CTA (default 100 KB, two
// CTAs per SM) sets the ring depth; each CTA owns up to 16/NT tiles, and the
// grid aims at >= 2 CTAs per SM. Tunable for sweeps via FISH_GEMV_SMEM_KB and
// FISH_GEMV_CTA_PER_SM.
template <int NT>
static int launch_stream(const GemvArgs* a, cudaStream_t st) {
    static const int budget = std::max(48, std::min(220, env_or("FISH_GEMV_SMEM_KB", 100))) * 1024;
    static const int want_cps = std::max(1, std::min(8, env_or("FISH_GEMV_CTA_PER_SM", 2)));
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(k_gemv_stream<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, budget) != cudaSuccess)
            return (int)cudaGetLastError();
        attr = true;
    }
    BulkJobs jobs{};
    int piece = 0;
    for (int s = 0; s < a->nseg; ++s)
        piece = std::max(piece, (int)group_bytes(a->seg[s].type, blocks_per_group(a->seg[s].type)));
    const int acc_bytes = kBulkConsumers * kMaxTiles * 32 * (int)sizeof(float);
    jobs.piece = piece;
    jobs.stages = std::min(kMaxStages, (budget - kBulkHeader - acc_bytes) / (piece * kBulkRows));
    if (jobs.stages < 2) return (int)cudaErrorInvalidValue;
    jobs.tile0[0] = 0;
    for (int s = 0; s < a->nseg; ++s) jobs.tile0[s + 1] = jobs.tile0[s] + (a->seg[s].rows + kBulkRows - 1) / kBulkRows;
    for (int s = a->nseg; s < kMaxSeg; ++s) jobs.tile0[s + 1] = jobs.tile0[s];
    jobs.n_groups = (a->K + kGroupValues - 1) / kGroupValues;
    jobs.err = fbk_gemv_error_flag();
    const int n_tiles = jobs.tile0[a->nseg];
    const int target = num_sms() * want_cps;
    jobs.tiles_per_cta = std::max(1, std::min(kMaxTiles / NT, (n_tiles + target - 1) / target));
    const int ctas = (n_tiles + jobs.tiles_per_cta - 1) / jobs.tiles_per_cta;
    const size_t smem = (size_t)kBulkHeader + acc_bytes + (size_t)jobs.stages * piece * kBulkRows;
    k_gemv_stream<NT><<<ctas, 32 * (kBulkConsumers + 1), smem, st>>>(*a, jobs);
    return (int)cudaGetLastError();
}

extern "C" int fbk_gemv(const GemvArgs* a, cudaStream_t st) {
    if (a->T <= 0 || a->nseg <= 0) return 0;
    if (a->T > 8) return (int)cudaErrorInvalidValue;
    bool quant = true;
    for (int s = 0; s < a->nseg; ++s) {
        const int t = a->seg[s].type;
        quant = quant && (t == T_Q4_K || t == T_Q6_K || t == T_Q8_0);
    }
    static const bool stream_off = getenv("FISH_GEMV_DIRECT") != nullptr;
    if (quant && !stream_off && a->T <= 4) {
        if (a->T == 1) return launch_stream<1>(a, st);
        if (a->T == 2) return launch_stream<2>(a, st);
        return launch_stream<4>(a, st);
    }
    int total = 0;
    for (int s = 0; s < a->nseg; ++s) total += a->seg[s].rows;
    int ctas = (total + 7) / 8;
    const int cap = num_sms() * 8;
    if (ctas > cap) ctas = cap;
    if (ctas < 1) ctas = 1;
    if (a->T == 1) k_gemv<1><<<ctas, 256, 0, st>>>(*a);
    else if (a->T == 2) k_gemv<2><<<ctas, 256, 0, st>>>(*a);
    else if (a->T <= 4) k_gemv<4><<<ctas, 256, 0, st>>>(*a);
    else k_gemv<8><<<ctas, 256, 0, st>>>(*a);
    return (int)cudaGetLastError();
}

extern "C" int fbk_block_sums(int type, const uint8_t* w, size_t stride, int rows, int K, const ActQ* a,
                              int32_t* sumi, int32_t* mins, cudaStream_t st) {
    const int ctas = (rows + 7) / 8;
    k_block_sums<<<ctas, 256, 0, st>>>(type, w, stride, rows, K, *a, sumi, mins);
    return (int)cudaGetLastError();
}
