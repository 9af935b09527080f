// gemv.cu — decode/small-batch quantised matrix-vector products.
//
// y[t][r] = W_r . x_t for T <= 8 tokens, W in Q8_0 / Q4_K / Q6_K (int8 path,
// src/quant_x86.cpp:299-309, 346-382, 431-495) or F32 / F16 (f32 path,
// src/ops.cpp:219-250).
//
// The work unit is 32 weight values of one row: a lane streams its unit's
// bytes with 128-bit (Q4_K, Q8_0) or 64-bit (Q6_K) loads, unpacks nibbles /
// 6-bit codes in registers and forms int32 dot products with dp4a. The lanes
// holding the units of one super-block then add their integer partials with
// shuffles, so every super-block's integer sums
//     Q4_K  sumi = sum_g sc_g sum_l q x,   mins = sum_g m_g bsums_g
//     Q6_K  sumi = sum_j sc_j sum (q6-32) x
//     Q8_0  s    = sum w x
// are formed exactly as the reference forms them before one float combine
// per block. The memory stream is the only bound: decode is HBM-bound.
#include "common.cuh"
#include "kernels.h"

namespace fb {

size_t dev_row_bytes(int type, int n) {
    size_t b = 0;
    switch (type) {
        case T_Q4_K: b = (size_t)(n / 256) * 144; break;
        case T_Q6_K: b = (size_t)(n / 256) * 208 + (size_t)(n / 256) * 2; break;
        case T_Q8_0: b = (size_t)(n / 32) * 32 + (size_t)(n / 32) * 2; break;
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
                for (int i = 0; i < 208; ++i) dst[(size_t)b * 208 + i] = src[(size_t)b * 210 + i];
                dst[(size_t)nb * 208 + 2 * b] = src[(size_t)b * 210 + 208];
                dst[(size_t)nb * 208 + 2 * b + 1] = src[(size_t)b * 210 + 209];
            }
            break;
        }
        case T_Q8_0: {
            const int nb = n / 32;
            for (int b = 0; b < nb; ++b) {
                for (int i = 0; i < 32; ++i) dst[(size_t)b * 32 + i] = src[(size_t)b * 34 + 2 + i];
                dst[(size_t)nb * 32 + 2 * b] = src[(size_t)b * 34];
                dst[(size_t)nb * 32 + 2 * b + 1] = src[(size_t)b * 34 + 1];
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

__device__ __forceinline__ uint32_t byte_of(const uint4& h, int k) {
    // bytes 4..15 of the Q4_K header (the packed scales) live in h.y, h.z, h.w
    const uint32_t w = k < 4 ? h.y : (k < 8 ? h.z : h.w);
    return (w >> (8 * (k & 3))) & 0xFFu;
}

// 6-bit scale and min of sub-block g (src/quant.cpp:136-144).
__device__ __forceinline__ void q4k_scale_min(const uint4& h, int g, int& sc, int& m) {
    if (g < 4) {
        sc = byte_of(h, g) & 63;
        m = byte_of(h, g + 4) & 63;
    } else {
        sc = (byte_of(h, g + 4) & 0x0F) | ((byte_of(h, g - 4) >> 6) << 4);
        m = (byte_of(h, g + 4) >> 4) | ((byte_of(h, g) >> 6) << 4);
    }
}

// ---------------------------------------------------------------- Q4_K
// unit u of a row: block b = u/4, sub-block pair p = u%4 (sub-blocks 2p, 2p+1,
// qs bytes 32p .. 32p+31: low nibbles = sub-block 2p, high = 2p+1).
template <int NT, bool SUMS>
__device__ __forceinline__ void row_q4k(const uint8_t* __restrict__ row, int nb, const ActQ& a, int lane,
                                        float (&acc)[NT], int32_t* sumi_out, int32_t* mins_out) {
    const int nunits = nb * 4;
    const int kb = a.K / 256, k32 = a.K / 32;
    for (int u0 = 0; u0 < nunits; u0 += 64) {
        uint4 hdr[2], q0[2], q1[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int u = u0 + lane + 32 * i;
            if (u < nunits) {
                const uint8_t* blk = row + (size_t)(u >> 2) * 144;
                hdr[i] = ldg_stream(blk);
                q0[i] = ldg_stream(blk + 16 + 32 * (u & 3));
                q1[i] = ldg_stream(blk + 32 + 32 * (u & 3));
            } else {
                hdr[i] = make_uint4(0, 0, 0, 0);
                q0[i] = hdr[i];
                q1[i] = hdr[i];
            }
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int u = u0 + lane + 32 * i;
            if (u0 + 32 * i >= nunits) break;  // warp-uniform
            const bool ok = u < nunits;
            const int b = u >> 2, p = u & 3;
            int sc0 = 0, sc1 = 0, m0 = 0, m1 = 0;
            if (ok) {
                q4k_scale_min(hdr[i], 2 * p, sc0, m0);
                q4k_scale_min(hdr[i], 2 * p + 1, sc1, m1);
            }
            const uint32_t lo[8] = {q0[i].x & 0x0F0F0F0Fu, q0[i].y & 0x0F0F0F0Fu, q0[i].z & 0x0F0F0F0Fu,
                                    q0[i].w & 0x0F0F0F0Fu, q1[i].x & 0x0F0F0F0Fu, q1[i].y & 0x0F0F0F0Fu,
                                    q1[i].z & 0x0F0F0F0Fu, q1[i].w & 0x0F0F0F0Fu};
            const uint32_t hi[8] = {(q0[i].x >> 4) & 0x0F0F0F0Fu, (q0[i].y >> 4) & 0x0F0F0F0Fu,
                                    (q0[i].z >> 4) & 0x0F0F0F0Fu, (q0[i].w >> 4) & 0x0F0F0F0Fu,
                                    (q1[i].x >> 4) & 0x0F0F0F0Fu, (q1[i].y >> 4) & 0x0F0F0F0Fu,
                                    (q1[i].z >> 4) & 0x0F0F0F0Fu, (q1[i].w >> 4) & 0x0F0F0F0Fu};
            const float dw = h2f((uint16_t)(hdr[i].x & 0xFFFFu));
            const float dmw = h2f((uint16_t)(hdr[i].x >> 16));
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                int si = 0, mi = 0;
                if (ok) {
                    const int8_t* xq = a.qk + (size_t)t * a.ld + (size_t)b * 256 + 64 * p;
                    const uint4 x0 = __ldg(reinterpret_cast<const uint4*>(xq));
                    const uint4 x1 = __ldg(reinterpret_cast<const uint4*>(xq + 16));
                    const uint4 x2 = __ldg(reinterpret_cast<const uint4*>(xq + 32));
                    const uint4 x3 = __ldg(reinterpret_cast<const uint4*>(xq + 48));
                    int s0 = 0, s1 = 0;
                    s0 = dp4a((int)lo[0], (int)x0.x, s0); s0 = dp4a((int)lo[1], (int)x0.y, s0);
                    s0 = dp4a((int)lo[2], (int)x0.z, s0); s0 = dp4a((int)lo[3], (int)x0.w, s0);
                    s0 = dp4a((int)lo[4], (int)x1.x, s0); s0 = dp4a((int)lo[5], (int)x1.y, s0);
                    s0 = dp4a((int)lo[6], (int)x1.z, s0); s0 = dp4a((int)lo[7], (int)x1.w, s0);
                    s1 = dp4a((int)hi[0], (int)x2.x, s1); s1 = dp4a((int)hi[1], (int)x2.y, s1);
                    s1 = dp4a((int)hi[2], (int)x2.z, s1); s1 = dp4a((int)hi[3], (int)x2.w, s1);
                    s1 = dp4a((int)hi[4], (int)x3.x, s1); s1 = dp4a((int)hi[5], (int)x3.y, s1);
                    s1 = dp4a((int)hi[6], (int)x3.z, s1); s1 = dp4a((int)hi[7], (int)x3.w, s1);
                    si = sc0 * s0 + sc1 * s1;
                    const uint32_t bs = __ldg(reinterpret_cast<const uint32_t*>(a.bsk + (size_t)t * k32 + (size_t)b * 8 + 2 * p));
                    mi = m0 * (int)(int16_t)(bs & 0xFFFFu) + m1 * (int)(int16_t)(bs >> 16);
                }
                si += __shfl_xor_sync(0xffffffffu, si, 1);
                si += __shfl_xor_sync(0xffffffffu, si, 2);
                mi += __shfl_xor_sync(0xffffffffu, mi, 1);
                mi += __shfl_xor_sync(0xffffffffu, mi, 2);
                if (ok && p == 0) {
                    if (SUMS) {
                        sumi_out[b] = si;
                        mins_out[b] = mi;
                    } else {
                        const float dx = __ldg(a.dk + (size_t)t * kb + b);
                        acc[t] += __fmul_rn(dw, dx) * (float)si - __fmul_rn(dmw, dx) * (float)mi;
                    }
                }
            }
        }
    }
}

// ---------------------------------------------------------------- Q6_K
// unit u: block b = u/8, j = u%8: half h = j/4, l0 = 8*(j%4); covers values
// l0..l0+7 of each of the half's four 32-value quads (src/quant.cpp:194-216).
__device__ __forceinline__ uint32_t q6_signed(uint32_t v) {
    // v: four 6-bit codes 0..63 per byte -> four int8 (code - 32), no borrows.
    return (v & 0x1F1F1F1Fu) | ((~v & 0x20202020u) * 7u);
}

template <int NT, bool SUMS>
__device__ __forceinline__ void row_q6k(const uint8_t* __restrict__ row, int nb, const ActQ& a, int lane,
                                        float (&acc)[NT], int32_t* sumi_out) {
    const int nunits = nb * 8;
    const int kb = a.K / 256;
    const uint8_t* dtab = row + (size_t)nb * 208;
    for (int u0 = 0; u0 < nunits; u0 += 64) {
        uint2 qa[2], qb[2], qh[2], sc[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int u = u0 + lane + 32 * i;
            if (u < nunits) {
                const int b = u >> 3, j = u & 7, h = j >> 2, jj = j & 3;
                const uint8_t* blk = row + (size_t)b * 208;
                qa[i] = ldg_stream2(blk + 64 * h + 8 * jj);
                qb[i] = ldg_stream2(blk + 64 * h + 32 + 8 * jj);
                qh[i] = ldg_stream2(blk + 128 + 32 * h + 8 * jj);
                sc[i] = ldg_stream2(blk + 192 + 8 * h);
            } else {
                qa[i] = make_uint2(0, 0); qb[i] = qa[i]; qh[i] = qa[i]; sc[i] = qa[i];
            }
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int u = u0 + lane + 32 * i;
            if (u0 + 32 * i >= nunits) break;
            const bool ok = u < nunits;
            const int b = u >> 3, j = u & 7, h = j >> 2, jj = j & 3;
            // codes of quad q, two words (values l0..l0+3, l0+4..l0+7)
            uint32_t v[4][2];
#pragma unroll
            for (int w = 0; w < 2; ++w) {
                const uint32_t a_ = w ? qa[i].y : qa[i].x;
                const uint32_t b_ = w ? qb[i].y : qb[i].x;
                const uint32_t h_ = w ? qh[i].y : qh[i].x;
                v[0][w] = q6_signed((a_ & 0x0F0F0F0Fu) | ((h_ & 0x03030303u) << 4));
                v[1][w] = q6_signed((b_ & 0x0F0F0F0Fu) | (((h_ >> 2) & 0x03030303u) << 4));
                v[2][w] = q6_signed(((a_ >> 4) & 0x0F0F0F0Fu) | (((h_ >> 4) & 0x03030303u) << 4));
                v[3][w] = q6_signed(((b_ >> 4) & 0x0F0F0F0Fu) | (((h_ >> 6) & 0x03030303u) << 4));
            }
            // scale of quad q for this l-range: scales[8h + 2q + (l0 >= 16)]
            int scq[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int k = 2 * q + (jj >> 1);
                const uint32_t w = k < 4 ? sc[i].x : sc[i].y;
                scq[q] = (int)(int8_t)((w >> (8 * (k & 3))) & 0xFFu);
            }
            const float dw = ok ? h2f(*reinterpret_cast<const uint16_t*>(dtab + 2 * b)) : 0.0f;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                int si = 0;
                if (ok) {
                    const int8_t* xq = a.qk + (size_t)t * a.ld + (size_t)b * 256 + 128 * h + 8 * jj;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint2 xv = __ldg(reinterpret_cast<const uint2*>(xq + 32 * q));
                        const int iq = dp4a((int)v[q][0], (int)xv.x, dp4a((int)v[q][1], (int)xv.y, 0));
                        si += scq[q] * iq;
                    }
                }
                si += __shfl_xor_sync(0xffffffffu, si, 1);
                si += __shfl_xor_sync(0xffffffffu, si, 2);
                si += __shfl_xor_sync(0xffffffffu, si, 4);
                if (ok && j == 0) {
                    if (SUMS) {
                        sumi_out[b] = si;
                    } else {
                        const float dx = __ldg(a.dk + (size_t)t * kb + b);
                        acc[t] += __fmul_rn(dw, dx) * (float)si;
                    }
                }
            }
        }
    }
}

// ---------------------------------------------------------------- Q8_0
template <int NT, bool SUMS>
__device__ __forceinline__ void row_q80(const uint8_t* __restrict__ row, int nb, const ActQ& a, int lane,
                                        float (&acc)[NT], int32_t* sumi_out) {
    const int k32 = a.K / 32;
    const uint8_t* dtab = row + (size_t)nb * 32;
    for (int b0 = 0; b0 < nb; b0 += 64) {
        uint4 w0[2], w1[2];
        float dw[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int b = b0 + lane + 32 * i;
            if (b < nb) {
                w0[i] = ldg_stream(row + (size_t)b * 32);
                w1[i] = ldg_stream(row + (size_t)b * 32 + 16);
                dw[i] = h2f(*reinterpret_cast<const uint16_t*>(dtab + 2 * b));
            } else {
                w0[i] = make_uint4(0, 0, 0, 0); w1[i] = w0[i]; dw[i] = 0.0f;
            }
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int b = b0 + lane + 32 * i;
            if (b >= nb) continue;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const int8_t* xq = a.q32 + (size_t)t * a.ld + (size_t)b * 32;
                const uint4 x0 = __ldg(reinterpret_cast<const uint4*>(xq));
                const uint4 x1 = __ldg(reinterpret_cast<const uint4*>(xq + 16));
                int s = 0;
                s = dp4a((int)w0[i].x, (int)x0.x, s); s = dp4a((int)w0[i].y, (int)x0.y, s);
                s = dp4a((int)w0[i].z, (int)x0.z, s); s = dp4a((int)w0[i].w, (int)x0.w, s);
                s = dp4a((int)w1[i].x, (int)x1.x, s); s = dp4a((int)w1[i].y, (int)x1.y, s);
                s = dp4a((int)w1[i].z, (int)x1.z, s); s = dp4a((int)w1[i].w, (int)x1.w, s);
                if (SUMS) {
                    sumi_out[b] = s;
                } else {
                    const float dx = __ldg(a.d32 + (size_t)t * k32 + b);
                    acc[t] += __fmul_rn(dw[i], dx) * (float)s;
                }
            }
        }
    }
}

// ---------------------------------------------------------------- F32 / F16
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
            float v = warp_sum(acc[t]);
            if (lane == 0 && t < args.T) {
                if (g.bias) v += g.bias[rr];
                float* yp = g.y + (size_t)t * g.ldy + rr;
                if (g.epi == EPI_ADD) *yp += v;
                else *yp = v;
            }
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

extern "C" int fbk_gemv(const GemvArgs* a, cudaStream_t st) {
    if (a->T <= 0 || a->nseg <= 0) return 0;
    int total = 0;
    for (int s = 0; s < a->nseg; ++s) total += a->seg[s].rows;
    const int warps_per_cta = 8;
    int ctas = (total + warps_per_cta - 1) / warps_per_cta;
    const int cap = num_sms() * 8;
    if (ctas > cap) ctas = cap;
    if (ctas < 1) ctas = 1;
    // tokens beyond 8 are processed in groups of 8 by the caller
    if (a->T == 1) k_gemv<1><<<ctas, 256, 0, st>>>(*a);
    else if (a->T == 2) k_gemv<2><<<ctas, 256, 0, st>>>(*a);
    else if (a->T <= 4) k_gemv<4><<<ctas, 256, 0, st>>>(*a);
    else if (a->T <= 8) k_gemv<8><<<ctas, 256, 0, st>>>(*a);
    else return (int)cudaErrorInvalidValue;
    return (int)cudaGetLastError();
}

extern "C" int fbk_block_sums(int type, const uint8_t* w, size_t stride, int rows, int K, const ActQ* a,
                              int32_t* sumi, int32_t* mins, cudaStream_t st) {
    const int ctas = (rows + 7) / 8;
    k_block_sums<<<ctas, 256, 0, st>>>(type, w, stride, rows, K, *a, sumi, mins);
    return (int)cudaGetLastError();
}
