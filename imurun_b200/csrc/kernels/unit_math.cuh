// unit_math.cuh — integer arithmetic of one 32-value work unit, shared by every
// GEMV variant so they all form exactly the reference's integer sums
// (src/quant_x86.cpp:299-309, 346-382, 431-495).
#pragma once

#include "common.cuh"

namespace fb {

__device__ __forceinline__ uint32_t q4k_byte(const uint4& h, int k) {
    // bytes 4..15 of a Q4_K block (the packed 6-bit scales / mins) are h.y, h.z, h.w
    const uint32_t w = k < 4 ? h.y : (k < 8 ? h.z : h.w);
    return (w >> (8 * (k & 3))) & 0xFFu;
}

// 6-bit scale and min of sub-block g (src/quant.cpp:136-144).
__device__ __forceinline__ void q4k_scale_min(const uint4& h, int g, int& sc, int& m) {
    if (g < 4) {
        sc = q4k_byte(h, g) & 63;
        m = q4k_byte(h, g + 4) & 63;
    } else {
        sc = (q4k_byte(h, g + 4) & 0x0F) | ((q4k_byte(h, g - 4) >> 6) << 4);
        m = (q4k_byte(h, g + 4) >> 4) | ((q4k_byte(h, g) >> 6) << 4);
    }
}

// Q4_K unit = sub-block pair p of a block: header h (d, dmin, scales),
// q0/q1 = qs bytes 32p .. 32p+31 (low nibbles sub-block 2p, high 2p+1),
// x = the 64 activation int8 of sub-blocks 2p, 2p+1, bs = their two bsums.
// si = sc_2p * sum q.x + sc_2p+1 * sum q.x;  mi = m_2p bs_2p + m_2p+1 bs_2p+1.
struct Q4kUnit {
    uint32_t lo[8], hi[8];
    int sc0, sc1, m0, m1;
    __device__ __forceinline__ void load(const uint4& h, const uint4& q0, const uint4& q1, int p) {
        q4k_scale_min(h, 2 * p, sc0, m0);
        q4k_scale_min(h, 2 * p + 1, sc1, m1);
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            lo[i] = w[i] & 0x0F0F0F0Fu;
            hi[i] = (w[i] >> 4) & 0x0F0F0F0Fu;
        }
    }
    __device__ __forceinline__ void dot(const uint4& x0, const uint4& x1, const uint4& x2, const uint4& x3, uint32_t bs,
                                        int& si, int& mi) const {
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
        mi = m0 * (int)(int16_t)(bs & 0xFFFFu) + m1 * (int)(int16_t)(bs >> 16);
    }
};

// four 6-bit codes 0..63 per byte -> four int8 (code - 32), no borrows
__device__ __forceinline__ uint32_t q6_signed(uint32_t v) { return (v & 0x1F1F1F1Fu) | ((~v & 0x20202020u) * 7u); }

// Q6_K unit j (0..7) of a block: half hh = j/4, values l0 = 8*(j%4) .. l0+7 of
// each of the half's four 32-value quads (src/quant.cpp:194-216).
// qa = ql[64hh + l0 ..+8] (quads 0, 2), qb = ql[64hh + 32 + l0 ..+8] (quads 1, 3),
// qh = qh[32hh + l0 ..+8], sc = scales[8hh .. 8hh+8].
// si = sum_q sc_q * sum (q6 - 32) x over the unit's four 8-value pieces.
struct Q6kUnit {
    uint32_t v[4][2];
    int scq[4];
    __device__ __forceinline__ void load(const uint2& qa, const uint2& qb, const uint2& qh, const uint2& sc, int jj) {
#pragma unroll
        for (int w = 0; w < 2; ++w) {
            const uint32_t a = w ? qa.y : qa.x, b = w ? qb.y : qb.x, h = w ? qh.y : qh.x;
            v[0][w] = q6_signed((a & 0x0F0F0F0Fu) | ((h & 0x03030303u) << 4));
            v[1][w] = q6_signed((b & 0x0F0F0F0Fu) | (((h >> 2) & 0x03030303u) << 4));
            v[2][w] = q6_signed(((a >> 4) & 0x0F0F0F0Fu) | (((h >> 4) & 0x03030303u) << 4));
            v[3][w] = q6_signed(((b >> 4) & 0x0F0F0F0Fu) | (((h >> 6) & 0x03030303u) << 4));
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int k = 2 * q + (jj >> 1);
            const uint32_t w = k < 4 ? sc.x : sc.y;
            scq[q] = (int)(int8_t)((w >> (8 * (k & 3))) & 0xFFu);
        }
    }
    // x[q] = the 8 activation int8 of quad q for this unit
    __device__ __forceinline__ int dot(const uint2 (&x)[4]) const {
        int si = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) si += scq[q] * dp4a((int)v[q][0], (int)x[q].x, dp4a((int)v[q][1], (int)x[q].y, 0));
        return si;
    }
};

// Q8_0 unit = one block: s = sum w.x over 32 values.
__device__ __forceinline__ int q80_dot(const uint4& w0, const uint4& w1, const uint4& x0, const uint4& x1) {
    int s = 0;
    s = dp4a((int)w0.x, (int)x0.x, s); s = dp4a((int)w0.y, (int)x0.y, s);
    s = dp4a((int)w0.z, (int)x0.z, s); s = dp4a((int)w0.w, (int)x0.w, s);
    s = dp4a((int)w1.x, (int)x1.x, s); s = dp4a((int)w1.y, (int)x1.y, s);
    s = dp4a((int)w1.z, (int)x1.z, s); s = dp4a((int)w1.w, (int)x1.w, s);
    return s;
}

}  // namespace fb
