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

// Scales and mins of sub-blocks 2p and 2p+1 at once (the same bit layout as
// q4k_scale_min, src/quant.cpp:136-144), as byte pairs: low byte = sub-block
// 2p, high byte = 2p+1. Branch-free so lanes with different p stay converged.
__device__ __forceinline__ void q4k_scale_pair(const uint4& h, int p, int& sc0, int& sc1, int& m0, int& m1) {
    const int sh = 16 * (p & 1);
    const uint32_t ys = h.y >> sh, zs = h.z >> sh, ws = h.w >> sh;
    const uint32_t sc_lo = ys & 0x3F3Fu, m_lo = zs & 0x3F3Fu;                                 // p < 2
    const uint32_t sc_hi = (ws & 0x0F0Fu) | ((ys >> 2) & 0x3030u);                              // p >= 2
    const uint32_t m_hi = ((ws >> 4) & 0x0F0Fu) | ((zs >> 2) & 0x3030u);
    const uint32_t scp = p < 2 ? sc_lo : sc_hi, mp = p < 2 ? m_lo : m_hi;
    sc0 = (int)(scp & 0xFFu);
    sc1 = (int)((scp >> 8) & 0xFFu);
    m0 = (int)(mp & 0xFFu);
    m1 = (int)((mp >> 8) & 0xFFu);
}

// Q4_K unit = sub-block pair p of a block: header h (d, dmin, scales),
// q0/q1 = qs bytes 32p .. 32p+31 (low nibbles sub-block 2p, high 2p+1),
// x = the 64 activation int8 of sub-blocks 2p, 2p+1, bs = their two bsums.
// si = sc_2p * sum q.x + sc_2p+1 * sum q.x;  mi = m_2p bs_2p + m_2p+1 bs_2p+1.
struct Q4kUnit {
    uint32_t lo[8], hi[8];
    int sc0, sc1, m0, m1;
    __device__ __forceinline__ void load(const uint4& h, const uint4& q0, const uint4& q1, int p) {
        q4k_scale_pair(h, p, sc0, sc1, m0, m1);
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

// Q6_K unit j (0..7) of a block: half hh = j/4, values l0 = 8*(j%4) .. l0+7 of
// each of the half's four 32-value quads (src/quant.cpp:194-216).
// qa = ql[64hh + l0 ..+8] (quads 0, 2), qb = ql[64hh + 32 + l0 ..+8] (quads 1, 3),
// qh = qh[32hh + l0 ..+8], sc = scales[8hh .. 8hh+8].
// si = sum_q sc_q * sum (q6 - 32) x over the unit's four 8-value pieces,
// formed as sum_q sc_q * (sum q6 x - 32 sum x): the same integer, with the
// unsigned 6-bit codes fed to dp4a directly (they are < 128) and sum x, which
// depends on the activations only, computed once per activation chunk.
struct Q6kUnit {
    uint32_t v[4][2];
    int scq[4];
    __device__ __forceinline__ void load(const uint2& qa, const uint2& qb, const uint2& qh, const uint2& sc, int jj) {
#pragma unroll
        for (int w = 0; w < 2; ++w) {
            const uint32_t a = w ? qa.y : qa.x, b = w ? qb.y : qb.x, h = w ? qh.y : qh.x;
            v[0][w] = (a & 0x0F0F0F0Fu) | ((h << 4) & 0x30303030u);
            v[1][w] = (b & 0x0F0F0F0Fu) | ((h << 2) & 0x30303030u);
            v[2][w] = ((a >> 4) & 0x0F0F0F0Fu) | (h & 0x30303030u);
            v[3][w] = ((b >> 4) & 0x0F0F0F0Fu) | ((h >> 2) & 0x30303030u);
        }
        const uint32_t s = (jj >> 1) ? 8u : 0u;   // byte 2q + (l0 >= 16) of the half's 8 scales
        scq[0] = (int)(int8_t)((sc.x >> s) & 0xFFu);
        scq[1] = (int)(int8_t)((sc.x >> (16 + s)) & 0xFFu);
        scq[2] = (int)(int8_t)((sc.y >> s) & 0xFFu);
        scq[3] = (int)(int8_t)((sc.y >> (16 + s)) & 0xFFu);
    }
    // x[q] = the 8 activation int8 of quad q, xs[q] = their sum
    __device__ __forceinline__ int dot(const uint2 (&x)[4], const int (&xs)[4]) const {
        int si = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q)
            si += scq[q] * (dp4a((int)v[q][0], (int)x[q].x, dp4a((int)v[q][1], (int)x[q].y, 0)) - 32 * xs[q]);
        return si;
    }
};

// sum of the 8 int8 in x
__device__ __forceinline__ int sum8(const uint2& x) { return dp4a((int)x.x, 0x01010101, dp4a((int)x.y, 0x01010101, 0)); }

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
