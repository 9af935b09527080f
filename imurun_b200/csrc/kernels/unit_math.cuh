// unit_math.cuh — integer arithmetic of one weight block against one int8
// activation block, shared by every GEMV variant and by the block-sum check so
// they all form exactly the reference's integer sums
// (src/quant_x86.cpp:299-309, 346-382, 431-495):
//   Q4_K  sumi = sum_g sc_g sum_l q x      mins = sum_g m_g bsums_g
//   Q6_K  sumi = sum_j sc_j sum_l (q6 - 32) x
//   Q8_0  s    = sum_l w x
// One thread owns a whole block, so each integer is complete in one register
// and is converted to float once, as the reference does.
#pragma once

#include "common.cuh"

namespace fb {

// dp4a with unsigned bytes in a and signed bytes in b.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ int byte_of(uint32_t v, int k) { return (int)((v >> (8 * k)) & 0xFFu); }
// component k (a compile-time constant after unrolling) of a uint4
__device__ __forceinline__ uint32_t word_of(const uint4& v, int k) { return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w; }

// Q4_K block (144 B as 9 uint4: h = d | dmin | 12 scale bytes, then qs[128])
// against activation block x (256 int8 as 16 uint4, through LD) and its eight
// 32-value sums bs. Sub-block g's 6-bit scale and min follow
// src/quant.cpp:136-144; qs[32p + l] holds sub-block 2p (low nibble) and
// 2p+1 (high nibble) value l. The high nibbles enter dp4a unshifted (16 q),
// and the sixteenfold sum is divided exactly once per block.
template <class LD>
__device__ __forceinline__ void q4k_block(const uint4 (&w)[9], const int8_t* x, uint4 bs, int& sumi, int& mins) {
    const uint4 h = w[0];
    const uint32_t sc_lo = h.y & 0x3F3F3F3Fu;                                  // sub-blocks 0..3
    const uint32_t m_lo = h.z & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);   // sub-blocks 4..7
    const uint32_t m_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
    int even = 0, odd16 = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint4 qa = w[1 + 2 * p], qb = w[2 + 2 * p];
        const uint4 x0 = LD::ld(x + 64 * p), x1 = LD::ld(x + 64 * p + 16);
        const uint4 x2 = LD::ld(x + 64 * p + 32), x3 = LD::ld(x + 64 * p + 48);
        int s0 = 0, s1 = 0;
        s0 = dp4a_us(qa.x & 0x0F0F0F0Fu, x0.x, s0); s0 = dp4a_us(qa.y & 0x0F0F0F0Fu, x0.y, s0);
        s0 = dp4a_us(qa.z & 0x0F0F0F0Fu, x0.z, s0); s0 = dp4a_us(qa.w & 0x0F0F0F0Fu, x0.w, s0);
        s0 = dp4a_us(qb.x & 0x0F0F0F0Fu, x1.x, s0); s0 = dp4a_us(qb.y & 0x0F0F0F0Fu, x1.y, s0);
        s0 = dp4a_us(qb.z & 0x0F0F0F0Fu, x1.z, s0); s0 = dp4a_us(qb.w & 0x0F0F0F0Fu, x1.w, s0);
        s1 = dp4a_us(qa.x & 0xF0F0F0F0u, x2.x, s1); s1 = dp4a_us(qa.y & 0xF0F0F0F0u, x2.y, s1);
        s1 = dp4a_us(qa.z & 0xF0F0F0F0u, x2.z, s1); s1 = dp4a_us(qa.w & 0xF0F0F0F0u, x2.w, s1);
        s1 = dp4a_us(qb.x & 0xF0F0F0F0u, x3.x, s1); s1 = dp4a_us(qb.y & 0xF0F0F0F0u, x3.y, s1);
        s1 = dp4a_us(qb.z & 0xF0F0F0F0u, x3.z, s1); s1 = dp4a_us(qb.w & 0xF0F0F0F0u, x3.w, s1);
        const uint32_t scv = p < 2 ? sc_lo : sc_hi;
        const int k0 = (2 * p) & 3, k1 = (2 * p + 1) & 3;
        even += byte_of(scv, k0) * s0;
        odd16 += byte_of(scv, k1) * s1;
    }
    sumi = even + (odd16 >> 4);   // odd16 is an exact multiple of 16
    const int b0 = (int)(int16_t)(bs.x & 0xFFFFu), b1 = (int)(int16_t)(bs.x >> 16);
    const int b2 = (int)(int16_t)(bs.y & 0xFFFFu), b3 = (int)(int16_t)(bs.y >> 16);
    const int b4 = (int)(int16_t)(bs.z & 0xFFFFu), b5 = (int)(int16_t)(bs.z >> 16);
    const int b6 = (int)(int16_t)(bs.w & 0xFFFFu), b7 = (int)(int16_t)(bs.w >> 16);
    mins = byte_of(m_lo, 0) * b0 + byte_of(m_lo, 1) * b1 + byte_of(m_lo, 2) * b2 + byte_of(m_lo, 3) * b3 +
           byte_of(m_hi, 0) * b4 + byte_of(m_hi, 1) * b5 + byte_of(m_hi, 2) * b6 + byte_of(m_hi, 3) * b7;
}

// Q6_K block (208 B as 13 uint4: ql[128], qh[64], int8 scales[16]; the fp16 d
// lives in the group's scale table) against x (256 int8) and xs16[j] = sum of
// x over values 16j .. 16j+15. Value l (0..31) of quad q (0..3) of half hh:
// ql nibble (ql[64hh + l + 32(q&1)], low for q < 2) | 2 bits of qh[32hh + l]
// at 2q, scale sc[8hh + 2q + l/16] (src/quant.cpp:194-216). The unsigned
// 6-bit codes go to dp4a as they are; sum (q6 - 32) x = sum q6 x - 32 sum x.
template <class LD>
__device__ __forceinline__ int q6k_block(const uint4 (&w)[13], const int8_t* x, const int16_t* xs16) {
    const uint4 scw = w[12];
    int sumi = 0, corr = 0;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
        for (int hl = 0; hl < 2; ++hl) {   // values l in [16 hl, 16 hl + 16)
            int s[4] = {0, 0, 0, 0};
            const uint4 xa = LD::ld(x + 128 * hh + 16 * hl);        // quad 0
            const uint4 xb = LD::ld(x + 128 * hh + 32 + 16 * hl);   // quad 1
            const uint4 xc = LD::ld(x + 128 * hh + 64 + 16 * hl);   // quad 2
            const uint4 xd = LD::ld(x + 128 * hh + 96 + 16 * hl);   // quad 3
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int wi = 4 * hl + i;
                const uint32_t a = word_of(w[(16 * hh + wi) >> 2], wi & 3);
                const uint32_t b = word_of(w[(16 * hh + 8 + wi) >> 2], wi & 3);
                const uint32_t hb = word_of(w[8 + ((8 * hh + wi) >> 2)], wi & 3);
                const uint32_t v0 = (a & 0x0F0F0F0Fu) | ((hb << 4) & 0x30303030u);
                const uint32_t v1 = (b & 0x0F0F0F0Fu) | ((hb << 2) & 0x30303030u);
                const uint32_t v2 = ((a >> 4) & 0x0F0F0F0Fu) | (hb & 0x30303030u);
                const uint32_t v3 = ((b >> 4) & 0x0F0F0F0Fu) | ((hb >> 2) & 0x30303030u);
                s[0] = dp4a_us(v0, word_of(xa, i), s[0]);
                s[1] = dp4a_us(v1, word_of(xb, i), s[1]);
                s[2] = dp4a_us(v2, word_of(xc, i), s[2]);
                s[3] = dp4a_us(v3, word_of(xd, i), s[3]);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int j = 8 * hh + 2 * q + hl;
                const int sc = (int)(int8_t)byte_of(word_of(scw, j >> 2), j & 3);
                sumi += sc * s[q];
                corr += sc * (int)xs16[j];
            }
        }
    }
    return sumi - 32 * corr;
}

// Quarter p (0..3) of a Q4_K block, for four lanes that share one block: qs
// bytes 32p .. 32p+31 (qa, qb), i.e. sub-blocks 2p (low nibbles, x0 x1) and
// 2p+1 (high nibbles, x2 x3), and bsw = the two 32-value sums of those
// sub-blocks (int16 pair). acc16 = 16 * (low part) + (unshifted high part);
// the four lanes' acc16 and mins add up, as integers, to 16 * sumi and to the
// mins of q4k_block, so sumi = (sum acc16) >> 4 exactly.
__device__ __forceinline__ void q4k_quarter(uint4 h, uint4 qa, uint4 qb, uint4 x0, uint4 x1, uint4 x2, uint4 x3,
                                            uint32_t bsw, int p, int& acc16, int& mins) {
    const uint32_t sc = p < 2 ? (h.y & 0x3F3F3F3Fu) : ((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u));
    const uint32_t mn = p < 2 ? (h.z & 0x3F3F3F3Fu) : (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u));
    const int k0 = (2 * p) & 3;
    int s0 = 0, s1 = 0;
    s0 = dp4a_us(qa.x & 0x0F0F0F0Fu, x0.x, s0); s0 = dp4a_us(qa.y & 0x0F0F0F0Fu, x0.y, s0);
    s0 = dp4a_us(qa.z & 0x0F0F0F0Fu, x0.z, s0); s0 = dp4a_us(qa.w & 0x0F0F0F0Fu, x0.w, s0);
    s0 = dp4a_us(qb.x & 0x0F0F0F0Fu, x1.x, s0); s0 = dp4a_us(qb.y & 0x0F0F0F0Fu, x1.y, s0);
    s0 = dp4a_us(qb.z & 0x0F0F0F0Fu, x1.z, s0); s0 = dp4a_us(qb.w & 0x0F0F0F0Fu, x1.w, s0);
    s1 = dp4a_us(qa.x & 0xF0F0F0F0u, x2.x, s1); s1 = dp4a_us(qa.y & 0xF0F0F0F0u, x2.y, s1);
    s1 = dp4a_us(qa.z & 0xF0F0F0F0u, x2.z, s1); s1 = dp4a_us(qa.w & 0xF0F0F0F0u, x2.w, s1);
    s1 = dp4a_us(qb.x & 0xF0F0F0F0u, x3.x, s1); s1 = dp4a_us(qb.y & 0xF0F0F0F0u, x3.y, s1);
    s1 = dp4a_us(qb.z & 0xF0F0F0F0u, x3.z, s1); s1 = dp4a_us(qb.w & 0xF0F0F0F0u, x3.w, s1);
    acc16 = 16 * byte_of(sc, k0) * s0 + byte_of(sc, k0 + 1) * s1;
    mins = byte_of(mn, k0) * (int)(int16_t)(bsw & 0xFFFFu) + byte_of(mn, k0 + 1) * (int)(int16_t)(bsw >> 16);
}

// Quarter (hh, hl) of a Q6_K block: values l in [16 hl, 16 hl + 16) of half hh
// of all four quads (the iteration (hh, hl) of q6k_block). a, b = ql bytes
// 64hh + 16hl and 64hh + 32 + 16hl, hb = qh bytes 32hh + 16hl, sc = the
// block's 16 scales, xa..xd = x at 128hh + 16hl + 32q, xs16 = sums of x over
// the same four 16-value runs. Returns sum (q6 - 32) x over those values; the
// four quarters add up to q6k_block's result.
__device__ __forceinline__ int q6k_quarter(uint4 a4, uint4 b4, uint4 h4, uint4 sc, uint4 xa, uint4 xb, uint4 xc,
                                           uint4 xd, const int (&xs16)[4], int hh, int hl) {
    int s[4] = {0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t a = word_of(a4, i), b = word_of(b4, i), hb = word_of(h4, i);
        const uint32_t v0 = (a & 0x0F0F0F0Fu) | ((hb << 4) & 0x30303030u);
        const uint32_t v1 = (b & 0x0F0F0F0Fu) | ((hb << 2) & 0x30303030u);
        const uint32_t v2 = ((a >> 4) & 0x0F0F0F0Fu) | (hb & 0x30303030u);
        const uint32_t v3 = ((b >> 4) & 0x0F0F0F0Fu) | ((hb >> 2) & 0x30303030u);
        s[0] = dp4a_us(v0, word_of(xa, i), s[0]);
        s[1] = dp4a_us(v1, word_of(xb, i), s[1]);
        s[2] = dp4a_us(v2, word_of(xc, i), s[2]);
        s[3] = dp4a_us(v3, word_of(xd, i), s[3]);
    }
    // scales j = 8hh + 2q + hl: bytes hl and 2 + hl of the halves of word 2hh (q < 2) and 2hh + 1 (q >= 2)
    const uint32_t w0 = hh ? sc.z : sc.x, w1 = hh ? sc.w : sc.y;
    const int c0 = (int)(int8_t)byte_of(w0, hl), c1 = (int)(int8_t)byte_of(w0, 2 + hl);
    const int c2 = (int)(int8_t)byte_of(w1, hl), c3 = (int)(int8_t)byte_of(w1, 2 + hl);
    const int sumi = c0 * s[0] + c1 * s[1] + c2 * s[2] + c3 * s[3];
    const int corr = c0 * xs16[0] + c1 * xs16[1] + c2 * xs16[2] + c3 * xs16[3];
    return sumi - 32 * corr;
}

// Q8_0 block (qs[32] as 2 uint4) against x (32 int8): s = sum w x.
template <class LD>
__device__ __forceinline__ int q80_block(uint4 w0, uint4 w1, const int8_t* x) {
    const uint4 x0 = LD::ld(x), x1 = LD::ld(x + 16);
    int s = 0;
    s = __dp4a((int)w0.x, (int)x0.x, s); s = __dp4a((int)w0.y, (int)x0.y, s);
    s = __dp4a((int)w0.z, (int)x0.z, s); s = __dp4a((int)w0.w, (int)x0.w, s);
    s = __dp4a((int)w1.x, (int)x1.x, s); s = __dp4a((int)w1.y, (int)x1.y, s);
    s = __dp4a((int)w1.z, (int)x1.z, s); s = __dp4a((int)w1.w, (int)x1.w, s);
    return s;
}

// sum of the 16 int8 in x
__device__ __forceinline__ int sum16(uint4 x) {
    int s = __dp4a((int)x.x, 0x01010101, 0);
    s = __dp4a((int)x.y, 0x01010101, s);
    s = __dp4a((int)x.z, 0x01010101, s);
    return __dp4a((int)x.w, 0x01010101, s);
}

// loaders: shared memory (plain), global weights (streaming, no L1
// allocation), global activations (read-only cache)
struct LdShared {
    static __device__ __forceinline__ uint4 ld(const void* p) { return *reinterpret_cast<const uint4*>(p); }
};
struct LdStream {
    static __device__ __forceinline__ uint4 ld(const void* p) { return ldg_stream(p); }
};
struct LdGlobal {
    static __device__ __forceinline__ uint4 ld(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
};

}  // namespace fb
