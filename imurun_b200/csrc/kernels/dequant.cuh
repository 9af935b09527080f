// dequant.cuh — single-value dequantisation of a device-layout matrix row.
#pragma once

#include "common.cuh"
#include "layout.cuh"

namespace fb {

// Value i of row `row` of a device-layout matrix, dequantised exactly like the
// reference's dequant_row (src/quant.cpp:129-216): same float operations in
// the same order.
__device__ __forceinline__ float dequant_at(int type, const uint8_t* w, int n, int row, int i) {
    switch (type) {
        case T_F32: return reinterpret_cast<const float*>(w + (size_t)row * (((size_t)n * 4 + 15) / 16 * 16))[i];
        case T_F16: return h2f(reinterpret_cast<const uint16_t*>(w + (size_t)row * (((size_t)n * 2 + 15) / 16 * 16))[i]);
        case T_Q8_0: {
            const int b = i / 32;
            const float d = h2f(*reinterpret_cast<const uint16_t*>(w + dscale_offset_tm(T_Q8_0, n, row, b)));
            return __fmul_rn(d, (float)reinterpret_cast<const int8_t*>(w + block_offset_tm(T_Q8_0, n, row, b))[i % 32]);
        }
        case T_Q4_K: {
            const int b = i / 256, r = i % 256, g = r / 32, l = r % 32;
            const uint8_t* blk = w + block_offset_tm(T_Q4_K, n, row, b);
            const float d = h2f(*reinterpret_cast<const uint16_t*>(blk));
            const float dm = h2f(*reinterpret_cast<const uint16_t*>(blk + 2));
            const uint8_t* s = blk + 4;
            int sc, m;
            if (g < 4) { sc = s[g] & 63; m = s[g + 4] & 63; }
            else { sc = (s[g + 4] & 0x0F) | ((s[g - 4] >> 6) << 4); m = (s[g + 4] >> 4) | ((s[g] >> 6) << 4); }
            const uint8_t qb = blk[16 + 32 * (g >> 1) + l];
            const int q = (g & 1) ? (qb >> 4) : (qb & 0x0F);
            return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dm, (float)m));
        }
        case T_Q6_K: {
            const int b = i / 256, r = i % 256, h = r / 128, rr = r % 128, quad = rr / 32, l = rr % 32;
            const uint8_t* blk = w + block_offset_tm(T_Q6_K, n, row, b);
            const float d = h2f(*reinterpret_cast<const uint16_t*>(w + dscale_offset_tm(T_Q6_K, n, row, b)));
            const uint8_t qlb = blk[64 * h + l + ((quad & 1) ? 32 : 0)];
            const int lo = quad < 2 ? (qlb & 0x0F) : (qlb >> 4);
            const int hi = (blk[128 + 32 * h + l] >> (2 * quad)) & 3;
            const int q = (lo | (hi << 4)) - 32;
            const int sc = (int)reinterpret_cast<const int8_t*>(blk + 192)[8 * h + 2 * quad + l / 16];
            return __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
        }
        default: return 0.0f;
    }
}

}  // namespace fb
