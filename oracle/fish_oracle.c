/*
 * fish_oracle.c — CPU restatement of FISH's decode/prefill arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (see fish_oracle.h). Plain C99, single threaded,
 * written from the reference's behaviour; every function cites the reference
 * file:line (relative to model/fish/) that it restates. Built with
 * -O2 -ffp-contract=off and without fast-math so the float steps that must be
 * byte-exact (activation quantisation) round exactly like the reference.
 */
#define _GNU_SOURCE
#include "fish_oracle.h"

#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

/* ======================================================================= fp16 */

/* quant.cpp:21-44: exact half -> float, subnormals renormalised. */
float or_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            int e = 127 - 15 + 1;
            while ((mant & 0x400u) == 0) { mant <<= 1; --e; }
            mant &= 0x3FFu;
            bits = sign | ((uint32_t)e << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((exp - 15 + 127) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* quantize.cpp:32-55: float -> half, round to nearest even, subnormals kept. */
uint16_t or_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int32_t e = (int32_t)((x >> 23) & 0xFF);
    uint32_t m = x & 0x7FFFFFu;
    if (e == 255) return (uint16_t)(sign | 0x7C00u | (m ? 0x200u : 0));
    const int32_t he = e - 127 + 15;
    if (he >= 31) return (uint16_t)(sign | 0x7C00u);
    if (he <= 0) {
        if (he < -10) return (uint16_t)sign;
        m |= 0x800000u;
        const int shift = 14 - he;
        uint32_t hm = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (hm & 1u))) ++hm;
        return (uint16_t)(sign | hm);
    }
    const uint32_t hm = m >> 13;
    const uint32_t rem = m & 0x1FFFu;
    uint32_t out = sign | ((uint32_t)he << 10) | hm;
    if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) ++out;
    return (uint16_t)out;
}

static inline float h2f_at(const uint8_t* p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return or_fp16_to_fp32(h);
}

/* ================================================================ type table */

/* gguf.cpp:215-275 (subset FISH's hot path uses). */
int or_block_elems(int t) {
    switch (t) {
        case OR_F32: case OR_F16: case OR_BF16: return 1;
        case OR_Q4_K: case OR_Q5_K: case OR_Q6_K: return 256;
        case OR_Q4_0: case OR_Q8_0: return 32;
        default: return 0;
    }
}

int or_block_bytes(int t) {
    switch (t) {
        case OR_F32: return 4;
        case OR_F16: case OR_BF16: return 2;
        case OR_Q4_0: return 18;
        case OR_Q8_0: return 34;
        case OR_Q4_K: return 144;
        case OR_Q5_K: return 176;
        case OR_Q6_K: return 210;
        default: return 0;
    }
}

uint64_t or_row_bytes(int t, uint64_t n) {
    const int be = or_block_elems(t), bb = or_block_bytes(t);
    if (!be || !bb) return 0;
    return (n / (uint64_t)be) * (uint64_t)bb;
}

/* ============================================================ dequantisation */

/* quant.cpp:83-90 */
static void deq_q4_0(const uint8_t* p, float* y) {
    const float d = h2f_at(p);
    const uint8_t* qs = p + 2;
    for (int j = 0; j < 16; ++j) {
        y[j] = d * (float)((qs[j] & 0x0F) - 8);
        y[j + 16] = d * (float)((qs[j] >> 4) - 8);
    }
}

/* quant.cpp:129-133 */
static void deq_q8_0(const uint8_t* p, float* y) {
    const float d = h2f_at(p);
    const int8_t* qs = (const int8_t*)(p + 2);
    for (int j = 0; j < 32; ++j) y[j] = d * (float)qs[j];
}

/* quant.cpp:136-144: 6-bit scale / min j of the 12 packed bytes. */
static void scale_min_k4(int j, const uint8_t* q, uint8_t* d, uint8_t* m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (uint8_t)((q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* quant.cpp:146-163. Block: d(2) dmin(2) scales(12) qs(128). */
static void deq_q4_K(const uint8_t* p, float* y) {
    const float d = h2f_at(p), mn = h2f_at(p + 2);
    const uint8_t* sc = p + 4;
    const uint8_t* q = p + 16;
    int is = 0;
    for (int j = 0; j < 256; j += 64) {
        uint8_t s, m;
        scale_min_k4(is + 0, sc, &s, &m);
        const float d1 = d * s, m1 = mn * m;
        scale_min_k4(is + 1, sc, &s, &m);
        const float d2 = d * s, m2 = mn * m;
        for (int l = 0; l < 32; ++l) y[j + l] = d1 * (float)(q[l] & 0x0F) - m1;
        for (int l = 0; l < 32; ++l) y[j + 32 + l] = d2 * (float)(q[l] >> 4) - m2;
        q += 32;
        is += 2;
    }
}

/* quant.cpp:165-192. Block: d dmin scales(12) qh(32) qs(128). */
static void deq_q5_K(const uint8_t* p, float* y) {
    const float d = h2f_at(p), mn = h2f_at(p + 2);
    const uint8_t* sc = p + 4;
    const uint8_t* qh = p + 16;
    const uint8_t* ql = p + 48;
    int is = 0;
    uint8_t u1 = 1, u2 = 2;
    for (int j = 0; j < 256; j += 64) {
        uint8_t s, m;
        scale_min_k4(is + 0, sc, &s, &m);
        const float d1 = d * s, m1 = mn * m;
        scale_min_k4(is + 1, sc, &s, &m);
        const float d2 = d * s, m2 = mn * m;
        for (int l = 0; l < 32; ++l)
            y[j + l] = d1 * (float)((ql[l] & 0x0F) + ((qh[l] & u1) ? 16 : 0)) - m1;
        for (int l = 0; l < 32; ++l)
            y[j + 32 + l] = d2 * (float)((ql[l] >> 4) + ((qh[l] & u2) ? 16 : 0)) - m2;
        ql += 32;
        is += 2;
        u1 = (uint8_t)(u1 << 2);
        u2 = (uint8_t)(u2 << 2);
    }
}

/* quant.cpp:194-216. Block: ql(128) qh(64) scales(16, int8) d(2) @208. */
static void deq_q6_K(const uint8_t* p, float* y) {
    const float d = h2f_at(p + 208);
    const uint8_t* ql = p;
    const uint8_t* qh = p + 128;
    const int8_t* sc = (const int8_t*)(p + 192);
    for (int n = 0; n < 256; n += 128) {
        for (int l = 0; l < 32; ++l) {
            const int is = l / 16;
            const int q1 = ((ql[l] & 0x0F) | (((qh[l] >> 0) & 3) << 4)) - 32;
            const int q2 = ((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
            const int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            const int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            y[n + l + 0] = d * (float)sc[is + 0] * (float)q1;
            y[n + l + 32] = d * (float)sc[is + 2] * (float)q2;
            y[n + l + 64] = d * (float)sc[is + 4] * (float)q3;
            y[n + l + 96] = d * (float)sc[is + 6] * (float)q4;
        }
        ql += 64;
        qh += 32;
        sc += 8;
    }
}

/* quant.cpp:470-506 (dequant_row). */
int or_dequant_row(int type, const void* src, float* dst, uint64_t n) {
    const uint8_t* p = (const uint8_t*)src;
    if (!src || !dst) return 0;
    if (type == OR_F32) { memcpy(dst, src, n * 4); return 1; }
    if (type == OR_F16) { for (uint64_t i = 0; i < n; ++i) dst[i] = h2f_at(p + 2 * i); return 1; }
    if (type == OR_BF16) {
        for (uint64_t i = 0; i < n; ++i) {
            uint16_t v; memcpy(&v, p + 2 * i, 2);
            uint32_t b = (uint32_t)v << 16; memcpy(dst + i, &b, 4);
        }
        return 1;
    }
    const int be = or_block_elems(type), bb = or_block_bytes(type);
    if (!be || n % (uint64_t)be) return 0;
    for (uint64_t i = 0; i < n; i += (uint64_t)be, p += bb) {
        switch (type) {
            case OR_Q4_0: deq_q4_0(p, dst + i); break;
            case OR_Q8_0: deq_q8_0(p, dst + i); break;
            case OR_Q4_K: deq_q4_K(p, dst + i); break;
            case OR_Q5_K: deq_q5_K(p, dst + i); break;
            case OR_Q6_K: deq_q6_K(p, dst + i); break;
            default: return 0;
        }
    }
    return 1;
}

/* ==================================================== activation quantisers */

static inline int8_t clamp127(long v) { return (int8_t)(v < -127 ? -127 : (v > 127 ? 127 : v)); }

/* quant.cpp:400-415: per 32 values, d = amax/127, id = 1/d (0 if d == 0),
 * q = clamp(lrintf(x * id), +-127) with round-half-to-even, sum = sum q. */
void or_quantize_acts(const float* x, uint64_t n, or_q8act* out) {
    for (uint64_t i = 0; i < n; i += 32, ++out) {
        float amax = 0.0f;
        for (int k = 0; k < 32; ++k) { const float a = fabsf(x[i + k]); if (a > amax) amax = a; }
        const float d = amax / 127.0f;
        const float id = d > 0.0f ? 1.0f / d : 0.0f;
        out->d = d;
        int32_t sum = 0;
        for (int k = 0; k < 32; ++k) {
            const float v = x[i + k] * id;
            out->qs[k] = clamp127(lrintf(v));
            sum += out->qs[k];
        }
        out->sum = sum;
    }
}

/* quant.cpp:417-434: one d per 256 values, bsums[8] = per-32 sums (int16). */
void or_quantize_acts_k(const float* x, uint64_t n, or_q8actk* out) {
    for (uint64_t i = 0; i < n; i += 256, ++out) {
        float amax = 0.0f;
        for (int k = 0; k < 256; ++k) { const float a = fabsf(x[i + k]); if (a > amax) amax = a; }
        const float d = amax / 127.0f;
        const float id = d > 0.0f ? 1.0f / d : 0.0f;
        out->d = d;
        for (int b = 0; b < 8; ++b) {
            int32_t sum = 0;
            for (int k = 0; k < 32; ++k) {
                const float v = x[i + b * 32 + k] * id;
                out->qs[b * 32 + k] = clamp127(lrintf(v));
                sum += out->qs[b * 32 + k];
            }
            out->bsums[b] = (int16_t)sum;
        }
    }
}

/* ======================================================= integer block sums */

/* quant_x86.cpp:317-327 / quant.cpp:136-144: sc[8], m[8] of a Q4_K/Q5_K block. */
static void k4_scales(const uint8_t* s12, int* sc, int* mn) {
    for (int j = 0; j < 8; ++j) {
        uint8_t a, b;
        scale_min_k4(j, s12, &a, &b);
        sc[j] = a;
        mn[j] = b;
    }
}

/* Sub-block g (0..7) value l (0..31) of a Q4_K block: nibble (g even: low,
 * odd: high) of qs[32*(g/2) + l]  (quant.cpp:146-163). */
static inline int q4k_val(const uint8_t* qs, int g, int l) {
    const uint8_t b = qs[32 * (g >> 1) + l];
    return (g & 1) ? (b >> 4) : (b & 0x0F);
}

/* Value i (0..255) of a Q6_K block as q6 - 32 (quant.cpp:194-216). */
static inline int q6k_val(const uint8_t* p, int i) {
    const int half = i / 128, r = i % 128, quad = r / 32, l = r % 32;
    const uint8_t* ql = p + 64 * half;
    const uint8_t* qh = p + 128 + 32 * half;
    int lo;
    if (quad == 0) lo = ql[l] & 0x0F;
    else if (quad == 1) lo = ql[l + 32] & 0x0F;
    else if (quad == 2) lo = ql[l] >> 4;
    else lo = ql[l + 32] >> 4;
    const int hi = (qh[l] >> (2 * quad)) & 3;
    return (lo | (hi << 4)) - 32;
}

/* Scale index of Q6_K value i: groups of 16 in value order (quant.cpp:200-210,
 * quant_x86.cpp:431-495: sc[is + 2*quad] with is = l/16 inside each half). */
static inline int q6k_scale_index(int i) {
    const int half = i / 128, r = i % 128, quad = r / 32, l = r % 32;
    return 8 * half + 2 * quad + l / 16;
}

int or_block_sums(int type, const void* row, const void* acts, uint64_t n,
                  int32_t* sumi, int32_t* mins) {
    const uint8_t* p = (const uint8_t*)row;
    if (type == OR_Q8_0 || type == OR_Q4_0) {
        const or_q8act* x = (const or_q8act*)acts;
        const int bb = or_block_bytes(type);
        for (uint64_t b = 0; b < n / 32; ++b, p += bb) {
            int32_t s = 0;
            if (type == OR_Q8_0) {
                const int8_t* qs = (const int8_t*)(p + 2);
                for (int k = 0; k < 32; ++k) s += (int32_t)qs[k] * x[b].qs[k];
            } else {
                /* quant_x86.cpp:279-294: low nibbles are values 0..15, high 16..31. */
                const uint8_t* qs = p + 2;
                for (int k = 0; k < 16; ++k) {
                    s += (int32_t)(qs[k] & 0x0F) * x[b].qs[k];
                    s += (int32_t)(qs[k] >> 4) * x[b].qs[k + 16];
                }
            }
            sumi[b] = s;
            if (mins) mins[b] = 0;
        }
        return 1;
    }
    if (type == OR_Q4_K || type == OR_Q5_K) {
        const or_q8actk* x = (const or_q8actk*)acts;
        const int bb = or_block_bytes(type);
        for (uint64_t b = 0; b < n / 256; ++b, p += bb) {
            int sc[8], mn[8];
            k4_scales(p + 4, sc, mn);
            int32_t s = 0, m = 0;
            for (int g = 0; g < 8; ++g) {
                int32_t gs = 0;
                for (int l = 0; l < 32; ++l) {
                    int q;
                    if (type == OR_Q4_K) {
                        q = q4k_val(p + 16, g, l);
                    } else {
                        const uint8_t* qh = p + 16;
                        const uint8_t* ql = p + 48;
                        const uint8_t bq = ql[32 * (g >> 1) + l];
                        q = ((g & 1) ? (bq >> 4) : (bq & 0x0F)) + (((qh[l] >> g) & 1) << 4);
                    }
                    gs += q * x[b].qs[32 * g + l];
                }
                s += sc[g] * gs;
                m += mn[g] * x[b].bsums[g];
            }
            sumi[b] = s;
            if (mins) mins[b] = m;
        }
        return 1;
    }
    if (type == OR_Q6_K) {
        const or_q8actk* x = (const or_q8actk*)acts;
        for (uint64_t b = 0; b < n / 256; ++b, p += 210) {
            const int8_t* sc = (const int8_t*)(p + 192);
            int32_t grp[16] = {0};
            for (int i = 0; i < 256; ++i) grp[q6k_scale_index(i)] += q6k_val(p, i) * x[b].qs[i];
            int32_t s = 0;
            for (int j = 0; j < 16; ++j) s += (int32_t)sc[j] * grp[j];
            sumi[b] = s;
            if (mins) mins[b] = 0;
        }
        return 1;
    }
    return 0;
}

/* quant.cpp:475-481 */
static int has_q8_kernel(int t) { return t == OR_Q4_0 || t == OR_Q8_0; }
static int has_q8k_kernel(int t) { return t == OR_Q4_K || t == OR_Q5_K || t == OR_Q6_K; }

/* quant_x86.cpp:279-309 (Q4_0 / Q8_0 against Q8Act). */
int or_vec_dot_q8(int type, const void* row, const or_q8act* x, uint64_t n, float* out) {
    if (!has_q8_kernel(type)) return 0;
    const uint8_t* p = (const uint8_t*)row;
    const int bb = or_block_bytes(type);
    double acc = 0.0;
    for (uint64_t b = 0; b < n / 32; ++b, p += bb) {
        int32_t s;
        or_block_sums(type, p, x + b, 32, &s, NULL);
        const float sc = h2f_at(p) * x[b].d;
        acc += (double)sc * (double)s;
        if (type == OR_Q4_0) acc -= (double)(sc * 8.0f) * (double)x[b].sum;
    }
    *out = (float)acc;
    return 1;
}

/* quant_x86.cpp:346-382 (Q4_K), 389-429 (Q5_K), 431-495 (Q6_K). */
int or_vec_dot_q8k(int type, const void* row, const or_q8actk* x, uint64_t n, float* out) {
    if (!has_q8k_kernel(type)) return 0;
    const uint8_t* p = (const uint8_t*)row;
    const int bb = or_block_bytes(type);
    double acc = 0.0;
    for (uint64_t b = 0; b < n / 256; ++b, p += bb) {
        int32_t s, m;
        or_block_sums(type, p, x + b, 256, &s, &m);
        if (type == OR_Q6_K) {
            acc += (double)(h2f_at(p + 208) * x[b].d) * (double)s;
        } else {
            acc += (double)(h2f_at(p) * x[b].d) * (double)s;
            acc -= (double)(h2f_at(p + 2) * x[b].d) * (double)m;
        }
    }
    *out = (float)acc;
    return 1;
}

/* ops.cpp:177-264: int8 path when the type has a kernel of the matching
 * layout (K-quants need n_in % 256 == 0, ops.cpp:166-174), else f32. */
void or_matmul(int type, const void* w, const float* x, int n_tok, int n_in,
               int n_out, float* y) {
    const uint64_t rb = or_row_bytes(type, (uint64_t)n_in);
    const uint8_t* base = (const uint8_t*)w;
    const int k_path = has_q8k_kernel(type) && (n_in % 256) == 0;
    const int q_path = has_q8_kernel(type) && (n_in % 32) == 0;
    if (k_path || q_path) {
        void* acts = malloc((size_t)n_tok * (size_t)(n_in / 32) * sizeof(or_q8act) + 16);
        for (int t = 0; t < n_tok; ++t) {
            const float* xt = x + (size_t)t * n_in;
            float* yt = y + (size_t)t * n_out;
            if (k_path) {
                or_q8actk* q = (or_q8actk*)acts;
                or_quantize_acts_k(xt, (uint64_t)n_in, q);
                for (int i = 0; i < n_out; ++i) or_vec_dot_q8k(type, base + (size_t)i * rb, q, (uint64_t)n_in, yt + i);
            } else {
                or_q8act* q = (or_q8act*)acts;
                or_quantize_acts(xt, (uint64_t)n_in, q);
                for (int i = 0; i < n_out; ++i) or_vec_dot_q8(type, base + (size_t)i * rb, q, (uint64_t)n_in, yt + i);
            }
        }
        free(acts);
        return;
    }
    float* row = (float*)malloc((size_t)n_in * sizeof(float));
    for (int i = 0; i < n_out; ++i) {
        or_dequant_row(type, base + (size_t)i * rb, row, (uint64_t)n_in);
        for (int t = 0; t < n_tok; ++t) {
            const float* xt = x + (size_t)t * n_in;
            double s = 0.0;
            for (int k = 0; k < n_in; ++k) s += (double)row[k] * xt[k];
            y[(size_t)t * n_out + i] = (float)s;
        }
    }
    free(row);
}

/* or_matmul with the activations given as records instead of quantised
 * here: qk (Q8ActK, rows of n_in/256 records) for types with a 256-layout
 * kernel, q32 (Q8Act, rows of n_in/32 records) for the 32-layout ones; other
 * weight types, or a NULL record array, take or_matmul's own path on x. */
static void matmul_acts(int type, const void* w, const float* x, const void* qk, const void* q32, int n_tok, int n_in,
                        int n_out, float* y) {
    const uint64_t rb = or_row_bytes(type, (uint64_t)n_in);
    const uint8_t* base = (const uint8_t*)w;
    const int k_path = has_q8k_kernel(type) && (n_in % 256) == 0 && qk;
    const int q_path = !k_path && has_q8_kernel(type) && (n_in % 32) == 0 && q32;
    if (!k_path && !q_path) {
        or_matmul(type, w, x, n_tok, n_in, n_out, y);
        return;
    }
    for (int t = 0; t < n_tok; ++t) {
        float* yt = y + (size_t)t * n_out;
        if (k_path) {
            const or_q8actk* a = (const or_q8actk*)qk + (size_t)t * (n_in / 256);
            for (int i = 0; i < n_out; ++i) or_vec_dot_q8k(type, base + (size_t)i * rb, a, (uint64_t)n_in, yt + i);
        } else {
            const or_q8act* a = (const or_q8act*)q32 + (size_t)t * (n_in / 32);
            for (int i = 0; i < n_out; ++i) or_vec_dot_q8(type, base + (size_t)i * rb, a, (uint64_t)n_in, yt + i);
        }
    }
}

/* ====================================================================== glue */

/* ops.cpp:18-23: the sum of squares is accumulated in double. */
void or_rmsnorm(float* out, const float* x, const float* w, int n, float eps) {
    double sum = 0.0;
    for (int i = 0; i < n; ++i) sum += (double)x[i] * x[i];
    const float scale = 1.0f / sqrtf((float)(sum / n) + eps);
    for (int i = 0; i < n; ++i) out[i] = x[i] * scale * w[i];
}

/* ops.cpp:25-31 */
void or_silu_inplace(float* x, int n) {
    for (int i = 0; i < n; ++i) { const float v = x[i]; x[i] = v / (1.0f + expf(-v)); }
}

/* ops.cpp:32-38: the tanh form of GELU */
void or_gelu_inplace(float* x, int n) {
    const float k = 0.7978845608028654f;
    for (int i = 0; i < n; ++i) {
        const float v = x[i];
        x[i] = 0.5f * v * (1.0f + tanhf(k * (v + 0.044715f * v * v * v)));
    }
}

/* ops.cpp:40-55 */
void or_softmax_inplace(float* x, int n) {
    if (n <= 0) return;
    float m = x[0];
    for (int i = 1; i < n; ++i) if (x[i] > m) m = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) { x[i] = expf(x[i] - m); sum += x[i]; }
    if (sum <= 0.0f) { for (int i = 0; i < n; ++i) x[i] = 1.0f / (float)n; return; }
    const float inv = 1.0f / sum;
    for (int i = 0; i < n; ++i) x[i] *= inv;
}

/* ops.cpp:61-70 */
static float yarn_corr_dim(int n_dims, int n_orig_ctx, float n_rot, float base) {
    return (float)n_dims * logf((float)n_orig_ctx / (n_rot * 2.0f * 3.14159265358979f)) / (2.0f * logf(base));
}
static float yarn_ramp(float low, float high, int i0) {
    const float den = (high - low) > 0.001f ? (high - low) : 0.001f;
    float y = ((float)i0 / 2.0f - low) / den;
    y = y < 0.0f ? 0.0f : (y > 1.0f ? 1.0f : y);
    return 1.0f - y;
}

/* ops.cpp:75-124: angles in double, cos/sin stored as float times mscale. */
void or_rope_build(float* cs, float* sn, int n_ctx, const or_rope_params* p) {
    const int rot = p->rot_dim > 0 && p->rot_dim < p->head_dim ? p->rot_dim : p->head_dim;
    const int half = rot / 2;
    const int yarn = p->yarn_factor > 0.0f && p->yarn_orig_ctx > 0;
    float corr_low = 0, corr_high = 0, mscale = 1.0f;
    if (yarn) {
        corr_low = floorf(yarn_corr_dim(rot, p->yarn_orig_ctx, p->yarn_beta_fast, p->freq_base));
        corr_high = ceilf(yarn_corr_dim(rot, p->yarn_orig_ctx, p->yarn_beta_slow, p->freq_base));
        if (corr_low < 0.0f) corr_low = 0.0f;
        if (corr_high > (float)(rot - 1)) corr_high = (float)(rot - 1);
        mscale = p->yarn_attn_factor * (1.0f + 0.1f * logf(p->yarn_factor));
    }
    double* inv = (double*)malloc(sizeof(double) * (size_t)(half > 0 ? half : 1));
    for (int i = 0; i < half; ++i) inv[i] = pow((double)p->freq_base, -2.0 * (double)i / (double)rot);
    for (int pos = 0; pos < n_ctx; ++pos) {
        float* c = cs + (size_t)pos * half;
        float* s = sn + (size_t)pos * half;
        for (int i = 0; i < half; ++i) {
            double te = (double)pos * inv[i];
            if (p->freq_factors) {
                const float ff = p->freq_factors[i];
                te /= (ff != 0.0f ? ff : 1.0f);
            }
            double theta;
            float m = p->mscale;
            if (yarn) {
                const double ti = te / p->yarn_factor;
                const float ramp = yarn_ramp(corr_low, corr_high, 2 * i);
                theta = ti * (1.0 - ramp) + te * ramp;
                m *= mscale;
            } else {
                theta = te * p->freq_scale;
            }
            c[i] = (float)cos(theta) * m;
            s[i] = (float)sin(theta) * m;
        }
    }
    free(inv);
}

/* ops.cpp:126-156 */
void or_rope_apply(float* q, float* k, int n_head, int n_head_kv, int D, int rot,
                   int neox, const float* c, const float* s) {
    const int half = rot / 2;
    for (int pass = 0; pass < 2; ++pass) {
        float* vec = pass == 0 ? q : k;
        const int nh = pass == 0 ? n_head : n_head_kv;
        if (!vec) continue;
        for (int h = 0; h < nh; ++h) {
            float* v = vec + (size_t)h * D;
            for (int i = 0; i < half; ++i) {
                const int a = neox ? i : 2 * i, b = neox ? i + half : 2 * i + 1;
                const float x0 = v[a], x1 = v[b];
                v[a] = x0 * c[i] - x1 * s[i];
                v[b] = x0 * s[i] + x1 * c[i];
            }
        }
    }
}

/* ops.cpp:303-356: per (token, head) scores over j <= pos, softmax, P.V. */
void or_attention(const float* q, const float* kc, const float* vc, int H, int HKV,
                  int D, int pos0, int n_tok, float* out, float scale, float softcap,
                  int window) {
    const int group = H / HKV, kvs = HKV * D, E = H * D;
    float* scores = (float*)malloc(sizeof(float) * (size_t)(pos0 + n_tok + 1));
    for (int t = 0; t < n_tok; ++t) {
        const int pos = pos0 + t;
        for (int h = 0; h < H; ++h) {
            const int kvh = h / group;
            const float* qh = q + (size_t)t * E + (size_t)h * D;
            float* oh = out + (size_t)t * E + (size_t)h * D;
            int t0 = 0;
            if (window > 0 && pos - window + 1 > 0) t0 = pos - window + 1;
            float mx = -INFINITY;
            for (int j = t0; j <= pos; ++j) {
                const float* kt = kc + (size_t)j * kvs + (size_t)kvh * D;
                double dd = 0.0;
                for (int d = 0; d < D; ++d) dd += (double)qh[d] * kt[d];
                float sc = (float)dd * scale;
                if (softcap > 0.0f) sc = softcap * tanhf(sc / softcap);
                scores[j] = sc;
                if (sc > mx) mx = sc;
            }
            double sum = 0.0;
            for (int j = t0; j <= pos; ++j) { scores[j] = expf(scores[j] - mx); sum += scores[j]; }
            const double inv = sum > 0.0 ? 1.0 / sum : 0.0;
            for (int d = 0; d < D; ++d) {
                double o = 0.0;
                for (int j = t0; j <= pos; ++j) o += (double)scores[j] * inv * vc[(size_t)j * kvs + (size_t)kvh * D + d];
                oh[d] = (float)o;
            }
        }
    }
    free(scores);
}

int or_argmax(const float* v, int n) {
    int best = 0;
    float bv = -INFINITY;
    for (int i = 0; i < n; ++i) if (v[i] > bv) { bv = v[i]; best = i; }
    return best;
}

/* ================================================================ GGUF reader */

typedef struct {
    char name[96];
    int type;
    uint64_t ne[4];
    int n_dims;
    uint64_t offset;
    const uint8_t* data;
} or_tensor;

typedef struct {
    char key[96];
    int vtype;            /* gguf value type id */
    uint64_t u; int64_t i; double f; int b;
    char s[96];
    uint64_t arr_count;
} or_kv;

typedef struct {
    const uint8_t* map;
    size_t size;
    or_tensor* tensors; int n_tensors;
    or_kv* kvs; int n_kv;
} or_gguf;

typedef struct { const uint8_t* p; size_t n, off; int ok; } rd;
static int rd_need(rd* r, size_t k) { if (!r->ok || k > r->n || r->off > r->n - k) { r->ok = 0; return 0; } return 1; }
static uint64_t rd_uint(rd* r, int bytes) {
    uint64_t v = 0;
    if (!rd_need(r, (size_t)bytes)) return 0;
    memcpy(&v, r->p + r->off, (size_t)bytes);
    r->off += (size_t)bytes;
    return v;
}
static void rd_str(rd* r, char* out, size_t cap) {
    const uint64_t len = rd_uint(r, 8);
    if (!rd_need(r, (size_t)len)) return;
    if (out && cap) {
        const size_t k = len < cap - 1 ? (size_t)len : cap - 1;
        memcpy(out, r->p + r->off, k);
        out[k] = 0;
    }
    r->off += (size_t)len;
}
static int vt_size(uint32_t t) {
    switch (t) { case 0: case 1: case 7: return 1; case 2: case 3: return 2;
                 case 4: case 5: case 6: return 4; case 10: case 11: case 12: return 8; default: return 0; }
}
/* gguf.cpp:86-170: one metadata value (arrays skipped, count kept). */
static int rd_value(rd* r, uint32_t t, or_kv* kv) {
    if (kv) kv->vtype = (int)t;
    switch (t) {
        case 0: case 2: case 4: case 10: { const uint64_t v = rd_uint(r, vt_size(t)); if (kv) { kv->u = v; kv->i = (int64_t)v; kv->f = (double)v; } break; }
        case 1: { const int8_t v = (int8_t)rd_uint(r, 1); if (kv) { kv->i = v; kv->u = (uint64_t)v; kv->f = v; } break; }
        case 3: { const int16_t v = (int16_t)rd_uint(r, 2); if (kv) { kv->i = v; kv->u = (uint64_t)v; kv->f = v; } break; }
        case 5: { const int32_t v = (int32_t)rd_uint(r, 4); if (kv) { kv->i = v; kv->u = (uint64_t)(int64_t)v; kv->f = v; } break; }
        case 11: { const int64_t v = (int64_t)rd_uint(r, 8); if (kv) { kv->i = v; kv->u = (uint64_t)v; kv->f = (double)v; } break; }
        case 6: { const uint32_t b = (uint32_t)rd_uint(r, 4); float f; memcpy(&f, &b, 4); if (kv) { kv->f = f; kv->i = (int64_t)f; kv->u = (uint64_t)f; } break; }
        case 12: { const uint64_t b = rd_uint(r, 8); double f; memcpy(&f, &b, 8); if (kv) { kv->f = f; kv->i = (int64_t)f; kv->u = (uint64_t)f; } break; }
        case 7: { const int v = (int)rd_uint(r, 1); if (kv) { kv->b = v != 0; kv->u = (uint64_t)v; kv->i = v; } break; }
        case 8: rd_str(r, kv ? kv->s : NULL, kv ? sizeof(kv->s) : 0); break;
        case 9: {
            const uint32_t et = (uint32_t)rd_uint(r, 4);
            const uint64_t cnt = rd_uint(r, 8);
            if (kv) kv->arr_count = cnt;
            if (et == 8) { for (uint64_t i = 0; i < cnt && r->ok; ++i) rd_str(r, NULL, 0); }
            else if (vt_size(et)) { if (!rd_need(r, (size_t)(cnt * (uint64_t)vt_size(et)))) return 0; r->off += (size_t)(cnt * (uint64_t)vt_size(et)); }
            else { for (uint64_t i = 0; i < cnt && r->ok; ++i) if (!rd_value(r, et, NULL)) return 0; }
            break;
        }
        default: return 0;
    }
    return r->ok;
}

/* gguf.cpp:336-421: header, metadata, tensor directory, aligned data section. */
static int gguf_open(const char* path, or_gguf* g, char* err, int cap) {
    memset(g, 0, sizeof(*g));
    const int fd = open(path, O_RDONLY);
    if (fd < 0) { snprintf(err, (size_t)cap, "cannot open %s", path); return 0; }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 0) { close(fd); snprintf(err, (size_t)cap, "cannot size"); return 0; }
    void* base = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (base == MAP_FAILED) { snprintf(err, (size_t)cap, "cannot map"); return 0; }
    g->map = (const uint8_t*)base;
    g->size = (size_t)st.st_size;
    rd r = {g->map, g->size, 0, 1};
    if (rd_uint(&r, 4) != 0x46554747u) { snprintf(err, (size_t)cap, "not a GGUF file"); return 0; }
    const uint32_t ver = (uint32_t)rd_uint(&r, 4);
    if (ver < 2 || ver > 3) { snprintf(err, (size_t)cap, "unsupported GGUF version"); return 0; }
    const uint64_t nt = rd_uint(&r, 8), nkv = rd_uint(&r, 8);
    if (!r.ok || nt > (1u << 20) || nkv > (1u << 20)) { snprintf(err, (size_t)cap, "bad header"); return 0; }
    g->kvs = (or_kv*)calloc((size_t)nkv + 1, sizeof(or_kv));
    g->n_kv = (int)nkv;
    uint64_t align = 32;
    for (uint64_t i = 0; i < nkv; ++i) {
        rd_str(&r, g->kvs[i].key, sizeof(g->kvs[i].key));
        const uint32_t t = (uint32_t)rd_uint(&r, 4);
        if (!rd_value(&r, t, &g->kvs[i])) { snprintf(err, (size_t)cap, "bad metadata value for %s", g->kvs[i].key); return 0; }
        if (!strcmp(g->kvs[i].key, "general.alignment") && g->kvs[i].u >= 1) align = g->kvs[i].u;
    }
    g->tensors = (or_tensor*)calloc((size_t)nt + 1, sizeof(or_tensor));
    g->n_tensors = (int)nt;
    for (uint64_t i = 0; i < nt; ++i) {
        or_tensor* t = &g->tensors[i];
        rd_str(&r, t->name, sizeof(t->name));
        t->n_dims = (int)rd_uint(&r, 4);
        if (t->n_dims < 1 || t->n_dims > 4) { snprintf(err, (size_t)cap, "bad tensor rank"); return 0; }
        for (int d = 0; d < 4; ++d) t->ne[d] = 1;
        for (int d = 0; d < t->n_dims; ++d) t->ne[d] = rd_uint(&r, 8);
        t->type = (int)rd_uint(&r, 4);
        t->offset = rd_uint(&r, 8);
    }
    if (!r.ok) { snprintf(err, (size_t)cap, "truncated tensor table"); return 0; }
    const uint64_t data_off = (r.off + align - 1) / align * align;
    for (int i = 0; i < g->n_tensors; ++i) {
        or_tensor* t = &g->tensors[i];
        uint64_t rows = 1;
        for (int d = 1; d < 4; ++d) rows *= t->ne[d];
        const uint64_t nb = or_row_bytes(t->type, t->ne[0]) * rows;
        if (data_off + t->offset + nb > g->size) { snprintf(err, (size_t)cap, "tensor %s past end of file", t->name); return 0; }
        t->data = g->map + data_off + t->offset;
    }
    return 1;
}

static const or_kv* gguf_kv(const or_gguf* g, const char* key) {
    for (int i = 0; i < g->n_kv; ++i) if (!strcmp(g->kvs[i].key, key)) return &g->kvs[i];
    return NULL;
}
static const or_tensor* gguf_tensor(const or_gguf* g, const char* name) {
    for (int i = 0; i < g->n_tensors; ++i) if (!strcmp(g->tensors[i].name, name)) return &g->tensors[i];
    return NULL;
}

/* ===================================================================== model */

typedef struct {
    const or_tensor *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    const or_tensor *gate_inp, *gate_exps, *up_exps, *down_exps;
    float *attn_norm, *ffn_norm, *bq, *bk, *bv, *q_norm, *k_norm;
    /* row views of fused tensors (phi3 attn_qkv, gate|up ffn_up): rows of
     * one output are independent, so a view's product is the fused one's */
    or_tensor vq, vk, vv, vg, vu;
    float *bo, *bqkv;                      /* attn_output.bias, attn_qkv.bias */
    float *post_attn_norm, *post_ffn_norm; /* gemma2 */
    const or_tensor *sh_gate, *sh_up, *sh_down, *sh_gate_inp;   /* qwen2moe shared expert */
} or_layer;

struct or_model {
    or_gguf g;
    or_model_info c;
    int kv_f16;
    const or_tensor *embd, *out_w;
    float* out_norm;
    or_layer* L;
    float *rope_cos, *rope_sin, *rope_freqs;
    float *k_cache, *v_cache;   /* [layer][n_ctx][kv_dim] */
    int kv_len;
    float* last_x;
    /* gemma2 (model.cpp:488-496) and MoE options */
    int gemma2, gelu, sliding_window, expert_weights_norm;
    float embd_scale, attn_softcap, final_softcap;
};

static float* load_vec(const or_tensor* t) {
    if (!t) return NULL;
    uint64_t n = 1;
    for (int d = 0; d < 4; ++d) n *= t->ne[d];
    float* v = (float*)malloc(sizeof(float) * (size_t)n);
    if (!or_dequant_row(t->type, t->data, v, n)) { free(v); return NULL; }
    return v;
}

static uint64_t kv_u(const or_gguf* g, const char* arch, const char* k, uint64_t def) {
    char key[160];
    snprintf(key, sizeof(key), "%s.%s", arch, k);
    const or_kv* v = gguf_kv(g, key);
    return v ? v->u : def;
}
static double kv_f(const or_gguf* g, const char* arch, const char* k, double def) {
    char key[160];
    snprintf(key, sizeof(key), "%s.%s", arch, k);
    const or_kv* v = gguf_kv(g, key);
    return v ? v->f : def;
}

/* model.cpp:393-645 (llama / qwen2 / qwen3 / their MoE variants with the
 * qwen2moe shared expert, gemma2, phi3). */
or_model* or_model_load(const char* path, int n_ctx, int kv_f16, char* err, int cap) {
    or_model* m = (or_model*)calloc(1, sizeof(or_model));
    if (!gguf_open(path, &m->g, err, cap)) { or_model_free(m); return NULL; }
    const or_gguf* g = &m->g;
    const or_kv* a = gguf_kv(g, "general.architecture");
    const char* arch = a ? a->s : "llama";
    or_model_info* c = &m->c;
    c->n_layers = (int)kv_u(g, arch, "block_count", 0);
    c->n_embd = (int)kv_u(g, arch, "embedding_length", 0);
    c->n_ff = (int)kv_u(g, arch, "feed_forward_length", 0);
    c->n_head = (int)kv_u(g, arch, "attention.head_count", 0);
    c->n_head_kv = (int)kv_u(g, arch, "attention.head_count_kv", (uint64_t)c->n_head);
    c->eps = (float)kv_f(g, arch, "attention.layer_norm_rms_epsilon", 1e-5);
    c->freq_base = (float)kv_f(g, arch, "rope.freq_base", 10000.0);
    const or_kv* b = gguf_kv(g, "tokenizer.ggml.bos_token_id");
    const or_kv* e = gguf_kv(g, "tokenizer.ggml.eos_token_id");
    c->bos = b ? (int)b->i : 1;
    c->eos = e ? (int)e->i : 2;
    const int ctx_train = (int)kv_u(g, arch, "context_length", 4096);
    c->vocab = (int)kv_u(g, arch, "vocab_size", 0);
    if (c->vocab <= 0) { const or_kv* tk = gguf_kv(g, "tokenizer.ggml.tokens"); if (tk) c->vocab = (int)tk->arr_count; }
    m->embd = gguf_tensor(g, "token_embd.weight");
    if (!m->embd) { snprintf(err, (size_t)cap, "missing token_embd.weight"); or_model_free(m); return NULL; }
    if (c->vocab <= 0) c->vocab = (int)m->embd->ne[1];
    c->head_dim = (int)kv_u(g, arch, "attention.key_length", 0);
    if (c->head_dim <= 0) c->head_dim = c->n_embd / c->n_head;
    c->n_experts = (int)kv_u(g, arch, "expert_count", 0);
    c->n_experts_per_tok = (int)kv_u(g, arch, "expert_used_count", 0);
    c->n_ff_exp = (int)kv_u(g, arch, "expert_feed_forward_length", (uint64_t)c->n_ff);
    if (c->n_experts > 0 && c->n_experts_per_tok <= 0) c->n_experts_per_tok = 2;
    if (c->n_experts_per_tok > c->n_experts) c->n_experts_per_tok = c->n_experts;
    c->rot_dim = (int)kv_u(g, arch, "rope.dimension_count", (uint64_t)c->head_dim);
    c->neox = !strcmp(arch, "qwen2") || !strcmp(arch, "qwen3") || !strcmp(arch, "qwen2moe") || !strcmp(arch, "qwen3moe") ||
              !strcmp(arch, "gemma2") || !strcmp(arch, "phi3");
    m->expert_weights_norm = (int)kv_u(g, arch, "expert_weights_norm", strcmp(arch, "qwen2moe") ? 1 : 0);
    m->embd_scale = 1.0f;
    if (!strcmp(arch, "gemma2")) {   /* model.cpp:488-496 */
        m->gemma2 = 1;
        m->gelu = 1;
        m->embd_scale = sqrtf((float)c->n_embd);
        m->attn_softcap = (float)kv_f(g, arch, "attn_logit_softcapping", 50.0);
        m->final_softcap = (float)kv_f(g, arch, "final_logit_softcapping", 30.0);
        m->sliding_window = (int)kv_u(g, arch, "attention.sliding_window", 4096);
    }
    c->n_ctx = n_ctx > 0 ? (n_ctx < ctx_train ? n_ctx : ctx_train) : (ctx_train < 4096 ? ctx_train : 4096);

    or_rope_params rp;
    memset(&rp, 0, sizeof(rp));
    rp.head_dim = c->head_dim;
    rp.rot_dim = c->rot_dim;
    rp.neox = c->neox;
    rp.freq_base = c->freq_base;
    rp.freq_scale = 1.0f;
    rp.mscale = 1.0f;
    rp.yarn_attn_factor = 1.0f;
    rp.yarn_beta_fast = 32.0f;
    rp.yarn_beta_slow = 1.0f;
    /* longrope (phi3, model.cpp:522-530): the long factor set beyond the
     * original context, else the short one; the attention factor scales the
     * rotation. Otherwise Llama-3 style rope_freqs (model.cpp:532-543). */
    const or_tensor* rf = NULL;
    {
        char key[160];
        snprintf(key, sizeof(key), "%s.rope.scaling.type", arch);
        const or_kv* st = gguf_kv(g, key);
        if (st && !strcmp(st->s, "longrope")) {
            const int orig = (int)kv_u(g, arch, "rope.scaling.original_context_length", 0);
            rf = (orig > 0 && c->n_ctx > orig) ? gguf_tensor(g, "rope_factors_long.weight")
                                               : gguf_tensor(g, "rope_factors_short.weight");
            if (!rf) rf = gguf_tensor(g, "rope_factors_short.weight");
            rp.mscale = (float)kv_f(g, arch, "rope.scaling.attn_factor", 1.0);
        } else {
            rf = gguf_tensor(g, "rope_freqs.weight");
        }
    }
    if (rf) { m->rope_freqs = load_vec(rf); rp.freq_factors = m->rope_freqs; }
    const int rot = c->rot_dim > 0 && c->rot_dim < c->head_dim ? c->rot_dim : c->head_dim;
    c->rot_dim = rot;
    m->rope_cos = (float*)malloc(sizeof(float) * (size_t)c->n_ctx * (size_t)(rot / 2));
    m->rope_sin = (float*)malloc(sizeof(float) * (size_t)c->n_ctx * (size_t)(rot / 2));
    or_rope_build(m->rope_cos, m->rope_sin, c->n_ctx, &rp);

    m->out_norm = load_vec(gguf_tensor(g, "output_norm.weight"));
    if (m->gemma2 && m->out_norm) for (int i = 0; i < c->n_embd; ++i) m->out_norm[i] += 1.0f;
    m->out_w = gguf_tensor(g, "output.weight");
    if (!m->out_w) { m->out_w = m->embd; c->tied_output = 1; }
    if (!m->out_norm) { snprintf(err, (size_t)cap, "missing output_norm.weight"); or_model_free(m); return NULL; }

    m->L = (or_layer*)calloc((size_t)c->n_layers, sizeof(or_layer));
    for (int i = 0; i < c->n_layers; ++i) {
        char nm[128];
        or_layer* L = &m->L[i];
#define T(field, suffix) do { snprintf(nm, sizeof(nm), "blk.%d." suffix, i); L->field = gguf_tensor(g, nm); } while (0)
#define V(field, suffix) do { snprintf(nm, sizeof(nm), "blk.%d." suffix, i); L->field = load_vec(gguf_tensor(g, nm)); } while (0)
        T(wq, "attn_q.weight"); T(wk, "attn_k.weight"); T(wv, "attn_v.weight"); T(wo, "attn_output.weight");
        T(wg, "ffn_gate.weight"); T(wu, "ffn_up.weight"); T(wd, "ffn_down.weight");
        T(gate_inp, "ffn_gate_inp.weight"); T(gate_exps, "ffn_gate_exps.weight");
        T(up_exps, "ffn_up_exps.weight"); T(down_exps, "ffn_down_exps.weight");
        V(attn_norm, "attn_norm.weight"); V(ffn_norm, "ffn_norm.weight");
        V(bq, "attn_q.bias"); V(bk, "attn_k.bias"); V(bv, "attn_v.bias");
        V(q_norm, "attn_q_norm.weight"); V(k_norm, "attn_k_norm.weight");
        V(bo, "attn_output.bias"); V(bqkv, "attn_qkv.bias");
        V(post_attn_norm, "post_attention_norm.weight"); V(post_ffn_norm, "post_ffw_norm.weight");
        T(sh_gate, "ffn_gate_shexp.weight"); T(sh_up, "ffn_up_shexp.weight"); T(sh_down, "ffn_down_shexp.weight");
        T(sh_gate_inp, "ffn_gate_inp_shexp.weight");
        if (m->gemma2) {   /* norm weights stored as w - 1 (model.cpp:241-245) */
            float* nv[4] = {L->attn_norm, L->ffn_norm, L->post_attn_norm, L->post_ffn_norm};
            for (int j = 0; j < 4; ++j) if (nv[j]) for (int e2 = 0; e2 < c->n_embd; ++e2) nv[j][e2] += 1.0f;
        }
        {
            const or_tensor* f = NULL;
            T(wq, "attn_qkv.weight");   /* phi3 fused q|k|v (model.cpp:253, 1665-1674) */
            f = L->wq;
            if (f) {
                const int Qd = c->n_head * c->head_dim, KVd = c->n_head_kv * c->head_dim;
                const uint64_t rb = or_row_bytes(f->type, f->ne[0]);
                L->vq = *f; L->vq.ne[1] = (uint64_t)Qd;
                L->vk = *f; L->vk.ne[1] = (uint64_t)KVd; L->vk.data = f->data + rb * (uint64_t)Qd;
                L->vv = *f; L->vv.ne[1] = (uint64_t)KVd; L->vv.data = f->data + rb * (uint64_t)(Qd + KVd);
                L->wq = &L->vq; L->wk = &L->vk; L->wv = &L->vv;
                if (L->bqkv && !L->bq) {
                    L->bq = (float*)malloc(sizeof(float) * (size_t)Qd);
                    L->bk = (float*)malloc(sizeof(float) * (size_t)KVd);
                    L->bv = (float*)malloc(sizeof(float) * (size_t)KVd);
                    memcpy(L->bq, L->bqkv, sizeof(float) * (size_t)Qd);
                    memcpy(L->bk, L->bqkv + Qd, sizeof(float) * (size_t)KVd);
                    memcpy(L->bv, L->bqkv + Qd + KVd, sizeof(float) * (size_t)KVd);
                }
            } else {
                T(wq, "attn_q.weight");
            }
        }
        if (!L->wg && L->wu && c->n_experts == 0 && L->wu->ne[1] == 2 * (uint64_t)c->n_ff) {
            /* phi3 fused gate|up: ffn_up holds 2 n_ff rows, gate first (model.cpp:1481-1489) */
            const or_tensor* f = L->wu;
            const uint64_t rb = or_row_bytes(f->type, f->ne[0]);
            L->vg = *f; L->vg.ne[1] = (uint64_t)c->n_ff;
            L->vu = *f; L->vu.ne[1] = (uint64_t)c->n_ff; L->vu.data = f->data + rb * (uint64_t)c->n_ff;
            L->wg = &L->vg; L->wu = &L->vu;
        }
#undef T
#undef V
        if (!L->attn_norm || !L->ffn_norm || !L->wq || !L->wk || !L->wv || !L->wo) {
            snprintf(err, (size_t)cap, "missing tensors in layer %d", i);
            or_model_free(m);
            return NULL;
        }
    }
    const size_t kvn = (size_t)c->n_layers * (size_t)c->n_ctx * (size_t)(c->n_head_kv * c->head_dim);
    m->k_cache = (float*)calloc(kvn, sizeof(float));
    m->v_cache = (float*)calloc(kvn, sizeof(float));
    m->last_x = (float*)calloc((size_t)c->n_embd, sizeof(float));
    m->kv_f16 = kv_f16;
    if (!m->k_cache || !m->v_cache) { snprintf(err, (size_t)cap, "out of memory for KV"); or_model_free(m); return NULL; }
    return m;
}

void or_model_free(or_model* m) {
    if (!m) return;
    if (m->L) {
        for (int i = 0; i < m->c.n_layers; ++i) {
            or_layer* L = &m->L[i];
            free(L->attn_norm); free(L->ffn_norm); free(L->bq); free(L->bk); free(L->bv);
            free(L->q_norm); free(L->k_norm);
            free(L->bo); free(L->bqkv); free(L->post_attn_norm); free(L->post_ffn_norm);
        }
        free(m->L);
    }
    free(m->out_norm); free(m->rope_cos); free(m->rope_sin); free(m->rope_freqs);
    free(m->k_cache); free(m->v_cache); free(m->last_x);
    free(m->g.tensors); free(m->g.kvs);
    if (m->g.map) munmap((void*)m->g.map, m->g.size);
    free(m);
}

int or_model_info_of(const or_model* m, or_model_info* out) { if (!m || !out) return -1; *out = m->c; return 0; }
void or_model_set_kv_len(or_model* m, int n) { m->kv_len = n; }
int or_model_kv_len(const or_model* m) { return m->kv_len; }
int or_model_last_hidden(const or_model* m, float* out, int n) {
    if (n > m->c.n_embd) n = m->c.n_embd;
    memcpy(out, m->last_x, sizeof(float) * (size_t)n);
    return n;
}

static void add_bias(float* y, int n_tok, int n, const float* b) {
    if (!b) return;
    for (int t = 0; t < n_tok; ++t) for (int i = 0; i < n; ++i) y[(size_t)t * n + i] += b[i];
}

/* Byte offset of expert e in a 3-D [n_in][n_out][n_expert] tensor (model.cpp:66-69). */
static const uint8_t* expert_ptr(const or_tensor* t, int e) {
    return t->data + or_row_bytes(t->type, t->ne[0]) * t->ne[1] * (uint64_t)e;
}

/* model.cpp:1474-1515 (separate gate / up). out[n_tok][n_in]. */
static void ffn_block_acts(int tg, const void* wg, int tu, const void* wu, int td, const void* wd,
                           const float* x, int n_tok, int n_in, int n_ff, float* out, const void* xk, const void* x32,
                           const void* hk, const void* h32, int gelu) {
    float* g = (float*)malloc(sizeof(float) * (size_t)n_tok * (size_t)n_ff);
    float* u = (float*)malloc(sizeof(float) * (size_t)n_tok * (size_t)n_ff);
    matmul_acts(tg, wg, x, xk, x32, n_tok, n_in, n_ff, g);
    matmul_acts(tu, wu, x, xk, x32, n_tok, n_in, n_ff, u);
    for (int t = 0; t < n_tok; ++t) {
        float* gr = g + (size_t)t * n_ff;
        if (gelu) or_gelu_inplace(gr, n_ff); else or_silu_inplace(gr, n_ff);
        for (int i = 0; i < n_ff; ++i) gr[i] *= u[(size_t)t * n_ff + i];
    }
    matmul_acts(td, wd, g, hk, h32, n_tok, n_ff, n_in, out);
    free(g);
    free(u);
}

/* model.cpp:1523-1580: softmax router, top-k by descending probability
 * (partial_sort), renormalise when expert_weights_norm, then every used
 * expert in ascending expert order runs its FFN and is scatter-added with its
 * weight, the same order of float additions as the reference. */
static void moe_ffn(or_model* m, const or_layer* L, const float* xb, int n_tok, float* out, const or_layer_acts* ov) {
    const or_model_info* c = &m->c;
    const int E = c->n_embd, NE = c->n_experts, K = c->n_experts_per_tok;
    float* r = (float*)malloc(sizeof(float) * (size_t)n_tok * (size_t)NE);
    or_matmul(L->gate_inp->type, L->gate_inp->data, xb, n_tok, E, NE, r);
    memset(out, 0, sizeof(float) * (size_t)n_tok * (size_t)E);
    float* tmp = (float*)malloc(sizeof(float) * (size_t)E);
    int* sel = (int*)malloc(sizeof(int) * (size_t)n_tok * (size_t)K);
    float* wsel = (float*)malloc(sizeof(float) * (size_t)n_tok * (size_t)K);
    for (int t = 0; t < n_tok; ++t) {
        float* lg = r + (size_t)t * NE;
        or_softmax_inplace(lg, NE);
        int used[256] = {0};
        float sum = 0.0f;
        for (int k = 0; k < K; ++k) {
            int best = -1;
            for (int e = 0; e < NE; ++e) if (!used[e] && (best < 0 || lg[e] > lg[best])) best = e;
            used[best] = 1;
            sel[t * K + k] = best;
            wsel[t * K + k] = lg[best];
            sum += lg[best];
        }
        if (m->expert_weights_norm && sum > 0.0f) for (int k = 0; k < K; ++k) wsel[t * K + k] /= sum;
    }
    for (int ex = 0; ex < NE; ++ex) {
        for (int t = 0; t < n_tok; ++t) {
            for (int k = 0; k < K; ++k) {
                if (sel[t * K + k] != ex) continue;
                const int F = c->n_ff_exp, r = t * K + k;
                ffn_block_acts(L->gate_exps->type, expert_ptr(L->gate_exps, ex),
                               L->up_exps->type, expert_ptr(L->up_exps, ex),
                               L->down_exps->type, expert_ptr(L->down_exps, ex),
                               xb + (size_t)t * E, 1, E, F, tmp,
                               ov && ov->qk[2] ? (const uint8_t*)ov->qk[2] + (size_t)t * (E / 256) * sizeof(or_q8actk) : NULL,
                               ov && ov->q32[2] ? (const uint8_t*)ov->q32[2] + (size_t)t * (E / 32) * sizeof(or_q8act) : NULL,
                               ov && ov->qk[3] ? (const uint8_t*)ov->qk[3] + (size_t)r * (F / 256) * sizeof(or_q8actk) : NULL,
                               ov && ov->q32[3] ? (const uint8_t*)ov->q32[3] + (size_t)r * (F / 32) * sizeof(or_q8act) : NULL, 0);
                const float w = wsel[t * K + k];
                for (int i = 0; i < E; ++i) out[(size_t)t * E + i] += w * tmp[i];
            }
        }
    }
    /* the shared expert (qwen2moe, model.cpp:1582-1599): every token, scaled
     * by the sigmoid of its one-row gate when the layer has one */
    if (L->sh_gate && L->sh_up && L->sh_down) {
        const int FS = (int)L->sh_gate->ne[1];
        float* d = (float*)malloc(sizeof(float) * (size_t)n_tok * (size_t)E);
        ffn_block_acts(L->sh_gate->type, L->sh_gate->data, L->sh_up->type, L->sh_up->data, L->sh_down->type,
                       L->sh_down->data, xb, n_tok, E, FS, d, NULL, NULL, NULL, NULL, 0);
        float* gate = (float*)malloc(sizeof(float) * (size_t)n_tok);
        for (int t = 0; t < n_tok; ++t) gate[t] = 1.0f;
        if (L->sh_gate_inp) {
            or_matmul(L->sh_gate_inp->type, L->sh_gate_inp->data, xb, n_tok, E, 1, gate);
            for (int t = 0; t < n_tok; ++t) gate[t] = 1.0f / (1.0f + expf(-gate[t]));
        }
        for (int t = 0; t < n_tok; ++t)
            for (int i = 0; i < E; ++i) out[(size_t)t * E + i] += gate[t] * d[(size_t)t * E + i];
        free(gate);
        free(d);
    }
    free(sel);
    free(wsel);
    free(tmp);
    free(r);
}

/* One iteration of the layer loop of model.cpp:1654-1785: x [n_tok][E] is
 * updated in place; layer li's K/V rows are stored at pos0..pos0+n_tok-1.
 * Work buffers: xb, pr [n_tok][E]; q, at [n_tok][H*D]; k, v [n_tok][HKV*D]. */
static void layer_forward(or_model* m, int li, float* x, int n_tok, int pos0, float* xb, float* q, float* k,
                          float* v, float* at, float* pr, const or_layer_acts* ov) {
    const void* const no[4] = {NULL, NULL, NULL, NULL};
    const void* const* ak = ov ? ov->qk : no;
    const void* const* a32 = ov ? ov->q32 : no;
    const or_model_info* c = &m->c;
    const int E = c->n_embd, H = c->n_head, HKV = c->n_head_kv, D = c->head_dim;
    const int Q = H * D, KV = HKV * D;
    const float scale = 1.0f / sqrtf((float)D);
    const int half = c->rot_dim / 2;
    {
        const or_layer* L = &m->L[li];
        for (int t = 0; t < n_tok; ++t) or_rmsnorm(xb + (size_t)t * E, x + (size_t)t * E, L->attn_norm, E, c->eps);
        matmul_acts(L->wq->type, L->wq->data, xb, ak[0], a32[0], n_tok, E, Q, q);
        matmul_acts(L->wk->type, L->wk->data, xb, ak[0], a32[0], n_tok, E, KV, k);
        matmul_acts(L->wv->type, L->wv->data, xb, ak[0], a32[0], n_tok, E, KV, v);
        add_bias(q, n_tok, Q, L->bq);
        add_bias(k, n_tok, KV, L->bk);
        add_bias(v, n_tok, KV, L->bv);
        if (L->q_norm && L->k_norm) {
            for (int t = 0; t < n_tok; ++t) {
                for (int h = 0; h < H; ++h) or_rmsnorm(q + (size_t)t * Q + h * D, q + (size_t)t * Q + h * D, L->q_norm, D, c->eps);
                for (int h = 0; h < HKV; ++h) or_rmsnorm(k + (size_t)t * KV + h * D, k + (size_t)t * KV + h * D, L->k_norm, D, c->eps);
            }
        }
        float* kc = m->k_cache + (size_t)li * c->n_ctx * KV;
        float* vc = m->v_cache + (size_t)li * c->n_ctx * KV;
        for (int t = 0; t < n_tok; ++t) {
            const int pos = pos0 + t;
            or_rope_apply(q + (size_t)t * Q, k + (size_t)t * KV, H, HKV, D, c->rot_dim, c->neox,
                          m->rope_cos + (size_t)pos * half, m->rope_sin + (size_t)pos * half);
            for (int i = 0; i < KV; ++i) {
                float kv_k = k[(size_t)t * KV + i], kv_v = v[(size_t)t * KV + i];
                if (m->kv_f16) {
                    kv_k = or_fp16_to_fp32(or_fp32_to_fp16(kv_k));
                    kv_v = or_fp16_to_fp32(or_fp32_to_fp16(kv_v));
                }
                kc[(size_t)pos * KV + i] = kv_k;
                vc[(size_t)pos * KV + i] = kv_v;
            }
        }
        /* gemma2: score soft cap, sliding window on the even layers (model.cpp:1735-1739) */
        const int window = (m->sliding_window > 0 && li % 2 == 0) ? m->sliding_window : 0;
        or_attention(q, kc, vc, H, HKV, D, pos0, n_tok, at, scale, m->attn_softcap, window);
        matmul_acts(L->wo->type, L->wo->data, at, ak[1], a32[1], n_tok, Q, E, pr);
        add_bias(pr, n_tok, E, L->bo);
        if (L->post_attn_norm)
            for (int t = 0; t < n_tok; ++t) or_rmsnorm(pr + (size_t)t * E, pr + (size_t)t * E, L->post_attn_norm, E, c->eps);
        for (size_t i = 0; i < (size_t)n_tok * E; ++i) x[i] += pr[i];
        for (int t = 0; t < n_tok; ++t) or_rmsnorm(xb + (size_t)t * E, x + (size_t)t * E, L->ffn_norm, E, c->eps);
        if (c->n_experts > 0) {
            moe_ffn(m, L, xb, n_tok, pr, ov);
        } else {
            ffn_block_acts(L->wg->type, L->wg->data, L->wu->type, L->wu->data, L->wd->type, L->wd->data,
                           xb, n_tok, E, c->n_ff, pr, ak[2], a32[2], ak[3], a32[3], m->gelu);
        }
        if (L->post_ffn_norm)
            for (int t = 0; t < n_tok; ++t) or_rmsnorm(pr + (size_t)t * E, pr + (size_t)t * E, L->post_ffn_norm, E, c->eps);
        for (size_t i = 0; i < (size_t)n_tok * E; ++i) x[i] += pr[i];
    }
}

/* model.cpp:1603-1811 */
int or_model_forward(or_model* m, const int32_t* tokens, int n_tok, int pos0,
                     float* logits, float* logits_all) {
    const or_model_info* c = &m->c;
    if (!tokens || n_tok <= 0 || pos0 < 0 || pos0 + n_tok > c->n_ctx) return 0;
    const int E = c->n_embd, H = c->n_head, HKV = c->n_head_kv, D = c->head_dim;
    const int Q = H * D, KV = HKV * D;
    float* x = (float*)malloc(sizeof(float) * (size_t)n_tok * E);
    float* xb = (float*)malloc(sizeof(float) * (size_t)n_tok * E);
    float* q = (float*)malloc(sizeof(float) * (size_t)n_tok * Q);
    float* k = (float*)malloc(sizeof(float) * (size_t)n_tok * KV);
    float* v = (float*)malloc(sizeof(float) * (size_t)n_tok * KV);
    float* at = (float*)malloc(sizeof(float) * (size_t)n_tok * Q);
    float* pr = (float*)malloc(sizeof(float) * (size_t)n_tok * E);
    const uint64_t erow = or_row_bytes(m->embd->type, (uint64_t)E);
    for (int t = 0; t < n_tok; ++t) {
        if (tokens[t] < 0 || tokens[t] >= c->vocab) return 0;
        or_dequant_row(m->embd->type, m->embd->data + (size_t)tokens[t] * erow, x + (size_t)t * E, (uint64_t)E);
        if (m->embd_scale != 1.0f)   /* gemma2 (model.cpp:1624-1627) */
            for (int i = 0; i < E; ++i) x[(size_t)t * E + i] *= m->embd_scale;
    }
    for (int li = 0; li < c->n_layers; ++li) layer_forward(m, li, x, n_tok, pos0, xb, q, k, v, at, pr, NULL);
    memcpy(m->last_x, x + (size_t)(n_tok - 1) * E, sizeof(float) * (size_t)E);
    const int rows = logits_all ? n_tok : 1;
    const int first = logits_all ? 0 : n_tok - 1;
    for (int t = 0; t < rows; ++t) or_rmsnorm(xb + (size_t)t * E, x + (size_t)(first + t) * E, m->out_norm, E, c->eps);
    float* out = logits_all ? logits_all : logits;
    or_matmul(m->out_w->type, m->out_w->data, xb, rows, E, c->vocab, out);
    if (m->final_softcap > 0.0f)   /* gemma2 (model.cpp:1802-1805) */
        for (size_t i = 0; i < (size_t)rows * c->vocab; ++i) out[i] = m->final_softcap * tanhf(out[i] / m->final_softcap);
    if (logits_all && logits) memcpy(logits, logits_all + (size_t)(n_tok - 1) * c->vocab, sizeof(float) * (size_t)c->vocab);
    m->kv_len = pos0 + n_tok;
    free(x); free(xb); free(q); free(k); free(v); free(at); free(pr);
    return 1;
}

int or_model_layer(or_model* m, int layer, const float* x_in, int n_tok, int pos0, float* x_out) {
    return or_model_layer_acts(m, layer, x_in, n_tok, pos0, NULL, x_out);
}

int or_model_layer_acts(or_model* m, int layer, const float* x_in, int n_tok, int pos0, const or_layer_acts* acts,
                        float* x_out) {
    if (!m) return 0;
    const or_model_info* c = &m->c;
    if (!x_in || !x_out || layer < 0 || layer >= c->n_layers || n_tok <= 0 || pos0 < 0 ||
        pos0 + n_tok > c->n_ctx)
        return 0;
    const int E = c->n_embd, Q = c->n_head * c->head_dim, KV = c->n_head_kv * c->head_dim;
    float* xb = (float*)malloc(sizeof(float) * (size_t)n_tok * E);
    float* q = (float*)malloc(sizeof(float) * (size_t)n_tok * Q);
    float* k = (float*)malloc(sizeof(float) * (size_t)n_tok * KV);
    float* v = (float*)malloc(sizeof(float) * (size_t)n_tok * KV);
    float* at = (float*)malloc(sizeof(float) * (size_t)n_tok * Q);
    float* pr = (float*)malloc(sizeof(float) * (size_t)n_tok * E);
    memcpy(x_out, x_in, sizeof(float) * (size_t)n_tok * E);
    layer_forward(m, layer, x_out, n_tok, pos0, xb, q, k, v, at, pr, acts);
    free(xb); free(q); free(k); free(v); free(at); free(pr);
    return 1;
}

const void* or_model_tensor(const or_model* m, const char* name, int* type, int64_t* ne0, int64_t* ne1,
                            int64_t* ne2) {
    const or_tensor* t = m && name ? gguf_tensor(&m->g, name) : NULL;
    if (!t) return NULL;
    if (type) *type = t->type;
    if (ne0) *ne0 = (int64_t)t->ne[0];
    if (ne1) *ne1 = (int64_t)t->ne[1];
    if (ne2) *ne2 = (int64_t)t->ne[2];
    return t->data;
}
