// gemm.cu — batched (prefill, T >= 16 tokens) quantised matrix products on
// the int8 tensor cores.
//
// Y[t][r] = W_r . x_t for Q4_K / Q6_K / Q8_0 rows (tile-major device layout)
// against the int8 activation planes (Q8ActK / Q8Act records, byte-exact
// with the reference's quantisers). The reference forms per block the
// integers (src/quant_x86.cpp:299-309, 346-382, 431-495)
//   Q4_K  sumi = sum_g sc_g sum_{32} q x,  mins = sum_g m_g bsums_g
//   Q6_K  sumi = sum_j sc_j sum_{16} (q6 - 32) x
//   Q8_0  s    = sum_{32} w x
// and here one mma.sync of K = 32 (Q4_K sub-block, Q8_0 block) or K = 16
// (Q6_K group) forms exactly one inner sum for a 16-row x 8-token fragment;
// the scales are applied to those int32 fragments, so every block's integers
// equal the reference's. Float steps per block are those of the GEMV
// kernels (q4k_term / scaled_term) and they are added in the GEMV kernels'
// order (a pairwise tree over the 8 blocks of each 2048-value group, then the
// groups in order; Q8_0: each eighth of a group summed in block order first),
// so a row's value does not depend on the number of tokens in the call.
//
// CTA tile BM (64, or 32 for small matrices) rows x BN tokens, warps of 16 FT
// rows x 8 JT tokens; BN = 64
// (warps of 32 x 16) for long prompts (compute-bound), 16 or 32 (warps of
// 16 x 8, 16 x 16) for batched decode and short prompts, which the weight
// stream bounds: narrower token tiles and a deeper pipeline. Each K step is one 256-value block (8 Q8_0 blocks): the CTA's
// 64 weight rows of that block and the BN tokens' 256 int8 activations are
// copied to shared memory with cp.async into an NS-stage ring. Nibbles /
// 6-bit codes are unpacked into A fragments in registers (Q4_K low nibbles of
// qs words are already four int8 in fragment order).
#include <algorithm>
#include <cstdint>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "layout.cuh"
#include "stream_common.cuh"
#include "unit_math.cuh"

namespace fb {

constexpr int kXStride = 272;   // bytes per token row of activations in shared memory (256 + pad)

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    const int n = valid ? 16 : 0;   // 0: the 16 bytes are zero-filled, nothing is read
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// D += A (16x32 s8, row) . B (32x8 s8, col)
__device__ __forceinline__ void mma_k32(int (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// D += A (16x16 s8, row) . B (16x8 s8, col)
__device__ __forceinline__ void mma_k16(int (&d)[4], const uint32_t (&a)[2], uint32_t b) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(b));
}

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

// Bytes per weight row of one K step in shared memory (row strides of 36, 60
// and 68 words put the 8 rows x 4 words of a fragment load in 32 banks).
template <int W>
struct Step;
template <>
struct Step<T_Q4_K> {
    static constexpr int wbytes = 144;   // one block
};
template <>
struct Step<T_Q6_K> {
    static constexpr int wbytes = 240;   // ql, qh, scales (208); the group's fp16 d table (16); pad: 60 words per row
                                         // keep fragment loads conflict-free
};
template <>
struct Step<T_Q8_0> {
    static constexpr int wbytes = 8 * 32 + 16;   // eight blocks' qs; then eight fp16 d
};


// Shared-memory stage of one K step: weights [BM][WB], activations
// [BN][272], per-token scales (dx, or 8 d32 for Q8_0) [BN][8] f32.
template <int W, int BM, int BN>
struct StageLayout {
    static constexpr int WB = Step<W>::wbytes;
    static constexpr int w_off = 0;
    static constexpr int x_off = BM * WB;
    static constexpr int d_off = x_off + BN * kXStride;
    static constexpr int bytes = d_off + BN * 8 * 4;
};

template <int W, int BM, int BN, int NS, int FT, int JT, bool SPLIT>
__global__ void __launch_bounds__(BM * BN / (4 * FT * JT)) k_gemm_q(GemvSeg g, ActQ a, int K, int T, int* err, int upc,
                                                                    float* part) {
    using L = StageLayout<W, BM, BN>;
    constexpr int WB = L::WB;
    // warps of 16 FT rows x 8 JT tokens: BM / (16 FT) along rows, BN / (8 JT) along tokens
    constexpr int kBM = BM, kBN = BN, WRN = BM / (16 * FT), kGemmThreads = 32 * WRN * (BN / (8 * JT));
    static_assert(WRN * 16 * FT == BM && (BN / (8 * JT)) * 8 * JT == BN, "warps tile the BM x BN tile");
    extern __shared__ __align__(128) uint8_t sm[];
    pdl_trigger();
    pdl_wait();
    const int row0 = blockIdx.x * kBM, t0 = blockIdx.y * kBN;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, tig = lane & 3;
    const int wr = warp % WRN, wc = warp / WRN;   // rows 16 FT wr .., tokens 8 JT wc ..
    // K split (SPLIT, compiled apart so the unsplit kernel keeps its
    // registers): this CTA takes the half-group units (4 blocks)
    // [z upc, (z + 1) upc) and writes each unit's tree value to
    // part[(unit * T + t) * rows + row] for k_gemm_unit_reduce
    constexpr bool split = SPLIT;
    const int sb0 = split ? 4 * (int)blockIdx.z * upc : 0;
    const int nsteps = split ? min(K / 256 - sb0, 4 * upc) : K / 256;
    const uint8_t* wend = g.w + g.w_bytes;

    // Issue the copies of step s into stage buffer b; returns this thread's
    // token scale for the step (K-quants: dk of token t0 + tid), stored by
    // the caller once the current step's arithmetic is done.
    auto issue = [&](int sl, uint8_t* b) -> float {
        const int s = sb0 + sl;   // block of the row
        constexpr int WCH = W == T_Q4_K ? 9 : (W == T_Q6_K ? 13 : 16);   // 16-byte chunks of codes per row
        constexpr int NCH = W == T_Q4_K ? WCH : WCH + 1;                 // + the scale-table chunk
        for (int i = tid; i < kBM * NCH; i += kGemmThreads) {
            const int r = i / NCH, c = i % NCH, row = row0 + r;
            const uint8_t* src = g.w;
            uint8_t* dst;
            bool ok = row < g.rows;
            if (c < WCH) {
                if (ok) src = g.w + block_offset_tm(W, K, row, W == T_Q8_0 ? 8 * s : s) + 16 * c;
                dst = b + L::w_off + r * WB + 16 * c;
            } else {   // Q6_K: the group's d table; Q8_0: the step's eight d
                if (ok) src = g.w + dscale_offset_tm(W, K, row, W == T_Q8_0 ? 8 * s : (s & ~7));
                dst = b + L::w_off + r * WB + (W == T_Q6_K ? 208 : 256);
            }
            if (ok && (src < g.w || src + 16 > wend)) {   // outside the matrix: skip (zero) and flag
                ok = false;
                src = g.w;
                if (err) atomicExch(err, 3);
            }
            cp_async16(dst, src, ok);
        }
        const int8_t* plane = W == T_Q8_0 ? a.q32 : a.qk;
        for (int i = tid; i < kBN * 16; i += kGemmThreads) {
            const int n = i >> 4, c = i & 15, t = t0 + n;
            const bool ok = t < T;
            const void* src = ok ? (const void*)(plane + (size_t)t * a.ld + (size_t)s * 256 + 16 * c) : (const void*)plane;
            cp_async16(b + L::x_off + n * kXStride + 16 * c, src, ok);
        }
        float dxv = 0.0f;
        if (W == T_Q8_0) {
            for (int i = tid; i < kBN * 2; i += kGemmThreads) {
                const int n = i >> 1, c = i & 1, t = t0 + n;
                const bool ok = t < T;
                const void* src = ok ? (const void*)(a.d32 + (size_t)t * (K / 32) + 8 * s + 4 * c) : (const void*)a.d32;
                cp_async16(b + L::d_off + n * 32 + 16 * c, src, ok);
            }
        } else {
            if (tid < kBN && t0 + tid < T) dxv = __ldg(a.dk + (size_t)(t0 + tid) * (K / 256) + s);
        }
        cp_async_commit();
        return dxv;
    };

    // Per output: the running row value and the pending nodes of the
    // current group's tree (block bi of the group: see tree_push).
    float acc[FT][JT][4], pa[FT][JT][4], pb[FT][JT][4], pc[FT][JT][4];
#pragma unroll
    for (int f = 0; f < FT; ++f)
#pragma unroll
        for (int j = 0; j < JT; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                acc[f][j][c] = 0.0f;
                pa[f][j][c] = pb[f][j][c] = pc[f][j][c] = 0.0f;
            }
    // The GEMV order for the 8 terms t0..t7 of a group:
    //   ((t0 + t1) + (t2 + t3)) + ((t4 + t5) + (t6 + t7)), then acc += group.
    // Block bi of the group is the same for the whole CTA: one branch per
    // block, every output inside it.
    // split mode: a finished half-group unit's value of output (f, j, c)
    auto unit_store = [&](int f, int j, int c, float v, int unit) {
        const int row = row0 + 16 * FT * wr + 16 * f + 8 * (c >> 1) + gid;
        const int t = t0 + 8 * JT * wc + 8 * j + 2 * tig + (c & 1);
        if (row < g.rows && t < T) part[((size_t)unit * T + t) * g.rows + row] = v;
    };
    // in split mode the half-group values ((t0 + t1) + (t2 + t3)) and
    // ((t4 + t5) + (t6 + t7)) go out at bi = 3 and 7 instead of acc += group
    auto tree_push = [&](const float (&t)[FT][JT][4], int bi, int unit) {
#define FB_EACH for (int f = 0; f < FT; ++f) for (int j = 0; j < JT; ++j) for (int c = 0; c < 4; ++c)
        switch (bi) {
            case 0: _Pragma("unroll") FB_EACH pa[f][j][c] = t[f][j][c]; break;
            case 1: _Pragma("unroll") FB_EACH pa[f][j][c] = __fadd_rn(pa[f][j][c], t[f][j][c]); break;
            case 2: _Pragma("unroll") FB_EACH pc[f][j][c] = t[f][j][c]; break;
            case 3:
                _Pragma("unroll") FB_EACH {
                    pa[f][j][c] = __fadd_rn(pa[f][j][c], __fadd_rn(pc[f][j][c], t[f][j][c]));
                    if (split) unit_store(f, j, c, pa[f][j][c], unit);
                }
                break;
            case 4: _Pragma("unroll") FB_EACH pb[f][j][c] = t[f][j][c]; break;
            case 5: _Pragma("unroll") FB_EACH pb[f][j][c] = __fadd_rn(pb[f][j][c], t[f][j][c]); break;
            case 6: _Pragma("unroll") FB_EACH pc[f][j][c] = t[f][j][c]; break;
            default:
                if (split) {
                    _Pragma("unroll") FB_EACH unit_store(f, j, c, __fadd_rn(pb[f][j][c], __fadd_rn(pc[f][j][c], t[f][j][c])), unit);
                } else {
                    _Pragma("unroll") FB_EACH acc[f][j][c] = __fadd_rn(
                        acc[f][j][c], __fadd_rn(pa[f][j][c], __fadd_rn(pb[f][j][c], __fadd_rn(pc[f][j][c], t[f][j][c]))));
                }
        }
#undef FB_EACH
    };
    // the same steps for one output (the Q6_K path: its 16 scale groups
    // leave fewer registers for a whole tile of terms)
    auto tree_push1 = [&](int f, int j, int c, float t, int bi, int unit) {
        switch (bi) {
            case 0: pa[f][j][c] = t; break;
            case 1: pa[f][j][c] = __fadd_rn(pa[f][j][c], t); break;
            case 2: pc[f][j][c] = t; break;
            case 3:
                pa[f][j][c] = __fadd_rn(pa[f][j][c], __fadd_rn(pc[f][j][c], t));
                if (split) unit_store(f, j, c, pa[f][j][c], unit);
                break;
            case 4: pb[f][j][c] = t; break;
            case 5: pb[f][j][c] = __fadd_rn(pb[f][j][c], t); break;
            case 6: pc[f][j][c] = t; break;
            default:
                if (split) unit_store(f, j, c, __fadd_rn(pb[f][j][c], __fadd_rn(pc[f][j][c], t)), unit);
                else acc[f][j][c] = __fadd_rn(acc[f][j][c], __fadd_rn(pa[f][j][c], __fadd_rn(pb[f][j][c], __fadd_rn(pc[f][j][c], t))));
        }
    };
    // after block bi of a group that ends there (the row's last group is
    // short; the GEMV adds +0 for its missing blocks), to the end of the
    // group, or of the half-group unit in split mode
    auto tree_close = [&](int bi, int unit) {
        float zero[FT][JT][4];
#pragma unroll
        for (int f = 0; f < FT; ++f)
#pragma unroll
            for (int j = 0; j < JT; ++j)
#pragma unroll
                for (int c = 0; c < 4; ++c) zero[f][j][c] = 0.0f;
        const int zend = split && bi < 4 ? 4 : 8;
        for (int z = bi + 1; z < zend; ++z) tree_push(zero, z, unit);
    };

    // steps 0 .. NS-2 in flight before the loop; every iteration commits one
    // group (the step NS-1 ahead, or an empty group past the end), so the
    // wait for all but the NS-1 newest groups always completes step s
#pragma unroll
    for (int p = 0; p < NS - 1; ++p) {
        if (p < nsteps) {
            const float dx0 = issue(p, sm + (size_t)p * L::bytes);
            if (W != T_Q8_0 && tid < kBN) reinterpret_cast<float*>(sm + (size_t)p * L::bytes + L::d_off)[tid] = dx0;
        } else {
            cp_async_commit();
        }
    }
    for (int s = 0; s < nsteps; ++s) {
        uint8_t* cur = sm + (size_t)(s % NS) * L::bytes;
        const int sn = s + NS - 1;   // the step issued now, into the stage step s - 1 used
        uint8_t* nxt = sm + (size_t)(sn % NS) * L::bytes;
        float dx_next = 0.0f;
        if (sn < nsteps) dx_next = issue(sn, nxt);
        else cp_async_commit();
        cp_async_wait<NS - 1>();
        __syncthreads();
        const uint8_t* sW = cur + L::w_off;
        const uint8_t* sX = cur + L::x_off;
        const float* sD = reinterpret_cast<const float*>(cur + L::d_off);
        const int sg = sb0 + s, unit = sg >> 2;
        const int bi = sg & 7;   // block (Q8_0: eighth) of the step within its group
        // this thread's rows (local): fragment f, h = 0: gid, h = 1: gid + 8;
        // tokens (local): fragment j, columns 2 tig, 2 tig + 1
        if (W == T_Q4_K) {
            // per row: fp16 d, dmin; 6-bit scales and mins of the 8 sub-blocks
            float dw[FT][2], dmw[FT][2];
            uint32_t sclo[FT][2], schi[FT][2], mlo[FT][2], mhi[FT][2];
#pragma unroll
            for (int f = 0; f < FT; ++f)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint4 hd = *reinterpret_cast<const uint4*>(sW + (16 * FT * wr + 16 * f + 8 * h + gid) * WB);
                    dw[f][h] = h2f((uint16_t)(hd.x & 0xFFFFu));
                    dmw[f][h] = h2f((uint16_t)(hd.x >> 16));
                    sclo[f][h] = hd.y & 0x3F3F3F3Fu;
                    mlo[f][h] = hd.z & 0x3F3F3F3Fu;
                    schi[f][h] = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
                    mhi[f][h] = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
                }
            // mins = sum_g m_g bsums_g = sum_l m_g(l) x_l: one more MMA per
            // sub-block with m_g in every byte of its A fragment, accumulated
            // in the MMA (exact integers, as sumi)
            int sumi[FT][JT][4], mn[FT][JT][4];
#pragma unroll
            for (int f = 0; f < FT; ++f)
#pragma unroll
                for (int j = 0; j < JT; ++j)
#pragma unroll
                    for (int c = 0; c < 4; ++c) sumi[f][j][c] = mn[f][j][c] = 0;
#pragma unroll
            for (int gq = 0; gq < 8; ++gq) {
                const int qoff = 16 + 32 * (gq >> 1), sh = (gq & 1) ? 4 : 0;
                uint32_t Am[FT][4];
#pragma unroll
                for (int f = 0; f < FT; ++f) {
                    Am[f][0] = Am[f][2] = (uint32_t)byte_of(gq < 4 ? mlo[f][0] : mhi[f][0], gq & 3) * 0x01010101u;
                    Am[f][1] = Am[f][3] = (uint32_t)byte_of(gq < 4 ? mlo[f][1] : mhi[f][1], gq & 3) * 0x01010101u;
                }
                uint32_t A[FT][4];
#pragma unroll
                for (int f = 0; f < FT; ++f) {
                    const uint8_t* r0p = sW + (16 * FT * wr + 16 * f + gid) * WB + qoff + 4 * tig;
                    const uint8_t* r1p = r0p + 8 * WB;
                    A[f][0] = (lds32(r0p) >> sh) & 0x0F0F0F0Fu;
                    A[f][1] = (lds32(r1p) >> sh) & 0x0F0F0F0Fu;
                    A[f][2] = (lds32(r0p + 16) >> sh) & 0x0F0F0F0Fu;
                    A[f][3] = (lds32(r1p + 16) >> sh) & 0x0F0F0F0Fu;
                }
#pragma unroll
                for (int j = 0; j < JT; ++j) {
                    const uint8_t* xp = sX + (8 * JT * wc + 8 * j + gid) * kXStride + 32 * gq + 4 * tig;
                    const uint32_t B[2] = {lds32(xp), lds32(xp + 16)};
#pragma unroll
                    for (int f = 0; f < FT; ++f) {
                        int c[4] = {0, 0, 0, 0};
                        mma_k32(c, A[f], B);
                        const int s0 = byte_of(gq < 4 ? sclo[f][0] : schi[f][0], gq & 3);
                        const int s1 = byte_of(gq < 4 ? sclo[f][1] : schi[f][1], gq & 3);
                        sumi[f][j][0] += s0 * c[0];
                        sumi[f][j][1] += s0 * c[1];
                        sumi[f][j][2] += s1 * c[2];
                        sumi[f][j][3] += s1 * c[3];
                        mma_k32(mn[f][j], Am[f], B);
                    }
                }
            }
            // the block's float terms
            float tt[FT][JT][4];
#pragma unroll
            for (int j = 0; j < JT; ++j) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const float dx = sD[8 * JT * wc + 8 * j + 2 * tig + e];
#pragma unroll
                    for (int f = 0; f < FT; ++f)
#pragma unroll
                        for (int h = 0; h < 2; ++h)
                            tt[f][j][2 * h + e] = q4k_term(dw[f][h], dmw[f][h], dx, sumi[f][j][2 * h + e], mn[f][j][2 * h + e]);
                }
            }
            tree_push(tt, bi, unit);
        } else if (W == T_Q6_K) {
            float dw[FT][2];
#pragma unroll
            for (int f = 0; f < FT; ++f)
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    dw[f][h] = h2f(*reinterpret_cast<const uint16_t*>(sW + (16 * FT * wr + 16 * f + 8 * h + gid) * WB + 208 + 2 * bi));
            int sumi[FT][JT][4];
#pragma unroll
            for (int f = 0; f < FT; ++f)
#pragma unroll
                for (int j = 0; j < JT; ++j)
#pragma unroll
                    for (int c = 0; c < 4; ++c) sumi[f][j][c] = 0;
#pragma unroll 4
            for (int jg = 0; jg < 16; ++jg) {   // 16-value group jg: values 16 jg .. 16 jg + 15 of the block
                const int hh = jg >> 3, quad = (jg & 7) >> 1, part = jg & 1;
                const int qlo = 64 * hh + 32 * (quad & 1) + 16 * part + 4 * tig;
                const int qho = 128 + 32 * hh + 16 * part + 4 * tig;
                const int nsh = quad < 2 ? 0 : 4, hsh = 2 * quad;
                uint32_t A[FT][2];
                int sc[FT][2];
#pragma unroll
                for (int f = 0; f < FT; ++f)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint8_t* rp = sW + (16 * FT * wr + 16 * f + 8 * h + gid) * WB;
                        const uint32_t v6 = ((lds32(rp + qlo) >> nsh) & 0x0F0F0F0Fu) | (((lds32(rp + qho) >> hsh) & 0x03030303u) << 4);
                        A[f][h] = __vsub4(v6, 0x20202020u);   // q6 - 32, per byte
                        sc[f][h] = (int)reinterpret_cast<const int8_t*>(rp + 192)[jg];
                    }
#pragma unroll
                for (int j = 0; j < JT; ++j) {
                    const uint32_t B = lds32(sX + (8 * JT * wc + 8 * j + gid) * kXStride + 16 * jg + 4 * tig);
#pragma unroll
                    for (int f = 0; f < FT; ++f) {
                        int c[4] = {0, 0, 0, 0};
                        mma_k16(c, A[f], B);
                        sumi[f][j][0] += sc[f][0] * c[0];
                        sumi[f][j][1] += sc[f][0] * c[1];
                        sumi[f][j][2] += sc[f][1] * c[2];
                        sumi[f][j][3] += sc[f][1] * c[3];
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < JT; ++j)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const float dx = sD[8 * JT * wc + 8 * j + 2 * tig + e];
#pragma unroll
                    for (int f = 0; f < FT; ++f)
#pragma unroll
                        for (int h = 0; h < 2; ++h)
                            tree_push1(f, j, 2 * h + e, scaled_term(dw[f][h], dx, sumi[f][j][2 * h + e]), bi, unit);
                }
        } else {   // Q8_0: eight 32-value blocks per step, summed in block order (a GEMV lane's share)
            float cs[FT][JT][4];
#pragma unroll
            for (int f = 0; f < FT; ++f)
#pragma unroll
                for (int j = 0; j < JT; ++j)
#pragma unroll
                    for (int c = 0; c < 4; ++c) cs[f][j][c] = 0.0f;
#pragma unroll 2
            for (int ib = 0; ib < 8; ++ib) {
                uint32_t A[FT][4];
                float dw[FT][2];
#pragma unroll
                for (int f = 0; f < FT; ++f) {
                    const uint8_t* r0p = sW + (16 * FT * wr + 16 * f + gid) * WB;
                    const uint8_t* r1p = r0p + 8 * WB;
                    A[f][0] = lds32(r0p + 32 * ib + 4 * tig);
                    A[f][1] = lds32(r1p + 32 * ib + 4 * tig);
                    A[f][2] = lds32(r0p + 32 * ib + 16 + 4 * tig);
                    A[f][3] = lds32(r1p + 32 * ib + 16 + 4 * tig);
                    dw[f][0] = h2f(*reinterpret_cast<const uint16_t*>(r0p + 256 + 2 * ib));
                    dw[f][1] = h2f(*reinterpret_cast<const uint16_t*>(r1p + 256 + 2 * ib));
                }
#pragma unroll
                for (int j = 0; j < JT; ++j) {
                    const uint8_t* xp = sX + (8 * JT * wc + 8 * j + gid) * kXStride + 32 * ib + 4 * tig;
                    const uint32_t B[2] = {lds32(xp), lds32(xp + 16)};
                    const float dx0 = sD[(8 * JT * wc + 8 * j + 2 * tig) * 8 + ib];
                    const float dx1 = sD[(8 * JT * wc + 8 * j + 2 * tig + 1) * 8 + ib];
#pragma unroll
                    for (int f = 0; f < FT; ++f) {
                        int c[4] = {0, 0, 0, 0};
                        mma_k32(c, A[f], B);
                        cs[f][j][0] = __fadd_rn(cs[f][j][0], scaled_term(dw[f][0], dx0, c[0]));
                        cs[f][j][1] = __fadd_rn(cs[f][j][1], scaled_term(dw[f][0], dx1, c[1]));
                        cs[f][j][2] = __fadd_rn(cs[f][j][2], scaled_term(dw[f][1], dx0, c[2]));
                        cs[f][j][3] = __fadd_rn(cs[f][j][3], scaled_term(dw[f][1], dx1, c[3]));
                    }
                }
            }
            tree_push(cs, bi, unit);
        }
        if (sg + 1 == K / 256 && bi != 7 && !(split && bi == 3)) tree_close(bi, unit);   // the row's short last group
        if (W != T_Q8_0 && sn < nsteps && tid < kBN) reinterpret_cast<float*>(nxt + L::d_off)[tid] = dx_next;
        __syncthreads();   // the stage is read; the next issue may overwrite it
    }
    // epilogue: bias, residual add (store_out)
    if (split) return;
#pragma unroll
    for (int f = 0; f < FT; ++f)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int row = row0 + 16 * FT * wr + 16 * f + 8 * h + gid;
            if (row >= g.rows) continue;
#pragma unroll
            for (int j = 0; j < JT; ++j)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int t = t0 + 8 * JT * wc + 8 * j + 2 * tig + e;
                    if (t < T) store_out(g, row, t, acc[f][j][2 * h + e]);
                }
        }
}

}  // namespace fb

using namespace fb;

static int gemm_num_sms() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 1;
}

template <int W, int BM, int BN, int NS, int FT, int JT>
static cudaError_t launch_gemm_tile(const GemvSeg& g, const ActQ& a, int K, int T, int* err, float* part,
                                    size_t part_floats, cudaStream_t st) {
    constexpr size_t smem = NS * (size_t)StageLayout<W, BM, BN>::bytes;
    constexpr int threads = BM * BN / (4 * FT * JT);   // 32 x warps
    static cudaError_t attr = [] {
        cudaError_t e = cudaFuncSetAttribute(k_gemm_q<W, BM, BN, NS, FT, JT, false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_gemm_q<W, BM, BN, NS, FT, JT, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem);
        return e;
    }();
    if (attr != cudaSuccess) return attr;
    // resident CTAs the device holds at once
    static const int capacity = [] {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_gemm_q<W, BM, BN, NS, FT, JT, true>, threads, smem) !=
            cudaSuccess)
            n = 1;
        return std::max(1, n) * gemm_num_sms();
    }();
    dim3 grid((g.rows + BM - 1) / BM, (T + BN - 1) / BN);
    // fewer tiles than resident CTAs: split K in half-group units so the
    // device fills (every unit's value is kept apart and the reduce adds them
    // in the unsplit order)
    static const bool no_split = getenv("FISH_GEMM_NO_SPLIT") != nullptr;
    const int tiles = (int)(grid.x * grid.y), n_units = (K / 256 + 3) / 4;
    int upc = 0;
    if (part && !no_split && tiles < capacity && n_units > 1 && (size_t)n_units * T * g.rows <= part_floats) {
        const int want = std::min(n_units, (capacity + tiles - 1) / tiles);
        if (want > 1) {
            upc = (n_units + want - 1) / want;
            grid.z = (n_units + upc - 1) / upc;
            if (grid.z <= 1) upc = 0, grid.z = 1;
        }
    }
    if (!upc) return fbk_launch(k_gemm_q<W, BM, BN, NS, FT, JT, false>, grid, dim3(threads), smem, st, g, a, K, T, err, 0,
                                (float*)nullptr);
    cudaError_t e = fbk_launch(k_gemm_q<W, BM, BN, NS, FT, JT, true>, grid, dim3(threads), smem, st, g, a, K, T, err, upc,
                               part);
    if (e != cudaSuccess) return e;
    return (cudaError_t)fbk_gemm_unit_reduce(&g, part, n_units, T, st);
}

// Token tile by call size: up to 32 tokens 16- or 32-token tiles with four
// stages in flight; longer prompts 64-token tiles (each weight step serves
// more tokens) double-buffered. At 33-64 tokens the 64-token tile (with the
// K split filling the device) wins on mid-sized matrices (Q6_K at 64 tokens:
// 18944x3584 221 -> 158 us, 14336x4096 181 -> 157 us) but not on very wide
// or narrow ones (152064 rows 909 vs 945 us, 512 rows 19 vs 25 us).
template <int W>
static cudaError_t launch_gemm(const GemvSeg& g, const ActQ& a, int K, int T, int* err, float* part, size_t pf,
                               cudaStream_t st) {
    static const int bn_env = [] {
        const char* e = getenv("FISH_GEMM_BN");
        return e ? atoi(e) : 0;
    }();
    static const int sms = gemm_num_sms();
    const bool mid = g.rows >= 2048 && g.rows <= 128 * sms && part;
    const int bn = bn_env == 16 || bn_env == 32 || bn_env == 64 ? bn_env
                                                              : (T <= 16 ? 16 : T <= 32 ? 32 : (T <= 64 && !mid) ? 32 : 64);
    // narrow token tiles on matrices with fewer 64-row tiles than SMs:
    // 32-row tiles, so twice the CTAs share the long K loop
    const bool rows32 = bn < 64 && (g.rows + 63) / 64 < sms;
    if (bn == 16) return rows32 ? launch_gemm_tile<W, 32, 16, 4, 1, 1>(g, a, K, T, err, part, pf, st)    // 4 warps of 16 x 8
                                : launch_gemm_tile<W, 64, 16, 4, 1, 1>(g, a, K, T, err, part, pf, st);   // 8 warps of 16 x 8
    if (bn == 32) return rows32 ? launch_gemm_tile<W, 32, 32, 4, 1, 2>(g, a, K, T, err, part, pf, st)    // 4 warps of 16 x 16
                                : launch_gemm_tile<W, 64, 32, 4, 1, 2>(g, a, K, T, err, part, pf, st);   // 8 warps of 16 x 16
    return launch_gemm_tile<W, 64, 64, 2, 2, 2>(g, a, K, T, err, part, pf, st);                           // 8 warps of 32 x 16
}

extern "C" int fbk_gemm_eligible(const GemvArgs* a) {
    if (a->T < 16 || a->pro.mode != PRO_ACT || a->swiglu || a->nseg <= 0) return 0;
    if (a->K % 256 || a->act.ld % 16) return 0;
    for (int s = 0; s < a->nseg; ++s) {
        const GemvSeg& g = a->seg[s];
        if (!(g.type == T_Q4_K || g.type == T_Q6_K || g.type == T_Q8_0) || g.expert || g.amax) return 0;
    }
    static const bool off = getenv("FISH_NO_GEMM") != nullptr;
    return off ? 0 : 1;
}

extern "C" int fbk_gemm(const GemvArgs* a, cudaStream_t st) {
    if (!fbk_gemm_eligible(a)) return (int)cudaErrorInvalidValue;
    int* err = a->err ? a->err : fbk_gemv_error_flag();
    for (int s = 0; s < a->nseg; ++s) {
        const GemvSeg& g = a->seg[s];
        cudaError_t e;
        // tcgen05 above 32 tokens; at 16-32 tokens only on narrow matrices
        // (at most 32 row tiles, K split over CTAs), where the mma.sync
        // kernel's few CTAs each walk all of K
        const bool narrow = (g.rows + 127) / 128 <= 32 && a->K >= 2048 && a->part;
        if (g.type == T_Q4_K && (a->T > 32 || narrow) && fbk_gemm_tc_eligible(&g, &a->act, a->K, a->T))
            e = (cudaError_t)fbk_gemm_tc(&g, &a->act, a->K, a->T, err, a->part, a->part_floats, st);
        else if (g.type == T_Q4_K) e = launch_gemm<T_Q4_K>(g, a->act, a->K, a->T, err, a->part, a->part_floats, st);
        else if (g.type == T_Q6_K) e = launch_gemm<T_Q6_K>(g, a->act, a->K, a->T, err, a->part, a->part_floats, st);
        else e = launch_gemm<T_Q8_0>(g, a->act, a->K, a->T, err, a->part, a->part_floats, st);
        if (e != cudaSuccess) return (int)e;
    }
    return 0;
}
