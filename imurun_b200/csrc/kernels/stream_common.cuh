// stream_common.cuh — device pieces shared by the streamed GEMV kernel and
// the persistent decode-step kernel: output epilogue, bounds check, the float
// steps of one block, tile -> segment mapping and the int8 activation image
// (layout and quantiser, the reference's arithmetic).
#pragma once

#include "common.cuh"
#include "kernels.h"
#include "layout.cuh"
#include "tma.cuh"
#include "trace.cuh"
#include "unit_math.cuh"

namespace fb {

constexpr int kXChunk = 272;   // bytes per 256 activation int8 (16 B pad: no bank conflicts)
constexpr int kConsumers = 8;            // consumer warps: 4 pairs, a pair per stage
constexpr int kPairs = kConsumers / 2;
constexpr int kMaxStages = 32;           // ring slots at most
constexpr int kMaxStreamTokens = 8;      // tokens of one streamed launch at most

__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory"); }


__device__ __forceinline__ float store_out(const GemvSeg& g, int rr, int t, float v) {
    if (g.bias) v += g.bias[rr];
    float* yp = g.y + (size_t)t * g.ldy + rr;
    if (g.epi == EPI_ADD) v += *yp;
    *yp = v;
    return v;
}

// true when [p, p + n) lies inside [lo, hi); otherwise the error flag is raised
__device__ __forceinline__ bool in_range(const uint8_t* p, size_t n, const uint8_t* lo, const uint8_t* hi, int* err) {
    if (p >= lo && p + n <= hi) return true;
    if (err) atomicExch(err, 3);
    return false;
}

// Float steps of one block, shared by both kernels (explicit roundings, so no
// multiply-add contraction can make the two kernels differ):
//   Q4_K  (dw dx) si - (dmin dx) mins      Q6_K, Q8_0  (dw dx) s
__device__ __forceinline__ float q4k_term(float dw, float dmw, float dx, int si, int mi) {
    return __fsub_rn(__fmul_rn(__fmul_rn(dw, dx), (float)si), __fmul_rn(__fmul_rn(dmw, dx), (float)mi));
}
__device__ __forceinline__ float scaled_term(float dw, float dx, int s) { return __fmul_rn(__fmul_rn(dw, dx), (float)s); }

// Segment of a tile (segments are copied to shared memory at kernel start,
// so no parameter array is indexed dynamically).
__device__ __forceinline__ int seg_index(const int* tile0, int nseg, int tile) {
    int sg = 0;
#pragma unroll
    for (int i = 1; i < kMaxSeg; ++i)
        if (i < nseg && tile >= tile0[i]) sg = i;
    return sg;
}
// Segment and segment-local tile of a tile: in pair mode tiles alternate
// (gate tile j, up tile j) so one CTA holds both halves of its output rows.
__device__ __forceinline__ void tile_seg(const int* tile0, int nseg, int pair, int tile, int& sg, int& lt) {
    if (pair) {
        sg = tile & 1;
        lt = tile >> 1;
    } else {
        sg = seg_index(tile0, nseg, tile);
        lt = tile - tile0[sg];
    }
}

// Activation image in shared memory, per token:
//   K layout (256-value blocks): q [n256][272], bsums [n256][8] i16,
//                                sum16 [n256][16] i16, d [n256] f32
//   32 layout:                   q [n256][272], d [n256][8] f32
struct XImage {
    uint8_t* base;
    int n256, xk, x32, T;
    __device__ int8_t* qk(int t, int c) const { return (int8_t*)(base + (size_t)t * xk + (size_t)c * kXChunk); }
    __device__ int16_t* bsk(int t, int c) const {
        return (int16_t*)(base + (size_t)t * xk + (size_t)n256 * kXChunk + 16 * c);
    }
    __device__ int16_t* s16(int t, int c) const {
        return (int16_t*)(base + (size_t)t * xk + (size_t)n256 * (kXChunk + 16) + 32 * c);
    }
    __device__ float* dk(int t, int c) const {
        return (float*)(base + (size_t)t * xk + (size_t)n256 * (kXChunk + 48) + 4 * c);
    }
    __device__ int8_t* q32(int t, int c) const {
        return (int8_t*)(base + (size_t)T * xk + (size_t)t * x32 + (size_t)c * kXChunk);
    }
    __device__ float* d32(int t, int c) const {
        return (float*)(base + (size_t)T * xk + (size_t)t * x32 + (size_t)n256 * kXChunk + 32 * c);
    }
};

static inline int ximg_k_bytes(int K) { return (((K + 255) / 256) * (kXChunk + 16 + 32 + 4) + 15) / 16 * 16; }
static inline int ximg_32_bytes(int K) { return (((K + 255) / 256) * (kXChunk + 32) + 15) / 16 * 16; }

__device__ __forceinline__ uint2 pack8q(const int (&q)[8]) {
    uint2 p;
    p.x = (q[0] & 0xFF) | ((q[1] & 0xFF) << 8) | ((q[2] & 0xFF) << 16) | ((uint32_t)(q[3] & 0xFF) << 24);
    p.y = (q[4] & 0xFF) | ((q[5] & 0xFF) << 8) | ((q[6] & 0xFF) << 16) | ((uint32_t)(q[7] & 0xFF) << 24);
    return p;
}

// Quantise one 256-value chunk (8 values per lane) into the image, both
// layouts as requested, with the reference's arithmetic (the same steps as
// quant_act.cu: d = amax/127, id = 1/d, round half to even, clamp).
__device__ __forceinline__ void ximg_quant_chunk(const float (&v)[8], int lane, int K, int t, int c,
                                                 const XImage& xi, bool wantk, bool want32) {
    const bool full = c * 256 + 256 <= K;
    float am = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(v[i]));
    if (wantk && full) {
        const float amax = warp_max(am);
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        int q[8], s = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            q[i] = max(-127, min(127, __float2int_rn(__fmul_rn(v[i], id))));
            s += q[i];
        }
        *reinterpret_cast<uint2*>(xi.qk(t, c) + 8 * lane) = pack8q(q);
        const int s16v = s + __shfl_xor_sync(0xffffffffu, s, 1);
        const int s32v = s16v + __shfl_xor_sync(0xffffffffu, s16v, 2);
        if ((lane & 1) == 0) xi.s16(t, c)[lane >> 1] = (int16_t)s16v;
        if ((lane & 3) == 0) xi.bsk(t, c)[lane >> 2] = (int16_t)s32v;
        if (lane == 0) *xi.dk(t, c) = d;
    }
    if (want32) {
        float b = am;
        b = fmaxf(b, __shfl_xor_sync(0xffffffffu, b, 1));
        b = fmaxf(b, __shfl_xor_sync(0xffffffffu, b, 2));
        const float d = __fdiv_rn(b, 127.0f);
        const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        int q[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = max(-127, min(127, __float2int_rn(__fmul_rn(v[i], id))));
        *reinterpret_cast<uint2*>(xi.q32(t, c) + 8 * lane) = pack8q(q);
        if ((lane & 3) == 0) xi.d32(t, c)[lane >> 2] = d;
    }
}

__device__ __forceinline__ void ld8(const float* p, int i0, int K, float (&v)[8]) {
    if (i0 + 8 <= K) {
        const float4 a = *reinterpret_cast<const float4*>(p + i0);
        const float4 b = *reinterpret_cast<const float4*>(p + i0 + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    }
}


// Norm weights a consumer lane keeps in registers: chunks warp + 8k, k < 2
// (all of them up to K = 4096), loaded before the wait for the previous kernel.
constexpr int kNormRegs = 2;
static_assert(kConsumers == kNormWarps, "the fused norm sums in the shared order of k_rmsnorm_quant");

// Consumer prologue: build the activation image for T tokens. PM >= 0 fixes
// the prologue mode at compile time (only that mode's code is emitted);
// PM < 0 reads it from the arguments.
template <int PM = -1>
__device__ __forceinline__ void build_ximage(const GemvArgs& args, const XImage& xi, bool wantk, bool want32,
                                             double* s_part, const float (&wv)[kNormRegs][8], int tseq) {
    const int ct = threadIdx.x, warp = ct >> 5, lane = ct & 31;
    const int K = args.K, T = args.T, n256 = xi.n256;
    const GemvPro& pro = args.pro;
    const int mode = PM >= 0 ? PM : pro.mode;
    if (mode == PRO_ACT) {
        const ActQ& a = args.act;
        for (int t = 0; t < T; ++t) {
            if (wantk) {
                for (int i = ct; i < n256 * 16; i += kConsumers * 32) {
                    const int c = i >> 4, j = i & 15;
                    const uint4 v =
                        __ldg(reinterpret_cast<const uint4*>(a.qk + (size_t)t * a.ld + (size_t)c * 256 + 16 * j));
                    *reinterpret_cast<uint4*>(xi.qk(t, c) + 16 * j) = v;
                    xi.s16(t, c)[j] = (int16_t)sum16(v);
                }
                for (int c = ct; c < n256; c += kConsumers * 32) {
                    *reinterpret_cast<uint4*>(xi.bsk(t, c)) =
                        __ldg(reinterpret_cast<const uint4*>(a.bsk + (size_t)t * (K / 32) + (size_t)c * 8));
                    *xi.dk(t, c) = __ldg(a.dk + (size_t)t * (K / 256) + c);
                }
            }
            if (want32) {
                for (int i = ct; i < K / 16; i += kConsumers * 32) {
                    const int c = i >> 4, j = i & 15;
                    *reinterpret_cast<uint4*>(xi.q32(t, c) + 16 * j) =
                        __ldg(reinterpret_cast<const uint4*>(a.q32 + (size_t)t * a.ld + 16 * (size_t)i));
                }
                for (int b = ct; b < K / 32; b += kConsumers * 32)
                    xi.d32(t, b >> 3)[b & 7] = __ldg(a.d32 + (size_t)t * (K / 32) + b);
            }
        }
        return;
    }
    const int n_chunks = (K + 255) / 256;
    if (mode == PRO_MERGE) {
        // decode-attention partials of C key chunks (one token): acc at
        // src[(c H + h) D ..], (m, l) at src[C H D + 2 (c H + h)]; the head's
        // output is sum_c e^(m_c - M) acc_c / sum_c e^(m_c - M) l_c,
        // accumulated online over the chunks in chunk order
        const int C = pro.ld, D = pro.ld2, H = K / D;
        const float* ml = pro.src + (size_t)C * H * D;
        for (int c = warp; c < n_chunks; c += kConsumers) {
            const int i0 = c * 256 + 8 * lane;
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = 0.0f;
            if (i0 < K) {
                const int h = i0 / D, d0 = i0 % D;
                float M = -INFINITY, den = 0.0f;
                for (int cc0 = 0; cc0 < C; cc0 += 2) {   // two chunks' loads in flight at once
                    float mb[2], lb[2];
                    float4 a0[2], a1[2];
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const size_t hc = (size_t)(cc0 + u) * H + h;
                        if (cc0 + u < C) {
                            mb[u] = ml[2 * hc];
                            lb[u] = ml[2 * hc + 1];
                            a0[u] = *reinterpret_cast<const float4*>(pro.src + hc * D + d0);
                            a1[u] = *reinterpret_cast<const float4*>(pro.src + hc * D + d0 + 4);
                        } else {
                            mb[u] = -INFINITY;
                        }
                    }
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const float m = mb[u];
                        if (!(m > -INFINITY)) continue;   // a chunk without keys, or past C
                        if (m > M) {
                            const float f = expf(M - m);
                            den *= f;
#pragma unroll
                            for (int i = 0; i < 8; ++i) v[i] *= f;
                            M = m;
                        }
                        const float wgt = expf(m - M);
                        den += wgt * lb[u];
                        v[0] += wgt * a0[u].x; v[1] += wgt * a0[u].y; v[2] += wgt * a0[u].z; v[3] += wgt * a0[u].w;
                        v[4] += wgt * a1[u].x; v[5] += wgt * a1[u].y; v[6] += wgt * a1[u].z; v[7] += wgt * a1[u].w;
                    }
                }
                const float inv = den > 0.0f ? 1.0f / den : 0.0f;
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] *= inv;
            }
            ximg_quant_chunk(v, lane, K, 0, c, xi, wantk, want32);
        }
        return;
    }
    if (mode == PRO_NORM) {
        // the reference's double sum (src/ops.cpp:18-23) in the order every
        // norm kernel shares (common.cuh); chunks that fit stay in registers
        // between the sum and the quantisation
        for (int t = 0; t < T; ++t) {
            const float* xr = pro.src + (size_t)t * pro.ld;
            float va[kNormRegs][8];
#pragma unroll
            for (int k = 0; k < kNormRegs; ++k) {
                const int c = warp + kConsumers * k;
                if (c < n_chunks) ld8(xr, c * 256 + 8 * lane, K, va[k]);
            }
            double s = 0.0;
#pragma unroll
            for (int k = 0; k < kNormRegs; ++k)
                if (warp + kConsumers * k < n_chunks) s = __dadd_rn(s, sumsq8(va[k]));
            for (int c = warp + kConsumers * kNormRegs; c < n_chunks; c += kConsumers) {
                float v[8];
                ld8(xr, c * 256 + 8 * lane, K, v);
                s = __dadd_rn(s, sumsq8(v));
            }
            s = warp_sum_d(s);
            if (lane == 0) s_part[warp] = s;
            consumers_sync();
            const float sc = norm_total(s_part, K, pro.eps);
            if (t == 0 && tseq >= 0 && ct == 0) trace_ev(TR_GEMV, EV_SCALE, tseq);
            consumers_sync();   // s_part is reused by the next token
#pragma unroll
            for (int k = 0; k < kNormRegs; ++k) {
                const int c = warp + kConsumers * k;
                if (c < n_chunks) {
                    const int i0 = c * 256 + 8 * lane;
                    float v[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[i] = i0 + i < K ? __fmul_rn(__fmul_rn(va[k][i], sc), wv[k][i]) : 0.0f;
                    ximg_quant_chunk(v, lane, K, t, c, xi, wantk, want32);
                }
            }
            for (int c = warp + kConsumers * kNormRegs; c < n_chunks; c += kConsumers) {
                const int i0 = c * 256 + 8 * lane;
                float xv[8], w8[8], v[8];
                ld8(xr, i0, K, xv);
                ld8(pro.w, i0, K, w8);
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = i0 + i < K ? __fmul_rn(__fmul_rn(xv[i], sc), w8[i]) : 0.0f;
                ximg_quant_chunk(v, lane, K, t, c, xi, wantk, want32);
            }
        }
        return;
    }
    // quantisation: warp w takes chunks w, w + 8, ...; each batch of up to 4
    // chunks loads everything it needs before computing
    constexpr int kB = 2;
    if (mode == PRO_QUANT) {   // one source: four chunks per batch
        constexpr int kQ = 4;
        for (int t = 0; t < T; ++t) {
            const float* xr = pro.src + (size_t)t * pro.ld;
            for (int c0 = warp; c0 < n_chunks; c0 += kConsumers * kQ) {
                float va[kQ][8];
#pragma unroll
                for (int k = 0; k < kQ; ++k) {
                    const int c = c0 + kConsumers * k;
                    if (c < n_chunks) ld8(xr, c * 256 + 8 * lane, K, va[k]);
                }
#pragma unroll
                for (int k = 0; k < kQ; ++k) {
                    const int c = c0 + kConsumers * k;
                    if (c < n_chunks) ximg_quant_chunk(va[k], lane, K, t, c, xi, wantk, want32);
                }
            }
        }
        return;
    }
    for (int t = 0; t < T; ++t) {
        const float* xr = pro.src + (size_t)t * pro.ld;
        const float* ur = mode == PRO_SILU ? pro.src2 + (size_t)t * pro.ld2 : nullptr;
        for (int c0 = warp; c0 < n_chunks; c0 += kConsumers * kB) {
            float va[kB][8], ua[kB][8];
#pragma unroll
            for (int k = 0; k < kB; ++k) {
                const int c = c0 + kConsumers * k;
                if (c < n_chunks) {
                    const int i0 = c * 256 + 8 * lane;
                    ld8(xr, i0, K, va[k]);
                    if (mode == PRO_SILU) ld8(ur, i0, K, ua[k]);
                }
            }
#pragma unroll
            for (int k = 0; k < kB; ++k) {
                const int c = c0 + kConsumers * k;
                if (c < n_chunks) {
                    float v[8];
                    if (mode == PRO_SILU) {
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            v[i] = __fmul_rn(__fdiv_rn(va[k][i], __fadd_rn(1.0f, expf(-va[k][i]))), ua[k][i]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 8; ++i) v[i] = va[k][i];
                    }
                    ximg_quant_chunk(v, lane, K, t, c, xi, wantk, want32);
                }
            }
        }
    }
}


// ------------------------------------------------------------ streamed jobs
//
// A streamed job is one GEMV as one CTA sees it: its 8-row tiles
// [t_begin, t_end), each split into G groups of 2048 values, one ring stage
// per (tile, group), in tile-major order. The producer warp (lane 0) issues
// the stages as one bulk copy each into a ring of shared-memory slots; four
// consumer warp pairs take every fourth stage.
//
// Ring stage g lives in slot g % S in phase g / S. A consumer must never wait
// on a slot for a phase two ahead of the barrier (a parity wait could not
// tell it apart from the phase behind). Two ways to guarantee that: S a
// multiple of the 4 pairs and a job starting at ring stage 0 (every slot is
// then only ever its own pair's, used phase after phase), or the guard: the
// consumer first waits until the producer has issued stage g, which implies
// the slot's previous phase completed (the producer waited for its release).


__device__ __forceinline__ void st_release_smem(volatile int* p, int v) {
    asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"((uint32_t)__cvta_generic_to_shared((const void*)p)), "r"(v)
                 : "memory");
}
__device__ __forceinline__ int ld_acquire_smem(volatile int* p) {
    int v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"((uint32_t)__cvta_generic_to_shared((const void*)p))
                 : "memory");
    return v;
}

struct RingView {
    uint8_t* base;
    uint64_t* full;
    uint64_t* empty;          // count 2: the two warps of the consuming pair
    int S, slot_bytes;
    volatile int* issued;     // ring stages the producer has issued
    volatile int* abort;      // CTA abort flag (shared)
    int guard;                // consumers wait for *issued > g first
    unsigned long long* pwait;   // optional: ns the producer waited for free slots
    unsigned long long* cwait;   // optional: ns consumer warp 0 waited for data
    long long* pclk = nullptr;   // optional: SM cycles in the producer's slot waits
    long long* cclk = nullptr;   // optional: SM cycles in thread 0's data waits
};

struct JobView {
    const GemvSeg* seg;       // shared copies
    const int* tile0;
    int nseg, pair, G, K, T;
    int t_begin, t_end;
};

// Weight-type sets a streamed kernel is compiled for (bit per type); a single
// type makes the per-stage type arithmetic constant, and the consumer loop
// carries only the arithmetic of the types in the set.
constexpr int TM_Q4K = 1, TM_Q6K = 2, TM_Q80 = 4, TM_ALL = 7;
__host__ __device__ constexpr int type_bit(int t) { return t == T_Q4_K ? TM_Q4K : t == T_Q6_K ? TM_Q6K : t == T_Q8_0 ? TM_Q80 : 0; }
template <int TM>
__device__ __forceinline__ int stage_type(int t) {
    return TM == TM_Q4K ? T_Q4_K : TM == TM_Q6K ? T_Q6_K : TM == TM_Q80 ? T_Q8_0 : t;
}

struct WaitFail {
    int stage, slot, parity;
    unsigned long long t0;
};

__device__ __forceinline__ int job_stages(const JobView& j) { return max(0, j.t_end - j.t_begin) * j.G; }

// Producer (one thread): the job's stages as ring stages gbase, gbase+1, ...
template <int TM = TM_ALL>
__device__ __forceinline__ bool produce_stages(const RingView& rg, const JobView& j, int gbase, int* err, WaitFail* wf) {
    const int n = job_stages(j);
    int tile = j.t_begin, gi = 0;
    int slot = gbase % rg.S, ph = gbase / rg.S;
    for (int l = 0; l < n; ++l) {
        int sg, lt;
        tile_seg(j.tile0, j.nseg, j.pair, tile, sg, lt);
        const GemvSeg& g = j.seg[sg];
        // expert index < 0: an expert held by another rank (expert
        // parallelism): nothing is streamed and the epilogue writes zeros
        const int eidx = g.expert ? __ldg(g.expert) : 0;
        const uint8_t* base = g.w + (size_t)max(eidx, 0) * g.expert_bytes;
        const int gt = stage_type<TM>(g.type);
        const int nb = row_blocks(gt, j.K);
        const uint32_t bytes = (uint32_t)(kTileRows * group_bytes(gt, group_blocks(gt, nb, gi)));
        if (ph > 0) {
            unsigned long long tw = 0;
            const long long c0 = rg.pclk ? clock64() : 0;
            const bool got = mbar_wait(&rg.empty[slot], (uint32_t)((ph - 1) & 1), rg.abort, &tw, rg.pwait);
            if (rg.pclk) *rg.pclk += clock64() - c0;
            if (!got) {
                wf->stage = gbase + l;
                wf->slot = slot;
                wf->parity = (ph - 1) & 1;
                wf->t0 = tw;
                return false;
            }
        }
        const uint8_t* src = base + (size_t)lt * kTileRows * g.row_stride + (size_t)kTileRows * group_offset(gt, gi);
        if (eidx >= 0 && bytes <= (uint32_t)rg.slot_bytes && in_range(src, bytes, g.w, g.w + g.w_bytes, err)) {
            mbar_expect_tx(&rg.full[slot], bytes);
            bulk_g2s(rg.base + (size_t)slot * rg.slot_bytes, src, bytes, &rg.full[slot]);
        } else {
            mbar_arrive(&rg.full[slot]);   // keep the ring moving; the stage holds stale bytes
        }
        st_release_smem(rg.issued, gbase + l + 1);
        if (++gi == j.G) {
            gi = 0;
            ++tile;
        }
        if (++slot == rg.S) {
            slot = 0;
            ++ph;
        }
    }
    return true;
}

// Consumer warps: pair pq = warp / 2 takes the job's local stages l with
// (gbase + l) % 4 == pq; warp half h of the pair rows 4h .. 4h+3 of the tile,
// lane = row * 8 + block. Row partials of local stage l go to
// part[(l * 8 + row) * NT + t]. False when a wait gave up (or the CTA aborted).
template <int NT, int TM = TM_ALL>
__device__ __forceinline__ bool consume_stages(const RingView& rg, const JobView& j, int gbase, const XImage& xi, float* part,
                                               WaitFail* wf, int tseq) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int half = warp & 1, pq = warp >> 1;
    const int r8 = 4 * half + (lane >> 3), bl = lane & 7;
    const int n = job_stages(j), G = j.G, K = j.K, T = j.T, S = rg.S;
    int l = (pq - (gbase & (kPairs - 1)) + kPairs) & (kPairs - 1);
    int tile = j.t_begin + l / G, gi = l % G;
    int slot = (gbase + l) % S, ph = (gbase + l) / S;
    for (; l < n; l += kPairs) {
        int sgc, ltc;
        tile_seg(j.tile0, j.nseg, j.pair, tile, sgc, ltc);
        const int type = stage_type<TM>(j.seg[sgc].type);
        const int nb = row_blocks(type, K), gbk = group_blocks(type, nb, gi);
        const int piece = (int)group_bytes(type, gbk);
        const uint8_t* pc = rg.base + (size_t)slot * rg.slot_bytes + (size_t)r8 * piece;
        if (rg.guard && ld_acquire_smem(rg.issued) <= gbase + l) {
            const unsigned long long t0 = gtimer();
            for (unsigned i = 1; ld_acquire_smem(rg.issued) <= gbase + l; ++i) {
                __nanosleep(64);
                if ((i & 63) == 0 && (*rg.abort || (long long)(gtimer() - t0) > kWaitNs)) {
                    wf->stage = gbase + l;
                    wf->slot = slot;
                    wf->parity = -1;
                    wf->t0 = t0;
                    return false;
                }
            }
        }
        {
            unsigned long long tw = 0;
            const long long c0 = rg.cclk && threadIdx.x == 0 ? clock64() : 0;
            const bool got = mbar_wait(&rg.full[slot], (uint32_t)(ph & 1), rg.abort, &tw, threadIdx.x == 0 ? rg.cwait : nullptr);
            if (rg.cclk && threadIdx.x == 0) *rg.cclk += clock64() - c0;
            if (!got) {
                wf->stage = gbase + l;
                wf->slot = slot;
                wf->parity = ph & 1;
                wf->t0 = tw;
                return false;
            }
        }
        if (tseq >= 0 && l == 0 && threadIdx.x == 0) trace_ev(TR_GEMV, EV_FIRST, tseq);
        float c[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) c[t] = 0.0f;
        // (the slot is released after the arithmetic: holding a whole block
        // in registers across an early release spills at the 96-register cap)
        if ((TM & TM_Q4K) && type == T_Q4_K) {
            if (bl < gbk) {
                uint4 w[9];
#pragma unroll
                for (int i = 0; i < 9; ++i) w[i] = *reinterpret_cast<const uint4*>(pc + bl * 144 + 16 * i);
                const float dw = h2f((uint16_t)(w[0].x & 0xFFFFu)), dmw = h2f((uint16_t)(w[0].x >> 16));
                const int kb = gi * 8 + bl;
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if (t >= T) break;
                    int si, mi;
                    q4k_block<LdShared>(w, xi.qk(t, kb), *reinterpret_cast<const uint4*>(xi.bsk(t, kb)), si, mi);
                    c[t] = q4k_term(dw, dmw, *xi.dk(t, kb), si, mi);
                }
            }
        } else if ((TM & TM_Q6K) && type == T_Q6_K) {
            if (bl < gbk) {
                uint4 w[13];
#pragma unroll
                for (int i = 0; i < 13; ++i) w[i] = *reinterpret_cast<const uint4*>(pc + bl * 208 + 16 * i);
                const float dw = h2f(*reinterpret_cast<const uint16_t*>(pc + gbk * 208 + 2 * bl));
                const int kb = gi * 8 + bl;
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if (t >= T) break;
                    const int si = q6k_block<LdShared>(w, xi.qk(t, kb), xi.s16(t, kb));
                    c[t] = scaled_term(dw, *xi.dk(t, kb), si);
                }
            }
        } else if (TM & TM_Q80) {   // Q8_0: lane takes blocks 8 bl .. 8 bl + 7 of the group, in block order
            const int kc = gi * 8 + bl;
            for (int i = 0; i < 8; ++i) {
                const int b = 8 * bl + i;
                if (b >= gbk) break;
                const uint4 w0 = *reinterpret_cast<const uint4*>(pc + 32 * b);
                const uint4 w1 = *reinterpret_cast<const uint4*>(pc + 32 * b + 16);
                const float dw = h2f(*reinterpret_cast<const uint16_t*>(pc + gbk * 32 + 2 * b));
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if (t >= T) break;
                    const int sv = q80_block<LdShared>(w0, w1, xi.q32(t, kc) + 32 * i);
                    c[t] = __fadd_rn(c[t], scaled_term(dw, xi.d32(t, kc)[i], sv));
                }
            }
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            c[t] += __shfl_xor_sync(0xffffffffu, c[t], 1);
            c[t] += __shfl_xor_sync(0xffffffffu, c[t], 2);
            c[t] += __shfl_xor_sync(0xffffffffu, c[t], 4);
        }
        if (bl == 0) {
#pragma unroll
            for (int t = 0; t < NT; ++t) part[((size_t)l * kTileRows + r8) * NT + t] = c[t];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&rg.empty[slot]);
        gi += kPairs;
        while (gi >= G) {
            gi -= G;
            ++tile;
        }
        slot += kPairs;
        while (slot >= S) {
            slot -= S;
            ++ph;
        }
    }
    return true;
}

// Warp-per-stage consumers (the persistent step kernel): warp w takes the
// job's local stages l with (gbase + l) % 8 == w, a whole stage each; lane =
// 8 * row pair + block, so a lane forms rows 2rp and 2rp+1 against one block
// of the activation image (its loads serve both rows) and loads weight words
// as it uses them. The integers are the quarter-block sums (unit_math.cuh)
// added up, i.e. exactly q4k_block / q6k_block; the float steps and the tree
// over blocks are those of consume_stages, so a row's value is the same.
// Empty barriers count 1 (the consuming warp); rg.guard must be set unless S
// is a multiple of 8 and the job starts at ring stage 0.
template <int NT, int TM = TM_ALL>
__device__ __forceinline__ bool consume_stages_w(const RingView& rg, const JobView& j, int gbase, const XImage& xi,
                                                 float* part, WaitFail* wf) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = 2 * (lane >> 3), bl = lane & 7;
    const int n = job_stages(j), G = j.G, K = j.K, T = j.T, S = rg.S;
    int l = (warp - (gbase & (kConsumers - 1)) + kConsumers) & (kConsumers - 1);
    int tile = j.t_begin + l / G, gi = l % G;
    int slot = (gbase + l) % S, ph = (gbase + l) / S;
    for (; l < n; l += kConsumers) {
        int sgc, ltc;
        tile_seg(j.tile0, j.nseg, j.pair, tile, sgc, ltc);
        const int type = stage_type<TM>(j.seg[sgc].type);
        const int nb = row_blocks(type, K), gbk = group_blocks(type, nb, gi);
        const int piece = (int)group_bytes(type, gbk);
        const uint8_t* p0 = rg.base + (size_t)slot * rg.slot_bytes + (size_t)r0 * piece;
        const uint8_t* p1 = p0 + piece;
        if (rg.guard && ld_acquire_smem(rg.issued) <= gbase + l) {
            const unsigned long long t0 = gtimer();
            for (unsigned i = 1; ld_acquire_smem(rg.issued) <= gbase + l; ++i) {
                __nanosleep(64);
                if ((i & 63) == 0 && (*rg.abort || (long long)(gtimer() - t0) > kWaitNs)) {
                    wf->stage = gbase + l;
                    wf->slot = slot;
                    wf->parity = -1;
                    wf->t0 = t0;
                    return false;
                }
            }
        }
        {
            unsigned long long tw = 0;
            if (!mbar_wait(&rg.full[slot], (uint32_t)(ph & 1), rg.abort, &tw, threadIdx.x == 0 ? rg.cwait : nullptr)) {
                wf->stage = gbase + l;
                wf->slot = slot;
                wf->parity = ph & 1;
                wf->t0 = tw;
                return false;
            }
        }
        float c0[NT], c1[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            c0[t] = 0.0f;
            c1[t] = 0.0f;
        }
        const int kb = gi * 8 + bl;
        if ((TM & TM_Q4K) && type == T_Q4_K) {
            if (bl < gbk) {
                const uint8_t* b0 = p0 + bl * 144;
                const uint8_t* b1 = p1 + bl * 144;
                const uint4 h0 = *reinterpret_cast<const uint4*>(b0), h1 = *reinterpret_cast<const uint4*>(b1);
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if (t >= T) break;
                    const int8_t* x = xi.qk(t, kb);
                    const uint4 bs = *reinterpret_cast<const uint4*>(xi.bsk(t, kb));
                    int a0 = 0, m0 = 0, a1 = 0, m1 = 0;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint4 x0 = *reinterpret_cast<const uint4*>(x + 64 * q);
                        const uint4 x1 = *reinterpret_cast<const uint4*>(x + 64 * q + 16);
                        const uint4 x2 = *reinterpret_cast<const uint4*>(x + 64 * q + 32);
                        const uint4 x3 = *reinterpret_cast<const uint4*>(x + 64 * q + 48);
                        const uint32_t bsw = word_of(bs, q);
                        int acc, mn;
                        q4k_quarter(h0, *reinterpret_cast<const uint4*>(b0 + 16 + 32 * q),
                                    *reinterpret_cast<const uint4*>(b0 + 32 + 32 * q), x0, x1, x2, x3, bsw, q, acc, mn);
                        a0 += acc;
                        m0 += mn;
                        q4k_quarter(h1, *reinterpret_cast<const uint4*>(b1 + 16 + 32 * q),
                                    *reinterpret_cast<const uint4*>(b1 + 32 + 32 * q), x0, x1, x2, x3, bsw, q, acc, mn);
                        a1 += acc;
                        m1 += mn;
                    }
                    const float dx = *xi.dk(t, kb);
                    c0[t] = q4k_term(h2f((uint16_t)(h0.x & 0xFFFFu)), h2f((uint16_t)(h0.x >> 16)), dx, a0 >> 4, m0);
                    c1[t] = q4k_term(h2f((uint16_t)(h1.x & 0xFFFFu)), h2f((uint16_t)(h1.x >> 16)), dx, a1 >> 4, m1);
                }
            }
        } else if ((TM & TM_Q6K) && type == T_Q6_K) {
            if (bl < gbk) {
                const uint8_t* b0 = p0 + bl * 208;
                const uint8_t* b1 = p1 + bl * 208;
                const uint4 sc0 = *reinterpret_cast<const uint4*>(b0 + 192), sc1 = *reinterpret_cast<const uint4*>(b1 + 192);
                const float dw0 = h2f(*reinterpret_cast<const uint16_t*>(p0 + gbk * 208 + 2 * bl));
                const float dw1 = h2f(*reinterpret_cast<const uint16_t*>(p1 + gbk * 208 + 2 * bl));
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if (t >= T) break;
                    int si0 = 0, si1 = 0;
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
                        for (int hl = 0; hl < 2; ++hl) {
                            const int8_t* x = xi.qk(t, kb) + 128 * hh + 16 * hl;
                            const uint4 xa = *reinterpret_cast<const uint4*>(x), xb = *reinterpret_cast<const uint4*>(x + 32);
                            const uint4 xc = *reinterpret_cast<const uint4*>(x + 64), xd = *reinterpret_cast<const uint4*>(x + 96);
                            const int16_t* s16 = xi.s16(t, kb) + 8 * hh + hl;
                            const int xs[4] = {(int)s16[0], (int)s16[2], (int)s16[4], (int)s16[6]};
                            const int oq = 64 * hh + 16 * hl, oh = 128 + 32 * hh + 16 * hl;
                            si0 += q6k_quarter(*reinterpret_cast<const uint4*>(b0 + oq), *reinterpret_cast<const uint4*>(b0 + oq + 32),
                                               *reinterpret_cast<const uint4*>(b0 + oh), sc0, xa, xb, xc, xd, xs, hh, hl);
                            si1 += q6k_quarter(*reinterpret_cast<const uint4*>(b1 + oq), *reinterpret_cast<const uint4*>(b1 + oq + 32),
                                               *reinterpret_cast<const uint4*>(b1 + oh), sc1, xa, xb, xc, xd, xs, hh, hl);
                        }
                    }
                    const float dx = *xi.dk(t, kb);
                    c0[t] = scaled_term(dw0, dx, si0);
                    c1[t] = scaled_term(dw1, dx, si1);
                }
            }
        } else if (TM & TM_Q80) {   // Q8_0: blocks 8 bl .. 8 bl + 7 of the group, in block order
            for (int i = 0; i < 8; ++i) {
                const int b = 8 * bl + i;
                if (b >= gbk) break;
                const uint4 wa0 = *reinterpret_cast<const uint4*>(p0 + 32 * b);
                const uint4 wa1 = *reinterpret_cast<const uint4*>(p0 + 32 * b + 16);
                const uint4 wb0 = *reinterpret_cast<const uint4*>(p1 + 32 * b);
                const uint4 wb1 = *reinterpret_cast<const uint4*>(p1 + 32 * b + 16);
                const float dwa = h2f(*reinterpret_cast<const uint16_t*>(p0 + gbk * 32 + 2 * b));
                const float dwb = h2f(*reinterpret_cast<const uint16_t*>(p1 + gbk * 32 + 2 * b));
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if (t >= T) break;
                    const int8_t* x = xi.q32(t, kb) + 32 * i;
                    const float dx = xi.d32(t, kb)[i];
                    c0[t] = __fadd_rn(c0[t], scaled_term(dwa, dx, q80_block<LdShared>(wa0, wa1, x)));
                    c1[t] = __fadd_rn(c1[t], scaled_term(dwb, dx, q80_block<LdShared>(wb0, wb1, x)));
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&rg.empty[slot]);   // every lane has read its words
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            c0[t] += __shfl_xor_sync(0xffffffffu, c0[t], 1);
            c0[t] += __shfl_xor_sync(0xffffffffu, c0[t], 2);
            c0[t] += __shfl_xor_sync(0xffffffffu, c0[t], 4);
            c1[t] += __shfl_xor_sync(0xffffffffu, c1[t], 1);
            c1[t] += __shfl_xor_sync(0xffffffffu, c1[t], 2);
            c1[t] += __shfl_xor_sync(0xffffffffu, c1[t], 4);
        }
        if (bl == 0) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                part[((size_t)l * kTileRows + r0) * NT + t] = c0[t];
                part[((size_t)l * kTileRows + r0 + 1) * NT + t] = c1[t];
            }
        }
        gi += kConsumers;
        while (gi >= G) {
            gi -= G;
            ++tile;
        }
        slot += kConsumers;
        while (slot >= S) {
            slot -= S;
            ++ph;
        }
    }
    return true;
}

// Consumer threads: the rows of the CTA's tiles, group partials summed in
// group order, through the epilogue: store/add (+bias), SwiGLU of (gate, up)
// tile pairs into segment 0, argmax keys (one atomic per token and CTA).
template <int NT>
__device__ __forceinline__ void reduce_rows(const JobView& j, const float* part,
                                            unsigned long long (*s_best)[kMaxStreamTokens]) {
    static_assert(NT <= kMaxStreamTokens, "argmax key slots per warp");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = j.G, T = j.T;
    unsigned long long best[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) best[t] = 0ull;
    const int n_rows = max(0, j.t_end - j.t_begin) * kTileRows;
    if (j.pair) {
        // tiles (2i, 2i+1) are (gate, up) tile i: h = silu(g) * u into segment 0's y
        const GemvSeg& g0 = j.seg[0];
        for (int idx = threadIdx.x; idx < n_rows / 2; idx += kConsumers * 32) {
            const int tp = idx / kTileRows, rr = idx % kTileRows;
            const int tl = 2 * tp, row = ((j.t_begin + tl) >> 1) * kTileRows + rr;
            if (row >= g0.rows) continue;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                if (t >= T) break;
                float gv = 0.0f, uv = 0.0f;
                for (int gi = 0; gi < G; ++gi) {
                    gv += part[((size_t)(tl * G + gi) * kTileRows + rr) * NT + t];
                    uv += part[((size_t)((tl + 1) * G + gi) * kTileRows + rr) * NT + t];
                }
                g0.y[(size_t)t * g0.ldy + row] = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), uv);
            }
        }
    }
    for (int idx = j.pair ? n_rows : threadIdx.x; idx < n_rows; idx += kConsumers * 32) {
        const int tl = idx / kTileRows, rr = idx % kTileRows, tile = j.t_begin + tl;
        const int sg = seg_index(j.tile0, j.nseg, tile);
        const GemvSeg& g = j.seg[sg];
        const int row = (tile - j.tile0[sg]) * kTileRows + rr;
        if (row >= g.rows) continue;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t >= T) break;
            float v = 0.0f;
            for (int gi = 0; gi < G; ++gi) v += part[((size_t)(tl * G + gi) * kTileRows + rr) * NT + t];
            if (g.expert && __ldg(g.expert) < 0) v = 0.0f;   // an expert of another rank
            v = store_out(g, row, t, v);
            if (g.amax) {
                const unsigned long long key = argmax_key(v, row + g.key_row0);
                best[t] = key > best[t] ? key : best[t];
            }
        }
    }
    if (j.seg[0].amax) {   // one segment (the output projection): merge the CTA's keys, one atomic per token
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            unsigned long long k = best[t];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long ok = __shfl_xor_sync(0xffffffffu, k, o);
                k = ok > k ? ok : k;
            }
            if (lane == 0) s_best[warp][t] = k;
        }
        consumers_sync();
        if (threadIdx.x < T) {
            unsigned long long k = 0ull;
            for (int w = 0; w < kConsumers; ++w) k = s_best[w][threadIdx.x] > k ? s_best[w][threadIdx.x] : k;
            if (k) atomicMax(&j.seg[0].amax[threadIdx.x], k);
        }
    }
}

}  // namespace fb
