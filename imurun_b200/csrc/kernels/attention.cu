// attention.cu — RoPE, KV append into the paged cache, causal GQA attention.
//
// Reference behaviour: RoPE from the
// precomputed cos/sin table with pairs (2i, 2i+1) or NeoX (i, i+half)
// (src/ops.cpp:126-156), K/V rows stored at their position
// (src/model.cpp:1723-1731), and per (token, head) softmax attention over
// positions 0..pos with scale 1/sqrt(D) (src/ops.cpp:303-356). The KV cache is
// paged (P positions per page, every layer of a position range in one page)
// and fp16 or f32.
#include <cooperative_groups.h>
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "tma.cuh"
#include "trace.cuh"

namespace fb {

__device__ __forceinline__ size_t kv_off(const KvView& kv, int layer, int head, int t, int pos) {
    int page = kv.pt[(size_t)kv.tok_seq[t] * kv.pt_stride + pos / kv.page_size];
    if (page < 0 || page >= kv.n_pages) {
        if (kv.err) atomicExch(kv.err, 5);
        page = 0;
    }
    return (size_t)page * kv.page_stride + (size_t)layer * kv.layer_stride + (size_t)head * kv.head_stride +
           (size_t)(pos % kv.page_size) * (kv.head_stride / kv.page_size);
}

// Gemma-2's attention-score soft cap (ops.cpp attention_batch): the scaled
// score s becomes cap * tanh(s / cap); cap 0 leaves it unchanged.
__device__ __forceinline__ float soft_cap(float s, float cap) {
    return cap > 0.0f ? __fmul_rn(cap, tanhf(__fdiv_rn(s, cap))) : s;
}
// First key a token at pos sees under a sliding window (0 without one).
__device__ __forceinline__ int window_lo(const KvView& kv, int pos) {
    return kv.window > 0 ? max(0, pos - kv.window + 1) : 0;
}

__global__ void k_rope_append(float* q, int ldq, const float* k, const float* v, int ldkv, int H, int HKV, int D,
                              int rot, int neox, const float* rcos, const float* rsin, KvView kv, int layer) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x;
    const int pos = kv.tok_pos[t];
    const int half = rot / 2;
    const float* c = rcos + (size_t)pos * half;
    const float* s = rsin + (size_t)pos * half;
    float* qr = q + (size_t)t * ldq;
    const float* kr = k + (size_t)t * ldkv;
    const float* vr = v + (size_t)t * ldkv;
    // q heads: rotate in place (biases were added by the projection epilogue)
    for (int idx = threadIdx.x; idx < H * (D / 2); idx += blockDim.x) {
        const int h = idx / (D / 2), i = idx % (D / 2);
        float* hv = qr + (size_t)h * D;
        if (i < half) {
            const int a = neox ? i : 2 * i, b = neox ? i + half : 2 * i + 1;
            const float x0 = hv[a], x1 = hv[b];
            hv[a] = __fsub_rn(__fmul_rn(x0, c[i]), __fmul_rn(x1, s[i]));
            hv[b] = __fadd_rn(__fmul_rn(x0, s[i]), __fmul_rn(x1, c[i]));
        }
    }
    // k heads: rotate and store; v heads: store
    for (int idx = threadIdx.x; idx < HKV * (D / 2); idx += blockDim.x) {
        const int h = idx / (D / 2), i = idx % (D / 2);
        const float* hk = kr + (size_t)h * D;
        const float* hvv = vr + (size_t)h * D;
        const size_t base = kv_off(kv, layer, h, t, pos);
        int a, b;
        float k0, k1;
        if (i < half) {
            a = neox ? i : 2 * i;
            b = neox ? i + half : 2 * i + 1;
            const float x0 = hk[a], x1 = hk[b];
            k0 = __fsub_rn(__fmul_rn(x0, c[i]), __fmul_rn(x1, s[i]));
            k1 = __fadd_rn(__fmul_rn(x0, s[i]), __fmul_rn(x1, c[i]));
        } else {
            a = 2 * i;
            b = 2 * i + 1;
            k0 = hk[a];
            k1 = hk[b];
        }
        const float v0 = hvv[2 * i], v1 = hvv[2 * i + 1];
        if (kv.f16) {
            __half* kp = reinterpret_cast<__half*>(kv.k) + base;
            __half* vp = reinterpret_cast<__half*>(kv.v) + base;
            kp[a] = __float2half_rn(k0);
            kp[b] = __float2half_rn(k1);
            vp[2 * i] = __float2half_rn(v0);
            vp[2 * i + 1] = __float2half_rn(v1);
        } else {
            float* kp = reinterpret_cast<float*>(kv.k) + base;
            float* vp = reinterpret_cast<float*>(kv.v) + base;
            kp[a] = k0;
            kp[b] = k1;
            vp[2 * i] = v0;
            vp[2 * i + 1] = v1;
        }
    }
}


// Split-K decode attention. CTA = (key split, kv head, query token); NW warps,
// each warp owns 32 consecutive keys (two 16-position pages). The CTA serves
// the G = H/HKV query heads of its kv head, so every K/V row is read once per
// group. Scores: lane = key, dot over D against q staged in shared memory.
// P.V: lane = a D-slice, 32 keys per warp with the probabilities shuffled.
// Each split writes (max, sum, o[D]) per head; k_attn_combine merges them.
constexpr int kMaxG = 8;
constexpr int kMaxD = 128;

template <bool F16, int NW>
__global__ void __launch_bounds__(32 * NW) k_attn_split(const float* __restrict__ q, int ldq, int H, int HKV, int D,
                                                        float scale, KvView kv, int layer, float* __restrict__ part,
                                                        int n_splits) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.z, hk = blockIdx.y, sp = blockIdx.x;
    const int G = H / HKV;
    const int n_keys = kv.tok_pos[t] + 1;
    const int j0 = sp * 32 * NW;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __shared__ __align__(16) float sq[kMaxG][kMaxD];
    __shared__ float sm[NW][kMaxG], sl[NW][kMaxG];
    __shared__ __align__(16) float so[NW][kMaxG][kMaxD];
    if (j0 >= n_keys) {
        if (threadIdx.x < G) {
            float* p = part + (((size_t)t * H + (size_t)hk * G + threadIdx.x) * n_splits + sp) * (D + 2);
            p[0] = -INFINITY;
            p[1] = 0.0f;
        }
        return;
    }
    for (int i = threadIdx.x; i < G * D; i += 32 * NW) sq[i / D][i % D] = q[(size_t)t * ldq + (size_t)hk * G * D + i];
    __syncthreads();
    const int jb = j0 + 32 * warp;
    const int j = jb + lane;
    const bool valid = j < n_keys;
    const bool live = valid && j >= window_lo(kv, n_keys - 1);
    float sc[kMaxG];
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) sc[g] = 0.0f;
    const size_t koff = valid ? kv_off(kv, layer, hk, t, j) : 0;
    if (valid) {
        const size_t off = koff;
        for (int d = 0; d < D; d += 8) {
            float kf[8];
            if (F16) {
                const uint4 raw = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(kv.k) + off + d);
                const __half2* hp = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(hp[e]);
                    kf[2 * e] = f.x;
                    kf[2 * e + 1] = f.y;
                }
            } else {
                const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(kv.k) + off + d);
                const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(kv.k) + off + d + 4);
                kf[0] = a.x; kf[1] = a.y; kf[2] = a.z; kf[3] = a.w; kf[4] = b.x; kf[5] = b.y; kf[6] = b.z; kf[7] = b.w;
            }
#pragma unroll
            for (int g = 0; g < kMaxG; ++g) {
                if (g < G) {
                    const float4 qa = *reinterpret_cast<const float4*>(&sq[g][d]);
                    const float4 qb = *reinterpret_cast<const float4*>(&sq[g][d + 4]);
                    float s = sc[g];
                    s = fmaf(qa.x, kf[0], s); s = fmaf(qa.y, kf[1], s); s = fmaf(qa.z, kf[2], s); s = fmaf(qa.w, kf[3], s);
                    s = fmaf(qb.x, kf[4], s); s = fmaf(qb.y, kf[5], s); s = fmaf(qb.z, kf[6], s); s = fmaf(qb.w, kf[7], s);
                    sc[g] = s;
                }
            }
        }
    }
    // softmax pieces of this warp's 32 keys (jb < n_keys, so lane 0 is valid)
    float m[kMaxG], l[kMaxG];
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
        if (g >= G) break;
        const float s = live ? soft_cap(__fmul_rn(sc[g], scale), kv.softcap) : -INFINITY;
        m[g] = warp_max(s);
        sc[g] = live ? expf(s - m[g]) : 0.0f;
        l[g] = warp_sum(sc[g]);
    }
    // P.V, lane owns dims [dper*lane, dper*lane + dper)
    const int dper = D / 32;
    float o[kMaxG][4];
#pragma unroll
    for (int g = 0; g < kMaxG; ++g)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[g][e] = 0.0f;
    const int nk = min(32, n_keys - jb);
    // each lane computed its own key's cache offset; broadcast them so the V
    // loads of 8 keys issue together with no dependent page-table reads
    for (int j8 = 0; j8 < nk; j8 += 8) {
        float vf[8][4];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int jj = j8 + u;
            const size_t off = (size_t)__shfl_sync(0xffffffffu, (long long)koff, jj & 31) + (size_t)lane * dper;
#pragma unroll
            for (int e = 0; e < 4; ++e) vf[u][e] = 0.0f;
            if (jj < nk) {
                if (F16) {
                    if (dper == 4) {
                        const uint2 raw = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(kv.v) + off);
                        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
                        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
                        vf[u][0] = a.x; vf[u][1] = a.y; vf[u][2] = b.x; vf[u][3] = b.y;
                    } else if (dper == 3) {
                        const __half* hv = reinterpret_cast<const __half*>(kv.v) + off;
#pragma unroll
                        for (int e = 0; e < 3; ++e) vf[u][e] = __half2float(hv[e]);
                    } else {
                        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(reinterpret_cast<const __half*>(kv.v) + off));
                        vf[u][0] = a.x; vf[u][1] = a.y;
                    }
                } else {
                    if (dper == 4) {
                        const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(kv.v) + off);
                        vf[u][0] = a.x; vf[u][1] = a.y; vf[u][2] = a.z; vf[u][3] = a.w;
                    } else if (dper == 3) {
                        const float* fv = reinterpret_cast<const float*>(kv.v) + off;
#pragma unroll
                        for (int e = 0; e < 3; ++e) vf[u][e] = fv[e];
                    } else {
                        const float2 a = *reinterpret_cast<const float2*>(reinterpret_cast<const float*>(kv.v) + off);
                        vf[u][0] = a.x; vf[u][1] = a.y;
                    }
                }
            }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
#pragma unroll
            for (int g = 0; g < kMaxG; ++g) {
                if (g >= G) break;
                const float p = __shfl_sync(0xffffffffu, sc[g], (j8 + u) & 31);   // 0 for keys >= nk
#pragma unroll
                for (int e = 0; e < 4; ++e) o[g][e] = fmaf(p, vf[u][e], o[g][e]);
            }
        }
    }
    float* pbase = part + (((size_t)t * H + (size_t)hk * G) * n_splits + sp) * (D + 2);
    if (NW == 1) {
#pragma unroll
        for (int g = 0; g < kMaxG; ++g) {
            if (g >= G) break;
            float* p = pbase + (size_t)g * n_splits * (D + 2);
            if (lane == 0) { p[0] = m[g]; p[1] = l[g]; }
#pragma unroll
            for (int e = 0; e < 4; ++e) if (e < dper) p[2 + lane * dper + e] = o[g][e];
        }
        return;
    }
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
        if (g >= G) break;
        if (lane == 0) { sm[warp][g] = jb < n_keys ? m[g] : -INFINITY; sl[warp][g] = l[g]; }
#pragma unroll
        for (int e = 0; e < 4; ++e) if (e < dper) so[warp][g][lane * dper + e] = o[g][e];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * D; i += 32 * NW) {
        const int g = i / D, d = i % D;
        float M = -INFINITY;
        for (int w = 0; w < NW; ++w) M = fmaxf(M, sm[w][g]);
        float L = 0.0f, O = 0.0f;
        for (int w = 0; w < NW; ++w) {
            if (sm[w][g] == -INFINITY) continue;
            const float c = expf(sm[w][g] - M);
            L += sl[w][g] * c;
            O += so[w][g][d] * c;
        }
        float* p = pbase + (size_t)g * n_splits * (D + 2);
        if (d == 0) { p[0] = M; p[1] = L; }
        p[2 + d] = O;
    }
}

// out[t][h][:] = sum_s w_s o_s / sum_s w_s l_s with w_s = exp(m_s - max m).
__global__ void k_attn_combine(const float* __restrict__ part, int H, int D, int n_splits, float* out, int ldo) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ float sw[];   // n_splits weights
    __shared__ float s_L;
    const int t = blockIdx.y, h = blockIdx.x;
    const float* p = part + ((size_t)t * H + h) * n_splits * (D + 2);
    float M = -INFINITY;
    for (int s = 0; s < n_splits; ++s) M = fmaxf(M, p[(size_t)s * (D + 2)]);
    for (int s = threadIdx.x; s < n_splits; s += blockDim.x) {
        const float ms = p[(size_t)s * (D + 2)];
        sw[s] = ms == -INFINITY ? 0.0f : expf(ms - M);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float L = 0.0f;
        for (int s = 0; s < n_splits; ++s) if (sw[s] != 0.0f) L += p[(size_t)s * (D + 2) + 1] * sw[s];
        s_L = L;
    }
    __syncthreads();
    const float L = s_L;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float O = 0.0f;
        for (int s = 0; s < n_splits; ++s) if (sw[s] != 0.0f) O += p[(size_t)s * (D + 2) + 2 + d] * sw[s];
        out[(size_t)t * ldo + (size_t)h * D + d] = L > 0.0f ? O / L : 0.0f;
    }
}


// ================================================================ fused decode
// Decode attention for T tokens of T distinct sequences, one kernel per layer:
// RoPE of q and of the new k, the append of the new K/V row into the cache,
// attention over the cached keys, and the merge of the partial results.
// A thread-block cluster of C CTAs serves one (token, kv head); CTA r takes
// the 64-key blocks r, r + C, ... of the context. A block's K and V page
// pieces (16 positions x D, contiguous in the paged layout) arrive by bulk
// copies into a two-slot ring while the previous block is computed. Scores:
// 8 lanes per key (D/8 dims each) reduced by shuffles; softmax is kept online
// per CTA (running max, sum and unnormalised output in shared memory); the C
// partials are merged through distributed shared memory. The CTA holding the
// token's own position rotates and stores the new k/v and patches its shared
// copy. Arithmetic follows k_rope_append, k_attn_split and k_attn_combine
// (src/ops.cpp:126-156, 303-356).
constexpr int kDecThreads = 128;
constexpr int kDecKeys = 64;

__device__ __forceinline__ float to_store(float x, const __half*) { return __half2float(__float2half_rn(x)); }
__device__ __forceinline__ float to_store(float x, const float*) { return x; }
__device__ __forceinline__ void put(__half* p, float x) { *p = __float2half_rn(x); }
__device__ __forceinline__ void put(float* p, float x) { *p = x; }

// Rows of the token's own sequence that this launch stores: when the tokens
// before t in the launch are the same sequence at positions pos-1, pos-2, ...
// (speculative verification runs a draft's tokens as one decode step), the
// K/V rows of those positions are being stored by other CTAs while this one
// runs, so the bulk copies may bring stale rows. Returns how many positions
// below pos are such rows (0 when every token is its own sequence).
__device__ __forceinline__ int fresh_rows(const KvView& kv, int t, int seq, int pos) {
    int nf = 0;
    while (nf < t && kv.tok_seq[t - 1 - nf] == seq && kv.tok_pos[t - 1 - nf] == pos - 1 - nf) ++nf;
    return nf;
}

// Rebuild the fresh rows that fall in block [j0, j0 + kb) of the shared K/V
// tiles (row stride rs elements) from the step's k/v projections, exactly as
// their owner CTAs store them: the rotation at the row's own position, then
// the rounding to the cache's element type.
template <class E>
__device__ void put_fresh_rows(E* K, E* V, int rs, int j0, int kb, int pos, int nf, int t, const float* knew,
                               const float* vnew, int ldkv, int hk, int D, int half, int neox, const float* rcos,
                               const float* rsin, int tid, int nt) {
    const int lo = max(j0, pos - nf), hi = min(j0 + kb, pos), pairs = D / 2;
    for (int idx = tid; idx < (hi - lo) * pairs; idx += nt) {
        const int j = lo + idx / pairs, i = idx % pairs, u = t - (pos - j);
        const float* kr = knew + (size_t)u * ldkv + (size_t)hk * D;
        const float* vr = vnew + (size_t)u * ldkv + (size_t)hk * D;
        E* kd = K + (size_t)(j - j0) * rs;
        E* vd = V + (size_t)(j - j0) * rs;
        int a = 2 * i, b = 2 * i + 1;
        float k0, k1;
        if (i < half) {
            a = neox ? i : 2 * i;
            b = neox ? i + half : 2 * i + 1;
            const float cs = rcos[(size_t)j * half + i], sn = rsin[(size_t)j * half + i];
            const float x0 = kr[a], x1 = kr[b];
            k0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
            k1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
        } else {
            k0 = kr[a];
            k1 = kr[b];
        }
        put(kd + a, k0);
        put(kd + b, k1);
        put(vd + 2 * i, vr[2 * i]);
        put(vd + 2 * i + 1, vr[2 * i + 1]);
    }
}
__device__ __forceinline__ float get(const __half* p) { return __half2float(*p); }
__device__ __forceinline__ float get(const float* p) { return *p; }

// n consecutive values (n = 8 or 16) of row p, as floats
template <int N>
__device__ __forceinline__ void ld_vals(const __half* p, float (&f)[16]) {
#pragma unroll
    for (int c = 0; c < N / 8; ++c) {
        const uint4 raw = *reinterpret_cast<const uint4*>(p + 8 * c);
        const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 v = __half22float2(h[e]);
            f[8 * c + 2 * e] = v.x;
            f[8 * c + 2 * e + 1] = v.y;
        }
    }
}
template <int N>
__device__ __forceinline__ void ld_vals(const float* p, float (&f)[16]) {
#pragma unroll
    for (int c = 0; c < N / 4; ++c) {
        const float4 a = *reinterpret_cast<const float4*>(p + 4 * c);
        f[4 * c] = a.x; f[4 * c + 1] = a.y; f[4 * c + 2] = a.z; f[4 * c + 3] = a.w;
    }
}

// 12 dims per lane (D = 96): halves at an 8-byte boundary, floats at 16
__device__ __forceinline__ void ld_vals12(const __half* p, float (&f)[16]) {
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const uint2 raw = *reinterpret_cast<const uint2*>(p + 4 * c);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
        f[4 * c] = a.x; f[4 * c + 1] = a.y; f[4 * c + 2] = b.x; f[4 * c + 3] = b.y;
    }
}
__device__ __forceinline__ void ld_vals12(const float* p, float (&f)[16]) { ld_vals<12>(p, f); }

template <class E>
struct DecSmem {
    static constexpr size_t kv_elems = (size_t)kDecKeys * kMaxD;
    static constexpr size_t off_k = 64;                                     // after 2 mbarriers + flags
    static constexpr size_t off_v = off_k + 2 * kv_elems * sizeof(E);
    static constexpr size_t off_q = off_v + 2 * kv_elems * sizeof(E);        // [G][D] f32
    static constexpr size_t off_s = off_q + sizeof(float) * kMaxG * kMaxD;   // [G][64] scores / probabilities
    static constexpr size_t off_o = off_s + sizeof(float) * kMaxG * kDecKeys;  // [G][D] output accumulator
    static constexpr size_t off_m = off_o + sizeof(float) * kMaxG * kMaxD;   // [G] running max
    static constexpr size_t off_l = off_m + sizeof(float) * kMaxG;           // [G] running sum
    static constexpr size_t off_c = off_l + sizeof(float) * kMaxG;           // [G] rescale of this block
    static constexpr size_t off_n = off_c + sizeof(float) * kMaxG;           // [2][D] new k, v (stored values)
    static constexpr size_t bytes = off_n + sizeof(float) * 2 * kMaxD;
};

template <class E>
__global__ void __launch_bounds__(kDecThreads) k_attn_decode(
    const float* __restrict__ q, int ldq, const float* __restrict__ knew, const float* __restrict__ vnew, int ldkv,
    int H, int HKV, int D, float scale, int rot, int neox, const float* __restrict__ rcos,
    const float* __restrict__ rsin, KvView kv, int layer, float* __restrict__ out, int ldo) {
    using L = DecSmem<E>;
    namespace cg = cooperative_groups;
    extern __shared__ __align__(128) uint8_t smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const int C = (int)cluster.num_blocks(), r = (int)cluster.block_rank();
    pdl_trigger();
    const bool tr = tracing() && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;
    __shared__ int s_tseq;
    if (tr && threadIdx.x == 0) {
        s_tseq = trace_launch(TR_ATTN);
        trace_ev(TR_ATTN, EV_START, s_tseq);
    }
    pdl_wait();
    if (tr && threadIdx.x == 0) trace_ev(TR_ATTN, EV_WAITED, s_tseq);
    const int t = blockIdx.z, hk = blockIdx.y, G = H / HKV;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
    volatile int* s_abort = reinterpret_cast<volatile int*>(smem + 16);
    E* sk = reinterpret_cast<E*>(smem + L::off_k);
    E* sv = reinterpret_cast<E*>(smem + L::off_v);
    float* sq = reinterpret_cast<float*>(smem + L::off_q);
    float* ss = reinterpret_cast<float*>(smem + L::off_s);
    float* so = reinterpret_cast<float*>(smem + L::off_o);
    float* sm = reinterpret_cast<float*>(smem + L::off_m);
    float* sl = reinterpret_cast<float*>(smem + L::off_l);
    float* sc = reinterpret_cast<float*>(smem + L::off_c);
    float* snew = reinterpret_cast<float*>(smem + L::off_n);
    const int pos = kv.tok_pos[t], n_keys = pos + 1;
    const int n_blocks = (n_keys + kDecKeys - 1) / kDecKeys;
    // blocks wholly below a sliding window are skipped: this rank's blocks
    // are b0 + r + C i
    const int jlo = window_lo(kv, pos), b0 = jlo / kDecKeys;
    const int nb_mine = r < n_blocks - b0 ? (n_blocks - b0 - r + C - 1) / C : 0;
    const int seq = kv.tok_seq[t];
    const size_t pblk = (size_t)16 * D;   // elements of one page's piece of this head
    const int b_own = pos / kDecKeys;
    const int nf = fresh_rows(kv, t, seq, pos);

    // bulk copies of my i-th block into slot i & 1: lane 0 sets the expected
    // bytes, lane pp (< 4) reads its page-table entry and copies that page
    auto issue = [&](int i) {   // called by all lanes of warp 0
        const int b = b0 + r + C * i, j0 = b * kDecKeys, kb = min(kDecKeys, n_keys - j0), np = (kb + 15) / 16;
        uint64_t* br = &bar[i & 1];
        if (lane == 0) mbar_expect_tx(br, (uint32_t)(2 * np * pblk * sizeof(E)));
        __syncwarp();
        if (lane < np) {
            const int pp = lane;
            int page = kv.pt[(size_t)seq * kv.pt_stride + j0 / 16 + pp];
            if (page < 0 || page >= kv.n_pages) {
                if (kv.err) atomicExch(kv.err, 5);
                page = 0;
            }
            const size_t off = (size_t)page * kv.page_stride + (size_t)layer * kv.layer_stride + (size_t)hk * kv.head_stride;
            bulk_g2s(sk + (size_t)(i & 1) * L::kv_elems + pp * pblk, reinterpret_cast<const E*>(kv.k) + off,
                     (uint32_t)(pblk * sizeof(E)), br);
            bulk_g2s(sv + (size_t)(i & 1) * L::kv_elems + pp * pblk, reinterpret_cast<const E*>(kv.v) + off,
                     (uint32_t)(pblk * sizeof(E)), br);
        }
    };
    if (tid == 0) {
        *s_abort = 0;
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (warp == 0) {
        if (nb_mine > 0) issue(0);
        if (nb_mine > 1) issue(1);
    }
    // q heads of this kv head, rotated (biases and q-norm were applied upstream)
    const int half = rot / 2;
    const float* cs = rcos + (size_t)pos * half;
    const float* sn = rsin + (size_t)pos * half;
    const float* qr = q + (size_t)t * ldq + (size_t)hk * G * D;
    for (int idx = tid; idx < G * (D / 2); idx += kDecThreads) {
        const int g = idx / (D / 2), i = idx % (D / 2);
        const float* hv = qr + (size_t)g * D;
        if (i < half) {
            const int a = neox ? i : 2 * i, b = neox ? i + half : 2 * i + 1;
            const float x0 = hv[a], x1 = hv[b];
            sq[g * kMaxD + a] = __fsub_rn(__fmul_rn(x0, cs[i]), __fmul_rn(x1, sn[i]));
            sq[g * kMaxD + b] = __fadd_rn(__fmul_rn(x0, sn[i]), __fmul_rn(x1, cs[i]));
        } else {
            sq[g * kMaxD + 2 * i] = hv[2 * i];
            sq[g * kMaxD + 2 * i + 1] = hv[2 * i + 1];
        }
    }
    // the token's own position: rotate k, store k and v, keep the stored values
    if ((b_own - b0) % C == r) {
        const float* kr = knew + (size_t)t * ldkv + (size_t)hk * D;
        const float* vr = vnew + (size_t)t * ldkv + (size_t)hk * D;
        const size_t base = kv_off(kv, layer, hk, t, pos);
        E* kp = reinterpret_cast<E*>(kv.k) + base;
        E* vp = reinterpret_cast<E*>(kv.v) + base;
        for (int i = tid; i < D / 2; i += kDecThreads) {
            int a, b;
            float k0, k1;
            if (i < half) {
                a = neox ? i : 2 * i;
                b = neox ? i + half : 2 * i + 1;
                const float x0 = kr[a], x1 = kr[b];
                k0 = __fsub_rn(__fmul_rn(x0, cs[i]), __fmul_rn(x1, sn[i]));
                k1 = __fadd_rn(__fmul_rn(x0, sn[i]), __fmul_rn(x1, cs[i]));
            } else {
                a = 2 * i;
                b = 2 * i + 1;
                k0 = kr[a];
                k1 = kr[b];
            }
            put(kp + a, k0);
            put(kp + b, k1);
            put(vp + 2 * i, vr[2 * i]);
            put(vp + 2 * i + 1, vr[2 * i + 1]);
            snew[a] = to_store(k0, kp);
            snew[b] = to_store(k1, kp);
            snew[kMaxD + 2 * i] = to_store(vr[2 * i], vp);
            snew[kMaxD + 2 * i + 1] = to_store(vr[2 * i + 1], vp);
        }
    }
    for (int i = tid; i < G * kMaxD; i += kDecThreads) so[i] = 0.0f;
    if (tid < G) {
        sm[tid] = -INFINITY;
        sl[tid] = 0.0f;
    }
    __syncthreads();
    if (tr && tid == 0) trace_ev(TR_ATTN, 4, s_tseq);   // q rotated, own row stored

    const int dpp = D / 8;                     // dims per lane in a key's dot
    const int part = lane & 7;
    int failed_at = -1;
    for (int i = 0; i < nb_mine; ++i) {
        const bool ok = mbar_wait(&bar[i & 1], (uint32_t)((i >> 1) & 1), s_abort);
        if (__syncthreads_or(!ok)) {
            failed_at = i;
            break;
        }
        if (tr && tid == 0 && i == 0) trace_ev(TR_ATTN, 5, s_tseq);   // first block landed
        const int b = b0 + r + C * i, j0 = b * kDecKeys, kb = min(kDecKeys, n_keys - j0);
        E* K = sk + (size_t)(i & 1) * L::kv_elems;
        E* V = sv + (size_t)(i & 1) * L::kv_elems;
        if (b == b_own) {
            const int rr = pos - j0;
            for (int d = tid; d < D; d += kDecThreads) {
                put(K + (size_t)rr * D + d, snew[d]);
                put(V + (size_t)rr * D + d, snew[kMaxD + d]);
            }
            __syncthreads();
        }
        if (nf > 0 && j0 < pos && j0 + kb > pos - nf) {
            put_fresh_rows(K, V, D, j0, kb, pos, nf, t, knew, vnew, ldkv, hk, D, half, neox, rcos, rsin, tid,
                           kDecThreads);
            __syncthreads();
        }
        // scores: warp w holds keys 16w .. 16w+15, four per pass, 8 lanes per key
#pragma unroll 1
        for (int ps = 0; ps < 4; ++ps) {
            const int key = 16 * warp + 4 * ps + (lane >> 3);
            const bool valid = key < kb;
            float acc[kMaxG];
#pragma unroll
            for (int g = 0; g < kMaxG; ++g) acc[g] = 0.0f;
            if (valid) {
                float kf[16];
                if (dpp == 16) ld_vals<16>(K + (size_t)key * D + 16 * part, kf);
                else if (dpp == 12) ld_vals12(K + (size_t)key * D + 12 * part, kf);
                else ld_vals<8>(K + (size_t)key * D + 8 * part, kf);
#pragma unroll
                for (int g = 0; g < kMaxG; ++g) {
                    if (g < G) {
                        const float* qq = sq + g * kMaxD + dpp * part;
                        float a = 0.0f;
#pragma unroll
                        for (int e4 = 0; e4 < 4; ++e4) {
                            if (4 * e4 < dpp) {
                                const float4 qv = *reinterpret_cast<const float4*>(qq + 4 * e4);
                                a = fmaf(qv.x, kf[4 * e4], a);
                                a = fmaf(qv.y, kf[4 * e4 + 1], a);
                                a = fmaf(qv.z, kf[4 * e4 + 2], a);
                                a = fmaf(qv.w, kf[4 * e4 + 3], a);
                            }
                        }
                        acc[g] = a;
                    }
                }
            }
#pragma unroll
            for (int g = 0; g < kMaxG; ++g) {
                if (g < G) {
                    float a = acc[g];
                    a += __shfl_xor_sync(0xffffffffu, a, 1);
                    a += __shfl_xor_sync(0xffffffffu, a, 2);
                    a += __shfl_xor_sync(0xffffffffu, a, 4);
                    if (part == 0 && valid)
                        ss[g * kDecKeys + key] = j0 + key >= jlo ? soft_cap(__fmul_rn(a, scale), kv.softcap) : -INFINITY;
                }
            }
        }
        __syncthreads();
        if (tr && tid == 0 && i == 0) trace_ev(TR_ATTN, 8, s_tseq);   // scores done
        // online softmax per head (warp g, g + 4)
        for (int g = warp; g < G; g += kDecThreads / 32) {
            const float s0 = lane < kb ? ss[g * kDecKeys + lane] : -INFINITY;
            const float s1 = lane + 32 < kb ? ss[g * kDecKeys + lane + 32] : -INFINITY;
            const float mb = warp_max(fmaxf(s0, s1));
            const float mo = sm[g], mn = fmaxf(mo, mb);
            const float p0 = s0 > -INFINITY ? expf(s0 - mn) : 0.0f;
            const float p1 = s1 > -INFINITY ? expf(s1 - mn) : 0.0f;
            const float sum = warp_sum(p0 + p1);
            ss[g * kDecKeys + lane] = p0;
            ss[g * kDecKeys + lane + 32] = p1;
            if (lane == 0) {
                const float corr = mo == -INFINITY ? 0.0f : expf(mo - mn);
                sl[g] = sl[g] * corr + sum;
                sm[g] = mn;
                sc[g] = corr;
            }
        }
        __syncthreads();
        if (tr && tid == 0 && i == 0) trace_ev(TR_ATTN, 9, s_tseq);   // softmax done
        // p.V: thread = one dim of one head (heads tid / D, tid / D + 128 / D, ...)
        for (int idx = tid; idx < G * D; idx += kDecThreads) {
            const int g = idx / D, d = idx % D;
            float o = so[g * kMaxD + d] * sc[g];
            const float* pg = ss + g * kDecKeys;
            for (int j = 0; j < kb; ++j) o = fmaf(pg[j], get(V + (size_t)j * D + d), o);
            so[g * kMaxD + d] = o;
        }
        __syncthreads();
        if (tr && tid == 0 && i == 0) trace_ev(TR_ATTN, 10, s_tseq);   // p.V done
        if (warp == 0 && i + 2 < nb_mine) issue(i + 2);
    }
    if (failed_at >= 0) {
        // let the copies still in flight (blocks failed_at, failed_at + 1) land before the CTA can exit
        if (tid == 0) {
            if (kv.err) atomicExch(kv.err, 6);
            for (int i = failed_at; i < nb_mine && i < failed_at + 2; ++i)
                mbar_wait_bounded(&bar[i & 1], (uint32_t)((i >> 1) & 1));
        }
        if (tid < G) { sm[tid] = -INFINITY; sl[tid] = 0.0f; }
    }
    if (tr && tid == 0) trace_ev(TR_ATTN, 6, s_tseq);   // blocks done
    cluster.sync();
    if (tr && tid == 0) trace_ev(TR_ATTN, 7, s_tseq);   // cluster barrier passed
    // merge the C partials through distributed shared memory: CTA r takes
    // outputs r*128 + tid (step C*128); every remote value is requested before
    // any is used
    for (int idx = r * kDecThreads + tid; idx < G * D; idx += C * kDecThreads) {
        const int g = idx / D, d = idx % D;
        float mv[16], lv[16], ov[16];
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) {
            if (rr < C) {
                mv[rr] = *cluster.map_shared_rank(sm + g, rr);
                lv[rr] = *cluster.map_shared_rank(sl + g, rr);
                ov[rr] = *cluster.map_shared_rank(so + g * kMaxD + d, rr);
            }
        }
        float M = -INFINITY;
#pragma unroll
        for (int rr = 0; rr < 16; ++rr)
            if (rr < C) M = fmaxf(M, mv[rr]);
        float Ls = 0.0f, O = 0.0f;
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) {
            if (rr < C && mv[rr] != -INFINITY) {
                const float w = expf(mv[rr] - M);
                Ls += lv[rr] * w;
                O += ov[rr] * w;
            }
        }
        out[(size_t)t * ldo + ((size_t)hk * G + g) * D + d] = Ls > 0.0f ? O / Ls : 0.0f;
    }
    cluster.sync();   // keep this CTA's shared memory alive until every remote read is done
    if (tr && threadIdx.x == 0) trace_ev(TR_ATTN, EV_END, s_tseq);
}


// ================================================================ fused decode, tensor cores (fp16 KV)
// Same structure as k_attn_decode, with both products on the tensor cores
// (mma.sync m16n8k16, f16 inputs, f32 accumulation): per warp and 64-key
// block, S^T[16 keys][8 heads] = K[16][D] . Q^T[D][8] and
// O^T[D][8 heads] += V^T[D][16 keys] . P^T[16][8]. q and p are split into
// f16 high and low parts (x = hi + lo to about 2^-22 relative) and both
// parts are multiplied, so the products keep f32 accuracy; K and V are the
// cache's f16 values. Every warp keeps its own online softmax state for its
// 16 keys of each block (the score and output fragments put the same two
// heads in each lane); the warps, then the cluster's CTAs, are merged at the
// end. K and V rows land in shared memory by one bulk copy per row, at a
// padded stride (D + 8 halves) so that ldmatrix reads are free of bank
// conflicts.
constexpr int kTcKeys = 64;
constexpr int kTcWarps = 4;
// floats of one rank partial: max[8], sum[8], O[G][D]
__host__ __device__ inline int dec_part_floats(int G, int D) { return 16 + G * D; }
constexpr int kTcRs = kMaxD + 8;   // padded row stride (halves) for D = 128; D = 64 uses 72

struct TcSmem {
    static constexpr size_t ring = (size_t)kTcKeys * kTcRs;                  // halves per slot
    static constexpr size_t off_k = 64;
    static constexpr size_t off_v = off_k + 2 * ring * 2;
    static constexpr size_t off_q = off_v + 2 * ring * 2;                     // [G][D] f32
    static constexpr size_t off_p = off_q + sizeof(float) * kMaxG * kMaxD;   // [warp][2][8 heads][16 keys] f16
    static constexpr size_t off_n = off_p + 2 * kTcWarps * 2 * 8 * 16;       // [2][D] f32 new k, v
    static constexpr size_t bytes = off_n + sizeof(float) * 2 * kMaxD;
    // after the last block the K ring holds the warps' partials and the V
    // ring the CTA's partial
    static constexpr size_t off_wm = off_k;                                   // [warp][8] f32
    static constexpr size_t off_wl = off_wm + sizeof(float) * kTcWarps * 8;
    static constexpr size_t off_wo = off_wl + sizeof(float) * kTcWarps * 8;  // [warp][8][D] f32
    static constexpr size_t off_cm = off_v;                                   // [8] f32
    static constexpr size_t off_cl = off_cm + sizeof(float) * 8;
    static constexpr size_t off_co = off_cl + sizeof(float) * 8;              // [8][D] f32
};
static_assert(TcSmem::off_wo + sizeof(float) * kTcWarps * 8 * kMaxD <= TcSmem::off_v, "warp partials fit the K ring");
static_assert(TcSmem::off_co + sizeof(float) * 8 * kMaxD <= TcSmem::off_q, "CTA partial fits the V ring");

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}
// x = hi + lo with hi, lo in f16
__device__ __forceinline__ void split_h(float x, float& hi, float& lo) {
    hi = __half2float(__float2half_rn(x));
    lo = x - hi;
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---- pieces shared by the decode kernel and the shared-prefix kernel; a
// token's arithmetic is the same wherever they run, so every path gives it
// the same bits

// q of one token rotated for its position (cs, sn: the position's table row)
// into sq[g * kMaxD + d]; threads tid of nt take the pairs in any order
__device__ __forceinline__ void tc_rotate_q(float* sq, const float* qr, int G, int qstride, int D, int half, int neox,
                                            const float* cs, const float* sn, int tid, int nt) {
    for (int idx = tid; idx < G * (D / 2); idx += nt) {
        const int g = idx / (D / 2), i = idx % (D / 2);
        const float* hv = qr + (size_t)g * qstride;
        if (i < half) {
            const int a = neox ? i : 2 * i, b = neox ? i + half : 2 * i + 1;
            const float x0 = hv[a], x1 = hv[b];
            sq[g * kMaxD + a] = __fsub_rn(__fmul_rn(x0, cs[i]), __fmul_rn(x1, sn[i]));
            sq[g * kMaxD + b] = __fadd_rn(__fmul_rn(x0, sn[i]), __fmul_rn(x1, cs[i]));
        } else {
            sq[g * kMaxD + 2 * i] = hv[2 * i];
            sq[g * kMaxD + 2 * i + 1] = hv[2 * i + 1];
        }
    }
}

// q as the B operand (k = dims, n = heads): lane holds head lane/4, dims
// 2(lane%4) + {0, 1, 8, 9} of each 16-dim step, as hi and lo halves
template <int KS>
__device__ __forceinline__ void tc_q_frags(const float* sq, int G, int lane, uint32_t (&qh)[KS][2], uint32_t (&ql)[KS][2]) {
    const int gq = lane >> 2, k0 = 2 * (lane & 3);
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int d = 16 * ks + k0 + 8 * e;
            const float x0 = gq < G ? sq[gq * kMaxD + d] : 0.0f, x1 = gq < G ? sq[gq * kMaxD + d + 1] : 0.0f;
            float h0, l0, h1, l1;
            split_h(x0, h0, l0);
            split_h(x1, h1, l1);
            qh[ks][e] = pack_h2(h0, h1);
            ql[ks][e] = pack_h2(l0, l1);
        }
    }
}

// One warp's 16 keys [kw, kw + 16) of a 64-key block (K, V: the block's
// rows at stride D + 8 halves; kb keys valid) into its online softmax state
// (m_r, l_r for the lane's two heads, O^T fragments acc).
template <int D>
__device__ __forceinline__ void tc_warp_block(const __half* K, const __half* V, int kw, int kb, int klo, float cap,
                                              float scale, const uint32_t (&qh)[D / 16][2],
                                              const uint32_t (&ql)[D / 16][2], float (&m_r)[2], float (&l_r)[2],
                                              float (&acc)[D / 16][4], __half* pw, int lane) {
    constexpr int RS = D + 8, KS = D / 16;
    if (kw >= kb || kw + 16 <= klo) return;
    const int gq = lane >> 2, k0 = 2 * (lane & 3), h0 = 2 * (lane & 3);
    const int r_in = (lane & 7) + ((lane >> 3) & 1) * 8, c_in = (lane >> 4) * 8;       // ldmatrix (K rows)
    const int key_in = (lane & 7) + ((lane >> 4) & 1) * 8, dim_in = ((lane >> 3) & 1) * 8;  // ldmatrix.trans (V)
    // scores S^T[16 keys][8 heads]: the q hi and lo products in two
    // independent accumulation chains, added at the end
    float c[4] = {0.0f, 0.0f, 0.0f, 0.0f}, cl4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
        uint32_t a[4];
        ldsm_x4(a, K + (size_t)(kw + r_in) * RS + 16 * ks + c_in);
        mma16816(c, a, qh[ks][0], qh[ks][1]);
        mma16816(cl4, a, ql[ks][0], ql[ks][1]);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) c[e] = __fadd_rn(c[e], cl4[e]);
    // c0: (key lane/4, head h0), c1: (lane/4, h0+1), c2: (lane/4+8, h0), c3: (lane/4+8, h0+1)
    const int ka = kw + (lane >> 2), kb2 = ka + 8;
    float sc[4];
    const bool va = ka < kb && ka >= klo, vb = kb2 < kb && kb2 >= klo;
    sc[0] = va ? soft_cap(__fmul_rn(c[0], scale), cap) : -INFINITY;
    sc[1] = va ? soft_cap(__fmul_rn(c[1], scale), cap) : -INFINITY;
    sc[2] = vb ? soft_cap(__fmul_rn(c[2], scale), cap) : -INFINITY;
    sc[3] = vb ? soft_cap(__fmul_rn(c[3], scale), cap) : -INFINITY;
    float corr[2], p[4];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        float mx = fmaxf(sc[e], sc[e + 2]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mn = fmaxf(m_r[e], mx);
        corr[e] = m_r[e] == -INFINITY ? 0.0f : expf(m_r[e] - mn);
        p[e] = sc[e] == -INFINITY ? 0.0f : expf(sc[e] - mn);
        p[e + 2] = sc[e + 2] == -INFINITY ? 0.0f : expf(sc[e + 2] - mn);
        float sum = p[e] + p[e + 2];
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        sum += __shfl_xor_sync(0xffffffffu, sum, 8);
        sum += __shfl_xor_sync(0xffffffffu, sum, 16);
        l_r[e] = __fmaf_rn(l_r[e], corr[e], sum);
        m_r[e] = mn;
    }
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
        acc[mt][0] = __fmul_rn(acc[mt][0], corr[0]);
        acc[mt][1] = __fmul_rn(acc[mt][1], corr[1]);
        acc[mt][2] = __fmul_rn(acc[mt][2], corr[0]);
        acc[mt][3] = __fmul_rn(acc[mt][3], corr[1]);
    }
    // P^T as the B operand of p.V (k = keys, n = heads): transpose through shared memory
    {
        const int kr = lane >> 2;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int hh = h0 + (e & 1), kk = kr + 8 * (e >> 1);
            float ph, pl;
            split_h(p[e], ph, pl);
            pw[(0 * 8 + hh) * 16 + kk] = __float2half_rn(ph);
            pw[(1 * 8 + hh) * 16 + kk] = __float2half_rn(pl);
        }
    }
    __syncwarp();
    const uint32_t pbh0 = *reinterpret_cast<const uint32_t*>(pw + (0 * 8 + gq) * 16 + k0);
    const uint32_t pbh1 = *reinterpret_cast<const uint32_t*>(pw + (0 * 8 + gq) * 16 + k0 + 8);
    const uint32_t pbl0 = *reinterpret_cast<const uint32_t*>(pw + (1 * 8 + gq) * 16 + k0);
    const uint32_t pbl1 = *reinterpret_cast<const uint32_t*>(pw + (1 * 8 + gq) * 16 + k0 + 8);
    __syncwarp();
    // O^T[D][8 heads] += V^T[D][16 keys] . P^T[16 keys][8 heads]
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
        uint32_t a[4];
        ldsm_x4_t(a, V + (size_t)(kw + key_in) * RS + 16 * mt + dim_in);
        mma16816(acc[mt], a, pbh0, pbh1);
        mma16816(acc[mt], a, pbl0, pbl1);
    }
}

// a warp's state (max, sum, O) into the CTA's per-warp partial arrays
template <int KS>
__device__ __forceinline__ void tc_store_warp(float* wm, float* wl, float* wo, int warp, int lane, const float (&m_r)[2],
                                              const float (&l_r)[2], const float (&acc)[KS][4]) {
    const int h0 = 2 * (lane & 3);
    if (lane < 4) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            wm[warp * 8 + h0 + e] = m_r[e];
            wl[warp * 8 + h0 + e] = l_r[e];
        }
    }
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
        const int d = 16 * mt + (lane >> 2);
        wo[((size_t)warp * 8 + h0) * kMaxD + d] = acc[mt][0];
        wo[((size_t)warp * 8 + h0 + 1) * kMaxD + d] = acc[mt][1];
        wo[((size_t)warp * 8 + h0) * kMaxD + d + 8] = acc[mt][2];
        wo[((size_t)warp * 8 + h0 + 1) * kMaxD + d + 8] = acc[mt][3];
    }
}

// the 4 warps' partials -> the CTA's (cm, cl, co); threads tid of nt
__device__ __forceinline__ void tc_merge_warps(const float* wm, const float* wl, const float* wo, float* cm, float* cl,
                                               float* co, int G, int D, int tid, int nt) {
    for (int idx = tid; idx < G * D; idx += nt) {
        const int g = idx / D, d = idx % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kTcWarps; ++w) M = fmaxf(M, wm[w * 8 + g]);
        float Ls = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < kTcWarps; ++w) {
            const float mw = wm[w * 8 + g];
            if (mw == -INFINITY) continue;
            const float cw = expf(mw - M);
            Ls = __fmaf_rn(wl[w * 8 + g], cw, Ls);
            O = __fmaf_rn(wo[((size_t)w * 8 + g) * kMaxD + d], cw, O);
        }
        co[g * kMaxD + d] = O;
        if (d == 0) { cm[g] = M; cl[g] = Ls; }
    }
}

// a warp's online-softmax state in global memory between the shared-prefix
// kernel and the decode kernel: floats [j][lane], j = m0 m1 l0 l1 acc...
__host__ __device__ constexpr int kStateFloats(int KS) { return 4 + 4 * KS; }
template <int KS, bool STORE>
__device__ __forceinline__ void tc_state_io(float* base, int lane, float (&m_r)[2], float (&l_r)[2], float (&acc)[KS][4]) {
    auto io = [&](int j, float& v) {
        if (STORE) base[j * 32 + lane] = v;
        else v = base[j * 32 + lane];
    };
    io(0, m_r[0]); io(1, m_r[1]); io(2, l_r[0]); io(3, l_r[1]);
#pragma unroll
    for (int mt = 0; mt < KS; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) io(4 + 4 * mt + e, acc[mt][e]);
}

// Shared-prefix blocks a rank of the prefix kernel keeps resident.
constexpr int kPreMaxBlocks = 4;

// GM (batched decode): the same C key ranks, launched as independent CTAs
// (x = rank) instead of one cluster, each writing its partial (max, sum,
// unnormalised O per head) to part[(t * HKV + hk) * C + r]; k_attn_decode_merge
// then merges the C partials with the cluster merge's arithmetic and order, so
// a token's output has the same bits on either path. Clusters of 16 CTAs are
// placed about one per GPC at a time, which serialises large batches.
template <int D, bool GM>
__global__ void __launch_bounds__(32 * kTcWarps) k_attn_decode_tc(
    const float* __restrict__ q, int ldq, const float* __restrict__ knew, const float* __restrict__ vnew, int ldkv,
    int H, int HKV, float scale, int rot, int neox, const float* __restrict__ rcos, const float* __restrict__ rsin,
    KvView kv, int layer, float* __restrict__ out, int ldo, float* __restrict__ part, const int* __restrict__ pre,
    const float* __restrict__ pstate) {
    using L = TcSmem;
    constexpr int RS = D + 8;        // padded row stride (halves)
    constexpr int KS = D / 16;       // k-steps of q.k, m-tiles of p.V
    namespace cg = cooperative_groups;
    extern __shared__ __align__(128) uint8_t smem[];
    const int C = GM ? (int)gridDim.x : (int)cg::this_cluster().num_blocks();
    const int r = GM ? (int)blockIdx.x : (int)cg::this_cluster().block_rank();
    pdl_trigger();
    // Blocks of this rank: b = r + C i. With a shared prefix (batched decode,
    // pre = its 64-key blocks, set before the step) the first i0 of them were
    // walked by k_attn_prefix_tc: their warp states wait in pstate, or, when
    // no block of the rank is left here, the rank partial is already in part.
    const int pos = kv.tok_pos[blockIdx.z], n_keys = pos + 1;
    const int n_blocks = (n_keys + kTcKeys - 1) / kTcKeys;
    // Blocks wholly below a sliding window are skipped the same way (the
    // rank's first i0 blocks, with no state to take over; a window and a
    // shared prefix never come together).
    const int bp = GM && pre ? min(*pre, C * kPreMaxBlocks) : 0;
    const int bs = bp > 0 ? bp : window_lo(kv, pos) / kTcKeys;
    const int i0 = r < bs ? (bs - r + C - 1) / C : 0;
    const int nb_all = r < n_blocks ? (n_blocks - r + C - 1) / C : 0;
    if (GM && bp > 0 && i0 > 0 && nb_all == i0) return;
    const int nb_mine = nb_all - i0;
    const unsigned long long t_kernel = gtimer();
    const bool tr = tracing() && !tracing_all() && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;
    __shared__ int s_tseq;
    if (tr && threadIdx.x == 0) {
        s_tseq = trace_launch(TR_ATTN);
        trace_ev(TR_ATTN, EV_START, s_tseq);
    }
    const int tcb = trace_cta_begin(3);
    if (tcb >= 0) {
        unsigned long long* r = g_trace.buf + 4 * (size_t)tcb;
        r[0] = t_kernel; r[1] = TR_ATTN; r[2] = EV_C_START;
        r[3] = (blockIdx.x + (unsigned long long)gridDim.x * (blockIdx.y + (unsigned long long)gridDim.y * blockIdx.z)) |
               ((unsigned long long)gridDim.x * gridDim.y * gridDim.z << 20);
    }
    // Before the dependency wait: everything written before this graph step
    // began (token positions, page tables, the KV cache of earlier positions,
    // the RoPE table). After it: q and the new k/v rows of the QKV projection.
    const int t = blockIdx.z, hk = blockIdx.y, G = H / HKV;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
    volatile int* s_abort = reinterpret_cast<volatile int*>(smem + 16);
    __half* sk = reinterpret_cast<__half*>(smem + L::off_k);
    __half* sv = reinterpret_cast<__half*>(smem + L::off_v);
    float* sq = reinterpret_cast<float*>(smem + L::off_q);
    __half* sp = reinterpret_cast<__half*>(smem + L::off_p);
    float* snew = reinterpret_cast<float*>(smem + L::off_n);
    const int seq = kv.tok_seq[t];
    const int b_own = pos / kTcKeys;
    const int nf = fresh_rows(kv, t, seq, pos);

    // warp 0: one bulk copy per K row and per V row of my i-th block (slot i & 1)
    auto issue = [&](int i) {
        const int b = r + C * (i0 + i), j0 = b * kTcKeys, kb = min(kTcKeys, n_keys - j0), np = (kb + 15) / 16;
        uint64_t* br = &bar[i & 1];
        int page = 0;
        if (lane < np) {
            page = kv.pt[(size_t)seq * kv.pt_stride + j0 / 16 + lane];
            if (page < 0 || page >= kv.n_pages) {
                if (kv.err) atomicExch(kv.err, 5);
                page = 0;
            }
        }
        if (lane == 0) mbar_expect_tx(br, (uint32_t)(2 * 16 * np * D * 2));
        __syncwarp();
        for (int k = 0; k < 2; ++k) {
            const int rr = lane + 32 * k;
            const int pg = __shfl_sync(0xffffffffu, page, (rr >> 4) & 3);
            if (rr < 16 * np) {
                const size_t off = (size_t)pg * kv.page_stride + (size_t)layer * kv.layer_stride +
                                   (size_t)hk * kv.head_stride + (size_t)(rr & 15) * D;
                bulk_g2s(sk + (size_t)(i & 1) * L::ring + (size_t)rr * RS, reinterpret_cast<const __half*>(kv.k) + off,
                         (uint32_t)(D * 2), br);
                bulk_g2s(sv + (size_t)(i & 1) * L::ring + (size_t)rr * RS, reinterpret_cast<const __half*>(kv.v) + off,
                         (uint32_t)(D * 2), br);
            }
        }
    };
    if (tid == 0) {
        *s_abort = 0;
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        mbar_fence_init();
    }
    __syncthreads();
    // the last warp issues the copies; the others rotate q and store the new row
    constexpr int kIssuer = kTcWarps - 1;
    if (warp == kIssuer) {
        if (nb_mine > 0) issue(0);
        if (nb_mine > 1) issue(1);
    }
    // this position's rotation table, staged in shared memory
    const int half = rot / 2;
    __shared__ float s_rot[2][kMaxD / 2];
    if (tid < half) {
        s_rot[0][tid] = rcos[(size_t)pos * half + tid];
        s_rot[1][tid] = rsin[(size_t)pos * half + tid];
    }
    __syncthreads();
    const float* cs = s_rot[0];
    const float* sn = s_rot[1];
    pdl_wait();
    trace_cta(tcb, 1, TR_ATTN, EV_C_WAITED);
    if (tr && threadIdx.x == 0) trace_ev(TR_ATTN, EV_WAITED, s_tseq);
    const float* qr = q + (size_t)t * ldq + (size_t)hk * G * D;
    const int wt = 32 * kIssuer;   // threads doing the rotation
    if (warp < kIssuer) tc_rotate_q(sq, qr, G, D, D, half, neox, cs, sn, tid, wt);
    if (b_own % C == r && warp < kIssuer) {
        const float* kr = knew + (size_t)t * ldkv + (size_t)hk * D;
        const float* vr = vnew + (size_t)t * ldkv + (size_t)hk * D;
        const size_t base = kv_off(kv, layer, hk, t, pos);
        __half* kp = reinterpret_cast<__half*>(kv.k) + base;
        __half* vp = reinterpret_cast<__half*>(kv.v) + base;
        for (int i = tid; i < D / 2; i += wt) {
            int a, b;
            float k0, k1;
            if (i < half) {
                a = neox ? i : 2 * i;
                b = neox ? i + half : 2 * i + 1;
                const float x0 = kr[a], x1 = kr[b];
                k0 = __fsub_rn(__fmul_rn(x0, cs[i]), __fmul_rn(x1, sn[i]));
                k1 = __fadd_rn(__fmul_rn(x0, sn[i]), __fmul_rn(x1, cs[i]));
            } else {
                a = 2 * i;
                b = 2 * i + 1;
                k0 = kr[a];
                k1 = kr[b];
            }
            kp[a] = __float2half_rn(k0);
            kp[b] = __float2half_rn(k1);
            vp[2 * i] = __float2half_rn(vr[2 * i]);
            vp[2 * i + 1] = __float2half_rn(vr[2 * i + 1]);
            snew[a] = __half2float(__float2half_rn(k0));
            snew[b] = __half2float(__float2half_rn(k1));
            snew[kMaxD + 2 * i] = __half2float(__float2half_rn(vr[2 * i]));
            snew[kMaxD + 2 * i + 1] = __half2float(__float2half_rn(vr[2 * i + 1]));
        }
    }
    __syncthreads();
    if (tr && tid == 0) trace_ev(TR_ATTN, 4, s_tseq);

    uint32_t qh[KS][2], ql[KS][2];
    tc_q_frags<KS>(sq, G, lane, qh, ql);
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.0f, 0.0f};
    float acc[KS][4];
#pragma unroll
    for (int mt = 0; mt < KS; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[mt][e] = 0.0f;
    if (bp > 0 && i0 > 0) {   // continue from the shared-prefix kernel's state of this warp
        float* sb = const_cast<float*>(pstate) + ((((size_t)t * HKV + hk) * C + r) * kTcWarps + warp) * 32 * kStateFloats(KS);
        tc_state_io<KS, false>(sb, lane, m_r, l_r, acc);
    }
    __half* pw = sp + (size_t)warp * 2 * 8 * 16;   // [hi/lo][8 heads][16 keys]
    int failed_at = -1;
    for (int i = 0; i < nb_mine; ++i) {
        const bool ok = mbar_wait(&bar[i & 1], (uint32_t)((i >> 1) & 1), s_abort);
        if (__syncthreads_or(!ok)) {
            failed_at = i;
            break;
        }
        const int b = r + C * (i0 + i), j0 = b * kTcKeys, kb = min(kTcKeys, n_keys - j0);
        __half* K = sk + (size_t)(i & 1) * L::ring;
        __half* V = sv + (size_t)(i & 1) * L::ring;
        if (b == b_own) {
            const int rr = pos - j0;
            for (int d = tid; d < D; d += 32 * kTcWarps) {
                K[(size_t)rr * RS + d] = __float2half_rn(snew[d]);
                V[(size_t)rr * RS + d] = __float2half_rn(snew[kMaxD + d]);
            }
            __syncthreads();
        }
        if (nf > 0 && j0 < pos && j0 + kb > pos - nf) {
            put_fresh_rows(K, V, RS, j0, kb, pos, nf, t, knew, vnew, ldkv, hk, D, half, neox, rcos, rsin, tid,
                           32 * kTcWarps);
            __syncthreads();
        }
        tc_warp_block<D>(K, V, 16 * warp, kb, window_lo(kv, pos) - j0, kv.softcap, scale, qh, ql, m_r, l_r, acc, pw,
                         lane);
        __syncthreads();
        if (warp == kIssuer && i + 2 < nb_mine) issue(i + 2);
    }
    if (tr && tid == 0) trace_ev(TR_ATTN, 6, s_tseq);
    float* wm = reinterpret_cast<float*>(smem + L::off_wm);
    float* wl = reinterpret_cast<float*>(smem + L::off_wl);
    float* wo = reinterpret_cast<float*>(smem + L::off_wo);
    float* cm = reinterpret_cast<float*>(smem + L::off_cm);
    float* cl = reinterpret_cast<float*>(smem + L::off_cl);
    float* co = reinterpret_cast<float*>(smem + L::off_co);
    if (failed_at >= 0) {
        if (tid == 0) {
            if (kv.err) atomicExch(kv.err, 6);
            for (int i = failed_at; i < nb_mine && i < failed_at + 2; ++i)
                mbar_wait_bounded(&bar[i & 1], (uint32_t)((i >> 1) & 1));
        }
        __syncthreads();
        if (tid < 8) { cm[tid] = -INFINITY; cl[tid] = 0.0f; }
    } else {
        // the warps' partials (max, sum, unnormalised O) -> the CTA's
        tc_store_warp<KS>(wm, wl, wo, warp, lane, m_r, l_r, acc);
        __syncthreads();
        tc_merge_warps(wm, wl, wo, cm, cl, co, G, D, tid, 32 * kTcWarps);
    }
    if constexpr (GM) {
        __syncthreads();
        float* pp = part + ((size_t)(t * HKV + hk) * C + r) * dec_part_floats(G, D);
        if (tid < G) { pp[tid] = cm[tid]; pp[8 + tid] = cl[tid]; }
        for (int idx = tid; idx < G * D; idx += 32 * kTcWarps) pp[16 + idx] = co[(idx / D) * kMaxD + idx % D];
        trace_cta(tcb, 2, TR_ATTN, EV_C_END);
        return;
    }
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (tr && tid == 0) trace_ev(TR_ATTN, 7, s_tseq);
    // merge the C partials through distributed shared memory
    for (int idx = r * 32 * kTcWarps + tid; idx < G * D; idx += C * 32 * kTcWarps) {
        const int g = idx / D, d = idx % D;
        float mv[16], lv[16], ov[16];
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) {
            if (rr < C) {
                mv[rr] = *cluster.map_shared_rank(cm + g, rr);
                lv[rr] = *cluster.map_shared_rank(cl + g, rr);
                ov[rr] = *cluster.map_shared_rank(co + g * kMaxD + d, rr);
            }
        }
        float M = -INFINITY;
#pragma unroll
        for (int rr = 0; rr < 16; ++rr)
            if (rr < C) M = fmaxf(M, mv[rr]);
        float Ls = 0.0f, O = 0.0f;
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) {
            if (rr < C && mv[rr] != -INFINITY) {
                const float w = expf(mv[rr] - M);
                Ls = __fmaf_rn(lv[rr], w, Ls);
                O = __fmaf_rn(ov[rr], w, O);
            }
        }
        out[(size_t)t * ldo + ((size_t)hk * G + g) * D + d] = Ls > 0.0f ? O / Ls : 0.0f;
    }
    cluster.sync();
    if (tr && tid == 0) trace_ev(TR_ATTN, EV_END, s_tseq);
    trace_cta(tcb, 2, TR_ATTN, EV_C_END);
}

// The C rank partials of one (token, kv head) written by k_attn_decode_tc<D,
// true>, merged as the cluster kernel merges them through distributed shared
// memory (same loops, same order, same roundings).
__global__ void __launch_bounds__(256) k_attn_decode_merge(const float* __restrict__ part, int C, int G, int D, int HKV,
                                                           float* __restrict__ out, int ldo) {
    pdl_trigger();
    pdl_wait();
    const int hk = blockIdx.x, t = blockIdx.y;
    const int pf = dec_part_floats(G, D);
    const float* pp = part + (size_t)(t * HKV + hk) * C * pf;
    for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
        const int g = idx / D, d = idx % D;
        float mv[16], lv[16], ov[16];
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) {
            if (rr < C) {
                mv[rr] = pp[(size_t)rr * pf + g];
                lv[rr] = pp[(size_t)rr * pf + 8 + g];
                ov[rr] = pp[(size_t)rr * pf + 16 + idx];
            }
        }
        float M = -INFINITY;
#pragma unroll
        for (int rr = 0; rr < 16; ++rr)
            if (rr < C) M = fmaxf(M, mv[rr]);
        float Ls = 0.0f, O = 0.0f;
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) {
            if (rr < C && mv[rr] != -INFINITY) {
                const float w = expf(mv[rr] - M);
                Ls = __fmaf_rn(lv[rr], w, Ls);
                O = __fmaf_rn(ov[rr], w, O);
            }
        }
        out[(size_t)t * ldo + ((size_t)hk * G + g) * D + d] = Ls > 0.0f ? O / Ls : 0.0f;
    }
}

// Shared prefix of a batched decode (the sessions' first bp 64-key blocks
// sit on the same pages): CTA (rank r, kv head, 8 tokens) brings the rank's
// prefix blocks (b = r + C i < bp, at most kPreMaxBlocks) into shared memory
// once and runs, for each token, the decode kernel's four warps over them
// (tc_warp_block, same order), so those keys cross HBM once per step instead
// of once per session. A token for which the rank has more blocks leaves its
// warps' states in pstate for k_attn_decode_tc; otherwise the CTA merges them
// as the decode kernel does and writes the rank partial. Eight warps: two
// tokens at a time.
struct PreSmem {
    static constexpr size_t tile = (size_t)kTcKeys * kTcRs;                   // halves of one K or V block
    static constexpr size_t off_k = 128;                                       // barriers + abort flag below
    static constexpr size_t off_v = off_k + kPreMaxBlocks * tile * 2;
    static constexpr size_t off_q = off_v + kPreMaxBlocks * tile * 2;           // [8 tokens][8][kMaxD] f32
    static constexpr size_t off_r = off_q + sizeof(float) * 8 * 8 * kMaxD;     // [8 tokens][cos, sin][kMaxD / 2]
    static constexpr size_t off_p = off_r + sizeof(float) * 8 * kMaxD;         // [8 warps][2][8][16] f16
    static constexpr size_t off_wm = off_p + 2 * 8 * 2 * 8 * 16;               // [2][4 warps][8]
    static constexpr size_t off_wl = off_wm + sizeof(float) * 2 * kTcWarps * 8;
    static constexpr size_t off_wo = off_wl + sizeof(float) * 2 * kTcWarps * 8; // [2][4][8][kMaxD]
    static constexpr size_t off_cm = off_wo + sizeof(float) * 2 * kTcWarps * 8 * kMaxD;  // [2][8]
    static constexpr size_t off_cl = off_cm + sizeof(float) * 2 * 8;
    static constexpr size_t off_co = off_cl + sizeof(float) * 2 * 8;           // [2][8][kMaxD]
    static constexpr size_t bytes = off_co + sizeof(float) * 2 * 8 * kMaxD;
};
constexpr int kPreTokens = 8;

template <int D>
__global__ void __launch_bounds__(256) k_attn_prefix_tc(const float* __restrict__ q, int ldq, int H, int HKV, float scale,
                                                        int rot, int neox, const float* __restrict__ rcos,
                                                        const float* __restrict__ rsin, KvView kv, int layer, int T,
                                                        const int* __restrict__ pre, float* __restrict__ pstate,
                                                        float* __restrict__ part) {
    using L = PreSmem;
    constexpr int RS = D + 8, KS = D / 16;
    extern __shared__ __align__(128) uint8_t smem[];
    pdl_trigger();
    const int C = (int)gridDim.x, r = (int)blockIdx.x, hk = (int)blockIdx.y, G = H / HKV;
    const int bp = min(*pre, C * kPreMaxBlocks);
    const int nbp = r < bp ? (bp - r + C - 1) / C : 0;
    const int tb = (int)blockIdx.z * kPreTokens;
    if (nbp == 0 || tb >= T) return;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ntok = min(kPreTokens, T - tb);
    __shared__ int s_pos[kPreTokens];
    if (tid < ntok) s_pos[tid] = kv.tok_pos[tb + tid];   // set before the step
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
    volatile int* s_abort = reinterpret_cast<volatile int*>(smem + 64);
    __half* sk = reinterpret_cast<__half*>(smem + L::off_k);
    __half* sv = reinterpret_cast<__half*>(smem + L::off_v);
    if (tid == 0) {
        *s_abort = 0;
        for (int i = 0; i < kPreMaxBlocks; ++i) mbar_init(&bar[i], 1);
        mbar_fence_init();
    }
    __syncthreads();
    // the prefix pages are the same for every token of the batch (set before
    // the step from the page tables): read them through the first token's
    if (warp == 0) {
        const int seq = kv.tok_seq[tb];
        for (int i = 0; i < nbp; ++i) {
            const int j0 = (r + C * i) * kTcKeys;   // a full block: 4 pages
            int page = 0;
            if (lane < 4) {
                page = kv.pt[(size_t)seq * kv.pt_stride + j0 / 16 + lane];
                if (page < 0 || page >= kv.n_pages) {
                    if (kv.err) atomicExch(kv.err, 5);
                    page = 0;
                }
            }
            if (lane == 0) mbar_expect_tx(&bar[i], (uint32_t)(2 * kTcKeys * D * 2));
            __syncwarp();
            for (int k = 0; k < 2; ++k) {
                const int rr = lane + 32 * k;
                const int pg = __shfl_sync(0xffffffffu, page, rr >> 4);
                const size_t off = (size_t)pg * kv.page_stride + (size_t)layer * kv.layer_stride +
                                   (size_t)hk * kv.head_stride + (size_t)(rr & 15) * D;
                bulk_g2s(sk + (size_t)i * L::tile + (size_t)rr * RS, reinterpret_cast<const __half*>(kv.k) + off,
                         (uint32_t)(D * 2), &bar[i]);
                bulk_g2s(sv + (size_t)i * L::tile + (size_t)rr * RS, reinterpret_cast<const __half*>(kv.v) + off,
                         (uint32_t)(D * 2), &bar[i]);
            }
        }
    }
    // the group's q rows (raw) and their positions' rotation rows, with
    // independent loads, then every row rotated in place
    const int half = rot / 2, GD = G * D;
    float* sqa = reinterpret_cast<float*>(smem + L::off_q);
    float* srot = reinterpret_cast<float*>(smem + L::off_r);
    for (int i = tid; i < ntok * half; i += 256) {
        const int u = i / half, j = i % half;
        srot[u * kMaxD + j] = rcos[(size_t)s_pos[u] * half + j];
        srot[u * kMaxD + kMaxD / 2 + j] = rsin[(size_t)s_pos[u] * half + j];
    }
    pdl_wait();
    for (int i = tid; i < ntok * (GD / 4); i += 256) {
        const int u = i / (GD / 4), j = 4 * (i % (GD / 4));
        const float4 v4 = *reinterpret_cast<const float4*>(q + (size_t)(tb + u) * ldq + (size_t)hk * GD + j);
        *reinterpret_cast<float4*>(sqa + (size_t)u * 8 * kMaxD + (j / D) * kMaxD + j % D) = v4;
    }
    __syncthreads();
    for (int u = 0; u < ntok; ++u)   // pairs (a, b) are disjoint: in place
        tc_rotate_q(sqa + (size_t)u * 8 * kMaxD, sqa + (size_t)u * 8 * kMaxD, G, kMaxD, D, half, neox,
                    srot + u * kMaxD, srot + u * kMaxD + kMaxD / 2, tid, 256);
    bool ok = true;
    for (int i = 0; i < nbp && ok; ++i) ok = mbar_wait(&bar[i], 0u, s_abort);
    if (__syncthreads_or(!ok)) {
        if (tid == 0) {
            if (kv.err) atomicExch(kv.err, 6);
            for (int i = 0; i < nbp; ++i) mbar_wait_bounded(&bar[i], 0u);
        }
        return;
    }
    const int slot = warp >> 2, w = warp & 3, stid = tid & 127;
    __half* pw = reinterpret_cast<__half*>(smem + L::off_p) + (size_t)warp * 2 * 8 * 16;
    float* wm = reinterpret_cast<float*>(smem + L::off_wm) + slot * kTcWarps * 8;
    float* wl = reinterpret_cast<float*>(smem + L::off_wl) + slot * kTcWarps * 8;
    float* wo = reinterpret_cast<float*>(smem + L::off_wo) + (size_t)slot * kTcWarps * 8 * kMaxD;
    float* cm = reinterpret_cast<float*>(smem + L::off_cm) + slot * 8;
    float* cl = reinterpret_cast<float*>(smem + L::off_cl) + slot * 8;
    float* co = reinterpret_cast<float*>(smem + L::off_co) + (size_t)slot * 8 * kMaxD;
    for (int pr = 0; pr < kPreTokens / 2; ++pr) {
        const int u = 2 * pr + slot, t = tb + u;
        const bool tv = t < T;
        const int pos = tv ? s_pos[u] : 0;
        const float* sq = sqa + (size_t)u * 8 * kMaxD;
        // does the rank have blocks of this token past the prefix?
        const int n_blocks = (pos + 1 + kTcKeys - 1) / kTcKeys;
        const bool more = (n_blocks - r + C - 1) / C > nbp;
        if (tv) {
            uint32_t qh[KS][2], ql[KS][2];
            tc_q_frags<KS>(sq, G, lane, qh, ql);
            float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.0f, 0.0f};
            float acc[KS][4];
#pragma unroll
            for (int mt = 0; mt < KS; ++mt)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[mt][e] = 0.0f;
            for (int i = 0; i < nbp; ++i)
                tc_warp_block<D>(sk + (size_t)i * L::tile, sv + (size_t)i * L::tile, 16 * w, kTcKeys, 0, 0.0f, scale, qh, ql, m_r,
                                 l_r, acc, pw, lane);
            if (more) {
                float* sb = pstate + ((((size_t)t * HKV + hk) * C + r) * kTcWarps + w) * 32 * kStateFloats(KS);
                tc_state_io<KS, true>(sb, lane, m_r, l_r, acc);
            } else {
                tc_store_warp<KS>(wm, wl, wo, w, lane, m_r, l_r, acc);
            }
        }
        // the two token slots share only the (read-only) prefix tiles: each
        // merges on its own 128-thread barrier (tv and more are the same for
        // the slot's four warps)
        if (tv && !more) {
            asm volatile("bar.sync %0, 128;" ::"r"(1 + slot) : "memory");   // warp partials written
            tc_merge_warps(wm, wl, wo, cm, cl, co, G, D, stid, 128);
            asm volatile("bar.sync %0, 128;" ::"r"(1 + slot) : "memory");   // the CTA partial written
            float* pp = part + ((size_t)(t * HKV + hk) * C + r) * dec_part_floats(G, D);
            if (stid < G) { pp[stid] = cm[stid]; pp[8 + stid] = cl[stid]; }
            for (int idx = stid; idx < G * D; idx += 128) pp[16 + idx] = co[(idx / D) * kMaxD + idx % D];
        }
    }
}

// ================================================================ prefill, tensor cores (fp16 KV)
// Causal attention for the T query tokens of one sequence (a prefill or a
// session's suffix): CTA = (16 consecutive query tokens, kv head); warp g
// takes query head g of the kv head's group, its 16 tokens as the MMA rows.
// 64-key K/V tiles of the sequence's pages come in by cp.async into a
// two-stage ring (rows padded to D + 8 halves); per tile the scores
// S[16 tokens][64 keys] = Q.K^T and O += P.V run on mma.sync m16n8k16 (f16
// in, f32 accumulation) in the register layout where the score accumulator
// is the next MMA's P operand; q and p are split into f16 high and low parts
// (x = hi + lo to about 2^-22 relative), both multiplied, so the products
// keep f32 accuracy; K and V are the cache's f16 values. Online softmax per
// row, causal mask j <= pos(token).
constexpr int kPfKeys = 64;
constexpr int kPfRows = 16;

template <int D>
struct PfSmem {
    static constexpr int RS = D + 8;                        // padded row (halves)
    static constexpr size_t tile = (size_t)kPfKeys * RS;    // halves of one K or V tile
    static constexpr size_t off_k = 0;                      // [2 stages][64][RS]
    static constexpr size_t off_v = off_k + 2 * tile * 2;
    static constexpr size_t bytes = off_v + 2 * tile * 2;
};

__device__ __forceinline__ void pf_cp16(void* dst, const void* src, bool valid) {
    const int n = valid ? 16 : 0;   // zero fill past the sequence
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void pf_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void pf_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int D>
__global__ void __launch_bounds__(32 * kMaxG) k_attn_prefill_tc(const float* __restrict__ q, int ldq, int T, int H,
                                                                 int HKV, float scale, KvView kv, int layer,
                                                                 float* __restrict__ out, int ldo) {
    using L = PfSmem<D>;
    constexpr int RS = L::RS, KS = D / 16, DN = D / 8;
    extern __shared__ __align__(128) uint8_t smem[];
    pdl_trigger();
    pdl_wait();
    const int G = H / HKV, hk = blockIdx.y, t0 = blockIdx.x * kPfRows;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, tig = lane & 3;
    const int nth = 32 * G;
    __half* sk = reinterpret_cast<__half*>(smem + L::off_k);
    __half* sv = reinterpret_cast<__half*>(smem + L::off_v);
    const int seq = kv.tok_seq[t0];
    const int tlast = min(T, t0 + kPfRows) - 1;
    const int pos_max = kv.tok_pos[tlast];
    const int n_tiles = (pos_max + kPfKeys) / kPfKeys;
    // this thread's two rows (tokens gid, gid + 8 of the tile) and their positions
    const int ta = t0 + gid, tb = t0 + gid + 8;
    const int pa = ta < T ? kv.tok_pos[ta] : -1, pb = tb < T ? kv.tok_pos[tb] : -1;
    // K and V rows of key tile kt (keys 64 kt ..) into stage st; rows past
    // pos_max are zero-filled (and masked below)
    auto load_tile = [&](int kt, int st) {
        constexpr int CH = D / 8;   // 16-byte chunks per row
        for (int i = tid; i < kPfKeys * CH; i += nth) {
            const int rr = i / CH, c = i % CH, j = kt * kPfKeys + rr;
            const bool ok = j <= pos_max;
            size_t off = 0;
            if (ok) {
                int page = kv.pt[(size_t)seq * kv.pt_stride + j / kv.page_size];
                if (page < 0 || page >= kv.n_pages) {
                    if (kv.err) atomicExch(kv.err, 5);
                    page = 0;
                }
                off = (size_t)page * kv.page_stride + (size_t)layer * kv.layer_stride + (size_t)hk * kv.head_stride +
                      (size_t)(j % kv.page_size) * D + 8 * c;
            }
            pf_cp16(sk + (size_t)st * L::tile + (size_t)rr * RS + 8 * c, reinterpret_cast<const __half*>(kv.k) + off, ok);
            pf_cp16(sv + (size_t)st * L::tile + (size_t)rr * RS + 8 * c, reinterpret_cast<const __half*>(kv.v) + off, ok);
        }
        pf_commit();
    };
    // key tiles wholly below every row's sliding window are skipped
    const int kt_lo = kv.window > 0 ? max(0, kv.tok_pos[t0] - kv.window + 1) / kPfKeys : 0;
    load_tile(kt_lo, kt_lo & 1);

    // q of this warp's head for the two rows as A fragments, hi and lo parts
    const int h = hk * G + warp;
    uint32_t qh[KS][4], ql[KS][4];
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int row = (e & 1) ? tb : ta, d = 16 * ks + 2 * tig + 8 * (e >> 1);
            const bool ok = row < T;
            const float x0 = ok ? q[(size_t)row * ldq + (size_t)h * D + d] : 0.0f;
            const float x1 = ok ? q[(size_t)row * ldq + (size_t)h * D + d + 1] : 0.0f;
            float h0, l0, h1, l1;
            split_h(x0, h0, l0);
            split_h(x1, h1, l1);
            qh[ks][e] = pack_h2(h0, h1);
            ql[ks][e] = pack_h2(l0, l1);
        }
    }
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.0f, 0.0f};
    float o[DN][4];
#pragma unroll
    for (int dn = 0; dn < DN; ++dn)
#pragma unroll
        for (int c = 0; c < 4; ++c) o[dn][c] = 0.0f;

    for (int kt = kt_lo; kt < n_tiles; ++kt) {
        if (kt + 1 < n_tiles) {
            load_tile(kt + 1, (kt + 1) & 1);
            pf_wait<1>();
        } else {
            pf_wait<0>();
        }
        __syncthreads();
        const __half* K = sk + (size_t)(kt & 1) * L::tile;
        const __half* V = sv + (size_t)(kt & 1) * L::tile;
        // S[16 rows][64 keys] in 8 n-tiles of 8 keys
        float s[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int c = 0; c < 4; ++c) s[nt][c] = 0.0f;
        const int mi = lane >> 3;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                uint32_t b[4];   // b0, b1 of n-tiles 2 np and 2 np + 1
                ldsm_x4(b, K + (size_t)(16 * np + (mi >> 1) * 8 + (lane & 7)) * RS + 16 * ks + (mi & 1) * 8);
                mma16816(s[2 * np], qh[ks], b[0], b[1]);
                mma16816(s[2 * np], ql[ks], b[0], b[1]);
                mma16816(s[2 * np + 1], qh[ks], b[2], b[3]);
                mma16816(s[2 * np + 1], ql[ks], b[2], b[3]);
            }
        }
        // scale, causal mask, online softmax per row (the row's 4 lanes hold its 64 keys)
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int j = kt * kPfKeys + 8 * nt + 2 * tig + (c & 1);
                const int pr = (c >> 1) ? pb : pa;
                s[nt][c] = j <= pr && (kv.window <= 0 || j > pr - kv.window)
                               ? soft_cap(__fmul_rn(s[nt][c], scale), kv.softcap) : -INFINITY;
                mx[c >> 1] = fmaxf(mx[c >> 1], s[nt][c]);
            }
        float corr[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 1));
            mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 2));
            const float mn = fmaxf(m_r[e], mx[e]);
            corr[e] = m_r[e] == -INFINITY ? 0.0f : expf(m_r[e] - mn);
            m_r[e] = mn;
        }
        float sum[2] = {0.0f, 0.0f};
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float p = s[nt][c] == -INFINITY ? 0.0f : expf(s[nt][c] - m_r[c >> 1]);
                s[nt][c] = p;
                sum[c >> 1] += p;
            }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            sum[e] += __shfl_xor_sync(0xffffffffu, sum[e], 1);
            sum[e] += __shfl_xor_sync(0xffffffffu, sum[e], 2);
            l_r[e] = __fmaf_rn(l_r[e], corr[e], sum[e]);
        }
#pragma unroll
        for (int dn = 0; dn < DN; ++dn) {
            o[dn][0] = __fmul_rn(o[dn][0], corr[0]);
            o[dn][1] = __fmul_rn(o[dn][1], corr[0]);
            o[dn][2] = __fmul_rn(o[dn][2], corr[1]);
            o[dn][3] = __fmul_rn(o[dn][3], corr[1]);
        }
        // O += P.V: P's accumulator fragments of n-tiles 2 kk, 2 kk + 1 are
        // the A fragment of k-step kk (keys 16 kk ..), hi and lo parts
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t ph[4], pl[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float* src = s[2 * kk + (e >> 1)] + 2 * (e & 1);
                float h0, l0, h1, l1;
                split_h(src[0], h0, l0);
                split_h(src[1], h1, l1);
                ph[e] = pack_h2(h0, h1);
                pl[e] = pack_h2(l0, l1);
            }
#pragma unroll
            for (int dp = 0; dp < DN / 2; ++dp) {
                uint32_t b[4];   // b0, b1 of d n-tiles 2 dp and 2 dp + 1
                ldsm_x4_t(b, V + (size_t)(16 * kk + (mi & 1) * 8 + (lane & 7)) * RS + 16 * dp + (mi >> 1) * 8);
                mma16816(o[2 * dp], ph, b[0], b[1]);
                mma16816(o[2 * dp], pl, b[0], b[1]);
                mma16816(o[2 * dp + 1], ph, b[2], b[3]);
                mma16816(o[2 * dp + 1], pl, b[2], b[3]);
            }
        }
        __syncthreads();   // the stage is read; the next load may overwrite it
    }
    // O / l for the two rows
#pragma unroll
    for (int dn = 0; dn < DN; ++dn)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int row = (c >> 1) ? tb : ta;
            if (row >= T) continue;
            const float l = l_r[c >> 1];
            out[(size_t)row * ldo + (size_t)h * D + 8 * dn + 2 * tig + (c & 1)] = l > 0.0f ? o[dn][c] / l : 0.0f;
        }
}

}  // namespace fb

using namespace fb;

extern "C" int fbk_rope_append(float* q, int ldq, const float* k, const float* v, int ldkv, int T, int H, int HKV,
                               int D, int rot, int neox, const float* rcos, const float* rsin, KvView kv, int layer,
                               cudaStream_t st) {
    if (T <= 0) return 0;
    return (int)fbk_launch(k_rope_append, dim3(T), dim3(256), 0, st, q, ldq, k, v, ldkv, H, HKV, D, rot, neox, rcos, rsin, kv,
                           layer);
}

// Keys per split: 32 per warp; contexts above 2048 use 4-warp CTAs so the
// number of splits (and the combine's work) stays <= 64.
static int attn_warps(int max_ctx) { return max_ctx > 2048 ? 4 : 1; }

// Scratch for calls of up to T tokens at any context up to max_ctx: a
// context of at most 2048 keys splits them 32 a CTA, a longer one 128 a CTA,
// so the most splits are at min(max_ctx, 2048) or at max_ctx.
extern "C" size_t fbk_attention_scratch_floats(int T, int H, int D, int max_ctx) {
    int n_splits = 0;
    for (const int ctx : {std::min(max_ctx, 2048), max_ctx}) {
        const int nw = attn_warps(ctx);
        n_splits = std::max(n_splits, (ctx + 32 * nw - 1) / (32 * nw));
    }
    return (size_t)T * H * n_splits * (D + 2);
}

// Scratch one fbk_attention call of T tokens with this max_ctx uses.
extern "C" size_t fbk_attention_call_floats(int T, int H, int D, int max_ctx) {
    const int nw = attn_warps(max_ctx);
    const int n_splits = (max_ctx + 32 * nw - 1) / (32 * nw);
    return (size_t)T * H * n_splits * (D + 2);
}

extern "C" int fbk_attention(const float* q, int ldq, int T, int H, int HKV, int D, float scale, KvView kv, int layer,
                             float* out, int ldo, float* scratch, size_t scratch_floats, int max_ctx, cudaStream_t st) {
    if (T <= 0) return 0;
    const int G = H / HKV;
    if (G > kMaxG || (D != 64 && D != 96 && D != 128)) return (int)cudaErrorInvalidValue;
    const int nw = attn_warps(max_ctx);
    const int n_splits = (max_ctx + 32 * nw - 1) / (32 * nw);
    if (fbk_attention_call_floats(T, H, D, max_ctx) > scratch_floats) return (int)cudaErrorInvalidValue;
    dim3 grid(n_splits, HKV, T);
    cudaError_t e;
    if (kv.f16) {
        if (nw == 1) e = fbk_launch(k_attn_split<true, 1>, grid, dim3(32), 0, st, q, ldq, H, HKV, D, scale, kv, layer, scratch, n_splits);
        else e = fbk_launch(k_attn_split<true, 4>, grid, dim3(128), 0, st, q, ldq, H, HKV, D, scale, kv, layer, scratch, n_splits);
    } else {
        if (nw == 1) e = fbk_launch(k_attn_split<false, 1>, grid, dim3(32), 0, st, q, ldq, H, HKV, D, scale, kv, layer, scratch, n_splits);
        else e = fbk_launch(k_attn_split<false, 4>, grid, dim3(128), 0, st, q, ldq, H, HKV, D, scale, kv, layer, scratch, n_splits);
    }
    if (e != cudaSuccess) return (int)e;
    return (int)fbk_launch(k_attn_combine, dim3(H, T), dim3(128), n_splits * sizeof(float), st, scratch, H, D, n_splits, out,
                           ldo);
}

// Cluster size of the decode attention: 16 CTAs when the device can host such
// clusters with this kernel's shared memory, else 8.
template <class E>
static int dec_cluster_size() {
    int c = 16;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(16, 1, 1);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = DecSmem<E>::bytes;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 16;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, k_attn_decode<E>, &cfg) != cudaSuccess || n < 1) {
        cudaGetLastError();
        c = 8;
    }
    return c;
}

template <class E>
static int launch_decode(const float* q, int ldq, const float* k, const float* v, int ldkv, int T, int H, int HKV,
                         int D, float scale, int rot, int neox, const float* rcos, const float* rsin, KvView kv,
                         int layer, float* out, int ldo, cudaStream_t st) {
    static int cluster = 0;
    if (!cluster) {
        cudaError_t e = cudaFuncSetAttribute(k_attn_decode<E>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)DecSmem<E>::bytes);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(k_attn_decode<E>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return (int)e;
        cluster = dec_cluster_size<E>();
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(cluster, HKV, T);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = DecSmem<E>::bytes;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = cluster;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    int na = 1;
    if (fbk_pdl_enabled()) {
        at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[1].val.programmaticStreamSerializationAllowed = 1;
        na = 2;
    }
    cfg.attrs = at;
    cfg.numAttrs = na;
    return (int)cudaLaunchKernelEx(&cfg, k_attn_decode<E>, q, ldq, k, v, ldkv, H, HKV, D, scale, rot, neox, rcos, rsin, kv,
                                   layer, out, ldo);
}

// Tensor-core decode attention for fp16 caches; cluster size as for the f32
// kernel. With part (batched decode) the ranks run as independent CTAs and a
// merge launch follows.
static int tc_cluster_size() {
    const char* ev = getenv("FISH_ATTN_CLUSTER");
    const int want = ev ? atoi(ev) : 16;
    return (want == 1 || want == 2 || want == 4 || want == 8) ? want : 16;
}

template <int D>
static int launch_decode_tc(const float* q, int ldq, const float* k, const float* v, int ldkv, int T, int H, int HKV,
                            float scale, int rot, int neox, const float* rcos, const float* rsin, KvView kv, int layer,
                            float* out, int ldo, float* part, const int* pre, float* pstate, cudaStream_t st) {
    static int cluster = 0;
    if (!cluster) {
        cudaError_t e = cudaFuncSetAttribute(k_attn_decode_tc<D, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)TcSmem::bytes);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_attn_decode_tc<D, false>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_attn_decode_tc<D, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)TcSmem::bytes);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_attn_prefix_tc<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)PreSmem::bytes);
        if (e != cudaSuccess) return (int)e;
        int c = tc_cluster_size();
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(c, 1, 1);
        cfg.blockDim = dim3(32 * kTcWarps);
        cfg.dynamicSmemBytes = TcSmem::bytes;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = c;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, k_attn_decode_tc<D, false>, &cfg) != cudaSuccess || n < 1) {
            cudaGetLastError();
            c = 8;
        }
        cluster = c;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(cluster, HKV, T);
    cfg.blockDim = dim3(32 * kTcWarps);
    cfg.dynamicSmemBytes = TcSmem::bytes;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    int na = 0;
    if (!part) {
        at[na].id = cudaLaunchAttributeClusterDimension;
        at[na].val.clusterDim.x = cluster;
        at[na].val.clusterDim.y = 1;
        at[na].val.clusterDim.z = 1;
        ++na;
    }
    if (fbk_pdl_enabled()) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = at;
    cfg.numAttrs = na;
    if (!part)
        return (int)cudaLaunchKernelEx(&cfg, k_attn_decode_tc<D, false>, q, ldq, k, v, ldkv, H, HKV, scale, rot, neox,
                                       rcos, rsin, kv, layer, out, ldo, (float*)nullptr, (const int*)nullptr,
                                       (const float*)nullptr);
    if (pre) {
        // the shared prefix once for all tokens (exits at once when there is none)
        cudaError_t e = fbk_launch(k_attn_prefix_tc<D>, dim3(cluster, HKV, (T + kPreTokens - 1) / kPreTokens), dim3(256),
                                   PreSmem::bytes, st, q, ldq, H, HKV, scale, rot, neox, rcos, rsin, kv, layer, T, pre,
                                   pstate, part);
        if (e != cudaSuccess) return (int)e;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_attn_decode_tc<D, true>, q, ldq, k, v, ldkv, H, HKV, scale, rot, neox,
                                       rcos, rsin, kv, layer, out, ldo, part, pre, (const float*)pstate);
    if (e != cudaSuccess) return (int)e;
    return (int)fbk_launch(k_attn_decode_merge, dim3(HKV, T), dim3(256), 0, st, (const float*)part, cluster, H / HKV,
                           D, HKV, out, ldo);
}

// Floats of the rank-partial scratch a batched decode of T tokens needs.
extern "C" size_t fbk_attention_decode_part_floats(int T, int H, int HKV, int D) {
    return (size_t)T * HKV * 16 * dec_part_floats(H / HKV, D);
}
extern "C" int fbk_attention_prefix_max_blocks(void) { return 16 * kPreMaxBlocks; }

template <int D>
static int launch_prefill_tc(const float* q, int ldq, int T, int H, int HKV, float scale, KvView kv, int layer,
                             float* out, int ldo, cudaStream_t st) {
    static const cudaError_t attr = cudaFuncSetAttribute(k_attn_prefill_tc<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                         (int)PfSmem<D>::bytes);
    if (attr != cudaSuccess) return (int)attr;
    return (int)fbk_launch(k_attn_prefill_tc<D>, dim3((T + kPfRows - 1) / kPfRows, HKV), dim3(32 * (H / HKV)),
                           PfSmem<D>::bytes, st, q, ldq, T, H, HKV, scale, kv, layer, out, ldo);
}

extern "C" int fbk_attention_prefill(const float* q, int ldq, int T, int H, int HKV, int D, float scale, KvView kv,
                                     int layer, float* out, int ldo, cudaStream_t st) {
    if (T <= 0) return 0;
    const int G = H / HKV;
    if (!kv.f16 || G > kMaxG || G * HKV != H || (D != 64 && D != 96 && D != 128) || kv.page_size != 16)
        return (int)cudaErrorInvalidValue;
    if (D == 128) return launch_prefill_tc<128>(q, ldq, T, H, HKV, scale, kv, layer, out, ldo, st);
    if (D == 96) return launch_prefill_tc<96>(q, ldq, T, H, HKV, scale, kv, layer, out, ldo, st);
    return launch_prefill_tc<64>(q, ldq, T, H, HKV, scale, kv, layer, out, ldo, st);
}
// Floats of the warp-state scratch of the shared-prefix kernel for T tokens.
extern "C" size_t fbk_attention_prefix_state_floats(int T, int HKV, int D) {
    return (size_t)T * HKV * 16 * kTcWarps * 32 * kStateFloats(D / 16);
}

extern "C" int fbk_attention_decode(const float* q, int ldq, const float* k, const float* v, int ldkv, int T, int H,
                                    int HKV, int D, float scale, int rot, int neox, const float* rcos, const float* rsin,
                                    KvView kv, int layer, float* out, int ldo, float* part, size_t part_floats,
                                    const int* pre, float* pstate, size_t pstate_floats, cudaStream_t st) {
    if (T <= 0) return 0;
    const int G = H / HKV;
    if (G > kMaxG || (D != 64 && D != 96 && D != 128) || kv.page_size != 16) return (int)cudaErrorInvalidValue;
    static const bool tc_off = getenv("FISH_ATTN_SIMT") != nullptr;
    static const bool batch_cluster = getenv("FISH_ATTN_CLUSTER_BATCH") != nullptr;
    if (kv.f16 && !tc_off) {
        // batches of tokens: independent rank CTAs + merge (same bits as one cluster per token)
        float* pp = (T > 1 && !batch_cluster && part && part_floats >= fbk_attention_decode_part_floats(T, H, HKV, D))
                        ? part : nullptr;
        static const bool no_prefix = getenv("FISH_ATTN_NO_PREFIX") != nullptr;
        // the shared-prefix kernel reads blocks for every token alike: no soft cap, no window
        const bool pf = pp && pre && pstate && !no_prefix && kv.softcap <= 0.0f && kv.window <= 0 &&
                        pstate_floats >= fbk_attention_prefix_state_floats(T, HKV, D);
        if (D == 128)
            return launch_decode_tc<128>(q, ldq, k, v, ldkv, T, H, HKV, scale, rot, neox, rcos, rsin, kv, layer, out, ldo,
                                         pp, pf ? pre : nullptr, pf ? pstate : nullptr, st);
        if (D == 96)
            return launch_decode_tc<96>(q, ldq, k, v, ldkv, T, H, HKV, scale, rot, neox, rcos, rsin, kv, layer, out, ldo,
                                        pp, pf ? pre : nullptr, pf ? pstate : nullptr, st);
        return launch_decode_tc<64>(q, ldq, k, v, ldkv, T, H, HKV, scale, rot, neox, rcos, rsin, kv, layer, out, ldo, pp,
                                    pf ? pre : nullptr, pf ? pstate : nullptr, st);
    }
    if (kv.f16) return launch_decode<__half>(q, ldq, k, v, ldkv, T, H, HKV, D, scale, rot, neox, rcos, rsin, kv, layer, out, ldo, st);
    return launch_decode<float>(q, ldq, k, v, ldkv, T, H, HKV, D, scale, rot, neox, rcos, rsin, kv, layer, out, ldo, st);
}

extern "C" int fbk_trace_set_attn(const fb::TraceState* s) { return (int)fb::trace_set(*s); }
