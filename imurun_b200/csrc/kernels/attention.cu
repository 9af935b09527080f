// attention.cu — RoPE, KV append into the paged cache, causal GQA attention.
//
// Reference behaviour: RoPE from the
// precomputed cos/sin table with pairs (2i, 2i+1) or NeoX (i, i+half)
// (src/ops.cpp:126-156), K/V rows stored at their position
// (src/model.cpp:1723-1731), and per (token, head) softmax attention over
// positions 0..pos with scale 1/sqrt(D) (src/ops.cpp:303-356). The KV cache is
// paged (P positions per page, every layer of a position range in one page)
// and fp16 or f32.
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "tma.cuh"

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
        const float s = valid ? __fmul_rn(sc[g], scale) : -INFINITY;
        m[g] = warp_max(s);
        sc[g] = valid ? expf(s - m[g]) : 0.0f;
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
                    } else {
                        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(reinterpret_cast<const __half*>(kv.v) + off));
                        vf[u][0] = a.x; vf[u][1] = a.y;
                    }
                } else {
                    if (dper == 4) {
                        const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(kv.v) + off);
                        vf[u][0] = a.x; vf[u][1] = a.y; vf[u][2] = a.z; vf[u][3] = a.w;
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
// split-K attention over the cached keys and the merge of the splits.
// CTA = (key split of KPS keys, kv head, token), 4 warps. The split's K and V
// page blocks (16 positions x D each, contiguous in the paged layout) land in
// shared memory by bulk copies; the CTA holding the token's own position
// rotates and stores the new k/v and patches its shared copy. Warps take 32
// keys each (lane = key for q.k, lane = a D-slice for p.V); the CTA merges
// its warps and writes (max, sum, o[D]) per head; the last CTA of a
// (token, kv head) to finish — an atomic counter, reset by that CTA — merges
// the splits into the output. Arithmetic follows k_rope_append, k_attn_split
// and k_attn_combine (src/ops.cpp:126-156, 303-356).
constexpr int kDecWarps = 4;

template <class E>
__device__ __forceinline__ void ld_chunk(const E* p, float (&f)[8]);
template <>
__device__ __forceinline__ void ld_chunk<__half>(const __half* p, float (&f)[8]) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float2 v = __half22float2(h[e]);
        f[2 * e] = v.x;
        f[2 * e + 1] = v.y;
    }
}
template <>
__device__ __forceinline__ void ld_chunk<float>(const float* p, float (&f)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
__device__ __forceinline__ float to_store(float x, __half*) { return __half2float(__float2half_rn(x)); }
__device__ __forceinline__ float to_store(float x, float*) { return x; }
__device__ __forceinline__ void put(__half* p, float x) { *p = __float2half_rn(x); }
__device__ __forceinline__ void put(float* p, float x) { *p = x; }

template <class E>
__host__ __device__ constexpr int dec_kps() { return sizeof(E) == 2 ? 128 : 64; }

// dynamic shared memory of k_attn_decode<E>
template <class E>
__host__ __device__ constexpr size_t dec_smem_bytes() {
    return 16 + 2 * (size_t)dec_kps<E>() * kMaxD * sizeof(E) +
           sizeof(float) * ((size_t)kMaxG * kMaxD + 2 * kDecWarps * kMaxG + (size_t)kDecWarps * kMaxG * kMaxD + 2 * kMaxD);
}

template <class E>
__global__ void __launch_bounds__(32 * kDecWarps) k_attn_decode(
    const float* __restrict__ q, int ldq, const float* __restrict__ knew, const float* __restrict__ vnew, int ldkv,
    int H, int HKV, int D, float scale, int rot, int neox, const float* __restrict__ rcos,
    const float* __restrict__ rsin, KvView kv, int layer, float* __restrict__ part, int n_splits,
    int* __restrict__ counters, float* __restrict__ out, int ldo) {
    constexpr int KPS = dec_kps<E>();
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_last;
    __shared__ volatile int s_abort;
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.z, hk = blockIdx.y, sp = blockIdx.x, G = H / HKV;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int pos = kv.tok_pos[t], n_keys = pos + 1, j0 = sp * KPS;
    if (j0 >= n_keys) return;
    const int n_active = (n_keys + KPS - 1) / KPS, nk = min(KPS, n_keys - j0);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
    E* sk = reinterpret_cast<E*>(smem + 16);
    E* sv = sk + (size_t)KPS * kMaxD;
    float* sq = reinterpret_cast<float*>(sv + (size_t)KPS * kMaxD);   // [G][D]
    float* swm = sq + kMaxG * kMaxD;                                    // [warp][G]
    float* swl = swm + kDecWarps * kMaxG;                               // [warp][G]
    float* swo = swl + kDecWarps * kMaxG;                               // [warp][G][D]
    float* snew = swo + kDecWarps * kMaxG * kMaxD;                     // [2][D]
    const int seq = kv.tok_seq[t];
    const int np = (nk + 15) / 16;
    const size_t blk = (size_t)16 * D;   // elements of one page's block of this head
    if (tid == 0) {
        s_abort = 0;
        mbar_init(bar, 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (tid == 0) {
        mbar_expect_tx(bar, (uint32_t)(2 * np * blk * sizeof(E)));
        for (int i = 0; i < np; ++i) {
            int page = kv.pt[(size_t)seq * kv.pt_stride + j0 / 16 + i];
            if (page < 0 || page >= kv.n_pages) {
                if (kv.err) atomicExch(kv.err, 5);
                page = 0;
            }
            const size_t off = (size_t)page * kv.page_stride + (size_t)layer * kv.layer_stride + (size_t)hk * kv.head_stride;
            bulk_g2s(sk + i * blk, reinterpret_cast<const E*>(kv.k) + off, (uint32_t)(blk * sizeof(E)), bar);
            bulk_g2s(sv + i * blk, reinterpret_cast<const E*>(kv.v) + off, (uint32_t)(blk * sizeof(E)), bar);
        }
    }
    // q heads of this kv head, rotated (biases and q-norm were applied upstream)
    const int half = rot / 2;
    const float* c = rcos + (size_t)pos * half;
    const float* s = rsin + (size_t)pos * half;
    const float* qr = q + (size_t)t * ldq + (size_t)hk * G * D;
    for (int idx = tid; idx < G * (D / 2); idx += 32 * kDecWarps) {
        const int g = idx / (D / 2), i = idx % (D / 2);
        const float* hv = qr + (size_t)g * D;
        if (i < half) {
            const int a = neox ? i : 2 * i, b = neox ? i + half : 2 * i + 1;
            const float x0 = hv[a], x1 = hv[b];
            sq[g * kMaxD + a] = __fsub_rn(__fmul_rn(x0, c[i]), __fmul_rn(x1, s[i]));
            sq[g * kMaxD + b] = __fadd_rn(__fmul_rn(x0, s[i]), __fmul_rn(x1, c[i]));
        } else {
            sq[g * kMaxD + 2 * i] = hv[2 * i];
            sq[g * kMaxD + 2 * i + 1] = hv[2 * i + 1];
        }
    }
    // the token's own position: rotate k, store k and v, keep their stored values
    const bool own = pos >= j0 && pos < j0 + KPS;
    if (own) {
        const float* kr = knew + (size_t)t * ldkv + (size_t)hk * D;
        const float* vr = vnew + (size_t)t * ldkv + (size_t)hk * D;
        const size_t base = kv_off(kv, layer, hk, t, pos);
        E* kp = reinterpret_cast<E*>(kv.k) + base;
        E* vp = reinterpret_cast<E*>(kv.v) + base;
        for (int i = tid; i < D / 2; i += 32 * kDecWarps) {
            int a, b;
            float k0, k1;
            if (i < half) {
                a = neox ? i : 2 * i;
                b = neox ? i + half : 2 * i + 1;
                const float x0 = kr[a], x1 = kr[b];
                k0 = __fsub_rn(__fmul_rn(x0, c[i]), __fmul_rn(x1, s[i]));
                k1 = __fadd_rn(__fmul_rn(x0, s[i]), __fmul_rn(x1, c[i]));
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
            snew[a] = to_store(k0, (E*)nullptr);
            snew[b] = to_store(k1, (E*)nullptr);
            snew[kMaxD + 2 * i] = to_store(vr[2 * i], (E*)nullptr);
            snew[kMaxD + 2 * i + 1] = to_store(vr[2 * i + 1], (E*)nullptr);
        }
    }
    const bool ok = mbar_wait(bar, 0, &s_abort);
    if (!ok) {
        s_abort = 1;
        if (kv.err) atomicExch(kv.err, 6);
    }
    __syncthreads();
    if (s_abort) {
        if (tid == 0) mbar_wait_bounded(bar, 0);   // let the copies land before the CTA exits
        return;
    }
    if (own) {
        const int r = pos - j0;
        for (int d = tid; d < D; d += 32 * kDecWarps) {
            put(sk + (size_t)r * D + d, snew[d]);
            put(sv + (size_t)r * D + d, snew[kMaxD + d]);
        }
    }
    __syncthreads();

    // scores: lane = key, 16-byte chunks visited in a lane-rotated order
    const int jw = 32 * warp;                    // this warp's first key in the split
    const int j = jw + lane;
    const bool valid = j < nk;
    const int nch = D / 8;                       // 8-element chunks per row
    float sc[kMaxG];
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) sc[g] = 0.0f;
    if (valid) {
        const E* krow = sk + (size_t)j * D;
        for (int cc = 0; cc < nch; ++cc) {
            const int ch = (cc + lane) % nch;
            float kf[8];
            ld_chunk<E>(krow + 8 * ch, kf);
#pragma unroll
            for (int g = 0; g < kMaxG; ++g) {
                if (g < G) {
                    const float4 qa = *reinterpret_cast<const float4*>(&sq[g * kMaxD + 8 * ch]);
                    const float4 qb = *reinterpret_cast<const float4*>(&sq[g * kMaxD + 8 * ch + 4]);
                    float v = sc[g];
                    v = fmaf(qa.x, kf[0], v); v = fmaf(qa.y, kf[1], v); v = fmaf(qa.z, kf[2], v); v = fmaf(qa.w, kf[3], v);
                    v = fmaf(qb.x, kf[4], v); v = fmaf(qb.y, kf[5], v); v = fmaf(qb.z, kf[6], v); v = fmaf(qb.w, kf[7], v);
                    sc[g] = v;
                }
            }
        }
    }
    const int nkw = max(0, min(32, nk - jw));    // keys of this warp
    float m[kMaxG], l[kMaxG];
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
        if (g >= G) break;
        const float sv_ = valid ? __fmul_rn(sc[g], scale) : -INFINITY;
        m[g] = warp_max(sv_);
        sc[g] = valid ? expf(sv_ - m[g]) : 0.0f;
        l[g] = warp_sum(sc[g]);
    }
    // p.V: lane owns dims [dper*lane, dper*lane + dper)
    const int dper = D / 32;
    float o[kMaxG][4];
#pragma unroll
    for (int g = 0; g < kMaxG; ++g)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[g][e] = 0.0f;
    for (int u = 0; u < nkw; ++u) {
        const E* vrow = sv + (size_t)(jw + u) * D + lane * dper;
        float vf[4];
        if (dper == 4) {
            if (sizeof(E) == 2) {
                const uint2 raw = *reinterpret_cast<const uint2*>(vrow);
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
                const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
                vf[0] = a.x; vf[1] = a.y; vf[2] = b.x; vf[3] = b.y;
            } else {
                const float4 a = *reinterpret_cast<const float4*>(vrow);
                vf[0] = a.x; vf[1] = a.y; vf[2] = a.z; vf[3] = a.w;
            }
        } else {
            if (sizeof(E) == 2) {
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(vrow));
                vf[0] = a.x; vf[1] = a.y;
            } else {
                const float2 a = *reinterpret_cast<const float2*>(vrow);
                vf[0] = a.x; vf[1] = a.y;
            }
            vf[2] = vf[3] = 0.0f;
        }
#pragma unroll
        for (int g = 0; g < kMaxG; ++g) {
            if (g >= G) break;
            const float p = __shfl_sync(0xffffffffu, sc[g], u);
#pragma unroll
            for (int e = 0; e < 4; ++e) o[g][e] = fmaf(p, vf[e], o[g][e]);
        }
    }
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
        if (g >= G) break;
        if (lane == 0) {
            swm[warp * kMaxG + g] = nkw > 0 ? m[g] : -INFINITY;
            swl[warp * kMaxG + g] = nkw > 0 ? l[g] : 0.0f;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e)
            if (e < dper) swo[((size_t)warp * kMaxG + g) * kMaxD + lane * dper + e] = o[g][e];
    }
    __syncthreads();
    // merge the warps into this split's (max, sum, o[D]) per head
    for (int idx = tid; idx < G * D; idx += 32 * kDecWarps) {
        const int g = idx / D, d = idx % D;
        float M = -INFINITY;
        for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, swm[w * kMaxG + g]);
        float L = 0.0f, O = 0.0f;
        for (int w = 0; w < kDecWarps; ++w) {
            const float mw = swm[w * kMaxG + g];
            if (mw == -INFINITY) continue;
            const float cw = expf(mw - M);
            L += swl[w * kMaxG + g] * cw;
            O += swo[((size_t)w * kMaxG + g) * kMaxD + d] * cw;
        }
        float* pp = part + (((size_t)t * H + (size_t)hk * G + g) * n_splits + sp) * (D + 2);
        if (d == 0) { pp[0] = M; pp[1] = L; }
        pp[2 + d] = O;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const int prev = atomicAdd(&counters[t * HKV + hk], 1);
        s_last = prev == n_active - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // last split of this (token, kv head): merge the splits (k_attn_combine)
    float* sw = swo;                      // [G][n_active] weights
    float* sL = swm;                      // [G]
    if (tid < G) {
        const int g = tid;
        const float* pg = part + ((size_t)t * H + (size_t)hk * G + g) * n_splits * (D + 2);
        float M = -INFINITY;
        for (int s2 = 0; s2 < n_active; ++s2) M = fmaxf(M, __ldcg(pg + (size_t)s2 * (D + 2)));
        float L = 0.0f;
        for (int s2 = 0; s2 < n_active; ++s2) {
            const float ms = __ldcg(pg + (size_t)s2 * (D + 2));
            const float w = ms == -INFINITY ? 0.0f : expf(ms - M);
            sw[g * n_active + s2] = w;
            if (w != 0.0f) L += __ldcg(pg + (size_t)s2 * (D + 2) + 1) * w;
        }
        sL[g] = L;
    }
    if (tid == 0) counters[t * HKV + hk] = 0;
    __syncthreads();
    for (int idx = tid; idx < G * D; idx += 32 * kDecWarps) {
        const int g = idx / D, d = idx % D;
        const float* pg = part + ((size_t)t * H + (size_t)hk * G + g) * n_splits * (D + 2);
        float O = 0.0f;
        for (int s2 = 0; s2 < n_active; ++s2) {
            const float w = sw[g * n_active + s2];
            if (w != 0.0f) O += __ldcg(pg + (size_t)s2 * (D + 2) + 2 + d) * w;
        }
        const float L = sL[g];
        out[(size_t)t * ldo + ((size_t)hk * G + g) * D + d] = L > 0.0f ? O / L : 0.0f;
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

extern "C" size_t fbk_attention_scratch_floats(int T, int H, int D, int max_ctx) {
    const int nw = attn_warps(max_ctx);
    const int n_splits = (max_ctx + 32 * nw - 1) / (32 * nw);
    return (size_t)T * H * n_splits * (D + 2);
}

extern "C" int fbk_attention(const float* q, int ldq, int T, int H, int HKV, int D, float scale, KvView kv, int layer,
                             float* out, int ldo, float* scratch, size_t scratch_floats, int max_ctx, cudaStream_t st) {
    if (T <= 0) return 0;
    const int G = H / HKV;
    if (G > kMaxG || (D != 64 && D != 128)) return (int)cudaErrorInvalidValue;
    const int nw = attn_warps(max_ctx);
    const int n_splits = (max_ctx + 32 * nw - 1) / (32 * nw);
    if ((size_t)T * H * n_splits * (D + 2) > scratch_floats) return (int)cudaErrorInvalidValue;
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

extern "C" size_t fbk_attention_decode_scratch_floats(int T, int H, int D, int max_ctx, int kv_f16) {
    const int kps = kv_f16 ? dec_kps<__half>() : dec_kps<float>();
    return (size_t)T * H * ((max_ctx + kps - 1) / kps) * (D + 2);
}

extern "C" int fbk_attention_decode(const float* q, int ldq, const float* k, const float* v, int ldkv, int T, int H,
                                    int HKV, int D, float scale, int rot, int neox, const float* rcos, const float* rsin,
                                    KvView kv, int layer, float* out, int ldo, float* scratch, size_t scratch_floats,
                                    int* counters, int max_ctx, cudaStream_t st) {
    if (T <= 0) return 0;
    const int G = H / HKV;
    if (G > kMaxG || (D != 64 && D != 128) || kv.page_size != 16 || !counters) return (int)cudaErrorInvalidValue;
    if (fbk_attention_decode_scratch_floats(T, H, D, max_ctx, kv.f16) > scratch_floats) return (int)cudaErrorInvalidValue;
    // the last split's merge keeps G x n_splits weights in the warp-output buffer
    const int kps = kv.f16 ? dec_kps<__half>() : dec_kps<float>();
    if ((size_t)G * ((max_ctx + kps - 1) / kps) > (size_t)kDecWarps * kMaxG * kMaxD) return (int)cudaErrorInvalidValue;
    cudaError_t e;
    if (kv.f16) {
        static bool attr = false;
        if (!attr) {
            e = cudaFuncSetAttribute(k_attn_decode<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)dec_smem_bytes<__half>());
            if (e != cudaSuccess) return (int)e;
            attr = true;
        }
        const int n_splits = (max_ctx + dec_kps<__half>() - 1) / dec_kps<__half>();
        e = fbk_launch(k_attn_decode<__half>, dim3(n_splits, HKV, T), dim3(32 * kDecWarps), dec_smem_bytes<__half>(), st,
                       q, ldq, k, v, ldkv, H, HKV, D, scale, rot, neox, rcos, rsin, kv, layer, scratch, n_splits,
                       counters, out, ldo);
    } else {
        static bool attr = false;
        if (!attr) {
            e = cudaFuncSetAttribute(k_attn_decode<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)dec_smem_bytes<float>());
            if (e != cudaSuccess) return (int)e;
            attr = true;
        }
        const int n_splits = (max_ctx + dec_kps<float>() - 1) / dec_kps<float>();
        e = fbk_launch(k_attn_decode<float>, dim3(n_splits, HKV, T), dim3(32 * kDecWarps), dec_smem_bytes<float>(), st,
                       q, ldq, k, v, ldkv, H, HKV, D, scale, rot, neox, rcos, rsin, kv, layer, scratch, n_splits,
                       counters, out, ldo);
    }
    return (int)e;
}
