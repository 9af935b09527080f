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
