// step.cu — persistent decode step: whole greedy decode steps of one
// sequence of a dense model in one cooperative launch.
//
// The decode step (reference src/model.cpp forward for one token: embedding,
// per layer RMSNorm -> q/k/v -> RoPE + KV append -> attention -> o + residual
// -> RMSNorm -> gate/up -> SwiGLU -> down + residual; final norm, output
// projection, argmax) runs as a sequence of phases separated by grid-wide
// barriers, one CTA per SM (its registers: no spills; its shared memory: a
// deep ring), all co-resident:
//   embed        x = dequantised embedding row of the token
//   GEMV phases  the streamed-GEMV job (stream_common.cuh) of one projection:
//                prologue (activation image), consumer pairs, row epilogue
//   attention    before each o projection: CTA (kv head, key chunk) items
//                write softmax partials; the o phase's prologue merges them
// The producer warp of each CTA never waits on a grid barrier: it walks the
// CTA's stages of every GEMV phase of every step in order and only waits for
// ring slots, so weight streaming runs on through prologues, attention and
// barriers (weights never depend on activations in a dense model). The
// argmax of step s becomes the token of step s + 1 without leaving the GPU.
//
// Every wait is bounded (ring slots, grid barriers: 2 s); a CTA that gives up
// records the failure in the control block, raises the abort flag and every
// CTA returns.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "dequant.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "layout.cuh"
#include "stream_common.cuh"
#include "tma.cuh"
#include "unit_math.cuh"

namespace fb {

constexpr int kStepThreads = 32 * (kConsumers + 1);
constexpr int kStepHdr = 1024;   // ring barriers (2 x kMaxStages x 8 B) and flags
constexpr int kAttnMinKeys = 64; // keys per attention work item at least

// Offset of a K/V row (sequence slot sid, position pos) in the paged pool.
__device__ __forceinline__ size_t kv_row(const KvView& kv, int sid, int layer, int head, int pos, volatile int* bad) {
    int page = kv.pt[(size_t)sid * kv.pt_stride + pos / kv.page_size];
    if (page < 0 || page >= kv.n_pages) {
        *bad = 1;
        page = 0;
    }
    return (size_t)page * kv.page_stride + (size_t)layer * kv.layer_stride + (size_t)head * kv.head_stride +
           (size_t)(pos % kv.page_size) * (kv.head_stride / kv.page_size);
}

__device__ __forceinline__ int attn_chunks(const StepArgs& A, int n_keys) {
    int c = (n_keys + kAttnMinKeys - 1) / kAttnMinKeys;
    return max(1, min(c, A.max_chunks));
}

// First failure wins the record; every failure raises the abort flag.
__device__ __noinline__ void step_fail(StepCtl* ctl, int code, int step, int phase, int stage, int slot,
                                       volatile int* s_abort) {
    if (atomicCAS(&ctl->err, 0, code) == 0) {
        ctl->info[0] = blockIdx.x;
        ctl->info[1] = step;
        ctl->info[2] = phase;
        ctl->info[3] = stage;
        ctl->info[4] = slot;
    }
    atomicExch(&ctl->abort, 1);
    *s_abort = 1;
}

// Grid barrier of the consumer warps (the producer warp never joins). Thread
// 0 publishes the CTA's writes (fence, then a release add) and spins with
// acquire loads; the CTA barriers around it order the other threads.
__device__ __forceinline__ bool grid_sync(const StepArgs& A, unsigned& target, volatile int* s_abort, int step,
                                          int phase) {
    consumers_sync();
    if (threadIdx.x == 0 && !*s_abort) {
        target += gridDim.x;
        __threadfence();
        atomicAdd(&A.ctl->bar, 1u);
        const unsigned long long t0 = gtimer();
        for (unsigned i = 1;; ++i) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(&A.ctl->bar) : "memory");
            if ((int)(v - target) >= 0) break;
            __nanosleep(32);
            if ((i & 255) == 0) {
                if (*reinterpret_cast<volatile int*>(&A.ctl->abort)) {
                    *s_abort = 1;
                    break;
                }
                if ((long long)(gtimer() - t0) > kWaitNs) {
                    step_fail(A.ctl, 2, step, phase, -1, -1, s_abort);
                    break;
                }
            }
        }
    }
    consumers_sync();
    return !*s_abort;
}

// Phase trace point (plain stores, no round trip): every thread counts the
// events, thread 0 of the first and the last CTA records the time.
__device__ __forceinline__ void strace(const StepArgs& A, int step, int& ev) {
    if (A.trace && threadIdx.x == 0 && (blockIdx.x == 0 || blockIdx.x == gridDim.x - 1) && ev < kStepTraceEvents)
        A.trace[((size_t)step * kStepTraceEvents + ev) * 2 + (blockIdx.x ? 1 : 0)] = gtimer();
    ++ev;
}

// x = embedding row tok (reference dequant_row): CTA b writes its slice.
__device__ __forceinline__ void embed_phase(const StepArgs& A, int tok) {
    const int E = A.E;
    const int i0 = (int)((long long)blockIdx.x * E / gridDim.x), i1 = (int)((long long)(blockIdx.x + 1) * E / gridDim.x);
    for (int i = i0 + (int)threadIdx.x; i < i1; i += kConsumers * 32) A.x[i] = dequant_at(A.emb_type, A.emb, E, tok, i);
}

// Attention of one token for one layer, work item (kv head h, key chunk c)
// per CTA (CTAs beyond HKV * C idle). q of the G heads of h and, in the chunk
// holding the token's own position, k are rotated with the RoPE table row
// (reference src/ops.cpp:126-156, the same float operations as
// k_rope_append); the token's K/V row is stored into the paged cache and used
// as stored (fp16-rounded for an fp16 cache). Scores q.k * scale, online
// softmax per warp (reference src/ops.cpp:303-356 computes the same softmax in
// two passes), then the warps' (m, l, acc) are merged into the CTA's partial.
// Warp w takes 8 keys per iteration (keys k0 + 8w .., stride 64): four lanes
// per key for the scores (32 dims each, lane = 4 key + part), one lane per 4
// output dims for P.V (D = 128). The chunk's page bases are read once into
// shared memory, and an iteration issues its K and V row loads together.
constexpr int kMaxChunkPages = 80;

template <int G, bool F16>
__device__ __forceinline__ void attention_phase(const StepArgs& A, int layer, int pos, float* scratch, volatile int* bad) {
    using E = typename std::conditional<F16, __half, float>::type;
    constexpr int D = 128, SQ = D + 4, KW = 8;
    const int H = A.H, HKV = A.HKV;
    const int n_keys = pos + 1;
    const int C = attn_chunks(A, n_keys);
    const int b = blockIdx.x;
    if (b >= HKV * C) return;
    const int h = b / C, c = b % C;
    const int k0 = (int)((long long)c * n_keys / C), k1 = (int)((long long)(c + 1) * n_keys / C);
    float* sq = scratch;                 // [G][D + 4]
    float* snew = sq + G * SQ;           // [2][D] k, v of the token as stored
    float* wpart = snew + 2 * D;         // [kConsumers][G][D + 2]
    size_t* sbase = reinterpret_cast<size_t*>(wpart + kConsumers * G * (D + 2));   // [kMaxChunkPages]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const KvView& kv = A.kv;
    const int ps = kv.page_size;
    const int pg0 = k0 / ps, np = (k1 - 1) / ps - pg0 + 1;
    const bool cached = np <= kMaxChunkPages;
    const size_t lh = (size_t)layer * kv.layer_stride + (size_t)h * kv.head_stride;
    if (cached) {
        for (int i = tid; i < np; i += kConsumers * 32) {
            int page = kv.pt[(size_t)A.sid * kv.pt_stride + pg0 + i];
            if (page < 0 || page >= kv.n_pages) {
                *bad = 1;
                page = 0;
            }
            sbase[i] = (size_t)page * kv.page_stride + lh;
        }
    }
    const int half = A.rot / 2;
    const float* cs = A.rcos + (size_t)pos * half;
    const float* sn = A.rsin + (size_t)pos * half;
    for (int idx = tid; idx < G * (D / 2); idx += kConsumers * 32) {
        const int g = idx / (D / 2), i = idx % (D / 2);
        const float* hv = A.q + (size_t)(h * G + g) * D;
        float* o = sq + g * SQ;
        if (i < half) {
            const int a = A.neox ? i : 2 * i, bb = A.neox ? i + half : 2 * i + 1;
            const float x0 = hv[a], x1 = hv[bb];
            o[a] = __fsub_rn(__fmul_rn(x0, cs[i]), __fmul_rn(x1, sn[i]));
            o[bb] = __fadd_rn(__fmul_rn(x0, sn[i]), __fmul_rn(x1, cs[i]));
        } else {
            o[2 * i] = hv[2 * i];
            o[2 * i + 1] = hv[2 * i + 1];
        }
    }
    if (k1 > pos) {   // the chunk holding the token's own position
        const float* kr = A.k + (size_t)h * D;
        const float* vr = A.v + (size_t)h * D;
        const size_t base = kv_row(kv, A.sid, layer, h, pos, bad);
        E* kp = reinterpret_cast<E*>(kv.k) + base;
        E* vp = reinterpret_cast<E*>(kv.v) + base;
        for (int i = tid; i < D / 2; i += kConsumers * 32) {
            int a, bb;
            float q0, q1;
            if (i < half) {
                a = A.neox ? i : 2 * i;
                bb = A.neox ? i + half : 2 * i + 1;
                const float x0 = kr[a], x1 = kr[bb];
                q0 = __fsub_rn(__fmul_rn(x0, cs[i]), __fmul_rn(x1, sn[i]));
                q1 = __fadd_rn(__fmul_rn(x0, sn[i]), __fmul_rn(x1, cs[i]));
            } else {
                a = 2 * i;
                bb = 2 * i + 1;
                q0 = kr[a];
                q1 = kr[bb];
            }
            const float v0 = vr[2 * i], v1 = vr[2 * i + 1];
            if (F16) {
                const __half hk0 = __float2half_rn(q0), hk1 = __float2half_rn(q1);
                const __half hv0 = __float2half_rn(v0), hv1 = __float2half_rn(v1);
                reinterpret_cast<__half*>(kp)[a] = hk0;
                reinterpret_cast<__half*>(kp)[bb] = hk1;
                reinterpret_cast<__half*>(vp)[2 * i] = hv0;
                reinterpret_cast<__half*>(vp)[2 * i + 1] = hv1;
                snew[a] = __half2float(hk0);
                snew[bb] = __half2float(hk1);
                snew[D + 2 * i] = __half2float(hv0);
                snew[D + 2 * i + 1] = __half2float(hv1);
            } else {
                reinterpret_cast<float*>(kp)[a] = q0;
                reinterpret_cast<float*>(kp)[bb] = q1;
                reinterpret_cast<float*>(vp)[2 * i] = v0;
                reinterpret_cast<float*>(vp)[2 * i + 1] = v1;
                snew[a] = q0;
                snew[bb] = q1;
                snew[D + 2 * i] = v0;
                snew[D + 2 * i + 1] = v1;
            }
        }
    }
    consumers_sync();

    auto row_off = [&](int j) -> size_t {
        const size_t base = cached ? sbase[j / ps - pg0] : kv_row(kv, A.sid, layer, h, j, bad) - (size_t)(j % ps) * D;
        return base + (size_t)(j % ps) * D;
    };
    const int kk = lane >> 2, part = lane & 3;
    float m[G], l[G], acc[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[g][i] = 0.0f;
    }
    constexpr int KV4 = F16 ? 4 : 8;   // 16-byte loads per lane for 32 dims of a K row
    for (int j0 = k0 + warp * KW; j0 < k1; j0 += kConsumers * KW) {
        const int j = j0 + kk;
        const bool valid = j < k1;
        const int nk = min(KW, k1 - j0);
        // loads first: this lane's 32 dims of its key's K row and (fp16
        // cache) the V rows of the iteration's keys, this lane's 4 dims; for
        // an fp32 cache the V loads follow the scores (register budget)
        using V4 = typename std::conditional<F16, uint2, float4>::type;
        V4 vr[KW];
        auto load_v = [&]() {
#pragma unroll
            for (int q2 = 0; q2 < KW; ++q2)
                if (q2 < nk && j0 + q2 != pos)
                    vr[q2] = *reinterpret_cast<const V4*>(reinterpret_cast<const E*>(kv.v) + row_off(j0 + q2) + 4 * lane);
        };
        uint4 kr4[KV4];
        const bool from_cache = valid && j != pos;
        if (from_cache) {
            const uint4* kp = reinterpret_cast<const uint4*>(reinterpret_cast<const E*>(kv.k) + row_off(j) + 32 * part);
#pragma unroll
            for (int i = 0; i < KV4; ++i) kr4[i] = kp[i];
        }
        if (F16) load_v();
        float s[G];
#pragma unroll
        for (int g = 0; g < G; ++g) s[g] = 0.0f;
        if (from_cache) {
#pragma unroll
            for (int i = 0; i < KV4; ++i) {
                if (F16) {
                    const __half2* hp = reinterpret_cast<const __half2*>(&kr4[i]);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = __half22float2(hp[e]);
#pragma unroll
                        for (int g = 0; g < G; ++g) {
                            const float2 q2v = *reinterpret_cast<const float2*>(sq + g * SQ + 32 * part + 8 * i + 2 * e);
                            s[g] = fmaf(q2v.x, f.x, s[g]);
                            s[g] = fmaf(q2v.y, f.y, s[g]);
                        }
                    }
                } else {
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const float4 q4 = *reinterpret_cast<const float4*>(sq + g * SQ + 32 * part + 4 * i);
                        s[g] = fmaf(q4.x, __uint_as_float(kr4[i].x), s[g]);
                        s[g] = fmaf(q4.y, __uint_as_float(kr4[i].y), s[g]);
                        s[g] = fmaf(q4.z, __uint_as_float(kr4[i].z), s[g]);
                        s[g] = fmaf(q4.w, __uint_as_float(kr4[i].w), s[g]);
                    }
                }
            }
        } else if (valid) {   // the token's own key
            for (int d = 0; d < 32; ++d) {
                const float kd = snew[32 * part + d];
#pragma unroll
                for (int g = 0; g < G; ++g) s[g] = fmaf(sq[g * SQ + 32 * part + d], kd, s[g]);
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float dot = s[g];
            dot += __shfl_xor_sync(0xffffffffu, dot, 1);
            dot += __shfl_xor_sync(0xffffffffu, dot, 2);
            s[g] = valid ? dot * A.scale : -INFINITY;
        }
        if (!F16) load_v();
        float p[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float mx = s[g];
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float mn = fmaxf(m[g], mx);   // finite: key j0 is valid
            const float fac = m[g] == -INFINITY ? 0.0f : expf(m[g] - mn);
            m[g] = mn;
            p[g] = valid ? expf(s[g] - mn) : 0.0f;
            float sum = p[g];
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            sum += __shfl_xor_sync(0xffffffffu, sum, 8);
            sum += __shfl_xor_sync(0xffffffffu, sum, 16);
            l[g] = l[g] * fac + sum;
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[g][i] *= fac;
        }
#pragma unroll
        for (int q2 = 0; q2 < KW; ++q2) {
            if (q2 >= nk) break;
            float vv[4];
            if (j0 + q2 == pos) {
#pragma unroll
                for (int i = 0; i < 4; ++i) vv[i] = snew[D + 4 * lane + i];
            } else if (F16) {
                const uint2 u = *reinterpret_cast<const uint2*>(&vr[q2]);
                const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
                const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
                vv[0] = f0.x; vv[1] = f0.y; vv[2] = f1.x; vv[3] = f1.y;
            } else {
                const float4 u = *reinterpret_cast<const float4*>(&vr[q2]);
                vv[0] = u.x; vv[1] = u.y; vv[2] = u.z; vv[3] = u.w;
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float pg = __shfl_sync(0xffffffffu, p[g], 4 * q2);
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[g][i] = fmaf(pg, vv[i], acc[g][i]);
            }
        }
    }
    // warp partials, then the CTA's partial of each head
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float* wp = wpart + (size_t)(warp * G + g) * (D + 2);
#pragma unroll
        for (int i = 0; i < 4; ++i) wp[4 * lane + i] = acc[g][i];
        if (lane == 0) {
            wp[D] = m[g];
            wp[D + 1] = l[g];
        }
    }
    consumers_sync();
    float* out_acc = A.att_part;
    float* out_ml = A.att_part + (size_t)C * H * D;
    for (int idx = tid; idx < G * D; idx += kConsumers * 32) {
        const int g = idx / D, d = idx % D;
        float M = -INFINITY;
        for (int w = 0; w < kConsumers; ++w) M = fmaxf(M, wpart[(size_t)(w * G + g) * (D + 2) + D]);
        float den = 0.0f, a = 0.0f;
        for (int w = 0; w < kConsumers; ++w) {
            const float* wp = wpart + (size_t)(w * G + g) * (D + 2);
            if (!(wp[D] > -INFINITY)) continue;   // a warp without keys
            const float f = expf(wp[D] - M);
            den += f * wp[D + 1];
            a += f * wp[d];
        }
        const size_t hq = (size_t)c * H + h * G + g;
        out_acc[hq * D + d] = a;
        if (d == 0) {
            out_ml[2 * hq] = M;
            out_ml[2 * hq + 1] = den;
        }
    }
}

// This CTA's tiles of a phase (balanced split of the units over the grid).
__device__ __forceinline__ void phase_tiles(int n_units, int pair, int n_tiles, int& t_begin, int& t_end) {
    const int unit = pair ? 2 : 1;
    t_begin = (int)((long long)blockIdx.x * n_units / gridDim.x) * unit;
    t_end = min(n_tiles, (int)((long long)(blockIdx.x + 1) * n_units / gridDim.x) * unit);
}

__device__ __forceinline__ int n_tiles_of(const int* tile0, int nseg) {
    int n = tile0[0];
#pragma unroll
    for (int i = 1; i <= kMaxSeg; ++i)
        if (i == nseg) n = tile0[i];
    return n;
}

// Copy a phase descriptor's GEMV job into shared memory (threads [t0, t0 + nt)).
__device__ __forceinline__ void load_phase(const StepPhase* gp, GemvArgs* s_args, int* s_tile0, int* s_meta, int tid,
                                           int nt) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(&gp->a);
    uint32_t* dst = reinterpret_cast<uint32_t*>(s_args);
    for (int i = tid; i < (int)(sizeof(GemvArgs) / 4); i += nt) dst[i] = __ldg(src + i);
    if (tid <= kMaxSeg) s_tile0[tid] = __ldg(gp->tile0 + tid);
    if (tid == 0) {
        s_meta[0] = __ldg(&gp->n_units);
        s_meta[1] = __ldg(&gp->G);
        s_meta[2] = __ldg(&gp->xk_bytes);
        s_meta[3] = __ldg(&gp->x32_bytes);
        s_meta[4] = __ldg(&gp->attn_layer);
    }
}

// Dynamic shared memory of the step kernel: [0, 256) full barriers, [256, 512)
// empty barriers, 512 abort flag, 516 issued-stage count, [1024, 1024 + U)
// the union area (activation image + row partials, or attention scratch),
// then the ring. Addressed from this symbol, so helpers need no pointers.
extern __shared__ __align__(128) uint8_t g_step_smem[];
__device__ __forceinline__ uint64_t* st_full() { return reinterpret_cast<uint64_t*>(g_step_smem); }
__device__ __forceinline__ uint64_t* st_empty() { return reinterpret_cast<uint64_t*>(g_step_smem) + kMaxStages; }
__device__ __forceinline__ volatile int* st_abort() { return reinterpret_cast<volatile int*>(g_step_smem + 2 * kMaxStages * 8); }
__device__ __forceinline__ volatile int* st_issued() {
    return reinterpret_cast<volatile int*>(g_step_smem + 2 * kMaxStages * 8 + 4);
}
__device__ __forceinline__ uint8_t* st_uni() { return g_step_smem + kStepHdr; }

__device__ __forceinline__ RingView step_ring(const StepArgs& A, unsigned long long* pw, unsigned long long* cw) {
    RingView rg;
    rg.base = st_uni() + A.union_bytes;
    rg.full = st_full();
    rg.empty = st_empty();
    rg.S = A.S;
    rg.slot_bytes = A.slot_bytes;
    rg.issued = st_issued();
    rg.abort = st_abort();
    rg.guard = 1;   // phases start at arbitrary ring stages
    rg.pwait = pw;
    rg.cwait = cw;
    return rg;
}

// Prologue of a GEMV phase, out of line with only shared-memory pointers and
// integers as parameters (no local copies): the activation image for K
// inputs, both layouts as requested.
__device__ __noinline__ void step_prologue(const GemvArgs* sa, int xk, int x32, double* s_part) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = sa->K;
    float wv[kNormRegs][8];
    if (sa->pro.mode == PRO_NORM) {
#pragma unroll
        for (int k = 0; k < kNormRegs; ++k) {
            const int c = warp + kConsumers * k;
            if (c * 256 < K) ld8(sa->pro.w, c * 256 + 8 * lane, K, wv[k]);
        }
    }
    XImage xi;
    xi.base = st_uni();
    xi.n256 = (K + 255) / 256;
    xi.xk = xk;
    xi.x32 = x32;
    xi.T = 1;
    build_ximage(*sa, xi, xk > 0, x32 > 0, s_part, wv, -1);
}

// Consumer side of one GEMV phase (descriptor in s_args / s_tile0 / s_meta):
// activation image, the CTA's stages from ring stage gbase on, row epilogue.
// Returns the phase's stage count of this CTA, or -1 when a wait gave up
// (failure recorded). The job and ring views are built after the prologue so
// they are not live across it.
__device__ __forceinline__ int gemv_phase(const StepArgs& A, GemvArgs& s_args, const int* s_tile0, const int* s_meta,
                                          double* s_part, unsigned long long (*s_best)[kMaxStreamTokens], unsigned long long* cw,
                                          int gbase, int step, int p, int& ev) {
    int t_begin, t_end;
    phase_tiles(s_meta[0], s_args.swiglu, n_tiles_of(s_tile0, s_args.nseg), t_begin, t_end);
    // a single residual-add segment (o, down): its y rows are read before the
    // stages, so the epilogue makes no dependent global read
    const int n_rows = max(0, t_end - t_begin) * kTileRows;
    const bool add1 = s_args.nseg == 1 && !s_args.swiglu && s_args.seg[0].epi == EPI_ADD && !s_args.seg[0].amax &&
                      n_rows <= 2 * kConsumers * 32;
    float ypre[2] = {0.0f, 0.0f};
    if (add1) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int idx = threadIdx.x + k * kConsumers * 32, row = t_begin * kTileRows + idx;
            if (idx < n_rows && row < s_args.seg[0].rows) ypre[k] = s_args.seg[0].y[row];
        }
    }
    step_prologue(&s_args, s_meta[2], s_meta[3], s_part);
    consumers_sync();
    strace(A, step, ev);
    JobView jv;
    jv.seg = s_args.seg;
    jv.tile0 = s_tile0;
    jv.nseg = s_args.nseg;
    jv.pair = s_args.swiglu;
    jv.G = s_meta[1];
    jv.K = s_args.K;
    jv.T = 1;
    jv.t_begin = t_begin;
    jv.t_end = t_end;
    XImage xi;
    xi.base = st_uni();
    xi.n256 = (jv.K + 255) / 256;
    xi.xk = s_meta[2];
    xi.x32 = s_meta[3];
    xi.T = 1;
    float* part = reinterpret_cast<float*>(st_uni() + xi.xk + xi.x32);
    {
        const RingView rg = step_ring(A, nullptr, cw);
        WaitFail wf{};
        if (!consume_stages_w<1>(rg, jv, gbase, xi, part, &wf)) {
            if (!*rg.abort) step_fail(A.ctl, 1, step, p, wf.stage, wf.slot, rg.abort);
            *rg.abort = 1;
        }
    }
    consumers_sync();
    strace(A, step, ev);
    if (*st_abort()) return -1;
    if (add1) {   // store_out's arithmetic: + bias, + y
        const GemvSeg& g0 = s_args.seg[0];
        const int G = jv.G;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int idx = threadIdx.x + k * kConsumers * 32, row = t_begin * kTileRows + idx;
            if (idx < n_rows && row < g0.rows) {
                const int tl = idx / kTileRows, rr = idx % kTileRows;
                float v = 0.0f;
                for (int gi = 0; gi < G; ++gi) v += part[(size_t)(tl * G + gi) * kTileRows + rr];
                if (g0.bias) v += g0.bias[row];
                v += ypre[k];
                g0.y[row] = v;
            }
        }
    } else {
        reduce_rows<1>(jv, part, s_best);
    }
    strace(A, step, ev);
    if (cw && threadIdx.x == 0 && p < 200) {   // consumer warp 0's wait for data in this phase
        A.trace[((size_t)step * kStepTraceEvents + 601 + 2 * p) * 2 + (blockIdx.x ? 1 : 0)] = *cw + 1;
        *cw = 0;
    }
    return job_stages(jv);
}

// G (q heads per kv head) and the KV element type are template parameters so
// only one attention variant is compiled into a kernel, and the whole kernel
// is inlined: it uses no local memory (with shared memory taking most of an
// SM's 256 KB, local memory would live in L2).
template <int G, bool F16>
__global__ void __launch_bounds__(kStepThreads, 1) k_step(StepArgs A) {
    uint64_t* full = st_full();
    uint64_t* empty = st_empty();
    volatile int* s_abort = st_abort();
    volatile int* s_issued = st_issued();
    uint8_t* uni = st_uni();
    __shared__ GemvArgs s_args2[2];      // consumers: current and next phase
    __shared__ int s_tile02[2][kMaxSeg + 1];
    __shared__ int s_meta2[2][8];
    __shared__ GemvArgs p_args;          // producer's current phase
    __shared__ int p_tile0[kMaxSeg + 1];
    __shared__ int p_meta[8];
    __shared__ double s_part[kNormWarps];
    __shared__ unsigned long long s_best[kConsumers][kMaxStreamTokens];
    __shared__ int s_bad;
    volatile int* sbad = &s_bad;
    __shared__ int s_gbase, s_tok;         // consumers: ring stage of the phase, current token
    __shared__ unsigned s_target;          // thread 0: barrier arrivals to wait for

    __shared__ unsigned long long s_pwait, s_cwait;
    const bool traced = A.trace && (blockIdx.x == 0 || blockIdx.x == gridDim.x - 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        *s_abort = 0;
        *s_issued = 0;
        s_bad = 0;
        s_pwait = 0;
        s_cwait = 0;
        for (int s = 0; s < A.S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);   // the consuming warp
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kConsumers) {   // producer warp: lane 0 issues, the warp copies descriptors
        int g = 0;
        bool ok = true;
        for (int step = 0; step < A.n_steps && ok; ++step) {
            for (int p = 0; p < A.n_ph && ok; ++p) {
                __syncwarp();
                load_phase(A.ph + p, &p_args, p_tile0, p_meta, lane, 32);
                __syncwarp();
                if (lane == 0) {
                    JobView jv;
                    jv.seg = p_args.seg;
                    jv.tile0 = p_tile0;
                    jv.nseg = p_args.nseg;
                    jv.pair = p_args.swiglu;
                    jv.G = p_meta[1];
                    jv.K = p_args.K;
                    jv.T = 1;
                    phase_tiles(p_meta[0], jv.pair, n_tiles_of(p_tile0, jv.nseg), jv.t_begin, jv.t_end);
                    WaitFail wf{};
                    const RingView rg = step_ring(A, traced ? &s_pwait : nullptr, nullptr);
                    if (!produce_stages(rg, jv, g, &A.ctl->err, &wf)) {
                        if (!*s_abort) step_fail(A.ctl, 1, step, p, wf.stage, wf.slot, s_abort);
                        // let the copies in flight land before the CTA can exit
                        for (int k = max(0, wf.stage - A.S); k < wf.stage; ++k)
                            mbar_wait_bounded(&full[k % A.S], (uint32_t)((k / A.S) & 1));
                        ok = false;
                    } else {
                        g += job_stages(jv);
                        if (traced && p < 200)   // cumulative producer wait when phase p was fully issued
                            A.trace[((size_t)step * kStepTraceEvents + 600 + 2 * p) * 2 + (blockIdx.x ? 1 : 0)] = s_pwait + 1;
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            }
        }
        return;
    }

    // consumers. Phase descriptors are double-buffered: each thread holds one
    // word of the next phase's descriptor in a register while the current
    // phase runs and stores it before the phase's grid barrier.
    constexpr int kArgWords = (int)(sizeof(GemvArgs) / 4);
    static_assert(kArgWords + (kMaxSeg + 1) + 5 <= kConsumers * 32, "descriptor words per thread");
    const int tid = threadIdx.x;
    auto desc_word = [&](int ph) -> uint32_t {
        const StepPhase* gp = A.ph + ph;
        if (tid < kArgWords) return __ldg(reinterpret_cast<const uint32_t*>(&gp->a) + tid);
        if (tid < kArgWords + kMaxSeg + 1) return (uint32_t)__ldg(gp->tile0 + (tid - kArgWords));
        switch (tid - kArgWords - (kMaxSeg + 1)) {
            case 0: return (uint32_t)__ldg(&gp->n_units);
            case 1: return (uint32_t)__ldg(&gp->G);
            case 2: return (uint32_t)__ldg(&gp->xk_bytes);
            case 3: return (uint32_t)__ldg(&gp->x32_bytes);
            case 4: return (uint32_t)__ldg(&gp->attn_layer);
            default: return 0u;
        }
    };
    auto desc_store = [&](int buf, uint32_t w) {
        if (tid < kArgWords) reinterpret_cast<uint32_t*>(&s_args2[buf])[tid] = w;
        else if (tid < kArgWords + kMaxSeg + 1) s_tile02[buf][tid - kArgWords] = (int)w;
        else if (tid < kArgWords + kMaxSeg + 6) s_meta2[buf][tid - kArgWords - (kMaxSeg + 1)] = (int)w;
    };
    desc_store(0, desc_word(0));
    if (tid == 0) {
        s_gbase = 0;
        s_tok = A.ids[0];
        s_target = 0;
    }
    consumers_sync();
    int cur = 0;
    for (int step = 0; step < A.n_steps; ++step) {
        const int pos = A.tok_pos[0] + step;
        const int tok = s_tok;
        if (tok < 0 || tok >= A.emb_rows) {
            if (threadIdx.x == 0) step_fail(A.ctl, 4, step, -1, tok, -1, s_abort);
            return;
        }
        int ev = 0;
        embed_phase(A, tok);
        if (!grid_sync(A, s_target, s_abort, step, -1)) return;
        strace(A, step, ev);
        if (blockIdx.x == 0 && threadIdx.x == 0) A.keys[(step + 1) & 1] = 0ull;   // every CTA has read it
        for (int p = 0; p < A.n_ph; ++p) {
            const uint32_t nxt = desc_word(p + 1 < A.n_ph ? p + 1 : 0);   // in flight during this phase
            GemvArgs& sa = s_args2[cur];
            const int attn_layer = s_meta2[cur][4];
            if (attn_layer >= 0) {
                attention_phase<G, F16>(A, attn_layer, pos, reinterpret_cast<float*>(uni), sbad);
                strace(A, step, ev);
                if (!grid_sync(A, s_target, s_abort, step, p)) return;
                strace(A, step, ev);
            }
            if (threadIdx.x == 0) {
                if (sa.seg[0].amax) sa.seg[0].amax = A.keys + (step & 1);
                if (sa.pro.mode == PRO_MERGE) sa.pro.ld = attn_chunks(A, pos + 1);
            }
            consumers_sync();
            const int n_st = gemv_phase(A, sa, s_tile02[cur], s_meta2[cur], s_part, s_best, traced ? &s_cwait : nullptr,
                                        s_gbase, step, p, ev);
            if (n_st < 0) return;
            desc_store(cur ^ 1, nxt);
            if (tid == 0) s_gbase += n_st;   // read again after the barrier
            if (!grid_sync(A, s_target, s_abort, step, p)) return;
            strace(A, step, ev);
            cur ^= 1;
        }
        // the output phase's argmax is the next token
        if (tid == 0) {
            const int nt = argmax_index(A.keys[step & 1]);
            s_tok = nt;
            if (blockIdx.x == 0) A.out[step] = nt;
        }
        consumers_sync();
    }
    if (threadIdx.x == 0 && s_bad) atomicCAS(&A.ctl->err, 0, 5);
}

}  // namespace fb

using namespace fb;

using StepKernel = void (*)(StepArgs);

static StepKernel step_kernel(int G, int f16) {
    switch (G * 2 + (f16 ? 1 : 0)) {
        case 2: return k_step<1, false>;
        case 3: return k_step<1, true>;
        case 4: return k_step<2, false>;
        case 5: return k_step<2, true>;
        case 8: return k_step<4, false>;
        case 9: return k_step<4, true>;
        case 16: return k_step<8, false>;
        case 17: return k_step<8, true>;
        default: return nullptr;
    }
}

extern "C" int fbk_step_plan(int G, int f16, int slot_bytes, int union_bytes, int* grid, int* stages, size_t* smem) {
    const StepKernel kern = step_kernel(G, f16);
    if (!kern) return -1;
    int dev = 0, sms = 0, per_sm = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa{};
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return (int)e;
    // one CTA per SM: the SM's shared memory less the per-CTA reservation and
    // the static part
    const int per_cta = std::min(optin, per_sm - 1024) - (int)fa.sharedSizeBytes;
    const int ring = per_cta - kStepHdr - ((union_bytes + 127) / 128 * 128);
    const int S = std::min(kMaxStages, ring > 0 ? ring / slot_bytes : 0);
    if (S < 2) return -1;
    const size_t dyn = (size_t)kStepHdr + (union_bytes + 127) / 128 * 128 + (size_t)S * slot_bytes;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
    if (e != cudaSuccess) return (int)e;
    int occ = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kStepThreads, dyn);
    if (e != cudaSuccess) return (int)e;
    if (occ < 1) return -1;
    *grid = sms;
    *stages = S;
    *smem = dyn;
    return 0;
}

extern "C" int fbk_step_decode(const StepArgs* a, int grid, size_t smem, cudaStream_t st) {
    const StepKernel kern = step_kernel(a->H / a->HKV, a->kv.f16);
    if (!kern) return (int)cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kStepThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return (int)cudaLaunchKernelEx(&cfg, kern, *a);
}
