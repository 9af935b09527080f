// misc.cu — embedding gather, residual add, argmax, MoE routing.
#include "common.cuh"
#include "dequant.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "layout.cuh"
#include "trace.cuh"

namespace fb {

// grid (ceil(E / 256), T): one value per thread
__global__ void k_embed(int type, const uint8_t* __restrict__ w, int E, int n_rows, const int32_t* __restrict__ ids,
                        float* __restrict__ x, int ldx, int* err) {
    pdl_trigger();
    const bool tr = tracing() && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0;
    const int tseq = tr ? trace_launch(TR_EMBED) : 0;
    if (tr) trace_ev(TR_EMBED, EV_START, tseq);
    pdl_wait();
    if (tr) trace_ev(TR_EMBED, EV_END, tseq);
    const int t = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
    int row = ids[t];
    if (row < 0 || row >= n_rows) {
        if (err && i == 0) atomicExch(err, 4);
        row = 0;
    }
    if (i < E) x[(size_t)t * ldx + i] = dequant_at(type, w, E, row, i);
}

__global__ void k_argmax_from_keys(unsigned long long* keys, int T, int32_t* out) {
    pdl_trigger();
    pdl_wait();
    const int t = threadIdx.x;
    if (t < T) {
        out[t] = argmax_index(keys[t]);
        keys[t] = 0ull;
    }
}

__global__ void k_greedy_from_keys(unsigned long long* keys, int32_t* ids, int32_t* tok_pos, int32_t* out,
                                   int32_t* step) {
    pdl_trigger();
    const int tseq = tracing() ? trace_launch(TR_KEYS) : 0;
    if (tracing()) trace_ev(TR_KEYS, EV_START, tseq);
    pdl_wait();
    if (tracing()) trace_ev(TR_KEYS, EV_END, tseq);
    const int bi = argmax_index(keys[0]);
    keys[0] = 0ull;
    ids[0] = bi;
    out[*step] = bi;
    *step += 1;
    tok_pos[0] += 1;
}

__global__ void k_add(float* __restrict__ y, const float* __restrict__ x, size_t n) {
    pdl_trigger();
    pdl_wait();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] += x[i];
}

// First index of the maximum (strict '>' scan, src/model.cpp:1939-1946).
__global__ void k_argmax(const float* __restrict__ x, int n, int ldx, int32_t* out) {
    pdl_trigger();
    pdl_wait();
    const float* r = x + (size_t)blockIdx.x * ldx;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = r[i];
        if (v > bv) { bv = v; bi = i; }
    }
    __shared__ float sv[32];
    __shared__ int si[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
        out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
    }
}

// Repetition penalty, then the first index of the maximum, over one row of
// logits: the greedy branch of the sampler on the device. Every occurrence of
// an id in `recent` (the sampler's window, oldest first) applies
// v = v > 0 ? v / p : v * p once (src/sampler.cpp: penalise, then argmax), so
// an id seen c times is penalised c times in a row. A bitmap of the window's
// ids in shared memory keeps the scan at one load per logit.
// One CTA per row: row r's window is the last `window` ids of
// hist[0 .. base + r), the sampler's window once the first r tokens of the
// forward that made these rows were accepted (speculative verification).
__global__ void k_argmax_penalized(const float* __restrict__ logits, int n, int ldx, const int32_t* __restrict__ hist,
                                   int base, int window, float penalty, int32_t* outs) {
    pdl_trigger();
    pdl_wait();
    const float* x = logits + (size_t)blockIdx.x * ldx;
    const int end = base + (int)blockIdx.x;
    const int n_recent = min(end, window);
    const int32_t* recent = hist + (end - n_recent);
    int32_t* out = outs + blockIdx.x;
    extern __shared__ uint32_t s_bits[];
    __shared__ int s_id[kMaxRecent];
    __shared__ float s_val[kMaxRecent];
    const int words = (n + 31) >> 5;
    for (int i = threadIdx.x; i < words; i += blockDim.x) s_bits[i] = 0u;
    __syncthreads();
    if (threadIdx.x < n_recent) {
        const int id = recent[threadIdx.x];
        int first = 1, count = 0;
        for (int j = 0; j < n_recent; ++j) {
            if (recent[j] == id) {
                if (j < (int)threadIdx.x) first = 0;
                ++count;
            }
        }
        s_id[threadIdx.x] = (first && id >= 0 && id < n) ? id : -1;
        if (s_id[threadIdx.x] >= 0) {
            float v = x[id];
            for (int c = 0; c < count; ++c) v = v > 0.0f ? __fdiv_rn(v, penalty) : __fmul_rn(v, penalty);
            s_val[threadIdx.x] = v;
            atomicOr(&s_bits[id >> 5], 1u << (id & 31));
        }
    }
    __syncthreads();
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = x[i];
        if (s_bits[i >> 5] & (1u << (i & 31))) {
            for (int j = 0; j < n_recent; ++j)
                if (s_id[j] == i) { v = s_val[j]; break; }
        }
        if (v > bv) { bv = v; bi = i; }
    }
    __shared__ float sv[32];
    __shared__ int si[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
        out[0] = bi == 0x7fffffff ? 0 : bi;
    }
}

// Router: softmax over NE logits (src/ops.cpp:40-55), top-K by probability
// (ties: lower expert first), renormalised when `norm` (src/model.cpp:1529-1550).
__global__ void k_moe_route(const float* __restrict__ logits, int T, int NE, int K, int norm, int32_t* sel,
                            float* wsel) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    float p[256];
    const float* lg = logits + (size_t)t * NE;
    float m = lg[0];
    for (int e = 1; e < NE; ++e) if (lg[e] > m) m = lg[e];
    float sum = 0.0f;
    for (int e = 0; e < NE; ++e) { p[e] = expf(lg[e] - m); sum += p[e]; }
    if (sum <= 0.0f) { for (int e = 0; e < NE; ++e) p[e] = 1.0f / NE; }
    else { const float inv = 1.0f / sum; for (int e = 0; e < NE; ++e) p[e] *= inv; }
    unsigned long long used[4] = {0, 0, 0, 0};
    float wsum = 0.0f;
    for (int k = 0; k < K; ++k) {
        int best = -1;
        for (int e = 0; e < NE; ++e) {
            if ((used[e >> 6] >> (e & 63)) & 1ull) continue;
            if (best < 0 || p[e] > p[best]) best = e;
        }
        used[best >> 6] |= 1ull << (best & 63);
        sel[(size_t)t * K + k] = best;
        wsel[(size_t)t * K + k] = p[best];
        wsum += p[best];
    }
    if (norm && wsum > 0.0f)
        for (int k = 0; k < K; ++k) wsel[(size_t)t * K + k] /= wsum;
}

// Per-head RMSNorm in place (qk-norm, src/model.cpp:1714-1721 with
// src/ops.cpp:18-23). One warp per (token, head).
__global__ void k_head_rmsnorm(float* x, int ldx, int T, int n_heads, int D, const float* __restrict__ w, float eps) {
    pdl_trigger();
    pdl_wait();
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (gw >= T * n_heads) return;
    float* r = x + (size_t)(gw / n_heads) * ldx + (size_t)(gw % n_heads) * D;
    double s = 0.0;
    for (int i = lane; i < D; i += 32) s += (double)r[i] * (double)r[i];
    s = warp_sum_d(s);
    const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(s / D), eps)));
    __syncwarp();
    for (int i = lane; i < D; i += 32) r[i] = __fmul_rn(__fmul_rn(r[i], sc), w[i]);
}

// Weighted scatter-add of the routed experts' outputs (src/model.cpp:1571-1578):
// ffn = sum_k w_k * d_k accumulated from zero, then x += ffn.
__global__ void k_moe_combine(float* x, int ldx, const float* __restrict__ eo, const float* __restrict__ wsel, int T,
                              int K, int E) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.y;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < E; i += gridDim.x * blockDim.x) {
        float acc = 0.0f;
        for (int k = 0; k < K; ++k) acc = __fadd_rn(acc, __fmul_rn(wsel[t * K + k], eo[((size_t)t * K + k) * E + i]));
        x[(size_t)t * ldx + i] = __fadd_rn(x[(size_t)t * ldx + i], acc);
    }
}

// ids[0] = argmax(logits); out[*step] = ids[0]; ++*step; ++tok_pos[0].
__global__ void k_greedy_advance(const float* __restrict__ x, int n, int32_t* ids, int32_t* tok_pos, int32_t* out,
                                 int32_t* step) {
    pdl_trigger();
    pdl_wait();
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = x[i];
        if (v > bv) { bv = v; bi = i; }
    }
    __shared__ float sv[32];
    __shared__ int si[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
        if (bi == 0x7fffffff) bi = 0;
        ids[0] = bi;
        out[*step] = bi;
        *step += 1;
        tok_pos[0] += 1;
    }
}

// Busy-wait for `ns` nanoseconds of device time (globaltimer), so a profiler
// can enqueue a whole step behind it; the loop ends once the time has passed
// and is additionally capped in iterations.
__global__ void k_delay(unsigned long long ns) {
    unsigned long long t0, t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (long long i = 0; i < (1LL << 30); ++i) {
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        if (t - t0 >= ns) break;
        __nanosleep(1000);
    }
}

}  // namespace fb

using namespace fb;

static bool g_pdl = false;
extern "C" void fbk_set_pdl(int on) { g_pdl = on != 0; }
extern "C" int fbk_pdl_enabled(void) { return g_pdl ? 1 : 0; }

extern "C" int fbk_delay(unsigned long long ns, cudaStream_t st) {
    k_delay<<<1, 1, 0, st>>>(ns);
    return (int)cudaGetLastError();
}

extern "C" int fbk_head_rmsnorm(float* x, int ldx, int T, int n_heads, int D, const float* w, float eps, cudaStream_t st) {
    const int warps = T * n_heads;
    if (warps <= 0) return 0;
    return (int)fbk_launch(k_head_rmsnorm, dim3((warps + 7) / 8), dim3(256), 0, st, x, ldx, T, n_heads, D, w, eps);
}

// Expert parallelism: global expert ids -> this rank's local ids (e - e0 for
// e in [e0, e0 + n), else -1: the expert GEMVs then write zero rows).
__global__ void k_moe_localize(const int32_t* __restrict__ sel, int n_sel, int e0, int n, int32_t* out) {
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n_sel) {
        out[i] = fb_localize_expert(sel[i], e0, n);
    }
}

// MoE router logits: out[t][e] = W_e . x_t for F32 router rows (row stride
// ws bytes), one warp per (token, expert). The reference sums f32 rows in
// float lanes (quant.cpp:67-80 scalar, quant_x86.cpp:242-251 AVX2), two
// orders that already differ from each other; here the products are summed
// in double in a fixed order (lane strides of 4 values, then a shuffle tree),
// so the logit is the exact dot product to within the final rounding. The
// same kernel serves every token count: a token's routing does not depend on
// the batch.
__global__ void k_router_f32(const uint8_t* __restrict__ w, size_t ws, const float* __restrict__ x, int ldx, int T,
                             int E, int NE, float* out, int ldo) {
    pdl_trigger();
    pdl_wait();
    const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (wid >= T * NE) return;
    const int t = wid / NE, e = wid % NE;
    const float* wr = reinterpret_cast<const float*>(w + (size_t)e * ws);
    const float* xr = x + (size_t)t * ldx;
    double s = 0.0;
    for (int k = 4 * lane; k < E; k += 128) {
        const float4 a = *reinterpret_cast<const float4*>(wr + k);
        const float4 b = *reinterpret_cast<const float4*>(xr + k);
        s += (double)a.x * b.x;
        s += (double)a.y * b.y;
        s += (double)a.z * b.z;
        s += (double)a.w * b.w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) out[(size_t)t * ldo + e] = (float)s;
}

extern "C" int fbk_router_f32(const uint8_t* w, size_t ws, const float* x, int ldx, int T, int E, int NE, float* out,
                              int ldo, cudaStream_t st) {
    if (T <= 0 || NE <= 0) return 0;
    if (E % 4 || ws % 16 || ldx % 4 || (reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(x) & 15))
        return (int)cudaErrorInvalidValue;
    const int warps = T * NE;
    return (int)fbk_launch(k_router_f32, dim3((warps + 7) / 8), dim3(256), 0, st, w, ws, x, ldx, T, E, NE, out, ldo);
}

// Expert grouping for batched MoE steps, packed in slots of S rows (S = 4 or
// 8, the GEMV launch's token count). Expert e owns ceil(count_e / S)
// consecutive slots from slot s0(e) = sum over e' < e of ceil(count_e' / S);
// the rows r = t K + k routed to it (ascending r) take packed rows
// S s0(e) + j: grp_src[S s0(e) + j] = r (-1 for the slot's pad rows and for
// unused slots), grp_pos[r] = S s0(e) + j (-1 for another
// rank's expert), grp_count[e] = count_e, chunk_exp[s] = the expert of slot s
// (-1 past the used slots: a GEMV given -1 fetches no weights). The caller
// sizes nslot with a bound on the used slots; dynamic shared memory holds
// nel + 1 ints.
__global__ void k_moe_group(const int32_t* __restrict__ esel, int T, int K, int nel, int32_t* grp_src,
                            int32_t* grp_pos, int32_t* grp_count, int32_t* chunk_exp, int nslot, int S) {
    extern __shared__ int s_slot[];   // [nel + 1]: first slot of each expert, then the total
    pdl_trigger();
    pdl_wait();
    const int n = T * K;
    for (int r = threadIdx.x; r < n; r += blockDim.x)
        if (esel[r] < 0 || esel[r] >= nel) grp_pos[r] = -1;
    for (int e = threadIdx.x; e < nel; e += blockDim.x) {
        int j = 0;
        for (int r = 0; r < n; ++r) j += esel[r] == e;
        grp_count[e] = j;
        s_slot[e + 1] = (j + S - 1) / S;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        s_slot[0] = 0;
        for (int e = 0; e < nel; ++e) s_slot[e + 1] += s_slot[e];
    }
    __syncthreads();
    const int used = min(s_slot[nel], nslot);
    for (int e = threadIdx.x; e < nel; e += blockDim.x) {
        const int s0 = s_slot[e], s1 = min(s_slot[e + 1], nslot), base = S * s0;
        int j = 0;
        for (int r = 0; r < n; ++r)
            if (esel[r] == e) {
                const bool fits = base + j < S * s1;
                if (fits) grp_src[base + j] = r;
                grp_pos[r] = fits ? base + j : -1;
                ++j;
            }
        for (int q = base + j; q < S * s1; ++q) grp_src[q] = -1;
        for (int s = s0; s < s1; ++s) chunk_exp[s] = e;
    }
    for (int s = used + threadIdx.x; s < nslot; s += blockDim.x) {
        chunk_exp[s] = -1;
        for (int q = 0; q < S; ++q) grp_src[S * s + q] = -1;
    }
}

// Grouped activation row g <- the int8 activations of token grp_src[g] / ksel
// (all layouts the planes hold; a zero row for -1).
__global__ void k_moe_gather(ActQ src, ActQ dst, const int32_t* __restrict__ grp_src, int ksel, int K) {
    pdl_trigger();
    pdl_wait();
    const int g = blockIdx.x;
    const int r = grp_src[g];
    const int t = r >= 0 ? r / ksel : -1;
    auto copy_bytes = [&](const int8_t* s, int8_t* d, int n) {   // n % 16 == 0, both 16-byte aligned
        for (int i = threadIdx.x; i < n / 16; i += blockDim.x)
            reinterpret_cast<uint4*>(d)[i] = t >= 0 ? reinterpret_cast<const uint4*>(s)[i] : make_uint4(0, 0, 0, 0);
    };
    if (src.qk && dst.qk) {
        copy_bytes(src.qk + (size_t)(t < 0 ? 0 : t) * src.ld, dst.qk + (size_t)g * dst.ld, K);
        for (int i = threadIdx.x; i < K / 256; i += blockDim.x)
            dst.dk[(size_t)g * (K / 256) + i] = t >= 0 ? src.dk[(size_t)t * (K / 256) + i] : 0.0f;
        for (int i = threadIdx.x; i < K / 32; i += blockDim.x)
            dst.bsk[(size_t)g * (K / 32) + i] = t >= 0 ? src.bsk[(size_t)t * (K / 32) + i] : (int16_t)0;
    }
    if (src.q32 && dst.q32) {
        copy_bytes(src.q32 + (size_t)(t < 0 ? 0 : t) * src.ld, dst.q32 + (size_t)g * dst.ld, K);
        for (int i = threadIdx.x; i < K / 32; i += blockDim.x) {
            dst.d32[(size_t)g * (K / 32) + i] = t >= 0 ? src.d32[(size_t)t * (K / 32) + i] : 0.0f;
            dst.s32[(size_t)g * (K / 32) + i] = t >= 0 ? src.s32[(size_t)t * (K / 32) + i] : 0;
        }
    }
}

// x[t] += sum_k w[t K + k] eo[grp_pos[t K + k]] (zero for another rank's
// expert), the float steps of k_moe_combine.
__global__ void k_moe_combine_grouped(float* x, int ldx, const float* __restrict__ eo, const int32_t* __restrict__ grp_pos,
                                      const float* __restrict__ wsel, int T, int K, int E) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.y;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < E; i += gridDim.x * blockDim.x) {
        float acc = 0.0f;
        for (int k = 0; k < K; ++k) {
            const int p = grp_pos[t * K + k];
            acc = __fadd_rn(acc, __fmul_rn(wsel[t * K + k], p >= 0 ? eo[(size_t)p * E + i] : 0.0f));
        }
        x[(size_t)t * ldx + i] = __fadd_rn(x[(size_t)t * ldx + i], acc);
    }
}

extern "C" int fbk_moe_group(const int32_t* esel, int T, int K, int nel, int32_t* grp_src, int32_t* grp_pos,
                             int32_t* grp_count, int32_t* chunk_exp, int nslot, int S, cudaStream_t st) {
    if (T <= 0 || nel <= 0) return 0;
    if (S != 4 && S != 8) return (int)cudaErrorInvalidValue;
    return (int)fbk_launch(k_moe_group, dim3(1), dim3(256), sizeof(int) * (nel + 1), st, esel, T, K, nel, grp_src,
                           grp_pos, grp_count, chunk_exp, nslot, S);
}

// Slots of S rows a grouping of T tokens x K selections over nel experts can
// use: each expert takes ceil(c / S) <= (c + S - 1) / S slots for its c <= T
// rows, so the sum is at most floor((T K + (S - 1) m) / S), m = experts with
// rows <= min(nel, T K), and at most nel ceil(T / S).
extern "C" int fbk_moe_slots(int T, int K, int nel, int S) {
    const int tk = T * K, m = nel < tk ? nel : tk;
    const int a = (tk + (S - 1) * m) / S, b = nel * ((T + S - 1) / S);
    return a < b ? a : b;
}

extern "C" int fbk_moe_gather(const ActQ* src, const ActQ* dst, const int32_t* grp_src, int ksel, int n_rows, int K,
                              cudaStream_t st) {
    if (n_rows <= 0) return 0;
    if (K % 256 && src->qk) return (int)cudaErrorInvalidValue;
    return (int)fbk_launch(k_moe_gather, dim3(n_rows), dim3(128), 0, st, *src, *dst, grp_src, ksel, K);
}

extern "C" int fbk_moe_combine_grouped(float* x, int ldx, const float* eo, const int32_t* grp_pos, const float* wsel,
                                       int T, int K, int E, cudaStream_t st) {
    if (T <= 0) return 0;
    return (int)fbk_launch(k_moe_combine_grouped, dim3((E + 255) / 256, T), dim3(256), 0, st, x, ldx, eo, grp_pos, wsel,
                           T, K, E);
}

extern "C" int fbk_moe_localize(const int32_t* sel, int n_sel, int e0, int n, int32_t* out, cudaStream_t st) {
    if (n_sel <= 0) return 0;
    return (int)fbk_launch(k_moe_localize, dim3((n_sel + 255) / 256), dim3(256), 0, st, sel, n_sel, e0, n, out);
}

extern "C" int fbk_moe_combine(float* x, int ldx, const float* eo, const float* wsel, int T, int K, int E, cudaStream_t st) {
    if (T <= 0) return 0;
    return (int)fbk_launch(k_moe_combine, dim3((E + 255) / 256, T), dim3(256), 0, st, x, ldx, eo, wsel, T, K, E);
}

extern "C" int fbk_greedy_advance(const float* logits, int V, int32_t* ids, int32_t* tok_pos, int32_t* out,
                                  int32_t* step, cudaStream_t st) {
    return (int)fbk_launch(k_greedy_advance, dim3(1), dim3(1024), 0, st, logits, V, ids, tok_pos, out, step);
}

extern "C" int fbk_embed(int type, const uint8_t* w, int E, int n_rows, const int32_t* ids, int T, float* x, int ldx,
                         int* err, cudaStream_t st) {
    if (T <= 0) return 0;
    return (int)fbk_launch(k_embed, dim3((E + 255) / 256, T), dim3(256), 0, st, type, w, E, n_rows, ids, x, ldx, err);
}

extern "C" int fbk_argmax_from_keys(unsigned long long* keys, int T, int32_t* out, cudaStream_t st) {
    if (T <= 0) return 0;
    if (T > 1024) return (int)cudaErrorInvalidValue;
    return (int)fbk_launch(k_argmax_from_keys, dim3(1), dim3(T), 0, st, keys, T, out);
}

extern "C" int fbk_greedy_from_keys(unsigned long long* keys, int32_t* ids, int32_t* tok_pos, int32_t* out,
                                    int32_t* step, cudaStream_t st) {
    return (int)fbk_launch(k_greedy_from_keys, dim3(1), dim3(1), 0, st, keys, ids, tok_pos, out, step);
}

extern "C" int fbk_add(float* y, const float* x, size_t n, cudaStream_t st) {
    if (!n) return 0;
    const int ctas = (int)((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184);
    return (int)fbk_launch(k_add, dim3(ctas), dim3(256), 0, st, y, x, n);
}

extern "C" int fbk_argmax(const float* x, int n, int rows, int ldx, int32_t* out, cudaStream_t st) {
    if (rows <= 0) return 0;
    return (int)fbk_launch(k_argmax, dim3(rows), dim3(1024), 0, st, x, n, ldx, out);
}

extern "C" int fbk_argmax_penalized(const float* x, int n, const int32_t* recent, int n_recent, float penalty,
                                    int32_t* out, cudaStream_t st) {
    return fbk_argmax_penalized_rows(x, n, 1, n, recent, n_recent, n_recent, penalty, out, st);
}

extern "C" int fbk_argmax_penalized_rows(const float* x, int n, int rows, int ldx, const int32_t* hist, int base,
                                         int window, float penalty, int32_t* out, cudaStream_t st) {
    if (rows <= 0) return 0;
    if (n <= 0 || ldx < n || base < 0 || window < 0 || window > kMaxRecent) return (int)cudaErrorInvalidValue;
    const size_t smem = sizeof(uint32_t) * (size_t)((n + 31) / 32);
    if (smem > 200 * 1024) return (int)cudaErrorInvalidValue;
    static bool attr = false;
    if (!attr) {
        const cudaError_t e = cudaFuncSetAttribute(k_argmax_penalized, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   200 * 1024);
        if (e != cudaSuccess) return (int)e;
        attr = true;
    }
    return (int)fbk_launch(k_argmax_penalized, dim3(rows), dim3(1024), smem, st, x, n, ldx, hist, base, window,
                           penalty, out);
}

extern "C" int fbk_moe_route(const float* logits, int T, int NE, int K, int norm, int32_t* sel, float* wsel,
                             cudaStream_t st) {
    if (T <= 0) return 0;
    if (NE > 256 || K > NE) return (int)cudaErrorInvalidValue;
    return (int)fbk_launch(k_moe_route, dim3((T + 63) / 64), dim3(64), 0, st, logits, T, NE, K, norm, sel, wsel);
}

extern "C" int fbk_trace_set_misc(const fb::TraceState* s) { return (int)fb::trace_set(*s); }

// Tracing for every kernel that records: a shared buffer of `cap` records,
// or off (cap <= 0). fbk_trace_dump copies the records out (4 values each:
// globaltimer ns, tag, event, launch number) and returns how many.
static unsigned long long* g_tbuf = nullptr;
static int* g_tcnt = nullptr;
static int g_tcap = 0;
extern "C" int fbk_trace_set_gemv(const fb::TraceState* s);
extern "C" int fbk_trace_set_attn(const fb::TraceState* s);
extern "C" int fbk_trace_enable(int cap) {
    fb::TraceState s{};
    if (cap > 0) {
        if (g_tcap < cap) {
            if (g_tbuf) cudaFree(g_tbuf);
            if (g_tcnt) cudaFree(g_tcnt);
            if (cudaMalloc(&g_tbuf, sizeof(unsigned long long) * 4 * (size_t)cap) != cudaSuccess) return -1;
            if (cudaMalloc(&g_tcnt, sizeof(int) * 9) != cudaSuccess) return -1;
            g_tcap = cap;
        }
        cudaMemset(g_tcnt, 0, sizeof(int) * 9);
        s.buf = g_tbuf;
        s.cap = cap;
        s.n = g_tcnt;
        s.seq = g_tcnt + 1;
        const char* all = getenv("FISH_TRACE_ALL");
        s.all = all && *all && *all != '0';
    }
    int rc = fbk_trace_set_gemv(&s);
    if (!rc) rc = fbk_trace_set_attn(&s);
    if (!rc) rc = fbk_trace_set_misc(&s);
    return rc;
}
extern "C" int fbk_trace_dump(unsigned long long* out, int cap) {
    if (!g_tbuf) return 0;
    int n = 0;
    if (cudaMemcpy(&n, g_tcnt, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    n = n < g_tcap ? n : g_tcap;
    n = n < cap ? n : cap;
    if (n > 0 && cudaMemcpy(out, g_tbuf, sizeof(unsigned long long) * 4 * (size_t)n, cudaMemcpyDeviceToHost) != cudaSuccess)
        return -1;
    return n;
}
