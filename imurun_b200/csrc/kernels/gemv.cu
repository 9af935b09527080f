// gemv.cu — decode/small-batch quantised matrix-vector products.
//
// y[t][r] = W_r . x_t for T <= 8 tokens, W in Q8_0 / Q4_K / Q6_K (int8 path,
// src/quant_x86.cpp:299-309, 346-382, 431-495) or F32 / F16 (f32 path,
// src/ops.cpp:219-250).
//
// Every integer the reference forms per block (Q4_K sumi and mins, Q6_K sumi,
// Q8_0 s) is formed whole by one thread (unit_math.cuh) and converted to float
// once. Two kernels:
//   k_gemv_stream  quantised rows, T <= 8 (decode). A producer warp streams
//                  (8-row tile x 2048-value group) stages — one contiguous
//                  bulk copy each, thanks to the tile-major layout — into a
//                  ring of shared-memory slots guarded by mbarriers. Eight
//                  consumer warps first build the activation image in shared
//                  memory (copied from quantised planes, or computed from f32
//                  rows: RMSNorm, SwiGLU or plain, then quantised), then each
//                  pair of them takes every fourth stage (4 rows x 8 blocks
//                  a warp, one block per lane). Per-stage row partials go to
//                  shared memory and are summed over groups at the end in a
//                  fixed order. Single-token launches use a variant compiled
//                  for their weight-type set and prologue mode.
//   k_gemv_direct  F32/F16 rows (up to 8 tokens), plain loads. Quantised
//                  calls of 5-15 tokens run as 4-token streamed launches
//                  (fbk_gemv_chunk); 16 or more go to the tensor-core
//                  kernel (gemm.cu).
// Launches carry the programmatic-dependent-launch attribute when the caller
// asks for it: the producer streams weights before the previous kernel has
// finished (weights never change); everything that reads activations or
// writes outputs waits for it first.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "layout.cuh"
#include "stream_common.cuh"
#include "tma.cuh"
#include "trace.cuh"
#include "unit_math.cuh"

namespace fb {

// ============================================================ host layouts

size_t dev_row_bytes(int type, int n) {
    size_t b = 0;
    switch (type) {
        case T_Q4_K: case T_Q6_K: case T_Q8_0: return row_bytes_dev(type, n);
        case T_F32: b = (size_t)n * 4; break;
        case T_F16: b = (size_t)n * 2; break;
        default: return 0;
    }
    return (b + 15) / 16 * 16;
}

size_t dev_matrix_bytes(int type, int n, int rows) {
    if (is_tiled(type)) return tiled_matrix_bytes(type, n, rows);
    return dev_row_bytes(type, n) * (size_t)rows;
}

static size_t ggml_block_bytes(int type) { return type == T_Q8_0 ? 34 : (type == T_Q4_K ? 144 : 210); }

void repack_rows(int type, const uint8_t* src, int rows, int n, uint8_t* dst, size_t src_stride) {
    const size_t total = dev_matrix_bytes(type, n, rows);
    std::memset(dst, 0, total);
    if (!is_tiled(type)) {
        const size_t sb = type == T_F32 ? (size_t)n * 4 : (size_t)n * 2, db = dev_row_bytes(type, n);
        const size_t ss = src_stride ? src_stride : sb;
        for (int r = 0; r < rows; ++r) std::memcpy(dst + (size_t)r * db, src + (size_t)r * ss, sb);
        return;
    }
    const int nb = row_blocks(type, n);
    const size_t srb = src_stride ? src_stride : (size_t)nb * ggml_block_bytes(type);
    for (int r = 0; r < rows; ++r) {
        const uint8_t* s = src + (size_t)r * srb;
        for (int b = 0; b < nb; ++b) {
            const uint8_t* sb = s + (size_t)b * ggml_block_bytes(type);
            uint8_t* q = dst + block_offset_tm(type, n, r, b);
            switch (type) {
                case T_Q4_K: std::memcpy(q, sb, 144); break;
                case T_Q6_K: {
                    std::memcpy(q, sb, 208);
                    uint8_t* d = dst + dscale_offset_tm(type, n, r, b);
                    d[0] = sb[208];
                    d[1] = sb[209];
                    break;
                }
                default: {   // Q8_0: fp16 d then qs[32]
                    std::memcpy(q, sb + 2, 32);
                    uint8_t* d = dst + dscale_offset_tm(type, n, r, b);
                    d[0] = sb[0];
                    d[1] = sb[1];
                    break;
                }
            }
        }
    }
}

// ============================================================ direct kernel

// Weights streamed from global memory, activations from the quantised planes
// through the read-only cache. One row, 8 lanes (bl = lane & 7). Summation order shared with
// k_gemv_stream, so a row's result does not depend on which kernel (which
// batch size) computed it: per 2048-value group, lane bl's term (the block
// gi*8 + bl for K-quants; for Q8_0 the sum, in block order, of blocks
// gi*64 + 8 bl .. + 7), then the tree over bl (xor 1, 2, 4), then the group
// sums added in group order. Every lane of the 8 runs every group (valid =
// row exists), so the shuffles never diverge.
template <int NT>
__device__ __forceinline__ void direct_rows_q(const GemvSeg& g, const uint8_t* base, int K, const ActQ& a, int T,
                                              int row, bool valid, int bl, float (&acc)[NT], int* err) {
    const int nb = row_blocks(g.type, K);
    const int G = row_groups(g.type, K);
    const uint8_t* wend = g.w + g.w_bytes;
    for (int gi = 0; gi < G; ++gi) {
        float c[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) c[t] = 0.0f;
        if (g.type == T_Q4_K) {
            const int kb = gi * 8 + bl;
            const uint8_t* p = base + block_offset_tm(T_Q4_K, K, row, kb);
            if (valid && kb < nb && in_range(p, 144, g.w, wend, err)) {
                uint4 w[9];
#pragma unroll
                for (int i = 0; i < 9; ++i) w[i] = ldg_stream(p + 16 * i);
                const float dw = h2f((uint16_t)(w[0].x & 0xFFFFu)), dmw = h2f((uint16_t)(w[0].x >> 16));
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if (t >= T) break;
                    int si, mi;
                    const uint4 bs = __ldg(reinterpret_cast<const uint4*>(a.bsk + (size_t)t * (K / 32) + (size_t)kb * 8));
                    q4k_block<LdGlobal>(w, a.qk + (size_t)t * a.ld + (size_t)kb * 256, bs, si, mi);
                    c[t] = q4k_term(dw, dmw, __ldg(a.dk + (size_t)t * (K / 256) + kb), si, mi);
                }
            }
        } else if (g.type == T_Q6_K) {
            const int kb = gi * 8 + bl;
            const uint8_t* p = base + block_offset_tm(T_Q6_K, K, row, kb);
            const uint8_t* pd = base + dscale_offset_tm(T_Q6_K, K, row, kb);
            if (valid && kb < nb && in_range(p, 208, g.w, wend, err) && in_range(pd, 2, g.w, wend, err)) {
                uint4 w[13];
#pragma unroll
                for (int i = 0; i < 13; ++i) w[i] = ldg_stream(p + 16 * i);
                const float dw = h2f(*reinterpret_cast<const uint16_t*>(pd));
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if (t >= T) break;
                    const int8_t* xq = a.qk + (size_t)t * a.ld + (size_t)kb * 256;
                    int16_t xs[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) xs[j] = (int16_t)sum16(__ldg(reinterpret_cast<const uint4*>(xq + 16 * j)));
                    const int si = q6k_block<LdGlobal>(w, xq, xs);
                    c[t] = scaled_term(dw, __ldg(a.dk + (size_t)t * (K / 256) + kb), si);
                }
            }
        } else {   // Q8_0: blocks gi*64 + 8 bl + i, i = 0..7, summed in block order
            for (int i = 0; i < 8; ++i) {
                const int b = gi * 64 + 8 * bl + i;
                if (!valid || b >= nb) break;
                const uint8_t* p = base + block_offset_tm(T_Q8_0, K, row, b);
                const uint8_t* pd = base + dscale_offset_tm(T_Q8_0, K, row, b);
                if (!in_range(p, 32, g.w, wend, err) || !in_range(pd, 2, g.w, wend, err)) continue;
                const uint4 w0 = ldg_stream(p), w1 = ldg_stream(p + 16);
                const float dw = h2f(*reinterpret_cast<const uint16_t*>(pd));
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if (t >= T) break;
                    const int s = q80_block<LdGlobal>(w0, w1, a.q32 + (size_t)t * a.ld + (size_t)b * 32);
                    c[t] = __fadd_rn(c[t], scaled_term(dw, __ldg(a.d32 + (size_t)t * (K / 32) + b), s));
                }
            }
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            c[t] += __shfl_xor_sync(0xffffffffu, c[t], 1);
            c[t] += __shfl_xor_sync(0xffffffffu, c[t], 2);
            c[t] += __shfl_xor_sync(0xffffffffu, c[t], 4);
            acc[t] += c[t];
        }
    }
}

template <int NT>
__device__ __forceinline__ void row_float(int type, const uint8_t* __restrict__ row, int K, const float* xf, int ldxf,
                                          int T, int lane, float (&acc)[NT]) {
    for (int k = lane; k < K; k += 32) {
        const float w = type == T_F32 ? reinterpret_cast<const float*>(row)[k]
                                      : h2f(reinterpret_cast<const uint16_t*>(row)[k]);
#pragma unroll
        for (int t = 0; t < NT; ++t)
            if (t < T) acc[t] += w * xf[(size_t)t * ldxf + k];
    }
}

// Quantised segments: a warp owns 4 rows (lane = row * 8 + block slot);
// float segments: a warp owns one row.
template <int NT>
__global__ void __launch_bounds__(256) k_gemv_direct(GemvArgs args) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    int items[kMaxSeg + 1];
    items[0] = 0;
#pragma unroll
    for (int s = 0; s < kMaxSeg; ++s) {
        const int r = s < args.nseg ? args.seg[s].rows : 0;
        const int n = s < args.nseg ? (is_tiled(args.seg[s].type) ? (r + 3) / 4 : r) : 0;
        items[s + 1] = items[s] + n;
    }
    for (int it = gw; it < items[args.nseg]; it += nw) {
        int s = 0;
        while (s < args.nseg - 1 && it >= items[s + 1]) ++s;
        const GemvSeg& g = args.seg[s];
        const int eidx = g.expert ? __ldg(g.expert) : 0;   // < 0: an expert of another rank (zero rows)
        const uint8_t* base = g.w + (size_t)max(eidx, 0) * g.expert_bytes;
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
        if (is_tiled(g.type)) {
            const int row = (it - items[s]) * 4 + (lane >> 3), bl = lane & 7;
            direct_rows_q<NT>(g, base, args.K, args.act, args.T, row, row < g.rows && eidx >= 0, bl, acc, args.err);
#pragma unroll
            for (int t = 0; t < NT; ++t)
                if (bl == 0 && row < g.rows && t < args.T) store_out(g, row, t, acc[t]);
        } else {
            const int row = it - items[s];
            if (eidx >= 0 &&
                in_range(base + (size_t)row * g.row_stride, g.row_stride, g.w, g.w + g.w_bytes, lane == 0 ? args.err : nullptr))
                row_float<NT>(g.type, base + (size_t)row * g.row_stride, args.K, args.xf, args.ldxf, args.T, lane, acc);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float v = warp_sum(acc[t]);
                if (lane == 0 && t < args.T) store_out(g, row, t, v);
            }
        }
    }
}

// Debug: the per-(row, block) integer sums, one thread per block, with the
// same block functions the GEMV kernels use.
__global__ void k_block_sums(int type, const uint8_t* __restrict__ w, int rows, int K, ActQ a, int32_t* sumi,
                             int32_t* mins) {
    const int nb = row_blocks(type, K);
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)rows * nb) return;
    const int row = (int)(i / nb), b = (int)(i % nb);
    if (type == T_Q4_K) {
        uint4 wr[9];
        const uint8_t* p = w + block_offset_tm(T_Q4_K, K, row, b);
#pragma unroll
        for (int k = 0; k < 9; ++k) wr[k] = ldg_stream(p + 16 * k);
        int si, mi;
        q4k_block<LdGlobal>(wr, a.qk + (size_t)b * 256, __ldg(reinterpret_cast<const uint4*>(a.bsk + (size_t)b * 8)),
                            si, mi);
        sumi[i] = si;
        if (mins) mins[i] = mi;
    } else if (type == T_Q6_K) {
        uint4 wr[13];
        const uint8_t* p = w + block_offset_tm(T_Q6_K, K, row, b);
#pragma unroll
        for (int k = 0; k < 13; ++k) wr[k] = ldg_stream(p + 16 * k);
        const int8_t* xq = a.qk + (size_t)b * 256;
        int16_t xs[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) xs[j] = (int16_t)sum16(__ldg(reinterpret_cast<const uint4*>(xq + 16 * j)));
        sumi[i] = q6k_block<LdGlobal>(wr, xq, xs);
    } else if (type == T_Q8_0) {
        const uint8_t* p = w + block_offset_tm(T_Q8_0, K, row, b);
        sumi[i] = q80_block<LdGlobal>(ldg_stream(p), ldg_stream(p + 16), a.q32 + (size_t)b * 32);
    }
}

// ============================================================ streamed kernel

constexpr int kHdrBytes = 2 * kMaxStages * 8 + 64;  // mbarriers, abort flag, norm scales


// Records of bounded waits that gave up (read with fbk_take_wait_record),
// up to kWaitRecs, 16 values each:
// [0] kind (1 producer/empty, 2 consumer/full), [1] CTA, [2] stage, [3] slot,
// [4] parity, [5] stages of the CTA, [6] ring slots, [7] stages the producer
// has issued, [8] ns spent waiting, [9] ns since the kernel started, [10] warp,
// [11] stage the producer is waiting to reuse (-1 none), [12] raw word of
// full[slot], [13] raw word of empty[slot], [14] SM id, [15] smem bytes
constexpr int kWaitRecs = 8;
__device__ long long g_wait_rec[kWaitRecs][16];
__device__ int g_wait_rec_n;

__device__ __noinline__ void record_wait_fail(int kind, int s, int slot, int parity, int n_stages, int S, int issued,
                                              unsigned long long t_start, unsigned long long t_kernel, int prod_wait,
                                              const uint64_t* full, const uint64_t* empty, int smem_bytes) {
    const int k = atomicAdd(&g_wait_rec_n, 1);
    if (k >= kWaitRecs) return;
    const unsigned long long now = gtimer();
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    long long* r = g_wait_rec[k];
    r[0] = kind; r[1] = blockIdx.x; r[2] = s; r[3] = slot; r[4] = parity; r[5] = n_stages; r[6] = S; r[7] = issued;
    r[8] = (long long)(now - t_start); r[9] = (long long)(now - t_kernel); r[10] = threadIdx.x >> 5;
    r[11] = prod_wait; r[12] = (long long)full[slot]; r[13] = (long long)empty[slot]; r[14] = smid; r[15] = smem_bytes;
    __threadfence();
}

// Ring slots: a FIFO, stage s in slot s % S, phase s / S, with S a multiple
// of the 4 consumer pairs. Pair q takes stages q, q + 4, ..., so every slot it
// touches is only ever its own (slot = s % S keeps s's residue mod 4), and it
// waits on each of them phase after phase: never for a phase two ahead of the
// barrier, which a parity wait could not tell apart.
__device__ __forceinline__ int ring_slot(int s, int S) { return s % S; }
__device__ __forceinline__ int ring_phase(int s, int S) { return s / S; }

struct StreamJobs {
    int tile0[kMaxSeg + 1];  // 8-row tiles: segment s owns tiles [tile0[s], tile0[s+1])
    int n_groups;            // 2048-value groups per row
    int stages;              // ring slots
    int slot_bytes;          // bytes per slot (8 x the largest piece)
    int tiles_per_cta;       // most tiles any CTA gets (sizes the partials)
    int n_units;             // work units (a tile, or a (gate, up) tile pair): CTA b takes
                             // units [b n_units / grid, (b+1) n_units / grid)
    int xk_bytes, x32_bytes; // per-token bytes of the two activation images (0 = not built)
    int* err;                // device error flag
    int wait_first;          // producer waits for the previous kernel (expert indices)
    int pair;                // tiles alternate between segments 0 and 1 (SwiGLU epilogue)
};

// TM: the weight types the kernel handles (TM_* bits); PM: the prologue mode,
// or -1 for any (read from the arguments).
template <int NT, int TM, int PM>
__global__ void __launch_bounds__(32 * (kConsumers + 1), NT == 1 ? 2 : 1) k_gemv_stream(GemvArgs args, StreamJobs jobs) {
    extern __shared__ __align__(128) uint8_t smem[];
    pdl_trigger();
    const unsigned long long t_kernel = gtimer();
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    volatile int* s_abort = reinterpret_cast<volatile int*>(smem + 2 * kMaxStages * 8);
    volatile int* s_issued = reinterpret_cast<volatile int*>(smem + 2 * kMaxStages * 8 + 4);
    volatile int* s_prod_wait = reinterpret_cast<volatile int*>(smem + 2 * kMaxStages * 8 + 8);
    unsigned dyn_smem;
    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn_smem));
    __shared__ double s_part[kNormWarps];
    __shared__ int s_tseq;
    __shared__ GemvSeg s_seg[kMaxSeg];
    __shared__ int s_tile0[kMaxSeg + 1];
    __shared__ unsigned long long s_best[kConsumers][kMaxStreamTokens];
    __shared__ long long s_pw, s_cw;   // summed wait cycles (all-CTA tracing)
    const int K = args.K, G = jobs.n_groups, S = jobs.stages;
    int n_tiles = jobs.tile0[0];
#pragma unroll
    for (int i = 1; i <= kMaxSeg; ++i)
        if (i == args.nseg) n_tiles = jobs.tile0[i];
    // balanced split: units of one tile, or of a (gate, up) tile pair
    const int unit = jobs.pair ? 2 : 1;
    JobView jv;
    jv.seg = s_seg;
    jv.tile0 = s_tile0;
    jv.nseg = args.nseg;
    jv.pair = jobs.pair;
    jv.G = G;
    jv.K = K;
    jv.T = args.T;
    jv.t_begin = (int)((long long)blockIdx.x * jobs.n_units / gridDim.x) * unit;
    jv.t_end = min(n_tiles, (int)((long long)(blockIdx.x + 1) * jobs.n_units / gridDim.x) * unit);
    const int n_stages = job_stages(jv);
    XImage xi;
    xi.base = smem + kHdrBytes;
    xi.n256 = (K + 255) / 256;
    xi.xk = jobs.xk_bytes;
    xi.x32 = jobs.x32_bytes;
    xi.T = args.T;
    float* part = reinterpret_cast<float*>(xi.base + (size_t)args.T * (jobs.xk_bytes + jobs.x32_bytes));
    RingView rg;
    rg.base = reinterpret_cast<uint8_t*>(part) + (((size_t)jobs.tiles_per_cta * G * kTileRows * NT * 4 + 127) / 128 * 128);
    rg.full = full;
    rg.empty = empty;
    rg.S = S;
    rg.slot_bytes = jobs.slot_bytes;
    rg.issued = s_issued;
    rg.abort = s_abort;
    rg.guard = 0;   // S is a multiple of the pairs and the job starts at ring stage 0
    rg.pwait = nullptr;
    rg.cwait = nullptr;
    rg.pclk = tracing_all() ? &s_pw : nullptr;
    rg.cclk = tracing_all() ? &s_cw : nullptr;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < kMaxSeg; ++i)
        if (threadIdx.x == i) s_seg[i] = args.seg[i];
#pragma unroll
    for (int i = 0; i <= kMaxSeg; ++i)
        if (threadIdx.x == i) s_tile0[i] = jobs.tile0[i];
    const bool tr = tracing() && !tracing_all() && blockIdx.x == 0;
    if (tr && threadIdx.x == 0) {
        s_tseq = trace_launch(TR_GEMV);
        trace_ev(TR_GEMV, EV_START, s_tseq);
    }
    if (threadIdx.x == 0) {
        *s_abort = 0;
        *s_issued = 0;
        *s_prod_wait = -1;
        s_pw = 0;
        s_cw = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 2);
        }
        mbar_fence_init();
    }
    __syncthreads();

    // every segment routed to an expert no row of this call uses (id -1:
    // another rank's expert, or an empty chunk of a grouped MoE step): no
    // weights, no arithmetic; the rows are zero, as the full path gives them
    if (jobs.wait_first && !args.swiglu) {
        pdl_wait();
        bool idle = true;
#pragma unroll
        for (int i = 0; i < kMaxSeg; ++i)
            if (i < args.nseg && (!args.seg[i].expert || __ldg(args.seg[i].expert) >= 0)) idle = false;
        if (idle) {
            if (warp < kConsumers) {
                const int n_rows = (jv.t_end - jv.t_begin) * kTileRows;
                for (int idx = threadIdx.x; idx < n_rows; idx += kConsumers * 32) {
                    const int tile = jv.t_begin + idx / kTileRows;
                    const int sg = seg_index(s_tile0, args.nseg, tile);
                    const GemvSeg& g = s_seg[sg];
                    const int row = (tile - s_tile0[sg]) * kTileRows + idx % kTileRows;
                    if (row >= g.rows) continue;
                    for (int t = 0; t < args.T; ++t) store_out(g, row, t, 0.0f);
                }
            }
            return;
        }
    }

    if (warp == kConsumers) {   // producer
        if (lane == 0) {
            if (jobs.wait_first) pdl_wait();
            WaitFail wf{};
            if (!produce_stages<TM>(rg, jv, 0, jobs.err, &wf)) {
                const int issued = wf.stage;   // stages issued before the one that waited
                record_wait_fail(1, wf.stage, wf.slot, wf.parity, n_stages, S, issued, wf.t0, t_kernel, wf.stage - S, full,
                                 empty, (int)dyn_smem);
                if (jobs.err) atomicExch(jobs.err, 1);
                *s_abort = 1;
                // let the copies in flight land before the CTA can exit
                for (int k = max(0, issued - S); k < issued; ++k)
                    mbar_wait_bounded(&full[ring_slot(k, S)], (uint32_t)(ring_phase(k, S) & 1));
            }
        }
        return;
    }

    // consumers: the norm weights are constant, so they are loaded before
    // waiting for the previous kernel
    const int tcb = trace_cta_begin(7);
    if (tcb >= 0) {
        unsigned long long* r = g_trace.buf + 4 * (size_t)tcb;
        r[0] = t_kernel; r[1] = TR_GEMV; r[2] = EV_C_START;
        r[3] = blockIdx.x | ((unsigned long long)gridDim.x << 20);
    }
    float wv[kNormRegs][8];
    if ((PM >= 0 ? PM : args.pro.mode) == PRO_NORM) {
#pragma unroll
        for (int k = 0; k < kNormRegs; ++k) {
            const int c = warp + kConsumers * k;
            if (c * 256 < K) ld8(args.pro.w, c * 256 + 8 * lane, K, wv[k]);
        }
    }
    pdl_wait();
    if (tr && threadIdx.x == 0) trace_ev(TR_GEMV, EV_WAITED, s_tseq);
    trace_cta(tcb, 1, TR_GEMV, EV_C_WAITED);
    const bool wantk = jobs.xk_bytes > 0, want32 = jobs.x32_bytes > 0;
    build_ximage<PM>(args, xi, wantk, want32, s_part, wv, tr ? s_tseq : -1);
    consumers_sync();
    if (args.img_dump && blockIdx.x == 0) {
        // debug record of the prologue's output (layer probes): the image is
        // the same in every CTA, so CTA 0's copy stands for all of them
        if (threadIdx.x == 0) {
            int* hdr = reinterpret_cast<int*>(args.img_dump);
            hdr[0] = jobs.xk_bytes;
            hdr[1] = jobs.x32_bytes;
            hdr[2] = args.T;
            hdr[3] = xi.n256;
        }
        const size_t nb = (size_t)args.T * (jobs.xk_bytes + jobs.x32_bytes);
        for (size_t i = (size_t)threadIdx.x * 16; i < nb; i += (size_t)kConsumers * 32 * 16)
            *reinterpret_cast<uint4*>(args.img_dump + 16 + i) = *reinterpret_cast<const uint4*>(xi.base + i);
    }
    if (tr && threadIdx.x == 0) trace_ev(TR_GEMV, EV_READY, s_tseq);
    trace_cta(tcb, 2, TR_GEMV, EV_C_READY);
    WaitFail wf{};
    const bool ok = consume_stages<NT, TM>(rg, jv, 0, xi, part, &wf, tr ? s_tseq : -1);
    if (!ok) {
        if (!*s_abort)
            record_wait_fail(2, wf.stage, wf.slot, wf.parity, n_stages, S, *s_issued, wf.t0, t_kernel, *s_prod_wait, full,
                             empty, (int)dyn_smem);
        if (jobs.err && lane == 0) atomicExch(jobs.err, 2);
        *s_abort = 1;
    }
    if (tr && threadIdx.x == 0) trace_ev(TR_GEMV, EV_LOOP, s_tseq);
    trace_cta(tcb, 3, TR_GEMV, EV_C_LOOP);
    trace_cta_val(tcb, 5, TR_GEMV, EV_C_CWAIT, (unsigned long long)s_cw);
    consumers_sync();
    if (*s_abort) return;
    reduce_rows<NT>(jv, part, s_best);
    if (tr) {
        consumers_sync();
        if (threadIdx.x == 0) trace_ev(TR_GEMV, EV_END, s_tseq);
    }
    if (tcb >= 0 || (tracing_all() && threadIdx.x < 32)) {
        __syncwarp();
        trace_cta(tcb, 4, TR_GEMV, EV_C_END);   // warp 0's rows are written
        trace_cta_val(tcb, 6, TR_GEMV, EV_C_PWAIT, (unsigned long long)s_pw);
    }
}
}  // namespace fb

using namespace fb;

static int g_num_sms = 0;

static int num_sms() {
    if (!g_num_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    return g_num_sms;
}

static int* g_err = nullptr;

extern "C" int* fbk_gemv_error_flag() {
    if (!g_err) {
        if (cudaMalloc(&g_err, sizeof(int)) != cudaSuccess) return nullptr;
        cudaMemset(g_err, 0, sizeof(int));
    }
    return g_err;
}

extern "C" int fbk_trace_set_gemv(const TraceState* s) { return (int)trace_set(*s); }

extern "C" int fbk_take_wait_record(long long* rec) {
    long long h[kWaitRecs][16] = {};
    int n = 0;
    if (cudaMemcpyFromSymbol(&n, g_wait_rec_n, sizeof(int)) != cudaSuccess) return -1;
    if (n) {
        if (cudaMemcpyFromSymbol(h, g_wait_rec, sizeof(h)) != cudaSuccess) return -1;
        const int zero = 0;
        cudaMemcpyToSymbol(g_wait_rec_n, &zero, sizeof(int));
    }
    for (int i = 0; i < kWaitRecs * 16; ++i) rec[i] = (&h[0][0])[i];
    return n;
}

extern "C" int fbk_take_error_flag() {
    if (!g_err) return 0;
    int v = 0;
    if (cudaMemcpy(&v, g_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (v) cudaMemset(g_err, 0, sizeof(int));
    return v;
}

static int env_or(const char* name, int def) {
    const char* v = getenv(name);
    return v && *v ? atoi(v) : def;
}

// Pipeline geometry: CTAs per SM (default 2) split the SM's shared memory;
// after the activation image and the row partials, the rest is ring slots.
using StreamKernel = void (*)(GemvArgs, StreamJobs);

// Single-token launches get a kernel compiled for their weight-type set and
// prologue mode: the variant that carries every type's consumer arithmetic
// and every prologue does not fit the instruction cache (a quarter of its
// fetches missed in a decode-sized launch). Other launches use that generic
// variant.
template <int NT>
static StreamKernel stream_variant(int tm, int pm) {
    if (NT == 1) {
        switch (pm * 8 + tm) {
#define FB_SV(P, T) \
    case P * 8 + T: return k_gemv_stream<1, T, P>;
            FB_SV(PRO_NORM, 1) FB_SV(PRO_NORM, 2) FB_SV(PRO_NORM, 3) FB_SV(PRO_NORM, 4)
            FB_SV(PRO_QUANT, 1) FB_SV(PRO_QUANT, 2) FB_SV(PRO_QUANT, 3) FB_SV(PRO_QUANT, 4)
            FB_SV(PRO_SILU, 1) FB_SV(PRO_SILU, 2) FB_SV(PRO_SILU, 4)
#undef FB_SV
            default: break;
        }
    }
    return k_gemv_stream<NT, TM_ALL, -1>;
}

// Dynamic shared memory opt-in, once per kernel variant.
static int stream_smem_optin(StreamKernel k, int dyn) {
    static std::mutex mu;
    static std::vector<StreamKernel> done;
    std::lock_guard<std::mutex> lock(mu);
    for (StreamKernel d : done)
        if (d == k) return 0;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn) != cudaSuccess)
        return (int)cudaGetLastError();
    done.push_back(k);
    return 0;
}

// Dynamic shared memory one streamed-GEMV CTA may take (the opt-in maximum
// less the kernel's static shared memory; 0 when unknown).
static int stream_max_smem() {
    static const int v = [] {
        int dev = 0, optin = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
            return 0;
        cudaFuncAttributes fa{};
        if (cudaFuncGetAttributes(&fa, k_gemv_stream<4, TM_ALL, -1>) != cudaSuccess) return 0;
        return std::max(0, optin - (int)fa.sharedSizeBytes);
    }();
    return v;
}

// The streamed launch of a call of NT tokens: jobs, CTAs, ring stages and
// shared memory; false when not even the minimum ring fits next to the
// activation images.
static bool stream_plan(const GemvArgs* a, int NT, StreamJobs* out, int* ctas_out, size_t* smem_out) {
    static const int want_cps = std::max(1, std::min(4, env_or("FISH_GEMV_CTA_PER_SM", 2)));
    const int max_smem = stream_max_smem();
    if (max_smem <= 0) return false;
    StreamJobs jobs{};
    bool wantk = false, want32 = false;
    int slot = 0;
    for (int s = 0; s < a->nseg; ++s) {
        const int t = a->seg[s].type;
        slot = std::max(slot, kTileRows * (int)group_bytes(t, blocks_per_group(t)));
        if (t == T_Q8_0) want32 = true; else wantk = true;
        if (a->seg[s].expert) jobs.wait_first = 1;
    }
    jobs.slot_bytes = slot;
    jobs.xk_bytes = wantk ? ximg_k_bytes(a->K) : 0;
    jobs.x32_bytes = want32 ? ximg_32_bytes(a->K) : 0;
    jobs.tile0[0] = 0;
    for (int s = 0; s < a->nseg; ++s) jobs.tile0[s + 1] = jobs.tile0[s] + (a->seg[s].rows + kTileRows - 1) / kTileRows;
    for (int s = a->nseg; s < kMaxSeg; ++s) jobs.tile0[s + 1] = jobs.tile0[s];
    jobs.pair = a->swiglu ? 1 : 0;
    if (jobs.pair && (a->nseg != 2 || a->seg[0].rows != a->seg[1].rows || a->seg[0].epi != EPI_STORE)) return false;
    jobs.n_groups = row_groups(a->seg[0].type, a->K);
    const int n_tiles = jobs.tile0[a->nseg];
    const int unit = jobs.pair ? 2 : 1;
    jobs.n_units = (n_tiles + unit - 1) / unit;
    const size_t xbytes = (size_t)a->T * (jobs.xk_bytes + jobs.x32_bytes);
    int ctas = 0, stages = 0;
    size_t smem = 0;
    for (int cps = NT == 1 ? want_cps : 1;; --cps) {
        const int budget = max_smem / cps - 2048;
        ctas = std::min(jobs.n_units, num_sms() * cps);
        jobs.tiles_per_cta = (jobs.n_units + ctas - 1) / ctas * unit;
        const size_t part = ((size_t)jobs.tiles_per_cta * jobs.n_groups * kTileRows * NT * 4 + 127) / 128 * 128;
        const long long left = (long long)budget - kHdrBytes - (long long)xbytes - (long long)part;
        stages = kPairs * (int)std::min<long long>(kMaxStages / kPairs, left > 0 ? left / (kPairs * (long long)slot) : 0);
        smem = kHdrBytes + xbytes + part + (size_t)stages * slot;
        if (stages >= kPairs || cps == 1) break;
    }
    if (stages < kPairs) return false;
    jobs.stages = stages;
    *out = jobs;
    *ctas_out = ctas;
    *smem_out = smem;
    return true;
}

template <int NT>
static int launch_stream(const GemvArgs* a, cudaStream_t st) {
    StreamJobs jobs{};
    int ctas = 0;
    size_t smem = 0;
    if (!stream_plan(a, NT, &jobs, &ctas, &smem)) return (int)cudaErrorInvalidValue;
    jobs.err = fbk_gemv_error_flag();
    int tm = 0;
    for (int s = 0; s < a->nseg; ++s) tm |= type_bit(a->seg[s].type);
    const StreamKernel kern = stream_variant<NT>(tm, a->pro.mode);
    if (const int e = stream_smem_optin(kern, stream_max_smem())) return e;
    return (int)fbk_launch(kern, dim3(ctas), dim3(32 * (kConsumers + 1)), smem, st, *a, jobs);
}

extern "C" int fbk_gemv_streamable(const GemvArgs* a) {
    if (a->T <= 0 || a->T > 8 || a->nseg <= 0) return 0;
    const int g0 = row_groups(a->seg[0].type, a->K);
    for (int s = 0; s < a->nseg; ++s) {
        const int t = a->seg[s].type;
        if (!is_tiled(t)) return 0;
        if (row_groups(t, a->K) != g0) return 0;
        if ((t == T_Q4_K || t == T_Q6_K) && a->K % 256) return 0;
    }
    if (a->K % 8) return 0;
    static const bool stream_off = getenv("FISH_GEMV_DIRECT") != nullptr;
    if (stream_off) return 0;
    if (a->T > 4) {   // an 8-token launch: its activation images must leave room for the ring
        StreamJobs j{};
        int c = 0;
        size_t m = 0;
        if (!stream_plan(a, 8, &j, &c, &m)) return 0;
    }
    return 1;
}

extern "C" int fbk_gemv_chunk(const GemvArgs* a) {
    GemvArgs p = *a;
    p.T = 8;
    if (fbk_gemv_streamable(&p)) return 8;
    p.T = 4;
    return fbk_gemv_streamable(&p) ? 4 : 8;
}

extern "C" int fbk_gemv(const GemvArgs* a, cudaStream_t st) {
    if (a->T <= 0 || a->nseg <= 0) return 0;
    if (a->T > 8) return (int)cudaErrorInvalidValue;
    if (fbk_gemv_streamable(a)) {
        if (a->T == 1) return launch_stream<1>(a, st);
        if (a->T == 2) return launch_stream<2>(a, st);
        if (a->T > 4) return launch_stream<8>(a, st);
        return launch_stream<4>(a, st);
    }
    if (a->pro.mode != PRO_ACT || a->swiglu) return (int)cudaErrorInvalidValue;
    GemvArgs ad = *a;
    if (!ad.err) ad.err = fbk_gemv_error_flag();
    a = &ad;
    int items = 0;
    for (int s = 0; s < a->nseg; ++s) items += is_tiled(a->seg[s].type) ? (a->seg[s].rows + 3) / 4 : a->seg[s].rows;
    int ctas = (items + 7) / 8;
    const int cap = num_sms() * 8;
    if (ctas > cap) ctas = cap;
    if (ctas < 1) ctas = 1;
    cudaError_t e;
    if (a->T == 1) e = fbk_launch(k_gemv_direct<1>, dim3(ctas), dim3(256), 0, st, *a);
    else if (a->T == 2) e = fbk_launch(k_gemv_direct<2>, dim3(ctas), dim3(256), 0, st, *a);
    else if (a->T <= 4) e = fbk_launch(k_gemv_direct<4>, dim3(ctas), dim3(256), 0, st, *a);
    else e = fbk_launch(k_gemv_direct<8>, dim3(ctas), dim3(256), 0, st, *a);
    return (int)e;
}

extern "C" int fbk_block_sums(int type, const uint8_t* w, int rows, int K, const ActQ* a, int32_t* sumi, int32_t* mins,
                              cudaStream_t st) {
    const long long n = (long long)rows * row_blocks(type, K);
    const int ctas = (int)((n + 255) / 256);
    k_block_sums<<<ctas, 256, 0, st>>>(type, w, rows, K, *a, sumi, mins);
    return (int)cudaGetLastError();
}
