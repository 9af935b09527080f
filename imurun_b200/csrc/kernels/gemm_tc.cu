// gemm_tc.cu — batched Q4_K products on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, accumulators in tensor memory, operands fed by TMA).
//
// Y[t][r] = W_r . x_t for Q4_K rows against the Q8ActK activation plane, with
// the reference's integers per 256-value block (src/quant_x86.cpp:346-382):
//   sumi = sum_g sc_g sum_{32} q x      mins = sum_g m_g bsums_g
// One MMA instruction sums over K = 32, so the per-sub-block 6-bit scale
// sc_g cannot ride along as is. It is split, sc_g = 8 hi_g + lo_g with
// hi_g, lo_g in 0..7, and each weight code q (0..15) is expanded in shared
// memory into three int8 planes whose K-sums over the whole block are exact
// integers:
//   plane 0: hi_g q  ->  D0 = sum_g hi_g sum q x
//   plane 1: lo_g q  ->  D1 = sum_g lo_g sum q x      sumi = 8 D0 + D1
//   plane 2: m_g     ->  D2 = sum_g m_g sum x = mins
// (all entries <= 105, int32 accumulation: the block integers equal the
// reference's bit for bit). The float steps per block and their order (the
// pairwise tree over the 8 blocks of a 2048-value group, then the groups in
// order) are those of the GEMV kernels, so a row's value does not depend on
// the kernel or on the number of tokens in the call.
//
// CTA tile: 128 weight rows (the TMEM lanes) x 64 tokens (the MMA N). Warps:
//   0      TMA producer: per block, the raw Q4_K bytes of the 128 rows (one
//          5-D tensor-map box over the tile-major device layout) and the 64
//          tokens' int8 activations (two 128-byte-swizzled 2-D boxes, the
//          UMMA K-major SW128 layout) into a 3-stage ring;
//   1      TMEM allocation and the MMA issue (one elected lane, descriptors
//          formed once and offset per instruction);
//   2..5   expansion of the raw block into the three planes (one row per
//          thread, written in the SW128 layout the MMA descriptors name);
//   6..21  epilogue: tcgen05.ld of the three accumulators, the block's float
//          term and the GEMV-order tree (a warp: 32 rows x 16 tokens), the
//          output rows.
// Tensor memory (all 512 columns): two accumulator sets of one block each
// (3 planes x 64 columns), so the MMAs of block s+1 run while block s is
// drained, and the tree's two pending partial sums of every (row, token)
// (columns 384..511); the running total and the third pending term stay in
// registers. Every wait is bounded; a CTA that gives up raises the error
// flag, lets its copies and MMAs land, frees its tensor memory and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "layout.cuh"
#include "stream_common.cuh"
#include "tma.cuh"

namespace fb {

namespace tc {

constexpr int BM = 128, BN = 64, NS = 3;
constexpr int kWBytes = BM * 144;                 // raw block of 128 rows
constexpr int kXHalf = BN * 128;                  // 64 tokens x 128 activations (one SW128 box)
constexpr int kStage = kWBytes + 2 * kXHalf;      // 34816 = 34 KiB
constexpr int kPlane = BM * 128;                  // 128 rows x 128 values
constexpr int kPlanes = 3 * kPlane;               // one half-block's three planes
constexpr int kRingOff = 0;
constexpr int kPlaneOff = NS * kStage;            // 104448 (1 KiB aligned)
constexpr int kBarOff = kPlaneOff + 2 * kPlanes;  // 202752
constexpr int kSmem = kBarOff + 256 + 1024;       // barriers + TMEM address + alignment slack
constexpr int kEpiWarps = 16;                     // 4 TMEM lane quarters x 4 runs of 16 tokens
constexpr int kThreads = (6 + kEpiWarps) * 32;
constexpr int kTmemCols = 512;
constexpr int kAccCols = 3 * BN;                  // one block's three accumulators
constexpr int kPaCol = 2 * kAccCols, kPbCol = kPaCol + BN;   // tree state: pending sums pa, pb
constexpr int kMaxBlocks = 128;                   // K <= 32768
static_assert(kStage % 1024 == 0 && kPlane % 1024 == 0, "SW128 atoms need 1 KiB alignment");
static_assert(kPbCol + BN <= kTmemCols, "tensor memory budget");

// barrier slots (uint64 each) at kBarOff
enum { B_FULL = 0, B_EMPTY = NS, B_PFULL = 2 * NS, B_PEMPTY = 2 * NS + 2, B_AFULL = 2 * NS + 4, B_AEMPTY = 2 * NS + 6,
       B_DRAIN = 2 * NS + 8, B_COUNT = 2 * NS + 9 };

// ---- PTX wrappers (tcgen05 / TMA), sm_100a
__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, int c4,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
        "%6}], [%7];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// D[tmem] (+)= A[smem] . B[smem]^T, int8 x int8 -> int32
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
// arrive on an mbarrier once every MMA issued so far by this thread completed
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// 16 consecutive 32-bit columns of this warp's 32 lanes
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
// 8 consecutive 32-bit columns of this warp's 32 lanes
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, int (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
                 "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
                 "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
                 : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms of
// 1 KiB (stride byte offset 1024), version 1 (sm_100).
__device__ __forceinline__ uint64_t sw128_desc(const void* p) {
    const uint32_t a = smem_u32(p);
    return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)2 << 61);
}
// Instruction descriptor: s8 x s8 -> s32, both K-major, M = 128, N = BN.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

// byte offset of (row, 16-byte chunk c) in a 128-byte-swizzled K-major tile
__device__ __forceinline__ uint32_t sw128_off(int row, int c) { return (uint32_t)(row * 128 + ((c ^ (row & 7)) << 4)); }

}  // namespace tc

struct TcArgs {
    GemvSeg g;
    const float* dk;     // [T][K/256] activation scales
    int K, T, nsteps, n_full;   // nsteps = K / 256; n_full = blocks in whole 2048-value groups
    int* err;
    // K split (narrow matrices): CTA z takes the half-group units (4 blocks)
    // [z U, (z + 1) U) and writes each unit's tree value to
    // part[(unit * T + t) * rows + row]; k_gemm_unit_reduce finishes the rows.
    // U = 0: one CTA per (row tile, token tile) over all of K.
    int units_per_cta;
    float* part;
};

__global__ void __launch_bounds__(tc::kThreads, 1)
    k_gemm_tc_q4k(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap wtail,
                  const __grid_constant__ CUtensorMap xmap, TcArgs args) {
    using namespace tc;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kBarOff);
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + kBarOff + 8 * B_COUNT);
    volatile int* s_abort = reinterpret_cast<volatile int*>(sm + kBarOff + 8 * B_COUNT + 8);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * BN, row0 = blockIdx.y * BM;
    const bool split = args.units_per_cta > 0;
    // this CTA's blocks [sb0, sb0 + nsteps) of the row (local step s = block sb0 + s)
    const int sb0 = split ? 4 * (int)blockIdx.z * args.units_per_cta : 0;
    const int nsteps = split ? min(args.nsteps - sb0, 4 * args.units_per_cta) : args.nsteps;
    pdl_trigger();

    if (threadIdx.x == 0) {
        *s_abort = 0;
        for (int s = 0; s < NS; ++s) {
            mbar_init(&bar[B_FULL + s], 1);
            mbar_init(&bar[B_EMPTY + s], 5);   // four expansion warps + the MMA commit
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bar[B_PFULL + i], 4);
            mbar_init(&bar[B_PEMPTY + i], 1);
            mbar_init(&bar[B_AFULL + i], 1);
            mbar_init(&bar[B_AEMPTY + i], kEpiWarps);
        }
        mbar_init(&bar[B_DRAIN], 1);
        mbar_fence_init();
    }
    if (warp == 1) tmem_alloc(s_tmem, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    pdl_wait();

    if (warp == 0) {
        // ---- TMA producer
        if (lane == 0) {
            int s = 0;
            for (; s < nsteps; ++s) {
                const int st = s % NS;
                if (s >= NS && !mbar_wait(&bar[B_EMPTY + st], (uint32_t)(((s / NS) - 1) & 1), s_abort)) break;
                uint8_t* stage = sm + kRingOff + st * kStage;
                const int sg = sb0 + s;
                mbar_expect_tx(&bar[B_FULL + st], (uint32_t)kStage);
                if (sg < args.n_full) tma_load_5d(stage, &wmap, 0, sg & 7, 0, sg >> 3, row0 / 8, &bar[B_FULL + st]);
                else tma_load_5d(stage, &wtail, 0, sg - args.n_full, 0, 0, row0 / 8, &bar[B_FULL + st]);
                tma_load_2d(stage + kWBytes, &xmap, sg * 256, t0, &bar[B_FULL + st]);
                tma_load_2d(stage + kWBytes + kXHalf, &xmap, sg * 256 + 128, t0, &bar[B_FULL + st]);
            }
            if (s < nsteps) {
                if (args.err) atomicExch(args.err, 4);
                *s_abort = 1;
            }
            // let the copies in flight land before the CTA can exit
            for (int k = (s > NS ? s - NS : 0); k < s; ++k)
                mbar_wait_bounded(&bar[B_FULL + k % NS], (uint32_t)((k / NS) & 1));
        }
    } else if (warp == 1) {
        // ---- MMA issue: block s accumulates into set s & 1
        if (lane == 0) {
            // descriptor = start address >> 4 in the low bits: a byte offset X
            // (16-byte multiple, inside shared memory) is + (X >> 4)
            const uint64_t a0 = sw128_desc(sm + kPlaneOff), b0 = sw128_desc(sm + kRingOff + kWBytes);
            bool ok = true;
            int s = 0;
            for (; s < nsteps && ok; ++s) {
                const int st = s % NS, ab = s & 1;
                if (s >= 2) {
                    ok = mbar_wait(&bar[B_AEMPTY + ab], (uint32_t)(((s >> 1) - 1) & 1), s_abort);
                    tc_fence_after();
                }
                if (ok) ok = mbar_wait(&bar[B_FULL + st], (uint32_t)((s / NS) & 1), s_abort);
                for (int h = 0; h < 2 && ok; ++h) {
                    const int q = 2 * s + h, pb = q & 1;
                    ok = mbar_wait(&bar[B_PFULL + pb], (uint32_t)((q >> 1) & 1), s_abort);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t ab0 = a0 + (uint64_t)((pb * kPlanes) >> 4);
                    const uint64_t bb0 = b0 + (uint64_t)((st * kStage + h * kXHalf) >> 4);
#pragma unroll
                    for (int j = 0; j < 3; ++j) {
                        const uint32_t d = tmem + (uint32_t)(ab * kAccCols + j * BN);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            umma_i8(d, ab0 + (uint64_t)((j * kPlane + 32 * kk) >> 4), bb0 + (uint64_t)((32 * kk) >> 4),
                                    kIdesc, (h > 0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit(&bar[B_PEMPTY + pb]);
                }
                if (!ok) break;
                umma_commit(&bar[B_EMPTY + st]);
                umma_commit(&bar[B_AFULL + ab]);
            }
            if (!ok) {
                if (args.err) atomicExch(args.err, 4);
                *s_abort = 1;
            }
            // the MMAs issued so far read shared memory and write tensor
            // memory: wait for them before anyone frees either
            umma_commit(&bar[B_DRAIN]);
            mbar_wait_bounded(&bar[B_DRAIN], 0u);
        }
    } else if (warp < 6) {
        // ---- expansion: row r of the raw block into the three planes
        const int r = threadIdx.x - 64;   // 0..127
        bool ok = true;
        for (int s = 0; s < nsteps && ok; ++s) {
            const int st = s % NS;
            ok = mbar_wait(&bar[B_FULL + st], (uint32_t)((s / NS) & 1), s_abort);
            if (!ok) break;
            const uint8_t* blk = sm + kRingOff + st * kStage + r * 144;
            const uint4 hd = *reinterpret_cast<const uint4*>(blk);   // d, dmin, 12 bytes of scales / mins
            // 6-bit scales and mins of the 8 sub-blocks (scale_min_k4, src/quant.cpp:136-144)
            const uint32_t sclo = hd.y & 0x3F3F3F3Fu, mlo = hd.z & 0x3F3F3F3Fu;
            const uint32_t schi = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
            const uint32_t mhi = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
            for (int h = 0; h < 2; ++h) {
                const int q = 2 * s + h, pb = q & 1;
                if (q >= 2 && !mbar_wait(&bar[B_PEMPTY + pb], (uint32_t)(((q >> 1) - 1) & 1), s_abort)) {
                    ok = false;
                    break;
                }
                uint8_t* planes = sm + kPlaneOff + pb * kPlanes;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    // values 16c .. 16c+15 of this half: sub-block g = 4h + c/2,
                    // codes qs[32 (g/2) + 16 (c%2) ..], low nibbles for even g
                    const int g = 4 * h + (c >> 1);
                    const uint4 raw = *reinterpret_cast<const uint4*>(blk + 16 + 32 * (g >> 1) + 16 * (c & 1));
                    const int sh = (g & 1) ? 4 : 0;
                    const uint32_t sc = (uint32_t)((g < 4 ? sclo : schi) >> (8 * (g & 3))) & 0xFFu;
                    const uint32_t mm = (uint32_t)((g < 4 ? mlo : mhi) >> (8 * (g & 3))) & 0xFFu;
                    const uint32_t hi = sc >> 3, lo = sc & 7u;
                    uint4 n;
                    n.x = (raw.x >> sh) & 0x0F0F0F0Fu;
                    n.y = (raw.y >> sh) & 0x0F0F0F0Fu;
                    n.z = (raw.z >> sh) & 0x0F0F0F0Fu;
                    n.w = (raw.w >> sh) & 0x0F0F0F0Fu;
                    const uint4 vh = make_uint4(n.x * hi, n.y * hi, n.z * hi, n.w * hi);   // bytes <= 105: no carries
                    const uint4 vl = make_uint4(n.x * lo, n.y * lo, n.z * lo, n.w * lo);
                    const uint32_t m4 = mm * 0x01010101u;
                    const uint32_t o = sw128_off(r, c);
                    *reinterpret_cast<uint4*>(planes + o) = vh;
                    *reinterpret_cast<uint4*>(planes + kPlane + o) = vl;
                    *reinterpret_cast<uint4*>(planes + 2 * kPlane + o) = make_uint4(m4, m4, m4, m4);
                }
                fence_async_smem();   // generic-proxy writes -> visible to the tensor cores
                __syncwarp();
                if (lane == 0) mbar_arrive(&bar[B_PFULL + pb]);
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar[B_EMPTY + st]);   // the raw block is expanded
        }
        if (!ok) {
            if (args.err && lane == 0) atomicExch(args.err, 4);
            *s_abort = 1;
        }
    } else {
        // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. (its rows),
        // columns of tokens 16 tq .. 16 tq + 15 of the tile
        const int lg = warp & 3, tq = (warp - 6) >> 2;
        const int row = row0 + 32 * lg + lane;
        const bool row_ok = row < args.g.rows;
        const int K = args.K, nb = K / 256;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * lg) << 16);
        // per (row, token): acc (the running row value) and pc (a group's
        // pending third term) in registers, pa / pb (its pending pair sums)
        // in tensor memory; the GEMV order of a group's 8 block terms t_b is
        //   ((t0 + t1) + (t2 + t3)) + ((t4 + t5) + (t6 + t7)), acc += group
        float acc[16], pc[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = pc[i] = 0.0f;
        // split mode: a finished half-group unit's value for tokens 8c..8c+7
        auto unit_out = [&](int unit, int c, const float (&v)[8]) {
            if (!row_ok) return;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int t = t0 + 16 * tq + 8 * c + k;
                if (t < args.T) args.part[((size_t)unit * args.T + t) * args.g.rows + row] = v[k];
            }
        };
        // one block's terms (t) into the tree: case bi of the group; in split
        // mode the half-group values ((t0 + t1) + (t2 + t3)) and
        // ((t4 + t5) + (t6 + t7)) go out at bi = 3 and 7 instead
        auto push = [&](int bi, int c, const float (&t)[8], int unit) {
            const uint32_t ca = lane_base + (uint32_t)(kPaCol + 16 * tq + 8 * c);
            const uint32_t cb = lane_base + (uint32_t)(kPbCol + 16 * tq + 8 * c);
            float v[8], w[8];
            int iv[8], iw[8];
            switch (bi) {
                case 0: tmem_st8(ca, t); break;
                case 1: case 3:
                    tmem_ld8(ca, iv);
                    tmem_ld_wait();
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        v[k] = __fadd_rn(__int_as_float(iv[k]), bi == 1 ? t[k] : __fadd_rn(pc[8 * c + k], t[k]));
                    tmem_st8(ca, v);
                    if (split && bi == 3) unit_out(unit, c, v);
                    break;
                case 2: case 6:
#pragma unroll
                    for (int k = 0; k < 8; ++k) pc[8 * c + k] = t[k];
                    break;
                case 4: tmem_st8(cb, t); break;
                case 5:
                    tmem_ld8(cb, iw);
                    tmem_ld_wait();
#pragma unroll
                    for (int k = 0; k < 8; ++k) w[k] = __fadd_rn(__int_as_float(iw[k]), t[k]);
                    tmem_st8(cb, w);
                    break;
                default:
                    if (split) {
                        tmem_ld8(cb, iw);
                        tmem_ld_wait();
#pragma unroll
                        for (int k = 0; k < 8; ++k) w[k] = __fadd_rn(__int_as_float(iw[k]), __fadd_rn(pc[8 * c + k], t[k]));
                        unit_out(unit, c, w);
                        break;
                    }
                    tmem_ld8(ca, iv);
                    tmem_ld8(cb, iw);
                    tmem_ld_wait();
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        acc[8 * c + k] = __fadd_rn(acc[8 * c + k],
                            __fadd_rn(__int_as_float(iv[k]), __fadd_rn(__int_as_float(iw[k]), __fadd_rn(pc[8 * c + k], t[k]))));
            }
        };
        bool ok = true;
        for (int s = 0; s < nsteps && ok; ++s) {
            const int sg = sb0 + s, ab = s & 1, bi = sg & 7;
            // this block's scales, fetched before the wait for its MMAs
            float dx[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int t = t0 + 16 * tq + i;
                dx[i] = t < args.T ? __ldg(args.dk + (size_t)t * nb + sg) : 0.0f;
            }
            const uint32_t hw =
                row_ok ? __ldg(reinterpret_cast<const uint32_t*>(args.g.w + block_offset_tm(T_Q4_K, K, row, sg))) : 0u;
            ok = mbar_wait(&bar[B_AFULL + ab], (uint32_t)((s >> 1) & 1), s_abort);
            if (!ok) break;
            tc_fence_after();
            const float dw = h2f((uint16_t)(hw & 0xFFFFu)), dmw = h2f((uint16_t)(hw >> 16));
            const uint32_t base = lane_base + (uint32_t)(ab * kAccCols + 16 * tq);
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                int d0[8], d1[8], d2[8];
                tmem_ld8(base + 8 * c, d0);
                tmem_ld8(base + BN + 8 * c, d1);
                tmem_ld8(base + 2 * BN + 8 * c, d2);
                tmem_ld_wait();
                if (c == 1) {   // the set's last read: let the next block's MMAs write it
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bar[B_AEMPTY + ab]);
                }
                float t[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) t[k] = q4k_term(dw, dmw, dx[8 * c + k], 8 * d0[k] + d1[k], d2[k]);
                push(bi, c, t, sg >> 2);
                // a row's last group may be short: its missing blocks add +0
                // (to the end of the group, or of the half-group unit)
                if (sg == nb - 1) {
                    float z[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) z[k] = 0.0f;
                    const int zend = split && bi < 4 ? 4 : 8;
                    for (int zb = bi + 1; zb < zend; ++zb) push(zb, c, z, sg >> 2);
                }
            }
            tmem_st_wait();
        }
        if (!ok) {
            if (args.err && lane == 0) atomicExch(args.err, 4);
            *s_abort = 1;
        }
        if (ok && !*s_abort && row_ok && !split) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int t = t0 + 16 * tq + i;
                if (t < args.T) store_out(args.g, row, t, acc[i]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// The rows of a K-split call: group g = unit 2g + unit 2g + 1 (a missing
// second half is +0, as the tree's zero pushes give), acc += group in order,
// then the output step of the unsplit kernel.
__global__ void __launch_bounds__(256) k_gemm_unit_reduce(GemvSeg g, const float* __restrict__ part, int n_units, int T) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.x * blockDim.x + threadIdx.x, t = blockIdx.y;
    if (row >= g.rows || t >= T) return;
    float acc = 0.0f;
    for (int u = 0; u < n_units; u += 2) {
        const float h0 = part[((size_t)u * T + t) * g.rows + row];
        const float h1 = u + 1 < n_units ? part[((size_t)(u + 1) * T + t) * g.rows + row] : 0.0f;
        acc = __fadd_rn(acc, __fadd_rn(h0, h1));
    }
    store_out(g, row, t, acc);
}

}  // namespace fb

using namespace fb;

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

bool encode_fn() {
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return g_encode != nullptr;
}

// Raw Q4_K blocks of 128 rows: the tile-major layout viewed as
// [tiles][groups][8 rows][blocks in group][144 bytes]; one box = one block
// of 16 tiles (128 rows), rows land contiguously at 144 bytes.
bool make_wmap(CUtensorMap* m, const uint8_t* base, int gb, int n_groups, int n_tiles, size_t tile_stride) {
    const cuuint64_t dims[5] = {144, (cuuint64_t)gb, 8, (cuuint64_t)n_groups, (cuuint64_t)n_tiles};
    const cuuint64_t gbytes = (cuuint64_t)group_bytes(T_Q4_K, gb);
    const cuuint64_t strides[4] = {144, gbytes, 8 * gbytes, (cuuint64_t)tile_stride};
    const cuuint32_t box[5] = {144, 1, 8, 1, 16};
    const cuuint32_t es[5] = {1, 1, 1, 1, 1};
    return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 5, const_cast<uint8_t*>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Whether the tcgen05 kernel can take a Q4_K call: K a multiple of 256,
// 16-byte aligned operands (TMA), at least 16 tokens. FISH_NO_TC=1 turns it
// off. fbk_gemm routes 16-32 tokens here only for narrow matrices (K split).
extern "C" int fbk_gemm_tc_eligible(const GemvSeg* g, const ActQ* a, int K, int T) {
    static const bool off = getenv("FISH_NO_TC") != nullptr;
    if (off || g->type != T_Q4_K || K % 256 || K / 256 > tc::kMaxBlocks || T < 16 || g->expert || g->amax) return 0;
    if ((reinterpret_cast<uintptr_t>(g->w) & 15) || (reinterpret_cast<uintptr_t>(a->qk) & 15) || a->ld % 16) return 0;
    return encode_fn() ? 1 : 0;
}

extern "C" int fbk_gemm_tc(const GemvSeg* g, const ActQ* a, int K, int T, int* err, float* part, size_t part_floats,
                           cudaStream_t st) {
    if (!fbk_gemm_tc_eligible(g, a, K, T)) return (int)cudaErrorInvalidValue;
    const int nb = K / 256, n_full_groups = nb / 8, tail = nb % 8;
    const int n_tiles = (g->rows + kTileRows - 1) / kTileRows;
    const size_t rb = row_bytes_dev(T_Q4_K, K);
    const size_t tile_stride = (size_t)kTileRows * rb;
    CUtensorMap wmap, wtail, xmap;
    std::memset(&wmap, 0, sizeof(wmap));
    std::memset(&wtail, 0, sizeof(wtail));
    if (n_full_groups > 0 && !make_wmap(&wmap, g->w, 8, n_full_groups, n_tiles, tile_stride))
        return (int)cudaErrorInvalidValue;
    if (tail > 0 &&
        !make_wmap(&wtail, g->w + (size_t)kTileRows * group_offset(T_Q4_K, n_full_groups), tail, 1, n_tiles, tile_stride))
        return (int)cudaErrorInvalidValue;
    if (n_full_groups == 0) wmap = wtail;
    if (tail == 0) wtail = wmap;
    {
        const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)T};
        const cuuint64_t strides[1] = {(cuuint64_t)a->ld};
        const cuuint32_t box[2] = {128, (cuuint32_t)tc::BN};
        const cuuint32_t es[2] = {1, 1};
        if (g_encode(&xmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a->qk, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return (int)cudaErrorInvalidValue;
    }
    static cudaError_t attr =
        cudaFuncSetAttribute(k_gemm_tc_q4k, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::kSmem);
    if (attr != cudaSuccess) return (int)attr;
    TcArgs args;
    args.g = *g;
    args.dk = a->dk;
    args.K = K;
    args.T = T;
    args.nsteps = nb;
    args.n_full = 8 * n_full_groups;
    args.err = err;
    args.units_per_cta = 0;
    args.part = part;
    // token tiles fastest: the CTAs that share a 128-row weight tile run
    // together, so its bytes come from HBM once and from L2 after
    dim3 grid((T + tc::BN - 1) / tc::BN, (g->rows + tc::BM - 1) / tc::BM);
    // fewer tiles than SMs (one CTA fits an SM): split K in half-group units
    // so about one CTA per SM streams the matrix
    static const int sms = [] {
        int dev = 0, n = 148;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            n = 148;
        return n;
    }();
    static const bool no_split = getenv("FISH_TC_NO_SPLIT") != nullptr;
    const int tiles = (int)(grid.x * grid.y), n_units = (nb + 3) / 4;
    if (part && !no_split && tiles < sms && n_units > 1 && (size_t)n_units * T * g->rows <= part_floats) {
        const int want = std::min(n_units, (sms + tiles - 1) / tiles);   // CTAs per tile
        const int U = (n_units + want - 1) / want;
        const int splits = (n_units + U - 1) / U;
        if (splits > 1) {
            args.units_per_cta = U;
            grid.z = splits;
        }
    }
    cudaError_t e = fbk_launch(k_gemm_tc_q4k, grid, dim3(tc::kThreads), (size_t)tc::kSmem, st, wmap, wtail, xmap, args);
    if (e != cudaSuccess || !args.units_per_cta) return (int)e;
    return fbk_gemm_unit_reduce(g, part, n_units, T, st);
}

extern "C" int fbk_gemm_unit_reduce(const GemvSeg* g, const float* part, int n_units, int T, cudaStream_t st) {
    return (int)fbk_launch(k_gemm_unit_reduce, dim3((g->rows + 255) / 256, T), dim3(256), 0, st, *g, part, n_units, T);
}
