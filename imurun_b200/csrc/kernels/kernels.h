// kernels.h — launch interface between the host engine and the CUDA kernels.
// Internal to libfish.so; the public C ABI lives in include/fish/c_api.h.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "common.cuh"

namespace fb {

// Device weight layouts (layout.cuh): quantised matrices are tile-major
// (8-row tiles, inside a tile group pieces ordered group first), F32/F16
// matrices row-major with rows padded to 16 bytes.
size_t dev_row_bytes(int type, int n_in);
size_t dev_matrix_bytes(int type, int n_in, int rows);
// Repack `rows` consecutive GGUF rows (the first one starting a tile) into
// the device layout at dst (dev_matrix_bytes(type, n_in, rows) bytes).
// Repack `rows` GGUF rows of n_in values into the device layout at dst (whole
// 8-row tiles). src_stride: bytes from one source row to the next (0 = the
// rows are contiguous; larger for a slice of K-blocks of wider rows).
void repack_rows(int type, const uint8_t* src, int rows, int n_in, uint8_t* dst, size_t src_stride = 0);

// Epilogue of a GEMV segment.
enum : int { EPI_STORE = 0, EPI_ADD = 1 };

struct GemvSeg {
    int type;
    const uint8_t* w;       // device matrix (tile-major for quantised types)
    size_t row_stride;
    int rows;               // output rows in this segment
    float* y;               // output [T][ldy]
    int ldy;
    const float* bias;      // optional per-row bias
    int epi;                // EPI_STORE / EPI_ADD
    const int32_t* expert;  // optional: rows start at w + (*expert) * expert_bytes
    size_t expert_bytes;
    size_t w_bytes;         // bytes readable from w (every expert); reads outside are skipped and flagged
    unsigned long long* amax;  // optional [T]: running argmax key per token (streamed kernel, EPI_STORE)
    int key_row0;           // added to the row index in argmax keys (a vocab slice's first global row)
};

constexpr int kMaxSeg = 4;

// Prologue of the streamed GEMV: where its int8 activations come from.
//   PRO_ACT    quantised planes already in global memory (GemvArgs::act)
//   PRO_NORM   RMSNorm of f32 rows src (weights w, eps), then quantised
//   PRO_QUANT  f32 rows src, quantised
//   PRO_SILU   silu(src) * src2, quantised
//   PRO_MERGE  one token's decode-attention partials of ld key chunks (head
//              dim ld2; acc [C][H][D] then (m, l) [C][H][2] at src), merged
//              and quantised (persistent decode step)
enum : int { PRO_ACT = 0, PRO_NORM = 1, PRO_QUANT = 2, PRO_SILU = 3, PRO_MERGE = 4 };
struct GemvPro {
    int mode;
    const float* src;
    int ld;
    const float* src2;
    int ld2;
    const float* w;
    float eps;
};

struct GemvArgs {
    GemvSeg seg[kMaxSeg];
    int nseg;
    int K;                  // input length
    int T;                  // tokens
    ActQ act;               // quantised activations (per type layout)
    const float* xf;        // f32 activations [T][ldxf] for F32/F16 weights
    int ldxf;
    GemvPro pro;            // streamed kernel only (T <= 8, quantised segments)
    int swiglu;             // streamed kernel, 2 segments of equal rows (gate, up): the output
                            // is h = silu(gate) * up into segment 0's y (src/model.cpp:1501-1506)
    int* err;               // device error flag (nullable): 3 = weight read out of range
    uint8_t* img_dump;      // debug (nullable, streamed kernel): CTA 0 copies its activation image here
                            // after the prologue: 16-byte header (xk bytes, x32 bytes, T, n256 as int32)
                            // then T * (xk + x32) bytes laid out as XImage (stream_common.cuh)
    float* part;            // tensor-core GEMM scratch for K-split calls (nullable: no split)
    size_t part_floats;
};

}  // namespace fb

extern "C" {
int fbk_quantize_rows(const float* x, int ldx, int T, int K, const fb::ActQ* a, int want32, int wantk, cudaStream_t st);
int fbk_rmsnorm_quant(const float* x, int ldx, const float* w, float eps, int T, int K, float* xb, int ldxb,
                      const fb::ActQ* a, int want32, int wantk, cudaStream_t st);
int fbk_silu_mul_quant(const float* g, int ldg, const float* u, int ldu, int T, int F, float* h, int ldh,
                       const fb::ActQ* a, int want32, int wantk, cudaStream_t st);
// h = act(g) * u, quantised: act = silu, or the tanh form of GELU (gelu = 1)
int fbk_act_mul_quant(const float* g, int ldg, const float* u, int ldu, int T, int F, float* h, int ldh,
                      const fb::ActQ* a, int want32, int wantk, int gelu, cudaStream_t st);
// x[t] += rmsnorm(y[t]) * w over K values (post norms)
int fbk_rmsnorm_add(float* x, int ldx, const float* y, int ldy, const float* w, float eps, int T, int K,
                    cudaStream_t st);
// x[i] *= s for n floats
int fbk_scale(float* x, size_t n, float s, cudaStream_t st);
// y[i] = sigmoid(x[i]) for n values (x null: y = 1)
int fbk_sigmoid(const float* x, float* y, int n, cudaStream_t st);
// rows of n logits (stride ldx): cap * tanh(x / cap)
int fbk_softcap(float* x, int n, int rows, int ldx, float cap, cudaStream_t st);
int fbk_gemv(const fb::GemvArgs* args, cudaStream_t st);
// Tokens per GEMV launch when a call has more than fit one: 8 (the streamed
// kernel's and the direct kernel's largest token count).
int fbk_gemv_chunk(const fb::GemvArgs* args);
// Batched products on the int8 tensor cores (gemm.cu): T >= 16 tokens,
// quantised planes already built (PRO_ACT), Q4_K / Q6_K / Q8_0 segments,
// K % 256 == 0. fbk_gemm_eligible says whether a job qualifies
// (FISH_NO_GEMM turns the path off).
int fbk_gemm_eligible(const fb::GemvArgs* args);
// Q4_K segments on the tcgen05 kernel (gemm_tc.cu): T >= 16, K % 256 == 0,
// 16-byte aligned operands; fbk_gemm takes it above 32 tokens, and at 16-32
// tokens for narrow matrices with K-split scratch.
int fbk_gemm_tc_eligible(const fb::GemvSeg* g, const fb::ActQ* a, int K, int T);
// part: scratch for a K split of narrow matrices (n_units * T * rows floats,
// n_units = ceil(K / 1024)); nullptr or too small runs unsplit.
int fbk_gemm_tc(const fb::GemvSeg* g, const fb::ActQ* a, int K, int T, int* err, float* part, size_t part_floats,
                cudaStream_t st);
int fbk_gemm(const fb::GemvArgs* args, cudaStream_t st);
// The rows of a K-split tensor-core call: the half-group unit values in part
// [n_units][T][rows] added as the unsplit kernels add them (group = first
// half + second half, then acc += group in order), then the output step.
int fbk_gemm_unit_reduce(const fb::GemvSeg* g, const float* part, int n_units, int T, cudaStream_t st);
// 1 if fbk_gemv runs this call on the streamed kernel (the only one that
// takes a prologue other than PRO_ACT).
int fbk_gemv_streamable(const fb::GemvArgs* args);
// Debug: per-(row, block) integer sums of one quantised matrix (bit-exact
// check of the GEMV's integer arithmetic). sumi/mins: [rows][nblocks].
int fbk_block_sums(int type, const uint8_t* w, int rows, int K, const fb::ActQ* a, int32_t* sumi, int32_t* mins,
                   cudaStream_t st);
// Programmatic dependent launch for every kernel launched after this call
// (in-order streams and graphs captured from them).
void fbk_set_pdl(int on);
// Device-time trace of kernel phases (diagnostics): enable with a record
// capacity (0 = off); dump returns the records (ns, tag, event, launch).
int fbk_trace_enable(int cap);
int fbk_trace_dump(unsigned long long* out, int cap);
int fbk_pdl_enabled(void);

// Embedding row gather + dequantisation: x[t][0..E) = dequant(embd row ids[t]).
int fbk_embed(int type, const uint8_t* w, int E, int n_rows, const int32_t* ids, int T, float* x, int ldx, int* err,
              cudaStream_t st);
// Shared device error flag of the kernels (0 = none); read-and-clear.
int* fbk_gemv_error_flag();
int fbk_take_error_flag();
// Bounded waits of the streamed GEMV that gave up since the last call: up to
// 8 records of 16 values (see gemv.cu) into rec[128]; returns how many
// occurred (may exceed 8).
int fbk_take_wait_record(long long* rec);

// Paged KV cache as the kernels see it. A page holds `page_size` positions of
// every layer: per layer a K block [HKV][page_size][D] then a V block of the
// same shape. Token t of a launch belongs to sequence slot tok_seq[t] (its page
// table is pt + tok_seq[t] * pt_stride) and sits at position tok_pos[t]; keys
// 0..tok_pos[t] are visible to it (causal).
struct KvView {
    void* k;                 // pool base + 0           (element type by f16)
    void* v;                 // pool base + HKV*P*D elements
    const int32_t* pt;       // page-table arena
    int pt_stride;           // entries per sequence slot
    const int32_t* tok_seq;  // [T]
    const int32_t* tok_pos;  // [T]
    int page_size;
    size_t page_stride;      // elements per page
    size_t layer_stride;     // elements per layer inside a page (2*HKV*P*D)
    size_t head_stride;      // elements per kv head block (P*D)
    int f16;
    int n_pages;             // pages in the pool (page indices outside are clamped and flagged)
    int* err;                // device error flag (nullable): 5 = page index out of range
    // gemma2: scores become softcap * tanh(score / softcap) (0: off), and a
    // token at pos sees keys pos - window + 1 .. pos only (0: all keys)
    float softcap = 0.0f;
    int window = 0;
};
// RoPE on q (in place) and k, then K/V stored at each token's position.
int fbk_rope_append(float* q, int ldq, const float* k, const float* v, int ldkv, int T, int H, int HKV, int D,
                    int rot, int neox, const float* rope_cos, const float* rope_sin, KvView kv, int layer,
                    cudaStream_t st);
// Scratch (floats) fbk_attention needs for T tokens at contexts <= max_ctx.
size_t fbk_attention_scratch_floats(int T, int H, int D, int max_ctx);
// scratch one fbk_attention call with exactly this max_ctx needs
size_t fbk_attention_call_floats(int T, int H, int D, int max_ctx);
// Causal GQA attention for T query tokens, output [T][H*D]; max_ctx bounds
// every tok_pos[t] + 1 (it sizes the key splits). D must be 64 or 128.
int fbk_attention(const float* q, int ldq, int T, int H, int HKV, int D, float scale, KvView kv, int layer,
                  float* out, int ldo, float* scratch, size_t scratch_floats, int max_ctx, cudaStream_t st);
// Decode attention for T tokens of T distinct sequences, RoPE and the K/V
// append fused: q and k/v are the raw projections [T][...]; the new rows are
// stored at each token's position; out [T][H*D]. Page size 16. One token:
// one cluster of CTAs per kv head, merged in distributed shared memory. More
// tokens with part (at least fbk_attention_decode_part_floats): the same key
// ranks as independent CTAs writing partials to part, then a merge launch;
// every token's output has the same bits on both paths.
// pre (device int, nullable): the number of leading 64-key blocks every
// token's sequence shares page for page, written before the step; with
// pstate (fbk_attention_prefix_state_floats) those blocks are read once for
// all tokens by a shared-prefix kernel whose warps continue into the decode
// kernel, again with the same bits per token.
int fbk_attention_decode(const float* q, int ldq, const float* k, const float* v, int ldkv, int T, int H, int HKV, int D,
                         float scale, int rot, int neox, const float* rope_cos, const float* rope_sin, KvView kv,
                         int layer, float* out, int ldo, float* part, size_t part_floats, const int* pre, float* pstate,
                         size_t pstate_floats, cudaStream_t st);
size_t fbk_attention_decode_part_floats(int T, int H, int HKV, int D);
// Prefill attention on tensor cores for the T tokens of ONE sequence at
// consecutive positions (kv.tok_seq / kv.tok_pos of token 0 ..), whose K/V
// rows are already in the fp16 cache (RoPE applied by fbk_rope_append): a
// CTA per (16 tokens, kv head), no scratch. D 64 or 128, G <= 8, page 16.
int fbk_attention_prefill(const float* q, int ldq, int T, int H, int HKV, int D, float scale, KvView kv, int layer,
                          float* out, int ldo, cudaStream_t st);
size_t fbk_attention_prefix_state_floats(int T, int HKV, int D);
// Blocks of 64 keys the shared-prefix kernel covers at most (16 key ranks x
// the blocks a rank keeps resident).
int fbk_attention_prefix_max_blocks(void);
// Per-head RMSNorm in place (q/k norm), rows [T][n_heads*D].
int fbk_head_rmsnorm(float* x, int ldx, int T, int n_heads, int D, const float* w, float eps, cudaStream_t st);
// MoE: x[t] += sum_k wsel[t][k] * eo[t][k][:]
int fbk_moe_combine(float* x, int ldx, const float* eo, const float* wsel, int T, int K, int E, cudaStream_t st);
// Greedy step bookkeeping for on-device decode loops: ids[0] = argmax,
// out[*step] = argmax, (*step)++, tok_pos[0]++.
int fbk_greedy_advance(const float* logits, int V, int32_t* ids, int32_t* tok_pos, int32_t* out, int32_t* step,
                       cudaStream_t st);
int fbk_add(float* y, const float* x, size_t n, cudaStream_t st);
// Device-side wait of ns nanoseconds (profiling aid).
int fbk_delay(unsigned long long ns, cudaStream_t st);
int fbk_argmax(const float* x, int n, int rows, int ldx, int32_t* out, cudaStream_t st);
// Greedy sampling with a repetition penalty on one row of n logits: each of
// the n_recent ids (device array, the sampler's window, <= kMaxRecent)
// penalises its logit once per occurrence, then out[0] = first index of the
// maximum. x is read, not modified.
constexpr int kMaxRecent = 256;
int fbk_argmax_penalized(const float* x, int n, const int32_t* recent, int n_recent, float penalty, int32_t* out,
                         cudaStream_t st);
// The same for `rows` rows of ldx floats: row r is penalised by the last
// `window` ids (<= kMaxRecent) of hist[0 .. base + r) and out[r] is its
// first maximum (the target's greedy choice after each accepted draft token).
int fbk_argmax_penalized_rows(const float* x, int n, int rows, int ldx, const int32_t* hist, int base, int window,
                              float penalty, int32_t* out, cudaStream_t st);
// Argmax keys (value, first index) accumulated by a GEMV's epilogue
// (GemvSeg::amax): decode them into out[t] / advance a greedy loop like
// fbk_greedy_advance, and reset the keys for the next step.
int fbk_argmax_from_keys(unsigned long long* keys, int T, int32_t* out, cudaStream_t st);
int fbk_greedy_from_keys(unsigned long long* keys, int32_t* ids, int32_t* tok_pos, int32_t* out, int32_t* step,
                         cudaStream_t st);
int fbk_moe_route(const float* logits, int T, int NE, int K, int norm, int32_t* sel, float* wsel, cudaStream_t st);
// Expert parallelism: out[i] = sel[i] - e0 when this rank holds that expert
// (e0 <= sel[i] < e0 + n), else -1 (the expert GEMVs write zero rows for -1).
int fbk_moe_localize(const int32_t* sel, int n_sel, int e0, int n, int32_t* out, cudaStream_t st);
}
// A routed expert as this rank's local id (experts [e0, e0 + n) live here),
// -1 for another rank's: the device kernel and host checks share it.
__host__ __device__ inline int fb_localize_expert(int e, int e0, int n) { return (e >= e0 && e < e0 + n) ? e - e0 : -1; }
extern "C" {
// MoE router logits over F32 router rows: one warp per (token, expert),
// double accumulation; any token count.
int fbk_router_f32(const uint8_t* w, size_t ws, const float* x, int ldx, int T, int E, int NE, float* out, int ldo,
                   cudaStream_t st);
// Expert grouping of a batched MoE step (misc.cu): rows routed to each local
// expert packed into consecutive slots of S = 4 or 8 rows (expert e from
// slot sum_{e' < e} ceil(count_e' / S)), the expert of every slot for GEMV
// launches of S rows (-1 past the used slots), and the weighted combine read
// back through grp_pos. nslot >= fbk_moe_slots(T, K, nel, S).
int fbk_moe_group(const int32_t* esel, int T, int K, int nel, int32_t* grp_src, int32_t* grp_pos, int32_t* grp_count,
                  int32_t* chunk_exp, int nslot, int S, cudaStream_t st);
int fbk_moe_slots(int T, int K, int nel, int S);
int fbk_moe_gather(const fb::ActQ* src, const fb::ActQ* dst, const int32_t* grp_src, int ksel, int n_rows, int K,
                   cudaStream_t st);
int fbk_moe_combine_grouped(float* x, int ldx, const float* eo, const int32_t* grp_pos, const float* wsel, int T, int K,
                            int E, cudaStream_t st);
}

// ---------------------------------------------------------------- persistent decode step (step.cu)
namespace fb {
// One GEMV phase of the step program: the same job the streamed GEMV kernel
// runs (segments, prologue, epilogue; T = 1), with its tile split.
struct StepPhase {
    GemvArgs a;
    int tile0[kMaxSeg + 1];   // 8-row tiles per segment (prefix sums; pair mode interleaves)
    int n_units;              // tiles, or (gate, up) tile pairs
    int G;                    // 2048-value groups per row
    int xk_bytes, x32_bytes;  // activation image layouts the segments need
    int attn_layer;           // >= 0: that layer's attention runs before this phase
};
// Control block in device memory (zeroed before each launch).
struct StepCtl {
    unsigned int bar;         // grid-barrier arrivals, monotonic
    int abort;                // set by the first CTA that gives up
    int err;                  // first error: 1 ring wait, 2 grid barrier, 3 weight range, 4 token id, 5 page index
    int info[5];              // CTA, step, phase, stage, slot of the first failure
};
struct StepArgs {
    const StepPhase* ph;      // [n_ph]: per layer qkv, o, gate+up, down; then the output projection
    int n_ph;
    // attention
    const float *q, *k, *v;   // raw projections of the token (written by the qkv phase)
    float* att_part;          // partials: acc [C][H][D], then (m, l) [C][H][2]
    const float *rcos, *rsin; // RoPE table [n_ctx][rot/2]
    int H, HKV, D, rot, neox;
    float scale;
    int max_chunks;           // key chunks per kv head at most (HKV * max_chunks <= grid)
    KvView kv;
    int sid;                  // sequence slot (page-table row)
    // embedding and residual stream
    int emb_type;
    const uint8_t* emb;
    int E, emb_rows;
    float* x;
    // token state
    const int32_t* ids;       // ids[0]: first token
    const int32_t* tok_pos;   // tok_pos[0]: its position
    int32_t* out;             // [n_steps] greedy tokens (argmax of each step)
    int n_steps;
    unsigned long long* keys; // [2] argmax keys of even / odd steps (zeroed before launch)
    StepCtl* ctl;
    int S, slot_bytes, union_bytes;
    // optional phase trace (nullable): thread 0 of the first and the last CTA
    // store %globaltimer at each phase boundary into
    // trace[(step * kStepTraceEvents + event) * 2 + (last CTA ? 1 : 0)]
    unsigned long long* trace;
};
constexpr int kStepTraceEvents = 1024;
}  // namespace fb

extern "C" {
// Launch shape of the step kernel (G = q heads per kv head, f16 = fp16 KV
// cache) for a ring slot size and a union area
// (activation image + partials, or attention scratch): CTAs (1 per SM), ring
// slots, dynamic shared memory. Returns 0, or a CUDA error / -1 when it does
// not fit.
int fbk_step_plan(int G, int f16, int slot_bytes, int union_bytes, int* grid, int* stages, size_t* smem);
// Cooperative launch of n_steps greedy decode steps.
int fbk_step_decode(const fb::StepArgs* a, int grid, size_t smem, cudaStream_t st);
}
