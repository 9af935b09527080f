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
void repack_rows(int type, const uint8_t* src, int rows, int n_in, uint8_t* dst);

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
};

constexpr int kMaxSeg = 4;

// Prologue of the streamed GEMV: where its int8 activations come from.
//   PRO_ACT    quantised planes already in global memory (GemvArgs::act)
//   PRO_NORM   RMSNorm of f32 rows src (weights w, eps), then quantised
//   PRO_QUANT  f32 rows src, quantised
//   PRO_SILU   silu(src) * src2, quantised
enum : int { PRO_ACT = 0, PRO_NORM = 1, PRO_QUANT = 2, PRO_SILU = 3 };
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
    GemvPro pro;            // streamed kernel only (T <= 4, quantised segments)
    int swiglu;             // streamed kernel, 2 segments of equal rows (gate, up): the output
                            // is h = silu(gate) * up into segment 0's y (src/model.cpp:1501-1506)
    int* err;               // device error flag (nullable): 3 = weight read out of range
};

}  // namespace fb

extern "C" {
int fbk_quantize_rows(const float* x, int ldx, int T, int K, const fb::ActQ* a, int want32, int wantk, cudaStream_t st);
int fbk_rmsnorm_quant(const float* x, int ldx, const float* w, float eps, int T, int K, float* xb, int ldxb,
                      const fb::ActQ* a, int want32, int wantk, cudaStream_t st);
int fbk_silu_mul_quant(const float* g, int ldg, const float* u, int ldu, int T, int F, float* h, int ldh,
                       const fb::ActQ* a, int want32, int wantk, cudaStream_t st);
int fbk_gemv(const fb::GemvArgs* args, cudaStream_t st);
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
};
// RoPE on q (in place) and k, then K/V stored at each token's position.
int fbk_rope_append(float* q, int ldq, const float* k, const float* v, int ldkv, int T, int H, int HKV, int D,
                    int rot, int neox, const float* rope_cos, const float* rope_sin, KvView kv, int layer,
                    cudaStream_t st);
// Scratch (floats) fbk_attention needs for T tokens at contexts <= max_ctx.
size_t fbk_attention_scratch_floats(int T, int H, int D, int max_ctx);
// Causal GQA attention for T query tokens, output [T][H*D]; max_ctx bounds
// every tok_pos[t] + 1 (it sizes the key splits). D must be 64 or 128.
int fbk_attention(const float* q, int ldq, int T, int H, int HKV, int D, float scale, KvView kv, int layer,
                  float* out, int ldo, float* scratch, size_t scratch_floats, int max_ctx, cudaStream_t st);
// Decode attention for T tokens of T distinct sequences, RoPE and the K/V
// append fused: q and k/v are the raw projections [T][...]; the new rows are
// stored at each token's position; out [T][H*D]. Page size 16. One cluster
// of CTAs per (token, kv head); no scratch.
int fbk_attention_decode(const float* q, int ldq, const float* k, const float* v, int ldkv, int T, int H, int HKV, int D,
                         float scale, int rot, int neox, const float* rope_cos, const float* rope_sin, KvView kv,
                         int layer, float* out, int ldo, cudaStream_t st);
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
// Argmax keys (value, first index) accumulated by a GEMV's epilogue
// (GemvSeg::amax): decode them into out[t] / advance a greedy loop like
// fbk_greedy_advance, and reset the keys for the next step.
int fbk_argmax_from_keys(unsigned long long* keys, int T, int32_t* out, cudaStream_t st);
int fbk_greedy_from_keys(unsigned long long* keys, int32_t* ids, int32_t* tok_pos, int32_t* out, int32_t* step,
                         cudaStream_t st);
int fbk_moe_route(const float* logits, int T, int NE, int K, int norm, int32_t* sel, float* wsel, cudaStream_t st);
}
