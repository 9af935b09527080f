// kernels.h — launch interface between the host engine and the CUDA kernels.
// Internal to libfish.so; the public C ABI lives in include/fish/c_api.h.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "common.cuh"

namespace fb {

// Device weight layouts (a bijective repack of the GGUF blocks so that every
// row starts 16-byte aligned and every load is 8 or 16 bytes):
//   Q4_K  row = nb x 144 B blocks, unchanged (144 = 9 x 16)
//   Q6_K  row = nb x 208 B (ql 128 | qh 64 | scales 16) then nb x fp16 d,
//         padded to 16 B
//   Q8_0  row = nb x 32 B qs then nb x fp16 d, padded to 16 B
//   F32 / F16  row = n_in values, padded to 16 B
size_t dev_row_bytes(int type, int n_in);
// Repack one GGUF row (src) into the device layout (dst, dev_row_bytes wide).
void repack_row(int type, const uint8_t* src, uint8_t* dst, int n_in);

// Epilogue of a GEMV segment.
enum : int { EPI_STORE = 0, EPI_ADD = 1 };

struct GemvSeg {
    int type;
    const uint8_t* w;       // device rows (dev_row_bytes stride)
    size_t row_stride;
    int rows;               // output rows in this segment
    float* y;               // output [T][ldy]
    int ldy;
    const float* bias;      // optional per-row bias
    int epi;                // EPI_STORE / EPI_ADD
    const int32_t* expert;  // optional: rows start at w + (*expert) * expert_bytes
    size_t expert_bytes;
};

constexpr int kMaxSeg = 4;

struct GemvArgs {
    GemvSeg seg[kMaxSeg];
    int nseg;
    int K;                  // input length
    int T;                  // tokens
    ActQ act;               // quantised activations (per type layout)
    const float* xf;        // f32 activations [T][ldxf] for F32/F16 weights
    int ldxf;
};

}  // namespace fb

extern "C" {
int fbk_quantize_rows(const float* x, int ldx, int T, int K, const fb::ActQ* a, int want32, int wantk, cudaStream_t st);
int fbk_rmsnorm_quant(const float* x, int ldx, const float* w, float eps, int T, int K, float* xb, int ldxb,
                      const fb::ActQ* a, int want32, int wantk, cudaStream_t st);
int fbk_silu_mul_quant(const float* g, int ldg, const float* u, int ldu, int T, int F, float* h, int ldh,
                       const fb::ActQ* a, int want32, int wantk, cudaStream_t st);
int fbk_gemv(const fb::GemvArgs* args, cudaStream_t st);
// Debug: per-(row, block) integer sums of one quantised row set (bit-exact
// check of the GEMV's integer arithmetic). sumi/mins: [rows][nblocks].
int fbk_block_sums(int type, const uint8_t* w, size_t row_stride, int rows, int K, const fb::ActQ* a,
                   int32_t* sumi, int32_t* mins, cudaStream_t st);

// Embedding row gather + dequantisation: x[t][0..E) = dequant(embd row ids[t]).
int fbk_embed(int type, const uint8_t* w, size_t row_stride, int E, const int32_t* ids, int T, float* x, int ldx,
              cudaStream_t st);

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
int fbk_moe_route(const float* logits, int T, int NE, int K, int norm, int32_t* sel, float* wsel, cudaStream_t st);
}
