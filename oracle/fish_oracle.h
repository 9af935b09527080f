/*
 * fish_oracle — CPU restatement of the FISH decode/prefill arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product library links or calls this
 * code; it exists so the tests, the smoke check and the CPU leg of bench.py can
 * check the CUDA path against an independent statement of the reference
 * algorithm. Each function names the reference file:line (paths relative to
 * the FISH project, model/fish/) whose behaviour it restates.
 *
 * Parity pin: the restatement is checked against the reference FISH build
 * (oracle/_ref, compiled from the reference sources by oracle/Makefile) on
 * seeded inputs, and against the reference's own known-answer tests
 * (test/test_m1.cpp:35-80, test/test_kernels.cpp:135-179); see
 * tests/test_oracle_pin.py.
 */
#ifndef FISH_ORACLE_H
#define FISH_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (include/fish/gguf.h:25-33). */
enum {
    OR_F32 = 0, OR_F16 = 1, OR_Q4_0 = 2, OR_Q8_0 = 8, OR_Q4_K = 12,
    OR_Q5_K = 13, OR_Q6_K = 14, OR_BF16 = 30
};

/* Activation blocks, byte layout identical to include/fish/quant.h:58-70. */
typedef struct { float d; int32_t sum; int8_t qs[32]; } or_q8act;          /* 40 B  */
typedef struct { float d; int16_t bsums[8]; int8_t qs[256]; } or_q8actk;   /* 276 B */

/* ---- scalars ------------------------------------------------------------ */
float    or_fp16_to_fp32(uint16_t h);           /* quant.cpp:21-44 */
uint16_t or_fp32_to_fp16(float f);              /* quantize.cpp:32-55 (RNE) */

/* ---- type table (gguf.cpp:215-275) ---------------------------------------- */
int      or_block_elems(int type);
int      or_block_bytes(int type);
uint64_t or_row_bytes(int type, uint64_t n);

/* ---- dequantisation (quant.cpp:83-216, 470-506) ---------------------------- */
int or_dequant_row(int type, const void* src, float* dst, uint64_t n);

/* ---- activation quantisers (quant.cpp:400-434) ------------------------------ */
void or_quantize_acts(const float* x, uint64_t n, or_q8act* out);
void or_quantize_acts_k(const float* x, uint64_t n, or_q8actk* out);

/* ---- integer block sums: the exact int32 quantities the reference's integer
 * kernels form per block (quant_x86.cpp:299-309, 346-382, 431-495).
 *   Q8_0 : s[b]    = sum_k w_k * x_k over the 32-block b
 *   Q4_0 : s[b]    = sum_k q_k * x_k (q in 0..15), offset 8*x.sum applied in fp
 *   Q4_K : sumi[b] = sum_g sc_g * sum_l q_gl * x_gl ; mins[b] = sum_g m_g * bsums_g
 *   Q6_K : sumi[b] = sum_j sc_j * sum_16 (q6 - 32) * x
 * `mins` may be NULL for types without a min term. Returns 0 for unsupported. */
int or_block_sums(int type, const void* row, const void* acts, uint64_t n,
                  int32_t* sumi, int32_t* mins);

/* Row dot products through the integer path, combined in double:
 * y = sum_b (fp16(d_w) * d_x) * sumi_b - (fp16(dmin_w) * d_x) * mins_b
 * (quant_x86.cpp:299-309, 346-382, 431-495). Returns 0 when the type has no
 * integer kernel of that layout (quant.cpp:475-481). */
int or_vec_dot_q8(int type, const void* row, const or_q8act* x, uint64_t n, float* out);
int or_vec_dot_q8k(int type, const void* row, const or_q8actk* x, uint64_t n, float* out);

/* Y[t][i] = W_i . X_t with the reference's choice of int8 path vs f32 path
 * (ops.cpp:177-264, incl. the K-layout rule ops.cpp:166-174). */
void or_matmul(int type, const void* w, const float* x, int n_tok, int n_in,
               int n_out, float* y);

/* ---- glue (ops.cpp:18-55) ----------------------------------------------------- */
void or_rmsnorm(float* out, const float* x, const float* w, int n, float eps);
void or_silu_inplace(float* x, int n);
void or_gelu_inplace(float* x, int n);
void or_softmax_inplace(float* x, int n);

/* RoPE table (ops.cpp:75-124): cos/sin [n_ctx][rot_dim/2]. */
typedef struct {
    int head_dim, rot_dim, neox;
    float freq_base, freq_scale, mscale;
    float yarn_factor, yarn_attn_factor, yarn_beta_fast, yarn_beta_slow;
    int yarn_orig_ctx;
    const float* freq_factors;     /* rot_dim/2 entries or NULL */
} or_rope_params;
void or_rope_build(float* cos_out, float* sin_out, int n_ctx, const or_rope_params* p);
/* ops.cpp:126-156, one token, q (n_head heads) and k (n_head_kv heads). */
void or_rope_apply(float* q, float* k, int n_head, int n_head_kv, int head_dim,
                   int rot_dim, int neox, const float* cos_row, const float* sin_row);

/* ops.cpp:303-356. Caches are [n_ctx][n_head_kv*head_dim] f32. */
void or_attention(const float* q, const float* k_cache, const float* v_cache,
                  int n_head, int n_head_kv, int head_dim, int pos0, int n_tok,
                  float* out, float scale, float softcap, int window);

/* ---- whole model (model.cpp:393-645 load, 1603-1811 forward) ------------------ */
typedef struct or_model or_model;

typedef struct {
    int n_layers, n_embd, n_ff, n_head, n_head_kv, head_dim, n_ctx, vocab;
    int n_experts, n_experts_per_tok, n_ff_exp, rot_dim, neox, tied_output;
    float eps, freq_base;
    int bos, eos;
} or_model_info;

/* kv_f16: 1 = round K/V through fp16 when they are stored (mirrors a device
 * fp16 KV cache); 0 = f32 like the reference (model.h:279-280). */
or_model* or_model_load(const char* path, int n_ctx, int kv_f16, char* err, int err_cap);
void      or_model_free(or_model* m);
int       or_model_info_of(const or_model* m, or_model_info* out);
/* Process n_tok tokens at pos0. When logits_all is non-NULL it receives
 * [n_tok][vocab] logits; `logits` always receives the last token's. */
int       or_model_forward(or_model* m, const int32_t* tokens, int n_tok, int pos0,
                           float* logits, float* logits_all);
void      or_model_set_kv_len(or_model* m, int n);
int       or_model_kv_len(const or_model* m);
/* int8 activations to use instead of the oracle's own quantisation, per
 * stage of a layer: 0 the attention-norm output (q/k/v input), 1 the
 * attention output (wo input), 2 the FFN-norm output (gate/up input, experts
 * included), 3 the SwiGLU product (down input; MoE: rows token * K + k in
 * selection order). qk: Q8ActK records [rows][K/256]; q32: Q8Act records
 * [rows][K/32]; a NULL entry leaves that stage to the oracle's quantiser. The
 * router (F32 weights) keeps the float path, as in the reference. */
typedef struct {
    const void* qk[4];
    const void* q32[4];
} or_layer_acts;

/* One layer alone (one iteration of the layer loop, model.cpp:1654-1785):
 * x_out = layer `layer` applied to x_in [n_tok][n_embd] at positions pos0..;
 * that layer's K/V rows are stored there. Returns 1, or 0 on a bad argument. */
int       or_model_layer(or_model* m, int layer, const float* x_in, int n_tok, int pos0, float* x_out);
/* The same with the int8 activations of `acts` (NULL: the oracle's own). */
int       or_model_layer_acts(or_model* m, int layer, const float* x_in, int n_tok, int pos0,
                              const or_layer_acts* acts, float* x_out);
/* The mapped GGUF data of a tensor (NULL when absent), its type and dims. */
const void* or_model_tensor(const or_model* m, const char* name, int* type, int64_t* ne0, int64_t* ne1,
                            int64_t* ne2);
/* Debug hook: copy of the final hidden state x (pre-norm) of the last token. */
int       or_model_last_hidden(const or_model* m, float* out, int n);
/* First index of the max value (model.cpp:1939-1946). */
int       or_argmax(const float* v, int n);

#ifdef __cplusplus
}
#endif
#endif
