#pragma once
/*
 * Kernel-level entry points of the B200 engine (libfish.so), for parity tests
 * and for callers that want a single hot-path step without a model.
 *
 * Every function takes HOST buffers, runs the same device code the engine's
 * forward pass runs, and copies the result back. Return 0 on success, a
 * negative value on bad arguments, or a positive CUDA error code.
 *
 * Type ids are ggml's (GGUF specification): 0 F32, 1 F16, 8 Q8_0, 12 Q4_K,
 * 14 Q6_K. Weight rows are passed in GGUF block order.
 */
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef FISH_API
#  define FISH_API __attribute__((visibility("default")))
#endif

/* Activation quantisers, the reference's records byte for byte:
 * q8act  = rows x (K/32)  x 40 B  (Q8Act,  reference quant.cpp:400-415)
 * q8actk = rows x (K/256) x 276 B (Q8ActK, reference quant.cpp:417-434)
 * Either output may be NULL. Replaces the reference's quantize_acts /
 * quantize_acts_k (include/fish/quant.h:75-76) and ActBatch::quantize
 * (include/fish/ops.h:64-81). */
FISH_API int fbx_quantize_acts(const float* x, int rows, int K, void* q8act, void* q8actk);

/* RMSNorm (reference ops.cpp:18-23) of rows x K, written to out. */
FISH_API int fbx_rmsnorm(const float* x, const float* w, int rows, int K, float eps, float* out);

/* y[t][r] = W_r . x_t through the int8 (Q8_0/Q4_K/Q6_K) or f32 (F32/F16)
 * path, activations quantised on the device first. Replaces matmul_batch
 * (reference include/fish/ops.h:89-91, ops.cpp:177-251). T <= 256. */
FISH_API int fbx_matmul(int type, const void* w, int n_in, int n_out, const float* x, int T, float* y);

/* Per-(row, block) integer sums of the device integer path on already
 * quantised activations (q8act for Q8_0, q8actk for K-quants, in the
 * reference's record layout): Q8_0 s_b, Q4_K sumi_b and mins_b, Q6_K sumi_b
 * (reference quant_x86.cpp:299-309, 346-382, 431-495). sumi/mins are
 * n_out x n_blocks; mins may be NULL. */
FISH_API int fbx_block_sums(int type, const void* w, int n_in, int n_out, const void* acts, int32_t* sumi,
                            int32_t* mins);

/* Causal GQA attention (reference ops.cpp:303-356) for T queries at
 * positions pos0.. against K/V caches [n_keys][HKV*D] (n_keys >= pos0+T),
 * stored into the paged device cache as fp16 (kv_f16=1) or f32. */
FISH_API int fbx_attention(const float* q, const float* k, const float* v, int n_keys, int H, int HKV, int D,
                           int pos0, int T, int kv_f16, float* out);

/* The same causal attention on the tensor-core prefill kernel the engine
 * uses for a prompt (fp16 cache; the T queries one sequence's tokens at
 * positions pos0..pos0+T-1; G = H/HKV <= 8). No reference counterpart beyond
 * fbx_attention's. */
FISH_API int fbx_attention_prefill(const float* q, const float* k, const float* v, int n_keys, int H, int HKV, int D,
                                   int pos0, int T, float* out);

/* One decode step of one sequence with the fused kernel the engine uses for
 * single-token steps: q [H*D] and the new k/v [HKV*D] are the raw
 * projections of the token at position pos; RoPE (reference ops.cpp:126-156,
 * table like rope_build ops.cpp:75-124) rotates q and k, the new K/V row is
 * stored in the paged cache at pos (reference model.cpp:1723-1731) after
 * caches k_cache/v_cache [pos][HKV*D] (already rotated, positions 0..pos-1),
 * and causal attention over positions 0..pos (reference ops.cpp:303-356)
 * writes out [H*D]. k_stored/v_stored (nullable) receive the row read back
 * from the cache at pos. */
FISH_API int fbx_attention_decode(const float* q, const float* k_cache, const float* v_cache, const float* k_new,
                                  const float* v_new, int pos, int H, int HKV, int D, int rot_dim, int neox,
                                  float freq_base, int kv_f16, float* out, float* k_stored, float* v_stored);

/* RoPE (reference ops.cpp:126-156) on q [T][H*D] and k [T][HKV*D] in place,
 * token t at position pos0+t, with a table built like rope_build
 * (ops.cpp:75-124) for freq_base and rot_dim. */
FISH_API int fbx_rope(float* q, float* k, int T, int H, int HKV, int D, int rot_dim, int neox, float freq_base,
                      int pos0);

/* Device time of the matmul kernel alone: `iters` back-to-back launches of
 * y = W x for T <= 256 tokens (the GEMV kernels up to 15 tokens, the int8
 * tensor-core kernel from 16 for quantised rows), timed with CUDA events on
 * the launching stream after
 * 3 warm-up launches. W is filled with a constant byte pattern and replicated
 * into enough copies (>= 512 MB) that consecutive launches read different
 * copies, so every launch streams its weights from HBM, not L2. Writes the
 * mean milliseconds per launch and the algorithmic bytes of one launch
 * (weight rows in GGUF encoding). */
FISH_API int fbx_time_matmul(int type, int n_in, int n_out, int T, int iters, float* ms_per_launch,
                             double* bytes_per_launch);

/* Marks the start (start != 0) or end of a profiler capture range
 * (cudaProfilerStart / cudaProfilerStop), for captures of one step with the
 * profiler set not to record from the program's start. No reference
 * counterpart. Returns the CUDA error. */
FISH_API int fbx_profiler(int start);

/* Causal GQA attention like fbx_attention, on DEVICE buffers, allocating
 * nothing. No counterpart in the reference: it serves callers that cannot
 * allocate device memory on the call path (a serving loop that gave all free
 * HBM to its KV page pool, code under a caching allocator that must not be
 * re-entered, a step that must not pay for cudaMalloc/cudaFree, which can
 * synchronise the device).
 *   q [T][H*D] f32, out [T][H*D] f32, k and v [n_keys][HKV*D] as fp16
 *   (kv_f16=1) or f32; every pointer 16-byte aligned; the call is queued on
 *   `stream` (a cudaStream_t, NULL = default stream) and returns without
 *   waiting for it. Token t sits at position pos0+t and attends to keys
 *   [0, pos0+t]; only rows [0, pos0+T) of k and v are read, so n_keys (which
 *   must be >= pos0+T) is only the caller's bound on those buffers.
 * Its scratch (split partials, positions, an identity page table) is one
 * fixed __device__ array per device, 8 MiB of partials: pos0+T <= 8192,
 * T <= 256 and T*H*n_splits*(D+2) <= 2^21 floats, n_splits = ceil((pos0+T)/32)
 * up to 2048 keys and ceil((pos0+T)/128) above; larger calls return -1.
 * The first call on a device resolves that array's address and initialises
 * it (a kernel on `stream`, then a wait for that stream); make it before any
 * stream capture. After cudaDeviceReset the next call does this again (the
 * device's new context is detected by its id). Partials need no clearing;
 * every split writes its own. Every call on a device shares the array, so
 * calls that overlap on the GPU (different streams, no ordering between
 * them) race and corrupt each other's output. */
FISH_API int fbx_attention_static(const float* q, const void* k, const void* v, int kv_f16, int n_keys, int H,
                                  int HKV, int D, int pos0, int T, float* out, void* stream);

/* First index of the maximum per row (reference model.cpp:1939-1946). */
FISH_API int fbx_argmax(const float* x, int rows, int n, int32_t* out);

/* The sampler's greedy branch on the device: every occurrence of an id in
 * recent[0..n_recent) (the penalty window, oldest first, n_recent <= 256)
 * applies the repetition penalty to its logit (v > 0 ? v / p : v * p), then
 * out[0] = the first index of the maximum of x[0..n). Reference
 * Sampler::penalise + greedy argmax (model/fish/src/sampler.cpp:42-132);
 * the generation loop runs it for temperature <= 0. Host buffers. */
FISH_API int fbx_argmax_penalized(const float* x, int n, const int32_t* recent, int n_recent, float penalty,
                                  int32_t* out);

/* Embedding row gather + dequantisation (reference dequant_row,
 * quant.cpp:470-506) for ids[0..T) of a [n_rows][E] table. */
FISH_API int fbx_embed(int type, const void* table, int E, int n_rows, const int32_t* ids, int T, float* out);

/* Debug probe of one transformer layer, for layer-wise parity tests (no
 * counterpart in the reference's ABI; it restates one iteration of
 * LlamaModel::forward's layer loop, model/fish/src/model.cpp:1654-1785). It
 * runs layer `layer` of the model loaded in ctx on n_tok hidden rows x_in
 * ([n_tok][n_embd] f32, host) at positions pos0.. of the context's sequence
 * (writing that layer's K/V rows there; pos0 <= the sequence length), with
 * the same kernels and fused prologues the forward uses for n_tok tokens,
 * launched eagerly. x_out receives the layer's output rows. Stages: 0 the
 * attention-norm input, 1 the attention output, 2 the FFN-norm input, 3 the
 * SwiGLU product (n_tok * n_experts_per_tok rows for MoE layers). For each
 * stage the caller may pass buffers (NULL = skip) for the float rows the
 * stage quantised (f; stages 0 and 2 before their RMSNorm) and for the int8
 * activations the kernels built, as the reference's Q8ActK records (qk,
 * 276 B per 256 values) and Q8Act records (q32, 40 B per 32 values). When
 * the SwiGLU product is formed inside the down projection's prologue, f[3]
 * stays unwritten and gate3 / up3 receive its two inputs. rows/K/has_k/
 * has_32 report what was recorded. Returns 0, or -1 with fish_last_error. */
typedef struct {
    float* f[4];
    uint8_t* qk[4];
    uint8_t* q32[4];
    float* gate3;
    float* up3;
    int rows[4];
    int K[4];
    int has_k[4];
    int has_32[4];
    int silu_in_prologue;
} fbx_layer_probe_out;
struct fish_ctx;
FISH_API int fbx_layer_probe(struct fish_ctx* ctx, int layer, int pos0, const float* x_in, int n_tok, float* x_out,
                             fbx_layer_probe_out* out);

/* Tensor / expert parallelism: rank `rank` of `world`'s slices, as the
 * loader takes them under fish_tp_init (host code, no device): out[14] =
 * head0, heads, kv_head0, kv_heads, q_row0, q_rows, kv_row0, kv_rows
 * (also attn_output's input slice), ff_row0, ff_rows (also ffn_down's input
 * slice; dense models), expert0, experts (MoE), vocab_row0, vocab_rows.
 * -1 when the counts do not split evenly over the ranks or the vocabulary
 * slice is not whole 8-row tiles. No counterpart in the reference, which
 * runs on one device. */
FISH_API int fbx_tp_plan(int n_head, int n_head_kv, int head_dim, int n_ff, int vocab, int n_experts, int rank,
                         int world, int32_t* out);
/* The routed experts sel[0..n) as local ids of the rank holding experts
 * [e0, e0 + n_local), -1 for another rank's (host code; the device step's
 * mapping). */
FISH_API int fbx_moe_localize_host(const int32_t* sel, int n, int e0, int n_local, int32_t* out);

/* Tokenizer of a GGUF file without loading its model: host code only, no
 * device needed. It is the tokenizer fish_load sets up for the same file
 * (vocabulary, merges or scores, special tokens, chat template), built from
 * the GGUF metadata on every call, for tokenizer parity tests and for tools
 * that only tokenize. Return values as fish_tokenize, fish_detokenize and
 * fish_chat_prompt (c_api.h), which replace the reference's
 * (model/fish/include/fish/c_api.h:108-121); -1 when the file or its
 * tokenizer cannot be read. */
FISH_API int fbx_tokenize_gguf(const char* gguf_path, const char* text, int add_bos, int32_t* out, int cap);
FISH_API int fbx_detokenize_gguf(const char* gguf_path, const int32_t* ids, int n, char* out, int cap);
FISH_API int fbx_chat_prompt_gguf(const char* gguf_path, const char* const* roles, const char* const* contents,
                                  int n, char* out, int cap);

/* The sampler of fish_generate on host logits (host code only): repetition
 * penalty over the last repeat_last_n of `recent`, temperature, top-k,
 * top-p, then a draw from a std::mt19937_64 seeded with `seed` (0: from the
 * clock), n_draws times with one generator, each draw on a fresh copy of the
 * logits. Replaces the reference's Sampler::sample
 * (model/fish/include/fish/sampler.h:26-33). Returns 0, or -1 on bad
 * arguments. */
FISH_API int fbx_sample(const float* logits, int n_vocab, float temperature, int top_k, float top_p,
                        float repeat_penalty, int repeat_last_n, const int32_t* recent, int n_recent, uint64_t seed,
                        int n_draws, int32_t* out);

/* The distribution fbx_sample draws from, as probabilities over the whole
 * vocabulary (host code only): after the penalty, a one-hot of the first
 * maximum when temperature <= 0, else the top-k softmax cut at top_p and
 * renormalised, zero elsewhere; speculative decoding compares the target's
 * and the draft's. Replaces the reference's Sampler::distribution
 * (model/fish/include/fish/sampler.h:32-37). Returns 0, or -1 on bad
 * arguments. */
FISH_API int fbx_sample_distribution(const float* logits, int n_vocab, float temperature, int top_k, float top_p,
                                     float repeat_penalty, int repeat_last_n, const int32_t* recent, int n_recent,
                                     float* probs);
/* n_draws indices drawn in proportion to the positive weights (-1 when there
 * are none) from one std::mt19937_64 seeded with `seed` (host code only).
 * Replaces the reference's Sampler::draw (model/fish/include/fish/sampler.h:39-40).
 * Returns 0, or -1 on bad arguments. */
FISH_API int fbx_sample_draw(const float* weights, int n, uint64_t seed, int n_draws, int32_t* out);

/* The token ids the context's last fish_generate* call emitted, in order (the
 * ids behind its token callbacks; test observability, host code only):
 * copies min(count, cap) of them and returns the count, -1 on bad
 * arguments. */
FISH_API int fbx_last_generated(struct fish_ctx* ctx, int32_t* out, int cap);

/* The rejection rule of speculative decoding on fixed distributions (host
 * code only): n_trials times, a draft token d is drawn from q and verified
 * against p (kept with probability min(1, p(d)/q(d)), else replaced by a draw
 * from max(0, p - q)); out[i] = the committed token, which is distributed as
 * p. One std::mt19937_64 seeded with `seed`. The step fish_generate takes per
 * draft token when a draft model is set (model/fish/src/c_api.cpp:719-741).
 * Returns 0, or -1 on bad arguments. */
FISH_API int fbx_speculative_draws(const float* p, const float* q, int n, uint64_t seed, int n_trials, int32_t* out);

/* fish_count_chat_tokens and fish_chat_format for the GGUF at gguf_path with
 * no model loaded (host code only, model/fish/src/c_api.cpp:384-397): returns
 * the token count of the formatted chat, and writes the chat format's name
 * to `format` as fish_detokenize writes strings; -1 when the file cannot be
 * read. */
FISH_API int fbx_chat_info_gguf(const char* gguf_path, const char* const* roles, const char* const* contents, int n,
                                char* format, int cap);

/* The token callback stream fish_generate produces for the generated ids
 * `ids` (host code only; the generation loop's own UTF-8 emitter and final
 * flush over the GGUF tokenizer's token texts, model/fish/src/c_api.cpp:81-101,
 * 774-779): every callback as "<token_id> <strlen(text)>\n<text>", in order.
 * Returns the record length, written as fish_detokenize writes strings; -1
 * when the file cannot be read. */
FISH_API int fbx_stream_gguf(const char* gguf_path, const int32_t* ids, int n, char* out, int cap);

/* The prompt decisions fish_generate makes before its first forward (host
 * code only, the same functions the generation loop calls): a state holding
 * the last head+tail cut and the ids whose KV the one-slot prefix cache holds
 * (model/fish/src/c_api.cpp:40-44, 516-567). fbx_prompt_plan fits `ids` into
 * n_ctx for `max_tokens` (<= 0: n_ctx) as fish_generate does, writes the kept
 * ids to `kept` and returns their count (fish_stats.prompt_tokens), with
 * *truncated (fish_stats.truncated) and *cached, the tokens the cache would
 * serve (fish_stats.cached_tokens); -1 on a bad argument or cap < the kept
 * count. fbx_prompt_commit sets the cached ids, as a finished turn leaves
 * them: the kept prompt followed by every generated token fed back. */
typedef struct fbx_prompt_state fbx_prompt_state;
FISH_API fbx_prompt_state* fbx_prompt_state_create(void);
FISH_API void fbx_prompt_state_destroy(fbx_prompt_state* s);
FISH_API int fbx_prompt_plan(fbx_prompt_state* s, const int32_t* ids, int n, int n_ctx, int max_tokens,
                             int32_t* kept, int cap, int* cached, int* truncated);
FISH_API int fbx_prompt_commit(fbx_prompt_state* s, const int32_t* ids, int n);

/* Digest of how this library reads a GGUF file (host code only): one line
 * per tensor in directory order, "T name type ne0,ne1,.. file_offset nbytes"
 * (the absolute offset of its data in the file), then one line per key in
 * `keys`, "K key kind value" (kind as in the GGUF metadata value kinds:
 * 0 uint, 1 int, 2 float, 3 bool, 4 string, 5 array; arrays as their length,
 * element counts per storage and an FNV-1a digest of the contents) or
 * "K key missing". For parity tests of the container reader against the
 * reference's GgufFile (model/fish/include/fish/gguf.h:77-116). Returns the
 * digest length, written as fish_detokenize writes strings; -1 when the file
 * cannot be read. */
FISH_API int fbx_gguf_digest(const char* gguf_path, const char* const* keys, int n_keys, char* out, int cap);

#ifdef __cplusplus
}
#endif
