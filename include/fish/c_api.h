#pragma once
/*
 * FISH C ABI, as exported by the B200 engine (libfish.so).
 *
 * ABI 4 (every function and struct below up to the "ABI 5" marker) is the
 * interface IMURUN's model/fish_native.py binds with ctypes; declarations,
 * struct layouts and return conventions are kept identical to the reference
 * header model/fish/include/fish/c_api.h so the Python server works
 * unchanged. Each declaration names the reference line it replaces.
 *
 * ABI 5 adds id-level prefill/decode, on-device greedy decode, and sessions
 * with a paged KV cache whose shared prefixes are referenced, not copied.
 * ABI rule (reference c_api.h:11-12): structs only grow at the end; new
 * functions are added, never changed.
 */
#include <stdint.h>

#ifdef _WIN32
#  define FISH_API __declspec(dllexport)
#else
#  define FISH_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FISH_ABI_VERSION 5

typedef struct fish_ctx fish_ctx;

/* reference c_api.h:30-32 */
typedef void (*fish_token_cb)(const char* text, int token_id, void* user);

/* reference c_api.h:34-70; sizeof == 1104 */
typedef struct fish_stats {
    double load_seconds;
    double prefill_seconds;
    double decode_seconds;
    double tokens_per_second;
    int    prompt_tokens;
    int    generated_tokens;
    int    context_used;
    int    context_size;
    unsigned long long weights_bytes;
    unsigned long long kv_bytes;
    double peak_rss_mb;
    int    truncated;
    int    cached_tokens;
    int    n_threads;
    int    streaming;
    double prefill_tokens_per_second;
    int    gpu_layers;
    int    ram_layers;
    int    disk_layers;
    unsigned long long gpu_bytes;
    char   gpu_name[64];
    int    draft_proposed;
    int    draft_accepted;
    int    draft_active;
    char   gpu_mix[160];
    char   placement[320];
    char   load_profile[400];
    unsigned long long vram_total;
    unsigned long long vram_free;
    unsigned long long vram_headroom;
} fish_stats;

/* reference c_api.h:72-90; sizeof == 168 */
typedef struct fish_model_info {
    char   arch[32];
    int    n_layers;
    int    n_embd;
    int    n_ff;
    int    n_head;
    int    n_head_kv;
    int    head_dim;
    int    n_ctx;
    int    vocab;
    int    tied_output;
    char   quant[64];
    int    n_experts;
    int    n_experts_per_tok;
    int    n_ctx_train;
    char   chat_format[16];
    char   tokenizer[8];
} fish_model_info;

FISH_API const char* fish_version(void);                         /* c_api.h:92 */
FISH_API int         fish_abi_version(void);                     /* c_api.h:93 */
FISH_API fish_ctx*   fish_create(void);                          /* c_api.h:95 */
FISH_API void        fish_destroy(fish_ctx* ctx);                /* c_api.h:96 */
FISH_API int         fish_load(fish_ctx* ctx, const char* path, int n_ctx);   /* c_api.h:100 */
FISH_API int         fish_loaded(fish_ctx* ctx);                 /* c_api.h:101 */
FISH_API const char* fish_last_error(fish_ctx* ctx);             /* c_api.h:102 */
FISH_API int         fish_model_info_of(fish_ctx* ctx, fish_model_info* out);   /* c_api.h:104 */
FISH_API int fish_tokenize(fish_ctx* ctx, const char* text, int add_bos,
                           int32_t* out, int cap);               /* c_api.h:108-109 */
FISH_API int fish_detokenize(fish_ctx* ctx, const int32_t* ids, int n,
                             char* out, int cap);                /* c_api.h:110-111 */
FISH_API int fish_chat_prompt(fish_ctx* ctx, const char* const* roles,
                              const char* const* contents, int n_messages,
                              char* out, int cap);               /* c_api.h:117-121 */
FISH_API const char* fish_chat_format(fish_ctx* ctx);            /* c_api.h:122 */
FISH_API int fish_generate(fish_ctx* ctx, const char* prompt, int add_bos,
                           int max_tokens, float temperature, int top_k,
                           float top_p, float repeat_penalty,
                           fish_token_cb cb, void* user);        /* c_api.h:128-131 */
FISH_API int fish_generate_chat(fish_ctx* ctx, const char* const* roles,
                                const char* const* contents, int n_messages,
                                int max_tokens, float temperature, int top_k,
                                float top_p, float repeat_penalty,
                                fish_token_cb cb, void* user);   /* c_api.h:136-142 */
FISH_API int fish_generate_to(fish_ctx* ctx, const char* prompt, int add_bos,
                              int max_tokens, float temperature, int top_k,
                              float top_p, float repeat_penalty,
                              char* out, int cap);               /* c_api.h:146-149 */
FISH_API void fish_cancel(fish_ctx* ctx);                        /* c_api.h:151 */
FISH_API void fish_reset(fish_ctx* ctx);                         /* c_api.h:152 */
FISH_API void fish_get_stats(fish_ctx* ctx, fish_stats* out);    /* c_api.h:153 */
FISH_API const char* fish_kernel_name(void);                     /* c_api.h:156 */
FISH_API const char* fish_specs_json(fish_ctx* ctx);             /* c_api.h:160 */
FISH_API const char* fish_supported_archs(void);                 /* c_api.h:163 */
FISH_API int  fish_set_threads(fish_ctx* ctx, int n);            /* c_api.h:177 */
FISH_API int  fish_set_draft(fish_ctx* ctx, const char* path, int k);   /* c_api.h:179 */
FISH_API void fish_clear_draft(fish_ctx* ctx);                   /* c_api.h:180 */
FISH_API int  fish_count_chat_tokens(fish_ctx* ctx, const char* const* roles,
                                     const char* const* contents, int n_messages);  /* c_api.h:185-186 */

/* reference c_api.h:208-224; sizeof == 208 */
typedef struct fish_adapter_info {
    int    active;
    int    pending;
    char   name[128];
    int    rank;
    int    rank_min;
    float  alpha;
    float  scale;
    float  effective_scale;
    int    tensors;
    unsigned long long merged_bytes;
    double merge_seconds;
    double retention;
    double residual;
    unsigned long long blocks;
    unsigned long long blocks_refit;
} fish_adapter_info;

FISH_API int  fish_set_adapter(fish_ctx* ctx, const char* path, float scale);   /* c_api.h:226 */
FISH_API int  fish_clear_adapter(fish_ctx* ctx);                 /* c_api.h:227 */
FISH_API int  fish_adapter_info_of(fish_ctx* ctx, fish_adapter_info* out);   /* c_api.h:228 */

/* ==================================================================== ABI 5
 * Id-level calls. The reference keeps prefill, decode and its one-slot prefix
 * cache inside generate_ids_locked (c_api.cpp:555-673); these expose the same
 * steps to callers that already hold token ids. All return 0 on success and a
 * negative value on error (fish_last_error says why). */

/* Forward `n` ids at positions pos0.. (chunks of <= 256, c_api.cpp:586-595)
 * after discarding any KV beyond pos0 (LlamaModel::set_kv_len). `logits`
 * (nullable, vocab floats) receives the last token's logits. */
FISH_API int fish_prefill_ids(fish_ctx* ctx, const int32_t* ids, int n, int pos0, float* logits);

/* Teacher-forced step(s): forward `n` ids at pos0 as one batch; logits_all
 * (nullable, n * vocab) receives every token's logits, argmax_out (nullable,
 * n) every token's greedy choice (first index of the maximum). */
FISH_API int fish_decode_ids(fish_ctx* ctx, const int32_t* ids, int n, int pos0,
                             float* logits_all, int32_t* argmax_out);

/* Greedy decode of n_steps tokens entirely on the device, starting by feeding
 * `first` at position kv_len. Writes the n_steps generated ids to out_ids.
 * Stops early only on error. Returns the number of ids written. */
FISH_API int fish_decode_greedy(fish_ctx* ctx, int32_t first, int n_steps, int32_t* out_ids);

/* Tensor parallelism (ABI 5 addition; no counterpart in the reference, which
 * runs one model per process on the CPU): one process per GPU, ranks
 * 0..world-1. fish_tp_unique_id writes a new 128-byte group id into out (on
 * one rank; every rank then receives it through the caller's own channel) and
 * returns its size (or the size needed when cap is too small, < 0 on error).
 * fish_tp_init records rank, world and id for the next fish_load, which
 * then joins the NCCL group and loads only this rank's shard: q/k/v and
 * gate/up rows split by heads and FFN rows, attn_output and ffn_down split
 * along their inputs (256-aligned), the output projection split by vocab
 * rows; two all-reduces per layer. MoE models split the experts instead of
 * the FFN rows (experts/world per rank; routing computed on every rank;
 * selections of other ranks' experts contribute zero rows) and all-reduce
 * the weighted expert outputs. Models whose kv heads, FFN rows (or experts)
 * and vocab divide by world. Every rank must make the same calls in the same
 * order (prefill, decode, greedy); logits and ids returned are the whole
 * model's. Returns 0, or -1 on bad arguments. */
FISH_API int fish_tp_unique_id(void* out, int cap);
FISH_API int fish_tp_init(fish_ctx* ctx, int rank, int world, const void* id, int id_bytes);

FISH_API int  fish_kv_len(fish_ctx* ctx);
FISH_API int  fish_set_kv_len(fish_ctx* ctx, int n);

/* Sessions over the paged KV cache. Session 0 is the context's own sequence
 * (the one fish_generate* and the calls above use). A fork references the
 * parent's full pages of the first `prefix_len` positions (refcounted, not
 * copied); a partially filled last page is copied so that appends never
 * touch a page another session reads. Returns the new id or < 0. */
FISH_API int  fish_session_open(fish_ctx* ctx);
FISH_API int  fish_session_fork(fish_ctx* ctx, int parent, int prefix_len);
FISH_API int  fish_session_close(fish_ctx* ctx, int session);
FISH_API int  fish_session_len(fish_ctx* ctx, int session);
/* Prefill ids onto the end of a session's KV; logits (nullable) = last token's. */
FISH_API int  fish_session_prefill(fish_ctx* ctx, int session, const int32_t* ids, int n, float* logits);
/* One decode step for n sessions at once (one token each, appended at each
 * session's length). argmax_out (nullable, n); logits (nullable, n * vocab). */
FISH_API int  fish_decode_batch(fish_ctx* ctx, const int* sessions, const int32_t* ids, int n,
                                int32_t* argmax_out, float* logits);
/* Page table of a session (page indices into the KV pool, in position order).
 * Returns the number of pages (or the required size when out is too small). */
FISH_API int  fish_session_pages(fish_ctx* ctx, int session, int32_t* out, int cap);
/* Positions per KV page. */
FISH_API int  fish_kv_page_size(fish_ctx* ctx);

/* Engine state as one JSON object: device, KV pool pages (total / free),
 * weight bytes on the device, kernels per captured step graph, the device
 * times (CUDA events on the engine's stream) of the last fish_decode_greedy
 * call (last_decode_device_ms) and of the last graph-launched
 * fish_decode_batch step (last_batch_device_ms), kernel error and wait
 * failure records, the persistent step kernel's state, and tp_world. The
 * pointer is valid until the next call on the same thread. */
FISH_API const char* fish_engine_json(fish_ctx* ctx);

/* Per-kernel-class device timing of n_steps single-token decode steps run
 * without graph replay (each launch bracketed by CUDA events), as JSON:
 * {"classes":[{"name","launches","ms","bytes"}...]}. GEMV bytes are the
 * algorithmic bytes (weight rows in GGUF encoding + outputs). Advances the
 * context's sequence by n_steps. NULL on error. */
FISH_API const char* fish_profile_decode_json(fish_ctx* ctx, int32_t first, int n_steps);

/* Device-time trace of n_steps graph-replayed greedy decode steps (like
 * fish_decode_greedy, which it performs): the first CTA of each traced kernel
 * records (globaltimer ns, kernel tag, event, launch number) into out
 * (4 values per record, at most cap records). Tags: 1 GEMV, 2 attention,
 * 3 embedding, 4 argmax/greedy. Events: 0 start, 1 dependency wait passed,
 * 2 operands ready, 3 end. When the persistent step kernel runs the decode,
 * records are (ns, tag 5, phase-boundary index, step * 2 + c) for thread 0 of
 * the first (c = 0) and the last (c = 1) CTA. Returns the number of records,
 * or < 0. */
FISH_API int fish_trace_decode(fish_ctx* ctx, int32_t first, int n_steps, uint64_t* out, int cap);

#ifdef __cplusplus
}
#endif
