// engine.h — the B200 decode/prefill engine behind the FISH C ABI.
//
// One Engine owns one model on one GPU: device weights (repacked GGUF
// blocks), a paged KV pool shared by all sequences of the model, work buffers
// for up to kMaxBatch tokens per forward, and CUDA graphs for single-token
// decode. It plays the role of the reference's LlamaModel
// (model/fish/include/fish/model.h:162-292): load, forward, set_kv_len /
// reset_kv, logits, argmax.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>   // types only: the library is loaded at run time (nccl_api)

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "gguf.h"
#include "kernels/kernels.h"

namespace fb {

constexpr int kMaxBatch = 256;   // tokens per forward (reference max_batch_, model.h:292)
constexpr int kPageSize = 16;    // KV positions per page
constexpr int kPrefixMaxBatch = 64;   // batched decode: sessions whose shared prefix attention reads once

struct Config {
    std::string arch = "llama";
    int n_layers = 0, n_embd = 0, n_ff = 0, n_head = 0, n_head_kv = 0, head_dim = 0;
    int n_ctx = 0, n_ctx_train = 0, vocab = 0, rot_dim = 0;
    float eps = 1e-5f, freq_base = 10000.0f;
    int bos = 1, eos = 2;
    bool tied_output = false, neox = false, qk_norm = false;
    // gemma2 (src/model.cpp:488-496): norm weights stored as w - 1, GELU in
    // the FFN, the embedding scaled by sqrt(n_embd), attention-score and
    // final-logit soft caps, a sliding window on the even layers, and
    // post-attention / post-FFN norms before the residual adds
    bool norm_plus_one = false, gelu = false, post_norms = false;
    float embd_scale = 1.0f, attn_softcap = 0.0f, final_softcap = 0.0f;
    int sliding_window = 0;
    int n_experts = 0, n_experts_per_tok = 0, n_ff_exp = 0;
    int n_ff_shexp = 0;   // qwen2moe: rows of the shared expert (0: none)
    // tensor parallelism: the head counts and n_ff above are this rank's
    // shares; the model's own values are kept here (equal without it)
    int n_head_model = 0, n_head_kv_model = 0, n_ff_model = 0;
    int out_rows = 0, out_row0 = 0;   // output-projection rows of this rank (vocab slice)
    bool expert_weights_norm = true;
    // RoPE scaling (src/model.cpp:508-537)
    float freq_scale = 1.0f, mscale = 1.0f;
    float yarn_factor = 0.0f, yarn_attn_factor = 1.0f, yarn_beta_fast = 32.0f, yarn_beta_slow = 1.0f;
    int yarn_orig_ctx = 0;
    int q_dim() const { return n_head * head_dim; }
    int kv_dim() const { return n_head_kv * head_dim; }
};

// This rank's slices under tensor / expert parallelism over `world` ranks
// (one process per GPU): heads and kv heads, the q / k / v rows and the
// matching input slice of attn_output, FFN rows and the input slice of
// ffn_down (dense), or experts (MoE), and vocab rows of the output
// projection. Every slice is contiguous and rank-ordered; false (with err)
// when the counts do not split evenly, the vocab slice is not whole 8-row
// tiles, or an input slice is not whole 256-value blocks.
struct TpPlan {
    int head0 = 0, heads = 0, kv_head0 = 0, kv_heads = 0;
    int q_row0 = 0, q_rows = 0, kv_row0 = 0, kv_rows = 0;   // also attn_output's input slice (q)
    int ff_row0 = 0, ff_rows = 0;                             // also ffn_down's input slice (dense)
    int expert0 = 0, experts = 0;                             // MoE
    int vocab_row0 = 0, vocab_rows = 0;
};
bool tp_plan(int n_head, int n_head_kv, int head_dim, int n_ff, int vocab, int n_experts, int rank, int world,
             TpPlan* out, std::string* err);

// RoPE cos/sin table [n_ctx][rot_dim/2] for c (uses n_ctx, rot_dim,
// freq_base and the scaling fields); ff = per-pair frequency factors or null.
void build_rope_table(const Config& c, const float* ff, std::vector<float>& cs, std::vector<float>& sn);

struct DevW {
    std::string name;   // the GGUF tensor it is uploaded from (a fused tensor for phi3's q/k/v and gate/up views)
    int type = -1;
    int n_in = 0, n_out = 0, n_exp = 1;   // this rank's shard (the whole tensor without tensor parallelism)
    // shard of the GGUF tensor: rows [row0, row0 + n_out) of its n_out_src,
    // values [k0, k0 + n_in) of its rows of n_in_src values (k0 a block edge)
    int row0 = 0, k0 = 0, n_in_src = 0, n_out_src = 0;
    int e0 = 0;   // first expert of this rank's slice (expert parallelism)
    size_t stride = 0;           // device row stride
    size_t expert_bytes = 0;     // bytes per expert slice (3-D tensors)
    uint8_t* d = nullptr;
    bool ok() const { return d != nullptr; }
};

struct DevLayer {
    DevW wq, wk, wv, wo, wg, wu, wd, gate_inp, gate_exps, up_exps, down_exps;
    DevW shexp_gate, shexp_up, shexp_down, shexp_gate_inp;   // qwen2moe shared expert (optional)
    float *attn_norm = nullptr, *ffn_norm = nullptr, *bq = nullptr, *bk = nullptr, *bv = nullptr;
    float *q_norm = nullptr, *k_norm = nullptr;
    float *post_attn_norm = nullptr, *post_ffn_norm = nullptr;   // gemma2
    float* bo = nullptr;   // attn_output.bias (added once: by rank 0 under tensor parallelism)
};

// Debug record of one layer's int8 activations (Engine::layer_probe). Stage
// s: 0 the attention-norm input, 1 the attention output, 2 the FFN-norm
// input, 3 the SwiGLU product. f[s]: the float rows the stage quantised
// (0, 2: before the RMSNorm); f[4], f[5]: gate and up rows when the product
// is formed inside the down projection's prologue (f[3] then stays empty).
// rk / r32: the int8 activations the kernels built, as the reference's
// Q8ActK (276 B per 256 values) / Q8Act (40 B per 32 values) records.
struct LayerProbe {
    std::vector<float> f[6];
    std::vector<uint8_t> rk[4], r32[4];
    int rows[6] = {}, K[6] = {};
    bool has_k[4] = {}, has_32[4] = {};
};
constexpr size_t kProbeChunkBytes = 589824;   // one GEMV launch's image dump (header + 8 tokens at K <= 28672)
constexpr int kXChunkBytes = 272;             // image bytes per 256 int8 values (stream_common.cuh kXChunk)

struct Seq {
    bool open = false;
    int len = 0;                 // positions holding valid KV
    std::vector<int> pages;      // page ids in position order
};

// NCCL entry points, resolved at run time (nccl_api() in engine.cpp); the
// types come from nccl.h.
struct NcclApi {
    bool ok = false;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};
const NcclApi* nccl_api(std::string* err);

class Engine {
public:
    Engine() = default;
    ~Engine();
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;

    // Tensor parallelism over `world` ranks (one process per GPU), before
    // load: q/k/v and gate/up rows split by heads / FFN rows, o and down split
    // along their inputs (256-aligned K slices) with an NCCL all-reduce after
    // each, the output projection split by vocab rows (argmax keys reduced by
    // max, logits gathered). id: the 128-byte NCCL unique id of the group.
    bool set_tp(int rank, int world, const void* id, std::string* err);
    int tp_rank() const { return tp_rank_; }
    int tp_world() const { return tp_world_; }

    bool load(const std::string& path, int n_ctx, std::string* err);
    const Config& cfg() const { return cfg_; }
    const Gguf& gguf() const { return *gguf_; }
    uint64_t weights_bytes() const { return weights_file_bytes_; }
    uint64_t device_weight_bytes() const { return weights_dev_bytes_; }
    uint64_t kv_bytes() const { return kv_pool_bytes_; }
    int device() const { return device_; }
    std::string device_name() const;
    double load_seconds_upload = 0.0;

    // ---- sequences (slot 0 always exists: the context's own sequence)
    int seq_open();
    int seq_fork(int parent, int prefix_len, std::string* err);
    bool seq_close(int sid);
    int seq_len(int sid) const;
    bool seq_truncate(int sid, int n);      // set_kv_len: drop positions >= n
    std::vector<int> seq_pages(int sid) const;
    int page_size() const { return kPageSize; }
    int free_pages() const { return (int)free_pages_.size(); }

    // Forward T tokens (host ids) onto sequence sid at its current length
    // (positions len .. len+T-1). Logits of the last token go to logits_last
    // (host, nullable); all_logits (host, T*vocab) and argmax (host, T)
    // are optional. Chunking to kMaxBatch is the caller's job.
    bool forward(int sid, const int32_t* ids, int T, float* logits_last, float* logits_all, int32_t* argmax,
                 std::string* err);
    // One token onto sid, then the sampler's greedy branch on the device:
    // the repetition penalty of the n_recent ids (the sampler's window) and
    // the first index of the maximum; only that id comes back to the host.
    bool decode_argmax(int sid, int32_t id, const int32_t* recent, int n_recent, float penalty, int32_t* out,
                       std::string* err);
    // Speculative verification: T tokens onto sid at consecutive positions
    // through the batched-decode step (each token's logits are the bits a
    // single-token decode at that position gives). argmax (host, T): the
    // sampler's greedy branch per row, row t penalised by the last `window`
    // ids of hist[0 .. base + t) (the window once the first t tokens were
    // accepted; no penalty when penalty is 1 or window 0). logits_all (host,
    // T*vocab) optional.
    bool verify(int sid, const int32_t* ids, int T, const int32_t* hist, int base, int window, float penalty,
                int32_t* argmax, float* logits_all, std::string* err);
    // Debug: run layer li alone on T hidden rows x_in (host, [T][E]) at
    // positions pos0.. of sequence 0 (its KV rows of that layer are written),
    // x_out = the layer's output rows; *p records every int8 activation the
    // kernels built and the float rows they came from. Eager launches, one GPU.
    bool layer_probe(int li, int pos0, const float* x_in, int T, float* x_out, LayerProbe* p, std::string* err);
    // One token for each of n sequences (n <= kMaxBatch).
    bool decode_batch(const int* sids, const int32_t* ids, int n, int32_t* argmax, float* logits, std::string* err);
    // Greedy decode of n_steps on the device with a captured CUDA graph.
    int decode_greedy(int sid, int32_t first, int n_steps, int32_t* out, std::string* err);
    // Device time (CUDA events on the engine stream) of the last greedy run.
    float last_greedy_ms() const { return last_greedy_ms_; }
    float last_batch_ms() const { return last_batch_ms_; }   // device time of the last batched decode step
    int last_prefix_blocks() const { return last_prefix_blocks_; }   // its shared-prefix 64-key blocks
    // Kernel nodes of the captured step graph for T tokens (0 if none yet).
    int graph_kernels(int T) const {
        auto it = graph_kernels_.find(T);
        return it == graph_kernels_.end() ? 0 : it->second;
    }

    // Per-launch device timing of non-graph single-token steps: each kernel
    // launch is bracketed by events on the engine stream and attributed to a
    // class; GEMV launches also carry their algorithmic bytes.
    struct ProfClass { std::string name; int launches = 0; double ms = 0.0; double bytes = 0.0; };
    bool profile_decode(int sid, int32_t first, int n_steps, std::vector<ProfClass>* out, std::string* err);

    // ---- kernel-level access for the parity entry points
    cudaStream_t stream() const { return stream_; }

    // Persistent decode step (k_step): used for single-sequence decode of
    // dense models it supports when FISH_PERSIST=1 is set. step_ready()
    // builds its phase program on first use; step_why() says why not.
    bool step_ready();
    const std::string& step_why() const { return step_why_; }
    int step_grid() const { return step_grid_; }
    int step_stages() const { return step_S_; }
    int step_slot_bytes() const { return step_slot_; }
    double step_weight_bytes() const { return step_wbytes_; }   // GGUF bytes streamed per step
    // Device time of the last step-kernel launch (CUDA events around it).
    float last_step_ms() const { return last_step_ms_; }
    // Phase trace of the step kernel (device buffer of kStepTraceEvents * 2
    // values per step, or null = off).
    void set_step_trace(unsigned long long* dev) { step_trace_ = dev; }

private:
    bool alloc_buffers(std::string* err);
    bool upload_weights(std::string* err);
    bool ensure_pages(int sid, int new_len, std::string* err);
    void write_page_table(int sid);
    // distinct: the T tokens belong to T different sequences (decode steps),
    // so attention can append each token's K/V inside the fused kernel
    bool run_layers(int T, int max_ctx, bool distinct, std::string* err, int l0 = 0, int l1 = -1);
    bool step_tokens(const int* sids, const int32_t* ids, const int* pos, int n, std::string* err);
    // embedding rows of the T ids in ids_ into x_ (scaled for gemma2)
    bool embed_rows(int T, std::string* err);
    bool probe_float(int idx, const float* dev, int rows, int K, std::string* err);
    bool probe_planes(int stage, const ActQ& a, int rows, int K, bool want32, bool wantk, std::string* err);
    bool probe_image(int stage, int rows, int K, std::string* err);
    bool probe_grouped(int stage, const ActQ& a, int grouped_rows, int rows, int K, std::string* err);
    LayerProbe* probe_ = nullptr;
    uint8_t* probe_img_ = nullptr;     // device: image dumps of the fused GEMV prologues
    size_t probe_img_bytes_ = 0;
    float* probe_h_ = nullptr;         // device: SwiGLU products of the unfused path
    uint8_t* dump_img_ = nullptr;      // set around a probed fused GEMV call
    // keys (nullable): argmax keys per row accumulated by the output GEMV;
    // returns in *keyed whether they were (streamed kernel only)
    // need_logits = false: with argmax keys and tensor parallelism, the
    // logits are not gathered (greedy steps)
    bool run_head(int rows_from, int n_rows, float* logits_dev, std::string* err,
                  unsigned long long* keys = nullptr, bool* keyed = nullptr, bool need_logits = true);
    bool gemv(const DevW& w, const ActQ& a, int T, float* y, int ldy, const float* bias, int epi,
              const float* xf, int ldxf, const int32_t* expert, std::string* err, const GemvPro* pro = nullptr,
              unsigned long long* keys = nullptr);
    bool gemv_group(const DevW* const* ws, float* const* ys, const int* ldys, const float* const* biases, int n,
                    const ActQ& a, int T, int epi, std::string* err, const GemvPro* pro = nullptr,
                    bool swiglu = false, const int32_t* expert = nullptr);
    // MoE FFN of a batched step (T > 1) with the tokens grouped per expert:
    // each expert's weights stream once over all rows routed to it
    bool moe_grouped(const DevLayer& L, const ActQ& a, int T, const int32_t* esel, int nel, float* out, std::string* err);
    // qwen2moe: x += gate * down(silu(gate(xb)) * up(xb)) for the T normed rows in xb_
    bool shared_expert(const DevLayer& L, ActQ a, int T, std::string* err);
    // true when a T-token GEMV over these matrices can build its own int8
    // activations (streamed kernel with a prologue)
    bool fusable(const DevW* const* ws, int n, int T) const;
    KvView kv_view() const;
    // Step graphs are sequence-agnostic (token -> sequence slot and position
    // come from device arrays): key T = T-token step with logits + argmax,
    // key 0 = single-token greedy step that feeds its own argmax back.
    bool capture_graph(int key, std::string* err);
    bool upload_tokens(const int32_t* ids, const int* sids, const int* pos, int T, std::string* err);
    void drop_graphs();
    void prof_begin();
    void prof_end(int cls, double bytes);

    Config cfg_;
    std::unique_ptr<Gguf> gguf_;
    int device_ = 0;
    cudaStream_t stream_ = nullptr;
    uint64_t weights_file_bytes_ = 0, weights_dev_bytes_ = 0, kv_pool_bytes_ = 0;

    // device weights (one arena)
    uint8_t* warena_ = nullptr;
    std::vector<DevLayer> layers_;
    DevW embd_, out_w_;
    float* out_norm_ = nullptr;
    float *rope_cos_ = nullptr, *rope_sin_ = nullptr;
    std::vector<float*> small_;   // small device vectors to free
    bool want32_e_ = false, wantk_e_ = false;   // activation layouts for E-wide inputs
    bool want32_q_ = false, wantk_q_ = false;   // ... for the attention output (wo)
    bool want32_f_ = false, wantk_f_ = false;   // ... for the FFN hidden (down)

    // work buffers
    int max_k_ = 0;
    float *x_ = nullptr, *xb_ = nullptr, *q_ = nullptr, *k_ = nullptr, *v_ = nullptr, *attn_ = nullptr;
    float *g_ = nullptr, *u_ = nullptr, *logits_ = nullptr, *router_ = nullptr, *eo_ = nullptr;
    int32_t *sel_ = nullptr;
    float* wsel_ = nullptr;
    ActQ act_{};
    int8_t* act_mem_ = nullptr;
    float* att_scratch_ = nullptr;
    size_t att_scratch_floats_ = 0;
    float* dec_part_ = nullptr;   // batched decode attention: rank partials
    size_t dec_part_floats_ = 0;
    float* gemm_part_ = nullptr;  // tensor-core GEMM: K-split unit values
    size_t gemm_part_floats_ = 0;
    int32_t* pre_blocks_ = nullptr;   // batched decode: shared-prefix 64-key blocks (set before each step)
    float* pre_state_ = nullptr;      // shared-prefix attention: warp states
    size_t pre_state_floats_ = 0;
    int last_prefix_blocks_ = 0;
    int att_chunk_ = 32;
    int32_t *ids_ = nullptr, *tok_seq_ = nullptr, *tok_pos_ = nullptr, *argmax_ = nullptr;
    int32_t *greedy_out_ = nullptr, *greedy_step_ = nullptr;
    unsigned long long* amax_keys_ = nullptr;   // [kMaxBatch] argmax keys, zero between steps
    int greedy_cap_ = 1 << 16;
    int32_t* h_pinned_ = nullptr;   // pinned staging for ids / tok_seq / tok_pos / the penalty window
    int32_t* recent_dev_ = nullptr;  // [kMaxRecent] penalty window of decode_argmax

    // KV pool
    void* kv_pool_ = nullptr;
    int n_pages_ = 0;
    size_t page_elems_ = 0;
    bool kv_f16_ = true;
    std::vector<int> page_ref_;
    std::vector<int> free_pages_;
    int32_t* pt_arena_ = nullptr;   // [max_seqs][pt_stride]
    int pt_stride_ = 0;
    int max_seqs_ = 0;
    std::vector<Seq> seqs_;

    std::map<int, cudaGraphExec_t> graphs_;
    std::map<int, int> graph_kernels_;
    // tensor parallelism
    int tp_rank_ = 0, tp_world_ = 1;
    void* nccl_ = nullptr;            // ncclComm_t
    float* tp_tmp_ = nullptr;         // [kMaxBatch][E] partial sums of o / down
    float* tp_logits_ = nullptr;      // [world][kMaxBatch][out_rows] gathered vocab slices
    int32_t* sel_loc_ = nullptr;      // expert parallelism: routed experts as local ids (-1: another rank's)
    // expert grouping (batched MoE steps): grouped rows e * T + j of local expert e
    ActQ gact_{};                     // int8 activations of the grouped rows
    int8_t* gact_mem_ = nullptr;
    float *gg_ = nullptr, *gu_ = nullptr, *geo_ = nullptr;   // grouped gate / up (then h) / down outputs
    int32_t *grp_src_ = nullptr, *grp_pos_ = nullptr, *grp_count_ = nullptr, *chunk_exp_ = nullptr;
    int grp_rows_ = 0;                // capacity: local experts x kMaxBatch
    int ep_e0_ = 0, ep_n_ = 0;        // this rank's experts [ep_e0_, ep_e0_ + ep_n_)
    bool tp_reduce_add(int T, std::string* err);   // x += all-reduce(tp_tmp_)
    bool tp_gather_logits(int rows, float* logits_dev, std::string* err);
    bool use_graphs_ = true;
    bool no_fuse_ = false;     // FISH_NO_FUSE: separate norm/quant kernels before every GEMV
    bool prefill_simt_ = false;   // FISH_ATTN_PREFILL_SIMT: prefill attention on the SIMT split-key kernel
    // persistent step
    bool run_step(int sid, int n_steps, int32_t* out_dev, std::string* err);
    int step_state_ = 0;       // 0 not built, 1 ready, -1 unavailable
    std::string step_why_;
    StepPhase* step_ph_ = nullptr;
    int step_nph_ = 0;
    StepCtl* step_ctl_ = nullptr;
    unsigned long long* step_keys_ = nullptr;
    float* att_part_ = nullptr;
    int step_grid_ = 0, step_S_ = 0, step_slot_ = 0, step_union_ = 0, att_max_chunks_ = 0;
    size_t step_smem_ = 0;
    double step_wbytes_ = 0.0;
    float last_step_ms_ = 0.0f;
    unsigned long long* step_trace_ = nullptr;
    float last_greedy_ms_ = 0.0f;
    float last_batch_ms_ = 0.0f;
    cudaEvent_t ev0_ = nullptr, ev1_ = nullptr;
    std::vector<ProfClass>* prof_ = nullptr;
    cudaEvent_t pe0_ = nullptr, pe1_ = nullptr;
    struct ProfRec { int cls; double bytes; int e0, e1; };
    std::vector<cudaEvent_t> prof_events_;   // pool, reused across profiles
    std::vector<ProfRec> prof_recs_;
    int prof_next_ = 0, prof_open_ = -1;
    int prof_event();
};

}  // namespace fb
