// engine.cpp — see engine.h.
#include "engine.h"

#include <dlfcn.h>
#include <mutex>
#include <nccl.h>
#include "kernels/layout.cuh"
#include "kernels/stream_common.cuh"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <thread>

namespace fb {

namespace {

const char* cerr_str(int e) { return cudaGetErrorString(static_cast<cudaError_t>(e)); }

#define CK(call)                                                                              \
    do {                                                                                      \
        const int rc_ = (int)(call);                                                          \
        if (rc_ != 0) {                                                                       \
            if (err) *err = std::string(#call) + ": " + cerr_str(rc_);                        \
            return false;                                                                     \
        }                                                                                     \
    } while (0)

// Like CK, and when a profile is being taken, time the launch on the stream.
#define CKP(cls, bytes, call)                                                                 \
    do {                                                                                      \
        if (prof_) prof_begin();                                                              \
        const int rc_ = (int)(call);                                                          \
        if (rc_ != 0) {                                                                       \
            if (err) *err = std::string(#call) + ": " + cerr_str(rc_);                        \
            return false;                                                                     \
        }                                                                                     \
        if (prof_) prof_end(cls, bytes);                                                      \
    } while (0)

enum { PC_GEMV = 0, PC_NORMQ = 1, PC_ROPE = 2, PC_ATTN = 3, PC_OTHER = 4 };

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

bool matmul_type_ok(int t) { return t == T_Q8_0 || t == T_Q4_K || t == T_Q6_K || t == T_F32 || t == T_F16; }

// Host dequantisation of a small vector (norm weights, biases, rope factors).
bool host_vec(const Tensor* t, std::vector<float>& out) {
    if (!t) return false;
    const uint64_t n = t->n_elements();
    out.resize(n);
    if (t->type == 0) {
        std::memcpy(out.data(), t->data, n * 4);
        return true;
    }
    if (t->type == 1 || t->type == 30) {
        for (uint64_t i = 0; i < n; ++i) {
            uint16_t h;
            std::memcpy(&h, t->data + 2 * i, 2);
            if (t->type == 30) {
                const uint32_t b = (uint32_t)h << 16;
                std::memcpy(&out[i], &b, 4);
            } else {
                const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
                uint32_t e = (h >> 10) & 0x1F, m = h & 0x3FF, bits;
                if (e == 0) {
                    if (m == 0) bits = sign;
                    else {
                        int ee = 113;
                        while (!(m & 0x400)) { m <<= 1; --ee; }
                        bits = sign | ((uint32_t)ee << 23) | ((m & 0x3FF) << 13);
                    }
                } else if (e == 31) bits = sign | 0x7F800000u | (m << 13);
                else bits = sign | ((e + 112) << 23) | (m << 13);
                std::memcpy(&out[i], &bits, 4);
            }
        }
        return true;
    }
    return false;
}

int env_int(const char* name, int def) {
    const char* v = std::getenv(name);
    return v && *v ? std::atoi(v) : def;
}

}  // namespace

// RoPE cos/sin table [n_ctx][rot/2], angles in double, stored as float times
// the attention factor (the reference's table, src/ops.cpp:75-124).
bool tp_plan(int n_head, int n_head_kv, int head_dim, int n_ff, int vocab, int n_experts, int rank, int world,
             TpPlan* out, std::string* err) {
    auto fail = [&](const char* why) {
        if (err) *err = std::string("tensor parallelism: ") + why;
        return false;
    };
    if (world < 1 || rank < 0 || rank >= world || !out) return fail("bad rank or world");
    const bool moe = n_experts > 0;   // experts split over the ranks (expert parallelism), not their rows
    if (n_head % world || n_head_kv % world || n_head % n_head_kv || (!moe && n_ff % world) ||
        (moe && n_experts % world) || vocab % world || (vocab / world) % 8)
        return fail("kv heads, FFN rows (experts) and vocab rows must split evenly over the ranks");
    TpPlan p;
    p.heads = n_head / world;
    p.head0 = rank * p.heads;
    p.kv_heads = n_head_kv / world;
    p.kv_head0 = rank * p.kv_heads;
    p.q_rows = p.heads * head_dim;
    p.q_row0 = p.head0 * head_dim;
    p.kv_rows = p.kv_heads * head_dim;
    p.kv_row0 = p.kv_head0 * head_dim;
    if (moe) {
        p.experts = n_experts / world;
        p.expert0 = rank * p.experts;
    } else {
        p.ff_rows = n_ff / world;
        p.ff_row0 = rank * p.ff_rows;
    }
    p.vocab_rows = vocab / world;
    p.vocab_row0 = rank * p.vocab_rows;
    // (the loader checks that attn_output's and ffn_down's input slices are
    // whole blocks of their weight type: then the per-block integer sums are
    // the unsharded ones)
    *out = p;
    return true;
}

void build_rope_table(const Config& c, const float* ff, std::vector<float>& cs, std::vector<float>& sn) {
    const int rot = c.rot_dim, half = rot / 2;
    cs.assign((size_t)c.n_ctx * half, 0.0f);
    sn.assign((size_t)c.n_ctx * half, 0.0f);
    const bool yarn = c.yarn_factor > 0.0f && c.yarn_orig_ctx > 0;
    float corr_low = 0, corr_high = 0, ym = 1.0f;
    auto corr_dim = [&](float n_rot) {
        return (float)rot * std::log((float)c.yarn_orig_ctx / (n_rot * 2.0f * 3.14159265358979f)) /
               (2.0f * std::log(c.freq_base));
    };
    if (yarn) {
        corr_low = std::max(0.0f, std::floor(corr_dim(c.yarn_beta_fast)));
        corr_high = std::min((float)(rot - 1), std::ceil(corr_dim(c.yarn_beta_slow)));
        ym = c.yarn_attn_factor * (1.0f + 0.1f * std::log(c.yarn_factor));
    }
    std::vector<double> inv(half);
    for (int i = 0; i < half; ++i) inv[i] = std::pow((double)c.freq_base, -2.0 * i / (double)rot);
    for (int pos = 0; pos < c.n_ctx; ++pos) {
        for (int i = 0; i < half; ++i) {
            double te = (double)pos * inv[i];
            if (ff) te /= (ff[i] != 0.0f ? ff[i] : 1.0f);
            double theta;
            float m = c.mscale;
            if (yarn) {
                const float den = std::max(0.001f, corr_high - corr_low);
                const float y = std::min(1.0f, std::max(0.0f, ((float)(2 * i) / 2.0f - corr_low) / den));
                const float ramp = 1.0f - y;
                theta = (te / c.yarn_factor) * (1.0 - ramp) + te * ramp;
                m *= ym;
            } else {
                theta = te * c.freq_scale;
            }
            cs[(size_t)pos * half + i] = (float)std::cos(theta) * m;
            sn[(size_t)pos * half + i] = (float)std::sin(theta) * m;
        }
    }
}

Engine::~Engine() {
    drop_graphs();
    if (device_ >= 0) cudaSetDevice(device_);
    if (stream_) cudaStreamSynchronize(stream_);
    for (float* p : small_) cudaFree(p);
    cudaFree(warena_);
    cudaFree(x_); cudaFree(xb_); cudaFree(q_); cudaFree(k_); cudaFree(v_); cudaFree(attn_);
    cudaFree(g_); cudaFree(u_); cudaFree(logits_); cudaFree(router_); cudaFree(eo_); cudaFree(sel_); cudaFree(wsel_);
    cudaFree(act_mem_); cudaFree(att_scratch_); cudaFree(dec_part_); cudaFree(gemm_part_);
    cudaFree(pre_blocks_); cudaFree(pre_state_);
    cudaFree(ids_); cudaFree(tok_seq_); cudaFree(tok_pos_); cudaFree(argmax_); cudaFree(greedy_out_); cudaFree(greedy_step_); cudaFree(amax_keys_);
    cudaFree(kv_pool_); cudaFree(pt_arena_);
    cudaFree(rope_cos_); cudaFree(rope_sin_); cudaFree(out_norm_);
    cudaFree(step_ph_); cudaFree(step_ctl_); cudaFree(step_keys_); cudaFree(att_part_);
    cudaFree(tp_tmp_); cudaFree(tp_logits_); cudaFree(sel_loc_);
    cudaFree(gg_); cudaFree(gu_); cudaFree(geo_); cudaFree(grp_src_); cudaFree(grp_pos_); cudaFree(grp_count_);
    cudaFree(chunk_exp_); cudaFree(gact_mem_);
    if (nccl_) nccl_api(nullptr)->comm_destroy((ncclComm_t)nccl_);   // after the graphs that hold its calls
    if (probe_img_) cudaFree(probe_img_);
    if (probe_h_) cudaFree(probe_h_);
    if (recent_dev_) cudaFree(recent_dev_);
    if (h_pinned_) cudaFreeHost(h_pinned_);
    if (ev0_) cudaEventDestroy(ev0_);
    if (ev1_) cudaEventDestroy(ev1_);
    if (pe0_) cudaEventDestroy(pe0_);
    if (pe1_) cudaEventDestroy(pe1_);
    for (cudaEvent_t e : prof_events_) cudaEventDestroy(e);
    if (stream_) cudaStreamDestroy(stream_);
}

std::string Engine::device_name() const {
    cudaDeviceProp p{};
    if (cudaGetDeviceProperties(&p, device_) != cudaSuccess) return "cuda";
    return p.name;
}

void Engine::drop_graphs() {
    for (auto& kv : graphs_) cudaGraphExecDestroy(kv.second);
    graphs_.clear();
    graph_kernels_.clear();
}

// Profiling records an event before and after each launch without waiting, so
// the GPU runs the launches back to back; the pairs are read after the run.
int Engine::prof_event() {
    if (prof_next_ == (int)prof_events_.size()) {
        cudaEvent_t e = nullptr;
        cudaEventCreate(&e);
        prof_events_.push_back(e);
    }
    return prof_next_++;
}

void Engine::prof_begin() {
    prof_open_ = prof_event();
    cudaEventRecord(prof_events_[prof_open_], stream_);
}

void Engine::prof_end(int cls, double bytes) {
    const int e1 = prof_event();
    cudaEventRecord(prof_events_[e1], stream_);
    prof_recs_.push_back({cls, bytes, prof_open_, e1});
}

// ------------------------------------------------------------------ load

bool Engine::load(const std::string& path, int n_ctx, std::string* err) {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0) {
        if (err) *err = "no CUDA device: the B200 engine has no CPU fallback";
        return false;
    }
    CK(cudaGetDevice(&device_));
    CK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    CK(cudaEventCreate(&ev0_));
    CK(cudaEventCreate(&ev1_));
    CK(cudaEventCreate(&pe0_));
    CK(cudaEventCreate(&pe1_));
    use_graphs_ = env_int("FISH_NO_GRAPHS", 0) == 0;
    no_fuse_ = env_int("FISH_NO_FUSE", 0) != 0;
    prefill_simt_ = env_int("FISH_ATTN_PREFILL_SIMT", 0) != 0;
    fbk_set_pdl(env_int("FISH_NO_PDL", 0) == 0 ? 1 : 0);
    gguf_ = Gguf::open(path, err);
    if (!gguf_) return false;
    const Gguf& g = *gguf_;
    Config& c = cfg_;
    // model.cpp:403-470: metadata under the architecture prefix
    c.arch = g.str("general.architecture", "llama");
    if (c.arch != "llama" && c.arch != "qwen2" && c.arch != "qwen3" && c.arch != "qwen2moe" && c.arch != "qwen3moe" &&
        c.arch != "gemma2" && c.arch != "phi3") {
        if (err) *err = "unsupported architecture: " + c.arch +
                        " (the B200 engine runs llama, qwen2, qwen3, their MoE variants, gemma2 and phi3)";
        return false;
    }
    auto key = [&](const char* k) { return c.arch + "." + k; };
    c.n_layers = (int)g.u64(key("block_count"), 0);
    c.n_embd = (int)g.u64(key("embedding_length"), 0);
    c.n_ff = (int)g.u64(key("feed_forward_length"), 0);
    c.n_head = (int)g.u64(key("attention.head_count"), 0);
    c.n_head_kv = (int)g.u64(key("attention.head_count_kv"), (uint64_t)c.n_head);
    c.eps = (float)g.f64(key("attention.layer_norm_rms_epsilon"), 1e-5);
    c.freq_base = (float)g.f64(key("rope.freq_base"), 10000.0);
    c.bos = (int)g.i64("tokenizer.ggml.bos_token_id", 1);
    c.eos = (int)g.i64("tokenizer.ggml.eos_token_id", 2);
    c.n_ctx_train = (int)g.u64(key("context_length"), 4096);
    c.vocab = (int)g.u64(key("vocab_size"), 0);
    if (c.vocab <= 0) if (const MetaValue* t = g.meta("tokenizer.ggml.tokens")) c.vocab = (int)t->sarr.size();
    const Tensor* embd = g.find("token_embd.weight");
    if (!embd) { if (err) *err = "missing token_embd.weight"; return false; }
    if (c.vocab <= 0 && embd->ne.size() > 1) c.vocab = (int)embd->ne[1];
    if (c.n_layers <= 0 || c.n_embd <= 0 || c.n_head <= 0 || c.n_ff <= 0 || c.vocab <= 0) {
        if (err) *err = "incomplete model metadata";
        return false;
    }
    if (c.n_head_kv <= 0 || c.n_head % c.n_head_kv != 0) { if (err) *err = "n_head is not a multiple of n_head_kv"; return false; }
    c.head_dim = (int)g.u64(key("attention.key_length"), 0);
    if (c.head_dim <= 0) c.head_dim = c.n_embd / c.n_head;
    c.n_experts = (int)g.u64(key("expert_count"), 0);
    c.n_experts_per_tok = (int)g.u64(key("expert_used_count"), 0);
    c.n_ff_exp = (int)g.u64(key("expert_feed_forward_length"), (uint64_t)c.n_ff);
    if (c.n_experts > 0 && c.n_experts_per_tok <= 0) c.n_experts_per_tok = 2;
    if (c.n_experts_per_tok > c.n_experts) c.n_experts_per_tok = c.n_experts;
    c.expert_weights_norm = g.flag(key("expert_weights_norm"), c.arch != "qwen2moe");
    c.rot_dim = (int)g.u64(key("rope.dimension_count"), (uint64_t)c.head_dim);
    if (c.rot_dim <= 0 || c.rot_dim > c.head_dim) c.rot_dim = c.head_dim;
    c.neox = c.arch != "llama";
    if (c.arch == "gemma2") {   // src/model.cpp:488-496
        if (tp_world_ > 1) { if (err) *err = "tensor parallelism is not supported for gemma2"; return false; }
        c.norm_plus_one = true;
        c.gelu = true;
        c.post_norms = true;
        c.embd_scale = std::sqrt((float)c.n_embd);
        c.attn_softcap = (float)g.f64(key("attn_logit_softcapping"), 50.0);
        c.final_softcap = (float)g.f64(key("final_logit_softcapping"), 30.0);
        c.sliding_window = (int)g.u64(key("attention.sliding_window"), 4096);
    }
    const int model_ctx = c.n_ctx_train;
    c.n_ctx = n_ctx > 0 ? std::min(n_ctx, model_ctx > 0 ? model_ctx : n_ctx) : std::min(4096, model_ctx);
    if (c.n_ctx < 32) { if (err) *err = "context too small"; return false; }
    if ((c.head_dim != 64 && c.head_dim != 96 && c.head_dim != 128) || c.n_head / c.n_head_kv > 8) {
        if (err) *err = "attention shape not supported by the B200 kernels (head_dim 64, 96 or 128, <= 8 q heads per kv head)";
        return false;
    }
    c.n_head_model = c.n_head;
    c.n_head_kv_model = c.n_head_kv;
    c.n_ff_model = c.n_ff;
    c.out_rows = c.vocab;
    c.out_row0 = 0;
    if (tp_world_ > 1) {   // this rank's heads, FFN rows and vocab rows
        TpPlan tp;
        if (!tp_plan(c.n_head, c.n_head_kv, c.head_dim, c.n_ff, c.vocab, c.n_experts, tp_rank_, tp_world_, &tp, err))
            return false;
        c.n_head = tp.heads;
        c.n_head_kv = tp.kv_heads;
        if (c.n_experts == 0) c.n_ff = tp.ff_rows;
        ep_n_ = tp.experts;
        ep_e0_ = tp.expert0;
        c.out_rows = tp.vocab_rows;
        c.out_row0 = tp.vocab_row0;
    }
    std::string longrope;   // the longrope factor tensor in use (phi3)
    {
        const std::string type = g.str(key("rope.scaling.type"), "none");
        const float factor = (float)g.f64(key("rope.scaling.factor"), 1.0);
        const int orig = (int)g.u64(key("rope.scaling.original_context_length"), 0);
        if (type == "linear" && factor > 0.0f) c.freq_scale = 1.0f / factor;
        else if (type == "yarn" && factor > 0.0f) {
            c.yarn_factor = factor;
            c.yarn_orig_ctx = orig > 0 ? orig : model_ctx;
            c.yarn_attn_factor = (float)g.f64(key("rope.scaling.attn_factor"), 1.0);
        } else if (type == "longrope") {
            // phi3 (src/model.cpp:522-530): per-pair factors, the long set
            // beyond the original context, the short set within it; the
            // attention factor scales the rotation
            longrope = (orig > 0 && c.n_ctx > orig) ? "rope_factors_long.weight" : "rope_factors_short.weight";
            if (!g.find(longrope)) longrope = "rope_factors_short.weight";
            c.mscale = (float)g.f64(key("rope.scaling.attn_factor"), 1.0);
        }
    }

    // weights
    auto bind = [&](const std::string& name, DevW& w, bool required) -> bool {
        const Tensor* t = g.find(name);
        if (!t) {
            if (required && err) *err = "missing tensor " + name;
            return !required;
        }
        if (!matmul_type_ok(t->type)) {
            if (err) *err = std::string("tensor type ") + ggml_type_name(t->type) + " is not supported on the B200 path yet (" + name + ")";
            return false;
        }
        w.name = name;
        w.type = t->type;
        w.n_in = (int)t->ne[0];
        w.n_out = t->ne.size() > 1 ? (int)t->ne[1] : 1;
        w.n_exp = t->ne.size() > 2 ? (int)t->ne[2] : 1;
        w.n_in_src = w.n_in;
        w.n_out_src = w.n_out;
        w.stride = dev_row_bytes(t->type, w.n_in);
        w.expert_bytes = dev_matrix_bytes(t->type, w.n_in, w.n_out);
        if (t->type == T_Q4_K || t->type == T_Q6_K) {
            if (w.n_in % 256) { if (err) *err = "K-quant row not a multiple of 256: " + name; return false; }
        }
        return true;
    };
    // tensor-parallel shards: a row range, or a range of input values (whole
    // blocks, so a shard's block integers are the unsharded ones)
    // (row0 adds to the view's own first row: a shard of one part of a fused tensor)
    auto shard_rows = [&](DevW& w, int n, int row0) {
        w.n_out = n;
        w.row0 += row0;
        w.expert_bytes = dev_matrix_bytes(w.type, w.n_in, w.n_out);
    };
    auto shard_k = [&](DevW& w, int n, int k0, const std::string& name) -> bool {
        const int blk = w.type == T_Q8_0 ? 32 : (w.type == T_Q4_K || w.type == T_Q6_K ? 256 : 8);
        if (k0 % blk || n % blk) {
            if (err) *err = "tensor parallelism: input slice of " + name + " is not block-aligned";
            return false;
        }
        w.n_in = n;
        w.k0 = k0;
        w.stride = dev_row_bytes(w.type, w.n_in);
        w.expert_bytes = dev_matrix_bytes(w.type, w.n_in, w.n_out);
        return true;
    };
    if (!bind("token_embd.weight", embd_, true)) return false;
    if (!bind("output.weight", out_w_, false)) return false;
    if (out_w_.type < 0) { out_w_ = embd_; c.tied_output = true; }
    else if (tp_world_ > 1) shard_rows(out_w_, c.out_rows, c.out_row0);
    layers_.resize(c.n_layers);
    for (int i = 0; i < c.n_layers; ++i) {
        const std::string p = "blk." + std::to_string(i) + ".";
        DevLayer& L = layers_[i];
        if (g.find(p + "attn_qkv.weight")) {
            // phi3: fused q|k|v rows (src/model.cpp:253, 1665-1674): three
            // views of one tensor, each uploaded as its own matrix
            const int Q = c.n_head_model * c.head_dim, KV = c.n_head_kv_model * c.head_dim;   // whole-model rows
            DevW f;
            if (!bind(p + "attn_qkv.weight", f, true)) return false;
            if (f.n_out != Q + 2 * KV) { if (err) *err = "fused attn_qkv has an unexpected shape in layer " + std::to_string(i); return false; }
            L.wq = L.wk = L.wv = f;
            shard_rows(L.wq, Q, 0);
            shard_rows(L.wk, KV, Q);
            shard_rows(L.wv, KV, Q + KV);
            if (!bind(p + "attn_output.weight", L.wo, true)) return false;
        } else if (!bind(p + "attn_q.weight", L.wq, true) || !bind(p + "attn_k.weight", L.wk, true) ||
                   !bind(p + "attn_v.weight", L.wv, true) || !bind(p + "attn_output.weight", L.wo, true)) {
            return false;
        }
        if (tp_world_ > 1) {
            const int Q = c.q_dim(), KV = c.kv_dim(), r = tp_rank_;
            shard_rows(L.wq, Q, r * Q);
            shard_rows(L.wk, KV, r * KV);
            shard_rows(L.wv, KV, r * KV);
            if (!shard_k(L.wo, Q, r * Q, p + "attn_output.weight")) return false;
        }
        if (c.n_experts > 0) {
            if (!bind(p + "ffn_gate_inp.weight", L.gate_inp, true) || !bind(p + "ffn_gate_exps.weight", L.gate_exps, true) ||
                !bind(p + "ffn_up_exps.weight", L.up_exps, true) || !bind(p + "ffn_down_exps.weight", L.down_exps, true))
                return false;
            c.n_ff_exp = L.gate_exps.n_out;
            // the shared expert every token also takes (qwen2moe, src/model.cpp:303-308, 1582-1599)
            if (!bind(p + "ffn_gate_shexp.weight", L.shexp_gate, false) || !bind(p + "ffn_up_shexp.weight", L.shexp_up, false) ||
                !bind(p + "ffn_down_shexp.weight", L.shexp_down, false) ||
                !bind(p + "ffn_gate_inp_shexp.weight", L.shexp_gate_inp, false))
                return false;
            if (L.shexp_gate.type >= 0 && L.shexp_up.type >= 0 && L.shexp_down.type >= 0) {
                if (L.shexp_up.n_out != L.shexp_gate.n_out || L.shexp_down.n_in != L.shexp_gate.n_out ||
                    (L.shexp_gate_inp.type >= 0 && (L.shexp_gate_inp.n_out != 1 || L.shexp_gate_inp.n_in != c.n_embd))) {
                    if (err) *err = "shared expert tensors of layer " + std::to_string(i) + " have inconsistent shapes";
                    return false;
                }
                c.n_ff_shexp = std::max(c.n_ff_shexp, L.shexp_gate.n_out);
            } else {
                L.shexp_gate = L.shexp_up = L.shexp_down = L.shexp_gate_inp = DevW{};
            }
            if (tp_world_ > 1) {   // this rank's experts
                for (DevW* w : {&L.gate_exps, &L.up_exps, &L.down_exps}) {
                    if (w->n_exp != c.n_experts) { if (err) *err = "expert tensor count differs from expert_count"; return false; }
                    w->n_exp = ep_n_;
                    w->e0 = ep_e0_;
                }
            }
        } else {
            if (!g.find(p + "ffn_gate.weight")) {
                // phi3: fused gate|up, ffn_up holding 2 n_ff rows, gate first
                // (src/model.cpp:310-316, 1481-1489)
                DevW f;
                if (!bind(p + "ffn_up.weight", f, true) || !bind(p + "ffn_down.weight", L.wd, true)) return false;
                const int Fm = c.n_ff_model;
                if (f.n_out != 2 * Fm) { if (err) *err = "missing tensor " + p + "ffn_gate.weight"; return false; }
                L.wg = L.wu = f;
                shard_rows(L.wg, Fm, 0);
                shard_rows(L.wu, Fm, Fm);
            } else if (!bind(p + "ffn_gate.weight", L.wg, true) || !bind(p + "ffn_up.weight", L.wu, true) ||
                       !bind(p + "ffn_down.weight", L.wd, true)) {
                return false;
            }
            if (tp_world_ > 1) {
                const int F = c.n_ff, r = tp_rank_;
                shard_rows(L.wg, F, r * F);
                shard_rows(L.wu, F, r * F);
                if (!shard_k(L.wd, F, r * F, p + "ffn_down.weight")) return false;
            }
        }
    }
    // activation layouts each consumer needs
    for (const DevLayer& L : layers_) {
        for (const DevW* w : {&L.wq, &L.wk, &L.wv, &L.wg, &L.wu, &L.gate_exps, &L.up_exps, &L.shexp_gate, &L.shexp_up,
                              &L.shexp_gate_inp}) {
            if (w->type == T_Q8_0) want32_e_ = true;
            if (w->type == T_Q4_K || w->type == T_Q6_K) wantk_e_ = true;
        }
        if (L.wo.type == T_Q8_0) want32_q_ = true;
        if (L.wo.type == T_Q4_K || L.wo.type == T_Q6_K) wantk_q_ = true;
        for (const DevW* w : {&L.wd, &L.down_exps, &L.shexp_down}) {
            if (w->type == T_Q8_0) want32_f_ = true;
            if (w->type == T_Q4_K || w->type == T_Q6_K) wantk_f_ = true;
        }
    }
    if (out_w_.type == T_Q8_0) want32_e_ = true;
    if (out_w_.type == T_Q4_K || out_w_.type == T_Q6_K) wantk_e_ = true;
    if (c.n_experts > 0 && c.n_experts_per_tok > 8) { if (err) *err = "more than 8 experts per token"; return false; }
    for (const Tensor& t : g.tensors()) weights_file_bytes_ += t.nbytes;

    const auto t0 = std::chrono::steady_clock::now();
    if (!upload_weights(err)) return false;
    load_seconds_upload = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();

    // small vectors
    // row0 / n: this rank's slice of the vector (biases of sharded rows)
    // plus_one: a norm weight stored as w - 1 (gemma2, src/model.cpp:241-245)
    auto dev_vec = [&](const std::string& name, float** out, bool required, int row0 = 0, int n = -1,
                       bool plus_one = false) -> bool {
        const Tensor* t = g.find(name);
        if (!t) {
            if (required && err) *err = "missing tensor " + name;
            return !required;
        }
        std::vector<float> v;
        if (!host_vec(t, v)) { if (err) *err = "bad vector " + name; return false; }
        if (plus_one) for (float& x : v) x += 1.0f;
        if (n >= 0) {
            if (row0 + n > (int)v.size()) { if (err) *err = "bad vector slice " + name; return false; }
            v = std::vector<float>(v.begin() + row0, v.begin() + row0 + n);
        }
        float* d = nullptr;
        CK(cudaMalloc(&d, v.size() * sizeof(float)));
        CK(cudaMemcpy(d, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice));
        small_.push_back(d);
        *out = d;
        return true;
    };
    for (int i = 0; i < c.n_layers; ++i) {
        const std::string p = "blk." + std::to_string(i) + ".";
        DevLayer& L = layers_[i];
        const int sq = tp_world_ > 1 ? c.q_dim() : -1, skv = tp_world_ > 1 ? c.kv_dim() : -1;
        const bool p1 = c.norm_plus_one;
        if (!dev_vec(p + "attn_norm.weight", &L.attn_norm, true, 0, -1, p1) ||
            !dev_vec(p + "ffn_norm.weight", &L.ffn_norm, true, 0, -1, p1) ||
            (c.post_norms && (!dev_vec(p + "post_attention_norm.weight", &L.post_attn_norm, true, 0, -1, p1) ||
                              !dev_vec(p + "post_ffw_norm.weight", &L.post_ffn_norm, true, 0, -1, p1))) ||
            !dev_vec(p + "attn_q.bias", &L.bq, false, tp_rank_ * c.q_dim(), sq) ||
            !dev_vec(p + "attn_k.bias", &L.bk, false, tp_rank_ * c.kv_dim(), skv) ||
            !dev_vec(p + "attn_v.bias", &L.bv, false, tp_rank_ * c.kv_dim(), skv) ||
            !dev_vec(p + "attn_output.bias", &L.bo, false) ||
            !dev_vec(p + "attn_q_norm.weight", &L.q_norm, false) ||
            !dev_vec(p + "attn_k_norm.weight", &L.k_norm, false))
            return false;
        if (L.q_norm && L.k_norm) c.qk_norm = true;
        if (g.find(p + "attn_qkv.bias")) {   // fused q|k|v bias (src/model.cpp:348): this rank's slices
            const int Qm = c.n_head_model * c.head_dim, KVm = c.n_head_kv_model * c.head_dim;
            const int Q = c.q_dim(), KV = c.kv_dim();
            if (!dev_vec(p + "attn_qkv.bias", &L.bq, true, tp_rank_ * Q, Q) ||
                !dev_vec(p + "attn_qkv.bias", &L.bk, true, Qm + tp_rank_ * KV, KV) ||
                !dev_vec(p + "attn_qkv.bias", &L.bv, true, Qm + KVm + tp_rank_ * KV, KV))
                return false;
        }
    }
    {
        const Tensor* t = g.find("output_norm.weight");
        std::vector<float> v;
        if (!t || !host_vec(t, v)) { if (err) *err = "missing output_norm.weight"; return false; }
        if (c.norm_plus_one) for (float& x : v) x += 1.0f;
        CK(cudaMalloc(&out_norm_, v.size() * sizeof(float)));
        CK(cudaMemcpy(out_norm_, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice));
    }
    {
        std::vector<float> ff, cs, sn;
        // longrope factors (phi3), else Llama-3 style rope_freqs (src/model.cpp:532-543)
        const Tensor* rf = g.find(longrope.empty() ? std::string("rope_freqs.weight") : longrope);
        if (rf && (!host_vec(rf, ff) || (int)ff.size() != c.rot_dim / 2)) { if (err) *err = "bad rope factors"; return false; }
        build_rope_table(c, ff.empty() ? nullptr : ff.data(), cs, sn);
        CK(cudaMalloc(&rope_cos_, cs.size() * sizeof(float)));
        CK(cudaMalloc(&rope_sin_, sn.size() * sizeof(float)));
        CK(cudaMemcpy(rope_cos_, cs.data(), cs.size() * sizeof(float), cudaMemcpyHostToDevice));
        CK(cudaMemcpy(rope_sin_, sn.data(), sn.size() * sizeof(float), cudaMemcpyHostToDevice));
    }
    if (!alloc_buffers(err)) return false;
    seqs_.assign(max_seqs_, Seq());
    seqs_[0].open = true;
    return true;
}

bool Engine::upload_weights(std::string* err) {
    const Gguf& g = *gguf_;
    struct Job { const Tensor* t; DevW* w; size_t off; };
    std::vector<Job> jobs;
    size_t total = 0;
    // every bound matrix, uploaded from the GGUF tensor it names (a fused
    // tensor's views each take their own rows)
    auto add = [&](DevW* w) {
        if (w->type < 0) return;
        const Tensor* t = g.find(w->name);
        if (!t) return;
        jobs.push_back({t, w, total});
        total = align_up(total + w->expert_bytes * (size_t)w->n_exp, 256);
    };
    add(&embd_);
    if (!cfg_.tied_output) add(&out_w_);
    for (DevLayer& L : layers_)
        for (DevW* w : {&L.wq, &L.wk, &L.wv, &L.wo, &L.wg, &L.wu, &L.wd, &L.gate_inp, &L.gate_exps, &L.up_exps,
                        &L.down_exps, &L.shexp_gate, &L.shexp_up, &L.shexp_down, &L.shexp_gate_inp})
            add(w);
    weights_dev_bytes_ = total;
    CK(cudaMalloc(&warena_, total + 256));
    for (Job& j : jobs) j.w->d = warena_ + j.off;
    if (cfg_.tied_output) {
        out_w_ = embd_;
        if (tp_world_ > 1) {   // this rank's vocab rows of the shared table: whole 8-row tiles
            out_w_.n_out = cfg_.out_rows;
            out_w_.row0 = cfg_.out_row0;
            out_w_.d = embd_.d + (size_t)(cfg_.out_row0 / 8) * dev_matrix_bytes(embd_.type, embd_.n_in, 8);
            out_w_.expert_bytes = dev_matrix_bytes(embd_.type, embd_.n_in, cfg_.out_rows);
        }
    }

    // staged, repacked upload: rows repacked by host threads into pinned
    // buffers, copied while the next buffer fills.
    const size_t stage = 64ull << 20;
    uint8_t* pin[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    CK(cudaMallocHost(&pin[0], stage));
    CK(cudaMallocHost(&pin[1], stage));
    CK(cudaEventCreate(&done[0]));
    CK(cudaEventCreate(&done[1]));
    const int nth = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    int cur = 0;
    bool ok = true;
    // chunks of whole 8-row tiles within one expert slice; each host thread
    // repacks a run of tiles
    for (const Job& j : jobs) {
        const DevW& w = *j.w;
        const size_t src_rb = ggml_row_bytes(j.t->type, (uint64_t)w.n_in_src);   // a whole source row
        const size_t k_off = ggml_row_bytes(j.t->type, (uint64_t)w.k0);          // the shard's first value
        const size_t tile_bytes = dev_matrix_bytes(w.type, w.n_in, 8);
        const int rows_per = (int)std::max<size_t>(8, stage / tile_bytes * 8);
        for (int e = 0; e < w.n_exp && ok; ++e) {
            for (int r0 = 0; r0 < w.n_out && ok; r0 += rows_per) {
                const int nr = std::min(rows_per, w.n_out - r0);
                const size_t nbytes = dev_matrix_bytes(w.type, w.n_in, nr);
                if (cudaEventSynchronize(done[cur]) != cudaSuccess) { ok = false; break; }
                uint8_t* dst = pin[cur];
                const uint8_t* src = j.t->data + ((size_t)(w.e0 + e) * w.n_out_src + w.row0 + r0) * src_rb + k_off;
                const int n_tiles = (nr + 7) / 8;
                auto work = [&](int tid) {
                    const int a = (int)((long long)n_tiles * tid / nth), b = (int)((long long)n_tiles * (tid + 1) / nth);
                    if (a >= b) return;
                    const int ra = 8 * a, rb = std::min(nr, 8 * b);
                    repack_rows(w.type, src + (size_t)ra * src_rb, rb - ra, w.n_in, dst + (size_t)a * tile_bytes, src_rb);
                };
                std::vector<std::thread> th;
                for (int i = 1; i < nth; ++i) th.emplace_back(work, i);
                work(0);
                for (auto& t : th) t.join();
                uint8_t* dev = w.d + (size_t)e * w.expert_bytes + (size_t)(r0 / 8) * tile_bytes;
                if (cudaMemcpyAsync(dev, dst, nbytes, cudaMemcpyHostToDevice, stream_) != cudaSuccess ||
                    cudaEventRecord(done[cur], stream_) != cudaSuccess) {
                    ok = false;
                    break;
                }
                cur ^= 1;
            }
        }
    }
    cudaStreamSynchronize(stream_);
    cudaEventDestroy(done[0]);
    cudaEventDestroy(done[1]);
    cudaFreeHost(pin[0]);
    cudaFreeHost(pin[1]);
    if (!ok) { if (err) *err = "weight upload failed"; return false; }
    return true;
}

bool Engine::alloc_buffers(std::string* err) {
    const Config& c = cfg_;
    const int E = c.n_embd, Q = c.q_dim(), KV = c.kv_dim();
    const int K = std::max(1, c.n_experts_per_tok);
    const int F = std::max(std::max(c.n_ff, c.n_ff_exp), c.n_ff_shexp);
    max_k_ = std::max(std::max(E, Q), F);
    const int R = kMaxBatch * K;   // rows of the expert-expanded activations
    const size_t ld = align_up((size_t)max_k_, 16);
    CK(cudaMalloc(&x_, sizeof(float) * kMaxBatch * E));
    CK(cudaMalloc(&xb_, sizeof(float) * kMaxBatch * E));
    CK(cudaMalloc(&q_, sizeof(float) * kMaxBatch * Q));
    CK(cudaMalloc(&k_, sizeof(float) * kMaxBatch * KV));
    CK(cudaMalloc(&v_, sizeof(float) * kMaxBatch * KV));
    CK(cudaMalloc(&attn_, sizeof(float) * kMaxBatch * Q));
    CK(cudaMalloc(&g_, sizeof(float) * (size_t)R * F));
    CK(cudaMalloc(&u_, sizeof(float) * (size_t)R * F));
    CK(cudaMalloc(&logits_, sizeof(float) * (size_t)kMaxBatch * c.vocab));
    if (tp_world_ > 1 || c.post_norms) {   // gemma2: the o / down rows before their post norm
        CK(cudaMalloc(&tp_tmp_, sizeof(float) * (size_t)kMaxBatch * E));
    }
    if (tp_world_ > 1) {
        CK(cudaMalloc(&tp_logits_, sizeof(float) * (size_t)tp_world_ * kMaxBatch * c.out_rows));
    }
    if (c.n_experts > 0) {
        CK(cudaMalloc(&router_, sizeof(float) * kMaxBatch * c.n_experts));
        CK(cudaMalloc(&eo_, sizeof(float) * (size_t)R * E));
        CK(cudaMalloc(&sel_, sizeof(int32_t) * R));
        if (tp_world_ > 1) CK(cudaMalloc(&sel_loc_, sizeof(int32_t) * R));
        CK(cudaMalloc(&wsel_, sizeof(float) * R));
        // expert grouping: local experts x kMaxBatch grouped rows
        const int nel = tp_world_ > 1 ? (c.n_experts + tp_world_ - 1) / tp_world_ : c.n_experts;
        grp_rows_ = nel * kMaxBatch;
        const int FE = std::max(E, c.n_ff_exp);
        const size_t gld = align_up((size_t)FE, 16);
        CK(cudaMalloc(&gg_, sizeof(float) * (size_t)grp_rows_ * c.n_ff_exp));
        CK(cudaMalloc(&gu_, sizeof(float) * (size_t)grp_rows_ * c.n_ff_exp));
        CK(cudaMalloc(&geo_, sizeof(float) * (size_t)grp_rows_ * E));
        CK(cudaMalloc(&grp_src_, sizeof(int32_t) * grp_rows_));
        CK(cudaMalloc(&grp_pos_, sizeof(int32_t) * R));
        CK(cudaMalloc(&grp_count_, sizeof(int32_t) * nel));
        CK(cudaMalloc(&chunk_exp_, sizeof(int32_t) * nel * (kMaxBatch / 4)));
        const size_t gq = (size_t)grp_rows_ * gld, g32 = (size_t)grp_rows_ * (FE / 32 + 1), g256 = (size_t)grp_rows_ * (FE / 256 + 1);
        CK(cudaMalloc(&gact_mem_, 2 * gq + g32 * (4 + 4 + 2) + g256 * 4 + 1024));
        uint8_t* gp = reinterpret_cast<uint8_t*>(gact_mem_);
        gact_.q32 = reinterpret_cast<int8_t*>(gp); gp += gq;
        gact_.qk = reinterpret_cast<int8_t*>(gp); gp += gq;
        gact_.d32 = reinterpret_cast<float*>(gp); gp += align_up(g32 * 4, 16);
        gact_.s32 = reinterpret_cast<int32_t*>(gp); gp += align_up(g32 * 4, 16);
        gact_.dk = reinterpret_cast<float*>(gp); gp += align_up(g256 * 4, 16);
        gact_.bsk = reinterpret_cast<int16_t*>(gp);
        gact_.ld = (int)gld;
    }
    // activation planes: q32 | qk (R x ld each), d32 | s32 | bsk (R x max_k/32), dk (R x max_k/256)
    const size_t nq = (size_t)R * ld, n32 = (size_t)R * (max_k_ / 32 + 1), n256 = (size_t)R * (max_k_ / 256 + 1);
    const size_t bytes = 2 * nq + n32 * (4 + 4 + 2) + n256 * 4 + 1024;
    CK(cudaMalloc(&act_mem_, bytes));
    uint8_t* p = reinterpret_cast<uint8_t*>(act_mem_);
    act_.q32 = reinterpret_cast<int8_t*>(p); p += nq;
    act_.qk = reinterpret_cast<int8_t*>(p); p += nq;
    act_.d32 = reinterpret_cast<float*>(p); p += align_up(n32 * 4, 16);
    act_.s32 = reinterpret_cast<int32_t*>(p); p += align_up(n32 * 4, 16);
    act_.dk = reinterpret_cast<float*>(p); p += align_up(n256 * 4, 16);
    act_.bsk = reinterpret_cast<int16_t*>(p);
    act_.ld = (int)ld;
    // attention scratch for att_chunk_ tokens per launch at the full context
    att_chunk_ = 64;
    att_scratch_floats_ = fbk_attention_scratch_floats(att_chunk_, c.n_head, c.head_dim, c.n_ctx);
    CK(cudaMalloc(&att_scratch_, sizeof(float) * att_scratch_floats_));
    // rank partials of batched decode attention (every token of a full batch)
    dec_part_floats_ = fbk_attention_decode_part_floats(kMaxBatch, c.n_head, c.n_head_kv, c.head_dim);
    CK(cudaMalloc(&dec_part_, sizeof(float) * dec_part_floats_));
    // K-split partial values of the tensor-core GEMM on narrow matrices
    gemm_part_floats_ = (size_t)16 << 20;
    CK(cudaMalloc(&gemm_part_, sizeof(float) * gemm_part_floats_));
    // shared-prefix attention of batched decode: the prefix length (set
    // before each step) and the warps' states, for batches of up to
    // kPrefixMaxBatch sessions
    CK(cudaMalloc(&pre_blocks_, sizeof(int32_t)));
    CK(cudaMemset(pre_blocks_, 0, sizeof(int32_t)));
    pre_state_floats_ = fbk_attention_prefix_state_floats(kPrefixMaxBatch, c.n_head_kv, c.head_dim);
    CK(cudaMalloc(&pre_state_, sizeof(float) * pre_state_floats_));
    CK(cudaMalloc(&ids_, sizeof(int32_t) * kMaxBatch));
    CK(cudaMalloc(&tok_seq_, sizeof(int32_t) * kMaxBatch));
    CK(cudaMalloc(&tok_pos_, sizeof(int32_t) * kMaxBatch));
    CK(cudaMalloc(&argmax_, sizeof(int32_t) * kMaxBatch));
    CK(cudaMalloc(&amax_keys_, sizeof(unsigned long long) * kMaxBatch));
    CK(cudaMemset(amax_keys_, 0, sizeof(unsigned long long) * kMaxBatch));
    CK(cudaMalloc(&greedy_out_, sizeof(int32_t) * greedy_cap_));
    CK(cudaMalloc(&greedy_step_, sizeof(int32_t)));
    CK(cudaMalloc(&recent_dev_, sizeof(int32_t) * kMaxRecent));
    CK(cudaMallocHost(&h_pinned_, sizeof(int32_t) * (3 * kMaxBatch + kMaxRecent + 4)));
    // the kernels' shared error flag is allocated on first use; make that use
    // now, so a context's first launches may be inside a graph capture
    if (!fbk_gemv_error_flag()) {
        if (err) *err = "error flag allocation failed";
        return false;
    }

    // KV pool
    kv_f16_ = env_int("FISH_KV_F32", 0) == 0;
    const size_t esz = kv_f16_ ? 2 : 4;
    page_elems_ = (size_t)c.n_layers * 2 * c.n_head_kv * kPageSize * c.head_dim;
    const size_t page_bytes = page_elems_ * esz;
    size_t free_b = 0, total_b = 0;
    cudaMemGetInfo(&free_b, &total_b);
    long long positions = env_int("FISH_KV_POSITIONS", 0);
    if (positions <= 0) positions = std::max<long long>(2LL * c.n_ctx, 65536);
    const long long cap_pos = (long long)((double)free_b * 0.45 / (double)page_bytes) * kPageSize;
    positions = std::max<long long>(std::min(positions, cap_pos), c.n_ctx + kPageSize);
    n_pages_ = (int)((positions + kPageSize - 1) / kPageSize);
    kv_pool_bytes_ = (uint64_t)n_pages_ * page_bytes;
    CK(cudaMalloc(&kv_pool_, kv_pool_bytes_));
    page_ref_.assign(n_pages_, 0);
    free_pages_.clear();
    for (int i = n_pages_ - 1; i >= 0; --i) free_pages_.push_back(i);
    max_seqs_ = std::max(1, env_int("FISH_MAX_SESSIONS", 256));
    pt_stride_ = (c.n_ctx + kPageSize - 1) / kPageSize + 1;
    CK(cudaMalloc(&pt_arena_, sizeof(int32_t) * (size_t)max_seqs_ * pt_stride_));
    CK(cudaMemset(pt_arena_, 0, sizeof(int32_t) * (size_t)max_seqs_ * pt_stride_));
    return true;
}

KvView Engine::kv_view() const {
    KvView kv{};
    const Config& c = cfg_;
    const size_t head = (size_t)kPageSize * c.head_dim;
    const size_t vofs = (size_t)c.n_head_kv * head;
    kv.f16 = kv_f16_ ? 1 : 0;
    kv.k = kv_pool_;
    kv.v = kv_f16_ ? (void*)(reinterpret_cast<__half*>(kv_pool_) + vofs) : (void*)(reinterpret_cast<float*>(kv_pool_) + vofs);
    kv.pt = pt_arena_;
    kv.pt_stride = pt_stride_;
    kv.tok_seq = tok_seq_;
    kv.tok_pos = tok_pos_;
    kv.page_size = kPageSize;
    kv.page_stride = page_elems_;
    kv.layer_stride = 2 * vofs;
    kv.head_stride = head;
    kv.n_pages = n_pages_;
    kv.err = fbk_gemv_error_flag();
    return kv;
}

// ------------------------------------------------------------------ sequences

int Engine::seq_open() {
    for (int i = 1; i < max_seqs_; ++i) {
        if (!seqs_[i].open) {
            seqs_[i] = Seq();
            seqs_[i].open = true;
            return i;
        }
    }
    return -1;
}

bool Engine::seq_close(int sid) {
    if (sid < 0 || sid >= max_seqs_ || !seqs_[sid].open) return false;
    seq_truncate(sid, 0);
    if (sid != 0) seqs_[sid].open = false;
    return true;
}

int Engine::seq_len(int sid) const {
    if (sid < 0 || sid >= max_seqs_ || !seqs_[sid].open) return -1;
    return seqs_[sid].len;
}

std::vector<int> Engine::seq_pages(int sid) const {
    if (sid < 0 || sid >= max_seqs_ || !seqs_[sid].open) return {};
    return seqs_[sid].pages;
}

void Engine::write_page_table(int sid) {
    const Seq& s = seqs_[sid];
    if (s.pages.empty()) return;
    // small synchronous copy: page tables change only when a page boundary is crossed
    std::vector<int32_t> row(s.pages.begin(), s.pages.end());
    cudaMemcpyAsync(pt_arena_ + (size_t)sid * pt_stride_, row.data(), row.size() * sizeof(int32_t),
                    cudaMemcpyHostToDevice, stream_);
    cudaStreamSynchronize(stream_);
}

bool Engine::seq_truncate(int sid, int n) {
    if (sid < 0 || sid >= max_seqs_ || !seqs_[sid].open) return false;
    Seq& s = seqs_[sid];
    if (n < 0) n = 0;
    if (n >= s.len) { s.len = std::min(n, s.len); return true; }
    s.len = n;
    const int keep = (n + kPageSize - 1) / kPageSize;
    while ((int)s.pages.size() > keep) {
        const int p = s.pages.back();
        s.pages.pop_back();
        if (--page_ref_[p] == 0) free_pages_.push_back(p);
    }
    return true;
}

bool Engine::ensure_pages(int sid, int new_len, std::string* err) {
    Seq& s = seqs_[sid];
    if (new_len > cfg_.n_ctx) {
        if (err) *err = "context full (" + std::to_string(new_len) + " > " + std::to_string(cfg_.n_ctx) + ")";
        return false;
    }
    bool changed = false;
    // copy-on-write: the page holding position s.len must be private before appending into it
    if (s.len % kPageSize != 0 && !s.pages.empty()) {
        const int pi = s.len / kPageSize;
        const int p = s.pages[pi];
        if (page_ref_[p] > 1) {
            if (free_pages_.empty()) { if (err) *err = "KV pool exhausted"; return false; }
            const int np = free_pages_.back();
            free_pages_.pop_back();
            const size_t pb = page_elems_ * (kv_f16_ ? 2 : 4);
            if (cudaMemcpyAsync(reinterpret_cast<uint8_t*>(kv_pool_) + (size_t)np * pb,
                                reinterpret_cast<uint8_t*>(kv_pool_) + (size_t)p * pb, pb, cudaMemcpyDeviceToDevice,
                                stream_) != cudaSuccess) {
                if (err) *err = "page copy failed";
                return false;
            }
            --page_ref_[p];
            page_ref_[np] = 1;
            s.pages[pi] = np;
            changed = true;
        }
    }
    const int need = (new_len + kPageSize - 1) / kPageSize;
    while ((int)s.pages.size() < need) {
        if (free_pages_.empty()) { if (err) *err = "KV pool exhausted"; return false; }
        const int p = free_pages_.back();
        free_pages_.pop_back();
        page_ref_[p] = 1;
        s.pages.push_back(p);
        changed = true;
    }
    if (changed) write_page_table(sid);
    return true;
}

int Engine::seq_fork(int parent, int prefix_len, std::string* err) {
    if (parent < 0 || parent >= max_seqs_ || !seqs_[parent].open) { if (err) *err = "bad parent session"; return -1; }
    const Seq& ps = seqs_[parent];
    if (prefix_len < 0 || prefix_len > ps.len) { if (err) *err = "prefix longer than the parent"; return -1; }
    const int sid = seq_open();
    if (sid < 0) { if (err) *err = "too many sessions"; return -1; }
    Seq& s = seqs_[sid];
    const int np = (prefix_len + kPageSize - 1) / kPageSize;
    for (int i = 0; i < np; ++i) {
        const int p = seqs_[parent].pages[i];
        ++page_ref_[p];
        s.pages.push_back(p);
    }
    s.len = prefix_len;
    write_page_table(sid);
    return sid;
}

// ------------------------------------------------------------------ matmuls

static double gemv_bytes(const DevW& w, int T) {
    // algorithmic bytes of one launch: the weight rows in GGUF encoding
    // (read once for all T tokens) plus the f32 outputs
    return (double)ggml_row_bytes(w.type, (uint64_t)w.n_in) * w.n_out + 4.0 * w.n_out * T;
}

static void set_act_rows(GemvArgs& g, const ActQ& a, int t0, int K) {
    g.act = a;
    g.act.K = K;
    if (a.q32) g.act.q32 = a.q32 + (size_t)t0 * a.ld;
    if (a.qk) g.act.qk = a.qk + (size_t)t0 * a.ld;
    if (a.d32) g.act.d32 = a.d32 + (size_t)t0 * (K / 32);
    if (a.s32) g.act.s32 = a.s32 + (size_t)t0 * (K / 32);
    if (a.dk) g.act.dk = a.dk + (size_t)t0 * (K / 256);
    if (a.bsk) g.act.bsk = a.bsk + (size_t)t0 * (K / 32);
}

bool Engine::fusable(const DevW* const* ws, int n, int T) const {
    if (no_fuse_) return false;
    GemvArgs g{};
    g.nseg = n;
    g.K = ws[0]->n_in;
    g.T = T;
    g.pro.mode = PRO_NORM;
    for (int i = 0; i < n; ++i) {
        if (ws[i]->n_in != g.K) return false;
        g.seg[i].type = ws[i]->type;
        g.seg[i].rows = ws[i]->n_out;
    }
    return fbk_gemv_streamable(&g) != 0;
}

bool Engine::gemv_group(const DevW* const* ws, float* const* ys, const int* ldys, const float* const* biases, int n,
                        const ActQ& a, int T, int epi, std::string* err, const GemvPro* pro, bool swiglu,
                        const int32_t* expert) {
    // T >= 16 tokens with quantised planes: one tensor-core launch per
    // segment; otherwise GEMV launches of up to 4 (streamed) or 8 tokens
    int chunk = 8;
    {
        GemvArgs p{};
        p.nseg = n;
        p.K = ws[0]->n_in;
        p.T = T;
        p.act = a;
        for (int i = 0; i < n; ++i) {
            p.seg[i].type = ws[i]->type;
            p.seg[i].rows = ws[i]->n_out;
        }
        chunk = fbk_gemv_chunk(&p);
        if (T >= 16 && !pro && !swiglu && !expert && fbk_gemm_eligible(&p)) chunk = T;
    }
    for (int t0 = 0; t0 < T; t0 += chunk) {
        const int nt = std::min(chunk, T - t0);
        GemvArgs g{};
        g.nseg = n;
        g.K = ws[0]->n_in;
        g.T = nt;
        set_act_rows(g, a, t0, g.K);
        if (pro) g.pro = *pro;
        g.swiglu = swiglu ? 1 : 0;
        g.img_dump = dump_img_ ? dump_img_ + (size_t)(t0 / chunk) * kProbeChunkBytes : nullptr;
        double bytes = 0.0;
        for (int i = 0; i < n; ++i) {
            GemvSeg& s = g.seg[i];
            s.type = ws[i]->type;
            s.w = ws[i]->d;
            s.row_stride = ws[i]->stride;
            s.w_bytes = ws[i]->expert_bytes * (size_t)ws[i]->n_exp;
            s.rows = ws[i]->n_out;
            s.y = ys[i] + (size_t)t0 * ldys[i];
            s.ldy = ldys[i];
            s.bias = biases ? biases[i] : nullptr;
            s.epi = epi;
            s.expert = expert;
            s.expert_bytes = ws[i]->expert_bytes;
            bytes += gemv_bytes(*ws[i], nt);
        }
        g.part = gemm_part_;
        g.part_floats = gemm_part_floats_;
        if (nt >= 16 && fbk_gemm_eligible(&g)) CKP(PC_GEMV, bytes, fbk_gemm(&g, stream_));
        else CKP(PC_GEMV, bytes, fbk_gemv(&g, stream_));
    }
    return true;
}

bool Engine::gemv(const DevW& w, const ActQ& a, int T, float* y, int ldy, const float* bias, int epi, const float* xf,
                  int ldxf, const int32_t* expert, std::string* err, const GemvPro* pro, unsigned long long* keys) {
    int chunk = 8;
    {
        GemvArgs p{};
        p.nseg = 1;
        p.K = w.n_in;
        p.T = T;
        p.act = a;
        p.seg[0].type = w.type;
        p.seg[0].rows = w.n_out;
        chunk = fbk_gemv_chunk(&p);
        if (T >= 16 && !pro && !expert && !keys && fbk_gemm_eligible(&p)) chunk = T;
    }
    for (int t0 = 0; t0 < T; t0 += chunk) {
        const int nt = std::min(chunk, T - t0);
        GemvArgs g{};
        g.nseg = 1;
        g.K = w.n_in;
        g.T = nt;
        set_act_rows(g, a, t0, g.K);
        if (pro) g.pro = *pro;
        g.img_dump = dump_img_ ? dump_img_ + (size_t)(t0 / chunk) * kProbeChunkBytes : nullptr;
        g.xf = xf ? xf + (size_t)t0 * ldxf : nullptr;
        g.ldxf = ldxf;
        GemvSeg& s = g.seg[0];
        s.type = w.type;
        s.w = w.d;
        s.row_stride = w.stride;
        s.w_bytes = w.expert_bytes * (size_t)w.n_exp;
        s.rows = w.n_out;
        s.y = y + (size_t)t0 * ldy;
        s.ldy = ldy;
        s.bias = bias;
        s.epi = epi;
        s.expert = expert;
        s.expert_bytes = w.expert_bytes;
        s.amax = keys ? keys + t0 : nullptr;
        s.key_row0 = keys ? cfg_.out_row0 : 0;   // argmax keys carry global vocab rows
        g.part = gemm_part_;
        g.part_floats = gemm_part_floats_;
        if (nt >= 16 && fbk_gemm_eligible(&g)) CKP(PC_GEMV, gemv_bytes(w, nt), fbk_gemm(&g, stream_));
        else CKP(PC_GEMV, gemv_bytes(w, nt), fbk_gemv(&g, stream_));
    }
    return true;
}

static ActQ act_row(const ActQ& a, int row, int K) {
    ActQ r = a;
    r.K = K;
    r.q32 = a.q32 + (size_t)row * a.ld;
    r.qk = a.qk + (size_t)row * a.ld;
    r.d32 = a.d32 + (size_t)row * (K / 32);
    r.s32 = a.s32 + (size_t)row * (K / 32);
    r.dk = a.dk + (size_t)row * (K / 256);
    r.bsk = a.bsk + (size_t)row * (K / 32);
    return r;
}

// ------------------------------------------------------------------ persistent step

// One streamed-GEMV job of the step program: the same segments, prologue and
// epilogue as the graph path's launch for one token.
static bool step_job(const DevW* const* ws, float* const* ys, const int* lds, const float* const* bs, const int* epis,
                     int n, const GemvPro& pro, bool swiglu, int grid, StepPhase* out, int* slot_max, int* union_need,
                     double* wbytes) {
    StepPhase ph{};
    GemvArgs& g = ph.a;
    g.nseg = n;
    g.K = ws[0]->n_in;
    g.T = 1;
    g.pro = pro;
    g.swiglu = swiglu ? 1 : 0;
    bool wantk = false, want32 = false;
    const int G = row_groups(ws[0]->type, g.K);
    ph.tile0[0] = 0;
    for (int i = 0; i < n; ++i) {
        const DevW& w = *ws[i];
        if (!is_tiled(w.type) || w.n_in != g.K || row_groups(w.type, g.K) != G) return false;
        if ((w.type == T_Q4_K || w.type == T_Q6_K) && g.K % 256) return false;
        GemvSeg& sg = g.seg[i];
        sg.type = w.type;
        sg.w = w.d;
        sg.row_stride = w.stride;
        sg.w_bytes = w.expert_bytes * (size_t)w.n_exp;
        sg.rows = w.n_out;
        sg.y = ys[i];
        sg.ldy = lds[i];
        sg.bias = bs ? bs[i] : nullptr;
        sg.epi = epis[i];
        ph.tile0[i + 1] = ph.tile0[i] + (w.n_out + kTileRows - 1) / kTileRows;
        *slot_max = std::max(*slot_max, kTileRows * (int)group_bytes(w.type, blocks_per_group(w.type)));
        if (w.type == T_Q8_0) want32 = true; else wantk = true;
        *wbytes += (double)ggml_row_bytes(w.type, (uint64_t)w.n_in) * w.n_out;
    }
    for (int i = n; i < kMaxSeg; ++i) ph.tile0[i + 1] = ph.tile0[i];
    if (g.K % 8) return false;
    const int unit = swiglu ? 2 : 1;
    if (swiglu && (n != 2 || ws[0]->n_out != ws[1]->n_out)) return false;
    ph.n_units = (ph.tile0[n] + unit - 1) / unit;
    ph.G = G;
    ph.xk_bytes = wantk ? ximg_k_bytes(g.K) : 0;
    ph.x32_bytes = want32 ? ximg_32_bytes(g.K) : 0;
    ph.attn_layer = -1;
    const int tiles_max = (ph.n_units + grid - 1) / grid * unit;
    const int part = ((tiles_max * G * kTileRows * 4) + 127) / 128 * 128;
    *union_need = std::max(*union_need, ph.xk_bytes + ph.x32_bytes + part);
    *out = ph;
    return true;
}

bool Engine::step_ready() {
    if (step_state_) return step_state_ > 0;
    step_state_ = -1;
    const Config& c = cfg_;
    if (!env_int("FISH_PERSIST", 0)) { step_why_ = "off (FISH_PERSIST=1 enables it)"; return false; }
    if (c.n_experts > 0) { step_why_ = "mixture of experts"; return false; }
    if (tp_world_ > 1) { step_why_ = "tensor parallel"; return false; }
    if (c.qk_norm) { step_why_ = "q/k norm"; return false; }
    for (const DevLayer& L : layers_)
        if (L.bo) { step_why_ = "attention output bias"; return false; }
    if (c.post_norms || c.gelu || c.attn_softcap > 0.0f || c.final_softcap > 0.0f || c.sliding_window > 0 ||
        c.embd_scale != 1.0f) {
        step_why_ = "gemma2 layer form";
        return false;
    }
    const int G = c.n_head_kv > 0 ? c.n_head / c.n_head_kv : 0;
    if (c.head_dim != 128 || c.n_head % c.n_head_kv || !(G == 1 || G == 2 || G == 4 || G == 8) || c.rot_dim > 128 ||
        c.rot_dim % 2) {
        step_why_ = "attention shape";
        return false;
    }
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int grid = sms;   // one CTA per SM
    const int E = c.n_embd, Q = c.q_dim(), KV = c.kv_dim(), F = c.n_ff, D = c.head_dim;
    std::vector<StepPhase> phs;
    int slot = 0, uni = 0;
    double wb = 0.0;
    for (int li = 0; li < c.n_layers; ++li) {
        const DevLayer& L = layers_[li];
        StepPhase ph{};
        {
            const DevW* ws[3] = {&L.wq, &L.wk, &L.wv};
            float* ys[3] = {q_, k_, v_};
            const int lds[3] = {Q, KV, KV};
            const float* bs[3] = {L.bq, L.bk, L.bv};
            const int ep[3] = {EPI_STORE, EPI_STORE, EPI_STORE};
            const GemvPro pro{PRO_NORM, x_, E, nullptr, 0, L.attn_norm, c.eps};
            if (!step_job(ws, ys, lds, bs, ep, 3, pro, false, grid, &ph, &slot, &uni, &wb)) { step_why_ = "qkv weights"; return false; }
            phs.push_back(ph);
        }
        {
            const DevW* ws[1] = {&L.wo};
            float* ys[1] = {x_};
            const int lds[1] = {E};
            const int ep[1] = {EPI_ADD};
            const GemvPro pro{PRO_MERGE, att_part_, 0, nullptr, D, nullptr, 0.0f};   // src patched below
            if (!step_job(ws, ys, lds, nullptr, ep, 1, pro, false, grid, &ph, &slot, &uni, &wb)) { step_why_ = "o weights"; return false; }
            ph.attn_layer = li;
            phs.push_back(ph);
        }
        {
            const DevW* ws[2] = {&L.wg, &L.wu};
            float* ys[2] = {g_, u_};
            const int lds[2] = {F, F};
            const int ep[2] = {EPI_STORE, EPI_STORE};
            const GemvPro pro{PRO_NORM, x_, E, nullptr, 0, L.ffn_norm, c.eps};
            if (!step_job(ws, ys, lds, nullptr, ep, 2, pro, true, grid, &ph, &slot, &uni, &wb)) { step_why_ = "ffn weights"; return false; }
            phs.push_back(ph);
        }
        {
            const DevW* ws[1] = {&L.wd};
            float* ys[1] = {x_};
            const int lds[1] = {E};
            const int ep[1] = {EPI_ADD};
            const GemvPro pro{PRO_QUANT, g_, F, nullptr, 0, nullptr, 0.0f};
            if (!step_job(ws, ys, lds, nullptr, ep, 1, pro, false, grid, &ph, &slot, &uni, &wb)) { step_why_ = "down weights"; return false; }
            phs.push_back(ph);
        }
    }
    {
        StepPhase ph{};
        const DevW* ws[1] = {&out_w_};
        float* ys[1] = {logits_};
        const int lds[1] = {c.vocab};
        const int ep[1] = {EPI_STORE};
        const GemvPro pro{PRO_NORM, x_, E, nullptr, 0, out_norm_, c.eps};
        if (!step_job(ws, ys, lds, nullptr, ep, 1, pro, false, grid, &ph, &slot, &uni, &wb)) { step_why_ = "output weights"; return false; }
        ph.a.seg[0].amax = reinterpret_cast<unsigned long long*>(1);   // patched per step on the device
        phs.push_back(ph);
    }
    // attention scratch in the same union area: q [G][D+4], own k/v [2][D], warp partials [8][G][D+2]
    // (+ page bases of a chunk: 80 x 8 bytes)
    uni = std::max(uni, (int)(sizeof(float) * (G * (D + 4) + 2 * D + 8 * G * (D + 2)) + 80 * sizeof(size_t)));
    uni = (uni + 127) / 128 * 128;   // the ring after it starts 128-byte aligned
    int g2 = 0, S = 0;
    size_t smem = 0;
    const int rc = fbk_step_plan(G, kv_f16_ ? 1 : 0, slot, uni, &g2, &S, &smem);
    if (rc != 0 || g2 != grid) { step_why_ = "step kernel does not fit (plan " + std::to_string(rc) + ")"; cudaGetLastError(); return false; }
    // key chunks per kv head: at most 8 (the o projection's prologue merges
    // them), more only when a chunk would exceed ~1024 keys
    att_max_chunks_ = std::min(grid / c.n_head_kv, std::max(8, (c.n_ctx + 1023) / 1024));
    const size_t part_floats = (size_t)att_max_chunks_ * c.n_head * (D + 2);
    if (cudaMalloc(&att_part_, part_floats * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&step_ctl_, sizeof(StepCtl)) != cudaSuccess ||
        cudaMalloc(&step_keys_, 2 * sizeof(unsigned long long)) != cudaSuccess ||
        cudaMalloc(&step_ph_, phs.size() * sizeof(StepPhase)) != cudaSuccess) {
        step_why_ = "allocation";
        cudaGetLastError();
        return false;
    }
    for (StepPhase& ph : phs)
        if (ph.a.pro.mode == PRO_MERGE) ph.a.pro.src = att_part_;
    if (cudaMemcpy(step_ph_, phs.data(), phs.size() * sizeof(StepPhase), cudaMemcpyHostToDevice) != cudaSuccess) {
        step_why_ = "upload";
        return false;
    }
    (void)Q;
    step_nph_ = (int)phs.size();
    step_grid_ = grid;
    step_S_ = S;
    step_slot_ = slot;
    step_union_ = uni;
    step_smem_ = smem;
    step_wbytes_ = wb;
    step_state_ = 1;
    step_why_.clear();
    return true;
}

// n_steps greedy steps of sequence sid from ids_[0] at tok_pos_[0] (already
// uploaded); argmax of step i -> out_dev[i]; logits of the last step in logits_.
bool Engine::run_step(int sid, int n_steps, int32_t* out_dev, std::string* err) {
    const Config& c = cfg_;
    StepArgs A{};
    A.ph = step_ph_;
    A.n_ph = step_nph_;
    A.q = q_;
    A.k = k_;
    A.v = v_;
    A.att_part = att_part_;
    A.rcos = rope_cos_;
    A.rsin = rope_sin_;
    A.H = c.n_head;
    A.HKV = c.n_head_kv;
    A.D = c.head_dim;
    A.rot = c.rot_dim;
    A.neox = c.neox ? 1 : 0;
    A.scale = 1.0f / std::sqrt((float)c.head_dim);
    A.max_chunks = att_max_chunks_;
    A.kv = kv_view();
    A.sid = sid;
    A.emb_type = embd_.type;
    A.emb = embd_.d;
    A.E = c.n_embd;
    A.emb_rows = embd_.n_out;
    A.x = x_;
    A.ids = ids_;
    A.tok_pos = tok_pos_;
    A.out = out_dev;
    A.n_steps = n_steps;
    A.keys = step_keys_;
    A.ctl = step_ctl_;
    A.S = step_S_;
    A.slot_bytes = step_slot_;
    A.union_bytes = step_union_;
    A.trace = step_trace_;
    CK(cudaMemsetAsync(step_ctl_, 0, sizeof(StepCtl), stream_));
    CK(cudaMemsetAsync(step_keys_, 0, 2 * sizeof(unsigned long long), stream_));
    cudaEventRecord(pe0_, stream_);
    CK(fbk_step_decode(&A, step_grid_, step_smem_, stream_));
    cudaEventRecord(pe1_, stream_);
    StepCtl h{};
    CK(cudaMemcpyAsync(&h, step_ctl_, sizeof(StepCtl), cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    cudaEventElapsedTime(&last_step_ms_, pe0_, pe1_);
    if (h.err) {
        if (err)
            *err = "step kernel failed: code " + std::to_string(h.err) + " (CTA " + std::to_string(h.info[0]) + ", step " +
                   std::to_string(h.info[1]) + ", phase " + std::to_string(h.info[2]) + ", stage " +
                   std::to_string(h.info[3]) + ", slot " + std::to_string(h.info[4]) + ")";
        return false;
    }
    return true;
}

// ------------------------------------------------------------------ MoE

// The expert FFNs of a batched step (model.cpp:1523-1599) with the rows
// routed to each local expert gathered together: grouped rows e * T + j
// (k_moe_group / k_moe_gather), gate/up and down over each expert's rows, so
// its weights stream once per step, then the weighted combine through
// grp_pos. Eager calls read the counts back and give each expert one call of
// exactly its rows (the tensor-core GEMM from 16 rows); inside a graph
// capture the counts stay on the device and every (expert, 4-row chunk)
// launch reads its expert id (-1: no rows, no weight bytes fetched). Rows are
// computed by the same kernels in either form, so the results are the same
// bits as the one-row-per-call path.
bool Engine::moe_grouped(const DevLayer& L, const ActQ& a, int T, const int32_t* esel, int nel, float* out,
                         std::string* err) {
    const Config& c = cfg_;
    const int K = c.n_experts_per_tok, F = c.n_ff_exp, E = c.n_embd;
    // slots of S rows (the streamed GEMV's token count: 8, or 4 for small
    // batches), packed per expert; in a captured graph every slot is a launch
    // whose expert is read on the device (idle slots exit at once)
    const int S = T > 4 ? 8 : 4;
    const int nslot = fbk_moe_slots(T, K, nel, S), rows = S * nslot;
    if (rows > grp_rows_ || nslot > nel * (kMaxBatch / 4)) { if (err) *err = "MoE grouping: batch too large"; return false; }
    CKP(PC_OTHER, 0, fbk_moe_group(esel, T, K, nel, grp_src_, grp_pos_, grp_count_, chunk_exp_, nslot, S, stream_));
    ActQ src = a, ga = gact_, gf = gact_;
    src.K = E;
    ga.K = E;
    gf.K = F;
    CKP(PC_OTHER, 0, fbk_moe_gather(&src, &ga, grp_src_, K, rows, E, stream_));
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    CK(cudaStreamIsCapturing(stream_, &cs));
    const bool exact = cs == cudaStreamCaptureStatusNone;
    std::vector<int32_t> cnt((size_t)nel, 0), row0((size_t)nel, 0);
    if (exact) {
        CK(cudaMemcpyAsync(cnt.data(), grp_count_, sizeof(int32_t) * nel, cudaMemcpyDeviceToHost, stream_));
        CK(cudaStreamSynchronize(stream_));
        for (int e = 1; e < nel; ++e) row0[e] = row0[e - 1] + S * ((cnt[e - 1] + S - 1) / S);   // the kernel's packing
    }
    const int nts = std::min(S, T);   // an expert has at most T rows: a slot's rows lie in its first nts
    auto view = [](const DevW& w, int e) {
        DevW v = w;
        v.d = w.d + (size_t)e * w.expert_bytes;
        v.n_exp = 1;
        return v;
    };
    if (exact) {
        for (int e = 0; e < nel; ++e) {
            if (!cnt[e]) continue;
            const int r0 = row0[e];
            const DevW gw = view(L.gate_exps, e), uw = view(L.up_exps, e);
            const DevW* ws[2] = {&gw, &uw};
            float* ys[2] = {gg_ + (size_t)r0 * F, gu_ + (size_t)r0 * F};
            const int lds[2] = {F, F};
            if (!gemv_group(ws, ys, lds, nullptr, 2, act_row(ga, r0, E), cnt[e], EPI_STORE, err)) return false;
        }
    } else {
        for (int sl = 0; sl < nslot; ++sl) {
            const int rr = S * sl;
            const DevW* ws[2] = {&L.gate_exps, &L.up_exps};
            float* ys[2] = {gg_ + (size_t)rr * F, gu_ + (size_t)rr * F};
            const int lds[2] = {F, F};
            if (!gemv_group(ws, ys, lds, nullptr, 2, act_row(ga, rr, E), nts, EPI_STORE, err, nullptr, false,
                            chunk_exp_ + sl))
                return false;
        }
    }
    CKP(PC_NORMQ, 0, fbk_silu_mul_quant(gg_, F, gu_, F, rows, F, probe_ ? probe_h_ : nullptr, F, &gf, want32_f_,
                                        wantk_f_, stream_));
    if (probe_ && !probe_grouped(3, gf, rows, T * K, F, err)) return false;
    if (exact) {
        for (int e = 0; e < nel; ++e) {
            if (!cnt[e]) continue;
            const int r0 = row0[e];
            const DevW dw = view(L.down_exps, e);
            if (!gemv(dw, act_row(gf, r0, F), cnt[e], geo_ + (size_t)r0 * E, E, nullptr, EPI_STORE, nullptr, 0, nullptr,
                      err))
                return false;
        }
    } else {
        for (int sl = 0; sl < nslot; ++sl) {
            const int rr = S * sl;
            if (!gemv(L.down_exps, act_row(gf, rr, F), nts, geo_ + (size_t)rr * E, E, nullptr, EPI_STORE, nullptr, 0,
                      chunk_exp_ + sl, err))
                return false;
        }
    }
    CKP(PC_OTHER, 0, fbk_moe_combine_grouped(out, E, geo_, grp_pos_, wsel_, T, K, E, stream_));
    return true;
}

// ------------------------------------------------------------------ forward

bool Engine::run_layers(int T, int max_ctx, bool distinct, std::string* err, int l0, int l1) {
    const Config& c = cfg_;
    const int E = c.n_embd, Q = c.q_dim(), KV = c.kv_dim(), H = c.n_head, HKV = c.n_head_kv, D = c.head_dim;
    const float scale = 1.0f / std::sqrt((float)D);
    KvView kv = kv_view();
    kv.softcap = c.attn_softcap;
    ActQ a = act_;
    if (l1 < 0) l1 = c.n_layers;
    for (int li = l0; li < l1; ++li) {
        const DevLayer& L = layers_[li];
        kv.window = (c.sliding_window > 0 && li % 2 == 0) ? c.sliding_window : 0;   // gemma2: even layers
        a.K = E;
        {
            const DevW* ws[3] = {&L.wq, &L.wk, &L.wv};
            float* ys[3] = {q_, k_, v_};
            const int lds[3] = {Q, KV, KV};
            const float* bs[3] = {L.bq, L.bk, L.bv};
            if (probe_ && !probe_float(0, x_, T, E, err)) return false;
            if (fusable(ws, 3, T)) {
                const GemvPro pro{PRO_NORM, x_, E, nullptr, 0, L.attn_norm, c.eps};
                if (probe_) dump_img_ = probe_img_;
                const bool ok = gemv_group(ws, ys, lds, bs, 3, a, T, EPI_STORE, err, &pro);
                dump_img_ = nullptr;
                if (!ok || (probe_ && !probe_image(0, T, E, err))) return false;
            } else {
                CKP(PC_NORMQ, 0, fbk_rmsnorm_quant(x_, E, L.attn_norm, c.eps, T, E, xb_, E, &a, want32_e_, wantk_e_, stream_));
                if (probe_ && !probe_planes(0, a, T, E, want32_e_, wantk_e_, err)) return false;
                if (!gemv_group(ws, ys, lds, bs, 3, a, T, EPI_STORE, err)) return false;
            }
        }
        if (L.q_norm && L.k_norm) {
            CKP(PC_OTHER, 0, fbk_head_rmsnorm(q_, Q, T, H, D, L.q_norm, c.eps, stream_));
            CKP(PC_OTHER, 0, fbk_head_rmsnorm(k_, KV, T, HKV, D, L.k_norm, c.eps, stream_));
        }
        if (distinct && !no_fuse_) {
            CKP(PC_ATTN, 0, fbk_attention_decode(q_, Q, k_, v_, KV, T, H, HKV, D, scale, c.rot_dim, c.neox ? 1 : 0,
                                                 rope_cos_, rope_sin_, kv, li, attn_, Q, dec_part_, dec_part_floats_,
                                                 pre_blocks_, pre_state_, pre_state_floats_, stream_));
        } else {
        CKP(PC_ROPE, 0, fbk_rope_append(q_, Q, k_, v_, KV, T, H, HKV, D, c.rot_dim, c.neox ? 1 : 0, rope_cos_,
                                        rope_sin_, kv, li, stream_));
        // one sequence (a prefill), fp16 cache: the tensor-core kernel over all T tokens
        if (!distinct && kv.f16 && !prefill_simt_) {
            CKP(PC_ATTN, 0, fbk_attention_prefill(q_, Q, T, H, HKV, D, scale, kv, li, attn_, Q, stream_));
        } else
        for (int t0 = 0; t0 < T; t0 += att_chunk_) {
            const int nt = std::min(att_chunk_, T - t0);
            KvView kvc = kv;
            kvc.tok_seq = tok_seq_ + t0;
            kvc.tok_pos = tok_pos_ + t0;
            CKP(PC_ATTN, 0, fbk_attention(q_ + (size_t)t0 * Q, Q, nt, H, HKV, D, scale, kvc, li, attn_ + (size_t)t0 * Q, Q,
                                          att_scratch_, att_scratch_floats_, max_ctx, stream_));
        }
        }
        a.K = Q;
        {
            // tensor parallelism: this rank's heads give a partial sum of o,
            // all-reduced before the residual add
            // gemma2: o rows into tp_tmp_, then x += post_norm(o)
            const bool tp = tp_world_ > 1, post = L.post_attn_norm != nullptr;
            float* oy = tp || post ? tp_tmp_ : x_;
            const int oepi = tp || post ? EPI_STORE : EPI_ADD;
            const float* bo = tp_rank_ == 0 ? L.bo : nullptr;   // partial sums of other ranks carry none
            const DevW* wo[1] = {&L.wo};
            if (probe_ && !probe_float(1, attn_, T, Q, err)) return false;
            if (fusable(wo, 1, T)) {
                const GemvPro pro{PRO_QUANT, attn_, Q, nullptr, 0, nullptr, 0.0f};
                if (probe_) dump_img_ = probe_img_;
                const bool ok = gemv(L.wo, a, T, oy, E, bo, oepi, nullptr, 0, nullptr, err, &pro);
                dump_img_ = nullptr;
                if (!ok || (probe_ && !probe_image(1, T, Q, err))) return false;
            } else {
                CKP(PC_NORMQ, 0, fbk_quantize_rows(attn_, Q, T, Q, &a, want32_q_, wantk_q_, stream_));
                if (probe_ && !probe_planes(1, a, T, Q, want32_q_, wantk_q_, err)) return false;
                if (!gemv(L.wo, a, T, oy, E, bo, oepi, nullptr, 0, nullptr, err)) return false;
            }
            if (tp && !tp_reduce_add(T, err)) return false;
            if (post) CKP(PC_NORMQ, 0, fbk_rmsnorm_add(x_, E, tp_tmp_, E, L.post_attn_norm, c.eps, T, E, stream_));
        }
        a.K = E;
        const DevW* wgu[2] = {&L.wg, &L.wu};
        const bool fuse_ffn = c.n_experts == 0 && fusable(wgu, 2, T);
        if (probe_ && !probe_float(2, x_, T, E, err)) return false;
        if (!fuse_ffn) {
            CKP(PC_NORMQ, 0, fbk_rmsnorm_quant(x_, E, L.ffn_norm, c.eps, T, E, xb_, E, &a, want32_e_, wantk_e_, stream_));
            if (probe_ && !probe_planes(2, a, T, E, want32_e_, wantk_e_, err)) return false;
        }
        if (c.n_experts > 0) {
            const int NE = c.n_experts, K = c.n_experts_per_tok, F = c.n_ff_exp;
            if (L.gate_inp.type == T_F32) {
                CKP(PC_OTHER, 0, fbk_router_f32(L.gate_inp.d, L.gate_inp.stride, xb_, E, T, E, NE, router_, NE, stream_));
            } else if (!gemv(L.gate_inp, a, T, router_, NE, nullptr, EPI_STORE, xb_, E, nullptr, err)) {
                return false;
            }
            CKP(PC_OTHER, 0, fbk_moe_route(router_, T, NE, K, c.expert_weights_norm ? 1 : 0, sel_, wsel_, stream_));
            // expert parallelism: experts of other ranks map to -1 (zero rows)
            const bool ep = tp_world_ > 1;
            const int32_t* esel = ep ? sel_loc_ : sel_;
            if (ep) CKP(PC_OTHER, 0, fbk_moe_localize(sel_, T * K, ep_e0_, ep_n_, sel_loc_, stream_));
            if (T > 1) {   // batched step: tokens grouped per expert
                float* out = x_;
                if (ep) {
                    CK(cudaMemsetAsync(tp_tmp_, 0, sizeof(float) * (size_t)T * E, stream_));
                    out = tp_tmp_;
                }
                if (!moe_grouped(L, a, T, esel, ep ? ep_n_ : NE, out, err)) return false;
                if (ep && !tp_reduce_add(T, err)) return false;
                if (L.shexp_gate.ok() && !shared_expert(L, a, T, err)) return false;
                continue;
            }
            for (int t = 0; t < T; ++t) {
                const ActQ ar = act_row(a, t, E);
                for (int k = 0; k < K; ++k) {
                    const int r = t * K + k;
                    if (!gemv(L.gate_exps, ar, 1, g_ + (size_t)r * F, F, nullptr, EPI_STORE, nullptr, 0, esel + r, err) ||
                        !gemv(L.up_exps, ar, 1, u_ + (size_t)r * F, F, nullptr, EPI_STORE, nullptr, 0, esel + r, err))
                        return false;
                }
            }
            a.K = F;
            CKP(PC_NORMQ, 0, fbk_silu_mul_quant(g_, F, u_, F, T * K, F, probe_ ? probe_h_ : nullptr, F, &a, want32_f_,
                                                wantk_f_, stream_));
            if (probe_ && (!probe_float(3, probe_h_, T * K, F, err) ||
                           !probe_planes(3, a, T * K, F, want32_f_, wantk_f_, err)))
                return false;
            for (int r = 0; r < T * K; ++r) {
                const ActQ ar = act_row(a, r, F);
                if (!gemv(L.down_exps, ar, 1, eo_ + (size_t)r * E, E, nullptr, EPI_STORE, nullptr, 0, esel + r, err))
                    return false;
            }
            if (ep) {   // this rank's weighted experts, summed over the ranks, then the residual add
                CK(cudaMemsetAsync(tp_tmp_, 0, sizeof(float) * (size_t)T * E, stream_));
                CKP(PC_OTHER, 0, fbk_moe_combine(tp_tmp_, E, eo_, wsel_, T, K, E, stream_));
                if (!tp_reduce_add(T, err)) return false;
            } else {
                CKP(PC_OTHER, 0, fbk_moe_combine(x_, E, eo_, wsel_, T, K, E, stream_));
            }
            if (L.shexp_gate.ok() && !shared_expert(L, a, T, err)) return false;
        } else {
            const int F = c.n_ff;
            {
                float* ys[2] = {g_, u_};
                const int lds[2] = {F, F};
                if (fuse_ffn) {
                    // SwiGLU in the epilogue; GELU (gemma2) in its own kernel below
                    const GemvPro pro{PRO_NORM, x_, E, nullptr, 0, L.ffn_norm, c.eps};
                    if (probe_) dump_img_ = probe_img_;
                    const bool ok = gemv_group(wgu, ys, lds, nullptr, 2, a, T, EPI_STORE, err, &pro, !c.gelu);
                    dump_img_ = nullptr;
                    if (!ok || (probe_ && !probe_image(2, T, E, err))) return false;
                } else {
                    if (!gemv_group(wgu, ys, lds, nullptr, 2, a, T, EPI_STORE, err)) return false;
                }
            }
            a.K = F;
            const bool tp = tp_world_ > 1, post = L.post_ffn_norm != nullptr;
            float* dy = tp || post ? tp_tmp_ : x_;
            const int depi = tp || post ? EPI_STORE : EPI_ADD;
            const DevW* wd[1] = {&L.wd};
            if (c.gelu) {   // h = gelu(g) * u, quantised, then the down projection
                CKP(PC_NORMQ, 0, fbk_act_mul_quant(g_, F, u_, F, T, F, probe_ ? probe_h_ : nullptr, F, &a, want32_f_,
                                                   wantk_f_, 1, stream_));
                if (probe_ && (!probe_float(3, probe_h_, T, F, err) ||
                               !probe_planes(3, a, T, F, want32_f_, wantk_f_, err)))
                    return false;
                if (!gemv(L.wd, a, T, dy, E, nullptr, depi, nullptr, 0, nullptr, err)) return false;
            } else if (fuse_ffn && fusable(wd, 1, T)) {   // h = silu(g) * u already in g_
                const GemvPro pro{PRO_QUANT, g_, F, nullptr, 0, nullptr, 0.0f};
                if (probe_ && !probe_float(3, g_, T, F, err)) return false;
                if (probe_) dump_img_ = probe_img_;
                const bool ok = gemv(L.wd, a, T, dy, E, nullptr, depi, nullptr, 0, nullptr, err, &pro);
                dump_img_ = nullptr;
                if (!ok || (probe_ && !probe_image(3, T, F, err))) return false;
            } else if (fusable(wd, 1, T)) {
                const GemvPro pro{PRO_SILU, g_, F, u_, F, nullptr, 0.0f};
                if (probe_ && (!probe_float(4, g_, T, F, err) || !probe_float(5, u_, T, F, err))) return false;
                if (probe_) dump_img_ = probe_img_;
                const bool ok = gemv(L.wd, a, T, dy, E, nullptr, depi, nullptr, 0, nullptr, err, &pro);
                dump_img_ = nullptr;
                if (!ok || (probe_ && !probe_image(3, T, F, err))) return false;
            } else {
                CKP(PC_NORMQ, 0, fbk_silu_mul_quant(g_, F, u_, F, T, F, probe_ ? probe_h_ : nullptr, F, &a, want32_f_,
                                                    wantk_f_, stream_));
                if (probe_ && (!probe_float(3, probe_h_, T, F, err) ||
                               !probe_planes(3, a, T, F, want32_f_, wantk_f_, err)))
                    return false;
                if (!gemv(L.wd, a, T, dy, E, nullptr, depi, nullptr, 0, nullptr, err)) return false;
            }
            if (tp && !tp_reduce_add(T, err)) return false;
            if (post) CKP(PC_NORMQ, 0, fbk_rmsnorm_add(x_, E, tp_tmp_, E, L.post_ffn_norm, c.eps, T, E, stream_));
        }
    }
    return true;
}

// The shared expert of a qwen2moe layer (src/model.cpp:1582-1599): every
// token's normed input (xb_, quantised again: the routed experts reused the
// activation planes) through gate/up, SwiGLU and down, scaled by the
// sigmoid of its own one-row gate when the layer has one, added to x. Every
// rank of an expert-parallel group holds it whole and adds it after the
// all-reduce of the routed experts.
bool Engine::shared_expert(const DevLayer& L, ActQ a, int T, std::string* err) {
    const Config& c = cfg_;
    const int E = c.n_embd, Fs = L.shexp_gate.n_out;
    a.K = E;
    CKP(PC_NORMQ, 0, fbk_quantize_rows(xb_, E, T, E, &a, want32_e_, wantk_e_, stream_));
    const DevW* gu[2] = {&L.shexp_gate, &L.shexp_up};
    float* ys[2] = {g_, u_};
    const int lds[2] = {Fs, Fs};
    if (!gemv_group(gu, ys, lds, nullptr, 2, a, T, EPI_STORE, err)) return false;
    // the gate before the planes are reused: one logit per token into router_
    const bool gated = L.shexp_gate_inp.ok();
    if (gated) {
        if (L.shexp_gate_inp.type == T_F32) {
            CKP(PC_OTHER, 0, fbk_router_f32(L.shexp_gate_inp.d, L.shexp_gate_inp.stride, xb_, E, T, E, 1, router_, 1,
                                            stream_));
        } else if (!gemv(L.shexp_gate_inp, a, T, router_, 1, nullptr, EPI_STORE, xb_, E, nullptr, err)) {
            return false;
        }
    }
    CKP(PC_OTHER, 0, fbk_sigmoid(gated ? router_ : nullptr, router_, T, stream_));
    a.K = Fs;
    CKP(PC_NORMQ, 0, fbk_silu_mul_quant(g_, Fs, u_, Fs, T, Fs, nullptr, Fs, &a, want32_f_, wantk_f_, stream_));
    if (!gemv(L.shexp_down, a, T, eo_, E, nullptr, EPI_STORE, nullptr, 0, nullptr, err)) return false;
    CKP(PC_OTHER, 0, fbk_moe_combine(x_, E, eo_, router_, T, 1, E, stream_));
    return true;
}

// ------------------------------------------------------------------ layer probe

static_assert(kXChunkBytes == kXChunk, "probe image parsing follows the streamed GEMV's image layout");

bool Engine::probe_float(int idx, const float* dev, int rows, int K, std::string* err) {
    LayerProbe& p = *probe_;
    p.f[idx].resize((size_t)rows * K);
    p.rows[idx] = rows;
    p.K[idx] = K;
    CK(cudaMemcpyAsync(p.f[idx].data(), dev, sizeof(float) * (size_t)rows * K, cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    return true;
}

namespace {
// Activation records in the reference's byte layout (quant.h:58-70).
void put_k_record(uint8_t* r, float d, const int16_t* bsums, const int8_t* qs) {
    std::memcpy(r, &d, 4);
    std::memcpy(r + 4, bsums, 16);
    std::memcpy(r + 20, qs, 256);
}
void put_32_record(uint8_t* r, float d, const int8_t* qs) {
    int32_t sum = 0;
    for (int i = 0; i < 32; ++i) sum += qs[i];
    std::memcpy(r, &d, 4);
    std::memcpy(r + 4, &sum, 4);
    std::memcpy(r + 8, qs, 32);
}
}  // namespace

bool Engine::probe_planes(int stage, const ActQ& a, int rows, int K, bool want32, bool wantk, std::string* err) {
    LayerProbe& p = *probe_;
    CK(cudaStreamSynchronize(stream_));
    p.has_k[stage] = wantk && K % 256 == 0;
    p.has_32[stage] = want32 && K % 32 == 0;
    p.rows[stage] = rows;
    p.K[stage] = K;
    if (p.has_k[stage]) {
        const int nb = K / 256;
        std::vector<int8_t> q((size_t)rows * a.ld);
        std::vector<float> d((size_t)rows * nb);
        std::vector<int16_t> bs((size_t)rows * (K / 32));
        CK(cudaMemcpy(q.data(), a.qk, q.size(), cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(d.data(), a.dk, sizeof(float) * d.size(), cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(bs.data(), a.bsk, sizeof(int16_t) * bs.size(), cudaMemcpyDeviceToHost));
        p.rk[stage].resize((size_t)rows * nb * 276);
        for (int t = 0; t < rows; ++t)
            for (int c = 0; c < nb; ++c)
                put_k_record(&p.rk[stage][((size_t)t * nb + c) * 276], d[(size_t)t * nb + c],
                             &bs[(size_t)t * (K / 32) + 8 * c], &q[(size_t)t * a.ld + 256 * c]);
    }
    if (p.has_32[stage]) {
        const int nb = K / 32;
        std::vector<int8_t> q((size_t)rows * a.ld);
        std::vector<float> d((size_t)rows * nb);
        CK(cudaMemcpy(q.data(), a.q32, q.size(), cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(d.data(), a.d32, sizeof(float) * d.size(), cudaMemcpyDeviceToHost));
        p.r32[stage].resize((size_t)rows * nb * 40);
        for (int t = 0; t < rows; ++t)
            for (int b = 0; b < nb; ++b)
                put_32_record(&p.r32[stage][((size_t)t * nb + b) * 40], d[(size_t)t * nb + b], &q[(size_t)t * a.ld + 32 * b]);
    }
    return true;
}

bool Engine::probe_image(int stage, int rows, int K, std::string* err) {
    LayerProbe& p = *probe_;
    CK(cudaStreamSynchronize(stream_));
    p.rows[stage] = rows;
    p.K[stage] = K;
    const int nbk = K / 256, nb32 = K / 32;
    int done = 0;
    std::vector<uint8_t> buf;
    for (int ch = 0; done < rows; ++ch) {
        if ((size_t)(ch + 1) * kProbeChunkBytes > probe_img_bytes_) { if (err) *err = "probe: too many chunks"; return false; }
        int hdr[4] = {0, 0, 0, 0};
        const uint8_t* src = probe_img_ + (size_t)ch * kProbeChunkBytes;
        CK(cudaMemcpy(hdr, src, sizeof(hdr), cudaMemcpyDeviceToHost));
        const int xk = hdr[0], x32 = hdr[1], tc = hdr[2], n256 = hdr[3];
        if (tc <= 0 || done + tc > rows || n256 != (K + 255) / 256 ||
            16 + (size_t)tc * (xk + x32) > kProbeChunkBytes) {
            if (err) *err = "probe: bad activation image header";
            return false;
        }
        buf.resize((size_t)tc * (xk + x32));
        CK(cudaMemcpy(buf.data(), src + 16, buf.size(), cudaMemcpyDeviceToHost));
        p.has_k[stage] = xk > 0 && K % 256 == 0;
        p.has_32[stage] = x32 > 0 && K % 32 == 0;
        if (p.has_k[stage]) {
            p.rk[stage].resize((size_t)rows * nbk * 276);
            for (int t = 0; t < tc; ++t) {
                const uint8_t* b = buf.data() + (size_t)t * xk;
                for (int c = 0; c < nbk; ++c) {
                    float d;
                    std::memcpy(&d, b + (size_t)n256 * (kXChunkBytes + 48) + 4 * c, 4);
                    put_k_record(&p.rk[stage][((size_t)(done + t) * nbk + c) * 276], d,
                                 reinterpret_cast<const int16_t*>(b + (size_t)n256 * kXChunkBytes + 16 * c),
                                 reinterpret_cast<const int8_t*>(b + (size_t)c * kXChunkBytes));
                }
            }
        }
        if (p.has_32[stage]) {
            p.r32[stage].resize((size_t)rows * nb32 * 40);
            for (int t = 0; t < tc; ++t) {
                const uint8_t* b = buf.data() + (size_t)tc * xk + (size_t)t * x32;
                for (int blk = 0; blk < nb32; ++blk) {
                    const int c = blk / 8, j = blk % 8;
                    float d;
                    std::memcpy(&d, b + (size_t)n256 * kXChunkBytes + 32 * c + 4 * j, 4);
                    put_32_record(&p.r32[stage][((size_t)(done + t) * nb32 + blk) * 40], d,
                                  reinterpret_cast<const int8_t*>(b + (size_t)c * kXChunkBytes + 32 * j));
                }
            }
        }
        done += tc;
    }
    return true;
}

// Stage records of grouped rows (expert-major) back in routed-row order
// r = t K + k, as the one-row-per-call path records them.
bool Engine::probe_grouped(int stage, const ActQ& a, int grouped_rows, int rows, int K, std::string* err) {
    LayerProbe& p = *probe_;
    if (!probe_float(stage, probe_h_, grouped_rows, K, err)) return false;
    if (!probe_planes(stage, a, grouped_rows, K, a.q32 && want32_f_, a.qk && wantk_f_, err)) return false;
    std::vector<int32_t> pos((size_t)rows);
    CK(cudaMemcpy(pos.data(), grp_pos_, sizeof(int32_t) * rows, cudaMemcpyDeviceToHost));
    auto regroup = [&](auto& v, size_t per_row) {
        if (v.empty()) return;
        std::remove_reference_t<decltype(v)> o(per_row * (size_t)rows);
        for (int r = 0; r < rows; ++r)
            if (pos[r] >= 0) std::copy_n(v.begin() + (size_t)pos[r] * per_row, per_row, o.begin() + (size_t)r * per_row);
        v.swap(o);
    };
    regroup(p.f[stage], (size_t)K);
    regroup(p.rk[stage], (size_t)(K / 256) * 276);
    regroup(p.r32[stage], (size_t)(K / 32) * 40);
    p.rows[stage] = rows;
    return true;
}

bool Engine::layer_probe(int li, int pos0, const float* x_in, int T, float* x_out, LayerProbe* p, std::string* err) {
    const Config& c = cfg_;
    if (li < 0 || li >= c.n_layers || T <= 0 || T > kMaxBatch || pos0 < 0 || !x_in || !x_out || !p) {
        if (err) *err = "probe: bad argument";
        return false;
    }
    if (tp_world_ > 1) { if (err) *err = "probe: single-GPU engines only"; return false; }
    Seq& s = seqs_[0];
    if (pos0 > s.len) { if (err) *err = "probe: pos0 beyond the sequence"; return false; }
    if (!ensure_pages(0, pos0 + T, err)) return false;
    const size_t img_need = (size_t)((T + 3) / 4 + 1) * kProbeChunkBytes;
    if (probe_img_bytes_ < img_need) {
        if (probe_img_) cudaFree(probe_img_);
        probe_img_ = nullptr;
        probe_img_bytes_ = 0;
        CK(cudaMalloc(&probe_img_, img_need));
        probe_img_bytes_ = img_need;
    }
    const int F = c.n_experts > 0 ? c.n_ff_exp : c.n_ff;
    const size_t h_need = (size_t)std::max(kMaxBatch * std::max(1, c.n_experts_per_tok), grp_rows_) * F;
    if (!probe_h_) CK(cudaMalloc(&probe_h_, sizeof(float) * h_need));
    std::vector<int32_t> ids(T, 0);
    std::vector<int> sids(T, 0), pos(T);
    for (int t = 0; t < T; ++t) pos[t] = pos0 + t;
    if (!upload_tokens(ids.data(), sids.data(), pos.data(), T, err)) return false;
    CK(cudaMemcpyAsync(x_, x_in, sizeof(float) * (size_t)T * c.n_embd, cudaMemcpyHostToDevice, stream_));
    *p = LayerProbe{};
    probe_ = p;
    const bool ok = run_layers(T, pos0 + T, T == 1, err, li, li + 1);
    probe_ = nullptr;
    dump_img_ = nullptr;
    if (!ok) return false;
    CK(cudaMemcpyAsync(x_out, x_, sizeof(float) * (size_t)T * c.n_embd, cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    s.len = std::max(s.len, pos0 + T);
    return true;
}

// Final norm + output projection for x rows [row0, row0+n) into logits rows 0..n-1.
bool Engine::run_head(int row0, int n, float* logits_dev, std::string* err, unsigned long long* keys, bool* keyed,
                      bool need_logits) {
    if (keyed) *keyed = false;
    const Config& c = cfg_;
    const int E = c.n_embd;
    ActQ a = act_;
    a.K = E;
    const DevW* wo[1] = {&out_w_};
    // tensor parallelism: this rank's vocab rows into its slice of
    // tp_logits_; argmax keys (global row ids) reduced by max over the ranks;
    // logits gathered when the caller needs them
    const bool tp = tp_world_ > 1;
    float* ydst = tp ? tp_logits_ + (size_t)tp_rank_ * n * c.out_rows : logits_dev;
    const int ldy = tp ? c.out_rows : c.vocab;
    bool k = false;
    // gemma2's final soft cap comes before any argmax: the GEMV's argmax keys
    // would see the uncapped logits
    if (c.final_softcap > 0.0f) keys = nullptr;
    if (fusable(wo, 1, n)) {
        const GemvPro pro{PRO_NORM, x_ + (size_t)row0 * E, E, nullptr, 0, out_norm_, c.eps};
        k = keys != nullptr;
        if (!gemv(out_w_, a, n, ydst, ldy, nullptr, EPI_STORE, nullptr, 0, nullptr, err, &pro, keys)) return false;
    } else {
        CKP(PC_NORMQ, 0, fbk_rmsnorm_quant(x_ + (size_t)row0 * E, E, out_norm_, c.eps, n, E, xb_, E, &a, want32_e_,
                                           wantk_e_, stream_));
        if (!gemv(out_w_, a, n, ydst, ldy, nullptr, EPI_STORE, xb_, E, nullptr, err)) return false;
    }
    if (c.final_softcap > 0.0f) CKP(PC_OTHER, 0, fbk_softcap(ydst, c.out_rows, n, ldy, c.final_softcap, stream_));
    if (keyed) *keyed = k;
    if (tp) {
        if (k && nccl_api(err)->all_reduce(keys, keys, (size_t)n, ncclUint64, ncclMax, (ncclComm_t)nccl_, stream_) !=
                     ncclSuccess) {
            if (err) *err = "NCCL all-reduce of argmax keys failed";
            return false;
        }
        if ((need_logits || !k) && !tp_gather_logits(n, logits_dev, err)) return false;
    }
    return true;
}

bool Engine::tp_reduce_add(int T, std::string* err) {
    const size_t n = (size_t)T * cfg_.n_embd;
    if (nccl_api(err)->all_reduce(tp_tmp_, tp_tmp_, n, ncclFloat, ncclSum, (ncclComm_t)nccl_, stream_) != ncclSuccess) {
        if (err) *err = "NCCL all-reduce failed";
        return false;
    }
    CKP(PC_OTHER, 0, fbk_add(x_, tp_tmp_, n, stream_));
    return true;
}

// tp_logits_ holds [world][rows][out_rows] after the gather; logits rows are
// [rows][vocab] with rank r's slice at columns r * out_rows.
bool Engine::tp_gather_logits(int rows, float* logits_dev, std::string* err) {
    const int R = cfg_.out_rows;
    const size_t cnt = (size_t)rows * R;
    if (nccl_api(err)->all_gather(tp_logits_ + (size_t)tp_rank_ * cnt, tp_logits_, cnt, ncclFloat, (ncclComm_t)nccl_,
                                  stream_) != ncclSuccess) {
        if (err) *err = "NCCL all-gather of logits failed";
        return false;
    }
    for (int r = 0; r < tp_world_; ++r)
        CK(cudaMemcpy2DAsync(logits_dev + (size_t)r * R, sizeof(float) * cfg_.vocab, tp_logits_ + (size_t)r * cnt,
                             sizeof(float) * R, sizeof(float) * R, rows, cudaMemcpyDeviceToDevice, stream_));
    return true;
}

// NCCL, loaded when tensor parallelism is first asked for (no link-time
// dependency: a process that also loads another NCCL build, e.g. a Python
// framework's, keeps whichever was loaded first). An NCCL already in the
// process is used as is.
const NcclApi* nccl_api(std::string* err) {
    static NcclApi api;
    static bool tried = false;
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    if (tried) {
        if (!api.ok && err) *err = "NCCL is not available";
        return api.ok ? &api : nullptr;
    }
    tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW);
    if (!h) { if (err) *err = "NCCL (libnccl.so.2) not found"; return nullptr; }
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce && api.all_gather &&
             api.error_string;
    if (!api.ok && err) *err = "NCCL library lacks an expected function";
    return api.ok ? &api : nullptr;
}

bool Engine::set_tp(int rank, int world, const void* id, std::string* err) {
    if (gguf_) { if (err) *err = "tensor parallelism must be set up before the model is loaded"; return false; }
    if (world < 1 || rank < 0 || rank >= world || (world > 1 && !id)) { if (err) *err = "bad tensor-parallel rank/world"; return false; }
    if (world == 1) return true;
    const NcclApi* nc = nccl_api(err);
    if (!nc) return false;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclComm_t comm = nullptr;
    const ncclResult_t r = nc->comm_init_rank(&comm, world, uid, rank);
    if (r != ncclSuccess) {
        if (err) *err = std::string("ncclCommInitRank: ") + nc->error_string(r);
        return false;
    }
    nccl_ = comm;
    tp_rank_ = rank;
    tp_world_ = world;
    return true;
}

bool Engine::upload_tokens(const int32_t* ids, const int* sids, const int* pos, int T, std::string* err) {
    int32_t* hp = h_pinned_;
    // the previous step's copies from this pinned buffer must have finished
    CK(cudaStreamSynchronize(stream_));
    for (int t = 0; t < T; ++t) {
        hp[t] = ids[t];
        hp[kMaxBatch + t] = sids[t];
        hp[2 * kMaxBatch + t] = pos[t];
    }
    CK(cudaMemcpyAsync(ids_, hp, sizeof(int32_t) * T, cudaMemcpyHostToDevice, stream_));
    CK(cudaMemcpyAsync(tok_seq_, hp + kMaxBatch, sizeof(int32_t) * T, cudaMemcpyHostToDevice, stream_));
    CK(cudaMemcpyAsync(tok_pos_, hp + 2 * kMaxBatch, sizeof(int32_t) * T, cudaMemcpyHostToDevice, stream_));
    return true;
}

bool Engine::embed_rows(int T, std::string* err) {
    const Config& c = cfg_;
    CKP(PC_OTHER, 0, fbk_embed(embd_.type, embd_.d, c.n_embd, embd_.n_out, ids_, T, x_, c.n_embd, fbk_gemv_error_flag(), stream_));
    if (c.embd_scale != 1.0f) CKP(PC_OTHER, 0, fbk_scale(x_, (size_t)T * c.n_embd, c.embd_scale, stream_));
    return true;
}

bool Engine::capture_graph(int key, std::string* err) {
    const int T = key == 0 ? 1 : key;
    cudaGraph_t graph = nullptr;
    CK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    std::string e2;
    bool ok = embed_rows(T, &e2);
    ok = ok && run_layers(T, cfg_.n_ctx, true, &e2);
    bool keyed = false;
    ok = ok && run_head(0, T, logits_, &e2, amax_keys_, &keyed, key != 0);
    if (key == 0)
        ok = ok && (keyed ? fbk_greedy_from_keys(amax_keys_, ids_, tok_pos_, greedy_out_, greedy_step_, stream_)
                          : fbk_greedy_advance(logits_, cfg_.vocab, ids_, tok_pos_, greedy_out_, greedy_step_, stream_)) == 0;
    else
        ok = ok && (keyed ? fbk_argmax_from_keys(amax_keys_, T, argmax_, stream_)
                          : fbk_argmax(logits_, cfg_.vocab, T, cfg_.vocab, argmax_, stream_)) == 0;
    const cudaError_t ce = cudaStreamEndCapture(stream_, &graph);
    if (!ok || ce != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        if (err) *err = "graph capture failed: " + (e2.empty() ? std::string(cudaGetErrorString(ce)) : e2);
        cudaGetLastError();
        return false;
    }
    size_t nodes = 0;
    cudaGraphGetNodes(graph, nullptr, &nodes);
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) { if (err) *err = std::string("graph instantiate: ") + cudaGetErrorString(ie); return false; }
    graphs_[key] = exec;
    graph_kernels_[key] = (int)nodes;
    return true;
}

bool Engine::forward(int sid, const int32_t* ids, int T, float* logits_last, float* logits_all, int32_t* argmax,
                     std::string* err) {
    if (sid < 0 || sid >= max_seqs_ || !seqs_[sid].open) { if (err) *err = "bad session"; return false; }
    if (T <= 0 || T > kMaxBatch) { if (err) *err = "bad token count"; return false; }
    const Config& c = cfg_;
    for (int t = 0; t < T; ++t)
        if (ids[t] < 0 || ids[t] >= c.vocab) { if (err) *err = "token id out of range"; return false; }
    Seq& s = seqs_[sid];
    const int pos0 = s.len;
    if (!ensure_pages(sid, pos0 + T, err)) return false;
    std::vector<int> sids(T, sid), pos(T);
    for (int t = 0; t < T; ++t) pos[t] = pos0 + t;
    if (!upload_tokens(ids, sids.data(), pos.data(), T, err)) return false;
    // profiling: hold the stream for 5 ms so every launch of the step is queued
    // before the first one runs and the event pairs time the kernels alone
    if (prof_) CK(fbk_delay(5000000ull, stream_));
    const bool all = logits_all != nullptr || argmax != nullptr;
    const int nrows = all ? T : 1;
    if (T == 1 && !prof_ && step_ready()) {
        if (!run_step(sid, 1, argmax_, err)) return false;
    } else if (T == 1 && use_graphs_ && !prof_) {
        if (!graphs_.count(1) && !capture_graph(1, err)) return false;
        CK(cudaGraphLaunch(graphs_[1], stream_));
    } else {
        if (!embed_rows(T, err)) return false;
        if (!run_layers(T, pos0 + T, T == 1, err)) return false;
        const int row0 = all ? 0 : T - 1;
        if (!run_head(row0, nrows, logits_, err)) return false;
        if (argmax) CKP(PC_OTHER, 0, fbk_argmax(logits_, c.vocab, nrows, c.vocab, argmax_, stream_));
    }
    if (logits_all) CK(cudaMemcpyAsync(logits_all, logits_, sizeof(float) * (size_t)T * c.vocab, cudaMemcpyDeviceToHost, stream_));
    if (logits_last)
        CK(cudaMemcpyAsync(logits_last, logits_ + (size_t)(nrows - 1) * c.vocab, sizeof(float) * c.vocab,
                           cudaMemcpyDeviceToHost, stream_));
    if (argmax) CK(cudaMemcpyAsync(argmax, argmax_, sizeof(int32_t) * T, cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    s.len = pos0 + T;
    return true;
}

bool Engine::decode_argmax(int sid, int32_t id, const int32_t* recent, int n_recent, float penalty, int32_t* out,
                           std::string* err) {
    const bool pen = n_recent > 0 && penalty > 0.0f && penalty != 1.0f;
    if (!pen) return forward(sid, &id, 1, nullptr, nullptr, out, err);
    if (n_recent > kMaxRecent) { if (err) *err = "penalty window too long"; return false; }
    if (sid < 0 || sid >= max_seqs_ || !seqs_[sid].open) { if (err) *err = "bad session"; return false; }
    const Config& c = cfg_;
    if (id < 0 || id >= c.vocab) { if (err) *err = "token id out of range"; return false; }
    Seq& s = seqs_[sid];
    const int pos0 = s.len;
    if (!ensure_pages(sid, pos0 + 1, err)) return false;
    if (!upload_tokens(&id, &sid, &pos0, 1, err)) return false;   // waits for the previous step's copies
    int32_t* hr = h_pinned_ + 3 * kMaxBatch;
    std::copy(recent, recent + n_recent, hr);
    CK(cudaMemcpyAsync(recent_dev_, hr, sizeof(int32_t) * n_recent, cudaMemcpyHostToDevice, stream_));
    if (use_graphs_) {
        if (!graphs_.count(1) && !capture_graph(1, err)) return false;
        CK(cudaGraphLaunch(graphs_[1], stream_));
    } else {
        if (!embed_rows(1, err)) return false;
        if (!run_layers(1, pos0 + 1, true, err)) return false;
        if (!run_head(0, 1, logits_, err)) return false;
    }
    CK(fbk_argmax_penalized(logits_, c.vocab, recent_dev_, n_recent, penalty, argmax_, stream_));
    CK(cudaMemcpyAsync(out, argmax_, sizeof(int32_t), cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    s.len = pos0 + 1;
    return true;
}

bool Engine::verify(int sid, const int32_t* ids, int T, const int32_t* hist, int base, int window, float penalty,
                    int32_t* argmax, float* logits_all, std::string* err) {
    if (sid < 0 || sid >= max_seqs_ || !seqs_[sid].open) { if (err) *err = "bad session"; return false; }
    if (T <= 0 || T > kMaxBatch) { if (err) *err = "bad token count"; return false; }
    const bool pen = argmax && penalty > 0.0f && penalty != 1.0f && window > 0;
    if (pen && (!hist || base < 0 || window > kMaxRecent || base + T - 1 > kMaxRecent)) {
        if (err) *err = "penalty window too long";
        return false;
    }
    const Config& c = cfg_;
    for (int t = 0; t < T; ++t)
        if (ids[t] < 0 || ids[t] >= c.vocab) { if (err) *err = "token id out of range"; return false; }
    Seq& s = seqs_[sid];
    const int pos0 = s.len;
    if (!ensure_pages(sid, pos0 + T, err)) return false;
    std::vector<int> sids(T, sid), pos(T);
    for (int t = 0; t < T; ++t) pos[t] = pos0 + t;
    if (!step_tokens(sids.data(), ids, pos.data(), T, err)) return false;   // its upload waited for the stream
    if (pen) {
        const int n_hist = base + T - 1;
        int32_t* hr = h_pinned_ + 3 * kMaxBatch;
        std::copy(hist, hist + n_hist, hr);
        if (n_hist > 0) CK(cudaMemcpyAsync(recent_dev_, hr, sizeof(int32_t) * n_hist, cudaMemcpyHostToDevice, stream_));
        CK(fbk_argmax_penalized_rows(logits_, c.vocab, T, c.vocab, recent_dev_, base, window, penalty, argmax_, stream_));
    }
    if (argmax) CK(cudaMemcpyAsync(argmax, argmax_, sizeof(int32_t) * T, cudaMemcpyDeviceToHost, stream_));
    if (logits_all) CK(cudaMemcpyAsync(logits_all, logits_, sizeof(float) * (size_t)T * c.vocab, cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    s.len = pos0 + T;
    return true;
}

// One decode step of n tokens, token i at position pos[i] of sequence
// sids[i] (pages already ensured): the batched-decode graph for n (or its
// eager launches), logits in logits_ and first-maximum ids in argmax_.
// Tokens of one sequence at consecutive positions attend causally: every
// token's K/V row is appended before the attention kernel reads keys up to
// its own position.
bool Engine::step_tokens(const int* sids, const int32_t* ids, const int* pos, int n, std::string* err) {
    const Config& c = cfg_;
    if (!upload_tokens(ids, sids, pos, n, err)) return false;
    // the 64-key blocks every token of the step holds on the same pages,
    // below every token's own position: attention reads them once for all
    {
        int bp = 0;
        if (n >= 2 && n <= kPrefixMaxBatch && c.attn_softcap <= 0.0f && c.sliding_window <= 0) {
            const std::vector<int>& p0 = seqs_[sids[0]].pages;
            size_t common = p0.size();
            for (int i = 1; i < n && common > 0; ++i) {
                const std::vector<int>& pi = seqs_[sids[i]].pages;
                size_t j = 0;
                while (j < common && j < pi.size() && pi[j] == p0[j]) ++j;
                common = j;
            }
            long long lp = (long long)common * kPageSize;
            for (int i = 0; i < n; ++i) lp = std::min<long long>(lp, pos[i]);
            bp = (int)std::min<long long>(lp / 64, fbk_attention_prefix_max_blocks());
        }
        int32_t* hb = h_pinned_ + 3 * kMaxBatch + kMaxRecent;
        *hb = bp;
        last_prefix_blocks_ = bp;
        CK(cudaMemcpyAsync(pre_blocks_, hb, sizeof(int32_t), cudaMemcpyHostToDevice, stream_));
    }
    if (use_graphs_) {
        if (!graphs_.count(n) && !capture_graph(n, err)) return false;
        CK(cudaEventRecord(ev0_, stream_));
        CK(cudaGraphLaunch(graphs_[n], stream_));
        CK(cudaEventRecord(ev1_, stream_));
    } else {
        int max_ctx = 0;
        for (int i = 0; i < n; ++i) max_ctx = std::max(max_ctx, pos[i] + 1);
        if (!embed_rows(n, err)) return false;
        if (!run_layers(n, max_ctx, true, err)) return false;
        if (!run_head(0, n, logits_, err)) return false;
        CK(fbk_argmax(logits_, c.vocab, n, c.vocab, argmax_, stream_));
    }
    return true;
}

bool Engine::decode_batch(const int* sids, const int32_t* ids, int n, int32_t* argmax, float* logits, std::string* err) {
    if (n <= 0 || n > kMaxBatch) { if (err) *err = "bad batch size"; return false; }
    const Config& c = cfg_;
    std::vector<int> pos(n);
    for (int i = 0; i < n; ++i) {
        const int sid = sids[i];
        if (sid < 0 || sid >= max_seqs_ || !seqs_[sid].open) { if (err) *err = "bad session in batch"; return false; }
        for (int j = 0; j < i; ++j) if (sids[j] == sid) { if (err) *err = "session repeated in one batch"; return false; }
        if (ids[i] < 0 || ids[i] >= c.vocab) { if (err) *err = "token id out of range"; return false; }
        if (!ensure_pages(sid, seqs_[sid].len + 1, err)) return false;
        pos[i] = seqs_[sid].len;
    }
    if (!step_tokens(sids, ids, pos.data(), n, err)) return false;
    if (argmax) CK(cudaMemcpyAsync(argmax, argmax_, sizeof(int32_t) * n, cudaMemcpyDeviceToHost, stream_));
    if (logits) CK(cudaMemcpyAsync(logits, logits_, sizeof(float) * (size_t)n * c.vocab, cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    if (use_graphs_) cudaEventElapsedTime(&last_batch_ms_, ev0_, ev1_);
    for (int i = 0; i < n; ++i) seqs_[sids[i]].len += 1;
    return true;
}

int Engine::decode_greedy(int sid, int32_t first, int n_steps, int32_t* out, std::string* err) {
    if (sid < 0 || sid >= max_seqs_ || !seqs_[sid].open) { if (err) *err = "bad session"; return -1; }
    if (n_steps <= 0) return 0;
    if (n_steps > greedy_cap_) { if (err) *err = "too many steps for one call"; return -1; }
    if (first < 0 || first >= cfg_.vocab) { if (err) *err = "token id out of range"; return -1; }
    Seq& s = seqs_[sid];
    if (!ensure_pages(sid, s.len + n_steps, err)) return -1;
    const int pos = s.len;
    if (!upload_tokens(&first, &sid, &pos, 1, err)) return -1;
    if (cudaMemsetAsync(greedy_step_, 0, sizeof(int32_t), stream_) != cudaSuccess) { if (err) *err = "memset failed"; return -1; }
    if (step_ready()) {
        if (!run_step(sid, n_steps, greedy_out_, err)) return -1;
        last_greedy_ms_ = last_step_ms_;
        if (cudaMemcpy(out, greedy_out_, sizeof(int32_t) * n_steps, cudaMemcpyDeviceToHost) != cudaSuccess) {
            if (err) *err = "copy failed";
            return -1;
        }
        s.len += n_steps;
        return n_steps;
    }
    if (!graphs_.count(0) && !capture_graph(0, err)) return -1;
    cudaGraphExec_t exec = graphs_[0];
    cudaEventRecord(ev0_, stream_);
    for (int i = 0; i < n_steps; ++i) {
        if (cudaGraphLaunch(exec, stream_) != cudaSuccess) {
            if (err) *err = "graph launch failed";
            cudaStreamSynchronize(stream_);
            return -1;
        }
    }
    cudaEventRecord(ev1_, stream_);
    if (cudaMemcpyAsync(out, greedy_out_, sizeof(int32_t) * n_steps, cudaMemcpyDeviceToHost, stream_) != cudaSuccess ||
        cudaStreamSynchronize(stream_) != cudaSuccess) {
        if (err) *err = std::string("decode failed: ") + cudaGetErrorString(cudaGetLastError());
        return -1;
    }
    cudaEventElapsedTime(&last_greedy_ms_, ev0_, ev1_);
    s.len += n_steps;
    return n_steps;
}

bool Engine::profile_decode(int sid, int32_t first, int n_steps, std::vector<ProfClass>* out, std::string* err) {
    std::vector<ProfClass> cls(5);
    cls[PC_GEMV].name = "gemv";
    cls[PC_NORMQ].name = "norm_quant";
    cls[PC_ROPE].name = "rope_kv_append";
    cls[PC_ATTN].name = "attention";
    cls[PC_OTHER].name = "other";
    prof_ = &cls;
    int32_t tok = first;
    bool ok = true;
    std::vector<int32_t> am(1);
    for (int i = 0; i < n_steps && ok; ++i) {
        prof_next_ = 0;
        prof_recs_.clear();
        ok = forward(sid, &tok, 1, nullptr, nullptr, am.data(), err);   // ends with a stream sync
        tok = am[0];
        for (const ProfRec& r : prof_recs_) {
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, prof_events_[r.e0], prof_events_[r.e1]);
            cls[r.cls].launches += 1;
            cls[r.cls].ms += ms;
            cls[r.cls].bytes += r.bytes;
        }
    }
    prof_ = nullptr;
    if (ok) *out = cls;
    return ok;
}

}  // namespace fb
