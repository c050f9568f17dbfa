// af_llama_cuda.cpp — llama_cuda_generate on the B200 decode path.
//
// Replaces the reference's stub (src/models/llama_cuda_model.cpp:7-17, which
// falls back to the CPU): llama_generate reaches this function when the
// engine was created with backend "cuda" and the model file is compiled with
// AXONFORGE_HAS_CUDA (src/models/llama_model.cpp:1633-1642).
//
// The model's tensors are uploaded byte-for-byte from the engine's zero-copy
// mmap views (Engine::weight, include/axonforge/engine.hpp:124) into a
// libaf_b200 engine, cached per Engine the way the reference caches its CPU
// weights (src/models/llama_model.cpp:1541-1548).  Generation keeps
// llama_generate_cpu_impl's semantics (src/models/llama_model.cpp:1502-1631):
// BOS prepended unless present, the hyper-parameter defaults it applies, the
// sampler's std::mt19937(42) stream, the repetition-penalty window, on_token
// per emitted token, stop at EOS (not emitted) or the context cap.  Sampling
// runs on the device (af_engine_sample); the draws come from the host rng.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "af_b200.h"
#include "axonforge/models/llama_cuda.hpp"

namespace axonforge {
namespace {

void check(cudaError_t st, const char* where) {
    if (st != cudaSuccess) {
        const char* msg = af_last_error();
        throw std::runtime_error(std::string("llama_cuda_generate: ") + where + ": " + cudaGetErrorString(st) +
                                 (msg && *msg ? std::string(" (") + msg + ")" : std::string()));
    }
}

int ggml_type_of(DType t) {
    switch (t) {
        case DType::F32: return AF_GGML_F32;
        case DType::Q4_K_M: return AF_GGML_Q4_K;
        case DType::Q6_K: return AF_GGML_Q6_K;
        default: return -1;
    }
}

// af_model_config with the defaults llama_generate_cpu_impl applies
// (src/models/llama_model.cpp:1507-1522).
af_model_config config_of(const Engine& engine, const LlamaConfig& cfg) {
    const ModelConfig& mc = engine.model_config();
    af_model_config c{};
    c.n_layer = mc.n_layers;
    c.n_embd = mc.hidden_dim;
    c.n_head = mc.n_heads;
    c.n_kv_head = mc.n_kv_heads > 0 ? mc.n_kv_heads : mc.n_heads;
    c.n_ctx = std::min(mc.max_seq_len, cfg.max_context_len);
    c.vocab = mc.vocab_size > 0 ? mc.vocab_size : 32000;
    c.eps = mc.rms_norm_eps > 0.f ? mc.rms_norm_eps : 1e-5f;
    c.theta = mc.rope_theta > 0.f ? mc.rope_theta : 10000.f;
    c.ffn = mc.ffn_dim > 0 ? mc.ffn_dim : 4 * mc.hidden_dim;
    c.qk_norm_order = mc.arch == "hunyuan-dense" ? 2 : (mc.arch == "qwen3" ? 1 : 0);
    c.bos_id = engine.bos_id();
    c.eos_id = engine.eos_id();
    return c;
}

void upload(af_engine* e, const Engine& engine, const char* name, bool required) {
    const Tensor* t = engine.weight(name);
    if (!t) {
        if (required) throw std::runtime_error(std::string("llama_cuda_generate: tensor '") + name + "' not found");
        return;
    }
    const int type = ggml_type_of(t->dtype());
    if (type < 0)
        throw std::runtime_error(std::string("llama_cuda_generate: tensor '") + name +
                                 "' has a type the B200 path does not take (F32, Q4_K, Q6_K)");
    const std::vector<int64_t> dims(t->shape().begin(), t->shape().end());  // GGML order: dims[0] = columns
    check(af_engine_load_tensor(e, name, type, dims.data(), static_cast<int>(dims.size()), t->raw_data(),
                                gguf_tensor_nbytes(t->dtype(), t->numel())),
          name);
}

// The tensors build_weights reads (src/models/llama_model.cpp:973-1004).
void upload_model(af_engine* e, const Engine& engine, int n_layer) {
    upload(e, engine, "token_embd.weight", true);
    upload(e, engine, "output_norm.weight", true);
    upload(e, engine, "output.weight", false);  // falls back to token_embd
    char name[128];
    for (int l = 0; l < n_layer; ++l) {
        for (const char* w : {"attn_norm", "ffn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate",
                              "ffn_up", "ffn_down"}) {
            std::snprintf(name, sizeof(name), "blk.%d.%s.weight", l, w);
            upload(e, engine, name, true);
        }
        for (const char* w : {"attn_q.bias", "attn_k.bias", "attn_v.bias", "attn_q_norm.weight", "attn_k_norm.weight"}) {
            std::snprintf(name, sizeof(name), "blk.%d.%s", l, w);
            upload(e, engine, name, false);
        }
    }
}

struct DeviceModel {
    const Engine* owner = nullptr;
    int n_ctx = 0;
    af_engine* e = nullptr;
    ~DeviceModel() {
        if (e) af_engine_destroy(e);
    }
};

}  // namespace

std::vector<int32_t> llama_cuda_generate(const Engine& engine, std::vector<int32_t> prompt_ids,
                                         const LlamaConfig& cfg) {
    if (prompt_ids.empty()) throw std::invalid_argument("llama_generate: empty prompt");
    const af_model_config c = config_of(engine, cfg);
    // device weights, cached per Engine (and context size)
    static DeviceModel dm;
    if (dm.owner != &engine || dm.n_ctx != c.n_ctx) {
        if (dm.e) af_engine_destroy(dm.e);
        dm.e = nullptr;
        dm.owner = nullptr;
        check(af_engine_create(&c, /*device*/ 0, /*tp_rank*/ 0, /*tp_size*/ 1, nullptr, &dm.e), "af_engine_create");
        upload_model(dm.e, engine, c.n_layer);
        // AF_Q8_ACTIVATIONS=1: the reference CPU path's production activation
        // format (Q8_0 before every GEMV) instead of the default 16-bit grid,
        // which tracks the F32-activation forward
        if (const char* q8 = std::getenv("AF_Q8_ACTIVATIONS"); q8 && q8[0] == '1')
            check(af_engine_set_q8_activations(dm.e, 1), "af_engine_set_q8_activations");
        check(af_engine_finalize(dm.e), "af_engine_finalize");
        dm.owner = &engine;
        dm.n_ctx = c.n_ctx;
        if (cfg.verbose)
            std::fprintf(stderr, "[AxonForge] B200 decode path: %d layers resident on the GPU\n", c.n_layer);
    }
    af_engine* e = dm.e;

    const af_sampling s{cfg.temperature, cfg.top_k, cfg.top_p, cfg.rep_penalty, cfg.rep_penalty_last_n};
    std::vector<int32_t> generated;
    generated.reserve(std::max(cfg.max_new_tokens, 0));
    if (cfg.temperature <= 0.f && cfg.rep_penalty == 1.0f && !cfg.on_token) {
        // greedy without a callback: the device-fed decode loop
        std::vector<int32_t> out(std::max(cfg.max_new_tokens, 1));
        int n = 0;
        check(af_engine_generate(e, prompt_ids.data(), static_cast<int>(prompt_ids.size()), cfg.max_new_tokens,
                                 out.data(), &n),
              "af_engine_generate");
        generated.assign(out.begin(), out.begin() + n);
        return generated;
    }

    // the sampling loop of llama_generate_cpu_impl (llama_model.cpp:1560-1624)
    std::mt19937 rng(42);
    std::uniform_real_distribution<float> dist(0.f, 1.f);
    const int32_t bos = engine.bos_id();
    if (prompt_ids[0] != bos) prompt_ids.insert(prompt_ids.begin(), bos);
    const int np = static_cast<int>(prompt_ids.size());
    if (np > c.n_ctx) throw std::runtime_error("llama_cuda_generate: prompt longer than the context");
    check(af_engine_prefill(e, prompt_ids.data(), np, 0, nullptr, nullptr), "af_engine_prefill");
    std::vector<int32_t> rep_ctx(prompt_ids.begin(), prompt_ids.end());
    auto pick = [&]() {
        const int win = cfg.rep_penalty != 1.0f ? std::min(cfg.rep_penalty_last_n, static_cast<int>(rep_ctx.size()))
                                                : 0;
        const float r = cfg.temperature > 0.f ? dist(rng) : 0.f;
        int32_t next = 0;
        check(af_engine_sample(e, &s, rep_ctx.data() + rep_ctx.size() - std::max(win, 0), std::max(win, 0), r, &next),
              "af_engine_sample");
        return next;
    };
    int32_t next_id = pick();
    int n_past = np;
    for (int step = 0; step < cfg.max_new_tokens; ++step) {
        if (next_id == engine.eos_id()) break;  // stop cleanly; EOS not emitted
        if (n_past >= c.n_ctx) break;
        generated.push_back(next_id);
        if (cfg.on_token) cfg.on_token(next_id);
        check(af_engine_step(e, next_id, n_past, nullptr, nullptr), "af_engine_step");
        ++n_past;
        rep_ctx.push_back(next_id);
        next_id = pick();
    }
    return generated;
}

}  // namespace axonforge
