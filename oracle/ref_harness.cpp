// ref_harness.cpp — test-infrastructure harness around the UNMODIFIED reference
// sources of songqiuyu/llm_core ("AxonForge"), compiled in place by oracle/ref.mk
// into oracle/_ref/libaxref.so.
//
// This file is a checker, never the product: only tests/, the smoke check and
// bench.py's CPU-baseline / reference arm load the library it builds.
//
// It #includes src/models/llama_model.cpp so that the file-static forward
// (`build_weights`, `LlamaState`, `llama_forward_token`, `llama_forward_batch`,
// `sample`) is reachable without editing the reference.  Every entry point is a
// plain extern "C" function so Python (ctypes) can drive it.
//
// Modes:
//   f32_mode = 1 : every WT::q8_fast = false after build_weights.  gemv_wt_q8
//                  then falls through to gemv_wt (llama_model.cpp:830), i.e. the
//                  F32-activation kernels gemv_q4k_avx2_range /
//                  gemv_q6k_avx2_range, and Fusion C is skipped
//                  (llama_model.cpp:1284).  This is the parity oracle mode.
//   f32_mode = 0 : the shipped production path (Q8_0 activations, r8 repack).

#include "src/models/llama_model.cpp"

#include <chrono>
#include <exception>

namespace {

struct RefModel {
    axonforge::Engine engine;
    std::unique_ptr<axonforge::ThreadPool> pool;
    std::unique_ptr<axonforge::LlamaState> state;
    int n_ctx{0};
    int vocab{0};
    bool f32_mode{true};
    // Engine has no move constructor; initialise it from the factory's prvalue.
    template <class F>
    explicit RefModel(F&& make) : engine(make()) {}
};

thread_local std::string g_last_error;

}  // namespace

using namespace axonforge;

extern "C" {

const char* axref_last_error() { return g_last_error.c_str(); }

// --- standalone GEMV kernels (reference x86 path) ---------------------------

// y[0:rows] = W(Q4_K) · x, F32 activations: gemv_q4k_avx2_range
// (src/backend/cpu_x86/kernels/gemv_q4k_avx2.cpp:230-238).
void axref_gemv_q4k_f32(float* y, const uint8_t* W, const float* x, int rows, int cols) {
    const size_t row_bytes = (size_t)(cols / 256) * 144;
    cpu_x86::gemv_q4k_avx2_range(y, W, x, 0, rows, cols, row_bytes);
}

// Scalar restatement inside the reference: q4k_dot_row (llama_model.cpp:476-504).
void axref_gemv_q4k_f32_scalar(float* y, const uint8_t* W, const float* x, int rows, int cols) {
    const size_t row_bytes = (size_t)(cols / 256) * 144;
    for (int o = 0; o < rows; ++o) y[o] = q4k_dot_row(W + (size_t)o * row_bytes, x, cols);
}

// y = W(Q6_K) · x, F32 activations: gemv_q6k_avx2_range (gemv_q6k_avx2.cpp:235-243).
void axref_gemv_q6k_f32(float* y, const uint8_t* W, const float* x, int rows, int cols) {
    const size_t row_bytes = (size_t)(cols / 256) * 210;
    cpu_x86::gemv_q6k_avx2_range(y, W, x, 0, rows, cols, row_bytes);
}

void axref_gemv_q6k_f32_scalar(float* y, const uint8_t* W, const float* x, int rows, int cols) {
    const size_t row_bytes = (size_t)(cols / 256) * 210;
    for (int o = 0; o < rows; ++o) y[o] = q6k_dot_row(W + (size_t)o * row_bytes, x, cols);
}

// Production GEMV (Q8_0 activations) exactly as gemv_wt_q8 runs it
// (llama_model.cpp:767-831), with an r8 repack when rows % 8 == 0.
// dtype: 12 = Q4_K, 14 = Q6_K (ggml type ids).
// The reference's own F32 -> Q8_0 quantiser (the kQ8Quant the production
// decode uses), unpacked into d[k/32] and q[k].
void axref_quantize_q8(const float* x, int k, float* d, int8_t* q) {
    std::vector<block_q8_0> blocks((size_t)(k / 32));
    kQ8Quant(blocks.data(), x, k);
    for (int i = 0; i < k / 32; ++i) {
        d[i] = blocks[i].d;
        std::memcpy(q + (size_t)32 * i, blocks[i].qs, 32);
    }
}

void axref_gemv_q8_production(float* y, const uint8_t* W, int ggml_type, const float* x,
                              int rows, int cols, int n_threads) {
    WT wt;
    wt.data = W;
    wt.dtype = ggml_type == 14 ? DType::Q6_K : DType::Q4_K_M;
    wt.q8_fast = true;
    repack_q4k_if_avx2(wt, rows, cols);
    std::vector<uint8_t> xq(sizeof(block_q8_0) * (cols / 32));
    kQ8Quant(reinterpret_cast<block_q8_0*>(xq.data()), x, cols);
    std::unique_ptr<ThreadPool> pool;
    if (n_threads > 1) pool = std::make_unique<ThreadPool>(n_threads - 1);
    gemv_wt_q8(y, wt, reinterpret_cast<block_q8_0*>(xq.data()), x, rows, cols, pool.get());
}

// --- whole-model forward ----------------------------------------------------

void* axref_open(const char* path, int n_threads, int f32_mode, int max_ctx) {
    try {
        EngineConfig ec;
        ec.backend = "cpu_x86";
        auto* m = new RefModel([&] { return Engine::from_gguf(path, ec); });
        const ModelConfig& mc = m->engine.model_config();
        const int L = mc.n_layers, E = mc.hidden_dim, H = mc.n_heads;
        const int KVH = mc.n_kv_heads > 0 ? mc.n_kv_heads : H;
        const int NC = std::min(mc.max_seq_len, max_ctx > 0 ? max_ctx : 4096);
        const int V = mc.vocab_size > 0 ? mc.vocab_size : 32000;
        const float eps = mc.rms_norm_eps > 0.f ? mc.rms_norm_eps : 1e-5f;
        const float rtheta = mc.rope_theta > 0.f ? mc.rope_theta : 10000.f;
        const int FD = mc.ffn_dim > 0 ? mc.ffn_dim : 4 * E;
        const QkNormOrder qk_order = mc.arch == "hunyuan-dense"
            ? QkNormOrder::AfterRope
            : (mc.arch == "qwen3" ? QkNormOrder::BeforeRope : QkNormOrder::None);
        if (n_threads > 1) m->pool = std::make_unique<ThreadPool>(n_threads - 1);
        m->state = std::make_unique<LlamaState>(L, NC, E, H, KVH, V, FD, eps, rtheta,
                                                n_threads, qk_order, m->pool.get());
        m->state->weights = build_weights(m->engine, L, E, H, KVH, FD);
        m->f32_mode = f32_mode != 0;
        if (m->f32_mode) {
            auto& w = m->state->weights;
            w.tok_embd.q8_fast = false;
            w.output.q8_fast = false;
            for (auto& lw : w.layers) {
                lw.wq.q8_fast = lw.wk.q8_fast = lw.wv.q8_fast = lw.wo.q8_fast = false;
                lw.wgate.q8_fast = lw.wup.q8_fast = lw.wdown.q8_fast = false;
            }
        }
        m->n_ctx = NC;
        m->vocab = V;
        return m;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return nullptr;
    }
}

void axref_close(void* h) { delete static_cast<RefModel*>(h); }

int axref_vocab(void* h) { return static_cast<RefModel*>(h)->vocab; }
int axref_n_ctx(void* h) { return static_cast<RefModel*>(h)->n_ctx; }
int axref_bos(void* h) { return static_cast<RefModel*>(h)->engine.bos_id(); }

// One decode step: llama_forward_token (llama_model.cpp:1207-1333); logits copied out.
int axref_forward_token(void* h, int token, int pos, float* logits) {
    auto* m = static_cast<RefModel*>(h);
    try {
        llama_forward_token(token, pos, *m->state);
        m->state->n_past = pos + 1;
        if (logits) std::memcpy(logits, m->state->logits.data(), sizeof(float) * m->vocab);
        return 0;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return -1;
    }
}

// Prefill: llama_forward_batch (llama_model.cpp:1339-1462); last-token logits.
int axref_forward_batch(void* h, const int32_t* tokens, int T, int pos0, float* logits) {
    auto* m = static_cast<RefModel*>(h);
    try {
        llama_forward_batch(tokens, T, pos0, *m->state);
        m->state->n_past = pos0 + T;
        if (logits) std::memcpy(logits, m->state->logits.data(), sizeof(float) * m->vocab);
        return 0;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return -1;
    }
}

// Copy of the fp32 residual stream after the last forward (LlamaState::x).
int axref_hidden(void* h, float* out) {
    auto* m = static_cast<RefModel*>(h);
    std::memcpy(out, m->state->x.data(), sizeof(float) * m->state->n_embd);
    return m->state->n_embd;
}

// Greedy generation with the decode-loop semantics of llama_generate_cpu_impl
// (llama_model.cpp:1562-1624): BOS prepend, prefill, argmax sampling, stop on
// EOS or the context cap.  Writes up to max_new ids, returns the count.
// If step_logits != NULL, the logits before every sampled token are appended
// (row i = logits that chose out[i]).
int axref_generate_greedy(void* h, const int32_t* prompt, int n_prompt, int max_new,
                          int32_t* out, float* step_logits) {
    auto* m = static_cast<RefModel*>(h);
    try {
        std::vector<int32_t> ids(prompt, prompt + n_prompt);
        const int32_t bos = m->engine.bos_id();
        if (ids.empty() || ids[0] != bos) ids.insert(ids.begin(), bos);
        auto& s = *m->state;
        const int np = (int)ids.size();
        if (np > 1) {
            llama_forward_batch(ids.data(), np, 0, s);
        } else {
            llama_forward_token(ids[0], 0, s);
        }
        s.n_past = np;
        std::mt19937 rng(42);
        int32_t next = sample(s.logits.data(), m->vocab, 0, 1.f, 0.f, rng);
        int n = 0;
        for (int step = 0; step < max_new; ++step) {
            if (next == m->engine.eos_id()) break;
            if (s.n_past >= m->n_ctx) break;
            if (step_logits)
                std::memcpy(step_logits + (size_t)n * m->vocab, s.logits.data(),
                            sizeof(float) * m->vocab);
            out[n++] = next;
            llama_forward_token(next, s.n_past, s);
            s.n_past++;
            next = sample(s.logits.data(), m->vocab, 0, 1.f, 0.f, rng);
        }
        return n;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return -1;
    }
}

// Timed decode: `steps` llama_forward_token calls continuing from the state's
// n_past, feeding back the argmax.  Returns the elapsed seconds.
double axref_time_decode(void* h, int first_token, int steps) {
    auto* m = static_cast<RefModel*>(h);
    auto& s = *m->state;
    int32_t tok = first_token;
    std::mt19937 rng(42);
    const auto t0 = std::chrono::steady_clock::now();
    for (int i = 0; i < steps && s.n_past < m->n_ctx; ++i) {
        llama_forward_token(tok, s.n_past, s);
        s.n_past++;
        tok = sample(s.logits.data(), m->vocab, 0, 1.f, 0.f, rng);
    }
    const auto t1 = std::chrono::steady_clock::now();
    return std::chrono::duration<double>(t1 - t0).count();
}

// The reference decode loop's repetition penalty, as the apply_rep_penalty
// lambda of llama_generate_cpu_impl states it (llama_model.cpp:1586-1598),
// over the window ids in order.
static void ref_rep_penalty(float* lp, int V, const int32_t* win, int n, float pen) {
    if (pen == 1.0f) return;
    for (int i = 0; i < n; i++) {
        const int32_t id = win[i];
        if (id < 0 || id >= V) continue;
        lp[id] = lp[id] > 0.f ? lp[id] / pen : lp[id] * pen;
    }
}

// One sampling step of the reference: the penalty over `win`, then sample()
// (llama_model.cpp:1466-1498) with a fresh std::mt19937(seed).
int axref_sample(const float* logits, int V, const int32_t* win, int n_win, float rep_penalty, int top_k,
                 float top_p, float temperature, uint32_t seed) {
    std::vector<float> lp(logits, logits + V);
    ref_rep_penalty(lp.data(), V, win, n_win, rep_penalty);
    std::mt19937 rng(seed);
    return sample(lp.data(), V, top_k, top_p, temperature, rng);
}

// Sampled generation: the loop of llama_generate_cpu_impl
// (llama_model.cpp:1562-1624) with its rng (mt19937(42)) and repetition
// window, on this harness's state (F32 activations when opened so).
int axref_generate_sampled(void* h, const int32_t* prompt, int n_prompt, int max_new, float temperature, int top_k,
                           float top_p, float rep_penalty, int rep_last_n, int32_t* out) {
    auto* m = static_cast<RefModel*>(h);
    try {
        std::vector<int32_t> ids(prompt, prompt + n_prompt);
        const int32_t bos = m->engine.bos_id();
        if (ids.empty() || ids[0] != bos) ids.insert(ids.begin(), bos);
        auto& s = *m->state;
        const int np = (int)ids.size();
        if (np > 1) {
            llama_forward_batch(ids.data(), np, 0, s);
        } else {
            llama_forward_token(ids[0], 0, s);
        }
        s.n_past = np;
        std::mt19937 rng(42);
        std::vector<int32_t> rep_ctx(ids.begin(), ids.end());
        auto pick = [&]() {
            const int win = std::min(rep_last_n, (int)rep_ctx.size());
            ref_rep_penalty(s.logits.data(), m->vocab, rep_ctx.data() + rep_ctx.size() - win, win, rep_penalty);
            return sample(s.logits.data(), m->vocab, top_k, top_p, temperature, rng);
        };
        int32_t next = pick();
        int n = 0;
        for (int step = 0; step < max_new; ++step) {
            if (next == m->engine.eos_id()) break;
            if (s.n_past >= m->n_ctx) break;
            out[n++] = next;
            llama_forward_token(next, s.n_past, s);
            s.n_past++;
            rep_ctx.push_back(next);
            next = pick();
        }
        return n;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return -1;
    }
}

// n draws of std::uniform_real_distribution<float>(0, 1) from std::mt19937(seed).
void axref_uniform(uint32_t seed, int n, float* out) {
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> dist(0.f, 1.f);
    for (int i = 0; i < n; ++i) out[i] = dist(rng);
}

int axref_n_past(void* h) { return static_cast<RefModel*>(h)->state->n_past; }
void axref_set_n_past(void* h, int n) { static_cast<RefModel*>(h)->state->n_past = n; }

}  // extern "C"
