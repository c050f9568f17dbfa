// integ_harness.cpp — test harness for the reference-side binding of the B200
// path (integration/af_cuda_backend.cpp, integration/af_llama_cuda.cpp).
//
// Test infrastructure: it drives the UNMODIFIED reference's public API —
// Engine::from_gguf with EngineConfig.backend, llama_generate,
// BackendRegistry / IBackend / IKernel — from extern "C" entry points that
// Python (ctypes) calls.  oracle/ref.mk links it with the reference's own
// objects (llama_model.cpp compiled with AXONFORGE_HAS_CUDA, so llama_generate
// dispatches to llama_cuda_generate for backend "cuda") and libaf_b200.so into
// oracle/_ref/libaxref_b200.so.
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <vector>

#include "axonforge/backend.hpp"
#include "axonforge/engine.hpp"
#include "axonforge/models/llama.hpp"

using namespace axonforge;

namespace {
thread_local std::string g_err;
}

extern "C" {

const char* axintg_last_error() { return g_err.c_str(); }

int axintg_has_backend(const char* id) { return BackendRegistry::instance().has_backend(id) ? 1 : 0; }

// llama_generate (src/models/llama_model.cpp:1633-1642) on a fresh Engine
// with the given backend; writes up to max_new ids, returns the count or -1.
int axintg_generate(const char* path, const char* backend, const int32_t* prompt, int n_prompt, int max_new,
                    float temperature, int top_k, float top_p, float rep_penalty, int rep_last_n, int32_t* out,
                    int32_t* streamed) {
    try {
        EngineConfig ec;
        ec.backend = backend;
        Engine engine = Engine::from_gguf(path, ec);
        LlamaConfig cfg;
        cfg.max_new_tokens = max_new;
        cfg.temperature = temperature;
        cfg.top_k = top_k;
        cfg.top_p = top_p;
        cfg.rep_penalty = rep_penalty;
        cfg.rep_penalty_last_n = rep_last_n;
        int n_cb = 0;
        if (streamed) cfg.on_token = [&](int32_t id) { streamed[n_cb++] = id; };
        const std::vector<int32_t> ids = llama_generate(engine, std::vector<int32_t>(prompt, prompt + n_prompt), cfg);
        std::memcpy(out, ids.data(), ids.size() * sizeof(int32_t));
        return static_cast<int>(ids.size());
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

// One MATMUL through the backend's IKernel: W (GGUF blocks, host) and x
// ([T][cols], host) transferred to the backend's memory, y ([T][rows]) back.
int axintg_matmul(const char* backend, int ggml_type, const void* w_host, int rows, int cols, const float* x_host,
                  int T, float* y_host) {
    try {
        auto be = BackendRegistry::instance().create(backend);
        if (!be->initialize()) throw std::runtime_error("backend failed to initialise");
        const DType wt = ggml_type == 14 ? DType::Q6_K : DType::Q4_K_M;
        const size_t wbytes = gguf_tensor_nbytes(wt, (int64_t)rows * cols);
        Tensor w_h = Tensor::from_raw_blob(const_cast<void*>(w_host), wbytes, {cols, rows}, wt);
        Tensor w_d = Tensor::from_storage(be->allocate(wbytes), {cols, rows}, wt);
        Shape xs = T > 1 ? Shape{T, cols} : Shape{cols};
        Shape ys = T > 1 ? Shape{T, rows} : Shape{rows};
        Tensor x_h = Tensor::from_blob(const_cast<float*>(x_host), xs, DType::F32);
        Tensor x_d = Tensor::from_storage(be->allocate((size_t)T * cols * 4), xs, DType::F32);
        Tensor y_d = Tensor::from_storage(be->allocate((size_t)T * rows * 4), ys, DType::F32);
        Tensor y_h = Tensor::from_blob(y_host, ys, DType::F32);
        be->transfer(w_h, w_d);
        be->transfer(x_h, x_d);
        const DType in_types[2] = {wt, DType::F32};
        if (!be->can_handle(OpType::MATMUL, in_types)) throw std::runtime_error("backend cannot handle MATMUL");
        AttributeMap attrs;
        attrs.set("row_bytes", (int64_t)(cols / 256) * (ggml_type == 14 ? 210 : 144));
        auto k = be->get_kernel(OpType::MATMUL, in_types, attrs);
        const Tensor ins[2] = {w_d, x_d};
        Tensor outs[1] = {y_d};
        k->execute(ins, outs, attrs);
        be->synchronize();
        be->transfer(y_d, y_h);
        be->finalize();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

// One RMS_NORM through the backend's IKernel (host in, host out).
int axintg_rms_norm(const char* backend, const float* x_host, const float* w_host, int n, float eps, float* y_host) {
    try {
        auto be = BackendRegistry::instance().create(backend);
        if (!be->initialize()) throw std::runtime_error("backend failed to initialise");
        Tensor x_h = Tensor::from_blob(const_cast<float*>(x_host), {n}, DType::F32);
        Tensor w_h = Tensor::from_blob(const_cast<float*>(w_host), {n}, DType::F32);
        Tensor y_h = Tensor::from_blob(y_host, {n}, DType::F32);
        Tensor x_d = Tensor::from_storage(be->allocate((size_t)n * 4), {n}, DType::F32);
        Tensor w_d = Tensor::from_storage(be->allocate((size_t)n * 4), {n}, DType::F32);
        Tensor y_d = Tensor::from_storage(be->allocate((size_t)n * 4), {n}, DType::F32);
        be->transfer(x_h, x_d);
        be->transfer(w_h, w_d);
        const DType in_types[2] = {DType::F32, DType::F32};
        AttributeMap attrs;
        attrs.set("eps", eps);
        auto k = be->get_kernel(OpType::RMS_NORM, in_types, attrs);
        const Tensor ins[2] = {x_d, w_d};
        Tensor outs[1] = {y_d};
        k->execute(ins, outs, attrs);
        be->synchronize();
        be->transfer(y_d, y_h);
        be->finalize();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

}  // extern "C"
