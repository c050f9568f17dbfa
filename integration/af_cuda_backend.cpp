// af_cuda_backend.cpp — AxonForge's "cuda" backend on the B200 decode path.
//
// The reference-side binding of libaf_b200.so (include/af_b200.h): an
// IBackend / IKernel pair (include/axonforge/backend.hpp:17-74) registered as
// "cuda" from a constructor function, exactly where the reference registers
// its sm_89 backend (src/backend/cuda/cuda_backend.cu:219-225).  Built
// against the reference's headers and linked with libaf_b200.so in place of
// src/backend/cuda/*, so `EngineConfig.backend = "cuda"` selects it.
//
// Op set: the reference CUDA backend's (src/backend/cuda/cuda_backend.cu:52-116,
// 184-198) — RMS_NORM, SILU, MUL, ROPE on F32, MATMUL on {Q4_K_M, F32} — plus
// MATMUL on {Q6_K, F32}, and a MATMUL whose activation is [T][K] (T > 1 rows)
// runs as one tensor-core GEMM (af_prefill_gemm_f32).
//
// MATMUL weights arrive as raw GGUF blocks (in[0], device memory, row_bytes
// per row).  The GEMV reads a packed layout, so each weight is packed once on
// first use into a buffer this backend owns, keyed by the weight's device
// address and shape; weights are assumed not to change in place (the
// reference never rewrites a loaded tensor).  Packs are freed in finalize().
//
// Errors: every C-ABI call returns a cudaError_t; failures throw
// std::runtime_error with af_last_error()'s text, as the reference backend
// does (src/backend/cuda/cuda_backend.cu:15-25).
#include <cuda_runtime.h>

#include <cstdio>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <tuple>

#include "af_b200.h"
#include "axonforge/backend.hpp"
#include "axonforge/dtype.hpp"

namespace axonforge::b200 {
namespace {

void check(cudaError_t st, const char* where) {
    if (st != cudaSuccess) {
        const char* msg = af_last_error();
        throw std::runtime_error(std::string(where) + ": " + cudaGetErrorString(st) +
                                 (msg && *msg ? std::string(" (") + msg + ")" : std::string()));
    }
}

int ggml_type_of(DType t) {
    switch (t) {
        case DType::Q4_K_M: return AF_GGML_Q4_K;
        case DType::Q6_K: return AF_GGML_Q6_K;
        default: return -1;
    }
}

// Device bytes a tensor occupies: exact block bytes for quantised types
// (gguf_tensor_nbytes, include/axonforge/dtype.hpp:136-155), not
// Tensor::nbytes, which is numel * an approximate element size for them.
size_t tensor_bytes(const Tensor& t) {
    return dtype_is_quantized(t.dtype()) ? gguf_tensor_nbytes(t.dtype(), t.numel()) : t.nbytes();
}

class DeviceStorage final : public TensorStorage {
public:
    DeviceStorage(size_t bytes, int device) : bytes_(bytes), device_(device) {
        if (bytes_ > 0) check(cudaMalloc(&ptr_, bytes_), "cudaMalloc");
    }
    ~DeviceStorage() override {
        if (ptr_) cudaFree(ptr_);
    }
    DeviceStorage(const DeviceStorage&) = delete;
    DeviceStorage& operator=(const DeviceStorage&) = delete;
    void* data() noexcept override { return ptr_; }
    const void* data() const noexcept override { return ptr_; }
    size_t byte_size() const noexcept override { return bytes_; }
    DeviceId device() const noexcept override { return DeviceId::cuda(device_); }

private:
    void* ptr_{nullptr};
    size_t bytes_{0};
    int device_{0};
};

// Packed copies of GGUF weight matrices, one per (address, type, rows, cols).
class PackCache {
public:
    const void* get(const void* gguf, int type, int rows, int cols, cudaStream_t st) {
        std::lock_guard<std::mutex> lock(mu_);
        const auto key = std::make_tuple(gguf, type, rows, cols);
        auto it = packs_.find(key);
        if (it != packs_.end()) return it->second;
        void* dst = nullptr;
        check(cudaMalloc(&dst, af_weight_bytes(type, rows, cols)), "cudaMalloc(packed weight)");
        const cudaError_t rc = af_weight_pack(dst, gguf, type, rows, cols, st);
        if (rc != cudaSuccess) {
            cudaFree(dst);
            check(rc, "af_weight_pack");
        }
        packs_.emplace(key, dst);
        return dst;
    }
    void clear() {
        std::lock_guard<std::mutex> lock(mu_);
        for (auto& kv : packs_) cudaFree(kv.second);
        packs_.clear();
    }

private:
    std::mutex mu_;
    std::map<std::tuple<const void*, int, int, int>, void*> packs_;
};

class B200Kernel final : public IKernel {
public:
    B200Kernel(OpType op, cudaStream_t stream, PackCache* packs) : op_(op), stream_(stream), packs_(packs) {}

    void execute(std::span<const Tensor> inputs, std::span<Tensor> outputs, const AttributeMap& attrs) override {
        if (outputs.empty()) throw std::runtime_error("B200Kernel::execute: no output tensor");
        float* y = static_cast<float*>(outputs[0].raw_data());
        switch (op_) {
            case OpType::RMS_NORM: {
                if (inputs.size() < 2) throw std::runtime_error("CUDA RMS_NORM requires x and weight");
                check(af_rms_norm_f32(y, static_cast<const float*>(inputs[0].raw_data()),
                                      static_cast<const float*>(inputs[1].raw_data()),
                                      static_cast<int>(inputs[0].numel()), attrs.get_or<float>("eps", 1e-5f),
                                      stream_),
                      "af_rms_norm_f32");
                break;
            }
            case OpType::SILU: {
                if (inputs.empty()) throw std::runtime_error("CUDA SILU requires input");
                check(af_silu_f32(y, static_cast<const float*>(inputs[0].raw_data()),
                                  static_cast<int>(inputs[0].numel()), stream_),
                      "af_silu_f32");
                break;
            }
            case OpType::MUL: {
                if (inputs.size() < 2) throw std::runtime_error("CUDA MUL requires two inputs");
                check(af_mul_f32(y, static_cast<const float*>(inputs[0].raw_data()),
                                 static_cast<const float*>(inputs[1].raw_data()),
                                 static_cast<int>(outputs[0].numel()), stream_),
                      "af_mul_f32");
                break;
            }
            case OpType::ROPE: {
                if (inputs.empty()) throw std::runtime_error("CUDA ROPE requires input/output alias tensor");
                const int n_heads = static_cast<int>(attrs.get_or<int64_t>("n_heads", 0));
                const int head_dim = static_cast<int>(attrs.get_or<int64_t>("head_dim", 0));
                const int pos = static_cast<int>(attrs.get_or<int64_t>("pos", 0));
                const float theta = attrs.get_or<float>("theta", 10000.0f);
                if (outputs[0].raw_data() != inputs[0].raw_data())
                    check(cudaMemcpyAsync(outputs[0].raw_data(), inputs[0].raw_data(), inputs[0].nbytes(),
                                          cudaMemcpyDeviceToDevice, stream_),
                          "cudaMemcpyAsync(ROPE)");
                check(af_rope_f32(y, n_heads, head_dim, pos, theta, stream_), "af_rope_f32");
                break;
            }
            case OpType::MATMUL: {
                if (inputs.size() < 2) throw std::runtime_error("CUDA MATMUL requires weight and x");
                const int type = ggml_type_of(inputs[0].dtype());
                if (type < 0 || inputs[1].dtype() != DType::F32)
                    throw std::runtime_error("CUDA MATMUL supports Q4_K_M / Q6_K weight x F32 activation");
                // x [T][K] (T = 1: one vector, the reference's v1 contract)
                const int64_t T = inputs[1].ndim() >= 2 ? inputs[1].dim(0) : 1;
                const int cols = static_cast<int>(inputs[1].numel() / (T > 0 ? T : 1));
                const int rows = static_cast<int>(outputs[0].numel() / (T > 0 ? T : 1));
                const int64_t dense = (int64_t)(cols / 256) * (type == AF_GGML_Q6_K ? 210 : 144);
                const int64_t row_bytes = attrs.get_or<int64_t>("row_bytes", dense);
                if (cols % 256 != 0 || row_bytes != dense)
                    throw std::runtime_error("CUDA MATMUL needs whole 256-value super-blocks in contiguous rows");
                const void* w = packs_->get(inputs[0].raw_data(), type, rows, cols, stream_);
                const float* x = static_cast<const float*>(inputs[1].raw_data());
                if (T > 1)
                    check(af_prefill_gemm_f32(y, w, type, x, rows, cols, static_cast<int>(T), stream_),
                          "af_prefill_gemm_f32");
                else
                    check(af_gemv_f32(y, w, type, x, rows, cols, stream_), "af_gemv_f32");
                break;
            }
            default:
                throw std::runtime_error("B200Kernel::execute: unsupported op");
        }
    }

private:
    OpType op_;
    cudaStream_t stream_{};
    PackCache* packs_;
};

class B200Backend final : public IBackend {
public:
    B200Backend() = default;
    ~B200Backend() override { finalize(); }

    std::string_view name() const noexcept override { return "cuda"; }
    DeviceId device_id() const noexcept override { return DeviceId::cuda(device_); }

    bool initialize() override {
        if (initialized_) return true;
        int count = 0;
        if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) return false;
        check(cudaSetDevice(device_), "cudaSetDevice");
        check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreateWithFlags");
        initialized_ = true;
        return true;
    }

    void finalize() override {
        packs_.clear();
        if (stream_) {
            cudaStreamDestroy(stream_);
            stream_ = nullptr;
        }
        initialized_ = false;
    }

    std::shared_ptr<TensorStorage> allocate(size_t bytes, size_t) override {
        return std::make_shared<DeviceStorage>(bytes, device_);
    }

    void transfer(const Tensor& src, Tensor& dst) override {
        const size_t bytes = tensor_bytes(src);
        if (bytes != tensor_bytes(dst)) throw std::runtime_error("B200Backend::transfer: size mismatch");
        check(cudaMemcpyAsync(dst.raw_data(), src.raw_data(), bytes, cudaMemcpyDefault, stream_),
              "cudaMemcpyAsync");
        synchronize();
    }

    void synchronize() override {
        if (stream_) check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
    }

    bool can_handle(OpType op, std::span<const DType> in) const override {
        switch (op) {
            case OpType::RMS_NORM:
            case OpType::SILU:
            case OpType::MUL:
            case OpType::ROPE:
                return in.empty() || in[0] == DType::F32;
            case OpType::MATMUL:
                return in.size() >= 2 && (in[0] == DType::Q4_K_M || in[0] == DType::Q6_K) && in[1] == DType::F32;
            default:
                return false;
        }
    }

    std::unique_ptr<IKernel> get_kernel(OpType op, std::span<const DType> in, const AttributeMap&) override {
        if (!can_handle(op, in))
            throw std::runtime_error("B200Backend::get_kernel: unsupported op/dtype combination");
        return std::make_unique<B200Kernel>(op, stream_, &packs_);
    }

private:
    bool initialized_{false};
    int device_{0};
    cudaStream_t stream_{};
    PackCache packs_;
};

}  // namespace
}  // namespace axonforge::b200

[[gnu::constructor]] static void axonforge_register_b200_backend() {
    ::axonforge::BackendRegistry::instance().register_backend(
        "cuda", []() -> std::unique_ptr<::axonforge::IBackend> {
            return std::make_unique<::axonforge::b200::B200Backend>();
        });
}
