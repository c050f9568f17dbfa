// af_ops.cuh — internal declarations shared by the engine and the launchers.
#pragma once
#include <string>

#include "af_common.cuh"
#include "af_gemv.cuh"

namespace af {

void set_last_error(const std::string& s);
int num_sms();
int gemv_grid();

cudaError_t weight_pack(void* d_dst, const void* d_src, int type, int rows, int cols, bool unpack, cudaStream_t st);
cudaError_t embed_launch(float* x, const uint8_t* W, int type, int cols, int row_stride, const int* token,
                         unsigned long long* argmax, uint8_t* xq, const float* xq_norm_w, cudaStream_t st,
                         bool pdl);

// Decode attention (af_attention.cu).
struct AttnParams {
    const float* q;        // [Hl*hd] projected (biased) queries
    const float* k;        // [KVl*hd] new key (before RoPE)
    const float* v;        // [KVl*hd] new value
    float* kc;             // layer K cache [n_ctx][KVl*hd]
    float* vc;             // layer V cache
    float* out;            // [Hl*hd]
    const float* cos_t;    // [n_ctx][hd/2]
    const float* sin_t;
    const float* q_norm;   // optional per-head RMSNorm weights [hd]
    const float* k_norm;
    float* part;           // scratch [Hl][nsplit][hd + 2]
    unsigned int* counter; // scratch [KVl], zero between launches
    const int* pos;        // device position of the new token
    int n_heads, n_kv_heads, head_dim, n_ctx, nsplit, qk_norm_order;
    float eps, scale;
    uint8_t* xq_out;       // optional: quantised copy of `out` for the next GEMV
};

cudaError_t attention_init();
cudaError_t attention_launch(const AttnParams& p, cudaStream_t st, bool pdl);
int attention_smem_bytes(const AttnParams& p);

// Argmax finalize: packed key -> token id, pos++ (af_attention.cu).
cudaError_t finalize_launch(const unsigned long long* key, int* token, int* pos, int* hist, cudaStream_t st,
                            bool pdl);

}  // namespace af
