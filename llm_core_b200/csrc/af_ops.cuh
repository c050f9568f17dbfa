// af_ops.cuh — internal declarations shared by the engine and the launchers.
#pragma once
#include <string>

#include "af_common.cuh"
#include "af_gemv.cuh"

namespace af {

void set_last_error(const std::string& s);
int num_sms();
int gemv_grid();

// Byte offset, inside a 512-byte fragment block of a unit, of byte i of
// word w (of a 32-byte chunk) of tile row r (see af_gemv.cuh).
__host__ __device__ inline int packed_frag_off(int r, int w, int i) {
    const int lane = 4 * (r & 7) + (w & 3), e = (r >> 3) + 2 * (w >> 2);
    return lane * 16 + e * 4 + i;
}

// 6-bit value k (0..255) of tile row r of a packed Q6_K unit.
__host__ __device__ inline int packed_q6_value(const uint8_t* unit, int r, int k) {
    const int P = k >> 6, kk = k & 63, l = kk & 31;
    const int lo = unit[P * 512 + packed_frag_off(r, l >> 2, l & 3)];
    const int Q = k >> 7, s = (k & 127) >> 5;
    const int hi = unit[kQ6Hi + Q * 512 + packed_frag_off(r, l >> 2, l & 3)];
    return ((kk >= 32 ? lo >> 4 : lo) & 0xF) | (((hi >> (2 * s)) & 3) << 4);
}

// Value v of packed row `tok` of an embedding matrix (nb super-blocks per
// row), dequantised as emb_lookup does (src/models/llama_model.cpp:882-934).
__device__ __forceinline__ float embed_value(const uint8_t* __restrict__ W, int type, int nb, int row_stride, int tok,
                                             int v) {
    const int b = v >> 8, k = v & 255, r = tok & (kPackTile - 1);
    const uint8_t* unit = W + (size_t)(tok / kPackTile) * kPackTile * row_stride + (size_t)b * unit_bytes(type);
    if (type == AF_GGML_Q6_K) {
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(unit + kQ6D + 2 * r));
        const int sc = (int8_t)unit[kQ6Sc + 16 * r + (k >> 4)];
        return d * sc * (packed_q6_value(unit, r, k) - 32);
    }
    const uint8_t* hdr = unit + kQ4Hdr + 16 * r;
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(hdr));
    const float dmin = half_bits_to_float(*reinterpret_cast<const uint16_t*>(hdr + 2));
    const uint8_t* sc = hdr + 4;
    const int chunk = k >> 6, rr = k & 63, j = chunk * 2 + (rr >> 5), l = rr & 31;
    int s, m;
    if (j < 4) {
        s = sc[j] & 63;
        m = sc[j + 4] & 63;
    } else {
        s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
    const int qb = unit[chunk * 512 + packed_frag_off(r, l >> 2, l & 3)];
    const int q = (rr < 32) ? (qb & 0xF) : (qb >> 4);
    return (d * s) * q - dmin * m;
}

cudaError_t weight_pack(void* d_dst, const void* d_src, int type, int rows, int cols, bool unpack, cudaStream_t st);
cudaError_t embed_launch(float* x, const uint8_t* W, int type, int cols, int row_stride, const int* token,
                         unsigned long long* argmax, uint8_t* xq, const float* xq_norm_w, cudaStream_t st,
                         bool pdl, bool q8 = false);

// Prefill (af_prefill.cu): the tcgen05 dequant-GEMM Y[T][rows] = X[T][cols]·Wᵀ
// and the row kernels of the batched prompt pass.
// Batched dequant GEMV (af_bgemv.cu): y[B][rows] for 1 <= B <= 32 vectors.
cudaError_t bgemv_launch(float* y, const uint8_t* w, int type, const float* x, int rows, int cols, int B,
                         cudaStream_t st);
bool bgemv_supported(int n_vec);
cudaError_t prefill_gemm_launch(float* y, const uint8_t* w, int type, const float* x, int rows, int cols, int T,
                                cudaStream_t st);
// Batched prompt attention (af_prefill.cu): per-head norms + RoPE of q/k,
// K/V rows stored at positions pos0.., then causal attention of the T tokens
// (head_dim 64 or 128).
bool prompt_attention_supported(int hd);
cudaError_t prompt_attention_launch(float* q, const float* k, const float* v, float* kc, float* vc, float* out,
                                   const float* cos_t, const float* sin_t, const float* q_norm, const float* k_norm,
                                   int T, int pos0, int H, int KV, int hd, int qk_order, float eps, cudaStream_t st);
cudaError_t prompt_embed_launch(float* x, const uint8_t* W, int type, int cols, int row_stride, const int* tokens,
                                int T, cudaStream_t st);
cudaError_t rows_rmsnorm_launch(float* y, const float* x, const float* w, int n, int T, float eps, cudaStream_t st);
cudaError_t rows_bias_launch(float* y, const float* b, int n, int T, cudaStream_t st);
cudaError_t rows_swiglu_launch(float* g, const float* u, long long count, cudaStream_t st);
cudaError_t rows_add_launch(float* x, const float* y, long long count, cudaStream_t st);

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
    unsigned long long* tpart;  // step kernel: tagged split partials [Hl][nsplit][hd + 2]
    const int* pos;        // device position of the new token
    int n_heads, n_kv_heads, head_dim, n_ctx, nsplit, qk_norm_order;
    float eps, scale;
    uint8_t* xq_out;       // optional: quantised copy of `out` for the next GEMV
    int q8;                // xq_out as Q8_0 blocks (see xq_store32w)
};

cudaError_t attention_init();
cudaError_t attention_launch(const AttnParams& p, cudaStream_t st, bool pdl);
int attention_smem_bytes(const AttnParams& p);

// Device sampling step (af_sample.cu).
cudaError_t sample_launch(float* d_logits, int vocab, const int* d_window, int n_window, const af_sampling& s, float r,
                          int* d_out, cudaStream_t st);
bool sample_supported(const af_sampling& s, int vocab, std::string* why);

// Argmax finalize: packed key -> token id, pos++ (af_attention.cu).
cudaError_t finalize_launch(const unsigned long long* key, int* token, int* pos, int* hist, cudaStream_t st,
                            bool pdl);

}  // namespace af
