// af_ops.cuh — internal declarations shared by the engine and the launchers.
#pragma once
#include <string>

#include "af_common.cuh"
#include "af_gemv.cuh"

namespace af {

void set_last_error(const std::string& s);
int num_sms();
int gemv_grid();

// Byte offset of (row, stage st) in the packed layout (see af_gemv.cuh).
__host__ __device__ inline size_t packed_off(int type, int nb, int row_stride, int row, int st) {
    const int nbs = min(8, nb - st * 8);
    const int seg = type == AF_GGML_Q6_K ? nbs * 208 + 16 : nbs * 144;
    const int full = type == AF_GGML_Q6_K ? 1680 : 1152;
    return (size_t)(row / kPackTile) * kPackTile * row_stride + (size_t)kPackTile * st * full +
           (size_t)(row % kPackTile) * seg;
}

// Value v of packed row `tok` of an embedding matrix (nb super-blocks per
// row), dequantised as emb_lookup does (src/models/llama_model.cpp:882-934).
__device__ __forceinline__ float embed_value(const uint8_t* __restrict__ W, int type, int nb, int row_stride, int tok,
                                             int v) {
    const int b = v >> 8, w = v & 255;
    const int st = b >> 3, k = b & 7, nbs = min(8, nb - st * 8);
    const uint8_t* seg = W + packed_off(type, nb, row_stride, tok, st);
    if (type == AF_GGML_Q6_K) {
        const uint8_t* blk = seg + k * 208;
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(seg + nbs * 208 + 2 * k));
        const int n = w >> 7, r = w & 127, s = r >> 5, l = r & 31;
        const uint8_t* ql = blk + 64 * n;
        const uint8_t* qh = blk + 128 + 32 * n;
        const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192 + 8 * n);
        const int qlb = (s & 1) ? ql[l + 32] : ql[l];
        const int nib = (s & 2) ? (qlb >> 4) : (qlb & 0xF);
        const int q = (nib | (((qh[l] >> (2 * s)) & 3) << 4)) - 32;
        return d * sc[(l >> 4) + 2 * s] * q;
    }
    const uint8_t* blk = seg + k * 144;
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(blk));
    const float dmin = half_bits_to_float(*reinterpret_cast<const uint16_t*>(blk + 2));
    const uint8_t* sc = blk + 4;
    const int chunk = w >> 6, r = w & 63, j = chunk * 2 + (r >> 5), l = r & 31;
    int s, m;
    if (j < 4) {
        s = sc[j] & 63;
        m = sc[j + 4] & 63;
    } else {
        s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
    const int qb = blk[16 + chunk * 32 + l];
    const int q = (r < 32) ? (qb & 0xF) : (qb >> 4);
    return (d * s) * q - dmin * m;
}

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
