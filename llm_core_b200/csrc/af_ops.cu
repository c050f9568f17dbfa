// af_ops.cu — C-ABI kernel launchers and the small decode kernels: Q6_K
// regroup, embedding-row dequant, and the reference CUDA backend's op set
// (RMSNorm, SiLU, Mul, RoPE; src/backend/cuda/cuda_kernels.hpp:8-19).
#include <cstdlib>
#include <mutex>
#include <string>

#include "af_gemv.cuh"
#include "af_ops.cuh"

namespace af {

thread_local std::string g_last_error;

void set_last_error(const std::string& s) { g_last_error = s; }

// CTAs per SM of the GEMV grid (AF_GEMV_CTAS_PER_SM, default 1).
int gemv_grid() {
    static int per_sm = [] {
        const char* v = std::getenv("AF_GEMV_CTAS_PER_SM");
        const int n = v ? std::atoi(v) : 1;
        return n < 1 ? 1 : (n > 4 ? 4 : n);
    }();
    return num_sms() * per_sm;
}

int num_sms() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

// ------------------------------------------------------- packed weight layout

// One CTA per unit (16-row tile × super-block): every output byte of the
// unit gathered from the GGUF rows (padding rows past `rows` are zero);
// `unpack` writes the GGUF bytes back from the unit (the inverse map).
__device__ __forceinline__ uint8_t q6_gguf_value(const uint8_t* blk, int k) {
    // 6-bit value k of a GGUF Q6_K block (q6k_row_to_f32, llama_model.cpp:560-592)
    const int n = k >> 7, kk = k & 127, s = kk >> 5, l = kk & 31;
    const int qlb = blk[64 * n + l + ((s & 1) ? 32 : 0)];
    const int lo = (s & 2) ? (qlb >> 4) : (qlb & 0xF);
    const int hi = (blk[128 + 32 * n + l] >> (2 * s)) & 3;
    return (uint8_t)(lo | (hi << 4));
}

__global__ void pack_kernel(uint8_t* __restrict__ packed, uint8_t* __restrict__ gguf, int type, int rows, int nb,
                            int unpack) {
    const int tile = blockIdx.x, b = blockIdx.y;
    const bool q6 = type == AF_GGML_Q6_K;
    const int BB = q6 ? 210 : 144, UB = 16 * BB;
    uint8_t* unit = packed + ((size_t)tile * nb + b) * UB;
    auto src_blk = [&](int r) { return gguf + ((size_t)(tile * 16 + r) * nb + b) * BB; };
    if (!unpack) {
        for (int o = threadIdx.x; o < UB; o += blockDim.x) {
            int r, v = 0;
            if (!q6) {
                if (o < kQ4Hdr) {
                    const int c = o >> 9, lane = (o >> 4) & 31, e = (o >> 2) & 3, i = o & 3;
                    r = (lane >> 2) + 8 * (e & 1);
                    const int w = (lane & 3) + 4 * (e >> 1);
                    if (tile * 16 + r < rows) v = src_blk(r)[16 + 32 * c + 4 * w + i];
                } else {
                    r = (o - kQ4Hdr) >> 4;
                    if (tile * 16 + r < rows) v = src_blk(r)[(o - kQ4Hdr) & 15];
                }
            } else if (o < kQ6Sc) {
                const int part = o < kQ6Hi ? 0 : 1, oo = part ? o - kQ6Hi : o;
                const int blkq = oo >> 9, lane = (oo >> 4) & 31, e = (oo >> 2) & 3, i = oo & 3;
                r = (lane >> 2) + 8 * (e & 1);
                const int w = (lane & 3) + 4 * (e >> 1);
                if (tile * 16 + r < rows) {
                    const uint8_t* blk = src_blk(r);
                    if (!part) {
                        const int k = 64 * blkq + 4 * w + i;
                        v = (q6_gguf_value(blk, k) & 0xF) | ((q6_gguf_value(blk, k + 32) & 0xF) << 4);
                    } else {
                        for (int sx = 0; sx < 4; ++sx)
                            v |= ((q6_gguf_value(blk, 128 * blkq + 32 * sx + 4 * w + i) >> 4) & 3) << (2 * sx);
                    }
                }
            } else if (o < kQ6D) {
                r = (o - kQ6Sc) >> 4;
                if (tile * 16 + r < rows) v = src_blk(r)[192 + ((o - kQ6Sc) & 15)];
            } else {
                r = (o - kQ6D) >> 1;
                if (tile * 16 + r < rows) v = src_blk(r)[208 + ((o - kQ6D) & 1)];
            }
            unit[o] = (uint8_t)v;
        }
        return;
    }
    // unpack: GGUF byte j of row r's block b
    for (int idx = threadIdx.x; idx < 16 * BB; idx += blockDim.x) {
        const int r = idx / BB, j = idx % BB;
        if (tile * 16 + r >= rows) continue;
        int v;
        if (!q6) {
            if (j < 16) {
                v = unit[kQ4Hdr + 16 * r + j];
            } else {
                const int c = (j - 16) >> 5, l = (j - 16) & 31;
                v = unit[c * 512 + packed_frag_off(r, l >> 2, l & 3)];
            }
        } else if (j < 128) {
            const int n = j >> 6, l = j & 63;
            const int k = 128 * n + l;  // low nibble value k, high nibble value k + 64
            v = (packed_q6_value(unit, r, k) & 0xF) | ((packed_q6_value(unit, r, k + 64) & 0xF) << 4);
        } else if (j < 192) {
            const int n = (j - 128) >> 5, l = (j - 128) & 31;
            v = 0;
            for (int sx = 0; sx < 4; ++sx) v |= ((packed_q6_value(unit, r, 128 * n + 32 * sx + l) >> 4) & 3) << (2 * sx);
        } else if (j < 208) {
            v = unit[kQ6Sc + 16 * r + (j - 192)];
        } else {
            v = unit[kQ6D + 2 * r + (j - 208)];
        }
        src_blk(r)[j] = (uint8_t)v;
    }
}

cudaError_t weight_pack(void* d_dst, const void* d_src, int type, int rows, int cols, bool unpack,
                        cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    const int nb = cols / 256;
    if (!unpack) AF_CUDA_TRY(cudaMemsetAsync(d_dst, 0, packed_bytes(type, rows, cols), st));
    uint8_t* packed = static_cast<uint8_t*>(unpack ? const_cast<void*>(d_src) : d_dst);
    uint8_t* gg = static_cast<uint8_t*>(unpack ? d_dst : const_cast<void*>(d_src));
    const dim3 grid((rows + kPackTile - 1) / kPackTile, nb);
    pack_kernel<<<grid, 256, 0, st>>>(packed, gg, type, rows, nb, unpack ? 1 : 0);
    return cudaGetLastError();
}

// --------------------------------------------------------- embedding lookup

// x[0:cols] = dequant(row `*token` of W): emb_lookup (src/models/llama_model.cpp:882-934)
// for Q4_K (GGUF rows) and Q6_K (regrouped rows).  Also resets the argmax
// key for the step (this is the step's first kernel).
__global__ void embed_kernel(float* __restrict__ x, const uint8_t* __restrict__ W, int type, int cols,
                             int row_stride, const int* __restrict__ token, unsigned long long* argmax,
                             uint8_t* xq, const float* xq_norm_w, int q8) {
    pdl_launch_dependents();
    pdl_wait();
    if (argmax && blockIdx.x == 0 && threadIdx.x == 0) *argmax = 0ull;
    const int nb = cols / 256;
    for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < cols; v += gridDim.x * blockDim.x) {
        x[v] = embed_value(W, type, nb, row_stride, *token, v);
    }
    if (xq) {
        // quantise this block's values (one 32-value group per warp) for the first GEMV
        __threadfence();
        __syncthreads();
        const int g = (blockIdx.x * blockDim.x) / 32 + (threadIdx.x >> 5);
        if (g < cols / 32) xq_quantize_group(xq, x, xq_norm_w, cols, g, q8 != 0);
    }
}

cudaError_t embed_launch(float* x, const uint8_t* W, int type, int cols, int row_stride, const int* token,
                         unsigned long long* argmax, uint8_t* xq, const float* xq_norm_w, cudaStream_t st,
                         bool pdl, bool q8) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((cols + 255) / 256);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, embed_kernel, x, W, type, cols, row_stride, token, argmax, xq, xq_norm_w,
                              q8 ? 1 : 0);
}

// -------------------------------------------------- reference CUDA op set

__global__ void rms_norm_kernel(float* __restrict__ y, const float* __restrict__ x, const float* __restrict__ w,
                                int n, float eps) {
    __shared__ float red[32];
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss += x[i] * x[i];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
    const float s = 1.f / sqrtf(tot / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = w[i] * (x[i] * s);
}

__global__ void silu_kernel(float* y, const float* x, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = x[i] / (1.f + expf(-x[i]));
}

__global__ void mul_kernel(float* y, const float* a, const float* b, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = a[i] * b[i];
}

// freq = 1/theta^(2i/hd), angle = pos*freq (RopeCache::build,
// src/models/llama_model.cpp:1024-1043); half-split pairs (i, i + hd/2).
__global__ void rope_kernel(float* q, int n_heads, int head_dim, int pos, float theta) {
    const int half = head_dim / 2;
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n_heads * half) return;
    const int h = idx / half, i = idx % half;
    const float freq = 1.f / powf(theta, (float)(2 * i) / (float)head_dim);
    const float ang = (float)pos * freq;
    const float c = cosf(ang), s = sinf(ang);
    float* hp = q + (size_t)h * head_dim;
    const float x0 = hp[i], x1 = hp[i + half];
    hp[i] = x0 * c - x1 * s;
    hp[i + half] = x0 * s + x1 * c;
}

}  // namespace af

using namespace af;

extern "C" {

const char* af_last_error(void) { return g_last_error.c_str(); }

cudaError_t af_device_error(int* h_code, int clear) {
    AF_CUDA_TRY(cudaMemcpyFromSymbol(h_code, g_err, sizeof(int)));
    if (clear) {
        const int z = 0;
        AF_CUDA_TRY(cudaMemcpyToSymbol(g_err, &z, sizeof(int)));
    }
    return cudaSuccess;
}

size_t af_row_stride(int ggml_type, int cols) {
    if (cols <= 0 || cols % 256) return 0;
    if (ggml_type == AF_GGML_Q4_K || ggml_type == AF_GGML_Q6_K) return (size_t)dev_row_stride(ggml_type, cols);
    if (ggml_type == AF_GGML_F32) return (size_t)cols * 4;
    return 0;
}

size_t af_weight_bytes(int ggml_type, int rows, int cols) {
    if (cols <= 0 || cols % 256 || rows < 0 || (ggml_type != AF_GGML_Q4_K && ggml_type != AF_GGML_Q6_K)) return 0;
    return packed_bytes(ggml_type, rows, cols);
}

cudaError_t af_weight_pack(void* d_dst, const void* d_src, int ggml_type, int rows, int cols, cudaStream_t stream) {
    if (!af_weight_bytes(ggml_type, rows, cols)) return cudaErrorInvalidValue;
    return weight_pack(d_dst, d_src, ggml_type, rows, cols, false, stream);
}

cudaError_t af_weight_unpack(void* d_dst, const void* d_src, int ggml_type, int rows, int cols, cudaStream_t stream) {
    if (!af_weight_bytes(ggml_type, rows, cols)) return cudaErrorInvalidValue;
    return weight_pack(d_dst, d_src, ggml_type, rows, cols, true, stream);
}

cudaError_t af_gemv_f32(float* d_y, const void* d_w, int ggml_type, const float* d_x, int rows, int cols,
                        cudaStream_t stream) {
    if ((ggml_type != AF_GGML_Q4_K && ggml_type != AF_GGML_Q6_K) || cols <= 0 || cols % 256 || rows < 0) {
        set_last_error("af_gemv_f32: need Q4_K/Q6_K weights and cols % 256 == 0");
        return cudaErrorInvalidValue;
    }
    if (cols > kGemvMaxK) {
        set_last_error("af_gemv_f32: cols > 12288 is not supported");
        return cudaErrorInvalidValue;
    }
    if ((reinterpret_cast<uintptr_t>(d_w) & 15) || (reinterpret_cast<uintptr_t>(d_x) & 15)) {
        set_last_error("af_gemv_f32: weights and x must be 16-byte aligned");
        return cudaErrorInvalidValue;
    }
    if (rows == 0) return cudaSuccess;
    GemvParams p = {};
    p.seg[0].w = static_cast<const uint8_t*>(d_w);
    p.seg[0].y = d_y;
    p.seg[0].type = ggml_type;
    p.seg[0].rows = rows;
    p.seg[0].row_stride = dev_row_stride(ggml_type, cols);
    p.nseg = 1;
    p.K = cols;
    p.x = d_x;
    p.epi = EPI_STORE;
    gemv_configure(p, gemv_grid());
    AF_CUDA_TRY(gemv_init());
    return gemv_launch(p, stream, false);
}

// Packed copy of the last raw matrix af_q4km_gemv_f32 was given, grown on
// demand (cudaMalloc: not during stream capture; calls on one device share it).
namespace {
std::mutex g_raw_mu;
int g_raw_dev = -1;
void* g_raw_packed = nullptr;
size_t g_raw_bytes = 0;
}  // namespace

cudaError_t af_q4km_gemv_f32(float* d_y, const uint8_t* d_w, const float* d_x, int rows, int cols, size_t row_bytes,
                             cudaStream_t stream) {
    if (cols <= 0 || cols % 256 || rows < 0 || cols > kGemvMaxK ||
        row_bytes != (size_t)dev_row_stride(AF_GGML_Q4_K, cols)) {
        set_last_error("af_q4km_gemv_f32: need cols % 256 == 0, cols <= 12288 and row_bytes == cols/256*144");
        return cudaErrorInvalidValue;
    }
    if ((reinterpret_cast<uintptr_t>(d_w) & 15) || (reinterpret_cast<uintptr_t>(d_x) & 15)) {
        set_last_error("af_q4km_gemv_f32: weights and x must be 16-byte aligned");
        return cudaErrorInvalidValue;
    }
    if (rows == 0) return cudaSuccess;
    int dev = 0;
    AF_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(g_raw_mu);
    const size_t need = packed_bytes(AF_GGML_Q4_K, rows, cols);
    if (g_raw_dev != dev) {
        g_raw_dev = dev;
        g_raw_packed = nullptr;  // a buffer of another device is not reused (it leaks with the process)
        g_raw_bytes = 0;
    }
    if (g_raw_bytes < need) {
        if (g_raw_packed) AF_CUDA_TRY(cudaFree(g_raw_packed));
        g_raw_packed = nullptr;
        g_raw_bytes = 0;
        AF_CUDA_TRY(cudaMalloc(&g_raw_packed, need));
        g_raw_bytes = need;
    }
    AF_CUDA_TRY(weight_pack(g_raw_packed, d_w, AF_GGML_Q4_K, rows, cols, false, stream));
    return af_gemv_f32(d_y, g_raw_packed, AF_GGML_Q4_K, d_x, rows, cols, stream);
}

cudaError_t af_gemv_q8_f32(float* d_y, const void* d_w, int ggml_type, const float* d_x, int rows, int cols,
                           cudaStream_t stream) {
    if ((ggml_type != AF_GGML_Q4_K && ggml_type != AF_GGML_Q6_K) || cols <= 0 || cols % 256 || rows < 0 ||
        cols > kGemvMaxK) {
        set_last_error("af_gemv_q8_f32: need Q4_K/Q6_K weights, cols % 256 == 0, cols <= 12288");
        return cudaErrorInvalidValue;
    }
    if ((reinterpret_cast<uintptr_t>(d_w) & 15) || (reinterpret_cast<uintptr_t>(d_x) & 15)) {
        set_last_error("af_gemv_q8_f32: weights and x must be 16-byte aligned");
        return cudaErrorInvalidValue;
    }
    if (rows == 0) return cudaSuccess;
    GemvParams p = {};
    p.seg[0].w = static_cast<const uint8_t*>(d_w);
    p.seg[0].y = d_y;
    p.seg[0].type = ggml_type;
    p.seg[0].rows = rows;
    p.seg[0].row_stride = dev_row_stride(ggml_type, cols);
    p.nseg = 1;
    p.K = cols;
    p.x = d_x;
    p.epi = EPI_STORE;
    p.q8 = 1;
    gemv_configure(p, gemv_grid());
    AF_CUDA_TRY(gemv_init());
    return gemv_launch(p, stream, false);
}

cudaError_t af_gemv_fused(const af_gemv_fused_args* a, cudaStream_t stream) {
    if (!a || a->nseg < 1 || a->nseg > 3 || a->cols <= 0 || a->cols % 256 || a->cols > kGemvMaxK || !a->x) {
        set_last_error("af_gemv_fused: need 1..3 segments, cols % 256 == 0, cols <= 12288");
        return cudaErrorInvalidValue;
    }
    if (a->epi < AF_EPI_STORE || a->epi > AF_EPI_ARGMAX || (a->epi == AF_EPI_SWIGLU && a->nseg != 2) ||
        (a->epi == AF_EPI_RESID && (!a->resid || a->nseg != 1)) || (a->epi == AF_EPI_ARGMAX && (!a->argmax || a->nseg != 1))) {
        set_last_error("af_gemv_fused: epilogue / segment combination not supported");
        return cudaErrorInvalidValue;
    }
    GemvParams p = {};
    for (int s = 0; s < a->nseg; ++s) {
        if ((a->type[s] != AF_GGML_Q4_K && a->type[s] != AF_GGML_Q6_K) || a->rows[s] < 0 ||
            (reinterpret_cast<uintptr_t>(a->w[s]) & 15)) {
            set_last_error("af_gemv_fused: bad segment");
            return cudaErrorInvalidValue;
        }
        p.seg[s].w = static_cast<const uint8_t*>(a->w[s]);
        p.seg[s].y = a->y[s];
        p.seg[s].bias = a->bias[s];
        p.seg[s].type = a->type[s];
        p.seg[s].rows = a->rows[s];
        p.seg[s].row_stride = dev_row_stride(a->type[s], a->cols);
    }
    if (a->epi == AF_EPI_SWIGLU && (a->rows[0] != a->rows[1] || a->type[0] != a->type[1])) {
        set_last_error("af_gemv_fused: SwiGLU needs gate/up of equal rows and type");
        return cudaErrorInvalidValue;
    }
    p.nseg = a->nseg;
    p.K = a->cols;
    p.x = a->x;
    p.x_add = a->x_add;
    p.x_store = a->x_store;
    p.norm_w = a->norm_w;
    p.eps = a->eps;
    p.epi = a->epi;
    p.resid = a->resid;
    p.argmax = a->argmax;
    p.argmax_base = a->argmax_base;
    gemv_configure(p, gemv_grid());
    AF_CUDA_TRY(gemv_init());
    return gemv_launch(p, stream, false);
}

cudaError_t af_attention_decode_f32(float* d_out, const float* d_q, const float* d_k, const float* d_v,
                                    float* d_kcache, float* d_vcache, const float* d_cos, const float* d_sin,
                                    const float* d_q_norm, const float* d_k_norm, const int* d_pos, int n_heads,
                                    int n_kv_heads, int head_dim, int n_ctx, int qk_norm_order, float eps,
                                    int nsplit, float* d_part, unsigned int* d_counter, cudaStream_t stream) {
    if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || nsplit <= 0 || n_ctx <= 0) {
        set_last_error("af_attention_decode_f32: bad shape");
        return cudaErrorInvalidValue;
    }
    AttnParams p = {};
    p.q = d_q; p.k = d_k; p.v = d_v; p.kc = d_kcache; p.vc = d_vcache; p.out = d_out;
    p.cos_t = d_cos; p.sin_t = d_sin; p.q_norm = d_q_norm; p.k_norm = d_k_norm;
    p.part = d_part; p.counter = d_counter; p.pos = d_pos;
    p.n_heads = n_heads; p.n_kv_heads = n_kv_heads; p.head_dim = head_dim; p.n_ctx = n_ctx;
    p.nsplit = nsplit; p.qk_norm_order = qk_norm_order; p.eps = eps;
    p.scale = 1.f / sqrtf((float)head_dim);
    AF_CUDA_TRY(attention_init());
    return attention_launch(p, stream, false);
}

cudaError_t af_rms_norm_f32(float* d_y, const float* d_x, const float* d_w, int n, float eps, cudaStream_t stream) {
    if (n <= 0) return cudaErrorInvalidValue;
    rms_norm_kernel<<<1, 1024, 0, stream>>>(d_y, d_x, d_w, n, eps);
    return cudaGetLastError();
}

cudaError_t af_silu_f32(float* d_y, const float* d_x, int n, cudaStream_t stream) {
    if (n <= 0) return n == 0 ? cudaSuccess : cudaErrorInvalidValue;
    silu_kernel<<<(n + 255) / 256, 256, 0, stream>>>(d_y, d_x, n);
    return cudaGetLastError();
}

cudaError_t af_mul_f32(float* d_y, const float* d_a, const float* d_b, int n, cudaStream_t stream) {
    if (n <= 0) return n == 0 ? cudaSuccess : cudaErrorInvalidValue;
    mul_kernel<<<(n + 255) / 256, 256, 0, stream>>>(d_y, d_a, d_b, n);
    return cudaGetLastError();
}

cudaError_t af_rope_f32(float* d_q, int n_heads, int head_dim, int pos, float theta, cudaStream_t stream) {
    if (n_heads <= 0 || head_dim <= 0 || head_dim % 2) return cudaErrorInvalidValue;
    const int n = n_heads * head_dim / 2;
    rope_kernel<<<(n + 127) / 128, 128, 0, stream>>>(d_q, n_heads, head_dim, pos, theta);
    return cudaGetLastError();
}

}  // extern "C"
