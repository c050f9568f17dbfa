/*
 * af_b200.h — C ABI of the B200 (sm_100a) decode path for AxonForge
 * (songqiuyu/llm_core).
 *
 * Plain pointers, sizes and a cudaStream_t; no C++ or torch types cross this
 * boundary.  Every function returns cudaSuccess (0) or an error code and never
 * throws.  Device pointers are marked `d_`; host pointers `h_`.
 *
 * Two layers:
 *   1. Kernel launchers — the op set of the reference CUDA backend
 *      (src/backend/cuda/cuda_kernels.hpp:8-19) plus the Q6_K GEMV it lacks.
 *   2. The decode engine — the GPU-resident replacement of
 *      llama_cuda_generate (include/axonforge/models/llama_cuda.hpp:25-28):
 *      weights uploaded byte-for-byte, fp32 KV cache on the device, one
 *      persistent kernel per decode step (captured in a CUDA graph), device
 *      sampling, optional tensor parallelism over NVLink peer memory.
 *
 * Weight layout on the device ("packed"): the GGUF super-blocks, byte for byte,
 * permuted once at upload by af_weight_pack so that every pipeline stage of the
 * GEMV is one contiguous range.  Rows are grouped in tiles of 16 (the last tile
 * zero-padded); a tile holds, stage after stage, the 16 rows' segments of 8
 * super-blocks (the last stage fewer).  A Q4_K segment is its 144-byte blocks
 * unchanged; a Q6_K segment is each block's ql/qh/scales (208 bytes) followed
 * by the blocks' f16 d values padded to 16 bytes, so every segment starts on a
 * 16-byte boundary.
 */
#ifndef AF_B200_H
#define AF_B200_H

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml tensor type ids used on this path (include/axonforge/dtype.hpp:80-96). */
#define AF_GGML_F32 0
#define AF_GGML_Q4_K 12
#define AF_GGML_Q6_K 14

/* ------------------------------------------------------------------ status */

/* Text of the last host-side error on this thread ("" if none). */
const char* af_last_error(void);

/* Device error word (0 = none).  Kernels never trap: a bounded wait that runs
 * out writes a code here and returns.  `clear` != 0 resets it. */
cudaError_t af_device_error(int* h_code, int clear);

/* ---------------------------------------------------------- weight layout */

/* Bytes of one packed row of `cols` values (Q4_K: cols/256*144; Q6_K:
 * cols/256*210), 0 for unsupported arguments. */
size_t af_row_stride(int ggml_type, int cols);
/* Device bytes of a packed rows x cols matrix (whole 16-row tiles). */
size_t af_weight_bytes(int ggml_type, int rows, int cols);

/* Pack `rows` GGUF rows (d_src, contiguous GGUF bytes) of a Q4_K or Q6_K
 * matrix into the packed layout at d_dst (af_weight_bytes bytes).
 * A bit-preserving permutation (Q4_K: of bytes; Q6_K: of the 6-bit values'
 * nibble and 2-bit fields); af_weight_unpack inverts it. */
cudaError_t af_weight_pack(void* d_dst, const void* d_src, int ggml_type, int rows, int cols,
                           cudaStream_t stream);
cudaError_t af_weight_unpack(void* d_dst, const void* d_src, int ggml_type, int rows, int cols,
                             cudaStream_t stream);

/* ------------------------------------------------------- kernel launchers */

/* y[rows] = W · x with W packed (af_weight_pack) and f32 x[cols]: the fused
 * dequant GEMV (fp32 accumulation).  Replaces q4km_gemv_f32
 * (src/backend/cuda/cuda_kernels.hpp:13-19, numerically wrong in the
 * reference) and adds Q6_K.  Parity target: gemv_q4k_avx2_range /
 * gemv_q6k_avx2_range (src/backend/cpu_x86/kernels/gemv_q4k_avx2.cpp:230-238,
 * gemv_q6k_avx2.cpp:235-243).  cols % 256 == 0. */
cudaError_t af_gemv_f32(float* d_y, const void* d_w, int ggml_type, const float* d_x, int rows,
                        int cols, cudaStream_t stream);

/* The reference CUDA backend's GEMV entry with its exact arguments:
 * q4km_gemv_f32(y, w, x, rows, cols, row_bytes, stream)
 * (src/backend/cuda/cuda_kernels.hpp:13-19, called for MATMUL by
 * cuda_backend.cu:98-111), w = raw GGUF Q4_K_M rows on the device.  Each call
 * repacks w into a shared device buffer and runs af_gemv_f32; callers that
 * keep a matrix resident pack it once with af_weight_pack instead (the
 * engine and the "cuda" IBackend do).  row_bytes must be cols/256*144 (GGUF
 * rows are contiguous). */
cudaError_t af_q4km_gemv_f32(float* d_y, const uint8_t* d_w, const float* d_x, int rows, int cols,
                             size_t row_bytes, cudaStream_t stream);

/* The same GEMV with x quantised to the reference's Q8_0 blocks first
 * (quantize_q8_avx2, src/backend/cpu_x86/kernels/quant_q8_avx2.cpp:33-84:
 * d = amax/127, q = round-half-even(x·127/amax) per 32 values): the
 * production decode GEMV gemv_wt_q8 (src/models/llama_model.cpp:767-831) with
 * its integer dots and min correction (gemv_q4k_r8_avx2.cpp:209-220,
 * gemv_q6k_q8_avx2.cpp:103).  cols % 256 == 0, cols <= 12288. */
cudaError_t af_gemv_q8_f32(float* d_y, const void* d_w, int ggml_type, const float* d_x, int rows,
                           int cols, cudaStream_t stream);

/* Prefill dequant-GEMM: y[n_tokens][rows] = x[n_tokens][cols] · Wᵀ with W
 * packed (af_weight_pack) and f32 x, on the tcgen05 tensor cores: W
 * dequantised to f16 in shared memory, each token of x scaled by a power of
 * two (undone exactly in the epilogue) and rounded to f16, f32 accumulation in
 * tensor memory (~2e-4 relative error).
 * The linear layers of the reference's batched prompt pass llama_forward_batch
 * (src/models/llama_model.cpp:1339-1462), whose Q4_K × Q8_0 GEMM is
 * gemm_q4k_q8_avx2_range (src/backend/cpu_x86/kernels/gemv_q4k_q8_avx2.cpp:257-346).
 * cols % 256 == 0; x and W 16-byte aligned.  n_tokens <= 32 runs the
 * batched GEMV instead (af_gemv_batched_f32: one weight pass, exact integer
 * dots), which is faster at that size. */
cudaError_t af_prefill_gemm_f32(float* d_y, const void* d_w, int ggml_type, const float* d_x, int rows,
                                int cols, int n_tokens, cudaStream_t stream);

/* Batched dequant GEMV: y[n][rows] = W · x[n] for 1 <= n_vec <= 32 vectors
 * x[n_vec][cols] against one pass over the packed weights (the reference's
 * many-token Q8 GEMM, gemm_q4k_q8_avx2_range,
 * src/backend/cpu_x86/kernels/gemv_q4k_q8_avx2.cpp:257-346).  Inputs are
 * quantised per token and 256 values to a 16-bit grid (~1e-5 relative);
 * integer dots and sub-block scales, f32 per super-block.  Deterministic.
 * Same arguments as af_prefill_gemm_f32. */
cudaError_t af_gemv_batched_f32(float* d_y, const void* d_w, int ggml_type, const float* d_x, int rows,
                                int cols, int n_vec, cudaStream_t stream);

/* The fused GEMV the decode step is built from: up to three matrices sharing
 * one input (e.g. attn_q/attn_k/attn_v), an optional residual add into the
 * input (x + x_add, stored to x_store), an optional RMSNorm of the input
 * (rms_norm_out, src/models/llama_model.cpp:393-419), and one epilogue:
 *   AF_EPI_STORE  y_s[r] = (W_s·x)[r] (+ bias_s[r])
 *   AF_EPI_SWIGLU y_0[r] = silu(W_0·x)[r] * (W_1·x)[r]   (gate, up; llama_model.cpp:344-368)
 *   AF_EPI_RESID  resid[r] += (W_0·x)[r]                   (residual add, :1277, :1324)
 *   AF_EPI_ARGMAX y_0 = W_0·x and *argmax = max over rows of the packed
 *                 (ordered value << 32 | ~(argmax_base + r)) key (greedy, :1466-1471). */
#define AF_EPI_STORE 0
#define AF_EPI_SWIGLU 1
#define AF_EPI_RESID 2
#define AF_EPI_ARGMAX 3
typedef struct {
    const void* w[3];
    int type[3];
    int rows[3];
    float* y[3];
    const float* bias[3];
    int nseg;
    int cols;
    const float* x;
    const float* x_add;
    float* x_store;
    const float* norm_w;
    float eps;
    int epi;
    float* resid;
    unsigned long long* argmax;
    int argmax_base;
} af_gemv_fused_args;
cudaError_t af_gemv_fused(const af_gemv_fused_args* args, cudaStream_t stream);

/* GQA decode attention for one new token at *d_pos (device int): RoPE of q and
 * k with the cos/sin tables [n_ctx][head_dim/2], optional per-head Q/K RMSNorm
 * (qk_norm_order 1 before / 2 after RoPE), K/V stored into the fp32 caches
 * [n_ctx][n_kv_heads*head_dim] at *d_pos, softmax attention over positions
 * 0..*d_pos, output [n_heads*head_dim].  Scratch: d_part
 * (n_heads*nsplit*(head_dim+2) floats) and d_counter (n_kv_heads uints, zero
 * on entry and on return).  llama_model.cpp:1236-1272. */
cudaError_t af_attention_decode_f32(float* d_out, const float* d_q, const float* d_k, const float* d_v,
                                    float* d_kcache, float* d_vcache, const float* d_cos,
                                    const float* d_sin, const float* d_q_norm, const float* d_k_norm,
                                    const int* d_pos, int n_heads, int n_kv_heads, int head_dim,
                                    int n_ctx, int qk_norm_order, float eps, int nsplit,
                                    float* d_part, unsigned int* d_counter, cudaStream_t stream);

/* af_attention_decode_f32 without caller-provided scratch, for callers that
 * cannot call cudaMalloc while serving (a host that owns a fixed device arena,
 * or a plugin only handed input and output pointers).  No counterpart in the
 * reference.  The split-K partials and counters live in a 1 MiB device array
 * of the library that every GPU loading it keeps until exit, so
 * n_heads*nsplit*(head_dim+2) <= 262144 and n_kv_heads <= 256 (larger calls
 * return cudaErrorInvalidValue).  The first call on a device looks the array's
 * address up (cudaGetSymbolAddress) and should come before any stream capture.
 * All calls share the array: calls that overlap on the GPU race.  Allocates
 * nothing (no cudaMalloc / cudaFree). */
cudaError_t af_attention_decode_f32_noalloc(float* d_out, const float* d_q, const float* d_k,
                                            const float* d_v, float* d_kcache, float* d_vcache,
                                            const float* d_cos, const float* d_sin,
                                            const float* d_q_norm, const float* d_k_norm,
                                            const int* d_pos, int n_heads, int n_kv_heads,
                                            int head_dim, int n_ctx, int qk_norm_order, float eps,
                                            int nsplit, cudaStream_t stream);

/* Sampling parameters of the reference's LlamaConfig
 * (include/axonforge/models/llama.hpp:17-35): temperature <= 0 is greedy;
 * top_k <= 0 (or >= vocab) keeps every token; top_p >= 1 disables the
 * nucleus cut; rep_penalty == 1 disables the penalty. */
typedef struct {
    float temperature;
    int top_k;
    float top_p;
    float rep_penalty;
    int rep_last_n;
} af_sampling;

/* One sampling step on the device, one CTA: the repetition penalty over the
 * n_window ids at d_window (applied in place to d_logits, in window order, as
 * apply_rep_penalty does, src/models/llama_model.cpp:1586-1598), then greedy
 * first-max at temperature <= 0, else temperature / top-k / top-p sampling
 * with the uniform draw r in [0, 1) (sample, llama_model.cpp:1466-1498).
 * Writes the id to *d_out.  With temperature > 0 the kept candidates must
 * number at most 1024 (top_k in 1..1024); otherwise cudaErrorNotSupported. */
cudaError_t af_sample_f32(float* d_logits, int vocab, const int32_t* d_window, int n_window,
                          const af_sampling* s, float r, int32_t* d_out, cudaStream_t stream);

/* n uniform draws of std::uniform_real_distribution<float>(0, 1) from
 * std::mt19937(seed) — the reference's sampler stream (llama_model.cpp:1560,
 * 1494-1495), computed by the host C++ library. */
cudaError_t af_mt19937_uniform(uint32_t seed, int n, float* h_out);

/* y = w ⊙ x / sqrt(mean(x²) + eps): rms_norm_f32 (cuda_kernels.hpp:8). */
cudaError_t af_rms_norm_f32(float* d_y, const float* d_x, const float* d_w, int n, float eps,
                            cudaStream_t stream);
/* y = x / (1 + e^-x): silu_f32 (cuda_kernels.hpp:9). */
cudaError_t af_silu_f32(float* d_y, const float* d_x, int n, cudaStream_t stream);
/* y = a ⊙ b: mul_f32 (cuda_kernels.hpp:10). */
cudaError_t af_mul_f32(float* d_y, const float* d_a, const float* d_b, int n, cudaStream_t stream);
/* In-place half-split RoPE of n_heads heads at position pos with base theta:
 * rope_f32 (cuda_kernels.hpp:11), same rotation as apply_rope
 * (src/models/llama_model.cpp:1046-1060). */
cudaError_t af_rope_f32(float* d_q, int n_heads, int head_dim, int pos, float theta,
                        cudaStream_t stream);

/* --------------------------------------------------------- decode engine */

typedef struct af_engine af_engine;

typedef struct {
    int n_layer, n_embd, n_head, n_kv_head, ffn, vocab;
    int n_ctx;            /* KV slots: min(context_length, max_context_len) */
    float eps, theta;
    int qk_norm_order;    /* 0 none, 1 before RoPE (qwen3), 2 after RoPE (hunyuan) */
    int bos_id, eos_id;
} af_model_config;

/* Write a fresh 128-byte ncclUniqueId to h_id (rank 0 calls this and sends the
 * bytes to the other ranks). */
cudaError_t af_nccl_unique_id(void* h_id);

/* Create an engine on `device`.  Tensor parallel when tp_size > 1: this process
 * is rank tp_rank and `nccl_id` points at the 128-byte ncclUniqueId that every
 * rank received from rank 0 (NULL when tp_size == 1). */
cudaError_t af_engine_create(const af_model_config* cfg, int device, int tp_rank, int tp_size,
                             const void* nccl_id, af_engine** out);
cudaError_t af_engine_destroy(af_engine* e);

/* Hand one GGUF tensor (host bytes, exact GGUF size) to the engine, which
 * copies this rank's shard to the device byte-for-byte (Q6_K then regrouped
 * on the device).  Names follow build_weights (src/models/llama_model.cpp:973-1004).
 * dims are in GGML order (dims[0] = columns). */
cudaError_t af_engine_load_tensor(af_engine* e, const char* name, int ggml_type,
                                  const int64_t* dims, int n_dims, const void* h_data,
                                  size_t nbytes);
/* Parse a GGUF file (mmap) and load every tensor; fills *cfg_out if non-NULL. */
cudaError_t af_gguf_read_config(const char* path, int max_context_len, af_model_config* cfg_out);
cudaError_t af_engine_load_gguf(af_engine* e, const char* path);
/* Activation format of the decode step, before af_engine_finalize: 0 (the
 * default) quantises every GEMV input to a 16-bit grid per 32 values (the
 * F32-activation reference within ~1e-5); 1 quantises them to Q8_0 blocks as
 * the reference's production path does (kQ8Quant before each gemv_wt_q8,
 * src/models/llama_model.cpp:1227,1275,1281,1322,1331).  The batched prompt
 * pass (af_engine_prefill_batched) keeps its own f16 GEMM numerics. */
cudaError_t af_engine_set_q8_activations(af_engine* e, int on);
/* Allocate activations/KV, check every required tensor, capture the step graph. */
cudaError_t af_engine_finalize(af_engine* e);

/* One decode step at position pos for token: logits (optional, host, vocab
 * floats; all ranks' shards gathered) and the greedy next id.  Host-driven:
 * token/pos go host->device and the id comes back every call. */
cudaError_t af_engine_step(af_engine* e, int32_t token, int32_t pos, float* h_logits,
                           int32_t* h_next);
/* Prefill tokens[0..n) at positions pos0.. (KV filled); last-token logits and
 * greedy id as in af_engine_step. */
cudaError_t af_engine_prefill(af_engine* e, const int32_t* h_tokens, int n, int32_t pos0,
                              float* h_logits, int32_t* h_next);

/* Same contract as af_engine_prefill, computed as one batched prompt pass:
 * tokens 0 .. n-2 through every layer as rows of the tcgen05 prefill GEMM
 * (af_prefill_gemm_f32), row kernels for norms / bias / SwiGLU / residuals,
 * attention per token in position order; the last token through the decode
 * step (its logits and the next token).  The reference's batched prompt pass
 * is llama_forward_batch (src/models/llama_model.cpp:1339-1462).  Numerics
 * differ from the per-token path by the GEMM's f16 rounding (~2e-4 relative).
 * Tensor-parallel engines fall back to af_engine_prefill. */
cudaError_t af_engine_prefill_batched(af_engine* e, const int32_t* h_tokens, int n, int32_t pos0,
                                      float* h_logits, int32_t* h_next);
/* Device-fed greedy decode: n_steps graph launches, each feeding its argmax to
 * the next; ids written to h_out (may be NULL).  No host round trip per step. */
cudaError_t af_engine_decode_greedy(af_engine* e, int32_t first_token, int32_t pos0, int n_steps,
                                    int32_t* h_out);
/* Greedy generation with llama_generate's decode-loop semantics
 * (src/models/llama_model.cpp:1562-1624): BOS prepended unless present, stop at
 * EOS or the context cap.  Returns the ids in h_out, count in *n_out. */
cudaError_t af_engine_generate(af_engine* e, const int32_t* h_prompt, int n_prompt, int max_new,
                               int32_t* h_out, int* n_out);
/* Sample the next token from the logits of the last step / prefill (all
 * ranks' shards): af_sample_f32 over the full vocabulary, with the penalty
 * window h_window[0..n_window) (host ids) and the draw r.  Tensor-parallel
 * ranks given the same arguments return the same id. */
cudaError_t af_engine_sample(af_engine* e, const af_sampling* s, const int32_t* h_window, int n_window, float r,
                             int32_t* h_next);
/* llama_generate with sampling (src/models/llama_model.cpp:1502-1631): BOS
 * prepended unless present, the prompt, then one sampling step per token
 * with the repetition window of the last rep_last_n ids of prompt +
 * generated, stopping at EOS (not emitted) or the context cap.  h_draws holds
 * the uniform draws in order (the reference consumes one per sampling step at
 * temperature > 0; e.g. af_mt19937_uniform(42, ...)); n_draws must cover
 * max_new + 1 of them then, and may be 0 when greedy. */
cudaError_t af_engine_generate_sampled(af_engine* e, const int32_t* h_prompt, int n_prompt, int max_new,
                                       const af_sampling* s, const float* h_draws, int n_draws, int32_t* h_out,
                                       int* n_out);
/* Copy the current residual stream (n_embd floats) to the host. */
cudaError_t af_engine_hidden(af_engine* e, float* h_out);
/* Copy layer l's fp32 K or V cache rows [0, n_pos) (local heads) to the host. */
cudaError_t af_engine_kv(af_engine* e, int layer, int which_v, int n_pos, float* h_out);
/* Launch kinds reported by af_engine_profile. */
#define AF_PROF_EMBED 0
#define AF_PROF_QKV 1
#define AF_PROF_ATTN 2
#define AF_PROF_O 3
#define AF_PROF_GATEUP 4
#define AF_PROF_DOWN 5
#define AF_PROF_LMHEAD 6
#define AF_PROF_FINAL 7
#define AF_PROF_COMM 8
#define AF_PROF_KINDS 9
/* Run n_steps decode steps eagerly (no graph) with a CUDA event after every
 * launch; per kind: total device ms, total algorithmic bytes and launch count
 * (arrays of AF_PROF_KINDS).  Positions pos0.. are written like a real step. */
cudaError_t af_engine_profile(af_engine* e, int32_t token, int32_t pos0, int n_steps, double* h_ms,
                              double* h_bytes, int* h_count);
/* Stream the step runs on (for event timing by the caller). */
cudaStream_t af_engine_stream(af_engine* e);
/* Kernel launches one decode step issues (graph nodes that are this library's). */
int af_engine_kernels_per_step(af_engine* e);
/* Per-step weight bytes this rank streams. */
size_t af_engine_weight_bytes(af_engine* e);

#ifdef __cplusplus
}
#endif
#endif /* AF_B200_H */
