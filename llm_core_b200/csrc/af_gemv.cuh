// af_gemv.cuh — the fused dequant GEMV for Q4_K / Q6_K super-blocks (sm_100a).
//
// Replaces the reference's x86 hot loop (gemv_q4k_avx2_range,
// src/backend/cpu_x86/kernels/gemv_q4k_avx2.cpp:230-238; gemv_q6k_avx2_range,
// gemv_q6k_avx2.cpp:235-243; production gemv_wt_q8, src/models/llama_model.cpp:767-831)
// and its incorrect CUDA v1 kernel (src/backend/cuda/cuda_kernels.cu:71-109).
//
// Design (HBM-bound; one launch streams each weight byte exactly once):
//  * Weights are "packed" once at upload (af_weight_pack): 16-row tiles, each
//    holding stage after stage the rows' segments of 8 super-blocks, so one
//    pipeline entry (a fragment of up to 30 rows × one stage) is a few
//    contiguous bulk copies.
//  * Grid = one CTA per SM.  Each CTA owns a byte-balanced contiguous range of
//    output rows (computed on the host) and walks it in fragments of up to 30
//    rows (15 gate/up pairs for SwiGLU), two fragments per K stage.
//  * Warp 15 is the producer: one thread streams every (fragment, K stage)
//    entry into a byte ring in shared memory with cp.async.bulk (the TMA
//    engine, no tensor map, no multicast), completion counted on an mbarrier,
//    L2 evict-first.  Weights do not depend on the previous kernel, so the
//    producer never waits for it (griddepcontrol.wait is the consumers' only).
//  * The input vector arrives already quantised ("XQ": x ≈ xs·(256·hi + lo)
//    per 64 values as two int8 planes, per-32 f32 sums, per-16 integer sums,
//    and for a normalised input the per-64 sums of squares); the consumers
//    copy it into shared memory with L2 loads.  The kernel that produced the
//    vector quantised each 64-value group once (the last CTA to finish a group
//    does it), so no CTA re-reads and re-quantises the whole input.  A legacy
//    in-CTA prologue quantises an f32 input for the standalone entry points
//    and tensor-parallel ranks.
//  * Warps 0-14 are consumers: lane = (super-block, 64-value chunk) of the
//    stage; each warp evaluates four rows (two per fragment) with exact integer
//    dp4a dots Σ q·(256·hi + lo) and applies the block scales in f32 — the
//    same w = d·sc·q − dmin·m (Q4_K) and w = d·sc·(q − 32) (Q6_K) the
//    reference dequantises, accumulated in fp32.
//  * Epilogues: plain store (+bias), in-place residual add, SwiGLU of a
//    gate/up row pair, LM-head logits with a fused first-max argmax; optionally
//    the output vector is quantised into the next GEMV's XQ buffer.
//  * The same building blocks (af_gemv_dev.cuh) run inside the persistent
//    decode-step kernel (af_step.cu), where the ring persists across phases.
#pragma once
#include "af_common.cuh"

namespace af {

enum GemvEpi : int { EPI_STORE = 0, EPI_SWIGLU = 1, EPI_RESID = 2, EPI_ARGMAX = 3 };

// 15 consumer warps + 1 producer = 16 warps: 4 per SM sub-partition, so each
// thread may use 128 registers (the register file is split across the 4).
constexpr int kGemvConsumerWarps = 15;
constexpr int kGemvThreads = (kGemvConsumerWarps + 1) * 32;
constexpr int kPackTile = 16;        // rows per tile of the packed weight layout
constexpr int kGemvFragRows = 2 * kGemvConsumerWarps;  // rows per pipeline stage
constexpr int kGemvSmemHdr = 1024;  // mbarriers, abort flag, group list
constexpr int kGemvMaxK = 12288;     // input length held in registers by the legacy prologue
constexpr int kGemvMaxGrid = 296;

struct GemvSeg {
    const uint8_t* w;      // packed rows
    float* y;              // output rows (EPI_STORE / EPI_ARGMAX / SWIGLU seg 0)
    const float* bias;     // optional per-row bias (EPI_STORE)
    int type;              // AF_GGML_Q4_K or AF_GGML_Q6_K
    int rows;
    int row_stride;        // bytes per row (sum of the row's stage segments)
};

struct GemvParams {
    GemvSeg seg[3];
    int nseg;
    int K;                 // input length, multiple of 256
    // input, quantised form (preferred): XQ layout of xq_bytes(K) bytes, and
    // with xq_norm the per-64 sums of squares after it (RMSNorm input)
    const uint8_t* xq;
    int xq_norm;
    // input, f32 form (legacy prologue): x (+ x_add, stored to x_store) [+ RMSNorm]
    const float* x;
    const float* x_add;
    float* x_store;
    const float* norm_w;
    float eps;
    int epi;
    float* resid;          // EPI_RESID: resid[row] += W·x
    unsigned long long* argmax;  // EPI_ARGMAX: packed (value, ~index) maximum
    int argmax_base;       // global index of row 0 (vocab shard offset)
    // optional: quantise the output vector (resid for EPI_RESID, y_0 otherwise)
    // into q_out for the next GEMV, with RMSNorm weights q_norm_w (NULL: plain)
    uint8_t* q_out;
    const float* q_norm_w;
    unsigned int* q_cnt;   // per-64-row-group arrival counters, zero between launches
    int ring_bytes;        // weight ring in shared memory (multiple of 16)
    int grid;
    int vrange[kGemvMaxGrid + 1];  // CTA i owns virtual rows [vrange[i], vrange[i+1])
};

__host__ __device__ inline int q6k_row_stride(int cols) {
    const int nb = cols / 256, full = nb / 8, rem = nb % 8;
    return full * 1680 + (rem ? rem * 208 + 16 : 0);
}

__host__ __device__ inline int dev_row_stride(int type, int cols) {
    return type == AF_GGML_Q6_K ? q6k_row_stride(cols) : (cols / 256) * 144;
}

// Device bytes of a packed matrix: whole 16-row tiles (the last one zero-padded).
__host__ __device__ inline size_t packed_bytes(int type, int rows, int cols) {
    return (size_t)((rows + kPackTile - 1) / kPackTile) * kPackTile * dev_row_stride(type, cols);
}

// Bytes of the quantised-input (XQ) layout for K values: per stage of 2048
// values: hi plane 2048, lo plane 2048, 32 f32 scales, 64 f32 sums of 32,
// 128 int sums of 16.  A normalised input appends K/64 f32 sums of squares.
__host__ __device__ inline int xq_bytes(int K) { return ((K / 256 + 7) / 8) * 4992; }
__host__ __device__ inline int xq_norm_bytes(int K) { return xq_bytes(K) + K / 16; }

// Shared-memory bytes of the standalone GEMV: header, ring, XQ input, misc.
__host__ __device__ inline int gemv_smem_bytes(int K, int ring_bytes) {
    return kGemvSmemHdr + ring_bytes + xq_norm_bytes(K) + 256;
}

// Per-device kernel attributes; call once per device before launching (and
// before any stream capture).
cudaError_t gemv_init();
// Fill ring size / grid / CTA ranges for the segments in p.
void gemv_configure(GemvParams& p, int grid);
cudaError_t gemv_launch(const GemvParams& p, cudaStream_t stream, bool pdl);

// Quantise an f32 vector (RMSNorm weights applied when norm_w is set) into XQ
// form, for inputs no producing kernel writes.
cudaError_t xq_quantize_launch(uint8_t* xq, const float* x, const float* norm_w, int K, cudaStream_t st, bool pdl);

// One warp quantises 64-value group g of src (global f32) into the XQ buffer;
// with norm_w, w·x is quantised and Σx² stored after the layout.
__device__ void xq_quantize_group(uint8_t* xq, const float* src, const float* norm_w, int K, int g);
// Same, from values already in registers: lane l holds group values 2l, 2l+1.
__device__ void xq_quantize_vals(uint8_t* xq, float a0, float a1, const float* norm_w, int K, int g);

}  // namespace af
