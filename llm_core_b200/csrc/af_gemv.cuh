// af_gemv.cuh — the fused dequant GEMV for Q4_K / Q6_K super-blocks (sm_100a).
//
// Replaces the reference's x86 hot loop (gemv_q4k_avx2_range,
// src/backend/cpu_x86/kernels/gemv_q4k_avx2.cpp:230-238; gemv_q6k_avx2_range,
// gemv_q6k_avx2.cpp:235-243; production gemv_wt_q8, src/models/llama_model.cpp:767-831)
// and its incorrect CUDA v1 kernel (src/backend/cuda/cuda_kernels.cu:71-109).
//
// Design (HBM-bound; one launch streams each weight byte exactly once):
//  * Grid = one CTA per SM.  Each CTA owns a byte-balanced contiguous range of
//    output rows and walks it in tiles of 16 rows (8 row pairs for SwiGLU).
//  * Warp 8 is the producer: it streams every (tile, 8-block K chunk) stage
//    into a ring of shared-memory slots with cp.async.bulk (the TMA engine,
//    no tensor map, no multicast), one bulk copy per row, completion counted
//    on an mbarrier.  Weights are read with an L2 evict-first policy.  The
//    first ring-full of stages is issued before griddepcontrol.wait, so under
//    programmatic dependent launch the weight stream overlaps the tail of the
//    previous kernel.
//  * Warps 0-7 are consumers.  Their prologue turns the f32 input (optionally
//    plus a pending residual, optionally RMS-normalised) into a shared-memory
//    copy split into two int8 planes: x ≈ xs·(256·hi + lo) per 64 values
//    (|error| ≤ 2^-16·max|x| of the group), plus per-32 f32 sums and per-16
//    integer sums for the min / offset terms.  Each lane then owns one
//    (super-block, 64-value chunk) of the stage and evaluates the exact
//    integer dot Σ q·(256·hi + lo) with dp4a, applying the block scales in
//    f32 — the same w = d·sc·q − dmin·m (Q4_K) and w = d·sc·(q − 32) (Q6_K)
//    the reference dequantises, accumulated in fp32.
//  * Epilogues: plain store (+bias), in-place residual add, SwiGLU of a
//    gate/up row pair, and LM-head logits with a fused first-max argmax.
#pragma once
#include "af_common.cuh"

namespace af {

enum GemvEpi : int { EPI_STORE = 0, EPI_SWIGLU = 1, EPI_RESID = 2, EPI_ARGMAX = 3 };

struct GemvSeg {
    const uint8_t* w;      // device rows (Q4_K GGUF rows or Q6_K regrouped rows)
    float* y;              // output rows (EPI_STORE / EPI_ARGMAX / SWIGLU seg 0)
    const float* bias;     // optional per-row bias (EPI_STORE)
    int type;              // AF_GGML_Q4_K or AF_GGML_Q6_K
    int rows;
    int row_stride;        // bytes
};

struct GemvParams {
    GemvSeg seg[3];
    int nseg;
    int K;                 // input length, multiple of 256
    const float* x;        // f32 input [K]
    const float* x_add;    // optional: input = x + x_add (deferred residual) ...
    float* x_store;        // ... and CTA 0 stores that sum here
    const float* norm_w;   // optional RMSNorm weight [K]
    float eps;
    int epi;
    float* resid;          // EPI_RESID: resid[row] += W·x
    unsigned long long* argmax;  // EPI_ARGMAX: packed (value, ~index) maximum
    int argmax_base;       // global index of row 0 (vocab shard offset)
    int pitch;             // shared-memory bytes per row slot
    int nslots;            // ring depth
};

constexpr int kGemvThreads = 288;  // 8 consumer warps + 1 producer warp
constexpr int kGemvTileRows = 16;
constexpr int kGemvMaxSlots = 6;
constexpr int kGemvMaxK = 12288;  // input length held in registers by the prologue

// Shared-memory bytes the GEMV needs for (K, pitch, nslots).
__host__ __device__ inline int gemv_smem_bytes(int K, int pitch, int nslots) {
    const int nst = (K / 256 + 7) / 8;
    return 128 + nslots * kGemvTileRows * pitch + nst * (2048 * 2 + 32 * 4 + 64 * 4 + 128 * 4) + 64 * 4;
}

__host__ __device__ inline int q6k_row_stride(int cols) {
    const int nb = cols / 256, full = nb / 8, rem = nb % 8;
    return full * 1680 + (rem ? rem * 208 + 16 : 0);
}

__host__ __device__ inline int dev_row_stride(int type, int cols) {
    return type == AF_GGML_Q6_K ? q6k_row_stride(cols) : (cols / 256) * 144;
}

// Device bytes of a packed matrix: whole 16-row tiles (the last one zero-padded).
__host__ __device__ inline size_t packed_bytes(int type, int rows, int cols) {
    return (size_t)((rows + kGemvTileRows - 1) / kGemvTileRows) * kGemvTileRows * dev_row_stride(type, cols);
}

// Per-device kernel attributes; call once per device before launching (and
// before any stream capture).
cudaError_t gemv_init();
cudaError_t gemv_launch(const GemvParams& p, int grid, cudaStream_t stream, bool pdl);
// Fill pitch / nslots for the segments in p; returns the dynamic smem bytes.
int gemv_configure(GemvParams& p);

}  // namespace af
