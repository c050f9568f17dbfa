// af_gemv.cuh — the fused dequant GEMV for Q4_K / Q6_K super-blocks (sm_100a).
//
// Replaces the reference's x86 hot loop (gemv_q4k_avx2_range,
// src/backend/cpu_x86/kernels/gemv_q4k_avx2.cpp:230-238; gemv_q6k_avx2_range,
// gemv_q6k_avx2.cpp:235-243; production gemv_wt_q8, src/models/llama_model.cpp:767-831)
// and its incorrect CUDA v1 kernel (src/backend/cuda/cuda_kernels.cu:71-109).
//
// Design (HBM-bound; one launch streams each weight byte exactly once):
//  * Weights are "packed" once at upload (af_weight_pack) into units of 16
//    rows × one 256-value super-block, laid out in the register order of the
//    tensor-core instruction mma.sync.m16n8k32 (u8 weights × s8 inputs, s32
//    accumulators): every lane fetches its A fragments with 16-byte shared
//    loads.  A tile (16 rows) is its units in K order, so a K stage of a tile
//    is one contiguous bulk copy.
//  * The input x is quantised per 32 values to a 16-bit grid
//    x ≈ xs·(256·hi + lo) (two int8 planes).  Each mma multiplies 16 rows ×
//    32 values of nibbles (or 6-bit values) by a block-diagonal B whose column
//    pairs hold the hi / lo planes of one 32-value sub-block (Q4_K) or 16-value
//    group (Q6_K), so the s32 accumulators come out as exact per-sub-block
//    integer dots Σ q·hi, Σ q·lo — the granularity at which the block scales
//    apply.  Scales are applied in f32 — the same w = d·sc·q − dmin·m (Q4_K)
//    and w = d·sc·(q − 32) (Q6_K) the reference dequantises.
//  * Grid = one CTA per SM.  Each CTA owns a byte-balanced contiguous range of
//    fragments (computed on the host): two 16-row tiles starting at an even
//    tile, i.e. 32 output rows (SwiGLU: the gate and the up tiles of the same
//    32 rows).
//  * One producer thread streams every (fragment, 8-super-block K stage)
//    entry into a byte ring in shared memory with cp.async.bulk (the TMA
//    engine, no tensor map, no multicast), completion counted on an mbarrier,
//    L2 evict-first.  Weights do not depend on the previous kernel, so the
//    producer never waits for it.
//  * 8 consumer warps: warp w evaluates super-block w of every stage for all
//    tiles of the fragment, accumulating per row in registers across stages;
//    at the end of a fragment the 8 warps' row sums are added in a fixed
//    order through shared memory (deterministic) and one warp (the duty
//    rotates) runs the epilogue for the fragment's 32 rows: plain store
//    (+bias), in-place residual add, SwiGLU of a gate/up pair, LM-head logits
//    with a fused first-max argmax.
//  * The input arrives either quantised ("XQ") or as an f32 vector the
//    consumers quantise in shared memory (RMSNorm folded in).  The GEMV that
//    produces a vector quantises each finished 32-row fragment in its
//    epilogue (RMSNorm-weighted for the next GEMV where it normalises), so the
//    consumer of the vector only copies it: no cross-CTA pass, counters or
//    second read of the f32 vector.
//  * The same building blocks (af_gemv_dev.cuh) run inside the persistent
//    decode-step kernel (af_step.cu), where the ring persists across phases.
#pragma once
#include "af_common.cuh"

namespace af {

enum GemvEpi : int { EPI_STORE = 0, EPI_SWIGLU = 1, EPI_RESID = 2, EPI_ARGMAX = 3 };

// 8 consumer warps + 1 producer warp.
constexpr int kGemvConsumerWarps = 8;
constexpr int kGemvThreads = (kGemvConsumerWarps + 1) * 32;
constexpr int kPackTile = 16;        // rows per tile of the packed weight layout
constexpr int kGemvFragTiles = 2;    // tiles per fragment (per gate / up part)
constexpr int kGemvStageBlocks = 8;  // super-blocks per K stage (one per consumer warp)
constexpr int kGemvMaxK = 12288;     // input length quantised by the f32 prologue
constexpr int kGemvMaxGrid = 296;
constexpr int kGemvSmemHdr = 6144;   // mbarriers, abort flag, phase parameters, reduction scratch
constexpr int kGemvMaxRanks = 8;     // tensor-parallel ranks a plain-store epilogue can send to

static_assert(kGemvStageBlocks == kGemvConsumerWarps, "one super-block per consumer warp");

// Bytes of one unit (16 rows × 256 values).
__host__ __device__ inline int unit_bytes(int type) { return type == AF_GGML_Q6_K ? 16 * 210 : 16 * 144; }

// Q4_K unit: [2048: qs words in fragment order][256: the 16 rows' 16-byte headers]
//   qs offset c*512 + lane*16 + e*4 (chunk c = 64 values) holds GGUF qs word
//   w of chunk c of row r, with g = lane/4, t = lane%4 and
//   e = 0: (r = g,   w = t)   e = 1: (r = g+8, w = t)
//   e = 2: (r = g,   w = t+4) e = 3: (r = g+8, w = t+4).
// Q6_K unit: [2048: low nibbles][1024: high bit pairs][256: row scales][32: row d]
//   low-nibble word at P*512 + lane*16 + e*4 (P = 64-value pair of tiles),
//   byte i = lo4(q(r, 64P + 4w + i)) | lo4(q(r, 64P + 32 + 4w + i)) << 4;
//   high word at 2048 + Q*512 + lane*16 + e*4 (Q = 128-value quad),
//   byte i = Σ_s hi2(q(r, 128Q + 32s + 4w + i)) << 2s;  (r, w) as for Q4_K.
constexpr int kQ4Hdr = 2048;
constexpr int kQ6Hi = 2048, kQ6Sc = 3072, kQ6D = 3328;

struct GemvSeg {
    const uint8_t* w;      // packed rows
    float* y;              // output rows (EPI_STORE / EPI_ARGMAX / SWIGLU seg 0)
    const float* bias;     // optional per-row bias (EPI_STORE)
    int type;              // AF_GGML_Q4_K or AF_GGML_Q6_K
    int rows;
    int row_stride;        // bytes per row = super-blocks × 144 (Q4_K) or 210 (Q6_K)
};

struct GemvParams {
    GemvSeg seg[3];
    int nseg;
    int K;                 // input length, multiple of 256
    // input, quantised form: XQ layout of xq_bytes(K) bytes, and with xq_norm
    // the per-32 sums of squares after it (RMSNorm input)
    const uint8_t* xq;
    int xq_norm;
    // input, f32 form (prologue): x (+ x_add, stored to x_store) [+ RMSNorm]
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
    // into q_out (XQ of the next GEMV), weighted by q_norm_w when set, with
    // the per-32 sums of squares for that GEMV's RMSNorm
    uint8_t* q_out;
    const float* q_norm_w;
    // tensor-parallel partial sums (xsend_n > 0, EPI_STORE): instead of y, the
    // epilogue stores each value v of row i as the 64-bit word
    // (xtag << 32) | bits(v) at xsend[r][i] for every rank r < xsend_n; the
    // tag makes the word its own arrival flag (no fence, no counter)
    unsigned long long* xsend[kGemvMaxRanks];
    int xsend_n;
    uint32_t xtag;
    // quantise inputs as Q8_0 blocks (the reference's production activation
    // format) instead of the 16-bit grid
    int q8;
    int ring_bytes;        // weight ring in shared memory (multiple of 16)
    int grid;
    int vrange[kGemvMaxGrid + 1];  // CTA i owns fragments [vrange[i], vrange[i+1])
};

__host__ __device__ inline int dev_row_stride(int type, int cols) {
    return (cols / 256) * (type == AF_GGML_Q6_K ? 210 : 144);
}

// Device bytes of a packed matrix: whole 16-row tiles (the last one zero-padded).
__host__ __device__ inline size_t packed_bytes(int type, int rows, int cols) {
    return (size_t)((rows + kPackTile - 1) / kPackTile) * kPackTile * dev_row_stride(type, cols);
}

// Quantised-input (XQ) layout for K values, per 256-value super-block
// (kXqSb bytes): hi plane [256] int8, lo plane [256] int8 (value order), then
// xs[8] f32 and sum32[8] f32 (Σx) per 32-value group, isum16[16] int32
// (Σ 256·hi + lo per 16 values).  A normalised input appends K/32 f32 sums of
// squares of the un-weighted values.
constexpr int kXqSb = 512 + 32 + 32 + 64;
constexpr int kXqXs = 512, kXqS32 = 544, kXqI16 = 576;
__host__ __device__ inline int xq_bytes(int K) { return (K / 256) * kXqSb; }
__host__ __device__ inline int xq_norm_bytes(int K) { return xq_bytes(K) + K / 8; }

// Shared-memory bytes of the standalone GEMV: header, ring, XQ input, misc.
__host__ __device__ inline int gemv_smem_bytes(int K, int ring_bytes) {
    return kGemvSmemHdr + ring_bytes + xq_norm_bytes(K) + 256;
}

// Per-device kernel attributes; call once per device before launching (and
// before any stream capture).
cudaError_t gemv_init();
// Fill ring size / grid / CTA tile ranges for the segments in p.
void gemv_configure(GemvParams& p, int grid);
cudaError_t gemv_launch(const GemvParams& p, cudaStream_t stream, bool pdl);

// Quantise an f32 vector (RMSNorm weights applied when norm_w is set) into XQ
// form, for inputs no producing kernel writes.
cudaError_t xq_quantize_launch(uint8_t* xq, const float* x, const float* norm_w, int K, cudaStream_t st, bool pdl,
                               bool q8 = false);

// Quantise value v (this lane's; the warp's 32 lanes hold one 32-value group,
// indices idx = 32·g + lane) into the XQ buffer, with the lane's RMSNorm
// weight already loaded (norm: the weighted value w·v is quantised and Σv²
// of the group stored after the layout).  All 32 lanes must call (lanes
// past the vector pass any v; they store nothing).  The 16-bit split matches
// the consumers' integer form: q = rint(v·32639/amax), hi = (q + 128) >> 8,
// lo = q − 256·hi.  Inline: it runs in the epilogues of the hot loops.
// With q8, the group is quantised as the reference's Q8_0 block instead
// (quantize_q8_avx2, src/backend/cpu_x86/kernels/quant_q8_avx2.cpp:33-84):
// d = amax/127, q = round-half-even(a · 127/amax), stored as hi = 0, lo = q,
// xs = d, and the group sum d·Σq (the min correction of the Q8 dot,
// gemv_q4k_r8_avx2.cpp:209-220).
__device__ __forceinline__ void xq_store32w(uint8_t* xq, float v, float wgt, bool norm, int K, int idx,
                                            bool q8 = false) {
    const int lane = threadIdx.x & 31;
    const bool in = idx >= 0 && idx < K;
    if (!in) v = 0.f;
    const float a = v * wgt;
    const float amax = warp_max(fabsf(a));
    int q, hi, lo;
    if (q8) {
        const float id = amax > 0.f ? 127.f / amax : 0.f;
        q = max(-127, min(127, __float2int_rn(a * id)));
        hi = 0;
        lo = q;
    } else {
        const float inv = amax > 0.f ? 32639.f / amax : 0.f;
        q = max(-32639, min(32639, __float2int_rn(a * inv)));
        hi = (q + 128) >> 8;
        lo = q - 256 * hi;
    }
    int is = q;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) is += __shfl_xor_sync(0xffffffffu, is, o);  // per 16
    const float fs = q8 ? (amax / 127.f) * (float)(is + __shfl_xor_sync(0xffffffffu, is, 16)) : warp_sum(a);
    const float ss = norm ? warp_sum(v * v) : 0.f;
    if (!in) return;
    uint8_t* sb = xq + (idx >> 8) * kXqSb;
    const int ko = idx & 255;
    sb[ko] = (uint8_t)(hi & 0xFF);
    sb[256 + ko] = (uint8_t)(lo & 0xFF);
    if ((lane & 15) == 0) reinterpret_cast<int*>(sb + kXqI16)[ko >> 4] = is;
    if (lane == 0) {
        reinterpret_cast<float*>(sb + kXqXs)[ko >> 5] = q8 ? amax / 127.f : amax / 32639.f;
        reinterpret_cast<float*>(sb + kXqS32)[ko >> 5] = fs;
        if (norm) reinterpret_cast<float*>(xq + xq_bytes(K))[idx >> 5] = ss;
    }
}

// Same, loading the weight from norm_w (nullptr: no norm).
__device__ __forceinline__ void xq_store32(uint8_t* xq, float v, const float* norm_w, int K, int idx,
                                           bool q8 = false) {
    const bool in = idx >= 0 && idx < K;
    xq_store32w(xq, v, norm_w && in ? __ldg(norm_w + idx) : 1.f, norm_w != nullptr, K, idx, q8);
}

// One warp quantises values [32·g, 32·g + 32) of src (global f32, written by
// other CTAs: read through L2).
__device__ __forceinline__ void xq_quantize_group(uint8_t* xq, const float* src, const float* norm_w, int K, int g,
                                                  bool q8 = false) {
    const int idx = 32 * g + (threadIdx.x & 31);
    xq_store32(xq, idx < K ? __ldcg(src + idx) : 0.f, norm_w, K, idx, q8);
}

}  // namespace af
