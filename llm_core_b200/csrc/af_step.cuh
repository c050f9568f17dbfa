// af_step.cuh — the persistent decode-step kernel: one launch per token.
//
// The separate-kernel step (embed, 5 kernels per layer, LM head, finalize)
// pays a kernel boundary per phase: the last CTA's tail, the grid drain and
// the next kernel's ramp, during which HBM idles.  Here one cooperative grid
// (one CTA per SM) runs every phase of the step.  The producer thread of each
// CTA streams the weight rows that CTA owns for ALL GEMV phases in order,
// limited only by the ring in shared memory, so weight streaming never waits
// for a phase boundary; the consumer warps wait for the previous phase on a
// grid-wide arrival counter (bounded spin) and then run the phase:
//
//   EMBED  token row dequant → x and its quantised form
//   GEMV   QKV(+bias) | O(+resid) | gate/up SwiGLU | down(+resid) | LM head+argmax
//   ATTN   RoPE, Q/K norm, KV store, split attention
//
// Every phase writes the next GEMV's input already quantised: the epilogue
// that finishes a 32-row fragment quantises it (one 32-value group,
// RMSNorm-weighted where the next GEMV normalises), so a phase ends with its
// epilogue stores and the next one copies its input with one L2 read: no
// cross-CTA pass, counters or fences between phases other than the arrival
// itself.  Under tensor parallelism the row-parallel GEMVs send tagged partial
// sums to every rank instead, and the GEMV after them reduces its input
// itself (XchgParams).  CTA 0, once every CTA has finished the last phase,
// turns the argmax into the next token and advances the position.
#pragma once
#include "af_gemv.cuh"
#include "af_ops.cuh"

namespace af {

enum StepPhaseKind : int { PH_EMBED = 0, PH_GEMV = 1, PH_ATTN = 2, PH_XRED = 3 };

constexpr int kStepMaxRanks = kGemvMaxRanks;

constexpr int kStepMaxG = 8;            // query heads per kv head
constexpr int kStepAttnChunk = 64;      // KV positions per attention chunk
constexpr int kStepAttnMaxSplit = 128;  // splits per kv head the attention merge stages in shared memory
constexpr int kStepAttnDistMerge = 8;   // splits above which the merge is spread over the splits
constexpr int kStepHdr = kGemvSmemHdr;  // mbarriers, flags, phase parameter copies, reduction scratch
constexpr int kStepUnion = 40 * 1024;   // XQ input of a GEMV phase / attention scratch, at most
// Attention scratch in the union area (AttnSmem, af_step.cu): q of the
// kv head's query heads, k, v, scores, the warps' P·V partials, per-head
// (max, sum, correction), the splits' (max, sum) and the merged output.
constexpr int kStepAttnScratch =
    (kStepMaxG * 128 + 256 + kStepMaxG * kStepAttnChunk + 8 * 128 + 3 * kStepMaxG + kStepMaxG * kStepAttnMaxSplit * 2 +
     kStepMaxG * 128 + 4) * 4;
static_assert(kStepAttnScratch <= kStepUnion, "attention scratch exceeds the union area");

// With Q8_0 activations the embedding phase normalises the first layer's
// input itself, in the reference's summation order (its embedding values are
// a discrete grid, where the Q8 rounding of x·127/amax often sits exactly on
// a tie, so the normalised values must be bit-identical); it stages the row
// in the union area, so n_embd·4 bytes must fit there.
__host__ __device__ inline bool step_q8_exact_embed(int n_embd) { return n_embd * 4 <= kStepUnion; }
constexpr int kStepSmem = 227 * 1024;

// Tensor-parallel exchanges (the outputs of the row-parallel O and down
// GEMVs, 2 per layer): the producing GEMV (k_out = k) sends each partial
// value tagged with the exchange's sequence number straight into every rank's
// receive area (slot [seq % 2][this rank]), and the GEMV that consumes the
// sum (k_in = k) waits for the tags instead of a grid barrier: each of its
// CTAs reads all ranks' partials, adds them in rank order to the residual
// (resid_in → resid_out, ping-pong so that no CTA overwrites what another
// still reads) and quantises the RMSNorm-weighted sum into its own shared
// memory.  No fence, counter or separate reduction phase.
struct XchgParams {
    int k_out;             // exchange this GEMV's partial sums feed (-1: none)
    int k_in;              // exchange whose sum is this GEMV's input (-1: none)
    const float* resid_in; // residual stream before the exchange [n]
    float* resid_out;      // after it (CTA g % grid writes group g)
    const float* norm_w;   // RMSNorm weights of the consuming GEMV
    int n;                 // values (n_embd)
    uint8_t* xq;           // PH_XRED: the quantised sum (XQ layout) for the consuming GEMV
};

// Two ways to consume an exchange: (1) the GEMV itself (k_in on a PH_GEMV):
// every CTA reads every rank's partials for the whole vector; (2) a PH_XRED
// phase before the GEMV: each 32-value group is reduced by one warp of one
// CTA (the ranks' tagged partials added in rank order to the residual),
// stored to resid_out and quantised (RMSNorm-weighted, with its Σx²) into
// x.xq; the GEMV then waits for the grid and copies the quantised vector like
// a single-GPU phase.  (2) reads n·tp words per rank instead of per CTA, for
// one more grid arrival.
struct StepPhase {
    int kind;
    GemvParams g;  // PH_GEMV
    AttnParams a;  // PH_ATTN (nsplit = splits per kv head)
    XchgParams x;  // PH_GEMV / PH_XRED: tensor-parallel exchanges
};

struct StepParams {
    const StepPhase* ph;  // device array
    int nph;
    unsigned int* bar;    // grid arrival counter, zeroed at launch
    // embedding
    const uint8_t* tok_w;
    int tok_type, tok_stride, n_embd, vocab;
    float* x;
    uint8_t* xq;
    const float* xq_norm_w;
    int q8;                          // activations as Q8_0 blocks (see xq_store32w)
    float eps;                       // RMSNorm epsilon (the Q8 embedding path normalises itself)
    int attn_dist;                   // attention splits per kv head can exceed kAttnDistMerge
    int union_bytes;                 // the union area this engine needs (the rest of shared memory is ring)
    // finalize
    unsigned long long* key;
    int* token;
    int* pos;
    int* hist;
    int ring_bytes;
    // tensor parallel (tp > 1): per rank r, its exchange area mapped into
    // this process (IPC): argmax arrival counter (u64, monotonic over the
    // engine's life), argmax keys [kStepMaxRanks], receive slots
    // [2][kStepMaxRanks][n_embd] of tagged partial sums
    int tp, rank;
    int n_buf;                       // partial-sum exchanges per step (2·layers)
    unsigned long long* xrecv[kStepMaxRanks];
    unsigned long long* xbar[kStepMaxRanks];
    unsigned long long* xkey[kStepMaxRanks];
    unsigned long long* epoch;       // steps run by this engine (this rank's memory)
};

// Bytes of one rank's exchange area for n_embd values.
inline size_t step_xchg_bytes(int n_embd) { return 256 + (size_t)2 * kStepMaxRanks * n_embd * sizeof(unsigned long long); }

// Whether a model shape runs on the step kernel (else: separate kernels).
// Tensor-parallel ranks need n_embd a multiple of 32 as well (checked by the engine).
bool step_supported(int n_heads, int n_kv_heads, int head_dim, int n_embd, int ffn);
cudaError_t step_init();
// Zero the arrival counter and launch the cooperative step grid on `st`.
cudaError_t step_launch(const StepParams& sp, cudaStream_t st);

}  // namespace af
