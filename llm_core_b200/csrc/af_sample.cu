// af_sample.cu — token sampling on the device: repetition penalty, greedy
// argmax or temperature / top-k / top-p sampling with a caller-supplied
// uniform draw, in one CTA.
//
// Mirrors the reference's decode-loop sampling step:
//   apply_rep_penalty (src/models/llama_model.cpp:1586-1598): for each id of
//     the window, in window order, logit /= penalty if positive else *= it
//     (an id present twice is penalised twice);
//   sample (src/models/llama_model.cpp:1466-1498): greedy first maximum at
//     temperature <= 0; otherwise the k = top_k largest of logit/temperature
//     in descending order, p_i = exp(s_i - s_0) summed and normalised in
//     order, the nucleus cut at the first cumulative p >= top_p and
//     renormalised, then the first i whose cumulative p exceeds the draw r.
// The sums and cumulative comparisons run in the reference's order on one
// thread, so a pick differs from the reference's only through expf rounding
// (a few ulp) when r lies within that distance of a cumulative boundary.  Ties
// at the k-th value keep the lowest indices (std::partial_sort leaves their
// order unspecified).
//
// The top k are found without sorting the vocabulary: a radix select on the
// order-preserving 32-bit keys of logit/temperature (four 8-bit passes with a
// shared histogram) finds the k-th largest key, the candidates are gathered
// (those above it, and the lowest-index ties) and a bitonic sort orders them.
#include <cuda_runtime.h>

#include "af_common.cuh"
#include "af_ops.cuh"

namespace af {
namespace {

constexpr int kSampleThreads = 1024;
constexpr int kSampleMaxK = 1024;  // candidates sorted in shared memory

__device__ __forceinline__ unsigned long long cand_key(float v, int idx) {
    // descending by value, then ascending by index
    return (static_cast<unsigned long long>(float_to_ordered(v)) << 32) | (0xFFFFFFFFu - (uint32_t)idx);
}

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(float* logits, int V, const int* window, int n_window,
                                                                 af_sampling s, float r, int* out) {
    __shared__ unsigned int hist[256];
    __shared__ unsigned long long cand[kSampleMaxK];
    __shared__ float prob[kSampleMaxK];
    __shared__ unsigned int s_prefix, s_mask, s_need, s_cnt;
    __shared__ int s_idx;
    __shared__ int tie_base[kSampleThreads / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    // ---- repetition penalty, sequentially in window order
    if (tid == 0 && s.rep_penalty != 1.f) {
        for (int i = 0; i < n_window; ++i) {
            const int id = window[i];
            if (id < 0 || id >= V) continue;
            const float v = logits[id];
            logits[id] = v > 0.f ? v / s.rep_penalty : v * s.rep_penalty;
        }
    }
    __syncthreads();

    // ---- greedy: first maximum
    if (!(s.temperature > 0.f)) {
        unsigned long long best = 0ull;
        for (int i = tid; i < V; i += kSampleThreads) {
            const unsigned long long k = cand_key(logits[i], i);
            best = k > best ? k : best;
        }
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long x = __shfl_xor_sync(0xffffffffu, best, o);
            best = x > best ? x : best;
        }
        if (lane == 0) cand[warp] = best;
        __syncthreads();
        if (tid == 0) {
            unsigned long long b = 0ull;
            for (int w = 0; w < kSampleThreads / 32; ++w) b = cand[w] > b ? cand[w] : b;
            *out = (int)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull));
        }
        return;
    }

    const float T = s.temperature;
    const int k = (s.top_k > 0 && s.top_k < V) ? s.top_k : V;  // the host keeps k <= kSampleMaxK

    // ---- radix select: key of the k-th largest scaled logit
    if (tid == 0) {
        s_prefix = 0u;
        s_mask = 0u;
        s_need = (unsigned)k;
    }
    for (int shift = 24; shift >= 0; shift -= 8) {
        if (tid < 256) hist[tid] = 0u;
        __syncthreads();
        const unsigned prefix = s_prefix, mask = s_mask;
        for (int i = tid; i < V; i += kSampleThreads) {
            const unsigned key = float_to_ordered(logits[i] / T);
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            unsigned need = s_need, above = 0u;
            int b = 255;
            for (; b > 0; --b) {
                if (above + hist[b] >= need) break;
                above += hist[b];
            }
            s_need = need - above;
            s_prefix = prefix | ((unsigned)b << shift);
            s_mask = mask | (255u << shift);
        }
        __syncthreads();
    }
    const unsigned kth = s_prefix;  // key of the k-th largest
    const unsigned need_ties = s_need;  // how many elements equal to it are taken

    // ---- gather: keys above the k-th, and the lowest-index ties
    if (tid == 0) s_cnt = 0u;
    // ties are ranked by index: thread t scans the contiguous block t of the vocabulary
    const int per = (V + kSampleThreads - 1) / kSampleThreads;
    const int b0 = tid * per, b1 = min(V, b0 + per);
    int my_ties = 0;
    for (int i = b0; i < b1; ++i) my_ties += float_to_ordered(logits[i] / T) == kth;
    // exclusive scan of the tie counts over the block (warp scan + warp totals)
    int incl = my_ties;
    for (int o = 1; o < 32; o <<= 1) {
        const int x = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += x;
    }
    if (lane == 31) tie_base[warp] = incl;
    __syncthreads();
    if (tid == 0) {
        int acc = 0;
        for (int w = 0; w < kSampleThreads / 32; ++w) {
            const int t = tie_base[w];
            tie_base[w] = acc;
            acc += t;
        }
    }
    __syncthreads();
    int rank = tie_base[warp] + incl - my_ties;
    for (int i = b0; i < b1; ++i) {
        const float v = logits[i] / T;
        const unsigned key = float_to_ordered(v);
        bool take = key > kth;
        if (key == kth) take = (unsigned)(rank++) < need_ties;
        if (take) {
            const unsigned slot = atomicAdd(&s_cnt, 1u);
            if (slot < (unsigned)kSampleMaxK) cand[slot] = cand_key(v, i);
        }
    }
    __syncthreads();
    // pad and bitonic-sort the candidates, descending
    for (int i = tid; i < kSampleMaxK; i += kSampleThreads)
        if (i >= k) cand[i] = 0ull;
    __syncthreads();
    for (int size = 2; size <= kSampleMaxK; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < kSampleMaxK; i += kSampleThreads) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool desc = (i & size) == 0;
                    const unsigned long long a = cand[i], c = cand[j];
                    if (desc ? a < c : a > c) {
                        cand[i] = c;
                        cand[j] = a;
                    }
                }
            }
            __syncthreads();
        }
    }

    // ---- probabilities, in the reference's order
    const float mx = ordered_to_float((uint32_t)(cand[0] >> 32));
    for (int i = tid; i < k; i += kSampleThreads) prob[i] = expf(ordered_to_float((uint32_t)(cand[i] >> 32)) - mx);
    __syncthreads();
    if (tid == 0) {
        float sum = 0.f;
        for (int i = 0; i < k; ++i) sum += prob[i];
        for (int i = 0; i < k; ++i) prob[i] /= sum;
        int kk = k;
        if (s.top_p < 1.0f) {
            float cum = 0.f;
            int cut = k;
            for (int i = 0; i < k; ++i) {
                cum += prob[i];
                if (cum >= s.top_p) {
                    cut = i + 1;
                    break;
                }
            }
            sum = 0.f;
            for (int i = 0; i < cut; ++i) sum += prob[i];
            for (int i = 0; i < cut; ++i) prob[i] /= sum;
            kk = cut;
        }
        float cum = 0.f;
        int pick = kk - 1;
        for (int i = 0; i < kk; ++i) {
            cum += prob[i];
            if (r < cum) {
                pick = i;
                break;
            }
        }
        s_idx = (int)(0xFFFFFFFFu - (uint32_t)(cand[pick] & 0xFFFFFFFFull));
        *out = s_idx;
    }
}

}  // namespace

cudaError_t sample_launch(float* d_logits, int vocab, const int* d_window, int n_window, const af_sampling& s, float r,
                          int* d_out, cudaStream_t st) {
    sample_kernel<<<1, kSampleThreads, 0, st>>>(d_logits, vocab, d_window, n_window, s, r, d_out);
    return cudaGetLastError();
}

bool sample_supported(const af_sampling& s, int vocab, std::string* why) {
    if (!(s.temperature > 0.f)) return true;
    const int k = (s.top_k > 0 && s.top_k < vocab) ? s.top_k : vocab;
    if (k > kSampleMaxK) {
        if (why) *why = "top_k must be in 1.." + std::to_string(kSampleMaxK) + " when temperature > 0 (got k = " +
                        std::to_string(k) + ")";
        return false;
    }
    if (s.rep_penalty <= 0.f) {
        if (why) *why = "rep_penalty must be positive";
        return false;
    }
    return true;
}

}  // namespace af

extern "C" cudaError_t af_sample_f32(float* d_logits, int vocab, const int32_t* d_window, int n_window,
                                     const af_sampling* s, float r, int32_t* d_out, cudaStream_t stream) {
    if (!d_logits || !s || !d_out || vocab <= 0 || n_window < 0 || (n_window > 0 && !d_window)) {
        af::set_last_error("af_sample_f32: bad arguments");
        return cudaErrorInvalidValue;
    }
    std::string why;
    if (!af::sample_supported(*s, vocab, &why)) {
        af::set_last_error("af_sample_f32: " + why);
        return cudaErrorNotSupported;
    }
    return af::sample_launch(d_logits, vocab, d_window, n_window, *s, r, d_out, stream);
}
