// af_step.cu — persistent decode-step kernel (see af_step.cuh for the design).
#include <cstddef>

#include "af_gemv_dev.cuh"
#include "af_step.cuh"

namespace af {

#ifdef AF_STEP_TRACE
// Timeline of one step (debug builds only): per CTA and phase, %globaltimer
// stamps at points of the phase (0 start, 1 input ready, 2 end, 3 producer
// done; the attention phase also 4-7 inside its item).
constexpr int kTracePh = 192;
__device__ unsigned long long g_trace[148][kTracePh][8];
__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
#define AF_TRACE(ph, k) \
    do { if (blockIdx.x < 148 && (ph) < kTracePh) g_trace[blockIdx.x][ph][k] = gtime(); } while (0)
#else
#define AF_TRACE(ph, k) do { } while (0)
#endif

namespace {

using namespace gdev;

constexpr int kParamOff = 1024;  // shared copies of the current phase's parameters
static_assert(offsetof(GemvParams, vrange) <= 448, "GemvParams head must fit its shared-memory slot");
static_assert(sizeof(AttnParams) <= 512, "AttnParams must fit its shared-memory slot");
static_assert(kParamOff + 512 + sizeof(AttnParams) <= kHdrRed, "step header overflow");
static_assert(kCW <= 16, "prologue scratch holds 16 warp sums");

// Spin limit of the grid-wide waits (each iteration is one L2 round trip,
// a few hundred ns: seconds in all).
constexpr uint32_t kGridSpinLimit = 1u << 24;

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid-wide phase arrivals: one release-reduction per CTA per phase on a
// counter that the waiters poll with acquire loads (a single L2 round trip
// on each side; no fence, no returned atomic on the critical path).
__device__ __forceinline__ void red_release(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Thread 0: count this CTA's arrival (its stores of the phase, ordered
// before by the consumer barrier, are released with it).
__device__ __forceinline__ void grid_arrive(unsigned* bar) { red_release(bar, 1u); }

// Consumer threads: wait until `target` arrivals have been counted.
// Thread 0 spins (bounded) and the consumer barrier publishes the result.
__device__ bool grid_wait(unsigned* bar, unsigned target, volatile int* flags) {
    if (threadIdx.x == 0) {
        bool ok = false;
        for (uint32_t i = 0; i < kGridSpinLimit; ++i) {
            if (ld_acquire(bar) >= target) {
                ok = true;
                break;
            }
            if ((i & 63) == 63 && flags[0]) break;
        }
        if (!ok) {
            if (!flags[0]) set_err(kErrMbarTimeout);
            flags[0] = 1;
        }
    }
    bar_consumers();
    return flags[0] == 0;
}

// ---- tensor-parallel exchanges (system scope: the counters and buffers of
// the other ranks are peer memory mapped into this process)
__device__ __forceinline__ void red_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ ulonglong2 ld_relaxed_sys2(const unsigned long long* p) {
    ulonglong2 v;
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}

// Input of a GEMV fed by tensor-parallel exchange `seq` (sequence number
// over the engine's life).  Thread t owns the float4 chunks j·kCT + t of the
// vector: it loads the residual chunks, then, RP ranks per pass, issues all
// its tagged-word loads of those ranks at once (16-byte vectors), re-polls
// the words whose tag is not yet this exchange's (bounded; every missing word
// per round trip), and adds the partials in rank order.  The sum goes to
// resid_out for the 32-value groups this CTA owns (group g: CTA g % grid) and
// is RMS-normalised and quantised into the shared XQ layout like an f32
// input.  False on a timeout or an abort.
template <int NIT>
__device__ bool xchg_input_t(const StepParams& sp, const XchgParams& x, unsigned long long seq, uint8_t* xqs,
                             float eps, volatile int* flags, float* red) {
    constexpr int RP = NIT <= 4 ? 2 : 1;  // ranks per pass: ≤ 16 vector loads in flight per thread
    const int tid = threadIdx.x;
    const int nvec = x.n / 4;
    const uint32_t tag = (uint32_t)(seq + 1ull);
    const unsigned long long* area = sp.xrecv[sp.rank] + (size_t)(seq & 1ull) * kStepMaxRanks * x.n;
    constexpr bool kEarlyW = NIT <= 4;  // norm weights in flight with the polls when registers allow
    float4 a[NIT], w[NIT];
#pragma unroll
    for (int j = 0; j < NIT; ++j) {
        const int v = j * kCT + tid;
        a[j] = v < nvec ? __ldcg(reinterpret_cast<const float4*>(x.resid_in) + v) : make_float4(0.f, 0.f, 0.f, 0.f);
        if (kEarlyW)
            w[j] = v < nvec ? __ldg(reinterpret_cast<const float4*>(x.norm_w) + v) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    bool ok = true;
    for (int r0 = 0; r0 < sp.tp && ok; r0 += RP) {
        ulonglong2 t[NIT][RP][2];
        auto word = [&](int j, int rr) { return area + (size_t)(r0 + rr) * x.n + 4 * (j * kCT + tid); };
        auto live = [&](int j, int rr) { return j * kCT + tid < nvec && r0 + rr < sp.tp; };
        auto have = [&](const ulonglong2& u) {
            return (uint32_t)(u.x >> 32) == tag && (uint32_t)(u.y >> 32) == tag;
        };
#pragma unroll
        for (int j = 0; j < NIT; ++j)
#pragma unroll
            for (int rr = 0; rr < RP; ++rr) {
                if (live(j, rr)) {
                    t[j][rr][0] = ld_relaxed_sys2(word(j, rr));
                    t[j][rr][1] = ld_relaxed_sys2(word(j, rr) + 2);
                } else {
                    t[j][rr][0] = t[j][rr][1] = make_ulonglong2((unsigned long long)tag << 32, (unsigned long long)tag << 32);
                }
            }
        for (uint32_t it = 0;; ++it) {
            bool all = true;
#pragma unroll
            for (int j = 0; j < NIT; ++j)
#pragma unroll
                for (int rr = 0; rr < RP; ++rr) all &= have(t[j][rr][0]) && have(t[j][rr][1]);
            if (all) break;
            if (it >= kGridSpinLimit || ((it & 15u) == 15u && flags[0])) {
                ok = false;
                break;
            }
#pragma unroll
            for (int j = 0; j < NIT; ++j)
#pragma unroll
                for (int rr = 0; rr < RP; ++rr)
#pragma unroll
                    for (int h = 0; h < 2; ++h)
                        if (!have(t[j][rr][h])) t[j][rr][h] = ld_relaxed_sys2(word(j, rr) + 2 * h);
        }
#pragma unroll
        for (int j = 0; j < NIT; ++j)
#pragma unroll
            for (int rr = 0; rr < RP; ++rr)
                if (r0 + rr < sp.tp) {
                    a[j].x += __uint_as_float((uint32_t)t[j][rr][0].x);
                    a[j].y += __uint_as_float((uint32_t)t[j][rr][0].y);
                    a[j].z += __uint_as_float((uint32_t)t[j][rr][1].x);
                    a[j].w += __uint_as_float((uint32_t)t[j][rr][1].y);
                }
    }
    if (!ok) {
        if (!flags[0]) set_err(kErrMbarTimeout);
        flags[0] = 1;
    }
    bar_consumers();
    if (flags[0]) return false;
#pragma unroll
    for (int j = 0; j < NIT; ++j) {
        const int v = j * kCT + tid;
        if (v < nvec && (v >> 3) % (int)gridDim.x == (int)blockIdx.x) reinterpret_cast<float4*>(x.resid_out)[v] = a[j];
        if (!kEarlyW)
            w[j] = v < nvec ? __ldg(reinterpret_cast<const float4*>(x.norm_w) + v) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    quantise_f4<NIT, true>(a, w, nvec, eps, xqs, red, sp.q8 != 0);
    bar_consumers();
    return true;
}

// PH_XRED: reduce exchange `seq` one 32-value group per warp (group
// w·grid + CTA, spread over the CTAs), store the new residual and quantise
// the RMSNorm-weighted sum into x.xq.  False on a timeout or an abort.
__device__ bool xred_phase(const StepParams& sp, const XchgParams& x, unsigned long long seq, volatile int* flags) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t tag = (uint32_t)(seq + 1ull);
    const unsigned long long* area = sp.xrecv[sp.rank] + (size_t)(seq & 1ull) * kStepMaxRanks * x.n;
    const int ng = x.n / 32;
    bool ok = true;
    for (int g = warp * (int)gridDim.x + (int)blockIdx.x; g < ng && ok; g += kCW * (int)gridDim.x) {
        const int v = 32 * g + lane;
        float a = __ldcg(x.resid_in + v);
        unsigned long long w[kStepMaxRanks];
#pragma unroll
        for (int r = 0; r < kStepMaxRanks; ++r)
            if (r < sp.tp) w[r] = ld_relaxed_sys(area + (size_t)r * x.n + v);
        for (uint32_t it = 0;; ++it) {
            bool all = true;
#pragma unroll
            for (int r = 0; r < kStepMaxRanks; ++r)
                if (r < sp.tp) all &= (uint32_t)(w[r] >> 32) == tag;
            if (__all_sync(0xffffffffu, all)) break;
            if (it >= kGridSpinLimit || ((it & 15u) == 15u && flags[0])) {
                ok = false;
                break;
            }
#pragma unroll
            for (int r = 0; r < kStepMaxRanks; ++r)
                if (r < sp.tp && (uint32_t)(w[r] >> 32) != tag) w[r] = ld_relaxed_sys(area + (size_t)r * x.n + v);
        }
        if (!ok) break;
#pragma unroll
        for (int r = 0; r < kStepMaxRanks; ++r)
            if (r < sp.tp) a += __uint_as_float((uint32_t)w[r]);
        x.resid_out[v] = a;
        xq_store32(x.xq, a, x.norm_w, x.n, v, sp.q8 != 0);
    }
    if (!ok) {
        if (!flags[0]) set_err(kErrMbarTimeout);
        flags[0] = 1;
    }
    return ok;
}

__device__ bool xchg_input(const StepParams& sp, const XchgParams& x, unsigned long long seq, uint8_t* xqs,
                           float eps, volatile int* flags, float* red) {
    switch ((x.n / 4 + kCT - 1) / kCT) {
        case 1: return xchg_input_t<1>(sp, x, seq, xqs, eps, flags, red);
        case 2: return xchg_input_t<2>(sp, x, seq, xqs, eps, flags, red);
        case 3: return xchg_input_t<3>(sp, x, seq, xqs, eps, flags, red);
        case 4: return xchg_input_t<4>(sp, x, seq, xqs, eps, flags, red);
        case 5: return xchg_input_t<5>(sp, x, seq, xqs, eps, flags, red);
        case 6: return xchg_input_t<6>(sp, x, seq, xqs, eps, flags, red);
        case 7: return xchg_input_t<7>(sp, x, seq, xqs, eps, flags, red);
        default: return xchg_input_t<8>(sp, x, seq, xqs, eps, flags, red);
    }
}

// Copy `bytes` (multiple of 4) of a parameter block into shared memory.
__device__ __forceinline__ void copy_params(void* dst, const void* src, int bytes) {
    for (int i = threadIdx.x; i < bytes / 4; i += kCT)
        reinterpret_cast<int*>(dst)[i] = __ldg(reinterpret_cast<const int*>(src) + i);
    bar_consumers();
}

// ------------------------------------------------------------------ embedding

// x = dequant(row token of the embedding) and its quantised, attn_norm-
// weighted form for the first QKV GEMV: one warp per 32 values.
__device__ void embed_phase(const StepParams& sp, int tok, float* row, float* red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (blockIdx.x == 0 && threadIdx.x == 0) *sp.key = 0ull;  // argmax of this step starts empty
    if (tok < 0 || tok >= sp.vocab) {  // never index outside the table
        if (blockIdx.x == 0 && threadIdx.x == 0) set_err(kErrBadToken);
        tok = 0;
    }
    const int nb = sp.n_embd / 256, ng = sp.n_embd / 32;
    if (sp.q8 && sp.xq && step_q8_exact_embed(sp.n_embd)) {
        // Q8_0 input of layer 0, exactly as the reference forms it:
        // rms_norm_out (src/models/llama_model.cpp:396-419) sums x² in 8
        // interleaved FMA chains added in lane order, then xn = w·(x·inv_rms)
        // is quantised; every CTA computes inv_rms itself (one row, cheap)
        const int E = sp.n_embd;
        for (int v = threadIdx.x; v < E; v += kCT) row[v] = embed_value(sp.tok_w, sp.tok_type, nb, sp.tok_stride, tok, v);
        bar_consumers();
        if (warp == 0) {
            float acc = 0.f;
            if (lane < 8)
                for (int i = lane; i < E; i += 8) acc = fmaf(row[i], row[i], acc);
            float ss = 0.f;
#pragma unroll
            for (int k = 0; k < 8; ++k) ss += __shfl_sync(0xffffffffu, acc, k);
            if (lane == 0) red[0] = 1.f / sqrtf(ss / (float)E + sp.eps);
        }
        bar_consumers();
        const float inv = red[0];
        for (int g = blockIdx.x * kCW + warp; g < ng; g += gridDim.x * kCW) {
            const int v = 32 * g + lane;
            const float a = row[v];
            sp.x[v] = a;
            xq_store32w(sp.xq, __ldg(sp.xq_norm_w + v) * (a * inv), 1.f, false, E, v, true);
        }
        return;
    }
    for (int g = blockIdx.x * kCW + warp; g < ng; g += gridDim.x * kCW) {
        const int v = 32 * g + lane;
        const float a = embed_value(sp.tok_w, sp.tok_type, nb, sp.tok_stride, tok, v);
        sp.x[v] = a;
        if (sp.xq) xq_store32(sp.xq, a, sp.xq_norm_w, sp.n_embd, v, sp.q8 != 0);
    }
}

// ------------------------------------------------------------------ attention

// Attention item: positions are taken in chunks of kStepAttnChunk; lane l of
// warp w holds K and V of positions w + kCW·i (i < kAttnPer) of the chunk at
// head dims 4l..4l+3 in registers, so the same thread needs its K rows for
// the scores and its V rows for P·V: no shared-memory staging of the cache.
constexpr int kAttnPer = kStepAttnChunk / kCW;
constexpr int kAttnMaxSplit = kStepAttnMaxSplit;
static_assert(kStepAttnChunk % kCW == 0 && kStepAttnChunk <= 64, "chunk: whole warps, two per lane at most");

// Shared scratch of one attention item (floats), inside the union area.
struct AttnSmem {
    float* qs;    // [G][hd]
    float* ks;    // [hd]
    float* vs;    // [hd]
    float* sc;    // [G][chunk] scores, then probabilities
    float* red;   // [kCW][hd] P·V partials of the warps
    float* mrow;  // [G]
    float* lrow;  // [G]
    float* corr;  // [G]
    float* ml;    // [G][nsplit][2] the splits' (max, sum), staged for the merge
    float* ob;    // [G][hd] the merged output, quantised from here
    int* last;
    __device__ explicit AttnSmem(uint8_t* base) {
        qs = reinterpret_cast<float*>(base);
        ks = qs + kStepMaxG * 128;
        vs = ks + 128;
        sc = vs + 128;
        red = sc + kStepMaxG * kStepAttnChunk;
        mrow = red + kCW * 128;
        lrow = mrow + kStepMaxG;
        corr = lrow + kStepMaxG;
        ml = corr + kStepMaxG;
        ob = ml + kStepMaxG * kAttnMaxSplit * 2;
        last = reinterpret_cast<int*>(ob + kStepMaxG * 128);
    }
};
static_assert(kCW == 8 && kAttnMaxSplit == kStepAttnMaxSplit, "kStepAttnScratch counts 8 warps");

// Per-thread K/V rows of the current chunk and the RoPE factors of the item.
struct AttnPre {
    float4 k[kAttnPer], v[kAttnPer];
    float c, s;
};

// Splits of each kv head's positions for this step: about one chunk per
// split, at most the configured maximum (the partial buffer's depth).
__device__ __forceinline__ int attn_splits(const AttnParams& a, int pos) {
    const int s = (pos + 1 + kStepAttnChunk - 1) / kStepAttnChunk;
    return max(1, min(a.nsplit, s));
}

// Range of positions of split `split` of `ns` for sequence length seq.
__device__ __forceinline__ void attn_range(int seq, int ns, int split, int& t0, int& t1) {
    const int chunk = (seq + ns - 1) / ns;
    t0 = min(seq, split * chunk);
    t1 = min(seq, t0 + chunk);
}

// One warp RMS-normalises one head in shared memory (qwen3 / hunyuan Q/K norm,
// rms_norm_out of src/models/llama_model.cpp:393-419 over hd values).
__device__ __forceinline__ void rms_norm_head(float* x, const float* w, int hd, float eps) {
    const int lane = threadIdx.x & 31;
    float ss = 0.f;
    for (int i = lane; i < hd; i += 32) ss += x[i] * x[i];
    ss = warp_sum(ss);
    const float s = 1.f / sqrtf(ss / (float)hd + eps);
    __syncwarp();
    for (int i = lane; i < hd; i += 32) x[i] = w[i] * (x[i] * s);
    __syncwarp();
}

// Request this thread's K (or V) registers of chunk positions [p0, p0 + n)
// that are older than pos (the new token's row comes from shared memory).
__device__ __forceinline__ void attn_load_rows(const float* cache, int hd, int kvd, int kvh, int p0, int n, int pos,
                                               float4 (&x)[kAttnPer]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < kAttnPer; ++i) {
        const int j = warp + kCW * i, p = p0 + j;
        x[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < n && p < pos && 4 * lane < hd)
            x[i] = __ldg(reinterpret_cast<const float4*>(cache + (size_t)p * kvd + (size_t)kvh * hd + 4 * lane));
    }
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Before the grid wait: pull into L2 everything of an item that does not
// depend on the QKV phase (its K/V rows older than the new token, the RoPE
// row), one bulk prefetch per cache row; no registers are held across the
// wait.
__device__ __forceinline__ void attn_prefetch(const AttnParams& a, int pos, int kvh, int split, int ns) {
    const int hd = a.head_dim, kvd = a.n_kv_heads * hd;
    int t0, t1;
    attn_range(pos + 1, ns, split, t0, t1);
    const int rows = min(t1, pos) - t0;  // rows in the cache (the new token is not yet)
    for (int i = threadIdx.x; i < 2 * rows; i += kCT) {
        const float* base = (i & 1) ? a.vc : a.kc;
        prefetch_l2(base + (size_t)(t0 + (i >> 1)) * kvd + (size_t)kvh * hd, (uint32_t)hd * 4);
    }
    if (threadIdx.x == kCT - 1) {
        prefetch_l2(a.cos_t + (size_t)pos * (hd / 2), (uint32_t)hd * 2);
        prefetch_l2(a.sin_t + (size_t)pos * (hd / 2), (uint32_t)hd * 2);
    }
}

constexpr int kAttnDistMerge = kStepAttnDistMerge;

// The spread merge of kv head kvh's ns split partials (every split published
// its un-normalised (o, max, sum) as tagged words): split `split` merges the
// 32-value output groups split, split + ns, ... of the head's G·hd outputs.
// For a group: the splits' (max, sum) of its head are polled into shared
// memory, M = max; warp w adds the splits q ≡ w (mod 8) for the group's 32
// dims (lane = dim; all its loads in flight, words whose tag is not this
// phase's re-polled, bounded), then warp 0 adds the 8 warps in order,
// normalises, stores and quantises the group for the O GEMV.
__device__ __forceinline__ void attn_merge_spread(const AttnParams& a, const AttnSmem& s, int kvh, int split, int ns,
                                               int G, int hd, unsigned long long tagw, volatile int* abort) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    auto poll = [&](const unsigned long long* p, unsigned long long w) {
        uint32_t it = 0;
        while ((w & ~0xFFFFFFFFull) != tagw && ++it < kGridSpinLimit && !*abort) w = ld_relaxed_gpu(p);
        if (it >= kGridSpinLimit) set_err(kErrMbarTimeout);
        return __uint_as_float((uint32_t)w);
    };
    constexpr int kPer = kAttnMaxSplit / kCW;  // splits per warp at most
    const int ngr = G * hd / 32;
    const int g0 = kvh * G * hd / 32;
    for (int gi = split; gi < ngr; gi += ns) {
        const int g = gi * 32 / hd, d0 = gi * 32 - g * hd;
        const unsigned long long* hb = a.tpart + (size_t)(kvh * G + g) * a.nsplit * (hd + 2);
        for (int q = tid; q < ns; q += kCT) {
            const unsigned long long* p = hb + (size_t)q * (hd + 2) + hd;
            s.ml[2 * q] = poll(p, ld_relaxed_gpu(p));
            s.ml[2 * q + 1] = poll(p + 1, ld_relaxed_gpu(p + 1));
        }
        bar_consumers();
        if (warp == 0) {
            float m = -INFINITY;
            for (int q = lane; q < ns; q += 32) m = fmaxf(m, s.ml[2 * q]);
            m = warp_max(m);
            if (lane == 0) s.corr[0] = m;
        }
        bar_consumers();
        const float M = s.corr[0];
        unsigned long long ov[kPer];
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int q = warp + kCW * k;
            ov[k] = q < ns ? ld_relaxed_gpu(hb + (size_t)q * (hd + 2) + d0 + lane) : 0ull;
        }
        float O = 0.f, L = 0.f;
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int q = warp + kCW * k;
            if (q >= ns) break;
            const float mq = s.ml[2 * q];
            if (mq == -INFINITY) continue;
            const float oq = poll(hb + (size_t)q * (hd + 2) + d0 + lane, ov[k]);
            const float w = expf(mq - M);
            L += s.ml[2 * q + 1] * w;
            O += oq * w;
        }
        s.red[warp * 32 + lane] = O;
        if (lane == 0) s.lrow[warp] = L;
        bar_consumers();
        if (warp == 0) {
            float Ot = 0.f, Lt = 0.f;
#pragma unroll
            for (int w = 0; w < kCW; ++w) {
                Ot += s.red[w * 32 + lane];
                Lt += s.lrow[w];
            }
            const float out = Ot / Lt;
            a.out[(size_t)kvh * G * hd + (size_t)gi * 32 + lane] = out;
            if (a.xq_out) xq_store32(a.xq_out, out, nullptr, a.n_heads * hd, 32 * (g0 + gi) + lane, a.q8 != 0);
        }
        bar_consumers();
    }
}

// One (kv head, split) item: llama_forward_token's attention
// (src/models/llama_model.cpp:1236-1272) for the G query heads of kv head kvh
// over positions [t0, t1), as an online softmax over chunks; the
// un-normalised partial (o, max, sum) goes to a.part and the last split of
// the kv head to finish merges them and quantises the output for the O GEMV.
// `r` holds the prefetched first chunk and RoPE factors.
// GM: query heads per kv head held in registers (G <= GM; the instance is
// chosen per model so that P·V accumulators cost 4·GM registers).
template <int GM, bool DIST>
__device__ __forceinline__ void attn_item(const AttnParams& a, const AttnSmem& s, int pos, int kvh, int split, int ns, AttnPre& r,
                                          int tph, uint32_t tag, volatile int* abort) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hd = a.head_dim, half = hd / 2, Q4 = hd / 4;
    const int G = a.n_heads / a.n_kv_heads;
    const int kvd = a.n_kv_heads * hd;
    const int seq = pos + 1;
    int t0, t1;
    attn_range(seq, ns, split, t0, t1);
    // first chunk's K/V rows and the RoPE factors (L2-resident after the
    // prefetch), in flight with the new token's q/k/v below.  RoPE pair i
    // of every head this thread rotates is tid % half (kCT is a multiple of half).
    attn_load_rows(a.kc, hd, kvd, kvh, t0, min(kStepAttnChunk, t1 - t0), pos, r.k);
    attn_load_rows(a.vc, hd, kvd, kvh, t0, min(kStepAttnChunk, t1 - t0), pos, r.v);
    r.c = __ldg(a.cos_t + (size_t)pos * half + tid % half);
    r.s = __ldg(a.sin_t + (size_t)pos * half + tid % half);

    // ---- q (G heads), k, v of the new token (written by the QKV phase)
    for (int i = tid; i < G * hd; i += kCT) s.qs[i] = __ldcg(a.q + (size_t)kvh * G * hd + i);
    for (int i = tid; i < hd; i += kCT) {
        s.ks[i] = __ldcg(a.k + (size_t)kvh * hd + i);
        s.vs[i] = __ldcg(a.v + (size_t)kvh * hd + i);
    }
    if (tid < kStepMaxG) {
        s.mrow[tid] = -INFINITY;
        s.lrow[tid] = 0.f;
    }
    bar_consumers();
    if (tid == 0) AF_TRACE(tph, 4);
    if (a.qk_norm_order == 1) {  // qwen3: per-head norm before RoPE
        for (int h = warp; h <= G; h += kCW) {
            if (h < G && a.q_norm) rms_norm_head(s.qs + h * hd, a.q_norm, hd, a.eps);
            if (h == G && a.k_norm) rms_norm_head(s.ks, a.k_norm, hd, a.eps);
        }
        bar_consumers();
    }
    // RoPE, half-split pairs (i, i + hd/2) (apply_rope, llama_model.cpp:1046-1080)
    for (int idx = tid; idx < (G + 1) * half; idx += kCT) {
        const int g = idx / half, i = idx % half;
        float* hp = g < G ? s.qs + g * hd : s.ks;
        const float x0 = hp[i], x1 = hp[i + half];
        hp[i] = x0 * r.c - x1 * r.s;
        hp[i + half] = x0 * r.s + x1 * r.c;
    }
    bar_consumers();
    if (a.qk_norm_order == 2) {  // hunyuan: per-head norm after RoPE
        for (int h = warp; h <= G; h += kCW) {
            if (h < G && a.q_norm) rms_norm_head(s.qs + h * hd, a.q_norm, hd, a.eps);
            if (h == G && a.k_norm) rms_norm_head(s.ks, a.k_norm, hd, a.eps);
        }
        bar_consumers();
    }
    if (split == 0) {
        for (int i = tid; i < hd; i += kCT) {
            a.kc[(size_t)pos * kvd + (size_t)kvh * hd + i] = s.ks[i];
            a.vc[(size_t)pos * kvd + (size_t)kvh * hd + i] = s.vs[i];
        }
    }

    // ---- chunks
    const bool dl = lane < Q4;  // this lane holds head dims 4·lane..4·lane+3
    float4 o[GM];
#pragma unroll
    for (int g = 0; g < GM; ++g) o[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p0 = t0; p0 < t1; p0 += kStepAttnChunk) {
        const int n = min(kStepAttnChunk, t1 - p0);
        if (p0 != t0) {
            attn_load_rows(a.kc, hd, kvd, kvh, p0, n, pos, r.k);
            attn_load_rows(a.vc, hd, kvd, kvh, p0, n, pos, r.v);
        }
        // the new token's row
#pragma unroll
        for (int i = 0; i < kAttnPer; ++i)
            if (p0 + warp + kCW * i == pos && dl) {
                r.k[i] = reinterpret_cast<const float4*>(s.ks)[lane];
                r.v[i] = reinterpret_cast<const float4*>(s.vs)[lane];
            }
        // scores q_g · k_j (lanes over the head dims, then a warp sum)
#pragma unroll
        for (int g = 0; g < GM; ++g) {
            if (g >= G) break;
            const float4 q = dl ? reinterpret_cast<const float4*>(s.qs + g * hd)[lane] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int i = 0; i < kAttnPer; ++i) {
                float d = q.x * r.k[i].x + q.y * r.k[i].y + q.z * r.k[i].z + q.w * r.k[i].w;
                d = warp_sum(d);
                const int j = warp + kCW * i;
                if (lane == 0 && j < n) s.sc[g * kStepAttnChunk + j] = d * a.scale;
            }
        }
        bar_consumers();
        // online softmax update, warp per head (max-subtracted exp, llama_model.cpp:445-451)
        static_assert(kStepMaxG <= kCW, "one warp per query head");
        if (warp < G) {
            float* sg = s.sc + warp * kStepAttnChunk;
            const float v0 = lane < n ? sg[lane] : -INFINITY;
            const float v1 = lane + 32 < n ? sg[lane + 32] : -INFINITY;
            const float m_old = s.mrow[warp];
            const float m_new = fmaxf(m_old, warp_max(fmaxf(v0, v1)));
            const float e0 = lane < n ? expf(v0 - m_new) : 0.f;
            const float e1 = lane + 32 < n ? expf(v1 - m_new) : 0.f;
            if (lane < n) sg[lane] = e0;
            if (lane + 32 < n) sg[lane + 32] = e1;
            const float l = warp_sum(e0 + e1);
            if (lane == 0) {
                const float c = expf(m_old - m_new);  // 0 on the first chunk (m_old = -inf)
                s.corr[warp] = c;
                s.lrow[warp] = s.lrow[warp] * c + l;
                s.mrow[warp] = m_new;
            }
        }
        bar_consumers();
        // P·V on this thread's rows
#pragma unroll
        for (int g = 0; g < GM; ++g) {
            if (g >= G) break;
            const float c = s.corr[g];
            o[g].x *= c;
            o[g].y *= c;
            o[g].z *= c;
            o[g].w *= c;
#pragma unroll
            for (int i = 0; i < kAttnPer; ++i) {
                const int j = warp + kCW * i;
                const float e = j < n ? s.sc[g * kStepAttnChunk + j] : 0.f;
                o[g].x = fmaf(e, r.v[i].x, o[g].x);
                o[g].y = fmaf(e, r.v[i].y, o[g].y);
                o[g].z = fmaf(e, r.v[i].z, o[g].z);
                o[g].w = fmaf(e, r.v[i].w, o[g].w);
            }
        }
        bar_consumers();  // sc is rewritten by the next chunk
    }
    if (tid == 0) AF_TRACE(tph, 5);
    if (tid == 0) AF_TRACE(tph, 5);
    // ---- reduce the warps.  Split 0 keeps its partial in shared memory; the
    // other splits publish theirs as tagged words (tag << 32 | bits) for it
    // and are done: no fence, counter or atomic.
    const unsigned long long tagw = (unsigned long long)tag << 32;
    // many splits (long context, few kv heads): every split publishes and the
    // merge is spread over the splits, one 32-value output group each, instead
    // of split 0 reading all of them
    const bool dist = DIST && ns > kAttnDistMerge;
#pragma unroll
    for (int g = 0; g < GM; ++g) {
        if (g >= G) break;
        if (dl) reinterpret_cast<float4*>(s.red + warp * hd)[lane] = o[g];
        bar_consumers();
        const int h = kvh * G + g;
        unsigned long long* dst = a.tpart + ((size_t)h * a.nsplit + split) * (hd + 2);
        for (int d = tid; d < hd; d += kCT) {
            float acc = 0.f;
#pragma unroll
            for (int w = 0; w < kCW; ++w) acc += s.red[w * hd + d];
            if (split == 0 && !dist) {
                s.ob[g * hd + d] = acc;
            } else {
                st_relaxed_gpu(dst + d, tagw | __float_as_uint(acc));
                if (d == 0) {
                    st_relaxed_gpu(dst + hd, tagw | __float_as_uint(s.mrow[g]));
                    st_relaxed_gpu(dst + hd + 1, tagw | __float_as_uint(s.lrow[g]));
                }
            }
        }
        bar_consumers();
    }
    if (dist) {
        attn_merge_spread(a, s, kvh, split, ns, G, hd, tagw, abort);
        if (tid == 0) AF_TRACE(tph, 7);
        return;
    }
    if (split != 0) return;
    // ---- split 0 merges the splits (exp(m_s − M) rescaling): the other
    // splits' (max, sum) staged in shared memory, then each output value
    // loads its splits' partials together; a word whose tag is not this
    // phase's yet is re-polled (bounded).  The output goes to global memory
    // and stays in shared memory, from where it is quantised.
    if (ns > 1) {
        auto poll = [&](const unsigned long long* p) {
            unsigned long long w = ld_relaxed_gpu(p);
            uint32_t it = 0;
            while ((w & ~0xFFFFFFFFull) != tagw && ++it < kGridSpinLimit && !*abort) w = ld_relaxed_gpu(p);
            if (it >= kGridSpinLimit) set_err(kErrMbarTimeout);
            return __uint_as_float((uint32_t)w);
        };
        for (int i = tid; i < G * ns; i += kCT) {
            const int g = i / ns, q = i - g * ns;
            if (q == 0) {
                s.ml[2 * i] = s.mrow[g];
                s.ml[2 * i + 1] = s.lrow[g];
            } else {
                const unsigned long long* b = a.tpart + ((size_t)(kvh * G + g) * a.nsplit + q) * (hd + 2);
                s.ml[2 * i] = poll(b + hd);
                s.ml[2 * i + 1] = poll(b + hd + 1);
            }
        }
        bar_consumers();
        constexpr int kBatch = 8;  // partial loads in flight per output value
        for (int idx = tid; idx < G * hd; idx += kCT) {
            const int g = idx / hd, dd = idx - g * hd;
            const unsigned long long* base = a.tpart + (size_t)(kvh * G + g) * a.nsplit * (hd + 2) + dd;
            const float* mlg = s.ml + 2 * g * ns;
            float M = -INFINITY;
            for (int q = 0; q < ns; ++q) M = fmaxf(M, mlg[2 * q]);
            float L = 0.f, O = 0.f;
            for (int q0 = 0; q0 < ns; q0 += kBatch) {
                unsigned long long ov[kBatch];
#pragma unroll
                for (int j = 0; j < kBatch; ++j)
                    ov[j] = q0 + j > 0 && q0 + j < ns ? ld_relaxed_gpu(base + (size_t)(q0 + j) * (hd + 2)) : 0ull;
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    const int q = q0 + j;
                    if (q >= ns || mlg[2 * q] == -INFINITY) continue;
                    float oq;
                    if (q == 0) {
                        oq = s.ob[idx];
                    } else if ((ov[j] & ~0xFFFFFFFFull) == tagw) {
                        oq = __uint_as_float((uint32_t)ov[j]);
                    } else {
                        oq = poll(base + (size_t)q * (hd + 2));
                    }
                    const float w = expf(mlg[2 * q] - M);
                    L += mlg[2 * q + 1] * w;
                    O += oq * w;
                }
            }
            s.ob[idx] = O / L;
        }
    } else {
        for (int idx = tid; idx < G * hd; idx += kCT) s.ob[idx] /= s.lrow[idx / hd];
    }
    bar_consumers();
    for (int idx = tid; idx < G * hd; idx += kCT) a.out[(size_t)kvh * G * hd + idx] = s.ob[idx];
    if (a.xq_out) {
        // quantise this kv head's G*hd outputs (32-value groups) for the O GEMV
        const int g0 = kvh * G * hd / 32, ng = G * hd / 32;
        for (int k = warp; k < ng; k += kCW)
            xq_store32(a.xq_out, s.ob[32 * k + lane], nullptr, a.n_heads * hd, 32 * (g0 + k) + lane, a.q8 != 0);
    }
    if (tid == 0) AF_TRACE(tph, 7);
}

// The whole attention phase of one layer for this CTA: the prefetch of what
// does not depend on the QKV phase, the grid wait, then the CTA's items.
template <int GM, bool DIST>
__device__ __forceinline__ bool attn_phase(const AttnParams& a, const AttnSmem& s, int pos, unsigned* bar,
                                           unsigned target, volatile int* abort, int tph, uint32_t tag) {
    const int ns = attn_splits(a, pos);
    const int items = a.n_kv_heads * ns;
    for (int item = blockIdx.x; item < items; item += gridDim.x) attn_prefetch(a, pos, item / ns, item % ns, ns);
    if (!grid_wait(bar, target, abort)) return false;
    if (threadIdx.x == 0) AF_TRACE(tph, 0);
    for (int item = blockIdx.x; item < items; item += gridDim.x) {
        AttnPre r;
        attn_item<GM, DIST>(a, s, pos, item / ns, item % ns, ns, r, tph, tag, abort);
        bar_consumers();
    }
    return true;
}

// ------------------------------------------------------------------ kernel

// DIST: the instance whose attention can spread the merge of more than
// kAttnDistMerge splits (engines whose kv heads allow that many splits); the
// other instance carries no code for it.
template <bool DIST>
__global__ void __launch_bounds__(kGemvThreads, 1) step_kernel(const __grid_constant__ StepParams sp) {
    extern __shared__ __align__(128) uint8_t smem[];
    Ring ring;
    ring.full = reinterpret_cast<uint64_t*>(smem);
    ring.empty = ring.full + kRingDesc;
    int* flags = reinterpret_cast<int*>(smem + kHdrFlags);  // [0] abort, [1..] group list
    GemvParams* gp = reinterpret_cast<GemvParams*>(smem + kParamOff);
    float* red = reinterpret_cast<float*>(smem + kParamOff + 448);  // 16 floats
    AttnParams* ap = reinterpret_cast<AttnParams*>(smem + kParamOff + 512);
    uint8_t* uni = smem + kStepHdr;
    ring.buf = uni + sp.union_bytes;
    ring.bytes = sp.ring_bytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRingDesc; ++i) {
            mbar_init(&ring.full[i], 1);
            mbar_init(&ring.empty[i], kCW);
        }
        flags[0] = 0;
        fence_mbar_init();
    }
    __syncthreads();
    volatile int* abort = flags;

    if (warp == kCW) {
        // ---- producer: the weights of every GEMV phase, in order
        if (lane != 0) return;
        Producer pr;
        const uint64_t pol = policy_evict_first();
        for (int i = 0; i < sp.nph; ++i) {
            const StepPhase& ph = sp.ph[i];
            if (ph.kind != PH_GEMV) continue;
            const int vbeg = ph.g.vrange[blockIdx.x], vend = ph.g.vrange[blockIdx.x + 1];
            if (!pr.produce(ph.g, vbeg, vend, ring, abort, pol)) {
                *abort = 1;
                pr.drain(ring);
                return;
            }
            AF_TRACE(i, 3);
        }
        return;
    }

    // ---- consumers: the phases, separated by grid-wide arrivals
    const int pos = __ldcg(sp.pos);
    const int tok = __ldcg(sp.token);
    const unsigned long long epoch = __ldcg(sp.epoch);
    // sequence number of partial-sum exchange k of this step
    auto xseq = [&](int k) { return epoch * (unsigned long long)sp.n_buf + (unsigned long long)k; };
    uint32_t consumed = 0;
    int head = 0;
    const unsigned grid = gridDim.x;
    for (int i = 0; i < sp.nph; ++i) {
        const StepPhase& ph = sp.ph[i];
        const int kind = ph.kind;
        if (kind == PH_ATTN) {
            copy_params(ap, &ph.a, sizeof(AttnParams));
            const int G = ap->n_heads / ap->n_kv_heads;
            const AttnSmem s(uni);
            const unsigned target = (unsigned)i * grid;
            // tag of this phase's split partials: unique per step and phase, never 0
            const uint32_t atag = (uint32_t)(epoch * (unsigned long long)sp.nph + (unsigned long long)i + 1ull);
            bool ok;
            if (G == 1) ok = attn_phase<1, DIST>(*ap, s, pos, sp.bar, target, abort, i, atag);
            else if (G == 2) ok = attn_phase<2, DIST>(*ap, s, pos, sp.bar, target, abort, i, atag);
            else if (G <= 4) ok = attn_phase<4, DIST>(*ap, s, pos, sp.bar, target, abort, i, atag);
            else ok = attn_phase<kStepMaxG, DIST>(*ap, s, pos, sp.bar, target, abort, i, atag);
            if (!ok) break;
        } else {
            // a GEMV fed by an exchange waits for the tagged partials instead
            // of the grid (the tags arrive only after every rank's producing
            // phase, and everything else it reads is older)
            const bool xin = (kind == PH_GEMV && ph.x.k_in >= 0) || kind == PH_XRED;
            // the phase's parameters and fragment range do not depend on the
            // previous phase: fetch them before waiting for it
            int vbeg = 0, vend = 0;
            if (kind == PH_GEMV) {
                copy_params(gp, &ph.g, offsetof(GemvParams, vrange));
                vbeg = __ldg(ph.g.vrange + blockIdx.x);
                vend = __ldg(ph.g.vrange + blockIdx.x + 1);
            }
            if (i > 0 && !xin && !grid_wait(sp.bar, (unsigned)i * grid, abort)) break;
            if (threadIdx.x == 0) AF_TRACE(i, 0);
            if (kind == PH_EMBED) {
                embed_phase(sp, tok, reinterpret_cast<float*>(uni), red);
            } else if (kind == PH_XRED) {
                if (!xred_phase(sp, ph.x, xseq(ph.x.k_in), abort)) {
                    *abort = 1;
                    break;
                }
            } else {
                if (ph.x.k_out >= 0) {  // row-parallel partial sums, sent to every rank
                    if (threadIdx.x == 0) {
                        const unsigned long long q = xseq(ph.x.k_out);
                        for (int r = 0; r < sp.tp; ++r)
                            gp->xsend[r] = sp.xrecv[r] + ((size_t)(q & 1ull) * kStepMaxRanks + sp.rank) * ph.x.n;
                        gp->xsend_n = sp.tp;
                        gp->xtag = (uint32_t)(q + 1ull);
                    }
                    bar_consumers();
                }
                float s_in = 1.f;
                if (xin) {
                    if (!xchg_input(sp, ph.x, xseq(ph.x.k_in), uni, gp->eps, abort, red)) break;
                } else if (gp->xq) {
                    s_in = load_xq(*gp, uni);
                } else {
                    input_prologue(*gp, uni, red);
                }
                if (threadIdx.x == 0) AF_TRACE(i, 1);
                if (!consume(*gp, vbeg, vend, ring, consumed, head, uni, s_in, smem)) {
                    *abort = 1;
                    break;
                }
            }
        }
        // arrive: every store of this phase by this CTA happens before the count
        bar_consumers();
        if (threadIdx.x == 0) AF_TRACE(i, 2);
        if (threadIdx.x == 0) grid_arrive(sp.bar);
    }
    // CTA 0 turns the step's argmax into the next token once every CTA has
    // finished the LM head, and advances the position.
    if (blockIdx.x == 0 && threadIdx.x == 0 && !*abort) {
        const unsigned target = (unsigned)sp.nph * grid;
        uint32_t it = 0;
        while (ld_acquire(sp.bar) < target && ++it < kGridSpinLimit) {
        }
        if (it >= kGridSpinLimit) {
            set_err(kErrMbarTimeout);
            return;
        }
        unsigned long long k = __ldcg(sp.key);
        if (sp.tp > 1) {
            // argmax over the ranks' vocabulary shards: publish this rank's key
            // in every rank's key slot and count one arrival per rank and step
            for (int r = 0; r < sp.tp; ++r) {
                sp.xkey[r][sp.rank] = k;
                red_release_sys(sp.xbar[r], 1ull);
            }
            const unsigned long long target = (unsigned long long)sp.tp * (epoch + 1ull);
            uint32_t it2 = 0;
            while (ld_acquire_sys(sp.xbar[sp.rank]) < target && ++it2 < kGridSpinLimit) {
            }
            if (it2 >= kGridSpinLimit) {
                set_err(kErrMbarTimeout);
                return;
            }
            for (int r = 0; r < sp.tp; ++r) {
                const unsigned long long kr = __ldcv(sp.xkey[sp.rank] + r);
                k = kr > k ? kr : k;
            }
        }
        *sp.epoch = epoch + 1ull;
        int id = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
        if (k == 0ull || id < 0 || id >= sp.vocab) {  // no finite logit reached the argmax
            set_err(kErrBadToken);
            id = 0;
        }
        *sp.token = id;
        if (sp.hist) sp.hist[pos] = id;
        *sp.pos = pos + 1;
    }
}

}  // namespace

bool step_supported(int n_heads, int n_kv_heads, int head_dim, int n_embd, int ffn) {
    const int G = n_kv_heads > 0 ? n_heads / n_kv_heads : 0;
    return G >= 1 && G <= kStepMaxG && (head_dim == 64 || head_dim == 128) && n_embd % 256 == 0 && ffn % 256 == 0 &&
           xq_norm_bytes(n_embd) <= kStepUnion && xq_norm_bytes(ffn) <= kStepUnion && (G * head_dim) % 64 == 0;
}

cudaError_t step_init() {
    AF_CUDA_TRY(cudaFuncSetAttribute(step_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kStepSmem));
    return cudaFuncSetAttribute(step_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kStepSmem);
}

cudaError_t step_launch(const StepParams& sp, cudaStream_t st) {
    AF_CUDA_TRY(cudaMemsetAsync(sp.bar, 0, sizeof(unsigned int), st));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms());
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = kStepSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (sp.attn_dist) return cudaLaunchKernelEx(&cfg, step_kernel<true>, sp);
    return cudaLaunchKernelEx(&cfg, step_kernel<false>, sp);
}

}  // namespace af

#ifdef AF_STEP_TRACE
extern "C" cudaError_t af_debug_step_trace(void* h_out, size_t bytes) {
    return cudaMemcpyFromSymbol(h_out, af::g_trace, bytes);
}
#endif
