// af_attention.cu — GQA decode attention over the fp32 KV cache, fused with
// RoPE, optional per-head Q/K RMSNorm and the KV-cache store of the new token.
//
// Reference: llama_forward_token (src/models/llama_model.cpp:1236-1272) —
// RoPE (half-split, apply_rope / rope_and_store_k, :1046-1080), V copy into the
// cache, then per head: scores = q·k_t / sqrt(hd), max-subtracted softmax
// (:445-451), o = Σ p_t v_t, with kv head h / (H / KVH).  The reference runs
// this serially on one thread; here it is split over (kv head, position chunk)
// CTAs ("flash decoding"): each CTA produces an un-normalised partial
// (o, running max, sum) and the last CTA of a kv head merges the partials with
// the usual exp(m_s − M) rescaling.  Cache layout is the reference's:
// [n_ctx][n_kv_heads * head_dim] per layer, fp32.
#include <cuda.h>
#include <mutex>
#include <string>

#include "af_ops.cuh"

namespace af {
namespace {

constexpr int kAttnThreads = 128;

// Score slots per head: positions per split rounded up to 4 floats so the
// areas after the scores stay 16-byte aligned for float4 access.
__host__ __device__ inline int attn_chunk_max(int n_ctx, int nsplit) {
    return ((n_ctx + nsplit - 1) / nsplit + 3) & ~3;
}

// Floats of the scratch area shared by the score partials [4][G][32] and the
// output partials [position groups][G][hd].
__host__ __device__ inline int attn_red1_floats(int G, int hd) {
    const int a = 4 * G * 32, b = (kAttnThreads / (hd / 4)) * G * hd;
    return a > b ? a : b;
}

__device__ __forceinline__ void rms_norm_head(float* x, const float* w, int hd, float eps, float* red) {
    // one warp (warp 0) normalises one head in shared memory
    const int lane = threadIdx.x & 31;
    float ss = 0.f;
    for (int i = lane; i < hd; i += 32) ss += x[i] * x[i];
    ss = warp_sum(ss);
    const float s = 1.f / sqrtf(ss / (float)hd + eps);
    __syncwarp();
    for (int i = lane; i < hd; i += 32) x[i] = w[i] * (x[i] * s);
    __syncwarp();
    (void)red;
}

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const __grid_constant__ AttnParams p) {
    extern __shared__ __align__(16) float sm[];
    const int hd = p.head_dim, half = hd / 2;
    const int G = p.n_heads / p.n_kv_heads;
    const int kvh = blockIdx.x, split = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kvd = p.n_kv_heads * hd;
    const int chunk_max = attn_chunk_max(p.n_ctx, p.nsplit);

    float* qs = sm;                 // [G][hd]
    float* ks = qs + G * hd;        // [hd]
    float* vs = ks + hd;            // [hd]
    float* sc = vs + hd;            // [G][chunk_max]
    float* red = sc + G * chunk_max + attn_red1_floats(G, hd);  // [64]

    pdl_launch_dependents();
    pdl_wait();
    const int pos = *p.pos;
    const int seq = pos + 1;
    const float* cr = p.cos_t + (size_t)pos * half;
    const float* sr = p.sin_t + (size_t)pos * half;

    // ---- load q (G heads), k, v of the new token
    for (int i = tid; i < G * hd; i += kAttnThreads) qs[i] = p.q[(size_t)kvh * G * hd + i];
    for (int i = tid; i < hd; i += kAttnThreads) {
        ks[i] = p.k[(size_t)kvh * hd + i];
        vs[i] = p.v[(size_t)kvh * hd + i];
    }
    __syncthreads();
    if (p.qk_norm_order == 1 && warp == 0) {  // qwen3: per-head norm before RoPE
        if (p.q_norm) for (int g = 0; g < G; ++g) rms_norm_head(qs + g * hd, p.q_norm, hd, p.eps, red);
        if (p.k_norm) rms_norm_head(ks, p.k_norm, hd, p.eps, red);
    }
    __syncthreads();
    // RoPE: pairs (i, i + hd/2)
    for (int idx = tid; idx < (G + 1) * half; idx += kAttnThreads) {
        const int g = idx / half, i = idx % half;
        float* hp = g < G ? qs + g * hd : ks;
        const float x0 = hp[i], x1 = hp[i + half];
        hp[i] = x0 * cr[i] - x1 * sr[i];
        hp[i + half] = x0 * sr[i] + x1 * cr[i];
    }
    __syncthreads();
    if (p.qk_norm_order == 2 && warp == 0) {  // hunyuan: per-head norm after RoPE
        if (p.q_norm) for (int g = 0; g < G; ++g) rms_norm_head(qs + g * hd, p.q_norm, hd, p.eps, red);
        if (p.k_norm) rms_norm_head(ks, p.k_norm, hd, p.eps, red);
    }
    __syncthreads();
    if (split == 0) {
        for (int i = tid; i < hd; i += kAttnThreads) {
            p.kc[(size_t)pos * kvd + (size_t)kvh * hd + i] = ks[i];
            p.vc[(size_t)pos * kvd + (size_t)kvh * hd + i] = vs[i];
        }
    }

    // ---- this CTA's positions
    const int chunk = (seq + p.nsplit - 1) / p.nsplit;
    const int t0 = split * chunk;
    const int t1 = min(seq, t0 + chunk);
    const int nt = max(0, t1 - t0);
    const int q4 = hd / 4;              // float4 per row
    float* red1 = sc + G * chunk_max;   // [4][G][32] partial scores, later [npg][G][hd]

    // scores: thread = (position lane, quarter of the head dims); all of a
    // thread's K loads are independent, so a tile costs one memory latency.
    for (int j0 = 0; j0 < nt; j0 += 32) {
        const int j = j0 + lane;
        const int quarter = warp;
        const int d0 = quarter * (q4 / 4);  // first float4 of this quarter
        float part[16];
#pragma unroll
        for (int g = 0; g < 16; ++g) part[g] = 0.f;
        if (j < nt) {
            const int t = t0 + j;
            const float4* kr = reinterpret_cast<const float4*>((t == pos) ? ks : p.kc + (size_t)t * kvd + (size_t)kvh * hd);
            float4 kv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (i < q4 / 4) kv[i] = kr[d0 + i];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (i >= q4 / 4) break;
#pragma unroll
                for (int g = 0; g < 16; ++g) {
                    if (g >= G) break;
                    const float4 qv = reinterpret_cast<const float4*>(qs + g * hd)[d0 + i];
                    part[g] += qv.x * kv[i].x + qv.y * kv[i].y + qv.z * kv[i].z + qv.w * kv[i].w;
                }
            }
        }
#pragma unroll
        for (int g = 0; g < 16; ++g)
            if (g < G) red1[(quarter * G + g) * 32 + lane] = part[g];
        __syncthreads();
        for (int idx = tid; idx < G * 32; idx += kAttnThreads) {
            const int g = idx / 32, l = idx % 32;
            if (j0 + l < nt) {
                const float s = red1[(0 * G + g) * 32 + l] + red1[(1 * G + g) * 32 + l] +
                                red1[(2 * G + g) * 32 + l] + red1[(3 * G + g) * 32 + l];
                sc[g * chunk_max + j0 + l] = s * p.scale;
            }
        }
        __syncthreads();
    }
    // softmax pieces per head: warp w handles heads w, w+4, ...
    float* mrow = red;       // [G] (G <= 32)
    float* lrow = red + 32;  // [G]
    for (int g = warp; g < G; g += kAttnThreads / 32) {
        float m = -INFINITY;
        for (int j = lane; j < nt; j += 32) m = fmaxf(m, sc[g * chunk_max + j]);
        m = warp_max(m);
        float l = 0.f;
        for (int j = lane; j < nt; j += 32) {
            const float e = expf(sc[g * chunk_max + j] - m);
            sc[g * chunk_max + j] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) { mrow[g] = m; lrow[g] = l; }
    }
    __syncthreads();
    // o_g[d] = Σ_t e_t v_t[d]: thread = (float4 of dims, position group);
    // positions unrolled by 4 so the V loads overlap.
    const int npg = kAttnThreads / q4;  // 4 (hd=128) or 8 (hd=64)
    const int d4 = tid % q4, pg = tid / q4;
    float4 acc[16];
#pragma unroll
    for (int g = 0; g < 16; ++g) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int jb = pg * 4; jb < nt; jb += npg * 4) {
        float4 vv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int j = jb + u;
            const int t = t0 + j;
            vv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (j < nt)
                vv[u] = (t == pos) ? reinterpret_cast<const float4*>(vs)[d4]
                                   : reinterpret_cast<const float4*>(p.vc + (size_t)t * kvd + (size_t)kvh * hd)[d4];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int j = jb + u;
            if (j >= nt) break;
#pragma unroll
            for (int g = 0; g < 16; ++g) {
                if (g >= G) break;
                const float e = sc[g * chunk_max + j];
                acc[g].x = fmaf(e, vv[u].x, acc[g].x);
                acc[g].y = fmaf(e, vv[u].y, acc[g].y);
                acc[g].z = fmaf(e, vv[u].z, acc[g].z);
                acc[g].w = fmaf(e, vv[u].w, acc[g].w);
            }
        }
    }
    // reduce the position groups through shared memory (red1 is free again)
    float* ored = red1;
#pragma unroll
    for (int g = 0; g < 16; ++g)
        if (g < G) reinterpret_cast<float4*>(ored + (pg * G + g) * hd)[d4] = acc[g];
    __syncthreads();
    for (int idx = tid; idx < G * hd; idx += kAttnThreads) {
        const int g = idx / hd, d = idx % hd;
        float o = 0.f;
        for (int q = 0; q < npg; ++q) o += ored[(q * G + g) * hd + d];
        const int h = kvh * G + g;
        float* dst = p.part + ((size_t)h * p.nsplit + split) * (hd + 2);
        dst[d] = o;
        if (d == 0) {
            dst[hd] = nt > 0 ? mrow[g] : -INFINITY;
            dst[hd + 1] = nt > 0 ? lrow[g] : 0.f;
        }
    }
    // ---- last CTA of this kv head merges the splits
    __threadfence();
    __syncthreads();
    __shared__ unsigned int last;
    if (tid == 0) last = (atomicAdd(&p.counter[kvh], 1u) == (unsigned)(p.nsplit - 1)) ? 1u : 0u;
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int idx = tid; idx < G * hd; idx += kAttnThreads) {
        const int g = idx / hd, dd = idx % hd;
        const int h = kvh * G + g;
        const float* base = p.part + (size_t)h * p.nsplit * (hd + 2);
        float M = -INFINITY;
        for (int s = 0; s < p.nsplit; ++s) M = fmaxf(M, base[s * (hd + 2) + hd]);
        float L = 0.f, O = 0.f;
        for (int s = 0; s < p.nsplit; ++s) {
            const float ms = base[s * (hd + 2) + hd];
            if (ms == -INFINITY) continue;
            const float w = expf(ms - M);
            L += base[s * (hd + 2) + hd + 1] * w;
            O += base[s * (hd + 2) + dd] * w;
        }
        p.out[(size_t)h * hd + dd] = O / L;
    }
    if (tid == 0) p.counter[kvh] = 0u;
    if (p.xq_out) {
        // quantise this kv head's G*hd outputs (whole 32-value groups) for the O projection
        __threadfence();
        __syncthreads();
        const int g0 = kvh * G * hd / 32, ng = G * hd / 32;  // 32-value warp groups
        for (int k = warp; k < ng; k += kAttnThreads / 32)
            xq_quantize_group(p.xq_out, p.out, nullptr, p.n_heads * hd, g0 + k, p.q8 != 0);
    }
}

__global__ void finalize_kernel(const unsigned long long* key, int* token, int* pos, int* hist) {
    pdl_launch_dependents();
    pdl_wait();
    const unsigned long long k = *key;
    const int id = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
    const int ps = *pos;
    *token = id;
    if (hist) hist[ps] = id;
    *pos = ps + 1;
}

}  // namespace

cudaError_t attention_init() {
    return cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

int attention_smem_bytes(const AttnParams& p) {
    const int G = p.n_heads / p.n_kv_heads;
    const int chunk_max = attn_chunk_max(p.n_ctx, p.nsplit);
    return (G * p.head_dim + 2 * p.head_dim + G * chunk_max + attn_red1_floats(G, p.head_dim) + 64) *
           (int)sizeof(float);
}

cudaError_t attention_launch(const AttnParams& p, cudaStream_t st, bool pdl) {
    const int G = p.n_heads / p.n_kv_heads;
    if (G > 16 || p.head_dim > 128 || (p.head_dim != 64 && p.head_dim != 128) || p.n_heads % p.n_kv_heads) {
        set_last_error("attention: need head_dim in {64,128} and n_heads/n_kv_heads <= 16");
        return cudaErrorInvalidValue;
    }
    const int smem = attention_smem_bytes(p);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.n_kv_heads, p.nsplit);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, attention_kernel, p);
}

cudaError_t finalize_launch(const unsigned long long* key, int* token, int* pos, int* hist, cudaStream_t st,
                            bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, finalize_kernel, key, token, pos, hist);
}

}  // namespace af

// ---------------------------------------------------------------------------
// Attention entry point that allocates nothing.
//
// Some callers cannot call cudaMalloc on the serving path: a host that owns a
// fixed device arena and forbids further allocation once it is serving, or a
// plugin that is only handed input/output pointers and must not change the
// process's memory footprint.  For them the split-K partials and the per-kv-head
// counters live in this file-scope device array instead of caller-provided
// scratch.  Every GPU that loads the library holds the array until exit.
namespace af {
namespace {

constexpr int kNoAllocPartFloats = 256 * 1024;  // 1 MiB of partials
constexpr int kNoAllocCounters = 256;

struct NoAllocScratch {
    float part[kNoAllocPartFloats];
    unsigned int counter[kNoAllocCounters];
};

static __device__ __align__(256) NoAllocScratch g_attn_scratch;

// Device addresses of g_attn_scratch, looked up once per device and context:
// a reset primary context reloads the module, so the address is looked up
// again when the current context is not the one it was taken in.
constexpr int kMaxDevices = 64;
struct ScratchAddr {
    CUcontext ctx = nullptr;
    NoAllocScratch* ptr = nullptr;
};
ScratchAddr g_scratch_addr[kMaxDevices];
std::mutex g_scratch_mu;

cudaError_t scratch_for_current_device(NoAllocScratch** out) {
    int dev = 0;
    AF_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    AF_CUDA_TRY(cudaSetDevice(dev));  // makes the device's primary context current
    // the driver's cuCtxGetCurrent through the runtime (the library does not link libcuda)
    using CtxGetCurrent = CUresult (*)(CUcontext*);
    static CtxGetCurrent get_ctx = nullptr;
    if (!get_ctx) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn) {
            set_last_error("af_attention_decode_f32_noalloc: cuCtxGetCurrent unavailable");
            return cudaErrorInitializationError;
        }
        get_ctx = reinterpret_cast<CtxGetCurrent>(fn);
    }
    CUcontext ctx = nullptr;
    if (get_ctx(&ctx) != CUDA_SUCCESS || !ctx) {
        set_last_error("af_attention_decode_f32_noalloc: no current CUDA context");
        return cudaErrorInitializationError;
    }
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    ScratchAddr& a = g_scratch_addr[dev];
    if (!a.ptr || a.ctx != ctx) {
        void* p = nullptr;
        const cudaError_t r = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (r != cudaSuccess) {
            set_last_error(std::string("af_attention_decode_f32_noalloc: cudaGetSymbolAddress: ") +
                           cudaGetErrorString(r));
            return r;
        }
        a.ptr = static_cast<NoAllocScratch*>(p);
        a.ctx = ctx;
    }
    *out = a.ptr;
    return cudaSuccess;
}

}  // namespace
}  // namespace af

extern "C" cudaError_t af_attention_decode_f32_noalloc(
    float* d_out, const float* d_q, const float* d_k, const float* d_v, float* d_kcache, float* d_vcache,
    const float* d_cos, const float* d_sin, const float* d_q_norm, const float* d_k_norm, const int* d_pos,
    int n_heads, int n_kv_heads, int head_dim, int n_ctx, int qk_norm_order, float eps, int nsplit,
    cudaStream_t stream) {
    using namespace af;
    if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || nsplit <= 0 || n_ctx <= 0 || head_dim <= 0) {
        set_last_error("af_attention_decode_f32_noalloc: bad shape");
        return cudaErrorInvalidValue;
    }
    if ((long long)n_heads * nsplit * (head_dim + 2) > kNoAllocPartFloats || n_kv_heads > kNoAllocCounters) {
        set_last_error("af_attention_decode_f32_noalloc: n_heads*nsplit*(head_dim+2) must be <= 262144 and "
                       "n_kv_heads <= 256 (fixed scratch of this entry point)");
        return cudaErrorInvalidValue;
    }
    NoAllocScratch* s = nullptr;
    AF_CUDA_TRY(scratch_for_current_device(&s));
    // The counters must start at zero; a call that ended early could have left
    // them dirty, so clear them on the stream (no allocation involved).
    AF_CUDA_TRY(cudaMemsetAsync(s->counter, 0, sizeof(unsigned int) * n_kv_heads, stream));
    AttnParams p = {};
    p.q = d_q; p.k = d_k; p.v = d_v; p.kc = d_kcache; p.vc = d_vcache; p.out = d_out;
    p.cos_t = d_cos; p.sin_t = d_sin; p.q_norm = d_q_norm; p.k_norm = d_k_norm;
    p.part = s->part; p.counter = s->counter; p.pos = d_pos;
    p.n_heads = n_heads; p.n_kv_heads = n_kv_heads; p.head_dim = head_dim; p.n_ctx = n_ctx;
    p.nsplit = nsplit; p.qk_norm_order = qk_norm_order; p.eps = eps;
    p.scale = 1.f / sqrtf((float)head_dim);
    AF_CUDA_TRY(attention_init());
    return attention_launch(p, stream, false);
}

