// af_engine.cu — GPU-resident LLaMA-family decode engine behind the C ABI.
//
// Replaces llama_cuda_generate (include/axonforge/models/llama_cuda.hpp:25-28,
// whose reference body falls back to the CPU, src/models/llama_cuda_model.cpp:7-17)
// with the forward of llama_forward_token (src/models/llama_model.cpp:1207-1333)
// on the device:
//
//   embed ─┬─ per layer: [RMSNorm→QKV GEMV(+bias)] → [RoPE+KV store+attention]
//          │             → [O GEMV + residual] → [RMSNorm→gate/up GEMV→SwiGLU]
//          │             → [down GEMV + residual]
//          └─ [final RMSNorm→LM head GEMV→argmax] → [id → next step's input]
//
// 5·L + 3 kernels per token, launched with programmatic dependent launch and
// captured once into a CUDA graph; the token id and position live in device
// memory, so consecutive steps chain on the device without a host round trip.
//
// Tensor parallelism (tp_size > 1, one process per GPU): attention heads and
// FFN rows are column-parallel, attn_output / ffn_down are row-parallel over
// whole 256-value super-blocks, the LM head is split over the vocabulary.
// attn_output and ffn_down write partial sums that one NCCL all-reduce (fp32
// sum) combines; the next GEMV's prologue adds them to the replicated residual.
// The argmax is one all-reduce (max) of a packed (value, ~index) key.
#include <nccl.h>

#include <cmath>
#include <cstdlib>
#include <thread>
#include <chrono>
#include <random>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "af_gemv.cuh"
#include "af_gguf.h"
#include "af_ops.cuh"
#include "af_step.cuh"

using namespace af;

namespace {

struct DevMat {
    uint8_t* w = nullptr;
    int type = -1;
    int rows = 0, cols = 0;  // local shard shape
    int stride = 0;
    bool present() const { return w != nullptr; }
};

struct LayerW {
    float *attn_norm = nullptr, *ffn_norm = nullptr, *bq = nullptr, *bk = nullptr, *bv = nullptr;
    float *q_norm = nullptr, *k_norm = nullptr;
    DevMat wq, wk, wv, wo, wg, wu, wd;
};

// [lo, hi) of `n` super-blocks for rank r of t, remainder to the low ranks
// (ffn_down K = 11008 = 43 blocks splits 22/21, 11/11/11/10, 6,6,6,5,5,5,5,5).
void block_split(int n, int r, int t, int& lo, int& hi) {
    const int base = n / t, rem = n % t;
    lo = r * base + (r < rem ? r : rem);
    hi = lo + base + (r < rem ? 1 : 0);
}

}  // namespace

struct af_engine {
    af_model_config cfg{};
    int device = 0, rank = 0, tp = 1;
    ncclComm_t comm = nullptr;
    cudaStream_t stream = nullptr;
    int sms = 148;
    int gemv_ctas = 148;
    bool pdl = true;  // programmatic dependent launch between the step's kernels (AF_PDL=0 disables)

    // local shard geometry
    int hd = 0, Hl = 0, KVl = 0, F0 = 0, F1 = 0, Fl = 0, V0 = 0, V1 = 0, Vl = 0, Vmax = 0;

    // weights
    DevMat tok_embd, output, tok_head;
    float* out_norm = nullptr;
    std::vector<LayerW> layers;
    std::vector<void*> allocs;
    size_t weight_bytes = 0;

    // activations / state
    float* x[2] = {nullptr, nullptr};
    float *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr, *h = nullptr, *ypart = nullptr;
    float *logits = nullptr, *logits_all = nullptr;
    float *kcache = nullptr, *vcache = nullptr, *cos_t = nullptr, *sin_t = nullptr, *apart = nullptr;
    unsigned int* acount = nullptr;
    uint8_t *xq_a = nullptr, *xq_o = nullptr, *xq_gu = nullptr, *xq_d = nullptr;  // quantised GEMV inputs
    unsigned long long* key = nullptr;
    int* tokpos = nullptr;  // [0] token, [1] pos
    int* hist = nullptr;
    int* d_window = nullptr;       // repetition-penalty window of the sampler [n_ctx + 1]
    int* d_sampled = nullptr;      // sampled id
    float* logits_full = nullptr;  // tensor parallel: the gathered vocabulary [vocab]
    int* h_tokpos = nullptr;  // pinned host mirror
    int* h_pin = nullptr;     // pinned prompt staging of af_engine_prefill (grown on demand)
    size_t h_pin_n = 0;
    void* pf_ws = nullptr;    // device rows of af_engine_prefill_batched (grown on demand)
    size_t pf_ws_bytes = 0;
    int nsplit = 1;

    // persistent step kernel (single GPU): phase table in device memory
    bool use_step = false;
    StepPhase* d_phases = nullptr;
    uint8_t* xchg = nullptr;                 // this rank's exchange area (tensor parallel)
    std::vector<void*> peer_maps;            // IPC mappings of the other ranks' areas
    unsigned int* step_bar = nullptr;
    unsigned long long* sepoch = nullptr;  // steps the step kernel has run (tags its inter-CTA words)
    unsigned long long* tpart = nullptr;   // tagged attention split partials of the step kernel
    StepParams step{};

    cudaGraph_t graph = nullptr;
    cudaGraphExec_t gexec = nullptr;
    bool finalized = false;
    int q8 = 0;  // activations as Q8_0 blocks (af_engine_set_q8_activations)
    int kernels_per_step = 0;

    void* dalloc(size_t bytes) {
        void* p = nullptr;
        if (cudaMalloc(&p, bytes ? bytes : 16) != cudaSuccess) throw std::runtime_error("cudaMalloc failed");
        allocs.push_back(p);
        return p;
    }
};

namespace {

cudaError_t fail(const std::string& msg, cudaError_t code = cudaErrorInvalidValue) {
    set_last_error(msg);
    return code;
}

#define ENG_TRY(x)                                                                          \
    do {                                                                                    \
        cudaError_t e_ = (x);                                                               \
        if (e_ != cudaSuccess) return fail(std::string(#x) + ": " + cudaGetErrorString(e_), e_); \
    } while (0)
// A call of this file's own functions, which set their message themselves.
#define ENG_CALL(x)                       \
    do {                                  \
        cudaError_t e_ = (x);             \
        if (e_ != cudaSuccess) return e_; \
    } while (0)

// Host-side limit of every wait on NCCL (AF_NCCL_INIT_TIMEOUT_S, default 300 s).
inline double nccl_limit_s() {
    const char* tv = std::getenv("AF_NCCL_INIT_TIMEOUT_S");
    return tv ? std::atof(tv) : 300.0;
}

// The communicator is non-blocking (see af_engine_create): a call may return
// ncclInProgress until NCCL has enqueued it (the first collective also sets up
// its connections, which can take a while); wait for that, bounded in time.
inline ncclResult_t nccl_settle(ncclComm_t comm, ncclResult_t r) {
    const auto t0 = std::chrono::steady_clock::now();
    while (r == ncclInProgress && comm) {
        if (ncclCommGetAsyncError(comm, &r) != ncclSuccess) return ncclSystemError;
        if (r != ncclInProgress) break;
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > nccl_limit_s())
            return ncclInProgress;
        std::this_thread::yield();
    }
    return r;
}
#define NCCL_TRY(x)                                                                         \
    do {                                                                                    \
        ncclResult_t r_ = nccl_settle(e->comm, (x));                                        \
        if (r_ != ncclSuccess) return fail(std::string(#x) + ": " + ncclGetErrorString(r_), cudaErrorUnknown); \
    } while (0)

// Upload rows [r0, r1) x blocks [b0, b1) of a GGUF matrix (rows of `cols`
// values) from host memory into a new device buffer in the device layout.
cudaError_t upload_matrix(af_engine* e, DevMat& m, int type, const uint8_t* h, int cols, int r0, int r1, int b0,
                          int b1) {
    const int bb = type == AF_GGML_Q6_K ? 210 : (type == AF_GGML_Q4_K ? 144 : 0);
    if (!bb) return fail("unsupported matrix type " + std::to_string(type) + " (Q4_K / Q6_K only)");
    const size_t src_rb = (size_t)(cols / 256) * bb;
    const int lcols = (b1 - b0) * 256, rows = r1 - r0;
    const size_t gg_rb = (size_t)(b1 - b0) * bb;
    m.type = type;
    m.rows = rows;
    m.cols = lcols;
    m.stride = dev_row_stride(type, lcols);
    m.w = static_cast<uint8_t*>(e->dalloc(packed_bytes(type, rows, lcols) + 64));
    uint8_t* stage = nullptr;
    ENG_TRY(cudaMalloc(&stage, (size_t)rows * gg_rb + 16));
    const uint8_t* src = h + (size_t)r0 * src_rb + (size_t)b0 * bb;
    // Copy and pack on the engine's (non-blocking) stream and wait: a
    // synchronous cudaMemcpy from pageable memory may return before its DMA
    // lands, and a non-blocking stream is not ordered after it.
    ENG_TRY(cudaMemcpy2DAsync(stage, gg_rb, src, src_rb, gg_rb, rows, cudaMemcpyHostToDevice, e->stream));
    ENG_TRY(weight_pack(m.w, stage, type, rows, lcols, false, e->stream));
    ENG_TRY(cudaStreamSynchronize(e->stream));
    cudaFree(stage);
    e->weight_bytes += (size_t)rows * m.stride;
    return cudaSuccess;
}

cudaError_t upload_f32(af_engine* e, float*& dst, const void* h, size_t n, size_t off = 0) {
    dst = static_cast<float*>(e->dalloc(n * 4));
    ENG_TRY(cudaMemcpyAsync(dst, static_cast<const float*>(h) + off, n * 4, cudaMemcpyHostToDevice, e->stream));
    ENG_TRY(cudaStreamSynchronize(e->stream));
    return cudaSuccess;
}

GemvParams base_params(const af_engine* e, int K) {
    GemvParams p = {};
    p.K = K;
    p.eps = e->cfg.eps;
    p.q8 = e->q8;
    return p;
}

GemvSeg seg_of(const DevMat& m, float* y, const float* bias) {
    GemvSeg s = {};
    s.w = m.w;
    s.y = y;
    s.bias = bias;
    s.type = m.type;
    s.rows = m.rows;
    s.row_stride = m.stride;
    return s;
}

// Event-bracketed eager launches for af_engine_profile: one event after every
// launch; kind k of launch i is kinds[i], its algorithmic bytes bytes[i].
struct Prof {
    std::vector<cudaEvent_t> ev;
    std::vector<int> kinds;
    std::vector<double> bytes;
    int pos = 0;
    cudaError_t mark(cudaStream_t st, int kind, double b) {
        cudaEvent_t x;
        AF_CUDA_TRY(cudaEventCreate(&x));
        AF_CUDA_TRY(cudaEventRecord(x, st));
        ev.push_back(x);
        kinds.push_back(kind);
        bytes.push_back(b);
        return cudaSuccess;
    }
};

double gemv_bytes(const GemvParams& p) {
    double b = (double)p.K * 4 * (p.x_add ? 2 : 1);
    for (int s = 0; s < p.nseg; ++s) b += (double)p.seg[s].rows * (p.seg[s].row_stride + 4);
    return b;
}

// Enqueue one decode step (token/pos read from device memory) on e->stream.
// With `prof`, every launch is followed by a timing event (no graph capture).
cudaError_t enqueue_step(af_engine* e, Prof* prof = nullptr) {
#define AF_MARK(kind, b) \
    if (prof) AF_CUDA_TRY(prof->mark(e->stream, kind, b))
    const auto& c = e->cfg;
    const int E = c.n_embd;
    const bool tp = e->tp > 1;
    int nk = 0;
    int cur = 0;  // residual buffer holding the current stream (TP ping-pong)
    // Single-GPU steps hand quantised inputs (XQ) from kernel to kernel; tensor
    // parallel ranks quantise inside each GEMV after the all-reduce.
    const bool xq = !tp;
    if (e->use_step && !prof) {
        ENG_TRY(step_launch(e->step, e->stream));
        e->kernels_per_step = 1;
        return cudaSuccess;
    }
    ENG_TRY(embed_launch(e->x[0], e->tok_embd.w, e->tok_embd.type, E, e->tok_embd.stride, &e->tokpos[0], e->key,
                         xq ? e->xq_a : nullptr, e->layers[0].attn_norm, e->stream, e->pdl, e->q8 != 0));
    ++nk;
    AF_MARK(AF_PROF_EMBED, (double)e->tok_embd.stride + E * 4.0);
    bool pending = false;  // TP: ypart holds an un-added partial sum
    for (int l = 0; l < c.n_layer; ++l) {
        const LayerW& L = e->layers[l];
        // --- RMSNorm + QKV
        {
            GemvParams p = base_params(e, E);
            p.seg[0] = seg_of(L.wq, e->q, L.bq);
            p.seg[1] = seg_of(L.wk, e->k, L.bk);
            p.seg[2] = seg_of(L.wv, e->v, L.bv);
            p.nseg = 3;
            p.x = e->x[cur];
            if (pending) {
                p.x_add = e->ypart;
                p.x_store = e->x[cur ^ 1];
                cur ^= 1;
            }
            p.norm_w = L.attn_norm;
            if (xq) {
                p.xq = e->xq_a;
                p.xq_norm = 1;
            }
            p.epi = EPI_STORE;
            gemv_configure(p, e->gemv_ctas);
            ENG_TRY(gemv_launch(p, e->stream, e->pdl));
            ++nk;
            AF_MARK(AF_PROF_QKV, gemv_bytes(p));
        }
        // --- attention (RoPE, KV store, GQA softmax)
        {
            AttnParams a = {};
            a.q = e->q;
            a.k = e->k;
            a.v = e->v;
            const size_t lsz = (size_t)c.n_ctx * e->KVl * e->hd;
            a.kc = e->kcache + (size_t)l * lsz;
            a.vc = e->vcache + (size_t)l * lsz;
            a.out = e->attn;
            a.cos_t = e->cos_t;
            a.sin_t = e->sin_t;
            a.q_norm = L.q_norm;
            a.k_norm = L.k_norm;
            a.part = e->apart;
            a.counter = e->acount;
            a.pos = &e->tokpos[1];
            a.n_heads = e->Hl;
            a.n_kv_heads = e->KVl;
            a.head_dim = e->hd;
            a.n_ctx = c.n_ctx;
            a.nsplit = e->nsplit;
            a.qk_norm_order = c.qk_norm_order;
            a.eps = c.eps;
            a.scale = 1.f / std::sqrt((float)e->hd);
            a.xq_out = xq ? e->xq_o : nullptr;
            a.q8 = e->q8;
            ENG_TRY(attention_launch(a, e->stream, e->pdl));
            ++nk;
            if (prof) {
                const double kvb = 2.0 * (prof->pos + 1) * e->KVl * e->hd * 4.0;
                AF_MARK(AF_PROF_ATTN, kvb + 2.0 * e->Hl * e->hd * 4.0);
            }
        }
        // --- O projection (+ residual)
        {
            GemvParams p = base_params(e, e->Hl * e->hd);
            p.seg[0] = seg_of(L.wo, e->ypart, nullptr);
            p.nseg = 1;
            p.x = e->attn;
            if (tp) {
                p.epi = EPI_STORE;
            } else {
                p.epi = EPI_RESID;
                p.resid = e->x[cur];
                p.xq = e->xq_o;
                p.q_out = e->xq_gu;
                p.q_norm_w = L.ffn_norm;
            }
            gemv_configure(p, e->gemv_ctas);
            ENG_TRY(gemv_launch(p, e->stream, e->pdl));
            ++nk;
            AF_MARK(AF_PROF_O, gemv_bytes(p));
            if (tp) {
                NCCL_TRY(ncclAllReduce(e->ypart, e->ypart, E, ncclFloat32, ncclSum, e->comm, e->stream));
                pending = true;
                AF_MARK(AF_PROF_COMM, E * 4.0);
            }
        }
        // --- RMSNorm + gate/up + SwiGLU
        {
            GemvParams p = base_params(e, E);
            p.seg[0] = seg_of(L.wg, e->h, nullptr);
            p.seg[1] = seg_of(L.wu, nullptr, nullptr);
            p.nseg = 2;
            p.x = e->x[cur];
            if (pending) {
                p.x_add = e->ypart;
                p.x_store = e->x[cur ^ 1];
                cur ^= 1;
                pending = false;
            }
            p.norm_w = L.ffn_norm;
            p.epi = EPI_SWIGLU;
            if (xq) {
                p.xq = e->xq_gu;
                p.xq_norm = 1;
                p.q_out = e->xq_d;
            }
            gemv_configure(p, e->gemv_ctas);
            ENG_TRY(gemv_launch(p, e->stream, e->pdl));
            ++nk;
            AF_MARK(AF_PROF_GATEUP, gemv_bytes(p) - 4.0 * p.seg[1].rows);
        }
        // --- down projection (+ residual)
        {
            GemvParams p = base_params(e, e->Fl);
            p.seg[0] = seg_of(L.wd, e->ypart, nullptr);
            p.nseg = 1;
            p.x = e->h;
            if (tp) {
                p.epi = EPI_STORE;
            } else {
                p.epi = EPI_RESID;
                p.resid = e->x[cur];
                p.xq = e->xq_d;
                p.q_out = e->xq_a;
                p.q_norm_w = l + 1 < c.n_layer ? e->layers[l + 1].attn_norm : e->out_norm;
            }
            gemv_configure(p, e->gemv_ctas);
            ENG_TRY(gemv_launch(p, e->stream, e->pdl));
            ++nk;
            AF_MARK(AF_PROF_DOWN, gemv_bytes(p));
            if (tp) {
                NCCL_TRY(ncclAllReduce(e->ypart, e->ypart, E, ncclFloat32, ncclSum, e->comm, e->stream));
                pending = true;
                AF_MARK(AF_PROF_COMM, E * 4.0);
            }
        }
    }
    // --- final RMSNorm + LM head + argmax
    {
        GemvParams p = base_params(e, E);
        p.seg[0] = seg_of(e->output, e->logits, nullptr);
        p.nseg = 1;
        p.x = e->x[cur];
        if (pending) {
            p.x_add = e->ypart;
            p.x_store = e->x[cur ^ 1];
            cur ^= 1;
        }
        p.norm_w = e->out_norm;
        if (xq) {
            p.xq = e->xq_a;
            p.xq_norm = 1;
        }
        p.epi = EPI_ARGMAX;
        p.argmax = e->key;
        p.argmax_base = e->V0;
        gemv_configure(p, e->gemv_ctas);
        ENG_TRY(gemv_launch(p, e->stream, e->pdl));
        ++nk;
        AF_MARK(AF_PROF_LMHEAD, gemv_bytes(p));
        if (tp) {
            NCCL_TRY(ncclAllReduce(e->key, e->key, 1, ncclUint64, ncclMax, e->comm, e->stream));
            AF_MARK(AF_PROF_COMM, 8.0);
        }
    }
    if (cur != 0) return fail("internal: residual ping-pong did not return to buffer 0");
    ENG_TRY(finalize_launch(e->key, &e->tokpos[0], &e->tokpos[1], e->hist, e->stream, e->pdl));
    ++nk;
    AF_MARK(AF_PROF_FINAL, 16.0);
    if (!prof) e->kernels_per_step = nk;
    return cudaSuccess;
#undef AF_MARK
}

// Tensor-parallel exchange areas: each rank allocates and zeroes its own,
// the CUDA IPC handles travel over the NCCL communicator (all-gather), and
// every rank maps the others' areas, so the step kernel reaches the peers'
// receive slots (tagged stores), argmax slots and counters over NVLink.
cudaError_t setup_exchange(af_engine* e) {
    const int E = e->cfg.n_embd;
    const size_t bytes = step_xchg_bytes(E);
    e->xchg = static_cast<uint8_t*>(e->dalloc(bytes));
    ENG_TRY(cudaMemset(e->xchg, 0, bytes));
    unsigned long long* epoch = static_cast<unsigned long long*>(e->dalloc(64));
    ENG_TRY(cudaMemset(epoch, 0, 64));
    ENG_TRY(cudaDeviceSynchronize());
    StepParams& sp = e->step;
    sp.epoch = epoch;
    cudaIpcMemHandle_t mine;
    ENG_TRY(cudaIpcGetMemHandle(&mine, e->xchg));
    const size_t hs = sizeof(cudaIpcMemHandle_t);
    uint8_t* d_h = nullptr;
    ENG_TRY(cudaMalloc(&d_h, hs * (e->tp + 1)));
    ENG_TRY(cudaMemcpy(d_h + hs * e->tp, &mine, hs, cudaMemcpyHostToDevice));
    NCCL_TRY(ncclAllGather(d_h + hs * e->tp, d_h, hs, ncclUint8, e->comm, e->stream));
    std::vector<cudaIpcMemHandle_t> all(e->tp);
    ENG_TRY(cudaStreamSynchronize(e->stream));
    ENG_TRY(cudaMemcpy(all.data(), d_h, hs * e->tp, cudaMemcpyDeviceToHost));
    cudaFree(d_h);
    for (int r = 0; r < e->tp; ++r) {
        uint8_t* base = e->xchg;
        if (r != e->rank) {
            void* p = nullptr;
            ENG_TRY(cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess));
            e->peer_maps.push_back(p);
            base = static_cast<uint8_t*>(p);
        }
        sp.xbar[r] = reinterpret_cast<unsigned long long*>(base);
        sp.xkey[r] = reinterpret_cast<unsigned long long*>(base + 128);
        sp.xrecv[r] = reinterpret_cast<unsigned long long*>(base + 256);
    }
    // every rank has mapped every area before any step runs
    int* dd = static_cast<int*>(e->dalloc(16));
    ENG_TRY(cudaMemset(dd, 0, 16));
    NCCL_TRY(ncclAllReduce(dd, dd, 1, ncclInt32, ncclSum, e->comm, e->stream));
    ENG_TRY(cudaStreamSynchronize(e->stream));
    return cudaSuccess;
}

// Phase table of the persistent step kernel (single GPU, quantised inputs
// handed from phase to phase), mirroring enqueue_step's kernel sequence.
cudaError_t build_step(af_engine* e) {
    const auto& c = e->cfg;
    const int E = c.n_embd;
    ENG_TRY(step_init());
    const bool tp = e->tp > 1;
    auto none = [](StepPhase& p) { p.x.k_out = p.x.k_in = -1; };
    // exchange k: input of the next normalised GEMV (norm weights norm_w);
    // the residual ping-pongs x[k % 2] -> x[(k + 1) % 2]
    std::vector<StepPhase> ph;
    // AF_TP_XRED=0: the consuming GEMV reads every rank's partials itself
    // (no separate phase); default: a reduction phase before it (StepPhase)
    const bool xred = [] {
        const char* v = std::getenv("AF_TP_XRED");
        return !(v && v[0] == '0');
    }();
    auto xin = [&](StepPhase& p, int k, const float* norm_w) {
        XchgParams x = {};
        x.k_out = -1;
        x.k_in = k;
        x.resid_in = e->x[k & 1];
        x.resid_out = e->x[(k + 1) & 1];
        x.norm_w = norm_w;
        x.n = E;
        if (xred) {
            StepPhase r = {};
            r.kind = PH_XRED;
            r.x = x;
            r.x.xq = const_cast<uint8_t*>(p.g.xq);  // the consuming GEMV copies the quantised sum
            ph.push_back(r);
        } else {
            x.k_out = p.x.k_out;
            p.x = x;
        }
    };
    e->sepoch = static_cast<unsigned long long*>(e->dalloc(sizeof(unsigned long long)));
    ENG_TRY(cudaMemset(e->sepoch, 0, sizeof(unsigned long long)));
    {
        const size_t n = (size_t)e->Hl * std::max(1, std::min(std::min(e->nsplit, e->sms / e->KVl), kStepAttnMaxSplit)) *
                         (e->hd + 2);
        e->tpart = static_cast<unsigned long long*>(e->dalloc(n * sizeof(unsigned long long)));
        ENG_TRY(cudaMemset(e->tpart, 0, n * sizeof(unsigned long long)));
    }
    StepPhase embed = {};
    embed.kind = PH_EMBED;
    none(embed);
    ph.push_back(embed);
    for (int l = 0; l < c.n_layer; ++l) {
        const LayerW& L = e->layers[l];
        StepPhase q = {};
        q.kind = PH_GEMV;
        none(q);
        q.g = base_params(e, E);
        q.g.seg[0] = seg_of(L.wq, e->q, L.bq);
        q.g.seg[1] = seg_of(L.wk, e->k, L.bk);
        q.g.seg[2] = seg_of(L.wv, e->v, L.bv);
        q.g.nseg = 3;
        q.g.xq = e->xq_a;
        // layer 0 in Q8 mode: the embedding phase stores the normalised input
        q.g.xq_norm = (l == 0 && e->q8 && step_q8_exact_embed(E)) ? 0 : 1;
        q.g.epi = EPI_STORE;
        if (tp && l > 0) xin(q, 2 * l - 1, L.attn_norm);
        gemv_configure(q.g, e->sms);
        ph.push_back(q);

        StepPhase at = {};
        at.kind = PH_ATTN;
        none(at);
        AttnParams& a = at.a;
        a.q = e->q;
        a.k = e->k;
        a.v = e->v;
        const size_t lsz = (size_t)c.n_ctx * e->KVl * e->hd;
        a.kc = e->kcache + (size_t)l * lsz;
        a.vc = e->vcache + (size_t)l * lsz;
        a.out = e->attn;
        a.cos_t = e->cos_t;
        a.sin_t = e->sin_t;
        a.q_norm = L.q_norm;
        a.k_norm = L.k_norm;
        a.part = e->apart;
        a.counter = e->acount;
        a.tpart = e->tpart;
        a.pos = &e->tokpos[1];
        a.n_heads = e->Hl;
        a.n_kv_heads = e->KVl;
        a.head_dim = e->hd;
        a.n_ctx = c.n_ctx;
        a.nsplit = std::max(1, std::min(std::min(e->nsplit, e->sms / e->KVl), kStepAttnMaxSplit));
        a.qk_norm_order = c.qk_norm_order;
        a.eps = c.eps;
        a.scale = 1.f / std::sqrt((float)e->hd);
        a.xq_out = e->xq_o;
        a.q8 = e->q8;
        ph.push_back(at);

        StepPhase o = {};
        o.kind = PH_GEMV;
        none(o);
        o.g = base_params(e, e->Hl * e->hd);
        o.g.seg[0] = seg_of(L.wo, e->ypart, nullptr);
        o.g.nseg = 1;
        o.g.xq = e->xq_o;
        if (tp) {  // row-parallel: partial sums into the exchange buffer, then the all-reduce
            o.g.epi = EPI_STORE;
            o.x.k_out = 2 * l;
            o.x.n = E;
        } else {
            o.g.epi = EPI_RESID;
            o.g.resid = e->x[0];
            o.g.q_out = e->xq_gu;
            o.g.q_norm_w = L.ffn_norm;
        }
        gemv_configure(o.g, e->sms);
        ph.push_back(o);

        StepPhase gu = {};
        gu.kind = PH_GEMV;
        none(gu);
        gu.g = base_params(e, E);
        gu.g.seg[0] = seg_of(L.wg, e->h, nullptr);
        gu.g.seg[1] = seg_of(L.wu, nullptr, nullptr);
        gu.g.nseg = 2;
        gu.g.epi = EPI_SWIGLU;
        gu.g.xq = e->xq_gu;
        gu.g.xq_norm = 1;
        gu.g.q_out = e->xq_d;
        if (tp) xin(gu, 2 * l, L.ffn_norm);
        gemv_configure(gu.g, e->sms);
        ph.push_back(gu);

        StepPhase d = {};
        d.kind = PH_GEMV;
        none(d);
        d.g = base_params(e, e->Fl);
        d.g.seg[0] = seg_of(L.wd, e->ypart, nullptr);
        d.g.nseg = 1;
        d.g.xq = e->xq_d;
        const float* next_norm = l + 1 < c.n_layer ? e->layers[l + 1].attn_norm : e->out_norm;
        if (tp) {
            d.g.epi = EPI_STORE;
            d.x.k_out = 2 * l + 1;
            d.x.n = E;
        } else {
            d.g.epi = EPI_RESID;
            d.g.resid = e->x[0];
            d.g.q_out = e->xq_a;
            d.g.q_norm_w = next_norm;
        }
        gemv_configure(d.g, e->sms);
        ph.push_back(d);
    }
    StepPhase lm = {};
    lm.kind = PH_GEMV;
    none(lm);
    lm.g = base_params(e, E);
    lm.g.seg[0] = seg_of(e->output, e->logits, nullptr);
    lm.g.nseg = 1;
    lm.g.xq = e->xq_a;
    lm.g.xq_norm = 1;
    lm.g.epi = EPI_ARGMAX;
    lm.g.argmax = e->key;
    lm.g.argmax_base = e->V0;
    if (tp) xin(lm, 2 * c.n_layer - 1, e->out_norm);
    gemv_configure(lm.g, e->sms);
    ph.push_back(lm);

    e->d_phases = static_cast<StepPhase*>(e->dalloc(ph.size() * sizeof(StepPhase)));
    ENG_TRY(cudaMemcpyAsync(e->d_phases, ph.data(), ph.size() * sizeof(StepPhase), cudaMemcpyHostToDevice,
                            e->stream));
    ENG_TRY(cudaStreamSynchronize(e->stream));
    e->step_bar = static_cast<unsigned int*>(e->dalloc(256));
    StepParams& sp = e->step;
    sp.ph = e->d_phases;
    sp.nph = (int)ph.size();
    sp.bar = e->step_bar;
    sp.tok_w = e->tok_embd.w;
    sp.tok_type = e->tok_embd.type;
    sp.tok_stride = e->tok_embd.stride;
    sp.n_embd = E;
    sp.vocab = c.vocab;
    sp.x = e->x[0];
    sp.xq = e->xq_a;
    sp.xq_norm_w = e->layers[0].attn_norm;
    sp.q8 = e->q8;
    sp.eps = c.eps;
    sp.attn_dist = std::max(1, std::min(std::min(e->nsplit, e->sms / e->KVl), kStepAttnMaxSplit)) > kStepAttnDistMerge ? 1 : 0;
    sp.key = e->key;
    sp.token = &e->tokpos[0];
    sp.pos = &e->tokpos[1];
    sp.hist = e->hist;
    // union area: the largest quantised GEMV input, the attention scratch and,
    // with Q8 activations, the staged embedding row; the rest is weight ring
    {
        int ub = std::max(kStepAttnScratch, std::max(xq_norm_bytes(E), xq_norm_bytes(e->Fl)));
        if (e->q8 && step_q8_exact_embed(E)) ub = std::max(ub, E * 4);
        ub = (ub + 127) & ~127;
        sp.union_bytes = std::min(ub, kStepUnion);
    }
    sp.ring_bytes = (kStepSmem - kStepHdr - sp.union_bytes) & ~15;
    sp.tp = e->tp;
    sp.rank = e->rank;
    sp.n_buf = tp ? 2 * c.n_layer : 0;
    sp.epoch = e->sepoch;
    if (tp) ENG_CALL(setup_exchange(e));
    return cudaSuccess;
}

cudaError_t gather_logits(af_engine* e, float* h_logits) {
    if (e->tp == 1) {
        ENG_TRY(cudaMemcpyAsync(h_logits, e->logits, (size_t)e->Vl * 4, cudaMemcpyDeviceToHost, e->stream));
        return cudaSuccess;
    }
    NCCL_TRY(ncclAllGather(e->logits, e->logits_all, e->Vmax, ncclFloat32, e->comm, e->stream));
    ENG_TRY(cudaStreamSynchronize(e->stream));
    int off = 0;
    for (int r = 0; r < e->tp; ++r) {
        int lo, hi;
        block_split(e->cfg.vocab, r, e->tp, lo, hi);
        ENG_TRY(cudaMemcpyAsync(h_logits + off, e->logits_all + (size_t)r * e->Vmax, (size_t)(hi - lo) * 4,
                                cudaMemcpyDeviceToHost, e->stream));
        off += hi - lo;
    }
    return cudaSuccess;
}

}  // namespace

extern "C" {

cudaError_t af_nccl_unique_id(void* h_id) {
    if (!h_id) return fail("af_nccl_unique_id: null");
    ncclUniqueId id;
    const ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return fail(std::string("ncclGetUniqueId: ") + ncclGetErrorString(r), cudaErrorUnknown);
    std::memcpy(h_id, &id, sizeof(id));
    return cudaSuccess;
}

cudaError_t af_engine_create(const af_model_config* cfg, int device, int tp_rank, int tp_size, const void* nccl_id,
                             af_engine** out) {
    if (!cfg || !out) return fail("af_engine_create: null argument");
    *out = nullptr;
    const auto& c = *cfg;
    if (c.n_embd % 256 || c.ffn % 256 || c.n_head <= 0 || c.n_embd % c.n_head || c.n_kv_head <= 0 ||
        c.n_head % c.n_kv_head || c.n_layer <= 0 || c.vocab <= 0 || c.n_ctx <= 0)
        return fail("af_engine_create: unsupported model shape (n_embd, ffn multiples of 256)");
    if (c.n_embd > kGemvMaxK || ((c.ffn / 256 + tp_size - 1) / tp_size) * 256 > kGemvMaxK)
        return fail("af_engine_create: n_embd and the per-rank ffn must be <= 12288");
    if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size) return fail("af_engine_create: bad tp rank/size");
    if (tp_size > 1 && (c.n_kv_head % tp_size || ((c.n_embd / tp_size) % 256)))
        return fail("af_engine_create: tensor parallel needs n_kv_head and n_embd/256 divisible by tp_size");
    std::unique_ptr<af_engine> e(new af_engine());
    e->cfg = c;
    e->device = device;
    e->rank = tp_rank;
    e->tp = tp_size;
    ENG_TRY(cudaSetDevice(device));
    ENG_TRY(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
    e->sms = num_sms();
    e->gemv_ctas = gemv_grid();
    if (const char* v = std::getenv("AF_PDL")) e->pdl = std::atoi(v) != 0;
    e->hd = c.n_embd / c.n_head;
    e->Hl = c.n_head / tp_size;
    e->KVl = c.n_kv_head / tp_size;
    int f0, f1;
    block_split(c.ffn / 256, tp_rank, tp_size, f0, f1);
    e->F0 = f0 * 256;
    e->F1 = f1 * 256;
    e->Fl = e->F1 - e->F0;
    block_split(c.vocab, tp_rank, tp_size, e->V0, e->V1);
    e->Vl = e->V1 - e->V0;
    e->Vmax = (c.vocab + tp_size - 1) / tp_size;
    e->layers.resize(c.n_layer);
    if (tp_size > 1) {
        if (!nccl_id) return fail("af_engine_create: tp_size > 1 needs an ncclUniqueId");
        ncclUniqueId id;
        std::memcpy(&id, nccl_id, sizeof(id));
        // non-blocking init with a host-side limit: a rank that never joins
        // ends this call with an error instead of a hang (AF_NCCL_INIT_TIMEOUT_S,
        // default 300 s), and the half-made communicator is aborted
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;
        ncclResult_t r = ncclCommInitRankConfig(&e->comm, tp_size, id, tp_rank, &cfg);
        const double limit = nccl_limit_s();
        const auto t0 = std::chrono::steady_clock::now();
        while (r == ncclInProgress || (r == ncclSuccess && e->comm)) {
            ncclResult_t st = ncclInProgress;
            if (ncclCommGetAsyncError(e->comm, &st) != ncclSuccess) st = ncclSystemError;
            if (st != ncclInProgress) {
                r = st;
                break;
            }
            if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > limit) {
                ncclCommAbort(e->comm);
                e->comm = nullptr;
                return fail("af_engine_create: NCCL init did not complete within AF_NCCL_INIT_TIMEOUT_S (a rank "
                            "did not join)", cudaErrorTimeout);
            }
            std::this_thread::sleep_for(std::chrono::milliseconds(1));
        }
        if (r != ncclSuccess) {
            if (e->comm) ncclCommAbort(e->comm);
            e->comm = nullptr;
            return fail(std::string("af_engine_create: ncclCommInitRankConfig: ") + ncclGetErrorString(r),
                        cudaErrorUnknown);
        }
    }
    *out = e.release();
    return cudaSuccess;
}

cudaError_t af_engine_destroy(af_engine* e) {
    if (!e) return cudaSuccess;
    cudaSetDevice(e->device);
    if (e->gexec) cudaGraphExecDestroy(e->gexec);
    if (e->graph) cudaGraphDestroy(e->graph);
    for (void* p : e->peer_maps) cudaIpcCloseMemHandle(p);
    for (void* p : e->allocs) cudaFree(p);
    if (e->h_tokpos) cudaFreeHost(e->h_tokpos);
    if (e->h_pin) cudaFreeHost(e->h_pin);
    if (e->pf_ws) cudaFree(e->pf_ws);
    if (e->comm) ncclCommDestroy(e->comm);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
    return cudaSuccess;
}

cudaError_t af_engine_load_tensor(af_engine* e, const char* name_c, int type, const int64_t* dims, int n_dims,
                                  const void* h_data, size_t nbytes) {
    if (!e || !name_c || !dims || !h_data) return fail("af_engine_load_tensor: null argument");
    if (e->finalized) return fail("af_engine_load_tensor: engine already finalized");
    ENG_TRY(cudaSetDevice(e->device));
    const std::string name(name_c);
    int64_t numel = 1;
    for (int i = 0; i < n_dims; ++i) numel *= dims[i];
    if (ggml_nbytes(type, numel) != nbytes)
        return fail("af_engine_load_tensor: " + name + ": byte size does not match its type and shape");
    const auto& c = e->cfg;
    const int cols = (int)dims[0];
    const int rows = n_dims > 1 ? (int)(numel / dims[0]) : 1;
    const uint8_t* hb = static_cast<const uint8_t*>(h_data);
    const int E = c.n_embd, hd = e->hd;
    auto need_f32 = [&](size_t n) -> bool { return type == AF_GGML_F32 && (size_t)numel == n; };
    if (name == "token_embd.weight") {
        if (cols != E || rows != c.vocab) return fail("token_embd.weight: shape mismatch");
        AF_CUDA_TRY(upload_matrix(e, e->tok_embd, type, hb, cols, 0, rows, 0, cols / 256));
        // A tied LM head needs this rank's vocabulary rows packed on their own
        // (the packed layout is tile-major); with one rank it aliases the table.
        if (e->tp > 1) return upload_matrix(e, e->tok_head, type, hb, cols, e->V0, e->V1, 0, cols / 256);
        return cudaSuccess;
    }
    if (name == "output.weight") {
        if (cols != E || rows != c.vocab) return fail("output.weight: shape mismatch");
        return upload_matrix(e, e->output, type, hb, cols, e->V0, e->V1, 0, cols / 256);
    }
    if (name == "output_norm.weight") {
        if (!need_f32(E)) return fail("output_norm.weight: need f32[n_embd]");
        return upload_f32(e, e->out_norm, h_data, E);
    }
    int l = -1;
    char field[96] = {0};
    if (std::sscanf(name_c, "blk.%d.%95s", &l, field) != 2 || l < 0 || l >= c.n_layer)
        return cudaSuccess;  // tensors outside the decode path are ignored
    LayerW& L = e->layers[l];
    const std::string f(field);
    const int q0 = e->rank * e->Hl * hd, q1 = q0 + e->Hl * hd;
    const int k0 = e->rank * e->KVl * hd, k1 = k0 + e->KVl * hd;
    if (f == "attn_norm.weight") return need_f32(E) ? upload_f32(e, L.attn_norm, h_data, E) : fail(name + ": need f32[n_embd]");
    if (f == "ffn_norm.weight") return need_f32(E) ? upload_f32(e, L.ffn_norm, h_data, E) : fail(name + ": need f32[n_embd]");
    if (f == "attn_q_norm.weight") return need_f32(hd) ? upload_f32(e, L.q_norm, h_data, hd) : fail(name + ": need f32[head_dim]");
    if (f == "attn_k_norm.weight") return need_f32(hd) ? upload_f32(e, L.k_norm, h_data, hd) : fail(name + ": need f32[head_dim]");
    if (f == "attn_q.bias") return need_f32(E) ? upload_f32(e, L.bq, h_data, q1 - q0, q0) : fail(name + ": shape");
    if (f == "attn_k.bias") return need_f32((size_t)c.n_kv_head * hd) ? upload_f32(e, L.bk, h_data, k1 - k0, k0) : fail(name + ": shape");
    if (f == "attn_v.bias") return need_f32((size_t)c.n_kv_head * hd) ? upload_f32(e, L.bv, h_data, k1 - k0, k0) : fail(name + ": shape");
    if (f == "attn_q.weight") {
        if (cols != E || rows != E) return fail(name + ": shape mismatch");
        return upload_matrix(e, L.wq, type, hb, cols, q0, q1, 0, cols / 256);
    }
    if (f == "attn_k.weight" || f == "attn_v.weight") {
        if (cols != E || rows != c.n_kv_head * hd) return fail(name + ": shape mismatch");
        return upload_matrix(e, f == "attn_k.weight" ? L.wk : L.wv, type, hb, cols, k0, k1, 0, cols / 256);
    }
    if (f == "attn_output.weight") {
        if (cols != E || rows != E) return fail(name + ": shape mismatch");
        return upload_matrix(e, L.wo, type, hb, cols, 0, rows, q0 / 256, q1 / 256);
    }
    if (f == "ffn_gate.weight" || f == "ffn_up.weight") {
        if (cols != E || rows != c.ffn) return fail(name + ": shape mismatch");
        return upload_matrix(e, f == "ffn_gate.weight" ? L.wg : L.wu, type, hb, cols, e->F0, e->F1, 0, cols / 256);
    }
    if (f == "ffn_down.weight") {
        if (cols != c.ffn || rows != E) return fail(name + ": shape mismatch");
        return upload_matrix(e, L.wd, type, hb, cols, 0, rows, e->F0 / 256, e->F1 / 256);
    }
    return cudaSuccess;
}

cudaError_t af_gguf_read_config(const char* path, int max_context_len, af_model_config* cfg_out) {
    try {
        GgufFile g;
        g.open(path);
        // Engine::from_gguf (src/engine.cpp:85-118)
        const std::string a = g.get_str("general.architecture", "unknown");
        af_model_config c = {};
        c.n_layer = (int)g.get_int(a + ".block_count", 0);
        c.n_embd = (int)g.get_int(a + ".embedding_length", 0);
        c.ffn = (int)g.get_int(a + ".feed_forward_length", 0);
        c.n_head = (int)g.get_int(a + ".attention.head_count", 0);
        c.n_kv_head = (int)g.get_int(a + ".attention.head_count_kv", c.n_head);
        const int ctx = (int)g.get_int(a + ".context_length", 4096);
        c.n_ctx = std::min(ctx, max_context_len > 0 ? max_context_len : 4096);
        c.eps = (float)g.get_float(a + ".attention.layer_norm_rms_epsilon", 1e-5);
        c.theta = (float)g.get_float(a + ".rope.freq_base", 10000.0);
        c.vocab = (int)g.array_count("tokenizer.ggml.tokens");
        if (c.vocab <= 0) c.vocab = 32000;
        if (c.eps <= 0.f) c.eps = 1e-5f;
        if (c.theta <= 0.f) c.theta = 10000.f;
        if (c.ffn <= 0) c.ffn = 4 * c.n_embd;
        c.qk_norm_order = a == "hunyuan-dense" ? 2 : (a == "qwen3" ? 1 : 0);
        c.bos_id = (int)g.get_int("tokenizer.ggml.bos_token_id", 1);
        c.eos_id = (int)g.get_int("tokenizer.ggml.eos_token_id", 2);
        if (cfg_out) *cfg_out = c;
        return cudaSuccess;
    } catch (const std::exception& ex) {
        return fail(ex.what());
    }
}

cudaError_t af_engine_load_gguf(af_engine* e, const char* path) {
    if (!e || !path) return fail("af_engine_load_gguf: null argument");
    try {
        GgufFile g;
        g.open(path);
        for (const auto& t : g.tensors()) {
            cudaError_t r = af_engine_load_tensor(e, t.name.c_str(), t.type, t.dims.data(), (int)t.dims.size(),
                                                  g.data(t), t.nbytes);
            if (r != cudaSuccess) return r;
        }
        return cudaSuccess;
    } catch (const std::exception& ex) {
        return fail(ex.what());
    }
}

cudaError_t af_engine_set_q8_activations(af_engine* e, int on) {
    if (!e) return fail("af_engine_set_q8_activations: null engine");
    if (e->finalized) return fail("af_engine_set_q8_activations: engine already finalized");
    e->q8 = on ? 1 : 0;
    return cudaSuccess;
}

cudaError_t af_engine_finalize(af_engine* e) {
    if (!e) return fail("af_engine_finalize: null engine");
    if (e->finalized) return cudaSuccess;
    ENG_TRY(cudaSetDevice(e->device));
    const auto& c = e->cfg;
    try {
        if (!e->tok_embd.present()) return fail("missing token_embd.weight");
        if (!e->out_norm) return fail("missing output_norm.weight");
        if (!e->output.present()) {
            // tied head: output falls back to token_embd (make_wt_opt, llama_model.cpp:979)
            if (e->tp > 1) {
                e->output = e->tok_head;
                e->weight_bytes -= (size_t)e->Vl * e->tok_embd.stride;  // counted below as the head
            } else {
                e->output = e->tok_embd;
            }
            e->weight_bytes += (size_t)e->Vl * e->tok_embd.stride;
        }
        // The embedding table is read one row per step: not part of the per-token stream.
        e->weight_bytes -= (size_t)c.vocab * e->tok_embd.stride;
        for (int l = 0; l < c.n_layer; ++l) {
            const LayerW& L = e->layers[l];
            if (!L.attn_norm || !L.ffn_norm || !L.wq.present() || !L.wk.present() || !L.wv.present() ||
                !L.wo.present() || !L.wg.present() || !L.wu.present() || !L.wd.present())
                return fail("missing weights for layer " + std::to_string(l));
            if (L.wg.type != L.wu.type)
                return fail("layer " + std::to_string(l) + ": ffn_gate and ffn_up must share a quantisation type");
        }
        const int E = c.n_embd, hd = e->hd;
        e->x[0] = static_cast<float*>(e->dalloc((size_t)E * 4));
        e->x[1] = static_cast<float*>(e->dalloc((size_t)E * 4));
        e->q = static_cast<float*>(e->dalloc((size_t)e->Hl * hd * 4));
        e->k = static_cast<float*>(e->dalloc((size_t)e->KVl * hd * 4));
        e->v = static_cast<float*>(e->dalloc((size_t)e->KVl * hd * 4));
        e->attn = static_cast<float*>(e->dalloc((size_t)e->Hl * hd * 4));
        e->h = static_cast<float*>(e->dalloc((size_t)e->Fl * 4));
        e->ypart = static_cast<float*>(e->dalloc((size_t)E * 4));
        e->logits = static_cast<float*>(e->dalloc((size_t)e->Vmax * 4));
        if (e->tp > 1) e->logits_all = static_cast<float*>(e->dalloc((size_t)e->Vmax * e->tp * 4));
        const size_t kvn = (size_t)c.n_layer * c.n_ctx * e->KVl * hd;
        e->kcache = static_cast<float*>(e->dalloc(kvn * 4));
        e->vcache = static_cast<float*>(e->dalloc(kvn * 4));
        ENG_TRY(cudaMemset(e->kcache, 0, kvn * 4));
        ENG_TRY(cudaMemset(e->vcache, 0, kvn * 4));
        // RoPE tables on the host with the reference's formula (RopeCache::build,
        // llama_model.cpp:1024-1043) so the device uses bit-identical cos/sin.
        const int half = hd / 2;
        std::vector<float> ct((size_t)c.n_ctx * half), st((size_t)c.n_ctx * half);
        for (int p = 0; p < c.n_ctx; ++p)
            for (int i = 0; i < half; ++i) {
                const float freq = 1.f / std::pow(c.theta, (float)(2 * i) / (float)hd);
                const float ang = (float)p * freq;
                ct[(size_t)p * half + i] = std::cos(ang);
                st[(size_t)p * half + i] = std::sin(ang);
            }
        ENG_TRY(upload_f32(e, e->cos_t, ct.data(), ct.size()));
        ENG_TRY(upload_f32(e, e->sin_t, st.data(), st.size()));
        int ns = (2 * e->sms + e->KVl - 1) / e->KVl;
        ns = std::max(1, std::min(ns, std::min(64, c.n_ctx)));
        e->nsplit = ns;
        e->apart = static_cast<float*>(e->dalloc((size_t)e->Hl * ns * (hd + 2) * 4));
        e->acount = static_cast<unsigned int*>(e->dalloc((size_t)e->KVl * 4));
        ENG_TRY(cudaMemset(e->acount, 0, (size_t)e->KVl * 4));
        e->xq_a = static_cast<uint8_t*>(e->dalloc(xq_norm_bytes(E)));
        e->xq_o = static_cast<uint8_t*>(e->dalloc(xq_norm_bytes(e->Hl * hd)));
        e->xq_gu = static_cast<uint8_t*>(e->dalloc(xq_norm_bytes(E)));
        e->xq_d = static_cast<uint8_t*>(e->dalloc(xq_norm_bytes(e->Fl)));
        ENG_TRY(cudaMemset(e->xq_a, 0, xq_norm_bytes(E)));
        ENG_TRY(cudaMemset(e->xq_o, 0, xq_norm_bytes(e->Hl * hd)));
        ENG_TRY(cudaMemset(e->xq_gu, 0, xq_norm_bytes(E)));
        ENG_TRY(cudaMemset(e->xq_d, 0, xq_norm_bytes(e->Fl)));
        e->key = static_cast<unsigned long long*>(e->dalloc(8));
        e->tokpos = static_cast<int*>(e->dalloc(8));
        e->hist = static_cast<int*>(e->dalloc((size_t)(c.n_ctx + 1) * 4));
        e->d_window = static_cast<int*>(e->dalloc((size_t)(c.n_ctx + 1) * 4));
        e->d_sampled = static_cast<int*>(e->dalloc(16));
        if (e->tp > 1) e->logits_full = static_cast<float*>(e->dalloc((size_t)c.vocab * 4));
        ENG_TRY(cudaMemset(e->tokpos, 0, 8));
        ENG_TRY(cudaMallocHost(&e->h_tokpos, 16));
        ENG_TRY(gemv_init());
        ENG_TRY(attention_init());
        const char* sv = std::getenv("AF_STEP_KERNEL");
        // tensor-parallel exchanges hold at most 8 float4 chunks per consumer thread
        e->use_step = (!sv || std::atoi(sv) != 0) && e->tp <= kStepMaxRanks && c.n_embd % 32 == 0 &&
                      (e->tp == 1 || c.n_embd <= 8192) &&
                      step_supported(e->Hl, e->KVl, e->hd, c.n_embd, e->Fl);
        if (e->use_step) ENG_CALL(build_step(e));
        ENG_TRY(cudaDeviceSynchronize());
        // Capture one step into a graph.
        ENG_TRY(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
        cudaError_t r = enqueue_step(e);
        cudaGraph_t g = nullptr;
        cudaError_t r2 = cudaStreamEndCapture(e->stream, &g);
        if (r != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            return r;
        }
        ENG_TRY(r2);
        e->graph = g;
        ENG_TRY(cudaGraphInstantiate(&e->gexec, g, 0));
        e->finalized = true;
        return cudaSuccess;
    } catch (const std::exception& ex) {
        return fail(ex.what(), cudaErrorMemoryAllocation);
    }
}

static cudaError_t check_ready(af_engine* e) {
    if (!e || !e->finalized) return fail("engine not finalized");
    ENG_TRY(cudaSetDevice(e->device));
    return cudaSuccess;
}

cudaError_t af_engine_step(af_engine* e, int32_t token, int32_t pos, float* h_logits, int32_t* h_next) {
    AF_CUDA_TRY(check_ready(e));
    if (pos < 0 || pos >= e->cfg.n_ctx) return fail("af_engine_step: position outside the context");
    if (token < 0 || token >= e->cfg.vocab) return fail("af_engine_step: token id outside the vocabulary");
    e->h_tokpos[0] = token;
    e->h_tokpos[1] = pos;
    ENG_TRY(cudaMemcpyAsync(e->tokpos, e->h_tokpos, 8, cudaMemcpyHostToDevice, e->stream));
    ENG_TRY(cudaGraphLaunch(e->gexec, e->stream));
    ENG_TRY(cudaMemcpyAsync(e->h_tokpos + 2, e->tokpos, 4, cudaMemcpyDeviceToHost, e->stream));
    if (h_logits) AF_CUDA_TRY(gather_logits(e, h_logits));
    ENG_TRY(cudaStreamSynchronize(e->stream));
    if (h_next) *h_next = e->h_tokpos[2];
    return cudaSuccess;
}

cudaError_t af_engine_prefill(af_engine* e, const int32_t* h_tokens, int n, int32_t pos0, float* h_logits,
                              int32_t* h_next) {
    AF_CUDA_TRY(check_ready(e));
    if (n <= 0 || pos0 < 0 || pos0 + n > e->cfg.n_ctx) return fail("af_engine_prefill: positions outside the context");
    for (int i = 0; i < n; ++i)
        if (h_tokens[i] < 0 || h_tokens[i] >= e->cfg.vocab) return fail("af_engine_prefill: token id outside the vocabulary");
    // Each token has its own pinned slot, so the async copies need no host sync.
    if (e->h_pin_n < (size_t)n + 1) {
        // the previous prefill's copies have completed (it synchronised)
        if (e->h_pin) cudaFreeHost(e->h_pin);
        e->h_pin = nullptr;
        e->h_pin_n = 0;
        ENG_TRY(cudaMallocHost(&e->h_pin, (size_t)(n + 1) * 4));
        e->h_pin_n = (size_t)n + 1;
    }
    int* pin = e->h_pin;
    std::memcpy(pin, h_tokens, (size_t)n * 4);
    pin[n] = pos0;
    ENG_TRY(cudaMemcpyAsync(&e->tokpos[1], &pin[n], 4, cudaMemcpyHostToDevice, e->stream));
    for (int i = 0; i < n; ++i) {
        ENG_TRY(cudaMemcpyAsync(&e->tokpos[0], &pin[i], 4, cudaMemcpyHostToDevice, e->stream));
        ENG_TRY(cudaGraphLaunch(e->gexec, e->stream));
    }
    ENG_TRY(cudaMemcpyAsync(e->h_tokpos + 2, e->tokpos, 4, cudaMemcpyDeviceToHost, e->stream));
    if (h_logits) AF_CUDA_TRY(gather_logits(e, h_logits));
    ENG_TRY(cudaStreamSynchronize(e->stream));
    if (h_next) *h_next = e->h_tokpos[2];
    return cudaSuccess;
}

// Batched prompt pass (one GPU): tokens 0 .. n-2 go through every layer as
// T = n-1 rows at once (llama_forward_batch, src/models/llama_model.cpp:1339-1462):
// the linear layers on the tcgen05 prefill GEMM (the batched GEMV below 33
// rows), norms / bias / SwiGLU / residuals as row kernels, and per layer one
// RoPE / K-V store launch plus one causal-attention launch over all T rows
// (head dims 64 and 128; other head dims run the decode attention kernel per
// token in position order, which stores each token's K/V row before attending
// over positions <= its own).  The last token then runs the decode step, which
// produces its logits and the next token exactly as af_engine_prefill does.
cudaError_t af_engine_prefill_batched(af_engine* e, const int32_t* h_tokens, int n, int32_t pos0, float* h_logits,
                                      int32_t* h_next) {
    AF_CUDA_TRY(check_ready(e));
    if (n <= 0 || pos0 < 0 || pos0 + n > e->cfg.n_ctx) return fail("af_engine_prefill_batched: positions outside the context");
    for (int i = 0; i < n; ++i)
        if (h_tokens[i] < 0 || h_tokens[i] >= e->cfg.vocab)
            return fail("af_engine_prefill_batched: token id outside the vocabulary");
    const auto& c = e->cfg;
    const int T = n - 1;
    if (T == 0 || e->tp != 1) return af_engine_prefill(e, h_tokens, n, pos0, h_logits, h_next);
    const int E = c.n_embd, QD = e->Hl * e->hd, KD = e->KVl * e->hd, F = e->Fl;
    // one workspace for the prompt rows, kept by the engine and grown on demand
    auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t need = 3 * al((size_t)T * E * 4) + 2 * al((size_t)T * QD * 4) + 2 * al((size_t)T * KD * 4) +
                        2 * al((size_t)T * F * 4) + al((size_t)2 * T * 4);
    if (e->pf_ws_bytes < need) {
        ENG_TRY(cudaStreamSynchronize(e->stream));
        if (e->pf_ws) cudaFree(e->pf_ws);
        e->pf_ws = nullptr;
        e->pf_ws_bytes = 0;
        if (cudaMalloc(&e->pf_ws, need) != cudaSuccess)
            return fail("af_engine_prefill_batched: out of device memory for the prompt rows",
                        cudaErrorMemoryAllocation);
        e->pf_ws_bytes = need;
    }
    size_t ws_off = 0;
    auto take = [&](size_t bytes) {
        void* p = static_cast<uint8_t*>(e->pf_ws) + ws_off;
        ws_off += al(bytes);
        return p;
    };
    float* x = static_cast<float*>(take((size_t)T * E * 4));
    float* xn = static_cast<float*>(take((size_t)T * E * 4));
    float* tmp = static_cast<float*>(take((size_t)T * E * 4));
    float* q = static_cast<float*>(take((size_t)T * QD * 4));
    float* k = static_cast<float*>(take((size_t)T * KD * 4));
    float* v = static_cast<float*>(take((size_t)T * KD * 4));
    float* att = static_cast<float*>(take((size_t)T * QD * 4));
    float* g = static_cast<float*>(take((size_t)T * F * 4));
    float* u = static_cast<float*>(take((size_t)T * F * 4));
    int* d_tp = static_cast<int*>(take((size_t)2 * T * 4));  // tokens, then positions
    cudaError_t err = cudaSuccess;
    auto run = [&]() -> cudaError_t {
        std::vector<int32_t> tp((size_t)2 * T);
        for (int t = 0; t < T; ++t) {
            tp[t] = h_tokens[t];
            tp[T + t] = pos0 + t;
        }
        ENG_TRY(cudaMemcpyAsync(d_tp, tp.data(), tp.size() * 4, cudaMemcpyHostToDevice, e->stream));
        ENG_TRY(prompt_embed_launch(x, e->tok_embd.w, e->tok_embd.type, E, e->tok_embd.stride, d_tp, T, e->stream));
        for (int l = 0; l < c.n_layer; ++l) {
            const LayerW& L = e->layers[l];
            ENG_TRY(rows_rmsnorm_launch(xn, x, L.attn_norm, E, T, c.eps, e->stream));
            ENG_TRY(prefill_gemm_launch(q, L.wq.w, L.wq.type, xn, QD, E, T, e->stream));
            ENG_TRY(prefill_gemm_launch(k, L.wk.w, L.wk.type, xn, KD, E, T, e->stream));
            ENG_TRY(prefill_gemm_launch(v, L.wv.w, L.wv.type, xn, KD, E, T, e->stream));
            if (L.bq) ENG_TRY(rows_bias_launch(q, L.bq, QD, T, e->stream));
            if (L.bk) ENG_TRY(rows_bias_launch(k, L.bk, KD, T, e->stream));
            if (L.bv) ENG_TRY(rows_bias_launch(v, L.bv, KD, T, e->stream));
            const size_t lsz = (size_t)c.n_ctx * KD;
            if (prompt_attention_supported(e->hd)) {
                // all T tokens at once: RoPE / Q-K norms, the KV rows, causal attention
                ENG_TRY(prompt_attention_launch(q, k, v, e->kcache + (size_t)l * lsz, e->vcache + (size_t)l * lsz, att,
                                                e->cos_t, e->sin_t, L.q_norm, L.k_norm, T, pos0, e->Hl, e->KVl, e->hd,
                                                c.qk_norm_order, c.eps, e->stream));
            }
            for (int t = 0; t < T && !prompt_attention_supported(e->hd); ++t) {
                AttnParams a = {};
                a.q = q + (size_t)t * QD;
                a.k = k + (size_t)t * KD;
                a.v = v + (size_t)t * KD;
                a.kc = e->kcache + (size_t)l * lsz;
                a.vc = e->vcache + (size_t)l * lsz;
                a.out = att + (size_t)t * QD;
                a.cos_t = e->cos_t;
                a.sin_t = e->sin_t;
                a.q_norm = L.q_norm;
                a.k_norm = L.k_norm;
                a.part = e->apart;
                a.counter = e->acount;
                a.pos = d_tp + T + t;
                a.n_heads = e->Hl;
                a.n_kv_heads = e->KVl;
                a.head_dim = e->hd;
                a.n_ctx = c.n_ctx;
                a.nsplit = e->nsplit;
                a.qk_norm_order = c.qk_norm_order;
                a.eps = c.eps;
                a.scale = 1.f / std::sqrt((float)e->hd);
                ENG_TRY(attention_launch(a, e->stream, false));
            }
            ENG_TRY(prefill_gemm_launch(tmp, L.wo.w, L.wo.type, att, E, QD, T, e->stream));
            ENG_TRY(rows_add_launch(x, tmp, (long long)T * E, e->stream));
            ENG_TRY(rows_rmsnorm_launch(xn, x, L.ffn_norm, E, T, c.eps, e->stream));
            ENG_TRY(prefill_gemm_launch(g, L.wg.w, L.wg.type, xn, F, E, T, e->stream));
            ENG_TRY(prefill_gemm_launch(u, L.wu.w, L.wu.type, xn, F, E, T, e->stream));
            ENG_TRY(rows_swiglu_launch(g, u, (long long)T * F, e->stream));
            ENG_TRY(prefill_gemm_launch(tmp, L.wd.w, L.wd.type, g, E, F, T, e->stream));
            ENG_TRY(rows_add_launch(x, tmp, (long long)T * E, e->stream));
        }
        ENG_TRY(cudaStreamSynchronize(e->stream));
        return cudaSuccess;
    };
    err = run();
    if (err != cudaSuccess) return err;
    return af_engine_prefill(e, h_tokens + T, 1, pos0 + T, h_logits, h_next);
}

cudaError_t af_engine_decode_greedy(af_engine* e, int32_t first_token, int32_t pos0, int n_steps, int32_t* h_out) {
    AF_CUDA_TRY(check_ready(e));
    if (n_steps < 0 || pos0 < 0 || pos0 + n_steps > e->cfg.n_ctx) return fail("af_engine_decode_greedy: context overflow");
    if (first_token < 0 || first_token >= e->cfg.vocab) return fail("af_engine_decode_greedy: bad token");
    if (n_steps == 0) return cudaSuccess;
    e->h_tokpos[0] = first_token;
    e->h_tokpos[1] = pos0;
    ENG_TRY(cudaMemcpyAsync(e->tokpos, e->h_tokpos, 8, cudaMemcpyHostToDevice, e->stream));
    for (int i = 0; i < n_steps; ++i) ENG_TRY(cudaGraphLaunch(e->gexec, e->stream));
    if (h_out)
        ENG_TRY(cudaMemcpyAsync(h_out, e->hist + pos0, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, e->stream));
    ENG_TRY(cudaStreamSynchronize(e->stream));
    return cudaSuccess;
}

cudaError_t af_engine_generate(af_engine* e, const int32_t* h_prompt, int n_prompt, int max_new, int32_t* h_out,
                               int* n_out) {
    AF_CUDA_TRY(check_ready(e));
    if (!n_out || (max_new > 0 && !h_out)) return fail("af_engine_generate: null output");
    if (n_prompt <= 0) return fail("llama_generate: empty prompt");
    *n_out = 0;
    std::vector<int32_t> ids(h_prompt, h_prompt + n_prompt);
    if (ids[0] != e->cfg.bos_id) ids.insert(ids.begin(), e->cfg.bos_id);
    const int np = (int)ids.size();
    if (np > e->cfg.n_ctx) return fail("af_engine_generate: prompt longer than the context");
    int32_t next = 0;
    AF_CUDA_TRY(af_engine_prefill(e, ids.data(), np, 0, nullptr, &next));
    // Every pushed token is forwarded (llama_model.cpp:1611-1624); ids stop at
    // EOS (not emitted) or when n_past reaches the context cap.
    const int budget = std::min(max_new, e->cfg.n_ctx - np);
    std::vector<int32_t> gen;
    if (budget > 0) {
        std::vector<int32_t> dev(budget);
        AF_CUDA_TRY(af_engine_decode_greedy(e, next, np, budget, dev.data()));
        gen.push_back(next);
        for (int i = 0; i + 1 < budget; ++i) gen.push_back(dev[i]);
    }
    int n = 0;
    for (int32_t id : gen) {
        if (id == e->cfg.eos_id) break;
        h_out[n++] = id;
    }
    *n_out = n;
    return cudaSuccess;
}

cudaError_t af_engine_sample(af_engine* e, const af_sampling* s, const int32_t* h_window, int n_window, float r,
                             int32_t* h_next) {
    AF_CUDA_TRY(check_ready(e));
    if (!s || !h_next || n_window < 0 || n_window > e->cfg.n_ctx + 1 || (n_window > 0 && !h_window))
        return fail("af_engine_sample: bad arguments");
    std::string why;
    if (!sample_supported(*s, e->cfg.vocab, &why)) {
        set_last_error("af_engine_sample: " + why);
        return cudaErrorNotSupported;
    }
    float* lg = e->logits;
    if (e->tp > 1) {
        // the full vocabulary, in rank order, on every rank
        NCCL_TRY(ncclAllGather(e->logits, e->logits_all, e->Vmax, ncclFloat32, e->comm, e->stream));
        int off = 0;
        for (int rk = 0; rk < e->tp; ++rk) {
            int lo, hi;
            block_split(e->cfg.vocab, rk, e->tp, lo, hi);
            ENG_TRY(cudaMemcpyAsync(e->logits_full + off, e->logits_all + (size_t)rk * e->Vmax, (size_t)(hi - lo) * 4,
                                    cudaMemcpyDeviceToDevice, e->stream));
            off += hi - lo;
        }
        lg = e->logits_full;
    }
    if (n_window > 0)
        ENG_TRY(cudaMemcpyAsync(e->d_window, h_window, (size_t)n_window * 4, cudaMemcpyHostToDevice, e->stream));
    ENG_TRY(sample_launch(lg, e->cfg.vocab, e->d_window, n_window, *s, r, e->d_sampled, e->stream));
    ENG_TRY(cudaMemcpyAsync(e->h_tokpos + 3, e->d_sampled, 4, cudaMemcpyDeviceToHost, e->stream));
    ENG_TRY(cudaStreamSynchronize(e->stream));
    *h_next = e->h_tokpos[3];
    return cudaSuccess;
}

cudaError_t af_engine_generate_sampled(af_engine* e, const int32_t* h_prompt, int n_prompt, int max_new,
                                       const af_sampling* s, const float* h_draws, int n_draws, int32_t* h_out,
                                       int* n_out) {
    AF_CUDA_TRY(check_ready(e));
    if (!s || !n_out || (max_new > 0 && !h_out)) return fail("af_engine_generate_sampled: null argument");
    if (n_prompt <= 0) return fail("llama_generate: empty prompt");
    const bool draws = s->temperature > 0.f;
    if (draws && (!h_draws || n_draws < max_new + 1))
        return fail("af_engine_generate_sampled: need max_new + 1 uniform draws at temperature > 0");
    *n_out = 0;
    std::vector<int32_t> ctx(h_prompt, h_prompt + n_prompt);
    if (ctx[0] != e->cfg.bos_id) ctx.insert(ctx.begin(), e->cfg.bos_id);
    const int np = (int)ctx.size();
    if (np > e->cfg.n_ctx) return fail("af_engine_generate_sampled: prompt longer than the context");
    int di = 0;
    // penalty window: the last rep_last_n ids of prompt + generated (llama_model.cpp:1588-1592)
    auto pick = [&](int32_t& next) -> cudaError_t {
        const int win = s->rep_penalty != 1.0f ? std::min(std::max(s->rep_last_n, 0), (int)ctx.size()) : 0;
        return af_engine_sample(e, s, ctx.data() + ctx.size() - win, win, draws ? h_draws[di++] : 0.f, &next);
    };
    AF_CUDA_TRY(af_engine_prefill(e, ctx.data(), np, 0, nullptr, nullptr));
    int32_t next = 0;
    AF_CUDA_TRY(pick(next));
    int n = 0, n_past = np;
    for (int step = 0; step < max_new; ++step) {
        if (next == e->cfg.eos_id) break;  // EOS is not emitted
        if (n_past >= e->cfg.n_ctx) break;
        h_out[n++] = next;
        AF_CUDA_TRY(af_engine_step(e, next, n_past, nullptr, nullptr));
        ++n_past;
        ctx.push_back(next);
        AF_CUDA_TRY(pick(next));
    }
    *n_out = n;
    return cudaSuccess;
}

cudaError_t af_mt19937_uniform(uint32_t seed, int n, float* h_out) {
    if (n < 0 || (n > 0 && !h_out)) return fail("af_mt19937_uniform: bad arguments");
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> dist(0.f, 1.f);
    for (int i = 0; i < n; ++i) h_out[i] = dist(rng);
    return cudaSuccess;
}

cudaError_t af_engine_hidden(af_engine* e, float* h_out) {
    AF_CUDA_TRY(check_ready(e));
    ENG_TRY(cudaMemcpyAsync(h_out, e->x[0], (size_t)e->cfg.n_embd * 4, cudaMemcpyDeviceToHost, e->stream));
    ENG_TRY(cudaStreamSynchronize(e->stream));
    return cudaSuccess;
}

cudaError_t af_engine_kv(af_engine* e, int layer, int which_v, int n_pos, float* h_out) {
    AF_CUDA_TRY(check_ready(e));
    if (layer < 0 || layer >= e->cfg.n_layer || n_pos < 0 || n_pos > e->cfg.n_ctx) return fail("af_engine_kv: range");
    const size_t row = (size_t)e->KVl * e->hd;
    const float* base = (which_v ? e->vcache : e->kcache) + (size_t)layer * e->cfg.n_ctx * row;
    ENG_TRY(cudaMemcpyAsync(h_out, base, (size_t)n_pos * row * 4, cudaMemcpyDeviceToHost, e->stream));
    ENG_TRY(cudaStreamSynchronize(e->stream));
    return cudaSuccess;
}

cudaError_t af_engine_profile(af_engine* e, int32_t token, int32_t pos0, int n_steps, double* h_ms, double* h_bytes,
                              int* h_count) {
    AF_CUDA_TRY(check_ready(e));
    if (n_steps <= 0 || pos0 < 0 || pos0 + n_steps > e->cfg.n_ctx) return fail("af_engine_profile: context overflow");
    for (int k = 0; k < AF_PROF_KINDS; ++k) {
        h_ms[k] = 0;
        h_bytes[k] = 0;
        h_count[k] = 0;
    }
    e->h_tokpos[0] = token;
    e->h_tokpos[1] = pos0;
    ENG_TRY(cudaMemcpyAsync(e->tokpos, e->h_tokpos, 8, cudaMemcpyHostToDevice, e->stream));
    for (int s = 0; s < n_steps; ++s) {
        Prof prof;
        prof.pos = pos0 + s;
        AF_CUDA_TRY(prof.mark(e->stream, -1, 0));
        cudaError_t r = enqueue_step(e, &prof);
        ENG_TRY(cudaStreamSynchronize(e->stream));
        for (size_t i = 1; i < prof.ev.size() && r == cudaSuccess; ++i) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, prof.ev[i - 1], prof.ev[i]);
            const int k = prof.kinds[i];
            h_ms[k] += ms;
            h_bytes[k] += prof.bytes[i];
            h_count[k] += 1;
        }
        for (cudaEvent_t x : prof.ev) cudaEventDestroy(x);
        AF_CUDA_TRY(r);
    }
    return cudaSuccess;
}

cudaStream_t af_engine_stream(af_engine* e) { return e ? e->stream : nullptr; }
int af_engine_kernels_per_step(af_engine* e) { return e ? e->kernels_per_step : 0; }
size_t af_engine_weight_bytes(af_engine* e) { return e ? e->weight_bytes : 0; }

}  // extern "C"
