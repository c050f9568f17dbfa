// af_gemv.cu — fused dequant GEMV kernel (see af_gemv.cuh for the design).
#include <algorithm>
#include <vector>

#include "af_gemv_dev.cuh"

namespace af {

__device__ int g_err = 0;

// Quantise value v (index idx = 32·g + lane) into the XQ layout.  The 16-bit
// split matches the consumers' integer form: q = rint(v·32639/amax),
// hi = (q + 128) >> 8, lo = q − 256·hi.
__device__ void xq_store32(uint8_t* xq, float v, const float* norm_w, int K, int idx) {
    const bool in = idx >= 0 && idx < K;
    xq_store32w(xq, v, norm_w && in ? __ldg(norm_w + idx) : 1.f, norm_w != nullptr, K, idx);
}

__device__ void xq_store32w(uint8_t* xq, float v, float wgt, bool norm, int K, int idx) {
    const int lane = threadIdx.x & 31;
    const bool in = idx >= 0 && idx < K;
    if (!in) v = 0.f;
    const float a = v * wgt;
    const float amax = warp_max(fabsf(a));
    const float inv = amax > 0.f ? 32639.f / amax : 0.f;
    const int q = max(-32639, min(32639, __float2int_rn(a * inv)));
    const int hi = (q + 128) >> 8, lo = q - 256 * hi;
    int is = q;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) is += __shfl_xor_sync(0xffffffffu, is, o);  // per 16
    const float fs = warp_sum(a);
    const float ss = norm ? warp_sum(v * v) : 0.f;
    if (!in) return;
    uint8_t* sb = xq + (idx >> 8) * kXqSb;
    const int ko = idx & 255;
    sb[ko] = (uint8_t)(hi & 0xFF);
    sb[256 + ko] = (uint8_t)(lo & 0xFF);
    if ((lane & 15) == 0) reinterpret_cast<int*>(sb + kXqI16)[ko >> 4] = is;
    if (lane == 0) {
        reinterpret_cast<float*>(sb + kXqXs)[ko >> 5] = amax / 32639.f;
        reinterpret_cast<float*>(sb + kXqS32)[ko >> 5] = fs;
        if (norm) reinterpret_cast<float*>(xq + xq_bytes(K))[idx >> 5] = ss;
    }
}

// One warp quantises values [32·g, 32·g + 32) of src (global f32, written by
// other CTAs: read through L2).
__device__ void xq_quantize_group(uint8_t* xq, const float* src, const float* norm_w, int K, int g) {
    const int idx = 32 * g + (threadIdx.x & 31);
    xq_store32(xq, idx < K ? __ldcg(src + idx) : 0.f, norm_w, K, idx);
}

namespace {

using namespace gdev;

__global__ void xq_quantize_kernel(uint8_t* xq, const float* x, const float* norm_w, int K) {
    pdl_launch_dependents();
    pdl_wait();
    const int g = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (g < (K + 31) / 32) xq_quantize_group(xq, x, norm_w, K, g);
}

__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    Ring ring;
    ring.full = reinterpret_cast<uint64_t*>(smem);
    ring.empty = ring.full + kRingDesc;
    int* flags = reinterpret_cast<int*>(smem + kHdrFlags);  // [0] abort, [1..] group list
    ring.buf = smem + kGemvSmemHdr;
    ring.bytes = p.ring_bytes;
    uint8_t* xqs = ring.buf + p.ring_bytes;
    float* misc = reinterpret_cast<float*>(xqs + xq_norm_bytes(p.K));  // 64 floats

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int vbeg = p.vrange[blockIdx.x], vend = p.vrange[blockIdx.x + 1];

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRingDesc; ++i) {
            mbar_init(&ring.full[i], 1);
            mbar_init(&ring.empty[i], kCW);
        }
        flags[0] = 0;
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();
    volatile int* abort = flags;

    if (warp == kCW) {
        // ---------------- producer: weights only, no wait on the previous kernel
        if (lane != 0) return;
        Producer pr;
        if (!pr.produce(p, vbeg, vend, ring, abort, policy_evict_first())) {
            *abort = 1;
            pr.drain(ring);
        }
        return;
    }

    // ---------------- consumer warps
    pdl_wait();
    float s_in = 1.f;  // RMSNorm scale folded into the per-group scales (XQ input)
    if (p.xq) {
        s_in = load_xq(p, xqs);
    } else {
        input_prologue(p, xqs, misc);
    }
    uint32_t consumed = 0;
    int head = 0;
    const bool ok = consume(p, vbeg, vend, ring, consumed, head, xqs, s_in, smem);
    if (!ok) *abort = 1;
}

}  // namespace

void gemv_configure(GemvParams& p, int grid) {
    // the rest of the 227 KB after the header, the XQ input and 256 B of scratch
    p.ring_bytes = (227 * 1024 - kGemvSmemHdr - xq_norm_bytes(p.K) - 256) & ~15;
    grid = grid < 1 ? 1 : (grid > kGemvMaxGrid ? kGemvMaxGrid : grid);
    p.grid = grid;
    // Fragment sizes in the order the kernel walks them (see FragIter), then
    // CTA ranges balanced by weight bytes at fragment boundaries.
    const bool sw = p.epi == EPI_SWIGLU;
    std::vector<long long> fb;
    for (int s = 0; s < (sw ? 1 : p.nseg); ++s) {
        const int tiles = (p.seg[s].rows + kPackTile - 1) / kPackTile;
        const long long tb = (long long)kPackTile * p.seg[s].row_stride * (sw ? 2 : 1);
        for (int t = 0; t < tiles; t += kGemvFragTiles) fb.push_back(tb * std::min(kGemvFragTiles, tiles - t));
    }
    std::vector<long long> pre(fb.size() + 1, 0);
    for (size_t i = 0; i < fb.size(); ++i) pre[i + 1] = pre[i] + fb[i];
    const long long total = pre.back();
    size_t f = 0;
    p.vrange[0] = 0;
    for (int i = 1; i <= grid; ++i) {
        const long long target = total * i / grid;
        // nearest fragment boundary at or after the previous one
        while (f < fb.size() && pre[f + 1] - target < target - pre[f]) ++f;
        p.vrange[i] = i == grid ? (int)fb.size() : (int)f;
    }
}

cudaError_t gemv_init() {
    return cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

cudaError_t gemv_launch(const GemvParams& p, cudaStream_t stream, bool pdl) {
    const int smem = gemv_smem_bytes(p.K, p.ring_bytes);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemv_kernel, p);
}

cudaError_t xq_quantize_launch(uint8_t* xq, const float* x, const float* norm_w, int K, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(((K + 31) / 32 + 3) / 4);
    cfg.blockDim = dim3(128);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, xq_quantize_kernel, xq, x, norm_w, K);
}

}  // namespace af
