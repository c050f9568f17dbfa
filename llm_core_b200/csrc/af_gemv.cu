// af_gemv.cu — fused dequant GEMV kernel (see af_gemv.cuh for the design).
#include <algorithm>
#include <vector>

#include "af_gemv_dev.cuh"

namespace af {

__device__ int g_err = 0;

namespace {

using namespace gdev;

__global__ void xq_quantize_kernel(uint8_t* xq, const float* x, const float* norm_w, int K, int q8) {
    pdl_launch_dependents();
    pdl_wait();
    const int g = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (g < (K + 31) / 32) xq_quantize_group(xq, x, norm_w, K, g, q8 != 0);
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

cudaError_t xq_quantize_launch(uint8_t* xq, const float* x, const float* norm_w, int K, cudaStream_t st, bool pdl,
                               bool q8) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(((K + 31) / 32 + 3) / 4);
    cfg.blockDim = dim3(128);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, xq_quantize_kernel, xq, x, norm_w, K, q8 ? 1 : 0);
}

}  // namespace af
