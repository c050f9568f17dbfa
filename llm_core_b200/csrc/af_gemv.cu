// af_gemv.cu — fused dequant GEMV kernel (see af_gemv.cuh for the design).
#include "af_gemv_dev.cuh"

namespace af {

__device__ int g_err = 0;

// Quantise one 64-value group (lane l holds values 2l, 2l+1) into the XQ
// layout.  The 16-bit split matches the consumers' integer form:
// q = rint(v·32639/amax), hi = (q + 128) >> 8, lo = q − 256·hi.  With norm_w,
// w·v is quantised and Σv² (of the un-weighted values) stored after the layout.
__device__ void xq_quantize_vals(uint8_t* xq, float a0, float a1, const float* norm_w, int K, int g) {
    const int lane = threadIdx.x & 31;
    const int v0 = 64 * g + 2 * lane;
    float ss = a0 * a0 + a1 * a1;
    if (norm_w) {
        a0 *= __ldg(norm_w + v0);
        a1 *= __ldg(norm_w + v0 + 1);
    }
    const float amax = warp_max(fmaxf(fabsf(a0), fabsf(a1)));
    const float inv = amax > 0.f ? 32639.f / amax : 0.f;
    const int q0 = max(-32639, min(32639, __float2int_rn(a0 * inv)));
    const int q1 = max(-32639, min(32639, __float2int_rn(a1 * inv)));
    const int h0 = (q0 + 128) >> 8, h1 = (q1 + 128) >> 8;
    const int l0 = q0 - 256 * h0, l1 = q1 - 256 * h1;
    uint8_t* sb = xq + (v0 >> 8) * kXqSb;
    const int ko = v0 & 255;
    *reinterpret_cast<uint16_t*>(sb + ko) = (uint16_t)((h0 & 0xFF) | ((h1 & 0xFF) << 8));
    *reinterpret_cast<uint16_t*>(sb + 256 + ko) = (uint16_t)((l0 & 0xFF) | ((l1 & 0xFF) << 8));
    float fs = a0 + a1;
    int is = q0 + q1;
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
        fs += __shfl_xor_sync(0xffffffffu, fs, o);
        is += __shfl_xor_sync(0xffffffffu, is, o);
    }
    fs += __shfl_xor_sync(0xffffffffu, fs, 8);  // 16 lanes = 32 values
    if ((lane & 7) == 0) reinterpret_cast<int*>(sb + kXqI16)[ko >> 4] = is;
    if ((lane & 15) == 0) reinterpret_cast<float*>(sb + kXqS32)[ko >> 5] = fs;
    if (lane == 0) reinterpret_cast<float*>(sb + kXqXs)[ko >> 6] = amax / 32639.f;
    if (norm_w) {
        ss = warp_sum(ss);
        if (lane == 0) reinterpret_cast<float*>(xq + xq_bytes(K))[g] = ss;
    }
}

// One warp quantises 64-value group g of src (global f32, written by other
// CTAs: read through L2).
__device__ void xq_quantize_group(uint8_t* xq, const float* src, const float* norm_w, int K, int g) {
    const int v0 = 64 * g + 2 * (threadIdx.x & 31);
    xq_quantize_vals(xq, __ldcg(src + v0), __ldcg(src + v0 + 1), norm_w, K, g);
}

namespace {

using namespace gdev;

__global__ void xq_quantize_kernel(uint8_t* xq, const float* x, const float* norm_w, int K) {
    pdl_launch_dependents();
    pdl_wait();
    const int g = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (g < K / 64) xq_quantize_group(xq, x, norm_w, K, g);
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
    if (p.q_out) quantise_output(p, vbeg, vend, flags + 1);
}

}  // namespace

void gemv_configure(GemvParams& p, int grid) {
    // the rest of the 227 KB after the header, the XQ input and 256 B of scratch
    p.ring_bytes = (227 * 1024 - kGemvSmemHdr - xq_norm_bytes(p.K) - 256) & ~15;
    // CTA tile ranges balanced by weight bytes (a gate/up pair is one virtual tile)
    grid = grid < 1 ? 1 : (grid > kGemvMaxGrid ? kGemvMaxGrid : grid);
    p.grid = grid;
    const bool sw = p.epi == EPI_SWIGLU;
    const int nvs = sw ? 1 : p.nseg;
    long long total = 0;
    long long tb[3], tiles[3];
    for (int s = 0; s < nvs; ++s) {
        const long long rs = sw ? (long long)p.seg[0].row_stride + p.seg[1].row_stride : p.seg[s].row_stride;
        tb[s] = rs * kPackTile;
        tiles[s] = (p.seg[s].rows + kPackTile - 1) / kPackTile;
        total += tb[s] * tiles[s];
    }
    for (int i = 0; i <= grid; ++i) {
        long long b = total * i / grid, base = 0;
        int v = 0;
        for (int s = 0; s < nvs; ++s) {
            const long long segb = tb[s] * tiles[s];
            if (b <= segb || s == nvs - 1) {
                long long t = (b + tb[s] / 2) / tb[s];  // nearest tile boundary
                if (t > tiles[s]) t = tiles[s];
                v = (int)(base + t);
                break;
            }
            b -= segb;
            base += tiles[s];
        }
        p.vrange[i] = i == 0 ? 0 : (v < p.vrange[i - 1] ? p.vrange[i - 1] : v);
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
    cfg.gridDim = dim3((K / 64 + 3) / 4);
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
