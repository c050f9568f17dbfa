// af_gemv.cu — fused dequant GEMV kernel (see af_gemv.cuh for the design).
#include "af_gemv_dev.cuh"

namespace af {

__device__ int g_err = 0;

// Quantise one 64-value group (lane l holds values 2l, 2l+1) into the XQ
// layout.  The 16-bit split matches the consumers' dp4a form:
// q = rint(v·32639/amax), hi = (q + 128) >> 8, lo = q − 256·hi.  With norm_w,
// w·v is quantised and Σv² (of the un-weighted values) stored after the layout.
__device__ void xq_quantize_vals(uint8_t* xq, float a0, float a1, const float* norm_w, int K, int g) {
    const int lane = threadIdx.x & 31;
    const int nst = (K / 256 + 7) / 8;
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
    const int s = v0 >> 11, w = v0 & 2047;
    const int b = w >> 8, c = (w >> 6) & 3, i = (w >> 4) & 3, e = w & 15;
    const int L = b * 4 + c;
    const int off = s * 2048 + i * 512 + L * 16 + e;
    *reinterpret_cast<uint16_t*>(xq + off) = (uint16_t)((h0 & 0xFF) | ((h1 & 0xFF) << 8));
    *reinterpret_cast<uint16_t*>(xq + nst * 2048 + off) = (uint16_t)((l0 & 0xFF) | ((l1 & 0xFF) << 8));
    float* XS = reinterpret_cast<float*>(xq + 2 * nst * 2048);
    float* XS32 = XS + nst * 32;
    int* XI16 = reinterpret_cast<int*>(XS32 + nst * 64);
    float fs = a0 + a1;
    int is = q0 + q1;
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
        fs += __shfl_xor_sync(0xffffffffu, fs, o);
        is += __shfl_xor_sync(0xffffffffu, is, o);
    }
    fs += __shfl_xor_sync(0xffffffffu, fs, 8);  // 16 lanes = 32 values
    if ((lane & 7) == 0) XI16[s * 128 + i * 32 + L] = is;
    if ((lane & 15) == 0) XS32[s * 64 + (i >> 1) * 32 + L] = fs;
    if (lane == 0) XS[s * 32 + L] = amax / 32639.f;
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

// Legacy prologue: f32 input (+ pending residual, optionally RMS-normalised)
// loaded with all NIT float4 loads per thread in flight, then quantised into
// the shared XQ layout (NST stages of 512 float4; the padded tail is zero).
template <int NST>
__device__ __forceinline__ void input_prologue(const GemvParams& p, uint8_t* xqs, float* red) {
    constexpr int NIT = (NST * 512 + kCT - 1) / kCT;
    static_assert(kCT % 16 == 0, "16 consecutive threads own one 64-value group");
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int nvec = p.K / 4;
    const int nst = NST;
    const int nslot = NST * 512;
    uint8_t* XH = xqs;
    uint8_t* XL = xqs + nst * 2048;
    float* XS = reinterpret_cast<float*>(xqs + 2 * nst * 2048);
    float* XS32 = XS + nst * 32;
    int* XI16 = reinterpret_cast<int*>(XS32 + nst * 64);
    float4 a[NIT];
#pragma unroll
    for (int j = 0; j < NIT; ++j) {
        const int v = j * kCT + tid;
        const int vc = v < nvec ? v : 0;
        a[j] = reinterpret_cast<const float4*>(p.x)[vc];
        if (p.x_add) {
            const float4 b = reinterpret_cast<const float4*>(p.x_add)[vc];
            a[j].x += b.x; a[j].y += b.y; a[j].z += b.z; a[j].w += b.w;
        }
        if (v >= nvec) a[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (p.x_store && blockIdx.x == 0) {
#pragma unroll
        for (int j = 0; j < NIT; ++j) {
            const int v = j * kCT + tid;
            if (v < nvec) reinterpret_cast<float4*>(p.x_store)[v] = a[j];
        }
    }
    if (p.norm_w) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < NIT; ++j)
            ss += a[j].x * a[j].x + a[j].y * a[j].y + a[j].z * a[j].z + a[j].w * a[j].w;
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        bar_consumers();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kCW; ++w) tot += red[w];
        // rms_norm_out (src/models/llama_model.cpp:393-419): 1/sqrt(ss/n + eps)
        const float inv_rms = 1.f / sqrtf(tot / (float)p.K + p.eps);
#pragma unroll
        for (int j = 0; j < NIT; ++j) {
            const int v = j * kCT + tid;
            const float4 w = reinterpret_cast<const float4*>(p.norm_w)[v < nvec ? v : 0];
            a[j].x = w.x * (a[j].x * inv_rms);
            a[j].y = w.y * (a[j].y * inv_rms);
            a[j].z = w.z * (a[j].z * inv_rms);
            a[j].w = w.w * (a[j].w * inv_rms);
        }
    }
    float amax[NIT];
#pragma unroll
    for (int j = 0; j < NIT; ++j)
        amax[j] = fmaxf(fmaxf(fabsf(a[j].x), fabsf(a[j].y)), fmaxf(fabsf(a[j].z), fabsf(a[j].w)));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1)
#pragma unroll
        for (int j = 0; j < NIT; ++j) amax[j] = fmaxf(amax[j], __shfl_xor_sync(0xffffffffu, amax[j], o));
    float fsum[NIT];
    int isum[NIT];
#pragma unroll
    for (int j = 0; j < NIT; ++j) {
        const int v = j * kCT + tid;
        isum[j] = 0;
        fsum[j] = 0.f;
        // 16-bit grid of ±32639 so that hi = (q + 128) >> 8 stays within int8.
        if (v >= nslot) continue;  // beyond the padded last stage (kCT does not divide 512)
        const float inv = amax[j] > 0.f ? 32639.f / amax[j] : 0.f;
        const float av[4] = {a[j].x, a[j].y, a[j].z, a[j].w};
        uint32_t hw = 0, lw = 0;
        int is = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            int q = __float2int_rn(av[e] * inv);
            q = max(-32639, min(32639, q));
            const int hi = (q + 128) >> 8;
            const int lo = q - hi * 256;
            hw |= (uint32_t)(hi & 0xFF) << (8 * e);
            lw |= (uint32_t)(lo & 0xFF) << (8 * e);
            is += q;
        }
        isum[j] = is;
        fsum[j] = a[j].x + a[j].y + a[j].z + a[j].w;
        const int val = v * 4;
        const int s = val >> 11, w = val & 2047;
        const int b = w >> 8, c = (w >> 6) & 3, i = (w >> 4) & 3, e = w & 15;
        const int off = s * 2048 + i * 512 + (b * 4 + c) * 16 + e;
        *reinterpret_cast<uint32_t*>(XH + off) = hw;
        *reinterpret_cast<uint32_t*>(XL + off) = lw;
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1)
#pragma unroll
        for (int j = 0; j < NIT; ++j) {
            fsum[j] += __shfl_xor_sync(0xffffffffu, fsum[j], o);
            isum[j] += __shfl_xor_sync(0xffffffffu, isum[j], o);
        }
#pragma unroll
    for (int j = 0; j < NIT; ++j) {
        const float fsum32 = fsum[j] + __shfl_xor_sync(0xffffffffu, fsum[j], 4);
        if (j * kCT + tid >= nslot) continue;
        const int val = (j * kCT + tid) * 4;
        const int s = val >> 11, w = val & 2047;
        const int b = w >> 8, c = (w >> 6) & 3, i = (w >> 4) & 3;
        const int L = b * 4 + c;
        if ((tid & 15) == 0) XS[s * 32 + L] = amax[j] / 32639.f;
        if ((tid & 7) == 0) XS32[s * 64 + (i >> 1) * 32 + L] = fsum32;
        if ((tid & 3) == 0) XI16[s * 128 + i * 32 + L] = isum[j];
    }
}

__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    Ring ring;
    ring.full = reinterpret_cast<uint64_t*>(smem);
    ring.empty = ring.full + kRingDesc;
    int* flags = reinterpret_cast<int*>(smem + 256);  // [0] abort, [1..] group list
    ring.buf = smem + kGemvSmemHdr;
    ring.bytes = p.ring_bytes;
    uint8_t* xqs = ring.buf + p.ring_bytes;
    float* misc = reinterpret_cast<float*>(xqs + xq_norm_bytes(p.K));  // 64 floats
    const int nst = (p.K / 256 + 7) / 8;

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
        switch (nst) {
            case 1: input_prologue<1>(p, xqs, misc); break;
            case 2: input_prologue<2>(p, xqs, misc); break;
            case 3: input_prologue<3>(p, xqs, misc); break;
            case 4: input_prologue<4>(p, xqs, misc); break;
            case 5: input_prologue<5>(p, xqs, misc); break;
            default: input_prologue<6>(p, xqs, misc); break;
        }
        bar_consumers();
    }
    uint32_t consumed = 0;
    int head = 0;
    const bool ok = consume(p, vbeg, vend, ring, consumed, head, xqs, s_in, abort);
    if (!ok) *abort = 1;
    if (p.q_out) quantise_output(p, vbeg, vend, flags + 1);
}

}  // namespace

void gemv_configure(GemvParams& p, int grid) {
    // the rest of the 227 KB after the header, the XQ input and 256 B of scratch
    p.ring_bytes = (227 * 1024 - kGemvSmemHdr - xq_norm_bytes(p.K) - 256) & ~15;
    // CTA row ranges balanced by weight bytes (a gate/up pair is one virtual row)
    grid = grid < 1 ? 1 : (grid > kGemvMaxGrid ? kGemvMaxGrid : grid);
    p.grid = grid;
    const bool sw = p.epi == EPI_SWIGLU;
    const int nvs = sw ? 1 : p.nseg;
    long long total = 0;
    long long rb[3], rows[3];
    for (int s = 0; s < nvs; ++s) {
        rb[s] = sw ? (long long)p.seg[0].row_stride + p.seg[1].row_stride : p.seg[s].row_stride;
        rows[s] = p.seg[s].rows;
        total += rb[s] * rows[s];
    }
    for (int i = 0; i <= grid; ++i) {
        long long b = total * i / grid, base = 0;
        int v = 0;
        for (int s = 0; s < nvs; ++s) {
            const long long segb = rb[s] * rows[s];
            if (b <= segb || s == nvs - 1) {
                long long r = (b + rb[s] - 1) / rb[s];
                if (r > rows[s]) r = rows[s];
                v = (int)(base + r);
                break;
            }
            b -= segb;
            base += rows[s];
        }
        p.vrange[i] = v;
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
