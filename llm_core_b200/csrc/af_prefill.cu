// af_prefill.cu — prefill dequant-GEMM on the 5th-generation tensor cores
// (tcgen05 + TMEM, sm_100a).
//
// Y[T][rows] = X[T][cols] · dequant(W)ᵀ for a packed Q4_K / Q6_K matrix W
// (af_weight_pack layout) and T tokens of f32 activations: the linear layers
// of a prompt, the reference's llama_forward_batch
// (src/models/llama_model.cpp:1339-1462) with its 4-row × 8-token Q8 GEMM
// tiles (gemm_q4k_q8_avx2_range, src/backend/cpu_x86/kernels/gemv_q4k_q8_avx2.cpp:257-346).
// Unlike decode, prefill is a dense contraction (2·rows·cols·T flops against
// rows·cols·0.56 weight bytes), so it belongs on the tensor cores:
//
//  * CTA tile: 128 weight rows × 128 tokens; the f32 accumulators live in
//    tensor memory (128 lanes × 128 columns), never in registers.
//  * K advances in stages of 64 values.  All 256 threads build a stage in
//    shared memory: the weight rows dequantised to bf16 (w = d·sc·q − dmin·m
//    for Q4_K, d·sc·(q − 32) for Q6_K, as the reference dequantises) and the
//    activations split into two bf16 planes, x ≈ hi + lo (the split keeps the
//    activation error near 2⁻¹⁶, so the bf16 rounding of the weights is the
//    only error that matters: ~1e-3 relative).
//  * Both operands are K-major in the no-swizzle canonical layout: 16-byte
//    core-matrix rows, 8-row groups 128 B apart (SBO), the two 16-byte K
//    halves of one MMA K-step 2 KiB apart (LBO).
//  * One elected thread issues 8 tcgen05.mma (kind::f16, bf16 × bf16 → f32,
//    M = 128, N = 128, K = 16: four K-steps × hi/lo) per stage and commits
//    them to the stage's mbarrier; the stage's buffer is rebuilt only after
//    that commit lands (two buffers, so building stage s + 1 overlaps the
//    tensor work of stage s).
//  * Epilogue: warps 0-3 read their 32 TMEM lanes (tcgen05.ld 32x32b) and
//    store token-major rows of Y (consecutive lanes = consecutive rows).
//  Every wait is bounded; on a timeout the kernel records an error, stops
//  issuing, and still frees its tensor memory.
#include <cuda_bf16.h>

#include <cstdint>

#include "af_ops.cuh"

namespace af {
namespace {

constexpr int kPfM = 128;       // weight rows per CTA tile (MMA M)
constexpr int kPfN = 128;       // tokens per CTA tile (MMA N, TMEM columns)
constexpr int kPfK = 64;        // K values per stage
constexpr int kPfThreads = 256;
constexpr int kPfPlane = kPfM * kPfK * 2;  // bytes of one bf16 operand plane of a stage (16 KiB)
constexpr int kPfStage = 3 * kPfPlane;     // A, B hi, B lo
constexpr int kPfHdr = 1024;               // mbarriers + TMEM address
constexpr int kPfSmem = kPfHdr + 2 * kPfStage;
static_assert(kPfM == kPfN, "A and B planes share the stage geometry");

__device__ __forceinline__ uint32_t bf16_bits(float f) {
    return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float bf16_val(uint32_t b) { return __uint_as_float(b << 16); }

// Shared-memory matrix descriptor: K-major, no swizzle; start, LBO, SBO in
// 16-byte units, descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::f16: f32 accumulate, bf16 A and B, both
// K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kPfIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kPfN >> 3) << 17) |
                              ((uint32_t)(kPfM >> 4) << 24);

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(kPfIdesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 16 consecutive f32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Eight consecutive dequantised values k0 .. k0+7 (k0 % 8 == 0) of packed row
// m (the reference's dequantisation: dequant_q4k_row / q6k_row_to_f32,
// src/models/llama_model.cpp:476-504, 560-592).
__device__ __forceinline__ void dequant8(const uint8_t* __restrict__ W, int type, int row_stride, int m, int k0,
                                         float (&w)[8]) {
    const int b = k0 >> 8, k = k0 & 255, r = m & (kPackTile - 1);
    const uint8_t* unit = W + (size_t)(m / kPackTile) * kPackTile * row_stride + (size_t)b * unit_bytes(type);
    const int l0 = k & 31;  // multiple of 8: words l0/4 and l0/4 + 1 of the 32-value chunk
    if (type == AF_GGML_Q6_K) {
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(unit + kQ6D + 2 * r));
        const int sc = (int8_t)unit[kQ6Sc + 16 * r + (k >> 4)];
        const int P = k >> 6, hiq = (k & 63) >= 32, Q = k >> 7, s = (k & 127) >> 5;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int wd = (l0 >> 2) + h;
            const uint32_t lo = *reinterpret_cast<const uint32_t*>(unit + P * 512 + packed_frag_off(r, wd, 0));
            const uint32_t hi = *reinterpret_cast<const uint32_t*>(unit + kQ6Hi + Q * 512 + packed_frag_off(r, wd, 0));
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int lb = (lo >> (8 * i)) & 0xFF, hb = (hi >> (8 * i)) & 0xFF;
                const int q = ((hiq ? lb >> 4 : lb) & 0xF) | (((hb >> (2 * s)) & 3) << 4);
                w[4 * h + i] = d * sc * (q - 32);
            }
        }
        return;
    }
    const uint8_t* hdr = unit + kQ4Hdr + 16 * r;
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(hdr));
    const float dmin = half_bits_to_float(*reinterpret_cast<const uint16_t*>(hdr + 2));
    const uint8_t* sc = hdr + 4;
    const int chunk = k >> 6, rr = k & 63, j = chunk * 2 + (rr >> 5);
    int s, mn;
    if (j < 4) {
        s = sc[j] & 63;
        mn = sc[j + 4] & 63;
    } else {
        s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
        mn = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
    const float ds = d * s, dm = dmin * mn;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t qw = *reinterpret_cast<const uint32_t*>(unit + chunk * 512 + packed_frag_off(r, (l0 >> 2) + h, 0));
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int qb = (qw >> (8 * i)) & 0xFF;
            const int q = rr < 32 ? (qb & 0xF) : (qb >> 4);
            w[4 * h + i] = ds * q - dm;
        }
    }
}

__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_gemm_kernel(float* __restrict__ Y, const uint8_t* __restrict__ W, int type, const float* __restrict__ X,
                        int rows, int cols, int T) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* done = reinterpret_cast<uint64_t*>(smem);          // [2] MMA completion per buffer
    uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + 64);    // TMEM base address
    volatile int* flag = reinterpret_cast<volatile int*>(smem + 128);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * kPfM, n0 = blockIdx.y * kPfN;
    const int tiles = (rows + kPackTile - 1) / kPackTile;
    const int row_stride = dev_row_stride(type, cols);
    const int nst = cols / kPfK;

    if (tid == 0) {
        mbar_init(&done[0], 1);
        mbar_init(&done[1], 1);
        *flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                     "r"((uint32_t)kPfN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    for (int s = 0; s < nst; ++s) {
        const int buf = s & 1;
        uint8_t* A = smem + kPfHdr + buf * kPfStage;
        uint8_t* Bh = A + kPfPlane;
        uint8_t* Bl = Bh + kPfPlane;
        if (s >= 2) {  // the MMAs that read this buffer (stage s - 2) have completed
            if (!mbar_wait(&done[buf], (uint32_t)((s - 2) >> 1) & 1u, flag)) {
                if (tid == 0 && !*flag) set_err(kErrMbarTimeout);
                *flag = 1;
            }
            tc_fence_after();
        }
        __syncthreads();
        if (*flag) break;
        const int kb = s * kPfK;
        // A: 128 rows × 8 sixteen-byte chunks; B: 128 tokens × 8 chunks (hi and lo planes)
        for (int it = tid; it < kPfM * (kPfK / 8); it += kPfThreads) {
            const int row = it & (kPfM - 1), c8 = it / kPfM;
            const int m = m0 + row;
            uint4 pk = make_uint4(0u, 0u, 0u, 0u);
            if (m < tiles * kPackTile) {
                float w[8];
                dequant8(W, type, row_stride, m, kb + 8 * c8, w);
                pk.x = bf16_bits(w[0]) | (bf16_bits(w[1]) << 16);
                pk.y = bf16_bits(w[2]) | (bf16_bits(w[3]) << 16);
                pk.z = bf16_bits(w[4]) | (bf16_bits(w[5]) << 16);
                pk.w = bf16_bits(w[6]) | (bf16_bits(w[7]) << 16);
            }
            *reinterpret_cast<uint4*>(A + c8 * (kPfM * 16) + row * 16) = pk;
        }
        for (int it = tid; it < kPfN * (kPfK / 8); it += kPfThreads) {
            const int tok = it & (kPfN - 1), c8 = it / kPfN;
            const int n = n0 + tok;
            uint4 ph = make_uint4(0u, 0u, 0u, 0u), pl = ph;
            if (n < T) {
                const float4* src = reinterpret_cast<const float4*>(X + (size_t)n * cols + kb + 8 * c8);
                const float4 a = __ldg(src), b = __ldg(src + 1);
                const float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
                uint32_t h[8], l[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    h[i] = bf16_bits(x[i]);
                    l[i] = bf16_bits(x[i] - bf16_val(h[i]));
                }
                ph = make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
                pl = make_uint4(l[0] | (l[1] << 16), l[2] | (l[3] << 16), l[4] | (l[5] << 16), l[6] | (l[7] << 16));
            }
            *reinterpret_cast<uint4*>(Bh + c8 * (kPfN * 16) + tok * 16) = ph;
            *reinterpret_cast<uint4*>(Bl + c8 * (kPfN * 16) + tok * 16) = pl;
        }
        fence_proxy_async_smem();  // generic-proxy stores → visible to the tensor core
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t a0 = smem_u32(A), h0 = smem_u32(Bh), l0 = smem_u32(Bl);
#pragma unroll
            for (int ks = 0; ks < kPfK / 16; ++ks) {
                const uint32_t off = (uint32_t)ks * 2 * (kPfM * 16);
                const uint64_t ad = smem_desc(a0 + off, kPfM * 16, 128);
                tc_mma(tmem, ad, smem_desc(h0 + off, kPfN * 16, 128), (s > 0 || ks > 0) ? 1u : 0u);
                tc_mma(tmem, ad, smem_desc(l0 + off, kPfN * 16, 128), 1u);
            }
            tc_commit(&done[buf]);
        }
    }
    // the last commit covers every MMA issued before it
    if (!*flag && nst > 0) {
        const int last = nst - 1;
        if (!mbar_wait(&done[last & 1], (uint32_t)(last >> 1) & 1u, flag)) {
            if (tid == 0 && !*flag) set_err(kErrMbarTimeout);
            *flag = 1;
        }
    }
    tc_fence_after();
    __syncthreads();
    if (!*flag && warp < 4) {
        const int row = warp * 32 + lane;
        const int m = m0 + row;
#pragma unroll 1
        for (int c = 0; c < kPfN; c += 16) {
            float v[16];
            tc_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, v);
            if (m < rows) {
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    if (n0 + c + i < T) Y[(size_t)(n0 + c + i) * rows + m] = v[i];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)kPfN)
                     : "memory");
    }
}

}  // namespace

cudaError_t prefill_gemm_launch(float* y, const uint8_t* w, int type, const float* x, int rows, int cols, int T,
                                cudaStream_t st) {
    static int attr_dev = -1;
    int dev = 0;
    AF_CUDA_TRY(cudaGetDevice(&dev));
    if (attr_dev != dev) {
        AF_CUDA_TRY(cudaFuncSetAttribute(prefill_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmem));
        attr_dev = dev;
    }
    const dim3 grid((rows + kPfM - 1) / kPfM, (T + kPfN - 1) / kPfN);
    prefill_gemm_kernel<<<grid, kPfThreads, kPfSmem, st>>>(y, w, type, x, rows, cols, T);
    return cudaGetLastError();
}

}  // namespace af

using namespace af;

extern "C" cudaError_t af_prefill_gemm_f32(float* d_y, const void* d_w, int ggml_type, const float* d_x, int rows,
                                           int cols, int n_tokens, cudaStream_t stream) {
    if ((ggml_type != AF_GGML_Q4_K && ggml_type != AF_GGML_Q6_K) || cols <= 0 || cols % 256 || rows < 0 ||
        n_tokens < 0) {
        set_last_error("af_prefill_gemm_f32: need Q4_K/Q6_K weights, cols % 256 == 0, rows, n_tokens >= 0");
        return cudaErrorInvalidValue;
    }
    if ((reinterpret_cast<uintptr_t>(d_w) & 15) || (reinterpret_cast<uintptr_t>(d_x) & 15)) {
        set_last_error("af_prefill_gemm_f32: weights and x must be 16-byte aligned");
        return cudaErrorInvalidValue;
    }
    if (rows == 0 || n_tokens == 0) return cudaSuccess;
    return prefill_gemm_launch(d_y, static_cast<const uint8_t*>(d_w), ggml_type, d_x, rows, cols, n_tokens, stream);
}
