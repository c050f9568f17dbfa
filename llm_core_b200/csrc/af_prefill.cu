// af_prefill.cu — prefill dequant-GEMM on the 5th-generation tensor cores
// (tcgen05 + TMEM, sm_100a).
//
// Y[T][rows] = X[T][cols] · dequant(W)ᵀ for a packed Q4_K / Q6_K matrix W
// (af_weight_pack layout) and T tokens of f32 activations: the linear layers
// of a prompt, the reference's llama_forward_batch
// (src/models/llama_model.cpp:1339-1462) with its 4-row × 8-token Q8 GEMM
// tiles (gemm_q4k_q8_avx2_range, src/backend/cpu_x86/kernels/gemv_q4k_q8_avx2.cpp:257-346).
// Unlike decode, prefill is a dense contraction (2·rows·cols·T flops against
// rows·cols·0.56 weight bytes), so it belongs on the tensor cores.
//
//  * X is staged once per call (prefill_pack_x): every token is scaled by a
//    power of two that puts its largest |x| in [2^14, 2^15) (exact, undone in
//    the epilogue; no f16 overflow whatever the activation range), converted
//    to f16 and laid out per (128-token tile, 64-value stage) exactly as the
//    tensor core reads it from shared memory, so one bulk copy moves a stage.
//  * CTA tile: 128 weight rows × 128 tokens, f32 accumulators in tensor
//    memory (128 lanes × 128 columns).  Four A/B stages and a two-super-block
//    ring of raw weight units per CTA, one CTA per SM.
//  * Warp roles (18 warps): a loader thread issues the bulk copies (TMA
//    engine, no tensor map, no multicast): per 256-value super-block one copy
//    of each of the CTA's 8 packed weight units (contiguous in the packed
//    layout; a ring of two super-blocks), per 64-value stage one X tile (small
//    copies cost the TMA engine a fixed time each, so they are made few and
//    large); 16 builder warps dequantise half a 16-row unit each from shared
//    memory into the f16 A tile
//    (w = d·sc·q − dmin·m for Q4_K, d·sc·(q − 32) for Q6_K, as the reference
//    dequantises); one thread issues the stage's 4 tcgen05.mma (kind::f16,
//    f16 × f16 → f32, M = N = 128, K = 16) and commits them to the stage's
//    "empty" barrier, which frees the buffers for the loader.
//  * f16 operands (11-bit significands) keep the GEMM at ~4e-4 relative error
//    with one MMA per K-step; bf16 would need a hi/lo split of x (twice the
//    tensor work) to stay inside the GEMV tolerance.
//  * Both operands are K-major in the no-swizzle canonical layout: 16-byte
//    core-matrix rows, 8-row groups 128 B apart (SBO), the two 16-byte K
//    halves of one MMA K-step 2 KiB apart (LBO).
//  * Epilogue: warps 0-3 read their 32 TMEM lanes (tcgen05.ld 32x32b), undo
//    the token scale and store token-major rows of Y.
//  Every wait is bounded; on a timeout the kernel records an error, stops
//  issuing, and still frees its tensor memory.
#include <cuda_fp16.h>

#include <cmath>
#include <cstdint>
#include <mutex>

#include "af_ops.cuh"

namespace af {
namespace {

constexpr int kPfM = 128;        // weight rows per CTA tile (MMA M): 8 units
constexpr int kPfN = 128;        // tokens per CTA tile (MMA N, TMEM columns)
constexpr int kPfK = 64;         // K values per stage
constexpr int kPfUnits = 8;      // 16-row units per CTA tile
constexpr int kPfBuilders = 16;  // builder warps: rows g (even warp) or g + 8 (odd warp) of one unit
constexpr int kPfMmaWarp = kPfBuilders, kPfLoadWarp = kPfBuilders + 1;
constexpr int kPfThreads = (kPfBuilders + 2) * 32;
constexpr int kPfPlane = kPfM * kPfK * 2;  // one f16 operand tile of a stage (16 KiB)
constexpr int kPfStage = 2 * kPfPlane;     // A, B
constexpr int kPfRawSlot = (kPfUnits * 3360 + 1023) / 1024 * 1024;  // one super-block of the CTA's 8 units (Q6_K size)
constexpr int kPfRawSlots = 2;
constexpr int kPfHdr = 1024;
// A/B stages in flight (one CTA per SM), plus the raw weight ring
constexpr int kPfStages = 4;
template <int S>
constexpr int pf_smem() { return kPfHdr + kPfRawSlots * kPfRawSlot + S * kPfStage; }
static_assert(kPfM == kPfN, "A and B tiles share the stage geometry");
static_assert(kPfStage % 1024 == 0 && kPfRawSlot % 1024 == 0, "stage alignment");
static_assert(pf_smem<kPfStages>() <= 227 * 1024, "stage budget");

// Shared-memory matrix descriptor: K-major, no swizzle; start, LBO, SBO in
// 16-byte units, descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::f16: f32 accumulate (bits 4-5 = 1), f16 A
// and B (formats 0), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kPfIdesc = (1u << 4) | ((uint32_t)(kPfN >> 3) << 17) | ((uint32_t)(kPfM >> 4) << 24);

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

__device__ __forceinline__ uint32_t h2bits(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Store 4 f16 values of A tile row `row` starting at K index k (k % 4 == 0).
__device__ __forceinline__ void st_a4(uint8_t* A, int row, int k, float a, float b, float c, float d) {
    *reinterpret_cast<uint2*>(A + (k >> 3) * (kPfM * 16) + row * 16 + (k & 7) * 2) = make_uint2(h2bits(a, b), h2bits(c, d));
}

// Builder lane's share of a Q4_K unit stage (chunk c of the super-block; a
// whole packed unit in shared memory): the 16-byte fragment word group of
// lane L holds rows g, g+8 × words t, t+4 (see af_gemv.cuh); low nibbles are
// sub-block 2c, high nibbles 2c + 1.
__device__ __forceinline__ void build_q4(uint8_t* A, const uint8_t* unit, int row0, int c, int lane, int h) {
    const int g = lane >> 2, t = lane & 3;
    const uint4 qv = *reinterpret_cast<const uint4*>(unit + c * 512 + lane * 16);
    const uint32_t qw0 = h ? qv.y : qv.x, qw1 = h ? qv.w : qv.z;  // words t, t + 4 of row g + 8h
    {  // row g (h = 0) or g + 8
        const int r = g + 8 * h;
        const uint8_t* hdr = unit + kQ4Hdr + 16 * r;
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(hdr));
        const float dmin = half_bits_to_float(*reinterpret_cast<const uint16_t*>(hdr + 2));
        const uint8_t* sc = hdr + 4;
        float ds[2], dm[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int j = 2 * c + q;
            int sv, mv;
            if (j < 4) {
                sv = sc[j] & 63;
                mv = sc[j + 4] & 63;
            } else {
                sv = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
                mv = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
            }
            ds[q] = d * sv;
            dm[q] = dmin * mv;
        }
#pragma unroll
        for (int ww = 0; ww < 2; ++ww) {  // word t (ww = 0) or t + 4
            const uint32_t wd = ww ? qw1 : qw0;
            const int k = 4 * (t + 4 * ww);
            float lo[4], hi[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int qb = (wd >> (8 * i)) & 0xFF;
                lo[i] = ds[0] * (qb & 0xF) - dm[0];
                hi[i] = ds[1] * (qb >> 4) - dm[1];
            }
            st_a4(A, row0 + r, k, lo[0], lo[1], lo[2], lo[3]);
            st_a4(A, row0 + r, 32 + k, hi[0], hi[1], hi[2], hi[3]);
        }
    }
}

// Q6_K unit stage P = c of the super-block (a whole packed unit in shared
// memory): low nibbles of the 64-value block P, the high 2-bit fields of its
// 128-value quad, the 16 rows' scales and d.
__device__ __forceinline__ void build_q6(uint8_t* A, const uint8_t* unit, int row0, int c, int lane, int h) {
    const int g = lane >> 2, t = lane & 3;
    const uint4 lv = *reinterpret_cast<const uint4*>(unit + c * 512 + lane * 16);
    const uint4 hv = *reinterpret_cast<const uint4*>(unit + kQ6Hi + (c >> 1) * 512 + lane * 16);
    const uint32_t lw0 = h ? lv.y : lv.x, lw1 = h ? lv.w : lv.z, hw0 = h ? hv.y : hv.x, hw1 = h ? hv.w : hv.z;
    const int s0 = 2 * (c & 1);  // 32-value group of the low nibbles within the quad (high: s0 + 1)
    {
        const int r = g + 8 * h;
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(unit + kQ6D + 2 * r));
        const int8_t* scr = reinterpret_cast<const int8_t*>(unit + kQ6Sc + 16 * r + 4 * c);
#pragma unroll
        for (int ww = 0; ww < 2; ++ww) {
            const uint32_t lo_w = ww ? lw1 : lw0, hi_w = ww ? hw1 : hw0;
            const int k = 4 * (t + 4 * ww);  // 0..31
            const int sc_lo = scr[k >> 4], sc_hi = scr[2 + (k >> 4)];
            float lo[4], hi[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int lb = (lo_w >> (8 * i)) & 0xFF, hb = (hi_w >> (8 * i)) & 0xFF;
                const int q0 = (lb & 0xF) | (((hb >> (2 * s0)) & 3) << 4);
                const int q1 = (lb >> 4) | (((hb >> (2 * s0 + 2)) & 3) << 4);
                lo[i] = d * sc_lo * (q0 - 32);
                hi[i] = d * sc_hi * (q1 - 32);
            }
            st_a4(A, row0 + r, k, lo[0], lo[1], lo[2], lo[3]);
            st_a4(A, row0 + r, 32 + k, hi[0], hi[1], hi[2], hi[3]);
        }
    }
}

template <int kPfS>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_gemm_kernel(float* __restrict__ Y, const uint8_t* __restrict__ W, int type, const uint8_t* __restrict__ Xp,
                        const int* __restrict__ xexp, int rows, int cols, int T) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full_b = reinterpret_cast<uint64_t*>(smem);        // [kPfS] X tile copy (tx)
    uint64_t* full_a = full_b + kPfS;                             // [kPfS] builder warps
    uint64_t* empty = full_a + kPfS;                              // [kPfS] MMA completion
    uint64_t* accf = empty + kPfS;                                // accumulators final
    uint64_t* raw_full = accf + 1;                                // [kPfRawSlots] unit copies (tx)
    uint64_t* raw_empty = raw_full + kPfRawSlots;                 // [kPfRawSlots] builder warps
    uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + 256);
    volatile int* flag = reinterpret_cast<volatile int*>(smem + 320);
    uint8_t* rawbase = smem + kPfHdr;
    uint8_t* stbase = rawbase + kPfRawSlots * kPfRawSlot;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * kPfM, nt = blockIdx.y, n0 = nt * kPfN;
    const int tiles = (rows + kPackTile - 1) / kPackTile;
    const int row_stride = dev_row_stride(type, cols);
    const int ub = unit_bytes(type);
    const int nst = cols / kPfK;
    const bool q6 = type == AF_GGML_Q6_K;

    if (tid == 0) {
        for (int i = 0; i < kPfS; ++i) {
            mbar_init(&full_b[i], 1);
            mbar_init(&full_a[i], kPfBuilders);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < kPfRawSlots; ++i) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], kPfBuilders);
        }
        mbar_init(accf, 1);
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

    if (warp == kPfLoadWarp) {
        // one thread: per super-block one copy of each of the CTA's units
        // (contiguous in the packed layout), per 64-value stage one X tile
        if (lane == 0) {
            const uint64_t pol_x = policy_evict_last(), pol_w = policy_evict_first();
            const int nu = max(0, min(kPfUnits, tiles - m0 / kPackTile));
            for (int j = 0; j < nst && !*flag; ++j) {
                if ((j & 3) == 0) {
                    const int sb = j >> 2, rs = sb % kPfRawSlots;
                    if (sb >= kPfRawSlots &&
                        !mbar_wait(&raw_empty[rs], (uint32_t)((sb / kPfRawSlots) - 1) & 1u, flag)) {
                        *flag = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&raw_full[rs], (uint32_t)(nu * ub));
                    for (int u = 0; u < nu; ++u)
                        bulk_g2s(rawbase + rs * kPfRawSlot + u * ub,
                                 W + (size_t)(m0 / kPackTile + u) * kPackTile * row_stride + (size_t)sb * ub,
                                 (uint32_t)ub, &raw_full[rs], pol_w);
                }
                const int slot = j % kPfS;
                if (j >= kPfS && !mbar_wait(&empty[slot], (uint32_t)((j / kPfS) - 1) & 1u, flag)) {
                    *flag = 1;
                    break;
                }
                // the staged X is the previous launch's output (programmatic
                // dependent launch: everything before this overlaps it)
                if (j == 0) pdl_wait();
                mbar_arrive_expect_tx(&full_b[slot], (uint32_t)kPfPlane);
                bulk_g2s(stbase + slot * kPfStage + kPfPlane, Xp + ((size_t)nt * nst + j) * kPfPlane, kPfPlane,
                         &full_b[slot], pol_x);
            }
        }
    } else if (warp == kPfMmaWarp) {
        if (lane == 0) {
            for (int j = 0; j < nst; ++j) {
                const int slot = j % kPfS;
                const uint32_t par = (uint32_t)(j / kPfS) & 1u;
                if (!mbar_wait(&full_b[slot], par, flag) || !mbar_wait(&full_a[slot], par, flag)) {
                    *flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t a0 = smem_u32(stbase + slot * kPfStage), b0 = a0 + kPfPlane;
#pragma unroll
                for (int ks = 0; ks < kPfK / 16; ++ks) {
                    const uint32_t off = (uint32_t)ks * 2 * (kPfM * 16);
                    tc_mma(tmem, smem_desc(a0 + off, kPfM * 16, 128), smem_desc(b0 + off, kPfN * 16, 128),
                           (j > 0 || ks > 0) ? 1u : 0u);
                }
                tc_commit(&empty[slot]);
            }
            tc_commit(accf);  // arrives once every MMA issued above has completed
        }
    } else {  // builder warps: half (rows g or g + 8 of each lane group) of unit warp / 2 of every stage
        const int un = warp >> 1, h = warp & 1;
        const int mt = m0 / kPackTile + un;
        for (int j = 0; j < nst; ++j) {
            const int slot = j % kPfS, sb = j >> 2, rs = sb % kPfRawSlots, c = j & 3;
            // the stage's A slot is free once the MMAs that last read it have
            // completed (the same signal the loader waits for before the X
            // copy, so building overlaps the copy instead of following it),
            // and at a super-block's first stage its raw units have landed
            if ((c == 0 && !mbar_wait(&raw_full[rs], (uint32_t)(sb / kPfRawSlots) & 1u, flag)) ||
                (j >= kPfS && !mbar_wait(&empty[slot], (uint32_t)((j / kPfS) - 1) & 1u, flag))) {
                *flag = 1;
                break;
            }
            uint8_t* A = stbase + slot * kPfStage;
            const uint8_t* unit = rawbase + rs * kPfRawSlot + un * ub;
            if (mt < tiles) {
                if (q6) build_q6(A, unit, un * kPackTile, c, lane, h);
                else build_q4(A, unit, un * kPackTile, c, lane, h);
            } else {  // rows past the matrix: zeros (this warp's 8 rows)
                for (int i = lane; i < 8 * (kPfK / 8); i += 32) {
                    const int r = (i & 7) + 8 * h, c8 = i >> 3;
                    *reinterpret_cast<uint4*>(A + c8 * (kPfM * 16) + (un * kPackTile + r) * 16) = make_uint4(0u, 0u, 0u, 0u);
                }
            }
            fence_proxy_async_smem();  // generic-proxy stores → visible to the tensor core
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&full_a[slot]);
                if (c == 3 || j == nst - 1) mbar_arrive(&raw_empty[rs]);  // done with this super-block's units
            }
        }
        // epilogue: warps 0-3 own TMEM lanes 32·warp .. 32·warp + 31
        if (warp < 4) {
            pdl_wait();  // xexp and the Y rows belong to earlier launches
            if (!*flag && !mbar_wait(accf, 0u, flag)) *flag = 1;
            tc_fence_after();
            if (!*flag) {
                const int row = warp * 32 + lane;
                const int m = m0 + row;
#pragma unroll 1
                for (int c0 = 0; c0 < kPfN; c0 += 16) {
                    float v[16];
                    tc_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
                    if (m < rows) {
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const int n = n0 + c0 + i;
                            if (n < T) Y[(size_t)n * rows + m] = ldexpf(v[i], -xexp[n]);
                        }
                    }
                }
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

// Per-token power-of-two exponent e with max|x|·2^e in [2^14, 2^15) (0 for
// an all-zero row): one warp per token.
__global__ void prefill_xexp_kernel(const float* __restrict__ X, int* __restrict__ xexp, int cols, int T) {
    pdl_launch_dependents();  // the X packing may start launching
    const int n = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (n >= T) return;
    float m = 0.f;
    for (int k = lane * 4; k < cols; k += 128) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(X + (size_t)n * cols + k));
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    m = warp_max(m);
    if (lane == 0) {
        int e = 0;
        if (m > 0.f && isfinite(m)) {
            const int E = (int)((__float_as_uint(m) >> 23) & 0xFF) - 127;  // m in [2^E, 2^(E+1)) (normal m)
            e = max(-120, min(120, 14 - E));
        }
        xexp[n] = e;
    }
}

// X f32 [T][cols] → f16 tiles: for token tile nt and stage s, 16 KiB at
// ((nt·nst + s)·16384) holding [8-value chunk c8][token][8 × f16], the
// K-major no-swizzle layout of one MMA B operand stage; tokens ≥ T are zero.
__global__ void prefill_pack_x_kernel(const float* __restrict__ X, const int* __restrict__ xexp, uint8_t* __restrict__ Xp,
                                      int cols, int T, int ntok) {
    pdl_launch_dependents();  // the GEMM's set-up and first weight copies overlap the packing
    pdl_wait();               // xexp from the previous launch
    const int kc = cols / 8;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)ntok * kc) return;
    const int n = (int)(i / kc), k0 = (int)(i % kc) * 8;
    uint4 o = make_uint4(0u, 0u, 0u, 0u);
    if (n < T) {
        const float* src = X + (size_t)n * cols + k0;
        const float4 a = __ldg(reinterpret_cast<const float4*>(src)), b = __ldg(reinterpret_cast<const float4*>(src) + 1);
        const int e = xexp[n];
        o = make_uint4(h2bits(ldexpf(a.x, e), ldexpf(a.y, e)), h2bits(ldexpf(a.z, e), ldexpf(a.w, e)),
                       h2bits(ldexpf(b.x, e), ldexpf(b.y, e)), h2bits(ldexpf(b.z, e), ldexpf(b.w, e)));
    }
    const int nst = cols / kPfK, s = k0 / kPfK, c8 = (k0 % kPfK) / 8;
    *reinterpret_cast<uint4*>(Xp + ((size_t)(n / kPfN) * nst + s) * kPfPlane + c8 * (kPfN * 16) + (n % kPfN) * 16) = o;
}

// ---- row kernels of the batched prompt pass (one token per row)

// x[t] = dequantised embedding row of token tokens[t] (emb_lookup,
// src/models/llama_model.cpp:882-934).
__global__ void prompt_embed_kernel(float* __restrict__ x, const uint8_t* __restrict__ W, int type, int cols,
                                    int row_stride, const int* __restrict__ tokens) {
    const int t = blockIdx.y;
    const int v = blockIdx.x * blockDim.x + threadIdx.x;
    if (v < cols) x[(size_t)t * cols + v] = embed_value(W, type, cols / 256, row_stride, tokens[t], v);
}

// y[t] = w ⊙ x[t] · 1/sqrt(Σx²/n + eps) (rms_norm_out, src/models/llama_model.cpp:393-419);
// one block per row, warp sums added in a fixed order.
__global__ void rows_rmsnorm_kernel(float* __restrict__ y, const float* __restrict__ x, const float* __restrict__ w,
                                    int n, float eps) {
    __shared__ float red[32];
    const float* xr = x + (size_t)blockIdx.x * n;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss += xr[i] * xr[i];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) tot += red[k];
    const float inv = 1.f / sqrtf(tot / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) y[(size_t)blockIdx.x * n + i] = w[i] * (xr[i] * inv);
}

// y[t][i] += b[i] (add_bias, src/models/llama_model.cpp:1082-1092).
__global__ void rows_bias_kernel(float* __restrict__ y, const float* __restrict__ b, int n, long long count) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) y[i] += b[i % n];
}

// g = silu(g) · u (swiglu, src/models/llama_model.cpp:319-368).
__global__ void rows_swiglu_kernel(float* __restrict__ g, const float* __restrict__ u, long long count) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) {
        const float v = g[i];
        g[i] = (v / (1.f + expf(-v))) * u[i];
    }
}

// x += y (residual adds, src/models/llama_model.cpp:1277, 1324).
__global__ void rows_add_kernel(float* __restrict__ x, const float* __restrict__ y, long long count) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) x[i] += y[i];
}

// ---- causal attention of the batched prompt pass

// Per (token, head row): the Q/K head norm (qwen3 before RoPE, hunyuan after
// it), half-split RoPE at the token's position, and for the K/V heads the
// store of the rotated k and the v row into the layer's cache — the RoPE and
// KV-fill loop of llama_forward_batch (src/models/llama_model.cpp:1387-1408).
// Block (t, r): rows r < H are q heads (rotated in place), r >= H kv heads.
__global__ void prompt_rope_kernel(float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                                   float* __restrict__ kc, float* __restrict__ vc, const float* __restrict__ cos_t,
                                   const float* __restrict__ sin_t, const float* __restrict__ q_norm,
                                   const float* __restrict__ k_norm, int pos0, int H, int KV, int hd, int qk_order,
                                   float eps) {
    __shared__ float row[256];
    __shared__ float red[32];
    const int t = blockIdx.x, r = blockIdx.y, tid = threadIdx.x;
    const int pos = pos0 + t, half = hd / 2, KD = KV * hd;
    const bool isq = r < H;
    const int kvh = r - H;
    const float* src = isq ? q + ((size_t)t * H + r) * hd : k + (size_t)t * KD + (size_t)kvh * hd;
    const float* nw = isq ? q_norm : k_norm;
    for (int i = tid; i < hd; i += blockDim.x) row[i] = src[i];
    __syncthreads();
    // per-head RMSNorm of hd values (rms_norm_avx2 per head): x = w·(x·s)
    auto head_norm = [&]() {
        float ss = 0.f;
        for (int i = tid; i < hd; i += blockDim.x) ss += row[i] * row[i];
        ss = warp_sum(ss);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        __syncthreads();
        float tot = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += red[w];
        const float sc = 1.f / sqrtf(tot / (float)hd + eps);
        __syncthreads();
        for (int i = tid; i < hd; i += blockDim.x) row[i] = nw[i] * (row[i] * sc);
        __syncthreads();
    };
    if (qk_order == 1 && nw) head_norm();
    for (int i = tid; i < half; i += blockDim.x) {
        const float c = cos_t[(size_t)pos * half + i], sn = sin_t[(size_t)pos * half + i];
        const float x0 = row[i], x1 = row[i + half];
        row[i] = x0 * c - x1 * sn;
        row[i + half] = x0 * sn + x1 * c;
    }
    __syncthreads();
    if (qk_order == 2 && nw) head_norm();
    if (isq) {
        float* dst = q + ((size_t)t * H + r) * hd;
        for (int i = tid; i < hd; i += blockDim.x) dst[i] = row[i];
    } else {
        float* kd = kc + (size_t)pos * KD + (size_t)kvh * hd;
        float* vd = vc + (size_t)pos * KD + (size_t)kvh * hd;
        const float* vs = v + (size_t)t * KD + (size_t)kvh * hd;
        for (int i = tid; i < hd; i += blockDim.x) {
            kd[i] = row[i];
            vd[i] = vs[i];
        }
    }
}

constexpr int kPaQ = 16;       // queries per block
constexpr int kPaK = 32;       // key positions per tile
constexpr int kPaThreads = 128;

// Causal attention of T prompt tokens at positions pos0 .. pos0+T-1 for one
// query head and a block of kPaQ tokens: token t attends to cache positions
// 0 .. pos0+t (the reference's per-token loop, llama_model.cpp:1410-1425:
// scores q·k·scale, softmax, Σ p·v), here as an online softmax over tiles of
// kPaK positions (fp32 throughout).  Thread (i = tid / 8, g = tid % 8) holds
// the 4 scores of query i at positions g, g+8, g+16, g+24 of a tile and the
// output columns 32c + 4g .. 32c + 4g + 3 (c = 0 .. HD/32 - 1) of query i.
template <int HD>
__global__ void __launch_bounds__(kPaThreads) prompt_attn_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                                               const float* __restrict__ vc, float* __restrict__ out,
                                                               int T, int pos0, int H, int KV, float scale) {
    constexpr int DPT = HD / 8;
    constexpr int KP = HD + 4;  // padded K rows: the 8 key rows a warp reads at once sit in distinct banks
    __shared__ __align__(16) float Qs[kPaQ][HD];
    __shared__ __align__(16) float Ks[kPaK][KP];
    __shared__ __align__(16) float Vs[kPaK][HD];
    __shared__ float Ps[kPaQ][kPaK];
    const int h = blockIdx.x, qb = blockIdx.y, tid = threadIdx.x;
    const int G = H / KV, kvh = h / G, KD = KV * HD;
    const int i = tid >> 3, g = tid & 7;
    const int t0 = qb * kPaQ;
    const int nq = min(kPaQ, T - t0);
    for (int x = tid; x < kPaQ * HD / 4; x += kPaThreads) {
        const int qi = x / (HD / 4), d = 4 * (x % (HD / 4));
        *reinterpret_cast<float4*>(&Qs[qi][d]) =
            qi < nq ? *reinterpret_cast<const float4*>(q + ((size_t)(t0 + qi) * H + h) * HD + d)
                    : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const int my_pos = pos0 + t0 + min(i, nq - 1);  // last position query i attends to
    const int last = pos0 + t0 + nq - 1;            // the block's last position
    float o[DPT];
#pragma unroll
    for (int e = 0; e < DPT; ++e) o[e] = 0.f;
    float m = -INFINITY, l = 0.f;
    for (int p0 = 0; p0 <= last; p0 += kPaK) {
        __syncthreads();
        for (int x = tid; x < kPaK * HD / 4; x += kPaThreads) {
            const int j = x / (HD / 4), d = 4 * (x % (HD / 4)), p = p0 + j;
            const bool in = p <= last;
            const size_t off = (size_t)p * KD + (size_t)kvh * HD + d;
            const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(&Ks[j][d]) = in ? *reinterpret_cast<const float4*>(kc + off) : z;
            *reinterpret_cast<float4*>(&Vs[j][d]) = in ? *reinterpret_cast<const float4*>(vc + off) : z;
        }
        __syncthreads();
        float sc[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) sc[r] = 0.f;
#pragma unroll 4
        for (int d = 0; d < HD; d += 4) {
            const float4 qv = *reinterpret_cast<const float4*>(&Qs[i][d]);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float4 kv = *reinterpret_cast<const float4*>(&Ks[g + 8 * r][d]);
                sc[r] = fmaf(qv.x, kv.x, sc[r]);
                sc[r] = fmaf(qv.y, kv.y, sc[r]);
                sc[r] = fmaf(qv.z, kv.z, sc[r]);
                sc[r] = fmaf(qv.w, kv.w, sc[r]);
            }
        }
        float tmax = -INFINITY;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int p = p0 + g + 8 * r;
            sc[r] = p <= my_pos ? sc[r] * scale : -INFINITY;
            tmax = fmaxf(tmax, sc[r]);
        }
        // the 8 lanes of query i are consecutive: reduce among them
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
        const float mn = fmaxf(m, tmax);
        const float corr = m == -INFINITY ? 0.f : expf(m - mn);
        float ps = 0.f;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const float pv = sc[r] == -INFINITY ? 0.f : expf(sc[r] - mn);
            Ps[i][g + 8 * r] = pv;
            ps += pv;
        }
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
        l = l * corr + ps;
        m = mn;
        __syncwarp();
#pragma unroll
        for (int e = 0; e < DPT; ++e) o[e] *= corr;
        for (int j = 0; j < kPaK; ++j) {
            const float pj = Ps[i][j];
#pragma unroll
            for (int e = 0; e < DPT; e += 4) {
                // columns 32·(e/4) + 4g .. +3: the 8 lanes of a query read one 128-byte row span
                const float4 vv = *reinterpret_cast<const float4*>(&Vs[j][8 * e + 4 * g]);
                o[e] = fmaf(pj, vv.x, o[e]);
                o[e + 1] = fmaf(pj, vv.y, o[e + 1]);
                o[e + 2] = fmaf(pj, vv.z, o[e + 2]);
                o[e + 3] = fmaf(pj, vv.w, o[e + 3]);
            }
        }
    }
    if (i < nq) {
        const float inv = 1.f / l;
        float* dst = out + ((size_t)(t0 + i) * H + h) * HD;
#pragma unroll
        for (int e = 0; e < DPT; e += 4)
            *reinterpret_cast<float4*>(dst + 8 * e + 4 * g) =
                make_float4(o[e] * inv, o[e + 1] * inv, o[e + 2] * inv, o[e + 3] * inv);
    }
}

// Staging buffers of X, grown on demand (cudaMalloc: not during stream capture).
struct PrefillScratch {
    std::mutex mu;
    int dev = -1;
    uint8_t* xp = nullptr;
    size_t xp_bytes = 0;
    int* xexp = nullptr;
    size_t xexp_n = 0;
};
PrefillScratch g_pf;

}  // namespace

cudaError_t prefill_gemm_launch(float* y, const uint8_t* w, int type, const float* x, int rows, int cols, int T,
                                cudaStream_t st) {
    // a few tokens stream the weights once through the batched GEMV instead
    // (faster below ~32 tokens, and exact integer dots)
    if (bgemv_supported(T)) return bgemv_launch(y, w, type, x, rows, cols, T, st);
    int dev = 0;
    AF_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(g_pf.mu);
    const int ntile = (T + kPfN - 1) / kPfN;
    const size_t xp_bytes = (size_t)ntile * (cols / kPfK) * kPfPlane;
    if (g_pf.dev != dev) {
        AF_CUDA_TRY(cudaFuncSetAttribute(prefill_gemm_kernel<kPfStages>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         pf_smem<kPfStages>()));
        g_pf.dev = dev;
        g_pf.xp = nullptr;  // buffers of another device are not reused (they leak with the process)
        g_pf.xp_bytes = 0;
        g_pf.xexp = nullptr;
        g_pf.xexp_n = 0;
    }
    if (g_pf.xp_bytes < xp_bytes) {
        if (g_pf.xp) AF_CUDA_TRY(cudaFree(g_pf.xp));
        g_pf.xp = nullptr;
        AF_CUDA_TRY(cudaMalloc(&g_pf.xp, xp_bytes));
        g_pf.xp_bytes = xp_bytes;
    }
    if (g_pf.xexp_n < (size_t)T) {
        if (g_pf.xexp) AF_CUDA_TRY(cudaFree(g_pf.xexp));
        g_pf.xexp = nullptr;
        AF_CUDA_TRY(cudaMalloc(&g_pf.xexp, (size_t)T * sizeof(int)));
        g_pf.xexp_n = (size_t)T;
    }
    prefill_xexp_kernel<<<(T + 7) / 8, 256, 0, st>>>(x, g_pf.xexp, cols, T);
    const long long items = (long long)ntile * kPfN * (cols / 8);
    AF_CUDA_TRY(cudaGetLastError());
    // the packing and the GEMM start under programmatic dependent launch:
    // each waits (griddepcontrol.wait) before it reads its predecessor's output
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((items + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    AF_CUDA_TRY(cudaLaunchKernelEx(&cfg, prefill_pack_x_kernel, x, (const int*)g_pf.xexp, g_pf.xp, cols, T,
                                   ntile * kPfN));
    cfg.gridDim = dim3((rows + kPfM - 1) / kPfM, ntile);
    cfg.blockDim = dim3(kPfThreads);
    cfg.dynamicSmemBytes = pf_smem<kPfStages>();
    return cudaLaunchKernelEx(&cfg, prefill_gemm_kernel<kPfStages>, y, w, type, (const uint8_t*)g_pf.xp,
                              (const int*)g_pf.xexp, rows, cols, T);
}

bool prompt_attention_supported(int hd) { return hd == 64 || hd == 128; }

cudaError_t prompt_attention_launch(float* q, const float* k, const float* v, float* kc, float* vc, float* out,
                                   const float* cos_t, const float* sin_t, const float* q_norm, const float* k_norm,
                                   int T, int pos0, int H, int KV, int hd, int qk_order, float eps, cudaStream_t st) {
    if (!prompt_attention_supported(hd)) return cudaErrorNotSupported;
    prompt_rope_kernel<<<dim3(T, H + KV), 128, 0, st>>>(q, k, v, kc, vc, cos_t, sin_t, q_norm, k_norm, pos0, H, KV, hd,
                                                       qk_order, eps);
    AF_CUDA_TRY(cudaGetLastError());
    const dim3 grid(H, (T + kPaQ - 1) / kPaQ);
    const float scale = 1.f / std::sqrt((float)hd);
    if (hd == 64) prompt_attn_kernel<64><<<grid, kPaThreads, 0, st>>>(q, kc, vc, out, T, pos0, H, KV, scale);
    else prompt_attn_kernel<128><<<grid, kPaThreads, 0, st>>>(q, kc, vc, out, T, pos0, H, KV, scale);
    return cudaGetLastError();
}

cudaError_t prompt_embed_launch(float* x, const uint8_t* W, int type, int cols, int row_stride, const int* tokens,
                                int T, cudaStream_t st) {
    prompt_embed_kernel<<<dim3((cols + 255) / 256, T), 256, 0, st>>>(x, W, type, cols, row_stride, tokens);
    return cudaGetLastError();
}

cudaError_t rows_rmsnorm_launch(float* y, const float* x, const float* w, int n, int T, float eps, cudaStream_t st) {
    rows_rmsnorm_kernel<<<T, 256, 0, st>>>(y, x, w, n, eps);
    return cudaGetLastError();
}

cudaError_t rows_bias_launch(float* y, const float* b, int n, int T, cudaStream_t st) {
    const long long count = (long long)n * T;
    rows_bias_kernel<<<(unsigned)((count + 255) / 256), 256, 0, st>>>(y, b, n, count);
    return cudaGetLastError();
}

cudaError_t rows_swiglu_launch(float* g, const float* u, long long count, cudaStream_t st) {
    rows_swiglu_kernel<<<(unsigned)((count + 255) / 256), 256, 0, st>>>(g, u, count);
    return cudaGetLastError();
}

cudaError_t rows_add_launch(float* x, const float* y, long long count, cudaStream_t st) {
    rows_add_kernel<<<(unsigned)((count + 255) / 256), 256, 0, st>>>(x, y, count);
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
