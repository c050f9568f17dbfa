// af_bgemv.cu — batched dequant GEMV: Y[B][rows] = X[B][cols] · dequant(W)ᵀ
// for 2 ≤ B ≤ 32 vectors against ONE pass over a packed Q4_K / Q6_K matrix.
//
// The reference computes several tokens against one weight pass with its
// many-token Q8 tile GEMM (gemm_q4k_q8_avx2_range,
// src/backend/cpu_x86/kernels/gemv_q4k_q8_avx2.cpp:257-346: 4 rows × 8 tokens,
// integer dots per 32-value sub-block, scales applied per sub-block) in
// llama_forward_batch (src/models/llama_model.cpp:1339-1462).  At a handful of
// tokens the work is still HBM-bound (≤ 57 flop per weight byte at B = 16),
// so this kernel is built like the single-vector GEMV, not like the
// tensor-memory GEMM: weights stream once through a shared-memory byte ring
// (cp.async.bulk on the TMA engine, no tensor map, no multicast), and each
// 16-row × 32-value weight fragment is multiplied, still as packed integers,
// by up to 8 tokens at a time with mma.sync (u8 weights × s8 inputs → s32):
//
//  * Tokens are the MMA's N dimension.  The inputs are quantised per token
//    and super-block to a 16-bit grid, x ≈ xs·(256·hi + lo), and the two int8
//    planes are two MMAs, so every accumulator is an exact integer dot
//    Σ q·hi, Σ q·lo of one row, one token and one 32-value sub-block (Q4_K)
//    or 16-value group (Q6_K, one m16n8k16 per group).  The sub-block scales
//    (6-bit Q4_K, int8 Q6_K) are applied in integer arithmetic and summed
//    over the super-block, the min / offset term from per-sub-block input
//    sums Σ(256·hi + lo); f32 only once per super-block:
//    w = d·sc·q − dmin·m (Q4_K), w = d·sc·(q − 32) (Q6_K).
//  * The packed layout (af_gemv.cuh) already holds each lane's A fragment
//    in one 16-byte word per 64 values; the input layout "XB" below is
//    arranged the same way: a lane's B words of one sub-block are one
//    16-byte load.
//  * Work: 8-tile groups (128 rows, one tile per consumer warp) × K
//    super-blocks, as (group, super-block) pairs split evenly over the grid
//    (one or two CTAs per SM).  A CTA streams its pairs as ring entries of
//    up to two super-blocks: the group's weights plus the inputs of all
//    tokens for them.  A group whose K range spans several CTAs is split-K:
//    each CTA writes its slice, and the last slice to arrive (an atomic
//    count, no waiting) adds all slices in slice order — the result does
//    not depend on the arrival order.
//  Every wait is bounded (kSpinLimit); a timeout records kErrMbarTimeout.
#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "af_gemv_dev.cuh"
#include "af_ops.cuh"

namespace af {
namespace {

using namespace gdev;

constexpr int kBgMaxVec = 32;          // tokens per call (4 MMA column octets)
constexpr int kBgGroupTiles = 8;       // tiles per group (one per consumer warp)
constexpr int kBgEntrySb = 2;          // super-blocks per ring entry
constexpr int kBgHdr = 256;            // mbarriers, abort and last-slice flags

// XB: the quantised inputs, per 256-value super-block (xb_sb_bytes):
//   planes [B tokens][512]: values x ≈ xs·(256·hi + lo) on a 16-bit grid
//     whose scale xs is per (token, super-block); sub-block j (32 values) at
//     j·64, lane-group t at +16·t: {hi word t, hi word t+4, lo word t,
//     lo word t+4}, where word w holds values 4w .. 4w+3 (one int8 each);
//   xs   [Bp] f32 (Bp = B rounded up to 8; padding tokens are zero);
//   is32 [8 sub-blocks][Bp] int32: Σ (256·hi + lo) over each sub-block;
//   is16 [16 groups][Bp] int32: the same over each 16-value group.
__host__ __device__ inline int bg_bp(int B) { return (B + 7) & ~7; }
__host__ __device__ inline int xb_sb_bytes(int B) { return B * 512 + 100 * bg_bp(B); }

struct BgemvParams {
    const uint8_t* w;  // packed rows
    float* y;          // [B][rows]
    const uint8_t* xb; // XB layout, K/256 super-blocks
    float* part;       // split-K partial sums [groups][maxs][8 tiles][32 lanes][4·NOCT]
    int* cnt;          // [groups] arrivals of split-K slices (zero between calls)
    int type;
    int rows;
    int K;
    int B;
    int row_stride;
    int ring_bytes;
    int groups;        // 8-tile groups
    int total;         // groups × super-blocks: the work pairs split over the grid
    int maxs;          // CTAs sharing one group at most
};

// CTA c owns work pairs [total·c/grid, total·(c+1)/grid) in (group,
// super-block) order; the CTA owning pair q:
__device__ __forceinline__ int bg_cta_of(long long q, int total) {
    return (int)(((q + 1) * gridDim.x - 1) / total);
}
__device__ __forceinline__ int bg_pair0(int c, int total) { return (int)((long long)total * c / gridDim.x); }

// d(16×8, s32) = a(16×16, u8) · b(16×8, s8)
__device__ __forceinline__ void mma_u8s8_k16(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    c[0] = c[1] = c[2] = c[3] = 0;
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(b0));
}

__device__ __forceinline__ void mma_k32(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    c[0] = c[1] = c[2] = c[3] = 0;
    mma_u8s8(c, a[0], a[1], a[2], a[3], b0, b1);
}

__device__ __forceinline__ int byte_of(uint32_t w, int i) { return (int)((w >> (8 * i)) & 0xFFu); }

// Integer partial sums of one unit for the lane's 4
// C slots per token octet: hi / lo plane dots weighted by the sub-block
// scales, and the min (Q4_K) or offset (Q6_K) term.
template <int NOCT>
struct BgInt {
    int hi[NOCT][4], lo[NOCT][4], m[NOCT][4];
};

// One Q4_K unit (16 rows × 256 values at u) against
// the token octets of one XB super-block (xsb); adds the item's f32 result
// to acc[o][e]: rows g (e < 2) / g + 8, tokens 8o + 2t + (e & 1).
// w = d·sc·q − dmin·m (q4k_dot_row, src/models/llama_model.cpp:476-504;
// scale/min unpacking of get_scale_min_k4, gemv_q4k_avx2.cpp:34-43).
template <int NOCT>
__device__ __forceinline__ void bg_q4(const uint8_t* u, const uint8_t* xsb, int B, int lane,
                                      float (&acc)[NOCT][4]) {
    const int g = lane >> 2, t = lane & 3, Bp = bg_bp(B);
    const uint4 h[2] = {lds128(u + kQ4Hdr + g * 16), lds128(u + kQ4Hdr + (g + 8) * 16)};
    // the 8 six-bit scales / mins of each row, as packed bytes
    uint32_t SC[2][2], MN[2][2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        SC[r][0] = h[r].y & 0x3F3F3F3Fu;
        MN[r][0] = h[r].z & 0x3F3F3F3Fu;
        SC[r][1] = (h[r].w & 0x0F0F0F0Fu) | ((h[r].y >> 2) & 0x30303030u);
        MN[r][1] = ((h[r].w >> 4) & 0x0F0F0F0Fu) | ((h[r].z >> 2) & 0x30303030u);
    }
    const uint8_t* pl = xsb + g * 512 + t * 16;
    const int* is32 = reinterpret_cast<const int*>(xsb + B * 512 + 4 * Bp);
    BgInt<NOCT> I;
#pragma unroll
    for (int o = 0; o < NOCT; ++o)
#pragma unroll
        for (int e = 0; e < 4; ++e) I.hi[o][e] = I.lo[o][e] = I.m[o][e] = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint4 q = lds128(u + (j >> 1) * 512 + lane * 16);
        const uint32_t qq[4] = {q.x, q.y, q.z, q.w};
        uint32_t a[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) a[e] = ((j & 1) ? (qq[e] >> 4) : qq[e]) & 0x0F0F0F0Fu;
        const int sc[2] = {byte_of(SC[0][j >> 2], j & 3), byte_of(SC[1][j >> 2], j & 3)};
        const int mn[2] = {byte_of(MN[0][j >> 2], j & 3), byte_of(MN[1][j >> 2], j & 3)};
#pragma unroll
        for (int o = 0; o < NOCT; ++o) {
            const uint4 hl = 8 * o + g < B ? lds128(pl + o * 8 * 512 + j * 64) : make_uint4(0u, 0u, 0u, 0u);
            int ch[4], cl[4];
            mma_k32(ch, a, hl.x, hl.y);
            mma_k32(cl, a, hl.z, hl.w);
            const int2 is = *reinterpret_cast<const int2*>(is32 + j * Bp + 8 * o + 2 * t);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int r = e >> 1;
                I.hi[o][e] += sc[r] * ch[e];
                I.lo[o][e] += sc[r] * cl[e];
                I.m[o][e] += mn[r] * ((e & 1) ? is.y : is.x);
            }
        }
    }
    const float d[2] = {half_bits_to_float(h[0].x & 0xFFFFu), half_bits_to_float(h[1].x & 0xFFFFu)};
    const float dmin[2] = {half_bits_to_float(h[0].x >> 16), half_bits_to_float(h[1].x >> 16)};
    const float* xs = reinterpret_cast<const float*>(xsb + B * 512);
#pragma unroll
    for (int o = 0; o < NOCT; ++o) {
        const float2 x2 = *reinterpret_cast<const float2*>(xs + 8 * o + 2 * t);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int r = e >> 1;
            const float xv = (e & 1) ? x2.y : x2.x;
            const float T = fmaf(256.f, (float)I.hi[o][e], (float)I.lo[o][e]);
            acc[o][e] = fmaf(d[r] * xv, T, acc[o][e]);
            acc[o][e] = fmaf(-dmin[r] * xv, (float)I.m[o][e], acc[o][e]);
        }
    }
}

// One Q6_K unit (eight 32-value ranges of two 16-value groups each):
// w = d·sc·(q − 32) (q6k_row_to_f32, src/models/llama_model.cpp:560-592).
template <int NOCT>
__device__ __forceinline__ void bg_q6(const uint8_t* u, const uint8_t* xsb, int B, int lane,
                                      float (&acc)[NOCT][4]) {
    const int g = lane >> 2, t = lane & 3, Bp = bg_bp(B);
    const uint4 S0 = lds128(u + kQ6Sc + 16 * g), S1 = lds128(u + kQ6Sc + 16 * (g + 8));
    const uint32_t SW[2][4] = {{S0.x, S0.y, S0.z, S0.w}, {S1.x, S1.y, S1.z, S1.w}};
    const uint8_t* pl = xsb + g * 512 + t * 16;
    const int* is16 = reinterpret_cast<const int*>(xsb + B * 512 + 36 * Bp);
    BgInt<NOCT> I;
#pragma unroll
    for (int o = 0; o < NOCT; ++o)
#pragma unroll
        for (int e = 0; e < 4; ++e) I.hi[o][e] = I.lo[o][e] = I.m[o][e] = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint4 L = lds128(u + (j >> 1) * 512 + lane * 16);
        const uint4 H = lds128(u + kQ6Hi + (j >> 2) * 512 + lane * 16);
        const uint32_t l[4] = {L.x, L.y, L.z, L.w}, hh[4] = {H.x, H.y, H.z, H.w};
        const int s = j & 3;
        uint32_t a[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const uint32_t lo = ((j & 1) ? (l[e] >> 4) : l[e]) & 0x0F0F0F0Fu;
            const uint32_t hi = s < 3 ? (hh[e] << (4 - 2 * s)) & 0x30303030u : (hh[e] >> 2) & 0x30303030u;
            a[e] = lo | hi;
        }
        // int8 scales of groups 2j, 2j + 1 for rows g, g + 8
        int sc[2][2];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int gg = 0; gg < 2; ++gg) sc[r][gg] = (int)(int8_t)byte_of(SW[r][(2 * j + gg) >> 2], (2 * j + gg) & 3);
#pragma unroll
        for (int o = 0; o < NOCT; ++o) {
            const uint4 hl = 8 * o + g < B ? lds128(pl + o * 8 * 512 + j * 64) : make_uint4(0u, 0u, 0u, 0u);
            int ch0[4], cl0[4], ch1[4], cl1[4];
            mma_u8s8_k16(ch0, a[0], a[1], hl.x);
            mma_u8s8_k16(cl0, a[0], a[1], hl.z);
            mma_u8s8_k16(ch1, a[2], a[3], hl.y);
            mma_u8s8_k16(cl1, a[2], a[3], hl.w);
            const int2 i0 = *reinterpret_cast<const int2*>(is16 + (2 * j) * Bp + 8 * o + 2 * t);
            const int2 i1 = *reinterpret_cast<const int2*>(is16 + (2 * j + 1) * Bp + 8 * o + 2 * t);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int r = e >> 1;
                I.hi[o][e] += sc[r][0] * ch0[e] + sc[r][1] * ch1[e];
                I.lo[o][e] += sc[r][0] * cl0[e] + sc[r][1] * cl1[e];
                I.m[o][e] += sc[r][0] * ((e & 1) ? i0.y : i0.x) + sc[r][1] * ((e & 1) ? i1.y : i1.x);
            }
        }
    }
    const float d[2] = {half_bits_to_float(*reinterpret_cast<const uint16_t*>(u + kQ6D + 2 * g)),
                        half_bits_to_float(*reinterpret_cast<const uint16_t*>(u + kQ6D + 2 * (g + 8)))};
    const float* xs = reinterpret_cast<const float*>(xsb + B * 512);
#pragma unroll
    for (int o = 0; o < NOCT; ++o) {
        const float2 x2 = *reinterpret_cast<const float2*>(xs + 8 * o + 2 * t);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int r = e >> 1;
            const float xv = (e & 1) ? x2.y : x2.x;
            // Σ sc·Σ (q − 32)·(256·hi + lo)
            const float T = fmaf(256.f, (float)I.hi[o][e], (float)I.lo[o][e]) - 32.f * (float)I.m[o][e];
            acc[o][e] = fmaf(d[r] * xv, T, acc[o][e]);
        }
    }
}

template <int NOCT, int CTAS>
__global__ void __launch_bounds__(kGemvThreads, CTAS) bgemv_kernel(const __grid_constant__ BgemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    Ring ring;
    ring.full = reinterpret_cast<uint64_t*>(smem);
    ring.empty = ring.full + kRingDesc;
    volatile int* abort = reinterpret_cast<volatile int*>(smem + 2 * kRingDesc * 8);
    volatile int* last = abort + 1;
    ring.buf = smem + kBgHdr;
    ring.bytes = p.ring_bytes;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kRingDesc; ++i) {
            mbar_init(&ring.full[i], 1);
            mbar_init(&ring.empty[i], kCW);
        }
        *abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    const int nsb = p.K / 256;
    const int tiles = (p.rows + kPackTile - 1) / kPackTile;
    const int ub = unit_bytes(p.type);
    const int xsbb = xb_sb_bytes(p.B);
    const int q0 = bg_pair0(blockIdx.x, p.total), q1 = bg_pair0(blockIdx.x + 1, p.total);

    if (warp == kCW) {
        // ---------------- producer: one thread issues every entry
        if (lane != 0) return;
        Producer pr;
        const uint64_t pol_w = policy_evict_first(), pol_x = policy_evict_last();
        for (int q = q0; q < q1;) {
            const int g = q / nsb, s0 = q % nsb, s1 = min(nsb, s0 + (q1 - q));
            const int nt = min(kBgGroupTiles, tiles - g * kBgGroupTiles);
            for (int sb = s0; sb < s1; sb += kBgEntrySb) {
                const int sc = min(kBgEntrySb, s1 - sb);
                const int bytes = nt * sc * ub + sc * xsbb;
                int at;
                if (*abort || !pr.reserve(ring, bytes, at, abort)) {
                    *abort = 1;
                    pr.drain(ring);
                    return;
                }
                uint64_t* bar = &ring.full[pr.issued % kRingDesc];
                mbar_arrive_expect_tx(bar, (uint32_t)bytes);
                for (int k = 0; k < nt; ++k)
                    bulk_g2s(ring.buf + at + k * sc * ub,
                             p.w + (size_t)(g * kBgGroupTiles + k) * kPackTile * p.row_stride + (size_t)sb * ub,
                             (uint32_t)(sc * ub), bar, pol_w);
                bulk_g2s(ring.buf + at + nt * sc * ub, p.xb + (size_t)sb * xsbb, (uint32_t)(sc * xsbb), bar, pol_x);
                ++pr.issued;
            }
            q += s1 - s0;
        }
        return;
    }

    // ---------------- consumer warps: warp w owns tile w of each group
    uint32_t consumed = 0;
    int head = 0;
    bool ok = true;
    const int g_ = lane >> 2, t_ = lane & 3;
    for (int q = q0; q < q1 && ok;) {
        const int g = q / nsb, s0 = q % nsb, s1 = min(nsb, s0 + (q1 - q));
        const int nt = min(kBgGroupTiles, tiles - g * kBgGroupTiles);
        float acc[NOCT][4];
#pragma unroll
        for (int o = 0; o < NOCT; ++o) acc[o][0] = acc[o][1] = acc[o][2] = acc[o][3] = 0.f;
        for (int sb = s0; sb < s1; sb += kBgEntrySb) {
            const int sc = min(kBgEntrySb, s1 - sb);
            const int at = ring_place(head, nt * sc * ub + sc * xsbb, ring.bytes);
            const uint32_t d = consumed % kRingDesc;
            if (lane == 0) ok = mbar_wait(&ring.full[d], (consumed / kRingDesc) & 1u, abort);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok || *abort) {
                ok = false;
                *abort = 1;
                break;
            }
            if (warp < nt) {
                for (int i = 0; i < sc; ++i) {
                    const uint8_t* u = ring.buf + at + (warp * sc + i) * ub;
                    const uint8_t* xsb = ring.buf + at + nt * sc * ub + i * xsbb;
                    if (p.type == AF_GGML_Q6_K) bg_q6<NOCT>(u, xsb, p.B, lane, acc);
                    else bg_q4<NOCT>(u, xsb, p.B, lane, acc);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&ring.empty[d]);
            ++consumed;
        }
        if (!ok) break;
        const int row0 = (g * kBgGroupTiles + warp) * kPackTile;
        if (s0 == 0 && s1 == nsb) {
            // the whole K of this group: store directly
            if (warp < nt) {
#pragma unroll
                for (int o = 0; o < NOCT; ++o)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int row = row0 + g_ + 8 * (e >> 1), tok = 8 * o + 2 * t_ + (e & 1);
                        if (row < p.rows && tok < p.B) p.y[(size_t)tok * p.rows + row] = acc[o][e];
                    }
            }
        } else {
            // split K: write this slice, and the last slice to arrive adds
            // all of them in slice order (deterministic) and stores
            const int c_lo = bg_cta_of((long long)g * nsb, p.total);
            const int c_hi = bg_cta_of((long long)g * nsb + nsb - 1, p.total);
            const int nslice = c_hi - c_lo + 1, slice = (int)blockIdx.x - c_lo;
            float4* pw = reinterpret_cast<float4*>(p.part) +
                         ((((size_t)g * p.maxs + slice) * kBgGroupTiles + warp) * 32 + lane) * NOCT;
            if (warp < nt) {
#pragma unroll
                for (int o = 0; o < NOCT; ++o) pw[o] = make_float4(acc[o][0], acc[o][1], acc[o][2], acc[o][3]);
            }
            __threadfence();
            bar_consumers();
            if (threadIdx.x == 0) *last = atomicAdd(p.cnt + g, 1) == nslice - 1;
            bar_consumers();
            if (*last) {
                __threadfence();
                if (warp < nt) {
                    float v[NOCT][4];
#pragma unroll
                    for (int o = 0; o < NOCT; ++o) v[o][0] = v[o][1] = v[o][2] = v[o][3] = 0.f;
                    for (int i = 0; i < nslice; ++i) {
                        const float4* pr = reinterpret_cast<const float4*>(p.part) +
                                           ((((size_t)g * p.maxs + i) * kBgGroupTiles + warp) * 32 + lane) * NOCT;
#pragma unroll
                        for (int o = 0; o < NOCT; ++o) {
                            const float4 f = __ldcg(pr + o);
                            v[o][0] += f.x;
                            v[o][1] += f.y;
                            v[o][2] += f.z;
                            v[o][3] += f.w;
                        }
                    }
#pragma unroll
                    for (int o = 0; o < NOCT; ++o)
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int row = row0 + g_ + 8 * (e >> 1), tok = 8 * o + 2 * t_ + (e & 1);
                            if (row < p.rows && tok < p.B) p.y[(size_t)tok * p.rows + row] = v[o][e];
                        }
                }
                if (threadIdx.x == 0) p.cnt[g] = 0;  // ready for the next call
            }
        }
        q += s1 - s0;
    }
}

// Quantise X [B][K] f32 into XB: one warp per (token, super-block); lane
// (j = lane / 4, t = lane % 4) owns words t and t + 4 of sub-block j and
// writes its 16-byte plane slot.  Tokens B .. Bp-1 write zero scales and sums.
__global__ void bg_quantize_kernel(uint8_t* __restrict__ xb, const float* __restrict__ x, int K, int B) {
    const int Bp = bg_bp(B), nsb = K / 256;
    const long long wid = (long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (wid >= (long long)Bp * nsb) return;
    const int tok = (int)(wid / nsb), sb = (int)(wid % nsb), lane = threadIdx.x & 31;
    const int j = lane >> 2, t = lane & 3;
    float v[8];
    if (tok < B) {
        const float* src = x + (size_t)tok * K + sb * 256 + 32 * j + 4 * t;
        const float4 a = __ldg(reinterpret_cast<const float4*>(src));
        const float4 b = __ldg(reinterpret_cast<const float4*>(src + 16));
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = warp_max(amax);
    const float inv = amax > 0.f ? 32639.f / amax : 0.f;
    uint32_t hw[2] = {0u, 0u}, lw[2] = {0u, 0u};
    int s16[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int q = max(-32639, min(32639, __float2int_rn(v[i] * inv)));
        const int hi = (q + 128) >> 8, lo = q - 256 * hi;
        hw[i >> 2] |= (uint32_t)(hi & 0xFF) << (8 * (i & 3));
        lw[i >> 2] |= (uint32_t)(lo & 0xFF) << (8 * (i & 3));
        s16[i >> 2] += q;
    }
    // groups 2j (words 0..3) and 2j + 1 (words 4..7) over the 4 lanes of j
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        s16[h] += __shfl_xor_sync(0xffffffffu, s16[h], 1);
        s16[h] += __shfl_xor_sync(0xffffffffu, s16[h], 2);
    }
    uint8_t* base = xb + (size_t)sb * xb_sb_bytes(B);
    if (tok < B) *reinterpret_cast<uint4*>(base + tok * 512 + j * 64 + t * 16) = make_uint4(hw[0], hw[1], lw[0], lw[1]);
    float* xs = reinterpret_cast<float*>(base + B * 512);
    int* is32 = reinterpret_cast<int*>(base + B * 512 + 4 * Bp);
    int* is16 = reinterpret_cast<int*>(base + B * 512 + 36 * Bp);
    if (lane == 0) xs[tok] = amax / 32639.f;
    if (t == 0) {
        is32[j * Bp + tok] = s16[0] + s16[1];
        is16[(2 * j) * Bp + tok] = s16[0];
        is16[(2 * j + 1) * Bp + tok] = s16[1];
    }
}

// Device buffers of the calls, grown on demand (cudaMalloc: not during stream
// capture).  Calls on one device share them: concurrent calls on two
// streams race.
struct BgScratch {
    std::mutex mu;
    int dev = -1;
    uint8_t* xb = nullptr;
    size_t xb_bytes = 0;
    float* part = nullptr;
    size_t part_bytes = 0;
    int* cnt = nullptr;
    size_t cnt_n = 0;
};
BgScratch g_bg;

template <typename T>
cudaError_t bg_grow(T*& ptr, size_t& have, size_t want, bool zero) {
    if (have >= want) return cudaSuccess;
    if (ptr) AF_CUDA_TRY(cudaFree(ptr));
    ptr = nullptr;
    have = 0;
    AF_CUDA_TRY(cudaMalloc(&ptr, want * sizeof(T)));
    if (zero) AF_CUDA_TRY(cudaMemset(ptr, 0, want * sizeof(T)));
    have = want;
    return cudaSuccess;
}

// CTAs per SM: 2 for one token octet (16 consumer warps per SM hide the
// MMA / shared-load latency; the registers fit), else 1;
// AF_BGEMV_CTAS_PER_SM = 1 or 2 overrides for up to two octets.
int bg_ctas_per_sm(int noct) {
    static const int env = [] {
        const char* v = std::getenv("AF_BGEMV_CTAS_PER_SM");
        return v ? std::atoi(v) : 0;
    }();
    if (env == 1 || env == 2) return noct > 2 ? 1 : env;
    return noct == 1 ? 2 : 1;
}

// The host's copy of bg_cta_of.
int host_cta_of(long long q, int total, int grid) { return (int)(((q + 1) * grid - 1) / total); }

template <int NOCT, int CTAS>
cudaError_t bg_launch_t(BgemvParams p, cudaStream_t st) {
    const int smem_total = (CTAS == 1 ? 227 * 1024 : 113 * 1024);
    p.ring_bytes = (smem_total - kBgHdr) & ~15;
    static int attr_dev = -1;  // the attribute is per device; set once
    if (attr_dev != g_bg.dev) {
        AF_CUDA_TRY(cudaFuncSetAttribute(bgemv_kernel<NOCT, CTAS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         smem_total));
        attr_dev = g_bg.dev;
    }
    const int nsb = p.K / 256;
    const int grid = std::min(num_sms() * CTAS, p.total);
    p.maxs = 1;
    for (int g = 0; g < p.groups; ++g)
        p.maxs = std::max(p.maxs, host_cta_of((long long)g * nsb + nsb - 1, p.total, grid) -
                                      host_cta_of((long long)g * nsb, p.total, grid) + 1);
    const size_t part_n = (size_t)p.groups * p.maxs * kBgGroupTiles * 32 * 4 * NOCT;
    AF_CUDA_TRY(bg_grow(g_bg.part, g_bg.part_bytes, part_n, false));
    AF_CUDA_TRY(bg_grow(g_bg.cnt, g_bg.cnt_n, (size_t)p.groups, true));
    p.part = g_bg.part;
    p.cnt = g_bg.cnt;
    bgemv_kernel<NOCT, CTAS><<<grid, kGemvThreads, smem_total, st>>>(p);
    return cudaGetLastError();
}

template <int NOCT>
cudaError_t bg_launch_n(const BgemvParams& p, cudaStream_t st) {
    if (NOCT <= 2 && bg_ctas_per_sm(NOCT) == 2) return bg_launch_t<NOCT, 2>(p, st);
    return bg_launch_t<NOCT, 1>(p, st);
}

}  // namespace

bool bgemv_supported(int n_vec) { return n_vec >= 1 && n_vec <= kBgMaxVec; }

cudaError_t bgemv_launch(float* y, const uint8_t* w, int type, const float* x, int rows, int cols, int B,
                         cudaStream_t st) {
    int dev = 0;
    AF_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(g_bg.mu);
    if (g_bg.dev != dev) {
        // buffers of another device are not reused (they leak with the process)
        g_bg.dev = dev;
        g_bg.xb = nullptr;
        g_bg.xb_bytes = 0;
        g_bg.part = nullptr;
        g_bg.part_bytes = 0;
        g_bg.cnt = nullptr;
        g_bg.cnt_n = 0;
    }
    AF_CUDA_TRY(bg_grow(g_bg.xb, g_bg.xb_bytes, (size_t)(cols / 256) * xb_sb_bytes(B), false));
    const long long warps = (long long)bg_bp(B) * (cols / 256);
    bg_quantize_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(g_bg.xb, x, cols, B);
    AF_CUDA_TRY(cudaGetLastError());
    BgemvParams p = {};
    p.w = w;
    p.y = y;
    p.xb = g_bg.xb;
    p.type = type;
    p.rows = rows;
    p.K = cols;
    p.B = B;
    p.row_stride = dev_row_stride(type, cols);
    const int tiles = (rows + kPackTile - 1) / kPackTile;
    p.groups = (tiles + kBgGroupTiles - 1) / kBgGroupTiles;
    p.total = p.groups * (cols / 256);
    switch (bg_bp(B) / 8) {
        case 1: return bg_launch_n<1>(p, st);
        case 2: return bg_launch_n<2>(p, st);
        case 3: return bg_launch_n<3>(p, st);
        default: return bg_launch_n<4>(p, st);
    }
}

}  // namespace af

using namespace af;

extern "C" cudaError_t af_gemv_batched_f32(float* d_y, const void* d_w, int ggml_type, const float* d_x, int rows,
                                           int cols, int n_vec, cudaStream_t stream) {
    if ((ggml_type != AF_GGML_Q4_K && ggml_type != AF_GGML_Q6_K) || cols <= 0 || cols % 256 || rows < 0 ||
        !bgemv_supported(n_vec)) {
        set_last_error("af_gemv_batched_f32: need Q4_K/Q6_K weights, cols % 256 == 0, rows >= 0, 1 <= n_vec <= 32");
        return cudaErrorInvalidValue;
    }
    if ((reinterpret_cast<uintptr_t>(d_w) & 15) || (reinterpret_cast<uintptr_t>(d_x) & 15)) {
        set_last_error("af_gemv_batched_f32: weights and x must be 16-byte aligned");
        return cudaErrorInvalidValue;
    }
    if (rows == 0) return cudaSuccess;
    return bgemv_launch(d_y, static_cast<const uint8_t*>(d_w), ggml_type, d_x, rows, cols, n_vec, stream);
}
