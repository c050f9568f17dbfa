// af_gemv_dev.cuh — device building blocks of the dequant GEMV, shared by the
// standalone GEMV kernel (af_gemv.cu) and the persistent decode-step kernel
// (af_step.cu).  Layouts are described in af_gemv.cuh.
//
// Weight streaming uses a byte ring in shared memory: entry i of a CTA's
// sequence (one fragment × one 8-super-block K stage) is placed at
//     h = head + size > ring_bytes ? 0 : head;   head = h + size
// which the producer thread and the consumer warps both evaluate, so the
// placement needs no communication.  Entry i completes on full[i % kRingDesc]
// (producer expect_tx + bulk copies) and is released on empty[i % kRingDesc]
// (one arrival per consumer warp).  The producer only overwrites bytes whose
// entries have been released, so Q4_K and Q6_K entries of any size share the
// whole ring.
#pragma once
#include "af_gemv.cuh"

namespace af {
namespace gdev {

constexpr int kCW = kGemvConsumerWarps;
constexpr int kCT = kCW * 32;
constexpr int kRingDesc = 8;  // entries in flight at most (a power of two)
static_assert((kRingDesc & (kRingDesc - 1)) == 0, "ring descriptors: power of two");

// Shared-memory header of the GEMV kernels (kGemvSmemHdr bytes).
constexpr int kHdrFlags = 256;    // int[0] abort
constexpr int kFragUnits = 2 * kGemvFragTiles;  // units of a fragment at most (SwiGLU)
constexpr int kHdrRed = 2048;     // [2 buffers][kFragUnits][kCW warps][16 rows] f32
static_assert(kHdrRed + 2 * kFragUnits * kCW * 16 * 4 <= kGemvSmemHdr, "GEMV header overflow");

// Named barrier 1 over the consumer warps only (the producer never joins).
__device__ __forceinline__ void bar_consumers() { asm volatile("bar.sync 1, %0;" ::"n"(kCT) : "memory"); }

// ---------------------------------------------------------------- fragments

// Fragment = up to two consecutive tiles of one segment starting at an even
// tile (32 output rows); SwiGLU: the same tiles of the gate (segment 0) and
// the up (segment 1) matrix, streamed gate tiles first.
struct Frag {
    int seg;    // segment (SwiGLU: 0)
    int tile;   // first tile within the segment (even)
    int nt;     // tiles per part (1 or 2)
    int parts;  // 1, or 2 for SwiGLU (gate, up)
    __device__ int units() const { return nt * parts; }
};

__device__ __forceinline__ int seg_tiles(const GemvSeg& s) { return (s.rows + kPackTile - 1) / kPackTile; }
__device__ __forceinline__ int seg_frags(const GemvSeg& s) { return (seg_tiles(s) + kGemvFragTiles - 1) / kGemvFragTiles; }

// Iterator over fragments [cur, end) of the virtual fragment space: the
// segments' fragments concatenated (SwiGLU: gate/up pairs).
struct FragIter {
    int cur, end;
    __device__ bool next(const GemvParams& p, Frag& t) {
        if (cur >= end) return false;
        const bool sw = p.epi == EPI_SWIGLU;
        int base = 0, s = 0;
        if (!sw) {
            for (; s < p.nseg - 1; ++s) {
                const int n = seg_frags(p.seg[s]);
                if (cur < base + n) break;
                base += n;
            }
        }
        t.seg = s;
        t.tile = (cur - base) * kGemvFragTiles;
        t.nt = min(kGemvFragTiles, seg_tiles(p.seg[s]) - t.tile);
        t.parts = sw ? 2 : 1;
        ++cur;
        return true;
    }
};

// Segment and tile of unit k (0 .. units-1) of a fragment.
__device__ __forceinline__ const GemvSeg& frag_seg(const GemvParams& p, const Frag& t, int k) {
    return p.seg[t.parts == 2 ? k / t.nt : t.seg];
}
__device__ __forceinline__ int frag_tile(const Frag& t, int k) { return t.tile + k % t.nt; }

__device__ __forceinline__ int ring_place(int& head, int size, int ring_bytes) {
    const int h = head + size > ring_bytes ? 0 : head;
    head = h + size;
    return h;
}

struct Ring {
    uint8_t* buf;
    int bytes;
    uint64_t* full;   // [kRingDesc]
    uint64_t* empty;  // [kRingDesc], kCW arrivals
};

// ---------------------------------------------------------------- producer

// Single-thread producer state; persists across the phases of a step.
// Ring space is accounted first-in first-out: `used` counts the bytes (with
// the waste a wrapped placement leaves at the end of the ring) of entries
// issued and not yet released, so making room costs O(1) per released entry.
// The producer thread shares an SM sub-partition with two busy consumer
// warps, so every instruction it spends per entry delays the stream.  The
// size table is indexed with compile-time slots only (registers, not local
// memory).
struct Producer {
    uint32_t issued = 0, released = 0;
    int head = 0;
    int used = 0;
    int size[kRingDesc];

    // Wait (bounded) until entry `released` has been consumed and free its bytes.
    __device__ bool release_oldest(const Ring& r, const volatile int* abort) {
        const uint32_t j = released;
        if (!mbar_wait(&r.empty[j % kRingDesc], (j / kRingDesc) & 1u, abort)) return false;
        int s = 0;
#pragma unroll
        for (int d = 0; d < kRingDesc; ++d)
            if (d == (int)(j % kRingDesc)) s = size[d];
        used -= s;
        ++released;
        return true;
    }

    // Reserve `bytes` at the next placement; false on timeout or abort.
    __device__ bool reserve(const Ring& r, int bytes, int& at, const volatile int* abort) {
        // the placement rule of ring_place: wrap to 0 when the entry does not
        // fit after head (head may sit exactly at the end: waste 0, still wrap)
        const bool wrap = head + bytes > r.bytes;
        const int waste = wrap ? r.bytes - head : 0;
        const int need = bytes + waste;
        while (used + need > r.bytes || issued - released >= (uint32_t)kRingDesc)
            if (!release_oldest(r, abort)) return false;
        at = wrap ? 0 : head;
        head = at + bytes;
        used += need;
        const int slot = issued % kRingDesc;
#pragma unroll
        for (int d = 0; d < kRingDesc; ++d)
            if (d == slot) size[d] = need;
        return true;
    }

    // Stream every (fragment, stage) entry of virtual tiles [vbeg, vend) of p
    // in the order the consumers take them.
    __device__ bool produce(const GemvParams& p, int vbeg, int vend, const Ring& r, volatile int* abort,
                            uint64_t pol) {
        const int nb = p.K / 256, nst = (nb + kGemvStageBlocks - 1) / kGemvStageBlocks;
        FragIter it{vbeg, vend};
        Frag t;
        while (it.next(p, t)) {
            const int ub = unit_bytes(p.seg[t.seg].type);
            for (int st = 0; st < nst; ++st) {
                const int nbs = min(kGemvStageBlocks, nb - st * kGemvStageBlocks);
                const int bytes = t.units() * nbs * ub;
                int at;
                if (*abort || !reserve(r, bytes, at, abort)) return false;
                uint64_t* bar = &r.full[issued % kRingDesc];
                mbar_arrive_expect_tx(bar, (uint32_t)bytes);
                for (int k = 0; k < t.units(); ++k) {
                    const GemvSeg& g = frag_seg(p, t, k);
                    const uint8_t* src = g.w + (size_t)frag_tile(t, k) * kPackTile * g.row_stride +
                                         (size_t)st * kGemvStageBlocks * ub;
                    bulk_g2s(r.buf + at + k * nbs * ub, src, (uint32_t)(nbs * ub), bar, pol);
                }
                ++issued;
            }
        }
        return true;
    }

    // After an abort: wait (bounded) for the copies still in flight so no
    // bulk copy lands in shared memory after the CTA exits.
    __device__ void drain(const Ring& r) {
        for (uint32_t i = released; i < issued; ++i) mbar_wait(&r.full[i % kRingDesc], (i / kRingDesc) & 1u);
    }
};

// ---------------------------------------------------------------- tensor-core units

// d(16×8, s32) += a(16×32, u8) · b(32×8, s8)
__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

// Exact int -> float for |v| < 2^22 on the FMA / ALU pipes (no conversion
// unit): the integer lands in the mantissa of 1.5·2^23.
__device__ __forceinline__ float i2f_small(int v) {
    return __int_as_float(0x4B400000 + v) - 12582912.f;
}

// The lane's share of one super-block of the quantised input, Q4_K form.
// Lane (g, t): B column g = (sub-block slot g/2, plane g%2); it supplies the
// plane's words of sub-blocks g/2 and 4 + g/2.  Its outputs (C slot t of the
// two accumulators) are sub-blocks t and 4 + t.
struct XQ4 {
    uint32_t b[8][2];  // B operands of tiles 0..7 (this lane's word where its column is the tile's, else 0)
    float xs0, xs1;    // xs of sub-blocks t and 4+t (1/16 folded in for odd t: high nibbles)
    float s0, s1;      // Σx of sub-blocks t and 4+t
};
__device__ __forceinline__ XQ4 load_xq4(const uint8_t* xsb, int lane, float s_in) {
    const int g = lane >> 2, t = lane & 3, m = g >> 1;
    const uint32_t* X = reinterpret_cast<const uint32_t*>(xsb + (g & 1) * 256);
    const float* XS = reinterpret_cast<const float*>(xsb + kXqXs);
    const float* S32 = reinterpret_cast<const float*>(xsb + kXqS32);
    XQ4 x;
    const uint32_t a0 = X[8 * m + t], a1 = X[8 * m + 4 + t];
    const uint32_t c0 = X[8 * (m + 4) + t], c1 = X[8 * (m + 4) + 4 + t];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const bool sel = (j & 3) == m;
        x.b[j][0] = sel ? (j < 4 ? a0 : c0) : 0u;
        x.b[j][1] = sel ? (j < 4 ? a1 : c1) : 0u;
    }
    const float f = (t & 1) ? s_in * 0.0625f : s_in;
    x.xs0 = XS[t] * f;
    x.xs1 = XS[4 + t] * f;
    x.s0 = S32[t] * s_in;
    x.s1 = S32[4 + t] * s_in;
    return x;
}

// One Q4_K unit (16 rows × 256 values at u): the lane's contribution to rows
// g and g+8 from its sub-blocks t and 4+t.  Block math of q4k_dot_row
// (src/models/llama_model.cpp:476-504) / get_scale_min_k4 (gemv_q4k_avx2.cpp:34-43).
__device__ __forceinline__ float2 q4_unit(const uint8_t* u, const XQ4& x, int lane) {
    const int g = lane >> 2, t = lane & 3;
    uint4 a[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) a[c] = lds128(u + c * 512 + lane * 16);
    int C0[4] = {0, 0, 0, 0}, C1[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t M = (j & 1) ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
        const uint4 q = a[j >> 1];
        if (j < 4) mma_u8s8(C0, q.x & M, q.y & M, q.z & M, q.w & M, x.b[j][0], x.b[j][1]);
        else mma_u8s8(C1, q.x & M, q.y & M, q.z & M, q.w & M, x.b[j][0], x.b[j][1]);
    }
    const int sh = 8 * t;
    float y[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint4 h = lds128(u + kQ4Hdr + (g + 8 * r) * 16);
        // exact integer dots Σ q·(256·hi + lo) of sub-blocks t and 4+t (|T| < 2^28)
        const float T0 = __int2float_rn(C0[2 * r] * 256 + C0[2 * r + 1]);
        const float T1 = __int2float_rn(C1[2 * r] * 256 + C1[2 * r + 1]);
        const uint32_t w0 = h.y >> sh, w1 = h.z >> sh, w2 = h.w >> sh;
        const float sc0 = __int2float_rn(w0 & 63), m0 = __int2float_rn(w1 & 63);
        const float sc1 = __int2float_rn((w2 & 0xF) | ((w0 >> 2) & 0x30));
        const float m1 = __int2float_rn(((w2 >> 4) & 0xF) | ((w1 >> 2) & 0x30));
        const float d = half_bits_to_float(h.x & 0xFFFFu), dmin = half_bits_to_float(h.x >> 16);
        y[r] = d * fmaf(x.xs0 * sc0, T0, x.xs1 * sc1 * T1) - dmin * fmaf(m0, x.s0, m1 * x.s1);
    }
    return make_float2(y[0], y[1]);
}

// The lane's share of one super-block, Q6_K form: B column g = (16-value
// group slot g/2, plane g%2); slot s of tile pair P is tile 2P + s/2, group
// s%2, so the lane supplies group (g/2)%2 of tiles g/4 + 2i.  Its outputs (C
// slot t of tile pair P) are group 4P + t, in tile 2P + t/2.
struct XQ6 {
    uint32_t w[4];
    float xs[4];   // xs of tile 2P + t/2
    float is32[4]; // 32·Σ(256·hi + lo) of group 4P + t
};
__device__ __forceinline__ XQ6 load_xq6(const uint8_t* xsb, int lane, float s_in) {
    const int g = lane >> 2, t = lane & 3, m = g >> 1;
    const uint32_t* X = reinterpret_cast<const uint32_t*>(xsb + (g & 1) * 256);
    const float* XS = reinterpret_cast<const float*>(xsb + kXqXs);
    const int* I16 = reinterpret_cast<const int*>(xsb + kXqI16);
    XQ6 x;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int j = (m >> 1) + 2 * i;
        x.w[i] = X[8 * j + 4 * (m & 1) + t];
        x.xs[i] = XS[2 * i + (t >> 1)] * s_in;
        x.is32[i] = 32.f * i2f_small(I16[4 * i + t]);
    }
    return x;
}

// One Q6_K unit: value mapping of q6k_row_to_f32 (src/models/llama_model.cpp:560-592),
// w = d·sc·(q − 32).
__device__ __forceinline__ float2 q6_unit(const uint8_t* u, const XQ6& x, int lane) {
    const int g = lane >> 2, t = lane & 3, m = g >> 1;
    uint4 L[4], H[2];
#pragma unroll
    for (int P = 0; P < 4; ++P) L[P] = lds128(u + P * 512 + lane * 16);
#pragma unroll
    for (int Q = 0; Q < 2; ++Q) H[Q] = lds128(u + kQ6Hi + Q * 512 + lane * 16);
    int C[4][4];
#pragma unroll
    for (int P = 0; P < 4; ++P) C[P][0] = C[P][1] = C[P][2] = C[P][3] = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int P = j >> 1, odd = j & 1, Q = j >> 2, s = j & 3;
        const uint32_t l[4] = {L[P].x, L[P].y, L[P].z, L[P].w};
        const uint32_t h[4] = {H[Q].x, H[Q].y, H[Q].z, H[Q].w};
        uint32_t a[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const uint32_t lo = (odd ? (l[e] >> 4) : l[e]) & 0x0F0F0F0Fu;
            const uint32_t hi = s < 3 ? (h[e] << (4 - 2 * s)) & 0x30303030u : (h[e] >> 2) & 0x30303030u;
            a[e] = lo | hi;
        }
        const bool own = (j & 1) == (m >> 1);
        const uint32_t wv = x.w[j >> 1];
        const uint32_t b0 = own && !(m & 1) ? wv : 0u;
        const uint32_t b1 = own && (m & 1) ? wv : 0u;
        mma_u8s8(C[P], a[0], a[1], a[2], a[3], b0, b1);
    }
    float y[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int row = g + 8 * r;
        const uint4 scw = lds128(u + kQ6Sc + row * 16);
        const uint32_t sw[4] = {scw.x, scw.y, scw.z, scw.w};
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(u + kQ6D + 2 * row));
        float acc = 0.f;
#pragma unroll
        for (int P = 0; P < 4; ++P) {
            // Σ (q − 32)·xint, exact in f32 (< 2^24)
            const float T = fmaf(256.f, i2f_small(C[P][2 * r]), i2f_small(C[P][2 * r + 1])) - x.is32[P];
            const float sc = i2f_small((int)(int8_t)((sw[P] >> (8 * t)) & 0xFF));
            acc = fmaf(x.xs[P] * sc, T, acc);
        }
        y[r] = d * acc;
    }
    return make_float2(y[0], y[1]);
}

// ---------------------------------------------------------------- input

// Quantise NIT float4 chunks per thread (chunk j of thread t holds values
// 4·(j·kCT + t) .. +3; chunks at or past nvec are zero) into the shared XQ
// layout, RMS-normalising first (weights w) when NORM.  `red` is kCW floats
// of shared scratch.
template <int NIT, bool NORM>
__device__ __forceinline__ void quantise_f4(float4 (&a)[NIT], const float4 (&w)[NORM ? NIT : 1], int nvec, float eps,
                                            uint8_t* xqs, float* red, bool q8 = false) {
    static_assert(kCT % 8 == 0, "8 consecutive threads own one 32-value group");
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    if (NORM) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < NIT; ++j) ss += a[j].x * a[j].x + a[j].y * a[j].y + a[j].z * a[j].z + a[j].w * a[j].w;
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        bar_consumers();
        float tot = 0.f;
#pragma unroll
        for (int k = 0; k < kCW; ++k) tot += red[k];
        // rms_norm_out (src/models/llama_model.cpp:393-419): 1/sqrt(ss/n + eps)
        const float inv_rms = 1.f / sqrtf(tot / (float)(4 * nvec) + eps);
#pragma unroll
        for (int j = 0; j < NIT; ++j) {
            const float4 wj = w[NORM ? j : 0];
            a[j].x = wj.x * (a[j].x * inv_rms);
            a[j].y = wj.y * (a[j].y * inv_rms);
            a[j].z = wj.z * (a[j].z * inv_rms);
            a[j].w = wj.w * (a[j].w * inv_rms);
        }
    }
#pragma unroll
    for (int j = 0; j < NIT; ++j) {
        const int v = j * kCT + tid;
        float amax = fmaxf(fmaxf(fabsf(a[j].x), fabsf(a[j].y)), fmaxf(fabsf(a[j].z), fabsf(a[j].w)));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));  // 8 threads = 32 values
        // 16-bit grid of ±32639 so that hi = (q + 128) >> 8 stays within int8;
        // q8: the Q8_0 block of the reference (see xq_store32w)
        const float inv = amax > 0.f ? (q8 ? 127.f : 32639.f) / amax : 0.f;
        const int qmax = q8 ? 127 : 32639;
        const float av[4] = {a[j].x, a[j].y, a[j].z, a[j].w};
        uint32_t hw = 0, lw = 0;
        int is = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            int q = __float2int_rn(av[e] * inv);
            q = max(-qmax, min(qmax, q));
            const int hi = q8 ? 0 : (q + 128) >> 8;
            const int lo = q - hi * 256;
            hw |= (uint32_t)(hi & 0xFF) << (8 * e);
            lw |= (uint32_t)(lo & 0xFF) << (8 * e);
            is += q;
        }
        float fs = a[j].x + a[j].y + a[j].z + a[j].w;
        is += __shfl_xor_sync(0xffffffffu, is, 1);
        is += __shfl_xor_sync(0xffffffffu, is, 2);  // 4 threads = 16 values
        fs += __shfl_xor_sync(0xffffffffu, fs, 1);
        fs += __shfl_xor_sync(0xffffffffu, fs, 2);
        fs += __shfl_xor_sync(0xffffffffu, fs, 4);
        if (q8) fs = (amax / 127.f) * (float)(is + __shfl_xor_sync(0xffffffffu, is, 4));
        if (v < nvec) {
            uint8_t* sb = xqs + (v >> 6) * kXqSb;
            const int ko = (4 * v) & 255;
            *reinterpret_cast<uint32_t*>(sb + ko) = hw;
            *reinterpret_cast<uint32_t*>(sb + 256 + ko) = lw;
            if ((tid & 3) == 0) reinterpret_cast<int*>(sb + kXqI16)[ko >> 4] = is;
            if ((tid & 7) == 0) {
                reinterpret_cast<float*>(sb + kXqXs)[ko >> 5] = amax / (q8 ? 127.f : 32639.f);
                reinterpret_cast<float*>(sb + kXqS32)[ko >> 5] = fs;
            }
        }
    }
}

// f32-input prologue: x (+ pending residual, optionally RMS-normalised)
// loaded with all NIT float4 loads per thread in flight (norm weights too),
// then quantised into the shared XQ layout.
template <int NIT, bool NORM>
__device__ __forceinline__ void input_prologue_t(const GemvParams& p, uint8_t* xqs, float* red) {
    const int tid = threadIdx.x;
    const int nvec = p.K / 4;
    float4 a[NIT], w[NORM ? NIT : 1];
#pragma unroll
    for (int j = 0; j < NIT; ++j) {
        const int v = j * kCT + tid;
        const int vc = v < nvec ? v : 0;
        a[j] = __ldcg(reinterpret_cast<const float4*>(p.x) + vc);
        if (p.x_add) {
            const float4 b = __ldcg(reinterpret_cast<const float4*>(p.x_add) + vc);
            a[j].x += b.x;
            a[j].y += b.y;
            a[j].z += b.z;
            a[j].w += b.w;
        }
        if (NORM) w[NORM ? j : 0] = __ldg(reinterpret_cast<const float4*>(p.norm_w) + vc);
        if (v >= nvec) a[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (p.x_store && blockIdx.x == 0) {
#pragma unroll
        for (int j = 0; j < NIT; ++j) {
            const int v = j * kCT + tid;
            if (v < nvec) reinterpret_cast<float4*>(p.x_store)[v] = a[j];
        }
    }
    quantise_f4<NIT, NORM>(a, w, nvec, p.eps, xqs, red, p.q8 != 0);
}

// Quantise the f32 input of p into the shared XQ layout (all consumer warps;
// `red` is kCW floats of shared scratch).  Ends with a consumer barrier.
__device__ __forceinline__ void input_prologue(const GemvParams& p, uint8_t* xqs, float* red) {
    const int nit = (p.K / 4 + kCT - 1) / kCT;
#define AF_PRO(N)                                                       \
    case N:                                                             \
        if (p.norm_w) input_prologue_t<N, true>(p, xqs, red);           \
        else input_prologue_t<N, false>(p, xqs, red);                   \
        break;
    switch (nit) {
        AF_PRO(1) AF_PRO(2) AF_PRO(3) AF_PRO(4) AF_PRO(5) AF_PRO(6)
        AF_PRO(7) AF_PRO(8) AF_PRO(9) AF_PRO(10) AF_PRO(11)
        default:
            if (p.norm_w) input_prologue_t<12, true>(p, xqs, red);
            else input_prologue_t<12, false>(p, xqs, red);
    }
#undef AF_PRO
    bar_consumers();
}

// RMSNorm scale 1/sqrt(Σx²/K + eps) of a quantised input in shared memory,
// from the per-32 sums of squares stored after the layout, added in a fixed
// order (deterministic; every lane returns the same value).
__device__ __forceinline__ float xq_norm_scale(const uint8_t* xqs, int K, float eps) {
    const float* pss = reinterpret_cast<const float*>(xqs + xq_bytes(K));
    float ss = 0.f;
    for (int g = (threadIdx.x & 31); g < K / 32; g += 32) ss += pss[g];
    ss = warp_sum(ss);
    return 1.f / sqrtf(ss / (float)K + eps);
}

// Copy the quantised input (XQ layout, written by other CTAs or an earlier
// kernel) from global memory into shared memory with L2 loads, and return
// the folded RMSNorm scale (1 without a norm).  Ends with a consumer barrier.
__device__ __forceinline__ float load_xq(const GemvParams& p, uint8_t* xqs) {
    const int bytes = p.xq_norm ? xq_norm_bytes(p.K) : xq_bytes(p.K);
    const int n16 = bytes / 16;
    const uint4* src = reinterpret_cast<const uint4*>(p.xq);
    uint4* dst = reinterpret_cast<uint4*>(xqs);
    const int tid = threadIdx.x;
    constexpr int kU = 8;
    for (int i0 = tid; i0 < n16; i0 += kU * kCT) {
        uint4 v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u)
            if (i0 + u * kCT < n16) v[u] = __ldcg(src + i0 + u * kCT);
#pragma unroll
        for (int u = 0; u < kU; ++u)
            if (i0 + u * kCT < n16) dst[i0 + u * kCT] = v[u];
    }
    bar_consumers();
    return p.xq_norm ? xq_norm_scale(xqs, p.K, p.eps) : 1.f;
}

// ---------------------------------------------------------------- consumers

// Consumer warps: evaluate virtual tiles [vbeg, vend) of p from the ring and
// apply the epilogue.  `consumed` / `head` persist across calls (the entry
// sequence of a step spans its phases).  `hdr` is the kernel's shared header.
// Returns false on a timeout or an abort.
__device__ __forceinline__ bool consume(const GemvParams& p, int vbeg, int vend, const Ring& r, uint32_t& consumed,
                                        int& head, const uint8_t* xqs, float s_in, uint8_t* hdr) {
    volatile int* abort = reinterpret_cast<volatile int*>(hdr + kHdrFlags);
    float* red = reinterpret_cast<float*>(hdr + kHdrRed);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = p.K / 256, nst = (nb + kGemvStageBlocks - 1) / kGemvStageBlocks;
    FragIter it{vbeg, vend};
    Frag t;
    bool ok = !*abort;
    float best = -INFINITY;
    uint32_t best_idx = 0;
    int fcount = 0;
    while (ok && it.next(p, t)) {
        const int type = p.seg[t.seg].type;
        const int ub = unit_bytes(type);
        const int nu = t.units();
        const bool sw = t.parts == 2;
        // the epilogue of fragment f is warp f % kCW's (the duty rotates so no
        // warp lags behind the others); lane l owns output row 32·frag + l,
        // i.e. row l%16 of unit l/16 (SwiGLU: of gate unit l/16 and up unit 2 + l/16)
        const bool ew = warp == fcount % kCW;
        const int ek = lane >> 4, er = lane & 15;
        const GemvSeg& eseg = p.seg[t.seg];
        const int erow = (t.tile + ek) * kPackTile + er;
        const bool evalid = ek < t.nt && erow < eseg.rows;
        // loads the epilogue needs, in flight during the stages
        float rpre = 0.f, qw = 1.f;
        if (ew && p.epi == EPI_RESID && evalid) rpre = __ldcg(p.resid + erow);
        if (ew && p.q_norm_w && evalid) qw = __ldg(p.q_norm_w + erow);
        float y[kFragUnits][2];
#pragma unroll
        for (int k = 0; k < kFragUnits; ++k) y[k][0] = y[k][1] = 0.f;
        for (int st = 0; st < nst; ++st) {
            const int nbs = min(kGemvStageBlocks, nb - st * kGemvStageBlocks);
            const int at = ring_place(head, nu * nbs * ub, r.bytes);
            const uint32_t d = consumed % kRingDesc;
            if (lane == 0) ok = mbar_wait(&r.full[d], (consumed / kRingDesc) & 1u, abort);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok || *abort) {
                ok = false;
                break;
            }
            if (warp < nbs) {
                const uint8_t* xsb = xqs + (st * kGemvStageBlocks + warp) * kXqSb;
                const uint8_t* u = r.buf + at + warp * ub;
                if (type == AF_GGML_Q6_K) {
                    const XQ6 x = load_xq6(xsb, lane, s_in);
#pragma unroll
                    for (int k = 0; k < kFragUnits; ++k) {
                        if (k < nu) {
                            const float2 v = q6_unit(u + k * nbs * ub, x, lane);
                            y[k][0] += v.x;
                            y[k][1] += v.y;
                        }
                    }
                } else {
                    const XQ4 x = load_xq4(xsb, lane, s_in);
#pragma unroll
                    for (int k = 0; k < kFragUnits; ++k) {
                        if (k < nu) {
                            const float2 v = q4_unit(u + k * nbs * ub, x, lane);
                            y[k][0] += v.x;
                            y[k][1] += v.y;
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&r.empty[d]);
            ++consumed;
        }
        if (!ok) break;
        // rows g, g+8 of each unit: sum the 4 lanes of a row group, then the
        // 8 warps in a fixed order (deterministic)
        float* rb = red + (fcount & 1) * kFragUnits * kCW * 16;
#pragma unroll
        for (int k = 0; k < kFragUnits; ++k)
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                float v = y[k][rr];
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                if ((lane & 3) == 0 && k < nu) rb[(k * kCW + warp) * 16 + (lane >> 2) + 8 * rr] = v;
            }
        bar_consumers();
        ++fcount;
        if (ew) {
            float v = 0.f, vu = 0.f;
#pragma unroll
            for (int w = 0; w < kCW; ++w) v += rb[(ek * kCW + w) * 16 + er];
            if (sw) {
#pragma unroll
                for (int w = 0; w < kCW; ++w) vu += rb[((t.nt + ek) * kCW + w) * 16 + er];
            }
            float out = 0.f;  // this lane's output value, quantised for the next GEMV
            if (evalid) {
                if (sw) {
                    out = (v / (1.f + expf(-v))) * vu;
                    p.seg[0].y[erow] = out;
                } else if (p.epi == EPI_RESID) {
                    out = rpre + v;
                    p.resid[erow] = out;
                } else {
                    if (eseg.bias) v += eseg.bias[erow];
                    out = v;
                    if (p.xsend_n) {
                        const unsigned long long wv = ((unsigned long long)p.xtag << 32) | __float_as_uint(v);
                        for (int rk = 0; rk < p.xsend_n; ++rk) st_relaxed_sys(p.xsend[rk] + erow, wv);
                    } else {
                        eseg.y[erow] = v;
                    }
                    if (p.epi == EPI_ARGMAX) {
                        // a lane's rows arrive in increasing order; ties keep the lowest index
                        const uint32_t gi = (uint32_t)(p.argmax_base + erow);
                        if (v > best || (v == best && gi < best_idx)) {
                            best = v;
                            best_idx = gi;
                        }
                    }
                }
            }
            // the fragment's 32 rows are one 32-value group of q_out
            if (p.q_out)
                xq_store32w(p.q_out, out, qw, p.q_norm_w != nullptr, p.seg[0].rows, evalid ? erow : -1, p.q8 != 0);
        }
    }
    if (p.epi == EPI_ARGMAX) {
        unsigned long long key = best > -INFINITY ? argmax_key(best, best_idx) : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
            key = other > key ? other : key;
        }
        if (lane == 0 && key) atomicMax(p.argmax, key);
    }
    return ok;
}

}  // namespace gdev
}  // namespace af
