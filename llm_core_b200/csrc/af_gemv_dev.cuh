// af_gemv_dev.cuh — device building blocks of the dequant GEMV, shared by the
// standalone GEMV kernel (af_gemv.cu) and the persistent decode-step kernel
// (af_step.cu).
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
constexpr int kRingDesc = 8;  // entries in flight at most

// Named barrier 1 over the consumer warps only (the producer never joins).
__device__ __forceinline__ void bar_consumers() { asm volatile("bar.sync 1, %0;" ::"n"(kCT) : "memory"); }

struct Frag {
    int seg;   // segment of the fragment's rows
    int row0;  // first row within the segment (virtual row for SwiGLU pairs)
    int n;     // rows (row pairs for SwiGLU)
};

__device__ __forceinline__ int n_vsegs(const GemvParams& p) { return p.epi == EPI_SWIGLU ? 1 : p.nseg; }

// Fragment iterator over [cur, end) of the concatenated virtual-row space.
struct FragIter {
    int cur, end;
    __device__ bool next(const GemvParams& p, Frag& t) {
        if (cur >= end) return false;
        int base = 0, s = 0;
        const int ns = n_vsegs(p);
        for (; s < ns - 1; ++s) {
            if (cur < base + p.seg[s].rows) break;
            base += p.seg[s].rows;
        }
        const int cap = p.epi == EPI_SWIGLU ? kGemvFragRows / 2 : kGemvFragRows;
        const int stop = min(min(cur + cap, end), base + p.seg[s].rows);
        t.seg = s;
        t.row0 = cur - base;
        t.n = stop - cur;
        cur = stop;
        return true;
    }
};

// Bytes of one row's segment for a stage of nbs super-blocks: Q4_K nbs*144;
// Q6_K nbs*208 + 16 (the group's d values).  Both are multiples of 16.
__device__ __forceinline__ uint32_t stage_seg_bytes(int type, int nbs) {
    return type == AF_GGML_Q6_K ? (uint32_t)nbs * 208u + 16u : (uint32_t)nbs * 144u;
}

// Address of row `row`, stage st in the packed (tile-major) layout: tile
// t = row / 16 occupies 16 * row_stride bytes; inside it stage st starts at
// 16 * st * full_seg and row i of the tile at i * seg(st).
__device__ __forceinline__ const uint8_t* packed_stage_ptr(const GemvSeg& g, int row, int st, uint32_t seg) {
    const uint32_t full = g.type == AF_GGML_Q6_K ? 1680u : 1152u;
    return g.w + (size_t)(row / kPackTile) * kPackTile * g.row_stride + (size_t)kPackTile * st * full +
           (size_t)(row % kPackTile) * seg;
}

// Copy rows [row0, row0 + n) of one segment's stage st into smem (dense,
// seg bytes per row): one bulk copy per packed tile the rows touch.
__device__ __forceinline__ void copy_rows(uint8_t* dst, const GemvSeg& g, int row0, int n, int st, uint32_t seg,
                                          uint64_t* bar, uint64_t pol) {
    int r = row0;
    while (r < row0 + n) {
        const int stop = min(row0 + n, (r / kPackTile + 1) * kPackTile);
        bulk_g2s(dst + (size_t)(r - row0) * seg, packed_stage_ptr(g, r, st, seg), (uint32_t)(stop - r) * seg, bar,
                 pol);
        r = stop;
    }
}

// Type of the rows a fragment streams (SwiGLU: gate and up share a type).
__device__ __forceinline__ int frag_type(const GemvParams& p, const Frag& t) {
    return p.seg[p.epi == EPI_SWIGLU ? 0 : t.seg].type;
}

// Ring bytes of one entry: (fragment t, stage of nbs super-blocks).  SwiGLU
// entries hold the gate rows then the up rows.
__device__ __forceinline__ int entry_bytes(const GemvParams& p, const Frag& t, int nbs) {
    return (p.epi == EPI_SWIGLU ? 2 : 1) * t.n * (int)stage_seg_bytes(frag_type(p, t), nbs);
}

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
struct Producer {
    uint32_t issued = 0, released = 0;
    int head = 0;
    int off[kRingDesc];
    int size[kRingDesc];

    // Wait (bounded) until entry `released` has been consumed.
    __device__ bool release_oldest(const Ring& r, const volatile int* abort) {
        const uint32_t j = released;
        if (!mbar_wait(&r.empty[j % kRingDesc], (j / kRingDesc) & 1u, abort)) return false;
        ++released;
        return true;
    }

    // Reserve `bytes` at the next placement; false on timeout.
    __device__ bool reserve(const Ring& r, int bytes, int& at, const volatile int* abort) {
        int h = head;
        at = ring_place(h, bytes, r.bytes);
        for (;;) {
            if (issued == released) break;
            bool clash = issued - released >= (uint32_t)kRingDesc;
            for (uint32_t i = released; !clash && i < issued; ++i) {
                const int o = off[i % kRingDesc], s = size[i % kRingDesc];
                clash = at < o + s && o < at + bytes;
            }
            if (!clash) break;
            if (!release_oldest(r, abort)) return false;
        }
        head = h;
        off[issued % kRingDesc] = at;
        size[issued % kRingDesc] = bytes;
        return true;
    }

    // Stream every (fragment, stage) entry of rows [vbeg, vend) of p, in the
    // order the consumers take them: fragment pairs, stage-major inside a pair.
    __device__ bool produce(const GemvParams& p, int vbeg, int vend, const Ring& r, volatile int* abort,
                            uint64_t pol) {
        const int nb = p.K / 256, nst = (nb + 7) / 8;
        FragIter it{vbeg, vend};
        Frag fr[2];
        while (it.next(p, fr[0])) {
            const int nf = it.next(p, fr[1]) ? 2 : 1;
            for (int st = 0; st < nst; ++st) {
                const int nbs = min(8, nb - st * 8);
                for (int f = 0; f < nf; ++f) {
                    const Frag& t = fr[f];
                    const int bytes = entry_bytes(p, t, nbs);
                    int at;
                    if (*abort || !reserve(r, bytes, at, abort)) return false;
                    uint64_t* bar = &r.full[issued % kRingDesc];
                    const GemvSeg& g0 = p.seg[p.epi == EPI_SWIGLU ? 0 : t.seg];
                    const uint32_t segb = stage_seg_bytes(g0.type, nbs);
                    mbar_arrive_expect_tx(bar, (uint32_t)bytes);
                    copy_rows(r.buf + at, g0, t.row0, t.n, st, segb, bar, pol);
                    if (p.epi == EPI_SWIGLU) copy_rows(r.buf + at + t.n * segb, p.seg[1], t.row0, t.n, st, segb, bar, pol);
                    ++issued;
                }
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

// ---------------------------------------------------------------- consumers

struct XRegs {
    uint4 h[4], l[4];
    float xs;
    float s32[2];
    int is16[4];
};

// Dot of one Q4_K (block b, chunk c) with the lane's x registers.
// Block: [d f16][dmin f16][scales 12][qs 128] (gemv_q4k_avx2.cpp:6-15).
__device__ __forceinline__ float q4k_lane_dot(const uint8_t* blk, int c, const XRegs& x) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
    const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16 + 32 * c);
    const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32 + 32 * c);
    const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const int* xh0 = reinterpret_cast<const int*>(&x.h[0]);
    const int* xl0 = reinterpret_cast<const int*>(&x.l[0]);
    // two interleaved accumulator sets (even / odd words) halve the dp4a chains
    int lh[2] = {0, 0}, ll[2] = {0, 0}, hh[2] = {0, 0}, hl[2] = {0, 0};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        // words 0-3: qs bytes 0-15 of the chunk -> x chunk 0 (lo) / 2 (hi);
        // words 4-7: bytes 16-31 -> x chunk 1 (lo) / 3 (hi).
        const uint32_t lo = qw[k] & 0x0F0F0F0Fu;
        const uint32_t hi = qw[k] & 0xF0F0F0F0u;  // 16 x high nibble
        const int e = k & 1;
        lh[e] = dp4a_us(lo, xh0[k], lh[e]);
        ll[e] = dp4a_us(lo, xl0[k], ll[e]);
        hh[e] = dp4a_us(hi, xh0[8 + k], hh[e]);
        hl[e] = dp4a_us(hi, xl0[8 + k], hl[e]);
    }
    const int tlo = (lh[0] + lh[1]) * 256 + (ll[0] + ll[1]);
    const int thi = ((hh[0] + hh[1]) * 256 + (hl[0] + hl[1])) >> 4;  // exact: every term is a multiple of 16
    // 6-bit scale/min pairs j = 2c (low nibbles) and 2c+1 (high nibbles):
    // get_scale_min_k4 (gemv_q4k_avx2.cpp:34-43) four bytes at a time.
    const uint32_t w0 = hdr.y, w1 = hdr.z, w2 = hdr.w;
    // branch-free: c is per lane, so a branch would diverge within the warp
    const bool upper = c >= 2;
    const uint32_t S = upper ? ((w2 & 0x0F0F0F0Fu) | ((w0 >> 2) & 0x30303030u)) : (w0 & 0x3F3F3F3Fu);
    const uint32_t M = upper ? (((w2 >> 4) & 0x0F0F0F0Fu) | ((w1 >> 2) & 0x30303030u)) : (w1 & 0x3F3F3F3Fu);
    const int sh = (c & 1) * 16;
    const int sc_lo = (S >> sh) & 0xFF, sc_hi = (S >> (sh + 8)) & 0xFF;
    const int m_lo = (M >> sh) & 0xFF, m_hi = (M >> (sh + 8)) & 0xFF;
    const float d = half_bits_to_float(hdr.x & 0xFFFFu);
    const float dmin = half_bits_to_float(hdr.x >> 16);
    const int T = sc_lo * tlo + sc_hi * thi;
    return (d * x.xs) * (float)T - dmin * ((float)m_lo * x.s32[0] + (float)m_hi * x.s32[1]);
}

// Dot of one Q6_K (block b, chunk c = 2n+u) with the lane's x registers.
// Regrouped block: [ql 128][qh 64][scales 16] (+ d in the group's d area);
// value mapping of q6k_row_to_f32 (src/models/llama_model.cpp:560-592).
__device__ __forceinline__ float q6k_lane_dot(const uint8_t* blk, float d, int c, const XRegs& x) {
    const int n = c >> 1, u = c & 1;
    const uint4 a0 = *reinterpret_cast<const uint4*>(blk + 64 * n);
    const uint4 a1 = *reinterpret_cast<const uint4*>(blk + 64 * n + 16);
    const uint4 b0 = *reinterpret_cast<const uint4*>(blk + 64 * n + 32);
    const uint4 b1 = *reinterpret_cast<const uint4*>(blk + 64 * n + 48);
    const uint4 h0 = *reinterpret_cast<const uint4*>(blk + 128 + 32 * n);
    const uint4 h1 = *reinterpret_cast<const uint4*>(blk + 128 + 32 * n + 16);
    const uint32_t scw = *reinterpret_cast<const uint32_t*>(blk + 192 + 4 * c);
    const uint32_t A[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const uint32_t B[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    const uint32_t H[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    const int* xh = reinterpret_cast<const int*>(&x.h[0]);
    const int* xl = reinterpret_cast<const int*>(&x.l[0]);
    const int s4 = 4 * u;
    int gh[4] = {0, 0, 0, 0}, gl[4] = {0, 0, 0, 0};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint32_t h = H[k] >> s4;
        // first stream (x local 0..31): ql[l] nibble u, qh bits 4u..4u+1
        const uint32_t q1 = ((A[k] >> s4) & 0x0F0F0F0Fu) | ((h << 4) & 0x30303030u);
        // second stream (x local 32..63): ql[l+32] nibble u, qh bits 4u+2..4u+3
        const uint32_t q2 = ((B[k] >> s4) & 0x0F0F0F0Fu) | ((h << 2) & 0x30303030u);
        const int g1 = k >> 2;        // group 0 or 1 (16 values each)
        const int g2 = 2 + (k >> 2);  // group 2 or 3
        gh[g1] = dp4a_us(q1, xh[k], gh[g1]);
        gl[g1] = dp4a_us(q1, xl[k], gl[g1]);
        gh[g2] = dp4a_us(q2, xh[8 + k], gh[g2]);
        gl[g2] = dp4a_us(q2, xl[8 + k], gl[g2]);
    }
    float acc = 0.f;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const int t = gh[g] * 256 + gl[g] - 32 * x.is16[g];  // Σ (q − 32)·xint
        const float sc = (float)(int8_t)((scw >> (8 * g)) & 0xFF);
        acc = fmaf(sc, (float)t, acc);
    }
    return (d * x.xs) * acc;
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
    constexpr int kU = 4;
    for (int i0 = tid; i0 < n16; i0 += kU * kCT) {
        uint4 v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u)
            if (i0 + u * kCT < n16) v[u] = __ldcg(src + i0 + u * kCT);
#pragma unroll
        for (int u = 0; u < kU; ++u)
            if (i0 + u * kCT < n16) dst[i0 + u * kCT] = v[u];
    }
    if (bytes % 16) {  // K/16 tail of the norm sums (K multiple of 256: never)
        for (int i = n16 * 16 + tid; i < bytes; i += kCT) xqs[i] = p.xq[i];
    }
    bar_consumers();
    float s_in = 1.f;
    if (p.xq_norm) {
        // s = 1/sqrt(Σx²/K + eps) from the producers' per-group sums, in a
        // fixed order (deterministic)
        const float* pss = reinterpret_cast<const float*>(xqs + xq_bytes(p.K));
        float ss = 0.f;
        for (int g = (tid & 31); g < p.K / 64; g += 32) ss += pss[g];
        ss = warp_sum(ss);
        s_in = 1.f / sqrtf(ss / (float)p.K + p.eps);
    }
    return s_in;
}

// Consumer warps: evaluate rows [vbeg, vend) of p from the ring, apply the
// epilogue.  `consumed` / `head` persist across calls (the entry sequence of
// a step spans its phases).  Returns false on a timeout or an abort.
__device__ __forceinline__ bool consume(const GemvParams& p, int vbeg, int vend, const Ring& r, uint32_t& consumed,
                                        int& head, const uint8_t* xqs, float s_in, volatile int* abort) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = p.K / 256, nst = (nb + 7) / 8;
    const uint8_t* XH = xqs;
    const uint8_t* XL = xqs + nst * 2048;
    const float* XS = reinterpret_cast<const float*>(xqs + 2 * nst * 2048);
    const float* XS32 = XS + nst * 32;
    const int* XI16 = reinterpret_cast<const int*>(XS32 + nst * 64);
    const int lb = lane >> 2, lc = lane & 3;
    FragIter it{vbeg, vend};
    Frag fr[2];
    bool ok = !*abort;
    float best = -INFINITY;
    uint32_t best_idx = 0;
    const int half = kGemvFragRows / 2;
    while (ok && it.next(p, fr[0])) {
        const int nf = it.next(p, fr[1]) ? 2 : 1;
        // rows of this warp: (fragment f, r) -> entry row warp + r*half
        // (SwiGLU: gate row warp, up row n + warp)
        float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
        bool rv[2][2];
        int row[2][2];
        int ty[2];
        for (int f = 0; f < 2; ++f) {
            const Frag& t = fr[f];
            const bool have = f < nf;
            if (p.epi == EPI_SWIGLU) {
                rv[f][0] = rv[f][1] = have && warp < t.n;
                row[f][0] = row[f][1] = t.row0 + warp;
                ty[f] = p.seg[0].type;
            } else {
                rv[f][0] = have && warp < t.n;
                rv[f][1] = have && warp + half < t.n;
                row[f][0] = t.row0 + warp;
                row[f][1] = t.row0 + warp + half;
                ty[f] = have ? p.seg[t.seg].type : p.seg[fr[0].seg].type;
            }
        }
        for (int st = 0; st < nst; ++st) {
            const int nbs = min(8, nb - st * 8);
            const uint32_t d0 = consumed % kRingDesc, d1 = (consumed + 1) % kRingDesc;
            const int at0 = ring_place(head, entry_bytes(p, fr[0], nbs), r.bytes);
            const int at1 = nf == 2 ? ring_place(head, entry_bytes(p, fr[1], nbs), r.bytes) : at0;
            if (lane == 0) {
                ok = mbar_wait(&r.full[d0], (consumed / kRingDesc) & 1u, abort);
                if (ok && nf == 2) ok = mbar_wait(&r.full[d1], ((consumed + 1) / kRingDesc) & 1u, abort);
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok || *abort) { ok = false; break; }
            // a fragment cut short at a segment end may precede a full one
            if (lb < nbs && (rv[0][0] || rv[1][0])) {
                XRegs x;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    x.h[i] = *reinterpret_cast<const uint4*>(XH + st * 2048 + i * 512 + lane * 16);
                    x.l[i] = *reinterpret_cast<const uint4*>(XL + st * 2048 + i * 512 + lane * 16);
                    x.is16[i] = XI16[st * 128 + i * 32 + lane];
                }
                x.xs = XS[st * 32 + lane] * s_in;
                x.s32[0] = XS32[st * 64 + lane] * s_in;
                x.s32[1] = XS32[st * 64 + 32 + lane] * s_in;
                // Up to four rows evaluated without branches so their dp4a
                // chains interleave.  Entries are packed end to end in the
                // ring, so a row past a fragment's end could lie past the ring
                // (and the shared allocation): an invalid row re-reads a valid
                // row of the same type instead, and its result is discarded.
                const uint8_t* rp[2][2];
#pragma unroll
                for (int f = 0; f < 2; ++f) {
                    const uint32_t segb = stage_seg_bytes(ty[f], nbs);
                    const uint8_t* row0 = r.buf + (f ? at1 : at0);
                    const uint8_t* own = row0 + warp * segb;
                    const uint8_t* safe = rv[f][0] ? own : row0;  // row 0 of an entry always exists
                    rp[f][0] = safe;
                    rp[f][1] = rv[f][1] ? own + (p.epi == EPI_SWIGLU ? fr[f].n : half) * segb : safe;
                }
                if (nf == 2 && ty[0] == ty[1]) {
                    if (ty[0] == AF_GGML_Q6_K) {
                        float d[4], a[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            d[k] = half_bits_to_float(
                                *reinterpret_cast<const uint16_t*>(rp[k >> 1][k & 1] + nbs * 208 + 2 * lb));
#pragma unroll
                        for (int k = 0; k < 4; ++k) a[k] = q6k_lane_dot(rp[k >> 1][k & 1] + lb * 208, d[k], lc, x);
#pragma unroll
                        for (int k = 0; k < 4; ++k) acc[k >> 1][k & 1] += a[k];
                    } else {
                        float a[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k) a[k] = q4k_lane_dot(rp[k >> 1][k & 1] + lb * 144, lc, x);
#pragma unroll
                        for (int k = 0; k < 4; ++k) acc[k >> 1][k & 1] += a[k];
                    }
                } else {
                    for (int f = 0; f < nf; ++f) {
                        if (ty[f] == AF_GGML_Q6_K) {
                            const float e0 = half_bits_to_float(
                                *reinterpret_cast<const uint16_t*>(rp[f][0] + nbs * 208 + 2 * lb));
                            const float e1 = half_bits_to_float(
                                *reinterpret_cast<const uint16_t*>(rp[f][1] + nbs * 208 + 2 * lb));
                            const float a0 = q6k_lane_dot(rp[f][0] + lb * 208, e0, lc, x);
                            const float a1 = q6k_lane_dot(rp[f][1] + lb * 208, e1, lc, x);
                            acc[f][0] += a0;
                            acc[f][1] += a1;
                        } else {
                            const float a0 = q4k_lane_dot(rp[f][0] + lb * 144, lc, x);
                            const float a1 = q4k_lane_dot(rp[f][1] + lb * 144, lc, x);
                            acc[f][0] += a0;
                            acc[f][1] += a1;
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&r.empty[d0]);
                if (nf == 2) mbar_arrive(&r.empty[d1]);
            }
            consumed += nf;
        }
        if (!ok) break;
        for (int f = 0; f < nf; ++f) {
            acc[f][0] = warp_sum(acc[f][0]);
            acc[f][1] = warp_sum(acc[f][1]);
            if (lane != 0) continue;
            if (p.epi == EPI_SWIGLU) {
                if (rv[f][0]) {
                    const float g = acc[f][0], u = acc[f][1];
                    p.seg[0].y[row[f][0]] = (g / (1.f + expf(-g))) * u;
                }
                continue;
            }
            const GemvSeg& sg = p.seg[fr[f].seg];
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                if (!rv[f][rr]) continue;
                float v = acc[f][rr];
                if (p.epi == EPI_RESID) {
                    p.resid[row[f][rr]] = __ldcg(p.resid + row[f][rr]) + v;
                } else {
                    if (sg.bias) v += sg.bias[row[f][rr]];
                    sg.y[row[f][rr]] = v;
                    if (p.epi == EPI_ARGMAX) {
                        // rows reach a lane in increasing order; ties keep the lowest index
                        const uint32_t gi = (uint32_t)(p.argmax_base + row[f][rr]);
                        if (v > best || (v == best && gi < best_idx)) {
                            best = v;
                            best_idx = gi;
                        }
                    }
                }
            }
        }
    }
    if (p.epi == EPI_ARGMAX && lane == 0 && best > -INFINITY) atomicMax(p.argmax, argmax_key(best, best_idx));
    return ok;
}

// After the epilogue stores of rows [vbeg, vend): every 64-row output group
// this CTA completes (per-group arrival counters) is quantised into q_out for
// the next GEMV.  Consumer warps only; `list` is shared scratch of at least
// (vend − vbeg) / 64 + 3 ints.
__device__ __forceinline__ void quantise_output(const GemvParams& p, int vbeg, int vend, int* list) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    bar_consumers();  // every epilogue store of this CTA is done
    if (threadIdx.x == 0) {
        __threadfence();
        int n = 0;
        for (int g = vbeg / 64; g * 64 < vend; ++g) {
            const int lo = max(vbeg, g * 64), hi = min(vend, g * 64 + 64);
            const unsigned int prev = atomicAdd(&p.q_cnt[g], (unsigned int)(hi - lo));
            if (prev + (unsigned int)(hi - lo) == 64u) list[++n] = g;
        }
        list[0] = n;
        __threadfence();
    }
    bar_consumers();
    const int n = list[0];
    const float* src = p.epi == EPI_RESID ? p.resid : p.seg[0].y;
    const int Kout = p.seg[0].rows;
    for (int k = warp; k < n; k += kCW) {
        const int g = list[1 + k];
        xq_quantize_group(p.q_out, src, p.q_norm_w, Kout, g);
        if (lane == 0) p.q_cnt[g] = 0u;
    }
}

}  // namespace gdev
}  // namespace af
