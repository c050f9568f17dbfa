// af_gemv.cu — fused dequant GEMV kernel (see af_gemv.cuh for the design).
#include "af_gemv.cuh"

namespace af {

__device__ int g_err = 0;

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
// float4 registers per consumer thread for the input: K <= 256*12*4 = 12288.
constexpr int kPrologueVec = kGemvMaxK / (kConsumerThreads * 4);

struct Tile {
    int seg;     // segment of the tile's rows
    int row0;    // first row within the segment (virtual row for SwiGLU pairs)
    int n;       // rows in the tile (row pairs for SwiGLU)
};

// Rows of a segment as seen by the CTA partition ("virtual rows": a SwiGLU
// gate/up pair counts as one).
__device__ __forceinline__ int n_vsegs(const GemvParams& p) { return p.epi == EPI_SWIGLU ? 1 : p.nseg; }

__device__ __forceinline__ long long vrow_bytes(const GemvParams& p, int s) {
    if (p.epi == EPI_SWIGLU) return (long long)p.seg[0].row_stride + p.seg[1].row_stride;
    return p.seg[s].row_stride;
}

// First virtual row whose starting byte is >= b.
__device__ long long vrow_at(const GemvParams& p, long long b) {
    long long base = 0;
    const int ns = n_vsegs(p);
    for (int s = 0; s < ns; ++s) {
        const long long rb = vrow_bytes(p, s);
        const long long segb = rb * p.seg[s].rows;
        if (b <= segb || s == ns - 1) {
            long long r = (b + rb - 1) / rb;
            if (r > p.seg[s].rows) r = p.seg[s].rows;
            return base + r;
        }
        b -= segb;
        base += p.seg[s].rows;
    }
    return base;
}

// Tile iterator over [vbeg, vend) of the concatenated virtual-row space.
struct TileIter {
    long long cur, end;
    __device__ bool next(const GemvParams& p, Tile& t) {
        if (cur >= end) return false;
        long long base = 0;
        const int ns = n_vsegs(p);
        int s = 0;
        for (; s < ns; ++s) {
            if (cur < base + p.seg[s].rows) break;
            base += p.seg[s].rows;
        }
        const int cap = p.epi == EPI_SWIGLU ? kGemvTileRows / 2 : kGemvTileRows;
        long long stop = cur + cap;
        if (stop > end) stop = end;
        if (stop > base + p.seg[s].rows) stop = base + p.seg[s].rows;
        // a fragment never crosses a 16-row tile of the packed layout, so each
        // of its stages is one contiguous range
        const long long tile_end = base + ((cur - base) / kGemvTileRows + 1) * kGemvTileRows;
        if (stop > tile_end) stop = tile_end;
        t.seg = s;
        t.row0 = (int)(cur - base);
        t.n = (int)(stop - cur);
        cur = stop;
        return true;
    }
};

// Physical row p (0..15) of a tile: segment, row index, validity.
__device__ __forceinline__ bool tile_row(const GemvParams& p, const Tile& t, int pr, int& seg, int& row) {
    if (p.epi == EPI_SWIGLU) {
        const int vr = pr & 7;
        seg = pr >> 3;
        row = t.row0 + vr;
        return vr < t.n;
    }
    seg = t.seg;
    row = t.row0 + pr;
    return pr < t.n;
}

// Bytes of one row's segment for stage `st` (8 super-blocks, fewer in the last
// stage): Q4_K nbs*144; Q6_K nbs*208 + 16 (the group's d values).
__device__ __forceinline__ uint32_t stage_seg_bytes(int type, int nbs) {
    return type == AF_GGML_Q6_K ? (uint32_t)nbs * 208u + 16u : (uint32_t)nbs * 144u;
}

// Address of rows [row, row + n) of stage `st` in the packed (tile-major) layout:
// tile t = row / 16 occupies 16 * row_stride bytes; inside it stage st starts at
// 16 * st * full_seg and row i of the tile at i * seg(st).
__device__ __forceinline__ const uint8_t* packed_stage_ptr(const GemvSeg& g, int row, int st, uint32_t seg) {
    const uint32_t full = g.type == AF_GGML_Q6_K ? 1680u : 1152u;
    return g.w + (size_t)(row / kGemvTileRows) * kGemvTileRows * g.row_stride +
           (size_t)kGemvTileRows * st * full + (size_t)(row % kGemvTileRows) * seg;
}

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
        const int xi_lo = k;
        const int xi_hi = 8 + k;
        const int e = k & 1;
        lh[e] = dp4a_us(lo, xh0[xi_lo], lh[e]);
        ll[e] = dp4a_us(lo, xl0[xi_lo], ll[e]);
        hh[e] = dp4a_us(hi, xh0[xi_hi], hh[e]);
        hl[e] = dp4a_us(hi, xl0[xi_hi], hl[e]);
    }
    const int tlo = (lh[0] + lh[1]) * 256 + (ll[0] + ll[1]);
    const int thi = ((hh[0] + hh[1]) * 256 + (hl[0] + hl[1])) >> 4;  // exact: every term is a multiple of 16
    // 6-bit scale/min pairs j = 2c (low nibbles) and 2c+1 (high nibbles):
    // get_scale_min_k4 (gemv_q4k_avx2.cpp:34-43) four bytes at a time.
    const uint32_t w0 = hdr.y, w1 = hdr.z, w2 = hdr.w;
    uint32_t S, M;
    if (c < 2) {
        S = w0 & 0x3F3F3F3Fu;
        M = w1 & 0x3F3F3F3Fu;
    } else {
        S = (w2 & 0x0F0F0F0Fu) | ((w0 >> 2) & 0x30303030u);
        M = ((w2 >> 4) & 0x0F0F0F0Fu) | ((w1 >> 2) & 0x30303030u);
    }
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

__device__ __forceinline__ void bar_consumers() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__global__ void __launch_bounds__(kGemvThreads, 2) gemv_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kGemvMaxSlots;
    int* abort_flag = reinterpret_cast<int*>(empty + kGemvMaxSlots);
    uint8_t* ring = smem + 128;
    const int nb = p.K / 256;
    const int nst = (nb + 7) / 8;
    uint8_t* XH = ring + p.nslots * kGemvTileRows * p.pitch;
    uint8_t* XL = XH + nst * 2048;
    float* XS = reinterpret_cast<float*>(XL + nst * 2048);
    float* XS32 = XS + nst * 32;
    int* XI16 = reinterpret_cast<int*>(XS32 + nst * 64);
    float* red = reinterpret_cast<float*>(XI16 + nst * 128);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // CTA row range, balanced by weight bytes.
    long long total = 0;
    for (int s = 0; s < n_vsegs(p); ++s) total += vrow_bytes(p, s) * p.seg[s].rows;
    const long long vbeg = vrow_at(p, total * blockIdx.x / gridDim.x);
    const long long vend = vrow_at(p, total * (blockIdx.x + 1) / gridDim.x);

    if (threadIdx.x == 0) {
        for (int i = 0; i < p.nslots; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kConsumerWarps);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kConsumerWarps) {
        // ---------------- producer warp ----------------
        const uint64_t pol = policy_evict_first();
        TileIter it{vbeg, vend};
        Tile t;
        uint32_t issued = 0;
        bool ok = true;
        while (ok && it.next(p, t)) {
            for (int st = 0; st < nst && ok; ++st) {
                const int slot = issued % p.nslots;
                const uint32_t ph = (issued / p.nslots) & 1u;
                if (lane == 0) ok = mbar_wait(&empty[slot], ph ^ 1u);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok || *(volatile int*)abort_flag) { ok = false; break; }
                // one bulk copy per segment per stage (two for a gate/up pair)
                if (lane == 0) {
                    const int nbs = min(8, nb - st * 8);
                    const GemvSeg& g0 = p.seg[p.epi == EPI_SWIGLU ? 0 : t.seg];
                    const uint32_t segb = stage_seg_bytes(g0.type, nbs);
                    const uint32_t bytes = (uint32_t)t.n * segb;
                    uint8_t* dst = ring + slot * kGemvTileRows * p.pitch;
                    mbar_arrive_expect_tx(&full[slot], p.epi == EPI_SWIGLU ? 2 * bytes : bytes);
                    bulk_g2s(dst, packed_stage_ptr(g0, t.row0, st, segb), bytes, &full[slot], pol);
                    if (p.epi == EPI_SWIGLU)
                        bulk_g2s(dst + 8 * segb, packed_stage_ptr(p.seg[1], t.row0, st, segb), bytes, &full[slot], pol);
                }
                __syncwarp();
                ++issued;
            }
        }
        if (!ok) {
            *(volatile int*)abort_flag = 1;
            // Drain: wait (bounded) for the copies still in flight.
            if (lane == 0) {
                const uint32_t first = issued > (uint32_t)p.nslots ? issued - p.nslots : 0u;
                for (uint32_t i = first; i < issued; ++i)
                    mbar_wait(&full[i % p.nslots], (i / p.nslots) & 1u);
            }
        }
        return;
    }

    // ---------------- consumer warps: input prologue ----------------
    // All global loads of the input are issued together (one memory latency),
    // held in registers, then normalised and quantised.
    pdl_wait();
    const int tid = threadIdx.x;  // 0..255
    const int nvec = p.K / 4;
    const int niter = nst * 2;    // float4 slots per thread incl. the padded last stage
    float4 a[kPrologueVec];
#pragma unroll
    for (int j = 0; j < kPrologueVec; ++j) {
        a[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        const int v = j * kConsumerThreads + tid;
        if (j < niter && v < nvec) {
            a[j] = reinterpret_cast<const float4*>(p.x)[v];
            if (p.x_add) {
                const float4 b = reinterpret_cast<const float4*>(p.x_add)[v];
                a[j].x += b.x; a[j].y += b.y; a[j].z += b.z; a[j].w += b.w;
            }
        }
    }
    if (p.x_store && blockIdx.x == 0) {
#pragma unroll
        for (int j = 0; j < kPrologueVec; ++j) {
            const int v = j * kConsumerThreads + tid;
            if (j < niter && v < nvec) reinterpret_cast<float4*>(p.x_store)[v] = a[j];
        }
    }
    if (p.norm_w) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < kPrologueVec; ++j)
            ss += a[j].x * a[j].x + a[j].y * a[j].y + a[j].z * a[j].z + a[j].w * a[j].w;
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        bar_consumers();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) tot += red[w];
        // rms_norm_out (src/models/llama_model.cpp:393-419): 1/sqrt(ss/n + eps)
        const float inv_rms = 1.f / sqrtf(tot / (float)p.K + p.eps);
#pragma unroll
        for (int j = 0; j < kPrologueVec; ++j) {
            const int v = j * kConsumerThreads + tid;
            if (j < niter && v < nvec) {
                const float4 w = reinterpret_cast<const float4*>(p.norm_w)[v];
                a[j].x = w.x * (a[j].x * inv_rms);
                a[j].y = w.y * (a[j].y * inv_rms);
                a[j].z = w.z * (a[j].z * inv_rms);
                a[j].w = w.w * (a[j].w * inv_rms);
            }
        }
    }
    // Quantise: 16 consecutive threads own one 64-value group.
#pragma unroll
    for (int j = 0; j < kPrologueVec; ++j) {
        if (j >= niter) break;
        const int v = j * kConsumerThreads + tid;
        const float4 q4 = a[j];
        float amax = fmaxf(fmaxf(fabsf(q4.x), fabsf(q4.y)), fmaxf(fabsf(q4.z), fabsf(q4.w)));
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        // 16-bit grid of ±32639 so that hi = (q + 128) >> 8 stays within int8.
        const float xs = amax / 32639.f;
        const float inv = amax > 0.f ? 32639.f / amax : 0.f;
        const float av[4] = {q4.x, q4.y, q4.z, q4.w};
        uint32_t hw = 0, lw = 0;
        int isum = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            int q = __float2int_rn(av[e] * inv);
            q = max(-32639, min(32639, q));
            const int hi = (q + 128) >> 8;
            const int lo = q - hi * 256;
            hw |= (uint32_t)(hi & 0xFF) << (8 * e);
            lw |= (uint32_t)(lo & 0xFF) << (8 * e);
            isum += q;
        }
        float fsum = q4.x + q4.y + q4.z + q4.w;
        fsum += __shfl_xor_sync(0xffffffffu, fsum, 1);
        fsum += __shfl_xor_sync(0xffffffffu, fsum, 2);
        isum += __shfl_xor_sync(0xffffffffu, isum, 1);
        isum += __shfl_xor_sync(0xffffffffu, isum, 2);
        const float fsum32 = fsum + __shfl_xor_sync(0xffffffffu, fsum, 4);
        // position -> lane-major layout [stage][chunk i][lane L][16 bytes]
        const int val = v * 4;
        const int s = val >> 11, w = val & 2047;
        const int b = w >> 8, c = (w >> 6) & 3, i = (w >> 4) & 3, e = w & 15;
        const int L = b * 4 + c;
        const int off = s * 2048 + i * 512 + L * 16 + e;
        *reinterpret_cast<uint32_t*>(XH + off) = hw;
        *reinterpret_cast<uint32_t*>(XL + off) = lw;
        if ((tid & 15) == 0) XS[s * 32 + L] = xs;
        if ((tid & 7) == 0) XS32[s * 64 + (i >> 1) * 32 + L] = fsum32;
        if ((tid & 3) == 0) XI16[s * 128 + i * 32 + L] = isum;
    }
    bar_consumers();

    // ---------------- consumer main loop ----------------
    const int lb = lane >> 2, lc = lane & 3;
    TileIter it{vbeg, vend};
    Tile t;
    uint32_t consumed = 0;
    bool ok = true;
    float best = -INFINITY;
    uint32_t best_idx = 0;
    while (ok && it.next(p, t)) {
        float acc[2] = {0.f, 0.f};
        int seg[2], row[2];
        bool rv[2];
        rv[0] = tile_row(p, t, warp, seg[0], row[0]);
        rv[1] = tile_row(p, t, warp + 8, seg[1], row[1]);
        const int ty0 = p.seg[seg[0]].type, ty1 = p.seg[seg[1]].type;
        for (int st = 0; st < nst; ++st) {
            const int slot = consumed % p.nslots;
            const uint32_t ph = (consumed / p.nslots) & 1u;
            if (lane == 0) ok = mbar_wait(&full[slot], ph);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok || *(volatile int*)abort_flag) { ok = false; break; }
            const int nbs = min(8, nb - st * 8);
            if (lb < nbs) {
                XRegs x;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    x.h[i] = *reinterpret_cast<const uint4*>(XH + st * 2048 + i * 512 + lane * 16);
                    x.l[i] = *reinterpret_cast<const uint4*>(XL + st * 2048 + i * 512 + lane * 16);
                    x.is16[i] = XI16[st * 128 + i * 32 + lane];
                }
                x.xs = XS[st * 32 + lane];
                x.s32[0] = XS32[st * 64 + lane];
                x.s32[1] = XS32[st * 64 + 32 + lane];
                // Both rows of the warp are evaluated without branches so their
                // independent dp4a chains interleave; an invalid row reads
                // stale shared memory and its result is discarded.
                const uint32_t segb = stage_seg_bytes(ty0, nbs);
                const uint8_t* rp0 = ring + slot * kGemvTileRows * p.pitch + warp * segb;
                const uint8_t* rp1 = rp0 + 8 * segb;
                if (ty0 == ty1 && ty0 == AF_GGML_Q6_K) {
                    const float d0 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(rp0 + nbs * 208 + 2 * lb));
                    const float d1 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(rp1 + nbs * 208 + 2 * lb));
                    const float a0 = q6k_lane_dot(rp0 + lb * 208, d0, lc, x);
                    const float a1 = q6k_lane_dot(rp1 + lb * 208, d1, lc, x);
                    acc[0] += a0;
                    acc[1] += a1;
                } else if (ty0 == ty1) {
                    const float a0 = q4k_lane_dot(rp0 + lb * 144, lc, x);
                    const float a1 = q4k_lane_dot(rp1 + lb * 144, lc, x);
                    acc[0] += a0;
                    acc[1] += a1;
                } else {
                    set_err(kErrBadArgs);  // a tile never mixes types (checked on the host)
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            ++consumed;
        }
        if (!ok) break;
        acc[0] = warp_sum(acc[0]);
        acc[1] = warp_sum(acc[1]);
        if (lane == 0) {
            if (p.epi == EPI_SWIGLU) {
                if (rv[0]) {
                    const float g = acc[0], u = acc[1];
                    p.seg[0].y[row[0]] = (g / (1.f + expf(-g))) * u;
                }
            } else {
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    if (!rv[r]) continue;
                    const GemvSeg& sg = p.seg[seg[r]];
                    float v = acc[r];
                    if (p.epi == EPI_RESID) {
                        p.resid[row[r]] += v;
                    } else {
                        if (sg.bias) v += sg.bias[row[r]];
                        sg.y[row[r]] = v;
                        if (p.epi == EPI_ARGMAX) {
                            // strict '>' keeps the first maximum within the warp's rows,
                            // which are visited in increasing order per warp.
                            const uint32_t gi = (uint32_t)(p.argmax_base + row[r]);
                            if (v > best || (v == best && gi < best_idx)) { best = v; best_idx = gi; }
                        }
                    }
                }
            }
        }
    }
    if (!ok) *(volatile int*)abort_flag = 1;
    if (p.epi == EPI_ARGMAX && lane == 0 && best > -INFINITY) atomicMax(p.argmax, argmax_key(best, best_idx));
}

}  // namespace

int gemv_configure(GemvParams& p) {
    int pitch = 0;
    const int nsegs = p.nseg;
    for (int s = 0; s < nsegs; ++s) {
        const int rb = p.seg[s].type == AF_GGML_Q6_K ? 8 * 208 + 16 : 8 * 144;
        pitch = pitch > rb ? pitch : rb;
    }
    // Ring budget keeps two CTAs (this kernel and the next one under PDL) per SM.
    const int budget = 84 * 1024;
    int ns = budget / (kGemvTileRows * pitch);
    ns = ns < 2 ? 2 : (ns > 4 ? 4 : ns);
    p.pitch = pitch;
    p.nslots = ns;
    return gemv_smem_bytes(p.K, pitch, ns);
}

cudaError_t gemv_init() {
    return cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

cudaError_t gemv_launch(const GemvParams& p, int grid, cudaStream_t stream, bool pdl) {
    const int smem = gemv_smem_bytes(p.K, p.pitch, p.nslots);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
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

}  // namespace af
