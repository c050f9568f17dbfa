// af_gemv.cu — fused dequant GEMV kernel (see af_gemv.cuh for the design).
#include "af_gemv.cuh"

namespace af {

__device__ int g_err = 0;

// One warp quantises 64-value group g of src into the XQ layout.  Values are
// read through L2 (other CTAs wrote them); the 16-bit split matches the
// consumers' dp4a form: q = rint(v·32639/amax), hi = (q + 128) >> 8, lo = q − 256·hi.
__device__ void xq_quantize_group(uint8_t* xq, const float* src, const float* norm_w, int K, int g) {
    const int lane = threadIdx.x & 31;
    const int nst = (K / 256 + 7) / 8;
    const int v0 = 64 * g + 2 * lane;
    float a0 = __ldcg(src + v0), a1 = __ldcg(src + v0 + 1);
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

namespace {

constexpr int kCW = kGemvConsumerWarps;
constexpr int kCT = kCW * 32;

__global__ void xq_quantize_kernel(uint8_t* xq, const float* x, const float* norm_w, int K) {
    pdl_launch_dependents();
    pdl_wait();
    const int g = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (g < K / 64) xq_quantize_group(xq, x, norm_w, K, g);
}

struct Frag {
    int seg;     // segment of the fragment's rows
    int row0;    // first row within the segment (virtual row for SwiGLU pairs)
    int n;       // rows (row pairs for SwiGLU)
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
        int stop = min(min(cur + cap, end), base + p.seg[s].rows);
        t.seg = s;
        t.row0 = cur - base;
        t.n = stop - cur;
        cur = stop;
        return true;
    }
};

// Bytes of one row's segment for a stage of nbs super-blocks: Q4_K nbs*144;
// Q6_K nbs*208 + 16 (the group's d values).
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


__device__ __forceinline__ void bar_consumers() { asm volatile("bar.sync 1, %0;" ::"n"(kCT) : "memory"); }

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
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kGemvMaxSlots;
    uint64_t* xbar = empty + kGemvMaxSlots;
    int* flags = reinterpret_cast<int*>(xbar + 1);  // [0] abort, [1..] group list
    uint8_t* ring = smem + 256;
    const int nb = p.K / 256;
    const int nst = (nb + 7) / 8;
    uint8_t* xqs = ring + p.nslots * kGemvFragRows * p.pitch;
    float* misc = reinterpret_cast<float*>(xqs + xq_norm_bytes(p.K));  // 64 floats

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int vbeg = p.vrange[blockIdx.x], vend = p.vrange[blockIdx.x + 1];

    if (threadIdx.x == 0) {
        for (int i = 0; i < p.nslots; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kCW);
        }
        mbar_init(xbar, 1);
        flags[0] = 0;
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kCW) {
        // ---------------- producer warp ----------------
        if (lane != 0) return;
        const uint64_t pol = policy_evict_first();
        const uint32_t xbytes = p.xq ? (uint32_t)(p.xq_norm ? xq_norm_bytes(p.K) : xq_bytes(p.K)) : 0u;
        bool xq_done = p.xq == nullptr;
        FragIter it{vbeg, vend};
        Frag fr[2];
        uint32_t issued = 0;
        bool ok = true;
        // fragments are taken in pairs; both fragments' stage st go to two
        // consecutive slots, so a consumer warp reuses one x load for 4 rows
        while (ok && it.next(p, fr[0])) {
            const int nf = it.next(p, fr[1]) ? 2 : 1;
            for (int st = 0; st < nst && ok; ++st) {
                for (int f = 0; f < nf && ok; ++f) {
                    const Frag& t = fr[f];
                    const int slot = issued % p.nslots;
                    const uint32_t ph = (issued / p.nslots) & 1u;
                    if (!xq_done && issued >= (uint32_t)p.nslots) {
                        // ring full of prefetched weights: now fetch the input
                        pdl_wait();
                        mbar_arrive_expect_tx(xbar, xbytes);
                        bulk_g2s(xqs, p.xq, xbytes, xbar, pol);
                        xq_done = true;
                    }
                    ok = mbar_wait(&empty[slot], ph ^ 1u);
                    if (!ok || *(volatile int*)flags) { ok = false; break; }
                    const int nbs = min(8, nb - st * 8);
                    const GemvSeg& g0 = p.seg[p.epi == EPI_SWIGLU ? 0 : t.seg];
                    const uint32_t segb = stage_seg_bytes(g0.type, nbs);
                    uint8_t* dst = ring + slot * kGemvFragRows * p.pitch;
                    mbar_arrive_expect_tx(&full[slot], (p.epi == EPI_SWIGLU ? 2u : 1u) * (uint32_t)t.n * segb);
                    copy_rows(dst, g0, t.row0, t.n, st, segb, &full[slot], pol);
                    if (p.epi == EPI_SWIGLU)
                        copy_rows(dst + (kGemvFragRows / 2) * segb, p.seg[1], t.row0, t.n, st, segb, &full[slot], pol);
                    ++issued;
                }
            }
        }
        if (!xq_done && ok) {
            pdl_wait();
            mbar_arrive_expect_tx(xbar, xbytes);
            bulk_g2s(xqs, p.xq, xbytes, xbar, pol);
            xq_done = true;
        }
        if (!ok) {
            *(volatile int*)flags = 1;
            // Drain: wait (bounded) for the copies still in flight.
            const uint32_t first = issued > (uint32_t)p.nslots ? issued - p.nslots : 0u;
            for (uint32_t i = first; i < issued; ++i) mbar_wait(&full[i % p.nslots], (i / p.nslots) & 1u);
            if (xq_done && p.xq) mbar_wait(xbar, 0);
        }
        return;
    }

    // ---------------- consumer warps: input ----------------
    pdl_wait();
    float s_in = 1.f;  // RMSNorm scale folded into the per-group scales (XQ input)
    if (p.xq) {
        bool ok = true;
        if (lane == 0) ok = mbar_wait(xbar, 0);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
            *(volatile int*)flags = 1;
        } else if (p.xq_norm) {
            // s = 1/sqrt(Σx²/K + eps) from the producer's per-group sums, in a
            // fixed order (deterministic)
            const float* pss = reinterpret_cast<const float*>(xqs + xq_bytes(p.K));
            float ss = 0.f;
            for (int g = lane; g < p.K / 64; g += 32) ss += pss[g];
            ss = warp_sum(ss);
            s_in = 1.f / sqrtf(ss / (float)p.K + p.eps);
        }
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
    const uint8_t* XH = xqs;
    const uint8_t* XL = xqs + nst * 2048;
    const float* XS = reinterpret_cast<const float*>(xqs + 2 * nst * 2048);
    const float* XS32 = XS + nst * 32;
    const int* XI16 = reinterpret_cast<const int*>(XS32 + nst * 64);

    // ---------------- consumer main loop ----------------
    const int lb = lane >> 2, lc = lane & 3;
    FragIter it{vbeg, vend};
    Frag fr[2];
    uint32_t consumed = 0;
    bool ok = !*(volatile int*)flags;
    float best = -INFINITY;
    uint32_t best_idx = 0;
    const int half = kGemvFragRows / 2;
    while (ok && it.next(p, fr[0])) {
        const int nf = it.next(p, fr[1]) ? 2 : 1;
        // rows of this warp: (fragment f, r) -> slot row warp + r*half
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
            const int slot0 = consumed % p.nslots;
            const int slot1 = (consumed + 1) % p.nslots;
            if (lane == 0) {
                ok = mbar_wait(&full[slot0], (consumed / p.nslots) & 1u);
                if (ok && nf == 2) ok = mbar_wait(&full[slot1], ((consumed + 1) / p.nslots) & 1u);
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok || *(volatile int*)flags) { ok = false; break; }
            const int nbs = min(8, nb - st * 8);
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
                // chains interleave; an invalid row reads stale shared memory
                // and its result is discarded.
                const uint8_t* rp[2][2];
#pragma unroll
                for (int f = 0; f < 2; ++f) {
                    const uint32_t segb = stage_seg_bytes(ty[f], nbs);
                    rp[f][0] = ring + (f ? slot1 : slot0) * kGemvFragRows * p.pitch + warp * segb;
                    rp[f][1] = rp[f][0] + half * segb;
                }
                if (nf == 2 && ty[0] == ty[1]) {
                    if (ty[0] == AF_GGML_Q6_K) {
                        float d[4], a[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            d[k] = half_bits_to_float(*reinterpret_cast<const uint16_t*>(rp[k >> 1][k & 1] + nbs * 208 + 2 * lb));
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
                            const float d0 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(rp[f][0] + nbs * 208 + 2 * lb));
                            const float d1 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(rp[f][1] + nbs * 208 + 2 * lb));
                            const float a0 = q6k_lane_dot(rp[f][0] + lb * 208, d0, lc, x);
                            const float a1 = q6k_lane_dot(rp[f][1] + lb * 208, d1, lc, x);
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
                mbar_arrive(&empty[slot0]);
                if (nf == 2) mbar_arrive(&empty[slot1]);
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
            for (int r = 0; r < 2; ++r) {
                if (!rv[f][r]) continue;
                float v = acc[f][r];
                if (p.epi == EPI_RESID) {
                    p.resid[row[f][r]] += v;
                } else {
                    if (sg.bias) v += sg.bias[row[f][r]];
                    sg.y[row[f][r]] = v;
                    if (p.epi == EPI_ARGMAX) {
                        // rows reach a lane in increasing order; ties keep the lowest index
                        const uint32_t gi = (uint32_t)(p.argmax_base + row[f][r]);
                        if (v > best || (v == best && gi < best_idx)) { best = v; best_idx = gi; }
                    }
                }
            }
        }
    }
    if (!ok) *(volatile int*)flags = 1;
    if (p.epi == EPI_ARGMAX && lane == 0 && best > -INFINITY) atomicMax(p.argmax, argmax_key(best, best_idx));

    // ---------------- quantise the output for the next GEMV ----------------
    if (p.q_out) {
        // Each 64-row group is quantised by the CTA that completes it.
        int* list = flags + 1;
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
}

}  // namespace

void gemv_configure(GemvParams& p, int grid) {
    int pitch = 0;
    for (int s = 0; s < p.nseg; ++s) {
        const int rb = p.seg[s].type == AF_GGML_Q6_K ? 8 * 208 + 16 : 8 * 144;
        pitch = pitch > rb ? pitch : rb;
    }
    const int budget = 165 * 1024;
    int ns = budget / (kGemvFragRows * pitch);
    ns = ns < 2 ? 2 : (ns > kGemvMaxSlots ? kGemvMaxSlots : ns);
    p.pitch = pitch;
    p.nslots = ns;
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
    const int smem = gemv_smem_bytes(p.K, p.pitch, p.nslots);
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
