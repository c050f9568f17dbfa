// af_common.cuh — shared device helpers for the sm_100a decode kernels:
// mbarrier + bulk-copy (TMA engine) PTX wrappers with bounded waits,
// programmatic dependent launch (PDL) controls, and the device error flag.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/af_b200.h"

namespace af {

// Device-side error word.  Kernels never trap: a wait that runs out sets a
// code here and the kernel returns; the host reads it with af_device_error().
extern __device__ int g_err;

constexpr int kErrMbarTimeout = 1;     // an mbarrier wait exceeded its limit
constexpr int kErrBadArgs = 2;         // launch arguments failed a device check
constexpr int kErrBadToken = 3;        // a step saw a token id outside the vocabulary (or no argmax)

// Iteration limit of every spin on an mbarrier.  Each try_wait suspends for
// up to the hardware time limit, so this is seconds of wall time at most.
constexpr uint32_t kSpinLimit = 1u << 26;

__device__ __forceinline__ void set_err(int code) { atomicCAS(&g_err, 0, code); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier -------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on phase `parity`.  Returns false (and sets g_err) on timeout.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// With `abort`, the wait also gives up (without an error code) once *abort
// is set by another thread of the CTA.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const volatile int* abort = nullptr) {
    if (mbar_test_wait(bar, parity)) return true;  // already complete: no suspend
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (abort && (i & 15) == 15 && *abort) return false;
    }
    set_err(kErrMbarTimeout);
    return false;
}

// ---- bulk copy global -> shared (TMA engine, no tensor map, no multicast) --

// L2 policy for streamed-once weights: evict-first keeps activations, the KV
// cache and the next kernel's inputs resident in L2.
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// L2 policy for inputs many CTAs read: keep them resident.
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// ---- programmatic dependent launch ------------------------------------------

// Block until the preceding kernel in the stream has completed and its memory
// is visible (no-op when the launch was not programmatic).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Allow the next kernel in the stream to begin launching.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- small math helpers ----------------------------------------------------

// a: four unsigned bytes, b: four signed bytes.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// System-scope relaxed 64-bit store / load: single-copy atomic words that a
// peer GPU (NVLink, IPC-mapped memory) observes without fences.
__device__ __forceinline__ void st_relaxed_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// GPU-scope relaxed 64-bit store / load: single-copy atomic words another
// CTA of this GPU observes without fences (a tag in the high half makes the
// word its own arrival flag).
__device__ __forceinline__ void st_relaxed_gpu(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_gpu(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
}

// Order-preserving map of a float to uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t float_to_ordered(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float ordered_to_float(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    return __uint_as_float(u);
}

// Packed argmax key: (ordered value << 32) | (~index) so that atomicMax picks
// the largest value and, among equal values, the smallest index — the
// first-maximum rule of std::max_element.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    return (static_cast<unsigned long long>(float_to_ordered(v)) << 32) | (0xFFFFFFFFu - idx);
}

}  // namespace af

// Host helper: launch with the programmatic-stream-serialization attribute.
#define AF_CUDA_TRY(x)                               \
    do {                                             \
        cudaError_t e_ = (x);                        \
        if (e_ != cudaSuccess) return e_;            \
    } while (0)
