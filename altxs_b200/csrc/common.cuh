// Internal helpers shared by the altxs_b200 CUDA sources (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/altxs_b200.h"

#define ALTXS_LAUNCH_CHECK()                                   \
    do {                                                       \
        cudaError_t e_ = cudaGetLastError();                   \
        if (e_ != cudaSuccess) {                               \
            ::altxs::note_cuda_error(e_);                      \
            return ALTXS_ECUDA;                                \
        }                                                      \
    } while (0)

namespace altxs {

// Records the CUDA error behind an ALTXS_ECUDA return (altxs_last_cuda_error).
void note_cuda_error(cudaError_t e);

constexpr uint64_t kTop = 1ull << 32;
constexpr uint64_t kHalf = 1ull << 31;
constexpr uint64_t kQuarter = 1ull << 30;
constexpr float kRmsEps = 1.1920928955078125e-07f;  // torch.finfo(float32).eps

__host__ __device__ inline int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ unsigned long long warp_sum_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Block-wide reductions with a fixed combination order (deterministic for a
// given block size).  `red` must hold >= 32 elements of the result type.
__device__ __forceinline__ float block_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float r = lane < nw ? red[lane] : 0.0f;
    r = warp_sum(r);
    return r;
}
__device__ __forceinline__ float block_max(float v, float *red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float r = lane < nw ? red[lane] : -INFINITY;
    return warp_max(r);
}
__device__ __forceinline__ unsigned long long block_sum_u64(unsigned long long v,
                                                            unsigned long long *red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum_u64(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    unsigned long long r = lane < nw ? red[lane] : 0ull;
    return warp_sum_u64(r);
}

// ---- fixed-point exp shared bit-exactly with oracle/coder.c ---------------
// 2^f on [0,1): Taylor series of e^(f ln2) through f^8, Horner with fma.
__device__ __forceinline__ float exp2_frac(float f) {
    float p = 1.32154867901443094e-06f;
    p = __fmaf_rn(p, f, 1.52527338040598403e-05f);
    p = __fmaf_rn(p, f, 1.54035303933816099e-04f);
    p = __fmaf_rn(p, f, 1.33335581464284434e-03f);
    p = __fmaf_rn(p, f, 9.61812910762847717e-03f);
    p = __fmaf_rn(p, f, 5.55041086648215800e-02f);
    p = __fmaf_rn(p, f, 2.40226506959100712e-01f);
    p = __fmaf_rn(p, f, 6.93147180559945309e-01f);
    p = __fmaf_rn(p, f, 1.0f);
    return p;
}
__device__ __forceinline__ float pow2i(int n) {  // exact 2^n for -126 <= n <= 127
    return __int_as_float((n + 127) << 23);
}
constexpr float kLog2e = 1.44269504088896341f;

// u = floor(2^24 * exp(l - mx)), l <= mx
__device__ __forceinline__ uint32_t fixed_weight(float l, float mx) {
    float x = __fsub_rn(l, mx);
    float t = __fmul_rn(x, kLog2e);
    float nf = floorf(t);
    if (nf < -25.0f) return 0u;
    float f = __fsub_rn(t, nf);
    float p = exp2_frac(f);
    int n = (int)nf;
    float scaled = __fmul_rn(p, pow2i(24 + n));
    return (uint32_t)floorf(scaled);
}
// e = exp(l - mx) with the same polynomial (reference-scale rule)
__device__ __forceinline__ float exp_rel(float l, float mx) {
    float x = __fsub_rn(l, mx);
    float t = __fmul_rn(x, kLog2e);
    float nf = floorf(t);
    if (nf < -126.0f) return 0.0f;
    float f = __fsub_rn(t, nf);
    return __fmul_rn(exp2_frac(f), pow2i((int)nf));
}
// reference mass rule max(1, floor((double)p * 1e6 + 0.5)) (gpu_ac.py:38-42)
__device__ __forceinline__ uint32_t ref_mass(float p) {
    double s = floor(__dadd_rn(__dmul_rn((double)p, 1000000.0), 0.5));
    long long v = (long long)s;
    return v < 1 ? 1u : (uint32_t)v;
}

// ---- shared-memory / TMA bulk copy helpers --------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// orders this thread's generic-proxy global accesses with async-proxy (TMA bulk) ones
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
__device__ __forceinline__ void mbar_inval(uint64_t *bar) {
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// Untiled bulk copy global -> shared, completion counted on `bar` (bytes % 16 == 0,
// both addresses 16-byte aligned; source is this GPU's own memory).
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: returns false if the phase did not complete within `limit` polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
constexpr uint32_t kWaitLimit = 1u << 22;
// Polls of the first wait of every pipeline stage (the data the kernel is
// waiting for).  A wait that gives up records ALTXS_ST_TIMEOUT; the drain
// waits that follow (the kernel's own copies and MMAs) keep kWaitLimit, so
// nothing is left in flight when a CTA exits.  One copy per translation unit,
// set for all of them by altxs_set_wait_limit (tests use 0: give up at once).
static __device__ uint32_t g_wait_limit = kWaitLimit;
__device__ __forceinline__ uint32_t wait_limit() { return *(volatile uint32_t *)&g_wait_limit; }

// fp16 bits -> float
__device__ __forceinline__ float h2f(uint16_t b) { return __half2float(__ushort_as_half(b)); }

}  // namespace altxs
