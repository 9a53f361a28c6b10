// tcgen05 tensor-core GEMM on hi/lo bf16 planes (sm_100a).
//
// C[b] = epi( sum_k A(b)[m][k] B(b)[n][k] ) with A and B given as hi/lo bf16
// planes (tc.cuh), each K-major or MN-major.  A persistent grid (one CTA per
// SM) walks 128 x BN output tiles:
//   warp 4      TMA producer: the four tiles (A hi, A lo, B hi, B lo) of each
//               64-wide K slice into a ring of shared-memory stages (128-byte
//               swizzle), one mbarrier per stage (full / empty), across tiles;
//   warp 5      MMA issuer: one thread issues tcgen05.mma (kind::f16, bf16 in,
//               fp32 accumulate in tensor memory) for Ahi*Bhi, Ahi*Blo, Alo*Bhi
//               over the four 16-wide K steps of a stage, then tcgen05.commit
//               frees the stage; two accumulators in tensor memory, so the
//               MMAs of tile i+1 run while the epilogue drains tile i;
//   warps 0-3   epilogue: tcgen05.ld of the accumulator in 32 x 32 blocks,
//               transposed through shared memory so that every warp store
//               writes one contiguous row segment.
// Every wait is bounded; a wait that gives up marks the rows of the tile with
// ALTXS_ST_TIMEOUT (when a status array is given), lets the CTA's own copies
// and MMAs drain (bounded) and frees the tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "gemm.cuh"
#include "model.cuh"
#include "prof.cuh"
#include "qmm.cuh"
#include "tc.cuh"
#include "tcgen05.cuh"

namespace altxs {
namespace {

constexpr int kBM = 128;         // tile rows = tensor-memory lanes
constexpr int kBK = 64;          // K per stage: one 128-byte swizzle row of bf16
constexpr unsigned kFull = 0xffffffffu;

constexpr int kSeg = 2304;  // one packed-code segment: 64 descriptors + up to 64 x 32 code bytes

template <int BN, int AMN, int BMN, int BQ = 0>
struct TcCfg {
    static constexpr int kATile = kBM * kBK * 2;  // bytes of one A plane tile
    static constexpr int kBTile = BN * kBK * 2;   // bytes of one B plane tile
    // packed weights: the tile's code segments (one per 64 rows) land here first
    static constexpr int kStg = BQ ? (BN / 64) * kSeg : 0;
    static constexpr int kStage = (2 * kATile + 2 * kBTile + kStg + 1023) / 1024 * 1024;
    static constexpr int kStages = BQ ? (BN == 64 ? 4 : 3) : (192 * 1024) / kStage;  // BN 64: 4, 128: 3
    // epilogue buffer: a 32 x 32 fp32 TMA-store box per warp, or the padded
    // 32 x 33 transpose block of the plain-store path (never both in one launch)
    static constexpr int kStore = 4 * 32 * 33 * 4;
    static constexpr int kSmem = kStages * kStage + kStore + 1024;  // + alignment slack
    static_assert(kSmem + 256 <= 227 * 1024, "shared memory");
    // kind::f16 instruction descriptor: fp32 accumulate, bf16 A and B,
    // A/B major-ness, M = 128, N = BN
    static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)AMN << 15) |
                                       ((uint32_t)BMN << 16) | ((uint32_t)(BN >> 3) << 17) |
                                       ((uint32_t)(kBM >> 4) << 24);
};

__device__ __forceinline__ float leaky2(float v) {  // leaky_relu(v, 0.5)^2 (model.py:874-882)
    const float t = v >= 0.0f ? v : __fmul_rn(v, 0.5f);
    return __fmul_rn(t, t);
}

// Dequantise the 64-wide group slice `kb` of packed weight row `wrow` into
// values i0 .. i0 + N1 - 1 (N1 = 64 / LPR) of that row in a K-major stage:
// hi/lo bf16 planes, 128 bytes per row, 16-byte chunk j of row r at
// (j ^ (r & 7)) (the 128-byte swizzle TMA would have produced).  The values
// are those of k_split_weights: w = level * scale, hi = bf16(w), lo = bf16(w - hi).
struct DqGroup {
    uint32_t d;     // group descriptor
    uint32_t w[8];  // packed codes (up to 8 x 32 bits: 2/3/4-bit groups)
};

__device__ __forceinline__ int dq_bits(uint32_t d) {
    const int c = (d >> 16) & 15;
    return c == 0 ? 0 : c == 1 ? 2 : c == 2 ? 3 : c == 3 ? 4 : 32;
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds_u64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts_v4(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}

// the row's descriptor and code words from its staged segment (shared-memory
// address seg: explicit shared loads, not generic ones)
__device__ __forceinline__ void dq_load(uint32_t seg, int j, DqGroup &q) {
    q.d = lds_u32(seg + 4 * j);
    const uint32_t p = seg + 256 + 8 * (q.d >> 20);
    const int b = dq_bits(q.d);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const uint2 x = w < b ? lds_u64(p + 8 * w) : make_uint2(0u, 0u);
        q.w[2 * w] = x.x;
        q.w[2 * w + 1] = x.y;
    }
}

// 8 values -> one 16-byte chunk of the hi plane and of the lo plane
// (hi = bf16(v), lo = bf16(v - hi), round to nearest even, two values per cvt)
__device__ __forceinline__ void dq_put8(uint32_t hrow, uint32_t lrow, int pos, const float *f) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const __nv_bfloat162 hb = __floats2bfloat162_rn(f[2 * u], f[2 * u + 1]);
        h[u] = *reinterpret_cast<const uint32_t *>(&hb);
        const float r0 = __fsub_rn(f[2 * u], __uint_as_float(h[u] << 16));
        const float r1 = __fsub_rn(f[2 * u + 1], __uint_as_float(h[u] & 0xffff0000u));
        const __nv_bfloat162 lb = __floats2bfloat162_rn(r0, r1);
        l[u] = *reinterpret_cast<const uint32_t *>(&lb);
    }
    sts_v4(hrow + pos, h[0], h[1], h[2], h[3]);
    sts_v4(lrow + pos, l[0], l[1], l[2], l[3]);
}

// w = (code - (2^B - 1)/2) * scale, exact in fp32 (a <= 4-bit half-integer
// times an fp16 scale).  The code becomes a float by its bits (2^23 + code),
// and fma(2^23 + code, s, -2^23 s) = code * s exactly; code * s - c * s is then
// the same exact value the plane builder forms as (code - c) * s.
template <int B, int N1>
__device__ __forceinline__ void dq_codes(const DqGroup &q, int i0, uint32_t hrow, uint32_t lrow, int r7) {
    const float s = h2f((uint16_t)(q.d & 0xffffu));
    const float k1 = __fmul_rn(-8388608.0f, s);
    const float cs = __fmul_rn((float)((1 << B) - 1) * 0.5f, s);
#pragma unroll
    for (int c = 0; c < N1 / 8; ++c) {
        float f[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = i0 + c * 8 + u;  // i0 is a literal 0 or 32: bit positions fold to constants
            const int bp = i * B, wi = bp >> 5, sh = bp & 31;
            uint32_t v;
            if (sh + B <= 32) v = q.w[wi] >> sh;
            else v = __funnelshift_r(q.w[wi], q.w[wi + 1], sh);
            const uint32_t code = v & ((1u << B) - 1u);
            f[u] = __fsub_rn(__fmaf_rn(__uint_as_float(0x4B000000u | code), s, k1), cs);
        }
        const int j = (i0 >> 3) + c;
        dq_put8(hrow, lrow, (j ^ r7) << 4, f);
    }
}

template <int N1>
__device__ __forceinline__ void dq_slice(const DqGroup &q, int i0, uint32_t hrow, uint32_t lrow, int r7) {
    const int b = dq_bits(q.d);
    if (b == 2) {
        if (i0 == 0) dq_codes<2, N1>(q, 0, hrow, lrow, r7);
        else dq_codes<2, N1>(q, 32, hrow, lrow, r7);
    } else if (b == 3) {
        if (i0 == 0) dq_codes<3, N1>(q, 0, hrow, lrow, r7);
        else dq_codes<3, N1>(q, 32, hrow, lrow, r7);
    } else if (b == 4) {
        if (i0 == 0) dq_codes<4, N1>(q, 0, hrow, lrow, r7);
        else dq_codes<4, N1>(q, 32, hrow, lrow, r7);
    } else {  // 0-bit group: zeros
        const float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < N1 / 8; ++c) dq_put8(hrow, lrow, ((((i0 >> 3) + c) ^ r7) << 4), z);
    }
}

struct Tile {
    int m0, n0, b, kb0, kb1;
    int id;      // output tile (unit without its split)
    int c0, c1;  // chunked K: the unit's chunks
    bool skip;
};

__device__ __forceinline__ int n_chunks(int nk) { return (nk + kTcChunkKb - 1) / kTcChunkKb; }
// chunks per unit (the accumulators a unit keeps in tensor memory)
__device__ __forceinline__ int unit_chunks(const TcGemm &g, int nk) {
    return g.chunked ? (n_chunks(nk) + g.splits - 1) / g.splits : 1;
}

// unit t: split slowest; within a split m-tile fastest (CTAs running at the
// same time share B tiles), then n-tile, then batch
__device__ __forceinline__ Tile tile_of(const TcGemm &g, int t, int mt, int ntl, int nk, int bn) {
    Tile T;
    const int ntiles = mt * ntl * g.batch;
    const int sp = t / ntiles;
    t -= sp * ntiles;
    T.id = t;
    T.m0 = (t % mt) * kBM;
    const int r = t / mt;
    T.n0 = (r % ntl) * bn;
    T.b = r / ntl;
    T.kb0 = 0;
    T.kb1 = nk;
    T.c0 = 0;
    T.c1 = 1;
    if (g.chunked) {
        const int nch = n_chunks(nk), per = unit_chunks(g, nk);
        T.c0 = min(nch, sp * per);
        T.c1 = min(nch, T.c0 + per);
        T.kb0 = T.c0 * kTcChunkKb;
        T.kb1 = min(nk, T.c1 * kTcChunkKb);
    }
    T.skip = g.causal == 1 && T.n0 > T.m0 + kBM - 1;
    if (g.causal == 2) T.kb1 = min(nk, (T.m0 + kBM + kBK - 1) / kBK);
    if (g.causal == 3) T.kb0 = min(nk, T.m0 / kBK);
    return T;
}

__device__ __forceinline__ int op_batch(const TcOp &o, int b) { return (b / o.div) * o.mul + o.add; }

// Epilogue of one 32 x 32 block (tile rows 32*warp .., columns c0 ..): v holds
// this lane's row (lane = tile row).  Applies the layer's epilogue and stores.
template <int BN>
__device__ __forceinline__ void emit_block(const TcGemm &g, const Tile &T, const CUtensorMap *tcm, int warp, int lane,
                                           int c0, const float *v, bool no_k, float (*eb)[33], float *sb, bool vec) {
    float *Cb = g.C ? g.C + (int64_t)T.b * g.sC : nullptr;
    if (g.tma_c) {
        // lane = tile row: its 32 columns become row `lane` of the box
        // (16-byte chunk j stored at j ^ (row & 7): the 128-byte swizzle),
        // then one asynchronous tensor store; the map clips rows >= M and
        // columns >= N.  The box is rewritten only after the previous
        // store has finished reading it.
        const int n0 = T.n0 + c0, mrow = T.m0 + warp * 32;
        if (n0 >= g.N || mrow >= g.M) return;
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
        char *rowp = reinterpret_cast<char *>(sb) + lane * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            float q[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float x = no_k ? 0.0f : v[4 * c + u];
                q[u] = g.alpha != 1.0f ? __fmul_rn(g.alpha, x) : x;
            }
            *reinterpret_cast<float4 *>(rowp + ((c ^ (lane & 7)) << 4)) = make_float4(q[0], q[1], q[2], q[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) tma_store_3d(tcm, sb, n0, mrow, T.b);
        return;
    }
#pragma unroll
    for (int u = 0; u < 32; ++u) eb[lane][u] = no_k ? 0.0f : v[u];
    __syncwarp();
    // lane -> 4 consecutive columns (c4) of rows it*4 + sub: one 16-byte store
    // per lane covers 4 rows x 32 columns per warp instruction.  All reads of
    // a block come before its stores (the residual input may be the output
    // array itself).
    const int sub = lane >> 3, c4 = (lane & 7) * 4;
    float4 vv[8];
#pragma unroll
    for (int it = 0; it < 8; ++it) {
        const float *e = eb[it * 4 + sub] + c4;
        vv[it] = make_float4(e[0], e[1], e[2], e[3]);
    }
    __syncwarp();  // the block buffer is free for the next block once every lane has its values
    const int n = T.n0 + c0 + c4;
    const int mb = T.m0 + warp * 32;
    if (n >= g.N) return;
    if (vec && n + 3 < g.N) {
        if (g.epi == kEpiResid) {
            const float4 cs = *reinterpret_cast<const float4 *>(g.colscale + n);
            float4 rv[8];
#pragma unroll
            for (int it = 0; it < 8; ++it) {
                const int m = mb + it * 4 + sub;
                rv[it] = m < g.M ? *reinterpret_cast<const float4 *>(g.R + (int64_t)m * g.ldr + n)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int it = 0; it < 8; ++it) {
                vv[it].x = __fadd_rn(rv[it].x, __fmul_rn(cs.x, vv[it].x));
                vv[it].y = __fadd_rn(rv[it].y, __fmul_rn(cs.y, vv[it].y));
                vv[it].z = __fadd_rn(rv[it].z, __fmul_rn(cs.z, vv[it].z));
                vv[it].w = __fadd_rn(rv[it].w, __fmul_rn(cs.w, vv[it].w));
            }
        } else {
            if (g.alpha != 1.0f) {
#pragma unroll
                for (int it = 0; it < 8; ++it) {
                    vv[it].x = __fmul_rn(g.alpha, vv[it].x);
                    vv[it].y = __fmul_rn(g.alpha, vv[it].y);
                    vv[it].z = __fmul_rn(g.alpha, vv[it].z);
                    vv[it].w = __fmul_rn(g.alpha, vv[it].w);
                }
            }
            if (g.beta != 0.0f) {
                float4 cv[8];
#pragma unroll
                for (int it = 0; it < 8; ++it) {
                    const int m = mb + it * 4 + sub;
                    cv[it] = m < g.M ? *reinterpret_cast<const float4 *>(Cb + (int64_t)m * g.ldc + n)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int it = 0; it < 8; ++it) {
                    vv[it].x = __fadd_rn(vv[it].x, __fmul_rn(g.beta, cv[it].x));
                    vv[it].y = __fadd_rn(vv[it].y, __fmul_rn(g.beta, cv[it].y));
                    vv[it].z = __fadd_rn(vv[it].z, __fmul_rn(g.beta, cv[it].z));
                    vv[it].w = __fadd_rn(vv[it].w, __fmul_rn(g.beta, cv[it].w));
                }
            }
            if (g.epi == kEpiLeaky2) {
#pragma unroll
                for (int it = 0; it < 8; ++it) {
                    vv[it].x = leaky2(vv[it].x);
                    vv[it].y = leaky2(vv[it].y);
                    vv[it].z = leaky2(vv[it].z);
                    vv[it].w = leaky2(vv[it].w);
                }
            }
        }
#pragma unroll
        for (int it = 0; it < 8; ++it) {
            const int64_t m = mb + it * 4 + sub;
            if (m >= g.M) continue;
            if (Cb) *reinterpret_cast<float4 *>(Cb + m * g.ldc + n) = vv[it];
            if (g.Y2) *reinterpret_cast<float4 *>(g.Y2 + m * g.ldy2 + n) = vv[it];
            if (g.p_hi) {
                const float f[4] = {vv[it].x, vv[it].y, vv[it].z, vv[it].w};
                uint32_t h2[2], l2[2];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const __nv_bfloat16 h0 = __float2bfloat16_rn(f[2 * u]), h1 = __float2bfloat16_rn(f[2 * u + 1]);
                    const __nv_bfloat16 l0 = __float2bfloat16_rn(__fsub_rn(f[2 * u], __bfloat162float(h0)));
                    const __nv_bfloat16 l1 = __float2bfloat16_rn(__fsub_rn(f[2 * u + 1], __bfloat162float(h1)));
                    h2[u] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
                    l2[u] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
                }
                *reinterpret_cast<uint2 *>(g.p_hi + m * g.ldp + n) = make_uint2(h2[0], h2[1]);
                *reinterpret_cast<uint2 *>(g.p_lo + m * g.ldp + n) = make_uint2(l2[0], l2[1]);
            }
        }
    } else {
        // ragged or unaligned edge: element by element, same arithmetic (unrolled,
        // so that vv stays in registers on every path)
#pragma unroll
        for (int it = 0; it < 8; ++it) {
            const int64_t m = mb + it * 4 + sub;
            if (m >= g.M) continue;
            const float f4[4] = {vv[it].x, vv[it].y, vv[it].z, vv[it].w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (n + u >= g.N) break;
                float x = f4[u];
                if (g.epi == kEpiResid) {
                    x = __fadd_rn(g.R[m * g.ldr + n + u], __fmul_rn(g.colscale[n + u], x));
                } else {
                    if (g.alpha != 1.0f) x = __fmul_rn(g.alpha, x);
                    if (g.beta != 0.0f) x = __fadd_rn(x, __fmul_rn(g.beta, Cb[m * g.ldc + n + u]));
                    if (g.epi == kEpiLeaky2) x = leaky2(x);
                }
                if (Cb) Cb[m * g.ldc + n + u] = x;
                if (g.Y2) g.Y2[m * g.ldy2 + n + u] = x;
                if (g.p_hi) split_store(g.p_hi, g.p_lo, m * g.ldp + n + u, x);
            }
        }
    }
}

template <int BQ>
struct TcThreads {
    // warps 0-3 epilogue, 4 TMA producer, 5 MMA issuer, 6-9 (BQ) dequantising producers
    static constexpr int kN = BQ ? 320 : 192;
};

template <int BN, int AMN, int BMN, int BQ>
__global__ void __launch_bounds__(TcThreads<BQ>::kN, 1)
    k_tc_gemm(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
              const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo,
              const __grid_constant__ CUtensorMap tc_map, TcGemm g) {
    using Cfg = TcCfg<BN, AMN, BMN, BQ>;
    constexpr int S = Cfg::kStages;
    static_assert(!BQ || !BMN, "packed weights are read K-major");
    extern __shared__ unsigned char tc_smem_raw[];
    __shared__ __align__(8) uint64_t full[S], empty[S], cfull[S], tfull[2], tempty[2], drainb;
    __shared__ uint32_t tmem_sh;
    __shared__ volatile int abort_sh;
    const uint32_t raw_s = smem_u32(tc_smem_raw);
    unsigned char *sm = tc_smem_raw + ((1024u - (raw_s & 1023u)) & 1023u);  // 1024-byte aligned stages
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = (g.K + kBK - 1) / kBK;
    const int mt = (g.M + kBM - 1) / kBM, ntl = (g.N + BN - 1) / BN;
    const int n_units = mt * ntl * g.batch * g.splits;
    // tensor memory: nbuf tiles in flight, each with `nacc` accumulators of BN columns
    const int nacc = unit_chunks(g, nk);
    const uint32_t bufcols = (uint32_t)(nacc * BN);
    const int nbuf = 2 * bufcols <= 512 ? 2 : 1;
    uint32_t tcols = 32;
    while (tcols < nbuf * bufcols) tcols <<= 1;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], BQ ? 5 : 1);  // the A copies' transaction arrival (+ 4 dequantising warps)
            mbar_init(&empty[s], 1);
            mbar_init(&cfull[s], 1);          // packed weights: the code segments' copies
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);  // one arrival per epilogue warp
        }
        mbar_init(&drainb, 1);
        abort_sh = 0;
        fence_mbar_init();
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_sh)),
                     "r"(tcols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_sh;

    if (warp == 4) {
        if (lane == 0) {
            int q = 0;  // stage fills issued by this CTA (all units)
            for (int t = blockIdx.x; t < n_units && !abort_sh; t += gridDim.x) {
                const Tile T = tile_of(g, t, mt, ntl, nk, BN);
                if (T.skip) continue;
                const int ab = op_batch(g.a, T.b), bb = op_batch(g.b, T.b);
                for (int kb = T.kb0; kb < T.kb1; ++kb, ++q) {
                    const int s = q % S, r = q / S;
                    if (r > 0 && !mbar_wait_bounded(&empty[s], (r - 1) & 1, wait_limit())) {
                        abort_sh = 1;
                        break;
                    }
                    if (abort_sh) break;
                    unsigned char *st = sm + s * Cfg::kStage;
                    unsigned char *sa = st, *sb = st + 2 * Cfg::kATile;
                    const int k0 = kb * kBK;
                    mbar_expect_tx(&full[s], BQ ? 2 * Cfg::kATile : Cfg::kStage);
                    if (!AMN) {
                        tma_load_3d(sa, &ta_hi, k0, (int)g.a.row_off + T.m0, ab, &full[s]);
                        tma_load_3d(sa + Cfg::kATile, &ta_lo, k0, (int)g.a.row_off + T.m0, ab, &full[s]);
                    } else {
#pragma unroll
                        for (int c = 0; c < kBM / 64; ++c) {
                            tma_load_3d(sa + c * 8192, &ta_hi, T.m0 + 64 * c, (int)g.a.row_off + k0, ab, &full[s]);
                            tma_load_3d(sa + Cfg::kATile + c * 8192, &ta_lo, T.m0 + 64 * c, (int)g.a.row_off + k0, ab,
                                        &full[s]);
                        }
                    }
                    if (BQ) {
                        // the tile's code segments of this K slice (one bulk copy per 64 rows;
                        // blocks past the matrix are not copied and read as zeros)
                        const int G = g.wt.cols / kBK, RB = (g.wt.rows + 63) / 64;
                        const int64_t rb0 = (g.wq_row0 + T.n0) / 64;
                        const int nb = (int)max((int64_t)0, min((int64_t)(BN / 64), (int64_t)RB - rb0));
                        mbar_expect_tx(&cfull[s], (uint32_t)(nb * kSeg));
                        unsigned char *stg = st + 2 * Cfg::kATile + 2 * Cfg::kBTile;
                        for (int blk = 0; blk < nb; ++blk)
                            bulk_g2s(stg + blk * kSeg, g.wt.data + ((rb0 + blk) * G + kb) * (int64_t)kSeg, kSeg,
                                     &cfull[s]);
                        continue;  // the dequantising warps fill B
                    }
                    if (!BMN) {
                        tma_load_3d(sb, &tb_hi, k0, (int)g.b.row_off + T.n0, bb, &full[s]);
                        tma_load_3d(sb + Cfg::kBTile, &tb_lo, k0, (int)g.b.row_off + T.n0, bb, &full[s]);
                    } else {
#pragma unroll
                        for (int c = 0; c < BN / 64; ++c) {
                            tma_load_3d(sb + c * 8192, &tb_hi, T.n0 + 64 * c, (int)g.b.row_off + k0, bb, &full[s]);
                            tma_load_3d(sb + Cfg::kBTile + c * 8192, &tb_lo, T.n0 + 64 * c, (int)g.b.row_off + k0, bb,
                                        &full[s]);
                        }
                    }
                }
            }
            if (abort_sh) {  // let this CTA's copies land before the CTA can exit
                for (int p = q - S > 0 ? q - S : 0; p < q; ++p) {
                    if (BQ) mbar_wait_bounded(&cfull[p % S], (p / S) & 1, kWaitLimit);
                    mbar_wait_bounded(&full[p % S], (p / S) & 1, kWaitLimit);
                }
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {
            bool ok = true;
            int q = 0, j = 0;  // stage fills consumed, units done by this CTA
            for (int t = blockIdx.x; t < n_units && ok; t += gridDim.x) {
                const Tile T = tile_of(g, t, mt, ntl, nk, BN);
                if (T.skip) continue;
                const int buf = j % nbuf, use = j / nbuf;
                ++j;
                if (use > 0 && !mbar_wait_bounded(&tempty[buf], (use - 1) & 1, wait_limit())) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t acc0 = tmem + buf * bufcols;
                for (int kb = T.kb0; kb < T.kb1; ++kb, ++q) {
                    const int s = q % S, r = q / S;
                    if (!mbar_wait_bounded(&full[s], r & 1, wait_limit())) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t ah = smem_u32(sm + s * Cfg::kStage);
                    const uint32_t al = ah + Cfg::kATile, bh = ah + 2 * Cfg::kATile, bl = bh + Cfg::kBTile;
                    // chunked K: each chunk starts its own accumulator from zero
                    const int ch = g.chunked ? kb / kTcChunkKb - T.c0 : 0;
                    const bool fresh = g.chunked ? kb % kTcChunkKb == 0 : kb == T.kb0;
                    const uint32_t acc = acc0 + (uint32_t)(ch * BN);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        const uint32_t first = fresh && kk == 0;
                        tc_mma(acc, op_desc<AMN>(ah, kk), op_desc<BMN>(bh, kk), Cfg::kIdesc, !first);
                        tc_mma(acc, op_desc<AMN>(ah, kk), op_desc<BMN>(bl, kk), Cfg::kIdesc, 1u);
                        tc_mma(acc, op_desc<AMN>(al, kk), op_desc<BMN>(bh, kk), Cfg::kIdesc, 1u);
                    }
                    tc_commit(&empty[s]);
                }
                if (ok) tc_commit(&tfull[buf]);
            }
            if (!ok) {  // no result for this unit: wait for the MMAs already issued, then leave
                abort_sh = 1;
                tc_commit(&drainb);
                mbar_wait_bounded(&drainb, 0, kWaitLimit);
            }
        }
    } else if (warp >= 6) {
        if constexpr (BQ != 0) {
            // B from the packed codes: warp w fills tile rows (w-6)*R .. of every
            // stage, LPR lanes per row, each lane 64/LPR consecutive values of the
            // row's 64-wide group.  Generic-proxy stores, then a proxy fence so the
            // tensor cores see them, then one arrival per warp on the stage's full
            // barrier.  The next slice's codes are fetched before this one is
            // expanded.
            constexpr int R = BN / 4, LPR = 32 / R, N1 = 64 / LPR;
            const int rloc = (warp - 6) * R + lane / LPR;
            const int i0 = (lane % LPR) * N1;
            const int r7 = rloc & 7;
            const int blk = rloc / 64, j = rloc % 64;
            const int RB = (g.wt.rows + 63) / 64;
            int q = 0;
            for (int t = blockIdx.x; t < n_units && !abort_sh; t += gridDim.x) {
                const Tile T = tile_of(g, t, mt, ntl, nk, BN);
                if (T.skip) continue;
                const bool have = (g.wq_row0 + T.n0) / 64 + blk < RB;  // this row's block was copied
                bool stop = false;
                for (int kb = T.kb0; kb < T.kb1; ++kb, ++q) {
                    const int s = q % S, r = q / S;
                    bool w_ok = true;
                    if (lane == 0) {
                        if (r > 0) w_ok = mbar_wait_bounded(&empty[s], (r - 1) & 1, wait_limit());
                        if (w_ok) w_ok = mbar_wait_bounded(&cfull[s], r & 1, wait_limit());
                    }
                    w_ok = __shfl_sync(kFull, w_ok ? 1 : 0, 0) != 0;
                    if (!w_ok) abort_sh = 1;
                    if (abort_sh) {
                        stop = true;
                        break;
                    }
                    const uint32_t st = smem_u32(sm + s * Cfg::kStage);
                    const uint32_t bh = st + 2 * Cfg::kATile;
                    const uint32_t hrow = bh + rloc * 128, lrow = bh + Cfg::kBTile + rloc * 128;
                    if (have) {
                        DqGroup cur;
                        dq_load(st + 2 * Cfg::kATile + 2 * Cfg::kBTile + blk * kSeg, j, cur);
                        dq_slice<N1>(cur, i0, hrow, lrow, r7);
                    } else {
                        const float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
                        for (int c = 0; c < N1 / 8; ++c) dq_put8(hrow, lrow, ((((i0 >> 3) + c) ^ r7) << 4), z);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&full[s]);
                }
                if (stop) break;
            }
        }
    } else {
        // epilogue: warp w reads tensor-memory lanes 32w .. 32w+31 = tile rows.
        // Per 32-column block: lane = tile row on the way out of tensor
        // memory, lane = column on the way to global memory.
        // TMA store path: this warp's [32 rows][32 fp32] box (4 KB, 1024-byte aligned:
        // the 128-byte swizzle); plain-store path: the padded 32 x 33 transpose
        // block.  One launch uses one of the two, so they share the bytes.
        float *ebase = reinterpret_cast<float *>(sm + S * Cfg::kStage);
        float *sb = ebase + warp * 32 * 32;
        float(*eb)[33] = reinterpret_cast<float(*)[33]>(ebase + warp * 32 * 33);
        // 16-byte stores and loads need 4-float row strides and 16-byte (8 for planes) bases
        auto al = [](const void *p, uintptr_t m) { return (reinterpret_cast<uintptr_t>(p) & m) == 0; };
        const bool vec = ((g.ldc | g.ldr | g.ldy2 | g.ldp | g.sC) & 3) == 0 && al(g.C, 15) && al(g.R, 15) &&
                         al(g.Y2, 15) && al(g.colscale, 15) && al(g.p_hi, 7) && al(g.p_lo, 7);
        int j = 0;
        for (int t = blockIdx.x; t < n_units; t += gridDim.x) {
            const Tile T = tile_of(g, t, mt, ntl, nk, BN);
            if (T.skip) continue;
            const int buf = j % nbuf, use = j / nbuf;
            ++j;
            const bool gave_up = __any_sync(kFull, abort_sh != 0);  // warp-uniform
            const bool ok = !gave_up && __all_sync(kFull, mbar_wait_bounded(&tfull[buf], use & 1, wait_limit()));
            if (!ok) {
                const int row = T.m0 + warp * 32 + lane;
                if (g.status && row < g.M) atomicOr(g.status + (int64_t)row * g.status_stride, ALTXS_ST_TIMEOUT);
                continue;
            }
            tc_fence_after();
            const bool no_k = T.kb0 >= T.kb1;  // nothing accumulated: the product is zero
            const uint32_t tl = tmem + buf * bufcols + ((uint32_t)(warp * 32) << 16);
            const int na = T.c1 - T.c0;  // accumulators of this unit
            if (g.splits == 1) {
                // the tile's chunk sums added in chunk order (one accumulator unless chunked)
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 32) {
                    float v[32];
                    __syncwarp();  // warp-collective load; the block buffer is free again
                    tc_ld32(tl + c0, v);
#pragma unroll 1
                    for (int a = 1; a < na; ++a) {
                        float w[32];
                        tc_ld32(tl + a * BN + c0, w);
#pragma unroll
                        for (int u = 0; u < 32; ++u) v[u] = __fadd_rn(v[u], w[u]);
                    }
                    if (c0 + 32 >= BN) {  // accumulators fully read: hand them back to the MMA warp
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[buf]);
                    }
                    emit_block<BN>(g, T, &tc_map, warp, lane, c0, v, no_k, eb, sb, vec);
                }
                continue;
            }
            // split K: this unit's chunk sums of the warp's 32 rows go to the
            // partials (float4 j of row `lane` at [j][lane]: every warp store is
            // 512 contiguous bytes); the slab's arrival counter picks the last
            // unit, which adds all chunk sums in chunk order and runs the epilogue
            const int nch = n_chunks(nk);
            constexpr int kSlab = 32 * BN / 4;  // float4 per warp slab of one chunk
            float4 *pbase = reinterpret_cast<float4 *>(g.part) + ((int64_t)T.id * nch * 4 + warp) * kSlab;
#pragma unroll 1
            for (int a = 0; a < na; ++a) {
                float4 *pw = pbase + (int64_t)(T.c0 + a) * 4 * kSlab;
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 32) {
                    float v[32];
                    __syncwarp();
                    tc_ld32(tl + a * BN + c0, v);
#pragma unroll
                    for (int u4 = 0; u4 < 8; ++u4)
                        __stcg(pw + (c0 / 4 + u4) * 32 + lane,
                               make_float4(v[4 * u4], v[4 * u4 + 1], v[4 * u4 + 2], v[4 * u4 + 3]));
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
            uint32_t old = 0;
            if (lane == 0) {
                // release: the warp's partials (ordered before by the warp barrier)
                // before the arrival; acquire: the other units' partials after it
                asm volatile("fence.acq_rel.gpu;" ::: "memory");
                old = atomicAdd(g.cnt + (int64_t)T.id * 4 + warp, 1u);
                asm volatile("fence.acq_rel.gpu;" ::: "memory");
            }
            old = __shfl_sync(kFull, old, 0);
            if (old != (uint32_t)g.splits - 1) continue;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                float v[32];
#pragma unroll
                for (int u4 = 0; u4 < 8; ++u4) {
                    const float4 p = __ldcg(pbase + (c0 / 4 + u4) * 32 + lane);
                    v[4 * u4] = p.x;
                    v[4 * u4 + 1] = p.y;
                    v[4 * u4 + 2] = p.z;
                    v[4 * u4 + 3] = p.w;
                }
#pragma unroll 1
                for (int c = 1; c < nch; ++c) {
                    const float4 *pr = pbase + (int64_t)c * 4 * kSlab + c0 / 4 * 32 + lane;
#pragma unroll
                    for (int u4 = 0; u4 < 8; ++u4) {
                        const float4 p = __ldcg(pr + u4 * 32);
                        v[4 * u4] = __fadd_rn(v[4 * u4], p.x);
                        v[4 * u4 + 1] = __fadd_rn(v[4 * u4 + 1], p.y);
                        v[4 * u4 + 2] = __fadd_rn(v[4 * u4 + 2], p.z);
                        v[4 * u4 + 3] = __fadd_rn(v[4 * u4 + 3], p.w);
                    }
                }
                __syncwarp();
                emit_block<BN>(g, T, &tc_map, warp, lane, c0, v, false, eb, sb, vec);
            }
            if (lane == 0) g.cnt[(int64_t)T.id * 4 + warp] = 0;  // ready for the next launch
        }
        if (g.tma_c && lane == 0) bulk_wait_all();  // every tensor store of this warp has landed
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols)
                     : "memory");
    }
}

__global__ void k_split_weights(altxs_qmat W, uint16_t *hi, uint16_t *lo) {
    const int row = blockIdx.x;
    for (int k = threadIdx.x; k < W.cols; k += blockDim.x)
        split_store(hi, lo, (int64_t)row * W.cols + k, qmat_elem(W, row, k));
}

// 8 consecutive output columns per thread (one 16-byte store per plane);
// planes compact [nb][rows][ldo], ldo a multiple of 8, zero past cols
__global__ void k_split_f32(const float *src, int64_t cols, int64_t ld, int64_t bs, int64_t rows, int64_t ldo,
                            int64_t n8, uint16_t *hi, uint16_t *lo) {
    const int64_t g8 = ldo / 8;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c0 = (i % g8) * 8, br = i / g8, r = br % rows, b = br / rows;
        const float *s = src + b * bs + r * ld;
        uint32_t h[4], l[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t c = c0 + 2 * u;
            const float v0 = c < cols ? s[c] : 0.0f, v1 = c + 1 < cols ? s[c + 1] : 0.0f;
            const __nv_bfloat16 h0 = __float2bfloat16_rn(v0), h1 = __float2bfloat16_rn(v1);
            const __nv_bfloat16 l0 = __float2bfloat16_rn(__fsub_rn(v0, __bfloat162float(h0)));
            const __nv_bfloat16 l1 = __float2bfloat16_rn(__fsub_rn(v1, __bfloat162float(h1)));
            h[u] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
            l[u] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
        }
        const int64_t o = br * ldo + c0;
        *reinterpret_cast<uint4 *>(hi + o) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4 *>(lo + o) = make_uint4(l[0], l[1], l[2], l[3]);
    }
}

// 3-D bf16 tensor map over [nb][rows][cols], box 64 (cols) x box_rows x 1, 128-byte swizzle
bool make_map(CUtensorMap *m, const uint16_t *p, const TcOp &o, int box_rows) {
    auto enc = encoder();
    if (!enc) return false;
    cuuint64_t dims[3] = {(cuuint64_t)o.cols, (cuuint64_t)o.rows, (cuuint64_t)(o.nb > 0 ? o.nb : 1)};
    cuuint64_t strides[2] = {(cuuint64_t)(o.ld * 2), (cuuint64_t)((o.bstride > 0 ? o.bstride : o.ld * o.rows) * 2)};
    cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<uint16_t *>(p), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Tensor map of C ([batch][M][ldc] fp32, boxes of 32 x 32, 128-byte swizzle)
// when the epilogue is a plain store that TMA can take: no accumulation into
// C, no residual, second output or planes, 16-byte aligned base and strides.
bool make_c_map(CUtensorMap *m, const TcGemm &g) {
    if (!g.C || g.epi != kEpiStore || g.beta != 0.0f || g.Y2 || g.p_hi || g.R) return false;
    if (!aligned16(g.C) || g.ldc % 4 || g.ldc < g.N || (g.batch > 1 && (g.sC % 4 || g.sC < g.ldc * g.M))) return false;
    auto enc = encoder();
    if (!enc) return false;
    cuuint64_t dims[3] = {(cuuint64_t)g.N, (cuuint64_t)g.M, (cuuint64_t)g.batch};
    const int64_t bs = g.batch > 1 ? g.sC : g.ldc * (int64_t)g.M;
    cuuint64_t strides[2] = {(cuuint64_t)(g.ldc * 4), (cuuint64_t)(bs * 4)};
    cuuint32_t box[3] = {32, 32, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, g.C, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool op_ok(const TcOp &o) {
    if (!o.hi || !o.lo || !aligned16(o.hi) || !aligned16(o.lo)) return false;
    if (o.ld % 8 || o.ld < o.cols || o.rows < 1 || o.cols < 1 || o.div < 1 || o.mul < 0 || o.add < 0) return false;
    if (o.nb > 1 && o.bstride % 8) return false;
    return o.row_off >= 0;
}

template <int BN, int AMN, int BMN, int BQ>
int launch_cfg(const TcGemm &g, int sms, cudaStream_t st) {
    using Cfg = TcCfg<BN, AMN, BMN, BQ>;
    static std::mutex mu;
    static bool attr_done[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ALTXS_ECUDA;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!attr_done[dev]) {
            if (cudaFuncSetAttribute(k_tc_gemm<BN, AMN, BMN, BQ>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     Cfg::kSmem) != cudaSuccess)
                return ALTXS_ECUDA;
            attr_done[dev] = true;
        }
    }
    CUtensorMap ta_hi, ta_lo, tb_hi, tb_lo, tc_map;
    const int abox = AMN ? 64 : kBM, bbox = BMN ? 64 : BN;
    if (!make_map(&ta_hi, g.a.hi, g.a, abox) || !make_map(&ta_lo, g.a.lo, g.a, abox)) return ALTXS_EINVAL;
    if (BQ) {
        tb_hi = ta_hi;  // unused: the producer warps expand B from the packed codes
        tb_lo = ta_lo;
    } else if (!make_map(&tb_hi, g.b.hi, g.b, bbox) || !make_map(&tb_lo, g.b.lo, g.b, bbox)) {
        return ALTXS_EINVAL;
    }
    TcGemm gk = g;
    gk.tma_c = make_c_map(&tc_map, g) ? 1 : 0;
    if (!gk.tma_c) tc_map = ta_hi;  // unused
    // persistent: at most one CTA per SM walks the units
    const int64_t units = (int64_t)((g.M + kBM - 1) / kBM) * ((g.N + BN - 1) / BN) * g.batch * g.splits;
    const int grid = (int)(units < sms ? units : sms);
    ALTXS_LAUNCH(::altxs::kKQmm, st,
                 k_tc_gemm<BN, AMN, BMN, BQ><<<grid, TcThreads<BQ>::kN, Cfg::kSmem, st>>>(ta_hi, ta_lo, tb_hi, tb_lo,
                                                                                          tc_map, gk));
    return ALTXS_OK;
}

template <int BN>
int launch_bn(const TcGemm &g, int sms, cudaStream_t st) {
    if (g.bq) return g.a.mn_major ? launch_cfg<BN, 1, 0, 1>(g, sms, st) : launch_cfg<BN, 0, 0, 1>(g, sms, st);
    if (!g.a.mn_major && !g.b.mn_major) return launch_cfg<BN, 0, 0, 0>(g, sms, st);
    if (!g.a.mn_major && g.b.mn_major) return launch_cfg<BN, 0, 1, 0>(g, sms, st);
    if (g.a.mn_major && !g.b.mn_major) return launch_cfg<BN, 1, 0, 0>(g, sms, st);
    return launch_cfg<BN, 1, 1, 0>(g, sms, st);
}

}  // namespace

int launch_tc_gemm(const TcGemm &g0, cudaStream_t st) {
    TcGemm g = g0;
    if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return ALTXS_OK;
    if (g.K <= 0 || !op_ok(g.a) || (!g.bq && !op_ok(g.b))) return ALTXS_EINVAL;
    if (g.causal < 0 || g.causal > 3) return ALTXS_EINVAL;
    if (g.bq && (!g.wt.data || g.wt.cols != g.K || g.K % kBK || g.wq_row0 < 0 || g.wq_row0 % 64 ||
                 g.wq_row0 + g.N > g.wt.rows || g.batch != 1 || g.b.mn_major ||
                 (reinterpret_cast<uintptr_t>(g.wt.data) & 15)))
        return ALTXS_EINVAL;
    if (g.epi == kEpiResid && (!g.R || !g.colscale || g.batch != 1)) return ALTXS_EINVAL;
    if ((g.p_hi && (!g.p_lo || g.ldp < g.N || g.batch != 1)) || (g.Y2 && g.batch != 1)) return ALTXS_EINVAL;
    if (g.beta != 0.0f && !g.C) return ALTXS_EINVAL;
    // the K extent of each operand must be covered by its stored array (zeros beyond come from the bounds)
    const int64_t ka = g.a.mn_major ? g.a.rows - g.a.row_off : g.a.cols;
    const int64_t kbx = g.bq ? g.wt.cols : g.b.mn_major ? g.b.rows - g.b.row_off : g.b.cols;
    if (ka < g.K || kbx < g.K) return ALTXS_EINVAL;
    // a K slice reads 64 values: past K they must come from the bounds (zeros), not from stored data
    if (g.K % kBK && (ka != g.K || kbx != g.K)) return ALTXS_EINVAL;
    static int sms[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return ALTXS_ECUDA;
    if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    const int64_t mt = (g.M + kBM - 1) / kBM;
    // chunked K: every chunk's accumulator stays in tensor memory until the epilogue
    const int nk = (g.K + kBK - 1) / kBK, nch = (nk + kTcChunkKb - 1) / kTcChunkKb;
    if (g.chunked && (g.causal != 0 || nch > kTcMaxChunks)) return ALTXS_EINVAL;
    g.splits = 1;
    // wide tiles when they still fill the device (and their chunks fit twice in
    // tensor memory), narrow ones otherwise
    if (mt * ((g.N + 127) / 128) * g.batch >= sms[dev] && (!g.chunked || nch <= 2))
        return launch_bn<128>(g, sms[dev], st);
    // few tiles: spread each tile's chunks over more CTAs (the sums do not depend on it)
    const int64_t tiles = mt * ((g.N + 63) / 64) * g.batch;
    if (g.chunked && g.part && g.cnt && nch >= 2 && tiles <= kTcSplitTiles && 2 * tiles <= sms[dev]) {
        if ((reinterpret_cast<uintptr_t>(g.part) & 15) || (reinterpret_cast<uintptr_t>(g.cnt) & 3))
            return ALTXS_EINVAL;
        const int s0 = (int)(sms[dev] / tiles < nch ? sms[dev] / tiles : nch);
        const int per = (nch + s0 - 1) / s0;
        g.splits = (nch + per - 1) / per;  // no unit without a chunk
    }
    return launch_bn<64>(g, sms[dev], st);
}

int launch_tc(const TcArgs &a, cudaStream_t st) {
    TcGemm g{};
    g.a.hi = a.a_hi;
    g.a.lo = a.a_lo;
    g.a.rows = a.M;
    g.a.cols = a.K;
    g.a.ld = a.lda;
    g.a.nb = 1;
    g.a.div = g.a.mul = 1;
    g.b.hi = a.b_hi;
    g.b.lo = a.b_lo;
    g.b.rows = a.b_rows;
    g.b.cols = a.K;
    g.b.ld = a.K;
    g.b.nb = 1;
    g.b.row_off = a.row0;
    g.b.div = g.b.mul = 1;
    if (a.row0 < 0 || a.row0 + a.N > a.b_rows || a.K % kBK) return ALTXS_EINVAL;
    g.M = a.M;
    g.N = a.N;
    g.K = a.K;
    g.batch = 1;
    g.alpha = 1.0f;
    g.epi = a.epi;
    g.C = a.Y;
    g.ldc = a.ldy;
    g.R = a.R;
    g.ldr = a.ldr;
    g.colscale = a.colscale;
    g.Y2 = a.Y2;
    g.ldy2 = a.ldy2;
    g.p_hi = a.p_hi;
    g.p_lo = a.p_lo;
    g.ldp = a.ldp;
    g.status = a.status;
    g.status_stride = a.status_stride;
    if (a.wt) {
        g.bq = 1;
        g.wt = *a.wt;
        g.wq_row0 = a.row0;
    }
    // chunked K whenever the chunks fit in tensor memory: a row's bits are then
    // the same whether its tile's K loop runs on one CTA or is split
    g.chunked = (a.K / kBK + kTcChunkKb - 1) / kTcChunkKb <= kTcMaxChunks ? 1 : 0;
    g.part = a.part;
    g.cnt = a.cnt;
    return launch_tc_gemm(g, st);
}

int64_t tc_linear_part_elems(int M, int N, int K) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    const int64_t nch = ((K + kBK - 1) / kBK + kTcChunkKb - 1) / kTcChunkKb;
    const int64_t tiles = (int64_t)((M + kBM - 1) / kBM) * ((N + 63) / 64);
    if (nch < 2 || nch > kTcMaxChunks || tiles > kTcSplitTiles) return 0;
    return tiles * nch * kBM * 64;
}

int64_t tc_linear_cnt_elems(int M, int N, int K) {
    if (tc_linear_part_elems(M, N, K) == 0) return 0;
    return (int64_t)((M + kBM - 1) / kBM) * ((N + 63) / 64) * 4;
}

int set_wait_limit_tc(uint32_t limit) {
    return cudaMemcpyToSymbol(g_wait_limit, &limit, sizeof(limit)) == cudaSuccess ? ALTXS_OK : ALTXS_ECUDA;
}

int launch_split_weights(const altxs_qmat &W, uint16_t *hi, uint16_t *lo, cudaStream_t st) {
    if (!hi || !lo || W.rows <= 0 || W.cols <= 0 || W.cols % 64) return ALTXS_EINVAL;
    ALTXS_LAUNCH(::altxs::kKQmm, st, k_split_weights<<<W.rows, 256, 0, st>>>(W, hi, lo));
    return ALTXS_OK;
}

int launch_split_f32(const float *src, int64_t rows, int64_t cols, int64_t ld, int nb, int64_t bs, uint16_t *hi,
                     uint16_t *lo, cudaStream_t st, int kernel_class) {
    if (rows <= 0 || cols <= 0 || nb <= 0) return ALTXS_OK;
    if (!src || !hi || !lo) return ALTXS_EINVAL;
    const int64_t ldo = align_up(cols, 8), n8 = (int64_t)nb * rows * (ldo / 8);
    if (!aligned16(hi) || !aligned16(lo)) return ALTXS_EINVAL;
    const int64_t blocks = (n8 + 255) / 256;
    const unsigned grid = (unsigned)(blocks < 148 * 16 ? blocks : 148 * 16);
    ALTXS_LAUNCH(kernel_class, st, k_split_f32<<<grid, 256, 0, st>>>(src, cols, ld, bs, rows, ldo, n8, hi, lo));
    return ALTXS_OK;
}

namespace {

// stored shape of an fp32 GemmArgs operand: op(A) is M x K, stored [M][lda] or [K][lda] (tA)
struct F32Op {
    int64_t rows, cols, ldo, nb;
};
F32Op f32_a(const GemmArgs &g) {
    F32Op o;
    o.rows = g.tA ? g.K : g.M;
    o.cols = g.tA ? g.M : g.K;
    o.ldo = align_up(o.cols, 8);
    o.nb = (g.batch + g.adiv - 1) / g.adiv;
    return o;
}
// op(B) is K x N, stored [K][ldb] or [N][ldb] (tB)
F32Op f32_b(const GemmArgs &g) {
    F32Op o;
    o.rows = g.tB ? g.N : g.K;
    o.cols = g.tB ? g.K : g.N;
    o.ldo = align_up(o.cols, 8);
    o.nb = (g.batch + g.bdiv - 1) / g.bdiv;
    return o;
}

}  // namespace

void tc_f32_scratch(const GemmArgs &g, int64_t *a_elems, int64_t *b_elems) {
    const F32Op a = f32_a(g), b = f32_b(g);
    *a_elems = 2 * align_up(a.nb * a.rows * a.ldo, 128);
    *b_elems = 2 * align_up(b.nb * b.rows * b.ldo, 128);
}

int tc_gemm_f32(const GemmArgs &g, uint16_t *a_scr, int64_t a_elems, uint16_t *b_scr, int64_t b_elems,
                cudaStream_t st, int kernel_class) {
    if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return ALTXS_OK;
    if (g.K <= 0 || g.adiv < 1 || g.bdiv < 1) return ALTXS_EINVAL;
    int64_t need_a, need_b;
    tc_f32_scratch(g, &need_a, &need_b);
    if (!a_scr || !b_scr || a_elems < need_a || b_elems < need_b) return ALTXS_EINVAL;
    const F32Op a = f32_a(g), b = f32_b(g);
    uint16_t *ahi = a_scr, *alo = a_scr + need_a / 2, *bhi = b_scr, *blo = b_scr + need_b / 2;
    int rc = launch_split_f32(g.A, a.rows, a.cols, g.lda, (int)a.nb, g.sA, ahi, alo, st, kernel_class);
    if (rc) return rc;
    rc = launch_split_f32(g.B, b.rows, b.cols, g.ldb, (int)b.nb, g.sB, bhi, blo, st, kernel_class);
    if (rc) return rc;
    TcGemm t{};
    t.a = TcOp{ahi, alo, g.tA ? 1 : 0, a.rows, a.cols, a.ldo, a.rows * a.ldo, (int)a.nb, 0, g.adiv, 1, 0};
    // tc reads B as [n][k]: stored [N][K] (tB) is K-major, stored [K][N] is MN-major
    t.b = TcOp{bhi, blo, g.tB ? 0 : 1, b.rows, b.cols, b.ldo, b.rows * b.ldo, (int)b.nb, 0, g.bdiv, 1, 0};
    t.M = g.M;
    t.N = g.N;
    t.K = g.K;
    t.batch = g.batch;
    t.causal = g.causal;
    t.alpha = g.alpha;
    t.beta = g.beta;
    t.epi = kEpiStore;
    t.C = g.C;
    t.ldc = g.ldc;
    t.sC = g.sC;
    return launch_tc_gemm(t, st);
}

}  // namespace altxs

// ---------------------------------------------------------------------------
namespace {

__global__ void k_split_rows(const float *X, int64_t ldx, int K, uint16_t *hi, uint16_t *lo) {
    const int64_t m = blockIdx.x;
    for (int k = threadIdx.x; k < K; k += blockDim.x) altxs::split_store(hi, lo, m * K + k, X[m * ldx + k]);
}

// X planes [M][K] x 2, then (when the call can split K) the partials and the
// arrival counters; the counters are zeroed on the stream.
int linear_scratch(void *workspace, int64_t bytes, int M, int N, int K, bool want_split, uint16_t **xh,
                   uint16_t **xl, altxs::TcArgs &t, cudaStream_t st) {
    using namespace altxs;
    unsigned char *p = static_cast<unsigned char *>(workspace);
    const int64_t xb = align_up((int64_t)M * K * 2, 256);
    *xh = reinterpret_cast<uint16_t *>(p);
    *xl = reinterpret_cast<uint16_t *>(p + xb);
    const int64_t pe = tc_linear_part_elems(M, N, K), ce = tc_linear_cnt_elems(M, N, K);
    if (!want_split || pe == 0 || bytes < altxs_linear_tc_workspace_bytes(M, N, K)) return ALTXS_OK;
    t.part = reinterpret_cast<float *>(p + 2 * xb);
    t.cnt = reinterpret_cast<uint32_t *>(p + 2 * xb + align_up(pe * 4, 256));
    return cudaMemsetAsync(t.cnt, 0, ce * 4, st) == cudaSuccess ? ALTXS_OK : ALTXS_ECUDA;
}
}  // namespace

extern "C" {

int altxs_split_weights(const altxs_qmat *m, uint16_t *hi, uint16_t *lo, altxs_stream_t stream) {
    if (!m) return ALTXS_EINVAL;
    if ((reinterpret_cast<uintptr_t>(hi) | reinterpret_cast<uintptr_t>(lo)) & 15) return ALTXS_EINVAL;
    return altxs::launch_split_weights(*m, hi, lo, reinterpret_cast<cudaStream_t>(stream));
}

int64_t altxs_gemm_workspace_bytes(int M, int N, int K, int tA, int tB, int batch) {
    if (M < 0 || N < 0 || K < 0 || batch < 0) return -1;
    altxs::GemmArgs g{};
    g.M = M;
    g.N = N;
    g.K = K;
    g.tA = tA;
    g.tB = tB;
    g.batch = batch;
    g.adiv = g.bdiv = 1;
    int64_t a, b;
    altxs::tc_f32_scratch(g, &a, &b);
    return altxs::align_up(a * 2, 256) + altxs::align_up(b * 2, 256);
}

int altxs_gemm(int M, int N, int K, const float *A, int64_t lda, int64_t sA, int tA, const float *B, int64_t ldb,
               int64_t sB, int tB, float *C, int64_t ldc, int64_t sC, int batch, float alpha, float beta, int causal,
               void *workspace, int64_t workspace_bytes, altxs_stream_t stream) {
    using namespace altxs;
    if (M < 0 || N < 0 || K < 0 || batch < 0 || !A || !B || !C || (tA | tB) & ~1) return ALTXS_EINVAL;
    if (M == 0 || N == 0 || batch == 0) return ALTXS_OK;
    if (workspace_bytes < altxs_gemm_workspace_bytes(M, N, K, tA, tB, batch) || !workspace) return ALTXS_EINVAL;
    GemmArgs g{};
    g.A = A;
    g.B = B;
    g.C = C;
    g.M = M;
    g.N = N;
    g.K = K;
    g.lda = lda;
    g.ldb = ldb;
    g.ldc = ldc;
    g.sA = sA;
    g.sB = sB;
    g.sC = sC;
    g.tA = tA;
    g.tB = tB;
    g.batch = batch;
    g.adiv = g.bdiv = 1;
    g.alpha = alpha;
    g.beta = beta;
    g.causal = causal;
    int64_t a, b;
    tc_f32_scratch(g, &a, &b);
    uint16_t *as = static_cast<uint16_t *>(workspace);
    uint16_t *bs = reinterpret_cast<uint16_t *>(static_cast<unsigned char *>(workspace) + align_up(a * 2, 256));
    return tc_gemm_f32(g, as, a, bs, b, reinterpret_cast<cudaStream_t>(stream), kKQmm);
}

int64_t altxs_linear_workspace_bytes(int M, int K) {
    if (M < 0 || K < 0) return -1;
    return altxs::align_up((int64_t)M * K * 2, 256) * 2;
}


int altxs_linear(const altxs_qmat *m, const uint16_t *w_hi, const uint16_t *w_lo, int row0, int N, const float *X,
                 int M, float *Y, void *workspace, int64_t workspace_bytes, altxs_stream_t stream) {
    using namespace altxs;
    if (!m || !X || !Y || M < 0 || N < 0 || row0 < 0 || row0 + N > m->rows) return ALTXS_EINVAL;
    if (M == 0 || N == 0) return ALTXS_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (!w_hi || !w_lo) {
        QmmArgs a{};
        a.X = X;
        a.ldx = m->cols;
        a.M = M;
        a.W = *m;
        a.row0 = row0;
        a.N = N;
        a.K = m->cols;
        a.Y = Y;
        a.ldy = N;
        a.epi = kEpiStore;
        return launch_qmm(a, st);
    }
    const int K = m->cols;
    if (!workspace || workspace_bytes < altxs_linear_workspace_bytes(M, K)) return ALTXS_EINVAL;
    TcArgs t{};
    uint16_t *xh, *xl;
    const int rc = linear_scratch(workspace, workspace_bytes, M, N, K, true, &xh, &xl, t, st);
    if (rc != ALTXS_OK) return rc;
    ALTXS_LAUNCH(::altxs::kKQmm, st, k_split_rows<<<M, 256, 0, st>>>(X, K, K, xh, xl));
    t.a_hi = xh;
    t.a_lo = xl;
    t.lda = K;
    t.M = M;
    t.b_hi = w_hi;
    t.b_lo = w_lo;
    t.b_rows = m->rows;
    t.row0 = row0;
    t.N = N;
    t.K = K;
    t.epi = kEpiStore;
    t.Y = Y;
    t.ldy = N;
    return launch_tc(t, st);
}

int64_t altxs_linear_tc_workspace_bytes(int M, int N, int K) {
    using namespace altxs;
    if (M < 0 || N < 0 || K < 0) return -1;
    return align_up((int64_t)M * K * 2, 256) * 2 + align_up(tc_linear_part_elems(M, N, K) * 4, 256) +
           align_up(tc_linear_cnt_elems(M, N, K) * 4, 256);
}

int altxs_linear_tc(const altxs_qtiles *w, int row0, int N, const float *X, int M, float *Y, void *workspace,
                    int64_t workspace_bytes, altxs_stream_t stream) {
    using namespace altxs;
    if (!w || !X || !Y || M < 0 || N < 0 || row0 < 0 || row0 + N > w->rows) return ALTXS_EINVAL;
    if (M == 0 || N == 0) return ALTXS_OK;
    const int K = w->cols;
    if (!workspace || workspace_bytes < altxs_linear_tc_workspace_bytes(M, N, K)) return ALTXS_EINVAL;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    TcArgs t{};
    uint16_t *xh, *xl;
    const int rc = linear_scratch(workspace, workspace_bytes, M, N, K, true, &xh, &xl, t, st);
    if (rc != ALTXS_OK) return rc;
    ALTXS_LAUNCH(::altxs::kKQmm, st, k_split_rows<<<M, 256, 0, st>>>(X, K, K, xh, xl));
    t.a_hi = xh;
    t.a_lo = xl;
    t.lda = K;
    t.M = M;
    t.b_rows = w->rows;
    t.row0 = row0;
    t.N = N;
    t.K = K;
    t.epi = kEpiStore;
    t.Y = Y;
    t.ldy = N;
    t.wt = w;
    return launch_tc(t, st);
}

}  // extern "C"
