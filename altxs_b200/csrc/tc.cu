// tcgen05 tensor-core GEMM for the mixed-bit linear layers (sm_100a).
//
// Y[m][n] = epi( sum_k X[m][k] W[row0+n][k] ) with X and W given as hi/lo
// bf16 planes (tc.cuh).  One CTA computes a 128 x BN tile:
//   warp 4      TMA producer: the four K-major tiles (X hi, X lo, W hi, W lo)
//               of each 64-wide K slice into a ring of shared-memory stages
//               (128-byte swizzle), one mbarrier per stage (full / empty);
//   warp 5      MMA issuer: one thread issues tcgen05.mma (kind::f16, bf16 in,
//               fp32 accumulate in tensor memory) for Xhi*Whi, Xhi*Wlo, Xlo*Whi
//               over the four 16-wide K steps of a stage, then tcgen05.commit
//               frees the stage; a final commit signals the epilogue;
//   warps 0-3   epilogue: tcgen05.ld of the accumulator (one tile row per
//               thread), the layer's epilogue, stores.
// Every wait is bounded; a wait that gives up marks the rows of the tile with
// ALTXS_ST_TIMEOUT (when a status array is given), lets the CTA's own copies
// and MMAs drain (bounded) and frees the tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "model.cuh"
#include "prof.cuh"
#include "qmm.cuh"
#include "tc.cuh"

namespace altxs {
namespace {

constexpr int kBM = 128;         // tile rows = tensor-memory lanes
constexpr int kBK = 64;          // K per stage: one 128-byte swizzle row of bf16
constexpr int kTcThreads = 192;  // warps 0-3 epilogue, 4 producer, 5 MMA
constexpr unsigned kFull = 0xffffffffu;

template <int BN>
struct TcCfg {
    static constexpr int kATile = kBM * kBK * 2;  // bytes of one X plane tile
    static constexpr int kBTile = BN * kBK * 2;   // bytes of one W plane tile
    static constexpr int kStage = 2 * kATile + 2 * kBTile;
    static constexpr int kStages = (192 * 1024) / kStage;  // BN 64: 4, 128: 3, 256: 2
    static constexpr int kSmem = kStages * kStage + 1024;  // + alignment slack
    static constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
    // kind::f16 instruction descriptor: fp32 accumulate, bf16 A and B, both
    // K-major, M = 128, N = BN
    static constexpr uint32_t kIdesc =
        (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
};

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory matrix descriptor of a K-major tile written by TMA with the
// 128-byte swizzle: 8-row x 128-byte swizzle atoms stacked every 1024 bytes.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);  // start address
    d |= (uint64_t)1 << 16;                           // leading byte offset (unused for this layout)
    d |= (uint64_t)(1024 >> 4) << 32;                 // stride byte offset: next 8-row group
    d |= (uint64_t)1 << 46;                           // descriptor version
    d |= (uint64_t)2 << 61;                           // 128-byte swizzle
    return d;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

// arrives once on `bar` when every tcgen05 operation issued so far by this thread has completed
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 8 consecutive fp32 accumulator columns of this thread's tensor-memory lane
__device__ __forceinline__ void tc_ld8(uint32_t taddr, float *v) {
    uint32_t r0, r1, r2, r3, r4, r5, r6, r7;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3), "=r"(r4), "=r"(r5), "=r"(r6), "=r"(r7)
                 : "r"(taddr));
    // the registers are defined once the wait returns: tie them to it
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r0), "+r"(r1), "+r"(r2), "+r"(r3), "+r"(r4), "+r"(r5), "+r"(r6), "+r"(r7)::"memory");
    v[0] = __uint_as_float(r0), v[1] = __uint_as_float(r1), v[2] = __uint_as_float(r2), v[3] = __uint_as_float(r3);
    v[4] = __uint_as_float(r4), v[5] = __uint_as_float(r5), v[6] = __uint_as_float(r6), v[7] = __uint_as_float(r7);
}

__device__ __forceinline__ float leaky2(float v) {  // leaky_relu(v, 0.5)^2 (model.py:874-882)
    const float t = v >= 0.0f ? v : __fmul_rn(v, 0.5f);
    return __fmul_rn(t, t);
}

template <int BN>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_tc_gemm(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
              const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo, TcArgs a) {
    using Cfg = TcCfg<BN>;
    constexpr int S = Cfg::kStages;
    extern __shared__ unsigned char tc_smem_raw[];
    __shared__ __align__(8) uint64_t full[S], empty[S], accb, drainb;
    __shared__ uint32_t tmem_sh;
    __shared__ volatile int abort_sh;
    const uint32_t raw_s = smem_u32(tc_smem_raw);
    unsigned char *sm = tc_smem_raw + ((1024u - (raw_s & 1023u)) & 1023u);  // 1024-byte aligned stages
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * BN;
    const int nk = a.K / kBK;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&accb, 1);
        mbar_init(&drainb, 1);
        abort_sh = 0;
        fence_mbar_init();
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_sh)),
                     "r"(Cfg::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_sh;

    if (warp == 4) {
        if (lane == 0) {
            int issued = 0;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % S, r = kb / S;
                if (r > 0 && !mbar_wait_bounded(&empty[s], (r - 1) & 1, kWaitLimit)) {
                    abort_sh = 1;
                    break;
                }
                if (abort_sh) break;
                unsigned char *st = sm + s * Cfg::kStage;
                mbar_expect_tx(&full[s], Cfg::kStage);
                tma_load_2d(st, &ta_hi, kb * kBK, m0, &full[s]);
                tma_load_2d(st + Cfg::kATile, &ta_lo, kb * kBK, m0, &full[s]);
                tma_load_2d(st + 2 * Cfg::kATile, &tb_hi, kb * kBK, a.row0 + n0, &full[s]);
                tma_load_2d(st + 2 * Cfg::kATile + Cfg::kBTile, &tb_lo, kb * kBK, a.row0 + n0, &full[s]);
                issued = kb + 1;
            }
            if (abort_sh) {  // let this CTA's copies land before the CTA can exit
                for (int kb = issued - S > 0 ? issued - S : 0; kb < issued; ++kb)
                    mbar_wait_bounded(&full[kb % S], (kb / S) & 1, kWaitLimit);
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {
            bool ok = true;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % S, r = kb / S;
                if (!mbar_wait_bounded(&full[s], r & 1, kWaitLimit)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t ah = smem_u32(sm + s * Cfg::kStage);
                const uint32_t al = ah + Cfg::kATile, bh = ah + 2 * Cfg::kATile, bl = bh + Cfg::kBTile;
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    const uint32_t off = kk * 32;  // 16 bf16 along K
                    tc_mma(tmem, sw128_desc(ah + off), sw128_desc(bh + off), Cfg::kIdesc, (kb | kk) != 0);
                    tc_mma(tmem, sw128_desc(ah + off), sw128_desc(bl + off), Cfg::kIdesc, 1u);
                    tc_mma(tmem, sw128_desc(al + off), sw128_desc(bh + off), Cfg::kIdesc, 1u);
                }
                tc_commit(&empty[s]);
            }
            if (ok) {
                tc_commit(&accb);
            } else {  // no result: wait for the MMAs already issued, then leave
                abort_sh = 1;
                tc_commit(&drainb);
                mbar_wait_bounded(&drainb, 0, kWaitLimit);
            }
        }
    } else {
        // epilogue: warp w reads tensor-memory lanes 32w .. 32w+31 = tile rows
        const bool ok = __all_sync(kFull, mbar_wait_bounded(&accb, 0, kWaitLimit));
        tc_fence_after();
        const int row = m0 + warp * 32 + lane;
        if (ok) {
            const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 8) {
                float v[8];
                __syncwarp();  // the load below is warp-collective
                tc_ld8(tl + c0, v);
                const int n = n0 + c0;
                if (row >= a.M || n >= a.N) continue;
                const int cnt = a.N - n < 8 ? a.N - n : 8;
                if (a.epi == kEpiLeaky2) {
#pragma unroll
                    for (int u = 0; u < 8; ++u) v[u] = leaky2(v[u]);
                } else if (a.epi == kEpiResid) {
                    const float *rr = a.R + (int64_t)row * a.ldr + n;
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        if (u < cnt) v[u] = __fadd_rn(rr[u], __fmul_rn(a.colscale[n + u], v[u]));
                }
                if (a.Y) {
                    float *yy = a.Y + (int64_t)row * a.ldy + n;
                    for (int u = 0; u < cnt; ++u) yy[u] = v[u];
                }
                if (a.Y2) {
                    float *yy = a.Y2 + (int64_t)row * a.ldy2 + n;
                    for (int u = 0; u < cnt; ++u) yy[u] = v[u];
                }
                if (a.p_hi) {
                    for (int u = 0; u < cnt; ++u) split_store(a.p_hi, a.p_lo, (int64_t)row * a.ldp + n + u, v[u]);
                }
            }
        } else if (a.status && row < a.M) {
            atomicOr(a.status + (int64_t)row * a.status_stride, ALTXS_ST_TIMEOUT);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Cfg::kTmemCols)
                     : "memory");
    }
}

__global__ void k_split_weights(altxs_qmat W, uint16_t *hi, uint16_t *lo) {
    const int row = blockIdx.x;
    for (int k = threadIdx.x; k < W.cols; k += blockDim.x)
        split_store(hi, lo, (int64_t)row * W.cols + k, qmat_elem(W, row, k));
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D bf16 tensor map over [rows][cols] (row stride ld elements), box 64 x box_rows, 128-byte swizzle
bool make_map(CUtensorMap *m, const uint16_t *p, int64_t cols, int64_t rows, int64_t ld, int box_rows) {
    auto enc = encoder();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
    cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t *>(p), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
int launch_bn(const TcArgs &a, cudaStream_t st) {
    using Cfg = TcCfg<BN>;
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return ALTXS_ECUDA;
    if (!attr_done[dev]) {
        if (cudaFuncSetAttribute(k_tc_gemm<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem) !=
            cudaSuccess)
            return ALTXS_ECUDA;
        attr_done[dev] = true;
    }
    CUtensorMap ta_hi, ta_lo, tb_hi, tb_lo;
    if (!make_map(&ta_hi, a.a_hi, a.K, a.M, a.lda, kBM) || !make_map(&ta_lo, a.a_lo, a.K, a.M, a.lda, kBM) ||
        !make_map(&tb_hi, a.b_hi, a.K, a.b_rows, a.K, BN) || !make_map(&tb_lo, a.b_lo, a.K, a.b_rows, a.K, BN))
        return ALTXS_EINVAL;
    dim3 grid((a.M + kBM - 1) / kBM, (a.N + BN - 1) / BN);
    ALTXS_LAUNCH(::altxs::kKQmm, st, k_tc_gemm<BN><<<grid, kTcThreads, Cfg::kSmem, st>>>(ta_hi, ta_lo, tb_hi, tb_lo, a));
    return ALTXS_OK;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

int launch_tc(const TcArgs &a, cudaStream_t st) {
    if (a.M <= 0 || a.N <= 0) return ALTXS_OK;
    if (a.K <= 0 || a.K % kBK || a.lda % 8 || a.lda < a.K || a.row0 < 0 || a.row0 + a.N > a.b_rows) return ALTXS_EINVAL;
    if (!a.a_hi || !a.a_lo || !a.b_hi || !a.b_lo || !aligned16(a.a_hi) || !aligned16(a.a_lo) || !aligned16(a.b_hi) ||
        !aligned16(a.b_lo))
        return ALTXS_EINVAL;
    if (a.p_hi && (!a.p_lo || a.ldp < a.N)) return ALTXS_EINVAL;
    if (a.epi == kEpiResid && (!a.R || !a.colscale)) return ALTXS_EINVAL;
    static int sms[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return ALTXS_ECUDA;
    if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    const int64_t mt = (a.M + kBM - 1) / kBM;
    // wide tiles when they still fill the device, narrow ones otherwise
    if (mt * ((a.N + 127) / 128) >= sms[dev]) return launch_bn<128>(a, st);
    return launch_bn<64>(a, st);
}

int launch_split_weights(const altxs_qmat &W, uint16_t *hi, uint16_t *lo, cudaStream_t st) {
    if (!hi || !lo || W.rows <= 0 || W.cols <= 0 || W.cols % 64) return ALTXS_EINVAL;
    ALTXS_LAUNCH(::altxs::kKQmm, st, k_split_weights<<<W.rows, 256, 0, st>>>(W, hi, lo));
    return ALTXS_OK;
}

}  // namespace altxs

// ---------------------------------------------------------------------------
namespace {

__global__ void k_split_rows(const float *X, int64_t ldx, int K, uint16_t *hi, uint16_t *lo) {
    const int64_t m = blockIdx.x;
    for (int k = threadIdx.x; k < K; k += blockDim.x) altxs::split_store(hi, lo, m * K + k, X[m * ldx + k]);
}

}  // namespace

extern "C" {

int altxs_split_weights(const altxs_qmat *m, uint16_t *hi, uint16_t *lo, altxs_stream_t stream) {
    if (!m) return ALTXS_EINVAL;
    if ((reinterpret_cast<uintptr_t>(hi) | reinterpret_cast<uintptr_t>(lo)) & 15) return ALTXS_EINVAL;
    return altxs::launch_split_weights(*m, hi, lo, reinterpret_cast<cudaStream_t>(stream));
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
    uint16_t *xh = static_cast<uint16_t *>(workspace);
    uint16_t *xl = reinterpret_cast<uint16_t *>(static_cast<unsigned char *>(workspace) +
                                                align_up((int64_t)M * K * 2, 256));
    ALTXS_LAUNCH(::altxs::kKQmm, st, k_split_rows<<<M, 256, 0, st>>>(X, K, K, xh, xl));
    TcArgs t{};
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

}  // extern "C"
