// Mixed-bit dequant GEMV / GEMM (fp32 FMA on CUDA cores).
//
// Canonical arithmetic for every output element (identical in both paths):
//     y = 0
//     for g in 0 .. K/64-1:                  # 64-wide groups along K
//         p = 0
//         for i in 0 .. 63: p = fma(lev[g][i], x[64g + i], p)
//         y = fma(scale[g], p, y)
// where lev is the group's level (code - (2^b-1)/2, a codebook entry, or the
// raw fp32 value of a dense group) and scale the group's fp16 scale.  The
// reference computes the same dot products from pre-multiplied dense weights
// (mixed_bit_delta.py:147-213 then F.linear); dequantised values are exact in
// fp32, so the two differ only in rounding order.
#include "qmm_body.cuh"
#include "prof.cuh"

namespace altxs {
namespace {

template <int MM>
__global__ void __launch_bounds__(kGemvThreads) k_qgemv(QmmArgs a) {
    extern __shared__ __align__(16) float xs[];  // [M][K + K/64]: one pad float per group
    // the lane's first group is fetched while X is staged (independent loads)
    QgemvPre pre;
    qgemv_prefetch(a, blockIdx.x, blockDim.x >> 5, threadIdx.x >> 5, pre);
    qgemv_stage_x(a, xs, blockDim.x);
    __syncthreads();
    qgemv_rows<MM>(a, xs, blockIdx.x, blockDim.x >> 5, threadIdx.x >> 5, &pre);
}

// ---------------------------------------------------------------------------
// Tiled path: CTA tile 64 (m) x 64 (n), 256 threads, 4x4 outputs per thread.
// Per 64-wide group: X tile and dequantised level tile staged in shared
// memory k-major, then 64 fma steps into p, then y = fma(scale, p, y).
constexpr int kTM = 64, kTN = 64, kTThreads = 256, kPad = 4;

__global__ void __launch_bounds__(kTThreads) k_qgemm(QmmArgs a) {
    __shared__ __align__(16) float Xs[64][kTM + kPad];
    __shared__ __align__(16) float Ws[64][kTN + kPad];
    __shared__ float Ss[kTN];
    const int t = threadIdx.x;
    const int m0 = blockIdx.y * kTM, n0 = blockIdx.x * kTN;
    const int K = a.K, G = K / 64;
    const int tx = t & 15, ty = t >> 4;  // 16 x 16 threads
    float y[4][4], p[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) y[i][j] = 0.0f;

    // loaders: X row lm = t/4, 16 columns at (t%4)*16; W row ln = t/4, codes (t%4)*16
    const int lr = t >> 2, lc = (t & 3) * 16;
    const int xm = m0 + lr;
    const int wn = n0 + lr;
    const int wrow = a.row0 + (wn < a.N ? wn : 0);

    for (int g = 0; g < G; ++g) {
        // stage X (k-major)
        {
            float v[16];
            if (xm < a.M) {
                const float4 *src = reinterpret_cast<const float4 *>(a.X + (int64_t)xm * a.ldx + g * 64 + lc);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 f = src[q];
                    v[4 * q] = f.x;
                    v[4 * q + 1] = f.y;
                    v[4 * q + 2] = f.z;
                    v[4 * q + 3] = f.w;
                }
            } else {
#pragma unroll
                for (int q = 0; q < 16; ++q) v[q] = 0.0f;
            }
#pragma unroll
            for (int q = 0; q < 16; ++q) Xs[lc + q][lr] = v[q];
        }
        // stage W levels (k-major) and scales
        {
            float lev[16];
            uint32_t d = 0;
            if (wn < a.N) {
                d = a.W.gdesc[(int64_t)wrow * G + g];
                qmm_group_levels<16>(a.W, wrow, g, G, d, lc, lev);
            } else {
#pragma unroll
                for (int q = 0; q < 16; ++q) lev[q] = 0.0f;
            }
#pragma unroll
            for (int q = 0; q < 16; ++q) Ws[lc + q][lr] = lev[q];
            if ((t & 3) == 0) Ss[lr] = h2f((uint16_t)(d & 0xffffu));
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) p[i][j] = 0.0f;
#pragma unroll 8
        for (int k = 0; k < 64; ++k) {
            const float4 xa = *reinterpret_cast<const float4 *>(&Xs[k][ty * 4]);
            const float4 wb = *reinterpret_cast<const float4 *>(&Ws[k][tx * 4]);
            const float xv[4] = {xa.x, xa.y, xa.z, xa.w};
            const float wv[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) p[i][j] = __fmaf_rn(wv[j], xv[i], p[i][j]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float s = Ss[tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i) y[i][j] = __fmaf_rn(s, p[i][j], y[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty * 4 + i;
        if (m >= a.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx * 4 + j;
            if (n < a.N) qmm_epilogue_store(a, m, n, y[i][j]);
        }
    }
}

}  // namespace

int launch_qmm_path(const QmmArgs &a, cudaStream_t stream, int force_path) {
    if (a.M <= 0 || a.N <= 0) return ALTXS_OK;
    if (a.K % 64 || a.K != a.W.cols || a.row0 < 0 || a.row0 + a.N > a.W.rows) return ALTXS_EINVAL;
    const bool gemv = force_path == 1 || (force_path == 0 && a.M < kGemvMaxM);
    if (gemv) {
        if (a.M > kGemvMaxM) return ALTXS_EINVAL;
        const int G = a.K / 64;
        const int lpr = qgemv_lanes_per_row(a.K);
        const int rows_per_cta = (kGemvThreads / 32) * (32 / lpr);
        const size_t sm = (size_t)a.M * (a.K + G) * sizeof(float);
        if (sm > 200 * 1024) return ALTXS_ENOTSUP;
        const int grid = (a.N + rows_per_cta - 1) / rows_per_cta;
        if (a.M <= 1) {
            if (sm > 48 * 1024) cudaFuncSetAttribute(k_qgemv<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
            ALTXS_LAUNCH(::altxs::kKQmm, stream, k_qgemv<1><<<grid, kGemvThreads, sm, stream>>>(a));
        } else if (a.M <= 4) {
            if (sm > 48 * 1024) cudaFuncSetAttribute(k_qgemv<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
            ALTXS_LAUNCH(::altxs::kKQmm, stream, k_qgemv<4><<<grid, kGemvThreads, sm, stream>>>(a));
        } else {
            if (sm > 48 * 1024) cudaFuncSetAttribute(k_qgemv<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
            ALTXS_LAUNCH(::altxs::kKQmm, stream, k_qgemv<16><<<grid, kGemvThreads, sm, stream>>>(a));
        }
    } else {
        if ((a.ldx % 4) || (reinterpret_cast<uintptr_t>(a.X) & 15)) return ALTXS_EINVAL;
        dim3 grid((a.N + kTN - 1) / kTN, (a.M + kTM - 1) / kTM);
        ALTXS_LAUNCH(::altxs::kKQmm, stream, k_qgemm<<<grid, kTThreads, 0, stream>>>(a));
    }
    ALTXS_LAUNCH_CHECK();
    return ALTXS_OK;
}

int launch_qmm(const QmmArgs &a, cudaStream_t stream) { return launch_qmm_path(a, stream, 0); }

}  // namespace altxs
