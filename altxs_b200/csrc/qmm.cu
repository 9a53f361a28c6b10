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
#include "qmm.cuh"
#include "prof.cuh"

namespace altxs {
namespace {

__device__ __forceinline__ int width_of(uint32_t d) {
    const int c = (d >> 16) & 15;
    return c == 0 ? 0 : c == 1 ? 2 : c == 2 ? 3 : c == 3 ? 4 : 32;
}

__device__ __forceinline__ float leaky2(float v) {
    const float t = v >= 0.0f ? v : __fmul_rn(v, 0.5f);
    return __fmul_rn(t, t);
}

__device__ __forceinline__ void epilogue_store(const QmmArgs &a, int m, int n, float acc) {
    float v = acc;
    if (a.epi == kEpiLeaky2) {
        v = leaky2(acc);
    } else if (a.epi == kEpiResid) {
        v = __fadd_rn(a.R[(int64_t)m * a.ldr + n], __fmul_rn(a.colscale[n], acc));
        if (a.Y2) a.Y2[(int64_t)m * a.ldy2 + n] = v;
    }
    a.Y[(int64_t)m * a.ldy + n] = v;
}

// Extract NC consecutive codes (LSB-first, width B) starting at bit sh0 of w[0].
template <int B, int NC>
__device__ __forceinline__ void unpack_codes(const uint32_t *w, int sh0, uint32_t *codes) {
#pragma unroll
    for (int j = 0; j < NC; ++j) {
        const int bp = sh0 + j * B, wi = bp >> 5, sh = bp & 31;
        uint32_t v = w[wi] >> sh;
        if (sh + B > 32) v |= w[wi + 1] << (32 - sh);
        codes[j] = v & ((1u << B) - 1u);
    }
}

// Levels of NC codes starting at code index c0 (multiple of NC) of one group.
template <int NC>
__device__ __forceinline__ void group_levels(const altxs_qmat &W, int row, int g, int G, uint32_t d, int c0,
                                             float *lev) {
    const int b = width_of(d);
    const uint8_t *gp = W.codes + 8ull * ((uint64_t)W.row_off8[row] + (d >> 20));
    if (b == 0) {
#pragma unroll
        for (int j = 0; j < NC; ++j) lev[j] = 0.0f;
        return;
    }
    if (b == 32) {
        const float2 *f = reinterpret_cast<const float2 *>(gp) + (c0 >> 1);
#pragma unroll
        for (int j = 0; j < NC / 2; ++j) {
            const float2 v = f[j];
            lev[2 * j] = v.x;
            lev[2 * j + 1] = v.y;
        }
        return;
    }
    constexpr int kMaxW = (NC * 4 + 31) / 32 + 1;
    uint32_t words[kMaxW];
    uint32_t codes[NC];
    const int bit0 = c0 * b;
    const uint32_t *wp = reinterpret_cast<const uint32_t *>(gp) + (bit0 >> 5);
    const int sh0 = bit0 & 31;
    const int nw = (sh0 + NC * b + 31) >> 5;
#pragma unroll
    for (int i = 0; i < kMaxW; ++i) words[i] = i < nw ? wp[i] : 0u;
    if (b == 2) unpack_codes<2, NC>(words, sh0, codes);
    else if (b == 3) unpack_codes<3, NC>(words, sh0, codes);
    else unpack_codes<4, NC>(words, sh0, codes);
    if (W.lut) {
        const uint16_t *lut = W.lut + 16ull * W.glut[(int64_t)row * G + g];
#pragma unroll
        for (int j = 0; j < NC; ++j) lev[j] = h2f(lut[codes[j]]);
    } else {
        const float center = (float)((1 << b) - 1) * 0.5f;
#pragma unroll
        for (int j = 0; j < NC; ++j) lev[j] = __fsub_rn((float)codes[j], center);
    }
}

// ---------------------------------------------------------------------------
// GEMV path: one lane computes one (row, group) partial p_g for every m; the
// lanes of a row then chain y = fma(s_g, p_g, y) in group order.
constexpr int kGemvThreads = 128;
constexpr int kGemvMaxM = 16;

template <int MM>
__global__ void __launch_bounds__(kGemvThreads) k_qgemv(QmmArgs a) {
    extern __shared__ __align__(16) float xs[];  // [M][K + K/64]: one pad float per group
    const int K = a.K, G = K / 64, M = a.M;
    const int kp = K + G;
    for (int idx = threadIdx.x; idx < M * K; idx += blockDim.x) {
        const int m = idx / K, k = idx - m * K;
        xs[m * kp + k + (k >> 6)] = a.X[(int64_t)m * a.ldx + k];
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // lanes per row: the power of two >= G, capped at 32 (then lanes loop over groups)
    int lpr = 1;
    while (lpr < G && lpr < 32) lpr <<= 1;
    const int rows_per_warp = 32 / lpr;
    const int warps = blockDim.x >> 5;
    const int row_local = lane / lpr, sub = lane % lpr;
    const int n = (blockIdx.x * warps + warp) * rows_per_warp + row_local;
    const bool valid = n < a.N;
    const int row = a.row0 + (valid ? n : 0);
    float y[MM];
#pragma unroll
    for (int m = 0; m < MM; ++m) y[m] = 0.0f;
    for (int g0 = 0; g0 < G; g0 += lpr) {
        const int g = g0 + sub;
        float p[MM];
#pragma unroll
        for (int m = 0; m < MM; ++m) p[m] = 0.0f;
        float s = 0.0f;
        if (valid && g < G) {
            const uint32_t d = a.W.gdesc[(int64_t)row * G + g];
            s = h2f((uint16_t)(d & 0xffffu));
#pragma unroll 1
            for (int c = 0; c < 64; c += 16) {
                float lev[16];
                group_levels<16>(a.W, row, g, G, d, c, lev);
#pragma unroll
                for (int m = 0; m < MM; ++m) {
                    if (m < M) {
                        const float *xr = xs + m * kp + g * 65 + c;
#pragma unroll
                        for (int j = 0; j < 16; ++j) p[m] = __fmaf_rn(lev[j], xr[j], p[m]);
                    }
                }
            }
        }
        // chain this round's groups in group order
        const int gl = min(lpr, G - g0);
        for (int j = 0; j < gl; ++j) {
            const int src = row_local * lpr + j;
            const float sj = __shfl_sync(0xffffffffu, s, src);
#pragma unroll
            for (int m = 0; m < MM; ++m) {
                const float pj = __shfl_sync(0xffffffffu, p[m], src);
                y[m] = __fmaf_rn(sj, pj, y[m]);
            }
        }
    }
    if (valid && sub == 0) {
#pragma unroll
        for (int m = 0; m < MM; ++m)
            if (m < M) epilogue_store(a, m, n, y[m]);
    }
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
                group_levels<16>(a.W, wrow, g, G, d, lc, lev);
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
            if (n < a.N) epilogue_store(a, m, n, y[i][j]);
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
        int lpr = 1;
        while (lpr < G && lpr < 32) lpr <<= 1;
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
