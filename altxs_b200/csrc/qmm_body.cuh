// Device bodies of the mixed-bit CUDA-core GEMV, shared by the GEMV kernel
// (qmm.cu) and the fused decode step (step.cu), so both compute every output
// with the same operation sequence:
//     y = 0
//     for g in 0 .. K/64-1:                  # 64-wide groups along K
//         p = 0
//         for i in 0 .. 63: p = fma(lev[g][i], x[64g + i], p)
//         y = fma(scale[g], p, y)
// where lev is the group's level (code - (2^b-1)/2, a codebook entry, or the
// raw fp32 value of a dense group) and scale the group's fp16 scale.
#pragma once

#include "qmm.cuh"

namespace altxs {

__device__ __forceinline__ int qmm_width_of(uint32_t d) {
    const int c = (d >> 16) & 15;
    return c == 0 ? 0 : c == 1 ? 2 : c == 2 ? 3 : c == 3 ? 4 : 32;
}

__device__ __forceinline__ float qmm_leaky2(float v) {
    const float t = v >= 0.0f ? v : __fmul_rn(v, 0.5f);
    return __fmul_rn(t, t);
}

__device__ __forceinline__ void qmm_epilogue_store(const QmmArgs &a, int m, int n, float acc) {
    float v = acc;
    if (a.epi == kEpiLeaky2) {
        v = qmm_leaky2(acc);
    } else if (a.epi == kEpiResid) {
        v = __fadd_rn(a.R[(int64_t)m * a.ldr + n], __fmul_rn(a.colscale[n], acc));
        if (a.Y2) a.Y2[(int64_t)m * a.ldy2 + n] = v;
    }
    a.Y[(int64_t)m * a.ldy + n] = v;
}

// Extract NC consecutive codes (LSB-first, width B) starting at bit sh0 of w[0].
template <int B, int NC>
__device__ __forceinline__ void qmm_unpack_codes(const uint32_t *w, int sh0, uint32_t *codes) {
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
__device__ __forceinline__ void qmm_group_levels(const altxs_qmat &W, int row, int g, int G, uint32_t d, int c0,
                                                 float *lev) {
    const int b = qmm_width_of(d);
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
    if (b == 2) qmm_unpack_codes<2, NC>(words, sh0, codes);
    else if (b == 3) qmm_unpack_codes<3, NC>(words, sh0, codes);
    else qmm_unpack_codes<4, NC>(words, sh0, codes);
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

// p[m] += lev[j] * x[m][j] for the 64 codes of one group of width B (2, 3 or
// 4 bits), in code order, from the group's packed words W (2B of them, loaded
// together); levels from the codebook lut when given, else code - (2^B-1)/2.
template <int B, int MM>
__device__ __forceinline__ void qmm_group_dot(const uint32_t *W, const uint16_t *lut, const float *xr, int kp, int M,
                                              float *p) {
    const float center = (float)((1 << B) - 1) * 0.5f;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
        constexpr int kMask = (1 << B) - 1;
        const int bp = j * B, wi = bp >> 5, sh = bp & 31;
        uint32_t v = W[wi] >> sh;
        if (sh + B > 32) v |= W[wi + 1] << (32 - sh);
        const uint32_t code = v & kMask;
        const float lev = lut ? h2f(lut[code]) : __fsub_rn((float)code, center);
#pragma unroll
        for (int m = 0; m < MM; ++m)
            if (m < M) p[m] = __fmaf_rn(lev, xr[m * kp + j], p[m]);
    }
}

// GEMV: one lane computes one (row, group) partial p_g for every m; the lanes
// of a row then chain y = fma(s_g, p_g, y) in group order.
constexpr int kGemvThreads = 128;
constexpr int kGemvMaxM = 16;

// lanes per row: the power of two >= K/64, capped at 32 (then lanes loop over groups)
__host__ __device__ __forceinline__ int qgemv_lanes_per_row(int K) {
    const int G = K / 64;
    int lpr = 1;
    while (lpr < G && lpr < 32) lpr <<= 1;
    return lpr;
}

// Stage X [M][K] into shared memory as [M][K + K/64] (one pad float per group)
// with the first nt threads of the block.
__device__ __forceinline__ void qgemv_stage_x(const QmmArgs &a, float *xs, int nt) {
    const int K = a.K, G = K / 64, kp = K + G;
    if ((int)threadIdx.x >= nt) return;
    for (int idx = threadIdx.x; idx < a.M * K; idx += nt) {
        const int m = idx / K, k = idx - m * K;
        xs[m * kp + k + (k >> 6)] = a.X[(int64_t)m * a.ldx + k];
    }
}

// A lane's first group (descriptor and packed 2/3/4-bit words), fetched before
// X is staged so that the two global latencies overlap.
struct QgemvPre {
    uint32_t d;
    uint32_t W[8];
};

__device__ __forceinline__ void qgemv_prefetch(const QmmArgs &a, int rb, int warps_per_block, int warp,
                                               QgemvPre &pre) {
    const int K = a.K, G = K / 64;
    const int lane = threadIdx.x & 31;
    const int lpr = qgemv_lanes_per_row(K);
    const int n = (rb * warps_per_block + warp) * (32 / lpr) + lane / lpr;
    const int g = lane % lpr;
    pre.d = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) pre.W[q] = 0u;
    if (n >= a.N || g >= G) return;
    const int row = a.row0 + n;
    pre.d = a.W.gdesc[(int64_t)row * G + g];
    const int b = qmm_width_of(pre.d);
    if (b >= 2 && b <= 4) {
        const uint2 *g2 =
            reinterpret_cast<const uint2 *>(a.W.codes + 8ull * ((uint64_t)a.W.row_off8[row] + (pre.d >> 20)));
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint2 u = q < b ? g2[q] : make_uint2(0u, 0u);
            pre.W[2 * q] = u.x;
            pre.W[2 * q + 1] = u.y;
        }
    }
}

// The rows of row block rb (warps_per_block warps of 32 / lpr rows each) from
// the staged X; warp `warp` of the block takes its rows.  `pre` (optional):
// this lane's first group, already fetched by qgemv_prefetch.
template <int MM>
__device__ __forceinline__ void qgemv_rows(const QmmArgs &a, const float *xs, int rb, int warps_per_block, int warp,
                                           const QgemvPre *pre = nullptr) {
    const int K = a.K, G = K / 64, M = a.M;
    const int kp = K + G;
    const int lane = threadIdx.x & 31;
    const int lpr = qgemv_lanes_per_row(K);
    const int rows_per_warp = 32 / lpr;
    const int row_local = lane / lpr, sub = lane % lpr;
    const int n = (rb * warps_per_block + warp) * rows_per_warp + row_local;
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
            const bool have = pre && g0 == 0;
            const uint32_t d = have ? pre->d : a.W.gdesc[(int64_t)row * G + g];
            s = h2f((uint16_t)(d & 0xffffu));
            const int b = qmm_width_of(d);
            if (b >= 2 && b <= 4) {
                // the group's packed words in one go (8-byte aligned), then its 64 codes in order
                uint32_t W[8];
                if (have) {
#pragma unroll
                    for (int q = 0; q < 8; ++q) W[q] = pre->W[q];
                } else {
                    const uint2 *g2 = reinterpret_cast<const uint2 *>(
                        a.W.codes + 8ull * ((uint64_t)a.W.row_off8[row] + (d >> 20)));
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint2 u = q < b ? g2[q] : make_uint2(0u, 0u);
                        W[2 * q] = u.x;
                        W[2 * q + 1] = u.y;
                    }
                }
                const uint16_t *lut = a.W.lut ? a.W.lut + 16ull * a.W.glut[(int64_t)row * G + g] : nullptr;
                const float *xr = xs + g * 65;
                if (b == 2) qmm_group_dot<2, MM>(W, lut, xr, kp, M, p);
                else if (b == 3) qmm_group_dot<3, MM>(W, lut, xr, kp, M, p);
                else qmm_group_dot<4, MM>(W, lut, xr, kp, M, p);
            } else {  // all-zero or dense fp32 group
#pragma unroll 1
                for (int c = 0; c < 64; c += 16) {
                    float lev[16];
                    qmm_group_levels<16>(a.W, row, g, G, d, c, lev);
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
            if (m < M) qmm_epilogue_store(a, m, n, y[m]);
    }
}

}  // namespace altxs
