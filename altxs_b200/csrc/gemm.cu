// fp32 batched GEMM and transposed mixed-bit GEMM (CUDA cores).
#include "gemm.cuh"
#include "prof.cuh"

namespace altxs {
namespace {

constexpr int BM = 64, BN = 64, BK = 32, NT = 256;

// One (m0, n0) tile of one batch entry over the K range [kb, ke).  The raw
// accumulators are returned in acc (alpha/beta applied by the caller).
__device__ __forceinline__ void gemm_tile(const GemmArgs &g, const float *A, const float *B, int m0, int n0,
                                          int kb, int ke, float (&acc)[4][4], float (*As)[BM + 4],
                                          float (*Bs)[BN + 4]) {
    const int t = threadIdx.x, tx = t & 15, ty = t >> 4;
    for (int k0 = kb; k0 < ke; k0 += BK) {
        // op(A)[m0..+63][k0..+31] -> As[k][m]; op(B)[k0..+31][n0..+63] -> Bs[k][n]
#pragma unroll
        for (int it = 0; it < (BM * BK) / NT; ++it) {
            const int idx = t + it * NT;
            int m, k;
            if (g.tA) {
                m = idx % BM;
                k = idx / BM;
            } else {
                k = idx % BK;
                m = idx / BK;
            }
            float v = 0.0f;
            if (m0 + m < g.M && k0 + k < ke)
                v = g.tA ? A[(int64_t)(k0 + k) * g.lda + m0 + m] : A[(int64_t)(m0 + m) * g.lda + k0 + k];
            As[k][m] = v;
        }
#pragma unroll
        for (int it = 0; it < (BN * BK) / NT; ++it) {
            const int idx = t + it * NT;
            int n, k;
            if (g.tB) {
                k = idx % BK;
                n = idx / BK;
            } else {
                n = idx % BN;
                k = idx / BN;
            }
            float v = 0.0f;
            if (n0 + n < g.N && k0 + k < ke)
                v = g.tB ? B[(int64_t)(n0 + n) * g.ldb + k0 + k] : B[(int64_t)(k0 + k) * g.ldb + n0 + n];
            Bs[k][n] = v;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < BK; ++k) {
            const float4 a4 = *reinterpret_cast<const float4 *>(&As[k][ty * 4]);
            const float4 b4 = *reinterpret_cast<const float4 *>(&Bs[k][tx * 4]);
            const float av[4] = {a4.x, a4.y, a4.z, a4.w};
            const float bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
}

// K range of an output tile under the causal modes (see GemmArgs::causal).
__device__ __forceinline__ void k_range(const GemmArgs &g, int m0, int &kb, int &ke) {
    kb = 0;
    ke = g.K;
    if (g.causal == 2) ke = min(g.K, m0 + BM);
    if (g.causal == 3) kb = (m0 / BK) * BK;
}

__global__ void __launch_bounds__(NT) k_gemm(GemmArgs g) {
    __shared__ __align__(16) float As[BK][BM + 4];
    __shared__ __align__(16) float Bs[BK][BN + 4];
    const int b = blockIdx.z;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    if (g.causal == 1 && n0 > m0 + BM - 1) return;  // tile entirely above the diagonal
    const float *A = g.A + (int64_t)(b / g.adiv) * g.sA;
    const float *B = g.B + (int64_t)(b / g.bdiv) * g.sB;
    float *C = g.C + (int64_t)b * g.sC;
    float acc[4][4] = {};
    int kb, ke;
    k_range(g, m0, kb, ke);
    gemm_tile(g, A, B, m0, n0, kb, ke, acc, As, Bs);
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty * 4 + i;
        if (m >= g.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx * 4 + j;
            if (n >= g.N) continue;
            float *c = C + (int64_t)m * g.ldc + n;
            const float v = __fmul_rn(g.alpha, acc[i][j]);
            *c = g.beta == 0.0f ? v : __fmaf_rn(g.beta, *c, v);
        }
    }
}

// split-K: blockIdx.z = batch * splits + split; raw partials into g.ws
__global__ void __launch_bounds__(NT) k_gemm_split(GemmArgs g, int splits, int kchunk) {
    __shared__ __align__(16) float As[BK][BM + 4];
    __shared__ __align__(16) float Bs[BK][BN + 4];
    const int b = blockIdx.z / splits, sp = blockIdx.z % splits;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const float *A = g.A + (int64_t)(b / g.adiv) * g.sA;
    const float *B = g.B + (int64_t)(b / g.bdiv) * g.sB;
    float acc[4][4] = {};
    int kb, ke;
    k_range(g, m0, kb, ke);
    const int sb = max(kb, sp * kchunk), se = min(ke, (sp + 1) * kchunk);
    if (sb < se) gemm_tile(g, A, B, m0, n0, sb, se, acc, As, Bs);
    float *P = g.ws + ((int64_t)b * splits + sp) * g.M * g.N;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty * 4 + i;
        if (m >= g.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx * 4 + j;
            if (n < g.N) P[(int64_t)m * g.N + n] = acc[i][j];
        }
    }
}

// fixed-order sum over splits, then alpha/beta into C
__global__ void k_split_reduce(GemmArgs g, int splits) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t mn = (int64_t)g.M * g.N;
    if (i >= mn * g.batch) return;
    const int b = (int)(i / mn);
    const int64_t r = i % mn;
    const int m = (int)(r / g.N), n = (int)(r % g.N);
    float s = 0.0f;
    for (int sp = 0; sp < splits; ++sp) s = __fadd_rn(s, g.ws[((int64_t)b * splits + sp) * mn + r]);
    float *c = g.C + (int64_t)b * g.sC + (int64_t)m * g.ldc + n;
    const float v = __fmul_rn(g.alpha, s);
    *c = g.beta == 0.0f ? v : __fmaf_rn(g.beta, *c, v);
}

__device__ __forceinline__ float qelem(const altxs_qmat &W, int row, int col) {
    const int G = W.cols / 64, gi = col >> 6, i = col & 63;
    const uint32_t d = W.gdesc[(int64_t)row * G + gi];
    const int c = (d >> 16) & 15;
    const int b = c == 0 ? 0 : c == 1 ? 2 : c == 2 ? 3 : c == 3 ? 4 : 32;
    if (b == 0) return 0.0f;
    const uint8_t *gp = W.codes + 8ull * ((uint64_t)W.row_off8[row] + (d >> 20));
    if (b == 32) return reinterpret_cast<const float *>(gp)[i];
    const int bp = i * b, wi = bp >> 5, sh = bp & 31;
    const uint32_t *w32 = reinterpret_cast<const uint32_t *>(gp);
    uint32_t v = w32[wi] >> sh;
    if (sh + b > 32) v |= w32[wi + 1] << (32 - sh);
    const uint32_t code = v & ((1u << b) - 1u);
    const float s = h2f((uint16_t)(d & 0xffffu));
    const float lev = W.lut ? h2f(W.lut[16ull * W.glut[(int64_t)row * G + gi] + code])
                            : __fsub_rn((float)code, (float)((1 << b) - 1) * 0.5f);
    return __fmul_rn(lev, s);
}

// dense fp32 copy of rows [row0, row0 + rows) of a mixed-bit matrix
__global__ void k_dequant(altxs_qmat W, int row0, int rows, float *out, int64_t ld) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)rows * W.cols) return;
    const int r = (int)(i / W.cols), c = (int)(i % W.cols);
    out[(int64_t)r * ld + c] = qelem(W, row0 + r, c);
}

// dX tile 64 (m) x 64 (k = one group column); reduction over W rows in chunks of 64
__global__ void __launch_bounds__(NT) k_qmm_t(QmmTArgs a) {
    __shared__ __align__(16) float Ys[64][64 + 4];  // [n][m]
    __shared__ __align__(16) float Ws[64][64 + 4];  // [n][k]
    const int m0 = blockIdx.y * 64, k0 = blockIdx.x * 64;
    const int t = threadIdx.x, tx = t & 15, ty = t >> 4;
    float acc[4][4] = {};
    for (int n0 = 0; n0 < a.N; n0 += 64) {
        for (int idx = t; idx < 64 * 64; idx += NT) {
            const int n = idx & 63, m = idx >> 6;  // coalesced along n
            float v = 0.0f;
            if (m0 + m < a.M && n0 + n < a.N) v = a.dY[(int64_t)(m0 + m) * a.lddy + n0 + n];
            Ys[n][m] = v;
        }
        for (int idx = t; idx < 64 * 64; idx += NT) {
            const int k = idx & 63, n = idx >> 6;
            float v = 0.0f;
            if (n0 + n < a.N && k0 + k < a.K) v = qelem(a.W, a.row0 + n0 + n, k0 + k);
            Ws[n][k] = v;
        }
        __syncthreads();
#pragma unroll 8
        for (int n = 0; n < 64; ++n) {
            const float4 y4 = *reinterpret_cast<const float4 *>(&Ys[n][ty * 4]);
            const float4 w4 = *reinterpret_cast<const float4 *>(&Ws[n][tx * 4]);
            const float yv[4] = {y4.x, y4.y, y4.z, y4.w};
            const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(yv[i], wv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty * 4 + i;
        if (m >= a.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int k = k0 + tx * 4 + j;
            if (k >= a.K) continue;
            float *c = a.dX + (int64_t)m * a.lddx + k;
            const float v = __fmul_rn(a.alpha, acc[i][j]);
            *c = a.beta == 0.0f ? v : __fmaf_rn(a.beta, *c, v);
        }
    }
}

}  // namespace

int launch_gemm(const GemmArgs &g, cudaStream_t s) {
    if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return ALTXS_OK;
    if (g.adiv < 1 || g.bdiv < 1) return ALTXS_EINVAL;
    const int tm = (g.M + BM - 1) / BM, tn = (g.N + BN - 1) / BN;
    const int64_t tiles = (int64_t)tm * tn * g.batch;
    // Split the reduction when the tile grid cannot fill the GPU and K is long.
    // The split count depends only on the shape, so results are deterministic.
    int splits = 1;
    if (g.ws && g.causal != 1 && tiles < 296 && g.K >= 4 * BK) {
        splits = (int)((592 + tiles - 1) / tiles);
        splits = min(splits, g.K / (2 * BK));
        const int64_t cap = g.ws_floats / ((int64_t)g.M * g.N * g.batch);
        if (splits > cap) splits = (int)cap;
    }
    if (splits > 1) {
        const int kchunk = ((g.K + splits - 1) / splits + BK - 1) / BK * BK;
        dim3 grid(tn, tm, g.batch * splits);
        ALTXS_LAUNCH(kKTtt, s, k_gemm_split<<<grid, NT, 0, s>>>(g, splits, kchunk));
        const int64_t total = (int64_t)g.M * g.N * g.batch;
        ALTXS_LAUNCH(kKTtt, s, k_split_reduce<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(g, splits));
        return ALTXS_OK;
    }
    dim3 grid(tn, tm, g.batch);
    ALTXS_LAUNCH(kKTtt, s, k_gemm<<<grid, NT, 0, s>>>(g));
    return ALTXS_OK;
}

int launch_qmm_t(const QmmTArgs &a, cudaStream_t s) {
    if (a.M <= 0 || a.K <= 0) return ALTXS_OK;
    if (a.K != a.W.cols || a.row0 < 0 || a.row0 + a.N > a.W.rows) return ALTXS_EINVAL;
    dim3 grid((a.K + 63) / 64, (a.M + 63) / 64);
    ALTXS_LAUNCH(kKTtt, s, k_qmm_t<<<grid, NT, 0, s>>>(a));
    return ALTXS_OK;
}

int launch_dequant(const altxs_qmat &W, int row0, int rows, float *out, int64_t ld, cudaStream_t s) {
    if (rows <= 0) return ALTXS_OK;
    if (row0 < 0 || row0 + rows > W.rows || ld < W.cols) return ALTXS_EINVAL;
    const int64_t n = (int64_t)rows * W.cols;
    ALTXS_LAUNCH(kKTtt, s, k_dequant<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(W, row0, rows, out, ld));
    return ALTXS_OK;
}

}  // namespace altxs
