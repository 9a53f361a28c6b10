// fp32 batched GEMM (CUDA cores) and the transposed mixed-bit product used by
// the test-time update's backward pass.
#pragma once

#include "common.cuh"

namespace altxs {

// C[b] = alpha * op(A[b]) op(B[b]) + beta * C[b]
//   op(A) is M x K: A stored [M][lda] (tA = 0) or [K][lda] read transposed (tA = 1)
//   op(B) is K x N: B stored [K][ldb] (tB = 0) or [N][ldb] read transposed (tB = 1)
// Batch b uses A + (b / adiv) * sA, B + (b / bdiv) * sB, C + b * sC.
// Reductions run in a fixed k order (deterministic); when the tile grid is
// too small to fill the GPU and `ws` is given, the K range is split into a
// shape-determined number of chunks whose partials are summed in order.
// causal: 0 none; 1 skip output tiles entirely above the diagonal (n > m);
// 2 op(A) is lower-triangular in (m, k): k < m0 + 64 only;
// 3 op(A) is upper-triangular in (m, k): k >= m0 only.
struct GemmArgs {
    const float *A;
    const float *B;
    float *C;
    int M, N, K;
    int64_t lda, ldb, ldc;
    int64_t sA, sB, sC;
    int tA, tB;
    int batch, adiv, bdiv;
    float alpha, beta;
    int causal;
    float *ws;
    int64_t ws_floats;
};
int launch_gemm(const GemmArgs &g, cudaStream_t s);

// Dense fp32 copy of rows [row0, row0 + rows) of a mixed-bit matrix (exact values).
int launch_dequant(const altxs_qmat &W, int row0, int rows, float *out, int64_t ld, cudaStream_t s);

// dX[m][k] = alpha * sum_n dY[m][n] * W[row0 + n][k]  (+ beta * dX)
// W is a mixed-bit matrix (groups along k); reduction over its rows.
struct QmmTArgs {
    const float *dY;
    int64_t lddy;
    int M;
    altxs_qmat W;
    int row0, N, K;
    float *dX;
    int64_t lddx;
    float alpha, beta;
};
int launch_qmm_t(const QmmTArgs &a, cudaStream_t s);

}  // namespace altxs
