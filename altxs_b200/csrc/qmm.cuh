// Mixed-bit group-dequant linear layers: Y[m][n] = epi(sum_k W[n][k] X[m][k]).
#pragma once

#include "common.cuh"

namespace altxs {

enum QmmEpi : int {
    kEpiStore = 0,   // Y = acc
    kEpiLeaky2 = 1,  // Y = leaky_relu(acc, 0.5)^2                 (model.py:874-882)
    kEpiResid = 2,   // Y = R + colscale[n] * acc (R may alias Y); Y2 = Y if set
};

struct QmmArgs {
    const float *X;
    int64_t ldx;
    int M;
    altxs_qmat W;
    int row0;  // first row of W used
    int N;     // rows of W used (= outputs)
    int K;     // = W.cols
    float *Y;
    int64_t ldy;
    int epi;
    const float *R;
    int64_t ldr;
    const float *colscale;
    float *Y2;
    int64_t ldy2;
};

// Launch on `stream`; picks the GEMV path for M < 16 and the tiled path
// otherwise.  Both compute every output with the same operation sequence
// (see qmm.cu), so results do not depend on M or on the batch composition.
int launch_qmm(const QmmArgs &a, cudaStream_t stream);
int launch_qmm_path(const QmmArgs &a, cudaStream_t stream, int force_path);  // 0 auto, 1 gemv, 2 tiled

}  // namespace altxs
