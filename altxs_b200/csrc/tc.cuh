// Tensor-core (tcgen05) form of the mixed-bit linear layers.
//
// Operands are kept as pairs of bf16 planes: an fp32 value v is stored as
// hi = bf16(v) and lo = bf16(v - hi) (v - hi is exact in fp32).  For the
// dequantised weights w = level * scale (a half-integer level of at most
// 4 bits times an fp16 scale, <= 15 significant bits) hi + lo == w exactly;
// for activations hi + lo keeps 16 of the 24 significand bits.  The product
// x*w is formed as hi_x*hi_w + hi_x*lo_w + lo_x*hi_w with fp32 accumulation
// in tensor memory; the dropped terms are below 2^-16 of |x*w|.
//
// Every output row is computed by the same instruction sequence whatever the
// number of rows in the batch and wherever the row sits in its 128-row tile,
// so results do not depend on the batch composition.
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace altxs {

// hi/lo bf16 split of v into planes at index idx
__device__ __forceinline__ void split_store(uint16_t *hi, uint16_t *lo, int64_t idx, float v) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    const float r = __fsub_rn(v, __bfloat162float(h));
    hi[idx] = __bfloat16_as_ushort(h);
    lo[idx] = __bfloat16_as_ushort(__float2bfloat16_rn(r));
}

struct TcArgs {
    const uint16_t *a_hi, *a_lo;  // activations [M][K] (row stride lda elements)
    int64_t lda;
    int M;
    const uint16_t *b_hi, *b_lo;  // weights [rows][K] (row stride K), rows row0 .. row0+N-1 used
    int64_t b_rows;
    int row0, N, K;
    int epi;  // QmmEpi
    float *Y;
    int64_t ldy;
    const float *R;
    int64_t ldr;
    const float *colscale;
    float *Y2;
    int64_t ldy2;
    uint16_t *p_hi, *p_lo;  // optional bf16 planes of the stored value (row stride ldp)
    int64_t ldp;
    uint32_t *status;        // optional per-row status word (ALTXS_ST_TIMEOUT on a wait that gave up)
    int64_t status_stride;   // in uint32 units
};

// 0 on success, a cudaError_t otherwise.  K must be a multiple of 64, lda a
// multiple of 8 and all plane pointers 16-byte aligned.
int launch_tc(const TcArgs &a, cudaStream_t stream);

// Expand rows [0, rows) of a mixed-bit matrix into hi/lo bf16 planes [rows][cols].
int launch_split_weights(const altxs_qmat &W, uint16_t *hi, uint16_t *lo, cudaStream_t stream);

}  // namespace altxs
