// Tensor-core (tcgen05) GEMM on hi/lo bf16 planes.
//
// Operands are kept as pairs of bf16 planes: an fp32 value v is stored as
// hi = bf16(v) and lo = bf16(v - hi) (v - hi is exact in fp32).  For the
// dequantised weights w = level * scale (a half-integer level of at most
// 4 bits times an fp16 scale, <= 15 significant bits) hi + lo == w exactly;
// for other values hi + lo keeps 16 of the 24 significand bits.  The product
// x*w is formed as hi_x*hi_w + hi_x*lo_w + lo_x*hi_w with fp32 accumulation
// in tensor memory; the dropped terms are below 2^-16 of |x*w|.
//
// Every output element is computed by the same instruction sequence whatever
// the number of rows in the batch and wherever the row sits in its 128-row
// tile, so results do not depend on the batch composition.
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
__device__ __forceinline__ float split_load(const uint16_t *hi, const uint16_t *lo, int64_t idx) {
    return __fadd_rn(__bfloat162float(__ushort_as_bfloat16(hi[idx])), __bfloat162float(__ushort_as_bfloat16(lo[idx])));
}

// One GEMM operand stored as planes of a [nb][rows][cols] array (row stride
// ld, batch stride bstride, elements).  K-major (mn_major = 0): the operand's
// element (i, k) is at [row_off + i][k]; MN-major (mn_major = 1): at
// [row_off + k][i].  Batch b of the GEMM reads stored batch (b / div) * mul + add.
struct TcOp {
    const uint16_t *hi, *lo;
    int mn_major;
    int64_t rows, cols, ld, bstride;
    int nb;
    int64_t row_off;
    int div, mul, add;
};

// C[b][m][n] = epi(alpha * sum_k A(b)[m][k] B(b)[n][k] (+ beta * C)) for m < M, n < N, b < batch.
// causal: 0 none; 1 skip output tiles entirely above the diagonal (n > m);
// 2 A is lower-triangular in (m, k): k < m0 + 128 only; 3 A is upper-triangular: k >= m0 only.
struct TcGemm {
    TcOp a, b;
    int M, N, K, batch;
    int causal;
    float alpha, beta;
    int epi;  // QmmEpi; kEpiResid uses R/colscale (no alpha/beta)
    float *C;
    int64_t ldc, sC;
    const float *R;
    int64_t ldr;
    const float *colscale;
    float *Y2;
    int64_t ldy2;
    uint16_t *p_hi, *p_lo;  // optional bf16 planes of the stored value (row stride ldp, batch 0 only)
    int64_t ldp;
    uint32_t *status;       // optional per-row status word (ALTXS_ST_TIMEOUT on a wait that gave up)
    int64_t status_stride;  // in uint32 units
    int tma_c;              // set by launch_tc_gemm: C is written by TMA tensor stores
    // bq: B is read from the packed mixed-bit codes (tile-stream layout,
    // altxs_qtiles) instead of planes: element (n, k) of B is row wq_row0 + n
    // of the matrix (K-major; batch 1; wq_row0 a multiple of 64).  Each K
    // slice's code segments arrive by bulk copy; producer warps expand them
    // into the stage as the same hi/lo planes k_split_weights writes, so the
    // products are unchanged.
    int bq;
    altxs_qtiles wt;
    int64_t wq_row0;
    // chunked K (the step's linears; causal 0): the K loop runs in chunks of
    // kTcChunkKb 64-wide slices, each accumulated from zero in its own
    // tensor-memory accumulator, and the chunk sums are added in chunk order,
    // so a result does not depend on how many CTAs share a tile's chunks.
    // splits > 1: a unit is a range of one tile's chunks; its chunk sums go to
    // part ([tile][chunk][4 warps][BN/4][32 rows] float4) and the last unit of
    // each 32-row slab (arrival counters cnt [tile][4], zero before the launch
    // and left zero after it) adds them and runs the epilogue.
    int chunked, splits;
    float *part;
    uint32_t *cnt;
};
constexpr int kTcChunkKb = 8;     // slices per chunk (512 of K)
constexpr int kTcMaxChunks = 8;   // chunks a tile's accumulators hold in tensor memory (K <= 4096)
constexpr int kTcSplitTiles = 80; // most 64-wide tiles a split launch has

// 0 on success.  K and the operands' K extents must be multiples of 8, plane
// pointers 16-byte aligned, ld and bstride multiples of 8.
int launch_tc_gemm(const TcGemm &g, cudaStream_t stream);

// The step's linear layer: Y = epi(X W[row0 .. row0+N)^T) with X planes [M][lda] and W planes [rows][K].
struct TcArgs {
    const uint16_t *a_hi, *a_lo;
    int64_t lda;
    int M;
    const uint16_t *b_hi, *b_lo;
    int64_t b_rows;
    int row0, N, K;
    int epi;
    float *Y;
    int64_t ldy;
    const float *R;
    int64_t ldr;
    const float *colscale;
    float *Y2;
    int64_t ldy2;
    uint16_t *p_hi, *p_lo;
    int64_t ldp;
    uint32_t *status;
    int64_t status_stride;
    // optional: the packed weights (B rows from wt instead of the planes)
    const altxs_qtiles *wt;
    // optional: split-K scratch (tc_linear_part_elems floats, tc_linear_cnt_elems
    // counters, zeroed before the call); without it the K loop is not split
    float *part;
    uint32_t *cnt;
};
int launch_tc(const TcArgs &a, cudaStream_t stream);
// Scratch of launch_tc's split K for an M x N x K linear (0 when it never splits).
int64_t tc_linear_part_elems(int M, int N, int K);
int64_t tc_linear_cnt_elems(int M, int N, int K);

// An fp32 GEMM with the semantics of GemmArgs (gemm.cuh: C[b] = alpha op(A)
// op(B) + beta C, batch b reading A batch b / adiv and B batch b / bdiv,
// causal modes) on the tensor cores: both operands are first split into
// compact planes in the scratch regions (uint16 elements; sizes from
// tc_f32_scratch), then one launch_tc_gemm.
struct GemmArgs;
void tc_f32_scratch(const GemmArgs &g, int64_t *a_elems, int64_t *b_elems);
int tc_gemm_f32(const GemmArgs &g, uint16_t *a_scr, int64_t a_elems, uint16_t *b_scr, int64_t b_elems,
                cudaStream_t stream, int kernel_class);

// The first-wait poll limit of this translation unit's kernels (altxs_set_wait_limit).
int set_wait_limit_tc(uint32_t limit);

// Expand rows [0, rows) of a mixed-bit matrix into hi/lo bf16 planes [rows][cols].
int launch_split_weights(const altxs_qmat &W, uint16_t *hi, uint16_t *lo, cudaStream_t stream);

// hi/lo planes [nb][rows][cols] (compact) of an fp32 array [nb][rows][cols] (row stride ld, batch stride bs).
int launch_split_f32(const float *src, int64_t rows, int64_t cols, int64_t ld, int nb, int64_t bs, uint16_t *hi,
                     uint16_t *lo, cudaStream_t stream, int kernel_class);

}  // namespace altxs
