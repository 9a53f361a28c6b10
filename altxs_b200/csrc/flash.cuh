// Causal attention over a whole window on the tensor cores, without the T x T
// scores: the context prefill and the window forward of the full-parameter
// update (which recomputes its probabilities in the backward).
#pragma once
#include "common.cuh"

namespace altxs {

// y[t][h*hd + c] = sum_{s <= t} softmax_s(scale * q_t . k_s) v_s[c] for query
// head h reading key/value head h / (H / Hkv); q [T][ldq] (head h at column
// h*hd), k [T][ldk] and v [T][ldv] (head g at column g*hd), y [T][ldy].
struct FlashArgs {
    int T, H, Hkv, hd;
    float scale;
    const float *q, *k, *v;
    int64_t ldq, ldk, ldv;
    float *y;
    int64_t ldy;
    uint16_t *scratch;  // flash_scratch_elems(T, H, Hkv, hd) elements, 16-byte aligned
    float *lse;         // optional [H][T]: log2 of each row's softmax sum of 2^(s * scale * log2 e)
};

// Gradient of the same attention: dq, dk, dv from dy (= d out), out and the
// forward's lse.  dk and dv sum over the query heads of a group.  Every sum
// runs in a fixed order (no atomics): the same inputs give the same bits.
struct FlashBwdArgs {
    int T, H, Hkv, hd;
    float scale;
    const float *q, *k, *v, *out, *dout, *lse;
    int64_t ldq, ldk, ldv, ldo, lddo;
    float *dq, *dk, *dv;
    int64_t lddq, lddk, lddv;
    uint16_t *scratch;  // flash_bwd_scratch_elems(T, H, Hkv) elements, 16-byte aligned
};

// Head sizes the kernel takes (others use the materialised path).
inline bool flash_ok(int hd) { return hd == 32 || hd == 64; }
int64_t flash_scratch_elems(int T, int H, int Hkv, int hd);
int launch_flash_fwd(const FlashArgs &a, cudaStream_t stream);
int64_t flash_bwd_scratch_elems(int T, int H, int Hkv);
int launch_flash_bwd(const FlashBwdArgs &a, cudaStream_t stream);
// The first-wait poll limit of this translation unit's kernels (altxs_set_wait_limit).
int set_wait_limit_flash(uint32_t limit);
// Process-wide switch (altxs_set_flash): 0 = the materialised attention everywhere.
int set_flash(int on);

}  // namespace altxs
