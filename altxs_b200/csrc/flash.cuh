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
};

// Head sizes the kernel takes (others use the materialised path).
inline bool flash_ok(int hd) { return hd == 32 || hd == 64; }
int64_t flash_scratch_elems(int T, int H, int Hkv, int hd);
int launch_flash_fwd(const FlashArgs &a, cudaStream_t stream);
// The first-wait poll limit of this translation unit's kernels (altxs_set_wait_limit).
int set_wait_limit_flash(uint32_t limit);
// Process-wide switch (altxs_set_flash): 0 = the materialised attention everywhere.
int set_flash(int on);

}  // namespace altxs
