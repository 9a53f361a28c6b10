// Model-level device helpers shared by the symbol step and the test-time update.
#pragma once

#include "common.cuh"

namespace altxs {

// LoRA arena offsets (floats) in TTTLoRA.parameters() order (its module
// registration order, ttt_lora.py:67-105): lm, q_s, v_s, k_s, mlp_s, o_s over
// the slots s (one per layer application).
struct LoraOff {
    int64_t lmA, lmB, qA, qB, vA, vB, kA, kB, mA, mB, oA, oB;  // per-slot blocks start; stride below
    int64_t q_stride, v_stride, k_stride, m_stride, o_stride, total;
};

__host__ __device__ inline LoraOff lora_offsets(const altxs_model_desc &dsc) {
    LoraOff o{};
    const int64_t r = dsc.lora_rank, d = dsc.d_model, kvd = (int64_t)dsc.n_kv_heads * dsc.head_dim;
    const int64_t V = dsc.vocab, L = dsc.n_virtual > 0 ? dsc.n_virtual : dsc.n_layers;
    int64_t cur = 0;
    if (r <= 0) return o;
    o.lmA = cur;
    cur += r * d;
    o.lmB = cur;
    cur += V * r;
    o.q_stride = r * d + d * r;
    o.qA = cur;
    o.qB = cur + r * d;
    cur += L * o.q_stride;
    o.v_stride = r * d + kvd * r;
    o.vA = cur;
    o.vB = cur + r * d;
    cur += L * o.v_stride;
    if (dsc.lora_mask & 2) {
        o.k_stride = r * d + kvd * r;
        o.kA = cur;
        o.kB = cur + r * d;
        cur += L * o.k_stride;
    }
    if (dsc.lora_mask & 32) {  // MLP adapter: d -> d on the MLP's normed input
        o.m_stride = r * d + d * r;
        o.mA = cur;
        o.mB = cur + r * d;
        cur += L * o.m_stride;
    }
    if (dsc.lora_mask & 8) {
        o.o_stride = r * d + d * r;
        o.oA = cur;
        o.oB = cur + r * d;
        cur += L * o.o_stride;
    }
    o.total = cur;
    return o;
}

__device__ __forceinline__ float rms_inv(float ss, int n) {
    const float ms = __fdiv_rn(ss, (float)n);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, kRmsEps)));
}

__device__ __forceinline__ float sigmoidf_(float v) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v))); }

// torch.lerp(start, end, weight)
__device__ __forceinline__ float lerp_t(float start, float end, float wgt) {
    const float diff = __fsub_rn(end, start);
    return wgt < 0.5f ? __fadd_rn(start, __fmul_rn(wgt, diff))
                      : __fsub_rn(end, __fmul_rn(diff, __fsub_rn(1.0f, wgt)));
}

// KV rows are stored in a 24-bit split format: fp32 rounded to nearest-even
// at bit 8, the high 16 bits (a bf16) and the next 8 mantissa bits kept in
// separate parts of the row: [hd x u16 high][hd x u8 low] = 3*hd bytes.
// fp16 K/V rounding moves the logits by up to ~1e-2 (the q_gain-scaled
// scores are sensitive to K); 24 bits keep them within ~3e-4 of fp32.
__device__ __forceinline__ uint32_t round24(float x) {
    const uint32_t b = __float_as_uint(x);
    return (b + 0x7Fu + ((b >> 8) & 1u)) >> 8;  // 24-bit pattern
}
__device__ __forceinline__ void store_kv_row(uint8_t *row, int hd, int k, float v) {
    const uint32_t r = round24(v);
    reinterpret_cast<uint16_t *>(row)[k] = (uint16_t)(r >> 8);
    row[2 * hd + k] = (uint8_t)(r & 0xFFu);
}

// dequantised W[row][col] (exact fp32 level*scale)
__device__ __forceinline__ float qmat_elem(const altxs_qmat &W, int row, int col) {
    const int G = W.cols / 64, g = col >> 6, i = col & 63;
    const uint32_t d = W.gdesc[(int64_t)row * G + g];
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
    float lev;
    if (W.lut) lev = h2f(W.lut[16ull * W.glut[(int64_t)row * G + g] + code]);
    else lev = __fsub_rn((float)code, (float)((1 << b) - 1) * 0.5f);
    return __fmul_rn(lev, s);
}


}  // namespace altxs
