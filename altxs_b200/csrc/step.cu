// One batched symbol step of the GPT model-and-code loop (sm_100a).
//
// Per layer (reference Block.forward, altxs src/xsa_ttt/model.py:948-979):
//   x_in = mix0*x + mix1*x0 ; n = rms(x_in)*ln
//   q,k,v = W n (+ LoRA) ; q,k = rms per head ; RoPE ; q *= q_gain
//   y = softmax(q k^T / sqrt(hd)) v over the sliding window ; o = W_o y (+ LoRA(n))
//   x = x_in + attn_scale*o ; x += mlp_scale * W_down leaky(W_up (rms(x)*ln), .5)^2
// with U-Net skips before decoder layers (model.py:1395-1436), then tied
// logits with tanh softcap (model.py:1460-1500), the integer CDF and the coder.
#include <math.h>

#include <algorithm>

#include <mutex>

#include "coder.cuh"
#include "flash.cuh"
#include "model.cuh"
#include "prof.cuh"
#include "qmm.cuh"
#include "qmm_body.cuh"
#include "tc.cuh"

using namespace altxs;

namespace {

#ifndef ALTXS_ATTN_SPLIT
#define ALTXS_ATTN_SPLIT 256
#endif
constexpr int kSplit = ALTXS_ATTN_SPLIT;  // keys per attention split (fixed: numerics independent of n)
constexpr int kCdfThreads = 512;

struct Dims {
    int n, V, L, d, H, Hkv, hd, F, ctx, rd, r, nsplit, enc, nskip, qkv_n, kvd;
    int64_t lora_stride;
    int Lv;        // layer applications (KV sets): L, or more with depth loops
    int xsa_from;  // physical layers >= xsa_from run XSA (L = none)
    int par;       // some decoder applications run the two parallel lanes
    int gw;        // gate window of the smear and sparse attention gates
    int mlora;     // MLP adapters (lora_mask bit 5)
};

// Per-application layout: which physical layer's weights run, at which KV set.
struct LayerApp {
    int p;     // physical layer
    int v;     // application index (KV set, skip slots)
    int mode;  // kAppPlain, kAppPar, kAppParFirst
};
constexpr int kAppPlain = 0;     // one residual stream
constexpr int kAppPar = 1;       // two lanes: attention reads lane 0, the MLP lane 1
constexpr int kAppParFirst = 2;  // first two-lane application: lane 1 starts as a copy of x

struct StepCtx {
    altxs_model_desc dsc;
    altxs_weights w;
    altxs_batch b;
    Dims D;
    LoraOff lo;
    // workspace
    float *x, *x0, *nrm, *nrm2, *skip, *qkv, *q, *part, *y, *ao, *hid, *logits, *lt;
    float *lane1, *mo;  // parallel lanes: the MLP lane; the MLP output (also with MLP adapters)
    float *lt2;         // MLP adapter: t = A n2 per stream [n][r]
    // tensor-core path: hi/lo bf16 planes of the linear layers' inputs; split-K
    // scratch of the linears (partials, arrival counters)
    int tc;
    uint16_t *nrm_h, *nrm_l, *y_h, *y_l, *nrm2_h, *nrm2_l, *hid_h, *hid_l;
    float *tcpart;
    uint32_t *tccnt;
    int64_t tccnt_elems;
};

__device__ __forceinline__ bool row_active(const altxs_batch &b, int i) { return !b.active || b.active[i]; }

// Kernel bodies take the block's item (bi, in place of blockIdx.x) and the
// thread count their arithmetic is written for (nt, in place of blockDim.x):
// the fused step runs them in larger blocks, where threads >= nt only join
// the barriers (their zero partials leave the block reductions unchanged).
#define ALTXS_TLOOP(k, lim) for (int k = (int)threadIdx.x < nt ? (int)threadIdx.x : (lim); k < (lim); k += nt)

// ---------------------------------------------------------------------------

// Embedding row, the smear gate when on (model.py:1350-1362: raw +=
// lambda * sigmoid(g . raw[:gate_window]) * raw of the previous token), RMSNorm.
__device__ void embed_body(const StepCtx &c, int bi, int nt) {
    __shared__ float red[32];
    __shared__ float gate;
    const int i = bi;
    if (!row_active(c.b, i)) return;
    const int d = c.D.d, tok = c.b.tok[i];
    float *x = c.x + (int64_t)i * d, *x0 = c.x0 + (int64_t)i * d;
    if (tok < 0 || tok >= c.D.V) {
        ALTXS_TLOOP(k, d) x[k] = x0[k] = 0.0f;
        return;
    }
    int prev = -1;
    if (c.dsc.smear_gate) {
        prev = c.b.prev_tok[i];
        if (threadIdx.x < 32) {
            float g = 0.0f;
            for (int k = threadIdx.x; k < c.D.gw; k += 32)
                g = __fmaf_rn(c.w.emb_dense ? c.w.emb_dense[(int64_t)tok * d + k] : qmat_elem(c.w.emb, tok, k),
                              c.w.smear_gate[k], g);
            g = warp_sum(g);
            if (threadIdx.x == 0) gate = __fmul_rn(c.w.smear_lambda[0], sigmoidf_(g));
        }
        __syncthreads();
    }
    const bool smear = prev >= 0 && prev < c.D.V;
    const float *ed = c.w.emb_dense;
    float ss = 0.0f;
    ALTXS_TLOOP(k, d) {
        float v = ed ? ed[(int64_t)tok * d + k] : qmat_elem(c.w.emb, tok, k);
        if (smear) v = __fadd_rn(v, __fmul_rn(gate, ed ? ed[(int64_t)prev * d + k] : qmat_elem(c.w.emb, prev, k)));
        x[k] = v;
        ss = __fmaf_rn(v, v, ss);
    }
    const float inv = rms_inv(block_sum(ss, red), d);
    __syncthreads();
    ALTXS_TLOOP(k, d) {
        const float v = __fmul_rn(x[k], inv);
        x[k] = v;
        x0[k] = v;
    }
}
__global__ void k_embed(StepCtx c) { embed_body(c, blockIdx.x, blockDim.x); }

// Skip lerp (decoder applications) + resid_mix + rms * ln -> x (= x_in), nrm.
// Two-lane applications (model.py:1293-1348) keep x as lane 0 after the skip
// (the lanes' residuals start from it, not from x_in) and also norm lane 1
// into nrm2 for the MLP, which reads lane 1 instead of the attention output.
__device__ void prenorm_body(const StepCtx &c, const LayerApp &a, int bi, int nt) {
    __shared__ float red[32];
    const int i = bi;
    if (!row_active(c.b, i)) return;
    const int d = c.D.d, n = c.D.n, l = a.p;
    float *x = c.x + (int64_t)i * d;
    const float *x0 = c.x0 + (int64_t)i * d;
    const float *mix = c.w.resid_mix + (int64_t)l * 2 * d;
    const int j = a.v - c.D.enc;  // decoder skip index
    const bool skip = j >= 0 && j < c.D.nskip;
    const float *sk = skip ? c.skip + ((int64_t)(c.D.nskip - 1 - j) * n + i) * d : nullptr;
    const bool par = a.mode != kAppPlain;
    float *l1 = par ? c.lane1 + (int64_t)i * d : nullptr;
    float ss = 0.0f, ss1 = 0.0f;
    ALTXS_TLOOP(k, d) {
        float xv = x[k];
        if (a.mode == kAppParFirst) l1[k] = xv;
        if (par) ss1 = __fmaf_rn(l1[k], l1[k], ss1);
        if (skip) {
            const float scaled = __fmul_rn(c.w.skip_weights[(int64_t)j * d + k], sk[k]);
            if (c.dsc.skip_gates) xv = lerp_t(scaled, xv, sigmoidf_(c.w.skip_gates[(int64_t)j * d + k]));
            else xv = __fadd_rn(xv, scaled);
        }
        const float xin = __fadd_rn(__fmul_rn(mix[k], xv), __fmul_rn(mix[d + k], x0[k]));
        x[k] = par ? xv : xin;
        ss = __fmaf_rn(xin, xin, ss);
    }
    const float inv = rms_inv(block_sum(ss, red), d);
    const float inv1 = par ? rms_inv(block_sum(ss1, red), d) : 0.0f;
    const float ln = c.w.ln_scale[l];
    __syncthreads();
    float *nr = c.nrm + (int64_t)i * d;
    ALTXS_TLOOP(k, d) {
        // x_in again from its parts (x now holds lane 0 on two-lane applications)
        const float xin = par ? __fadd_rn(__fmul_rn(mix[k], x[k]), __fmul_rn(mix[d + k], x0[k])) : x[k];
        const float v = __fmul_rn(__fmul_rn(xin, inv), ln);
        nr[k] = v;
        if (c.tc) split_store(c.nrm_h, c.nrm_l, (int64_t)i * d + k, v);
        if (par) {
            const float v1 = __fmul_rn(__fmul_rn(l1[k], inv1), ln);
            c.nrm2[(int64_t)i * d + k] = v1;
            if (c.tc) split_store(c.nrm2_h, c.nrm2_l, (int64_t)i * d + k, v1);
        }
    }
}
__global__ void k_prenorm(StepCtx c, LayerApp a) { prenorm_body(c, a, blockIdx.x, blockDim.x); }

// t[r] = A[r] . x  (warp per rank row; each lane sums its 16-byte chunks of
// the row in order, then a fixed warp tree; the chunk loads of a row are
// issued before the sums).  Unaligned operands take the scalar order.
__device__ inline void lora_t(const float *A, const float *x, int rank, int d, float *t) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(x)) & 15) || (d & 3)) {
        for (int r = wid; r < rank; r += nw) {
            float s = 0.0f;
            for (int k = lane; k < d; k += 32) s = __fmaf_rn(x[k], A[(int64_t)r * d + k], s);
            s = warp_sum(s);
            if (lane == 0) t[r] = s;
        }
        return;
    }
    const int d4 = d >> 2;
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    for (int r = wid; r < rank; r += nw) {
        const float4 *a4 = reinterpret_cast<const float4 *>(A + (int64_t)r * d);
        float s = 0.0f;
#pragma unroll 4
        for (int k = lane; k < d4; k += 32) {
            const float4 a = a4[k], xv = x4[k];
            s = __fmaf_rn(xv.x, a.x, s);
            s = __fmaf_rn(xv.y, a.y, s);
            s = __fmaf_rn(xv.z, a.z, s);
            s = __fmaf_rn(xv.w, a.w, s);
        }
        s = warp_sum(s);
        if (lane == 0) t[r] = s;
    }
}
// delta = (B[j] . t) * scale (ascending r; 16-byte loads when the rank allows)
__device__ __forceinline__ float lora_u(const float *B, const float *t, int rank, int j, float scale) {
    float u = 0.0f;
    if ((rank & 3) == 0 && !(reinterpret_cast<uintptr_t>(B) & 15)) {
        const float4 *b4 = reinterpret_cast<const float4 *>(B + (int64_t)j * rank);
        for (int r4 = 0; r4 < (rank >> 2); ++r4) {
            const float4 b = b4[r4];
            u = __fmaf_rn(b.x, t[4 * r4], u);
            u = __fmaf_rn(b.y, t[4 * r4 + 1], u);
            u = __fmaf_rn(b.z, t[4 * r4 + 2], u);
            u = __fmaf_rn(b.w, t[4 * r4 + 3], u);
        }
    } else {
        for (int r = 0; r < rank; ++r) u = __fmaf_rn(B[(int64_t)j * rank + r], t[r], u);
    }
    return __fmul_rn(u, scale);
}

// LoRA on q/k/v, per-head RMSNorm, partial RoPE, q_gain, KV ring write.
// Layers that run XSA get their new V rows (fp32, after LoRA) back in qkv.
// (no block-wide reductions: its arithmetic does not depend on the block size)
// part/nparts: this block takes heads [part*nh/nparts, (part+1)*nh/nparts) of the
// row's nh = H + 2 Hkv heads (a few streams spread one row over many blocks);
// every block computes the adapters' t itself, so the values do not change.
__device__ void qkv_post_body(const StepCtx &c, const LayerApp &a, int bi, int part = 0, int nparts = 1) {
    extern __shared__ __align__(16) float sm[];
    const int i = bi;
    if (!row_active(c.b, i)) return;
    const int tok = c.b.tok[i];
    if (tok < 0) return;
    const Dims &D = c.D;
    const int d = D.d, kvd = D.kvd, hd = D.hd, R = D.r, l = a.p;
    float *v = sm;                   // [qkv_n]
    float *tq = sm + D.qkv_n;        // [3][R]
    float *nx = tq + 3 * (R > 0 ? R : 1);  // [d]
    const float *src = c.qkv + (int64_t)i * D.qkv_n;
    for (int k = threadIdx.x; k < D.qkv_n; k += blockDim.x) v[k] = src[k];
    if (R > 0 && c.b.lora) {
        const float *nr = c.nrm + (int64_t)i * d;
        for (int k = threadIdx.x; k < d; k += blockDim.x) nx[k] = nr[k];
        __syncthreads();
        const float *P = c.b.lora + (int64_t)i * c.b.lora_stride;
        const LoraOff &o = c.lo;
        const int s = a.v;  // adapter slot: one per layer application (ttt_lora.py:73-77)
        lora_t(P + o.qA + s * o.q_stride, nx, R, d, tq);
        if (c.dsc.lora_mask & 2) lora_t(P + o.kA + s * o.k_stride, nx, R, d, tq + R);
        lora_t(P + o.vA + s * o.v_stride, nx, R, d, tq + 2 * R);
        __syncthreads();
        const float sc = c.dsc.lora_scale;
        const int nh = D.H + 2 * D.Hkv;
        const int k0 = part * nh / nparts * hd, k1 = (part + 1) * nh / nparts * hd;
        for (int k = k0 + threadIdx.x; k < k1; k += blockDim.x) {
            if (k < d) {
                v[k] = __fadd_rn(v[k], lora_u(P + o.qB + s * o.q_stride, tq, R, k, sc));
            } else if (k < d + kvd) {
                if (c.dsc.lora_mask & 2)
                    v[k] = __fadd_rn(v[k], lora_u(P + o.kB + s * o.k_stride, tq + R, R, k - d, sc));
            } else {
                v[k] = __fadd_rn(v[k], lora_u(P + o.vB + s * o.v_stride, tq + 2 * R, R, k - d - kvd, sc));
            }
        }
    }
    __syncthreads();
    const int nhead = D.H + 2 * D.Hkv;
    const int h0 = part * nhead / nparts, h1 = (part + 1) * nhead / nparts;
    if (l >= D.xsa_from && R > 0 && c.b.lora) {
        float *dst = c.qkv + (int64_t)i * D.qkv_n;
        const int k0 = max(d + kvd, h0 * hd), k1 = min(D.qkv_n, h1 * hd);
        for (int k = k0 + threadIdx.x; k < k1; k += blockDim.x) dst[k] = v[k];
    }
    const int64_t pos = c.b.pos[i];
    if (pos < 0 || pos >= c.w.rope_positions) {
        if (threadIdx.x == 0) atomicOr(&c.b.ac[i].status, ALTXS_ST_BAD_POS);
        return;
    }
    const int slot = (int)(pos % D.ctx);
    const int half = D.rd / 2;
    const float *cs = c.w.rope_cos + pos * half, *sn = c.w.rope_sin + pos * half;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    // heads: 0..H-1 q, H..H+Hkv-1 k (normed + rope), H+Hkv.. v (copy)
    const int64_t rb = 3 * (int64_t)hd;  // bytes per KV row
    uint8_t *kvbase = c.b.kv + ((int64_t)i * D.Lv + a.v) * 2 * D.Hkv * D.ctx * rb;
    for (int h = h0 + wid; h < h1; h += nw) {
        float *e = v + h * hd;  // q heads, then k heads, then v heads are contiguous
        if (h >= D.H + D.Hkv) {
            const int kvh = h - D.H - D.Hkv;
            uint8_t *dst = kvbase + (((int64_t)D.Hkv + kvh) * D.ctx + slot) * rb;
            for (int k = lane; k < hd; k += 32) store_kv_row(dst, hd, k, e[k]);
            continue;
        }
        float ss = 0.0f;
        for (int k = lane; k < hd; k += 32) ss = __fmaf_rn(e[k], e[k], ss);
        const float inv = rms_inv(warp_sum(ss), hd);
        float outv[4];  // hd <= 128 -> <= 4 per lane
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int k = lane + 32 * u;
            if (k >= hd) break;
            const float a = __fmul_rn(e[k], inv);
            float r = a;
            if (k < D.rd) {
                if (k < half) {
                    const float b2 = __fmul_rn(e[k + half], inv);
                    r = __fadd_rn(__fmul_rn(a, cs[k]), __fmul_rn(b2, sn[k]));
                } else {
                    const float a1 = __fmul_rn(e[k - half], inv);
                    r = __fadd_rn(__fmul_rn(a1, -sn[k - half]), __fmul_rn(a, cs[k - half]));
                }
            }
            outv[u] = r;
        }
        __syncwarp();
        if (h < D.H) {
            const float g = c.w.q_gain[(int64_t)l * D.H + h];
            float *qd = c.q + ((int64_t)i * D.H + h) * hd;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int k = lane + 32 * u;
                if (k < hd) qd[k] = __fmul_rn(outv[u], g);
            }
        } else {
            const int kvh = h - D.H;
            uint8_t *dst = kvbase + ((int64_t)kvh * D.ctx + slot) * rb;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int k = lane + 32 * u;
                if (k < hd) store_kv_row(dst, hd, k, outv[u]);
            }
        }
    }
}

// two floats from a u32 of two bf16 high halves and two low bytes (24-bit split)
__device__ __forceinline__ void unpack24x2(uint32_t h, uint32_t lo2, float &f0, float &f1) {
    // lo2: low byte of element 0 in bits 0-7, element 1 in bits 8-15, zeros above
    f0 = __uint_as_float(__byte_perm(h, lo2, 0x1046));
    f1 = __uint_as_float(__byte_perm(h, lo2, 0x3256));
}
__global__ void __launch_bounds__(256, 5) k_qkv_post(StepCtx c, LayerApp a) {
    qkv_post_body(c, a, blockIdx.x, blockIdx.y, gridDim.y);
}


// ---------------------------------------------------------------------------
// Warp-pipelined split attention.  Item t of a layer (stream, kv head, split
// of kSplit keys; split fastest) is taken by warp t mod (total warps).  A warp
// streams its items' keys in chunks of 32 rows: lane 0 issues the TMA bulk
// copies of a chunk's K and V rows into one of the warp's `slots` shared-memory
// slots (one mbarrier each), and the warp computes on the oldest slot while
// the others are in flight, so each warp keeps slots-1 chunks of HBM reads
// outstanding with no CTA-wide barrier.  Within an item the softmax runs
// online over its chunks (running max, rescaled sums).  The arithmetic of an
// item is fixed, so the partials do not depend on the number of streams or on
// which warp took the item.
//
// Lane layout (LPK = hd/8 lanes per key, 32/LPK keys per pass, LPK passes per
// chunk): lane (kl = lane/LPK, ds = lane%LPK) holds dims ds*8..ds*8+7 of key
// kl + (32/LPK)*p in pass p.  The LPK partial dots of a lane are summed across
// its LPK-lane group by recursive halving, which leaves lane (kl, ds) with the
// full score of key kl + (32/LPK)*ds: one score, one exp per lane per chunk.
constexpr int kRingChunk = 32;     // key rows per TMA chunk
constexpr int kRingMaxWarps = 8;   // warps per CTA
constexpr int kRingMaxSlots = 8;   // chunk slots per warp
#ifndef ALTXS_RING_WARPS
#define ALTXS_RING_WARPS 2  // 2 warps x 2 slots x 12 KB (hd 64): four CTAs per SM
#endif
#ifndef ALTXS_RING_SLOTS
#define ALTXS_RING_SLOTS 2
#endif

struct RingItem {
    int i, kvh, sp, nvalid;
    bool live;
};

__device__ __forceinline__ RingItem ring_item(const StepCtx &c, int t) {
    const Dims &D = c.D;
    RingItem it;
    it.sp = t % D.nsplit;
    const int r = t / D.nsplit;
    it.kvh = r % D.Hkv;
    it.i = r / D.Hkv;
    it.live = row_active(c.b, it.i) && c.b.tok[it.i] >= 0;
    it.nvalid = 0;
    if (it.live) {
        const int64_t pos = c.b.pos[it.i];
        const int npos = (int)(pos + 1 < (int64_t)D.ctx ? pos + 1 : (int64_t)D.ctx);
        const int k0 = it.sp * kSplit;
        it.nvalid = max(0, min(min(kSplit, D.ctx - k0), npos - k0));
    }
    return it;
}

// One warp's share of a layer's items: warp gw of GW takes items gw, gw+GW, ..
// with its slots in wbuf and its mbarriers in bar (l: the application's KV set).
// False when a copy did not land in time (the barriers are then left as they
// are).  kReuse: the caller initialises the same barriers again later (the
// fused step), so they are invalidated at the end.
template <int LPK, int G, bool kReuse = false>
__device__ bool attn_ring_warp(const StepCtx &c, int l, int n_items, int slots, int gw, int GW, uint8_t *wbuf,
                               uint64_t *bar) {
    constexpr int KPP = 32 / LPK;  // keys per pass
    constexpr int HD = LPK * 8, RB = 3 * HD;
    constexpr uint32_t kChunkBytes = (uint32_t)kRingChunk * RB;  // K (or V) rows of one chunk
    constexpr unsigned FULL = 0xffffffffu;
    const Dims &D = c.D;
    const int lane = threadIdx.x & 31;
    const int ds = lane % LPK, kl = lane / LPK;
    if (lane == 0) {
        for (int s = 0; s < slots; ++s) mbar_init(&bar[s], 1);
        fence_mbar_init();
    }
    __syncwarp();
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));

    // Load cursor (tracked by every lane, issued by lane 0): chunk lc of the
    // lnch chunks of item lt.  After seek(), lt >= n_items or lc < lnch.
    int lt = gw, lc = 0, lnch = 0;
    RingItem lit{};
    if (lt < n_items) {
        lit = ring_item(c, lt);
        lnch = (lit.nvalid + kRingChunk - 1) / kRingChunk;
    }
    auto seek = [&]() {
        while (lt < n_items && lc >= lnch) {
            lt += GW;
            lc = 0;
            lnch = 0;
            if (lt < n_items) {
                lit = ring_item(c, lt);
                lnch = (lit.nvalid + kRingChunk - 1) / kRingChunk;
            }
        }
    };
    auto issue = [&](int s) {
        if (lane == 0) {
            const int rows = min(kRingChunk, lit.nvalid - lc * kRingChunk);
            const uint32_t bytes = (uint32_t)rows * RB;
            const int64_t k0 = (int64_t)lit.sp * kSplit + lc * kRingChunk;
            const uint8_t *kvb = c.b.kv + ((int64_t)lit.i * D.Lv + l) * 2 * D.Hkv * D.ctx * RB;
            uint8_t *dst = wbuf + (int64_t)s * 2 * kChunkBytes;
            mbar_expect_tx(&bar[s], 2 * bytes);
            bulk_g2s(dst, kvb + ((int64_t)lit.kvh * D.ctx + k0) * RB, bytes, &bar[s]);
            bulk_g2s(dst + kChunkBytes, kvb + ((int64_t)(D.Hkv + lit.kvh) * D.ctx + k0) * RB, bytes, &bar[s]);
        }
        ++lc;
        seek();
    };
    seek();
    uint32_t par = 0, pend = 0;  // bit s: parity of slot s's next completion / a copy into s in flight
    for (int s = 0; s < slots && lt < n_items; ++s) {
        issue(s);
        pend |= 1u << s;
    }
    int slot = 0;
    for (int t = gw; t < n_items; t += GW) {
        const RingItem it = ring_item(c, t);
        if (!it.live) continue;
        float *part_base = c.part + (((int64_t)it.i * D.H + (int64_t)it.kvh * G) * D.nsplit + it.sp) * (HD + 2);
        if (it.nvalid == 0) {
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float *pp = part_base + (int64_t)g * D.nsplit * (HD + 2);
                for (int k = lane; k < HD; k += 32) pp[k] = 0.0f;
                if (lane == 0) {
                    pp[HD] = -INFINITY;
                    pp[HD + 1] = 0.0f;
                }
            }
            continue;
        }
        float qv[G][8], M[G], Ls[G], acc[G][8];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            M[g] = -INFINITY;
            Ls[g] = 0.0f;
            const float4 *qh =
                reinterpret_cast<const float4 *>(c.q + ((int64_t)it.i * D.H + it.kvh * G + g) * HD + ds * 8);
            const float4 a = qh[0], b2 = qh[1];
            qv[g][0] = a.x, qv[g][1] = a.y, qv[g][2] = a.z, qv[g][3] = a.w;
            qv[g][4] = b2.x, qv[g][5] = b2.y, qv[g][6] = b2.z, qv[g][7] = b2.w;
#pragma unroll
            for (int u = 0; u < 8; ++u) acc[g][u] = 0.0f;
        }
        const int nch = (it.nvalid + kRingChunk - 1) / kRingChunk;
        for (int cc = 0; cc < nch; ++cc) {
            const bool ok = __all_sync(FULL, mbar_wait_bounded(&bar[slot], (par >> slot) & 1u, wait_limit()));
            if (!ok) {  // a copy did not land in time: record it, let this warp's copies drain, leave
                if (lane == 0) atomicOr(&c.b.ac[it.i].status, ALTXS_ST_TIMEOUT);
                for (int s = 0; s < slots; ++s)
                    if (pend & (1u << s)) mbar_wait_bounded(&bar[s], (par >> s) & 1u, kWaitLimit);
                return false;
            }
            par ^= 1u << slot;
            pend &= ~(1u << slot);
            const uint8_t *Kc = wbuf + (int64_t)slot * 2 * kChunkBytes;
            const uint8_t *Vc = Kc + kChunkBytes;
            const int nv = min(kRingChunk, it.nvalid - cc * kRingChunk);
            // ---- scores: partial dots over this lane's 8 dims, one per pass
            float pd[G][LPK];
#pragma unroll
            for (int p = 0; p < LPK; ++p) {
                const int j = kl + KPP * p;
                float f[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) f[u] = 0.0f;
                if (j < nv) {
                    const uint8_t *row = Kc + j * RB;
                    const uint4 hi = *reinterpret_cast<const uint4 *>(row + ds * 16);
                    const uint2 lo = *reinterpret_cast<const uint2 *>(row + 2 * HD + ds * 8);
                    unpack24x2(hi.x, lo.x & 0xFFFFu, f[0], f[1]);
                    unpack24x2(hi.y, lo.x >> 16, f[2], f[3]);
                    unpack24x2(hi.z, lo.y & 0xFFFFu, f[4], f[5]);
                    unpack24x2(hi.w, lo.y >> 16, f[6], f[7]);
                }
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float dot = 0.0f;
#pragma unroll
                    for (int u = 0; u < 8; ++u) dot = __fmaf_rn(qv[g][u], f[u], dot);
                    pd[g][p] = dot;
                }
            }
            // ---- recursive-halving sum across the LPK lanes of a key group,
            // then the online softmax update with this chunk's scores
            const int jd = kl + KPP * ds;  // the key whose score this lane ends with
            float e[G];
#pragma unroll
            for (int g = 0; g < G; ++g) {
#pragma unroll
                for (int o = LPK / 2; o >= 1; o >>= 1) {
                    const bool up = (ds & o) != 0;
#pragma unroll
                    for (int q = 0; q < o; ++q) {
                        const float send = up ? pd[g][q] : pd[g][q + o];
                        const float keep = up ? pd[g][q + o] : pd[g][q];
                        pd[g][q] = __fadd_rn(keep, __shfl_xor_sync(FULL, send, o));
                    }
                }
                const float s = jd < nv ? __fmul_rn(pd[g][0], scale) : -INFINITY;
                const float mn = fmaxf(M[g], warp_max(s));
                const float alpha = expf(__fsub_rn(M[g], mn));
                e[g] = jd < nv ? expf(__fsub_rn(s, mn)) : 0.0f;
                Ls[g] = __fmaf_rn(Ls[g], alpha, e[g]);
#pragma unroll
                for (int u = 0; u < 8; ++u) acc[g][u] = __fmul_rn(acc[g][u], alpha);
                M[g] = mn;
            }
            // ---- weighted V rows
#pragma unroll
            for (int p = 0; p < LPK; ++p) {
                const int j = kl + KPP * p;
                float ej[G];
#pragma unroll
                for (int g = 0; g < G; ++g) ej[g] = __shfl_sync(FULL, e[g], kl * LPK + p);
                if (j < nv) {
                    const uint8_t *row = Vc + j * RB;
                    const uint4 hi = *reinterpret_cast<const uint4 *>(row + ds * 16);
                    const uint2 lo = *reinterpret_cast<const uint2 *>(row + 2 * HD + ds * 8);
                    float f[8];
                    unpack24x2(hi.x, lo.x & 0xFFFFu, f[0], f[1]);
                    unpack24x2(hi.y, lo.x >> 16, f[2], f[3]);
                    unpack24x2(hi.z, lo.y & 0xFFFFu, f[4], f[5]);
                    unpack24x2(hi.w, lo.y >> 16, f[6], f[7]);
#pragma unroll
                    for (int g = 0; g < G; ++g)
#pragma unroll
                        for (int u = 0; u < 8; ++u) acc[g][u] = __fmaf_rn(ej[g], f[u], acc[g][u]);
                }
            }
            __syncwarp();  // every lane is done with this slot: refill it
            if (lt < n_items) {
                issue(slot);
                pend |= 1u << slot;
            }
            slot = slot + 1 == slots ? 0 : slot + 1;
        }
        // ---- item partial: (max, sum of exp, unnormalised weighted V)
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
            for (int o = LPK; o < 32; o <<= 1)
#pragma unroll
                for (int u = 0; u < 8; ++u) acc[g][u] = __fadd_rn(acc[g][u], __shfl_xor_sync(FULL, acc[g][u], o));
            const float lsum = warp_sum(Ls[g]);
            float *pp = part_base + (int64_t)g * D.nsplit * (HD + 2);
            if (kl == 0) {
#pragma unroll
                for (int u = 0; u < 8; ++u) pp[ds * 8 + u] = acc[g][u];
            }
            if (lane == 0) {
                pp[HD] = M[g];
                pp[HD + 1] = lsum;
            }
        }
    }
    if (kReuse) {  // every copy this warp issued has been waited for: release the barriers
        __syncwarp();
        if (lane == 0)
            for (int s = 0; s < slots; ++s) mbar_inval(&bar[s]);
    }
    return true;
}

template <int LPK, int G>
__global__ void __launch_bounds__(kRingMaxWarps * 32) k_attn_ring(StepCtx c, int l, int n_items, int slots) {
    constexpr uint32_t kChunkBytes = (uint32_t)kRingChunk * 3 * (LPK * 8);
    extern __shared__ __align__(128) unsigned char smraw[];
    __shared__ __align__(8) uint64_t bars[kRingMaxWarps * kRingMaxSlots];
    const int w = threadIdx.x >> 5, W = blockDim.x >> 5;
    attn_ring_warp<LPK, G>(c, l, n_items, slots, blockIdx.x * W + w, gridDim.x * W,
                           smraw + (int64_t)w * slots * 2 * kChunkBytes, bars + w * kRingMaxSlots);
}

// Launch of the ring kernel for this model's head size and group size:
// a persistent grid of as many CTAs as fit on the device at once.
// Few items (a few streams: at most one item per warp of the device) keep every
// chunk of an item in flight (8 slots = one 256-key split) at one CTA per SM;
// many items keep 2 slots per warp at four CTAs per SM.  The slot count only
// changes how far ahead a warp's copies run, not an item's arithmetic.
template <int LPK, int G>
cudaError_t launch_ring(const StepCtx &c, int l, cudaStream_t st) {
    const Dims &D = c.D;
    const int warps = ALTXS_RING_WARPS;
    static std::mutex mu;
    static int grid_max[64][2] = {};
    static int sms_of[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    const size_t row = (size_t)2 * kRingChunk * 3 * (LPK * 8);  // bytes of one slot (K and V rows)
    {
        std::lock_guard<std::mutex> lk(mu);
        if (grid_max[dev][0] == 0) {
            cudaError_t e = cudaFuncSetAttribute(k_attn_ring<LPK, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)(warps * kRingMaxSlots * row));
            if (e != cudaSuccess) return e;
            cudaDeviceGetAttribute(&sms_of[dev], cudaDevAttrMultiProcessorCount, dev);
            for (int k = 0; k < 2; ++k) {
                const int sl = k ? kRingMaxSlots : ALTXS_RING_SLOTS;
                int per_sm = 0;
                e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_attn_ring<LPK, G>, warps * 32,
                                                                  warps * sl * row);
                if (e != cudaSuccess) return e;
                grid_max[dev][k] = (per_sm > 0 ? per_sm : 1) * (sms_of[dev] > 0 ? sms_of[dev] : 1);
            }
        }
    }
    const int n_items = D.n * D.Hkv * D.nsplit;
    const int deep = n_items <= warps * (sms_of[dev] > 0 ? sms_of[dev] : 1) ? 1 : 0;
    const int slots = deep ? kRingMaxSlots : ALTXS_RING_SLOTS;
    const size_t smem = (size_t)warps * slots * row;
    const int need = (n_items + warps - 1) / warps;
    const int grid = need < grid_max[dev][deep] ? need : grid_max[dev][deep];
    k_attn_ring<LPK, G><<<grid, warps * 32, smem, st>>>(c, l, n_items, slots);
    return cudaGetLastError();
}

cudaError_t launch_attn(const StepCtx &c, int l, cudaStream_t st) {
    const int G = c.D.H / c.D.Hkv;
#define ALTXS_RING_G(LPK)                               \
    switch (G) {                                        \
        case 1: return launch_ring<LPK, 1>(c, l, st);   \
        case 2: return launch_ring<LPK, 2>(c, l, st);   \
        case 3: return launch_ring<LPK, 3>(c, l, st);   \
        case 4: return launch_ring<LPK, 4>(c, l, st);   \
        default: return cudaErrorInvalidValue;          \
    }
    switch (c.D.hd / 8) {
        case 2: ALTXS_RING_G(2)
        case 4: ALTXS_RING_G(4)
        case 8: ALTXS_RING_G(8)
        case 16: ALTXS_RING_G(16)
        default: return cudaErrorInvalidValue;
    }
#undef ALTXS_RING_G
}

// Fixed-order merge of the split partials -> y [n][H*hd], then on XSA layers
// y -= (y . v^) v^ with v^ = v/max(|v|, 1e-12) of the head's own new V row,
// and with the sparse attention gate y *= sigmoid(scale * w_h . n[:gate_window])
// (model.py:760-768, 845-862).  One CTA of hd threads per (stream, head).
// (item bi = stream * H + head; nt = hd threads, one element each)
__device__ void merge_body(const StepCtx &c, int p, int bi, int nt) {
    __shared__ float red[32];
    const Dims &D = c.D;
    const int i = bi / D.H, h = bi % D.H;
    const bool act = (int)threadIdx.x < nt;
    const int k = act ? (int)threadIdx.x : 0;
    if (!row_active(c.b, i) || c.b.tok[i] < 0) return;
    const float *pp = c.part + ((int64_t)i * D.H + h) * D.nsplit * (D.hd + 2);
    float M = -INFINITY;
    for (int s = 0; s < D.nsplit; ++s)
        if (pp[s * (D.hd + 2) + D.hd + 1] > 0.0f) M = fmaxf(M, pp[s * (D.hd + 2) + D.hd]);
    float l = 0.0f, a = 0.0f;
    for (int s = 0; s < D.nsplit; ++s) {
        const float *q = pp + s * (D.hd + 2);
        if (q[D.hd + 1] > 0.0f) {
            const float f = expf(__fsub_rn(q[D.hd], M));
            l = __fmaf_rn(q[D.hd + 1], f, l);
            a = __fmaf_rn(q[k], f, a);
        }
    }
    float yv = act && l > 0.0f ? __fdiv_rn(a, l) : 0.0f;
    if (p >= D.xsa_from) {
        const float vn = act ? c.qkv[(int64_t)i * D.qkv_n + D.d + D.kvd + (h / (D.H / D.Hkv)) * D.hd + k] : 0.0f;
        const float nv = fmaxf(__fsqrt_rn(block_sum(__fmul_rn(vn, vn), red)), 1e-12f);
        const float vh = __fdiv_rn(vn, nv);
        const float dot = block_sum(__fmul_rn(yv, vh), red);
        yv = __fsub_rn(yv, __fmul_rn(dot, vh));
    }
    if (c.dsc.sparse_gate) {
        const float *gw = c.w.attn_gate_w + ((int64_t)p * D.H + h) * D.gw;
        const float *nr = c.nrm + (int64_t)i * D.d;
        // gate_window <= head_dim (checked on the host): thread k takes n[k]
        const float g = block_sum(act && k < D.gw ? __fmul_rn(nr[k], gw[k]) : 0.0f, red);
        yv = __fmul_rn(yv, sigmoidf_(__fmul_rn(c.dsc.sparse_gate_scale, g)));
    }
    if (!act) return;
    c.y[(int64_t)i * D.d + h * D.hd + k] = yv;
    if (c.tc) split_store(c.y_h, c.y_l, (int64_t)i * D.d + h * D.hd + k, yv);
}
__global__ void k_attn_merge(StepCtx c, int p) { merge_body(c, p, blockIdx.x, blockDim.x); }

// o-LoRA on the pre-attention normed input, residual, rms*ln for the MLP
// (layer l, adapter slot s).
__device__ void post_attn_body(const StepCtx &c, int l, int s, int bi, int nt) {
    extern __shared__ __align__(16) float sm[];
    __shared__ float red[32];
    const int i = bi;
    if (!row_active(c.b, i)) return;
    const int d = c.D.d, R = c.D.r;
    float *x = c.x + (int64_t)i * d;
    const float *ao = c.ao + (int64_t)i * d;
    const float *as = c.w.attn_scale + (int64_t)l * d;
    float *t = sm;  // [R]
    const bool has_o = R > 0 && c.b.lora && (c.dsc.lora_mask & 8);
    const float *P = R > 0 && c.b.lora ? c.b.lora + (int64_t)i * c.b.lora_stride : nullptr;
    // the o adapter reads the block's normed input, or with lora_mask bit 6 the
    // attention output y (ttt_o_lora_on_y, ttt_lora.py:168-170)
    const float *o_in = (c.dsc.lora_mask & 64) ? c.y + (int64_t)i * d : c.nrm + (int64_t)i * d;
    if (has_o) lora_t(P + c.lo.oA + s * c.lo.o_stride, o_in, R, d, t);
    __syncthreads();
    float ss = 0.0f;
    ALTXS_TLOOP(k, d) {
        float o = ao[k];
        if (has_o) o = __fadd_rn(o, lora_u(P + c.lo.oB + s * c.lo.o_stride, t, R, k, c.dsc.lora_scale));
        const float xv = __fadd_rn(x[k], __fmul_rn(as[k], o));
        x[k] = xv;
        ss = __fmaf_rn(xv, xv, ss);
    }
    const float inv = rms_inv(block_sum(ss, red), d);
    const float ln = c.w.ln_scale[l];
    __syncthreads();
    float *nr = c.nrm2 + (int64_t)i * d;
    ALTXS_TLOOP(k, d) {
        const float v = __fmul_rn(__fmul_rn(x[k], inv), ln);
        nr[k] = v;
        if (c.tc) split_store(c.nrm2_h, c.nrm2_l, (int64_t)i * d + k, v);
    }
    if (c.D.mlora && P) {  // MLP adapter's t = A n2 (the row is read back after the barrier)
        __syncthreads();
        lora_t(P + c.lo.mA + s * c.lo.m_stride, nr, R, d, c.lt2 + (int64_t)i * R);
    }
}
__global__ void k_post_attn(StepCtx c, int l, int s) { post_attn_body(c, l, s, blockIdx.x, blockDim.x); }

// MLP output with its adapter, then the residual (ttt_lora.py:171-175):
// x = x_mid + mlp_scale * (down + s * B t); encoder applications also keep the
// result as a skip source.
__device__ void mlp_resid_body(const StepCtx &c, int l, int s, float *skip, int bi, int nt) {
    const int i = bi;
    if (!row_active(c.b, i)) return;
    const int d = c.D.d, R = c.D.r;
    const float *P = c.b.lora ? c.b.lora + (int64_t)i * c.b.lora_stride + c.lo.mB + s * c.lo.m_stride : nullptr;
    const float *t = c.lt2 + (int64_t)i * R;
    float *x = c.x + (int64_t)i * d;
    const float *mo = c.mo + (int64_t)i * d, *ms = c.w.mlp_scale + (int64_t)l * d;
    ALTXS_TLOOP(k, d) {
        float m = mo[k];
        if (P) m = __fadd_rn(m, lora_u(P, t, R, k, c.dsc.lora_scale));
        const float v = __fadd_rn(x[k], __fmul_rn(ms[k], m));
        x[k] = v;
        if (skip) skip[(int64_t)i * d + k] = v;
    }
}
__global__ void k_mlp_resid(StepCtx c, int l, int s, float *skip) { mlp_resid_body(c, l, s, skip, blockIdx.x, blockDim.x); }

// Two-lane residual update (model.py:1293-1348; ttt_lora.py:181-250 with adapters):
//   a = attn_scale*(ao + o-adapter) ; m = mlp_scale*(mo + MLP adapter)
//   lane0 = r0*lane0 + p00*a + p10*m ; lane1 = r1*lane1 + p01*a + p11*m
// (layer l, adapter slot s)
__device__ void par_combine_body(const StepCtx &c, int l, int s, int bi, int nt) {
    extern __shared__ __align__(16) float tsm[];  // [2][R]: o- and MLP-adapter t
    const int i = bi;
    if (!row_active(c.b, i)) return;
    const int d = c.D.d, R = c.D.r;
    const float *pp = c.w.parallel_post + (int64_t)l * 4, *pr = c.w.parallel_resid + (int64_t)l * 2;
    const float p00 = pp[0], p01 = pp[1], p10 = pp[2], p11 = pp[3], r0 = pr[0], r1 = pr[1];
    float *x = c.x + (int64_t)i * d, *l1 = c.lane1 + (int64_t)i * d;
    const float *ao = c.ao + (int64_t)i * d, *mo = c.mo + (int64_t)i * d;
    const float *as = c.w.attn_scale + (int64_t)l * d, *ms = c.w.mlp_scale + (int64_t)l * d;
    const float *P = R > 0 && c.b.lora ? c.b.lora + (int64_t)i * c.b.lora_stride : nullptr;
    const bool has_o = P && (c.dsc.lora_mask & 8), has_m = P && c.D.mlora;
    if (has_o) {
        const float *o_in = (c.dsc.lora_mask & 64) ? c.y + (int64_t)i * d : c.nrm + (int64_t)i * d;
        lora_t(P + c.lo.oA + s * c.lo.o_stride, o_in, R, d, tsm);
    }
    if (has_m) lora_t(P + c.lo.mA + s * c.lo.m_stride, c.nrm2 + (int64_t)i * d, R, d, tsm + R);
    __syncthreads();
    ALTXS_TLOOP(k, d) {
        float ov = ao[k], mv = mo[k];
        if (has_o) ov = __fadd_rn(ov, lora_u(P + c.lo.oB + s * c.lo.o_stride, tsm, R, k, c.dsc.lora_scale));
        if (has_m) mv = __fadd_rn(mv, lora_u(P + c.lo.mB + s * c.lo.m_stride, tsm + R, R, k, c.dsc.lora_scale));
        const float a = __fmul_rn(as[k], ov), m = __fmul_rn(ms[k], mv);
        x[k] = __fadd_rn(__fadd_rn(__fmul_rn(r0, x[k]), __fmul_rn(p00, a)), __fmul_rn(p10, m));
        l1[k] = __fadd_rn(__fadd_rn(__fmul_rn(r1, l1[k]), __fmul_rn(p01, a)), __fmul_rn(p11, m));
    }
}
__global__ void k_par_combine(StepCtx c, int l, int s) { par_combine_body(c, l, s, blockIdx.x, blockDim.x); }

// final RMSNorm (+ lm_head LoRA t).  lanes: -1 one residual stream; after
// two-lane applications 0 the lanes' mean, 1 lane 0, 2 lane 1 (model.py:1437-1443).
__device__ void final_body(const StepCtx &c, int lanes, int bi, int nt) {
    extern __shared__ __align__(16) float sm[];
    __shared__ float red[32];
    const int i = bi;
    if (!row_active(c.b, i)) return;
    const int d = c.D.d, R = c.D.r;
    const float *x = lanes == 2 ? c.lane1 + (int64_t)i * d : c.x + (int64_t)i * d;
    const float *x1 = c.lane1 + (int64_t)i * d;
    float *nr = c.nrm + (int64_t)i * d;
    float ss = 0.0f;
    ALTXS_TLOOP(k, d) {
        float v = x[k];
        if (lanes == 0) v = __fmul_rn(0.5f, __fadd_rn(v, x1[k]));
        sm[k] = v;
        ss = __fmaf_rn(v, v, ss);
    }
    const float inv = rms_inv(block_sum(ss, red), d);
    ALTXS_TLOOP(k, d) {
        const float v = __fmul_rn(sm[k], inv);
        nr[k] = v;
        sm[k] = v;
        if (c.tc) split_store(c.nrm_h, c.nrm_l, (int64_t)i * d + k, v);
    }
    __syncthreads();
    if (R > 0 && c.b.lora && (c.dsc.lora_mask & 16)) {
        const float *P = c.b.lora + (int64_t)i * c.b.lora_stride;
        lora_t(P + c.lo.lmA, sm, R, d, c.lt + (int64_t)i * R);
    }
}
__global__ void k_final(StepCtx c, int lanes) { final_body(c, lanes, blockIdx.x, blockDim.x); }

// logits (+ lm LoRA) -> softcap -> integer CDF -> encode / decode; written for
// (and called only with) blocks of kCdfThreads threads
// The head's logits of row i, entries [k0, k1): the LM-head adapter's delta,
// then the (asymmetric) tanh softcap (model.py:1478-1500); into dst (and the
// caller's logits_out).
__device__ __forceinline__ void head_logits(const StepCtx &c, int i, int k0, int k1, float *dst, const float *tl) {
    const Dims &D = c.D;
    const int V = D.V, R = D.r, tok = c.b.tok[i];
    const float cap = c.dsc.logit_softcap;
    const bool has_lm = R > 0 && c.b.lora && (c.dsc.lora_mask & 16) && tok >= 0;
    const float *P = has_lm ? c.b.lora + (int64_t)i * c.b.lora_stride + c.lo.lmB : nullptr;
    const float *raw = c.logits + (int64_t)i * V;
    const float cap_n = c.dsc.asym_softcap ? c.w.softcap[1] : cap;
    const float cap_p = c.dsc.asym_softcap ? c.w.softcap[0] : cap;
    for (int k = k0 + threadIdx.x; k < k1; k += blockDim.x) {
        float lg = 0.0f;
        if (tok >= 0) {
            float v = raw[k];
            if (has_lm) v = __fadd_rn(v, lora_u(P, tl, R, k, c.dsc.lora_scale));
            const float cp = v >= 0.0f ? cap_p : cap_n;
            lg = __fmul_rn(cp, tanhf(__fdiv_rn(v, cp)));
        }
        dst[k - k0] = lg;
        if (c.b.logits_out) c.b.logits_out[(int64_t)i * V + k] = lg;
    }
}

// A few streams: the head's logits of each row in parallel over many blocks
// (part of nparts), written over the raw logits; the CDF kernel then reads them.
__global__ void k_head_rows(StepCtx c) {
    __shared__ float tl[128];
    const int i = blockIdx.x;
    if (!row_active(c.b, i)) return;
    const Dims &D = c.D;
    const int R = D.r;
    if (R > 0 && c.b.lora && (c.dsc.lora_mask & 16) && c.b.tok[i] >= 0 && threadIdx.x < R)
        tl[threadIdx.x] = c.lt[(int64_t)i * R + threadIdx.x];
    __syncthreads();
    const int k0 = blockIdx.y * D.V / gridDim.y, k1 = (blockIdx.y + 1) * D.V / gridDim.y;
    head_logits(c, i, k0, k1, c.logits + (int64_t)i * D.V + k0, tl);
}

// pre: the head's logits are already final in c.logits (k_head_rows)
__device__ void cdf_code_body(const StepCtx &c, int mode, int bi, int pre = 0) {
    extern __shared__ __align__(16) float buf[];  // [V]
    __shared__ CdfScratch sc;
    __shared__ float tl[128];
    const int i = bi;
    if (!row_active(c.b, i)) return;
    const Dims &D = c.D;
    const int V = D.V, R = D.r, tok = c.b.tok[i];
    if (pre) {
        if (mode == ALTXS_STEP_LOGITS) return;
        for (int k = threadIdx.x; k < V; k += blockDim.x) buf[k] = c.logits[(int64_t)i * V + k];
    } else {
        const bool has_lm = R > 0 && c.b.lora && (c.dsc.lora_mask & 16) && tok >= 0;
        if (has_lm && threadIdx.x < R) tl[threadIdx.x] = c.lt[(int64_t)i * R + threadIdx.x];
        __syncthreads();
        head_logits(c, i, 0, V, buf, tl);
    }
    __syncthreads();
    if (mode == ALTXS_STEP_LOGITS) return;
    uint32_t status = 0;
    const uint64_t total = logits_to_masses(buf, V, c.dsc.cdf_mode, c.dsc.cdf_bits, sc, status);
    const uint32_t *m = reinterpret_cast<const uint32_t *>(buf);
    altxs_ac_state st = c.b.ac[i];
    uint32_t *bits = c.b.bits + (int64_t)i * c.b.words_per_stream;
    int sym;
    if (mode == ALTXS_STEP_ENCODE) {
        sym = c.b.sym[i];
        if (sym < 0 || sym >= V) {
            if (threadIdx.x == 0) {
                st.status |= ALTXS_ST_BAD_SYMBOL | status;
                c.b.ac[i] = st;
            }
            return;
        }
        const uint64_t sl = mass_below(m, V, sym, sc);
        if (threadIdx.x == 0) {
            if (total == 0 || total > kQuarter) {
                st.status |= ALTXS_ST_BAD_TOTAL;
            } else {
                BitWriter bw;
                bw.begin(bits, c.b.words_per_stream, st.nbits);
                enc_symbol(st, bw, sl, sl + m[sym], total);
                bw.end();
                st.nbits = bw.nbits;
                st.status |= bw.status;
            }
        }
    } else {
        if (threadIdx.x == 0) sc.bcast[2] = dec_offset(st, total);
        __syncthreads();
        const uint64_t off = sc.bcast[2];
        uint64_t sl, sh;
        find_symbol(m, V, off, sc, sym, sl, sh);
        if (threadIdx.x == 0) {
            dec_symbol(st, bits, sl, sh, total);
            c.b.sym[i] = sym;
        }
    }
    if (threadIdx.x == 0) {
        st.status |= status;
        c.b.ac[i] = st;
        int64_t p = c.b.pos[i];
        if (tok >= 0) p += 1;
        c.b.pos[i] = p;
        c.b.tok[i] = sym;
        if (c.b.prev_tok && tok >= 0) c.b.prev_tok[i] = tok;
        if (c.b.hist) {
            const int64_t ap = p + (c.b.pos_base ? c.b.pos_base[i] : 0);  // absolute symbol index
            c.b.hist[(int64_t)i * c.b.hist_len + (ap % c.b.hist_len)] = sym;
        }
    }
}
__global__ void __launch_bounds__(kCdfThreads) k_cdf_code(StepCtx c, int mode, int pre) {
    cdf_code_body(c, mode, blockIdx.x, pre);
}


// ---------------------------------------------------------------------------
// Fused step for a few streams on the CUDA-core path: one persistent,
// cooperatively launched kernel runs the whole step (every layer application,
// the logits, the CDF and the coder) as the same sequence of phases that
// altxs_step launches one kernel each, calling the same bodies with the same
// thread counts and item order, with a grid-wide barrier between phases.  Its
// results are therefore bit-identical to the multi-launch step; what goes
// away is the ~76 launches per symbol.  Every barrier wait is bounded: a wait
// that gives up (or a block that saw a TMA copy time out) marks every stream
// ALTXS_ST_TIMEOUT and all blocks return.

constexpr int kFusedThreads = 512;  // = kCdfThreads: the CDF body runs at its own width
// Attention in the fused step: few streams give few items (n * Hkv * splits),
// so each warp keeps all chunks of its item in flight (8 slots of 32 rows =
// one 256-key split) instead of 2; 2 warps per block hold 2 x 8 slots.
constexpr int kFusedAttnWarps = 2;
constexpr int kFusedAttnSlots = 8;
constexpr int kFusedMaxApps = 64;
constexpr uint32_t kGridWaitLimit = 1u << 24;  // polls of one barrier wait (~0.2 us each: a few seconds)

struct GridSync {
    unsigned count, err, pad0, pad1;
};

struct FusedProg {
    GridSync *sync;
    int mode;
    int sched[kFusedMaxApps];  // physical layer of each application
};

// All blocks meet; ok = 0 from any thread of any block aborts the kernel.
// One arrival word: every block adds 1 except block 0, which adds
// 0x80000000 - (blocks - 1), so the word's top bit flips when the last block
// arrives; a block waits for the flip relative to the value it saw.  Release
// before the arrive, a fence after the wait: the next phase's loads see every
// block's stores of this one.
__device__ bool grid_sync(GridSync *g, int ok) {
    __shared__ int res;
    ok = __syncthreads_and(ok);
    if (threadIdx.x == 0) {
        if (!ok) atomicOr(&g->err, 1u);
        const unsigned add = blockIdx.x == 0 ? 0x80000000u - (gridDim.x - 1) : 1u;
        __threadfence();
        const unsigned old = atomicAdd(&g->count, add);
        bool flipped = false;
        for (uint32_t spins = 0;; ++spins) {
            if ((old ^ *(volatile unsigned *)&g->count) & 0x80000000u) {
                flipped = true;
                break;
            }
            if ((spins & 255u) == 255u && (spins > kGridWaitLimit || *(volatile unsigned *)&g->err)) break;
        }
        if (!flipped) atomicOr(&g->err, 1u);
        __threadfence();
        res = flipped && !*(volatile unsigned *)&g->err;
    }
    __syncthreads();
    return res != 0;
}

// One linear layer on the CUDA-core GEMV: the same rows, the same per-row
// arithmetic as k_qgemv; a block stages X once and takes row blocks rb =
// blockIdx.x, + gridDim.x, ..
__device__ void fused_gemv(const QmmArgs &a, float *xs) {
    const int warps = kFusedThreads / 32;
    const int rows_per_block = warps * (32 / qgemv_lanes_per_row(a.K));
    const int nrb = (a.N + rows_per_block - 1) / rows_per_block;
    if ((int)blockIdx.x >= nrb) return;
    qgemv_stage_x(a, xs, kFusedThreads);
    __syncthreads();
    for (int rb = blockIdx.x; rb < nrb; rb += gridDim.x) {
        if (a.M <= 1) qgemv_rows<1>(a, xs, rb, warps, threadIdx.x >> 5);
        else qgemv_rows<4>(a, xs, rb, warps, threadIdx.x >> 5);  // the fused step takes <= 4 streams
    }
    __syncthreads();
}

__device__ QmmArgs fused_lin(const float *X, int64_t ldx, int M, const altxs_qmat &W, int row0, int N, int K, float *Y,
                             int64_t ldy, int epi) {
    QmmArgs a{};
    a.X = X;
    a.ldx = ldx;
    a.M = M;
    a.W = W;
    a.row0 = row0;
    a.N = N;
    a.K = K;
    a.Y = Y;
    a.ldy = ldy;
    a.epi = epi;
    return a;
}

template <int LPK, int G>
__global__ void __launch_bounds__(kFusedThreads, 1) k_step_fused(StepCtx c, FusedProg fp) {
    constexpr uint32_t kChunkBytes = (uint32_t)kRingChunk * 3 * (LPK * 8);
    extern __shared__ __align__(128) unsigned char fsm[];
    __shared__ __align__(8) uint64_t fbars[kFusedAttnWarps * kFusedAttnSlots];
    const Dims &D = c.D;
    const int nb = gridDim.x, w = threadIdx.x >> 5;
    float *xs = reinterpret_cast<float *>(fsm);
    int ok = 1;
#define ALTXS_FUSED_SYNC()                                                              \
    do {                                                                                \
        if (!grid_sync(fp.sync, ok)) {                                                  \
            if (blockIdx.x == 0 && c.b.ac)                                              \
                for (int i_ = threadIdx.x; i_ < D.n; i_ += blockDim.x)                  \
                    atomicOr(&c.b.ac[i_].status, ALTXS_ST_TIMEOUT);                     \
            return;                                                                     \
        }                                                                               \
    } while (0)
#define ALTXS_FUSED_ITEMS(cnt, ...)                                        \
    do {                                                                   \
        for (int it = blockIdx.x; it < (cnt); it += nb) {                  \
            __VA_ARGS__;                                                   \
            __syncthreads();                                               \
        }                                                                  \
    } while (0)

    ALTXS_FUSED_ITEMS(D.n, embed_body(c, it, 128));
    ALTXS_FUSED_SYNC();
    bool lanes_on = false;
    for (int v = 0; v < D.Lv; ++v) {
        const int l = fp.sched[v];
        LayerApp app{l, v, kAppPlain};
        if (v >= D.enc && c.dsc.parallel_start > 0 && l >= c.dsc.parallel_start) {
            app.mode = lanes_on ? kAppPar : kAppParFirst;
            lanes_on = true;
        }
        const bool par = app.mode != kAppPlain;
        ALTXS_FUSED_ITEMS(D.n, prenorm_body(c, app, it, 128));
        ALTXS_FUSED_SYNC();
        fused_gemv(fused_lin(c.nrm, D.d, D.n, c.w.qkv, l * D.qkv_n, D.qkv_n, D.d, c.qkv, D.qkv_n, kEpiStore), xs);
        ALTXS_FUSED_SYNC();
        ALTXS_FUSED_ITEMS(D.n, qkv_post_body(c, app, it));
        fence_proxy_async_global();  // the new K/V rows, read next by TMA bulk copies on other SMs
        ALTXS_FUSED_SYNC();
        fence_proxy_async_global();
        if (w < kFusedAttnWarps)
            ok &= attn_ring_warp<LPK, G, true>(c, v, D.n * D.Hkv * D.nsplit, kFusedAttnSlots,
                                               blockIdx.x * kFusedAttnWarps + w, nb * kFusedAttnWarps,
                                               fsm + (int64_t)w * kFusedAttnSlots * 2 * kChunkBytes,
                                               fbars + w * kFusedAttnSlots)
                      ? 1
                      : 0;
        ALTXS_FUSED_SYNC();
        ALTXS_FUSED_ITEMS(D.n * D.H, merge_body(c, l, it, D.hd));
        ALTXS_FUSED_SYNC();
        fused_gemv(fused_lin(c.y, D.d, D.n, c.w.o, l * D.d, D.d, D.d, c.ao, D.d, kEpiStore), xs);
        ALTXS_FUSED_SYNC();
        if (!par) {
            ALTXS_FUSED_ITEMS(D.n, post_attn_body(c, l, v, it, 128));
            ALTXS_FUSED_SYNC();
        }
        fused_gemv(fused_lin(c.nrm2, D.d, D.n, c.w.up, l * D.F, D.F, D.d, c.hid, D.F, kEpiLeaky2), xs);
        ALTXS_FUSED_SYNC();
        const int skip_slot = v - (D.enc - D.nskip);
        float *skip_out = v < D.enc && skip_slot >= 0 ? c.skip + (int64_t)skip_slot * D.n * D.d : nullptr;
        const bool mres = !par && D.mlora && c.b.lora;
        QmmArgs dn = fused_lin(c.hid, D.F, D.n, c.w.down, l * D.d, D.d, D.F, par || mres ? c.mo : c.x, D.d,
                               par || mres ? kEpiStore : kEpiResid);
        if (!(par || mres)) {
            dn.R = c.x;
            dn.ldr = D.d;
            dn.colscale = c.w.mlp_scale + (int64_t)l * D.d;
            dn.Y2 = skip_out;
            dn.ldy2 = D.d;
        }
        fused_gemv(dn, xs);
        ALTXS_FUSED_SYNC();
        if (par) {
            ALTXS_FUSED_ITEMS(D.n, par_combine_body(c, l, v, it, 128));
            ALTXS_FUSED_SYNC();
        }
        if (mres) {
            ALTXS_FUSED_ITEMS(D.n, mlp_resid_body(c, l, v, skip_out, it, 128));
            ALTXS_FUSED_SYNC();
        }
    }
    const int lanes = lanes_on ? c.dsc.parallel_final : -1;
    ALTXS_FUSED_ITEMS(D.n, final_body(c, lanes, it, 128));
    ALTXS_FUSED_SYNC();
    fused_gemv(fused_lin(c.nrm, D.d, D.n, c.w.emb, 0, D.V, D.d, c.logits, D.V, kEpiStore), xs);
    ALTXS_FUSED_SYNC();
    ALTXS_FUSED_ITEMS(D.n, cdf_code_body(c, fp.mode, it));
#undef ALTXS_FUSED_SYNC
#undef ALTXS_FUSED_ITEMS
}

// Dynamic shared memory of the fused step: the largest phase (the attention
// slots of kFusedAttnWarps warps, the CDF row, a staged GEMV input, the
// qkv_post row).
inline size_t fused_smem(const Dims &D) {
    size_t s = (size_t)kFusedAttnWarps * kFusedAttnSlots * 2 * kRingChunk * 3 * D.hd;
    auto mx = [&](size_t v) { s = v > s ? v : s; };
    mx((size_t)D.V * 4);
    mx((size_t)D.n * (D.F + D.F / 64) * 4);
    mx((size_t)D.n * (D.d + D.d / 64) * 4);
    mx(((size_t)D.qkv_n + 3 * (D.r > 0 ? D.r : 1) + D.d) * 4);
    mx((size_t)2 * (D.r > 0 ? D.r : 1) * 4);
    return s;
}

// altxs_set_step_fusion; off by default: on a B200 the 33M single-stream step
// measured 0.75 ms fused against 0.56 ms for the CUDA-graph replay of the
// launch-per-phase step (each phase costs inside the kernel what it costs as
// its own launch, and the grid barrier eats the launch gap it saves)
int g_fused_max_streams = 0;
// altxs_set_linear_packed: the tensor-core linears read the packed codes (1) or
// the dense hi/lo planes (0); both give the same bits
int g_linear_packed = 0;

template <int LPK, int G>
int launch_fused_t(const StepCtx &c, const FusedProg &fp, cudaStream_t st) {
    // per-device launch shape, set up once per (device, shared-memory size);
    // the lock keeps a second host thread from reading a half-written entry
    static std::mutex mu;
    static int blocks[64] = {};
    static size_t smem_set[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return ALTXS_ECUDA;
    if (dev < 0 || dev >= 64) return ALTXS_ENOTSUP;
    const size_t smem = fused_smem(c.D);
    int nblk = 0;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (smem_set[dev] < smem) {
            if (cudaFuncSetAttribute(k_step_fused<LPK, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem) != cudaSuccess)
                return ALTXS_ENOTSUP;
            int per_sm = 0, sms = 0, coop = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_step_fused<LPK, G>, kFusedThreads, smem) !=
                cudaSuccess)
                return ALTXS_ENOTSUP;
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
            blocks[dev] = coop && per_sm > 0 ? sms : 0;  // one block per SM: all co-resident
            smem_set[dev] = smem;
        }
        nblk = blocks[dev];
    }
    if (nblk <= 0) return ALTXS_ENOTSUP;
    if (cudaMemsetAsync(fp.sync, 0, sizeof(GridSync), st) != cudaSuccess) return ALTXS_ECUDA;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(nblk);
    cfg.blockDim = dim3(kFusedThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaSuccess;
    ALTXS_LAUNCH(::altxs::kKFused, st, e = cudaLaunchKernelEx(&cfg, k_step_fused<LPK, G>, c, fp));
    return e == cudaSuccess ? ALTXS_OK : ALTXS_ECUDA;
}

// ENOTSUP: not a shape the fused step covers (the caller launches the phases one by one)
int launch_fused(const StepCtx &c, const altxs_model_desc *desc, int mode, GridSync *sync, cudaStream_t st) {
    const Dims &D = c.D;
    if (c.tc || D.n < 1 || D.n > g_fused_max_streams || D.n > 4 || D.Lv > kFusedMaxApps) return ALTXS_ENOTSUP;
    FusedProg fp{};
    fp.sync = sync;
    fp.mode = mode;
    for (int v = 0; v < D.Lv; ++v) fp.sched[v] = desc->schedule ? desc->schedule[v] : v;
    const int G = D.H / D.Hkv;
    if (D.hd == 64 && G == 1) return launch_fused_t<8, 1>(c, fp, st);
    if (D.hd == 64 && G == 2) return launch_fused_t<8, 2>(c, fp, st);
    if (D.hd == 32 && G == 1) return launch_fused_t<4, 1>(c, fp, st);
    if (D.hd == 32 && G == 2) return launch_fused_t<4, 2>(c, fp, st);
    return ALTXS_ENOTSUP;
}

// ---------------------------------------------------------------------------

// split-K scratch of the step's tensor-core linears (qkv, o, up, down, tied head)
inline int64_t tc_scratch(const Dims &D, bool counters) {
    const int NK[5][2] = {{D.qkv_n, D.d}, {D.d, D.d}, {D.F, D.d}, {D.d, D.F}, {D.V, D.d}};
    int64_t m = 0;
    for (const auto &nk : NK) {
        const int64_t e = counters ? tc_linear_cnt_elems(D.n, nk[0], nk[1]) : tc_linear_part_elems(D.n, nk[0], nk[1]);
        m = e > m ? e : m;
    }
    return m;
}

inline int64_t ws_size(const Dims &D) {
    auto A = [](int64_t x) { return align_up(x * 4, 256); };
    int64_t s = 0;
    s += 4 * A((int64_t)D.n * D.d);                   // x, x0, nrm, nrm2
    s += A((int64_t)D.nskip * D.n * D.d);             // skip
    s += A((int64_t)D.n * D.qkv_n);                   // qkv
    s += A((int64_t)D.n * D.H * D.hd);                // q
    s += A((int64_t)D.n * D.H * D.nsplit * (D.hd + 2));  // attention partials
    s += 2 * A((int64_t)D.n * D.d);                   // y, ao
    s += A((int64_t)D.n * D.F);                       // hid
    s += A((int64_t)D.n * D.V);                       // logits
    s += A((int64_t)D.n * (D.r > 0 ? D.r : 1));       // lm LoRA t
    s += 3 * A((int64_t)D.n * D.d);                   // hi/lo bf16 planes of nrm, y, nrm2
    if (D.par) s += A((int64_t)D.n * D.d);            // lane 1
    if (D.par || D.mlora) s += A((int64_t)D.n * D.d);  // MLP output
    if (D.mlora) s += A((int64_t)D.n * D.r);          // MLP adapter t
    s += A(tc_scratch(D, false)) + A(tc_scratch(D, true));  // split K of the tensor-core linears
    s += 256;                                         // grid barrier words of the fused step
    return s;
}

int fill_dims(const altxs_model_desc *dsc, int n, Dims &D) {
    if (!dsc || n < 0) return ALTXS_EINVAL;
    D.n = n;
    D.V = dsc->vocab;
    D.L = dsc->n_layers;
    D.d = dsc->d_model;
    D.H = dsc->n_heads;
    D.Hkv = dsc->n_kv_heads;
    D.hd = dsc->head_dim;
    D.F = dsc->mlp_hidden;
    D.ctx = dsc->ctx;
    D.rd = dsc->rope_dims;
    D.r = dsc->lora_rank;
    if (D.V < 2 || D.L < 1 || D.d % 64 || D.F % 64 || D.H < 1 || D.Hkv < 1 || D.H % D.Hkv) return ALTXS_EINVAL;
    if (D.hd * D.H != D.d || D.hd % 16 || D.hd > 128 || 32 % (D.hd / 8) || D.H / D.Hkv > 4) return ALTXS_ENOTSUP;
    if (D.rd % 2 || D.rd > D.hd || D.ctx < 1 || D.r < 0 || D.r > 128) return ALTXS_EINVAL;
    D.mlora = D.r > 0 && (dsc->lora_mask & 32) != 0;
    if ((int64_t)D.V * 4 > 160 * 1024) return ALTXS_ENOTSUP;
    if (dsc->cdf_mode != ALTXS_CDF_FIXED && dsc->cdf_mode != ALTXS_CDF_REF) return ALTXS_EINVAL;
    if (dsc->cdf_mode == ALTXS_CDF_FIXED && (dsc->cdf_bits > 30 || (1ll << dsc->cdf_bits) <= D.V))
        return ALTXS_EINVAL;
    D.kvd = D.Hkv * D.hd;
    D.qkv_n = D.d + 2 * D.kvd;
    D.nsplit = (D.ctx + kSplit - 1) / kSplit;
    D.Lv = dsc->n_virtual > 0 ? dsc->n_virtual : D.L;
    if (D.Lv != D.L && !dsc->schedule) return ALTXS_EINVAL;
    if (D.Lv > 4 * D.L + 64) return ALTXS_EINVAL;
    if (dsc->schedule)
        for (int v = 0; v < D.Lv; ++v)
            if (dsc->schedule[v] < 0 || dsc->schedule[v] >= D.L) return ALTXS_EINVAL;
    D.enc = dsc->n_encoder > 0 ? dsc->n_encoder : D.Lv / 2;
    if (D.enc > D.Lv) return ALTXS_EINVAL;
    D.nskip = D.enc < D.Lv - D.enc ? D.enc : D.Lv - D.enc;
    if (dsc->xsa_last_n < 0 || dsc->xsa_last_n > D.L || dsc->parallel_start < 0) return ALTXS_EINVAL;
    D.xsa_from = D.L - dsc->xsa_last_n;
    D.par = 0;
    if (dsc->parallel_start > 0)
        for (int v = D.enc; v < D.Lv; ++v)
            if ((dsc->schedule ? dsc->schedule[v] : v) >= dsc->parallel_start) D.par = 1;
    if (dsc->parallel_final < 0 || dsc->parallel_final > 2) return ALTXS_EINVAL;
    D.gw = 0;
    if (dsc->smear_gate || dsc->sparse_gate) {
        D.gw = dsc->gate_window;
        if (D.gw < 1 || D.gw > D.d || (dsc->sparse_gate && D.gw > D.hd)) return ALTXS_EINVAL;
    }
    return ALTXS_OK;
}

}  // namespace

extern "C" {

int altxs_set_wait_limit(uint32_t limit) {
    if (cudaMemcpyToSymbol(g_wait_limit, &limit, sizeof(limit)) != cudaSuccess) return ALTXS_ECUDA;
    if (altxs::set_wait_limit_flash(limit) != ALTXS_OK) return ALTXS_ECUDA;
    return altxs::set_wait_limit_tc(limit);
}

uint32_t altxs_default_wait_limit(void) { return altxs::kWaitLimit; }

int altxs_set_flash(int on) { return altxs::set_flash(on); }

int altxs_set_linear_packed(int on) {
    g_linear_packed = on ? 1 : 0;
    return ALTXS_OK;
}

int altxs_set_step_fusion(int max_streams) {
    if (max_streams < 0) return ALTXS_EINVAL;
    g_fused_max_streams = max_streams;
    return ALTXS_OK;
}

int64_t altxs_workspace_bytes(const altxs_model_desc *desc, int n_streams) {
    Dims D{};
    if (fill_dims(desc, n_streams, D) != ALTXS_OK) return -1;
    return ws_size(D);
}

int64_t altxs_lora_floats(const altxs_model_desc *desc) {
    if (!desc) return -1;
    return lora_offsets(*desc).total;
}

int altxs_step(const altxs_model_desc *desc, const altxs_weights *w, const altxs_batch *b, int mode,
               altxs_stream_t stream) {
    if (!desc || !w || !b) return ALTXS_EINVAL;
    if (mode < ALTXS_STEP_LOGITS || mode > ALTXS_STEP_DECODE) return ALTXS_EINVAL;
    StepCtx c{};
    c.dsc = *desc;
    c.w = *w;
    c.b = *b;
    int rc = fill_dims(desc, b->n_streams, c.D);
    if (rc) return rc;
    Dims &D = c.D;
    if (D.n == 0) return ALTXS_OK;
    if (!b->tok || !b->pos || !b->kv || !b->workspace || b->workspace_bytes < ws_size(D)) return ALTXS_EINVAL;
    if (mode != ALTXS_STEP_LOGITS && (!b->ac || !b->bits || !b->sym || b->words_per_stream < 1))
        return ALTXS_EINVAL;
    if (b->hist && b->hist_len < 1) return ALTXS_EINVAL;
    if (reinterpret_cast<uintptr_t>(b->kv) & 15) return ALTXS_EINVAL;
    if (w->emb.rows != D.V || w->emb.cols != D.d || w->qkv.rows != D.L * D.qkv_n || w->qkv.cols != D.d ||
        w->o.rows != D.L * D.d || w->o.cols != D.d || w->up.rows != D.L * D.F || w->up.cols != D.d ||
        w->down.rows != D.L * D.d || w->down.cols != D.F)
        return ALTXS_EINVAL;
    if ((desc->smear_gate && (!w->smear_gate || !w->smear_lambda || !b->prev_tok)) ||
        (desc->sparse_gate && !w->attn_gate_w) || (desc->asym_softcap && !w->softcap) ||
        (D.par && (!w->parallel_post || !w->parallel_resid)))
        return ALTXS_EINVAL;
    c.lo = lora_offsets(*desc);
    if (D.r > 0 && b->lora && b->lora_stride < c.lo.total) return ALTXS_EINVAL;
    D.lora_stride = b->lora_stride;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // carve workspace
    unsigned char *p = static_cast<unsigned char *>(b->workspace);
    auto take = [&](int64_t nfl) {
        float *r = reinterpret_cast<float *>(p);
        p += align_up(nfl * 4, 256);
        return r;
    };
    c.x = take((int64_t)D.n * D.d);
    c.x0 = take((int64_t)D.n * D.d);
    c.nrm = take((int64_t)D.n * D.d);
    c.nrm2 = take((int64_t)D.n * D.d);
    c.skip = take((int64_t)D.nskip * D.n * D.d);
    c.qkv = take((int64_t)D.n * D.qkv_n);
    c.q = take((int64_t)D.n * D.H * D.hd);
    c.part = take((int64_t)D.n * D.H * D.nsplit * (D.hd + 2));
    c.y = take((int64_t)D.n * D.d);
    c.ao = take((int64_t)D.n * D.d);
    c.hid = take((int64_t)D.n * D.F);
    c.logits = take((int64_t)D.n * D.V);
    c.lt = take((int64_t)D.n * (D.r > 0 ? D.r : 1));
    {
        const int64_t nd = (int64_t)D.n * D.d;
        c.nrm_h = reinterpret_cast<uint16_t *>(take(nd));
        c.nrm_l = c.nrm_h + nd;
        c.y_h = reinterpret_cast<uint16_t *>(take(nd));
        c.y_l = c.y_h + nd;
        c.nrm2_h = reinterpret_cast<uint16_t *>(take(nd));
        c.nrm2_l = c.nrm2_h + nd;
        // the MLP hidden planes take the place of the fp32 hidden buffer (unused on this path)
        c.hid_h = reinterpret_cast<uint16_t *>(c.hid);
        c.hid_l = c.hid_h + (int64_t)D.n * D.F;
    }
    if (D.par) c.lane1 = take((int64_t)D.n * D.d);
    if (D.par || D.mlora) c.mo = take((int64_t)D.n * D.d);
    if (D.mlora) c.lt2 = take((int64_t)D.n * D.r);
    c.tcpart = take(tc_scratch(D, false));
    c.tccnt_elems = tc_scratch(D, true);
    c.tccnt = reinterpret_cast<uint32_t *>(take(c.tccnt_elems));
    GridSync *gsync = reinterpret_cast<GridSync *>(p);
    p += 256;
    const altxs_split_planes *sp = w->split;
    c.tc = sp != nullptr;
    if (sp && (!sp->emb_hi || !sp->emb_lo || !sp->qkv_hi || !sp->qkv_lo || !sp->o_hi || !sp->o_lo || !sp->up_hi ||
               !sp->up_lo || !sp->down_hi || !sp->down_lo))
        return ALTXS_EINVAL;
    // a few streams on the CUDA-core path: the whole step as one fused launch
    if (!c.tc) {
        rc = launch_fused(c, desc, mode, gsync, st);
        if (rc != ALTXS_ENOTSUP) return rc;
    }
    // one linear layer: tensor cores from the bf16 planes, or CUDA cores from the packed codes
    auto linear = [&](const QmmArgs &q, const uint16_t *xh, const uint16_t *xl, const uint16_t *wh, const uint16_t *wl,
                      uint16_t *ph, uint16_t *pl, const altxs_qtiles *wt) -> int {
        if (!c.tc) return launch_qmm(q, st);
        TcArgs t{};
        t.a_hi = xh;
        t.a_lo = xl;
        t.lda = q.ldx;
        t.M = q.M;
        t.b_hi = wh;
        t.b_lo = wl;
        t.b_rows = q.W.rows;
        t.row0 = q.row0;
        t.N = q.N;
        t.K = q.K;
        t.epi = q.epi;
        t.Y = ph ? nullptr : q.Y;
        t.ldy = q.ldy;
        t.R = q.R;
        t.ldr = q.ldr;
        t.colscale = q.colscale;
        t.Y2 = q.Y2;
        t.ldy2 = q.ldy2;
        t.p_hi = ph;
        t.p_lo = pl;
        t.ldp = q.N;
        if (b->ac) {
            t.status = &b->ac[0].status;
            t.status_stride = sizeof(altxs_ac_state) / sizeof(uint32_t);
        }
        // the producer warps expand B from the packed codes
        if (!w->planes_live && g_linear_packed && wt && q.row0 % 64 == 0) t.wt = wt;
        if (c.tccnt_elems > 0) {
            t.part = c.tcpart;
            t.cnt = c.tccnt;
        }
        return launch_tc(t, st);
    };

    // the linears' split-K counters start from zero (each launch also leaves them zero)
    if (c.tc && c.tccnt_elems > 0 && cudaMemsetAsync(c.tccnt, 0, c.tccnt_elems * 4, st) != cudaSuccess)
        return ALTXS_ECUDA;
    ALTXS_LAUNCH(::altxs::kKEmbed, st, k_embed<<<D.n, 128, 0, st>>>(c));
    {
        static bool attr_done[64] = {};
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev < 0 || dev >= 64 || !attr_done[dev]) {
            cudaFuncSetAttribute(k_cdf_code, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
            if (dev >= 0 && dev < 64) attr_done[dev] = true;
        }
    }
    const size_t qkv_sm = ((size_t)D.qkv_n + 3 * (D.r > 0 ? D.r : 1) + D.d) * 4;
    // applications in schedule order: weights by physical layer p, KV set and
    // skip slot by application v (model.py:1064-1077, 1377-1436)
    bool lanes_on = false;
    for (int v = 0; v < D.Lv; ++v) {
        const int l = desc->schedule ? desc->schedule[v] : v;
        LayerApp app{l, v, kAppPlain};
        if (v >= D.enc && desc->parallel_start > 0 && l >= desc->parallel_start) {
            app.mode = lanes_on ? kAppPar : kAppParFirst;
            lanes_on = true;
        }
        const bool par = app.mode != kAppPlain;
        ALTXS_LAUNCH(::altxs::kKPrenorm, st, k_prenorm<<<D.n, 128, 0, st>>>(c, app));
        QmmArgs a{};
        a.X = c.nrm;
        a.ldx = D.d;
        a.M = D.n;
        a.W = w->qkv;
        a.row0 = l * D.qkv_n;
        a.N = D.qkv_n;
        a.K = D.d;
        a.Y = c.qkv;
        a.ldy = D.qkv_n;
        a.epi = kEpiStore;
        if ((rc = linear(a, c.nrm_h, c.nrm_l, c.tc ? sp->qkv_hi : nullptr, c.tc ? sp->qkv_lo : nullptr, nullptr, nullptr, w->tiles ? &w->tiles->qkv : nullptr))) return rc;
        {
            // a few streams: one block per head of each row, so the row's heads run in parallel
            const int nh = D.H + 2 * D.Hkv;
            const int parts = (int64_t)D.n * nh <= 296 ? nh : 1;
            ALTXS_LAUNCH(::altxs::kKQkvPost, st, k_qkv_post<<<dim3(D.n, parts), 256, qkv_sm, st>>>(c, app));
        }
        {
            cudaError_t ae = cudaSuccess;
            ALTXS_LAUNCH(::altxs::kKAttn, st, ae = launch_attn(c, v, st));
            if (ae != cudaSuccess) return ALTXS_ECUDA;
        }
        ALTXS_LAUNCH(::altxs::kKAttnMerge, st, k_attn_merge<<<D.n * D.H, D.hd, 0, st>>>(c, l));
        a.X = c.y;
        a.W = w->o;
        a.row0 = l * D.d;
        a.N = D.d;
        a.Y = c.ao;
        a.ldy = D.d;
        if ((rc = linear(a, c.y_h, c.y_l, c.tc ? sp->o_hi : nullptr, c.tc ? sp->o_lo : nullptr, nullptr, nullptr, w->tiles ? &w->tiles->o : nullptr))) return rc;
        // two-lane applications normed lane 1 for the MLP in k_prenorm
        if (!par)
            ALTXS_LAUNCH(::altxs::kKPostAttn, st, k_post_attn<<<D.n, 128, (D.r > 0 ? D.r : 1) * 4, st>>>(c, l, v));
        a.X = c.nrm2;
        a.W = w->up;
        a.row0 = l * D.F;
        a.N = D.F;
        a.Y = c.hid;
        a.ldy = D.F;
        a.epi = kEpiLeaky2;
        if ((rc = linear(a, c.nrm2_h, c.nrm2_l, c.tc ? sp->up_hi : nullptr, c.tc ? sp->up_lo : nullptr, c.tc ? c.hid_h : nullptr, c.tc ? c.hid_l : nullptr, w->tiles ? &w->tiles->up : nullptr))) return rc;
        a.X = c.hid;
        a.ldx = D.F;
        a.W = w->down;
        a.row0 = l * D.d;
        a.N = D.d;
        a.K = D.F;
        a.ldy = D.d;
        // encoder outputs the decoder's skips read (the last nskip of them)
        const int skip_slot = v - (D.enc - D.nskip);
        float *skip_out = v < D.enc && skip_slot >= 0 ? c.skip + (int64_t)skip_slot * D.n * D.d : nullptr;
        const bool mres = !par && D.mlora && b->lora;  // MLP adapter: the residual in k_mlp_resid
        if (par || mres) {
            a.Y = c.mo;
            a.epi = kEpiStore;
        } else {
            a.Y = c.x;
            a.epi = kEpiResid;
            a.R = c.x;
            a.ldr = D.d;
            a.colscale = w->mlp_scale + (int64_t)l * D.d;
            a.Y2 = skip_out;
            a.ldy2 = D.d;
        }
        if ((rc = linear(a, c.hid_h, c.hid_l, c.tc ? sp->down_hi : nullptr, c.tc ? sp->down_lo : nullptr, nullptr, nullptr, w->tiles ? &w->tiles->down : nullptr))) return rc;
        if (par)
            ALTXS_LAUNCH(::altxs::kKPostAttn, st,
                         k_par_combine<<<D.n, 128, 2 * (D.r > 0 ? D.r : 1) * 4, st>>>(c, l, v));
        if (mres) ALTXS_LAUNCH(::altxs::kKPostAttn, st, k_mlp_resid<<<D.n, 128, 0, st>>>(c, l, v, skip_out));
    }
    const int lanes = lanes_on ? desc->parallel_final : -1;
    ALTXS_LAUNCH(::altxs::kKFinal, st, k_final<<<D.n, 128, D.d * 4, st>>>(c, lanes));
    QmmArgs a{};
    a.X = c.nrm;
    a.ldx = D.d;
    a.M = D.n;
    a.W = w->emb;
    a.row0 = 0;
    a.N = D.V;
    a.K = D.d;
    a.Y = c.logits;
    a.ldy = D.V;
    a.epi = kEpiStore;
    if ((rc = linear(a, c.nrm_h, c.nrm_l, c.tc ? sp->emb_hi : nullptr, c.tc ? sp->emb_lo : nullptr, nullptr, nullptr, w->tiles ? &w->tiles->emb : nullptr))) return rc;
    {
        // a few streams: the head's logits of each row over many blocks first
        const int pre = D.n <= 8 ? 1 : 0;
        if (pre)
            ALTXS_LAUNCH(::altxs::kKCdfCode, st, k_head_rows<<<dim3(D.n, 32), 256, 0, st>>>(c));
        ALTXS_LAUNCH(::altxs::kKCdfCode, st, k_cdf_code<<<D.n, kCdfThreads, (size_t)D.V * 4, st>>>(c, mode, pre));
    }
    return ALTXS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of altxs_step.
//
// The step's scratch (activations, attention split partials, logits) normally
// lives in a workspace the caller allocates.  Some callers cannot allocate
// device memory at all: a host framework that owns the whole device budget
// through its own allocator and refuses allocations from plugins, or a
// latency-critical caller that must not risk the device-wide synchronisation
// cudaMalloc/cudaFree may imply.  For them the scratch below is a fixed
// array in this module's device memory: every GPU that loads the library
// holds these 16 MiB until the process exits, and no call allocates.
// Calls share the one array, so calls that overlap on a GPU (two streams,
// two host threads) race on it; run them one after another.  No scratch value
// needs to start at zero: the step writes every scratch value it reads.

namespace {
constexpr int64_t kNoAllocScratchBytes = 16ll << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void *g_noalloc_addr[64] = {};

// Device address of the scratch array on the current device, resolved once
// per device with that device current.
int noalloc_scratch(void **out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ALTXS_ECUDA;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return ALTXS_ECUDA;
        g_noalloc_addr[dev] = p;
    }
    *out = g_noalloc_addr[dev];
    return ALTXS_OK;
}
}  // namespace

extern "C" int64_t altxs_step_noalloc_max_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int altxs_step_noalloc(const altxs_model_desc *desc, const altxs_weights *w, const altxs_batch *b,
                                  int mode, altxs_stream_t stream) {
    if (!desc || !w || !b) return ALTXS_EINVAL;
    Dims D{};
    const int rc = fill_dims(desc, b->n_streams, D);
    if (rc) return rc;
    if (ws_size(D) > kNoAllocScratchBytes) return ALTXS_ENOSPC;  // too many streams for the fixed scratch
    void *scratch = nullptr;
    const int rs = noalloc_scratch(&scratch);
    if (rs) return rs;
    altxs_batch bb = *b;
    bb.workspace = scratch;
    bb.workspace_bytes = kNoAllocScratchBytes;
    return altxs_step(desc, w, &bb, mode, stream);
}
