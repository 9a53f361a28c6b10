// Test-time updates of one stream over a window (sm_100a): the LoRA update,
// the full-parameter gradient of replenish / "full", and the context prefill.
//
// Restates the reference online update in lora mode (altxs
// src/xsa_ttt/compress.py:1104-1137 with ttt_lora.py:124-250, 258-374):
// teacher-forced forward over x = window[0..T), targets window[1..T] with
// positions 0..T-1 and causal attention, LoRA deltas (x A^T B^T) * alpha/r on
// q/k/v/o/MLP (o on the block's normed input or on y) per layer application
// and on the tied LM head, softcap, mean cross-entropy; backward into the
// adapters only (frozen mixed-bit base); global-norm clip; AdamW step.  The
// full-parameter gradient (compress.py:611-1146) trains every parameter of the
// same forward.  The reference motifs (model.py:760-868, 1293-1500) run in
// both.  Every reduction runs in a fixed order (no atomics), so encoder and
// decoder compute identical updates.
#include <math.h>

#include "flash.cuh"
#include "gemm.cuh"
#include "model.cuh"
#include "prof.cuh"
#include "qmm.cuh"
#include "tc.cuh"

using namespace altxs;

namespace {

// Per-application tape entries are indexed by the layer application a (depth
// loops apply a physical layer i more than once); weights by i.
struct TD {
    int T, V, L, d, H, Hkv, hd, kvd, F, qn, r, G, rd;
    int A;          // layer applications (= L without depth loops)
    int enc, nskip; // encoder applications (the skips' sources); skips taken by the decoder
    int first;      // first scored position of the loss (rows before it are context only)
    int omask;      // lora_mask
    int full;       // full-parameter gradient (replenish): extra tape, P recomputed per layer
    // motifs (full-parameter gradient only)
    int smear, gw, xsa_from, sgate, asym, par, pfinal;
    float sgs;
};

constexpr int kMaxApps = 64;

enum FillMode { kFillLora, kFillPrefill, kFillFull };

struct Tape {
    // forward state
    float *x0, *x, *skip;  // skip [enc][T][d]
    // per layer application [A][...]
    float *xin, *inv1, *n, *qkv, *hinv, *qr, *kr, *P, *tq, *tk, *tv, *to, *tm, *xmid, *inv2, *n2, *u;
    // scratch
    float *y, *ao, *hbuf;
    // head
    float *invf, *hf, *logits, *tlm, *rowloss;
    // backward
    float *dx, *dskip, *dd, *dh, *dn, *dn2, *dqkv, *dqr, *dkr, *dy, *dao, *dS, *dt, *grad, *red;
    // full-parameter gradient only: layer inputs before skip and mix, attention
    // outputs, o- and down-projection outputs [L][T][d]; raw embedding rows and
    // their inverse rms; d(x0); per-row products [T][4d] and their column partials
    float *xraw, *yl, *aol, *doutl, *eraw, *inv0, *dx0, *colbuf, *cpart;
    // motifs: smeared embedding rows before the norm [T][d]; attention outputs
    // before XSA and the gate [A][T][d]; the second lane and its gradient, the
    // gradient of the attention read of a parallel block [T][d]; XSA's d(v) [T][kvd]
    float *esm, *yraw, *lane1, *dl1, *dread, *dvx;
    // flash attention: each application's rows' log-sum-exp [A][H][T] (the backward's input)
    float *lse;
};

constexpr int kColChunks = 64;  // row chunks of a column sum (summed in order)

int fill(const altxs_model_desc &dsc, int T, TD &D, FillMode mode = kFillLora) {
    const bool prefill = mode == kFillPrefill;
    D.T = T;
    D.V = dsc.vocab;
    D.L = dsc.n_layers;
    D.d = dsc.d_model;
    D.H = dsc.n_heads;
    D.Hkv = dsc.n_kv_heads;
    D.hd = dsc.head_dim;
    D.kvd = D.Hkv * D.hd;
    D.F = dsc.mlp_hidden;
    D.qn = D.d + 2 * D.kvd;
    D.r = dsc.lora_rank;
    D.G = D.H / (D.Hkv > 0 ? D.Hkv : 1);
    D.rd = dsc.rope_dims;
    D.first = 0;
    D.full = mode == kFillFull;
    D.omask = dsc.lora_mask;
    // an adapter update trains over >= 2 positions; a context prefill needs neither;
    // the full-parameter gradient trains the base itself (no adapters)
    if (mode == kFillFull) {
        if (T < 1 || D.r != 0) return ALTXS_EINVAL;
        if (D.d > 1024) return ALTXS_ENOTSUP;  // embedding scatter: 8 columns per thread of 128
    } else if (T < (prefill ? 1 : 2) || D.r < (prefill ? 0 : 1) || D.r > 128) {
        return ALTXS_EINVAL;
    }
    if (D.d % 64 || D.F % 64 || D.H % D.Hkv || D.hd * D.H != D.d) return ALTXS_EINVAL;
    if (D.hd > 128 || D.rd > D.hd || D.rd % 2) return ALTXS_EINVAL;
    D.A = dsc.n_virtual > 0 ? dsc.n_virtual : D.L;
    if (D.A != D.L && !dsc.schedule) return ALTXS_EINVAL;
    if (D.A > kMaxApps || D.L > kMaxApps) return ALTXS_ENOTSUP;
    if (dsc.schedule)
        for (int a = 0; a < D.A; ++a)
            if (dsc.schedule[a] < 0 || dsc.schedule[a] >= D.L) return ALTXS_EINVAL;
    D.enc = dsc.n_encoder > 0 ? dsc.n_encoder : D.A / 2;
    if (D.enc > D.A) return ALTXS_EINVAL;
    D.nskip = D.enc < D.A - D.enc ? D.enc : D.A - D.enc;
    if (dsc.xsa_last_n < 0 || dsc.xsa_last_n > D.L || dsc.parallel_start < 0) return ALTXS_EINVAL;
    if (dsc.parallel_final < 0 || dsc.parallel_final > 2) return ALTXS_EINVAL;
    D.smear = dsc.smear_gate != 0;
    D.sgate = dsc.sparse_gate != 0;
    D.sgs = dsc.sparse_gate_scale;
    D.xsa_from = dsc.xsa_last_n > 0 ? D.L - dsc.xsa_last_n : D.L;
    D.asym = dsc.asym_softcap != 0;
    D.par = dsc.parallel_start;
    D.pfinal = dsc.parallel_final;
    D.gw = 0;
    if (D.smear || D.sgate) {
        D.gw = dsc.gate_window;
        if (D.gw < 1 || D.gw > D.d || (D.sgate && (D.gw > D.hd || D.H > 128))) return ALTXS_EINVAL;
    }
    // parallel lanes: once a decoder application runs two lanes, every later one
    // must (the reference would run a plain block on its stale single stream)
    if (D.par > 0) {
        bool on = false;
        for (int a = D.enc; a < D.A; ++a) {
            const bool p = (dsc.schedule ? dsc.schedule[a] : a) >= D.par;
            if (on && !p) return ALTXS_ENOTSUP;
            on = on || p;
        }
    }
    return ALTXS_OK;
}

// the layer application a runs two lanes (a decoder application of a layer >= parallel_start)
inline bool par_app(const TD &D, const int *sched, int a) { return D.par > 0 && a >= D.enc && sched[a] >= D.par; }
// attention output rewritten before the o-projection (XSA on this layer, or the sparse gate)
inline bool ymotif(const TD &D, int i) { return i >= D.xsa_from || D.sgate; }

int64_t carve(const TD &D, void *base, Tape *tp) {
    unsigned char *p = static_cast<unsigned char *>(base);
    int64_t off = 0;
    auto take = [&](int64_t nfl) -> float * {
        float *r = base ? reinterpret_cast<float *>(p + off) : nullptr;
        off += align_up(nfl * 4, 256);
        return r;
    };
    const int64_t T = D.T, L = D.A, d = D.d;  // per-application arrays
    Tape t{};
    t.x0 = take(T * d);
    t.x = take(T * d);
    t.skip = take((int64_t)(D.enc > 0 ? D.enc : 1) * T * d);
    t.xin = take(L * T * d);
    t.inv1 = take(L * T);
    t.n = take(L * T * d);
    t.qkv = take(L * T * D.qn);
    t.hinv = take(L * T * (D.H + D.Hkv));
    t.qr = take(L * T * d);
    t.kr = take(L * T * D.kvd);
    // fp32 [H][T][T], or bf16 hi/lo planes [2][H][T][align8(T)], per layer; one layer
    // (recomputed in the backward) for the full-parameter gradient
    t.P = take((D.full ? 1 : L) * D.H * T * align_up(T, 8));
    t.tq = take(L * T * D.r);
    t.tk = take(L * T * D.r);
    t.tv = take(L * T * D.r);
    t.to = take(L * T * D.r);
    t.tm = take(L * T * D.r);
    t.xmid = take(L * T * d);
    t.inv2 = take(L * T);
    t.n2 = take(L * T * d);
    t.u = take(L * T * D.F);
    t.y = take(T * d);
    t.ao = take(T * d);
    t.hbuf = take(T * D.F);
    t.invf = take(T);
    t.hf = take(T * d);
    t.logits = take(T * D.V);
    t.tlm = take(T * D.r);
    t.rowloss = take(T);
    t.dx = take(T * d);
    t.dskip = take((int64_t)(D.enc > 0 ? D.enc : 1) * T * d);
    t.dd = take(T * d);
    t.dh = take(T * D.F);
    t.dn = take(T * d);
    t.dn2 = take(T * d);
    t.dqkv = take(T * D.qn);
    t.dqr = take(T * d);
    t.dkr = take(T * D.kvd);
    t.dy = take(T * d);
    t.dao = take(T * d);
    t.dS = take((int64_t)D.H * T * align_up(T, 8));  // fp32 scores / dP, rows of stride align8(T) on the tensor-core path
    t.dt = take(T * 3 * (D.r > 0 ? D.r : 1));  // up to three adapters sharing an input
    t.grad = nullptr;  // set by caller (lora_floats)
    t.red = take(1024);
    t.lse = take(L * D.H * T);
    // the attention output per layer (the o adapter's input on y, and the flash
    // backward's; the full-parameter gradient takes it below)
    if (!D.full) t.yl = take(L * T * d);
    if (D.par && !D.full) {  // the lanes' combine and its backward read each application's outputs
        t.aol = take(L * T * d);
        t.doutl = take(L * T * d);
    }
    if (D.xsa_from < D.L || D.sgate) t.yraw = take(L * T * d);
    if (D.par) {
        t.lane1 = take(T * d);
        t.dl1 = take(T * d);
        t.dread = take(T * d);
    }
    if (D.xsa_from < D.L) t.dvx = take(T * D.kvd);
    if (D.full) {
        t.xraw = take(L * T * d);
        t.yl = take(L * T * d);
        t.aol = take(L * T * d);
        t.doutl = take(L * T * d);
        t.eraw = take(T * d);
        t.inv0 = take(T);
        t.dx0 = take(T * d);
        int64_t cw = 4 * d > D.H ? 4 * d : D.H;
        cw = cw > (int64_t)D.H * D.gw ? cw : (int64_t)D.H * D.gw;  // sparse gate weights
        cw = cw > D.gw + 1 ? cw : D.gw + 1;                          // smear gate, lambda
        t.colbuf = take(T * cw);
        t.cpart = take((int64_t)kColChunks * cw);
        if (D.smear) t.esm = take(T * d);
    }
    if (tp) *tp = t;
    return off;
}

// ---- forward row kernels -------------------------------------------------

// embedding rows (dense fp32 copy when given, else the mixed-bit codes) + RMSNorm;
// the full-parameter gradient keeps the raw rows and their inverse rms.  Smear
// gate (model.py:1364-1375): row t >= 1 adds lambda*sigmoid(raw_t[:gw] . g) times
// row t-1; the window's first row is left alone.
__device__ __forceinline__ float emb_row_elem(const TD &D, altxs_qmat emb, const float *embd, int tk, int k) {
    if (tk < 0 || tk >= D.V) return 0.0f;
    return embd ? embd[(int64_t)tk * D.d + k] : qmat_elem(emb, tk, k);
}
__global__ void t_embed(TD D, const int32_t *tok, altxs_qmat emb, const float *embd, float *x0, float *x, Tape tp,
                        altxs_weights w) {
    __shared__ float red[32];
    const int t = blockIdx.x;
    const int tk = tok[t];
    float gate = 0.0f;
    if (D.smear && t > 0) {
        float z = 0.0f;
        for (int k = threadIdx.x; k < D.gw; k += blockDim.x) z = __fmaf_rn(emb_row_elem(D, emb, embd, tk, k), w.smear_gate[k], z);
        z = block_sum(z, red);
        gate = __fmul_rn(w.smear_lambda[0], sigmoidf_(z));
        __syncthreads();
    }
    float ss = 0.0f;
    for (int k = threadIdx.x; k < D.d; k += blockDim.x) {
        float v = emb_row_elem(D, emb, embd, tk, k);
        if (tp.eraw) tp.eraw[(int64_t)t * D.d + k] = v;
        if (D.smear && t > 0) v = __fadd_rn(v, __fmul_rn(gate, emb_row_elem(D, emb, embd, tok[t - 1], k)));
        if (tp.esm) tp.esm[(int64_t)t * D.d + k] = v;
        x0[(int64_t)t * D.d + k] = v;
        ss = __fmaf_rn(v, v, ss);
    }
    const float inv = rms_inv(block_sum(ss, red), D.d);
    if (tp.inv0 && threadIdx.x == 0) tp.inv0[t] = inv;
    __syncthreads();
    for (int k = threadIdx.x; k < D.d; k += blockDim.x) {
        const float v = __fmul_rn(x0[(int64_t)t * D.d + k], inv);
        x0[(int64_t)t * D.d + k] = v;
        x[(int64_t)t * D.d + k] = v;
    }
}

// application a of layer i: the skip of decoder application j (-1: none) into
// the stream, then x_in = mix0 * x + mix1 * x0 and its normed, ln-scaled form.
// A parallel application (par) keeps lane 0 (after the skip) as its stream and
// x_in only as the attention's read (model.py:1310-1317).
__global__ void t_prenorm(TD D, int a, int i, int j, int par, Tape tp, altxs_weights w, int skip_gates) {
    __shared__ float red[32];
    const int t = blockIdx.x, d = D.d, l = a;
    float *x = tp.x + (int64_t)t * d;
    const float *x0 = tp.x0 + (int64_t)t * d;
    const float *mix = w.resid_mix + (int64_t)i * 2 * d;
    const bool skip = j >= 0;
    const float *sk = skip ? tp.skip + ((int64_t)(D.enc - 1 - j) * D.T + t) * d : nullptr;
    float *xin = tp.xin + ((int64_t)l * D.T + t) * d;
    float *xr = tp.xraw ? tp.xraw + ((int64_t)l * D.T + t) * d : nullptr;
    float ss = 0.0f;
    for (int k = threadIdx.x; k < d; k += blockDim.x) {
        float xv = x[k];
        if (xr) xr[k] = xv;
        if (skip) {
            const float scaled = __fmul_rn(w.skip_weights[(int64_t)j * d + k], sk[k]);
            xv = skip_gates ? lerp_t(scaled, xv, sigmoidf_(w.skip_gates[(int64_t)j * d + k])) : __fadd_rn(xv, scaled);
        }
        const float v = __fadd_rn(__fmul_rn(mix[k], xv), __fmul_rn(mix[d + k], x0[k]));
        xin[k] = v;
        x[k] = par ? xv : v;
        ss = __fmaf_rn(v, v, ss);
    }
    const float inv = rms_inv(block_sum(ss, red), d);
    const float ln = w.ln_scale[i];
    if (threadIdx.x == 0) tp.inv1[(int64_t)l * D.T + t] = inv;
    __syncthreads();
    float *nr = tp.n + ((int64_t)l * D.T + t) * d;
    for (int k = threadIdx.x; k < d; k += blockDim.x) nr[k] = __fmul_rn(__fmul_rn(xin[k], inv), ln);
}

// per-head RMSNorm + RoPE (positions 0..T-1) + q_gain; one warp per head
__global__ void t_qk(TD D, int l, int i, Tape tp, altxs_weights w) {
    const int t = blockIdx.x, hd = D.hd, half = D.rd / 2;
    const float *qkv = tp.qkv + ((int64_t)l * D.T + t) * D.qn;
    const float *cs = w.rope_cos + (int64_t)t * half, *sn = w.rope_sin + (int64_t)t * half;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int h = wid; h < D.H + D.Hkv; h += nw) {
        const float *e = qkv + (int64_t)h * hd;
        float ss = 0.0f;
        for (int k = lane; k < hd; k += 32) ss = __fmaf_rn(e[k], e[k], ss);
        const float inv = rms_inv(warp_sum(ss), hd);
        if (lane == 0) tp.hinv[((int64_t)l * D.T + t) * (D.H + D.Hkv) + h] = inv;
        float *dst;
        float g = 1.0f;
        if (h < D.H) {
            dst = tp.qr + ((int64_t)l * D.T + t) * D.d + (int64_t)h * hd;
            g = w.q_gain[(int64_t)i * D.H + h];
        } else {
            dst = tp.kr + ((int64_t)l * D.T + t) * D.kvd + (int64_t)(h - D.H) * hd;
        }
        for (int k = lane; k < hd; k += 32) {
            const float a = __fmul_rn(e[k], inv);
            float r = a;
            if (k < D.rd) {
                if (k < half) {
                    r = __fadd_rn(__fmul_rn(a, cs[k]), __fmul_rn(__fmul_rn(e[k + half], inv), sn[k]));
                } else {
                    r = __fadd_rn(__fmul_rn(__fmul_rn(e[k - half], inv), -sn[k - half]), __fmul_rn(a, cs[k - half]));
                }
            }
            dst[k] = h < D.H ? __fmul_rn(r, g) : r;
        }
    }
}

// causal softmax over rows of S (in place): one block per (head, t)
__global__ void t_softmax(TD D, float *P) {
    __shared__ float red[32];
    const int row = blockIdx.x;  // h * T + t
    const int t = row % D.T;
    float *s = P + (int64_t)row * D.T;
    float m = -INFINITY;
    for (int j = threadIdx.x; j <= t; j += blockDim.x) m = fmaxf(m, s[j]);
    m = block_max(m, red);
    __syncthreads();
    float sum = 0.0f;
    for (int j = threadIdx.x; j < D.T; j += blockDim.x) {
        const float e = j <= t ? expf(__fsub_rn(s[j], m)) : 0.0f;
        s[j] = e;
        sum = __fadd_rn(sum, e);
    }
    sum = block_sum(sum, red);
    __syncthreads();
    const float inv = __fdiv_rn(1.0f, sum);
    for (int j = threadIdx.x; j < D.T; j += blockDim.x) s[j] = __fmul_rn(s[j], inv);
}

// MLP input of application l (layer i): x_in + attn_scale * attention output, or
// in a parallel application lane 1 (model.py:1337-1339); kept with its inverse rms
__global__ void t_post_attn(TD D, int l, int i, Tape tp, altxs_weights w, const float *aob, int par) {
    __shared__ float red[32];
    const int t = blockIdx.x, d = D.d;
    const float *xin = tp.xin + ((int64_t)l * D.T + t) * d;
    const float *ao = aob + (int64_t)t * d;
    const float *as = w.attn_scale + (int64_t)i * d;
    float *xm = tp.xmid + ((int64_t)l * D.T + t) * d;
    float ss = 0.0f;
    for (int k = threadIdx.x; k < d; k += blockDim.x) {
        const float v = par ? tp.lane1[(int64_t)t * d + k] : __fadd_rn(xin[k], __fmul_rn(as[k], ao[k]));
        xm[k] = v;
        ss = __fmaf_rn(v, v, ss);
    }
    const float inv = rms_inv(block_sum(ss, red), d);
    const float ln = w.ln_scale[i];
    if (threadIdx.x == 0) tp.inv2[(int64_t)l * D.T + t] = inv;
    __syncthreads();
    float *n2 = tp.n2 + ((int64_t)l * D.T + t) * d;
    for (int k = threadIdx.x; k < d; k += blockDim.x) n2[k] = __fmul_rn(__fmul_rn(xm[k], inv), ln);
}

__global__ void t_leaky(int64_t n, const float *u, float *h) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = u[i];
    const float a = v >= 0.0f ? v : __fmul_rn(v, 0.5f);
    h[i] = __fmul_rn(a, a);
}

// final RMSNorm; after parallel lanes the hidden state is first their mean,
// lane 0 or lane 1 (model.py:1357-1362), written back into the stream
__global__ void t_final(TD D, Tape tp, int lanes) {
    __shared__ float red[32];
    const int t = blockIdx.x, d = D.d;
    float *x = tp.x + (int64_t)t * d;
    if (lanes) {
        const float *l1 = tp.lane1 + (int64_t)t * d;
        for (int k = threadIdx.x; k < d; k += blockDim.x)
            x[k] = D.pfinal == 0 ? __fmul_rn(0.5f, __fadd_rn(x[k], l1[k])) : D.pfinal == 1 ? x[k] : l1[k];
        __syncthreads();
    }
    float ss = 0.0f;
    for (int k = threadIdx.x; k < d; k += blockDim.x) ss = __fmaf_rn(x[k], x[k], ss);
    const float inv = rms_inv(block_sum(ss, red), d);
    if (threadIdx.x == 0) tp.invf[t] = inv;
    for (int k = threadIdx.x; k < d; k += blockDim.x) tp.hf[(int64_t)t * d + k] = __fmul_rn(x[k], inv);
}

// softcap + cross-entropy; logits row -> d(loss)/d(raw logits) in place.  With
// the asymmetric softcap (sc = {positive, negative} caps, model.py:1478-1493) the
// row's contributions to d(cap) go to scrow[t][2].
__global__ void t_ce(TD D, const int32_t *tgt, Tape tp, float cap, const float *sc, float *scrow) {
    __shared__ float red[32];
    const int t = blockIdx.x;
    float *l = tp.logits + (int64_t)t * D.V;
    if (t < D.first) {  // context row: not scored
        for (int j = threadIdx.x; j < D.V; j += blockDim.x) l[j] = 0.0f;
        if (threadIdx.x == 0) tp.rowloss[t] = 0.0f;
        if (scrow && threadIdx.x < 2) scrow[2 * t + threadIdx.x] = 0.0f;
        return;
    }
    const float cp = sc ? sc[0] : cap, cn = sc ? sc[1] : cap;
    const int y = tgt[t];
    float m = -INFINITY;
    for (int j = threadIdx.x; j < D.V; j += blockDim.x) {
        const float c = l[j] >= 0.0f ? cp : cn;
        const float z = __fmul_rn(c, tanhf(__fdiv_rn(l[j], c)));
        m = fmaxf(m, z);
    }
    m = block_max(m, red);
    __syncthreads();
    float s = 0.0f;
    for (int j = threadIdx.x; j < D.V; j += blockDim.x) {
        const float c = l[j] >= 0.0f ? cp : cn;
        const float z = __fmul_rn(c, tanhf(__fdiv_rn(l[j], c)));
        s = __fadd_rn(s, expf(__fsub_rn(z, m)));
    }
    s = block_sum(s, red);
    __syncthreads();
    const float lse = __fadd_rn(m, logf(s));
    const float invT = __fdiv_rn(1.0f, (float)(D.T - D.first));
    float gp = 0.0f, gn = 0.0f;
    for (int j = threadIdx.x; j < D.V; j += blockDim.x) {
        const float lj = l[j];
        const bool pos = lj >= 0.0f;
        const float c = pos ? cp : cn;
        const float u = __fdiv_rn(lj, c);
        const float th = tanhf(u);
        const float z = __fmul_rn(c, th);
        if (j == y) tp.rowloss[t] = __fsub_rn(lse, z);
        float p = __fdiv_rn(expf(__fsub_rn(z, m)), s);
        if (j == y) p = __fsub_rn(p, 1.0f);
        const float dz = __fmul_rn(p, invT);
        const float sech2 = __fsub_rn(1.0f, __fmul_rn(th, th));
        l[j] = __fmul_rn(dz, sech2);
        if (scrow) {  // d(c tanh(l/c))/dc = tanh(u) - u (1 - tanh(u)^2)
            const float dc = __fmul_rn(dz, __fsub_rn(th, __fmul_rn(u, sech2)));
            if (pos) gp = __fadd_rn(gp, dc);
            else gn = __fadd_rn(gn, dc);
        }
    }
    if (scrow) {
        gp = block_sum(gp, red);
        gn = block_sum(gn, red);
        if (threadIdx.x == 0) {
            scrow[2 * t] = gp;
            scrow[2 * t + 1] = gn;
        }
    }
}

// XSA and the sparse attention gate on one row of application l, layer i
// (model.py:760-768, 845-862): per head, y -= (y . v^) v^ with v^ the head's KV
// group value at the same position over its norm (floored at 1e-12), when
// layer i is one of the last xsa_last_n; then y *= sigmoid(scale * w_h . n[:gw])
// with n the block's normed attention input.  yraw -> yl; one warp per head.
__global__ void t_xsa_gate(TD D, int l, int i, Tape tp, altxs_weights w, float *yout) {
    const int t = blockIdx.x, hd = D.hd, lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int64_t row = (int64_t)l * D.T + t;
    const float *yr = tp.yraw + row * D.d, *nr = tp.n + row * D.d;
    const float *vr = tp.qkv + row * D.qn + D.d + D.kvd;
    float *yo = yout + (int64_t)t * D.d;
    const bool xsa = i >= D.xsa_from;
    for (int h = wid; h < D.H; h += nw) {
        float y[4], v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int k = lane + 32 * u;
            y[u] = k < hd ? yr[(int64_t)h * hd + k] : 0.0f;
            v[u] = k < hd ? vr[(int64_t)(h / D.G) * hd + k] : 0.0f;
        }
        if (xsa) {
            float ss = 0.0f;
#pragma unroll
            for (int u = 0; u < 4; ++u) ss = __fmaf_rn(v[u], v[u], ss);
            const float den = fmaxf(__fsqrt_rn(warp_sum(ss)), 1e-12f);
            float dot = 0.0f;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                v[u] = __fdiv_rn(v[u], den);
                dot = __fmaf_rn(y[u], v[u], dot);
            }
            dot = warp_sum(dot);
#pragma unroll
            for (int u = 0; u < 4; ++u) y[u] = __fsub_rn(y[u], __fmul_rn(dot, v[u]));
        }
        if (D.sgate) {
            const float *gwr = w.attn_gate_w + ((int64_t)i * D.H + h) * D.gw;
            float z = 0.0f;
            for (int k = lane; k < D.gw; k += 32) z = __fmaf_rn(nr[k], gwr[k], z);
            const float g = sigmoidf_(__fmul_rn(D.sgs, warp_sum(z)));
#pragma unroll
            for (int u = 0; u < 4; ++u) y[u] = __fmul_rn(y[u], g);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (lane + 32 * u < hd) yo[(int64_t)h * hd + lane + 32 * u] = y[u];
    }
}

// parallel lanes after application l of layer i (model.py:1336-1351):
// lane0 = r0 lane0 + p00 a + p10 m, lane1 = r1 lane1 + p01 a + p11 m with
// a = attn_scale * (o-projection), m = mlp_scale * (down-projection)
__global__ void t_par_combine(int64_t n, int d, int l, int i, Tape tp, altxs_weights w, int T) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= n) return;
    const int k = (int)(e % d);
    const float A = __fmul_rn(w.attn_scale[(int64_t)i * d + k], tp.aol[(int64_t)l * T * d + e]);
    const float M = __fmul_rn(w.mlp_scale[(int64_t)i * d + k], tp.doutl[(int64_t)l * T * d + e]);
    const float *pr = w.parallel_resid + 2 * i, *pp = w.parallel_post + 4 * i;
    tp.x[e] = __fadd_rn(__fadd_rn(__fmul_rn(pr[0], tp.x[e]), __fmul_rn(pp[0], A)), __fmul_rn(pp[2], M));
    tp.lane1[e] = __fadd_rn(__fadd_rn(__fmul_rn(pr[1], tp.lane1[e]), __fmul_rn(pp[1], A)), __fmul_rn(pp[3], M));
}

// mean of the scored rows' losses (rows before `first` hold 0)
__global__ void t_loss_sum(int T, int first, const float *rowloss, float *out) {
    __shared__ float red[32];
    float s = 0.0f;
    for (int t = threadIdx.x; t < T; t += blockDim.x) s = __fadd_rn(s, rowloss[t]);
    s = block_sum(s, red);
    if (threadIdx.x == 0 && out) *out = __fdiv_rn(s, (float)(T - first));
}

// ---- backward row kernels -----------------------------------------------

// out = (add ? add : 0) + d/dx[rms(x) * scale] applied to g
__global__ void t_rms_bwd(int d, const float *g, int64_t ldg, const float *x, const float *inv,
                          const float *scale_ptr, const float *add, float *out) {
    __shared__ float red[32];
    const int t = blockIdx.x;
    const float scale = scale_ptr ? *scale_ptr : 1.0f;
    const float *gr = g + (int64_t)t * ldg, *xr = x + (int64_t)t * d;
    const float iv = inv[t];
    float dot = 0.0f;
    for (int k = threadIdx.x; k < d; k += blockDim.x) dot = __fmaf_rn(__fmul_rn(gr[k], scale), xr[k], dot);
    dot = block_sum(dot, red);
    const float c = __fdiv_rn(__fmul_rn(__fmul_rn(iv, iv), __fmul_rn(iv, dot)), (float)d);
    for (int k = threadIdx.x; k < d; k += blockDim.x) {
        float v = __fsub_rn(__fmul_rn(iv, __fmul_rn(gr[k], scale)), __fmul_rn(xr[k], c));
        if (add) v = __fadd_rn(add[(int64_t)t * d + k], v);
        out[(int64_t)t * d + k] = v;
    }
}

__global__ void t_scale_cols(int64_t n, int d, const float *a, const float *col, float *out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    out[i] = __fmul_rn(a[i], col[i % d]);
}

__global__ void t_leaky_bwd(int64_t n, const float *dh, const float *u, float *du) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = u[i];
    du[i] = __fmul_rn(dh[i], v >= 0.0f ? __fmul_rn(2.0f, v) : __fmul_rn(0.5f, v));
}

// dS = P * (dP - sum_j dP P) * scale, per (head, row), in place over dP.
// Only j <= t is read (dP above the diagonal is never computed); dS there is 0.
__global__ void t_softmax_bwd(TD D, const float *P, float *dS, float scale) {
    __shared__ float red[32];
    const int row = blockIdx.x;
    const int t = row % D.T;
    const float *p = P + (int64_t)row * D.T;
    float *g = dS + (int64_t)row * D.T;
    float s = 0.0f;
    for (int j = threadIdx.x; j <= t; j += blockDim.x) s = __fmaf_rn(g[j], p[j], s);
    s = block_sum(s, red);
    for (int j = threadIdx.x; j < D.T; j += blockDim.x)
        g[j] = j <= t ? __fmul_rn(__fmul_rn(p[j], __fsub_rn(g[j], s)), scale) : 0.0f;
}

// Plane forms of the two softmax kernels (tensor-core path).  The scores S
// (and dP) come in fp32 rows of stride ldp = align8(T); P (and dS) leave as
// hi/lo bf16 planes [H][T][ldp].  Row t is written only up to the end of its
// 128-column diagonal tile (zero past t): the products that read the planes
// (P v and dS k with k < m0 + 128, P^T dy and dS^T q with k >= m0) never read
// further.  Each thread takes 8 consecutive columns per pass with 16-byte loads
// and stores; one CTA per (head, t) row.
__device__ __forceinline__ void load8(const float *p, float *v) {
    const float4 a = reinterpret_cast<const float4 *>(p)[0], b = reinterpret_cast<const float4 *>(p)[1];
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
__device__ __forceinline__ void store8_planes(uint16_t *hi, uint16_t *lo, int64_t idx, const float *v) {
    uint16_t h[8], l[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const __nv_bfloat16 b = __float2bfloat16_rn(v[u]);
        h[u] = __bfloat16_as_ushort(b);
        l[u] = __bfloat16_as_ushort(__float2bfloat16_rn(__fsub_rn(v[u], __bfloat162float(b))));
    }
    *reinterpret_cast<uint4 *>(hi + idx) = *reinterpret_cast<const uint4 *>(h);
    *reinterpret_cast<uint4 *>(lo + idx) = *reinterpret_cast<const uint4 *>(l);
}
__device__ __forceinline__ void load8_planes(const uint16_t *hi, const uint16_t *lo, int64_t idx, float *v) {
    const uint4 a = *reinterpret_cast<const uint4 *>(hi + idx), b = *reinterpret_cast<const uint4 *>(lo + idx);
    const uint16_t *h = reinterpret_cast<const uint16_t *>(&a), *l = reinterpret_cast<const uint16_t *>(&b);
#pragma unroll
    for (int u = 0; u < 8; ++u)
        v[u] = __fadd_rn(__bfloat162float(__ushort_as_bfloat16(h[u])), __bfloat162float(__ushort_as_bfloat16(l[u])));
}
__device__ __forceinline__ int64_t diag_end(int n, int64_t ldp) {
    const int64_t e = ((int64_t)n + 127) / 128 * 128;
    return e < ldp ? e : ldp;
}

__global__ void __launch_bounds__(256) t_softmax_pl(TD D, const float *S, uint16_t *ph, uint16_t *pl, int64_t ldp) {
    __shared__ float red[32];
    const int row = blockIdx.x;  // h * T + t
    const int n = row % D.T + 1;  // scores 0..t
    const float *s = S + (int64_t)row * ldp;
    const int nc = (n + 7) / 8;
    float v[8];
    float m = -INFINITY;
    for (int c = threadIdx.x; c < nc; c += blockDim.x) {
        load8(s + 8 * c, v);
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (8 * c + u < n) m = fmaxf(m, v[u]);
    }
    m = block_max(m, red);
    float sum = 0.0f;
    for (int c = threadIdx.x; c < nc; c += blockDim.x) {
        load8(s + 8 * c, v);
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (8 * c + u < n) sum = __fadd_rn(sum, expf(__fsub_rn(v[u], m)));
    }
    sum = block_sum(sum, red);
    const float inv = __fdiv_rn(1.0f, sum);
    const int64_t o = (int64_t)row * ldp;
    const int wc = (int)(diag_end(n, ldp) / 8);
    for (int c = threadIdx.x; c < wc; c += blockDim.x) {
        if (c < nc) load8(s + 8 * c, v);
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = 8 * c + u < n ? __fmul_rn(expf(__fsub_rn(v[u], m)), inv) : 0.0f;
        store8_planes(ph, pl, o + 8 * c, v);
    }
}

// dS = P * (dP - sum_j dP P) * scale over j <= t (dP above the diagonal is never computed)
__global__ void __launch_bounds__(256) t_softmax_bwd_pl(TD D, const uint16_t *ph, const uint16_t *pl, int64_t ldp,
                                                        const float *dP, uint16_t *gh, uint16_t *gl, float scale) {
    __shared__ float red[32];
    const int row = blockIdx.x;
    const int n = row % D.T + 1;
    const int64_t o = (int64_t)row * ldp;
    const float *g = dP + o;
    const int nc = (n + 7) / 8;
    float pv[8], gv[8];
    float sdot = 0.0f;
    for (int c = threadIdx.x; c < nc; c += blockDim.x) {
        load8_planes(ph, pl, o + 8 * c, pv);
        load8(g + 8 * c, gv);
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (8 * c + u < n) sdot = __fmaf_rn(gv[u], pv[u], sdot);
    }
    sdot = block_sum(sdot, red);
    const int wc = (int)(diag_end(n, ldp) / 8);
    for (int c = threadIdx.x; c < wc; c += blockDim.x) {
        float out[8];
        if (c < nc) {
            load8_planes(ph, pl, o + 8 * c, pv);
            load8(g + 8 * c, gv);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
            out[u] = 8 * c + u < n ? __fmul_rn(__fmul_rn(pv[u], __fsub_rn(gv[u], sdot)), scale) : 0.0f;
        store8_planes(gh, gl, o + 8 * c, out);
    }
}

// context prefill: K (normed, roped) and V rows of position t, layer
// application l into slot t % ctx of one stream's ring [A][2][Hkv][ctx][3*hd]
// (24-bit rows; depth loops give each application its own K/V set)
__global__ void t_kv_write(TD D, Tape tp, uint8_t *kv, int64_t ctx) {
    const int t = blockIdx.x, l = blockIdx.y, hd = D.hd;
    const int64_t rb = 3 * (int64_t)hd, slot = t % ctx;
    const float *kr = tp.kr + ((int64_t)l * D.T + t) * D.kvd;
    const float *v = tp.qkv + ((int64_t)l * D.T + t) * D.qn + D.d + D.kvd;
    uint8_t *base = kv + (int64_t)l * 2 * D.Hkv * ctx * rb;
    for (int e = threadIdx.x; e < D.kvd; e += blockDim.x) {
        const int h = e / hd, c = e - h * hd;
        store_kv_row(base + ((int64_t)h * ctx + slot) * rb, hd, c, kr[e]);
        store_kv_row(base + ((int64_t)(D.Hkv + h) * ctx + slot) * rb, hd, c, v[e]);
    }
}

// x = r + colscale * y (row stride d), optional copy into y2
__global__ void t_resid(int64_t n, int d, const float *r, const float *col, const float *y, float *x, float *y2) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = __fadd_rn(r[i], __fmul_rn(col[i % d], y[i]));
    x[i] = v;
    if (y2) y2[i] = v;
}

// q/k: undo gain, RoPE transpose, per-head RMSNorm backward -> dqkv
__global__ void t_qk_bwd(TD D, int l, int i, Tape tp, altxs_weights w) {
    const int t = blockIdx.x, hd = D.hd, half = D.rd / 2;
    const float *qkv = tp.qkv + ((int64_t)l * D.T + t) * D.qn;
    const float *cs = w.rope_cos + (int64_t)t * half, *sn = w.rope_sin + (int64_t)t * half;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float *dq = tp.dqkv + (int64_t)t * D.qn;
    for (int h = wid; h < D.H + D.Hkv; h += nw) {
        const float *e = qkv + (int64_t)h * hd;
        const float inv = tp.hinv[((int64_t)l * D.T + t) * (D.H + D.Hkv) + h];
        const float *gsrc;
        float g = 1.0f;
        if (h < D.H) {
            gsrc = tp.dqr + (int64_t)t * D.d + (int64_t)h * hd;
            g = w.q_gain[(int64_t)i * D.H + h];
        } else {
            gsrc = tp.dkr + (int64_t)t * D.kvd + (int64_t)(h - D.H) * hd;
        }
        // grad wrt the normed (pre-rope) vector a_k, then RMS backward
        float dot = 0.0f;
        float ga[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int k = lane + 32 * u;
            float v = 0.0f;
            if (k < hd) {
                if (k < D.rd) {
                    if (k < half) {  // a_k feeds out_k (cos) and out_{k+half} (-sin)
                        v = __fsub_rn(__fmul_rn(__fmul_rn(gsrc[k], g), cs[k]), __fmul_rn(__fmul_rn(gsrc[k + half], g), sn[k]));
                    } else {  // a_k feeds out_{k-half} (sin) and out_k (cos)
                        v = __fadd_rn(__fmul_rn(__fmul_rn(gsrc[k - half], g), sn[k - half]), __fmul_rn(__fmul_rn(gsrc[k], g), cs[k - half]));
                    }
                } else {
                    v = __fmul_rn(gsrc[k], g);
                }
                dot = __fmaf_rn(v, e[k], dot);
            }
            ga[u] = v;
        }
        dot = warp_sum(dot);
        if (D.full && h < D.H) {  // d q_gain[h] = sum_k dout_k * (roped, normed q)_k
            float gd = 0.0f;
            for (int k = lane; k < hd; k += 32) {
                const float a = __fmul_rn(e[k], inv);
                float r = a;
                if (k < D.rd) {
                    if (k < half)
                        r = __fadd_rn(__fmul_rn(a, cs[k]), __fmul_rn(__fmul_rn(e[k + half], inv), sn[k]));
                    else
                        r = __fadd_rn(__fmul_rn(__fmul_rn(e[k - half], inv), -sn[k - half]), __fmul_rn(a, cs[k - half]));
                }
                gd = __fmaf_rn(gsrc[k], r, gd);
            }
            gd = warp_sum(gd);
            if (lane == 0) tp.colbuf[(int64_t)t * D.H + h] = gd;
        }
        const float c = __fdiv_rn(__fmul_rn(__fmul_rn(inv, inv), __fmul_rn(inv, dot)), (float)hd);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int k = lane + 32 * u;
            if (k < hd) dq[(int64_t)h * hd + k] = __fsub_rn(__fmul_rn(inv, ga[u]), __fmul_rn(e[k], c));
        }
    }
}

// residual mix and skip lerp backward of application l (layer i, skip of
// decoder application j or -1): dx <- d(loss)/d(input of the application).  In
// a sequential block dx holds d(x_in); in a parallel one d(x_in) (the
// attention read) comes in tp.dread and dx holds the residual lane's r0 * d(lane0).
// The full-parameter gradient also adds mix1 * d(x_in) into d(x0) and leaves
// per-row products for the column sums: [0,d) d(mix0), [d,2d) d(mix1), [2d,3d)
// d(skip_weights), [3d,4d) d(skip_gates).
__global__ void t_mix_bwd(TD D, int l, int i, int j, int par, Tape tp, altxs_weights w, int skip_gates) {
    const int t = blockIdx.x, d = D.d;
    const float *mix = w.resid_mix + (int64_t)i * 2 * d;
    const bool skip = j >= 0;
    float *dx = tp.dx + (int64_t)t * d;
    const float *gread = par ? tp.dread + (int64_t)t * d : dx;
    float *ds = skip ? tp.dskip + ((int64_t)(D.enc - 1 - j) * D.T + t) * d : nullptr;
    const float *sk = skip ? tp.skip + ((int64_t)(D.enc - 1 - j) * D.T + t) * d : nullptr;
    for (int k = threadIdx.x; k < d; k += blockDim.x) {
        const float gin = gread[k];
        // d(stream after the skip): through the mix, plus the parallel lane's residual
        const float gx = par ? __fadd_rn(__fmul_rn(gin, mix[k]), dx[k]) : __fmul_rn(gin, mix[k]);
        if (D.full) {
            const float xr = tp.xraw[((int64_t)l * D.T + t) * d + k];
            float xv = xr, scaled = 0.0f, gg = 0.0f;
            if (skip) {
                scaled = __fmul_rn(w.skip_weights[(int64_t)j * d + k], sk[k]);
                if (skip_gates) {
                    gg = sigmoidf_(w.skip_gates[(int64_t)j * d + k]);
                    xv = lerp_t(scaled, xr, gg);
                } else {
                    xv = __fadd_rn(xr, scaled);
                }
            }
            float *cb = tp.colbuf + (int64_t)t * 4 * d;
            cb[k] = __fmul_rn(gin, xv);
            cb[d + k] = __fmul_rn(gin, tp.x0[(int64_t)t * d + k]);
            float *g0 = tp.dx0 + (int64_t)t * d + k;
            *g0 = __fadd_rn(*g0, __fmul_rn(mix[d + k], gin));
            if (skip) {
                const float gv = gx;
                if (skip_gates) {
                    cb[2 * d + k] = __fmul_rn(__fmul_rn(gv, __fsub_rn(1.0f, gg)), sk[k]);
                    cb[3 * d + k] = __fmul_rn(__fmul_rn(gv, __fsub_rn(xr, scaled)), __fmul_rn(gg, __fsub_rn(1.0f, gg)));
                } else {
                    cb[2 * d + k] = __fmul_rn(gv, sk[k]);
                    cb[3 * d + k] = 0.0f;
                }
            }
        }
        if (skip) {
            const float sw = w.skip_weights[(int64_t)j * d + k];
            if (skip_gates) {
                const float gg = sigmoidf_(w.skip_gates[(int64_t)j * d + k]);
                ds[k] = __fmul_rn(__fmul_rn(gx, __fsub_rn(1.0f, gg)), sw);
                dx[k] = __fmul_rn(gx, gg);
            } else {
                ds[k] = __fmul_rn(gx, sw);
                dx[k] = gx;
            }
        } else {
            dx[k] = gx;
        }
    }
}

__global__ void t_add(int64_t n, float *a, const float *b) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) a[i] = __fadd_rn(a[i], b[i]);
}

// Column sums over rows t < T of A[t][c] (times B[t][c] when B is given), in a
// fixed order: each of the gridDim.y row chunks sums its rows in order, then
// t_colsum_fin adds the chunk partials in order.
__global__ void t_colsum_part(int T, int ncol, const float *A, int64_t lda, const float *B, int64_t ldb,
                              float *part) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= ncol) return;
    const int per = (T + gridDim.y - 1) / gridDim.y;
    const int t0 = blockIdx.y * per, t1 = t0 + per < T ? t0 + per : T;
    float s = 0.0f;
    for (int t = t0; t < t1; ++t)
        s = B ? __fmaf_rn(A[(int64_t)t * lda + c], B[(int64_t)t * ldb + c], s) : __fadd_rn(s, A[(int64_t)t * lda + c]);
    part[(int64_t)blockIdx.y * ncol + c] = s;
}
// adds into out: a layer applied several times (depth loops) sums its applications
__global__ void t_colsum_fin(int ncol, int nch, const float *part, float *out) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= ncol) return;
    float s = 0.0f;
    for (int i = 0; i < nch; ++i) s = __fadd_rn(s, part[(int64_t)i * ncol + c]);
    out[c] = __fadd_rn(out[c], s);
}

// Backward of t_xsa_gate for one row: tp.dy (d of the o-projection input) is
// rewritten in place as d of the attention output; d(v) of XSA goes to tp.dvx,
// d(n[:gw]) of the gate is added into tp.dn, and the gate-weight products
// dz_h * n[k] to colbuf [t][H*gw].  One warp per KV group, heads in order.
__global__ void t_xsa_gate_bwd(TD D, int l, int i, Tape tp, altxs_weights w) {
    __shared__ float dzs[128];
    const int t = blockIdx.x, hd = D.hd, lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int64_t row = (int64_t)l * D.T + t;
    const float *yr = tp.yraw + row * D.d, *nr = tp.n + row * D.d;
    const float *vr = tp.qkv + row * D.qn + D.d + D.kvd;
    float *dy = tp.dy + (int64_t)t * D.d;
    const bool xsa = i >= D.xsa_from;
    for (int g = wid; g < D.Hkv; g += nw) {
        float vn[4], dvn[4];
        float nrm = 0.0f, den = 1.0f;
        if (xsa) {
            float ss = 0.0f;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int k = lane + 32 * u;
                vn[u] = k < hd ? vr[(int64_t)g * hd + k] : 0.0f;
                ss = __fmaf_rn(vn[u], vn[u], ss);
            }
            nrm = __fsqrt_rn(warp_sum(ss));
            den = fmaxf(nrm, 1e-12f);
#pragma unroll
            for (int u = 0; u < 4; ++u) vn[u] = __fdiv_rn(vn[u], den);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) dvn[u] = 0.0f;
        for (int h = g * D.G; h < (g + 1) * D.G; ++h) {
            float y0[4], y1[4], gy[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int k = lane + 32 * u;
                y0[u] = k < hd ? yr[(int64_t)h * hd + k] : 0.0f;
                gy[u] = k < hd ? dy[(int64_t)h * hd + k] : 0.0f;
            }
            float c = 0.0f;
            if (xsa) {
#pragma unroll
                for (int u = 0; u < 4; ++u) c = __fmaf_rn(y0[u], vn[u], c);
                c = warp_sum(c);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) y1[u] = xsa ? __fsub_rn(y0[u], __fmul_rn(c, vn[u])) : y0[u];
            if (D.sgate) {
                const float *gwr = w.attn_gate_w + ((int64_t)i * D.H + h) * D.gw;
                float z = 0.0f;
                for (int k = lane; k < D.gw; k += 32) z = __fmaf_rn(nr[k], gwr[k], z);
                const float gt = sigmoidf_(__fmul_rn(D.sgs, warp_sum(z)));
                float dg = 0.0f;
#pragma unroll
                for (int u = 0; u < 4; ++u) dg = __fmaf_rn(gy[u], y1[u], dg);
                dg = warp_sum(dg);
                if (lane == 0) dzs[h] = __fmul_rn(__fmul_rn(dg, __fmul_rn(gt, __fsub_rn(1.0f, gt))), D.sgs);
#pragma unroll
                for (int u = 0; u < 4; ++u) gy[u] = __fmul_rn(gy[u], gt);
            }
            if (xsa) {  // y1 = y0 - (y0 . vn) vn: d y0 = P d y1, d vn -= (d y1 . vn) y0 + c d y1
                float e = 0.0f;
#pragma unroll
                for (int u = 0; u < 4; ++u) e = __fmaf_rn(gy[u], vn[u], e);
                e = warp_sum(e);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    dvn[u] = __fsub_rn(dvn[u], __fadd_rn(__fmul_rn(e, y0[u]), __fmul_rn(c, gy[u])));
                    gy[u] = __fsub_rn(gy[u], __fmul_rn(e, vn[u]));
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (lane + 32 * u < hd) dy[(int64_t)h * hd + lane + 32 * u] = gy[u];
        }
        if (xsa) {  // vn = v / max(|v|, eps)
            float pd = 0.0f;
#pragma unroll
            for (int u = 0; u < 4; ++u) pd = __fmaf_rn(dvn[u], vn[u], pd);
            pd = warp_sum(pd);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int k = lane + 32 * u;
                const float dv = nrm > 1e-12f ? __fdiv_rn(__fsub_rn(dvn[u], __fmul_rn(pd, vn[u])), den)
                                              : __fdiv_rn(dvn[u], den);
                if (k < hd) tp.dvx[(int64_t)t * D.kvd + (int64_t)g * hd + k] = dv;
            }
        }
    }
    if (!D.sgate) return;
    __syncthreads();
    float *dn = tp.dn + (int64_t)t * D.d;
    for (int k = threadIdx.x; k < D.gw; k += blockDim.x) {
        float acc = 0.0f;
        for (int h = 0; h < D.H; ++h) acc = __fmaf_rn(dzs[h], w.attn_gate_w[((int64_t)i * D.H + h) * D.gw + k], acc);
        dn[k] = __fadd_rn(dn[k], acc);
    }
    if (!tp.colbuf) return;  // gate-weight products: the full-parameter gradient only
    float *cb = tp.colbuf + (int64_t)t * D.H * D.gw;
    for (int e = threadIdx.x; e < D.H * D.gw; e += blockDim.x) cb[e] = __fmul_rn(dzs[e / D.gw], nr[e % D.gw]);
}

// d(v part of qkv) += XSA's d(v)
__global__ void t_add_v(int64_t n, int kvd, int qn, int voff, float *dqkv, const float *dvx) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= n) return;
    const int64_t t = e / kvd;
    float *p = dqkv + t * qn + voff + (e - t * kvd);
    *p = __fadd_rn(*p, dvx[e]);
}

// Backward of t_par_combine for application l (layer i, skip j) per row: from
// d(lane0') in tp.dx and d(lane1') in tp.dl1 to d(o-projection) (tp.dao),
// d(down-projection) (tp.dd), the lanes' residual parts (tp.dx = r0 d lane0',
// tp.dl1 = r1 d lane1') and per-row products: [0,d) d(attn_scale), [d,2d)
// d(mlp_scale), [2d,2d+2) d(parallel_resid[i]), [2d+2,2d+6) d(parallel_post[i]).
__global__ void t_par_bwd(TD D, int l, int i, int j, Tape tp, altxs_weights w, int skip_gates) {
    __shared__ float red[32];
    const int t = blockIdx.x, d = D.d;
    const int64_t row = ((int64_t)l * D.T + t) * d;
    const float *pr = w.parallel_resid + 2 * i, *pp = w.parallel_post + 4 * i;
    const float *sk = j >= 0 ? tp.skip + ((int64_t)(D.enc - 1 - j) * D.T + t) * d : nullptr;
    float *dx = tp.dx + (int64_t)t * d, *dl1 = tp.dl1 + (int64_t)t * d;
    float *cb = tp.colbuf ? tp.colbuf + (int64_t)t * 4 * d : nullptr;  // parameter products (full gradient)
    float s[6] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    for (int k = threadIdx.x; k < d; k += blockDim.x) {
        const float g0 = dx[k], g1 = dl1[k];
        const float as = w.attn_scale[(int64_t)i * d + k], ms = w.mlp_scale[(int64_t)i * d + k];
        const float ao = tp.aol[row + k], mo = tp.doutl[row + k];
        const float A = __fmul_rn(as, ao), M = __fmul_rn(ms, mo);
        float l0 = cb ? tp.xraw[row + k] : 0.0f;  // lane 0 after the skip
        if (cb && sk) {
            const float scaled = __fmul_rn(w.skip_weights[(int64_t)j * d + k], sk[k]);
            l0 = skip_gates ? lerp_t(scaled, l0, sigmoidf_(w.skip_gates[(int64_t)j * d + k])) : __fadd_rn(l0, scaled);
        }
        const float da = __fadd_rn(__fmul_rn(pp[0], g0), __fmul_rn(pp[1], g1));
        const float dm = __fadd_rn(__fmul_rn(pp[2], g0), __fmul_rn(pp[3], g1));
        tp.dao[(int64_t)t * d + k] = __fmul_rn(as, da);
        tp.dd[(int64_t)t * d + k] = __fmul_rn(ms, dm);
        if (cb) {
            cb[k] = __fmul_rn(da, ao);
            cb[d + k] = __fmul_rn(dm, mo);
        }
        s[0] = __fmaf_rn(g0, l0, s[0]);
        s[1] = __fmaf_rn(g1, tp.xmid[row + k], s[1]);
        s[2] = __fmaf_rn(g0, A, s[2]);
        s[3] = __fmaf_rn(g1, A, s[3]);
        s[4] = __fmaf_rn(g0, M, s[4]);
        s[5] = __fmaf_rn(g1, M, s[5]);
        dx[k] = __fmul_rn(pr[0], g0);
        dl1[k] = __fmul_rn(pr[1], g1);
    }
    if (!cb) return;
#pragma unroll
    for (int q = 0; q < 6; ++q) {
        const float v = block_sum(s[q], red);
        if (threadIdx.x == 0) cb[2 * d + q] = v;
    }
}

// d(final hidden) -> the two lanes (mean, lane 0 or lane 1)
__global__ void t_lane_split(int64_t n, int pfinal, float *dx, float *dl1) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= n) return;
    const float g = dx[e];
    dx[e] = pfinal == 0 ? __fmul_rn(0.5f, g) : pfinal == 1 ? g : 0.0f;
    dl1[e] = pfinal == 0 ? __fmul_rn(0.5f, g) : pfinal == 2 ? g : 0.0f;
}

// Smear gate backward per row t: dxs = d(smeared rows) -> draw = d(raw rows)
// (x_t = raw_t + lambda*sig(z_t)*raw_{t-1}, z_t = raw_t[:gw] . g), and per-row
// products [0] d(lambda), [1, 1+gw) d(g) into colbuf [t][1+gw].
__global__ void t_smear_bwd(TD D, Tape tp, altxs_weights w, const float *dxs, float *draw) {
    __shared__ float red[32];
    const int t = blockIdx.x, d = D.d, gw = D.gw;
    const float *raw = tp.eraw + (int64_t)t * d;
    const float lam = w.smear_lambda[0];
    float z = 0.0f, zn = 0.0f, dg = 0.0f;
    for (int k = threadIdx.x; k < gw; k += blockDim.x) {
        z = __fmaf_rn(raw[k], w.smear_gate[k], z);
        if (t + 1 < D.T) zn = __fmaf_rn(raw[d + k], w.smear_gate[k], zn);
    }
    if (t > 0)
        for (int k = threadIdx.x; k < d; k += blockDim.x) dg = __fmaf_rn(dxs[(int64_t)t * d + k], raw[k - d], dg);
    z = block_sum(z, red);
    zn = block_sum(zn, red);
    dg = block_sum(dg, red);
    const float sg = sigmoidf_(z);
    const float gn = t + 1 < D.T ? __fmul_rn(lam, sigmoidf_(zn)) : 0.0f;
    const float dz = t > 0 ? __fmul_rn(__fmul_rn(dg, lam), __fmul_rn(sg, __fsub_rn(1.0f, sg))) : 0.0f;
    for (int k = threadIdx.x; k < d; k += blockDim.x) {
        float v = dxs[(int64_t)t * d + k];
        if (t + 1 < D.T) v = __fadd_rn(v, __fmul_rn(gn, dxs[(int64_t)(t + 1) * d + k]));
        if (k < gw) v = __fadd_rn(v, __fmul_rn(dz, w.smear_gate[k]));
        draw[(int64_t)t * d + k] = v;
    }
    float *cb = tp.colbuf + (int64_t)t * (gw + 1);
    if (threadIdx.x == 0) cb[0] = t > 0 ? __fmul_rn(dg, sg) : 0.0f;
    for (int k = threadIdx.x; k < gw; k += blockDim.x) cb[1 + k] = __fmul_rn(dz, raw[k]);
}

// Input-embedding gradient of the tied table: gemb[v] += sum over positions t
// with tok[t] == v of draw[t], in increasing t.  Each warp finds the matching
// positions 32 at a time with a ballot; thread k owns columns k, k+128, ..
// (d <= 1024, 128 threads).
__global__ void __launch_bounds__(128) t_emb_scatter(int T, int d, int V, const int32_t *tok, const float *draw,
                                                     float *gemb) {
    constexpr unsigned FULL = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    for (int v = blockIdx.x; v < V; v += gridDim.x) {
        float acc[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) acc[u] = 0.0f;
        bool hit = false;
        for (int base = 0; base < T; base += 32) {
            const int t = base + lane;
            unsigned m = __ballot_sync(FULL, t < T && tok[t] == v);
            hit |= m != 0u;
            while (m) {
                const int b = __ffs(m) - 1;
                m &= m - 1u;
                const float *row = draw + (int64_t)(base + b) * d;
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int k = threadIdx.x + 128 * u;
                    if (k < d) acc[u] = __fadd_rn(acc[u], row[k]);
                }
            }
        }
        if (hit) {
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int k = threadIdx.x + 128 * u;
                if (k < d) gemb[(int64_t)v * d + k] = __fadd_rn(gemb[(int64_t)v * d + k], acc[u]);
            }
        }
    }
}


// ---- fused LoRA products (rank <= kLoraFused) ---------------------------
// The adapters that read the same input (q, k and v on the block's normed
// input) are one launch: a warp per row computes t = X A^T for every adapter
// (warp reductions over the input in a fixed order) and adds s t B^T to each
// adapter's output; the backward is a per-row kernel (dt = s G B, dX += dt A)
// and the two row reductions dB = s G^T t and dA = dt^T X as chunked outer
// sums added in a fixed chunk order.  Rows are independent, every sum has a
// fixed order: results do not depend on anything but the window.
constexpr int kLoraFused = 16;   // largest rank of the fused kernels
constexpr int kLoraMaxIn = 1024; // largest adapter input width
constexpr int kOuterChunks = 16; // row chunks of the outer sums

struct LoraJob {
    const float *A, *B;  // A [r][din], B [dout][r]
    float *t;            // [T][r]: t = X A^T (forward: written; backward: read)
    float *Y;            // forward: output columns (ld ldy), += s t B^T
    const float *G;      // backward: d(output) columns (ld ldg)
    int64_t ldy, ldg;
    int dout;
    float *dA, *dB;      // backward: gradients (written)
};
struct LoraGroup {
    const float *X;
    int64_t ldx;
    int din, r, n;  // input width, rank, adapters (<= 3)
    float s;
    LoraJob j[3];
    float *dX;      // backward: += sum_j dt_j A_j (may be NULL)
    float *dt;      // backward: [T][n * r] scratch
};

__global__ void __launch_bounds__(256) t_lora_fwd(int T, LoraGroup g) {
    const int lane = threadIdx.x & 31;
    const int nw = blockDim.x >> 5;
    constexpr int E = kLoraMaxIn / 32;
    for (int row = blockIdx.x * nw + (threadIdx.x >> 5); row < T; row += gridDim.x * nw) {
        float x[E];
        const float *xr = g.X + (int64_t)row * g.ldx;
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] = lane + 32 * e < g.din ? xr[lane + 32 * e] : 0.0f;
        for (int a = 0; a < g.n; ++a) {
            const LoraJob &J = g.j[a];
            float t[kLoraFused];
#pragma unroll
            for (int p = 0; p < kLoraFused; ++p) {
                float acc = 0.0f;
                if (p < g.r) {
                    const float *ar = J.A + (int64_t)p * g.din;
#pragma unroll
                    for (int e = 0; e < E; ++e)
                        if (lane + 32 * e < g.din) acc = __fmaf_rn(x[e], __ldg(ar + lane + 32 * e), acc);
                }
                t[p] = warp_sum(acc);
            }
            if (lane < g.r) {
#pragma unroll
                for (int p = 0; p < kLoraFused; ++p)
                    if (p == lane) J.t[(int64_t)row * g.r + p] = t[p];
            }
            float *yr = J.Y + (int64_t)row * J.ldy;
            for (int o = lane; o < J.dout; o += 32) {
                const float *br = J.B + (int64_t)o * g.r;
                float acc = 0.0f;
#pragma unroll
                for (int p = 0; p < kLoraFused; ++p)
                    if (p < g.r) acc = __fmaf_rn(t[p], __ldg(br + p), acc);
                yr[o] = __fadd_rn(yr[o], __fmul_rn(g.s, acc));
            }
        }
    }
}

// backward, per row: dt_j = s G_j B_j (into g.dt), dX += sum_j dt_j A_j
__global__ void __launch_bounds__(256) t_lora_bwd_rows(int T, LoraGroup g) {
    const int lane = threadIdx.x & 31;
    const int nw = blockDim.x >> 5;
    constexpr int E = kLoraMaxIn / 32;
    for (int row = blockIdx.x * nw + (threadIdx.x >> 5); row < T; row += gridDim.x * nw) {
        float dx[E];
#pragma unroll
        for (int e = 0; e < E; ++e) dx[e] = 0.0f;
        for (int a = 0; a < g.n; ++a) {
            const LoraJob &J = g.j[a];
            float acc[kLoraFused];
#pragma unroll
            for (int p = 0; p < kLoraFused; ++p) acc[p] = 0.0f;
            const float *gr = J.G + (int64_t)row * J.ldg;
            for (int o = lane; o < J.dout; o += 32) {
                const float gv = gr[o];
                const float *br = J.B + (int64_t)o * g.r;
#pragma unroll
                for (int p = 0; p < kLoraFused; ++p)
                    if (p < g.r) acc[p] = __fmaf_rn(gv, __ldg(br + p), acc[p]);
            }
            float dt[kLoraFused];
#pragma unroll
            for (int p = 0; p < kLoraFused; ++p) dt[p] = __fmul_rn(g.s, warp_sum(acc[p]));
            if (lane < g.r) {
#pragma unroll
                for (int p = 0; p < kLoraFused; ++p)
                    if (p == lane) g.dt[(int64_t)row * g.n * g.r + a * g.r + p] = dt[p];
            }
            if (g.dX) {
#pragma unroll
                for (int p = 0; p < kLoraFused; ++p) {
                    if (p >= g.r) break;
                    const float *ar = J.A + (int64_t)p * g.din;
#pragma unroll
                    for (int e = 0; e < E; ++e)
                        if (lane + 32 * e < g.din) dx[e] = __fmaf_rn(dt[p], __ldg(ar + lane + 32 * e), dx[e]);
                }
            }
        }
        if (g.dX) {
            float *xr = g.dX + (int64_t)row * g.din;
#pragma unroll
            for (int e = 0; e < E; ++e)
                if (lane + 32 * e < g.din) xr[lane + 32 * e] = __fadd_rn(xr[lane + 32 * e], dx[e]);
        }
    }
}

// Outer sums out[p][q] = scale * sum over rows of U[t][p] V[t][q] for the
// adapter gradients: job 2a is dB_a (U = t_a, V = G_a, stored [q][p] = B's
// layout), job 2a+1 is dA_a (U = dt_a, V = X, stored [p][q]).  Part: chunk c
// of the rows, one thread per (job, p, q), partials [c][job][p][qmax].
__device__ __forceinline__ void lora_outer_job(const LoraGroup &g, int job, const float *&U, int64_t &ldu,
                                               const float *&V, int64_t &ldv, int &Q) {
    const LoraJob &J = g.j[job >> 1];
    if ((job & 1) == 0) {
        U = J.t;
        ldu = g.r;
        V = J.G;
        ldv = J.ldg;
        Q = J.dout;
    } else {
        U = g.dt + (job >> 1) * g.r;
        ldu = (int64_t)g.n * g.r;
        V = g.X;
        ldv = g.ldx;
        Q = g.din;
    }
}

__global__ void __launch_bounds__(256) t_lora_outer_part(int T, LoraGroup g, int qmax, float *part) {
    const int job = blockIdx.z / g.r, p = blockIdx.z % g.r, c = blockIdx.y;
    const int q = blockIdx.x * blockDim.x + threadIdx.x;
    const float *U, *V;
    int64_t ldu, ldv;
    int Q;
    lora_outer_job(g, job, U, ldu, V, ldv, Q);
    if (q >= Q) return;
    const int rows = (T + kOuterChunks - 1) / kOuterChunks;
    const int t0 = c * rows, t1 = min(T, t0 + rows);
    float acc = 0.0f;
    for (int t = t0; t < t1; ++t) acc = __fmaf_rn(U[(int64_t)t * ldu + p], V[(int64_t)t * ldv + q], acc);
    part[(((int64_t)c * 2 * g.n + job) * g.r + p) * qmax + q] = acc;
}

__global__ void __launch_bounds__(256) t_lora_outer_fin(LoraGroup g, int qmax, const float *part) {
    const int job = blockIdx.z / g.r, p = blockIdx.z % g.r;
    const int q = blockIdx.x * blockDim.x + threadIdx.x;
    const float *U, *V;
    int64_t ldu, ldv;
    int Q;
    lora_outer_job(g, job, U, ldu, V, ldv, Q);
    if (q >= Q) return;
    float acc = 0.0f;
    for (int c = 0; c < kOuterChunks; ++c) acc = __fadd_rn(acc, part[(((int64_t)c * 2 * g.n + job) * g.r + p) * qmax + q]);
    const LoraJob &J = g.j[job >> 1];
    if ((job & 1) == 0) J.dB[(int64_t)q * g.r + p] = __fmul_rn(g.s, acc);
    else J.dA[(int64_t)p * g.din + q] = acc;
}

// out = a + s * b (two roundings, as the reference's w + s * dw)
__global__ void t_axpy(int64_t n, const float *a, float s, const float *b, float *out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __fadd_rn(a[i], __fmul_rn(s, b[i]));
}
// p -= (p - w0) * pull
__global__ void t_anchor(int64_t n, float *p, const float *w0, const float *pull) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        p[i] = __fsub_rn(p[i], __fmul_rn(__fsub_rn(p[i], w0[i]), pull[i]));
}

// global grad norm: partial sums over fixed chunks, then a single-block sum
__global__ void t_sqsum_part(int64_t n, const float *g, float *part) {
    __shared__ float red[32];
    const int64_t chunk = (n + gridDim.x - 1) / gridDim.x;
    const int64_t b0 = (int64_t)blockIdx.x * chunk, b1 = b0 + chunk < n ? b0 + chunk : n;
    float s = 0.0f;
    for (int64_t i = b0 + threadIdx.x; i < b1; i += blockDim.x) s = __fmaf_rn(g[i], g[i], s);
    s = block_sum(s, red);
    if (threadIdx.x == 0) part[blockIdx.x] = s;
}

__global__ void t_adam(int64_t n, float *p, const float *g, float *m, float *v, const float *part, int nparts,
                       altxs_ttt_hparams hp, int step) {
    __shared__ float coef_s;
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int i = 0; i < nparts; ++i) s = __fadd_rn(s, part[i]);
        const float norm = __fsqrt_rn(s);
        const float c = __fdiv_rn(hp.grad_clip, __fadd_rn(norm, 1e-6f));
        coef_s = c < 1.0f ? c : 1.0f;
    }
    __syncthreads();
    const float coef = coef_s;
    const float bc1 = 1.0f - powf(hp.beta1, (float)step);
    const float bc2 = 1.0f - powf(hp.beta2, (float)step);
    const float step_size = __fdiv_rn(hp.lr, bc1);
    const float bc2s = __fsqrt_rn(bc2);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float gi = __fmul_rn(g[i], coef);
        float pi = p[i];
        if (hp.weight_decay != 0.0f) pi = __fmul_rn(pi, __fsub_rn(1.0f, __fmul_rn(hp.lr, hp.weight_decay)));
        const float mi = lerp_t(m[i], gi, __fsub_rn(1.0f, hp.beta1));  // exp_avg.lerp_(grad, 1 - beta1)
        const float vi = __fadd_rn(__fmul_rn(v[i], hp.beta2), __fmul_rn(__fmul_rn(__fsub_rn(1.0f, hp.beta2), gi), gi));
        const float den = __fadd_rn(__fdiv_rn(__fsqrt_rn(vi), bc2s), hp.eps);
        p[i] = __fsub_rn(pi, __fmul_rn(step_size, __fdiv_rn(mi, den)));
        m[i] = mi;
        v[i] = vi;
    }
}

inline int g1(int64_t n, int t) { return (int)((n + t - 1) / t); }

#define TRY(x)                 \
    do {                       \
        int rc_ = (x);         \
        if (rc_) return rc_;   \
    } while (0)

struct Run {
    TD D;
    const altxs_model_desc *desc;
    const altxs_weights *w;
    const altxs_dense_weights *dw;  // dense fp32 base, or NULL
    Tape tp;
    float *splitk;
    int64_t splitk_floats;
    // tensor-core path (weights given as hi/lo planes): operand plane scratch
    const altxs_split_planes *sp;
    uint16_t *tca, *tcb;
    int64_t tca_n, tcb_n;
    bool no_lora;  // context prefill of a model without adapters, or the full-parameter gradient
    cudaStream_t st;
    // full-parameter gradient: the window's tokens, the gradient arena and its layout
    const int32_t *tok;
    float *fg;
    altxs_param_layout lay;
    // physical layer of every application
    int sched[kMaxApps];
};

void plan(Run &R) {
    for (int a = 0; a < R.D.A; ++a) R.sched[a] = R.desc->schedule ? R.desc->schedule[a] : a;
}
// skip slot taken by application a (a decoder application), or -1
inline int skip_of(const TD &D, int a) { return a >= D.enc && a - D.enc < D.nskip ? a - D.enc : -1; }

// Batched/causal GEMMs of the update: tensor cores when the model carries
// bf16 planes, CUDA cores otherwise (the two differ in the last bits; the
// choice is the caller's and is the same at the encoder and the decoder).
int gemm(const Run &R, const GemmArgs &g) {
    if (R.sp) return tc_gemm_f32(g, R.tca, R.tca_n, R.tcb, R.tcb_n, R.st, kKTtt);
    return launch_gemm(g, R.st);
}

// A = X (split into planes in the A scratch), B = weight planes rows row0..: Y (+)= X W^T or dX (+)= dY W
int tc_lin(const Run &R, const uint16_t *wh, const uint16_t *wl, int64_t wrows, int row0, int N, int K,
           const float *X, int64_t ldx, float *Y, int64_t ldy, bool transposed_w, float beta) {
    const int T = R.D.T;
    const int kx = transposed_w ? N : K;  // columns of the fp32 input
    const int64_t ldo = align_up(kx, 8);
    if (R.tca_n < 2 * align_up((int64_t)T * ldo, 128)) return ALTXS_EINVAL;
    uint16_t *xh = R.tca, *xl = R.tca + align_up((int64_t)T * ldo, 128);
    TRY(launch_split_f32(X, T, kx, ldx, 1, 0, xh, xl, R.st, kKTtt));
    TcGemm t{};
    t.a = TcOp{xh, xl, 0, T, kx, ldo, T * ldo, 1, 0, 1, 1, 0};
    // forward: B[n][k] = W[row0 + n][k] (K-major); backward: B[n][k] = W[row0 + k][n] (MN-major)
    t.b = TcOp{wh, wl, transposed_w ? 1 : 0, wrows, K, K, wrows * (int64_t)K, 1, row0, 1, 1, 0};
    t.M = T;
    t.N = transposed_w ? K : N;
    t.K = kx;
    t.batch = 1;
    t.alpha = 1.0f;
    t.beta = beta;
    t.epi = kEpiStore;
    t.C = Y;
    t.ldc = ldy;
    return launch_tc_gemm(t, R.st);
}

// GEMM with the common fields (split-K scratch attached)
GemmArgs G(const Run &R, const float *A, int64_t lda, int tA, const float *B, int64_t ldb, int tB, float *C,
           int64_t ldc, int M, int N, int K, float alpha = 1.0f, float beta = 0.0f) {
    GemmArgs g{};
    g.A = A;
    g.B = B;
    g.C = C;
    g.M = M;
    g.N = N;
    g.K = K;
    g.lda = lda;
    g.ldb = ldb;
    g.ldc = ldc;
    g.tA = tA;
    g.tB = tB;
    g.batch = 1;
    g.adiv = 1;
    g.bdiv = 1;
    g.alpha = alpha;
    g.beta = beta;
    g.ws = R.splitk;
    g.ws_floats = R.splitk_floats;
    return g;
}

// B operand from an fp32 array [nb][rows][cols] (row stride ld, batch stride bs), split into the B scratch
int split_b(const Run &R, const float *src, int64_t rows, int64_t cols, int64_t ld, int nb, int64_t bs, int mn_major,
            int div, int mul, int add, TcOp &op) {
    const int64_t ldo = align_up(cols, 8), n = align_up((int64_t)nb * rows * ldo, 128);
    if (2 * n > R.tcb_n) return ALTXS_EINVAL;
    TRY(launch_split_f32(src, rows, cols, ld, nb, bs, R.tcb, R.tcb + n, R.st, kKTtt));
    op = TcOp{R.tcb, R.tcb + n, mn_major, rows, cols, ldo, rows * ldo, nb, 0, div, mul, add};
    return ALTXS_OK;
}

// one attention product on the tensor cores: per-head [T][T] planes (P or dS) with a split right operand
int tc_att(const Run &R, const TcOp &a, const TcOp &b, int M, int N, int K, int batch, int causal, float beta,
           float *C, int64_t ldc, int64_t sC) {
    TcGemm t{};
    t.a = a;
    t.b = b;
    t.M = M;
    t.N = N;
    t.K = K;
    t.batch = batch;
    t.causal = causal;
    t.alpha = 1.0f;
    t.beta = beta;
    t.epi = kEpiStore;
    t.C = C;
    t.ldc = ldc;
    t.sC = sC;
    return launch_tc_gemm(t, R.st);
}

// Y[T][N] = X[T][K] W[row0.., :]^T  (tensor cores from the planes wh/wl, else the dense
// copy of the base if present, else the packed codes)
int lin_fwd(const Run &R, const altxs_qmat &Wq, const float *Wd, const uint16_t *wh, const uint16_t *wl, int row0,
            int N, int K, const float *X, int64_t ldx, float *Y, int64_t ldy) {
    if (R.sp) return tc_lin(R, wh, wl, Wq.rows, row0, N, K, X, ldx, Y, ldy, false, 0.0f);
    if (Wd) return launch_gemm(G(R, X, ldx, 0, Wd + (int64_t)row0 * K, K, 1, Y, ldy, R.D.T, N, K), R.st);
    QmmArgs a{};
    a.X = X;
    a.ldx = ldx;
    a.M = R.D.T;
    a.W = Wq;
    a.row0 = row0;
    a.N = N;
    a.K = K;
    a.Y = Y;
    a.ldy = ldy;
    a.epi = kEpiStore;
    return launch_qmm(a, R.st);
}

// dX[T][K] (= or +=) dY[T][N] W[row0.., :]
int lin_bwd(const Run &R, const altxs_qmat &Wq, const float *Wd, const uint16_t *wh, const uint16_t *wl, int row0,
            int N, int K, const float *dY, int64_t lddy, float *dX, int64_t lddx, float beta) {
    if (R.sp) return tc_lin(R, wh, wl, Wq.rows, row0, N, K, dY, lddy, dX, lddx, true, beta);
    if (Wd)
        return launch_gemm(G(R, dY, lddy, 0, Wd + (int64_t)row0 * K, K, 0, dX, lddx, R.D.T, K, N, 1.0f, beta), R.st);
    QmmTArgs q{};
    q.dY = dY;
    q.lddy = lddy;
    q.M = R.D.T;
    q.W = Wq;
    q.row0 = row0;
    q.N = N;
    q.K = K;
    q.dX = dX;
    q.lddx = lddx;
    q.alpha = 1.0f;
    q.beta = beta;
    return launch_qmm_t(q, R.st);
}

// fused adapters sharing one input X: forward (t and Y += s t B^T)
int lora_fwd_group(const Run &R, const LoraGroup &g) {
    if (R.no_lora || g.n == 0) return ALTXS_OK;
    const int T = R.D.T;
    const int grid = (T + 7) / 8 < 148 * 8 ? (T + 7) / 8 : 148 * 8;
    ALTXS_LAUNCH(kKTtt, R.st, t_lora_fwd<<<grid, 256, 0, R.st>>>(T, g));
    return ALTXS_OK;
}

// fused adapters sharing one input X: backward (dt, dX += dt A, dA, dB)
int lora_bwd_group(const Run &R, const LoraGroup &g) {
    if (R.no_lora || g.n == 0) return ALTXS_OK;
    const int T = R.D.T;
    const int grid = (T + 7) / 8 < 148 * 8 ? (T + 7) / 8 : 148 * 8;
    ALTXS_LAUNCH(kKTtt, R.st, t_lora_bwd_rows<<<grid, 256, 0, R.st>>>(T, g));
    int qmax = g.din;
    for (int a = 0; a < g.n; ++a) qmax = qmax > g.j[a].dout ? qmax : g.j[a].dout;
    if ((int64_t)kOuterChunks * 2 * g.n * g.r * qmax > R.splitk_floats) return ALTXS_EINVAL;
    const dim3 grid2((qmax + 255) / 256, kOuterChunks, 2 * g.n * g.r);
    ALTXS_LAUNCH(kKTtt, R.st, t_lora_outer_part<<<grid2, 256, 0, R.st>>>(T, g, qmax, R.splitk));
    ALTXS_LAUNCH(kKTtt, R.st,
                 t_lora_outer_fin<<<dim3((qmax + 255) / 256, 1, 2 * g.n * g.r), 256, 0, R.st>>>(g, qmax, R.splitk));
    return ALTXS_OK;
}

// small adapters on the layers' inputs; the LM-head adapter (V outputs) keeps
// the GEMM path, whose tiles make the T x V read-modify-write of the logits
// and the V-wide reductions cheaper than a warp per row
bool lora_fusable(const Run &R, int din, int dout = 0) {
    return R.D.r > 0 && R.D.r <= kLoraFused && din <= kLoraMaxIn && dout <= kLoraMaxIn;
}

// one forward adapter job: A, B, the t tape, the output columns
LoraJob fjob(const float *A, const float *B, float *t, float *Y, int64_t ldy, int dout) {
    LoraJob j{};
    j.A = A;
    j.B = B;
    j.t = t;
    j.Y = Y;
    j.ldy = ldy;
    j.dout = dout;
    return j;
}
// one backward adapter job: A, B, the t tape, d(output) columns, gradients
LoraJob bjob(const float *A, const float *B, float *t, const float *Gy, int64_t ldg, int dout, float *dA, float *dB) {
    LoraJob j{};
    j.A = A;
    j.B = B;
    j.t = t;
    j.G = Gy;
    j.ldg = ldg;
    j.dout = dout;
    j.dA = dA;
    j.dB = dB;
    return j;
}
LoraGroup lgroup(const Run &R, const float *X, int din, float *dX = nullptr) {
    LoraGroup g{};
    g.X = X;
    g.ldx = din;
    g.din = din;
    g.r = R.D.r;
    g.s = R.desc->lora_scale;
    g.dX = dX;
    g.dt = R.tp.dt;
    return g;
}

// LoRA forward for one target: t = X A^T ; Y += s * t B^T
int lora_fwd(const Run &R, const float *X, int din, const float *A, const float *B, int dout, float s, float *t,
             float *Y, int64_t ldy) {
    if (R.no_lora) return ALTXS_OK;
    const int T = R.D.T, r = R.D.r;
    if (lora_fusable(R, din, dout) && s == R.desc->lora_scale) {
        LoraGroup g = lgroup(R, X, din);
        g.j[g.n++] = fjob(A, B, t, Y, ldy, dout);
        return lora_fwd_group(R, g);
    }
    TRY(launch_gemm(G(R, X, din, 0, A, din, 1, t, r, T, r, din), R.st));
    TRY(launch_gemm(G(R, t, r, 0, B, r, 1, Y, ldy, T, dout, r, s, 1.0f), R.st));
    return ALTXS_OK;
}

// LoRA backward: grads dA, dB (written), dX += dt A (if dX)
int lora_bwd(const Run &R, const float *X, int din, const float *A, const float *B, int dout, float s,
             const float *t, const float *Gy, int64_t ldg, float *dA, float *dB, float *dX) {
    if (R.no_lora) return ALTXS_OK;
    const int T = R.D.T, r = R.D.r;
    if (lora_fusable(R, din, dout) && s == R.desc->lora_scale) {
        LoraGroup g = lgroup(R, X, din, dX);
        g.j[g.n++] = bjob(A, B, const_cast<float *>(t), Gy, ldg, dout, dA, dB);
        return lora_bwd_group(R, g);
    }
    float *dt = R.tp.dt;
    TRY(launch_gemm(G(R, Gy, ldg, 1, t, r, 0, dB, r, dout, r, T, s), R.st));  // dB = s G^T t
    TRY(launch_gemm(G(R, Gy, ldg, 0, B, r, 0, dt, r, T, r, dout, s), R.st));  // dt = s G B
    TRY(launch_gemm(G(R, dt, r, 1, X, din, 0, dA, din, r, din, T), R.st));    // dA = dt^T X
    if (dX) TRY(launch_gemm(G(R, dt, r, 0, A, din, 0, dX, din, T, din, r, 1.0f, 1.0f), R.st));  // dX += dt A
    return ALTXS_OK;
}


// the weight planes of matrix field f (NULL on the CUDA-core path)
#define PL(f) (R.sp ? R.sp->f : nullptr)

// attention probabilities of layer l (causal softmax of q k^T / sqrt(hd)): fp32
// [H][T][T], or hi/lo planes [2][H][T][align8(T)] on the tensor-core path.  The
// full-parameter gradient keeps one layer's worth and recomputes it in the backward.
float *p_f32(const Run &R, int l) {
    return R.tp.P + (R.D.full ? 0 : (int64_t)l * R.D.H * R.D.T * R.D.T);
}
uint16_t *p_planes(const Run &R, int l) {
    return reinterpret_cast<uint16_t *>(R.tp.P + (R.D.full ? 0 : (int64_t)l * R.D.H * R.D.T * align_up(R.D.T, 8)));
}
int attn_probs(const Run &R, int l) {
    const TD &D = R.D;
    const Tape &tp = R.tp;
    const int Tn = D.T, d = D.d;
    cudaStream_t st = R.st;
    const float att_scale = 1.0f / __builtin_sqrtf((float)D.hd);
    const float *qr = tp.qr + (int64_t)l * Tn * d, *kr = tp.kr + (int64_t)l * Tn * D.kvd;
    const int64_t ldp = align_up(Tn, 8);
    // tensor cores: S in fp32 scratch (rows of stride ldp), P leaves as planes
    float *S = R.sp ? tp.dS : p_f32(R, l);
    const int64_t lds = R.sp ? ldp : Tn;
    GemmArgs g = G(R, qr, D.H * D.hd, 0, kr, D.kvd, 1, S, lds, Tn, Tn, D.hd, att_scale);  // S = q k^T
    g.batch = D.H;
    g.sA = D.hd;
    g.sB = D.hd;
    g.bdiv = D.G;
    g.sC = (int64_t)Tn * lds;
    g.causal = 1;
    TRY(gemm(R, g));
    if (R.sp) {
        uint16_t *Ph = p_planes(R, l), *Pl = Ph + D.H * Tn * ldp;
        ALTXS_LAUNCH(kKTtt, st, t_softmax_pl<<<D.H * Tn, 256, 0, st>>>(D, tp.dS, Ph, Pl, ldp));
    } else {
        ALTXS_LAUNCH(kKTtt, st, t_softmax<<<D.H * Tn, 256, 0, st>>>(D, S));
    }
    return ALTXS_OK;
}

// Window attention without the T x T probabilities (the flash kernels): the
// context prefill, and the forward and backward of the update and of the
// full-parameter gradient (the backward reads the forward's output and
// log-sum-exp instead of the probabilities).
int g_flash = 1;
}  // namespace

int altxs::set_flash(int on) {
    g_flash = on ? 1 : 0;
    return ALTXS_OK;
}

namespace {
bool use_flash(const Run &R) {
    const TD &D = R.D;
    return g_flash && R.sp && flash_ok(D.hd) && flash_scratch_elems(D.T, D.H, D.Hkv, D.hd) <= R.tca_n;
}

int forward(const Run &R, const int32_t *tok, const int32_t *tgt, const float *lora, float *loss_out,
            bool head = true) {
    const TD &D = R.D;
    const Tape &tp = R.tp;
    const altxs_weights *w = R.w;
    const altxs_dense_weights *dw = R.dw;
    const LoraOff lo = lora_offsets(*R.desc);
    const int mask = R.desc->lora_mask;
    const float s = R.desc->lora_scale;
    const int Tn = D.T, d = D.d, r = D.r;
    cudaStream_t st = R.st;
    ALTXS_LAUNCH(kKTtt, st, t_embed<<<Tn, 128, 0, st>>>(D, tok, w->emb, dw ? dw->emb : w->emb_dense, tp.x0, tp.x, tp, *w));
    bool lanes = false;
    // l: the layer application (tape index; the LoRA update has one per layer), i: its layer
    for (int l = 0; l < D.A; ++l) {
        const int i = R.sched[l];
        const bool par = par_app(D, R.sched, l);
        if (par && !lanes) {  // the stream splits into two lanes (model.py:1404-1407)
            cudaMemcpyAsync(tp.lane1, tp.x, (size_t)Tn * d * 4, cudaMemcpyDeviceToDevice, st);
            lanes = true;
        }
        ALTXS_LAUNCH(kKTtt, st, t_prenorm<<<Tn, 128, 0, st>>>(D, l, i, skip_of(D, l), par, tp, *w, R.desc->skip_gates));
        const float *n = tp.n + (int64_t)l * Tn * d;
        float *qkv = tp.qkv + (int64_t)l * Tn * D.qn;
        TRY(lin_fwd(R, w->qkv, dw ? dw->qkv : nullptr, PL(qkv_hi), PL(qkv_lo), i * D.qn, D.qn, d, n, d, qkv, D.qn));
        if (lora_fusable(R, d, d > D.kvd ? d : D.kvd)) {  // q, k, v read the same input: one launch
            LoraGroup g = lgroup(R, n, d);
            g.j[g.n++] = fjob(lora + lo.qA + l * lo.q_stride, lora + lo.qB + l * lo.q_stride,
                              tp.tq + (int64_t)l * Tn * r, qkv, D.qn, d);
            if (mask & 2)
                g.j[g.n++] = fjob(lora + lo.kA + l * lo.k_stride, lora + lo.kB + l * lo.k_stride,
                                  tp.tk + (int64_t)l * Tn * r, qkv + d, D.qn, D.kvd);
            g.j[g.n++] = fjob(lora + lo.vA + l * lo.v_stride, lora + lo.vB + l * lo.v_stride,
                              tp.tv + (int64_t)l * Tn * r, qkv + d + D.kvd, D.qn, D.kvd);
            TRY(lora_fwd_group(R, g));
        } else {
            TRY(lora_fwd(R, n, d, lora + lo.qA + l * lo.q_stride, lora + lo.qB + l * lo.q_stride, d, s,
                         tp.tq + (int64_t)l * Tn * r, qkv, D.qn));
            if (mask & 2)
                TRY(lora_fwd(R, n, d, lora + lo.kA + l * lo.k_stride, lora + lo.kB + l * lo.k_stride, D.kvd, s,
                             tp.tk + (int64_t)l * Tn * r, qkv + d, D.qn));
            TRY(lora_fwd(R, n, d, lora + lo.vA + l * lo.v_stride, lora + lo.vB + l * lo.v_stride, D.kvd, s,
                         tp.tv + (int64_t)l * Tn * r, qkv + d + D.kvd, D.qn));
        }
        ALTXS_LAUNCH(kKTtt, st, t_qk<<<Tn, 256, 0, st>>>(D, l, i, tp, *w));
        const bool flash = use_flash(R);
        if (!flash) TRY(attn_probs(R, l));
        // the full-parameter gradient keeps every application's attention output and projections
        const bool o_on_y = r > 0 && (mask & 64);
        float *yb = D.full || o_on_y || flash ? tp.yl + (int64_t)l * Tn * d : tp.y;
        float *aob = tp.aol ? tp.aol + (int64_t)l * Tn * d : tp.ao;
        const bool ym = ymotif(D, i);
        float *ya = ym ? tp.yraw + (int64_t)l * Tn * d : yb;  // P v, before XSA and the gate
        const int64_t ldp = align_up(Tn, 8);
        if (flash) {  // y = softmax(q k^T / sqrt(hd)) v without the scores leaving the SM
            FlashArgs fa{};
            fa.T = Tn;
            fa.H = D.H;
            fa.Hkv = D.Hkv;
            fa.hd = D.hd;
            fa.scale = 1.0f / __builtin_sqrtf((float)D.hd);
            fa.q = tp.qr + (int64_t)l * Tn * d;
            fa.ldq = d;
            fa.k = tp.kr + (int64_t)l * Tn * D.kvd;
            fa.ldk = D.kvd;
            fa.v = qkv + d + D.kvd;
            fa.ldv = D.qn;
            fa.y = ya;
            fa.ldy = d;
            fa.scratch = R.tca;
            fa.lse = head ? tp.lse + (int64_t)l * D.H * Tn : nullptr;  // for the flash backward
            TRY(launch_flash_fwd(fa, st));
        } else if (R.sp) {
            const uint16_t *Ph = p_planes(R, l), *Pl = Ph + D.H * Tn * ldp;
            TcOp a{Ph, Pl, 0, Tn, Tn, ldp, Tn * ldp, D.H, 0, 1, 1, 0}, b{};
            TRY(split_b(R, qkv + d + D.kvd, Tn, D.hd, D.qn, D.Hkv, D.hd, 1, D.G, 1, 0, b));  // v, [n=c][k=t']
            TRY(tc_att(R, a, b, Tn, D.hd, Tn, D.H, 2, 0.0f, ya, d, D.hd));                   // y = P v
        } else {
            GemmArgs g = G(R, p_f32(R, l), Tn, 0, qkv + d + D.kvd, D.qn, 0, ya, d, Tn, D.hd, Tn);  // y = P v
            g.batch = D.H;
            g.sA = (int64_t)Tn * Tn;
            g.sB = D.hd;
            g.bdiv = D.G;
            g.sC = D.hd;
            g.causal = 2;
            TRY(gemm(R, g));
        }
        if (ym) ALTXS_LAUNCH(kKTtt, st, t_xsa_gate<<<Tn, 256, 0, st>>>(D, l, i, tp, *w, yb));
        TRY(lin_fwd(R, w->o, dw ? dw->o : nullptr, PL(o_hi), PL(o_lo), i * d, d, d, yb, d, aob, d));
        if (mask & 8)
            TRY(lora_fwd(R, o_on_y ? yb : n, d, lora + lo.oA + l * lo.o_stride, lora + lo.oB + l * lo.o_stride, d, s,
                         tp.to + (int64_t)l * Tn * r, aob, d));
        ALTXS_LAUNCH(kKTtt, st, t_post_attn<<<Tn, 128, 0, st>>>(D, l, i, tp, *w, aob, par));
        float *u = tp.u + (int64_t)l * Tn * D.F;
        TRY(lin_fwd(R, w->up, dw ? dw->up : nullptr, PL(up_hi), PL(up_lo), i * D.F, D.F, d, tp.n2 + (int64_t)l * Tn * d, d, u, D.F));
        ALTXS_LAUNCH(kKTtt, st, t_leaky<<<g1((int64_t)Tn * D.F, 256), 256, 0, st>>>((int64_t)Tn * D.F, u, tp.hbuf));
        float *sk = l < D.enc ? tp.skip + (int64_t)l * Tn * d : nullptr;
        const float *xm = tp.xmid + (int64_t)l * Tn * d;
        if (dw || R.sp || (mask & 32) || par) {
            float *db = tp.doutl ? tp.doutl + (int64_t)l * Tn * d : tp.dd;
            TRY(lin_fwd(R, w->down, dw ? dw->down : nullptr, PL(down_hi), PL(down_lo), i * d, d, D.F, tp.hbuf, D.F, db, d));
            if (mask & 32)  // MLP adapter on the MLP's normed input, added to its output
                TRY(lora_fwd(R, tp.n2 + (int64_t)l * Tn * d, d, lora + lo.mA + l * lo.m_stride,
                             lora + lo.mB + l * lo.m_stride, d, s, tp.tm + (int64_t)l * Tn * r, db, d));
            if (par)
                ALTXS_LAUNCH(kKTtt, st, t_par_combine<<<g1((int64_t)Tn * d, 256), 256, 0, st>>>((int64_t)Tn * d, d, l,
                                                                                                 i, tp, *w, Tn));
            else
                ALTXS_LAUNCH(kKTtt, st, t_resid<<<g1((int64_t)Tn * d, 256), 256, 0, st>>>(
                                            (int64_t)Tn * d, d, xm, w->mlp_scale + (int64_t)i * d, db, tp.x, sk));
        } else {
            QmmArgs a{};
            a.X = tp.hbuf;
            a.ldx = D.F;
            a.M = Tn;
            a.W = w->down;
            a.row0 = i * d;
            a.N = d;
            a.K = D.F;
            a.Y = tp.x;
            a.ldy = d;
            a.epi = kEpiResid;
            a.R = xm;
            a.ldr = d;
            a.colscale = w->mlp_scale + (int64_t)i * d;
            a.Y2 = sk;
            a.ldy2 = d;
            TRY(launch_qmm(a, st));
        }
    }
    if (!head) return ALTXS_OK;  // context prefill: the layers' K/V rows are all it needs
    ALTXS_LAUNCH(kKTtt, st, t_final<<<Tn, 128, 0, st>>>(D, tp, lanes ? 1 : 0));
    TRY(lin_fwd(R, w->emb, dw ? dw->emb : nullptr, PL(emb_hi), PL(emb_lo), 0, D.V, d, tp.hf, d, tp.logits, D.V));
    if (mask & 16) TRY(lora_fwd(R, tp.hf, d, lora + lo.lmA, lora + lo.lmB, D.V, s, tp.tlm, tp.logits, D.V));
    const float *sc = D.asym ? w->softcap : nullptr;
    ALTXS_LAUNCH(kKTtt, st, t_ce<<<Tn, 512, 0, st>>>(D, tgt, tp, R.desc->logit_softcap, sc,
                                                     D.asym && D.full ? tp.colbuf : nullptr));
    ALTXS_LAUNCH(kKTtt, st, t_loss_sum<<<1, 1024, 0, st>>>(Tn, D.first, tp.rowloss, loss_out));
    return ALTXS_OK;
}

// Backward of the window loss: into the adapters (grad in the LoRA arena
// layout), or with R.fg into every parameter (the full arena layout R.lay,
// zeroed by the caller: a layer's applications add up).
int backward(const Run &R, const float *lora, float *grad) {
    const TD &D = R.D;
    const Tape &tp = R.tp;
    const altxs_weights *w = R.w;
    const altxs_dense_weights *dw = R.dw;
    const LoraOff lo = lora_offsets(*R.desc);
    const int mask = R.desc->lora_mask;
    const float s = R.desc->lora_scale;
    const int Tn = D.T, d = D.d, r = D.r;
    const int64_t Td = (int64_t)Tn * d;
    const float att_scale = 1.0f / __builtin_sqrtf((float)D.hd);
    cudaStream_t st = R.st;
    const bool full = D.full;
    float *FG = R.fg;
    const altxs_param_layout &lay = R.lay;
    // out[c] += sum over rows of A[t][c] (* B[t][c])
    auto colsum = [&](const float *A, int64_t lda, const float *B, int64_t ldb, int ncol, float *out) -> int {
        ALTXS_LAUNCH(kKTtt, st, t_colsum_part<<<dim3(g1(ncol, 128), kColChunks), 128, 0, st>>>(Tn, ncol, A, lda, B,
                                                                                                 ldb, tp.cpart));
        ALTXS_LAUNCH(kKTtt, st, t_colsum_fin<<<g1(ncol, 128), 128, 0, st>>>(ncol, kColChunks, tp.cpart, out));
        return ALTXS_OK;
    };
    // weight gradient out[N][K] (+)= dY^T X (dY [T][N], X [T][K]): the reduction runs over positions
    auto wgrad = [&](const float *dY, int N, const float *X, int K, float *out, bool acc) -> int {
        return gemm(R, G(R, dY, N, 1, X, K, 0, out, K, N, K, Tn, 1.0f, acc ? 1.0f : 0.0f));
    };
    bool seen[kMaxApps] = {};  // layer i already has gradient from a later application
    int first_par = -1;
    for (int l = 0; l < D.A; ++l)
        if (first_par < 0 && par_app(D, R.sched, l)) first_par = l;
    if (full) {
        cudaMemsetAsync(tp.dx0, 0, (size_t)Td * 4, st);
        if (D.asym) TRY(colsum(tp.colbuf, 2, nullptr, 0, 2, FG + lay.softcap));  // rows left by t_ce
        TRY(wgrad(tp.logits, D.V, tp.hf, d, FG + lay.emb, false));  // the tied table as the LM head
    }
    // LM head: dhf = dlogits E (+ LoRA)
    TRY(lin_bwd(R, w->emb, dw ? dw->emb : nullptr, PL(emb_hi), PL(emb_lo), 0, D.V, d, tp.logits, D.V, tp.dn, d, 0.0f));
    if (mask & 16)
        TRY(lora_bwd(R, tp.hf, d, lora + lo.lmA, lora + lo.lmB, D.V, s, tp.tlm, tp.logits, D.V, grad + lo.lmA,
                     grad + lo.lmB, tp.dn));
    ALTXS_LAUNCH(kKTtt, st, t_rms_bwd<<<Tn, 128, 0, st>>>(d, tp.dn, d, tp.x, tp.invf, nullptr, nullptr, tp.dx));
    if (first_par >= 0)
        ALTXS_LAUNCH(kKTtt, st, t_lane_split<<<g1(Td, 256), 256, 0, st>>>(Td, D.pfinal, tp.dx, tp.dl1));
    for (int l = D.A - 1; l >= 0; --l) {
        const int i = R.sched[l], j = skip_of(D, l);
        const bool par = par_app(D, R.sched, l);
        const bool acc = seen[i];
        seen[i] = true;
        if (l < D.enc)
            ALTXS_LAUNCH(kKTtt, st, t_add<<<g1(Td, 256), 256, 0, st>>>(Td, tp.dx, tp.dskip + (int64_t)l * Td));
        // MLP: d(down-projection output) into dd
        if (par) {  // both lanes' gradients -> the two branches, the residual parts, the lane products
            ALTXS_LAUNCH(kKTtt, st, t_par_bwd<<<Tn, 128, 0, st>>>(D, l, i, j, tp, *w, R.desc->skip_gates));
            if (full) {
                TRY(colsum(tp.colbuf, 4 * d, nullptr, 0, d, FG + lay.attn_scale + (int64_t)i * d));
                TRY(colsum(tp.colbuf + d, 4 * d, nullptr, 0, d, FG + lay.mlp_scale + (int64_t)i * d));
                TRY(colsum(tp.colbuf + 2 * d, 4 * d, nullptr, 0, 2, FG + lay.parallel_resid + 2 * i));
                TRY(colsum(tp.colbuf + 2 * d + 2, 4 * d, nullptr, 0, 4, FG + lay.parallel_post + 4 * i));
            }
        } else {
            ALTXS_LAUNCH(kKTtt, st, t_scale_cols<<<g1(Td, 256), 256, 0, st>>>(Td, d, tp.dx, w->mlp_scale + (int64_t)i * d,
                                                                             tp.dd));
            if (full) TRY(colsum(tp.dx, d, tp.doutl + (int64_t)l * Td, d, d, FG + lay.mlp_scale + (int64_t)i * d));
        }
        if (full) {
            ALTXS_LAUNCH(kKTtt, st, t_leaky<<<g1((int64_t)Tn * D.F, 256), 256, 0, st>>>(
                                        (int64_t)Tn * D.F, tp.u + (int64_t)l * Tn * D.F, tp.hbuf));
            TRY(wgrad(tp.dd, d, tp.hbuf, D.F, FG + lay.down + (int64_t)i * d * D.F, acc));
        }
        TRY(lin_bwd(R, w->down, dw ? dw->down : nullptr, PL(down_hi), PL(down_lo), i * d, d, D.F, tp.dd, d, tp.dh, D.F, 0.0f));
        ALTXS_LAUNCH(kKTtt, st, t_leaky_bwd<<<g1((int64_t)Tn * D.F, 256), 256, 0, st>>>(
                                    (int64_t)Tn * D.F, tp.dh, tp.u + (int64_t)l * Tn * D.F, tp.dh));
        if (full) TRY(wgrad(tp.dh, D.F, tp.n2 + (int64_t)l * Td, d, FG + lay.up + (int64_t)i * D.F * d, acc));
        TRY(lin_bwd(R, w->up, dw ? dw->up : nullptr, PL(up_hi), PL(up_lo), i * D.F, D.F, d, tp.dh, D.F, tp.dn2, d, 0.0f));
        if (mask & 32)
            TRY(lora_bwd(R, tp.n2 + (int64_t)l * Td, d, lora + lo.mA + l * lo.m_stride, lora + lo.mB + l * lo.m_stride,
                         d, s, tp.tm + (int64_t)l * Tn * r, tp.dd, d, grad + lo.mA + l * lo.m_stride,
                         grad + lo.mB + l * lo.m_stride, tp.dn2));
        // the MLP read: x_mid (sequential) or lane 1 (parallel)
        float *dmid = par ? tp.dl1 : tp.dx;
        ALTXS_LAUNCH(kKTtt, st, t_rms_bwd<<<Tn, 128, 0, st>>>(d, tp.dn2, d, tp.xmid + (int64_t)l * Td,
                                                             tp.inv2 + (int64_t)l * Tn, w->ln_scale + i, dmid, dmid));
        if (!par) {
            if (full) TRY(colsum(tp.dx, d, tp.aol + (int64_t)l * Td, d, d, FG + lay.attn_scale + (int64_t)i * d));
            ALTXS_LAUNCH(kKTtt, st, t_scale_cols<<<g1(Td, 256), 256, 0, st>>>(Td, d, tp.dx,
                                                                             w->attn_scale + (int64_t)i * d, tp.dao));
        }
        const float *n = tp.n + (int64_t)l * Td;
        cudaMemsetAsync(tp.dn, 0, (size_t)Td * 4, st);
        const bool o_on_y = r > 0 && (mask & 64);
        if ((mask & 8) && !o_on_y)
            TRY(lora_bwd(R, n, d, lora + lo.oA + l * lo.o_stride, lora + lo.oB + l * lo.o_stride, d, s,
                         tp.to + (int64_t)l * Tn * r, tp.dao, d, grad + lo.oA + l * lo.o_stride,
                         grad + lo.oB + l * lo.o_stride, tp.dn));
        if (full) TRY(wgrad(tp.dao, d, tp.yl + (int64_t)l * Td, d, FG + lay.o + (int64_t)i * d * d, acc));
        TRY(lin_bwd(R, w->o, dw ? dw->o : nullptr, PL(o_hi), PL(o_lo), i * d, d, d, tp.dao, d, tp.dy, d, 0.0f));
        if ((mask & 8) && o_on_y)  // the o adapter read y: its d(input) joins d(y)
            TRY(lora_bwd(R, tp.yl + (int64_t)l * Td, d, lora + lo.oA + l * lo.o_stride, lora + lo.oB + l * lo.o_stride,
                         d, s, tp.to + (int64_t)l * Tn * r, tp.dao, d, grad + lo.oA + l * lo.o_stride,
                         grad + lo.oB + l * lo.o_stride, tp.dy));
        const bool ym = ymotif(D, i);
        if (ym) {  // XSA / sparse gate: dy becomes d(P v); d(v) and d(n[:gw]) on the side
            ALTXS_LAUNCH(kKTtt, st, t_xsa_gate_bwd<<<Tn, 256, 0, st>>>(D, l, i, tp, *w));
            if (full && D.sgate) TRY(colsum(tp.colbuf, (int64_t)D.H * D.gw, nullptr, 0, D.H * D.gw,
                                    FG + lay.attn_gate_w + (int64_t)i * D.H * D.gw));
        }
        // attention backward: the flash kernels from the forward's output and
        // log-sum-exp, or the probabilities recomputed (full-parameter gradient)
        // or kept (update) and the products over them
        const bool fwd_flash = use_flash(R);
        const bool fbwd = fwd_flash && flash_bwd_scratch_elems(Tn, D.H, D.Hkv) <= R.tca_n;
        if (fbwd) {
            FlashBwdArgs fb{};
            fb.T = Tn;
            fb.H = D.H;
            fb.Hkv = D.Hkv;
            fb.hd = D.hd;
            fb.scale = att_scale;
            fb.q = tp.qr + (int64_t)l * Td;
            fb.ldq = d;
            fb.k = tp.kr + (int64_t)l * Tn * D.kvd;
            fb.ldk = D.kvd;
            fb.v = tp.qkv + (int64_t)l * Tn * D.qn + d + D.kvd;
            fb.ldv = D.qn;
            fb.out = ym ? tp.yraw + (int64_t)l * Tn * d : tp.yl + (int64_t)l * Tn * d;  // the forward's P v
            fb.ldo = d;
            fb.lse = tp.lse + (int64_t)l * D.H * Tn;
            fb.dout = tp.dy;
            fb.lddo = d;
            fb.dq = tp.dqr;
            fb.lddq = d;
            fb.dk = tp.dkr;
            fb.lddk = D.kvd;
            fb.dv = tp.dqkv + d + D.kvd;
            fb.lddv = D.qn;
            fb.scratch = R.tca;
            TRY(launch_flash_bwd(fb, st));
        } else {
        if (full || fwd_flash) TRY(attn_probs(R, l));
        const float *P = p_f32(R, l);
        const float *qkv = tp.qkv + (int64_t)l * Tn * D.qn;
        const float *qr = tp.qr + (int64_t)l * Td, *kr = tp.kr + (int64_t)l * Tn * D.kvd;
        if (R.sp) {  // tensor cores: P and dS as planes, K-major or read transposed (MN-major)
            const int64_t ldp = align_up(Tn, 8);
            const uint16_t *Ph = p_planes(R, l);
            const uint16_t *Pl = Ph + D.H * Tn * ldp;
            GemmArgs g = G(R, tp.dy, d, 0, qkv + d + D.kvd, D.qn, 1, tp.dS, ldp, Tn, Tn, D.hd);  // dP = dy v^T
            g.batch = D.H;
            g.sA = D.hd;
            g.sB = D.hd;
            g.bdiv = D.G;
            g.sC = (int64_t)Tn * ldp;
            g.causal = 1;
            TRY(gemm(R, g));
            TcOp b{};
            TRY(split_b(R, tp.dy, Tn, D.hd, d, D.H, D.hd, 1, 1, 1, 0, b));  // dy per head, [n=c][k=t]
            for (int gi = 0; gi < D.G; ++gi) {  // dv = sum over the group's heads of P^T dy
                TcOp a{Ph, Pl, 1, Tn, Tn, ldp, Tn * ldp, D.H, 0, 1, D.G, gi};
                b.mul = D.G;
                b.add = gi;
                TRY(tc_att(R, a, b, Tn, D.hd, Tn, D.Hkv, 3, gi ? 1.0f : 0.0f, tp.dqkv + d + D.kvd, D.qn, D.hd));
            }
            uint16_t *Gh = R.tca, *Gl = R.tca + D.H * Tn * ldp;  // dS planes
            ALTXS_LAUNCH(kKTtt, st,
                         t_softmax_bwd_pl<<<D.H * Tn, 256, 0, st>>>(D, Ph, Pl, ldp, tp.dS, Gh, Gl, att_scale));
            TRY(split_b(R, kr, Tn, D.hd, D.kvd, D.Hkv, D.hd, 1, D.G, 1, 0, b));  // k, [n=c][k=t']
            TRY(tc_att(R, TcOp{Gh, Gl, 0, Tn, Tn, ldp, Tn * ldp, D.H, 0, 1, 1, 0}, b, Tn, D.hd, Tn, D.H, 2, 0.0f,
                       tp.dqr, d, D.hd));  // dq = dS k
            TRY(split_b(R, qr, Tn, D.hd, d, D.H, D.hd, 1, 1, 1, 0, b));  // q per head, [n=c][k=t]
            for (int gi = 0; gi < D.G; ++gi) {  // dk = sum over the group's heads of dS^T q
                b.mul = D.G;
                b.add = gi;
                TRY(tc_att(R, TcOp{Gh, Gl, 1, Tn, Tn, ldp, Tn * ldp, D.H, 0, 1, D.G, gi}, b, Tn, D.hd, Tn, D.Hkv, 3,
                           gi ? 1.0f : 0.0f, tp.dkr, D.kvd, D.hd));
            }
        } else {
            {
                GemmArgs g = G(R, tp.dy, d, 0, qkv + d + D.kvd, D.qn, 1, tp.dS, Tn, Tn, Tn, D.hd);  // dP = dy v^T
                g.batch = D.H;
                g.sA = D.hd;
                g.sB = D.hd;
                g.bdiv = D.G;
                g.sC = (int64_t)Tn * Tn;
                g.causal = 1;
                TRY(gemm(R, g));
            }
            for (int gi = 0; gi < D.G; ++gi) {  // dv = sum over the group's heads of P^T dy
                GemmArgs g = G(R, P + (int64_t)gi * Tn * Tn, Tn, 1, tp.dy + gi * D.hd, d, 0, tp.dqkv + d + D.kvd,
                               D.qn, Tn, D.hd, Tn, 1.0f, gi ? 1.0f : 0.0f);
                g.batch = D.Hkv;
                g.sA = (int64_t)D.G * Tn * Tn;
                g.sB = (int64_t)D.G * D.hd;
                g.sC = D.hd;
                g.causal = 3;
                TRY(gemm(R, g));
            }
            ALTXS_LAUNCH(kKTtt, st, t_softmax_bwd<<<D.H * Tn, 256, 0, st>>>(D, P, tp.dS, att_scale));
            {
                GemmArgs g = G(R, tp.dS, Tn, 0, kr, D.kvd, 0, tp.dqr, d, Tn, D.hd, Tn);  // dq = dS k
                g.batch = D.H;
                g.sA = (int64_t)Tn * Tn;
                g.sB = D.hd;
                g.bdiv = D.G;
                g.sC = D.hd;
                g.causal = 2;
                TRY(gemm(R, g));
            }
            for (int gi = 0; gi < D.G; ++gi) {  // dk = sum over the group's heads of dS^T q
                GemmArgs g = G(R, tp.dS + (int64_t)gi * Tn * Tn, Tn, 1, qr + gi * D.hd, d, 0, tp.dkr, D.kvd, Tn, D.hd,
                               Tn, 1.0f, gi ? 1.0f : 0.0f);
                g.batch = D.Hkv;
                g.sA = (int64_t)D.G * Tn * Tn;
                g.sB = (int64_t)D.G * D.hd;
                g.sC = D.hd;
                g.causal = 3;
                TRY(gemm(R, g));
            }
        }
        }
        if (ym && i >= D.xsa_from)
            ALTXS_LAUNCH(kKTtt, st, t_add_v<<<g1((int64_t)Tn * D.kvd, 256), 256, 0, st>>>(
                                        (int64_t)Tn * D.kvd, D.kvd, D.qn, d + D.kvd, tp.dqkv, tp.dvx));
        ALTXS_LAUNCH(kKTtt, st, t_qk_bwd<<<Tn, 256, 0, st>>>(D, l, i, tp, *w));
        if (full) TRY(colsum(tp.colbuf, D.H, nullptr, 0, D.H, FG + lay.q_gain + (int64_t)i * D.H));
        if (lora_fusable(R, d, d > D.kvd ? d : D.kvd) && !R.no_lora) {  // q, k, v read the same input: one group
            LoraGroup g = lgroup(R, n, d, tp.dn);
            g.j[g.n++] = bjob(lora + lo.qA + l * lo.q_stride, lora + lo.qB + l * lo.q_stride,
                              tp.tq + (int64_t)l * Tn * r, tp.dqkv, D.qn, d, grad + lo.qA + l * lo.q_stride,
                              grad + lo.qB + l * lo.q_stride);
            if (mask & 2)
                g.j[g.n++] = bjob(lora + lo.kA + l * lo.k_stride, lora + lo.kB + l * lo.k_stride,
                                  tp.tk + (int64_t)l * Tn * r, tp.dqkv + d, D.qn, D.kvd,
                                  grad + lo.kA + l * lo.k_stride, grad + lo.kB + l * lo.k_stride);
            g.j[g.n++] = bjob(lora + lo.vA + l * lo.v_stride, lora + lo.vB + l * lo.v_stride,
                              tp.tv + (int64_t)l * Tn * r, tp.dqkv + d + D.kvd, D.qn, D.kvd,
                              grad + lo.vA + l * lo.v_stride, grad + lo.vB + l * lo.v_stride);
            TRY(lora_bwd_group(R, g));
        } else {
            TRY(lora_bwd(R, n, d, lora + lo.qA + l * lo.q_stride, lora + lo.qB + l * lo.q_stride, d, s,
                         tp.tq + (int64_t)l * Tn * r, tp.dqkv, D.qn, grad + lo.qA + l * lo.q_stride,
                         grad + lo.qB + l * lo.q_stride, tp.dn));
            if (mask & 2)
                TRY(lora_bwd(R, n, d, lora + lo.kA + l * lo.k_stride, lora + lo.kB + l * lo.k_stride, D.kvd, s,
                             tp.tk + (int64_t)l * Tn * r, tp.dqkv + d, D.qn, grad + lo.kA + l * lo.k_stride,
                             grad + lo.kB + l * lo.k_stride, tp.dn));
            TRY(lora_bwd(R, n, d, lora + lo.vA + l * lo.v_stride, lora + lo.vB + l * lo.v_stride, D.kvd, s,
                         tp.tv + (int64_t)l * Tn * r, tp.dqkv + d + D.kvd, D.qn, grad + lo.vA + l * lo.v_stride,
                         grad + lo.vB + l * lo.v_stride, tp.dn));
        }
        if (full) TRY(wgrad(tp.dqkv, D.qn, n, d, FG + lay.qkv + (int64_t)i * D.qn * d, acc));
        TRY(lin_bwd(R, w->qkv, dw ? dw->qkv : nullptr, PL(qkv_hi), PL(qkv_lo), i * D.qn, D.qn, d, tp.dqkv, D.qn, tp.dn, d, 1.0f));
        // d(x_in): added to the stream's gradient (sequential), or the attention read alone (parallel)
        ALTXS_LAUNCH(kKTtt, st, t_rms_bwd<<<Tn, 128, 0, st>>>(d, tp.dn, d, tp.xin + (int64_t)l * Td,
                                                             tp.inv1 + (int64_t)l * Tn, w->ln_scale + i,
                                                             par ? nullptr : tp.dx, par ? tp.dread : tp.dx));
        ALTXS_LAUNCH(kKTtt, st, t_mix_bwd<<<Tn, 128, 0, st>>>(D, l, i, j, par, tp, *w, R.desc->skip_gates));
        if (full) {
            TRY(colsum(tp.colbuf, 4 * d, nullptr, 0, 2 * d, FG + lay.resid_mix + (int64_t)i * 2 * d));
            if (j >= 0) {
                TRY(colsum(tp.colbuf + 2 * d, 4 * d, nullptr, 0, d, FG + lay.skip_weights + (int64_t)j * d));
                TRY(colsum(tp.colbuf + 3 * d, 4 * d, nullptr, 0, d, FG + lay.skip_gates + (int64_t)j * d));
            }
        }
        if (l == first_par)  // before the split both lanes were the one stream
            ALTXS_LAUNCH(kKTtt, st, t_add<<<g1(Td, 256), 256, 0, st>>>(Td, tp.dx, tp.dl1));
    }
    if (full) {  // embedding: d(x0) over every use, through x0 = rms(raw or smeared), into the tied table's rows
        ALTXS_LAUNCH(kKTtt, st, t_add<<<g1(Td, 256), 256, 0, st>>>(Td, tp.dx0, tp.dx));
        ALTXS_LAUNCH(kKTtt, st, t_rms_bwd<<<Tn, 128, 0, st>>>(d, tp.dx0, d, D.smear ? tp.esm : tp.eraw, tp.inv0,
                                                             nullptr, nullptr, tp.dn));
        const float *draw = tp.dn;
        if (D.smear) {
            ALTXS_LAUNCH(kKTtt, st, t_smear_bwd<<<Tn, 128, 0, st>>>(D, tp, *w, tp.dn, tp.dd));
            TRY(colsum(tp.colbuf, D.gw + 1, nullptr, 0, 1, FG + lay.smear_lambda));
            TRY(colsum(tp.colbuf + 1, D.gw + 1, nullptr, 0, D.gw, FG + lay.smear_gate));
            draw = tp.dd;
        }
        ALTXS_LAUNCH(kKTtt, st, t_emb_scatter<<<D.V < 148 * 16 ? D.V : 148 * 16, 128, 0, st>>>(Tn, d, D.V, R.tok,
                                                                                             draw, FG + lay.emb));
    }
    return ALTXS_OK;
}

constexpr int64_t kSplitkFloats = 16ll << 20;  // 64 MiB of split-K partials

// plane scratch of the tensor-core path (uint16 elements): A = the largest
// split operand (P, dS [H][T][T]; dlogits [T][V]; MLP [T][F]), B = the
// attention right operands ([T][H*hd] at most)
void tc_scratch(const TD &D, int64_t *a_n, int64_t *b_n) {
    const int64_t T = D.T;
    int64_t a = (int64_t)D.H * T * align_up(T, 8);
    a = a > T * align_up(D.V, 8) ? a : T * align_up(D.V, 8);
    a = a > T * align_up(D.F, 8) ? a : T * align_up(D.F, 8);
    a = a > T * align_up(D.qn, 8) ? a : T * align_up(D.qn, 8);
    *a_n = 2 * align_up(a, 128);
    int64_t b = T * align_up(D.hd, 8) * (D.H > D.Hkv ? D.H : D.Hkv);
    if (D.full) b = b > T * align_up(D.F, 8) ? b : T * align_up(D.F, 8);  // weight-gradient inputs [T][F]
    *b_n = 2 * align_up(b, 128);
}

// Segments of the full parameter arena (floats, each 64-aligned).
altxs_param_layout param_layout(const altxs_model_desc &dsc) {
    const int64_t V = dsc.vocab, L = dsc.n_layers, d = dsc.d_model, H = dsc.n_heads, F = dsc.mlp_hidden;
    const int64_t qn = d + 2 * (int64_t)dsc.n_kv_heads * dsc.head_dim;
    const int64_t A = dsc.n_virtual > 0 ? dsc.n_virtual : L, E = dsc.n_encoder > 0 ? dsc.n_encoder : A / 2;
    const int64_t S = E < A - E ? E : A - E;
    const int64_t gw = (dsc.smear_gate || dsc.sparse_gate) ? dsc.gate_window : 0;
    altxs_param_layout o{};
    int64_t off = 0;
    auto seg = [&](int64_t n) {
        const int64_t r = off;
        off += align_up(n, 64);
        return r;
    };
    o.emb = seg(V * d);
    o.qkv = seg(L * qn * d);
    o.o = seg(L * d * d);
    o.up = seg(L * F * d);
    o.down = seg(L * d * F);
    o.q_gain = seg(L * H);
    o.attn_scale = seg(L * d);
    o.mlp_scale = seg(L * d);
    o.resid_mix = seg(L * 2 * d);
    o.skip_weights = seg(S * d);
    o.skip_gates = seg(S * d);
    o.smear_gate = seg(dsc.smear_gate ? gw : 0);
    o.smear_lambda = seg(dsc.smear_gate ? 1 : 0);
    o.attn_gate_w = seg(dsc.sparse_gate ? L * H * gw : 0);
    o.softcap = seg(dsc.asym_softcap ? 2 : 0);
    o.parallel_post = seg(dsc.parallel_start > 0 ? L * 4 : 0);
    o.parallel_resid = seg(dsc.parallel_start > 0 ? L * 2 : 0);
    o.total = off;
    return o;
}

}  // namespace

extern "C" {

int64_t altxs_ttt_workspace_bytes(const altxs_model_desc *desc, int T) {
    TD D{};
    if (!desc || fill(*desc, T, D)) return -1;
    int64_t a_n, b_n;
    tc_scratch(D, &a_n, &b_n);
    return carve(D, nullptr, nullptr) + align_up(lora_offsets(*desc).total * 4, 256) + kSplitkFloats * 4 +
           align_up(a_n * 2, 256) + align_up(b_n * 2, 256);
}

int altxs_dequant(const altxs_qmat *m, float *out, int64_t ld, altxs_stream_t stream) {
    if (!m || !out) return ALTXS_EINVAL;
    return launch_dequant(*m, 0, m->rows, out, ld, reinterpret_cast<cudaStream_t>(stream));
}

int64_t altxs_prefill_workspace_bytes(const altxs_model_desc *desc, int T) {
    TD D{};
    if (!desc || T < 1 || fill(*desc, T, D, kFillPrefill)) return -1;
    const int64_t lo_total = D.r > 0 ? lora_offsets(*desc).total : 1;
    int64_t a_n, b_n;
    tc_scratch(D, &a_n, &b_n);
    return carve(D, nullptr, nullptr) + align_up(lo_total * 4, 256) + kSplitkFloats * 4 + align_up(a_n * 2, 256) +
           align_up(b_n * 2, 256);
}

int altxs_prefill(const altxs_model_desc *desc, const altxs_weights *w, const altxs_dense_weights *dense,
                  const int32_t *tokens, int T, const float *lora, uint8_t *kv, void *workspace,
                  int64_t workspace_bytes, altxs_stream_t stream) {
    if (!desc || !w || !kv || T < 0) return ALTXS_EINVAL;
    if (T == 0) return ALTXS_OK;
    if (!tokens || !workspace) return ALTXS_EINVAL;
    Run R{};
    TRY(fill(*desc, T, R.D, kFillPrefill));
    if (desc->ctx < 1 || w->rope_positions < T) return ALTXS_EINVAL;
    if (R.D.r > 0 && !lora) return ALTXS_EINVAL;
    if (dense && (!dense->emb || !dense->qkv || !dense->o || !dense->up || !dense->down)) return ALTXS_EINVAL;
    if (workspace_bytes < altxs_prefill_workspace_bytes(desc, T)) return ALTXS_EINVAL;
    R.desc = desc;
    plan(R);
    R.w = w;
    R.dw = dense;
    R.no_lora = R.D.r == 0 || !lora;
    R.st = reinterpret_cast<cudaStream_t>(stream);
    const int64_t tape_bytes = carve(R.D, workspace, &R.tp);
    const LoraOff lo = lora_offsets(*desc);
    R.splitk = reinterpret_cast<float *>(static_cast<unsigned char *>(workspace) + tape_bytes +
                                         align_up((R.no_lora ? 1 : lo.total) * 4, 256));
    R.splitk_floats = kSplitkFloats;
    R.sp = w->split;
    if (R.sp) {
        tc_scratch(R.D, &R.tca_n, &R.tcb_n);
        R.tca = reinterpret_cast<uint16_t *>(R.splitk + kSplitkFloats);
        R.tcb = R.tca + align_up(R.tca_n, 128);
    }
    TRY(forward(R, tokens, nullptr, lora, nullptr, false));
    ALTXS_LAUNCH(kKTtt, R.st, t_kv_write<<<dim3(T, R.D.A), 128, 0, R.st>>>(R.D, R.tp, kv, desc->ctx));
    return ALTXS_OK;
}

int altxs_ttt_update(const altxs_model_desc *desc, const altxs_weights *w, const altxs_dense_weights *dense,
                     const altxs_ttt_hparams *hp, const int32_t *tokens, int T, float *lora, float *adam_m,
                     float *adam_v, int step, float *loss_out, void *workspace, int64_t workspace_bytes,
                     altxs_stream_t stream) {
    if (!desc || !w || !hp || !tokens || !lora || !adam_m || !adam_v || !workspace || step < 1) return ALTXS_EINVAL;
    Run R{};
    TRY(fill(*desc, T, R.D));
    if (workspace_bytes < altxs_ttt_workspace_bytes(desc, T)) return ALTXS_EINVAL;
    if (w->rope_positions < T) return ALTXS_EINVAL;
    if (dense && (!dense->emb || !dense->qkv || !dense->o || !dense->up || !dense->down)) return ALTXS_EINVAL;
    R.desc = desc;
    plan(R);
    R.w = w;
    R.dw = dense;
    R.st = reinterpret_cast<cudaStream_t>(stream);
    const int64_t tape_bytes = carve(R.D, workspace, &R.tp);
    const LoraOff lo = lora_offsets(*desc);
    float *grad = reinterpret_cast<float *>(static_cast<unsigned char *>(workspace) + tape_bytes);
    R.tp.grad = grad;
    R.splitk = reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(grad) + align_up(lo.total * 4, 256));
    R.splitk_floats = kSplitkFloats;
    R.sp = w->split;
    if (R.sp) {
        tc_scratch(R.D, &R.tca_n, &R.tcb_n);
        R.tca = reinterpret_cast<uint16_t *>(R.splitk + kSplitkFloats);
        R.tcb = R.tca + align_up(R.tca_n, 128);
    }
    cudaStream_t st = R.st;
    cudaMemsetAsync(grad, 0, lo.total * 4, st);
    TRY(forward(R, tokens, tokens + 1, lora, loss_out));
    TRY(backward(R, lora, grad));
    // global-norm clip + AdamW
    const int nparts = 256;
    ALTXS_LAUNCH(kKTtt, st, t_sqsum_part<<<nparts, 256, 0, st>>>(lo.total, grad, R.tp.red));
    ALTXS_LAUNCH(kKTtt, st, t_adam<<<g1(lo.total, 1024), 1024, 0, st>>>(lo.total, lora, grad, adam_m, adam_v,
                                                                         R.tp.red, nparts, *hp, step));
    return ALTXS_OK;
}

int altxs_param_layout_of(const altxs_model_desc *desc, altxs_param_layout *out) {
    TD D{};
    if (!desc || !out) return ALTXS_EINVAL;
    TRY(fill(*desc, 1, D, kFillFull));
    *out = param_layout(*desc);
    return ALTXS_OK;
}

int64_t altxs_full_workspace_bytes(const altxs_model_desc *desc, int n) {
    TD D{};
    if (!desc || n < 2 || fill(*desc, n - 1, D, kFillFull)) return -1;
    int64_t a_n, b_n;
    tc_scratch(D, &a_n, &b_n);
    return carve(D, nullptr, nullptr) + kSplitkFloats * 4 + align_up(a_n * 2, 256) + align_up(b_n * 2, 256);
}

int altxs_full_loss_grad(const altxs_model_desc *desc, const altxs_weights *w, const altxs_dense_weights *dense,
                         const int32_t *tokens, int n, int first, float *loss_out, float *grad, void *workspace,
                         int64_t workspace_bytes, altxs_stream_t stream) {
    if (!desc || !w || !dense || !tokens || !workspace || n < 2 || first < 0 || first >= n - 1) return ALTXS_EINVAL;
    if (!dense->emb || !dense->qkv || !dense->o || !dense->up || !dense->down) return ALTXS_EINVAL;
    Run R{};
    TRY(fill(*desc, n - 1, R.D, kFillFull));
    R.D.first = first;
    if (workspace_bytes < altxs_full_workspace_bytes(desc, n)) return ALTXS_EINVAL;
    if (w->rope_positions < n - 1) return ALTXS_EINVAL;
    R.desc = desc;
    plan(R);
    R.w = w;
    R.dw = dense;
    R.no_lora = true;
    R.st = reinterpret_cast<cudaStream_t>(stream);
    R.tok = tokens;
    R.fg = grad;
    R.lay = param_layout(*desc);
    const int64_t tape_bytes = carve(R.D, workspace, &R.tp);
    R.splitk = reinterpret_cast<float *>(static_cast<unsigned char *>(workspace) + tape_bytes);
    R.splitk_floats = kSplitkFloats;
    R.sp = w->split;
    if (R.sp) {
        tc_scratch(R.D, &R.tca_n, &R.tcb_n);
        R.tca = reinterpret_cast<uint16_t *>(R.splitk + kSplitkFloats);
        R.tcb = R.tca + align_up(R.tca_n, 128);
    }
    TRY(forward(R, tokens, tokens + 1, nullptr, loss_out));
    if (grad) {
        cudaMemsetAsync(grad, 0, (size_t)R.lay.total * 4, R.st);
        TRY(backward(R, nullptr, nullptr));
    }
    return cudaGetLastError() == cudaSuccess ? ALTXS_OK : ALTXS_ECUDA;
}

int altxs_adamw(int64_t n, float *params, const float *grad, float *m, float *v, const altxs_ttt_hparams *hp, int step,
                float *partials, altxs_stream_t stream) {
    if (n < 0 || !hp || step < 1) return ALTXS_EINVAL;
    if (n == 0) return ALTXS_OK;
    if (!params || !grad || !m || !v || !partials) return ALTXS_EINVAL;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int nparts = 256;
    ALTXS_LAUNCH(kKTtt, st, t_sqsum_part<<<nparts, 256, 0, st>>>(n, grad, partials));
    const int64_t blocks = (n + 1023) / 1024;
    ALTXS_LAUNCH(kKTtt, st, t_adam<<<(unsigned)(blocks < 148 * 32 ? blocks : 148 * 32), 1024, 0, st>>>(
                                n, params, grad, m, v, partials, nparts, *hp, step));
    return ALTXS_OK;
}

int altxs_params_axpy(int64_t n, const float *a, float s, const float *b, float *out, altxs_stream_t stream) {
    if (n < 0 || (n && (!a || !b || !out))) return ALTXS_EINVAL;
    if (n == 0) return ALTXS_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int64_t blocks = (n + 255) / 256;
    ALTXS_LAUNCH(kKTtt, st, t_axpy<<<(unsigned)(blocks < 148 * 64 ? blocks : 148 * 64), 256, 0, st>>>(n, a, s, b, out));
    return ALTXS_OK;
}

int altxs_params_anchor(int64_t n, float *p, const float *w0, const float *pull, altxs_stream_t stream) {
    if (n < 0 || (n && (!p || !w0 || !pull))) return ALTXS_EINVAL;
    if (n == 0) return ALTXS_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int64_t blocks = (n + 255) / 256;
    ALTXS_LAUNCH(kKTtt, st, t_anchor<<<(unsigned)(blocks < 148 * 64 ? blocks : 148 * 64), 256, 0, st>>>(n, p, w0, pull));
    return ALTXS_OK;
}

int altxs_split_params(const altxs_model_desc *desc, const float *params, const altxs_split_planes *planes,
                       altxs_stream_t stream) {
    TD D{};
    if (!desc || !params || !planes) return ALTXS_EINVAL;
    TRY(fill(*desc, 1, D, kFillFull));
    const altxs_param_layout lay = param_layout(*desc);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    struct M {
        int64_t off, rows, cols;
        uint16_t *hi, *lo;
    } ms[5] = {
        {lay.emb, D.V, D.d, const_cast<uint16_t *>(planes->emb_hi), const_cast<uint16_t *>(planes->emb_lo)},
        {lay.qkv, (int64_t)D.L * D.qn, D.d, const_cast<uint16_t *>(planes->qkv_hi), const_cast<uint16_t *>(planes->qkv_lo)},
        {lay.o, (int64_t)D.L * D.d, D.d, const_cast<uint16_t *>(planes->o_hi), const_cast<uint16_t *>(planes->o_lo)},
        {lay.up, (int64_t)D.L * D.F, D.d, const_cast<uint16_t *>(planes->up_hi), const_cast<uint16_t *>(planes->up_lo)},
        {lay.down, (int64_t)D.L * D.d, D.F, const_cast<uint16_t *>(planes->down_hi), const_cast<uint16_t *>(planes->down_lo)},
    };
    for (const M &m : ms) TRY(launch_split_f32(params + m.off, m.rows, m.cols, m.cols, 1, 0, m.hi, m.lo, st, kKTtt));
    return ALTXS_OK;
}

}  // extern "C"
