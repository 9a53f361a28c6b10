/*
 * CPU restatement of the altxs range coder and of the probability -> integer
 * CDF rules.  TEST INFRASTRUCTURE ONLY: this file is the checker that the
 * CUDA path is compared against.  Nothing in the product links it.
 *
 * Reference behaviour restated here (file:line inside the altxs project):
 *   - 32-bit Witten-Neal-Cleary coder constants   src/model/arithmetic_coder_lm.py:15-18
 *   - probs -> masses  max(1, floor(p*1e6+0.5))   src/model/arithmetic_coder_lm.py:49-64
 *                                                 src/xsa_ttt/gpu_ac.py:38-42
 *   - interval update + E1/E2/E3 renorm + pending src/model/arithmetic_coder_lm.py:90-112,175-180
 *   - flush (pending+1, one bit + pending run)    src/model/arithmetic_coder_lm.py:182-193
 *   - MSB-first bit packing, zero padded          src/model/arithmetic_coder_lm.py:115-128
 *   - decode: value from first 32 bits, offset =
 *     ((v-l+1)*total-1)/range, largest s with
 *     cum[s] <= offset, zeros past the end        src/model/arithmetic_coder_lm.py:131-137,198-284
 *
 * The fixed-point CDF rule (cdf_fixed) has no counterpart in the reference;
 * it is this framework's deterministic rule and is restated here exactly as
 * the CUDA kernel computes it (explicit fp32 fma/mul/add, no contraction;
 * build with -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define OC_TOP     (1ull << 32)
#define OC_HALF    (1ull << 31)
#define OC_QUARTER (1ull << 30)

enum { OC_ST_OVERFLOW = 1, OC_ST_BAD_SYMBOL = 2, OC_ST_BAD_TOTAL = 4 };

typedef struct {
    uint64_t low, high, pending, nbits;
    int32_t status;
} oc_enc;

static void put_bit(uint8_t *out, uint64_t cap_bits, oc_enc *s, int bit) {
    if (s->nbits >= cap_bits) {
        s->status |= OC_ST_OVERFLOW;
        return;
    }
    if (bit) out[s->nbits >> 3] |= (uint8_t)(0x80u >> (s->nbits & 7));
    s->nbits++;
}

static void enc_interval(oc_enc *s, uint8_t *out, uint64_t cap_bits,
                         uint64_t sl, uint64_t sh, uint64_t total) {
    uint64_t range = s->high - s->low + 1;
    s->high = s->low + (range * sh) / total - 1;
    s->low = s->low + (range * sl) / total;
    for (;;) {
        if (s->high < OC_HALF) {
            put_bit(out, cap_bits, s, 0);
            for (; s->pending; s->pending--) put_bit(out, cap_bits, s, 1);
        } else if (s->low >= OC_HALF) {
            put_bit(out, cap_bits, s, 1);
            for (; s->pending; s->pending--) put_bit(out, cap_bits, s, 0);
            s->low -= OC_HALF;
            s->high -= OC_HALF;
        } else if (s->low >= OC_QUARTER && s->high < 3 * OC_QUARTER) {
            s->pending++;
            s->low -= OC_QUARTER;
            s->high -= OC_QUARTER;
        } else {
            break;
        }
        s->low <<= 1;
        s->high = (s->high << 1) | 1;
    }
}

static void enc_flush(oc_enc *s, uint8_t *out, uint64_t cap_bits) {
    s->pending++;
    if (s->low < OC_QUARTER) {
        put_bit(out, cap_bits, s, 0);
        for (; s->pending; s->pending--) put_bit(out, cap_bits, s, 1);
    } else {
        put_bit(out, cap_bits, s, 1);
        for (; s->pending; s->pending--) put_bit(out, cap_bits, s, 0);
    }
}

/* Encode n symbols, row i coded with the integer CDF cum[i*(V+1) .. +V].
 * out must hold cap_bytes zeroed bytes.  Returns the number of bits written
 * (bytes = ceil(bits/8)), or a negative status on error. */
int64_t oc_encode_cum(int64_t n, int32_t V, const uint64_t *cum,
                      const int32_t *syms, uint8_t *out, int64_t cap_bytes) {
    oc_enc s = {0, OC_TOP - 1, 0, 0, 0};
    uint64_t cap_bits = (uint64_t)cap_bytes * 8;
    memset(out, 0, (size_t)cap_bytes);
    for (int64_t i = 0; i < n; i++) {
        const uint64_t *c = cum + i * (int64_t)(V + 1);
        int32_t sym = syms[i];
        if (sym < 0 || sym >= V) return -OC_ST_BAD_SYMBOL;
        uint64_t total = c[V];
        if (total == 0 || total > OC_QUARTER) return -OC_ST_BAD_TOTAL;
        if (c[sym + 1] <= c[sym]) return -OC_ST_BAD_SYMBOL;
        enc_interval(&s, out, cap_bits, c[sym], c[sym + 1], total);
    }
    enc_flush(&s, out, cap_bits);
    if (s.status) return -s.status;
    return (int64_t)s.nbits;
}

static inline int get_bit(const uint8_t *in, uint64_t n_bits, uint64_t k) {
    if (k >= n_bits) return 0;
    return (in[k >> 3] >> (7 - (k & 7))) & 1;
}

/* Decode n symbols from in (n_bytes bytes) with per-row integer CDFs. */
int64_t oc_decode_cum(int64_t n, int32_t V, const uint64_t *cum,
                      const uint8_t *in, int64_t n_bytes, int32_t *syms_out) {
    uint64_t n_bits = (uint64_t)n_bytes * 8;
    uint64_t low = 0, high = OC_TOP - 1, value = 0, bpos = 0;
    for (int i = 0; i < 32; i++) value = (value << 1) | (uint64_t)get_bit(in, n_bits, bpos++);
    for (int64_t i = 0; i < n; i++) {
        const uint64_t *c = cum + i * (int64_t)(V + 1);
        uint64_t total = c[V];
        if (total == 0 || total > OC_QUARTER) return -OC_ST_BAD_TOTAL;
        uint64_t range = high - low + 1;
        uint64_t offset = ((value - low + 1) * total - 1) / range;
        /* largest s with cum[s] <= offset (binary search over cum[0..V-1]) */
        int32_t lo = 0, hi = V, sym = 0;
        while (lo < hi) {
            int32_t mid = (lo + hi) / 2;
            if (c[mid] <= offset) { sym = mid; lo = mid + 1; } else { hi = mid; }
        }
        syms_out[i] = sym;
        high = low + (range * c[sym + 1]) / total - 1;
        low = low + (range * c[sym]) / total;
        for (;;) {
            if (high < OC_HALF) {
            } else if (low >= OC_HALF) {
                low -= OC_HALF; high -= OC_HALF; value -= OC_HALF;
            } else if (low >= OC_QUARTER && high < 3 * OC_QUARTER) {
                low -= OC_QUARTER; high -= OC_QUARTER; value -= OC_QUARTER;
            } else {
                break;
            }
            low <<= 1;
            high = (high << 1) | 1;
            value = (value << 1) | (uint64_t)get_bit(in, n_bits, bpos++);
        }
    }
    return 0;
}

/* ---- incremental forms (one symbol per call) for model-in-the-loop use --- */
typedef struct {
    uint64_t low, high, value, bpos, n_bits;
    const uint8_t *in;
} oc_dec;

void oc_dec_begin(oc_dec *d, const uint8_t *in, int64_t n_bytes) {
    d->low = 0;
    d->high = OC_TOP - 1;
    d->value = 0;
    d->bpos = 0;
    d->n_bits = (uint64_t)n_bytes * 8;
    d->in = in;
    for (int i = 0; i < 32; i++) d->value = (d->value << 1) | (uint64_t)get_bit(in, d->n_bits, d->bpos++);
}

int32_t oc_dec_next(oc_dec *d, int32_t V, const uint64_t *c) {
    uint64_t total = c[V];
    if (total == 0 || total > OC_QUARTER) return -1;
    uint64_t range = d->high - d->low + 1;
    uint64_t offset = ((d->value - d->low + 1) * total - 1) / range;
    int32_t lo = 0, hi = V, sym = 0;
    while (lo < hi) {
        int32_t mid = (lo + hi) / 2;
        if (c[mid] <= offset) { sym = mid; lo = mid + 1; } else { hi = mid; }
    }
    d->high = d->low + (range * c[sym + 1]) / total - 1;
    d->low = d->low + (range * c[sym]) / total;
    for (;;) {
        if (d->high < OC_HALF) {
        } else if (d->low >= OC_HALF) {
            d->low -= OC_HALF; d->high -= OC_HALF; d->value -= OC_HALF;
        } else if (d->low >= OC_QUARTER && d->high < 3 * OC_QUARTER) {
            d->low -= OC_QUARTER; d->high -= OC_QUARTER; d->value -= OC_QUARTER;
        } else {
            break;
        }
        d->low <<= 1;
        d->high = (d->high << 1) | 1;
        d->value = (d->value << 1) | (uint64_t)get_bit(d->in, d->n_bits, d->bpos++);
    }
    return sym;
}

typedef struct {
    oc_enc s;
    uint8_t *out;
    uint64_t cap_bits;
} oc_enc_inc;

void oc_enc_begin(oc_enc_inc *e, uint8_t *out, int64_t cap_bytes) {
    e->s.low = 0;
    e->s.high = OC_TOP - 1;
    e->s.pending = 0;
    e->s.nbits = 0;
    e->s.status = 0;
    e->out = out;
    e->cap_bits = (uint64_t)cap_bytes * 8;
    memset(out, 0, (size_t)cap_bytes);
}

int oc_enc_next(oc_enc_inc *e, int32_t V, const uint64_t *c, int32_t sym) {
    if (sym < 0 || sym >= V || c[sym + 1] <= c[sym]) return -OC_ST_BAD_SYMBOL;
    if (c[V] == 0 || c[V] > OC_QUARTER) return -OC_ST_BAD_TOTAL;
    enc_interval(&e->s, e->out, e->cap_bits, c[sym], c[sym + 1], c[V]);
    return -e->s.status;
}

int64_t oc_enc_finish(oc_enc_inc *e) {
    enc_flush(&e->s, e->out, e->cap_bits);
    if (e->s.status) return -e->s.status;
    return (int64_t)e->s.nbits;
}

int64_t oc_dec_state_size(void) { return (int64_t)sizeof(oc_dec); }
int64_t oc_enc_state_size(void) { return (int64_t)sizeof(oc_enc_inc); }

/* Reference mass rule: freq = max(1, floor((double)p * 1e6 + 0.5)). */
void oc_cum_from_probs_ref(int64_t n, int32_t V, const float *probs, uint64_t *cum) {
    for (int64_t r = 0; r < n; r++) {
        const float *p = probs + r * V;
        uint64_t *c = cum + r * (int64_t)(V + 1);
        uint64_t acc = 0;
        c[0] = 0;
        for (int32_t i = 0; i < V; i++) {
            double s = floor((double)p[i] * 1000000.0 + 0.5);
            int64_t f = (int64_t)s;
            if (f < 1) f = 1;
            acc += (uint64_t)f;
            c[i + 1] = acc;
        }
    }
}

/* ---- framework CDF rules over softcapped fp32 logits --------------------
 * exp2 of the fractional part uses the Taylor series of 2^f = e^(f ln 2)
 * truncated after the f^8 term (coefficients (ln 2)^k / k!, rounded to
 * fp32), evaluated by Horner's rule with one fma per term.  Any fixed
 * fp32 operation sequence is bit-reproducible on CPU and GPU; this one is
 * accurate to a few fp32 ulps on [0, 1). */
static const float OC_EXP2_C[9] = {
    1.0f,
    0.693147180559945309f,
    0.240226506959100712f,
    0.0555041086648215800f,
    0.00961812910762847717f,
    0.00133335581464284434f,
    0.000154035303933816099f,
    0.0000152527338040598403f,
    0.00000132154867901443094f,
};
#define OC_LOG2E 1.44269504088896341f

static inline float oc_exp2_frac(float f) {
    float p = OC_EXP2_C[8];
    for (int k = 7; k >= 0; k--) p = fmaf(p, f, OC_EXP2_C[k]);
    return p;
}

/* u = floor(2^24 * exp(x)) for x = l - max <= 0, as the kernel computes it. */
static inline uint32_t oc_fixed_weight(float l, float mx) {
    float x = l - mx;            /* fp32 subtract */
    float t = x * OC_LOG2E;      /* fp32 multiply */
    float nf = floorf(t);
    if (nf < -25.0f) return 0u;
    float f = t - nf;            /* exact */
    float p = oc_exp2_frac(f);   /* in [1, 2) */
    int n = (int)nf;             /* -25 .. 0 */
    float scaled = ldexpf(p, 24 + n); /* exact power-of-two scaling */
    return (uint32_t)floorf(scaled);
}

/* Fixed-point rule: u_i = floor(2^24 exp(l_i - max)), S = sum u_i (u64,
 * order independent), freq_i = 1 + floor(u_i * (2^cdf_bits - V) / S). */
int oc_cum_from_logits_fixed(int64_t n, int32_t V, const float *logits,
                             int32_t cdf_bits, uint64_t *cum) {
    uint64_t T = 1ull << cdf_bits;
    if ((uint64_t)V >= T) return -1;
    uint64_t budget = T - (uint64_t)V;
    for (int64_t r = 0; r < n; r++) {
        const float *l = logits + r * V;
        uint64_t *c = cum + r * (int64_t)(V + 1);
        float mx = -INFINITY;
        for (int32_t i = 0; i < V; i++) mx = l[i] > mx ? l[i] : mx;
        uint64_t S = 0;
        for (int32_t i = 0; i < V; i++) S += oc_fixed_weight(l[i], mx);
        uint64_t acc = 0;
        c[0] = 0;
        for (int32_t i = 0; i < V; i++) {
            uint64_t u = oc_fixed_weight(l[i], mx);
            acc += 1 + (u * budget) / S;
            c[i + 1] = acc;
        }
    }
    return 0;
}

/* Reference-scale rule over logits: p_i = e_i / sum(e) with e_i the same
 * exp as above (as fp32, e_i = p(f) * 2^n) and the sum taken in the
 * kernel's canonical order: sequential sums over chunks of 32 consecutive
 * entries, then a tree over chunk sums padded to a power of two in which
 * step `stride` adds s[i + stride] into s[i] for i < stride.
 * Then freq_i = max(1, floor((double)p_i * 1e6 + 0.5)). */
static inline float oc_exp_rel(float l, float mx) {
    float x = l - mx;
    float t = x * OC_LOG2E;
    float nf = floorf(t);
    if (nf < -126.0f) return 0.0f;
    float f = t - nf;
    return ldexpf(oc_exp2_frac(f), (int)nf);
}

int oc_cum_from_logits_ref(int64_t n, int32_t V, const float *logits, uint64_t *cum) {
    int32_t nchunk = (V + 31) / 32;
    int32_t np2 = 1;
    while (np2 < nchunk) np2 <<= 1;
    float part[65536];
    if (np2 > 65536) return -1;
    for (int64_t r = 0; r < n; r++) {
        const float *l = logits + r * V;
        uint64_t *c = cum + r * (int64_t)(V + 1);
        float mx = -INFINITY;
        for (int32_t i = 0; i < V; i++) mx = l[i] > mx ? l[i] : mx;
        for (int32_t k = 0; k < np2; k++) {
            float s = 0.0f;
            for (int32_t j = 0; j < 32; j++) {
                int32_t i = k * 32 + j;
                if (k < nchunk && i < V) s = s + oc_exp_rel(l[i], mx);
            }
            part[k] = s;
        }
        for (int32_t stride = np2 / 2; stride >= 1; stride /= 2)
            for (int32_t i = 0; i < stride; i++) part[i] = part[i] + part[i + stride];
        float sum = part[0];
        uint64_t acc = 0;
        c[0] = 0;
        for (int32_t i = 0; i < V; i++) {
            float p = oc_exp_rel(l[i], mx) / sum;
            double s = floor((double)p * 1000000.0 + 0.5);
            int64_t f = (int64_t)s;
            if (f < 1) f = 1;
            acc += (uint64_t)f;
            c[i + 1] = acc;
        }
    }
    return 0;
}
