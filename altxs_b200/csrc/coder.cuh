// Range coder (32-bit Witten-Neal-Cleary) and per-row integer CDF machinery.
//
// Coder arithmetic follows the reference host coder
// (altxs src/model/arithmetic_coder_lm.py:90-137, 175-195, 235-284): the
// interval update high = low + range*sh/total - 1, low = low + range*sl/total,
// E1/E2/E3 renormalisation with a pending counter, the pending+1 flush, and
// MSB-first bits.  One thread runs the serial coder; the CTA computes the
// V-wide CDF around it.
#pragma once

#include "common.cuh"

namespace altxs {

// Writes bits MSB-first into the byte stream image held in uint32 words.
struct BitWriter {
    uint32_t *base;
    uint64_t cap_bits;
    uint64_t nbits;
    uint32_t word;
    uint32_t status;

    __device__ __forceinline__ void begin(uint32_t *b, int64_t words, uint64_t nb) {
        base = b;
        cap_bits = (uint64_t)words * 32ull;
        nbits = nb;
        status = 0;
        word = ((nb & 31ull) && nb < cap_bits) ? base[nb >> 5] : 0u;
    }
    __device__ __forceinline__ void put(uint32_t bit) {
        if (nbits >= cap_bits) {
            status |= ALTXS_ST_OVERFLOW;
            return;
        }
        if (bit) {
            const uint32_t k = (uint32_t)(nbits & 31ull);
            word |= 1u << (((k >> 3) << 3) + 7u - (k & 7u));
        }
        ++nbits;
        if ((nbits & 31ull) == 0) {
            base[(nbits >> 5) - 1] = word;
            word = 0u;
        }
    }
    __device__ __forceinline__ void put_run(uint32_t bit, uint64_t n) {
        for (uint64_t i = 0; i < n; ++i) put(bit);
    }
    __device__ __forceinline__ void end() {
        if ((nbits & 31ull) && nbits <= cap_bits) base[nbits >> 5] = word;
    }
};

__device__ __forceinline__ uint32_t read_bit(const uint32_t *base, uint64_t n_in_bits, uint64_t k) {
    if (k >= n_in_bits) return 0u;
    const uint32_t w = base[k >> 5];
    const uint32_t kk = (uint32_t)(k & 31ull);
    return (w >> (((kk >> 3) << 3) + 7u - (kk & 7u))) & 1u;
}

// Encode one symbol with [sl, sh) of `total` into the stream state.
__device__ __forceinline__ void enc_symbol(altxs_ac_state &s, BitWriter &bw, uint64_t sl, uint64_t sh,
                                           uint64_t total) {
    const uint64_t range = s.high - s.low + 1;
    s.high = s.low + (range * sh) / total - 1;
    s.low = s.low + (range * sl) / total;
    for (;;) {
        if (s.high < kHalf) {
            bw.put(0);
            bw.put_run(1, s.pending);
            s.pending = 0;
        } else if (s.low >= kHalf) {
            bw.put(1);
            bw.put_run(0, s.pending);
            s.pending = 0;
            s.low -= kHalf;
            s.high -= kHalf;
        } else if (s.low >= kQuarter && s.high < 3 * kQuarter) {
            s.pending += 1;
            s.low -= kQuarter;
            s.high -= kQuarter;
        } else {
            break;
        }
        s.low <<= 1;
        s.high = (s.high << 1) | 1ull;
    }
}

__device__ __forceinline__ void enc_flush(altxs_ac_state &s, BitWriter &bw) {
    s.pending += 1;
    if (s.low < kQuarter) {
        bw.put(0);
        bw.put_run(1, s.pending);
    } else {
        bw.put(1);
        bw.put_run(0, s.pending);
    }
    s.pending = 0;
}

// Decoder: offset of the current value inside the interval, scaled to total.
__device__ __forceinline__ uint64_t dec_offset(const altxs_ac_state &s, uint64_t total) {
    const uint64_t range = s.high - s.low + 1;
    return ((s.value - s.low + 1) * total - 1) / range;
}
__device__ __forceinline__ void dec_symbol(altxs_ac_state &s, const uint32_t *bits, uint64_t sl, uint64_t sh,
                                           uint64_t total) {
    const uint64_t range = s.high - s.low + 1;
    s.high = s.low + (range * sh) / total - 1;
    s.low = s.low + (range * sl) / total;
    for (;;) {
        if (s.high < kHalf) {
        } else if (s.low >= kHalf) {
            s.low -= kHalf;
            s.high -= kHalf;
            s.value -= kHalf;
        } else if (s.low >= kQuarter && s.high < 3 * kQuarter) {
            s.low -= kQuarter;
            s.high -= kQuarter;
            s.value -= kQuarter;
        } else {
            break;
        }
        s.low <<= 1;
        s.high = (s.high << 1) | 1ull;
        s.value = (s.value << 1) | read_bit(bits, s.n_in_bits, s.bpos);
        s.bpos += 1;
    }
}

// ---------------------------------------------------------------------------
// CTA-wide integer CDF over a row held in shared memory.
//
// `buf` holds V entries.  fill_masses() turns them in place into uint32
// masses; the remaining helpers work on masses.  Threads own contiguous
// chunks [t*C, (t+1)*C) with C = ceil(V / blockDim.x) for the decode search.

struct CdfScratch {
    float fred[32];
    unsigned long long ured[32];
    unsigned long long uscan[1024];
    float part[2048];  // ref-rule chunk sums (V <= 65536)
    uint64_t bcast[4];
    int32_t ibcast[4];
};

// In-place: buf[i] (softcapped logits as float) -> masses (uint32) for the
// framework rules.  Returns total (sum of masses) in every thread.
__device__ inline uint64_t logits_to_masses(float *buf, int V, int mode, int cdf_bits, CdfScratch &sc,
                                            uint32_t &status) {
    const int tid = threadIdx.x, nt = blockDim.x;
    float mx = -INFINITY;
    bool bad = false;
    for (int i = tid; i < V; i += nt) {
        const float l = buf[i];
        bad |= !isfinite(l);
        mx = fmaxf(mx, l);
    }
    mx = block_max(mx, sc.fred);
    const int anybad = __syncthreads_or(bad);
    if (anybad) {
        // non-finite logits: fall back to the uniform distribution, flag it
        status |= ALTXS_ST_NONFINITE;
        __syncthreads();
        for (int i = tid; i < V; i += nt) reinterpret_cast<uint32_t *>(buf)[i] = 1u;
        __syncthreads();
        return (uint64_t)V;
    }
    uint32_t *m = reinterpret_cast<uint32_t *>(buf);
    if (mode == ALTXS_CDF_FIXED) {
        unsigned long long S = 0;
        for (int i = tid; i < V; i += nt) {
            const uint32_t u = fixed_weight(buf[i], mx);
            m[i] = u;  // in place: same thread reads then writes element i
            S += u;
        }
        S = block_sum_u64(S, sc.ured);
        const uint64_t budget = (1ull << cdf_bits) - (uint64_t)V;
        // floor(u * budget / S) for every entry: a double-precision estimate
        // (off by at most one or two) corrected with exact integer products
        const double inv = (double)budget / (double)S;
        unsigned long long tot = 0;
        for (int i = tid; i < V; i += nt) {
            const uint64_t a = (uint64_t)m[i] * budget;
            uint64_t q = (uint64_t)((double)m[i] * inv);
            while (q > 0 && q * S > a) --q;
            while ((q + 1) * S <= a) ++q;
            const uint32_t f = 1u + (uint32_t)q;
            m[i] = f;
            tot += f;
        }
        tot = block_sum_u64(tot, sc.ured);
        __syncthreads();
        return tot;
    }
    // reference-scale rule: canonical fp32 sum (32-element chunks, then a
    // tree over chunk sums padded to a power of two)
    const int nchunk = (V + 31) >> 5;
    int np2 = 1;
    while (np2 < nchunk) np2 <<= 1;
    for (int c = tid; c < np2; c += nt) {
        float s = 0.0f;
        if (c < nchunk) {
            for (int j = 0; j < 32; ++j) {
                const int i = c * 32 + j;
                if (i < V) s = __fadd_rn(s, exp_rel(buf[i], mx));
            }
        }
        sc.part[c] = s;
    }
    __syncthreads();
    for (int stride = np2 >> 1; stride >= 1; stride >>= 1) {
        for (int i = tid; i < stride; i += nt) sc.part[i] = __fadd_rn(sc.part[i], sc.part[i + stride]);
        __syncthreads();
    }
    const float sum = sc.part[0];
    unsigned long long tot = 0;
    for (int i = tid; i < V; i += nt) {
        const float p = __fdiv_rn(exp_rel(buf[i], mx), sum);
        const uint32_t f = ref_mass(p);
        m[i] = f;
        tot += f;
    }
    tot = block_sum_u64(tot, sc.ured);
    __syncthreads();
    return tot;
}

// Sum of masses of symbols < sym (every thread gets it).
__device__ inline uint64_t mass_below(const uint32_t *m, int V, int sym, CdfScratch &sc) {
    unsigned long long s = 0;
    for (int i = threadIdx.x; i < V && i < sym; i += blockDim.x) s += m[i];
    return block_sum_u64(s, sc.ured);
}

// Exclusive prefix over threads of a per-thread u64 value (block scan).
__device__ inline unsigned long long block_exclusive_scan_u64(unsigned long long v, CdfScratch &sc) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    unsigned long long inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long n = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += n;
    }
    __syncthreads();
    if (lane == 31) sc.ured[wid] = inc;
    __syncthreads();
    if (wid == 0) {
        unsigned long long w = lane < nw ? sc.ured[lane] : 0ull;
        unsigned long long wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long n = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += n;
        }
        if (lane < nw) sc.uscan[lane] = wi - w;
    }
    __syncthreads();
    return sc.uscan[wid] + inc - v;
}

// Largest s with cum[s] <= offset given masses m; every thread gets sym and
// its [sl, sh).  Threads own contiguous chunks of ceil(V / blockDim) entries.
__device__ inline void find_symbol(const uint32_t *m, int V, uint64_t offset, CdfScratch &sc, int &sym,
                                   uint64_t &sl, uint64_t &sh) {
    const int tid = threadIdx.x, nt = blockDim.x;
    const int C = (V + nt - 1) / nt;
    const int b0 = min(V, tid * C), b1 = min(V, b0 + C);
    unsigned long long mine = 0;
    for (int i = b0; i < b1; ++i) mine += m[i];
    if (tid == 0) {
        sc.ibcast[0] = V - 1;
        sc.bcast[0] = 0;
        sc.bcast[1] = 0;
    }
    const unsigned long long start = block_exclusive_scan_u64(mine, sc);
    if (b0 < b1 && offset >= start && offset < start + mine) {
        unsigned long long acc = start;
        int s = b0;
        for (; s < b1 - 1; ++s) {
            if (acc + m[s] > offset) break;
            acc += m[s];
        }
        sc.ibcast[0] = s;
        sc.bcast[0] = acc;
        sc.bcast[1] = acc + m[s];
    }
    __syncthreads();
    sym = sc.ibcast[0];
    sl = sc.bcast[0];
    sh = sc.bcast[1];
    __syncthreads();
}

}  // namespace altxs
