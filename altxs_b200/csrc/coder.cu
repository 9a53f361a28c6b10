// Batched range-coder entry points (one stream per CTA or per thread).
#include "coder.cuh"
#include "prof.cuh"

using namespace altxs;

namespace {

constexpr int kCoderThreads = 256;

__device__ __forceinline__ int row_of(const int32_t *rows, int i) { return rows ? rows[i] : i; }

__global__ void k_ac_init(int n, const int32_t *rows, altxs_ac_state *st) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    altxs_ac_state s{};
    s.high = kTop - 1;
    st[row_of(rows, i)] = s;
}

__global__ void k_ac_flush(int n, const int32_t *rows, altxs_ac_state *st, uint32_t *bits, int64_t wps) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int r = row_of(rows, i);
    altxs_ac_state s = st[r];
    BitWriter bw;
    bw.begin(bits + (int64_t)r * wps, wps, s.nbits);
    enc_flush(s, bw);
    bw.end();
    s.nbits = bw.nbits;
    s.status |= bw.status;
    st[r] = s;
}

__global__ void k_ac_begin_decode(int n, const int32_t *rows, altxs_ac_state *st, const uint32_t *bits,
                                  const uint64_t *n_bits, int64_t wps) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int r = row_of(rows, i);
    altxs_ac_state s{};
    s.high = kTop - 1;
    s.n_in_bits = n_bits[i];
    if (s.n_in_bits > (uint64_t)wps * 32ull) {
        s.status |= ALTXS_ST_OVERFLOW;
        s.n_in_bits = (uint64_t)wps * 32ull;
    }
    const uint32_t *b = bits + (int64_t)r * wps;
    uint64_t v = 0;
    for (int k = 0; k < 32; ++k) v = (v << 1) | read_bit(b, s.n_in_bits, (uint64_t)k);
    s.value = v;
    s.bpos = 32;
    st[r] = s;
}

// one thread per stream: caller-supplied integer CDFs
__global__ void k_ac_encode_cum(int n, const int32_t *rows, int V, const uint32_t *cum, int64_t ld,
                                const int32_t *syms, altxs_ac_state *st, uint32_t *bits, int64_t wps) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int r = row_of(rows, i);
    altxs_ac_state s = st[r];
    const uint32_t *c = cum + (int64_t)i * ld;
    const int sym = syms[i];
    const uint64_t total = c[V];
    if (sym < 0 || sym >= V || c[sym + 1] <= c[sym]) {
        s.status |= ALTXS_ST_BAD_SYMBOL;
        st[r] = s;
        return;
    }
    if (total == 0 || total > kQuarter) {
        s.status |= ALTXS_ST_BAD_TOTAL;
        st[r] = s;
        return;
    }
    BitWriter bw;
    bw.begin(bits + (int64_t)r * wps, wps, s.nbits);
    enc_symbol(s, bw, c[sym], c[sym + 1], total);
    bw.end();
    s.nbits = bw.nbits;
    s.status |= bw.status;
    st[r] = s;
}

__global__ void k_ac_decode_cum(int n, const int32_t *rows, int V, const uint32_t *cum, int64_t ld,
                                int32_t *syms_out, altxs_ac_state *st, const uint32_t *bits, int64_t wps) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int r = row_of(rows, i);
    altxs_ac_state s = st[r];
    const uint32_t *c = cum + (int64_t)i * ld;
    const uint64_t total = c[V];
    if (total == 0 || total > kQuarter) {
        s.status |= ALTXS_ST_BAD_TOTAL;
        st[r] = s;
        syms_out[i] = 0;
        return;
    }
    const uint64_t off = dec_offset(s, total);
    int lo = 0, hi = V, sym = 0;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if ((uint64_t)c[mid] <= off) {
            sym = mid;
            lo = mid + 1;
        } else {
            hi = mid;
        }
    }
    dec_symbol(s, bits + (int64_t)r * wps, c[sym], c[sym + 1], total);
    syms_out[i] = sym;
    st[r] = s;
}

// one CTA per stream: reference mass rule over fp32 probabilities
__global__ void k_ac_probs(int n, const int32_t *rows, int V, const float *probs, int64_t ld, int32_t *syms,
                           altxs_ac_state *st, uint32_t *bits, int64_t wps, int decode) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint32_t *m = reinterpret_cast<uint32_t *>(smem_raw);
    __shared__ CdfScratch sc;
    const int i = blockIdx.x;
    const int r = row_of(rows, i);
    const float *p = probs + (int64_t)i * ld;
    unsigned long long tot = 0;
    for (int k = threadIdx.x; k < V; k += blockDim.x) {
        const uint32_t f = ref_mass(p[k]);
        m[k] = f;
        tot += f;
    }
    tot = block_sum_u64(tot, sc.ured);
    __syncthreads();
    altxs_ac_state s = st[r];
    if (tot == 0 || tot > kQuarter) {
        if (threadIdx.x == 0) {
            s.status |= ALTXS_ST_BAD_TOTAL;
            st[r] = s;
            if (decode) syms[i] = 0;
        }
        return;
    }
    const uint32_t *b = bits + (int64_t)r * wps;
    if (!decode) {
        const int sym = syms[i];
        if (sym < 0 || sym >= V) {
            if (threadIdx.x == 0) {
                s.status |= ALTXS_ST_BAD_SYMBOL;
                st[r] = s;
            }
            return;
        }
        const uint64_t sl = mass_below(m, V, sym, sc);
        if (threadIdx.x == 0) {
            BitWriter bw;
            bw.begin(bits + (int64_t)r * wps, wps, s.nbits);
            enc_symbol(s, bw, sl, sl + m[sym], tot);
            bw.end();
            s.nbits = bw.nbits;
            s.status |= bw.status;
            st[r] = s;
        }
        return;
    }
    const uint64_t off = dec_offset(s, tot);
    int sym;
    uint64_t sl, sh;
    find_symbol(m, V, off, sc, sym, sl, sh);
    if (threadIdx.x == 0) {
        dec_symbol(s, b, sl, sh, tot);
        syms[i] = sym;
        st[r] = s;
    }
}

// one CTA per row: framework CDF rule -> cumulative table
__global__ void k_cdf_rows(int V, const float *logits, int64_t ld, int mode, int cdf_bits, uint32_t *cum,
                           int64_t cld) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float *buf = reinterpret_cast<float *>(smem_raw);
    __shared__ CdfScratch sc;
    const int i = blockIdx.x;
    for (int k = threadIdx.x; k < V; k += blockDim.x) buf[k] = logits[(int64_t)i * ld + k];
    __syncthreads();
    uint32_t status = 0;
    logits_to_masses(buf, V, mode, cdf_bits, sc, status);
    const uint32_t *m = reinterpret_cast<const uint32_t *>(buf);
    const int nt = blockDim.x, C = (V + nt - 1) / nt;
    const int b0 = min(V, (int)threadIdx.x * C), b1 = min(V, b0 + C);
    unsigned long long mine = 0;
    for (int k = b0; k < b1; ++k) mine += m[k];
    unsigned long long acc = block_exclusive_scan_u64(mine, sc);
    uint32_t *c = cum + (int64_t)i * cld;
    if (threadIdx.x == 0) c[0] = 0;
    for (int k = b0; k < b1; ++k) {
        acc += m[k];
        c[k + 1] = (uint32_t)acc;
    }
}

inline cudaStream_t S(altxs_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }
inline int grid1(int n, int t) { return (n + t - 1) / t; }

}  // namespace

extern "C" {

int altxs_ac_init(int n, const int32_t *rows, altxs_ac_state *st, altxs_stream_t stream) {
    if (n < 0 || (n > 0 && !st)) return ALTXS_EINVAL;
    if (n == 0) return ALTXS_OK;
    ALTXS_LAUNCH(::altxs::kKCoder, S(stream), k_ac_init<<<grid1(n, 128), 128, 0, S(stream)>>>(n, rows, st));
    return ALTXS_OK;
}

static int probs_smem_ok(int V) { return V >= 1 && (int64_t)V * 4 <= 160 * 1024; }

int altxs_ac_encode_probs(int n, const int32_t *rows, int vocab, const float *probs, int64_t ld,
                          const int32_t *syms, altxs_ac_state *st, uint32_t *bits, int64_t wps,
                          altxs_stream_t stream) {
    if (n < 0 || !probs_smem_ok(vocab) || ld < vocab || wps < 1) return ALTXS_EINVAL;
    if (n == 0) return ALTXS_OK;
    const size_t sm = (size_t)vocab * 4;
    if (sm > 48 * 1024)
        cudaFuncSetAttribute(k_ac_probs, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    ALTXS_LAUNCH(::altxs::kKCoder, S(stream), k_ac_probs<<<n, kCoderThreads, sm, S(stream)>>>(n, rows, vocab, probs, ld, const_cast<int32_t *>(syms), st,
                                                    bits, wps, 0));
    return ALTXS_OK;
}

int altxs_ac_decode_probs(int n, const int32_t *rows, int vocab, const float *probs, int64_t ld,
                          int32_t *syms_out, altxs_ac_state *st, const uint32_t *bits, int64_t wps,
                          altxs_stream_t stream) {
    if (n < 0 || !probs_smem_ok(vocab) || ld < vocab || wps < 1) return ALTXS_EINVAL;
    if (n == 0) return ALTXS_OK;
    const size_t sm = (size_t)vocab * 4;
    if (sm > 48 * 1024)
        cudaFuncSetAttribute(k_ac_probs, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    ALTXS_LAUNCH(::altxs::kKCoder, S(stream), k_ac_probs<<<n, kCoderThreads, sm, S(stream)>>>(n, rows, vocab, probs, ld, syms_out, st,
                                                    const_cast<uint32_t *>(bits), wps, 1));
    return ALTXS_OK;
}

int altxs_ac_encode_cum(int n, const int32_t *rows, int vocab, const uint32_t *cum, int64_t ld,
                        const int32_t *syms, altxs_ac_state *st, uint32_t *bits, int64_t wps,
                        altxs_stream_t stream) {
    if (n < 0 || vocab < 1 || ld < vocab + 1 || wps < 1) return ALTXS_EINVAL;
    if (n == 0) return ALTXS_OK;
    ALTXS_LAUNCH(::altxs::kKCoder, S(stream), k_ac_encode_cum<<<grid1(n, 128), 128, 0, S(stream)>>>(n, rows, vocab, cum, ld, syms, st, bits, wps));
    return ALTXS_OK;
}

int altxs_ac_decode_cum(int n, const int32_t *rows, int vocab, const uint32_t *cum, int64_t ld,
                        int32_t *syms_out, altxs_ac_state *st, const uint32_t *bits, int64_t wps,
                        altxs_stream_t stream) {
    if (n < 0 || vocab < 1 || ld < vocab + 1 || wps < 1) return ALTXS_EINVAL;
    if (n == 0) return ALTXS_OK;
    ALTXS_LAUNCH(::altxs::kKCoder, S(stream), k_ac_decode_cum<<<grid1(n, 128), 128, 0, S(stream)>>>(n, rows, vocab, cum, ld, syms_out, st, bits, wps));
    return ALTXS_OK;
}

int altxs_ac_flush(int n, const int32_t *rows, altxs_ac_state *st, uint32_t *bits, int64_t wps,
                   altxs_stream_t stream) {
    if (n < 0 || wps < 1) return ALTXS_EINVAL;
    if (n == 0) return ALTXS_OK;
    ALTXS_LAUNCH(::altxs::kKCoder, S(stream), k_ac_flush<<<grid1(n, 128), 128, 0, S(stream)>>>(n, rows, st, bits, wps));
    return ALTXS_OK;
}

int altxs_ac_begin_decode(int n, const int32_t *rows, altxs_ac_state *st, const uint32_t *bits,
                          const uint64_t *n_bits, int64_t wps, altxs_stream_t stream) {
    if (n < 0 || wps < 1) return ALTXS_EINVAL;
    if (n == 0) return ALTXS_OK;
    ALTXS_LAUNCH(::altxs::kKCoder, S(stream), k_ac_begin_decode<<<grid1(n, 128), 128, 0, S(stream)>>>(n, rows, st, bits, n_bits, wps));
    return ALTXS_OK;
}

int altxs_cdf_from_logits(int n, int vocab, const float *logits, int64_t ld, int mode, int cdf_bits,
                          uint32_t *cum, int64_t cum_ld, altxs_stream_t stream) {
    if (n < 0 || !probs_smem_ok(vocab) || ld < vocab || cum_ld < vocab + 1) return ALTXS_EINVAL;
    if (mode != ALTXS_CDF_FIXED && mode != ALTXS_CDF_REF) return ALTXS_EINVAL;
    if (mode == ALTXS_CDF_FIXED && (cdf_bits > 30 || (1ll << cdf_bits) <= vocab)) return ALTXS_EINVAL;
    if (n == 0) return ALTXS_OK;
    const size_t sm = (size_t)vocab * 4;
    if (sm > 48 * 1024)
        cudaFuncSetAttribute(k_cdf_rows, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    ALTXS_LAUNCH(::altxs::kKCoder, S(stream), k_cdf_rows<<<n, kCoderThreads, sm, S(stream)>>>(vocab, logits, ld, mode, cdf_bits, cum, cum_ld));
    return ALTXS_OK;
}

const char *altxs_version(void) { return "altxs_b200 0.1 (sm_100a)"; }

}  // extern "C"
