// Causal window attention on the tensor cores (sm_100a), one CTA per
// (128-query tile, head), the scores never leaving the SM.
//
// Operands are hi/lo bf16 planes (tc.cuh: x = hi + lo to 16 significand
// bits; a product is hi*hi + hi*lo + lo*hi with fp32 accumulation), written by
// a split pass: Q and K as [head][T][64] (head dim zero-padded to one 128-byte
// swizzle row), V transposed as [kv head][hd][align8(T)] so that every MMA
// operand is K-major.  Per key tile j (128 keys):
//   warp 8  TMA: Q once; K_j and V_j^T into a two-stage ring;
//   warp 9  MMA: S_j = Q K_j^T into one of two tensor-memory score buffers,
//           then (once the softmax has written P_{j-1}) O_h = P_h V_h of
//           each 64-key half h into its accumulator: S_{j+1} runs while the
//           softmax works on S_j;
//   warps 0-7  softmax: warp w takes query rows 32 (w % 4) .. and key half
//           w / 4, with that half's own running max, sum and output: the
//           max of the scaled, causally masked scores, the previous tile's
//           P_h V_h folded in with its rescale, then p = 2^(x - m), the sum,
//           and p as hi/lo planes in shared memory (the A operand of P V).
// After the last tile the two halves of each row are combined: y = O / l
// (and, on request, the row's log-sum-exp for the backward).  Every wait is
// bounded; a wait that gives up stops the CTA's roles, drains its copies and
// MMAs, frees the tensor memory and leaves y unwritten.  The backward kernels
// (dq; dk and dv) follow after the forward, below.
//
// The rows are the reference's causal softmax attention over the window
// (model.py CausalSelfAttention via F.scaled_dot_product_attention, is_causal,
// fp32), formed online instead of as a T x T matrix.
#include "flash.cuh"
#include "prof.cuh"
#include "tc.cuh"
#include "tcgen05.cuh"

namespace altxs {
namespace {

constexpr int kFM = 128;  // queries per CTA
constexpr int kFN = 128;  // keys per tile
constexpr int kFD = 64;   // head dim of the Q/K planes (zero-padded)
constexpr int kQT = kFM * kFD * 2;          // one Q plane tile: 16 KB
constexpr int kKT = kFN * kFD * 2;          // one K plane tile: 16 KB
constexpr int kVAtom = 64 * 128;            // one V^T plane atom (64 keys x up to 64 dims): 8 KB
constexpr int kVT = 2 * kVAtom;             // one V^T plane tile: 16 KB
constexpr int kStage = 2 * kKT + 2 * kVT;   // K hi, K lo, V^T hi, V^T lo
constexpr int kPAtom = kFM * 128;           // one P plane atom (128 rows x 64 keys): 16 KB
constexpr int kPT = 2 * kPAtom;             // one P plane: 32 KB
constexpr int kSmem = 2 * kQT + 2 * kStage + 2 * kPT + 1024;
static_assert(kSmem + 256 <= 227 * 1024, "shared memory");
constexpr uint32_t kTmemCols = 512;  // S buffers at 0 and 128, O at 256
constexpr unsigned kAll = 0xffffffffu;

template <int N>
constexpr uint32_t idesc_kmajor() {  // kind::f16: fp32 accumulate, bf16 A and B, both K-major, M = 128
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kFM >> 4) << 24);
}

__device__ __forceinline__ void sts_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
// hi/lo bf16 planes of 8 consecutive values at element e (16-byte aligned)
__device__ __forceinline__ void store8_split(uint16_t *hi, uint16_t *lo, int64_t e, const float *x) {
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const __nv_bfloat162 h2 = __floats2bfloat162_rn(x[2 * k], x[2 * k + 1]);
        const float2 hf = __bfloat1622float2(h2);
        const __nv_bfloat162 l2 = __floats2bfloat162_rn(__fsub_rn(x[2 * k], hf.x), __fsub_rn(x[2 * k + 1], hf.y));
        hw[k] = *reinterpret_cast<const uint32_t *>(&h2);
        lw[k] = *reinterpret_cast<const uint32_t *>(&l2);
    }
    *reinterpret_cast<uint4 *>(hi + e) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4 *>(lo + e) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
}

// Q and K rows as zero-padded planes, V^T through a shared-memory transpose.
// grid (32-row blocks of T, H + 2 Hkv): y < H a Q head, then K heads, then V heads.
__global__ void __launch_bounds__(256) k_flash_split(FlashArgs a, int64_t tp, uint16_t *qh, uint16_t *ql,
                                                     uint16_t *kh, uint16_t *kl, uint16_t *vh, uint16_t *vl) {
    __shared__ float tile[32][65];
    const int t0 = blockIdx.x * 32, hd = a.hd, y = blockIdx.y;
    if (y < a.H + a.Hkv) {  // Q [H][T][64], K [Hkv][T][64]
        const bool isq = y < a.H;
        const int hh = isq ? y : y - a.H;
        const float *src = isq ? a.q : a.k;
        const int64_t ld = isq ? a.ldq : a.ldk;
        uint16_t *dh = isq ? qh : kh, *dl = isq ? ql : kl;
        // one 16-byte store per plane and thread: 8 consecutive columns of one row
        for (int i = threadIdx.x; i < 32 * (kFD / 8); i += blockDim.x) {
            const int c8 = (i % (kFD / 8)) * 8, t = t0 + i / (kFD / 8);
            if (t >= a.T) break;
            float x[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) x[e] = c8 + e < hd ? src[(int64_t)t * ld + hh * hd + c8 + e] : 0.0f;
            store8_split(dh, dl, ((int64_t)hh * a.T + t) * kFD + c8, x);
        }
        return;
    }
    // V^T [Hkv][hd][tp]: columns T .. tp are zero (keys past T read as zero)
    const int g = y - a.H - a.Hkv;
    for (int i = threadIdx.x; i < 32 * hd; i += blockDim.x) {
        const int r = i / hd, c = i % hd, t = t0 + r;
        tile[r][c] = t < a.T ? a.v[(int64_t)t * a.ldv + g * hd + c] : 0.0f;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 4 * hd; i += blockDim.x) {  // 8 consecutive keys of one dim per thread
        const int c = i / 4, r8 = (i % 4) * 8;
        if (t0 + r8 >= tp) continue;  // tp is a multiple of 8: a group is all below tp or all past it
        float x[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = tile[r8 + e][c];
        store8_split(vh, vl, ((int64_t)g * hd + c) * tp + t0 + r8, x);
    }
}

__device__ __forceinline__ float ex2(float x) {  // 2^x (the SFU instruction; 2^-inf = 0)
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int HD>
__global__ void __launch_bounds__(320, 1)
    k_flash_fwd(const __grid_constant__ CUtensorMap tq_hi, const __grid_constant__ CUtensorMap tq_lo,
                const __grid_constant__ CUtensorMap tk_hi, const __grid_constant__ CUtensorMap tk_lo,
                const __grid_constant__ CUtensorMap tv_hi, const __grid_constant__ CUtensorMap tv_lo, FlashArgs a) {
    extern __shared__ unsigned char fl_smem_raw[];
    __shared__ __align__(8) uint64_t q_full, kv_full[2], kv_empty[2], s_full[2], p_full[2], o_full[2], drainb,
        xbar[4];
    __shared__ uint32_t tmem_sh;
    __shared__ volatile int abort_sh;
    const uint32_t raw_s = smem_u32(fl_smem_raw);
    unsigned char *sm = fl_smem_raw + ((1024u - (raw_s & 1023u)) & 1023u);
    const uint32_t sq = smem_u32(sm), sst = sq + 2 * kQT, sp = sst + 2 * kStage;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * kFM, h = blockIdx.y, g = h / (a.H / a.Hkv);
    const int last_q = min(a.T, q0 + kFM) - 1;
    const int n = last_q / kFN + 1;  // key tiles up to the diagonal
    if (threadIdx.x == 0) {
        mbar_init(&q_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
            mbar_init(&s_full[s], 1);
        }
        for (int hh = 0; hh < 2; ++hh) {
            mbar_init(&p_full[hh], 4);  // one arrival per softmax warp of the key half
            mbar_init(&o_full[hh], 1);
        }
        for (int qq = 0; qq < 4; ++qq) mbar_init(&xbar[qq], 1);  // the key-half-1 warp of a lane quarter
        mbar_init(&drainb, 1);
        abort_sh = 0;
        fence_mbar_init();
    }
    if (warp == 9) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_sh)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_sh;

    if (warp == 8) {
        if (lane == 0) {
            mbar_expect_tx(&q_full, 2 * kQT);
            tma_load_3d(sm, &tq_hi, 0, q0, h, &q_full);
            tma_load_3d(sm + kQT, &tq_lo, 0, q0, h, &q_full);
            int j = 0;
            for (; j < n && !abort_sh; ++j) {
                const int s = j & 1;
                if (j >= 2 && !mbar_wait_bounded(&kv_empty[s], ((j - 2) >> 1) & 1, wait_limit())) {
                    abort_sh = 1;
                    break;
                }
                unsigned char *st = sm + 2 * kQT + s * kStage;
                mbar_expect_tx(&kv_full[s], 2 * kKT + 4 * 128 * HD);
                tma_load_3d(st, &tk_hi, 0, j * kFN, g, &kv_full[s]);
                tma_load_3d(st + kKT, &tk_lo, 0, j * kFN, g, &kv_full[s]);
#pragma unroll
                for (int at = 0; at < 2; ++at) {
                    tma_load_3d(st + 2 * kKT + at * kVAtom, &tv_hi, j * kFN + 64 * at, 0, g, &kv_full[s]);
                    tma_load_3d(st + 2 * kKT + kVT + at * kVAtom, &tv_lo, j * kFN + 64 * at, 0, g, &kv_full[s]);
                }
            }
            if (abort_sh) {  // let the copies in flight land before the CTA can exit
                mbar_wait_bounded(&q_full, 0, kWaitLimit);
                for (int p = j - 2 > 0 ? j - 2 : 0; p < j; ++p) mbar_wait_bounded(&kv_full[p & 1], (p >> 1) & 1, kWaitLimit);
            }
        }
    } else if (warp == 9) {
        if (lane == 0) {
            bool ok = mbar_wait_bounded(&q_full, 0, wait_limit());
            for (int j = 0; j <= n && ok && !abort_sh; ++j) {
                if (j < n) {  // S_j = Q K_j^T (buffer j & 1, free once P_{j-2} was written)
                    const int s = j & 1;
                    if (!mbar_wait_bounded(&kv_full[s], (j >> 1) & 1, wait_limit())) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t kb = sst + s * kStage;
#pragma unroll
                    for (int kk = 0; kk < kFD / 16; ++kk) {
                        const uint64_t qh = sw128_desc(sq + kk * 32, 16), qlo = sw128_desc(sq + kQT + kk * 32, 16);
                        const uint64_t kh = sw128_desc(kb + kk * 32, 16), klo = sw128_desc(kb + kKT + kk * 32, 16);
                        const uint32_t d = tmem + s * kFN;
                        tc_mma(d, qh, kh, idesc_kmajor<kFN>(), kk != 0);
                        tc_mma(d, qh, klo, idesc_kmajor<kFN>(), 1u);
                        tc_mma(d, qlo, kh, idesc_kmajor<kFN>(), 1u);
                    }
                    tc_commit(&s_full[s]);
                }
                if (j >= 1) {  // O_h = P_h V_h of tile j-1 for each key half h (P_h written, O_h of j-2 read)
                    const int jp = j - 1, s = jp & 1;
                    const uint32_t vb = sst + s * kStage + 2 * kKT;
                    for (int hh = 0; hh < 2 && ok; ++hh) {
                        if (!mbar_wait_bounded(&p_full[hh], jp & 1, wait_limit())) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            const uint64_t ph = sw128_desc(sp + hh * kPAtom + kk * 32, 16);
                            const uint64_t pl = sw128_desc(sp + kPT + hh * kPAtom + kk * 32, 16);
                            const uint64_t vh = sw128_desc(vb + hh * kVAtom + kk * 32, 16);
                            const uint64_t vl = sw128_desc(vb + kVT + hh * kVAtom + kk * 32, 16);
                            const uint32_t d = tmem + 2 * kFN + hh * 64;
                            tc_mma(d, ph, vh, idesc_kmajor<HD>(), kk != 0);
                            tc_mma(d, ph, vl, idesc_kmajor<HD>(), 1u);
                            tc_mma(d, pl, vh, idesc_kmajor<HD>(), 1u);
                        }
                        tc_commit(&o_full[hh]);
                    }
                    if (!ok) break;
                    tc_commit(&kv_empty[s]);
                }
            }
            if (!ok) abort_sh = 1;
            // every MMA this thread issued has completed before the CTA can exit
            tc_commit(&drainb);
            mbar_wait_bounded(&drainb, 0, kWaitLimit);
        }
    } else {
        // softmax, warps 0-7: warp w reads tensor-memory lanes 32 (w % 4) ..
        // (query rows) and key half h = w / 4 of every score tile, with its own
        // running max m_h, sum l_h and output o_h = sum over its keys of p v
        // (the tensor cores form P_h V_h per half).  At the end the half-1 warp
        // of each lane quarter hands (m_1, l_1, o_1) to the half-0 warp through a
        // free shared-memory stage, which combines and stores y.  Scores in
        // log2 units: x = s * scale * log2(e), p = 2^(x - m).
        const int quarter = warp & 3, half = warp >> 2;
        const int r = quarter * 32 + lane;
        const int qi = min(q0 + r, a.T - 1);  // rows past T mask like the last row and are not stored
        const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
        const float c2 = __fmul_rn(a.scale, 1.4426950408889634f);  // log2(e)
        float o[HD];
#pragma unroll
        for (int c = 0; c < HD; ++c) o[c] = 0.0f;
        float m = -INFINITY, l = 0.0f, a_prev = 0.0f;
        bool ok = true;
        for (int j = 0; j <= n; ++j) {
            float m_new = m;
            const uint32_t sb = tmem + lanes + (j & 1) * kFN + half * 64;
            const int kb = j * kFN + half * 64;  // first key of this warp's half
            const bool whole = kb + 63 <= q0;    // every row of the tile sees all 64 keys
            if (j < n) {  // pass 1: the max of this half's scaled, masked scores (log2 units)
                ok = __all_sync(kAll, ok && !abort_sh && mbar_wait_bounded(&s_full[j & 1], (j >> 1) & 1, wait_limit()));
                if (!ok) break;
                tc_fence_after();
#pragma unroll
                for (int c0 = 0; c0 < 64; c0 += 32) {
                    float v[32];
                    tc_ld32(sb + c0, v);
#pragma unroll
                    for (int u = 0; u < 32; ++u)
                        m_new = fmaxf(m_new, whole || kb + c0 + u <= qi ? __fmul_rn(v[u], c2) : -INFINITY);
                }
            }
            if (j >= 1) {  // fold the previous tile: o = o * 2^(m_{j-2} - m_{j-1}) + (P_h V_h)_{j-1}
                ok = __all_sync(kAll, ok && !abort_sh && mbar_wait_bounded(&o_full[half], (j - 1) & 1, wait_limit()));
                if (!ok) break;
                tc_fence_after();
                const uint32_t ob = tmem + lanes + 2 * kFN + half * 64;
#pragma unroll
                for (int c0 = 0; c0 < HD; c0 += 32) {
                    float v[32];
                    tc_ld32(ob + c0, v);
#pragma unroll
                    for (int u = 0; u < 32; ++u) o[c0 + u] = __fmaf_rn(o[c0 + u], a_prev, v[u]);
                }
            }
            if (j == n) break;
            // pass 2: p = 2^(x - m_j) as hi/lo planes (atom `half` of P), this half's sum;
            // a half that has seen no key yet keeps m = -inf, p = 0 and alpha = 0
            const bool seen = m_new != -INFINITY;
            const float alpha = seen ? ex2(__fsub_rn(m, m_new)) : 0.0f;
            float sum = 0.0f;
            const uint32_t row = sp + half * kPAtom + r * 128;
#pragma unroll
            for (int c0 = 0; c0 < 64; c0 += 32) {
                float v[32];
                tc_ld32(sb + c0, v);  // the scores again (tensor-memory reads are cheaper than 64 more registers)
#pragma unroll
                for (int u = 0; u < 32; ++u) {
                    v[u] = seen && (whole || kb + c0 + u <= qi) ? ex2(__fsub_rn(__fmul_rn(v[u], c2), m_new)) : 0.0f;
                    sum = __fadd_rn(sum, v[u]);
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {  // 16-byte chunk c0 / 8 + k of the row, swizzled
                    uint32_t hw[4], lw[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float x0 = v[8 * k + 2 * e], x1 = v[8 * k + 2 * e + 1];
                        const __nv_bfloat162 hi2 = __floats2bfloat162_rn(x0, x1);
                        const float2 hf = __bfloat1622float2(hi2);
                        const __nv_bfloat162 lo2 = __floats2bfloat162_rn(__fsub_rn(x0, hf.x), __fsub_rn(x1, hf.y));
                        hw[e] = *reinterpret_cast<const uint32_t *>(&hi2);
                        lw[e] = *reinterpret_cast<const uint32_t *>(&lo2);
                    }
                    const uint32_t off = (uint32_t)((((c0 / 8 + k) ^ (r & 7))) << 4);
                    sts_v4(row + off, hw[0], hw[1], hw[2], hw[3]);
                    sts_v4(row + kPT + off, lw[0], lw[1], lw[2], lw[3]);
                }
            }
            l = __fmaf_rn(l, alpha, sum);
            m = m_new;
            a_prev = alpha;
            // the tensor cores read P through the async proxy; S_j and O_h of j-1 are consumed
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[half]);
        }
        // combine the halves: y = (o_0 2^(m_0 - M) + o_1 2^(m_1 - M)) / (l_0 2^(m_0 - M) + l_1 2^(m_1 - M)).
        // Hand-off region: the stage of tile n-2 (or the unused stage when n == 1), free once this
        // warp saw its last P V complete (the tensor cores finish MMAs in issue order, tile by tile).
        float *xf = reinterpret_cast<float *>(sm + 2 * kQT + (n & 1) * kStage) + quarter * 32 * (HD + 2);
        if (ok && half == 1) {
            xf[lane] = m;
            xf[32 + lane] = l;
#pragma unroll
            for (int c = 0; c < HD; ++c) xf[(c + 2) * 32 + lane] = o[c];
            __syncwarp();
            if (lane == 0) mbar_arrive(&xbar[quarter]);
        }
        if (ok && half == 0) {
            ok = __all_sync(kAll, mbar_wait_bounded(&xbar[quarter], 0, wait_limit()));
            if (ok && q0 + r < a.T) {
                const float m1 = xf[lane], l1 = xf[32 + lane];
                const float mx = fmaxf(m, m1);  // m (half 0) is finite: key 0 of tile 0 is seen by every row
                const float f0 = ex2(__fsub_rn(m, mx)), f1 = m1 == -INFINITY ? 0.0f : ex2(__fsub_rn(m1, mx));
                const float lt = __fadd_rn(__fmul_rn(l, f0), __fmul_rn(l1, f1));
                if (a.lse) a.lse[(int64_t)h * a.T + q0 + r] = __fadd_rn(mx, log2f(lt));
                float *y = a.y + (int64_t)(q0 + r) * a.ldy + (int64_t)h * HD;
#pragma unroll
                for (int c = 0; c < HD; c += 4) {
                    float w[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        w[e] = __fdiv_rn(__fadd_rn(__fmul_rn(o[c + e], f0), __fmul_rn(xf[(c + e + 2) * 32 + lane], f1)),
                                         lt);
                    *reinterpret_cast<float4 *>(y + c) = make_float4(w[0], w[1], w[2], w[3]);
                }
            }
        }
        if (!ok) abort_sh = 1;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// ---- backward --------------------------------------------------------------
//
// dS = P o (dP - D) * scale with P = 2^(s * scale * log2 e - lse), dP = dy v^T
// and D = rowsum(dy o out); dq = dS k, dk = dS^T q, dv = P^T dy.  Two kernels,
// each sum in a fixed order:
//   dq: one CTA per (128 queries, head), key tiles 0 .. diagonal;
//   dk, dv: one CTA per (128 keys, kv head), the group's heads one after
//       another, each over its 64-query tiles from the diagonal on.
// Both are one template: rows R (q and dy, or k and v) stay in shared memory,
// column tiles C (k and v, or q and dy) stream through; X = R1 C1^T and
// Y = R2 C2^T (the scores and dP, or their transposes) go to tensor memory,
// the eight compute warps form P and dS as hi/lo planes in shared memory, and
// the tensor cores add dS C1 (and P C2) into the row accumulators, reading C
// as an MN-major operand (its rows are the reduction index).

// Row planes [heads][T][64] of q, dy, k and v (head dim zero-padded).
// grid (32-row blocks of T, 2 H + 2 Hkv): q heads, dy heads, k heads, v heads.
__global__ void __launch_bounds__(256) k_flash_bwd_split(FlashBwdArgs a, uint16_t *qh, uint16_t *ql, uint16_t *oh,
                                                         uint16_t *ol, uint16_t *kh, uint16_t *kl, uint16_t *vh,
                                                         uint16_t *vl) {
    const int t0 = blockIdx.x * 32, hd = a.hd, y = blockIdx.y;
    const float *src;
    int64_t ld;
    uint16_t *dh, *dl;
    int hh;
    if (y < a.H) {
        src = a.q, ld = a.ldq, dh = qh, dl = ql, hh = y;
    } else if (y < 2 * a.H) {
        src = a.dout, ld = a.lddo, dh = oh, dl = ol, hh = y - a.H;
    } else if (y < 2 * a.H + a.Hkv) {
        src = a.k, ld = a.ldk, dh = kh, dl = kl, hh = y - 2 * a.H;
    } else {
        src = a.v, ld = a.ldv, dh = vh, dl = vl, hh = y - 2 * a.H - a.Hkv;
    }
    for (int i = threadIdx.x; i < 32 * (kFD / 8); i += blockDim.x) {
        const int c8 = (i % (kFD / 8)) * 8, t = t0 + i / (kFD / 8);
        if (t >= a.T) break;
        float x[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = c8 + e < hd ? src[(int64_t)t * ld + hh * hd + c8 + e] : 0.0f;
        store8_split(dh, dl, ((int64_t)hh * a.T + t) * kFD + c8, x);
    }
}

// dsum[h][t] = dy_t,h . out_t,h: one warp per (t, h), a fixed lane tree
__global__ void k_flash_dsum(FlashBwdArgs a, float *dsum) {
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= (int64_t)a.T * a.H) return;
    const int t = (int)(w / a.H), h = (int)(w % a.H);
    float s = 0.0f;
    for (int c = lane; c < a.hd; c += 32)
        s = __fmaf_rn(a.dout[(int64_t)t * a.lddo + h * a.hd + c], a.out[(int64_t)t * a.ldo + h * a.hd + c], s);
    s = warp_sum(s);
    if (lane == 0) dsum[(int64_t)h * a.T + t] = s;
}

template <int KV>
struct BwdCfg {
    static constexpr int CN = KV ? 64 : 128;     // columns per tile (queries, or keys)
    static constexpr int RT = 128 * 128;         // one row plane tile: 128 rows x 128 bytes
    static constexpr int CT = CN * 128;          // one column plane tile
    static constexpr int NST = KV ? 2 : 1;       // column stages
    static constexpr int Stage = 4 * CT;         // C1 hi, C1 lo, C2 hi, C2 lo
    static constexpr int PPlane = 128 * CN * 2;  // one P or dS plane
    static constexpr int NP = KV ? 4 : 2;        // (P hi, P lo,) dS hi, dS lo
    static constexpr int Smem = 4 * RT + NST * Stage + NP * PPlane + 1024;
    static constexpr int NBUF = KV ? 2 : 1;      // X / Y buffers in tensor memory
    static constexpr int XY = 2 * CN;            // columns of one X / Y buffer
    static constexpr int ACC = NBUF * XY;        // first accumulator column
    static_assert(Smem + 256 <= 227 * 1024, "shared memory");
    static_assert(ACC + (KV ? 2 : 1) * kFD <= 512, "tensor memory");
};

// kind::f16, M = 128, N = 64, A K-major, B MN-major
constexpr uint32_t kIdescAccMN = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(kFD >> 3) << 17) |
                                 ((uint32_t)(kFM >> 4) << 24);

template <int KV>
__global__ void __launch_bounds__(320, 1)
    k_flash_bwd(const __grid_constant__ CUtensorMap r1_hi, const __grid_constant__ CUtensorMap r1_lo,
                const __grid_constant__ CUtensorMap r2_hi, const __grid_constant__ CUtensorMap r2_lo,
                const __grid_constant__ CUtensorMap c1_hi, const __grid_constant__ CUtensorMap c1_lo,
                const __grid_constant__ CUtensorMap c2_hi, const __grid_constant__ CUtensorMap c2_lo, FlashBwdArgs a,
                const float *dsum) {
    using Cf = BwdCfg<KV>;
    constexpr int CN = Cf::CN, NST = Cf::NST, NBUF = Cf::NBUF;
    extern __shared__ unsigned char fb_smem_raw[];
    __shared__ __align__(8) uint64_t r_full, c_full[2], c_empty[2], xy_full[2], pd_full, pd_empty, acc_full, drainb;
    __shared__ uint32_t tmem_sh;
    __shared__ volatile int abort_sh;
    const uint32_t raw_s = smem_u32(fb_smem_raw);
    unsigned char *sm = fb_smem_raw + ((1024u - (raw_s & 1023u)) & 1023u);
    const uint32_t sr = smem_u32(sm), sc = sr + 4 * Cf::RT, spd = sc + NST * Cf::Stage;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = a.H / a.Hkv;
    const int r0 = blockIdx.x * 128, hr = blockIdx.y;  // rows: queries of head hr, or keys of kv head hr
    const int cfirst = KV ? r0 / CN : 0;
    const int ncol = KV ? (a.T + CN - 1) / CN - cfirst : (min(a.T, r0 + 128) - 1) / CN + 1;
    const int steps = KV ? G * ncol : ncol;
    if (threadIdx.x == 0) {
        mbar_init(&r_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&c_full[s], 1);
            mbar_init(&c_empty[s], 1);
            mbar_init(&xy_full[s], 1);
        }
        mbar_init(&pd_full, 8);  // one arrival per compute warp
        mbar_init(&pd_empty, 1);
        mbar_init(&acc_full, 1);
        mbar_init(&drainb, 1);
        abort_sh = 0;
        fence_mbar_init();
    }
    if (warp == 9) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_sh)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_sh;
    // column tile of step t: first column and the head it belongs to
    auto col_of = [&](int t, int &col0, int &ch) {
        if (KV) {
            col0 = (cfirst + t % ncol) * CN;
            ch = hr * G + t / ncol;
        } else {
            col0 = t * CN;
            ch = hr / G;
        }
    };

    if (warp == 8) {
        if (lane == 0) {
            mbar_expect_tx(&r_full, 4 * Cf::RT);
            tma_load_3d(sm, &r1_hi, 0, r0, hr, &r_full);
            tma_load_3d(sm + Cf::RT, &r1_lo, 0, r0, hr, &r_full);
            tma_load_3d(sm + 2 * Cf::RT, &r2_hi, 0, r0, hr, &r_full);
            tma_load_3d(sm + 3 * Cf::RT, &r2_lo, 0, r0, hr, &r_full);
            int t = 0;
            for (; t < steps && !abort_sh; ++t) {
                const int s = t % NST;
                if (t >= NST && !mbar_wait_bounded(&c_empty[s], ((t - NST) / NST) & 1, wait_limit())) {
                    abort_sh = 1;
                    break;
                }
                int col0, ch;
                col_of(t, col0, ch);
                unsigned char *st = sm + 4 * Cf::RT + s * Cf::Stage;
                mbar_expect_tx(&c_full[s], Cf::Stage);
                tma_load_3d(st, &c1_hi, 0, col0, ch, &c_full[s]);
                tma_load_3d(st + Cf::CT, &c1_lo, 0, col0, ch, &c_full[s]);
                tma_load_3d(st + 2 * Cf::CT, &c2_hi, 0, col0, ch, &c_full[s]);
                tma_load_3d(st + 3 * Cf::CT, &c2_lo, 0, col0, ch, &c_full[s]);
            }
            if (abort_sh) {  // let the copies in flight land before the CTA can exit
                mbar_wait_bounded(&r_full, 0, kWaitLimit);
                for (int p = t - NST > 0 ? t - NST : 0; p < t; ++p)
                    mbar_wait_bounded(&c_full[p % NST], (p / NST) & 1, kWaitLimit);
            }
        }
    } else if (warp == 9) {
        if (lane == 0) {
            bool ok = mbar_wait_bounded(&r_full, 0, wait_limit());
            // the accumulators' products of step u: dS C1 (and P C2), C read MN-major
            auto acc_step = [&](int u) -> bool {
                if (!mbar_wait_bounded(&pd_full, u & 1, wait_limit())) return false;
                tc_fence_after();
                const uint32_t cb = sc + (u % NST) * Cf::Stage;
                const uint32_t ds = spd + (KV ? 2 : 0) * Cf::PPlane;
#pragma unroll
                for (int kk = 0; kk < CN / 16; ++kk) {
                    const uint32_t ao = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
                    const uint64_t dh = sw128_desc(ds + ao, 16), dl = sw128_desc(ds + Cf::PPlane + ao, 16);
                    const uint64_t c1h = sw128_desc(cb + kk * 2048, 8192), c1l = sw128_desc(cb + Cf::CT + kk * 2048, 8192);
                    const uint32_t acc = !(u == 0 && kk == 0);
                    tc_mma(tmem + Cf::ACC, dh, c1h, kIdescAccMN, acc);
                    tc_mma(tmem + Cf::ACC, dh, c1l, kIdescAccMN, 1u);
                    tc_mma(tmem + Cf::ACC, dl, c1h, kIdescAccMN, 1u);
                    if (KV) {
                        const uint64_t ph = sw128_desc(spd + ao, 16), pl = sw128_desc(spd + Cf::PPlane + ao, 16);
                        const uint64_t c2h = sw128_desc(cb + 2 * Cf::CT + kk * 2048, 8192);
                        const uint64_t c2l = sw128_desc(cb + 3 * Cf::CT + kk * 2048, 8192);
                        tc_mma(tmem + Cf::ACC + kFD, ph, c2h, kIdescAccMN, acc);
                        tc_mma(tmem + Cf::ACC + kFD, ph, c2l, kIdescAccMN, 1u);
                        tc_mma(tmem + Cf::ACC + kFD, pl, c2h, kIdescAccMN, 1u);
                    }
                }
                tc_commit(&c_empty[u % NST]);
                tc_commit(&pd_empty);
                return true;
            };
            for (int t = 0; t <= steps && ok && !abort_sh; ++t) {
                if (NBUF == 1 && t >= 1 && !(ok = acc_step(t - 1))) break;
                if (t < steps) {  // X = R1 C1^T, Y = R2 C2^T into buffer t % NBUF
                    const int s = t % NST, b = t % NBUF;
                    if (!mbar_wait_bounded(&c_full[s], (t / NST) & 1, wait_limit())) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t cb = sc + s * Cf::Stage;
#pragma unroll
                    for (int kk = 0; kk < kFD / 16; ++kk) {
                        const uint32_t o = kk * 32;
                        const uint64_t r1h = sw128_desc(sr + o, 16), r1l = sw128_desc(sr + Cf::RT + o, 16);
                        const uint64_t r2h = sw128_desc(sr + 2 * Cf::RT + o, 16), r2l = sw128_desc(sr + 3 * Cf::RT + o, 16);
                        const uint64_t c1h = sw128_desc(cb + o, 16), c1l = sw128_desc(cb + Cf::CT + o, 16);
                        const uint64_t c2h = sw128_desc(cb + 2 * Cf::CT + o, 16), c2l = sw128_desc(cb + 3 * Cf::CT + o, 16);
                        const uint32_t dx = tmem + b * Cf::XY, dy = dx + CN;
                        tc_mma(dx, r1h, c1h, idesc_kmajor<CN>(), kk != 0);
                        tc_mma(dx, r1h, c1l, idesc_kmajor<CN>(), 1u);
                        tc_mma(dx, r1l, c1h, idesc_kmajor<CN>(), 1u);
                        tc_mma(dy, r2h, c2h, idesc_kmajor<CN>(), kk != 0);
                        tc_mma(dy, r2h, c2l, idesc_kmajor<CN>(), 1u);
                        tc_mma(dy, r2l, c2h, idesc_kmajor<CN>(), 1u);
                    }
                    tc_commit(&xy_full[b]);
                }
                if (NBUF == 2 && t >= 1 && !(ok = acc_step(t - 1))) break;
            }
            if (ok) tc_commit(&acc_full);
            else abort_sh = 1;
            tc_commit(&drainb);
            mbar_wait_bounded(&drainb, 0, kWaitLimit);
        }
    } else {
        // compute warps 0-7: rows 32 (w % 4) .. (tensor-memory lanes), columns
        // [(w / 4) CN / 2, +CN / 2) of each tile
        const int quarter = warp & 3, half = warp >> 2;
        const int r = quarter * 32 + lane, row = r0 + r;
        const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
        const float c2 = __fmul_rn(a.scale, 1.4426950408889634f);  // log2(e)
        const int rq = min(row, a.T - 1);
        const float lse_r = KV ? 0.0f : a.lse[(int64_t)hr * a.T + rq];
        const float d_r = KV ? 0.0f : dsum[(int64_t)hr * a.T + rq];
        bool ok = true;
        for (int t = 0; t < steps; ++t) {
            const int b = t % NBUF;
            ok = __all_sync(kAll, ok && !abort_sh && mbar_wait_bounded(&xy_full[b], (t / NBUF) & 1, wait_limit()));
            if (!ok) break;
            if (t >= 1) {  // the previous step's products have read the P / dS planes
                ok = __all_sync(kAll, mbar_wait_bounded(&pd_empty, (t - 1) & 1, wait_limit()));
                if (!ok) break;
            }
            tc_fence_after();
            int col0, ch;
            col_of(t, col0, ch);
            // dk / dv: the 32 columns' lse and D, one coalesced load per lane, shared by shuffle
            float lse_c = 0.0f, d_c = 0.0f;
            if (KV) {
                const int cq = col0 + half * (CN / 2) + lane;
                if (cq < a.T) {
                    lse_c = a.lse[(int64_t)ch * a.T + cq];
                    d_c = dsum[(int64_t)ch * a.T + cq];
                }
            }
#pragma unroll
            for (int c0 = 0; c0 < CN / 2; c0 += 32) {
                const int cl = half * (CN / 2) + c0;  // first local column of this block
                float xv[32], yv[32];
                tc_ld32(tmem + lanes + b * Cf::XY + cl, xv);
                tc_ld32(tmem + lanes + b * Cf::XY + CN + cl, yv);
#pragma unroll
                for (int u = 0; u < 32; ++u) {
                    const int col = col0 + cl + u;
                    float lse, dd;
                    bool in;
                    if (KV) {  // row = key, col = query of head ch (CN / 2 = 32: lane u holds column u)
                        in = col < a.T && row <= col;
                        lse = __shfl_sync(kAll, lse_c, u);
                        dd = __shfl_sync(kAll, d_c, u);
                    } else {  // row = query, col = key
                        in = col <= rq;
                        lse = lse_r;
                        dd = d_r;
                    }
                    const float p = in ? ex2(__fsub_rn(__fmul_rn(xv[u], c2), lse)) : 0.0f;
                    xv[u] = p;
                    yv[u] = __fmul_rn(__fmul_rn(p, __fsub_rn(yv[u], dd)), a.scale);
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {  // 16-byte chunks of the row, swizzled
                    const int cc = cl + 8 * k;
                    const uint32_t off = (uint32_t)((cc / 64) * (128 * 128) + r * 128 + ((((cc % 64) / 8) ^ (r & 7)) << 4));
                    uint32_t hw[4], lw[4];
#pragma unroll
                    for (int pass = 0; pass < (KV ? 2 : 1); ++pass) {
                        const float *vv = (KV && pass == 0) ? xv : yv;  // P (dk / dv kernel only), then dS
                        const uint32_t pl = spd + (KV && pass == 1 ? 2 : 0) * Cf::PPlane;
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float x0 = vv[8 * k + 2 * e], x1 = vv[8 * k + 2 * e + 1];
                            const __nv_bfloat162 hi2 = __floats2bfloat162_rn(x0, x1);
                            const float2 hf = __bfloat1622float2(hi2);
                            const __nv_bfloat162 lo2 = __floats2bfloat162_rn(__fsub_rn(x0, hf.x), __fsub_rn(x1, hf.y));
                            hw[e] = *reinterpret_cast<const uint32_t *>(&hi2);
                            lw[e] = *reinterpret_cast<const uint32_t *>(&lo2);
                        }
                        sts_v4(pl + off, hw[0], hw[1], hw[2], hw[3]);
                        sts_v4(pl + Cf::PPlane + off, lw[0], lw[1], lw[2], lw[3]);
                    }
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&pd_full);
        }
        if (ok) ok = __all_sync(kAll, !abort_sh && mbar_wait_bounded(&acc_full, 0, wait_limit()));
        if (!ok) {
            abort_sh = 1;
        } else if (half * 32 < a.hd) {  // warp-uniform: the tensor-memory loads are warp-collective
            tc_fence_after();
#pragma unroll
            for (int which = 0; which < (KV ? 2 : 1); ++which) {
                float v[32];
                tc_ld32(tmem + lanes + Cf::ACC + which * kFD + half * 32, v);
                if (row >= a.T) continue;
                float *out = KV ? (which ? a.dv + (int64_t)row * a.lddv : a.dk + (int64_t)row * a.lddk)
                                : a.dq + (int64_t)row * a.lddq;
                out += (int64_t)hr * a.hd + half * 32;
#pragma unroll
                for (int c = 0; c < 32; c += 4)
                    *reinterpret_cast<float4 *>(out + c) = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// 3-D bf16 tensor map over [nb][rows][cols] (row stride cols), box 64 x box_rows x 1, 128-byte swizzle
bool map3(CUtensorMap *m, const uint16_t *p, int64_t cols, int64_t rows, int64_t nb, int box_rows) {
    auto enc = encoder();
    if (!enc) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)nb};
    cuuint64_t strides[2] = {(cuuint64_t)(cols * 2), (cuuint64_t)(cols * rows * 2)};
    cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<uint16_t *>(p), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int HD>
int launch_hd(const FlashArgs &a, const CUtensorMap (&m)[6], cudaStream_t st) {
    static bool attr_done[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ALTXS_ECUDA;
    if (!attr_done[dev]) {
        if (cudaFuncSetAttribute(k_flash_fwd<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
            return ALTXS_ECUDA;
        attr_done[dev] = true;
    }
    const dim3 grid((a.T + kFM - 1) / kFM, a.H);
    ALTXS_LAUNCH(kKTtt, st, k_flash_fwd<HD><<<grid, 320, kSmem, st>>>(m[0], m[1], m[2], m[3], m[4], m[5], a));
    return ALTXS_OK;
}

template <int KV>
int launch_bwd_kernel(const FlashBwdArgs &a, const CUtensorMap (&m)[8], const float *dsum, cudaStream_t st) {
    static bool attr_done[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ALTXS_ECUDA;
    if (!attr_done[dev]) {
        if (cudaFuncSetAttribute(k_flash_bwd<KV>, cudaFuncAttributeMaxDynamicSharedMemorySize, BwdCfg<KV>::Smem) !=
            cudaSuccess)
            return ALTXS_ECUDA;
        attr_done[dev] = true;
    }
    const dim3 grid((a.T + 127) / 128, KV ? a.Hkv : a.H);
    ALTXS_LAUNCH(kKTtt, st,
                 k_flash_bwd<KV><<<grid, 320, BwdCfg<KV>::Smem, st>>>(m[0], m[1], m[2], m[3], m[4], m[5], m[6], m[7],
                                                                      a, dsum));
    return ALTXS_OK;
}

}  // namespace

int64_t flash_bwd_scratch_elems(int T, int H, int Hkv) {
    if (T <= 0 || H <= 0 || Hkv <= 0) return 0;
    // q, dy, k, v planes (hi and lo), then dsum [H][T] fp32
    return 4 * align_up((int64_t)H * T * kFD, 8) + 4 * align_up((int64_t)Hkv * T * kFD, 8) +
           2 * align_up((int64_t)H * T, 8);
}

int launch_flash_bwd(const FlashBwdArgs &a, cudaStream_t st) {
    if (a.T <= 0) return ALTXS_OK;
    auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!flash_ok(a.hd) || a.H <= 0 || a.Hkv <= 0 || a.H % a.Hkv || !a.q || !a.k || !a.v || !a.out || !a.dout ||
        !a.lse || !a.dq || !a.dk || !a.dv || !a.scratch || !al16(a.scratch) || !al16(a.dq) || !al16(a.dk) ||
        !al16(a.dv) || a.lddq % 4 || a.lddk % 4 || a.lddv % 4)
        return ALTXS_EINVAL;
    const int64_t nq = align_up((int64_t)a.H * a.T * kFD, 8), nk = align_up((int64_t)a.Hkv * a.T * kFD, 8);
    uint16_t *qh = a.scratch, *ql = qh + nq, *oh = ql + nq, *ol = oh + nq;
    uint16_t *kh = ol + nq, *kl = kh + nk, *vh = kl + nk, *vl = vh + nk;
    float *dsum = reinterpret_cast<float *>(vl + nk);
    ALTXS_LAUNCH(kKTtt, st,
                 k_flash_bwd_split<<<dim3((a.T + 31) / 32, 2 * a.H + 2 * a.Hkv), 256, 0, st>>>(a, qh, ql, oh, ol, kh,
                                                                                              kl, vh, vl));
    const int64_t warps = (int64_t)a.T * a.H;
    ALTXS_LAUNCH(kKTtt, st, k_flash_dsum<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(a, dsum));
    CUtensorMap kv[8], dq[8];
    // dk, dv: rows k, v (128-row boxes); columns q, dy (64-row boxes)
    if (!map3(&kv[0], kh, kFD, a.T, a.Hkv, 128) || !map3(&kv[1], kl, kFD, a.T, a.Hkv, 128) ||
        !map3(&kv[2], vh, kFD, a.T, a.Hkv, 128) || !map3(&kv[3], vl, kFD, a.T, a.Hkv, 128) ||
        !map3(&kv[4], qh, kFD, a.T, a.H, 64) || !map3(&kv[5], ql, kFD, a.T, a.H, 64) ||
        !map3(&kv[6], oh, kFD, a.T, a.H, 64) || !map3(&kv[7], ol, kFD, a.T, a.H, 64))
        return ALTXS_EINVAL;
    // dq: rows q, dy; columns k, v (128-row boxes)
    if (!map3(&dq[0], qh, kFD, a.T, a.H, 128) || !map3(&dq[1], ql, kFD, a.T, a.H, 128) ||
        !map3(&dq[2], oh, kFD, a.T, a.H, 128) || !map3(&dq[3], ol, kFD, a.T, a.H, 128))
        return ALTXS_EINVAL;
    for (int i = 0; i < 4; ++i) dq[4 + i] = kv[i];
    int rc = launch_bwd_kernel<1>(a, kv, dsum, st);
    if (rc != ALTXS_OK) return rc;
    return launch_bwd_kernel<0>(a, dq, dsum, st);
}

int set_wait_limit_flash(uint32_t limit) {
    return cudaMemcpyToSymbol(g_wait_limit, &limit, sizeof(limit)) == cudaSuccess ? ALTXS_OK : ALTXS_ECUDA;
}

int64_t flash_scratch_elems(int T, int H, int Hkv, int hd) {
    if (T <= 0 || H <= 0 || Hkv <= 0 || hd <= 0) return 0;
    const int64_t tp = align_up((int64_t)T, 8);
    // Q, K and V^T planes (hi and lo), each part 16-byte aligned
    return 2 * (align_up((int64_t)H * T * kFD, 8) + align_up((int64_t)Hkv * T * kFD, 8) + (int64_t)Hkv * hd * tp);
}

int launch_flash_fwd(const FlashArgs &a, cudaStream_t st) {
    if (a.T <= 0) return ALTXS_OK;
    if (!flash_ok(a.hd) || a.H <= 0 || a.Hkv <= 0 || a.H % a.Hkv || !a.q || !a.k || !a.v || !a.y || !a.scratch ||
        (reinterpret_cast<uintptr_t>(a.scratch) & 15) || (reinterpret_cast<uintptr_t>(a.y) & 15) || a.ldy % 4)
        return ALTXS_EINVAL;
    const int64_t tp = align_up((int64_t)a.T, 8);
    const int64_t nq = align_up((int64_t)a.H * a.T * kFD, 8), nk = align_up((int64_t)a.Hkv * a.T * kFD, 8);
    const int64_t nv = (int64_t)a.Hkv * a.hd * tp;
    uint16_t *qh = a.scratch, *ql = qh + nq, *kh = ql + nq, *kl = kh + nk, *vh = kl + nk, *vl = vh + nv;
    ALTXS_LAUNCH(kKTtt, st,
                 k_flash_split<<<dim3((a.T + 31) / 32, a.H + 2 * a.Hkv), 256, 0, st>>>(a, tp, qh, ql, kh, kl, vh, vl));
    CUtensorMap m[6];
    if (!map3(&m[0], qh, kFD, a.T, a.H, kFM) || !map3(&m[1], ql, kFD, a.T, a.H, kFM) ||
        !map3(&m[2], kh, kFD, a.T, a.Hkv, kFN) || !map3(&m[3], kl, kFD, a.T, a.Hkv, kFN) ||
        !map3(&m[4], vh, tp, a.hd, a.Hkv, a.hd) || !map3(&m[5], vl, tp, a.hd, a.Hkv, a.hd))
        return ALTXS_EINVAL;
    return a.hd == 32 ? launch_hd<32>(a, m, st) : launch_hd<64>(a, m, st);
}

}  // namespace altxs

extern "C" {

int64_t altxs_window_attention_workspace_bytes(int T, int H, int Hkv, int hd) {
    if (T < 0 || H <= 0 || Hkv <= 0 || hd <= 0) return -1;
    return altxs::flash_scratch_elems(T, H, Hkv, hd) * 2;
}

int altxs_window_attention(int T, int H, int Hkv, int hd, float scale, const float *q, int64_t ldq, const float *k,
                           int64_t ldk, const float *v, int64_t ldv, float *y, int64_t ldy, float *lse,
                           void *workspace, int64_t workspace_bytes, altxs_stream_t stream) {
    using namespace altxs;
    if (T < 0 || H <= 0 || Hkv <= 0 || H % Hkv || ldq < (int64_t)H * hd || ldk < (int64_t)Hkv * hd ||
        ldv < (int64_t)Hkv * hd || ldy < (int64_t)H * hd)
        return ALTXS_EINVAL;
    if (!flash_ok(hd)) return ALTXS_ENOTSUP;
    if (T == 0) return ALTXS_OK;
    if (!workspace || workspace_bytes < altxs_window_attention_workspace_bytes(T, H, Hkv, hd)) return ALTXS_EINVAL;
    FlashArgs a{};
    a.T = T;
    a.H = H;
    a.Hkv = Hkv;
    a.hd = hd;
    a.scale = scale;
    a.q = q;
    a.k = k;
    a.v = v;
    a.ldq = ldq;
    a.ldk = ldk;
    a.ldv = ldv;
    a.y = y;
    a.ldy = ldy;
    a.lse = lse;
    a.scratch = static_cast<uint16_t *>(workspace);
    return launch_flash_fwd(a, reinterpret_cast<cudaStream_t>(stream));
}

int64_t altxs_window_attention_backward_workspace_bytes(int T, int H, int Hkv, int hd) {
    if (T < 0 || H <= 0 || Hkv <= 0 || hd <= 0) return -1;
    return altxs::flash_bwd_scratch_elems(T, H, Hkv) * 2;
}

int altxs_window_attention_backward(int T, int H, int Hkv, int hd, float scale, const float *q, int64_t ldq,
                                    const float *k, int64_t ldk, const float *v, int64_t ldv, const float *y,
                                    int64_t ldy, const float *lse, const float *dy, int64_t lddy, float *dq,
                                    int64_t lddq, float *dk, int64_t lddk, float *dv, int64_t lddv, void *workspace,
                                    int64_t workspace_bytes, altxs_stream_t stream) {
    using namespace altxs;
    if (T < 0 || H <= 0 || Hkv <= 0 || H % Hkv || ldq < (int64_t)H * hd || ldk < (int64_t)Hkv * hd ||
        ldv < (int64_t)Hkv * hd || ldy < (int64_t)H * hd || lddy < (int64_t)H * hd || lddq < (int64_t)H * hd ||
        lddk < (int64_t)Hkv * hd || lddv < (int64_t)Hkv * hd)
        return ALTXS_EINVAL;
    if (!flash_ok(hd)) return ALTXS_ENOTSUP;
    if (T == 0) return ALTXS_OK;
    if (!workspace || workspace_bytes < altxs_window_attention_backward_workspace_bytes(T, H, Hkv, hd))
        return ALTXS_EINVAL;
    FlashBwdArgs a{};
    a.T = T;
    a.H = H;
    a.Hkv = Hkv;
    a.hd = hd;
    a.scale = scale;
    a.q = q;
    a.k = k;
    a.v = v;
    a.out = y;
    a.dout = dy;
    a.lse = lse;
    a.ldq = ldq;
    a.ldk = ldk;
    a.ldv = ldv;
    a.ldo = ldy;
    a.lddo = lddy;
    a.dq = dq;
    a.dk = dk;
    a.dv = dv;
    a.lddq = lddq;
    a.lddk = lddk;
    a.lddv = lddv;
    a.scratch = static_cast<uint16_t *>(workspace);
    return launch_flash_bwd(a, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
