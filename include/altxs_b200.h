/*
 * altxs_b200 -- C ABI of the B200 model-and-code loop.
 *
 * Plain pointers and sizes only.  Every pointer marked "device" is CUDA
 * device memory owned by the caller; the library never allocates, never
 * synchronises the stream (except where stated) and enqueues all work on the
 * stream it is given (a cudaStream_t passed as void*, NULL = legacy default
 * stream).  Return values: 0 on success, a negative errno-style code
 * otherwise.  Device-side faults of the data (bit buffer full, symbol out of
 * range, bad CDF total, non-finite logits, bounded wait expired) are recorded
 * in the per-stream status word of altxs_ac_state and never trap the GPU.
 *
 * Bit buffers hold the reference's byte stream: stream s owns
 * words_per_stream uint32 words at bits + s*words_per_stream and byte k of
 * that region (little-endian word order) is byte k of the payload the
 * reference's _pack_bits would produce (MSB-first bits, zero padded).
 */
#ifndef ALTXS_B200_H
#define ALTXS_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ALTXS_OK 0
#define ALTXS_EINVAL (-22)
#define ALTXS_ENOSPC (-28)
#define ALTXS_ENOTSUP (-95)
#define ALTXS_ECUDA (-5)
#define ALTXS_ENOMEM (-12)
#define ALTXS_EMISMATCH (-71) /* decoder settings differ from the encoder's (altxs_set_lockstep) */

/* per-stream device status bits (altxs_ac_state.status) */
#define ALTXS_ST_OVERFLOW 1u    /* bit buffer full: further bits dropped */
#define ALTXS_ST_BAD_SYMBOL 2u  /* symbol outside [0, V) or zero mass */
#define ALTXS_ST_BAD_TOTAL 4u   /* CDF total 0 or above 2^30 */
#define ALTXS_ST_NONFINITE 8u   /* NaN/inf logits */
#define ALTXS_ST_TIMEOUT 16u    /* a bounded device wait gave up */
#define ALTXS_ST_BAD_POS 32u    /* position beyond weights->rope_positions */

/* CDF rules */
#define ALTXS_CDF_FIXED 0 /* integer fixed-point softmax, total <= 2^cdf_bits */
#define ALTXS_CDF_REF 1   /* reference masses max(1, floor(p*1e6 + 0.5)) */

/* altxs_step modes */
#define ALTXS_STEP_LOGITS 0 /* model only: logits into batch->logits_out */
#define ALTXS_STEP_ENCODE 1
#define ALTXS_STEP_DECODE 2

typedef void *altxs_stream_t;

/* Range-coder state of one stream (64 bytes). */
typedef struct altxs_ac_state {
    uint64_t low, high, pending, nbits; /* encoder */
    uint64_t value, bpos, n_in_bits;    /* decoder: value, next bit, payload bits */
    uint32_t status, reserved;
} altxs_ac_state;

/* ---- range coder ---------------------------------------------------------
 * Replaces the reference's single-stream CUDA coder module xsa_gpu_ac
 * (altxs src/xsa_ttt/gpu_ac.py:26-341): one 1-thread kernel per symbol with
 * one int64 per bit becomes one CTA per stream over many streams, 32 bits per
 * word, with error status instead of silent truncation.  `rows` (device,
 * optional) selects which streams a call touches; NULL = streams 0..n-1.
 */

/* Reset encoders (low = 0, high = 2^32 - 1, pending = nbits = status = 0).
 * Replaces GpuRangeCoder.__init__ state setup (gpu_ac.py:400-415). */
int altxs_ac_init(int n, const int32_t *rows, altxs_ac_state *st, altxs_stream_t stream);

/* Encode one symbol per stream from fp32 probabilities with the reference
 * mass rule.  probs: device [n][ld] (row i for stream rows[i]).
 * Replaces encode_sym / launch_encode_sym (gpu_ac.py:84-116, 224-230, 271-290). */
int altxs_ac_encode_probs(int n, const int32_t *rows, int vocab, const float *probs, int64_t ld,
                          const int32_t *syms, altxs_ac_state *st, uint32_t *bits,
                          int64_t words_per_stream, altxs_stream_t stream);

/* Encode with caller-supplied integer CDFs: cum device [n][ld] uint32,
 * cum[0] = 0, cum[V] = total <= 2^30.  Same coder arithmetic as
 * arithmetic_coder_lm.encode_with_probs (arithmetic_coder_lm.py:175-180). */
int altxs_ac_encode_cum(int n, const int32_t *rows, int vocab, const uint32_t *cum, int64_t ld,
                        const int32_t *syms, altxs_ac_state *st, uint32_t *bits,
                        int64_t words_per_stream, altxs_stream_t stream);

/* Final flush (pending+1, one bit and the pending run).
 * Replaces flush_bits / flush_kernel (gpu_ac.py:118-142, 292-304). */
int altxs_ac_flush(int n, const int32_t *rows, altxs_ac_state *st, uint32_t *bits,
                   int64_t words_per_stream, altxs_stream_t stream);

/* Start decoding: n_bits device [n] payload length in bits, value = first
 * 32 bits.  Replaces seed_value / begin_decode (gpu_ac.py:144-156, 448-466). */
int altxs_ac_begin_decode(int n, const int32_t *rows, altxs_ac_state *st, const uint32_t *bits,
                          const uint64_t *n_bits, int64_t words_per_stream, altxs_stream_t stream);

/* Decode one symbol per stream (reference mass rule / supplied CDFs).
 * Replaces decode_sym / decode_sym_kernel (gpu_ac.py:158-222, 306-330). */
int altxs_ac_decode_probs(int n, const int32_t *rows, int vocab, const float *probs, int64_t ld,
                          int32_t *syms_out, altxs_ac_state *st, const uint32_t *bits,
                          int64_t words_per_stream, altxs_stream_t stream);
int altxs_ac_decode_cum(int n, const int32_t *rows, int vocab, const uint32_t *cum, int64_t ld,
                        int32_t *syms_out, altxs_ac_state *st, const uint32_t *bits,
                        int64_t words_per_stream, altxs_stream_t stream);

/* Integer CDFs of softcapped logits under a framework rule (parity/debug).
 * Replaces the host rule _scale_cum_np over torch.softmax rows
 * (arithmetic_coder_lm.py:49-64, incremental.py:603-633). */
int altxs_cdf_from_logits(int n, int vocab, const float *logits, int64_t ld, int mode, int cdf_bits,
                          uint32_t *cum, int64_t cum_ld, altxs_stream_t stream);

/* ---- model ------------------------------------------------------------- */

/* One mixed-bit matrix W[rows][cols] in 64-wide groups along cols.
 * gdesc[r][g] = fp16 scale | width code << 16 (0:0 1:2 2:3 3:4 4:fp32 bits)
 *               | in-row offset in 8-byte units << 20.
 * Replaces the dense bf16 banks + F.linear of the reference step
 * (model.py:997-1011, 1183-1236; ac_gemv.py:27-60) and the host-side
 * dequantisation of the v5 codec (mixed_bit_delta.py:96-229). */
typedef struct altxs_qmat {
    const uint8_t *codes;     /* device: packed codes, 16-byte aligned */
    const uint32_t *row_off8; /* device [rows]: row start in 8-byte units */
    const uint32_t *gdesc;    /* device [rows][cols/64] */
    const uint16_t *lut;      /* device fp16 [n][16] codebooks, NULL = symmetric */
    const uint32_t *glut;     /* device [rows][cols/64] codebook index, or NULL */
    int32_t rows, cols;
} altxs_qmat;

/* The packed codes of one matrix re-laid for the tensor-core GEMM (built
 * once at load, about 0.56 bytes per weight): fixed-size segments of 2304
 * bytes, [ceil(rows/64)][cols/64], one per 64-row block and 64-wide group:
 * 64 uint32 descriptors (fp16 scale | width code << 16 (0:0 1:2 2:3 3:4 bits)
 * | offset of the row's code bytes within the segment's code area in 8-byte
 * units << 20), then the rows' code bytes (8*b each, LSB-first as in the
 * packed rows).  Rows past the matrix are 0-bit.  A tile's K slice is then
 * one bulk copy per 64 rows with no table lookups.  Only 0/2/3/4-bit
 * symmetric groups; no counterpart in the reference (its banks are dense). */
typedef struct altxs_qtiles {
    const uint8_t *data; /* device, 16-byte aligned */
    int32_t rows, cols;
} altxs_qtiles;

typedef struct altxs_tile_weights {
    altxs_qtiles emb, qkv, o, up, down;
} altxs_tile_weights;

typedef struct altxs_model_desc {
    int32_t vocab, n_layers, d_model, n_heads, n_kv_heads, head_dim, mlp_hidden;
    int32_t ctx;        /* sliding window (reference block_size) */
    int32_t rope_dims;  /* partial RoPE width */
    int32_t skip_gates; /* sigmoid-gated U-Net skips */
    int32_t lora_rank;  /* 0 = no adapters */
    int32_t lora_mask;  /* bit0 q, bit1 k, bit2 v, bit3 o, bit4 lm_head, bit5 MLP (d -> d on the
                           MLP's normed input, added to the MLP output), bit6 the o adapter
                           reads the attention output y instead of the block's normed input */
    int32_t cdf_mode, cdf_bits;
    float logit_softcap, lora_scale;
    /* Reference motifs (altxs src/xsa_ttt/model.py:760-768, 845-862, 1064-1077,
     * 1293-1362, 1404-1500); all zero = the plain GPT.  The step, the
     * updates (altxs_ttt_update, altxs_full_loss_grad) and the context
     * prefill (altxs_prefill) compute them. */
    int32_t n_virtual;          /* layer applications (depth loops repeat layers); 0 = n_layers */
    int32_t n_encoder;          /* encoder applications (the U-Net skips' sources); 0 = n_virtual/2 */
    const int32_t *schedule;    /* host [n_virtual]: physical layer of each application, or NULL */
    int32_t smear_gate;         /* raw embedding += lambda*sigmoid(g . raw[:gate_window]) * previous raw */
    int32_t gate_window;
    int32_t xsa_last_n;         /* on the last n physical layers: y_h -= (y_h . v^) v^, v^ = v/|v| */
    int32_t sparse_gate;        /* y_h *= sigmoid(sparse_gate_scale * w_h . n[:gate_window]) */
    float sparse_gate_scale;
    int32_t asym_softcap;       /* logits: sp*tanh(l/sp) for l >= 0, sn*tanh(l/sn) below */
    int32_t parallel_start;     /* decoder applications of layers >= this run two lanes; 0 = off */
    int32_t parallel_final;     /* final hidden: 0 mean of the lanes, 1 attention lane, 2 MLP lane */
} altxs_model_desc;

/* Tensor-core operand form of the five mixed-bit matrices: every dequantised
 * weight w = level*scale as two bf16 planes hi = bf16(w), lo = bf16(w - hi)
 * ([rows][cols], row stride cols), filled once by altxs_split_weights.
 * hi + lo == w exactly for the 2/3/4-bit symmetric levels.  No counterpart
 * in the reference, which multiplies dequantised fp32/bf16 tensors. */
typedef struct altxs_split_planes {
    const uint16_t *emb_hi, *emb_lo;
    const uint16_t *qkv_hi, *qkv_lo;
    const uint16_t *o_hi, *o_lo;
    const uint16_t *up_hi, *up_lo;
    const uint16_t *down_hi, *down_lo;
} altxs_split_planes;

typedef struct altxs_weights {
    altxs_qmat emb;  /* [V][d], tied LM head */
    altxs_qmat qkv;  /* [L*(d+2*kv)][d]: per layer q rows, k rows, v rows */
    altxs_qmat o;    /* [L*d][d] */
    altxs_qmat up;   /* [L*F][d] */
    altxs_qmat down; /* [L*d][F] */
    const float *q_gain;       /* [L][H] */
    const float *attn_scale;   /* [L][d] */
    const float *mlp_scale;    /* [L][d] */
    const float *resid_mix;    /* [L][2][d] */
    const float *ln_scale;     /* [L] (1/sqrt(i+1) or 1) */
    const float *skip_weights; /* [L/2][d] */
    const float *skip_gates;   /* [L/2][d] */
    const float *rope_cos;     /* [rope_positions][rope_dims/2] */
    const float *rope_sin;
    int64_t rope_positions;
    /* NULL: the step's linear layers run on CUDA cores in exact fp32 order
     * (sum over 64-wide groups of scale * sum of level*x).  Non-NULL: they run
     * on the tensor cores (products within 2^-16 relative), expanding the
     * packed codes of the five matrices in the GEMM's producer warps; the
     * planes themselves are read only with planes_live (below) and by the
     * test-time updates.  Either way results do not depend on the batch; an
     * encoder and its decoder must make the same choice. */
    const altxs_split_planes *split;
    /* motif parameters (device; NULL when the motif is off) */
    const float *smear_gate;     /* [gate_window] */
    const float *smear_lambda;   /* [1] */
    const float *attn_gate_w;    /* [L][H][gate_window] */
    const float *softcap;        /* [2]: positive, negative */
    const float *parallel_post;  /* [L][2][2]: (attention, MLP) output into (lane 0, lane 1) */
    const float *parallel_resid; /* [L][2]: lane 0, lane 1 residual scales */
    /* dense fp32 embedding [V][d] for the step's input rows, or NULL (rows from
     * the emb codes).  A model whose weights change (full-parameter replenish)
     * points it at its parameter arena and refreshes split with altxs_split_params. */
    const float *emb_dense;
    /* 1: the tensor-core linears read the split planes instead of the packed
     * codes, because the planes hold weights updated after loading (a
     * full-parameter model's arena, re-split by altxs_split_params); 0: the
     * planes equal the codes and the codes are read (0.43 instead of 4 bytes
     * per weight). */
    int32_t planes_live;
    /* The five matrices in the tile-stream layout for the packed tensor-core
     * linears (altxs_set_linear_packed), or NULL (planes). */
    const altxs_tile_weights *tiles;
} altxs_weights;

/* Per-stream state and scratch of a batch of n streams.  Stream i of the
 * batch lives in slot i of every per-stream array. */
typedef struct altxs_batch {
    int32_t n_streams;
    int32_t *tok;           /* [n] token consumed this step (<0: none, uniform row) */
    int64_t *pos;           /* [n] position tok is written at (tokens consumed) */
    const uint8_t *active;  /* [n] 0 = leave the stream untouched (NULL = all) */
    uint8_t *kv;            /* [n][n_virtual][2 (K,V)][Hkv][ctx][3*hd] sliding-window ring, rows in
                               24-bit split format: hd x u16 (bf16 high half of the
                               round-to-nearest 24-bit value) then hd x u8 (low byte) */
    float *lora;            /* [n][lora_floats] adapters (NULL if lora_rank = 0) */
    int64_t lora_stride;    /* floats per stream */
    altxs_ac_state *ac;     /* [n] */
    uint32_t *bits;         /* [n][words_per_stream] */
    int64_t words_per_stream;
    int32_t *sym;           /* [n] encode: input symbols; decode: output */
    int32_t *hist;          /* [n][hist_len] coded-symbol ring (TTT windows) or NULL */
    int32_t hist_len;
    float *logits_out;      /* [n][V] final logits copy, or NULL */
    void *workspace;        /* >= altxs_workspace_bytes(desc, n) bytes, 256-aligned */
    int64_t workspace_bytes;
    const int64_t *pos_base; /* [n] absolute index of position 0 for the hist ring, or NULL
                                (= 0).  Segment-reset context (positions restart at every
                                segment) keeps hist in absolute symbol order with it. */
    int32_t *prev_tok;       /* [n] token consumed by the previous step (-1: none), read by
                                the smear gate and advanced with pos by the encode and
                                decode modes; NULL when the gate is off */
} altxs_batch;

/* Allocation-free altxs_step for callers that cannot allocate device memory
 * (a host framework that owns the device budget through its own allocator
 * and refuses allocations from plugins, or a latency-critical caller that
 * must not risk the device-wide synchronisation an allocation may imply).
 * No counterpart in the reference.  Same arguments and results as
 * altxs_step, but b->workspace / b->workspace_bytes are ignored: the scratch
 * is a fixed 16 MiB array inside the library's device image (held on every
 * GPU that loads the library until exit; altxs_step_noalloc_max_bytes()).
 * Batches whose scratch would exceed it return ALTXS_ENOSPC (at the 33M
 * shapes, 125 streams fit).  The first call on a device resolves the
 * array's device address with that device current; make that first call
 * before any stream capture.  The address is kept for the life of the
 * process, so do not call this entry point again on a device after
 * cudaDeviceReset (the library's device image, and with it the array, is
 * reloaded at a new address).  All calls share the array: calls that overlap
 * on one GPU race, so issue them one after another.  Nothing in the scratch
 * needs to start at zero. */
int altxs_step_noalloc(const altxs_model_desc *desc, const altxs_weights *w, const altxs_batch *b, int mode,
                       altxs_stream_t stream);
int64_t altxs_step_noalloc_max_bytes(void);

/* Workspace needed by altxs_step for n streams (bytes). */
int64_t altxs_workspace_bytes(const altxs_model_desc *desc, int n_streams);

/* Floats per stream in the LoRA arena: adapters in the reference
 * TTTLoRA.parameters() order lm(A,B), q_s(A,B).., v_s.., k_s.., mlp_s.., o_s..
 * over the slots s = 0..n_virtual-1, one per layer application
 * (ttt_lora.py:67-105), A [r][in] then B [out][r]. */
int64_t altxs_lora_floats(const altxs_model_desc *desc);

/* One symbol step for every active stream: embed tok, run the L-layer GPT
 * step over the sliding KV window (writing tok's K/V at pos), tied logits with
 * tanh softcap, integer CDF, then range-code sym (encode) or decode it
 * (decode).  Afterwards tok = coded symbol and pos advances if a token was
 * consumed.  Replaces one W=1 window step plus coder call of the reference
 * engine (incremental.py:1083-1130 run_decode_row_dev + gpu_ac decode_sym,
 * and the encode-side run_window + encode_sym, :1268-1290). */
int altxs_step(const altxs_model_desc *desc, const altxs_weights *w, const altxs_batch *b, int mode,
               altxs_stream_t stream);

/* ---- test-time LoRA update ------------------------------------------------ */

typedef struct altxs_ttt_hparams {
    float lr, beta1, beta2, eps, weight_decay, grad_clip;
} altxs_ttt_hparams;

/* Optional dense fp32 copies of the frozen base (same row layout as the
 * altxs_qmat views), built once with altxs_dequant; the update's linear
 * layers then run as plain fp32 GEMMs instead of re-dequantising per tile. */
typedef struct altxs_dense_weights {
    const float *emb, *qkv, *o, *up, *down;
} altxs_dense_weights;

/* out[r][c] = exact fp32 value of m[r][c] (row stride ld floats). */
int altxs_dequant(const altxs_qmat *m, float *out, int64_t ld, altxs_stream_t stream);

/* hi/lo bf16 planes [m->rows][m->cols] of a mixed-bit matrix (see
 * altxs_split_planes); both 16-byte aligned. */
int altxs_split_weights(const altxs_qmat *m, uint16_t *hi, uint16_t *lo, altxs_stream_t stream);

/* Batched fp32 GEMM on the tensor cores (hi/lo bf16 planes, fp32
 * accumulate; products within 2^-16 relative):
 *   C[b] = alpha * op(A[b]) op(B[b]) + beta * C[b],  b < batch,
 * op(A) M x K: A stored [M][lda] (tA = 0) or [K][lda] (tA = 1), batch stride sA;
 * op(B) K x N: B stored [K][ldb] (tB = 0) or [N][ldb] (tB = 1), batch stride sB;
 * C [M][ldc], batch stride sC.  causal: 0 all of C; 1 output tiles wholly
 * above the diagonal (n > m) may be left unwritten; 2 op(A) is zero for
 * k > m; 3 op(A) is zero for k < m.  These are the products of the
 * test-time update's forward and backward (the reference's torch matmuls in
 * ttt_lora.py and the training attention, train_attn.py:578). */
int64_t altxs_gemm_workspace_bytes(int M, int N, int K, int tA, int tB, int batch);
int altxs_gemm(int M, int N, int K, const float *A, int64_t lda, int64_t sA, int tA, const float *B, int64_t ldb,
               int64_t sB, int tB, float *C, int64_t ldc, int64_t sC, int batch, float alpha, float beta, int causal,
               void *workspace, int64_t workspace_bytes, altxs_stream_t stream);

/* One linear layer, Y[i][j] = sum_k X[i][k] * m[row0 + j][k] for i < M,
 * j < N (X row stride m->cols, Y row stride N): the reference's
 * F.linear on the dequantised weight (altxs src/xsa_ttt/model.py:123-127,
 * CastedLinear.forward).  With w_hi/w_lo (planes
 * of m from altxs_split_weights) it runs on the tensor cores and needs
 * altxs_linear_workspace_bytes(M, m->cols) of device workspace; without, on
 * CUDA cores (workspace unused). */
int64_t altxs_linear_workspace_bytes(int M, int K);
int altxs_linear(const altxs_qmat *m, const uint16_t *w_hi, const uint16_t *w_lo, int row0, int N, const float *X,
                 int M, float *Y, void *workspace, int64_t workspace_bytes, altxs_stream_t stream);

/* The layer on the tensor cores with the weights read as packed 2/3/4-bit
 * codes and fp16 group scales (the reference's mixed-bit GEMV/GEMM, altxs
 * src/xsa_ttt/ac_gemv.py:27 _gemv_row_tiles, on the format of
 * src/hyperflow_distillation/mixed_bit_delta.py:96-229): the GEMM's own
 * producer warps expand each 64-wide group slice in shared memory into the
 * hi/lo bf16 operands (no dense copy of the weights is read), so the result
 * is bit-identical to altxs_linear with the planes.  The decode step takes
 * this path under altxs_set_linear_packed(1).  row0 a multiple of 64.  Needs
 * altxs_linear_tc_workspace_bytes(M, N, w->cols) of device workspace. */
int64_t altxs_linear_tc_workspace_bytes(int M, int N, int K);
int altxs_linear_tc(const altxs_qtiles *w, int row0, int N, const float *X, int M, float *Y, void *workspace,
                    int64_t workspace_bytes, altxs_stream_t stream);

/* Causal attention over a window on the tensor cores (the flash kernel of the
 * context prefill and the full-parameter forward; the reference's
 * F.scaled_dot_product_attention(q, k, v, is_causal=True) inside
 * CausalSelfAttention.forward, altxs src/xsa_ttt/model.py, and its training
 * attention train_attn.py:67 _train_attn_fwd):
 *   y[t][h*hd + c] = sum_{s <= t} softmax_s(scale * q_t,h . k_s,g) v_s,g[c],
 * g = h / (H / Hkv); q [T][ldq], k [T][ldk], v [T][ldv], y [T][ldy] fp32
 * (ldy a multiple of 4, y 16-byte aligned).  hd 32 or 64 (else
 * ALTXS_ENOTSUP).  Products as hi/lo bf16 planes with fp32 accumulation, an
 * online softmax per 128-key tile; no T x T buffer. */
int64_t altxs_window_attention_workspace_bytes(int T, int H, int Hkv, int hd);
/* lse: optional [H][T] output (NULL to skip), each row's log2 of its softmax
 * sum of 2^(scale * log2(e) * q . k), the input of the backward. */
int altxs_window_attention(int T, int H, int Hkv, int hd, float scale, const float *q, int64_t ldq, const float *k,
                           int64_t ldk, const float *v, int64_t ldv, float *y, int64_t ldy, float *lse,
                           void *workspace, int64_t workspace_bytes, altxs_stream_t stream);

/* Gradient of altxs_window_attention (the backward of the reference's
 * training attention, train_attn.py:578 triton_causal_sdpa / autograd of
 * F.scaled_dot_product_attention): dq, dk, dv from dy (= d y), y and lse of
 * the forward, in the same layouts (dk and dv sum over the query heads of
 * each group).  dq, dk, dv 16-byte aligned with row strides a multiple of 4.
 * Flash-style on the tensor cores (no T x T buffer); every sum in a fixed
 * order, so equal inputs give equal bits. */
int64_t altxs_window_attention_backward_workspace_bytes(int T, int H, int Hkv, int hd);
int altxs_window_attention_backward(int T, int H, int Hkv, int hd, float scale, const float *q, int64_t ldq,
                                    const float *k, int64_t ldk, const float *v, int64_t ldv, const float *y,
                                    int64_t ldy, const float *lse, const float *dy, int64_t lddy, float *dq,
                                    int64_t lddq, float *dk, int64_t lddk, float *dv, int64_t lddv, void *workspace,
                                    int64_t workspace_bytes, altxs_stream_t stream);

/* Segment-reset context (the reference's reset_segment, altxs
 * src/xsa_ttt/incremental.py:858-897, with _chunk_ctx_start, compress.py:122-125):
 * after a boundary update the stream's context is rebuilt from its last
 * block_size symbols at positions 0..  This writes the key and value rows of
 * tokens[0..T) at positions 0..T-1 (slots 0..T-1) of one stream's ring
 * kv ([n_virtual][2][Hkv][desc->ctx][3*hd]: one K/V set per layer
 * application), computed with the stream's adapters and the model's motifs
 * (the smear gate leaves tokens[0] alone, as at a sequence start); the caller
 * then steps the context's last token at position T with the previous token
 * tokens[T-1] for the smear gate.  lora may be NULL when desc->lora_rank is 0. */
int64_t altxs_prefill_workspace_bytes(const altxs_model_desc *desc, int T);
int altxs_prefill(const altxs_model_desc *desc, const altxs_weights *w, const altxs_dense_weights *dense,
                  const int32_t *tokens, int T, const float *lora, uint8_t *kv, void *workspace,
                  int64_t workspace_bytes, altxs_stream_t stream);

/* Workspace for one update over a T-token window (bytes). */
int64_t altxs_ttt_workspace_bytes(const altxs_model_desc *desc, int T);

/* One boundary update of one stream's adapters: teacher-forced forward over
 * tokens[0..T) (positions 0..T-1, causal), targets tokens[1..T], tied logits
 * with tanh softcap, mean cross-entropy, backward into the adapters only,
 * global-norm clip, AdamW step number `step` (1-based).  lora / adam_m /
 * adam_v: device [altxs_lora_floats] in the arena layout; loss_out: device
 * float or NULL; dense: NULL or the dense base copies.  Replaces the lora
 * branch of online_retrain (compress.py:1104-1137: ce_with_lora, backward,
 * clip_grad_norm_, AdamW step; ttt_lora.py:124-179, 258-374) on the window
 * of _window_xy (compress.py:301-320). */
int altxs_ttt_update(const altxs_model_desc *desc, const altxs_weights *w, const altxs_dense_weights *dense,
                     const altxs_ttt_hparams *hp, const int32_t *tokens, int T, float *lora, float *adam_m,
                     float *adam_v, int step, float *loss_out, void *workspace, int64_t workspace_bytes,
                     altxs_stream_t stream);

/* ---- full-parameter replenish -------------------------------------------------
 * The reference's production update trains every weight of the model
 * (online_retrain with retrain_mode "replenish", altxs src/xsa_ttt/compress.py:
 * 816-1073, and its Forward-XM boundary :611-718).  One stream's parameters
 * live in a single fp32 arena whose segments (floats from its start, each
 * 64-aligned) altxs_param_layout_of gives:
 *   emb [V][d] (the tied table), qkv [L][d+2*kvd][d] (each layer's q, k, v
 *   rows), o [L][d][d], up [L][F][d], down [L][d][F], q_gain [L][H],
 *   attn_scale [L][d], mlp_scale [L][d], resid_mix [L][2][d],
 *   skip_weights [S][d], skip_gates [S][d]   (S = min(encoder, decoder)
 *   applications), and the motif parameters of the model (empty segments when
 *   a motif is off): smear_gate [gate_window], smear_lambda [1], attn_gate_w
 *   [L][H][gate_window], softcap [2] (positive, negative), parallel_post
 *   [L][2][2], parallel_resid [L][2]
 * The gradient and the AdamW moments use the same layout.  The host keeps the
 * boundary schedule (anneal, warmup, replay draws, XM candidates and probe
 * windows), which is integer and float arithmetic of a few values. */
typedef struct altxs_param_layout {
    int64_t emb, qkv, o, up, down, q_gain, attn_scale, mlp_scale, resid_mix, skip_weights, skip_gates;
    int64_t smear_gate, smear_lambda, attn_gate_w, softcap, parallel_post, parallel_resid;
    int64_t total;
} altxs_param_layout;
int altxs_param_layout_of(const altxs_model_desc *desc, altxs_param_layout *out);

/* Workspace of one altxs_full_loss_grad call over windows of up to n tokens. */
int64_t altxs_full_workspace_bytes(const altxs_model_desc *desc, int n);

/* Teacher-forced forward over tokens[0..n-1) (positions 0.., causal) and the
 * mean cross-entropy of targets tokens[first+1..n) — the chunk loss of
 * chunk_tf_train_loss (compress.py:128-170; tokens = arr[ctx_start:chunk_end],
 * first = p0 - ctx_start - 1) and of the XM probes (_xm_probe_ce, :523-583).
 * With grad non-NULL, also d(loss)/d(every parameter) into grad
 * [layout.total] (all entries written).  The forward reads the five matrices
 * from dense (tensor cores from w->split when set) and the small parameters
 * from w; the caller points both into its parameter arena.  desc->lora_rank
 * must be 0.  The motifs of desc run in the forward and the backward as in the
 * reference's training forward (GPT._forward_hidden, model.py:1377-1476, with
 * the depth-loop schedule): the smear gate from the window's first position,
 * XSA, the sparse attention gate, parallel lanes, the asymmetric softcap; their
 * parameters get gradients like every other.  loss_out: device float or NULL. */
int altxs_full_loss_grad(const altxs_model_desc *desc, const altxs_weights *w, const altxs_dense_weights *dense,
                         const int32_t *tokens, int n, int first, float *loss_out, float *grad, void *workspace,
                         int64_t workspace_bytes, altxs_stream_t stream);

/* clip_grad_norm_(grad, hp->grad_clip) then AdamW step `step` (1-based) over
 * n floats, as torch.optim.AdamW (decoupled decay, bias corrections, eps
 * outside the square root).  partials: device scratch of >= 256 floats. */
int altxs_adamw(int64_t n, float *params, const float *grad, float *m, float *v, const altxs_ttt_hparams *hp, int step,
                float *partials, altxs_stream_t stream);

/* out[i] = a[i] + s * b[i]: ΔW = W - W0 (s = -1) and the XM candidates W0 + s ΔW. */
int altxs_params_axpy(int64_t n, const float *a, float s, const float *b, float *out, altxs_stream_t stream);

/* Anchor pull toward the first boundary's weights: p[i] -= (p[i] - w0[i]) * pull[i]
 * (_apply_replenish_anchor, compress.py:439-445; pull = mask * rate). */
int altxs_params_anchor(int64_t n, float *p, const float *w0, const float *pull, altxs_stream_t stream);

/* Rewrites the step's tensor-core planes (written through planes' pointers)
 * from the five matrices of a parameter arena. */
int altxs_split_params(const altxs_model_desc *desc, const float *params, const altxs_split_planes *planes,
                       altxs_stream_t stream);

/* ---- runtime context ----------------------------------------------------------
 * A handle over the calls above for callers that want the engine's state kept
 * for them: the reference's compress_full_sha_incremental /
 * decompress_full_sha_incremental drivers (altxs src/xsa_ttt/incremental.py:
 * 1561-1976) call create / load_weights / streams_init once, then per symbol
 * step_encode or step_decode, and at every segment boundary flush (encoder) or
 * begin_decode (decoder) around ttt_boundary (online_retrain, lora branch,
 * compress.py:1104-1137); the device coder module xsa_gpu_ac (gpu_ac.py:
 * 26-365) and StaticACEngine's state (incremental.py:203-1218) are what it
 * replaces.  All allocation happens in create, load_weights and streams_init;
 * the per-symbol and boundary calls allocate nothing and never synchronise the
 * host (get_status does).  Errors: negative return codes for arguments, device
 * errors per stream in the status words.  Not thread-safe per context. */
typedef struct altxs_ctx altxs_ctx;

/* NULL on failure (*status = error code). */
altxs_ctx *altxs_create(const altxs_model_desc *desc, int device, int *status);
/* Device views of the weights (caller-owned, kept alive by the caller); with
 * tensor_cores the context builds the hi/lo planes (4 bytes per weight),
 * without it and with adapters, dense fp32 copies for the update. */
int altxs_load_weights(altxs_ctx *ctx, const altxs_weights *view, int tensor_cores);
/* The adapters every stream starts from (device, altxs_lora_floats floats:
 * the reference's seeded initial A matrices, B = 0). */
int altxs_set_adapters(altxs_ctx *ctx, const float *d_init);
/* Hyperparameters of the boundary update (no update when never set). */
int altxs_set_ttt(altxs_ctx *ctx, const altxs_ttt_hparams *hp);
/* Symbols per segment (online_retrain_every): sizes the bit buffers. */
int altxs_set_segment(altxs_ctx *ctx, int64_t segment_symbols);
/* Allocate and reset n streams (ids unused: streams are independent). */
int altxs_streams_init(altxs_ctx *ctx, int n_streams, const uint64_t *ids);
/* One symbol per stream: d_tokens [n] device (encode input / decode output). */
int altxs_step_encode(altxs_ctx *ctx, const int32_t *d_tokens, altxs_stream_t stream);
int altxs_step_decode(altxs_ctx *ctx, int32_t *d_tokens_out, altxs_stream_t stream);
/* One AdamW step of every stream's adapters on its last window of coded symbols. */
int altxs_ttt_boundary(altxs_ctx *ctx, altxs_stream_t stream);
/* Finish the segments: d_bits [n][altxs_ctx_words_per_stream], d_nbits [n]
 * (device, segment k of stream i = the first nbits[i] bits of row i, MSB-first);
 * the coders restart for the next segment. */
int altxs_flush(altxs_ctx *ctx, uint32_t *d_bits, uint64_t *d_nbits, altxs_stream_t stream);
/* Load one segment per stream and seed the decoders.  Returns ALTXS_EMISMATCH
 * (loading nothing) when an expected lockstep id was set and differs. */
int altxs_begin_decode(altxs_ctx *ctx, const uint32_t *d_bits, const uint64_t *d_nbits, altxs_stream_t stream);
/* Lockstep identity of a context: a 64-bit hash of everything that changes
 * the coded bits (model description, layer schedule, linear path, segment
 * length, update hyper-parameters, the caller's weights_id and the library's
 * numerics version).  An encoder stores altxs_lockstep_id with its payload; a
 * decoder passes it as expect_id, and altxs_begin_decode then refuses a
 * context that would decode with other settings instead of desyncing.
 * weights_id identifies the weights (e.g. a hash of the codec file); 0 is
 * allowed.  The reference has no such check: its decoder silently desyncs
 * when a config field or environment switch differs (src/xsa_ttt/config.py:
 * 271-420). */
int altxs_set_lockstep(altxs_ctx *ctx, uint64_t weights_id, uint64_t expect_id);
int altxs_lockstep_id(altxs_ctx *ctx, uint64_t *id);
/* Waits; status (host [n] or NULL) gets each stream's status word; returns their OR. */
int altxs_get_status(altxs_ctx *ctx, int32_t *status);
int64_t altxs_ctx_words_per_stream(const altxs_ctx *ctx);
void altxs_destroy(altxs_ctx *ctx);

/* ---- failure detection ------------------------------------------------------
 * No counterpart in the reference (its device waits do not exist; its coder
 * drops bits silently).  Every device wait of this library is bounded: the
 * first wait of a pipeline stage polls at most `limit` times
 * (altxs_default_wait_limit() unless changed), then the kernel records
 * ALTXS_ST_TIMEOUT in the affected streams' status words, lets its own
 * copies and tensor-core operations finish (with the default bound) and
 * returns.  Setting the limit to 0 makes every such wait give up at once:
 * tests use it to exercise the timeout path on a real step without faulting
 * or hanging the GPU.  Applies to later launches on the current device. */
int altxs_set_wait_limit(uint32_t limit);
uint32_t altxs_default_wait_limit(void);

/* ---- fused step -------------------------------------------------------------
 * Counterpart of the reference's W=1 fused paths (persistent_step.py,
 * mega_step.py) for a few streams: on the CUDA-core path (weights->split
 * NULL) with 1 <= n_streams <= max_streams (at most 4), head_dim 32 or 64 and
 * n_heads/n_kv_heads 1 or 2, altxs_step runs the whole step as one persistent
 * cooperative kernel: the same phases and arithmetic as the launch-per-phase
 * step, so results are bit-identical, with a grid-wide barrier (bounded wait,
 * ALTXS_ST_TIMEOUT on giving up) instead of each launch.  Off by default
 * (max_streams 0): measured slower than the CUDA-graph replay of the
 * launch-per-phase step on a B200.  Process-wide. */
int altxs_set_step_fusion(int max_streams);

/* Operand source of the step's tensor-core linears: 1 = the packed codes,
 * expanded in the GEMM's producer warps; 0 (default) = the dense hi/lo bf16
 * planes.  Both feed the tensor cores the same values in the same order, so
 * the results are bit-identical; only the speed differs.  Process-wide. */
int altxs_set_linear_packed(int on);

/* Window attention of the context prefill (altxs_prefill) and of the
 * full-parameter gradient's forward (altxs_full_loss_grad) on the tensor-core
 * path: 1 (default) = the flash kernel (scores and probabilities stay in
 * tensor and shared memory; head_dim 32 or 64), 0 = the materialised T x T
 * probabilities (every head size).  The two agree to fp32 rounding, not bit
 * for bit: an encoder and its decoder use the same setting.  Replaces the
 * reference's causal attention over the window (model.py
 * CausalSelfAttention.forward, F.scaled_dot_product_attention is_causal).
 * Process-wide. */
int altxs_set_flash(int on);

/* The cudaError_t code behind the calling thread's last ALTXS_ECUDA from a
 * failed kernel launch (0 when none): a diagnostic only. */
int altxs_last_cuda_error(void);

/* ---- accounting -----------------------------------------------------------
 * No counterpart in the reference (which has no tracing); these
 * give the benchmark per-kernel device time measured live on the launch
 * stream and the number of kernels launched. */

/* Kernels launched by this library since load (monotonic). */
int64_t altxs_launch_count(void);

/* 1: reset and start recording a CUDA event pair around every launch
 * (host-side only, at most 16384 launches); 0: stop. */
int altxs_profile(int enable);

/* Synchronises the recorded events and returns, per kernel class c <
 * n_classes, the summed duration ms[c] and launch count counts[c].  Classes:
 * 0 embed, 1 prenorm, 2 mixed-bit linear, 3 qkv post, 4 attention partials,
 * 5 attention merge, 6 post-attention, 7 final norm, 8 logits->CDF->coder,
 * 9 standalone coder, 10 test-time LoRA.  Returns the number of pairs read. */
int altxs_profile_read(int n_classes, double *ms, int64_t *counts);

/* Restrict recording to the classes whose bit is set in mask (bit c = class
 * c above; default all).  A benchmark times one class live without paying for
 * event pairs around every other launch. */
int altxs_profile_mask(uint32_t mask);

/* Library build string (for logs). */
const char *altxs_version(void);

#ifdef __cplusplus
}
#endif
#endif /* ALTXS_B200_H */
