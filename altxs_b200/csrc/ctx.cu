// Handle-based runtime API over the stateless C ABI: one context per model and
// GPU holds the weight views (and the tensor-core planes or dense copies it
// builds from them), the per-stream device state of a batch of streams (KV
// rings, adapters and their AdamW moments, coder states, bit buffers, the
// symbol ring the update reads) and every workspace.  Everything is allocated
// by altxs_create / altxs_load_weights / altxs_streams_init; the per-symbol
// calls, the boundary update and the segment flush/load allocate nothing and
// do not synchronise the host (altxs_get_status does).
//
// The sequence is the reference engine's (altxs src/xsa_ttt/incremental.py
// compress_full_sha_incremental / decompress_full_sha_incremental,
// :1561-1976): streams advance together one symbol per step; at a segment
// boundary the encoder flushes its segments, re-seeds its coders and updates
// every stream's adapters on its last window (online_retrain, lora branch,
// compress.py:1104-1137 with _window_xy :301-320); the decoder updates, then
// loads the next segments.  Not thread-safe per context.
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "../../include/altxs_b200.h"

namespace {

// hist[start .. start+count) of one stream's symbol ring (indices mod len)
__global__ void k_ring_window(const int32_t *ring, int64_t len, int64_t start, int count, int32_t *out) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x)
        out[i] = ring[(start + i) % len];
}

// nbits of every coder state, and the OR of the status words (device)
__global__ void k_ac_fields(int n, const altxs_ac_state *st, uint64_t *nbits, int32_t *status) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        if (nbits) nbits[i] = st[i].nbits;
        if (status) status[i] = (int32_t)st[i].status;
    }
}

__global__ void k_fill_i32(int32_t *p, int64_t n, int32_t v) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        p[i] = v;
}

// every stream's adapters start as the same initial arena
__global__ void k_broadcast(float *dst, int n, int64_t len, const float *src) {
    const int64_t total = (int64_t)n * len;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = src[i % len];
}

}  // namespace

struct altxs_ctx {
    int device = 0;
    altxs_model_desc desc{};
    std::vector<int32_t> schedule;
    altxs_weights w{};
    bool weights = false;
    altxs_split_planes planes{};
    altxs_dense_weights dense{};
    bool have_dense = false;
    std::vector<void *> owned;  // device buffers freed by altxs_destroy
    float *lora_init = nullptr;
    int64_t lora_floats = 0;
    altxs_ttt_hparams hp{};
    bool ttt = false;
    int64_t words = 0;     // bit-buffer words per stream (one segment)
    int32_t hist_len = 0;  // symbol ring length
    // streams
    int n = 0;
    altxs_batch b{};
    float *m = nullptr, *v = nullptr;  // AdamW moments of the adapters
    std::vector<int> steps;            // AdamW step per stream
    void *ttt_ws = nullptr;
    int64_t ttt_ws_bytes = 0;
    int32_t *window = nullptr;  // one stream's update window
    float *loss = nullptr;
    uint64_t *nbits = nullptr;
    int32_t *status = nullptr;
    int64_t t = 0;  // symbols coded per stream so far
    bool tensor_cores = false;
    uint64_t weights_id = 0;  // the caller's identifier of the weights (altxs_set_lockstep)
    uint64_t expect_id = 0;   // the encoder's lockstep id a decoder must match (0 = unchecked)

    void *alloc(size_t bytes) {
        void *p = nullptr;
        if (cudaMalloc(&p, bytes ? bytes : 16) != cudaSuccess) return nullptr;
        owned.push_back(p);
        return p;
    }
};

namespace {

int use_device(const altxs_ctx *c) { return cudaSetDevice(c->device) == cudaSuccess ? ALTXS_OK : ALTXS_ECUDA; }

// Bumped whenever a kernel change alters any result bit of the step or the
// update (the same number as the Python engine's payload fingerprint).
constexpr uint64_t kNumerics = 3;

struct Fnv {
    uint64_t h = 1469598103934665603ull;
    void bytes(const void *p, size_t n) {
        const unsigned char *b = static_cast<const unsigned char *>(p);
        for (size_t i = 0; i < n; ++i) h = (h ^ b[i]) * 1099511628211ull;
    }
    template <typename T>
    void v(const T &x) {
        bytes(&x, sizeof(x));
    }
};

// Everything of a context that changes the coded bits: the model description
// field by field (no padding or pointers), the layer schedule, the linear
// path, the segment length, the update and its hyper-parameters, the caller's
// weights identifier and the numerics version.
uint64_t lockstep_id(const altxs_ctx *c) {
    const altxs_model_desc &d = c->desc;
    Fnv f;
    f.v(kNumerics);
    const int32_t ints[] = {d.vocab, d.n_layers, d.d_model, d.n_heads, d.n_kv_heads, d.head_dim, d.mlp_hidden, d.ctx,
                            d.rope_dims, d.skip_gates, d.lora_rank, d.lora_mask, d.cdf_mode, d.cdf_bits, d.n_virtual,
                            d.n_encoder, d.smear_gate, d.gate_window, d.xsa_last_n, d.sparse_gate, d.asym_softcap,
                            d.parallel_start, d.parallel_final};
    f.bytes(ints, sizeof(ints));
    const float fl[] = {d.logit_softcap, d.lora_scale, d.sparse_gate_scale};
    f.bytes(fl, sizeof(fl));
    for (int32_t x : c->schedule) f.v(x);
    f.v((int32_t)c->tensor_cores);
    f.v(c->words);
    f.v((int32_t)c->ttt);
    if (c->ttt) {
        const float hp[] = {c->hp.lr, c->hp.beta1, c->hp.beta2, c->hp.eps, c->hp.weight_decay, c->hp.grad_clip};
        f.bytes(hp, sizeof(hp));
    }
    f.v(c->weights_id);
    return f.h ? f.h : 1;  // never 0: 0 means "unchecked"
}

}  // namespace

extern "C" {

altxs_ctx *altxs_create(const altxs_model_desc *desc, int device, int *status) {
    auto fail = [&](int rc) -> altxs_ctx * {
        if (status) *status = rc;
        return nullptr;
    };
    if (!desc || device < 0) return fail(ALTXS_EINVAL);
    if (cudaSetDevice(device) != cudaSuccess) return fail(ALTXS_ECUDA);
    if (altxs_workspace_bytes(desc, 1) < 0) return fail(ALTXS_ENOTSUP);
    altxs_ctx *c = new (std::nothrow) altxs_ctx();
    if (!c) return fail(ALTXS_ENOMEM);
    c->device = device;
    c->desc = *desc;
    if (desc->schedule) {
        const int nv = desc->n_virtual > 0 ? desc->n_virtual : desc->n_layers;
        c->schedule.assign(desc->schedule, desc->schedule + nv);
        c->desc.schedule = c->schedule.data();
    }
    c->lora_floats = desc->lora_rank > 0 ? altxs_lora_floats(desc) : 0;
    if (status) *status = ALTXS_OK;
    return c;
}

int altxs_load_weights(altxs_ctx *c, const altxs_weights *view, int tensor_cores) {
    if (!c || !view) return ALTXS_EINVAL;
    if (int rc = use_device(c)) return rc;
    c->w = *view;
    c->w.split = nullptr;
    cudaStream_t st = 0;
    const altxs_qmat *mats[5] = {&view->emb, &view->qkv, &view->o, &view->up, &view->down};
    if (tensor_cores) {
        if (view->split) {
            c->planes = *view->split;
        } else {
            uint16_t *hl[10];
            for (int i = 0; i < 5; ++i) {
                const size_t bytes = (size_t)mats[i]->rows * mats[i]->cols * 2;
                hl[2 * i] = static_cast<uint16_t *>(c->alloc(bytes));
                hl[2 * i + 1] = static_cast<uint16_t *>(c->alloc(bytes));
                if (!hl[2 * i] || !hl[2 * i + 1]) return ALTXS_ENOMEM;
                if (int rc = altxs_split_weights(mats[i], hl[2 * i], hl[2 * i + 1], st)) return rc;
            }
            c->planes = altxs_split_planes{hl[0], hl[1], hl[2], hl[3], hl[4], hl[5], hl[6], hl[7], hl[8], hl[9]};
        }
        c->w.split = &c->planes;
    } else if (c->desc.lora_rank > 0) {
        // the update's products on CUDA cores read dense fp32 copies of the base
        float *d[5];
        for (int i = 0; i < 5; ++i) {
            d[i] = static_cast<float *>(c->alloc((size_t)mats[i]->rows * mats[i]->cols * 4));
            if (!d[i]) return ALTXS_ENOMEM;
            if (int rc = altxs_dequant(mats[i], d[i], mats[i]->cols, st)) return rc;
        }
        c->dense = altxs_dense_weights{d[0], d[1], d[2], d[3], d[4]};
        c->have_dense = true;
    }
    if (cudaStreamSynchronize(st) != cudaSuccess) return ALTXS_ECUDA;
    c->tensor_cores = tensor_cores != 0;
    c->weights = true;
    return ALTXS_OK;
}

int altxs_set_lockstep(altxs_ctx *c, uint64_t weights_id, uint64_t expect_id) {
    if (!c) return ALTXS_EINVAL;
    c->weights_id = weights_id;
    c->expect_id = expect_id;
    return ALTXS_OK;
}

int altxs_lockstep_id(altxs_ctx *c, uint64_t *id) {
    if (!c || !id || !c->weights) return ALTXS_EINVAL;
    *id = lockstep_id(c);
    return ALTXS_OK;
}

int altxs_set_adapters(altxs_ctx *c, const float *d_init) {
    if (!c || !d_init || c->lora_floats <= 0) return ALTXS_EINVAL;
    if (int rc = use_device(c)) return rc;
    if (!c->lora_init) c->lora_init = static_cast<float *>(c->alloc((size_t)c->lora_floats * 4));
    if (!c->lora_init) return ALTXS_ENOMEM;
    return cudaMemcpy(c->lora_init, d_init, (size_t)c->lora_floats * 4, cudaMemcpyDeviceToDevice) == cudaSuccess
               ? ALTXS_OK
               : ALTXS_ECUDA;
}

int altxs_set_ttt(altxs_ctx *c, const altxs_ttt_hparams *hp) {
    if (!c || !hp || c->desc.lora_rank <= 0) return ALTXS_EINVAL;
    c->hp = *hp;
    c->ttt = true;
    return ALTXS_OK;
}

int altxs_set_segment(altxs_ctx *c, int64_t segment_symbols) {
    if (!c || segment_symbols < 1 || c->n) return ALTXS_EINVAL;
    const int64_t bits = c->desc.cdf_bits > 20 ? c->desc.cdf_bits : 20;
    c->words = segment_symbols * (bits + 2) / 32 + 4;  // <= cdf_bits + 2 bits per symbol
    return ALTXS_OK;
}

}  // extern "C"

extern "C" {

int altxs_streams_init(altxs_ctx *c, int n, const uint64_t *ids) {
    (void)ids;  // streams are independent; their order is the caller's
    if (!c || n < 1 || !c->weights || c->n || c->words < 1) return ALTXS_EINVAL;
    if (c->desc.lora_rank > 0 && !c->lora_init) return ALTXS_EINVAL;
    if (int rc = use_device(c)) return rc;
    const altxs_model_desc &d = c->desc;
    const int64_t Lv = d.n_virtual > 0 ? d.n_virtual : d.n_layers;
    const int64_t kv_bytes = (int64_t)n * Lv * 2 * d.n_kv_heads * d.ctx * 3 * d.head_dim;
    const int64_t ws = altxs_workspace_bytes(&d, n);
    if (ws < 0) return ALTXS_ENOTSUP;
    c->hist_len = d.ctx + 2;
    altxs_batch &b = c->b;
    b = altxs_batch{};
    b.n_streams = n;
    b.tok = static_cast<int32_t *>(c->alloc((size_t)n * 4));
    b.pos = static_cast<int64_t *>(c->alloc((size_t)n * 8));
    b.kv = static_cast<uint8_t *>(c->alloc((size_t)kv_bytes));
    b.ac = static_cast<altxs_ac_state *>(c->alloc((size_t)n * sizeof(altxs_ac_state)));
    b.bits = static_cast<uint32_t *>(c->alloc((size_t)n * c->words * 4));
    b.words_per_stream = c->words;
    b.sym = static_cast<int32_t *>(c->alloc((size_t)n * 4));
    b.hist = static_cast<int32_t *>(c->alloc((size_t)n * c->hist_len * 4));
    b.hist_len = c->hist_len;
    b.workspace = c->alloc((size_t)ws);
    b.workspace_bytes = ws;
    if (d.smear_gate) b.prev_tok = static_cast<int32_t *>(c->alloc((size_t)n * 4));
    c->nbits = static_cast<uint64_t *>(c->alloc((size_t)n * 8));
    c->status = static_cast<int32_t *>(c->alloc((size_t)n * 4));
    if (!b.tok || !b.pos || !b.kv || !b.ac || !b.bits || !b.sym || !b.hist || !b.workspace || !c->nbits ||
        !c->status || (d.smear_gate && !b.prev_tok))
        return ALTXS_ENOMEM;
    cudaStream_t st = 0;
    k_fill_i32<<<64, 256, 0, st>>>(b.tok, n, -1);  // the first symbol of a stream is coded uniformly
    if (b.prev_tok) k_fill_i32<<<64, 256, 0, st>>>(b.prev_tok, n, -1);
    cudaMemsetAsync(b.pos, 0, (size_t)n * 8, st);
    cudaMemsetAsync(b.kv, 0, (size_t)kv_bytes, st);
    cudaMemsetAsync(b.hist, 0, (size_t)n * c->hist_len * 4, st);
    if (c->lora_floats > 0) {
        b.lora = static_cast<float *>(c->alloc((size_t)n * c->lora_floats * 4));
        b.lora_stride = c->lora_floats;
        c->m = static_cast<float *>(c->alloc((size_t)n * c->lora_floats * 4));
        c->v = static_cast<float *>(c->alloc((size_t)n * c->lora_floats * 4));
        if (!b.lora || !c->m || !c->v) return ALTXS_ENOMEM;
        k_broadcast<<<256, 256, 0, st>>>(b.lora, n, c->lora_floats, c->lora_init);
        cudaMemsetAsync(c->m, 0, (size_t)n * c->lora_floats * 4, st);
        cudaMemsetAsync(c->v, 0, (size_t)n * c->lora_floats * 4, st);
        c->steps.assign(n, 0);
        c->ttt_ws_bytes = altxs_ttt_workspace_bytes(&d, d.ctx);
        if (c->ttt_ws_bytes < 0) return ALTXS_ENOTSUP;
        c->ttt_ws = c->alloc((size_t)c->ttt_ws_bytes);
        c->window = static_cast<int32_t *>(c->alloc((size_t)(d.ctx + 1) * 4));
        c->loss = static_cast<float *>(c->alloc(4));
        if (!c->ttt_ws || !c->window || !c->loss) return ALTXS_ENOMEM;
    }
    if (int rc = altxs_ac_init(n, nullptr, b.ac, st)) return rc;
    if (cudaStreamSynchronize(st) != cudaSuccess) return ALTXS_ECUDA;
    c->n = n;
    c->t = 0;
    return ALTXS_OK;
}

int altxs_step_encode(altxs_ctx *c, const int32_t *d_tokens, altxs_stream_t stream) {
    if (!c || !c->n || !d_tokens) return ALTXS_EINVAL;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(c->b.sym, d_tokens, (size_t)c->n * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return ALTXS_ECUDA;
    if (int rc = altxs_step(&c->desc, &c->w, &c->b, ALTXS_STEP_ENCODE, stream)) return rc;
    ++c->t;
    return ALTXS_OK;
}

int altxs_step_decode(altxs_ctx *c, int32_t *d_tokens_out, altxs_stream_t stream) {
    if (!c || !c->n || !d_tokens_out) return ALTXS_EINVAL;
    if (int rc = altxs_step(&c->desc, &c->w, &c->b, ALTXS_STEP_DECODE, stream)) return rc;
    ++c->t;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    return cudaMemcpyAsync(d_tokens_out, c->b.sym, (size_t)c->n * 4, cudaMemcpyDeviceToDevice, st) == cudaSuccess
               ? ALTXS_OK
               : ALTXS_ECUDA;
}

// One AdamW step of every stream's adapters on its last window of the coded
// symbols: x = s[end-T-1 .. end-1), y = s[end-T .. end), T = min(ctx, end-1),
// nothing when T < 2 (end = symbols coded per stream so far).
int altxs_ttt_boundary(altxs_ctx *c, altxs_stream_t stream) {
    if (!c || !c->n) return ALTXS_EINVAL;
    if (!c->ttt || c->lora_floats <= 0) return ALTXS_OK;
    const int64_t end = c->t;
    const int T = (int)(end - 1 < c->desc.ctx ? end - 1 : c->desc.ctx);
    if (T < 2) return ALTXS_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    for (int r = 0; r < c->n; ++r) {
        k_ring_window<<<1, 256, 0, st>>>(c->b.hist + (int64_t)r * c->hist_len, c->hist_len, end - T - 1, T + 1,
                                         c->window);
        const int64_t o = (int64_t)r * c->lora_floats;
        const int rc = altxs_ttt_update(&c->desc, &c->w, c->have_dense ? &c->dense : nullptr, &c->hp, c->window, T,
                                        c->b.lora + o, c->m + o, c->v + o, ++c->steps[r], c->loss, c->ttt_ws,
                                        c->ttt_ws_bytes, stream);
        if (rc) return rc;
    }
    return cudaGetLastError() == cudaSuccess ? ALTXS_OK : ALTXS_ECUDA;
}

// Flush every coder; bits [n][words] and n_bits [n] of the finished segments
// (device); the coders restart for the next segment.
int altxs_flush(altxs_ctx *c, uint32_t *d_bits, uint64_t *d_nbits, altxs_stream_t stream) {
    if (!c || !c->n || !d_bits || !d_nbits) return ALTXS_EINVAL;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (int rc = altxs_ac_flush(c->n, nullptr, c->b.ac, c->b.bits, c->words, stream)) return rc;
    k_ac_fields<<<(c->n + 255) / 256, 256, 0, st>>>(c->n, c->b.ac, d_nbits, nullptr);
    if (cudaMemcpyAsync(d_bits, c->b.bits, (size_t)c->n * c->words * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return ALTXS_ECUDA;
    return altxs_ac_init(c->n, nullptr, c->b.ac, stream);
}

// Load one segment per stream (bits [n][words], n_bits [n], device) and seed the decoders.
int altxs_begin_decode(altxs_ctx *c, const uint32_t *d_bits, const uint64_t *d_nbits, altxs_stream_t stream) {
    if (!c || !c->n || !d_bits || !d_nbits) return ALTXS_EINVAL;
    if (c->expect_id && c->expect_id != lockstep_id(c)) return ALTXS_EMISMATCH;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(c->b.bits, d_bits, (size_t)c->n * c->words * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return ALTXS_ECUDA;
    return altxs_ac_begin_decode(c->n, nullptr, c->b.ac, c->b.bits, d_nbits, c->words, stream);
}

// Waits for the context's work; status (host, [n], may be NULL) receives each
// stream's status word.  Returns the OR of the words (0: every stream healthy).
int altxs_get_status(altxs_ctx *c, int32_t *status) {
    if (!c || !c->n) return ALTXS_EINVAL;
    if (int rc = use_device(c)) return rc;
    k_ac_fields<<<(c->n + 255) / 256, 256>>>(c->n, c->b.ac, nullptr, c->status);
    std::vector<int32_t> h(c->n);
    if (cudaMemcpy(h.data(), c->status, (size_t)c->n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return ALTXS_ECUDA;
    int32_t any = 0;
    for (int i = 0; i < c->n; ++i) any |= h[i];
    if (status) std::memcpy(status, h.data(), (size_t)c->n * 4);
    return any;
}

int64_t altxs_ctx_words_per_stream(const altxs_ctx *c) { return c ? c->words : -1; }

void altxs_destroy(altxs_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->device);
    cudaDeviceSynchronize();
    for (void *p : c->owned) cudaFree(p);
    delete c;
}

}  // extern "C"
