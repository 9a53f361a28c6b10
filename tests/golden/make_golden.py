"""Generate the golden fixtures by running the altxs reference itself.

Run in a container where the reference checkout is importable:

    ALTXS_REFERENCE=/path/to/altxs python tests/golden/make_golden.py

The fixtures pin the CPU oracle (``oracle/``) to the reference:

* ``coder_probs.npz``  reference ``encode_with_probs`` bitstreams for float
  probability rows (the reference's own test vector, n=64 V=256 rng(0),
  plus a peaked V=1024 case);
* ``coder_cum.npz``    reference coder bitstreams for given integer CDFs
  (``_scale_cum_np`` replaced by a lookup of the supplied tables), including
  extreme tables (one dominant symbol, total = 2^30, V = 2);
* ``model_small.npz``  sliding-window logits from the reference ``GPT``
  (``prefill_cache`` + ``extend_cache`` with the KV tuples truncated to
  ``ctx-1`` rows before each extend) for seeded synthetic mixed-bit weights;
* ``lora_small.npz``   reference ``TTTLoRA`` init and one
  ``ce_with_lora`` -> backward -> clip -> AdamW step, plus the updated
  window logits;
* ``codec_small.json`` checks that the reference ``dequantize_channels``
  decodes this framework's codec writer output to the same dense weights.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
if "ALTXS_REFERENCE" not in os.environ:
    sys.exit("set ALTXS_REFERENCE to the root of a read-only altvectra/altxs checkout")
REF = Path(os.environ["ALTXS_REFERENCE"])
sys.path.insert(0, str(REPO))
for p in (REF / "src", REF / "src" / "model"):
    sys.path.insert(0, str(p))

import arithmetic_coder_lm as acl  # noqa: E402  (reference)
from hyperflow_distillation.mixed_bit_delta import dequantize_channels  # noqa: E402
from xsa_ttt.config import XsaTttConfig  # noqa: E402
from xsa_ttt.model import GPT  # noqa: E402
from xsa_ttt.ttt_lora import TTTLoRA, _forward_logits_lora, ce_with_lora, make_ttt_optimizer  # noqa: E402

from altxs_b200 import codec as C  # noqa: E402
from altxs_b200.config import ModelConfig  # noqa: E402
from oracle import coder as oc  # noqa: E402

SMALL = dict(
    vocab_size=512, num_layers=3, model_dim=128, num_heads=4, num_kv_heads=2,
    mlp_mult=4.0, rope_dims=16, block_size=32, online_retrain_every=64, seed=11,
    ttt_lora_rank=4, ttt_lora_lr=1e-3, ttt_k_lora=True, ttt_o_lora=True,
)


def small_cfg() -> ModelConfig:
    return ModelConfig(**SMALL)


def ref_cfg(cfg: ModelConfig) -> XsaTttConfig:
    h = XsaTttConfig(seed=cfg.seed)
    for k in ("vocab_size", "num_layers", "model_dim", "num_heads", "num_kv_heads", "mlp_mult",
              "rope_base", "rope_dims", "qk_gain_init", "logit_softcap", "ln_scale",
              "skip_gates_enabled", "block_size", "online_retrain_every", "ttt_lora_rank",
              "ttt_lora_alpha", "ttt_lora_lr", "ttt_beta1", "ttt_beta2", "ttt_weight_decay",
              "ttt_k_lora", "ttt_o_lora", "ttt_mlp_lora", "ttt_use_rslora", "grad_clip"):
        setattr(h, k, getattr(cfg, k))
    # plain GPT: every reference motif off (the engine's supported subset)
    h.xsa_last_n = 0
    h.num_loops = 0
    h.parallel_start_layer = 0
    h.smear_gate_enabled = False
    h.sparse_attn_gate_enabled = False
    h.attn_out_gate_enabled = False
    h.gated_attn_enabled = False
    h.asym_logit_rescale = False
    h.rope_yarn = False
    h.tie_embeddings = True
    h.ttt_warm_start_a = True
    h.retrain_mode = "lora"
    h.gradient_checkpointing = False
    return h


def ref_model(cfg: ModelConfig, weights: C.ModelWeights) -> GPT:
    torch.manual_seed(0)
    m = GPT(ref_cfg(cfg))
    sd = m.state_dict()
    for k, v in weights.dense().items():
        sd[k] = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32))
    m.load_state_dict(sd, strict=True)
    m.eval()
    return m


# ---------------------------------------------------------------------------


def gen_coder_probs() -> None:
    rng = np.random.default_rng(0)
    n, v = 64, 256
    rows = rng.random((n, v)).astype(np.float32)
    rows /= rows.sum(axis=1, keepdims=True)
    syms = rng.integers(0, v, size=n, dtype=np.int64)
    bs_a = acl.encode_with_probs(syms, lambda i, _p: rows[i], alphabet_size=v)
    rng = np.random.default_rng(1)
    n2, v2 = 64, 1024
    lg = rng.normal(0, 4.0, size=(n2, v2))
    p2 = np.exp(lg - lg.max(axis=1, keepdims=True))
    p2 = (p2 / p2.sum(axis=1, keepdims=True)).astype(np.float32)
    p64 = p2.astype(np.float64)
    syms2 = np.array([rng.choice(v2, p=p64[i] / p64[i].sum()) for i in range(n2)])
    bs_b = acl.encode_with_probs(syms2, lambda i, _p: p2[i], alphabet_size=v2)
    np.savez_compressed(
        HERE / "coder_probs.npz",
        a_probs=rows, a_syms=syms.astype(np.int32), a_bits=np.frombuffer(bs_a, np.uint8),
        b_probs=p2, b_syms=syms2.astype(np.int32), b_bits=np.frombuffer(bs_b, np.uint8),
    )


def _ref_encode_cum(cum: np.ndarray, syms: np.ndarray) -> bytes:
    """Reference coder with the supplied integer tables as its masses."""
    v = cum.shape[1] - 1
    orig = acl._scale_cum_np
    rows = iter(range(cum.shape[0]))

    def fake(_probs, *, alphabet_size):
        i = next(rows)
        return cum[i].astype(np.int64), int(cum[i][v])

    acl._scale_cum_np = fake
    try:
        carrier = np.zeros(v, dtype=np.float32)
        return acl.encode_with_probs(syms.astype(np.int64), lambda i, _p: carrier, alphabet_size=v)
    finally:
        acl._scale_cum_np = orig


def gen_coder_cum() -> None:
    out = {}
    rng = np.random.default_rng(2)
    # (a) framework fixed-point CDFs of random logits, V=512 (tables are
    # recomputed from the stored logits by the oracle rule)
    n, v = 96, 512
    lg = (30 * np.tanh(rng.normal(0, 3.0, size=(n, v)) / 30)).astype(np.float32)
    cum = oc.cum_from_logits(lg, "fixed", 20)
    syms = rng.integers(0, v, size=n).astype(np.int32)
    out["a_logits"], out["a_syms"] = lg, syms
    out["a_bits"] = np.frombuffer(_ref_encode_cum(cum, syms), np.uint8)
    # (b) reference-scale rule on the same logits
    cumr = oc.cum_from_logits(lg, "ref")
    out["b_bits"] = np.frombuffer(_ref_encode_cum(cumr, syms), np.uint8)
    # (c) extreme tables: one dominant symbol (long pending runs), total 2^30
    n3, v3 = 300, 64
    cum3 = np.zeros((n3, v3 + 1), dtype=np.uint64)
    syms3 = np.zeros(n3, dtype=np.int32)
    for i in range(n3):
        f = np.ones(v3, dtype=np.uint64)
        dom = int(rng.integers(0, v3))
        f[dom] = (1 << 30) - (v3 - 1)
        cum3[i, 1:] = np.cumsum(f)
        syms3[i] = dom if rng.random() < 0.97 else int(rng.integers(0, v3))
    out["c_cum"], out["c_syms"] = cum3, syms3
    out["c_bits"] = np.frombuffer(_ref_encode_cum(cum3, syms3), np.uint8)
    # (d) binary alphabet, balanced and skewed masses
    n4 = 400
    cum4 = np.zeros((n4, 3), dtype=np.uint64)
    p = rng.integers(1, 1 << 20, size=n4).astype(np.uint64)
    cum4[:, 1] = p
    cum4[:, 2] = p + rng.integers(1, 1 << 20, size=n4).astype(np.uint64)
    syms4 = rng.integers(0, 2, size=n4).astype(np.int32)
    out["d_cum"], out["d_syms"] = cum4, syms4
    out["d_bits"] = np.frombuffer(_ref_encode_cum(cum4, syms4), np.uint8)
    np.savez_compressed(HERE / "coder_cum.npz", **out)


def gen_codec() -> dict:
    cfg = small_cfg()
    w = C.synth_weights(cfg, seed=7)
    res = {}
    for name, mats in C._bank_mats(w).items():
        bits = np.concatenate([m.bits.reshape(-1) for m in mats])
        codes = np.concatenate([m.codes.reshape(-1, 64) for m in mats])
        scales = np.concatenate([m.scales.reshape(-1) for m in mats])
        packed = {b: C._pack_lsb(codes[bits == b], b).reshape(-1) for b in (2, 3, 4)}
        cbs = {b: scales[bits == b].reshape(-1, 1).astype(np.float16) for b in (2, 3, 4)}
        ref_ch = dequantize_channels(bits, cbs, packed, channel_width=64, codebook_mode="symmetric")
        mine = np.concatenate([m.dequant().reshape(-1, 64) for m in mats])
        res[name] = bool(np.array_equal(ref_ch, mine))
    dense = w.dense()
    h = hashlib.sha256()
    for k in sorted(dense):
        h.update(np.ascontiguousarray(dense[k], dtype=np.float32).tobytes())
    res["dense_sha256"] = h.hexdigest()
    (HERE / "codec_small.json").write_text(json.dumps(res, indent=1) + "\n")
    assert all(v for k, v in res.items() if k != "dense_sha256"), res
    return res


def gen_model() -> None:
    cfg = small_cfg()
    w = C.synth_weights(cfg, seed=7)
    m = ref_model(cfg, w)
    rng = np.random.default_rng(5)
    n = 80
    toks = rng.integers(0, cfg.vocab_size, size=n).astype(np.int64)
    logits = np.zeros((n, cfg.vocab_size), dtype=np.float32)
    keep = cfg.block_size - 1
    with torch.no_grad():
        cache = m.prefill_cache(torch.tensor([[int(toks[0])]]))
        logits[0] = m.logits_from_cache(cache)[0, -1].numpy()
        for i in range(1, n):
            cache.kv_slots = [(k[:, -keep:], v[:, -keep:]) for (k, v) in cache.kv_slots]
            cache, lg = m.extend_cache(cache, int(toks[i]))
            logits[i] = lg[0, -1].numpy()
    np.savez_compressed(HERE / "model_small.npz", tokens=toks.astype(np.int32), logits=logits)


def gen_lora() -> None:
    cfg = small_cfg()
    w = C.synth_weights(cfg, seed=7)
    m = ref_model(cfg, w)
    h = m.cfg
    for p in m.parameters():
        p.requires_grad_(False)
    torch.manual_seed(int(h.seed) ^ 0xA5A51070)
    lora = TTTLoRA(m, h)
    init = {k: v.detach().clone().numpy() for k, v in lora.state_dict().items()}
    opt = make_ttt_optimizer(lora, h)
    rng = np.random.default_rng(9)
    arr = rng.integers(0, cfg.vocab_size, size=100).astype(np.int64)
    end = 64
    t = min(cfg.block_size, end - 1)
    s0 = end - t - 1
    x = torch.tensor(arr[s0: s0 + t])[None]
    y = torch.tensor(arr[s0 + 1: s0 + 1 + t])[None]
    losses = []
    for _ in range(2):  # two boundaries on the same window: A moves on the 2nd
        opt.zero_grad(set_to_none=True)
        loss = ce_with_lora(m, x, y, lora)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(lora.parameters(), h.grad_clip)
        opt.step()
        losses.append(float(loss.detach()))
    with torch.no_grad():
        after = _forward_logits_lora(m, x, lora)[0].numpy()
    fin = {k: v.detach().clone().numpy() for k, v in lora.state_dict().items()}
    out = {"arr": arr.astype(np.int32), "end": np.array(end), "losses": np.array(losses),
           "logits_after": after.astype(np.float32)}
    out.update({f"init/{k}": v for k, v in init.items()})
    out.update({f"final/{k}": v for k, v in fin.items()})
    np.savez_compressed(HERE / "lora_small.npz", **out)


def gen_lora_steps() -> None:
    """The reference's online_retrain in lora mode with several steps per
    boundary (replay windows after the first, _replay_window_end) driven like
    its stream driver: adapters after two boundaries, the losses."""
    from xsa_ttt.compress import _init_online_state, _online_steps_at, online_retrain

    cfg = small_cfg()
    w = C.synth_weights(cfg, seed=7)
    m = ref_model(cfg, w)
    h = m.cfg
    h.online_retrain_steps = 3
    h.online_retrain_replay = True
    dev = torch.device("cpu")
    lora, opt = _init_online_state(m, h, dev, True)
    init = {k: v.detach().clone().numpy() for k, v in lora.state_dict().items()}
    arr = np.random.default_rng(10).integers(0, cfg.vocab_size, size=200).astype(np.int64)
    every = int(h.online_retrain_every)
    out = {"arr": arr.astype(np.int32)}
    for end in (every, 2 * every):
        steps = _online_steps_at(end, h, every)
        loss = online_retrain(m, arr, end=end, cfg=h, device=dev, optimizer=opt, lora=lora, seed=h.seed,
                              steps_override=steps, n_total=len(arr))
        out[f"{end}/loss"] = np.float64(loss)
    out.update({f"init/{k}": v for k, v in init.items()})
    out.update({f"final/{k}": v.detach().clone().numpy() for k, v in lora.state_dict().items()})
    np.savez_compressed(HERE / "lora_steps.npz", **out)


LORA_DEFAULTS = [  # the reference's LoRA defaults: rank 80, k off, o and MLP adapters on
    ("base", dict(ttt_lora_rank=80, ttt_k_lora=False, ttt_o_lora=True, ttt_mlp_lora=True, ttt_lora_lr=1e-3,
                  online_retrain_steps=2, online_retrain_replay=True)),
    ("o_on_y", dict(ttt_lora_rank=80, ttt_k_lora=False, ttt_o_lora=True, ttt_mlp_lora=True, ttt_o_lora_on_y=True,
                    ttt_lora_lr=1e-3, online_retrain_steps=2, online_retrain_replay=True)),
]


def gen_lora_defaults() -> None:
    """The reference's online_retrain in lora mode with its default adapter set
    (rank 80, q/v/o + MLP + lm_head adapters, k off), with the o adapter on the
    normed input and on the attention output: per-boundary losses, adapters
    after two boundaries of two steps (replay window on the second)."""
    from xsa_ttt.compress import _init_online_state, _online_steps_at, online_retrain

    arr = np.random.default_rng(12).integers(0, SMALL["vocab_size"], size=200).astype(np.int64)
    out = {"arr": arr.astype(np.int32)}
    for name, over in LORA_DEFAULTS:
        cfg = ModelConfig(**{**SMALL, **over})
        w = C.synth_weights(cfg, seed=7)
        m = ref_model(cfg, w)
        h = m.cfg
        h.ttt_o_lora_on_y = bool(over.get("ttt_o_lora_on_y", False))
        h.online_retrain_steps = over["online_retrain_steps"]
        h.online_retrain_replay = over["online_retrain_replay"]
        dev = torch.device("cpu")
        lora, opt = _init_online_state(m, h, dev, True)
        out.update({f"{name}/init/{k}": v.detach().clone().numpy() for k, v in lora.state_dict().items()})
        every = int(h.online_retrain_every)
        for end in (every, 2 * every):
            steps = _online_steps_at(end, h, every)
            loss = online_retrain(m, arr, end=end, cfg=h, device=dev, optimizer=opt, lora=lora, seed=h.seed,
                                  steps_override=steps, n_total=len(arr))
            out[f"{name}/{end}/loss"] = np.float64(loss)
        out.update({f"{name}/final/{k}": v.detach().clone().numpy() for k, v in lora.state_dict().items()})
        out[f"{name}/over"] = np.frombuffer(json.dumps(over).encode(), dtype=np.uint8)
    np.savez_compressed(HERE / "lora_defaults.npz", **out)


MOTIFS = dict(
    vocab_size=256, num_layers=6, model_dim=64, num_heads=4, num_kv_heads=2, mlp_mult=2.0,
    rope_dims=16, block_size=64, online_retrain_every=128, seed=3, retrain_mode="none",
    smear_gate_enabled=True, xsa_last_n=3, sparse_attn_gate_enabled=True, asym_logit_rescale=True,
    num_loops=1, loop_start=1, loop_end=2, parallel_start_layer=4, parallel_final_lane="mean",
)


def gen_model_motifs() -> None:
    """The reference GPT with its motifs on (smear gate, XSA on the last 3
    layers, sparse attention gate, asymmetric softcap, one depth loop over
    layers 1-2, parallel lanes from layer 4), random weights rounded to fp16
    (stored as fp16, loaded exactly), full-forward logits of one sequence."""
    h = XsaTttConfig(seed=MOTIFS["seed"])
    for k, v in MOTIFS.items():
        setattr(h, k, v)
    h.rope_base = 1e4
    h.qk_gain_init = 5.0
    h.logit_softcap = 30.0
    h.ln_scale = True
    h.skip_gates_enabled = True
    h.attn_out_gate_enabled = False
    h.gated_attn_enabled = False
    h.rope_yarn = False
    h.tie_embeddings = True
    h.gradient_checkpointing = False
    torch.manual_seed(0)
    m = GPT(h)
    m.enable_looping(True)
    g = torch.Generator().manual_seed(11)
    sd = m.state_dict()
    for k, v in sd.items():
        if v.dtype != torch.float32:
            continue
        if v.ndim >= 2 and v.numel() > 64:  # weight banks / embedding: fresh random
            v = torch.randn(v.shape, generator=g) * (0.5 / v.shape[-1] ** 0.5 if "emb" not in k else 0.3)
        elif k in ("smear_lambda",):
            v = torch.full_like(v, 0.7)
        elif k.startswith("smear_gate") or k.endswith("attn_gate_w"):
            v = torch.randn(v.shape, generator=g) * 0.5
        elif k.startswith("parallel_"):
            v = v + 0.1 * torch.randn(v.shape, generator=g)
        elif k == "softcap_pos":
            v = torch.tensor(25.0)
        elif k == "softcap_neg":
            v = torch.tensor(35.0)
        elif "skip_gates" in k or "resid_mix" in k or k.endswith("q_gain") or "scale" in k:
            v = v + 0.05 * torch.randn(v.shape, generator=g)
        sd[k] = v.half().float()
    m.load_state_dict(sd, strict=True)
    m.eval()
    rng = np.random.default_rng(8)
    T = 48
    toks = rng.integers(0, h.vocab_size, size=T).astype(np.int64)
    with torch.no_grad():
        logits = m.forward_logits(torch.tensor(toks)[None])[0].float().numpy()
    out = {"tokens": toks.astype(np.int32), "logits": logits.astype(np.float32),
           "config": np.frombuffer(json.dumps(MOTIFS).encode(), dtype=np.uint8)}
    out.update({f"w/{k}": v.half().numpy() for k, v in sd.items()})
    np.savez_compressed(HERE / "model_motifs.npz", **out)


REPLENISH = dict(
    vocab_size=64, num_layers=2, model_dim=64, num_heads=4, num_kv_heads=2, mlp_mult=2.0,
    rope_dims=8, block_size=16, online_retrain_every=24, seed=13, retrain_mode="none",
)
# reference replenish scenarios: (name, XsaTttConfig overrides, boundaries)
REPLENISH_CASES = [
    ("xm", dict(ttt_replenish_xm_k=3, ttt_replenish_warmup_steps=1, ttt_replenish_xm_4x_until_bytes=60,
                ttt_weight_decay=0.01, ttt_lora_lr=2e-3), [24, 48, 72, 96]),
    ("xm_probe2_anchor", dict(ttt_replenish_xm_k=2, ttt_replenish_warmup_steps=0, ttt_replenish_xm_probe_chunks=2,
                              ttt_replenish_xm_4x_until_bytes=0, ttt_replenish_anneal="exp",
                              ttt_replenish_lr_half_mb=1e-4, ttt_replenish_lr_min=1e-4, ttt_lora_lr=3e-3,
                              ttt_replenish_anchor_rate=0.3), [24, 48, 72, 96]),
    ("replay", dict(ttt_replenish_xm_k=0, ttt_replenish_warmup_steps=0, online_retrain_steps=2,
                    online_retrain_replay=True, ttt_replenish_replay_recent_mb=0.0, ttt_lora_lr=2e-3,
                    ttt_beta1=0.9), [24, 48, 72, 96]),
]


def gen_replenish() -> None:
    """Full-parameter replenish boundaries of the reference (online_retrain in
    retrain_mode="replenish", Forward-XM, anchor, anneal, replay) on a tiny
    GPT: the returned loss and the XM scores/choice at every boundary and the
    weights after the last one, from the reference's own code on CPU."""
    import copy
    import tempfile

    from safetensors.torch import save_file
    from xsa_ttt.compress import _init_online_state, online_retrain

    cfg = ModelConfig(**REPLENISH)
    w = C.synth_weights(cfg, seed=21)
    base = ref_model(cfg, w)
    rng = np.random.default_rng(5)
    arr = rng.integers(0, cfg.vocab_size, size=100).astype(np.int64)
    out = {"arr": arr.astype(np.int32), "config": np.frombuffer(json.dumps(REPLENISH).encode(), dtype=np.uint8)}
    out.update({f"w0/{k}": v.detach().numpy() for k, v in base.state_dict().items()})
    tmp = Path(tempfile.mkdtemp())
    masks = {"qo_bank": torch.rand(base.qo_bank.shape, generator=torch.Generator().manual_seed(3)),
             "blocks.0.attn_scale": torch.ones(base.blocks[0].attn_scale.shape)}
    save_file(masks, str(tmp / "anchor.safetensors"))
    out.update({f"anchor/{k}": v.numpy() for k, v in masks.items()})
    for name, over, ends in REPLENISH_CASES:
        m = copy.deepcopy(base)
        h = ref_cfg(cfg)
        h.retrain_mode = "replenish"
        for k, v in over.items():
            setattr(h, k, v)
        if "anchor" in name:
            h.ttt_replenish_anchor = str(tmp / "anchor.safetensors")
        dev = torch.device("cpu")
        _, opt = _init_online_state(m, h, dev, True)
        out[f"{name}/over"] = np.frombuffer(json.dumps(over).encode(), dtype=np.uint8)
        for end in ends:
            m.train()
            loss = online_retrain(m, arr, end=end, cfg=h, device=dev, optimizer=opt, lora=None, seed=h.seed,
                                  n_total=len(arr))
            xm = getattr(m, "_xm_last", None)
            out[f"{name}/{end}/loss"] = np.float64(loss)
            if xm is not None and int(xm["end"]) == end:
                out[f"{name}/{end}/xm_chosen"] = np.int32(xm["chosen"])
                out[f"{name}/{end}/xm_scores"] = np.asarray(xm["scores"], dtype=np.float64)
        # the per-boundary losses and scores pin the trajectory; the weights are kept at its end
        for k, v in m.state_dict().items():
            out[f"{name}/w/{k}"] = v.detach().numpy().copy()
    np.savez_compressed(HERE / "replenish.npz", **out)


FULL_CASES = [
    ("full_plain", dict(ttt_lora_lr=2e-3, ttt_weight_decay=0.01)),
    ("full_replay", dict(online_retrain_steps=3, online_retrain_replay=True, ttt_lora_lr=1e-3, ttt_beta1=0.9)),
    ("full_burst", dict(ttt_burst_schedule="50:3", ttt_burst_lr=1e-3, ttt_lora_lr=2e-3)),
]


def gen_full() -> None:
    """The reference's default retrain mode ("full": every weight on the last
    block window, replay windows, burst steps on their own AdamW) through its
    own online_retrain, driven like its stream driver (steps from
    _online_steps_at, one persistent burst state): per-boundary loss, final weights."""
    import copy

    from xsa_ttt.compress import _init_online_state, _online_steps_at, online_retrain

    cfg = ModelConfig(**REPLENISH)
    w = C.synth_weights(cfg, seed=21)
    base = ref_model(cfg, w)
    arr = np.random.default_rng(5).integers(0, cfg.vocab_size, size=100).astype(np.int64)
    out = {"arr": arr.astype(np.int32), "config": np.frombuffer(json.dumps(REPLENISH).encode(), dtype=np.uint8)}
    out.update({f"w0/{k}": v.detach().numpy() for k, v in base.state_dict().items()})
    dev = torch.device("cpu")
    for name, over in FULL_CASES:
        m = copy.deepcopy(base)
        h = ref_cfg(cfg)
        h.retrain_mode = "full"
        for k, v in over.items():
            setattr(h, k, v)
        _, opt = _init_online_state(m, h, dev, True)
        burst: dict = {}
        out[f"{name}/over"] = np.frombuffer(json.dumps(over).encode(), dtype=np.uint8)
        for end in (24, 48, 72, 96):
            steps = _online_steps_at(end, h, int(h.online_retrain_every))
            m.train()
            loss = online_retrain(m, arr, end=end, cfg=h, device=dev, optimizer=opt, lora=None, seed=h.seed,
                                  steps_override=steps, burst_state=burst, n_total=len(arr))
            out[f"{name}/{end}/loss"] = np.float64(loss)
        for k, v in m.state_dict().items():
            out[f"{name}/w/{k}"] = v.detach().numpy().copy()
    np.savez_compressed(HERE / "full_retrain.npz", **out)


MOTIF_RETRAIN = dict(
    vocab_size=64, num_layers=4, model_dim=64, num_heads=4, num_kv_heads=2, mlp_mult=2.0, rope_dims=8,
    block_size=16, online_retrain_every=24, seed=17, retrain_mode="none", smear_gate_enabled=True, gate_window=8,
    xsa_last_n=2, sparse_attn_gate_enabled=True, sparse_attn_gate_scale=0.5, asym_logit_rescale=True, num_loops=1,
    loop_start=1, loop_end=2, parallel_start_layer=3, parallel_final_lane="mean",
)
MOTIF_RETRAIN_CASES = [
    ("m_full", "full", dict(online_retrain_steps=2, online_retrain_replay=True, ttt_lora_lr=2e-3, ttt_beta1=0.9)),
    ("m_xm", "replenish", dict(ttt_replenish_xm_k=3, ttt_replenish_warmup_steps=1,
                               ttt_replenish_xm_4x_until_bytes=60, ttt_lora_lr=2e-3, ttt_weight_decay=0.01)),
    ("m_lora", "lora", dict(ttt_lora_rank=8, ttt_k_lora=True, ttt_o_lora=True, ttt_mlp_lora=True, ttt_lora_lr=2e-3,
                            online_retrain_steps=2, online_retrain_replay=True)),
]


def gen_motif_retrain() -> None:
    """The reference's retrain modes ("full" with replay windows; replenish
    with Forward-XM; lora with an adapter slot per layer application, MLP
    adapters, replay) through its own online_retrain on a GPT with every
    supported motif on (smear gate, XSA on the last 2 layers,
    sparse attention gate, asymmetric softcap, one depth loop over layers 1-2
    with looping active as at compression, parallel lanes from layer 3), random
    weights: per-boundary loss, XM choice and scores, final weights (adapters in lora mode)."""
    import copy

    from xsa_ttt.compress import _init_online_state, _online_steps_at, online_retrain

    h0 = XsaTttConfig(seed=MOTIF_RETRAIN["seed"])
    for k, v in MOTIF_RETRAIN.items():
        setattr(h0, k, v)
    h0.rope_base = 1e4
    h0.qk_gain_init = 5.0
    h0.logit_softcap = 30.0
    h0.ln_scale = True
    h0.skip_gates_enabled = True
    h0.attn_out_gate_enabled = False
    h0.gated_attn_enabled = False
    h0.rope_yarn = False
    h0.tie_embeddings = True
    h0.gradient_checkpointing = False
    h0.ttt_lora_rank = 0
    torch.manual_seed(0)
    base = GPT(h0)
    base.enable_looping(True)
    g = torch.Generator().manual_seed(23)
    sd = base.state_dict()
    for k, v in sd.items():
        if v.dtype != torch.float32:
            continue
        if v.ndim >= 2 and v.numel() > 64:
            v = torch.randn(v.shape, generator=g) * (0.5 / v.shape[-1] ** 0.5 if "emb" not in k else 0.3)
        elif k == "smear_lambda":
            v = torch.full_like(v, 0.6)
        elif k.startswith("smear_gate") or k.endswith("attn_gate_w"):
            v = torch.randn(v.shape, generator=g) * 0.5
        elif k.startswith("parallel_"):
            v = v + 0.1 * torch.randn(v.shape, generator=g)
        elif k == "softcap_pos":
            v = torch.tensor(12.0)
        elif k == "softcap_neg":
            v = torch.tensor(18.0)
        elif "skip_gates" in k or "resid_mix" in k or k.endswith("q_gain") or "scale" in k:
            v = v + 0.05 * torch.randn(v.shape, generator=g)
        sd[k] = v
    base.load_state_dict(sd, strict=True)
    arr = np.random.default_rng(6).integers(0, h0.vocab_size, size=100).astype(np.int64)
    out = {"arr": arr.astype(np.int32), "config": np.frombuffer(json.dumps(MOTIF_RETRAIN).encode(), dtype=np.uint8)}
    out.update({f"w0/{k}": v.detach().numpy().copy() for k, v in base.state_dict().items()})
    dev = torch.device("cpu")
    for name, mode, over in MOTIF_RETRAIN_CASES:
        m = copy.deepcopy(base)
        h = copy.deepcopy(h0)
        h.retrain_mode = mode
        for k, v in over.items():
            setattr(h, k, v)
        lora, opt = _init_online_state(m, h, dev, True)
        if lora is not None:
            out.update({f"{name}/init/{k}": v.detach().clone().numpy() for k, v in lora.state_dict().items()})
        burst: dict = {}
        out[f"{name}/over"] = np.frombuffer(json.dumps({"retrain_mode": mode, **over}).encode(), dtype=np.uint8)
        for end in (24, 48, 72, 96):
            steps = _online_steps_at(end, h, int(h.online_retrain_every))
            m.train()
            loss = online_retrain(m, arr, end=end, cfg=h, device=dev, optimizer=opt, lora=lora, seed=h.seed,
                                  steps_override=steps, burst_state=burst, n_total=len(arr))
            out[f"{name}/{end}/loss"] = np.float64(loss)
            xm = getattr(m, "_xm_last", None)
            if xm is not None and int(xm["end"]) == end:
                out[f"{name}/{end}/xm_chosen"] = np.int32(xm["chosen"])
                out[f"{name}/{end}/xm_scores"] = np.asarray(xm["scores"], dtype=np.float64)
        if lora is not None:
            out.update({f"{name}/final/{k}": v.detach().clone().numpy() for k, v in lora.state_dict().items()})
        for k, v in m.state_dict().items():
            out[f"{name}/w/{k}"] = v.detach().numpy().copy()
    np.savez_compressed(HERE / "motif_retrain.npz", **out)


CODEC_REF = dict(
    vocab_size=256, num_layers=4, model_dim=64, num_heads=4, num_kv_heads=2, mlp_mult=2.0, rope_dims=16,
    block_size=64, online_retrain_every=128, seed=77, smear_gate_enabled=True, xsa_last_n=2,
    sparse_attn_gate_enabled=True, sparse_attn_gate_init_std=0.02, asym_logit_rescale=True, num_loops=1,
    loop_start=1, loop_end=2, parallel_start_layer=3, parallel_final_lane="mean",
)


def gen_codec_ref() -> None:
    """A reference-format codec as the reference ships them: residual over
    Init(seed), channels along the reference layout (rows; o and mlp_down as
    columns), lloyd codebooks (2^b fp16 centroids per channel), some 0-bit
    channels, the motif small parameters; decoded by the reference's own
    load_codec (its deterministic Init(seed) + delta) and run by its GPT."""
    import dataclasses

    from hyperflow_distillation.mixed_bit_delta import load_codec
    from safetensors.numpy import save_file

    h = XsaTttConfig(seed=CODEC_REF["seed"])
    for k, v in CODEC_REF.items():
        setattr(h, k, v)
    h.tie_embeddings = True
    h.attn_out_gate_enabled = False
    h.gated_attn_enabled = False
    h.rope_yarn = False
    h.gradient_checkpointing = False
    L, d, V = h.num_layers, h.model_dim, h.vocab_size
    kv = h.num_kv_heads * (d // h.num_heads)
    F = int(h.mlp_mult * d)
    shapes = {"qo_bank": [2 * L, d, d], "kv_bank": [2 * L, kv, d], "mlp_up_bank": [L, F, d],
              "mlp_down_bank": [L, d, F], "tok_emb.weight": [V, d]}
    rng = np.random.default_rng(19)
    tensors, layouts = {}, {}
    for name, shape in shapes.items():
        n_ch = int(np.prod(shape)) // d
        bits = rng.choice([0, 2, 3, 4], size=n_ch, p=[0.05, 0.3, 0.35, 0.3]).astype(np.uint8)
        tensors[f"bits/{name}"] = bits
        for b in (2, 3, 4):
            idx = np.flatnonzero(bits == b)
            codes = rng.integers(0, 1 << b, size=(idx.size, d)).astype(np.uint8)
            tensors[f"packed/{name}/b{b}"] = C._pack_lsb(codes, b).reshape(-1) if idx.size else np.zeros(0, np.uint8)
            cb = np.sort(rng.normal(0, 0.01, size=(idx.size, 1 << b)), axis=1).astype(np.float16)
            tensors[f"codebook/{name}/b{b}"] = cb
        layouts[name] = {"shape": shape, "channels": n_ch, "channel_width": d}
    small = {}
    for i in range(L):
        small[f"blocks.{i}.attn_scale"] = (1 + 0.1 * rng.normal(size=d)).astype(np.float16)
        small[f"blocks.{i}.mlp_scale"] = (1 + 0.1 * rng.normal(size=d)).astype(np.float32)
        small[f"blocks.{i}.resid_mix"] = np.stack([1 + 0.1 * rng.normal(size=d), 0.1 * rng.normal(size=d)]).astype(np.float16)
        small[f"blocks.{i}.attn.q_gain"] = (5 + rng.normal(size=h.num_heads)).astype(np.float32)
        if i:  # layer 0 keeps the gate weights Init(seed) drew
            small[f"blocks.{i}.attn.attn_gate_w"] = (0.5 * rng.normal(size=(h.num_heads, h.gate_window))).astype(np.float32)
    S = min(len(range(4)) // 2, 3)
    small["skip_weights"] = (1 + 0.1 * rng.normal(size=(3, d))).astype(np.float32)
    small["skip_gates"] = (0.3 * rng.normal(size=(3, d))).astype(np.float32)
    small["smear_gate.weight"] = (0.5 * rng.normal(size=(1, h.gate_window))).astype(np.float32)
    small["smear_lambda"] = np.array([0.6], dtype=np.float32)
    small["softcap_pos"] = np.array(22.0, dtype=np.float32)
    small["softcap_neg"] = np.array(33.0, dtype=np.float32)
    small["parallel_post_lambdas"] = (1 + 0.1 * rng.normal(size=(L, 2, 2))).astype(np.float32)
    small["parallel_resid_lambdas"] = (1.1 + 0.1 * rng.normal(size=(L, 2))).astype(np.float32)
    del S
    for k, v in small.items():
        tensors[f"small/{k}"] = v
    path = HERE / "codec_ref_v256.safetensors"
    save_file(tensors, str(path))
    cfg_d = {k: v for k, v in dataclasses.asdict(h).items() if isinstance(v, (int, float, str, bool)) or v is None}
    meta = {"format": "hope_mixed_bit_delta", "format_version": 5, "codebook_mode": "lloyd", "seed": h.seed,
            "cfg": cfg_d, "n_layers": L, "layouts": layouts, "small_params": sorted(small)}
    path.with_suffix(".json").write_text(json.dumps(meta, indent=1) + "\n")
    model, _, _ = load_codec(path, device=torch.device("cpu"))
    model.eval()
    toks = np.random.default_rng(3).integers(0, V, size=40).astype(np.int64)
    with torch.no_grad():
        logits = model.forward_logits(torch.tensor(toks)[None])[0].float().numpy()
    out = {"tokens": toks.astype(np.int32), "logits": logits.astype(np.float32)}
    out.update({f"w/{k}": v.detach().float().numpy() for k, v in model.state_dict().items()})
    np.savez_compressed(HERE / "codec_ref_v256.npz", **out)


def gen_zipf() -> None:
    from altxs_b200.synth import zipf_markov

    s = zipf_markov(256, 4096, [1, 2, 3])
    np.savez_compressed(HERE / "zipf_markov.npz", seeds=np.array([1, 2, 3]), streams=s)


# positions whose reference probability rows the C1 fixture keeps (both
# segment sides of several boundaries, the stream start and end)
C1_ROWS = (1, 2, 3, 255, 256, 257, 4095, 4096, 4097, 4100, 8191, 8192, 8193, 20000, 32767, 32768,
           32769, 61439, 61440, 61441, 65534, 65535)


C1_BANKS = ("tok_emb.weight", "qo_bank", "kv_bank", "mlp_up_bank", "mlp_down_bank")


def gen_c1_stream() -> None:
    """BASELINE config C1 through the reference's own coder path.

    Model: the reference ``GPT`` at the C1 shapes from ``torch.manual_seed(0)``
    (its own random init).  Stream: 65,536 symbols of the order-2 Zipf-Markov
    source, seed 1.  Run: ``compress_bytes`` (compress.py:1363) with rank-4
    q/v LoRA, lr 1e-3, an update at every multiple of 4096 (``online_retrain``
    lora branch), probability rows from the chunked teacher-forced forward
    (``_chunk_tf_probs``: each segment with the previous block as context at
    positions from 0), masses ``max(1, round(p*1e6))``.  Kept: bits/symbol,
    payload size and hash, and the log-probability rows at ``C1_ROWS``."""
    import time

    import xsa_ttt.compress as rc

    from altxs_b200.config import c1_config
    from altxs_b200.synth import zipf_markov

    cfg = c1_config()
    h = ref_cfg(cfg)
    torch.manual_seed(0)
    m = GPT(h)
    m.eval()
    sd = {k: v.detach().float().numpy() for k, v in m.state_dict().items()}
    mine = C.reference_init(cfg, 0)
    for k in C1_BANKS:
        assert np.array_equal(sd[k], mine[k]), k
    wsha = hashlib.sha256()
    for k in C1_BANKS:
        wsha.update(np.ascontiguousarray(sd[k], dtype=np.float32).tobytes())
    arr = zipf_markov(65536, cfg.vocab_size, [1])[0].astype(np.uint16)
    cache: dict = {}
    t0 = time.time()
    res = rc.compress_bytes(m, arr, cfg=h, device=torch.device("cpu"), online_retrain_enabled=True,
                            progress=False, prob_cache=cache)
    t_enc = time.time() - t0
    rows = []
    for p in C1_ROWS:
        st = (p // 4096) * 4096
        r = cache[(st, min(65536, st + 4096))][p - st].astype(np.float64)
        rows.append(np.log(np.maximum(r, 1e-45)))
    out = dict(
        stream_sha=np.frombuffer(hashlib.sha256(arr.astype("<u2").tobytes()).digest(), np.uint8),
        bank_sha=np.frombuffer(wsha.digest(), np.uint8),
        bits_per_symbol=np.float64(res["bits_per_symbol"]),
        payload_bytes=np.int64(res["payload_bytes"]),
        payload_sha=np.frombuffer(hashlib.sha256(res["payload"]).digest(), np.uint8),
        retrain_count=np.int64(res["retrain_count"]),
        chunk_bits=np.array([r["bpb"] for r in res["chunk_bpb_rows"]]),
        row_pos=np.array(C1_ROWS, dtype=np.int64),
        row_logp=np.stack(rows).astype(np.float32),
    )
    np.savez_compressed(HERE / "c1_stream.npz", **out)
    print(f"c1: {res['bits_per_symbol']:.5f} bits/sym, {res['payload_bytes']} B, "
          f"{res['retrain_count']} updates, encode {t_enc:.1f} s")


def gen_incr_stream() -> None:
    """Bits/symbol and probability rows of the reference's own incremental
    entry point, ``compress_full_sha_incremental`` (incremental.py:1561), run
    eagerly on the CPU (``XSA_AC_FUSED=0 XSA_AC_GPU_AC=0 XSA_AC_GRAPH=0``).

    Same stream as C1 (65,536 Zipf-Markov symbols, seed 1) and the C1 shapes.
    The weights are this framework's seeded mixed-bit synthetic model at those
    shapes (seed 3; dense fp32 in the reference ``GPT``): the reference's own
    seed-0 init has zero output and down projections and stays at log2(V)
    bits under every update, which would not tell a right update from a wrong
    one.  Two runs: no update (the reference engine's segment reset and
    prefill alone), and ``retrain_mode="replenish"`` (its production update;
    this entry point refuses LoRA, incremental.py:1553) with an update every
    4096 symbols, 2 steps per boundary (replay on), lr 1e-3, no warmup.  Each
    run keeps bits/symbol, payload size and hash, and the log-probabilities
    the reference engine coded with at ``C1_ROWS`` (from its
    ``_segment_rows_tf``, which runs ``reset_segment`` then the W-windows)."""
    import time

    os.environ.update(XSA_AC_FUSED="0", XSA_AC_GPU_AC="0", XSA_AC_GRAPH="0")
    import xsa_ttt.incremental as inc

    from altxs_b200.config import c1_config
    from altxs_b200.synth import zipf_markov

    cfg = c1_config()
    arr = zipf_markov(65536, cfg.vocab_size, [1])[0].astype(np.uint16)
    out = {"row_pos": np.array(C1_ROWS, dtype=np.int64)}
    orig = inc._segment_rows_tf
    for tag, online in (("none", False), ("replenish", True)):
        w = C.synth_weights(cfg, seed=3)
        m = ref_model(cfg, w)
        h = m.cfg
        h.retrain_mode = "replenish"
        h.online_retrain_every = 4096
        h.online_retrain_steps = 2
        h.ttt_lora_lr = 1e-3
        h.ttt_replenish_warmup_steps = 0
        got: dict[int, np.ndarray] = {}

        def rec(engine, a, seg, *, start):
            rows = orig(engine, a, seg, start=start)
            for p in C1_ROWS:
                if start <= p < start + len(seg):
                    got[p] = np.log(np.maximum(rows[p - start].astype(np.float64), 1e-45))
            return rows

        inc._segment_rows_tf = rec
        try:
            t0 = time.time()
            res = inc.compress_full_sha_incremental(m, arr, cfg=h, device=torch.device("cpu"),
                                                    online_retrain_enabled=online, progress=False)
        finally:
            inc._segment_rows_tf = orig
        out[f"{tag}_bits_per_symbol"] = np.float64(res["bits_per_symbol"])
        out[f"{tag}_payload_bytes"] = np.int64(res["payload_bytes"])
        out[f"{tag}_payload_sha"] = np.frombuffer(hashlib.sha256(res["payload"]).digest(), np.uint8)
        out[f"{tag}_retrain_count"] = np.int64(res["retrain_count"])
        out[f"{tag}_segment_bits"] = np.array([r["bpb"] for r in res["chunk_bpb_rows"]])
        out[f"{tag}_row_logp"] = np.stack([got[p] for p in C1_ROWS]).astype(np.float32)
        print(f"incr {tag}: {res['bits_per_symbol']:.5f} bits/sym, {res['payload_bytes']} B, "
              f"{res['retrain_count']} updates, {time.time() - t0:.1f} s")
    np.savez_compressed(HERE / "incr_stream.npz", **out)


if __name__ == "__main__":
    GEN = [gen_coder_probs, gen_coder_cum, gen_codec, gen_model, gen_lora, gen_lora_steps, gen_lora_defaults,
           gen_model_motifs, gen_replenish, gen_full, gen_motif_retrain, gen_codec_ref, gen_zipf, gen_c1_stream,
           gen_incr_stream]
    # no argument: every fixture; otherwise only the named generators (e.g. gen_c1_stream)
    pick = sys.argv[1:]
    for fn in GEN:
        if not pick or fn.__name__ in pick:
            r = fn()
            if r is not None:
                print(r)
    for f in sorted(HERE.glob("*.npz")) + sorted(HERE.glob("*.json")):
        print(f.name, f.stat().st_size)
