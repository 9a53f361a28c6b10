"""The CPU oracle against golden vectors produced by the altxs reference.

These pin the oracle before it is trusted as the checker of the CUDA path
(fixtures: ``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from altxs_b200 import codec as C
from altxs_b200.config import ModelConfig
from oracle import coder as oc
from oracle.model import OracleModel, OracleTTT, OracleWeights
from tests.conftest import GOLDEN

SMALL = dict(
    vocab_size=512, num_layers=3, model_dim=128, num_heads=4, num_kv_heads=2,
    mlp_mult=4.0, rope_dims=16, block_size=32, online_retrain_every=64, seed=11,
    ttt_lora_rank=4, ttt_lora_lr=1e-3, ttt_k_lora=True, ttt_o_lora=True,
)


def _bits(a) -> bytes:
    return np.asarray(a, dtype=np.uint8).tobytes()


def test_coder_probs_matches_reference(golden):
    g = golden("coder_probs.npz")
    for c in ("a", "b"):
        probs, syms, ref = g[f"{c}_probs"], g[f"{c}_syms"], _bits(g[f"{c}_bits"])
        got = oc.encode_probs(probs, syms)
        assert got == ref
        assert np.array_equal(oc.decode_probs(probs, got, len(syms)), syms)


def test_coder_cum_matches_reference(golden):
    g = golden("coder_cum.npz")
    lg, syms = g["a_logits"], g["a_syms"]
    for rule, key in (("fixed", "a_bits"), ("ref", "b_bits")):
        cum = oc.cum_from_logits(lg, rule, 20) if rule == "fixed" else oc.cum_from_logits(lg, "ref")
        got = oc.encode_cum(cum, syms)
        assert got == _bits(g[key]), rule
        assert np.array_equal(oc.decode_cum(cum, got, len(syms)), syms)
    for c in ("c", "d"):
        cum, s = g[f"{c}_cum"], g[f"{c}_syms"]
        got = oc.encode_cum(cum, s)
        assert got == _bits(g[f"{c}_bits"]), c
        assert np.array_equal(oc.decode_cum(cum, got, len(s)), s)


def test_fixed_cdf_rule_properties():
    rng = np.random.default_rng(0)
    lg = (30 * np.tanh(rng.normal(0, 4, size=(50, 300)) / 30)).astype(np.float32)
    for bits in (16, 20, 24, 30):
        cum = oc.cum_from_logits(lg, "fixed", bits)
        f = np.diff(cum.astype(np.int64), axis=1)
        assert (f >= 1).all()
        assert (cum[:, -1] <= (1 << bits)).all()
        # order independence: permuting the alphabet permutes the masses
        perm = rng.permutation(300)
        cum_p = oc.cum_from_logits(lg[:, perm], "fixed", bits)
        assert np.array_equal(np.diff(cum_p.astype(np.int64), axis=1), f[:, perm])


def test_codec_golden():
    res = json.loads((GOLDEN / "codec_small.json").read_text())
    w = C.synth_weights(ModelConfig(**SMALL), seed=7)
    import hashlib

    d = w.dense()
    h = hashlib.sha256()
    for k in sorted(d):
        h.update(np.ascontiguousarray(d[k], dtype=np.float32).tobytes())
    assert h.hexdigest() == res["dense_sha256"]
    assert all(v for k, v in res.items() if k != "dense_sha256")


def test_codec_roundtrip(tmp_path):
    w = C.synth_weights(ModelConfig(**SMALL), seed=7)
    p = C.write_codec(w, tmp_path / "m")
    w2 = C.read_codec(p)
    a, b = w.dense(), w2.dense()
    for k in a:
        assert np.array_equal(np.asarray(a[k]), np.asarray(b[k])), k


def test_oracle_step_matches_reference_sliding_window(golden):
    g = golden("model_small.npz")
    cfg = ModelConfig(**SMALL)
    m = OracleModel(OracleWeights.from_model_weights(C.synth_weights(cfg, seed=7)))
    st = m.new_stream()
    toks = g["tokens"]
    ref = g["logits"]
    got = np.stack([m.step(st, int(t)).numpy() for t in toks])
    err = np.abs(got - ref).max()
    assert err < 2e-4, err


def test_oracle_lora_matches_reference(golden):
    g = golden("lora_small.npz")
    cfg = ModelConfig(**SMALL)
    m = OracleModel(OracleWeights.from_model_weights(C.synth_weights(cfg, seed=7)))
    ttt = OracleTTT(m)
    # init: bit-identical A matrices, in the reference's parameter order
    names = {"lm": "lm_head_lora"}
    for i in range(cfg.num_layers):
        for t in ("q", "k", "v", "o"):
            names[f"{t}{i}"] = f"{t}_loras.{i}"
    for ours, ref in names.items():
        assert torch.equal(ttt.lora.A[ours], torch.from_numpy(g[f"init/{ref}.A"])), ours
    arr, end = g["arr"], int(g["end"])
    losses = [ttt.update(arr, end) for _ in range(2)]
    np.testing.assert_allclose(losses, g["losses"], rtol=1e-5)
    for ours, ref in names.items():
        np.testing.assert_allclose(ttt.lora.A[ours].detach().numpy(), g[f"final/{ref}.A"], atol=1e-6)
        np.testing.assert_allclose(ttt.lora.B[ours].detach().numpy(), g[f"final/{ref}.B"], atol=1e-6)
    t = min(cfg.block_size, end - 1)
    x = torch.from_numpy(arr[end - t - 1: end - 1].astype(np.int64))
    with torch.no_grad():
        after = m.window_logits(x, ttt.lora).numpy()
    assert np.abs(after - g["logits_after"]).max() < 2e-4


def test_zipf_markov_fixture(golden):
    from altxs_b200.synth import zipf_markov

    g = golden("zipf_markov.npz")
    assert np.array_equal(zipf_markov(256, 4096, g["seeds"]), g["streams"])


@pytest.mark.parametrize("vocab", [2, 7, 256])
def test_oracle_coder_roundtrip_edge(vocab):
    rng = np.random.default_rng(vocab)
    n = 257
    lg = rng.normal(0, 6, size=(n, vocab)).astype(np.float32)
    syms = rng.integers(0, vocab, size=n).astype(np.int32)
    for rule in ("fixed", "ref"):
        cum = oc.cum_from_logits(lg, rule, 20)
        bs = oc.encode_cum(cum, syms)
        assert np.array_equal(oc.decode_cum(cum, bs, n), syms)
    # empty input: flush only
    cum0 = np.zeros((0, vocab + 1), dtype=np.uint64)
    assert len(oc.encode_cum(cum0, np.zeros(0, np.int32))) == 1


def _motif_model(g):
    import json

    from altxs_b200 import codec as C
    from altxs_b200.config import ModelConfig

    cfg = ModelConfig(**json.loads(bytes(g["config"])))
    tensors = {k[2:]: g[k].astype(np.float32) for k in g.files if k.startswith("w/")}
    return cfg, C.dense_weights(cfg, tensors)


def test_oracle_motifs_match_reference(golden):
    """Step-by-step oracle logits of the reference GPT with every supported
    motif on (smear, XSA, sparse gate, asymmetric softcap, depth loop,
    parallel lanes) against the reference's own full forward."""
    from oracle.model import OracleModel, OracleWeights

    g = golden("model_motifs.npz")
    cfg, w = _motif_model(g)
    assert cfg.num_virtual_layers == 8 and cfg.motifs
    om = OracleModel(OracleWeights.from_model_weights(w))
    st = om.new_stream()
    got = np.stack([om.step(st, int(t)).numpy() for t in g["tokens"]])
    err = float(np.abs(got - g["logits"]).max())
    assert err < 1e-4, err
    # one causal pass gives the same last row
    st2 = om.new_stream()
    last = om.prefill(st2, g["tokens"]).numpy()
    assert float(np.abs(last - g["logits"][-1]).max()) < 1e-4


def replenish_case(g, name):
    """Config, initial state and anchor masks of one golden replenish scenario."""
    import json

    from altxs_b200.config import ModelConfig

    base = json.loads(bytes(g["config"]))
    over = json.loads(bytes(g[f"{name}/over"]))
    cfg = ModelConfig(**{**base, "retrain_mode": "replenish", **over})
    w0 = {k[3:]: g[k] for k in g.files if k.startswith("w0/")}
    masks = {k[7:]: g[k] for k in g.files if k.startswith("anchor/")} if "anchor" in name else None
    if masks:
        cfg.ttt_replenish_anchor = "anchor.safetensors"
    return cfg, w0, masks


@pytest.mark.parametrize("name", ["xm", "xm_probe2_anchor", "replay"])
def test_oracle_replenish_matches_reference(golden, name):
    """Full-parameter replenish boundaries (Forward-XM with a 4x head and a
    warmup boundary; XM over two probe chunks with anchor masks and an
    annealed lr; plain replenish with replay draws) against the reference's
    own online_retrain: loss and XM scores/choice per boundary, weights at the end."""
    from oracle.replenish import OracleReplenish

    g = golden("replenish.npz")
    cfg, w0, masks = replenish_case(g, name)
    o = OracleReplenish(cfg, w0, masks)
    arr = g["arr"].astype(np.int64)
    for end in (24, 48, 72, 96):
        loss = o.boundary(arr, end, n_total=len(arr))
        assert abs(loss - float(g[f"{name}/{end}/loss"])) < 1e-5, (end, loss)
        if f"{name}/{end}/xm_chosen" in g.files:
            assert o.xm_last["chosen"] == int(g[f"{name}/{end}/xm_chosen"])
            assert np.abs(np.array(o.xm_last["scores"]) - g[f"{name}/{end}/xm_scores"]).max() < 1e-5
    st = o.state()
    err = max(float(np.abs(st[k] - g[f"{name}/w/{k}"]).max()) for k in st)
    assert err < 1e-6, err


def test_reference_codec_decodes_like_the_reference(golden):
    """A reference-format V=256 codec as shipped (residual over Init(seed),
    reference channel layout with o / mlp_down as columns, lloyd codebooks,
    0-bit channels, motif small parameters): read_codec rebuilds the
    reference's deterministic Init(seed) and adds the decoded delta, giving the
    reference load_codec's weights bit for bit; the oracle then reproduces the
    reference GPT's logits."""
    from altxs_b200 import codec as C
    from tests.conftest import GOLDEN

    g = golden("codec_ref_v256.npz")
    w = C.read_codec(GOLDEN / "codec_ref_v256.safetensors")
    assert w.cfg.vocab_size == 256 and w.cfg.motifs and w.cfg.num_virtual_layers == 6
    dense = w.dense()
    for k in ("tok_emb.weight", "qo_bank", "kv_bank", "mlp_up_bank", "mlp_down_bank"):
        assert np.array_equal(dense[k], g["w/" + k]), k
    sm = w.small
    for i in range(w.cfg.num_layers):
        assert np.array_equal(sm["attn_gate_w"][i], g[f"w/blocks.{i}.attn.attn_gate_w"])  # layer 0: Init draw
        assert np.array_equal(sm["resid_mix"][i], g[f"w/blocks.{i}.resid_mix"])
    assert np.array_equal(sm["smear_gate"], g["w/smear_gate.weight"].reshape(-1))
    om = OracleModel(OracleWeights.from_model_weights(w))
    st = om.new_stream()
    got = np.stack([om.step(st, int(t)).numpy() for t in g["tokens"]])
    assert float(np.abs(got - g["logits"]).max()) < 1e-4


def full_case(g, name):
    """Config and initial state of one golden full-mode scenario."""
    import json

    from altxs_b200.config import ModelConfig

    base = json.loads(bytes(g["config"]))
    over = json.loads(bytes(g[f"{name}/over"]))
    cfg = ModelConfig(**{**base, "retrain_mode": "full", **over})
    return cfg, {k[3:]: g[k] for k in g.files if k.startswith("w0/")}


@pytest.mark.parametrize("name", ["full_plain", "full_replay", "full_burst"])
def test_oracle_full_retrain_matches_reference(golden, name):
    """The reference's default retrain mode ("full": every weight on the last
    block window; replay windows; burst steps on their own AdamW walking the
    boundaries) against its own online_retrain: loss per boundary, final weights."""
    from oracle.replenish import OracleReplenish

    g = golden("full_retrain.npz")
    cfg, w0 = full_case(g, name)
    o = OracleReplenish(cfg, w0)
    arr = g["arr"].astype(np.int64)
    for end in (24, 48, 72, 96):
        loss = o.boundary(arr, end, n_total=len(arr))
        assert abs(loss - float(g[f"{name}/{end}/loss"])) < 1e-5, (end, loss)
    st = o.state()
    err = max(float(np.abs(st[k] - g[f"{name}/w/{k}"]).max()) for k in st)
    # Adam moves an entry by about lr per step whatever its gradient's size, so
    # rounding on entries whose gradient is ~0 (they do not move the loss: the
    # losses above agree to 1e-5) shows up as a fraction of a step
    lr = min(cfg.ttt_lora_lr, cfg.ttt_burst_lr)
    assert err < 0.1 * lr, (err, lr)


def motif_case(g, name):
    """Config and initial state of one golden retrain scenario on the motif model."""
    import json

    base = json.loads(bytes(g["config"]))
    over = json.loads(bytes(g[f"{name}/over"]))
    cfg = ModelConfig(**{**base, **over})
    return cfg, {k[3:]: g[k] for k in g.files if k.startswith("w0/")}


@pytest.mark.parametrize("name", ["m_full", "m_xm"])
def test_oracle_motif_retrain_matches_reference(golden, name):
    """Both full-parameter retrain modes on a model with every supported motif
    on (smear gate, XSA, sparse attention gate, asymmetric softcap, a depth
    loop, parallel lanes) against the reference's own online_retrain: loss and
    XM choice per boundary, every parameter (the motifs' own included) at the end."""
    from oracle.replenish import OracleReplenish

    g = golden("motif_retrain.npz")
    cfg, w0 = motif_case(g, name)
    o = OracleReplenish(cfg, w0)
    assert {"smear_gate.weight", "softcap_pos", "parallel_post_lambdas", "blocks.1.attn.attn_gate_w"} <= set(o.p)
    arr = g["arr"].astype(np.int64)
    for end in (24, 48, 72, 96):
        loss = o.boundary(arr, end, n_total=len(arr))
        assert abs(loss - float(g[f"{name}/{end}/loss"])) < 1e-5, (end, loss)
        if f"{name}/{end}/xm_chosen" in g.files:
            assert o.xm_last["chosen"] == int(g[f"{name}/{end}/xm_chosen"])
            assert np.abs(np.array(o.xm_last["scores"]) - g[f"{name}/{end}/xm_scores"]).max() < 1e-5
    st = o.state()
    assert set(st) == {k[len(name) + 3:] for k in g.files if k.startswith(f"{name}/w/")}
    err = max(float(np.abs(st[k] - g[f"{name}/w/{k}"]).max()) for k in st)
    assert err < 0.1 * cfg.ttt_lora_lr, err


def lora_ref_names(cfg) -> dict:
    """Our adapter names -> the reference TTTLoRA module names."""
    names = {"lm": "lm_head_lora"}
    for i in range(cfg.num_layers):
        for t, mod in (("q", "q_loras"), ("k", "k_loras"), ("v", "v_loras"), ("o", "o_loras"), ("mlp", "mlp_loras")):
            names[f"{t}{i}"] = f"{mod}.{i}"
    return names


@pytest.mark.parametrize("name", ["base", "o_on_y"])
def test_oracle_lora_defaults_match_reference(golden, name):
    """The reference's default adapter set (rank 80, MLP adapters, k off; the o
    adapter on the normed input or on the attention output) through its own
    online_retrain in lora mode: initial A bit-identical, losses per boundary,
    adapters after two boundaries of two steps."""
    import json

    g = golden("lora_defaults.npz")
    cfg = ModelConfig(**{**SMALL, **json.loads(bytes(g[f"{name}/over"]))})
    m = OracleModel(OracleWeights.from_model_weights(C.synth_weights(cfg, seed=7)))
    ttt = OracleTTT(m)
    names = lora_ref_names(cfg)
    for ours in ttt.lora.A:
        assert torch.equal(ttt.lora.A[ours], torch.from_numpy(g[f"{name}/init/{names[ours]}.A"])), ours
    assert any(k.startswith("mlp") for k in ttt.lora.A)
    arr = g["arr"].astype(np.int64)
    every = cfg.online_retrain_every
    for end in (every, 2 * every):
        loss = ttt.update(arr, end)
        assert abs(loss - float(g[f"{name}/{end}/loss"])) < 1e-5, (end, loss)
    err = 0.0
    for ours in ttt.lora.A:
        for part, t in (("A", ttt.lora.A[ours]), ("B", ttt.lora.B[ours])):
            err = max(err, float(np.abs(t.detach().numpy() - g[f"{name}/final/{names[ours]}.{part}"]).max()))
    assert err < 0.05 * cfg.ttt_lora_lr, err


def motif_lora_model(cfg, w0):
    """OracleModel of a reference state (detached fp32 tensors)."""
    import dataclasses

    from oracle.replenish import OracleReplenish

    w = OracleReplenish(cfg, w0).weights()
    det = lambda v: [t.detach() for t in v] if isinstance(v, list) else v.detach()  # noqa: E731
    w = dataclasses.replace(w, **{f.name: det(getattr(w, f.name)) for f in dataclasses.fields(w)
                                  if f.name not in ("cfg", "small")},
                            small={k: v.detach() for k, v in w.small.items()})
    return OracleModel(w)


def test_oracle_motif_lora_matches_reference(golden):
    """The reference's lora mode on its motif model (one adapter slot per layer
    application with the depth loop active, MLP adapters, replay steps) through
    its own online_retrain: initial A bit-identical, loss per boundary, adapters."""
    g = golden("motif_retrain.npz")
    cfg, w0 = motif_case(g, "m_lora")
    assert cfg.num_virtual_layers == 6 and cfg.lora_enabled
    ttt = OracleTTT(motif_lora_model(cfg, w0))
    names = {"lm": "lm_head_lora"}
    for sl in range(cfg.num_virtual_layers):
        for t, mod in (("q", "q_loras"), ("k", "k_loras"), ("v", "v_loras"), ("o", "o_loras"), ("mlp", "mlp_loras")):
            names[f"{t}{sl}"] = f"{mod}.{sl}"
    assert len([k for k in ttt.lora.A if k.startswith("q")]) == 6
    for ours in ttt.lora.A:
        assert torch.equal(ttt.lora.A[ours], torch.from_numpy(g[f"m_lora/init/{names[ours]}.A"])), ours
    arr = g["arr"].astype(np.int64)
    for end in (24, 48, 72, 96):
        loss = ttt.update(arr, end)
        assert abs(loss - float(g[f"m_lora/{end}/loss"])) < 1e-5, (end, loss)
    err = 0.0
    for ours in ttt.lora.A:
        for part, t in (("A", ttt.lora.A[ours]), ("B", ttt.lora.B[ours])):
            err = max(err, float(np.abs(t.detach().numpy() - g[f"m_lora/final/{names[ours]}.{part}"]).max()))
    assert err < 0.05 * cfg.ttt_lora_lr, err


def test_oracle_lora_steps_match_reference(golden):
    """Three LoRA steps per boundary (replay windows after the first) against
    the reference's own online_retrain in lora mode: losses and adapters."""
    g = golden("lora_steps.npz")
    cfg = ModelConfig(**{**SMALL, "online_retrain_steps": 3, "online_retrain_replay": True})
    m = OracleModel(OracleWeights.from_model_weights(C.synth_weights(cfg, seed=7)))
    ttt = OracleTTT(m)
    names = {"lm": "lm_head_lora"}
    for i in range(cfg.num_layers):
        for t in ("q", "k", "v", "o"):
            names[f"{t}{i}"] = f"{t}_loras.{i}"
    for ours, ref in names.items():
        assert torch.equal(ttt.lora.A[ours], torch.from_numpy(g[f"init/{ref}.A"])), ours
    arr = g["arr"].astype(np.int64)
    every = cfg.online_retrain_every
    for end in (every, 2 * every):
        loss = ttt.update(arr, end)
        assert abs(loss - float(g[f"{end}/loss"])) < 1e-5, (end, loss)
    for ours, ref in names.items():
        np.testing.assert_allclose(ttt.lora.A[ours].detach().numpy(), g[f"final/{ref}.A"], atol=1e-6)
        np.testing.assert_allclose(ttt.lora.B[ours].detach().numpy(), g[f"final/{ref}.B"], atol=1e-6)
